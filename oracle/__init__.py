"""CPU oracle for the single-transformer-layer forward. TEST INFRASTRUCTURE ONLY.

This package restates, in plain PyTorch-on-CPU fp32 ops, what the reference
harness `torch_transformer_benchmark.py` computes for the layer forward
(`BaselineTransformer`, lines 70-272), its input generator (lines 500-540) and
its accuracy rule (`compare_outputs`, lines 557-624).

It is the checker, never the product: only `tests/`, `__graft_entry__.smoke()`
and `bench.py` (its CPU-baseline leg and `--impl reference`) may import it. The
shipped path (`kernel_ext` / `optimized` in the package directory) never
imports it and raises when its CUDA library is missing.

Parity of this restatement with the reference itself is pinned by the golden
fixtures in `tests/golden/`, produced by `tests/golden/make_golden.py` from the
unmodified reference `BaselineTransformer` and `generate_random_case`.
"""

from .layer import (  # noqa: F401
    AccuracyResult,
    TransformerConfig,
    attention_reference,
    baseline_forward,
    compare_outputs,
    fp16_operand_forward,
    generate_random_case,
    init_params,
    param_checksum,
    BASELINE_CONFIGS,
)
