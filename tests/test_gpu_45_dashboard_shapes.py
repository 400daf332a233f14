"""The reference dashboard's official shapes (4-layer causal models, ffn_dim =
d_model; the shapes are listed with the reference's published results) through
the whole multi-layer model, gpu.

Every shape is checked (head_dim 32/64/128 on the tcgen05 attention, 8 and 256
on the CUDA-core kernel) on a few batch rows (rows never interact) with the
reference harness's pass rule against the reference's fp16 kernel arithmetic,
and against the fp32 baseline no worse than that arithmetic is itself.
The last shape (S = 100,000, two layers) is beyond what the CPU oracle can
check in a test and is left to the benchmark.
"""

import pytest
import torch

from oracle import layer as O

pytestmark = pytest.mark.gpu

ATOL, RTOL = 2e-3, 0.02

# (B, S, d_model, heads, ffn_dim, layers)
SHAPES = {
    1: (64, 128, 128, 4, 128, 4),
    2: (1, 128, 128, 4, 128, 4),
    3: (4, 128, 128, 4, 128, 4),
    4: (16, 128, 128, 4, 128, 4),
    5: (128, 128, 128, 4, 128, 4),
    6: (10000, 128, 128, 4, 128, 4),
    7: (64, 128, 32, 4, 32, 4),
    8: (64, 128, 1024, 4, 1024, 4),
    9: (64, 128, 128, 1, 128, 4),
    10: (64, 128, 128, 2, 128, 4),
    11: (64, 128, 128, 16, 128, 4),
    12: (64, 32, 128, 4, 128, 4),
    13: (64, 1024, 128, 4, 128, 4),
}
UNSUPPORTED = set()   # head_dim 8 (shapes 7, 11) and 256 (shape 8) run on the CUDA-core attention


def _model(cfg, seed):
    from optimized import OptimizedTransformer

    params = O.init_params(cfg, seed)
    m = OptimizedTransformer(cfg)
    m.load_state_dict(params, strict=True)
    return m.cuda().eval(), params


@pytest.mark.parametrize("shape", sorted(SHAPES))
def test_dashboard_shape(kernels, shape):
    B, S, d, H, F, L = SHAPES[shape]
    cfg = O.TransformerConfig(B, S, d, H, F, L, True)
    model, params = _model(cfg, 100 + shape)
    x, mask = O.generate_random_case(cfg, 200 + shape, 0.25, 1.0)
    if shape in UNSUPPORTED:
        with pytest.raises(RuntimeError, match="head_dim"):
            with torch.inference_mode():
                model(x.cuda(), mask.cuda())
        return
    with torch.inference_mode():
        out = model(x.cuda(), mask.cuda()).cpu()
    assert torch.isfinite(out).all()
    rows = sorted({0, B // 2, B - 1})
    idx = torch.tensor(rows)
    sub = O.TransformerConfig(len(rows), S, d, H, F, L, True)
    got = out[idx]
    # (1) Parity: the harness rule against the reference's fp16 kernel
    # arithmetic (fp16 operands where its kernels round them, exact otherwise).
    ref16 = O.fp16_operand_forward(params, sub, x[idx], mask[idx])
    r16 = O.compare_outputs(ref16, got, rtol=RTOL, atol=ATOL)
    assert r16.passed, (shape, r16.failed_elements, r16.max_abs_error, r16.worst_index)
    # (2) Against the fp32 baseline, a sanity bound. Over 4 layers fp16
    # operands alone can miss the 2e-3 bound on a few elements (e.g. 1-4 of
    # 49,152 on shapes 1-5 with these seeds). The rule here: at most twice the
    # misses of the reference's own fp16 arithmetic plus 4 (counts this small
    # are rounding noise: shape 7, d_model 32, has 4 against its 1 of 12,288),
    # and the largest error at most 1.25x the larger of atol and its largest error.
    ref = O.baseline_forward(params, sub, x[idx], mask[idx])
    r32 = O.compare_outputs(ref, got, rtol=RTOL, atol=ATOL)
    e32 = O.compare_outputs(ref, ref16, rtol=RTOL, atol=ATOL)
    detail = (shape, r32.failed_elements, r32.max_abs_error, e32.failed_elements, e32.max_abs_error)
    assert r32.failed_elements <= 2 * e32.failed_elements + 4, detail
    assert r32.max_abs_error <= 1.25 * max(ATOL, e32.max_abs_error), detail
