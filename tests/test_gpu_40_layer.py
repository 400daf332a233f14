"""The whole layer against the oracle and the golden fixtures (gpu).

The pass rule is the reference harness's (torch_transformer_benchmark.py:
557-624): every element within 2e-3 absolute OR 2% relative of the
reference, both finite, zero failures.
"""

import dataclasses
import os

import numpy as np
import pytest
import torch

from conftest import GOLDEN
from oracle import layer as O

pytestmark = pytest.mark.gpu

ATOL, RTOL = 2e-3, 0.02


def _model(cfg, seed):
    from optimized import OptimizedTransformer

    params = O.init_params(cfg, seed)
    m = OptimizedTransformer(cfg)
    m.load_state_dict(params, strict=True)
    return m.cuda().eval(), params


GOLDEN_CASES = sorted(f[:-4] for f in os.listdir(GOLDEN) if f.endswith(".npz"))


@pytest.mark.parametrize("name", GOLDEN_CASES)
@pytest.mark.parametrize("graph", ["off", "always"])
def test_layer_matches_golden(kernels, name, graph):
    from optimized import config

    z = np.load(os.path.join(GOLDEN, f"{name}.npz"))
    B, S, d, H, F, L, causal = (int(v) for v in z["cfg"])
    cfg = O.TransformerConfig(B, S, d, H, F, L, bool(causal))
    model, params = _model(cfg, int(z["seed"]))
    assert abs(O.param_checksum(params) - float(z["param_checksum"])) < 1e-9
    x = torch.from_numpy(z["x"]).cuda()
    mask = torch.from_numpy(z["mask"]).cuda()
    old = config.CUDA_GRAPH
    config.CUDA_GRAPH = graph
    try:
        with torch.inference_mode():
            out = model(x, mask)
            out2 = model(x, mask)
    finally:
        config.CUDA_GRAPH = old
    torch.cuda.synchronize()
    assert torch.equal(out, out2), "two identical calls must give identical bits"
    r = O.compare_outputs(torch.from_numpy(z["out"]), out.cpu(), rtol=RTOL, atol=ATOL)
    assert r.passed, (r.failed_elements, r.max_abs_error, r.worst_index)
    if graph == "always":
        assert len(model._graphs) == 1, "graph capture declined"


@pytest.mark.parametrize("cfg_id", [1, 2, 3, 4, 5])
def test_baseline_configs_full_size(kernels, cfg_id):
    """Each BASELINE config at its full size on the GPU; the oracle checks a
    subset of batch rows (rows never interact, so a row's output does not
    depend on the rest of the batch)."""
    cfg, pad = O.BASELINE_CONFIGS[cfg_id]
    model, params = _model(cfg, 1234)
    x, mask = O.generate_random_case(cfg, 1234, pad, 1.0)
    with torch.inference_mode():
        out = model(x.cuda(), mask.cuda()).cpu()
    rows = {1: 2, 2: 4, 3: 2, 4: 256, 5: 2}[cfg_id]
    sub = dataclasses.replace(cfg, batch_size=rows)
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    ref = O.baseline_forward(params, sub, x[:rows], mask[:rows] if pad > 0 else None,
                             query_block=256)
    r = O.compare_outputs(ref, out[:rows], rtol=RTOL, atol=ATOL)
    assert r.passed, (r.failed_elements, r.max_abs_error, r.worst_index)
    assert torch.isfinite(out).all()
    if pad > 0:
        assert torch.all(out[~mask] == 0)


def test_batch_rows_independent(kernels):
    """A batch row's output is bit-identical whether it runs alone or in a batch."""
    cfg, pad = O.BASELINE_CONFIGS[1]
    model, _ = _model(cfg, 7)
    x, mask = O.generate_random_case(cfg, 99, pad, 1.0)
    x, mask = x.cuda(), mask.cuda()
    with torch.inference_mode():
        full = model(x, mask)
        one = model(x[1:2].contiguous(), mask[1:2].contiguous())
    assert torch.equal(full[1:2], one)


def test_all_valid_mask_matches_no_mask(kernels):
    """A given all-valid mask takes the masked kernels; the output is the same
    bits as with no mask (the reference instead skips the mask after a host
    check)."""
    cfg, _ = O.BASELINE_CONFIGS[2]
    cfg = dataclasses.replace(cfg, batch_size=2)
    model, _ = _model(cfg, 5)
    x, mask = O.generate_random_case(cfg, 21, 0.0, 1.0)
    assert bool(mask.all())
    x, mask = x.cuda(), mask.cuda()
    with torch.inference_mode():
        a = model(x, mask)
        b = model(x, None)
    assert torch.equal(a, b)


@pytest.mark.parametrize("cfg_id", [1, 2])
def test_host_pipeline_matches_forward(kernels, cfg_id):
    """HostPipeline (pinned host batches in and out, copies overlapped with
    the neighbouring batches' forwards) returns exactly model(x, mask) per batch."""
    from optimized import HostPipeline

    cfg, pad = O.BASELINE_CONFIGS[cfg_id]
    model, _ = _model(cfg, 3)
    cases = [O.generate_random_case(cfg, 40 + i, pad, 1.0) for i in range(5)]
    xs = [x.pin_memory() for x, _ in cases]
    ms = [m.pin_memory() for _, m in cases]
    outs = [torch.empty(x.shape, dtype=torch.float32).pin_memory() for x in xs]
    pipe = HostPipeline(model, torch.device("cuda", 0))
    with torch.inference_mode():
        pipe.run(xs, ms, outs)
        ref = [model(x.cuda(), m.cuda()).cpu() for x, m in zip(xs, ms)]
    for o, r in zip(outs, ref):
        assert torch.equal(o, r)


@pytest.mark.parametrize("name", GOLDEN_CASES)
def test_layer_fused_ln_path_matches_golden(kernels, name, monkeypatch):
    """The layer with every out_proj / ffn_out taking the GEMM + LayerNorm
    kernel wherever it covers d_model (the shape rule normally keeps it to
    large row counts), against the reference's golden outputs."""
    from optimized import config, layers

    z = np.load(os.path.join(GOLDEN, f"{name}.npz"))
    B, S, d, H, F, L, causal = (int(v) for v in z["cfg"])
    if not kernels.linear_ln_supported(d):
        pytest.skip(f"d_model {d} is outside the fused kernel's cluster shapes")
    monkeypatch.setattr(layers, "_linear_ln_ok", lambda rows, n: kernels.linear_ln_supported(n))
    cfg = O.TransformerConfig(B, S, d, H, F, L, bool(causal))
    model, _ = _model(cfg, int(z["seed"]))
    x = torch.from_numpy(z["x"]).cuda()
    mask = torch.from_numpy(z["mask"]).cuda()
    old = config.CUDA_GRAPH
    config.CUDA_GRAPH = "off"
    try:
        with torch.inference_mode():
            out = model(x, mask)
    finally:
        config.CUDA_GRAPH = old
    r = O.compare_outputs(torch.from_numpy(z["out"]), out.cpu(), rtol=RTOL, atol=ATOL)
    assert r.passed, (r.failed_elements, r.max_abs_error, r.worst_index)


def test_graph_replay_semantics(kernels):
    """scripts/verify_graph.py's checks: the replay counter fires; three
    different inputs give three different outputs, each bit-identical to eager
    (no stale input copy); a returned result survives later replays (the output
    is copied out of the graph's buffer); mask modes capture separately."""
    from optimized import config

    cfg = O.TransformerConfig(2, 64, 128, 4, 256, 1, True)
    model, _ = _model(cfg, 5)
    g = torch.Generator(device="cuda").manual_seed(6)
    xs = [torch.randn(2, 64, 128, device="cuda", generator=g) for _ in range(3)]
    mask = torch.ones(2, 64, dtype=torch.bool, device="cuda")
    mask[1, 40:] = False
    old = config.CUDA_GRAPH
    config.CUDA_GRAPH = "always"
    try:
        with torch.inference_mode():
            outs = [model(x, None) for x in xs]
            runner = next(iter(model._graphs.values()))
            assert runner.replays >= 2, "the graph did not replay"
            for i in range(3):
                for j in range(i + 1, 3):
                    assert not torch.equal(outs[i], outs[j]), "stale input copy"
            for x, o in zip(xs, outs):
                assert torch.equal(o, model._forward_eager(x, None, False)), "an earlier result changed"
            om = model(xs[0], mask)
            assert len(model._graphs) == 2, "mask modes must key separately"
            assert torch.equal(om, model._forward_eager(xs[0], mask, True))
    finally:
        config.CUDA_GRAPH = old
        model.release_graphs()
