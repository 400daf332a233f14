"""Host-side logic of the drop-in package, on the CPU (no GPU)."""

import argparse

import pytest
import torch

from oracle import layer as O


def test_state_dict_names_match_the_reference_model():
    """One state_dict loads into OptimizedTransformer with strict=True
    (layers.py:1-5, model.py:24-30 upstream)."""
    from optimized import OptimizedTransformer

    cfg = O.TransformerConfig(2, 16, 64, 4, 128, 2, True)
    params = O.init_params(cfg, 1)
    model = OptimizedTransformer(cfg)
    model.load_state_dict(params, strict=True)
    assert set(model.state_dict()) == set(params)
    assert torch.equal(model.layers[1].ffn_in.weight, params["layers.1.ffn_in.weight"])


def test_usermixin_declaration_works():
    """The harness's `class UserOptimizedTransformer(OptimizedTransformer, BaselineTransformer)`."""
    import torch.nn as nn

    from optimized import OptimizedTransformer

    class BaselineTransformer(nn.Module):
        pass

    class UserOptimizedTransformer(OptimizedTransformer, BaselineTransformer):
        pass

    m = UserOptimizedTransformer(O.TransformerConfig(1, 8, 32, 2, 64, 1, False))
    assert isinstance(m, BaselineTransformer)


def test_qkv_weight_cache_rebuilds_on_version_change():
    from optimized import OptimizedTransformer

    cfg = O.TransformerConfig(1, 8, 32, 2, 64, 1, False)
    m = OptimizedTransformer(cfg)
    m.load_state_dict(O.init_params(cfg, 2), strict=True)
    attn = m.layers[0].attention
    w1, b1 = attn._get_qkv_weight()
    assert w1.dtype == torch.float16 and w1.shape == (96, 32) and b1.dtype == torch.float32
    assert attn._get_qkv_weight()[0] is w1
    with torch.no_grad():
        attn.k_proj.weight.mul_(2.0)
    w2, _ = attn._get_qkv_weight()
    assert w2 is not w1
    assert torch.equal(w2[32:64], (attn.k_proj.weight.half()))


def test_config_validate_refuses_fallbacks():
    from optimized import config

    config.validate()
    for knob, bad in (("ATTENTION_IMPL", "scalar"), ("ATTENTION_PRECISION", "bf16"),
                      ("LINEAR_GELU", "off"), ("LINEAR_BIAS", "tf32"), ("LAYERNORM", "off"),
                      ("CUDA_GRAPH", "sometimes")):
        old = getattr(config, knob)
        setattr(config, knob, bad)
        try:
            with pytest.raises(ValueError):
                config.validate()
        finally:
            setattr(config, knob, old)
    config.validate()


def test_cli_hooks():
    from optimized import cli, config

    parser = argparse.ArgumentParser()
    cli.add_arguments(parser)
    args = parser.parse_args(["--cuda-graph", "off", "--attn-impl", "wmma"])
    with pytest.raises(ValueError, match="CUDA"):
        cli.validate_args(args, torch.device("cpu"), torch.float32)
    assert config.CUDA_GRAPH == "auto", "validate_args must not leave overrides applied"
    old = (config.CUDA_GRAPH, config.ATTENTION_IMPL)
    try:
        cli.apply_overrides(args)
        assert (config.CUDA_GRAPH, config.ATTENTION_IMPL) == ("off", "wmma")
        bad = parser.parse_args(["--linear-gelu", "off"])
        with pytest.raises(ValueError, match="LINEAR_GELU"):
            cli.validate_args(bad, torch.device("cuda"), torch.float32)
    finally:
        config.CUDA_GRAPH, config.ATTENTION_IMPL = old


def test_graph_key_and_gate():
    from optimized import config, graphs

    x = torch.empty(2, 8, 32)
    k1 = graphs._graph_key(x, True)
    k2 = graphs._graph_key(x, False)
    assert k1 != k2 and k1 == graphs._graph_key(torch.empty(2, 8, 32), True)
    assert not graphs._graph_eligible(x, 0), "CPU tensors never capture"
    old = config.CUDA_GRAPH
    config.CUDA_GRAPH = "off"
    try:
        assert not graphs._graph_eligible(x, 0)
    finally:
        config.CUDA_GRAPH = old


def test_mask_is_trivial():
    from optimized import OptimizedTransformer

    m = OptimizedTransformer(O.TransformerConfig(1, 8, 32, 2, 64, 1, False))
    mask = torch.ones(1, 8, dtype=torch.bool)
    assert m._mask_is_trivial(mask) is True
    assert m._mask_is_trivial(None) is False
    mask[0, 3] = False
    assert m._mask_is_trivial(mask) is False, "an in-place edit is seen"


def test_half_weight_cache_semantics():
    import dotl_ops

    cache = dotl_ops._HalfWeightCache()
    w = torch.randn(8, 8)
    h1 = cache.get(w)
    assert h1.dtype == torch.float16 and cache.get(w) is h1
    with torch.no_grad():
        w.add_(1.0)
    h2 = cache.get(w)
    assert h2 is not h1 and torch.equal(h2, w.half())


def test_missing_library_raises(monkeypatch):
    """The product path fails loudly without libdotl: no torch or CPU fallback."""
    import kernel_ext
    from optimized import kernels

    monkeypatch.setattr(kernel_ext, "get_kernels", lambda verbose=False: None)
    with pytest.raises(RuntimeError, match="no fallback"):
        kernels._custom_kernels()


def test_get_kernels_without_cuda_reports_why(monkeypatch):
    import kernel_ext

    monkeypatch.setattr(kernel_ext, "_load_attempted", False)
    monkeypatch.setattr(kernel_ext, "_kernels", None)
    monkeypatch.setattr(torch.cuda, "is_available", lambda: False)
    assert kernel_ext.get_kernels() is None
    assert "CUDA is not available" in str(kernel_ext.load_error())
    monkeypatch.setattr(kernel_ext, "_load_attempted", False)


def test_reference_named_functions_exist():
    import dotl_ops

    for name in ("smoke_test_identity", "fused_layernorm", "fused_add_layernorm", "linear_bias",
                 "linear_gelu", "fused_attention_forward", "fused_ffn_block", "wmma_set_fp16",
                 "wmma_set_cp_async", "layernorm_set_warp_width"):
        assert callable(getattr(dotl_ops, name)), name


def test_attention_refuses_uncovered_requests_on_host():
    """Refusals that need no device: impl/precision/layout codes (the CUDA check
    comes first upstream too, so use meta tensors' shape errors only)."""
    import dotl_ops

    q = torch.empty(1, 1, 8, 64)
    with pytest.raises(RuntimeError, match="out_layout"):
        dotl_ops.fused_attention_forward(q, q, q, out_layout=3)
    with pytest.raises(RuntimeError, match="impl must be"):
        dotl_ops.fused_attention_forward(q, q, q, impl=9)
    with pytest.raises(RuntimeError, match="CUDA"):
        dotl_ops.fused_attention_forward(q, q, q)


class _FakeRunner:
    def __init__(self, fingerprint=None):
        self.released = False
        self.fingerprint = fingerprint

    def release(self):
        self.released = True


def test_reloading_or_moving_weights_drops_captured_graphs():
    """A graph bakes in the fp16 weight copies: load_state_dict and module
    moves drop the model's graphs so the next forward captures the new weights."""
    from optimized import OptimizedTransformer

    cfg = O.TransformerConfig(2, 16, 64, 4, 128, 1, True)
    params = O.init_params(cfg, 1)
    model = OptimizedTransformer(cfg)
    model.load_state_dict(params, strict=True)          # no graphs yet: nothing to drop
    r = _FakeRunner()
    model._graphs.runners[("key",)] = r
    model.load_state_dict(O.init_params(cfg, 2), strict=True)
    assert r.released and not model._graphs
    r2 = _FakeRunner()
    model._graphs.runners[("key",)] = r2
    model.float()                                       # any _apply (to, cuda, half, ...)
    assert r2.released and not model._graphs
    r3 = _FakeRunner()
    model._graphs.runners[("key",)] = r3
    model.eval()                                        # mode switches keep them
    assert not r3.released and model._graphs


def test_in_place_weight_edit_retires_the_graph():
    """An in-place update (optimizer step, copy_, mul_ under no_grad) bumps a
    parameter's version: the graph captured under the old weights is released
    at the next lookup instead of replaying stale fp16 copies."""
    from optimized import OptimizedTransformer
    from optimized.graphs import _weights_fingerprint

    cfg = O.TransformerConfig(2, 16, 64, 4, 128, 1, True)
    model = OptimizedTransformer(cfg)
    model.load_state_dict(O.init_params(cfg, 1), strict=True)
    fp = lambda: _weights_fingerprint(model)  # noqa: E731
    r = _FakeRunner(fp())
    model._graphs.runners[("key",)] = r
    assert model._graphs.get(("key",), fp) is r and not r.released
    with torch.no_grad():
        model.layers[0].ffn_out.weight.mul_(0.5)
    assert model._graphs.get(("key",), fp) is None
    assert r.released and not model._graphs
    r2 = _FakeRunner(fp())
    model._graphs.runners[("key",)] = r2
    with torch.no_grad():
        model.layers[0].attention.q_proj.bias.copy_(torch.ones(64))
    assert model._graphs.get(("key",), fp) is None and r2.released


def test_graph_cache_releases_with_its_model():
    """The model's graphs go when the model is collected (no global registry)."""
    import gc

    from optimized import OptimizedTransformer

    model = OptimizedTransformer(O.TransformerConfig(1, 8, 32, 2, 64, 1, False))
    r = _FakeRunner()
    model._graphs.runners[("key",)] = r
    del model
    gc.collect()
    assert r.released
