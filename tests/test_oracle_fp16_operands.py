"""The oracle's fp16-operand restatement of the reference's kernel arithmetic (cpu)."""

import torch

from oracle import layer as O


def _case(causal):
    cfg = O.TransformerConfig(2, 48, 64, 4, 96, 2, causal)
    params = O.init_params(cfg, 3)
    x, mask = O.generate_random_case(cfg, 4, 0.4, 1.0)
    return cfg, params, x, mask


def test_without_rounding_it_is_the_baseline(monkeypatch):
    """With the fp16 rounding taken out, the graph is the baseline's exactly."""
    monkeypatch.setattr(O, "_r16", lambda t: t.double())
    for causal in (False, True):
        cfg, params, x, mask = _case(causal)
        ref = O.baseline_forward(params, cfg, x, mask)
        got = O.fp16_operand_forward(params, cfg, x, mask)
        assert (got - ref).abs().max().item() < 1e-5


def test_rounding_moves_it_by_fp16_amounts():
    cfg, params, x, mask = _case(True)
    ref = O.baseline_forward(params, cfg, x, mask)
    got = O.fp16_operand_forward(params, cfg, x, mask)
    diff = (got - ref).abs().max().item()
    assert 1e-5 < diff < 1e-2, diff
    assert torch.all(got[~mask] == 0)
