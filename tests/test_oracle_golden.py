"""The CPU oracle against fixtures generated from the reference itself (no GPU).

tests/golden/*.npz were produced by tests/golden/make_golden.py from the
unmodified reference BaselineTransformer and generate_random_case; these tests
pin the oracle (inputs, parameters and outputs) to them bit for bit.
"""

import os

import numpy as np
import pytest
import torch

from conftest import GOLDEN
from oracle import layer as O

CASES = sorted(f[:-4] for f in os.listdir(GOLDEN) if f.endswith(".npz"))


def _load(name):
    z = np.load(os.path.join(GOLDEN, f"{name}.npz"))
    B, S, d, H, F, L, causal = (int(v) for v in z["cfg"])
    return z, O.TransformerConfig(B, S, d, H, F, L, bool(causal))


def test_fixtures_present():
    assert {"cfg1", "small_causal", "odd_causal_pad", "short_seq", "hd128_causal",
            "two_layer_pad"} <= set(CASES)


@pytest.mark.parametrize("name", CASES)
def test_inputs_regenerate_bit_exact(name):
    z, cfg = _load(name)
    x, mask = O.generate_random_case(cfg, int(z["input_seed"]), float(z["padding_ratio"]), 1.0)
    assert np.array_equal(x.numpy(), z["x"])
    assert np.array_equal(mask.numpy(), z["mask"])


@pytest.mark.parametrize("name", CASES)
def test_params_regenerate(name):
    z, cfg = _load(name)
    params = O.init_params(cfg, int(z["seed"]))
    assert O.param_checksum(params) == pytest.approx(float(z["param_checksum"]), abs=1e-9)


@pytest.mark.parametrize("name", CASES)
def test_oracle_matches_reference_output(name):
    z, cfg = _load(name)
    params = O.init_params(cfg, int(z["seed"]))
    x = torch.from_numpy(z["x"])
    mask = torch.from_numpy(z["mask"])
    out = O.baseline_forward(params, cfg, x, mask)
    ref = torch.from_numpy(z["out"])
    # Same ops in the same order on the same CPU build: expect identity;
    # allow a few ulp for a different CPU (vector width changes reductions).
    assert (out - ref).abs().max().item() <= 1e-5
    if not float(z["padding_ratio"]) > 0:
        return
    assert torch.all(out[~mask] == 0), "padded rows must be zero"


def test_chunked_attention_is_same_math():
    """ChunkedBaselineSelfAttention semantics: scoring queries in blocks gives the same rows."""
    cfg = O.TransformerConfig(2, 96, 64, 4, 128, 1, True)
    params = O.init_params(cfg, 5)
    x, mask = O.generate_random_case(cfg, 6, 0.5, 1.0)
    a = O.baseline_forward(params, cfg, x, mask)
    b = O.baseline_forward(params, cfg, x, mask, query_block=32)
    assert (a - b).abs().max().item() <= 1e-5


def test_compare_outputs_rule():
    """|d| <= atol OR |d| <= rtol*|ref|, both finite, zero failures
    (torch_transformer_benchmark.py:557-624)."""
    ref = torch.tensor([1.0, 100.0, 0.0, 0.5, float("nan")])
    ok = torch.tensor([1.0015, 101.5, 0.0019, 0.5, float("nan")])
    r = O.compare_outputs(ref[:4], ok[:4])
    assert r.passed and r.failed_elements == 0
    bad = torch.tensor([1.03, 103.0, 0.0021, 0.5])
    r = O.compare_outputs(ref[:4], bad)
    assert not r.passed and r.failed_elements == 3
    r = O.compare_outputs(ref, ok)
    assert not r.passed and r.failed_elements == 1, "non-finite elements fail"
    with pytest.raises(AssertionError, match="shape mismatch"):
        O.compare_outputs(ref[:2], ok[:3])


def test_generate_random_case_lengths():
    """padding_ratio 0.5 gives lengths in [S/2, S] and zeroed padded rows (D3)."""
    cfg, pad = O.BASELINE_CONFIGS[1]
    x, mask = O.generate_random_case(cfg, 1234, pad, 1.0)
    lengths = mask.sum(1)
    assert torch.all(lengths >= 64) and torch.all(lengths <= 128)
    assert torch.all(mask == (torch.arange(128)[None, :] < lengths[:, None]))
    assert torch.all(x[~mask] == 0)


def test_baseline_config_shapes():
    shapes = {k: (c.batch_size, c.seq_len, c.d_model, c.num_heads, c.ffn_dim, c.causal, p)
              for k, (c, p) in O.BASELINE_CONFIGS.items()}
    assert shapes == {
        1: (2, 128, 256, 4, 1024, False, 0.5),
        2: (4, 512, 512, 8, 2048, True, 0.0),
        3: (8, 2048, 1024, 16, 4096, False, 0.5),
        4: (8192, 32, 256, 4, 1024, False, 0.0),
        5: (16, 1024, 2048, 16, 8192, True, 0.0),
    }
