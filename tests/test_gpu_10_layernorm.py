"""LayerNorm / add+LayerNorm kernels against torch fp32 (gpu).

Cases follow the reference's scripts/verify_layernorm_warp.py: narrow and wide
rows, D not a multiple of 32, ragged row counts, and large-mean rows that
catch a naive one-pass variance.
"""

import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu

TOL = 1e-5


def _ref_ln(x, w, b, eps=1e-5):
    return F.layer_norm(x.double(), (x.shape[-1],), w.double(), b.double(), eps).float()


@pytest.mark.parametrize("rows,D", [(1, 64), (7, 256), (300, 512), (33, 1024), (16, 2048),
                                    (5, 100), (9, 1000), (64, 32), (3, 48)])
def test_layernorm_plain(kernels, rows, D):
    g = torch.Generator(device="cuda").manual_seed(rows * 1000 + D)
    x = torch.randn(rows, D, device="cuda", generator=g)
    w = torch.randn(D, device="cuda", generator=g)
    b = torch.randn(D, device="cuda", generator=g)
    out = kernels.fused_layernorm(x, w, b, 1e-5)
    torch.testing.assert_close(out, _ref_ln(x, w, b), atol=TOL, rtol=TOL)


@pytest.mark.parametrize("rows,D", [(11, 256), (128, 512), (2, 2048), (17, 96)])
def test_add_layernorm(kernels, rows, D):
    g = torch.Generator(device="cuda").manual_seed(7 + D)
    x = torch.randn(rows, D, device="cuda", generator=g)
    s = torch.randn(rows, D, device="cuda", generator=g)
    w = torch.rand(D, device="cuda", generator=g) + 0.5
    b = torch.randn(D, device="cuda", generator=g)
    x_new, normed = kernels.fused_add_layernorm(x, s, w, b, 1e-5)
    assert torch.equal(x_new, x + s)
    torch.testing.assert_close(normed, _ref_ln(x + s, w, b), atol=TOL, rtol=TOL)


def test_large_mean_rows(kernels):
    """Rows with mean 1e4 and unit spread: a sum-then-square variance loses it."""
    g = torch.Generator(device="cuda").manual_seed(3)
    x = torch.randn(64, 512, device="cuda", generator=g) + 1e4
    w = torch.ones(512, device="cuda")
    b = torch.zeros(512, device="cuda")
    out = kernels.fused_layernorm(x, w, b, 1e-5)
    torch.testing.assert_close(out, _ref_ln(x, w, b), atol=2e-3, rtol=0)


def test_normed_half_and_row_mask(kernels):
    g = torch.Generator(device="cuda").manual_seed(5)
    x = torch.randn(4, 32, 256, device="cuda", generator=g)
    w = torch.randn(256, device="cuda", generator=g)
    b = torch.randn(256, device="cuda", generator=g)
    out16 = kernels.fused_layernorm(x, w, b, 1e-5, True)
    assert out16.dtype == torch.float16
    assert torch.equal(out16, _ref_ln(x, w, b).half()) or \
        (out16.float() - _ref_ln(x, w, b)).abs().max().item() <= 2e-3
    valid = torch.rand(4, 32, device="cuda", generator=g) > 0.3
    out = kernels.layernorm_rows(x, w, b, 1e-5, row_valid=valid.reshape(-1))
    ref = _ref_ln(x, w, b).masked_fill(~valid[..., None], 0)
    torch.testing.assert_close(out, ref, atol=TOL, rtol=TOL)


def test_zero_rows(kernels):
    x = torch.empty(0, 256, device="cuda")
    w = torch.ones(256, device="cuda")
    out = kernels.fused_layernorm(x, w, torch.zeros_like(w))
    assert out.shape == (0, 256)


def test_bad_shape_raises(kernels):
    x = torch.randn(4, 256, device="cuda")
    with pytest.raises(RuntimeError, match="weight/bias must have 256 elements"):
        kernels.fused_layernorm(x, torch.ones(128, device="cuda"), torch.zeros(128, device="cuda"))
    with pytest.raises(RuntimeError, match="2048"):
        big = torch.randn(2, 4096, device="cuda")
        kernels.fused_layernorm(big, torch.ones(4096, device="cuda"), torch.zeros(4096, device="cuda"))


def test_identity_smoke(kernels):
    x = torch.randn(1000, device="cuda")
    assert torch.equal(kernels.smoke_test_identity(x), x)
