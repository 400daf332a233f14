"""GEMM + residual + LayerNorm in one kernel (dotl_linear_ln), gpu.

x_new is checked against a float64 GEMM of the same fp16 operands (bound
relative to the row's scale, as the plain GEMM tests), normed against a
float64 LayerNorm of that x_new. The cluster shapes cover every cluster size
the layer uses (1 for d_model 256 at tile 256, 2, 4 and 8), partial M tiles,
every residual mode, both normed dtypes, and x_new not stored.
"""

import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu

EPS = 1e-5


def _operands(M, N, K, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    a = torch.randn(M, K, device="cuda", generator=g).half()
    w = (torch.randn(N, K, device="cuda", generator=g) * K ** -0.5).half()
    b = torch.randn(N, device="cuda", generator=g) * 0.1
    resid = torch.randn(M, N, device="cuda", generator=g)
    lw = 1.0 + 0.1 * torch.randn(N, device="cuda", generator=g)
    lb = 0.1 * torch.randn(N, device="cuda", generator=g)
    rv = torch.rand(M, device="cuda", generator=g) > 0.3
    return a, w, b, resid, lw, lb, rv


def _x_ref(a, w, b, resid, rv, mode):
    y = a.double() @ w.double().t() + b.double()
    if mode == 0:
        return y
    r = resid.double()
    v = rv.double()[:, None]
    if mode == 1:
        return r + y
    if mode == 2:
        return r + y * v
    return (r + y) * v


def _scale(a, w, resid):
    return (a.double().abs() @ w.double().abs().t()).clamp_min(1e-3) + resid.double().abs()


@pytest.mark.parametrize("M,N,K,tile", [
    (2048, 512, 512, 0),      # cfg2 out_proj: tile 64, cluster 8
    (2048, 512, 2048, 0),     # cfg2 ffn_out
    (300, 256, 256, 0),       # cfg1-like, partial M tile, cluster 4
    (1000, 256, 256, 256),    # cluster 1
    (640, 1024, 512, 256),    # cluster 4
    (384, 2048, 256, 256),    # cluster 8 at tile 256
    (256, 512, 128, 128),     # cluster 4 at tile 128
    (129, 512, 64, 256),      # cluster 2, one row past a tile
])
@pytest.mark.parametrize("mode", [1, 2, 3])
def test_linear_ln_matches_reference(kernels, M, N, K, tile, mode):
    a, w, b, resid, lw, lb, rv = _operands(M, N, K, M + N + K + mode)
    rvu = rv.to(torch.uint8)
    x, n = kernels.linear_ln(a, w, b, lw, lb, EPS, resid=resid, row_valid=rvu, resid_mode=mode,
                             normed_half=False, tile_n=tile)
    xr = _x_ref(a, w, b, resid, rv, mode)
    err = ((x.double() - xr).abs() / _scale(a, w, resid)).max().item()
    assert err < 1e-5, err
    nr = F.layer_norm(x.double(), (N,), lw.double(), lb.double(), EPS)
    nerr = (n.double() - nr).abs().max().item()
    assert nerr < 1e-4, nerr


@pytest.mark.parametrize("store_x", [True, False])
def test_linear_ln_f16_and_row_mask(kernels, store_x):
    M, N, K = 1024, 512, 1024
    a, w, b, resid, lw, lb, rv = _operands(M, N, K, 5)
    rvu = rv.to(torch.uint8)
    x_ref, _ = kernels.linear_ln(a, w, b, lw, lb, EPS, resid=resid, row_valid=rvu, resid_mode=3,
                                 normed_half=False)
    x, n = kernels.linear_ln(a, w, b, lw, lb, EPS, resid=resid, row_valid=rvu, resid_mode=3,
                             store_x=store_x, normed_half=True, normed_row_valid=rvu)
    assert n.dtype == torch.float16
    if store_x:
        assert torch.equal(x, x_ref)
    else:
        assert x is None
    nr = F.layer_norm(x_ref.double(), (N,), lw.double(), lb.double(), EPS)
    nr[~rv] = 0.0
    err = (n.double() - nr).abs() / (nr.abs() + 1e-2)
    assert err.max().item() < 2 ** -10
    assert torch.all(n[~rv] == 0)


def test_linear_ln_matches_unfused_pair(kernels):
    """The fused kernel against the two it replaces (GEMM with residual, then
    the LayerNorm kernel): same x_new bits, normed within fp32 rounding."""
    M, N, K = 2048, 512, 2048
    a, w, b, resid, lw, lb, rv = _operands(M, N, K, 9)
    x_u = kernels.linear_fp16(a, w, b, resid=resid, resid_mode=1)
    n_u = kernels.layernorm_rows(x_u, lw, lb, EPS, out_half=False)
    x_f, n_f = kernels.linear_ln(a, w, b, lw, lb, EPS, resid=resid, resid_mode=1, normed_half=False)
    assert (x_f - x_u).abs().max().item() < 1e-5
    assert (n_f - n_u).abs().max().item() < 1e-4


def test_linear_ln_repeatable(kernels):
    """Two calls give the same bits (the cluster merges statistics in rank order)."""
    M, N, K = 1536, 1024, 512
    a, w, b, resid, lw, lb, rv = _operands(M, N, K, 13)
    _, n1 = kernels.linear_ln(a, w, b, lw, lb, EPS, resid=resid, resid_mode=1, normed_half=False)
    _, n2 = kernels.linear_ln(a, w, b, lw, lb, EPS, resid=resid, resid_mode=1, normed_half=False)
    assert torch.equal(n1, n2)


def test_linear_ln_rejects(kernels):
    a, w, b, resid, lw, lb, rv = _operands(128, 96, 64, 1)
    with pytest.raises(RuntimeError, match="cluster"):
        kernels.linear_ln(a, w, b, lw, lb, EPS)
    assert not kernels.linear_ln_supported(96)
    assert kernels.linear_ln_supported(512) and kernels.linear_ln_supported(2048)
    assert not kernels.linear_ln_supported(4096)
