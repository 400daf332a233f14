"""tcgen05 GEMM with fused epilogues against a float64 reference (gpu).

The reference product uses the same fp16-rounded operands, so the only
differences are fp32 accumulation order and the output rounding: the bound is
relative to the row's scale (sum |a||w|), 1e-5 for fp32 output and one fp16
ulp (2^-10 relative) for fp16 output.
"""

import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu


def _operands(M, N, K, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    a = torch.randn(M, K, device="cuda", generator=g).half()
    w = (torch.randn(N, K, device="cuda", generator=g) * K ** -0.5).half()
    b = torch.randn(N, device="cuda", generator=g) * 0.1
    return a, w, b


def _ref(a, w, b, act=False):
    y = a.double() @ w.double().t() + b.double()
    if act:
        y = F.gelu(y, approximate="none")
    return y


def _scale(a, w):
    return (a.double().abs() @ w.double().abs().t()).clamp_min(1e-3)


@pytest.mark.parametrize("M,N,K,tile", [
    (128, 128, 64, 128), (256, 256, 64, 256), (300, 384, 256, 0), (1, 128, 64, 0),
    (129, 136, 72, 128), (2048, 1536, 512, 0), (512, 1024, 2048, 256), (1000, 8, 8, 128),
    (4096, 2048, 8192, 0)])
def test_linear_bias_f32(kernels, M, N, K, tile):
    a, w, b = _operands(M, N, K, M + N + K)
    out = kernels.linear_fp16(a, w, b, tile_n=tile)
    ref = _ref(a, w, b)
    err = ((out.double() - ref).abs() / _scale(a, w)).max().item()
    assert err < 1e-5, err


@pytest.mark.parametrize("M,N,K", [(256, 1024, 256), (2048, 2048, 512), (77, 264, 128)])
def test_linear_gelu_f16(kernels, M, N, K):
    a, w, b = _operands(M, N, K, 11)
    out = kernels.linear_fp16(a, w, b, act=1, out_half=True)
    assert out.dtype == torch.float16
    ref = _ref(a, w, b, act=True)
    err = (out.double() - ref).abs() / (ref.abs() + 1e-2)
    assert err.max().item() < 2 ** -10


@pytest.mark.parametrize("mode", [1, 2, 3])
def test_linear_residual_modes(kernels, mode):
    M, N, K = 384, 512, 256
    a, w, b = _operands(M, N, K, 21)
    g = torch.Generator(device="cuda").manual_seed(4)
    resid = torch.randn(M, N, device="cuda", generator=g)
    valid = torch.rand(M, device="cuda", generator=g) > 0.25
    out = kernels.linear_fp16(a, w, b, resid=resid, row_valid=valid, resid_mode=mode)
    proj = _ref(a, w, b)
    if mode == 1:
        ref = resid.double() + proj
    elif mode == 2:
        ref = resid.double() + proj.masked_fill(~valid[:, None], 0)
    else:
        ref = (resid.double() + proj).masked_fill(~valid[:, None], 0)
    err = ((out.double() - ref).abs() / (_scale(a, w) + resid.double().abs())).max().item()
    assert err < 1e-5, err
    if mode == 3:
        assert torch.all(out[~valid] == 0)


@pytest.mark.parametrize("N", [384, 320, 448])
def test_partial_last_tile_f16_many_tiles(kernels, N):
    """fp16 output, width-256 tiles whose last N tile is partial, ~34 tiles per
    CTA (the dashboard's B=10000 QKV shape): the chunks past N stage nothing, so
    the double-buffered staging never overwrites a half a store still reads."""
    M, K = 320000, 128
    a, w, b = _operands(M, N, K, N)
    out = kernels.linear_fp16(a, w, b, out_half=True, tile_n=256)
    ref = _ref(a, w, b)
    err = (out.double() - ref).abs() / (ref.abs() + _scale(a, w) * 1e-3)
    assert err.max().item() < 2 ** -10, err.max().item()


def test_reference_named_entry_points(kernels):
    """linear_bias / linear_gelu take fp32 x and fp32 nn.Linear weights, as upstream."""
    g = torch.Generator(device="cuda").manual_seed(9)
    x = torch.randn(2, 64, 256, device="cuda", generator=g)
    w = torch.randn(512, 256, device="cuda", generator=g) * 0.05
    b = torch.randn(512, device="cuda", generator=g) * 0.02
    y = kernels.linear_bias(x, w, b)
    assert y.shape == (2, 64, 512) and y.dtype == torch.float32
    ref = x.half().double() @ w.half().double().t() + b.double()
    assert (y.double() - ref).abs().max().item() < 1e-4
    y16 = kernels.linear_bias(x, w, b, -1, -1, True)
    assert y16.dtype == torch.float16
    yg = kernels.linear_gelu(x, w, b)
    refg = F.gelu(ref, approximate="none")
    assert (yg.double() - refg).abs().max().item() < 1e-4
    # deterministic: the same call gives the same bits
    assert torch.equal(kernels.linear_bias(x, w, b), y)


def test_rows_independent_of_m(kernels):
    """A row's result does not depend on how many rows share the launch."""
    a, w, b = _operands(1024, 512, 512, 5)
    full = kernels.linear_fp16(a, w, b)
    part = kernels.linear_fp16(a[100:357].contiguous(), w, b)
    assert torch.equal(full[100:357], part)


def test_gemm_rejects(kernels):
    a, w, b = _operands(64, 64, 64, 1)
    with pytest.raises(RuntimeError, match="multiples? of 8"):
        kernels.linear_fp16(a[:, :60], w[:, :60], b)
    with pytest.raises(RuntimeError, match="x's last dimension must match"):
        kernels.linear_bias(torch.randn(4, 32, device="cuda"), torch.randn(8, 16, device="cuda"),
                            torch.randn(8, device="cuda"))


def test_gelu_epilogue_matches_exact_erf(kernels):
    """The epilogue's GELU (erf from Abramowitz & Stegun 7.1.28, |error| <= 3e-7)
    against the exact erf GELU in float64, over every fp16 value in [-12, 12]."""
    v = torch.arange(-12.0, 12.0, 2.0 ** -9, device="cuda").half().unique()
    M = v.numel()
    a = torch.zeros(M, 8, device="cuda", dtype=torch.float16)
    a[:, 0] = v
    w = torch.zeros(8, 8, device="cuda", dtype=torch.float16)
    w[0, 0] = 1.0
    b = torch.zeros(8, device="cuda")
    out = kernels.linear_fp16(a, w, b, act=1)[:, 0].double()
    ref = F.gelu(v.double(), approximate="none")
    err = (out - ref).abs()
    assert (err <= 1e-6 * (1.0 + v.double().abs())).all(), err.max().item()


@pytest.mark.parametrize("M,N,K", [(2048, 512, 2048), (300, 392, 576), (128, 128, 128), (1000, 256, 1088)])
@pytest.mark.parametrize("mode", [0, 1, 3])
def test_split_k_pair(kernels, M, N, K, mode):
    """tile_n=-128: two CTAs of a cluster split K and add their partial sums
    (ragged M and N tiles, odd k-block counts, every epilogue kind)."""
    a, w, b = _operands(M, N, K, M + K + mode)
    g = torch.Generator(device="cuda").manual_seed(6)
    resid = torch.randn(M, N, device="cuda", generator=g)
    valid = torch.rand(M, device="cuda", generator=g) > 0.25
    if mode == 0:
        out = kernels.linear_fp16(a, w, b, act=1, out_half=True, tile_n=-128)
        ref = _ref(a, w, b, act=True)
        err = (out.double() - ref).abs() / (ref.abs() + 1e-2)
        assert err.max().item() < 2 ** -10
    else:
        out = kernels.linear_fp16(a, w, b, resid=resid, row_valid=valid, resid_mode=mode, tile_n=-128)
        proj = _ref(a, w, b)
        ref = resid.double() + proj if mode == 1 else (resid.double() + proj).masked_fill(~valid[:, None], 0)
        err = ((out.double() - ref).abs() / (_scale(a, w) + resid.double().abs())).max().item()
        assert err < 1e-5, err
        again = kernels.linear_fp16(a, w, b, resid=resid, row_valid=valid, resid_mode=mode, tile_n=-128)
        assert torch.equal(out, again), "the pair's sum must not depend on timing"


def test_split_k_is_auto_for_long_k_few_tiles(kernels):
    """The shape rule takes the split pair for the config-2 ffn_out GEMM
    (128 tiles of width 64 and 32 k-blocks): auto and forced give the same bits."""
    a, w, b = _operands(2048, 512, 2048, 77)
    assert torch.equal(kernels.linear_fp16(a, w, b), kernels.linear_fp16(a, w, b, tile_n=-128))


@pytest.mark.parametrize("M,N,K,mode,act,half_out", [
    (256, 256, 64, 0, 0, False), (512, 1024, 512, 1, 0, False), (300, 512, 256, 3, 0, False),
    (1000, 768, 1024, 0, 1, True), (2048, 2048, 2048, 2, 0, False), (129, 256, 72, 0, 0, True),
    (4096, 6144, 512, 0, 0, True)])
def test_cta_pair_tiles(kernels, M, N, K, mode, act, half_out):
    """tile_n=-256: two CTAs of a cluster run each 256 x 256 tile with M = 256
    MMAs, each staging half of W; every epilogue against float64."""
    a, w, b = _operands(M, N, K, 40 + M)
    g = torch.Generator(device="cuda").manual_seed(41)
    resid = torch.randn(M, N, device="cuda", generator=g) if mode else None
    valid = (torch.rand(M, device="cuda", generator=g) > 0.3) if mode >= 2 else None
    out = kernels.linear_fp16(a, w, b, act=act, resid=resid, row_valid=valid, resid_mode=mode,
                              out_half=half_out, tile_n=-256)
    one = kernels.linear_fp16(a, w, b, act=act, resid=resid, row_valid=valid, resid_mode=mode,
                              out_half=half_out, tile_n=256)
    y = _ref(a, w, b, act=bool(act))
    if mode == 1:
        y = resid.double() + y
    elif mode == 2:
        y = resid.double() + torch.where(valid[:, None], y, torch.zeros_like(y))
    elif mode == 3:
        y = torch.where(valid[:, None], resid.double() + y, torch.zeros_like(y))
    scale = _scale(a, w) + (resid.double().abs() if resid is not None else 0)
    tol = 2 ** -10 if half_out else 1e-5
    assert ((out.double() - y).abs() / (scale if not half_out else y.abs() + 1e-2)).max().item() < tol
    assert ((out.double() - one.double()).abs() / scale).max().item() < 1e-5


@pytest.mark.parametrize("tile", [160, 192, 224])
@pytest.mark.parametrize("M,N,K,mode,act,half_out", [
    (300, 512, 256, 0, 0, False), (257, 1000, 128, 1, 0, False), (2048, 2048, 512, 3, 0, False),
    (129, 456, 72, 2, 0, False), (1000, 768, 1024, 0, 1, True), (64, 8, 64, 0, 0, True)])
def test_intermediate_tile_widths(kernels, tile, M, N, K, mode, act, half_out):
    """tile_n 160/192/224 (two accumulators in a 512-column TMEM allocation,
    the second at column 256; last N tile partial on most shapes): every
    epilogue against float64, and the same bits as width 256, since each
    output element's k loop is the same whatever the tile's width."""
    a, w, b = _operands(M, N, K, 60 + M + tile)
    g = torch.Generator(device="cuda").manual_seed(61)
    resid = torch.randn(M, N, device="cuda", generator=g) if mode else None
    valid = (torch.rand(M, device="cuda", generator=g) > 0.3) if mode >= 2 else None
    out = kernels.linear_fp16(a, w, b, act=act, resid=resid, row_valid=valid, resid_mode=mode,
                              out_half=half_out, tile_n=tile)
    wide = kernels.linear_fp16(a, w, b, act=act, resid=resid, row_valid=valid, resid_mode=mode,
                               out_half=half_out, tile_n=256)
    y = _ref(a, w, b, act=bool(act))
    if mode == 1:
        y = resid.double() + y
    elif mode == 2:
        y = resid.double() + torch.where(valid[:, None], y, torch.zeros_like(y))
    elif mode == 3:
        y = torch.where(valid[:, None], resid.double() + y, torch.zeros_like(y))
    scale = _scale(a, w) + (resid.double().abs() if resid is not None else 0)
    tol = 2 ** -10 if half_out else 1e-5
    assert ((out.double() - y).abs() / (scale if not half_out else y.abs() + 1e-2)).max().item() < tol
    assert torch.equal(out, wide)


@pytest.mark.parametrize("tile", [160, 224])
def test_intermediate_tile_widths_pair_operands(kernels, tile):
    """The three-product mode at a width that leaves the last N tile partial:
    its W rows past N come from the lo plane (the map covers both planes) into
    columns that are never stored."""
    g = torch.Generator(device="cuda").manual_seed(62)
    M, N, K = 300, 456, 192
    a = torch.randn(M, K, device="cuda", generator=g)
    w = torch.randn(N, K, device="cuda", generator=g) * K ** -0.5
    b = torch.randn(N, device="cuda", generator=g) * 0.1

    def pair(t):
        hi = t.half()
        return torch.stack([hi, (t - hi.float()).half()]).contiguous()

    out = kernels.linear_fp16(pair(a), pair(w), b, pair_operands=True, tile_n=tile)
    wide = kernels.linear_fp16(pair(a), pair(w), b, pair_operands=True, tile_n=256)
    assert torch.equal(out, wide)
    y = a.double() @ w.double().t() + b.double()
    assert ((out.double() - y).abs() / (a.double().abs() @ w.double().abs().t())).max().item() < 4e-6
