"""dotl_ffn, the MLP in one kernel (gpu), against float64 and against the
unfused kernels (linear GELU -> linear + residual -> LayerNorm).

The float64 reference rounds the hidden to fp16 where the kernel does (the
GEMM2 operand); the GELU is the kernel's erf approximation against the exact
one (<= 1e-6 relative), so a hidden value near an fp16 rounding boundary may
round the other way: bounds are relative to the row's scale."""

import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu

RESID_NONE, RESID_ADD, RESID_ADD_MASKSUB, RESID_ADD_MASKALL = 0, 1, 2, 3


def _case(M, D, Fd, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    a = torch.randn(M, D, device="cuda", generator=g).half()
    w1 = (torch.randn(Fd, D, device="cuda", generator=g) * D ** -0.5).half()
    b1 = torch.randn(Fd, device="cuda", generator=g) * 0.1
    w2 = (torch.randn(D, Fd, device="cuda", generator=g) * Fd ** -0.5).half()
    b2 = torch.randn(D, device="cuda", generator=g) * 0.1
    resid = torch.randn(M, D, device="cuda", generator=g)
    valid = torch.rand(M, device="cuda", generator=g) > 0.25
    nvalid = torch.rand(M, device="cuda", generator=g) > 0.25
    lw = torch.randn(D, device="cuda", generator=g) * 0.2 + 1.0
    lb = torch.randn(D, device="cuda", generator=g) * 0.1
    return a, w1, b1, w2, b2, resid, valid, nvalid, lw, lb


def _ref(a, w1, b1, w2, b2, resid, valid, mode, lw, lb, nvalid):
    h = F.gelu(a.double() @ w1.double().t() + b1.double(), approximate="none").half().double()
    proj = h @ w2.double().t() + b2.double()
    if mode == RESID_NONE:
        x = proj
    elif mode == RESID_ADD:
        x = resid.double() + proj
    elif mode == RESID_ADD_MASKSUB:
        x = resid.double() + proj * valid[:, None]
    else:
        x = (resid.double() + proj) * valid[:, None]
    y = F.layer_norm(x, (x.shape[1],), lw.double(), lb.double(), 1e-5)
    if nvalid is not None:
        y = y * nvalid[:, None]
    scale = h.abs() @ w2.double().abs().t() + resid.double().abs() + 1.0
    return x, y, scale


@pytest.mark.parametrize("M,D,Fd", [(128, 128, 128), (300, 256, 1024), (1000, 128, 384), (129, 256, 256),
                                    (5000, 256, 1024), (77, 128, 128)])
@pytest.mark.parametrize("mode", [RESID_NONE, RESID_ADD, RESID_ADD_MASKSUB, RESID_ADD_MASKALL])
def test_ffn_against_float64(kernels, M, D, Fd, mode):
    a, w1, b1, w2, b2, resid, valid, nvalid, lw, lb = _case(M, D, Fd, M + D + Fd + mode)
    x_out = torch.full((M, D), float("nan"), device="cuda")
    normed = kernels.ffn(a, w1, b1, w2, b2, lw, lb, 1e-5, resid=resid if mode else None,
                         row_valid=valid if mode in (2, 3) else None, resid_mode=mode, x_out=x_out,
                         normed_row_valid=nvalid)
    x, y, scale = _ref(a, w1, b1, w2, b2, resid, valid, mode, lw, lb, nvalid)
    assert ((x_out.double() - x).abs() / scale).max().item() < 1e-4
    # LN output: x_new error / row std, amplified by |gamma|
    std = x.std(dim=1, keepdim=True) + 1e-3
    err = (normed.double() - y).abs() * std / (scale * 1.5)
    assert err.max().item() < 1e-4
    assert torch.all(normed[~nvalid] == 0)


@pytest.mark.parametrize("D,Fd", [(128, 128), (256, 1024)])
def test_ffn_matches_unfused_kernels(kernels, D, Fd):
    """Same operands through linear_fp16(GELU, fp16 out) -> linear_fp16(residual)
    -> layernorm_rows: the kernels round at the same points, so they agree to
    accumulation order."""
    M = 4096
    a, w1, b1, w2, b2, resid, valid, nvalid, lw, lb = _case(M, D, Fd, 9)
    x_out = torch.empty(M, D, device="cuda")
    normed = kernels.ffn(a, w1, b1, w2, b2, lw, lb, 1e-5, resid=resid, row_valid=valid,
                         resid_mode=RESID_ADD_MASKALL, x_out=x_out, normed_half=True)
    h = kernels.linear_fp16(a, w1, b1, act=1, out_half=True)
    x2 = kernels.linear_fp16(h, w2, b2, resid=resid, row_valid=valid, resid_mode=RESID_ADD_MASKALL)
    n2 = kernels.layernorm_rows(x2, lw, lb, 1e-5, out_half=True)
    assert (x_out - x2).abs().max().item() < 1e-4
    assert torch.all((normed.float() - n2.float()).abs() <= 2 ** -9 * (n2.float().abs() + 0.25))


def test_ffn_repeatable_and_rows_independent(kernels):
    a, w1, b1, w2, b2, resid, valid, nvalid, lw, lb = _case(3000, 256, 512, 5)
    n1 = kernels.ffn(a, w1, b1, w2, b2, lw, lb, 1e-5, resid=resid, resid_mode=RESID_ADD)
    n2 = kernels.ffn(a, w1, b1, w2, b2, lw, lb, 1e-5, resid=resid, resid_mode=RESID_ADD)
    assert torch.equal(n1, n2)
    part = kernels.ffn(a[1000:1300].contiguous(), w1, b1, w2, b2, lw, lb, 1e-5,
                       resid=resid[1000:1300].contiguous(), resid_mode=RESID_ADD)
    assert torch.equal(part, n1[1000:1300])


def test_ffn_rejects(kernels):
    a, w1, b1, w2, b2, resid, valid, nvalid, lw, lb = _case(64, 128, 128, 1)
    with pytest.raises(RuntimeError, match="128 or 256"):
        kernels.ffn(torch.zeros(64, 64, device="cuda").half(), w1[:, :64].contiguous(), b1,
                    w2[:64].contiguous(), b2[:64].contiguous(), lw[:64].contiguous(), lb[:64].contiguous(), 1e-5)
    with pytest.raises(RuntimeError, match="multiple of 128"):
        kernels.ffn(a, w1[:96].contiguous(), b1[:96].contiguous(), w2[:, :96].contiguous(), b2, lw, lb, 1e-5)
    with pytest.raises(RuntimeError, match="needs row_valid"):
        kernels.ffn(a, w1, b1, w2, b2, lw, lb, 1e-5, resid=resid, resid_mode=RESID_ADD_MASKALL)


@pytest.mark.parametrize("D,Fd", [(256, 1024), (64, 256)])
def test_reference_fused_ffn_block(kernels, D, Fd):
    """The reference-named entry point: [x2, LN2(x2)] for x + attn_out -> LN1 ->
    Linear+GELU -> Linear -> + residual -> LN2 (ffn_block.cuh:270-311 upstream),
    fp32 weights in; d_model 256 takes the one-kernel MLP, 64 the GEMM path."""
    g = torch.Generator(device="cuda").manual_seed(D)
    M = 4096
    x = torch.randn(M, D, device="cuda", generator=g)
    attn = torch.randn(M, D, device="cuda", generator=g) * 0.5
    n1w, n1b = torch.ones(D, device="cuda"), torch.zeros(D, device="cuda")
    n2w = torch.randn(D, device="cuda", generator=g) * 0.1 + 1.0
    n2b = torch.randn(D, device="cuda", generator=g) * 0.1
    w1 = torch.randn(Fd, D, device="cuda", generator=g) * D ** -0.5
    b1 = torch.randn(Fd, device="cuda", generator=g) * 0.02
    w2 = torch.randn(D, Fd, device="cuda", generator=g) * Fd ** -0.5
    b2 = torch.randn(D, device="cuda", generator=g) * 0.02
    x2, n2 = kernels.fused_ffn_block(x, attn, n1w, n1b, w1, b1, w2, b2, n2w, n2b, 1e-5)
    x1 = (x + attn).double()
    a = F.layer_norm(x1, (D,), eps=1e-5).half().double()
    h = F.gelu(a @ w1.half().double().t() + b1.double(), approximate="none").half().double()
    rx2 = x1 + h @ w2.half().double().t() + b2.double()
    rn2 = F.layer_norm(rx2, (D,), n2w.double(), n2b.double(), 1e-5)
    assert (x2.double() - rx2).abs().max().item() < 1e-3
    assert (n2.double() - rn2).abs().max().item() < 2e-3
