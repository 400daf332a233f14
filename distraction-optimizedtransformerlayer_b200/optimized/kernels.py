"""Dispatch into libdotl (optimized/kernels.py upstream).

The boundary between torch and the sm_100a kernels: every helper here calls
the library through `kernel_ext.get_kernels()` and raises when it is missing.
There is no torch fallback for any op (the reference fell back to cuBLAS and
ATen for the GEMMs and LayerNorm; the B200 build refuses instead).
"""

from __future__ import annotations

from typing import Optional, Tuple

import torch

from . import config


def _custom_kernels():
    """The kernel module; raises if the library cannot be loaded."""
    import kernel_ext

    kernels = kernel_ext.get_kernels()
    if kernels is None:
        raise RuntimeError(
            "libdotl (the sm_100a kernel library) failed to load, and there is no fallback: "
            "this project implements every op of the layer itself. Build it with "
            f"kernel_ext.build(). Cause: {kernel_ext.load_error()}")
    return kernels


def _f32_param(module, name: str) -> torch.Tensor:
    """A parameter as a contiguous fp32 tensor, cached per parameter version
    (parameters may have been moved to fp16/bf16 by model.to(dtype))."""
    p = getattr(module, name)
    if p.dtype == torch.float32 and p.is_contiguous():
        return p
    cache = module.__dict__.setdefault("_f32_cache", {})
    key = (name, p.data_ptr(), p.device, p.dtype, getattr(p, "_version", None))
    hit = cache.get(name)
    if hit is not None and hit[0] == key:
        return hit[1]
    t = p.detach().float().contiguous()
    cache[name] = (key, t)
    return t


def _layernorm(x: torch.Tensor, norm, out_half: bool = False,
               row_valid: Optional[torch.Tensor] = None, out_pair: bool = False) -> torch.Tensor:
    """LayerNorm(x) * w + b over the last dim of fp32 x; padded rows -> 0 if
    row_valid; out_pair: an fp16 pair [2, *x.shape] for three-product GEMMs."""
    k = _custom_kernels()
    return k.layernorm_rows(x, _f32_param(norm, "weight"), _f32_param(norm, "bias"), norm.eps,
                            out_half=out_half, row_valid=row_valid, out_pair=out_pair)


def _add_layernorm(x: torch.Tensor, sub: torch.Tensor, norm,
                   normed_half: bool = False) -> Tuple[torch.Tensor, torch.Tensor]:
    """(x + sub, norm(x + sub)) in one kernel."""
    k = _custom_kernels()
    return k.layernorm_rows(x, _f32_param(norm, "weight"), _f32_param(norm, "bias"), norm.eps,
                            sub=sub, out_half=normed_half)


def _linear(a16: torch.Tensor, w16: torch.Tensor, bias32: torch.Tensor, act: int = 0,
            resid: Optional[torch.Tensor] = None, row_valid: Optional[torch.Tensor] = None,
            resid_mode: int = 0, out_half: bool = False, pairs: bool = False,
            out_pair: bool = False) -> torch.Tensor:
    """epilogue(a16 @ w16^T + bias) on the tcgen05 GEMM (pairs: a16 and w16
    are fp16 pairs, the three-product mode; out_pair: an fp16 pair out)."""
    k = _custom_kernels()
    return k.linear_fp16(a16, w16, bias32, act=act, resid=resid, row_valid=row_valid,
                         resid_mode=resid_mode, out_half=out_half, pair_operands=pairs, out_pair=out_pair)


def _linear_ln_ok(rows: int, n: int) -> bool:
    """Whether the layer takes the GEMM + LayerNorm kernel for rows x n outputs
    (where it beats the GEMM and LayerNorm kernels run one after the other)."""
    return _custom_kernels().linear_ln_preferred(rows, n)


def _ffn_ok(rows: int, d: int, f: int) -> bool:
    """Whether the layer runs its MLP (ffn_in, GELU, ffn_out, residual, next
    LayerNorm) as the one dotl_ffn kernel."""
    return _custom_kernels().ffn_preferred(rows, d, f)


def _ffn(n2: torch.Tensor, ffn_in, ffn_out, norm, resid: torch.Tensor,
         row_valid: Optional[torch.Tensor], resid_mode: int, store_x: bool, normed_half: bool,
         normed_row_valid: Optional[torch.Tensor] = None):
    """(x_new, norm(x_new)) with x_new = resid-mode(GELU(n2 W1^T + b1) W2^T + b2),
    the hidden never leaving the chip (x_new None when store_x is False)."""
    k = _custom_kernels()
    x_out = torch.empty_like(resid) if store_x else None
    normed = k.ffn(n2, ffn_in.half_weight(), _f32_param(ffn_in, "bias"), ffn_out.half_weight(),
                   _f32_param(ffn_out, "bias"), _f32_param(norm, "weight"), _f32_param(norm, "bias"),
                   norm.eps, resid=resid, row_valid=row_valid, resid_mode=resid_mode, x_out=x_out,
                   normed_half=normed_half, normed_row_valid=normed_row_valid)
    return x_out, normed


def _linear_ln(a16: torch.Tensor, w16: torch.Tensor, bias32: torch.Tensor, norm,
               resid: Optional[torch.Tensor] = None, row_valid: Optional[torch.Tensor] = None,
               resid_mode: int = 0, store_x: bool = True, normed_half: bool = True,
               normed_row_valid: Optional[torch.Tensor] = None, pairs: bool = False,
               normed_pair: bool = False):
    """(x_new, norm(x_new)) from one kernel: x_new = epilogue(a16 @ w16^T + bias)
    as _linear computes it (fp32; None when store_x is False), then the
    LayerNorm over its rows (fp16 or fp32, padded rows 0 with normed_row_valid)."""
    k = _custom_kernels()
    return k.linear_ln(a16, w16, bias32, _f32_param(norm, "weight"), _f32_param(norm, "bias"), norm.eps,
                       resid=resid, row_valid=row_valid, resid_mode=resid_mode, store_x=store_x,
                       normed_half=normed_half, normed_row_valid=normed_row_valid, pair_operands=pairs,
                       normed_pair=normed_pair)


def _linear_bias(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor,
                 out_half: bool = False) -> torch.Tensor:
    """x @ weight^T + bias with the reference signature (fp32 weight)."""
    return _custom_kernels().linear_bias(x, weight, bias, -1, -1, out_half)


def _linear_gelu(x: torch.Tensor, lin) -> torch.Tensor:
    """GELU(lin(x)) with the reference signature."""
    return _custom_kernels().linear_gelu(x, lin.weight, lin.bias, -1, -1)


def _attention_dispatch(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                        key_mask: Optional[torch.Tensor], is_causal: bool, scale: float,
                        out: Optional[torch.Tensor] = None, out_pair: bool = False) -> torch.Tensor:
    """Attention on the tcgen05 kernel; q/k/v fp16 [B,H,S,hd] views; returns [B,S,H*hd] fp16.

    key_mask: bool [B,S], True = may attend (the [B,1,1,S] mask upstream).
    """
    config.validate()
    kernels = _custom_kernels()
    return kernels.attention_packed(q, k, v, is_causal, scale, key_mask=key_mask,
                                    out_layout=config._OUT_LAYOUT_BSHD, out=out, out_pair=out_pair)
