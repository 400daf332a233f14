"""Drop-in replacements for the baseline's submodules (optimized/layers.py upstream).

Parameter and submodule names match BaselineTransformer exactly, so one
state_dict loads into either model with strict=True.

Data flow of one block (T = B*S rows, d = d_model):

    normed [T,d] fp16 --QKV GEMM--> qkv [T,3d] fp16 --attention--> ctx [T,d] fp16
    ctx --out_proj GEMM, epilogue: + bias, padded rows -> 0, + residual x--> x1 [T,d] fp32
    x1 --LayerNorm--> n2 fp16 --ffn_in GEMM, epilogue: + bias, GELU--> h [T,F] fp16
    h --ffn_out GEMM, epilogue: + bias + residual x1, padded rows -> 0--> x2 [T,d] fp32
    x2 --next_norm (fp16 for a next block; fp32 with padded rows -> 0 if final)--> normed

Every residual add and masked_fill of the reference block
(torch_transformer_benchmark.py:234-245) is folded into a GEMM epilogue or a
LayerNorm, so a block is at most 8 kernels and never writes an intermediate
it reads back only to add it. Where the shape allows, out_proj -> norm2 and
ffn_out -> next norm are each one GEMM + LayerNorm kernel (6 kernels), and for
d_model 128/256 the whole MLP (ffn_in, GELU, ffn_out, residual, next norm) is
one kernel that keeps h on chip (5 kernels with the former).
"""

from __future__ import annotations

from typing import Optional, Tuple

import torch
import torch.nn as nn

from .kernels import (_attention_dispatch, _f32_param, _ffn, _ffn_ok, _layernorm, _linear, _linear_bias,
                      _linear_ln, _linear_ln_ok)
from .util import _version_or_none

RESID_ADD, RESID_ADD_MASKSUB, RESID_ADD_MASKALL = 1, 2, 3


def fp16_pair(w: torch.Tensor) -> torch.Tensor:
    """[2, *w.shape] fp16: hi = fp16(w) and lo = fp16(w - hi), both round to
    nearest even (the DOTL_F16X2 layout, planes back to back)."""
    w = w.float()
    hi = w.to(torch.float16)
    lo = (w - hi.float()).to(torch.float16)
    return torch.stack([hi, lo]).contiguous()


class MyLinear(nn.Module):
    """A linear layer whose `weight` [out, in] and `bias` [out] are laid out as
    nn.Linear's, so a baseline state_dict loads with strict=True; the GEMM runs
    on libdotl with the weight narrowed to fp16 once per version."""

    def __init__(self, in_features: int, out_features: int, bias: bool = True) -> None:
        super().__init__()
        self.weight = nn.Parameter(torch.empty(out_features, in_features))
        self.bias = nn.Parameter(torch.empty(out_features)) if bias else None
        self._w16_key = None
        self._w16: Optional[torch.Tensor] = None
        self._wpair_key = None
        self._wpair: Optional[torch.Tensor] = None

    def half_weight(self) -> torch.Tensor:
        """The weight narrowed to fp16 once per version (the GEMM's B operand)."""
        w = self.weight
        key = (w.device, w.dtype, w.data_ptr(), _version_or_none(w))
        if self._w16_key != key:
            self._w16 = w.detach().to(torch.float16).contiguous()
            self._w16_key = key
        return self._w16

    def pair_weight(self) -> torch.Tensor:
        """The weight as an fp16 pair [2, out, in] (hi = fp16(w), lo = fp16(w - hi)),
        the B operand of the three-product GEMM mode, once per version."""
        w = self.weight
        key = (w.device, w.dtype, w.data_ptr(), _version_or_none(w))
        if self._wpair_key != key:
            self._wpair = fp16_pair(w.detach())
            self._wpair_key = key
        return self._wpair

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if self.bias is None:
            raise RuntimeError("MyLinear: the GEMM epilogue always adds a bias; every Linear "
                               "of this model has one")
        return _linear_bias(x, self.weight, self.bias)


class MyLayerNorm(nn.Module):
    """LayerNorm parameters `weight` and `bias` [d_model] as nn.LayerNorm keeps
    them (strict state_dict loading works); normalises on libdotl's kernels."""

    def __init__(self, d_model: int, eps: float = 1e-5) -> None:
        super().__init__()
        self.weight = nn.Parameter(torch.ones(d_model))
        self.bias = nn.Parameter(torch.zeros(d_model))
        self.eps = eps

    def forward(self, x: torch.Tensor, out_half: bool = False) -> torch.Tensor:
        return _layernorm(x.float().contiguous(), self, out_half=out_half)


class MySelfAttention(nn.Module):
    """Multi-head self-attention with q/k/v/out projections named as the
    baseline's (strict state_dict loading works): one fused QKV GEMM, the
    tcgen05 attention kernel, and out_proj with its residual folded in."""

    def __init__(self, d_model: int, num_heads: int) -> None:
        super().__init__()
        self.num_heads = num_heads
        self.head_dim = d_model // num_heads
        self.scale = self.head_dim ** -0.5
        self.q_proj = MyLinear(d_model, d_model)
        self.k_proj = MyLinear(d_model, d_model)
        self.v_proj = MyLinear(d_model, d_model)
        self.out_proj = MyLinear(d_model, d_model)
        self._qkv_key: Optional[Tuple] = None
        self._qkv_weight: Optional[torch.Tensor] = None
        self._qkv_bias: Optional[torch.Tensor] = None
        self._qkv_pair_key: Optional[Tuple] = None
        self._qkv_pair: Optional[torch.Tensor] = None

    def _get_qkv_weight(self) -> Tuple[torch.Tensor, torch.Tensor]:
        """Q, K and V as one fp16 [3d, d] weight and one fp32 [3d] bias
        (layers.py:88-110 upstream: one wide GEMM instead of three narrow
        ones), rebuilt when any of the three weights changes version."""
        w_q, w_k, w_v = self.q_proj.weight, self.k_proj.weight, self.v_proj.weight
        key = (w_q.device, w_q.dtype, _version_or_none(w_q), _version_or_none(w_k),
               _version_or_none(w_v), _version_or_none(self.q_proj.bias),
               _version_or_none(self.k_proj.bias), _version_or_none(self.v_proj.bias),
               w_q.data_ptr(), w_k.data_ptr(), w_v.data_ptr())
        if self._qkv_key != key:
            self._qkv_weight = torch.cat([w_q, w_k, w_v], dim=0).detach().to(torch.float16).contiguous()
            self._qkv_bias = torch.cat([self.q_proj.bias, self.k_proj.bias, self.v_proj.bias],
                                       dim=0).detach().float().contiguous()
            self._qkv_key = key
        return self._qkv_weight, self._qkv_bias

    def _get_qkv_pair(self) -> Tuple[torch.Tensor, torch.Tensor]:
        """The fused QKV weight as an fp16 pair [2, 3d, d] and the fp32 bias."""
        _w, bias = self._get_qkv_weight()
        if self._qkv_pair_key != self._qkv_key:
            w_q, w_k, w_v = self.q_proj.weight, self.k_proj.weight, self.v_proj.weight
            self._qkv_pair = fp16_pair(torch.cat([w_q, w_k, w_v], dim=0).detach())
            self._qkv_pair_key = self._qkv_key
        return self._qkv_pair, bias

    def forward(self, x: torch.Tensor, valid_token_mask: Optional[torch.Tensor] = None,
                causal: bool = False, mask_is_trivial: bool = False,
                residual: Optional[torch.Tensor] = None, norm: Optional["MyLayerNorm"] = None,
                pairs: bool = False):
        """out_proj(attention(x)) with padded rows zeroed, plus `residual` if given.

        x is the block's normalised input [B,S,d] (fp16 or fp32), or with
        `pairs` an fp16 pair [2,B,S,d] for the three-product GEMM mode. With
        `residual`, the add x + attn happens in the out_proj epilogue and the
        fp32 sum is returned; without it, the attention output alone. With
        `norm` as well, returns (sum, norm(sum)) from one GEMM + LayerNorm
        kernel, norm(sum) fp16 (an fp16 pair with `pairs`).
        """
        if pairs:
            batch, seq_len, d_model = x.shape[1:]
            qkv_w, qkv_b = self._get_qkv_pair()
            wo = self.out_proj.pair_weight()
            a = x
        else:
            batch, seq_len, d_model = x.shape
            qkv_w, qkv_b = self._get_qkv_weight()
            wo = self.out_proj.half_weight()
            a = (x if x.dtype == torch.float16 else x.to(torch.float16)).contiguous()
        qkv = _linear(a, qkv_w, qkv_b, out_half=True, pairs=pairs)   # [B, S, 3d] fp16
        q, k, v = (qkv.view(batch, seq_len, 3, self.num_heads, self.head_dim)
                   .permute(2, 0, 3, 1, 4).unbind(0))              # [B, H, S, hd] views
        use_mask = valid_token_mask is not None and not mask_is_trivial
        key_mask = valid_token_mask if use_mask else None
        # [B, S, d] fp16, or its fp16 pair [2, B, S, d]
        context = _attention_dispatch(q, k, v, key_mask, causal, self.scale, out_pair=pairs)
        row_valid = valid_token_mask.reshape(-1) if use_mask else None
        bo = _f32_param(self.out_proj, "bias")
        mode = RESID_ADD_MASKSUB if use_mask else RESID_ADD
        if residual is None:
            # Plain attention output, padded rows zeroed: residual is zero.
            zeros = torch.zeros(batch, seq_len, d_model, device=x.device, dtype=torch.float32)
            return _linear(context, wo, bo, resid=zeros, row_valid=row_valid, resid_mode=mode, pairs=pairs)
        if norm is not None:
            return _linear_ln(context, wo, bo, norm, resid=residual, row_valid=row_valid, resid_mode=mode,
                              pairs=pairs, normed_pair=pairs)
        return _linear(context, wo, bo, resid=residual, row_valid=row_valid, resid_mode=mode, pairs=pairs)


class MyTransformerBlock(nn.Module):
    """One Pre-LN block (norm1, attention, norm2, ffn_in, ffn_out, named as the
    baseline block's submodules) run as 5 to 8 fused kernels."""

    def __init__(self, d_model: int, num_heads: int, ffn_dim: int, causal: bool) -> None:
        super().__init__()
        self.norm1 = MyLayerNorm(d_model)
        self.attention = MySelfAttention(d_model, num_heads)
        self.norm2 = MyLayerNorm(d_model)
        self.ffn_in = MyLinear(d_model, ffn_dim)
        self.ffn_out = MyLinear(ffn_dim, d_model)
        self.causal = causal

    def forward(self, x: torch.Tensor, normed: torch.Tensor, next_norm: "MyLayerNorm",
                valid_token_mask: Optional[torch.Tensor] = None, mask_is_trivial: bool = False,
                next_norm_is_output: bool = False, pairs: bool = False) -> Tuple[torch.Tensor, torch.Tensor]:
        """Returns (residual stream, next_norm applied to it) (layers.py:206-262 upstream).

        `normed` is norm1(x), produced by whoever produced x. `next_norm` is
        the next block's norm1 or the model's final_norm; when it is the final
        norm (next_norm_is_output) its output is fp32 with padded rows zeroed
        (the model's final masked_fill), otherwise fp16 for the next QKV GEMM
        (an fp16 pair [2, B, S, d] with `pairs`, the three-product GEMM mode,
        in which `normed` is one too). After the last block the residual
        stream is only returned when the unfused path ran (None otherwise:
        nothing reads it).
        """
        use_mask = valid_token_mask is not None and not mask_is_trivial
        row_valid = valid_token_mask.reshape(-1) if use_mask else None
        rows, d = x.numel() // x.shape[-1], x.shape[-1]
        # out_proj + residual + norm2, and ffn_out + residual + next norm, each
        # as one GEMM whose epilogue also normalises (a thread-block cluster
        # shares each row's statistics) on the shapes where that is faster.
        fused = _linear_ln_ok(rows, d)
        if fused:
            x1, n2 = self.attention(normed, valid_token_mask, self.causal, mask_is_trivial, residual=x,
                                    norm=self.norm2, pairs=pairs)
        else:
            x1 = self.attention(normed, valid_token_mask, self.causal, mask_is_trivial, residual=x, pairs=pairs)
            n2 = _layernorm(x1, self.norm2, out_half=True, out_pair=pairs)
        # x1 + ffn_out(h); padded rows of the whole sum zeroed (the block's
        # trailing masked_fill), before the next LayerNorm reads it.
        mode = RESID_ADD_MASKALL if use_mask else RESID_ADD
        last = next_norm_is_output
        if not pairs and _ffn_ok(rows, d, self.ffn_in.weight.shape[0]):
            # ffn_in + GELU + ffn_out + residual + next norm in one kernel
            x2, out = _ffn(n2, self.ffn_in, self.ffn_out, next_norm, x1, row_valid, mode,
                           store_x=not last, normed_half=not last,
                           normed_row_valid=row_valid if last else None)
            return (x2.view(x.shape) if x2 is not None else None), out
        w1 = self.ffn_in.pair_weight() if pairs else self.ffn_in.half_weight()
        w2 = self.ffn_out.pair_weight() if pairs else self.ffn_out.half_weight()
        b2 = _f32_param(self.ffn_out, "bias")
        h = _linear(n2, w1, _f32_param(self.ffn_in, "bias"), act=1, out_half=True, pairs=pairs, out_pair=pairs)
        if fused:
            # after the last block x2 itself is not needed, only its final norm
            return _linear_ln(h, w2, b2, next_norm, resid=x1, row_valid=row_valid, resid_mode=mode,
                              store_x=not last, normed_half=not last,
                              normed_row_valid=row_valid if last else None, pairs=pairs,
                              normed_pair=pairs and not last)
        x2 = _linear(h, w2, b2, resid=x1, row_valid=row_valid, resid_mode=mode, pairs=pairs)
        if last:
            return x2, _layernorm(x2, next_norm, out_half=False, row_valid=row_valid)
        return x2, _layernorm(x2, next_norm, out_half=True, out_pair=pairs)
