"""Tensor-level entry points over libdotl's C ABI (include/dotl.h), via ctypes.

This module is what `kernel_ext.get_kernels()` returns. Its public functions
have the names, arguments and error behaviour of the reference's pybind module
`transformer_kernels` (csrc/fused_attention.cu:118-376 upstream):

    smoke_test_identity, fused_layernorm, fused_add_layernorm, linear_bias,
    linear_gelu, fused_attention_forward, fused_ffn_block, and the process-wide
    knob setters/getters scripts call (accepted, recorded, no effect).

Torch is only the allocator and the stream source here: outputs are torch
tensors, their data pointers go to the C ABI together with the current
stream, and every launch is enqueued on that stream. A failed call raises
RuntimeError with the library's message. There is no fallback to any other
implementation: the functions either run libdotl's kernels or raise.

The model path in `optimized/` uses the lower-level helpers at the bottom
(`linear_fp16`, `attention_packed`, `layernorm_rows`), which take weights
already narrowed to fp16 and fuse the residual adds and padded-row masks into
the GEMM epilogues.
"""

from __future__ import annotations

import ctypes
import weakref
from typing import Dict, List, Optional, Tuple

import torch

_lib: Optional[ctypes.CDLL] = None

F32, F16, F16X2 = 0, 1, 2
RESID_NONE, RESID_ADD, RESID_ADD_MASKSUB, RESID_ADD_MASKALL, MASK_ROWS = 0, 1, 2, 3, 4
MASK_NONE, MASK_KEY, MASK_FULL = 0, 1, 2

_vp, _i64, _i32, _f32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_float
_P64 = ctypes.POINTER(ctypes.c_int64)

_SIGNATURES = {
    "dotl_abi_version": ([], _i32),
    "dotl_last_error": ([], ctypes.c_char_p),
    "dotl_num_sms": ([ctypes.POINTER(ctypes.c_int)], _i32),
    "dotl_device_error": ([_i32, ctypes.POINTER(ctypes.c_uint)], _i32),
    "dotl_identity_f32": ([_vp, _vp, _i64, _vp], _i32),
    "dotl_cast_f32_f16": ([_vp, _vp, _i64, _vp], _i32),
    "dotl_cast_f16_f32": ([_vp, _vp, _i64, _vp], _i32),
    "dotl_layernorm": ([_vp, _vp, _vp, _vp, _vp, _vp, _i32, _vp, _i64, _i64, _f32, _vp], _i32),
    "dotl_linear": ([_vp, _i64, _i64, _i64, _vp, _i64, _i64, _vp, _i32, _vp, _i64, _vp, _i32,
                     _vp, _i32, _i64, _i32, _i32, _vp], _i32),
    "dotl_linear_ln": ([_vp, _i64, _i64, _i64, _vp, _i64, _i64, _vp, _vp, _i64, _vp, _i32, _vp, _i64,
                        _vp, _vp, _f32, _vp, _i32, _i64, _vp, _i32, _i32, _vp], _i32),
    "dotl_attention": ([_vp, _vp, _vp, _i32, _i32, _i32, _i32, _P64, _P64, _P64, _vp, _i32, _P64,
                        _i32, _f32, _vp, _i32, _i32, _vp, _i64, _vp], _i32),
    "dotl_attention_workspace_bytes": ([_i32, _i32, _i32, _i32, _i32, _P64], _i32),
    "dotl_attention_static_scratch": ([_vp, _vp, _vp, _i32, _i32, _i32, _i32, _P64, _P64, _P64, _vp, _i32, _P64,
                                       _i32, _f32, _vp, _i32, _i32, _vp], _i32),
    "dotl_ffn": ([_vp, _i64, _i64, _i64, _vp, _i64, _i64, _vp, _vp, _i64, _vp, _vp, _i64, _vp, _i32,
                  _vp, _i64, _vp, _vp, _f32, _vp, _i32, _i64, _vp, _vp], _i32),
    "dotl_peer_alloc": ([_i64, ctypes.POINTER(_vp)], _i32),
    "dotl_peer_free": ([_vp], _i32),
    "dotl_ipc_handle": ([_vp, _vp], _i32),
    "dotl_ipc_open": ([_vp, ctypes.POINTER(_vp)], _i32),
    "dotl_ipc_close": ([_vp], _i32),
    "dotl_peer_blocks": ([ctypes.POINTER(ctypes.c_int)], _i32),
    "dotl_peer_signal_bytes": ([_i32, _P64], _i32),
    "dotl_allreduce_ln": ([_i32, _i32, _vp, _vp, _vp, _vp, _i32, _i32, _i32, _vp, _vp, _vp, _vp, _vp, _f32, _vp,
                           _i64, _i64, _i32, _i64, _vp, _i32, _vp], _i32),
    "dotl_linear_peer": ([_vp, _i64, _i64, _i64, _vp, _i64, _i64, _vp, _i32, _vp, _i64, _i64, _vp], _i32),
}

IPC_HANDLE_BYTES = 64
ABI_VERSION = 2


def load(path: str) -> ctypes.CDLL:
    """Open libdotl and declare its signatures. Idempotent."""
    global _lib
    if _lib is not None:
        return _lib
    lib = ctypes.CDLL(path)
    for name, (argtypes, restype) in _SIGNATURES.items():
        fn = getattr(lib, name)
        fn.argtypes = argtypes
        fn.restype = restype
    if lib.dotl_abi_version() != ABI_VERSION:
        raise RuntimeError(f"libdotl ABI version {lib.dotl_abi_version()} is not {ABI_VERSION}")
    _lib = lib
    return lib


def lib() -> ctypes.CDLL:
    if _lib is None:
        raise RuntimeError("libdotl is not loaded; call kernel_ext.get_kernels() first")
    return _lib


def _check(rc: int) -> None:
    if rc != 0:
        raise RuntimeError(lib().dotl_last_error().decode(errors="replace"))


def _stream(device: torch.device) -> int:
    # The raw handle of torch's current stream on that device (the one a
    # torch.cuda.stream() context or a graph capture has made current),
    # without building a torch.cuda.Stream object on every kernel call.
    if device.type != "cuda":
        raise ValueError(f"libdotl kernels take CUDA tensors, got a tensor on {device}")
    index = device.index
    if index is None:
        index = torch.cuda.current_device()
    return torch._C._cuda_getCurrentRawStream(index)


def _ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


def _i64arr(vals) -> ctypes.Array:
    return (ctypes.c_int64 * len(vals))(*[int(v) for v in vals])


def device_error(clear: bool = True) -> int:
    """The sticky device error word (nonzero = a kernel gave up a wait)."""
    word = ctypes.c_uint(0)
    _check(lib().dotl_device_error(1 if clear else 0, ctypes.byref(word)))
    return int(word.value)


def num_sms() -> int:
    n = ctypes.c_int(0)
    _check(lib().dotl_num_sms(ctypes.byref(n)))
    return int(n.value)


# --------------------------------------------------------------- weights ---

class _HalfWeightCache:
    """fp16 copies of fp32 weights, keyed on the weight object and its version.

    The reference's GEMM narrows W to fp16 while staging every tile
    (linear_gelu.cuh:108-128); the tensor cores here read fp16 operands from
    TMA, so the narrowing happens once per weight version instead. Keyed on a
    weakref plus the version counter, like the reference's _mask_is_trivial
    cache (optimized/model.py:68-93): an address alone could be recycled.
    """

    def __init__(self) -> None:
        self._entries: Dict[int, Tuple[weakref.ReferenceType, object, torch.Tensor]] = {}

    def get(self, w: torch.Tensor) -> torch.Tensor:
        if w.dtype == torch.float16 and w.is_contiguous():
            return w
        try:
            version = w._version
        except RuntimeError:
            version = None
        key = id(w)
        hit = self._entries.get(key)
        if hit is not None and hit[0]() is w and hit[1] == version and version is not None:
            return hit[2]
        half = w.detach().to(torch.float16).contiguous()
        self._entries = {k: v for k, v in self._entries.items() if v[0]() is not None}
        self._entries[key] = (weakref.ref(w), version, half)
        return half


_half_weights = _HalfWeightCache()


# ------------------------------------------------------- low-level helpers ---

def to_f16(x: torch.Tensor) -> torch.Tensor:
    """fp32 -> fp16 with this library's cast kernel (RNE), contiguous."""
    x = x.contiguous()
    if x.dtype == torch.float16:
        return x
    if x.dtype != torch.float32:
        x = x.float()
    out = torch.empty(x.shape, dtype=torch.float16, device=x.device)
    _check(lib().dotl_cast_f32_f16(x.data_ptr(), out.data_ptr(), x.numel(), _stream(x.device)))
    return out


def to_f32(x: torch.Tensor) -> torch.Tensor:
    x = x.contiguous()
    if x.dtype == torch.float32:
        return x
    out = torch.empty(x.shape, dtype=torch.float32, device=x.device)
    _check(lib().dotl_cast_f16_f32(x.data_ptr(), out.data_ptr(), x.numel(), _stream(x.device)))
    return out


def _pair_planes(t: torch.Tensor) -> Tuple[int, int]:
    """(rows, ld) of one plane of an fp16 pair: a contiguous fp16 tensor
    [2, ..., cols] whose lo plane starts rows * cols elements after its hi
    plane (the C ABI's DOTL_F16X2 layout)."""
    if t.dim() < 3 or t.shape[0] != 2 or t.dtype != torch.float16 or not t.is_contiguous():
        raise RuntimeError("an fp16 pair is a contiguous fp16 tensor [2, ..., cols] (hi plane, lo plane)")
    cols = t.shape[-1]
    return (t[0].numel() // cols if cols else 0), cols


def layernorm_rows(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor, eps: float,
                   sub: Optional[torch.Tensor] = None, out_half: bool = False,
                   row_valid: Optional[torch.Tensor] = None,
                   x_new: Optional[torch.Tensor] = None,
                   out: Optional[torch.Tensor] = None, out_pair: bool = False):
    """(x + sub, LN(x + sub)) or LN(x) over the last dim of an fp32 tensor.

    row_valid: optional bool/uint8 tensor with one entry per row; rows with 0
    get a zero LN output (the final masked_fill). out_pair: the output is an
    fp16 pair [2, *x.shape] (hi, lo) for the three-product GEMM mode.
    """
    D = x.shape[-1]
    rows = x.numel() // D if D else 0
    if out is None:
        if out_pair:
            out = torch.empty((2, *x.shape), dtype=torch.float16, device=x.device)
        else:
            out = torch.empty(x.shape, dtype=torch.float16 if out_half else torch.float32, device=x.device)
    if out_pair and (out.shape[0] != 2 or not out.is_contiguous()):
        raise RuntimeError("layernorm_rows: a pair output must be a contiguous [2, *x.shape] fp16 tensor")
    if sub is not None and x_new is None:
        x_new = torch.empty_like(x)
    dtype = F16X2 if out_pair else (F16 if out.dtype == torch.float16 else F32)
    rc = lib().dotl_layernorm(
        x.data_ptr(), _ptr(sub), weight.data_ptr(), bias.data_ptr(), _ptr(x_new), out.data_ptr(),
        dtype, _ptr(row_valid), rows, D, float(eps), _stream(x.device))
    _check(rc)
    return (x_new, out) if sub is not None else out


def linear_fp16(a16: torch.Tensor, w16: torch.Tensor, bias: torch.Tensor, act: int = 0,
                resid: Optional[torch.Tensor] = None, row_valid: Optional[torch.Tensor] = None,
                resid_mode: int = RESID_NONE, out_half: bool = False,
                out: Optional[torch.Tensor] = None, tile_n: int = 0, pair_operands: bool = False,
                out_pair: bool = False) -> torch.Tensor:
    """epilogue(a16 @ w16^T + bias) on the tcgen05 GEMM, a16 [..., K] fp16.

    pair_operands: a16 is an fp16 pair [2, ..., K] and w16 one [2, N, K] (the
    three-product mode). out_pair: fp16 pair output [2, ..., N]."""
    K = a16.shape[-1]
    if pair_operands:
        M, lda = _pair_planes(a16)
        _pair_planes(w16)
        lead = a16.shape[1:-1]
        N, ldw = w16.shape[1], w16.stride(-2)
    else:
        M, lda = a16.numel() // K, (a16.stride(-2) if a16.dim() >= 2 else K)
        lead = a16.shape[:-1]
        N, ldw = w16.shape[0], w16.stride(0)
    if out is None:
        if out_pair:
            out = torch.empty((2, *lead, N), dtype=torch.float16, device=a16.device)
        else:
            out = torch.empty((*lead, N), dtype=torch.float16 if out_half else torch.float32, device=a16.device)
    if out_pair:
        _, ldo = _pair_planes(out)
        odt = F16X2
    else:
        ldo = out.stride(-2) if out.dim() >= 2 else N
        odt = F16 if out.dtype == torch.float16 else F32
    rc = lib().dotl_linear(
        a16.data_ptr(), M, K, lda, w16.data_ptr(), N, ldw,
        bias.data_ptr(), act, _ptr(resid), resid.stride(-2) if resid is not None and resid.dim() >= 2 else N,
        _ptr(row_valid), resid_mode, out.data_ptr(), odt, ldo, tile_n, F16X2 if pair_operands else F16,
        _stream(a16.device))
    _check(rc)
    return out


def ffn_supported(d: int, f: int) -> bool:
    """Whether dotl_ffn covers d_model d and ffn_dim f."""
    return d in (128, 256) and f > 0 and f % 128 == 0


def ffn_preferred(rows: int, d: int, f: int) -> bool:
    """The layer's rule for the one-kernel MLP: covered, and at least 32 row
    blocks of 128 (below that one block per SM runs its whole F serially and
    the two GEMMs' wider grids win: 36 vs 24 us at 256 x 256 x 1024; from 64
    blocks on it wins, 15 vs 20 us at 8192 x 128 x 128, 412 vs 504 us at
    262144 x 256 x 1024)."""
    return ffn_supported(d, f) and (rows + 127) // 128 >= 32


def ffn(a16: torch.Tensor, w1_16: torch.Tensor, b1: torch.Tensor, w2_16: torch.Tensor, b2: torch.Tensor,
        ln_w: torch.Tensor, ln_b: torch.Tensor, eps: float, resid: Optional[torch.Tensor] = None,
        row_valid: Optional[torch.Tensor] = None, resid_mode: int = RESID_NONE,
        x_out: Optional[torch.Tensor] = None, normed_half: bool = False,
        normed_row_valid: Optional[torch.Tensor] = None, normed: Optional[torch.Tensor] = None) -> torch.Tensor:
    """The MLP in one kernel: normed = LN(resid-mode(GELU(a w1^T + b1) w2^T + b2)),
    x_new into x_out when given. a16 [..., D] fp16; returns normed (a16's shape)."""
    D = a16.shape[-1]
    M = a16.numel() // D
    F = w1_16.shape[0]
    if normed is None:
        normed = torch.empty(a16.shape, dtype=torch.float16 if normed_half else torch.float32, device=a16.device)
    rc = lib().dotl_ffn(
        a16.data_ptr(), M, D, a16.stride(-2) if a16.dim() >= 2 else D, w1_16.data_ptr(), F, w1_16.stride(0),
        b1.data_ptr(), w2_16.data_ptr(), w2_16.stride(0), b2.data_ptr(), _ptr(resid),
        resid.stride(-2) if resid is not None and resid.dim() >= 2 else D, _ptr(row_valid), resid_mode,
        _ptr(x_out), x_out.stride(-2) if x_out is not None and x_out.dim() >= 2 else D, ln_w.data_ptr(),
        ln_b.data_ptr(), float(eps), normed.data_ptr(), F16 if normed.dtype == torch.float16 else F32,
        normed.stride(-2) if normed.dim() >= 2 else D, _ptr(normed_row_valid), _stream(a16.device))
    _check(rc)
    return normed


def linear_ln_supported(N: int) -> bool:
    """Whether dotl_linear_ln covers a row of N columns (64, 128 or 256 times
    a cluster of at most 8 CTAs)."""
    return any(N % bn == 0 and N // bn <= 8 for bn in (64, 128, 256))


_SMS: Optional[int] = None


def linear_ln_preferred(M: int, N: int) -> bool:
    """Whether the layer should take dotl_linear_ln over the GEMM + LayerNorm
    kernel pair for an [M, N] output. The fused kernel saves the LayerNorm's
    HBM round trip but holds each row block in a cluster of N / tile CTAs that
    must exchange statistics; measured on B200 it wins when a 256-wide tile
    covers the row with at most 4 CTAs per cluster and the row blocks fill at
    least two waves of the SMs, and loses on small or 8-wide-cluster shapes."""
    global _SMS
    if N % 256 != 0 or N // 256 > 4:
        return False
    if _SMS is None:
        _SMS = num_sms()
    return ((M + 127) // 128) * (N // 256) >= 2 * _SMS


def linear_ln(a16: torch.Tensor, w16: torch.Tensor, bias: torch.Tensor, ln_w: torch.Tensor,
              ln_b: torch.Tensor, eps: float, resid: Optional[torch.Tensor] = None,
              row_valid: Optional[torch.Tensor] = None, resid_mode: int = RESID_NONE,
              store_x: bool = True, normed_half: bool = True,
              normed_row_valid: Optional[torch.Tensor] = None, out: Optional[torch.Tensor] = None,
              normed: Optional[torch.Tensor] = None, tile_n: int = 0, pair_operands: bool = False,
              normed_pair: bool = False):
    """(x_new, normed): x_new = resid epilogue(a16 @ w16^T + bias) in fp32 (None
    when store_x is False) and normed = LayerNorm(x_new) * ln_w + ln_b, from one
    kernel whose CTA cluster shares each row's statistics. pair_operands /
    normed_pair: fp16 pairs as linear_fp16 takes and gives them."""
    K = a16.shape[-1]
    if pair_operands:
        M, lda = _pair_planes(a16)
        _pair_planes(w16)
        lead = a16.shape[1:-1]
        N, ldw = w16.shape[1], w16.stride(-2)
    else:
        M, lda = a16.numel() // K, (a16.stride(-2) if a16.dim() >= 2 else K)
        lead = a16.shape[:-1]
        N, ldw = w16.shape[0], w16.stride(0)
    if store_x and out is None:
        out = torch.empty((*lead, N), dtype=torch.float32, device=a16.device)
    if normed is None:
        if normed_pair:
            normed = torch.empty((2, *lead, N), dtype=torch.float16, device=a16.device)
        else:
            normed = torch.empty((*lead, N), dtype=torch.float16 if normed_half else torch.float32,
                                 device=a16.device)
    if normed_pair:
        _, ldn = _pair_planes(normed)
        ndt = F16X2
    else:
        ldn = normed.stride(-2) if normed.dim() >= 2 else N
        ndt = F16 if normed.dtype == torch.float16 else F32
    rc = lib().dotl_linear_ln(
        a16.data_ptr(), M, K, lda, w16.data_ptr(), N, ldw,
        bias.data_ptr(), _ptr(resid), resid.stride(-2) if resid is not None and resid.dim() >= 2 else N,
        _ptr(row_valid), resid_mode, out.data_ptr() if store_x else None,
        out.stride(-2) if store_x and out.dim() >= 2 else N, ln_w.data_ptr(), ln_b.data_ptr(), float(eps),
        normed.data_ptr(), ndt, ldn, _ptr(normed_row_valid), tile_n, F16X2 if pair_operands else F16,
        _stream(a16.device))
    _check(rc)
    return (out if store_x else None), normed


def attention_packed(q16: torch.Tensor, k16: torch.Tensor, v16: torch.Tensor, causal: bool,
                     scale: float, key_mask: Optional[torch.Tensor] = None,
                     full_mask: Optional[torch.Tensor] = None, out_layout: int = 1,
                     out: Optional[torch.Tensor] = None, out_pair: bool = False,
                     split_kv: bool = True) -> torch.Tensor:
    """Flash attention over fp16 [B,H,S,hd] views (head_dim stride 1).

    key_mask: bool [B,S] (True = may attend), any strides.
    full_mask: bool tensor already expanded to [B,H,S,S] (any strides).
    out_pair: the output is an fp16 pair [2, *shape] (hi, lo planes).
    split_kv: give the kernel a workspace (from torch's caching allocator) so
    shapes with few query tiles and long key ranges run split-KV.
    """
    B, H, S, hd = q16.shape
    shape = (B, S, H * hd) if out_layout == 1 else (B, H, S, hd)
    if out is None:
        out = torch.empty(((2,) if out_pair else ()) + shape, dtype=torch.float16, device=q16.device)
    if out_pair and (tuple(out.shape) != (2, *shape) or not out.is_contiguous()):
        raise RuntimeError("attention_packed: a pair output must be a contiguous [2, *shape] fp16 tensor")
    ws = None
    if split_kv:
        nbytes = attention_workspace_bytes(B, H, S, hd, causal, q16.device)
        if nbytes:
            ws = torch.empty(nbytes, dtype=torch.uint8, device=q16.device)
    if key_mask is not None:
        kind, mptr, ms = MASK_KEY, key_mask.data_ptr(), (key_mask.stride(0), 0, 0, key_mask.stride(1))
    elif full_mask is not None:
        kind, mptr, ms = MASK_FULL, full_mask.data_ptr(), tuple(full_mask.stride())
    else:
        kind, mptr, ms = MASK_NONE, None, (0, 0, 0, 0)
    rc = lib().dotl_attention(
        q16.data_ptr(), k16.data_ptr(), v16.data_ptr(), B, H, S, hd,
        _i64arr(q16.stride()[:3]), _i64arr(k16.stride()[:3]), _i64arr(v16.stride()[:3]),
        mptr, kind, _i64arr(ms), 1 if causal else 0, float(scale), out.data_ptr(), out_layout,
        F16X2 if out_pair else F16, None if ws is None else ws.data_ptr(), 0 if ws is None else ws.numel(),
        _stream(q16.device))
    _check(rc)
    return out


_WS_BYTES: Dict[Tuple, int] = {}


def attention_workspace_bytes(B: int, H: int, S: int, hd: int, causal: bool, device: torch.device) -> int:
    """Split-KV workspace dotl_attention uses for this shape (0: none),
    memoised per shape and device."""
    key = (B, H, S, hd, bool(causal), torch.device(device).index)
    n = _WS_BYTES.get(key)
    if n is None:
        out = ctypes.c_int64(0)
        with torch.cuda.device(device):
            _check(lib().dotl_attention_workspace_bytes(B, H, S, hd, 1 if causal else 0, ctypes.byref(out)))
        n = _WS_BYTES[key] = int(out.value)
    return n


# -------------------------------------------- reference-named entry points ---

def smoke_test_identity(x: torch.Tensor) -> torch.Tensor:
    """Copy through a trivial kernel (fused_attention.cu:97-116 upstream)."""
    if not x.is_cuda:
        raise RuntimeError("smoke_test_identity: input must be a CUDA tensor")
    if x.dtype != torch.float32:
        raise RuntimeError("smoke_test_identity: only float32 is wired up for the smoke test")
    xc = x.contiguous()
    out = torch.empty_like(xc)
    _check(lib().dotl_identity_f32(xc.data_ptr(), out.data_ptr(), xc.numel(), _stream(x.device)))
    return out


def _ln_checks(x, weight, bias, who, sub=None):
    if not x.is_cuda:
        raise RuntimeError(f"{who}: x must be CUDA")
    if sub is not None:
        if not sub.is_cuda:
            raise RuntimeError(f"{who}: sub must be CUDA")
        if x.shape != sub.shape:
            raise RuntimeError(f"{who}: x and sub must have identical shapes, got "
                               f"{tuple(x.shape)} and {tuple(sub.shape)}")
        if x.dtype != sub.dtype:
            raise RuntimeError(f"{who}: x and sub must share a dtype")
    if x.dim() < 1:
        raise RuntimeError(f"{who}: x needs at least one dimension")
    D = x.shape[-1]
    if weight.numel() != D or bias.numel() != D:
        raise RuntimeError(f"{who}: weight/bias must have {D} elements")
    if weight.dtype != x.dtype or bias.dtype != x.dtype:
        raise RuntimeError(f"{who}: weight/bias must share x's dtype")


def fused_add_layernorm(x: torch.Tensor, sub: torch.Tensor, weight: torch.Tensor,
                        bias: torch.Tensor, eps: float = 1e-5,
                        normed_half: bool = False) -> List[torch.Tensor]:
    """[x + sub, LayerNorm(x + sub)] (add_layernorm.cuh:663-672 upstream)."""
    _ln_checks(x, weight, bias, "fused_add_layernorm", sub)
    if normed_half and x.dtype != torch.float32:
        raise RuntimeError(f"fused_add_layernorm: normed_half is only defined for an fp32 input, got {x.dtype}")
    dtype = x.dtype
    xs, ss = x.float().contiguous(), sub.float().contiguous()
    x_new, normed = layernorm_rows(xs, weight.float().contiguous(), bias.float().contiguous(), eps,
                                   sub=ss, out_half=normed_half)
    if dtype != torch.float32:
        return [x_new.to(dtype), normed.to(dtype)]
    return [x_new, normed]


def fused_layernorm(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor, eps: float = 1e-5,
                    out_half: bool = False) -> torch.Tensor:
    """LayerNorm(x) over the last dimension (add_layernorm.cuh:687-692 upstream)."""
    _ln_checks(x, weight, bias, "fused_layernorm")
    if out_half and x.dtype != torch.float32:
        raise RuntimeError(f"fused_layernorm: normed_half is only defined for an fp32 input, got {x.dtype}")
    dtype = x.dtype
    out = layernorm_rows(x.float().contiguous(), weight.float().contiguous(), bias.float().contiguous(),
                         eps, out_half=out_half)
    return out.to(dtype) if (dtype != torch.float32 and not out_half) else out


def _gemm_checks(x, weight, bias, who):
    if not (x.is_cuda and weight.is_cuda and bias.is_cuda):
        raise RuntimeError(f"{who}: all inputs must be CUDA tensors")
    if weight.dim() != 2:
        raise RuntimeError(f"{who}: weight must be 2-D [N, K]")
    if x.dim() < 1 or x.shape[-1] != weight.shape[1]:
        raise RuntimeError(f"{who}: x's last dimension must match weight's, got "
                           f"{tuple(x.shape)} and {tuple(weight.shape)}")
    if bias.numel() != weight.shape[0]:
        raise RuntimeError(f"{who}: bias must have {weight.shape[0]} elements")


def _gemm(x, weight, bias, act, out_half, tile, who):
    _gemm_checks(x, weight, bias, who)
    a16 = to_f16(x)
    w16 = _half_weights.get(weight)
    b32 = bias.float().contiguous()
    tile_n = 0 if tile is None or int(tile) < 0 else int(tile)
    return linear_fp16(a16, w16, b32, act=act, out_half=out_half, tile_n=tile_n)


def linear_bias(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor, tile: int = -1,
                math: int = -1, out_half: bool = False) -> torch.Tensor:
    """x @ weight^T + bias (linear_gelu.cuh:751-756 upstream).

    fp16 operands, fp32 accumulation. `tile` -1 = auto, else the N tile (128
    or 256). `math` is accepted for signature compatibility; the only
    arithmetic here is fp16 (the reference's default, kGemmMathAuto), and an
    explicit tf32 request (0) raises rather than silently computing fp16.
    """
    if math not in (-1, None):
        raise RuntimeError("linear_bias: only fp16 fragments (math=-1) exist on this build")
    return _gemm(x, weight, bias, 0, out_half, tile, "linear_bias")


def linear_gelu(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor, tile: int = -1,
                math: int = -1) -> torch.Tensor:
    """GELU_erf(x @ weight^T + bias) (linear_gelu.cuh:726-730 upstream). fp32 out."""
    if math not in (-1, None):
        raise RuntimeError("linear_gelu: only fp16 fragments (math=-1) exist on this build")
    return _gemm(x, weight, bias, 1, False, tile, "linear_gelu")


def fused_ffn_block(x, attn_out, norm1_w, norm1_b, ffn_in_w, ffn_in_b, ffn_out_w, ffn_out_b,
                    norm2_w, norm2_b, eps) -> List[torch.Tensor]:
    """[x2, normed2] for add+LN -> Linear+GELU -> Linear -> add+LN
    (ffn_block.cuh:270-311 upstream). Covers every shape (the reference
    declined above d_model 64): LN, then for d_model 128/256 the one-kernel
    MLP (dotl_ffn), elsewhere two tcgen05 GEMMs with the GELU and residual
    fused into their epilogues and a final LN."""
    if not x.is_cuda:
        raise RuntimeError("fused_ffn_block: x must be CUDA")
    if x.shape != attn_out.shape:
        raise RuntimeError(f"fused_ffn_block: x and attn_out must match, got {tuple(x.shape)} "
                           f"and {tuple(attn_out.shape)}")
    if x.dtype != torch.float32:
        raise RuntimeError(f"fused_ffn_block: float32 only, got {x.dtype}")
    D = x.shape[-1]
    F = ffn_in_w.shape[0]
    if ffn_in_w.shape[1] != D or ffn_out_w.shape[0] != D or ffn_out_w.shape[1] != F:
        raise RuntimeError(f"fused_ffn_block: weight shapes disagree with d_model={D} ffn_dim={F}")
    x1, n1 = layernorm_rows(x.contiguous(), norm1_w.float().contiguous(), norm1_b.float().contiguous(),
                            eps, sub=attn_out.contiguous(), out_half=True)
    if ffn_supported(D, F):
        # the MLP and the second LayerNorm in one kernel, the hidden on chip
        x2 = torch.empty_like(x1)
        n2 = ffn(n1, _half_weights.get(ffn_in_w), ffn_in_b.float().contiguous(), _half_weights.get(ffn_out_w),
                 ffn_out_b.float().contiguous(), norm2_w.float().contiguous(), norm2_b.float().contiguous(), eps,
                 resid=x1, resid_mode=RESID_ADD, x_out=x2)
        return [x2, n2]
    h = linear_fp16(n1, _half_weights.get(ffn_in_w), ffn_in_b.float().contiguous(), act=1, out_half=True)
    x2 = linear_fp16(h, _half_weights.get(ffn_out_w), ffn_out_b.float().contiguous(), resid=x1,
                     resid_mode=RESID_ADD)
    n2 = layernorm_rows(x2, norm2_w.float().contiguous(), norm2_b.float().contiguous(), eps)
    return [x2, n2]


# impl codes (config._IMPL_CODE upstream) and precision codes (AttnPrecision)
_IMPL_NAMES = {0: "auto", 1: "scalar", 2: "wmma", 3: "tile"}
_PREC_NAMES = {0: "auto", 1: "fp32", 2: "tf32", 3: "fp16", 4: "bf16"}


def fused_attention_forward(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                            attn_mask: Optional[torch.Tensor] = None, is_causal: bool = False,
                            scale: float = None, impl: int = 0, out_layout: int = 0,
                            precision: int = 0) -> torch.Tensor:
    """Fused scaled-dot-product attention (attention_dispatch.cuh:332-519 upstream).

    q, k, v: [B, H, S, head_dim] CUDA tensors of one dtype; strided views are
    taken as they are when head_dim is stride-1 (the fused-QKV views).
    attn_mask: optional bool, broadcastable to [B,H,S,S], True = may attend;
    may be combined with is_causal. Output: layout 0 [B,H,S,hd] or 1
    [B,S,H*hd], in q's dtype. Fully masked rows are 0.

    impl 0 (auto) and 2 (the tensor-core kernel, named "wmma" upstream) run
    the tcgen05 kernel with fp16 operands (precision auto or fp16). There is
    no scalar, tile, tf32 or bf16 arithmetic in this build: asking for one
    raises, as the reference raises for a forced impl lacking a precision.
    """
    if out_layout not in (0, 1):
        raise RuntimeError("fused_attention_forward: out_layout must be 0 ([B,H,S,head_dim]) or 1 ([B,S,H*head_dim])")
    if impl not in _IMPL_NAMES:
        raise RuntimeError("fused_attention_forward: impl must be 0 (auto), 1 (scalar), 2 (wmma) or 3 (tile)")
    if precision not in _PREC_NAMES:
        raise RuntimeError("fused_attention_forward: precision must be 0 (auto), 1 (fp32), 2 (tf32), 3 (fp16) or 4 (bf16)")
    if not (q.is_cuda and k.is_cuda and v.is_cuda):
        raise RuntimeError("fused_attention_forward: q/k/v must be CUDA tensors")
    if q.dim() != 4 or k.dim() != 4 or v.dim() != 4:
        raise RuntimeError("fused_attention_forward: q/k/v must be 4-D [B, H, S, head_dim]")
    if q.shape != k.shape or q.shape != v.shape:
        raise RuntimeError("fused_attention_forward: q/k/v must have identical shapes")
    if q.dtype != k.dtype or q.dtype != v.dtype:
        raise RuntimeError("fused_attention_forward: q/k/v must share a dtype")
    if impl in (1, 3) or precision in (1, 2, 4):
        raise RuntimeError(
            f"fused_attention_forward: impl={impl} ({_IMPL_NAMES[impl]}), precision="
            f"{_PREC_NAMES[precision]} is not covered: this build's attention kernels compute "
            "with fp16 operands (impl 0 or 2, precision 0 or 3)")
    B, H, S, hd = q.shape
    if scale is None:
        scale = hd ** -0.5
    if hd % 8 or not 8 <= hd <= 256:
        raise RuntimeError(
            f"fused_attention_forward: impl={impl} ({_IMPL_NAMES[impl]}) does not cover "
            f"dtype={q.dtype}, head_dim={hd}: head_dim must be a multiple of 8 up to 256 "
            "(32, 64 and 128 on the tcgen05 kernel, the others on the CUDA-core kernel)")
    dtype = q.dtype

    def prep(t):
        if t.dtype != torch.float16:
            t = t.to(torch.float16)
        st = t.stride()
        if st[3] != 1 or any(s % 8 for s in st[:3]) or t.data_ptr() % 16:
            t = t.contiguous()
        return t

    q16, k16, v16 = prep(q), prep(k), prep(v)
    key_mask = full_mask = None
    if attn_mask is not None:
        if attn_mask.dtype != torch.bool:
            raise RuntimeError("fused_attention_forward: attn_mask must be a bool tensor")
        m = attn_mask.contiguous().expand(B, H, S, S)
        if m.stride(1) == 0 and m.stride(2) == 0:
            key_mask = m[:, 0, 0, :]
        else:
            full_mask = m
    out = attention_packed(q16, k16, v16, bool(is_causal), float(scale), key_mask=key_mask,
                           full_mask=full_mask, out_layout=out_layout)
    return out if dtype == torch.float16 else out.to(dtype)


# ------------------------------------------------------------- knob shims ---
# The reference exposes process-global tuning knobs for its wmma/LN kernels
# (fused_attention.cu:163-364). Tile shapes here are chosen per call by the
# host dispatcher, so the setters are accepted and recorded but change
# nothing; the getters report what was set.

_knobs: Dict[str, object] = {}


def _setter(name):
    def set_knob(value):
        _knobs[name] = value
    set_knob.__name__ = name
    return set_knob


def _getter(name, default):
    def get_knob(*_args):
        return _knobs.get(name, default)
    get_knob.__name__ = name
    return get_knob


wmma_set_fp16 = _setter("wmma_fp16")
wmma_fp16 = _getter("wmma_fp16", True)
wmma_set_cp_async = _setter("wmma_cp_async_mode")
wmma_cp_async_mode = _getter("wmma_cp_async_mode", 2)
wmma_set_softmax_mode = _setter("wmma_softmax_mode")
wmma_softmax_mode = _getter("wmma_softmax_mode", 1)
wmma_set_mask_classify = _setter("wmma_mask_classify")
wmma_mask_classify_enabled = _getter("wmma_mask_classify", True)
wmma_set_direct_o = _setter("wmma_direct_o")
wmma_direct_o_enabled = _getter("wmma_direct_o", True)
wmma_set_split_kv = _setter("wmma_split_kv")
wmma_split_kv_enabled = _getter("wmma_split_kv", False)
wmma_set_causal_reverse = _setter("wmma_causal_reverse")
wmma_causal_reverse_enabled = _getter("wmma_causal_reverse", True)
layernorm_set_warp_width = _setter("layernorm_warp_width")
layernorm_warp_width = _getter("layernorm_warp_width", 2048)
layernorm_set_block_threads = _setter("layernorm_block_threads")
layernorm_set_fused_reduce = _setter("layernorm_fused_reduce")
layernorm_fused_reduce_enabled = _getter("layernorm_fused_reduce", True)


# ------------------------------------------------------------ peer memory ---

def peer_alloc(nbytes: int) -> int:
    """A zeroed device buffer whose IPC handle other processes can open."""
    p = ctypes.c_void_p(0)
    _check(lib().dotl_peer_alloc(int(nbytes), ctypes.byref(p)))
    return int(p.value)


def peer_free(ptr: int) -> None:
    _check(lib().dotl_peer_free(ptr))


def ipc_handle(ptr: int) -> bytes:
    buf = ctypes.create_string_buffer(IPC_HANDLE_BYTES)
    _check(lib().dotl_ipc_handle(ptr, buf))
    return buf.raw


def ipc_open(handle: bytes) -> int:
    if len(handle) != IPC_HANDLE_BYTES:
        raise ValueError(f"an IPC handle is {IPC_HANDLE_BYTES} bytes, got {len(handle)}")
    buf = ctypes.create_string_buffer(handle, IPC_HANDLE_BYTES)
    p = ctypes.c_void_p(0)
    _check(lib().dotl_ipc_open(buf, ctypes.byref(p)))
    return int(p.value)


def ipc_close(ptr: int) -> None:
    _check(lib().dotl_ipc_close(ptr))


def peer_blocks() -> int:
    n = ctypes.c_int(0)
    _check(lib().dotl_peer_blocks(ctypes.byref(n)))
    return int(n.value)


def peer_signal_bytes(blocks: int) -> int:
    n = ctypes.c_int64(0)
    _check(lib().dotl_peer_signal_bytes(int(blocks), ctypes.byref(n)))
    return int(n.value)


def _ptrarr(vals) -> ctypes.Array:
    return (ctypes.c_void_p * len(vals))(*[None if v is None else int(v) for v in vals])


def allreduce_ln(world: int, rank: int, parts, signals, x_new, normed, normed_half: bool, push: bool,
                 x: torch.Tensor, bias: Optional[torch.Tensor], ln_w: torch.Tensor, ln_b: torch.Tensor,
                 eps: float, sum_row_valid: Optional[torch.Tensor], normed_row_valid: Optional[torch.Tensor],
                 rows: int, D: int, blocks: int, timeout_ms: int, parts_local: bool = False,
                 signal_bytes: Optional[int] = None, status: Optional[int] = None) -> None:
    """dotl_allreduce_ln: parts / signals / x_new / normed are per-rank lists of
    device addresses as this process sees them (None where not used).
    signal_bytes: the size the signal areas were allocated with (default: the
    size `blocks` needs). status: address of a device-visible uint32 that a
    timed-out wait sets (e.g. a pinned host word), or None."""
    if signal_bytes is None:
        signal_bytes = peer_signal_bytes(blocks)
    _check(lib().dotl_allreduce_ln(
        world, rank, _ptrarr(parts), _ptrarr(signals), None if x_new is None else _ptrarr(x_new),
        _ptrarr(normed), F16 if normed_half else F32, 1 if push else 0, 1 if parts_local else 0,
        x.data_ptr(), _ptr(bias),
        _ptr(sum_row_valid), ln_w.data_ptr(), ln_b.data_ptr(), float(eps), _ptr(normed_row_valid),
        int(rows), int(D), int(blocks), int(signal_bytes), status, int(timeout_ms), _stream(x.device)))


def linear_peer(a16: torch.Tensor, w16: torch.Tensor, bias: Optional[torch.Tensor], outs, rows_per_rank: int,
                ldo: int) -> None:
    """dotl_linear_peer: a16 @ w16^T (+ bias), fp32, each 128-row tile stored
    into the receive slot of the rank owning its rows (outs: per-rank device
    addresses as this process sees them)."""
    K = a16.shape[-1]
    M = a16.numel() // K
    _check(lib().dotl_linear_peer(
        a16.data_ptr(), M, K, a16.stride(-2) if a16.dim() >= 2 else K, w16.data_ptr(), w16.shape[0],
        w16.stride(0), _ptr(bias), len(outs), _ptrarr(outs), int(rows_per_rank), int(ldo), _stream(a16.device)))
