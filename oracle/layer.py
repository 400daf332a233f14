"""CPU fp32 restatement of the reference layer forward. TEST INFRASTRUCTURE ONLY.

Every function cites the reference file:line it restates. Paths are relative
to the reference project root (jazwinn/Distraction-OptimizedTransformerLayer).

Nothing here touches a GPU. It runs in fp32 on CPU, with the same op order as
the reference, so its output is what the reference's `BaselineTransformer`
produces on a CPU for the same parameters and inputs (pinned bit-for-bit by
tests/test_oracle_golden.py against fixtures generated from the reference).
"""

from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Dict, List, Optional, Tuple

import torch
import torch.nn.functional as F


@dataclass(frozen=True)
class TransformerConfig:
    """Same fields and validation as torch_transformer_benchmark.py:40-67."""

    batch_size: int
    seq_len: int
    d_model: int
    num_heads: int
    ffn_dim: int
    num_layers: int
    causal: bool

    def validate(self) -> None:
        if self.batch_size <= 0:
            raise ValueError("batch_size must be positive")
        if self.seq_len <= 0:
            raise ValueError("seq_len must be positive")
        if self.d_model <= 0:
            raise ValueError("d_model must be positive")
        if self.num_heads <= 0:
            raise ValueError("num_heads must be positive")
        if self.d_model % self.num_heads != 0:
            raise ValueError(
                f"d_model ({self.d_model}) must be divisible by "
                f"num_heads ({self.num_heads})")
        if self.ffn_dim <= 0:
            raise ValueError("ffn_dim must be positive")
        if self.num_layers <= 0:
            raise ValueError("num_layers must be positive")


# The five benchmark configurations, one layer each, with the padding ratio
# that reproduces their valid-length ranges through generate_random_case
# (0.5 gives lengths U[S/2, S]; 0 gives an all-valid mask).
BASELINE_CONFIGS: Dict[int, Tuple[TransformerConfig, float]] = {
    1: (TransformerConfig(2, 128, 256, 4, 1024, 1, False), 0.5),
    2: (TransformerConfig(4, 512, 512, 8, 2048, 1, True), 0.0),
    3: (TransformerConfig(8, 2048, 1024, 16, 4096, 1, False), 0.5),
    4: (TransformerConfig(8192, 32, 256, 4, 1024, 1, False), 0.0),
    5: (TransformerConfig(16, 1024, 2048, 16, 8192, 1, True), 0.0),
}


def _param_names(cfg: TransformerConfig) -> List[Tuple[str, Tuple[int, ...], str]]:
    """(name, shape, kind) for every parameter of BaselineTransformer, in
    state_dict order (torch_transformer_benchmark.py:222-260)."""
    d, f = cfg.d_model, cfg.ffn_dim
    out = []
    for i in range(cfg.num_layers):
        p = f"layers.{i}."
        out += [(p + "norm1.weight", (d,), "ln_w"), (p + "norm1.bias", (d,), "ln_b")]
        for proj in ("q_proj", "k_proj", "v_proj", "out_proj"):
            out += [(p + f"attention.{proj}.weight", (d, d), "w"),
                    (p + f"attention.{proj}.bias", (d,), "b")]
        out += [(p + "norm2.weight", (d,), "ln_w"), (p + "norm2.bias", (d,), "ln_b"),
                (p + "ffn_in.weight", (f, d), "w"), (p + "ffn_in.bias", (f,), "b"),
                (p + "ffn_out.weight", (d, f), "w"), (p + "ffn_out.bias", (d,), "b")]
    out += [("final_norm.weight", (d,), "ln_w"), ("final_norm.bias", (d,), "ln_b")]
    return out


def init_params(cfg: TransformerConfig, seed: int) -> Dict[str, torch.Tensor]:
    """The benchmark's parameter initialisation, as a state_dict.

    Xavier-uniform on every Linear weight, U(-0.02, 0.02) on every Linear bias,
    LayerNorm gamma = 1 and beta = 0, drawn in state_dict order from one seeded
    CPU generator. The names are exactly BaselineTransformer's, so the dict
    loads with strict=True into the reference model and into
    `optimized.OptimizedTransformer` (optimized/model.py:24-30 upstream).
    """
    g = torch.Generator(device="cpu")
    g.manual_seed(seed)
    params: Dict[str, torch.Tensor] = {}
    for name, shape, kind in _param_names(cfg):
        if kind == "ln_w":
            t = torch.ones(shape)
        elif kind == "ln_b":
            t = torch.zeros(shape)
        elif kind == "w":
            fan_out, fan_in = shape
            bound = math.sqrt(6.0 / float(fan_in + fan_out))
            t = (torch.rand(shape, generator=g) * 2.0 - 1.0) * bound
        else:
            t = (torch.rand(shape, generator=g) * 2.0 - 1.0) * 0.02
        params[name] = t.float().contiguous()
    return params


def param_checksum(params: Dict[str, torch.Tensor]) -> float:
    """float64 sum of (index+1) * sum(param) over the state_dict, a cheap
    fingerprint that regenerated parameters are the fixture's parameters."""
    total = 0.0
    for i, name in enumerate(sorted(params)):
        total += (i + 1) * float(params[name].double().sum())
    return total


def generate_random_case(
    cfg: TransformerConfig,
    seed: int,
    padding_ratio: float,
    input_scale: float = 1.0,
    rows: Optional[int] = None,
) -> Tuple[torch.Tensor, torch.Tensor]:
    """torch_transformer_benchmark.py:500-540 on the CPU, fp32.

    x ~ N(0,1) * input_scale; a prefix key-padding mask with per-row valid
    lengths randint(round(S*(1-p)), S+1) drawn from the same generator after x;
    padded rows of x zeroed. Same generator calls in the same order, so it is
    bit-identical to the reference's CPU output for the same seed.
    """
    g = torch.Generator(device="cpu")
    g.manual_seed(seed)
    batch = cfg.batch_size if rows is None else rows
    x = torch.randn(batch, cfg.seq_len, cfg.d_model, generator=g,
                    dtype=torch.float32)
    x = x * input_scale
    if padding_ratio <= 0:
        return x, torch.ones(batch, cfg.seq_len, dtype=torch.bool)
    min_valid = max(1, int(round(cfg.seq_len * (1.0 - padding_ratio))))
    lengths = torch.randint(low=min_valid, high=cfg.seq_len + 1, size=(batch,),
                            generator=g)
    positions = torch.arange(cfg.seq_len)[None, :]
    mask = positions < lengths[:, None]
    x = x.masked_fill(~mask[..., None], 0)
    return x, mask


def attention_reference(q, k, v, attn_mask, is_causal: bool, scale: float,
                        query_block: int = 0):
    """softmax(q k^T * scale + masks) v per head, as the reference computes it.

    torch_transformer_benchmark.py:108-125 (BaselineSelfAttention.forward) and
    scripts/verify_kernel.py:58-68 (reference_attention): scores scaled after
    the matmul, causal triangle then the key mask applied as -inf, fp32
    softmax, probabilities times v. `attn_mask` is a bool tensor broadcastable
    to [B,H,S,S], True = may attend. q/k/v are [B,H,S,hd].

    query_block > 0 scores that many queries at a time, which is the reference's
    ChunkedBaselineSelfAttention (torch_transformer_benchmark.py:146-219): the
    same rows, with less memory. A fully masked row yields NaN here, as it does
    in the reference (0/0 in the softmax).
    """
    S = q.shape[2]
    block = S if query_block <= 0 else query_block
    out = torch.empty_like(q)
    for lo in range(0, S, block):
        hi = min(lo + block, S)
        scores = torch.matmul(q[:, :, lo:hi], k.transpose(-2, -1)) * scale
        if is_causal:
            qpos = torch.arange(lo, hi)[:, None]
            kpos = torch.arange(S)[None, :]
            scores = scores.masked_fill(kpos > qpos, float("-inf"))
        if attn_mask is not None:
            m = attn_mask
            if m.dim() == 4 and m.shape[2] != 1:
                m = m[:, :, lo:hi]
            scores = scores.masked_fill(~m, float("-inf"))
        probs = torch.softmax(scores.float(), dim=-1).to(q.dtype)
        out[:, :, lo:hi] = torch.matmul(probs, v)
    return out


def _layer_norm(x, params, prefix):
    return F.layer_norm(x, (x.shape[-1],), params[prefix + ".weight"],
                        params[prefix + ".bias"], 1e-5)


def _self_attention(params, prefix, x, mask, causal, num_heads, query_block):
    """BaselineSelfAttention.forward, torch_transformer_benchmark.py:96-133."""
    batch, seq_len, d_model = x.shape
    hd = d_model // num_heads
    scale = hd ** -0.5  # :81

    def proj(name, t):
        return F.linear(t, params[f"{prefix}.{name}.weight"],
                        params[f"{prefix}.{name}.bias"])

    def split(t):  # _split_heads, :88-94
        return t.view(batch, seq_len, num_heads, hd).transpose(1, 2).contiguous()

    q = split(proj("q_proj", x))
    k = split(proj("k_proj", x))
    v = split(proj("v_proj", x))
    key_mask = mask[:, None, None, :] if mask is not None else None
    ctx = attention_reference(q, k, v, key_mask, causal, scale, query_block)
    ctx = ctx.transpose(1, 2).contiguous().view(batch, seq_len, d_model)
    out = proj("out_proj", ctx)
    if mask is not None:
        out = out.masked_fill(~mask[..., None], 0)
    return out


@torch.inference_mode()
def baseline_forward(params: Dict[str, torch.Tensor], cfg: TransformerConfig,
                     x: torch.Tensor, mask: Optional[torch.Tensor],
                     query_block: int = 0) -> torch.Tensor:
    """BaselineTransformer.forward (torch_transformer_benchmark.py:262-272) with
    BaselineTransformerBlock.forward (:234-245) per layer:

        x = x + attn(norm1(x)); x = x + ffn_out(gelu(ffn_in(norm2(x))))
        x = masked_fill(x, pad, 0)           per layer, when a mask is given
        out = masked_fill(final_norm(x), pad, 0)

    Pre-LN with a final LayerNorm; GELU is the exact erf form.
    """
    x = x.float()
    for i in range(cfg.num_layers):
        p = f"layers.{i}"
        x = x + _self_attention(params, p + ".attention", _layer_norm(x, params, p + ".norm1"),
                                mask, cfg.causal, cfg.num_heads, query_block)
        h = F.linear(_layer_norm(x, params, p + ".norm2"),
                     params[p + ".ffn_in.weight"], params[p + ".ffn_in.bias"])
        h = F.gelu(h, approximate="none")
        x = x + F.linear(h, params[p + ".ffn_out.weight"], params[p + ".ffn_out.bias"])
        if mask is not None:
            x = x.masked_fill(~mask[..., None], 0)
    x = _layer_norm(x, params, "final_norm")
    if mask is not None:
        x = x.masked_fill(~mask[..., None], 0)
    return x


def _r16(t: torch.Tensor) -> torch.Tensor:
    """Round to fp16 (round to nearest even) and widen back to float64."""
    return t.half().double()


@torch.inference_mode()
def fp16_operand_forward(params: Dict[str, torch.Tensor], cfg: TransformerConfig,
                         x: torch.Tensor, mask: torch.Tensor) -> torch.Tensor:
    """The reference's fp16 kernel path, in exact (float64) arithmetic.

    Same graph as `baseline_forward`, with the operands rounded to fp16 where
    the reference's own CUDA kernels round them in their fp16 configuration,
    and nothing else rounded:
      - every GEMM stages A and W as __half (csrc/linear_gelu.cuh:66-71), so
        the LayerNorm outputs, the attention context and the GELU output meet
        their GEMM as fp16 (csrc/add_layernorm.cuh:30-43 stores `normed` fp16
        for that reason);
      - attention contracts fp32 q/k/v as __half
        (csrc/attention_wmma.cuh:2049-2066) and stores the unnormalised
        probabilities exp(s - max) as __half before the P.V product, while the
        row sum adds the unrounded values (csrc/attention_wmma.cuh:1420-1431);
      - the residual stream, LayerNorm statistics, softmax and GELU stay wide.
    Used to separate the error that fp16 operands cause on their own from
    anything a kernel adds: over several layers that error alone can pass the
    harness's 2e-3 absolute bound on a few elements. `mask` is required here
    (an all-True mask for none).
    """
    def ln(t, pre):
        return F.layer_norm(t, (t.shape[-1],), params[pre + ".weight"].double(),
                            params[pre + ".bias"].double(), 1e-5)

    def lin(t, name):
        return _r16(t) @ _r16(params[name + ".weight"].double()).t() + params[name + ".bias"].double()

    B, S, d = x.shape
    H = cfg.num_heads
    hd = d // H
    allow = mask[:, None, None, :].expand(B, H, S, S)
    if cfg.causal:
        allow = allow & torch.ones(S, S, dtype=torch.bool).tril()
    keep = mask[..., None]
    h = x.double()
    for i in range(cfg.num_layers):
        pre = f"layers.{i}"
        n1 = ln(h, pre + ".norm1")

        def heads(name):
            return _r16(lin(n1, f"{pre}.attention.{name}").view(B, S, H, hd).transpose(1, 2))

        q, k, v = heads("q_proj"), heads("k_proj"), heads("v_proj")
        s = (q @ k.transpose(-1, -2)) * hd ** -0.5
        s = s.masked_fill(~allow, float("-inf"))
        m = s.amax(-1, keepdim=True).clamp_min(-1e300)
        e = torch.exp(s - m)
        l = e.sum(-1, keepdim=True)
        ctx = (_r16(e) @ v) / l.clamp_min(1e-300)
        ctx = ctx.masked_fill(l == 0, 0.0).transpose(1, 2).reshape(B, S, d)
        h = h + lin(ctx, f"{pre}.attention.out_proj").masked_fill(~keep, 0)
        f = F.gelu(lin(ln(h, pre + ".norm2"), pre + ".ffn_in"), approximate="none")
        h = (h + lin(f, pre + ".ffn_out")).masked_fill(~keep, 0)
    return ln(h, "final_norm").masked_fill(~keep, 0).float()


@dataclass
class AccuracyResult:
    """Fields of the reference's AccuracyResult (torch_transformer_benchmark.py:543-554)."""

    passed: bool
    total_elements: int
    failed_elements: int
    max_abs_error: float
    max_relative_error: float
    mean_abs_error: float
    worst_index: Tuple[int, ...]
    reference_at_worst: float
    optimized_at_worst: float


def compare_outputs(reference: torch.Tensor, optimized: torch.Tensor,
                    rtol: float = 0.02, atol: float = 0.002) -> AccuracyResult:
    """The harness's elementwise rule, torch_transformer_benchmark.py:557-624.

    An element passes when both values are finite and
    |opt - ref| <= atol OR |opt - ref| <= rtol * |ref|. The run passes only
    with zero failing elements. Defaults are the harness defaults
    (:1077-1078): atol 2e-3, rtol 2%.
    """
    if reference.shape != optimized.shape:
        raise AssertionError(f"shape mismatch: baseline={tuple(reference.shape)}, "
                             f"optimized={tuple(optimized.shape)}")
    ref = reference.detach().float().cpu()
    opt = optimized.detach().float().cpu()
    finite = torch.isfinite(ref) & torch.isfinite(opt)
    abs_error = (opt - ref).abs()
    passed = finite & ((abs_error <= atol) | (abs_error <= rtol * ref.abs()))
    failed = int((~passed).sum())
    if ref.numel() == 0:
        return AccuracyResult(True, 0, 0, 0.0, 0.0, 0.0, (), 0.0, 0.0)
    flat = int(torch.nan_to_num(abs_error, nan=float("inf")).reshape(-1).argmax())
    idx = []
    rem = flat
    for size in reversed(ref.shape):
        idx.append(rem % size)
        rem //= size
    worst = tuple(reversed(idx))
    rel = abs_error / ref.abs().clamp_min(1e-12)
    return AccuracyResult(
        passed=failed == 0,
        total_elements=ref.numel(),
        failed_elements=failed,
        max_abs_error=float(abs_error.max()),
        max_relative_error=float(rel.max()),
        mean_abs_error=float(abs_error.mean()),
        worst_index=worst,
        reference_at_worst=float(ref[worst]),
        optimized_at_worst=float(opt[worst]),
    )
