"""Tensor parallelism across the GPUs of one box.

The reference runs on one GPU and has no parallel code
asks for the wide-head layer "8-way head-sharded tensor parallel with one NCCL
all-reduce over NVLink after the out-proj and after FFN2". With P ranks (one
process per GPU, torch.distributed over NCCL), rank r holds:

    attention  q/k/v rows and out_proj columns of heads [r H/P, (r+1) H/P)
    ffn_in     rows [r F/P, (r+1) F/P)        (column-parallel, GELU local)
    ffn_out    columns [r F/P, (r+1) F/P)     (row-parallel)
    biases of out_proj / ffn_out on rank 0 only (added once by the sum)
    LayerNorm parameters on every rank (the norms run replicated)

Per layer, on every rank (x replicated, fp32):

    n1 = LN1(x) fp16; qkv_r = n1 Wqkv_r^T + b; ctx_r = attention(local heads)
    part = mask(ctx_r Wo_r^T + [bo]) fp32   -> all_reduce(sum) over NVLink
    x1, n2 = x + part, LN2(x + part)
    h_r = GELU(n2 W1_r^T + b1_r); part = mask(h_r W2_r^T + [b2]) -> all_reduce
    x2, out = x1 + part, next LN(x1 + part)

With fused=True (the default at 2 ranks, where it measured faster than NCCL;
NCCL is the default above that) each all_reduce + add + LN
pair is one dotl_allreduce_ln kernel over peer memory (optimized/peer.py):
the GEMMs write bias-free partial sums and the kernel adds the full bias once,
on valid rows only. Otherwise NCCL all-reduces partials that carry the bias on
rank 0 and are zeroed on padded rows.

Failure: the fused reduction's waits for peers are bounded (timeout_ms). A
timed-out wait leaves that forward's outputs invalid and the peer group's
counters out of step. With error_check="sync" (the default) forward()
synchronises the stream at its end and raises PeerTimeoutError, so no invalid
output is returned. With "deferred" (no per-forward sync, for pipelined
serving and timing loops) the next forward() or check() raises instead. After
the error the group is poisoned: the next forward rebuilds it, which is
collective, so every rank must take that path (every rank sees the timeout
when a peer stops calling).

The partial sums stay fp32 through the reduction. Padded rows add nothing;
the residual stream keeps x there, which differs from the reference's zeroed
rows only on padded rows, which no valid row attends to and the final
LayerNorm writes as 0.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Dict, Optional

import torch

RESID_NONE, MASK_ROWS = 0, 4


@dataclass(frozen=True)
class TPShardPlan:
    """Which slices of each weight rank `rank` of `world` holds."""

    d_model: int
    num_heads: int
    ffn_dim: int
    world: int
    rank: int

    def __post_init__(self):
        if self.num_heads % self.world or self.ffn_dim % self.world:
            raise ValueError(f"heads ({self.num_heads}) and ffn_dim ({self.ffn_dim}) must divide "
                             f"by the tensor-parallel size {self.world}")
        if not 0 <= self.rank < self.world:
            raise ValueError(f"rank {self.rank} outside [0, {self.world})")
        if (self.d_model // self.world) % 8 or (self.ffn_dim // self.world) % 8:
            raise ValueError("each rank's slice of d_model and ffn_dim must be a multiple of 8")

    @property
    def head_dim(self) -> int:
        return self.d_model // self.num_heads

    @property
    def local_heads(self) -> int:
        return self.num_heads // self.world

    @property
    def d_slice(self) -> slice:
        w = self.d_model // self.world
        return slice(self.rank * w, (self.rank + 1) * w)

    @property
    def f_slice(self) -> slice:
        w = self.ffn_dim // self.world
        return slice(self.rank * w, (self.rank + 1) * w)

    def shard(self, state: Dict[str, torch.Tensor], num_layers: int) -> Dict[str, torch.Tensor]:
        """This rank's tensors from a full BaselineTransformer state_dict."""
        ds, fs = self.d_slice, self.f_slice
        out: Dict[str, torch.Tensor] = {}
        for i in range(num_layers):
            p = f"layers.{i}."
            a = p + "attention."
            out[p + "wqkv"] = torch.cat([state[a + f"{n}_proj.weight"][ds] for n in "qkv"], 0)
            out[p + "bqkv"] = torch.cat([state[a + f"{n}_proj.bias"][ds] for n in "qkv"], 0)
            out[p + "wo"] = state[a + "out_proj.weight"][:, ds]
            bo = state[a + "out_proj.bias"]
            out[p + "bo"] = bo if self.rank == 0 else torch.zeros_like(bo)
            out[p + "w1"] = state[p + "ffn_in.weight"][fs]
            out[p + "b1"] = state[p + "ffn_in.bias"][fs]
            out[p + "w2"] = state[p + "ffn_out.weight"][:, fs]
            b2 = state[p + "ffn_out.bias"]
            out[p + "b2"] = b2 if self.rank == 0 else torch.zeros_like(b2)
            for n in ("norm1", "norm2"):
                out[p + n + ".weight"] = state[p + n + ".weight"]
                out[p + n + ".bias"] = state[p + n + ".bias"]
        out["final_norm.weight"] = state["final_norm.weight"]
        out["final_norm.bias"] = state["final_norm.bias"]
        return out


class TensorParallelTransformer:
    """The layer stack split over the ranks of a process group (one per GPU).

    forward(x, valid_token_mask) takes the same replicated input on every rank
    and returns the same [B, S, d_model] fp32 output on every rank. Every rank
    must call it with the same shapes in the same order (it runs collectives).
    """

    def __init__(self, config, state_dict: Dict[str, torch.Tensor], group=None,
                 device: Optional[torch.device] = None, eps: float = 1e-5,
                 fused: Optional[bool] = None, push: Optional[bool] = None,
                 timeout_ms: int = 2000, scatter: Optional[bool] = None,
                 error_check: str = "sync") -> None:
        import torch.distributed as dist

        self.dist = dist
        self.group = group
        self.config = config
        self.eps = eps
        world = dist.get_world_size(group)
        rank = dist.get_rank(group)
        self.plan = TPShardPlan(config.d_model, config.num_heads, config.ffn_dim, world, rank)
        dev = device or torch.device("cuda", torch.cuda.current_device())
        self.device = dev
        shards = self.plan.shard(state_dict, config.num_layers)
        self.w: Dict[str, torch.Tensor] = {}
        for k, t in shards.items():
            half = k.split(".")[-1] in ("wqkv", "wo", "w1", "w2")
            self.w[k] = t.detach().to(dev, torch.float16 if half else torch.float32).contiguous()
        d = config.d_model
        if fused is None:
            # measured on B200s at config 5: the fused reduction wins at 2 ranks
            # (12.6 vs 10.6 M tokens/s), NCCL's bulk transfers at 8 (12.7 vs 10.3)
            fused = d % 4 == 0 and d <= 2048 and world <= 2
        if error_check not in ("sync", "deferred"):
            raise ValueError(f"error_check must be 'sync' or 'deferred', not {error_check!r}")
        self.error_check = error_check
        self.fused, self.push, self.timeout_ms = bool(fused), push, timeout_ms
        self.scatter = scatter   # None: wherever the rows allow it
        self.peer = None
        if self.fused:
            # the fused reduction adds the full biases itself; the GEMMs get zeros
            for i in range(config.num_layers):
                p = f"layers.{i}."
                self.w[p + "bo_full"] = state_dict[p + "attention.out_proj.bias"].detach().to(dev, torch.float32).contiguous()
                self.w[p + "b2_full"] = state_dict[p + "ffn_out.bias"].detach().to(dev, torch.float32).contiguous()
            self.w["zero_d"] = torch.zeros(d, dtype=torch.float32, device=dev)

    def _kernels(self):
        from .kernels import _custom_kernels

        return _custom_kernels()

    def _peer_group(self, rows: int):
        from .peer import PeerGroup

        if self.peer is None or self.peer.rows < rows or self.peer.poisoned:
            if self.peer is not None:
                self.peer.close()
                self.peer = None
            self.peer = PeerGroup(self.group, rows, self.config.d_model, self.device, self.push,
                                  self.timeout_ms)
        return self.peer

    def check(self) -> None:
        """Raise PeerTimeoutError if a finished forward of the fused path gave up
        waiting for a peer (reads a pinned host word: no device sync). Its
        output was not valid; the next forward rebuilds the peer group."""
        if self.peer is not None:
            self.peer.check()

    def close(self) -> None:
        """Collective: releases the peer-mapped buffers of the fused path."""
        if self.peer is not None:
            self.peer.close()
            self.peer = None

    def _forward_fused(self, x: torch.Tensor, valid_token_mask: Optional[torch.Tensor]) -> torch.Tensor:
        """The layer with each all-reduce + add + LayerNorm as one
        dotl_allreduce_ln over peer memory. Returns the group's `out` buffer
        viewed as [B, S, d]: it is overwritten by the next forward."""
        k = self._kernels()
        cfg, plan, w = self.config, self.plan, self.w
        B, S, d = x.shape
        T = B * S
        pg = self._peer_group(T)
        use_mask = valid_token_mask is not None and not bool(valid_token_mask.all())
        mask = valid_token_mask.contiguous() if use_mask else None
        rv = mask.reshape(-1) if use_mask else None
        hd, hl = plan.head_dim, plan.local_heads
        bufs = {n: pg.view(n, T) for n in ("part", "xa", "xb", "n16", "out")}
        part, n16 = bufs["part"], bufs["n16"]
        # the row-parallel GEMMs scatter their tiles to the row owners while they
        # run (the reduce-scatter inside the GEMM), or write locally for the
        # reduction kernel to pull
        scatter = self.scatter is not False and pg.scatter_ok(T)

        def row_parallel(a16, w16):
            if scatter:
                pg.gemm_to_owners(a16, w16, T)
            else:
                k.linear_fp16(a16, w16, w["zero_d"], out=part)
        bufs["xa"].copy_(x.reshape(T, d))
        k.layernorm_rows(bufs["xa"], w["layers.0.norm1.weight"], w["layers.0.norm1.bias"], self.eps, out=n16)
        cur, alt = "xa", "xb"
        for i in range(cfg.num_layers):
            p = f"layers.{i}."
            qkv = k.linear_fp16(n16.view(B, S, d), w[p + "wqkv"], w[p + "bqkv"], out_half=True)
            q, kk, v = qkv.view(B, S, 3, hl, hd).permute(2, 0, 3, 1, 4).unbind(0)
            ctx = k.attention_packed(q, kk, v, cfg.causal, hd ** -0.5, key_mask=mask)
            row_parallel(ctx.reshape(T, -1), w[p + "wo"])
            pg.allreduce_ln(bufs[cur], w[p + "bo_full"], w[p + "norm2.weight"], w[p + "norm2.bias"], self.eps,
                            alt, "n16", T, sum_row_valid=rv, from_owners=scatter)
            h = k.linear_fp16(n16, w[p + "w1"], w[p + "b1"], act=1, out_half=True)
            row_parallel(h, w[p + "w2"])
            last = i == cfg.num_layers - 1
            nn_ = "final_norm." if last else f"layers.{i + 1}.norm1."
            pg.allreduce_ln(bufs[alt], w[p + "b2_full"], w[nn_ + "weight"], w[nn_ + "bias"], self.eps,
                            None if last else cur, "out" if last else "n16", T, sum_row_valid=rv,
                            normed_row_valid=rv if last else None, from_owners=scatter)
        return bufs["out"].view(B, S, d)

    def forward(self, x: torch.Tensor, valid_token_mask: Optional[torch.Tensor] = None) -> torch.Tensor:
        if self.fused:
            if self.peer is not None and not self.peer.poisoned:
                self.peer.check()          # an earlier (deferred) forward that timed out
            out = self._forward_fused(x.float().contiguous(), valid_token_mask)
            if self.error_check == "sync":
                torch.cuda.current_stream(self.device).synchronize()
                self.peer.check()
            return out
        k = self._kernels()
        cfg, plan, w = self.config, self.plan, self.w
        B, S, d = x.shape
        x = x.float().contiguous()
        use_mask = valid_token_mask is not None and not bool(valid_token_mask.all())
        mask = valid_token_mask.contiguous() if use_mask else None
        rv = mask.reshape(-1) if use_mask else None
        mode = MASK_ROWS if use_mask else RESID_NONE
        hd, hl = plan.head_dim, plan.local_heads
        normed = k.layernorm_rows(x, w["layers.0.norm1.weight"], w["layers.0.norm1.bias"], self.eps,
                                  out_half=True)
        for i in range(cfg.num_layers):
            p = f"layers.{i}."
            qkv = k.linear_fp16(normed, w[p + "wqkv"], w[p + "bqkv"], out_half=True)
            q, kk, v = qkv.view(B, S, 3, hl, hd).permute(2, 0, 3, 1, 4).unbind(0)
            ctx = k.attention_packed(q, kk, v, cfg.causal, hd ** -0.5, key_mask=mask)
            part = k.linear_fp16(ctx, w[p + "wo"], w[p + "bo"], row_valid=rv, resid_mode=mode)
            self.dist.all_reduce(part, group=self.group)
            x1, n2 = k.layernorm_rows(x, w[p + "norm2.weight"], w[p + "norm2.bias"], self.eps, sub=part,
                                      out_half=True)
            h = k.linear_fp16(n2, w[p + "w1"], w[p + "b1"], act=1, out_half=True)
            part2 = k.linear_fp16(h, w[p + "w2"], w[p + "b2"], row_valid=rv, resid_mode=mode)
            self.dist.all_reduce(part2, group=self.group)
            last = i == cfg.num_layers - 1
            nn_ = "final_norm." if last else f"layers.{i + 1}.norm1."
            x, normed = k.layernorm_rows(x1, w[nn_ + "weight"], w[nn_ + "bias"], self.eps, sub=part2,
                                         out_half=not last, row_valid=rv if last else None)
        return normed

    __call__ = forward
