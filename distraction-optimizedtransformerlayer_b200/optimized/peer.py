"""Peer-mapped buffers for the fused all-reduce + LayerNorm of the
tensor-parallel layer (one process per GPU, one box).

No reference counterpart: the reference runs on one GPU. This replaces, for
`TensorParallelTransformer`, each NCCL all-reduce of fp32 partial sums and the
add+LayerNorm kernel after it with one `dotl_allreduce_ln` launch that reads
the peers' partial sums over NVLink (plain loads from each peer, one CTA at a time).

Every rank allocates the same named buffers with `dotl_peer_alloc`, publishes
their CUDA IPC handles through the process group (all_gather_object) and
maps every peer's with `dotl_ipc_open`:

    part      fp32 [rows, d]  the rank's partial sums (a row-parallel GEMM writes here)
    recv      fp32 [rows, d]  slots [world][rows / world, d]: every rank's partial sums of
                              this rank's rows, stored there by dotl_linear_peer
    xa, xb    fp32 [rows, d]  residual stream, ping-pong
    n16       fp16 [rows, d]  LayerNorm output feeding the next GEMM
    out       fp32 [rows, d]  the final LayerNorm output
    signal    the per-CTA handshake flags

push=True (two-shot, the default): each rank reduces 1/world of the rows and
stores them into every rank's buffers. push=False (one-shot): each rank
reduces every row and writes its own buffers only; at 2 ranks it moves fewer
NVLink bytes (4 vs 5 per element) but measured slower on config 5 (309 vs
307 us per launch, 11.4 vs 12.1 M tokens/s per step), and above 2 ranks it
reads (P-1) whole partials per rank.

Every rank must create the group, and call `allreduce_ln`, with the same
arguments in the same order. `close()` unmaps and frees collectively.

Failure: every wait inside the kernel is bounded by `timeout_ms`. A wait that
runs out stores a bit into `status`, a pinned host word the kernel writes
through its device mapping, so the host sees it without a device sync once
the kernel has finished (`failed()`). The ranks' call counters then disagree,
so the group is unusable: `check()` raises PeerTimeoutError and marks the
group `poisoned`, and its owner must rebuild it (collectively) before the
next call.
"""

from __future__ import annotations

from typing import Dict, List, Optional

import torch

_NAMES = ("part", "recv", "xa", "xb", "n16", "out")


class PeerTimeoutError(RuntimeError):
    """A fused all-reduce gave up waiting for a peer; its outputs are not valid."""


class _DeviceView:
    """Exposes library-owned device memory to torch.as_tensor (zero copy)."""

    _TYPESTR = {torch.float32: "<f4", torch.float16: "<f2"}

    def __init__(self, ptr: int, shape, dtype: torch.dtype) -> None:
        self.__cuda_array_interface__ = {
            "shape": tuple(int(s) for s in shape), "typestr": self._TYPESTR[dtype],
            "data": (int(ptr), False), "version": 3, "strides": None,
        }


class PeerGroup:
    def __init__(self, group, rows: int, d: int, device: torch.device, push: Optional[bool] = None,
                 timeout_ms: int = 2000) -> None:
        import torch.distributed as dist

        from .kernels import _custom_kernels

        self.k = _custom_kernels()
        self.dist, self.group = dist, group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if not 1 <= self.world <= 8:
            raise ValueError(f"the fused all-reduce covers 1..8 ranks, not {self.world}")
        if d % 4 or d > 2048:
            raise ValueError(f"the fused all-reduce needs d_model % 4 == 0 and <= 2048, got {d}")
        self.rows, self.d, self.device = int(rows), int(d), device
        self.push = True if push is None else bool(push)
        self.timeout_ms = int(timeout_ms)
        self.poisoned = False
        # Host word the kernel sets when a wait times out (pinned memory is
        # mapped into the device's address space at the same address).
        self.status = torch.zeros(1, dtype=torch.int32, pin_memory=torch.cuda.is_available())
        k = self.k
        with torch.cuda.device(device):
            blocks = torch.tensor([k.peer_blocks()], dtype=torch.int64, device=device)
            dist.all_reduce(blocks, op=dist.ReduceOp.MIN, group=group)
            self.blocks = int(blocks.item())
            sizes = {n: self.rows * d * (2 if n == "n16" else 4) for n in _NAMES}
            sizes["signal"] = self.signal_bytes = k.peer_signal_bytes(self.blocks)
            self._own: Dict[str, int] = {}
            self._opened: List[int] = []
            try:
                for n, nbytes in sizes.items():
                    self._own[n] = k.peer_alloc(max(nbytes, 16))
                handles = {n: k.ipc_handle(p) for n, p in self._own.items()}
                everyone: List[Optional[dict]] = [None] * self.world
                dist.all_gather_object(everyone, handles, group=group)
                self.ptrs: Dict[str, List[int]] = {n: [0] * self.world for n in sizes}
                for r in range(self.world):
                    for n in sizes:
                        if r == self.rank:
                            self.ptrs[n][r] = self._own[n]
                        else:
                            p = k.ipc_open(everyone[r][n])
                            self._opened.append(p)
                            self.ptrs[n][r] = p
            except Exception:
                self._release()
                raise
            dist.barrier(group=group)

    def view(self, name: str, rows: Optional[int] = None) -> torch.Tensor:
        """This rank's buffer `name` as a [rows, d] tensor (fp16 for n16)."""
        rows = self.rows if rows is None else rows
        if rows > self.rows:
            raise ValueError(f"{rows} rows exceed the group's {self.rows}")
        dtype = torch.float16 if name == "n16" else torch.float32
        return torch.as_tensor(_DeviceView(self._own[name], (rows, self.d), dtype), device=self.device)

    def allreduce_ln(self, x: torch.Tensor, bias: Optional[torch.Tensor], ln_w: torch.Tensor,
                     ln_b: torch.Tensor, eps: float, x_new: Optional[str], normed: str, rows: int,
                     sum_row_valid: Optional[torch.Tensor] = None,
                     normed_row_valid: Optional[torch.Tensor] = None, from_owners: bool = False) -> None:
        """x_new := x + valid * (sum over ranks of `part` + bias); normed := LN(x_new).

        x is this rank's residual (a [rows, d] fp32 tensor, the same values on
        every rank); x_new names a buffer ('xa' / 'xb') or None, normed names
        'n16' (fp16) or 'out' (fp32)."""
        if rows > self.rows:
            raise ValueError(f"{rows} rows exceed the group's {self.rows}")
        if self.poisoned:
            raise PeerTimeoutError("this peer group timed out earlier and must be rebuilt")
        if x_new is not None and self._own[x_new] == x.data_ptr():
            raise ValueError("x_new must not be the buffer x is read from")
        dsts = range(self.world) if self.push else (self.rank,)
        mask = [r in dsts for r in range(self.world)]
        pick = lambda n: [p if m else None for p, m in zip(self.ptrs[n], mask)]  # noqa: E731
        if from_owners:
            # the GEMMs left rank s's partial sums of this rank's rows in slot s
            per = rows // self.world
            base = self.ptrs["recv"][self.rank]
            parts = [base + s * per * self.d * 4 for s in range(self.world)]
        else:
            parts = self.ptrs["part"]
        self.k.allreduce_ln(
            self.world, self.rank, parts, self.ptrs["signal"],
            None if x_new is None else pick(x_new), pick(normed), normed == "n16", self.push,
            x, bias, ln_w, ln_b, eps, sum_row_valid, normed_row_valid, rows, self.d, self.blocks,
            self.timeout_ms, parts_local=from_owners, signal_bytes=self.signal_bytes,
            status=self.status.data_ptr())

    def failed(self) -> bool:
        """Whether a finished call of this group timed out (no device sync:
        reads the pinned status word; a call still running is not seen)."""
        return int(self.status[0]) != 0

    def check(self) -> None:
        """Raise PeerTimeoutError (and mark the group poisoned) if a call timed out."""
        if self.poisoned or self.failed():
            self.poisoned = True
            raise PeerTimeoutError(
                f"dotl_allreduce_ln on rank {self.rank} of {self.world} gave up waiting for a peer "
                f"(timeout {self.timeout_ms} ms); its outputs are not valid and the peer group must be "
                "rebuilt by every rank")

    def scatter_ok(self, rows: int) -> bool:
        """Whether row-parallel GEMMs over `rows` rows can scatter their tiles
        to the row owners (dotl_linear_peer): push mode, and 128-row blocks
        that never straddle two ranks."""
        return self.push and rows <= self.rows and rows % (128 * self.world) == 0

    def gemm_to_owners(self, a16: torch.Tensor, w16: torch.Tensor, rows: int) -> None:
        """part = a16 @ w16^T, each 128-row tile stored into the `recv` slot
        (this rank's) of the rank that owns its rows."""
        per = rows // self.world
        slot = self.rank * per * self.d * 4
        self.k.linear_peer(a16, w16, None, [p + slot for p in self.ptrs["recv"]], per, self.d)

    def _release(self) -> None:
        for p in self._opened:
            self.k.ipc_close(p)
        self._opened = []
        for p in self._own.values():
            self.k.peer_free(p)
        self._own = {}

    def close(self) -> None:
        """Collective: every rank unmaps its peers' buffers, then frees its own."""
        if not self._own:
            return
        torch.cuda.synchronize(self.device)
        for p in self._opened:
            self.k.ipc_close(p)
        self._opened = []
        self.dist.barrier(group=self.group)
        for p in self._own.values():
            self.k.peer_free(p)
        self._own = {}
