"""Whole-forward CUDA graph capture and replay (optimized/graphs.py upstream).

The forward is recorded once per key (shape, dtype, device, mask mode) and
replayed afterwards: one graph launch plus two input copies instead of
1 + 6 * num_layers kernel launches. Replay is verified bit-identical to eager
before a graph is installed; on any doubt capture declines and the caller
stays eager. Re-derived for B200: graphs are captured per device (one process
per GPU) and the size gate is B200's (config._GRAPH_MAX_ACTIVATION).
"""

from __future__ import annotations

import atexit
import weakref
from typing import Optional, Tuple

import torch

from . import config
from .kernels import _custom_kernels

_graph_warned = False


class _GraphRunner:
    """One captured CUDA graph plus the buffers whose addresses it baked in."""

    __slots__ = ("graph", "stream", "static_x", "static_mask", "static_out", "needs_mask",
                 "replays", "pinned", "__weakref__")

    def __init__(self, graph, stream, static_x, static_mask, static_out, needs_mask, pinned):
        self.graph = graph
        self.stream = stream
        self.static_x = static_x
        self.static_mask = static_mask
        self.static_out = static_out
        self.needs_mask = needs_mask
        self.pinned = pinned
        self.replays = 0

    def replay(self, x: torch.Tensor, mask: Optional[torch.Tensor],
               out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """Copy the inputs in, replay, return the output copied out of the
        graph's buffer (the next replay overwrites static_out in place): into
        `out` when given, else into a new tensor."""
        self.static_x.copy_(x)
        if self.needs_mask:
            self.static_mask.copy_(mask)
        self.graph.replay()
        self.replays += 1
        if out is None:
            return self.static_out.clone()
        out.copy_(self.static_out)
        return out

    def release(self) -> None:
        try:
            self.graph.reset()
        except Exception:  # noqa: BLE001 - reset on a half-captured graph may throw
            pass
        self.graph = None
        self.stream = None
        self.static_x = self.static_mask = self.static_out = None
        self.pinned = None


def _graph_key(x: torch.Tensor, use_mask: bool) -> Tuple:
    """What makes two calls interchangeable to one captured graph."""
    return (tuple(x.shape), x.dtype, x.device.index, use_mask, config.ATTENTION_IMPL,
            config.ATTENTION_PRECISION)


def _graph_eligible(x: torch.Tensor, entries: int) -> bool:
    """Cheap per-call gate; pure Python, no GPU calls."""
    if config.CUDA_GRAPH == "off":
        return False
    if x.device.type != "cuda" or x.dim() != 3:
        return False
    if torch.compiler.is_compiling() or torch.cuda.is_current_stream_capturing():
        return False
    if entries >= config._GRAPH_MAX_ENTRIES:
        return False
    if config.CUDA_GRAPH == "always":
        return True
    return x.shape[0] * x.shape[1] * x.shape[2] <= config._GRAPH_MAX_ACTIVATION


def _graph_cache_ptrs(model) -> Tuple:
    out = []
    for layer in model.layers:
        attn = layer.attention
        for t in (attn._qkv_weight, attn._qkv_bias, attn.out_proj._w16, layer.ffn_in._w16,
                  layer.ffn_out._w16):
            out.append(None if t is None else t.data_ptr())
    return tuple(out)


def _graph_pinned_refs(model) -> Tuple:
    out = []
    for layer in model.layers:
        attn = layer.attention
        out.extend((attn._qkv_weight, attn._qkv_bias, attn.out_proj._w16, layer.ffn_in._w16,
                    layer.ffn_out._w16))
    return tuple(out)


def _capture_graph(model, x: torch.Tensor, mask: Optional[torch.Tensor],
                   use_mask: bool) -> Optional[_GraphRunner]:
    """Capture model._forward_eager, or return None and leave the run eager."""
    global _graph_warned
    dev = x.device
    g = None
    try:
        _custom_kernels()
        free_bytes, _ = torch.cuda.mem_get_info(dev)
        if free_bytes < config._GRAPH_MIN_FREE_BYTES:
            return None
        with torch.inference_mode(False), torch.no_grad():
            static_x = torch.empty(x.shape, dtype=x.dtype, device=dev)
            static_mask = torch.empty(mask.shape, dtype=torch.bool, device=dev) if use_mask else None
            gen = torch.Generator(device=dev)
            gen.manual_seed(config._GRAPH_SEED)
            static_x.normal_(generator=gen)
            if use_mask:
                static_mask.fill_(True)
                static_mask[:, static_mask.shape[1] // 2:] = False
            side = torch.cuda.Stream(device=dev)
            side.wait_stream(torch.cuda.current_stream(dev))
            with torch.cuda.stream(side):
                for _ in range(config._GRAPH_WARMUP_ITERS):
                    model._forward_eager(static_x, static_mask, use_mask)
            torch.cuda.current_stream(dev).wait_stream(side)
            torch.cuda.synchronize(dev)
            ptrs_before = _graph_cache_ptrs(model)
            ref = model._forward_eager(static_x, static_mask, use_mask).clone()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=side):
                static_out = model._forward_eager(static_x, static_mask, use_mask)
            g.replay()
            torch.cuda.synchronize(dev)
            exact = torch.equal(static_out, ref)
            ptrs_after = _graph_cache_ptrs(model)
        if ptrs_after != ptrs_before or not exact:
            _graph_release(g)
            if not _graph_warned:
                _graph_warned = True
                print("[info] CUDA graph replay did not reproduce eager exactly (or a weight "
                      "cache moved during capture); this shape stays eager.")
            return None
        runner = _GraphRunner(g, side, static_x, static_mask, static_out, use_mask,
                              _graph_pinned_refs(model))
        _graph_register(runner)
        return runner
    except Exception as exc:  # noqa: BLE001
        _graph_release(g)
        try:
            if torch.cuda.is_current_stream_capturing():
                raise RuntimeError("stream is still capturing")
            torch.cuda.synchronize(dev)
        except Exception as fatal:  # noqa: BLE001
            raise RuntimeError("CUDA graph capture failed and left the CUDA context unusable. "
                               f"Original failure: {exc}") from fatal
        if not _graph_warned:
            _graph_warned = True
            print(f"[info] CUDA graph capture failed for shape {tuple(x.shape)}, running eagerly. "
                  f"Reason: {type(exc).__name__}: {exc}")
        return None


def _graph_release(g) -> None:
    if g is not None:
        try:
            g.reset()
        except Exception:  # noqa: BLE001
            pass


_graph_live: "weakref.WeakSet" = weakref.WeakSet()
_graph_atexit_registered = False


def _graph_register(runner: _GraphRunner) -> None:
    global _graph_atexit_registered
    _graph_live.add(runner)
    if not _graph_atexit_registered:
        _graph_atexit_registered = True
        atexit.register(_graph_release_all)


def _graph_release_all() -> None:
    """Drop every surviving graph while CUDA is still up. Safe to re-run."""
    for runner in list(_graph_live):
        try:
            runner.release()
        except Exception:  # noqa: BLE001
            pass
    _graph_live.clear()
