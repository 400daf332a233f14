"""Whole-forward CUDA graph capture and replay (the role of optimized/graphs.py
upstream: `_graph_key`, `_graph_eligible`, `_capture_graph`, `_GraphRunner`).

A forward of 1 + 5..8 * num_layers kernel launches becomes one graph launch
plus the copy of x (and the mask) into the graph's input buffers and the copy
of its output out. How this build does it:

* What a graph depends on. The kernels read fp16 / fp32 copies of the weights
  that the layers cache per parameter version, and a graph bakes in the
  addresses of those copies. So a runner records the fingerprint of the
  parameters it was captured under (each parameter's storage address and
  version counter). `OptimizedTransformer.forward` compares it with the live
  fingerprint before every replay, so an in-place update (optimizer.step,
  param.copy_ or mul_ under no_grad) or a reload retires the runner, and the
  next call captures again from the new weights.
* How it is captured. The capturing call runs the forward eagerly on a side
  stream with the caller's own input first. That run builds every lazily
  created cache, and its output, which the call returns, is also the reference
  for a bit-exact check of one replay. A graph whose replay differs, or whose
  capture rebuilt a weight cache, is dropped and the key stays eager.
* Lifetime. The graphs belong to their model. A `weakref.finalize` on the
  model releases them when the model is collected, and at interpreter exit
  while CUDA is still up; `release_graphs()` does it on demand (before a
  process group that a graph's kernels use is torn down, for instance).
"""

from __future__ import annotations

import weakref
from typing import Dict, Optional, Tuple

import torch

from . import config
from .kernels import _custom_kernels
from .util import _version_or_none

_warned = False


def _note_once(msg: str) -> None:
    global _warned
    if not _warned:
        _warned = True
        print(f"[info] {msg}")


class _GraphRunner:
    """One captured forward: the graph, the input/output buffers whose
    addresses it holds, and the weight fingerprint it is valid for."""

    __slots__ = ("graph", "stream", "static_x", "static_mask", "static_out", "needs_mask",
                 "fingerprint", "keep_alive", "replays")

    def __init__(self, graph, stream, static_x, static_mask, static_out, needs_mask, fingerprint,
                 keep_alive):
        self.graph = graph
        self.stream = stream
        self.static_x = static_x
        self.static_mask = static_mask
        self.static_out = static_out
        self.needs_mask = needs_mask
        self.fingerprint = fingerprint
        self.keep_alive = keep_alive      # the weight caches the kernels read
        self.replays = 0

    def replay(self, x: torch.Tensor, mask: Optional[torch.Tensor],
               out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """Copy the inputs in, replay, and return the output copied out of the
        graph's buffer (the next replay rewrites that buffer): into `out`
        when given, else into a new tensor."""
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
        if self.graph is not None:
            try:
                self.graph.reset()
            except Exception:  # noqa: BLE001 - a graph whose capture failed may refuse reset
                pass
        self.graph = self.stream = None
        self.static_x = self.static_mask = self.static_out = None
        self.keep_alive = ()


def _graph_key(x: torch.Tensor, use_mask: bool) -> Tuple:
    """What makes two calls interchangeable to one captured graph."""
    return (tuple(x.shape), x.dtype, x.device.index, use_mask, config.ATTENTION_IMPL,
            config.ATTENTION_PRECISION, config.GEMM_PRECISION)


def _graph_eligible(x: torch.Tensor, entries: int, gemm_flops: float = 0.0) -> bool:
    """Cheap per-call gate; pure Python, no GPU calls. gemm_flops: the
    forward's GEMM work, for the size gate."""
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
    return (x.shape[0] * x.shape[1] * x.shape[2] <= config._GRAPH_MAX_ACTIVATION
            and gemm_flops <= config._GRAPH_MAX_GEMM_FLOPS)


def _weights_fingerprint(model) -> Tuple:
    """(storage address, version) of every parameter: changes whenever a
    weight is edited in place, reloaded or moved."""
    return tuple((p.data_ptr(), _version_or_none(p)) for p in model.parameters())


def _weight_caches(model) -> Tuple:
    """The cached weight copies the kernels read (the tensors a graph holds
    the addresses of)."""
    out = []
    for layer in model.layers:
        attn = layer.attention
        out += [attn._qkv_weight, attn._qkv_bias, attn.out_proj._w16, layer.ffn_in._w16, layer.ffn_out._w16,
                attn._qkv_pair, attn.out_proj._wpair, layer.ffn_in._wpair, layer.ffn_out._wpair]
        for mod in (layer.norm1, layer.norm2, attn.out_proj, layer.ffn_in, layer.ffn_out):
            out += [entry[1] for entry in mod.__dict__.get("_f32_cache", {}).values()]
    out += [entry[1] for entry in model.final_norm.__dict__.get("_f32_cache", {}).values()]
    return tuple(out)


def _capture_graph(model, x: torch.Tensor, mask: Optional[torch.Tensor],
                   use_mask: bool) -> Tuple[Optional[_GraphRunner], torch.Tensor]:
    """Runs model._forward_eager(x, mask) and tries to capture it.

    Returns (runner or None, this call's output). The output is the eager
    result, so the capturing call costs one eager forward plus the capture."""
    dev = x.device
    _custom_kernels()
    side = torch.cuda.Stream(device=dev)
    side.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(side):
        eager = model._forward_eager(x, mask, use_mask)
    torch.cuda.current_stream(dev).wait_stream(side)
    eager.record_stream(torch.cuda.current_stream(dev))   # made on `side`, read by the caller's stream
    free, _total = torch.cuda.mem_get_info(dev)
    if free < config._GRAPH_MIN_FREE_BYTES:
        return None, eager
    graph = None
    try:
        with torch.inference_mode(False), torch.no_grad():
            static_x = x.detach().clone()
            static_mask = mask.detach().clone() if use_mask else None
            fingerprint = _weights_fingerprint(model)
            caches = _weight_caches(model)
            torch.cuda.synchronize(dev)
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=side):
                static_out = model._forward_eager(static_x, static_mask, use_mask)
            graph.replay()
            torch.cuda.synchronize(dev)
            same_caches = all(a is b for a, b in zip(caches, _weight_caches(model)))
            if not same_caches or fingerprint != _weights_fingerprint(model):
                raise RuntimeError("a weight cache was rebuilt during capture")
            if not torch.equal(static_out, eager):
                raise RuntimeError("graph replay did not reproduce the eager forward bit for bit")
    except Exception as exc:  # noqa: BLE001
        if graph is not None:
            try:
                graph.reset()
            except Exception:  # noqa: BLE001
                pass
        if torch.cuda.is_current_stream_capturing():
            raise RuntimeError(f"CUDA graph capture failed and left the stream capturing: {exc}") from exc
        torch.cuda.synchronize(dev)   # surfaces a broken context instead of hiding it
        _note_once(f"shape {tuple(x.shape)} stays eager (no CUDA graph): {type(exc).__name__}: {exc}")
        return None, eager
    return _GraphRunner(graph, side, static_x, static_mask, static_out, use_mask, fingerprint, caches), eager


class GraphCache:
    """A model's captured graphs by key, released with the model."""

    def __init__(self, owner) -> None:
        self.runners: Dict[Tuple, _GraphRunner] = {}
        self.declined: set = set()
        # runs when the owner is collected, or at interpreter exit
        self._finalizer = weakref.finalize(owner, GraphCache._release_all, self.runners)

    @staticmethod
    def _release_all(runners: Dict[Tuple, _GraphRunner]) -> None:
        for runner in runners.values():
            runner.release()
        runners.clear()

    def clear(self) -> None:
        self._release_all(self.runners)
        self.declined.clear()

    def get(self, key: Tuple, fingerprint_of) -> Optional[_GraphRunner]:
        """The runner for `key` if it was captured under the current weights;
        a runner whose weights changed is released and forgotten."""
        runner = self.runners.get(key)
        if runner is not None and runner.fingerprint != fingerprint_of():
            runner.release()
            del self.runners[key]
            runner = None
        return runner

    def __len__(self) -> int:
        return len(self.runners)

    def values(self):
        return self.runners.values()
