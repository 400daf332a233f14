"""The optimized transformer layer on B200 (optimized/__init__.py upstream).

Same modules and reading order as the reference package:

    config.py    the knobs (names kept; values this build lacks are refused)
    cli.py       --attn-impl / --cuda-graph / ... overrides
    model.py     OptimizedTransformer, the whole forward pass
    layers.py    the submodules, baseline-name-compatible
    kernels.py   dispatch into libdotl through kernel_ext (no fallbacks)
    graphs.py    CUDA graph capture and replay
    util.py      small shared helpers
    pipeline.py  HostPipeline: host-in/host-out batches with the copies
                 overlapped (no upstream counterpart)
    tensor_parallel.py  the layer split over the GPUs of one box (no
                 upstream counterpart)

A harness declares `class UserOptimizedTransformer(OptimizedTransformer,
BaselineTransformer)` exactly as upstream. The directory holding this package
(with kernel_ext.py and dotl_ops.py beside it) goes on sys.path, as the
reference's project root did.
"""

from . import cli, config, graphs, kernels, layers, util
from .model import OptimizedTransformer
from .pipeline import HostPipeline

__all__ = ["OptimizedTransformer", "HostPipeline", "cli", "config", "graphs", "kernels", "layers", "util"]
