"""Command-line overrides for the knobs in config.py (optimized/cli.py upstream).

Same three hooks, so a harness written for the reference works unchanged:

    parse_args()     -> add_arguments(parser)
    validate_args()  -> validate_args(args, device, dtype)
    main()           -> apply_overrides(args)

The choices are the reference's. Values that would select an implementation
this build does not have are rejected by validate_args with the reason.
"""

from __future__ import annotations

import argparse

import torch

from . import config

_FLAGS = (
    ("--attn-backend", "attn_backend", ("custom",), "ATTENTION_BACKEND"),
    ("--attn-impl", "attn_impl", ("auto", "scalar", "wmma", "tile"), "ATTENTION_IMPL"),
    ("--attn-precision", "attn_precision", ("auto", "fp32", "tf32", "fp16", "bf16"), "ATTENTION_PRECISION"),
    ("--linear-gelu", "linear_gelu", ("auto", "tf32", "off"), "LINEAR_GELU"),
    ("--linear-bias", "linear_bias", ("auto", "tf32", "off"), "LINEAR_BIAS"),
    ("--layernorm", "layernorm", ("auto", "off"), "LAYERNORM"),
    ("--qkv-fp16", "qkv_fp16", ("auto", "off"), "QKV_FP16"),
    ("--normed-fp16", "normed_fp16", ("auto", "off"), "NORMED_FP16"),
    ("--cp-async", "cp_async", ("auto", "sync", "off"), "CP_ASYNC"),
    ("--cuda-graph", "cuda_graph", ("off", "auto", "always"), "CUDA_GRAPH"),
)


def add_arguments(parser: argparse.ArgumentParser) -> None:
    """Add the optimization flags to the harness's own parser."""
    for flag, dest, choices, knob in _FLAGS:
        parser.add_argument(flag, dest=dest, choices=choices, default=None,
                            help=f"override {knob} for this run only")


def apply_overrides(args: argparse.Namespace) -> None:
    """Write the requested overrides into config, before any model is built."""
    for _flag, dest, _choices, knob in _FLAGS:
        value = getattr(args, dest, None)
        if value is not None:
            setattr(config, knob, value)


def validate_args(args: argparse.Namespace, device: torch.device, dtype: torch.dtype) -> None:
    """Reject combinations this build cannot run, before anything is built."""
    saved = {knob: getattr(config, knob) for _f, _d, _c, knob in _FLAGS}
    try:
        apply_overrides(args)
        config.validate()
    finally:
        for knob, value in saved.items():
            setattr(config, knob, value)
    if device.type != "cuda":
        raise ValueError("the optimized model runs on CUDA (sm_100a) only")
