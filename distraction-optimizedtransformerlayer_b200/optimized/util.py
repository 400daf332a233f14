"""Small shared helpers (optimized/util.py upstream)."""

from __future__ import annotations

from typing import Optional

import torch


def _version_or_none(t: torch.Tensor) -> Optional[int]:
    """t._version, or None when the tensor does not track one (inference tensors)."""
    try:
        return t._version
    except RuntimeError:
        return None
