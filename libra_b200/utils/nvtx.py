"""NVTX ranges around the trainer's phases and the engines' hot regions.

Off unless ``LIBRA_NVTX=1`` (one environment read at import; ``set_enabled``
switches it at run time), so the default path costs one boolean test.  When
on, a profiler that records NVTX (Nsight Systems, ``ncu --nvtx``) sees the
phase names of the step: ``collect_batch``, ``recompute_logprobs``,
``grpo_update`` with ``forward_backward`` / ``grad_reduce`` /
``optimizer_step`` inside, ``weight_sync``, and the rollout engine's
``prefill`` / ``decode`` steps.

``nvtx_range`` nests (push/pop); ``range_start``/``range_end`` return and take
a handle, for phases whose start and end do not nest with others.
"""

from __future__ import annotations

import contextlib
import os
from typing import Optional

_enabled = os.environ.get("LIBRA_NVTX", "0") == "1"


def set_enabled(on: bool) -> None:
    global _enabled
    _enabled = bool(on)


def enabled() -> bool:
    return _enabled


def _nvtx():
    import torch

    return torch.cuda.nvtx


@contextlib.contextmanager
def nvtx_range(name: str):
    if not _enabled:
        yield
        return
    nv = _nvtx()
    nv.range_push(name)
    try:
        yield
    finally:
        nv.range_pop()


def range_start(name: str) -> Optional[int]:
    return _nvtx().range_start(name) if _enabled else None


def range_end(handle: Optional[int]) -> None:
    if handle is not None:
        _nvtx().range_end(handle)
