"""Plain, bounded snapshots of trainer state for ``torch.save``.

The trainer's stats hold nested records (planner decisions, reconfiguration
results, per-phase timings) that may share or even contain one another.  A
checkpoint must never fail to pickle because of that, nor grow without bound,
so ``snapshot`` turns a value into plain containers of scalars and strings:

* dicts (keys as strings), lists and tuples are copied element by element;
* tensors become Python numbers (one element) or lists (small), otherwise a
  short ``"<tensor shape dtype>"`` description;
* dataclasses become dicts; anything else becomes its ``repr`` (cut short);
* a container met again on its own path is replaced by
  ``"<recursive-reference>"``; below ``max_depth`` nested levels a container
  becomes ``"<max-depth>"``.

Reference behaviour: ``trainer/async_rl_trainer.py`` keeps checkpoint
snapshots acyclic and depth-limited (``tests/test_checkpoint_snapshot.py``).
"""

from __future__ import annotations

import dataclasses
import math
from typing import Any

RECURSIVE = "<recursive-reference>"
TOO_DEEP = "<max-depth>"


def snapshot(value: Any, max_depth: int = 32, max_tensor_elems: int = 64, max_repr: int = 200) -> Any:
    def go(v: Any, depth: int, path: frozenset) -> Any:
        if v is None or isinstance(v, (bool, int, str)):
            return v
        if isinstance(v, float):
            return v if math.isfinite(v) else str(v)
        try:
            import torch

            if isinstance(v, torch.Tensor):
                if v.numel() == 1:
                    return v.detach().cpu().item()
                if v.numel() <= max_tensor_elems:
                    return v.detach().cpu().tolist()
                return f"<tensor {tuple(v.shape)} {str(v.dtype).replace('torch.', '')}>"
        except ImportError:  # pragma: no cover
            pass
        if dataclasses.is_dataclass(v) and not isinstance(v, type):
            v = {f.name: getattr(v, f.name) for f in dataclasses.fields(v)}
        if isinstance(v, (dict, list, tuple, set, frozenset)):
            if id(v) in path:
                return RECURSIVE
            if depth >= max_depth:
                return TOO_DEEP
            inner = path | {id(v)}
            if isinstance(v, dict):
                return {str(k): go(x, depth + 1, inner) for k, x in v.items()}
            return [go(x, depth + 1, inner) for x in v]
        r = repr(v)
        return r if len(r) <= max_repr else r[:max_repr - 3] + "..."

    return go(value, 0, frozenset())
