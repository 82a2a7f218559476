"""Weight-sync copy plans: trainer TP-k shards -> rollout TP-m slices, checked
against slicing the full tensors (CPU), plus the kernel work list."""

import itertools

import pytest
import torch

from libra_b200.infra.sync.reshard import apply_plan, build_plan, plan_bytes, plan_items
from libra_b200.models.qwen3 import ParamLayout, get_config, param_shapes
from libra_b200.parallel.tensor_parallel import shard_full_params


def _full_params(cfg, seed=0):
    g = torch.Generator().manual_seed(seed)
    lay = ParamLayout(param_shapes(cfg, 1, 0))
    return {n: torch.randn(lay.shapes[n], generator=g).bfloat16() for n in lay.order}


def _flat(cfg, tp, rank, params):
    lay = ParamLayout(param_shapes(cfg, tp, rank))
    flat = torch.zeros(lay.numel, dtype=torch.bfloat16)
    views = lay.views(flat)
    for n, v in shard_full_params(params, cfg, tp, rank).items():
        views[n].copy_(v)
    return flat


@pytest.mark.parametrize("model,src_tp,dst_tp", [
    (m, s, d) for m in ("tiny",) for s, d in itertools.product((1, 2, 4), (1, 2, 4))
] + [("tiny-moe", 1, 2), ("tiny-moe", 2, 1), ("tiny-moe", 2, 2)])
def test_plan_reproduces_tp_slices(model, src_tp, dst_tp):
    cfg = get_config(model)
    full = _full_params(cfg)
    srcs = [_flat(cfg, src_tp, r, full) for r in range(src_tp)]
    for dst_rank in range(dst_tp):
        rects = build_plan(cfg, src_tp, dst_tp, dst_rank)
        want = _flat(cfg, dst_tp, dst_rank, full)
        got = torch.zeros_like(want)
        apply_plan(rects, srcs, got)
        assert torch.equal(got, want), (model, src_tp, dst_tp, dst_rank)
        # every element of the destination slice is written exactly once
        lay = ParamLayout(param_shapes(cfg, dst_tp, dst_rank))
        assert plan_bytes(rects) == 2 * sum(torch.Size(s).numel() for s in lay.shapes.values())


def test_kernel_items_cover_the_plan():
    """Replay the kernel's work list on host memory: same result as the plan."""
    cfg = get_config("tiny")
    full = _full_params(cfg, seed=3)
    srcs = [_flat(cfg, 2, r, full) for r in range(2)]
    want = _flat(cfg, 4, 1, full)
    rects = build_plan(cfg, 2, 4, 1)
    # fake address space: source r at 1 << 40 * (r + 1), destination at 1 << 44
    bases = [(1 << 40) * (r + 1) for r in range(2)]
    dst_base = 1 << 44
    items = plan_items(rects, bases, [2, 2], dst_base, item_bytes=4096)
    got = torch.zeros_like(want)
    for src, dst, shape, pitch, flags in items.tolist():
        rows, row_elems = shape >> 32, shape & 0xFFFFFFFF
        sp, dp = pitch >> 32, pitch & 0xFFFFFFFF
        r = max(i for i, b in enumerate(bases) if src >= b)
        so, do = (src - bases[r]) // 2, (dst - dst_base) // 2
        assert flags == 0 and rows * row_elems * 2 <= 4096 or rows == 1
        for k in range(rows):
            got[do + k * dp:do + k * dp + row_elems] = srcs[r][so + k * sp:so + k * sp + row_elems]
    assert torch.equal(got, want)


def test_request_validation_rejects_pickles():
    from libra_b200.infra.sync.peer_weight_sync import _validate

    with pytest.raises(ValueError):
        _validate({"src_tp": 1, "sources": ["gASVAAAAAAAAAAA="]})
    with pytest.raises(ValueError):
        _validate({"src_tp": 2, "sources": [{"dtype": "bfloat16"}]})
    _validate({"src_tp": 1, "sources": [{"dtype": "bfloat16", "ipc": "", "offset": 0}]})
