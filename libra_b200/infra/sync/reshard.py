"""Copy plans for resharding trainer weights into rollout tensor-parallel slices.

The trainer holds its weights as ``k`` tensor-parallel shards, each a flat
bf16 buffer laid out by ``ParamLayout(param_shapes(cfg, k, r))``; a rollout
bucket of TP degree ``m`` needs, on each of its ranks, a flat buffer laid out
by ``param_shapes(cfg, m, r')``.  Every TP-split parameter is split along one
axis of its full (TP=1) matrix, in *sections*: the q / k / v head blocks of
QKV, the gate / up halves of the gate-up projection, the whole vocabulary of
the embedding, the input columns of the o- and down-projections.  A rank holds
one contiguous range of every section, and its local tensor is those ranges
concatenated.  With more TP ranks than KV heads, neighbouring ranks hold the
same KV head (replicated).

``build_plan`` intersects, parameter by parameter, the ranges a destination
rank needs with the ranges each source rank holds (taking a replicated range
from the first source that has it) and emits 2-D rectangles in element
offsets of the two flat buffers.  ``apply_plan`` runs them with torch (the CPU
path and the oracle); ``DeviceReshard`` turns them into the address list of
the ``weight_reshard`` kernel, whose sources may be peer GPUs' buffers mapped
with CUDA IPC, so every byte moves once, over NVLink, with no gather on the
trainer side (the reference gathers full HF tensors on trainer rank 0 and
broadcasts them through a separate NCCL communicator,
``infra/sync/nccl_weight_sync.py:126-197``).
"""

from __future__ import annotations

import base64
import math
from dataclasses import dataclass
from typing import Dict, List, Optional, Sequence, Tuple

import torch

from libra_b200.models.qwen3 import ParamLayout, Qwen3Config, param_shapes

# item rows are capped so one item moves at most this many bytes (grid balance)
ITEM_BYTES = 256 * 1024


@dataclass(frozen=True)
class Rect:
    """``rows`` rows of ``row_elems`` elements: source rank ``src`` at element
    offset ``src_off`` (pitch ``src_pitch``) -> destination offset ``dst_off``
    (pitch ``dst_pitch``)."""

    src: int
    src_off: int
    dst_off: int
    rows: int
    row_elems: int
    src_pitch: int
    dst_pitch: int


def _base(name: str) -> str:
    return name.split(".", 2)[-1] if name.startswith("layers.") else name


def split_axis(name: str) -> Optional[int]:
    """Axis of the local tensor along which TP splits ``name`` (None: replicated)."""
    b = _base(name)
    if b in ("qkv_proj", "gate_up_proj", "embed_tokens", "lm_head"):
        return 0
    if b in ("o_proj", "down_proj", "experts.w1"):
        return 1
    if b == "experts.w2":
        return 2
    return None


def local_ranges(name: str, cfg: Qwen3Config, tp: int, rank: int) -> List[Tuple[int, int, int]]:
    """(full start, length, local start) along the split axis for TP rank ``rank`` of ``tp``."""
    b = _base(name)
    D = cfg.head_dim
    nq, nkv = cfg.num_attention_heads, cfg.num_key_value_heads
    if b == "qkv_proj":
        nq_l, kv_l = nq // tp, max(1, nkv // tp)
        kv0 = rank * nkv // tp
        return [(rank * nq_l * D, nq_l * D, 0),
                (nq * D + kv0 * D, kv_l * D, nq_l * D),
                ((nq + nkv) * D + kv0 * D, kv_l * D, (nq_l + kv_l) * D)]
    if b == "gate_up_proj":
        F = cfg.intermediate_size
        Fl = F // tp
        return [(rank * Fl, Fl, 0), (F + rank * Fl, Fl, Fl)]
    if b == "experts.w1":
        F = cfg.moe_intermediate_size
        Fl = F // tp
        return [(rank * Fl, Fl, 0), (F + rank * Fl, Fl, Fl)]
    if b in ("embed_tokens", "lm_head"):
        Vl = cfg.vocab_size // tp
        return [(rank * Vl, Vl, 0)]
    if b == "o_proj":
        c = nq // tp * D
        return [(rank * c, c, 0)]
    if b == "down_proj":
        Fl = cfg.intermediate_size // tp
        return [(rank * Fl, Fl, 0)]
    if b == "experts.w2":
        Fl = cfg.moe_intermediate_size // tp
        return [(rank * Fl, Fl, 0)]
    raise ValueError(f"{name} is not split by tensor parallelism")


def _geometry(shape: Sequence[int], axis: int) -> Tuple[int, int, int]:
    """(outer count, local extent along axis, elements per axis step) of a row-major tensor."""
    outer = math.prod(shape[:axis])
    inner = math.prod(shape[axis + 1:])
    return outer, shape[axis], inner


def build_plan(cfg: Qwen3Config, src_tp: int, dst_tp: int, dst_rank: int) -> List[Rect]:
    """Rectangles that fill rank ``dst_rank`` of a TP-``dst_tp`` bucket from the
    ``src_tp`` trainer shards (element offsets in the flat buffers)."""
    src_layouts = [ParamLayout(param_shapes(cfg, src_tp, r)) for r in range(src_tp)]
    dst_layout = ParamLayout(param_shapes(cfg, dst_tp, dst_rank))
    rects: List[Rect] = []
    for name in dst_layout.order:
        dshape = dst_layout.shapes[name]
        doff = dst_layout.offsets[name]
        axis = split_axis(name)
        if axis is None:
            n = math.prod(dshape)
            rects.append(Rect(0, src_layouts[0].offsets[name], doff, 1, n, n, n))
            continue
        d_outer, d_ext, inner = _geometry(dshape, axis)
        for full0, length, local0 in local_ranges(name, cfg, dst_tp, dst_rank):
            need = [(full0, full0 + length)]
            for s in range(src_tp):
                if not need:
                    break
                sshape = src_layouts[s].shapes[name]
                s_outer, s_ext, s_inner = _geometry(sshape, axis)
                soff = src_layouts[s].offsets[name]
                still = []
                for lo, hi in need:
                    covered = []
                    for sf0, slen, sl0 in local_ranges(name, cfg, src_tp, s):
                        a, b = max(lo, sf0), min(hi, sf0 + slen)
                        if a >= b:
                            continue
                        covered.append((a, b))
                        src_pos, dst_pos = sl0 + (a - sf0), local0 + (a - full0)
                        if inner == 1 or axis == len(dshape) - 1:
                            # the split axis is the innermost one: a column range of every outer row
                            rects.append(Rect(s, soff + src_pos, doff + dst_pos, d_outer, b - a, s_ext, d_ext))
                        else:
                            # a run of whole rows inside every outer block
                            rects.append(Rect(s, soff + src_pos * inner, doff + dst_pos * inner, d_outer,
                                              (b - a) * inner, s_ext * inner, d_ext * inner))
                    still += _subtract((lo, hi), covered)
                need = still
            if need:
                raise RuntimeError(f"{name}: ranges {need} are held by no source shard")
    return rects


def _subtract(span: Tuple[int, int], covered: List[Tuple[int, int]]) -> List[Tuple[int, int]]:
    out, cur = [], span[0]
    for a, b in sorted(covered):
        if a > cur:
            out.append((cur, a))
        cur = max(cur, b)
    if cur < span[1]:
        out.append((cur, span[1]))
    return out


def plan_bytes(rects: Sequence[Rect], dst_elem_bytes: int = 2) -> int:
    return sum(r.rows * r.row_elems for r in rects) * dst_elem_bytes


def apply_plan(rects: Sequence[Rect], src_flats: Sequence[torch.Tensor], dst_flat: torch.Tensor) -> None:
    """Execute a plan with torch strided copies (CPU path; oracle for the kernel)."""
    with torch.no_grad():
        for r in rects:
            src = src_flats[r.src]
            s = torch.as_strided(src, (r.rows, r.row_elems), (r.src_pitch, 1), src.storage_offset() + r.src_off)
            d = torch.as_strided(dst_flat, (r.rows, r.row_elems), (r.dst_pitch, 1),
                                 dst_flat.storage_offset() + r.dst_off)
            d.copy_(s)


def plan_items(rects: Sequence[Rect], src_addrs: Sequence[int], src_elem_bytes: Sequence[int], dst_addr: int,
               item_bytes: int = ITEM_BYTES) -> torch.Tensor:
    """Kernel work list (int64 [n, 5]): absolute addresses, shapes and pitches,
    with every rectangle cut into items of at most ``item_bytes`` destination bytes."""
    rows_out = []
    cap = max(8, item_bytes // 2)  # destination elements per item
    for r in rects:
        se = int(src_elem_bytes[r.src])
        flags = 1 if se == 4 else 0
        src0, dst0 = int(src_addrs[r.src]) + r.src_off * se, dst_addr + r.dst_off * 2
        if r.row_elems >= cap:  # long rows: split each row into segments
            seg = cap // 8 * 8
            for row in range(r.rows):
                for c in range(0, r.row_elems, seg):
                    n = min(seg, r.row_elems - c)
                    rows_out.append((src0 + (row * r.src_pitch + c) * se, dst0 + (row * r.dst_pitch + c) * 2,
                                     (1 << 32) | n, (r.src_pitch << 32) | r.dst_pitch, flags))
        else:  # short rows: group whole rows
            per = max(1, cap // r.row_elems)
            for row in range(0, r.rows, per):
                n = min(per, r.rows - row)
                rows_out.append((src0 + row * r.src_pitch * se, dst0 + row * r.dst_pitch * 2,
                                 (n << 32) | r.row_elems, (r.src_pitch << 32) | r.dst_pitch, flags))
    return torch.tensor(rows_out, dtype=torch.int64).view(-1, 5)


class DeviceReshard:
    """A plan bound to concrete buffers on the destination GPU: ``run`` launches
    the ``weight_reshard`` kernel on the current stream.  ``src_addrs`` are
    device addresses readable from the destination GPU (its own memory or
    peer buffers mapped into its context)."""

    def __init__(self, cfg: Qwen3Config, src_tp: int, dst_tp: int, dst_rank: int, src_addrs: Sequence[int],
                 dst_flat: torch.Tensor, src_elem_bytes: Optional[Sequence[int]] = None, grid: int = 0):
        if dst_flat.dtype != torch.bfloat16 or not dst_flat.is_cuda:
            raise ValueError("the destination must be a bf16 CUDA buffer")
        self.rects = build_plan(cfg, src_tp, dst_tp, dst_rank)
        need = ParamLayout(param_shapes(cfg, dst_tp, dst_rank)).numel
        if dst_flat.numel() < need:
            raise ValueError(f"destination holds {dst_flat.numel()} elements, the layout needs {need}")
        se = list(src_elem_bytes) if src_elem_bytes is not None else [2] * src_tp
        self.items = plan_items(self.rects, src_addrs, se, int(dst_flat.data_ptr())).to(dst_flat.device)
        self.bytes = plan_bytes(self.rects)
        self.dst = dst_flat
        self.grid = int(grid)

    def run(self) -> int:
        from libra_b200 import ops

        ops.ext().weight_reshard(self.items, self.grid)
        return self.bytes


# ---------------------------------------------------------------------------
# handles: plain JSON descriptions of exported buffers (no pickled objects)
# ---------------------------------------------------------------------------

def export_buffer(t: torch.Tensor) -> Dict[str, object]:
    """JSON-safe description of a CUDA buffer for another process on this box:
    the IPC handle of its allocation (base64), the byte offset, dtype, numel."""
    from libra_b200 import ops

    handle, offset = ops.ext().ipc_export(t)
    return {"ipc": base64.b64encode(bytes(handle)).decode("ascii"), "offset": int(offset),
            "dtype": str(t.dtype).replace("torch.", ""), "numel": int(t.numel()), "device": int(t.device.index)}


_OPEN: Dict[Tuple[int, str], int] = {}


def open_buffer(desc: Dict[str, object], device: torch.device) -> int:
    """Map an exported buffer into ``device``'s context; returns the address of
    its first element (mappings are cached per (device, handle))."""
    from libra_b200 import ops

    if not isinstance(desc.get("ipc"), str) or not isinstance(desc.get("offset"), int):
        raise ValueError("malformed buffer description")
    raw = base64.b64decode(desc["ipc"], validate=True)
    key = (int(device.index), desc["ipc"])
    base = _OPEN.get(key)
    if base is None:
        with torch.cuda.device(device):
            base = ops.ext().ipc_open(raw)
        _OPEN[key] = base
    return base + int(desc["offset"])
