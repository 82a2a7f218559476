"""Paged KV cache with reference-counted, content-addressed (prefix-cached) blocks.

Layout per layer: K and V pools of shape [num_blocks, block_size, kv_heads, head_dim]
(bf16 on GPU).  A sequence owns a block table (list of block ids).  Full blocks
are hashed by (parent hash, token ids) so a new request whose prompt shares a
prefix with a cached sequence (the GRPO group members, or the next turn of a
multi-turn episode) reuses those blocks instead of recomputing them.
Replaces vLLM's paged KV + prefix cache used by the reference's rollout servers.
"""

from __future__ import annotations

import hashlib
from collections import OrderedDict
from dataclasses import dataclass, field
from typing import Dict, List, Optional, Tuple

import torch


def _block_hash(parent: str, tokens: List[int]) -> str:
    h = hashlib.blake2b(digest_size=16)
    h.update(parent.encode())
    h.update(",".join(map(str, tokens)).encode())
    return h.hexdigest()


@dataclass
class SequenceBlocks:
    blocks: List[int] = field(default_factory=list)
    num_tokens: int = 0          # tokens whose KV is written
    hashes: List[str] = field(default_factory=list)  # hash of each full block


class BlockAllocator:
    """Free list + refcounts + an LRU of unreferenced cached blocks."""

    def __init__(self, num_blocks: int, block_size: int):
        self.num_blocks, self.block_size = num_blocks, block_size
        self.refcount = [0] * num_blocks
        self.free: List[int] = list(range(num_blocks - 1, -1, -1))
        self.cached: Dict[str, int] = {}            # hash -> block
        self.block_hash: Dict[int, str] = {}
        self.evictable: "OrderedDict[int, None]" = OrderedDict()  # cached blocks with refcount 0

    def num_free(self) -> int:
        return len(self.free) + len(self.evictable)

    def allocate(self) -> int:
        if self.free:
            b = self.free.pop()
        elif self.evictable:
            b, _ = self.evictable.popitem(last=False)
            h = self.block_hash.pop(b, None)
            if h is not None and self.cached.get(h) == b:
                del self.cached[h]
        else:
            raise MemoryError("KV cache out of blocks")
        self.refcount[b] = 1
        return b

    def lookup(self, h: str) -> Optional[int]:
        b = self.cached.get(h)
        if b is None:
            return None
        if self.refcount[b] == 0:
            self.evictable.pop(b, None)
        self.refcount[b] += 1
        return b

    def register(self, b: int, h: str) -> None:
        if h not in self.cached:
            self.cached[h] = b
            self.block_hash[b] = h

    def release(self, b: int) -> None:
        self.refcount[b] -= 1
        if self.refcount[b] == 0:
            if b in self.block_hash:
                self.evictable[b] = None
            else:
                self.free.append(b)

    def clear_cache(self) -> None:
        """Forget every content hash (after a weight update the cached KV is stale)."""
        for b in list(self.evictable):
            self.free.append(b)
        self.evictable.clear()
        self.cached.clear()
        self.block_hash.clear()


class PagedKVCache:
    def __init__(self, num_layers: int, num_blocks: int, block_size: int, kv_heads: int, head_dim: int,
                 device, dtype=torch.bfloat16):
        self.num_layers, self.block_size = num_layers, block_size
        self.kv_heads, self.head_dim = kv_heads, head_dim
        shape = (num_layers, num_blocks, block_size, kv_heads, head_dim)
        self.k = torch.zeros(shape, dtype=dtype, device=device)
        self.v = torch.zeros(shape, dtype=dtype, device=device)
        self.alloc = BlockAllocator(num_blocks, block_size)
        self.seqs: Dict[str, SequenceBlocks] = {}

    @staticmethod
    def blocks_for_budget(budget_bytes: float, num_layers: int, block_size: int, kv_heads: int, head_dim: int,
                          dtype_bytes: int = 2) -> int:
        per_block = 2 * num_layers * block_size * kv_heads * head_dim * dtype_bytes
        return max(1, int(budget_bytes // per_block))

    # -------------------------------------------------------------- sequence ops
    def match_prefix(self, seq_id: str, tokens: List[int]) -> int:
        """Attach cached full blocks for the longest cached prefix; returns cached token count."""
        sb = self.seqs.setdefault(seq_id, SequenceBlocks())
        assert not sb.blocks, "prefix match only on a fresh sequence"
        parent = ""
        bs = self.block_size
        # never reuse the block holding the last prompt token: its logits must be recomputed
        limit = (max(len(tokens) - 1, 0) // bs) * bs
        for s in range(0, limit, bs):
            h = _block_hash(parent, tokens[s:s + bs])
            b = self.alloc.lookup(h)
            if b is None:
                break
            sb.blocks.append(b)
            sb.hashes.append(h)
            parent = h
        sb.num_tokens = len(sb.blocks) * bs
        return sb.num_tokens

    def reserve(self, seq_id: str, new_total_tokens: int) -> None:
        sb = self.seqs.setdefault(seq_id, SequenceBlocks())
        need = -(-new_total_tokens // self.block_size)
        while len(sb.blocks) < need:
            sb.blocks.append(self.alloc.allocate())

    def can_reserve(self, seq_id: str, new_total_tokens: int) -> bool:
        sb = self.seqs.get(seq_id)
        have = len(sb.blocks) if sb else 0
        return -(-new_total_tokens // self.block_size) - have <= self.alloc.num_free()

    def commit(self, seq_id: str, tokens: List[int]) -> None:
        """Mark KV of ``tokens`` (the full token list of the sequence so far) as written and
        publish newly completed full blocks to the prefix cache."""
        sb = self.seqs[seq_id]
        sb.num_tokens = len(tokens)
        bs = self.block_size
        while len(sb.hashes) < len(tokens) // bs:
            i = len(sb.hashes)
            parent = sb.hashes[-1] if sb.hashes else ""
            h = _block_hash(parent, tokens[i * bs:(i + 1) * bs])
            sb.hashes.append(h)
            self.alloc.register(sb.blocks[i], h)

    def commit_block(self, seq_id: str, num_tokens: int, block_tokens: List[int]) -> None:
        """Decode-path commit: ``num_tokens`` tokens now have KV; when that
        completes a block, ``block_tokens`` are its tokens and it is published
        to the prefix cache (same hash chain as ``commit``)."""
        sb = self.seqs[seq_id]
        sb.num_tokens = num_tokens
        bs = self.block_size
        if num_tokens % bs == 0 and len(sb.hashes) == num_tokens // bs - 1:
            parent = sb.hashes[-1] if sb.hashes else ""
            h = _block_hash(parent, block_tokens)
            sb.hashes.append(h)
            self.alloc.register(sb.blocks[len(sb.hashes) - 1], h)

    def free(self, seq_id: str) -> None:
        sb = self.seqs.pop(seq_id, None)
        if sb:
            for b in sb.blocks:
                self.alloc.release(b)

    def block_table(self, seq_ids: List[str], device) -> torch.Tensor:
        width = max((len(self.seqs[s].blocks) for s in seq_ids), default=1)
        tbl = torch.full((len(seq_ids), max(width, 1)), 0, dtype=torch.int32)
        for i, s in enumerate(seq_ids):
            bl = self.seqs[s].blocks
            if bl:
                tbl[i, :len(bl)] = torch.tensor(bl, dtype=torch.int32)
        return tbl.to(device, non_blocking=True)

    def slot_mapping(self, seq_id: str, start: int, end: int) -> torch.Tensor:
        """Flat slot index (block * block_size + offset) for token positions [start, end)."""
        bl = self.seqs[seq_id].blocks
        pos = torch.arange(start, end)
        blocks = torch.tensor(bl, dtype=torch.long)[pos // self.block_size]
        return blocks * self.block_size + pos % self.block_size

    def gather(self, layer: int, seq_id: str, length: int) -> Tuple[torch.Tensor, torch.Tensor]:
        """Contiguous K/V [length, kv_heads, D] of one sequence (prefill/extend attention)."""
        slots = self.slot_mapping(seq_id, 0, length).to(self.k.device)
        kf = self.k[layer].view(-1, self.kv_heads, self.head_dim)
        vf = self.v[layer].view(-1, self.kv_heads, self.head_dim)
        return kf.index_select(0, slots), vf.index_select(0, slots)

    def write(self, layer: int, slots: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> None:
        self.k[layer].view(-1, self.kv_heads, self.head_dim).index_copy_(0, slots, k)
        self.v[layer].view(-1, self.kv_heads, self.head_dim).index_copy_(0, slots, v)

    # -------------------------------------------------------------- migration between instances
    def cached_blocks(self, tokens: List[int]) -> List[Tuple[int, str]]:
        """(block, hash) of the longest run of full blocks of ``tokens`` that
        this cache holds in its prefix cache (read only: refcounts unchanged)."""
        out, parent, bs = [], "", self.block_size
        for s in range(0, (len(tokens) // bs) * bs, bs):
            h = _block_hash(parent, tokens[s:s + bs])
            b = self.alloc.cached.get(h)
            if b is None:
                break
            out.append((b, h))
            parent = h
        return out

    def import_blocks(self, src: "PagedKVCache", blocks: List[Tuple[int, str]]) -> int:
        """Copy ``src``'s cached blocks (a hash chain from ``cached_blocks``)
        into this cache as prefix-cached blocks, so the next request with that
        prefix here skips its prefill.  Every layer's K and V move in one
        gather + one peer copy + one scatter each (NVLink when the caches sit
        on different GPUs).  Stops at the free capacity.  Returns the tokens
        now cached here for that prefix."""
        if (src.num_layers, src.block_size, src.kv_heads, src.head_dim) != \
                (self.num_layers, self.block_size, self.kv_heads, self.head_dim):
            raise ValueError("KV caches of different shapes: migrate through a head reshard")

        def fetch(pos: List[int]):
            si = torch.tensor([blocks[i][0] for i in pos], dtype=torch.long, device=src.k.device)
            return src.k.index_select(1, si), src.v.index_select(1, si)

        return self._import([h for _, h in blocks], fetch)

    def block_hashes(self, tokens: List[int]) -> List[str]:
        """Prefix-cache hash chain of the full blocks of ``tokens``."""
        out, parent, bs = [], "", self.block_size
        for s in range(0, (len(tokens) // bs) * bs, bs):
            parent = _block_hash(parent, tokens[s:s + bs])
            out.append(parent)
        return out

    def export_blocks(self, blocks: List[Tuple[int, str]]) -> Tuple[torch.Tensor, torch.Tensor]:
        """K and V of ``blocks`` as [layers, blocks, block_size, kv_heads, head_dim]."""
        idx = torch.tensor([b for b, _ in blocks], dtype=torch.long, device=self.k.device)
        return self.k.index_select(1, idx), self.v.index_select(1, idx)

    def import_block_tensors(self, tokens: List[int], k: torch.Tensor, v: torch.Tensor) -> int:
        """Prefix-cache the blocks of ``tokens`` from K/V given as
        [layers, blocks, block_size, kv_heads, head_dim] (this cache's heads);
        block j holds tokens [j * block_size, (j + 1) * block_size)."""
        if k.shape != v.shape or tuple(k.shape[:1]) + tuple(k.shape[2:]) != \
                (self.num_layers, self.block_size, self.kv_heads, self.head_dim):
            raise ValueError(f"KV blocks of shape {tuple(k.shape)} do not fit this cache")
        hashes = self.block_hashes(tokens)[:k.shape[1]]

        def fetch(pos: List[int]):
            i = torch.tensor(pos, dtype=torch.long, device=k.device)
            return k.index_select(1, i), v.index_select(1, i)

        return self._import(hashes, fetch)

    def _import(self, hashes: List[str], fetch) -> int:
        """Register a hash chain as prefix-cached blocks; ``fetch(positions)``
        gives the K/V of the chain positions that are not cached here yet."""
        pinned, todo, have = [], [], 0
        for i, h in enumerate(hashes):
            if not todo and h in self.alloc.cached:
                pinned.append(self.alloc.lookup(h))  # keep the present head of the chain while allocating
                have += 1
            else:
                todo.append(i)
        todo = todo[:max(0, self.alloc.num_free())]
        dst = [self.alloc.allocate() for _ in todo]
        if todo:
            kk, vv = fetch(todo)
            di = torch.tensor(dst, dtype=torch.long, device=self.k.device)
            self.k.index_copy_(1, di, kk.to(self.k.device, self.k.dtype))
            self.v.index_copy_(1, di, vv.to(self.v.device, self.v.dtype))
        for b, i in zip(dst, todo):
            self.alloc.register(b, hashes[i])
            self.alloc.release(b)  # unreferenced and cached: reusable by a matching prefix
        for b in pinned:
            self.alloc.release(b)
        return (have + len(todo)) * self.block_size

    def usage(self) -> float:
        return 1.0 - self.alloc.num_free() / max(1, self.alloc.num_blocks)
