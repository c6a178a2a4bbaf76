"""Paged KV cache: read lists over a pool of physical slots.

The reference's expansion walk can store physical KV slots instead of positions: with
MAP_SLOTS it loads row r's slot-table row ``slot_rows[r]`` and writes
``slot_table[slot_row, id]`` for the walked members and for the window / sink tail
(``src/lsa_rocm_lab/port/select_fused.py:147-148, 177-199``). ``map_slots`` is that mapping
as a pass over finished read lists (``lsa_map_slots``), so every selection arm composes
with it. ``PagedKV`` holds a slot pool ``k``/``v`` [1, slots, Hkv, D] and a slot table
[sequences, max_len] int32 (position -> slot, -1 unmapped); reading mapped lists over the
pool equals reading the position lists over each sequence's own cache.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from . import _lib
from ._lib import check, lib, ptr, require_cuda, stream_of


@dataclass
class PagedKV:
    k: torch.Tensor  # [1, slots, Hkv, D]
    v: torch.Tensor  # [1, slots, Hkv, D]
    slot_table: torch.Tensor  # [sequences, max_len] int32, -1 unmapped


def map_slots(lists: torch.Tensor, lengths: torch.Tensor, slot_table: torch.Tensor,
              slot_rows: torch.Tensor) -> torch.Tensor:
    """lists [R, width] int32 positions -> [R, width] int32 slots (a new tensor): entry j < length
    of row r becomes slot_table[slot_rows[r], lists[r, j]]; -1 past the length, for positions
    outside the table, or for a slot row outside it."""
    require_cuda(lists, lengths, slot_table, slot_rows, what="map_slots")
    if lists.dim() != 2 or slot_table.dim() != 2:
        raise ValueError("map_slots takes lists [R, width] and a slot table [rows, cols]")
    R, width = lists.shape
    lists = lists.to(torch.int32).contiguous()
    lengths = lengths.reshape(-1).to(torch.int32).contiguous()
    table = slot_table.to(torch.int32).contiguous()
    rows = slot_rows.reshape(-1).to(torch.int32).contiguous()
    if lengths.numel() != R or rows.numel() != R:
        raise ValueError("map_slots: one length and one slot row per list row")
    out = torch.empty_like(lists)
    check(lib().lsa_map_slots(ptr(lists), ptr(lengths), R, width, ptr(table), table.shape[0], table.shape[1],
                              table.shape[1], ptr(rows), ptr(out), stream_of(lists)), "map_slots")
    return out


def pack_paged(k: torch.Tensor, v: torch.Tensor, lengths, page: int = 64, generator=None, spare_pages: int = 0):
    """Copy per-sequence caches k/v [B, T, Hkv, D] (sequence b holds lengths[b] positions) into a
    paged pool: every sequence gets ceil(length / page) pages drawn from a shuffled free list
    (a page allocator's state after churn), positions map to slots page by page."""
    B, T, Hkv, D = k.shape
    dev = k.device
    lengths = [int(x) for x in lengths]
    n_pages = [(L + page - 1) // page for L in lengths]
    total = sum(n_pages) + spare_pages
    order = torch.randperm(total, generator=generator, device="cpu").to(dev)
    pool_k = torch.zeros(1, total * page, Hkv, D, dtype=k.dtype, device=dev)
    pool_v = torch.zeros_like(pool_k)
    table = torch.full((B, T), -1, dtype=torch.int32, device=dev)
    at = 0
    for b, (L, n) in enumerate(zip(lengths, n_pages)):
        pages = order[at:at + n]
        at += n
        pos = torch.arange(L, device=dev)
        slots = pages[pos // page] * page + pos % page
        table[b, :L] = slots.to(torch.int32)
        pool_k[0, slots] = k[b, :L]
        pool_v[0, slots] = v[b, :L]
    return PagedKV(pool_k, pool_v, table)


def paged_read(q: torch.Tensor, kv: PagedKV, lists: torch.Tensor, lengths: torch.Tensor, slot_rows: torch.Tensor,
               scale=None) -> torch.Tensor:
    """Read position lists [R, width] of query rows q [R, 1, Hq, D] over the pool: map, then one
    batched read with every row in the pool's single batch row. Output like q."""
    from .read_kernel_tiled import _read

    slots = map_slots(lists, lengths, kv.slot_table, slot_rows)
    R = q.shape[0]
    out = _read(q.reshape(1, R, q.shape[2], q.shape[3]), kv.k, kv.v, slots[None], lengths.reshape(1, R),
                q.shape[-1] ** -0.5 if scale is None else scale)
    return out.reshape(q.shape)
