"""The D-LSA tree select on B200 - drop-in for ``lsa_rocm_lab.port._tree``.

Reference: AIwork4me/latent-sparse-attention-rocm, ``src/lsa_rocm_lab/port/_tree.py``
(switch ``:34-60``, beam ``:318-373``, growth replay ``:100-142``).

The beam runs as one ``lsa_tree_select`` call: for up to 64 rows one thread-block cluster
per row walks every level in one launch, else a launch per node level, top down, and one
for the buckets, each ordering its candidates in the row's last CTA (packed keys: score
first, the lower id on ties). The growth each query's page saw is computed in closed form
on the device - no host sync, CUDA-graph safe. ``tree_select_batched`` goes through
``lsa_tree_select_lists``: the cluster form expands the picks into read lists in the same
launch (the flat select's walk); otherwise the picks go through the expansion kernel.

``LSA_TREE_IMPL`` (``per_page`` default / ``batched``) names the reference's two torch
walks; both map to this one kernel, which is set-equal to either by construction. This
build emits only unique, valid picks (a short level pads with -1; the reference's batched
walk does the same, ``_tree.py:279-282``).
"""

from __future__ import annotations

import ctypes
import os

import torch

from . import _lib
from ._lib import check, lib, ptr, require_cuda, stream_of


def _beam(index_queries, positions, buckets, hierarchy, config):
    """The beam's operands (kept alive by the caller while the launch is queued) and the
    leading ctypes arguments of lsa_tree_select / lsa_tree_select_lists."""
    require_cuda(index_queries, positions, what="tree_select")
    if positions.shape[0] != index_queries.shape[0]:
        raise ValueError(f"a position a query: {index_queries.shape[0]} queries, {positions.shape[0]} positions")
    if config.start_nodes is not None:
        raise ValueError("the beam covers start_nodes=None (the top level down), as the reference's exact walk")
    if buckets.centroids_f32 is None:
        raise ValueError("tree_select scores buckets with centroids_f32")
    q = index_queries.float().contiguous()
    pos = positions.to(torch.int32).contiguous()
    R, d = q.shape
    levels = hierarchy.levels
    n = len(levels)
    counts = (ctypes.c_int64 * max(n, 1))(*[lv.centroids.shape[0] for lv in levels])
    cents = [lv.centroids.float().contiguous() for lv in levels]
    kids = [lv.children.to(torch.int64).contiguous() for lv in levels]
    cptrs = (ctypes.c_void_p * max(n, 1))(*[c.data_ptr() for c in cents])
    kptrs = (ctypes.c_void_p * max(n, 1))(*[c.data_ptr() for c in kids])
    bc = buckets.centroids_f32.float().contiguous()
    keep = (q, pos, cents, kids, bc, counts, cptrs, kptrs)
    lead = (ptr(q), R, d, ptr(pos), config.cluster_block_size, config.block_bucket_count, buckets.rows, n, cptrs, kptrs,
            counts, ptr(bc), config.node_bucket_size, config.node_cluster_block_size, config.top_level,
            config.beam_width, config.top_p)
    return keep, lead, R, n, counts


def _workspace(R, n, counts, config, dev, what):
    sb, nc = ctypes.c_int64(), ctypes.c_int64()
    check(lib().lsa_tree_plan(R, n, counts, config.beam_width, config.node_bucket_size,
                              config.node_cluster_block_size, config.block_bucket_count, config.top_p,
                              ctypes.byref(sb), ctypes.byref(nc)), what)
    return _lib.scratch(sb.value, dev), _lib.counters(nc.value, dev)


def tree_picks(index_queries, positions, buckets, hierarchy, config) -> torch.Tensor:
    """Best-first bucket picks [R, top_p] int32 (-1 padded) of the beam."""
    keep, lead, R, n, counts = _beam(index_queries, positions, buckets, hierarchy, config)
    dev = keep[0].device
    picks = torch.empty(R, config.top_p, dtype=torch.int32, device=dev)
    if R == 0:
        return picks
    sc, ct = _workspace(R, n, counts, config, dev, "tree_select")
    check(lib().lsa_tree_select(*lead, ptr(picks), ptr(sc), sc.numel(), ptr(ct), ct.numel(), stream_of(keep[0])),
          "tree_select")
    _lib.after_call(dev, "tree_select")
    return picks


def tree_select_batched(index_queries, positions, buckets, hierarchy, config, top_k=None):
    """Select by the beam, expand the picks into read lists (ref ``_tree.py:34-60``): one
    ``lsa_tree_select_lists`` call, one launch when the beam's cluster form takes the rows and
    the picked member rows fit its shared memory (else the beam, then the expansion kernel;
    the same lists)."""
    os.environ.get("LSA_TREE_IMPL", "per_page")  # both walks are this one kernel
    top_k = config.top_k if top_k is None else top_k
    keep, lead, R, n, counts = _beam(index_queries, positions, buckets, hierarchy, config)
    dev = keep[0].device
    width = top_k + config.window_size + config.sink_size
    lists = torch.empty(R, width, dtype=torch.int32, device=dev)
    lengths = torch.empty(R, dtype=torch.int32, device=dev)
    if R == 0:
        return lists, lengths
    mem = buckets.members.to(torch.int32).contiguous()
    picks = torch.empty(R, config.top_p, dtype=torch.int32, device=dev)
    sc, ct = _workspace(R, n, counts, config, dev, "tree_select")
    check(lib().lsa_tree_select_lists(*lead, ptr(mem), mem.shape[0], mem.shape[1], config.window_size,
                                      config.sink_size, top_k, ptr(picks), ptr(lists), ptr(lengths), ptr(sc),
                                      sc.numel(), ptr(ct), ct.numel(), stream_of(keep[0])), "tree_select")
    _lib.after_call(dev, "tree_select")
    return lists, lengths


def tree_select_per_page(index_queries, positions, buckets, hierarchy, config, top_k=None):
    """The reference's per-page walk entry (ref ``_tree.py:63-85``) - the same kernel."""
    return tree_select_batched(index_queries, positions, buckets, hierarchy, config, top_k)


__all__ = ["tree_picks", "tree_select_batched", "tree_select_per_page", "_lib"]
