"""Incremental index maintenance: keep a growing cache's buckets and node hierarchy current.

The reference rebuilds the index of the whole cache before selecting (its bench calls
``build_buckets_gpu`` / ``build_hierarchy_gpu`` on all index keys,
``src/lsa_rocm_lab/port/pipeline.py:71-116, 136-181``), and its tree decode replays the
hierarchy's growth page by page (``_growth_replay``, ``src/lsa_rocm_lab/port/_tree.py:100-142``).
Both builds are local: a cluster block's buckets depend only on that block's keys (pools,
Ward merge, member rows made absolute by the block's start), and a node block of a level
depends only on its ``node_cluster_block_size`` rows of the level below. So an append that
closes blocks only builds those blocks:

* positions arrive with their index keys (``IndexState.append``); keys of the open block wait
  in a block-sized buffer;
* every block that closes is built alone (``lsa_build_buckets`` over its keys, members
  offset by its start) and its buckets are appended;
* every node block that completes at any level is paired alone (``lsa_pair_to_size``,
  children offset by the block's first row) and its nodes are appended, up to ``top_level``.

The state after any sequence of appends equals ``build_buckets_gpu`` + ``build_hierarchy_gpu``
on all keys so far, bit for bit (tested). Tables live in capacity-doubling buffers; the
``buckets`` / ``hierarchy`` properties return views of the filled rows.
"""

from __future__ import annotations

import torch

from . import pipeline


class _Rows:
    """A row table [rows, *shape] that grows by doubling; ``view`` is the filled part."""

    def __init__(self, shape, dtype, device, capacity=64):
        self.buf = torch.empty((capacity, *shape), dtype=dtype, device=device)
        self.n = 0

    def extend(self, rows: torch.Tensor) -> None:
        need = self.n + rows.shape[0]
        if need > self.buf.shape[0]:
            cap = max(need, 2 * self.buf.shape[0])
            grown = torch.empty((cap, *self.buf.shape[1:]), dtype=self.buf.dtype, device=self.buf.device)
            grown[: self.n] = self.buf[: self.n]
            self.buf = grown
        self.buf[self.n:need] = rows
        self.n = need

    @property
    def view(self) -> torch.Tensor:
        return self.buf[: self.n]


class IndexState:
    """The index of one growing sequence (index dim d) under ``config``."""

    def __init__(self, d: int, config, device):
        pipeline._validate_build(config, d)
        self.config, self.d, self.device = config, d, torch.device(device)
        cap = config.bucket_cap
        self.positions = 0  # positions appended
        self.closed = 0  # positions covered by closed blocks
        self._pend = torch.empty(config.cluster_block_size, d, dtype=torch.float32, device=self.device)
        self._npend = 0  # keys of the open block, at the front of _pend
        self._cf = _Rows((d,), torch.float32, self.device)
        self._cb = _Rows((d,), torch.bfloat16, self.device)
        self._members = _Rows((cap,), torch.int32, self.device)
        self._sizes = _Rows((), torch.int32, self.device)
        self._sums = _Rows((d,), torch.float32, self.device)
        # per level: node centroids, children, key sums, and the child rows already paired
        self._levels: list[tuple[_Rows, _Rows, _Rows]] = []
        self._paired: list[int] = []

    # ---------------------------------------------------------------- views

    @property
    def buckets(self) -> pipeline.Buckets:
        return pipeline.Buckets(self._cb.view, self._members.view, self._sizes.view, centroids_f32=self._cf.view,
                                key_sums=self._sums.view)

    @property
    def hierarchy(self) -> pipeline.Hierarchy:
        h = pipeline.Hierarchy(bucket_key_sums=self._sums.view)
        for cent, kids, sums in self._levels:
            h.levels.append(pipeline.NodeLevel(cent.view, kids.view, sums.view))
        return h

    # ---------------------------------------------------------------- appends

    def append(self, index_keys: torch.Tensor) -> int:
        """Append the index keys [n, d] of the next n positions; returns the buckets added.

        Keys of the open block are copied into a block-sized buffer (one copy per call); a
        block closes as soon as its last key arrives."""
        pipeline.require_cuda(index_keys, what="IndexState.append")
        keys = index_keys.float().reshape(-1, self.d)
        n = keys.shape[0]
        self.positions += n
        block = self.config.cluster_block_size
        i, added = 0, 0
        if self._npend:  # complete the open block first
            take = min(block - self._npend, n)
            self._pend[self._npend:self._npend + take] = keys[:take]
            self._npend += take
            i = take
            if self._npend == block:
                added += self._close_blocks(self._pend)
                self._npend = 0
        whole = (n - i) // block * block  # whole blocks straight from the input
        if whole:
            added += self._close_blocks(keys[i:i + whole].contiguous())
            i += whole
        if i < n:  # the start of the next open block
            self._pend[: n - i] = keys[i:]
            self._npend = n - i
        return added

    def _close_blocks(self, keys: torch.Tensor) -> int:
        """Build the buckets of the closed blocks in ``keys`` (starting at ``self.closed``)."""
        b = pipeline.build_buckets_gpu(keys, self.config)
        start = self.closed
        members = torch.where(b.members >= 0, b.members + start, b.members)
        self._cf.extend(b.centroids_f32)
        self._cb.extend(b.centroids)
        self._members.extend(members)
        self._sizes.extend(b.sizes)
        self._sums.extend(b.key_sums)
        self.closed += keys.shape[0]
        self._grow_levels()
        return b.rows

    def _grow_levels(self) -> None:
        """Pair every node block completed at any level since the last append."""
        cfg = self.config
        size, block = cfg.node_bucket_size, cfg.node_cluster_block_size
        below = self._sums.view
        for level in range(cfg.top_level):
            done = self._paired[level] if level < len(self._paired) else 0
            full = below.shape[0] // block * block
            if full > done:
                blocks = (full - done) // block
                _, order, node_sums = pipeline._pair_to_size(below[done:full].reshape(blocks, block, -1), size)
                if level == len(self._levels):
                    self._levels.append((_Rows((self.d,), torch.float32, self.device),
                                         _Rows((size,), torch.int64, self.device),
                                         _Rows((self.d,), torch.float32, self.device)))
                    self._paired.append(0)
                sums = node_sums.reshape(-1, self.d)
                cent, kids, ksum = self._levels[level]
                cent.extend(pipeline._normalize(sums))
                kids.extend((order + done).view(-1, size))
                ksum.extend(sums)
                self._paired[level] = full
            if level >= len(self._levels):
                break
            below = self._levels[level][2].view
