"""Paged KV cache: the slot mapping of the expansion (select_fused.py MAP_SLOTS path) and
reads over a shuffled slot pool.

* ``lsa_map_slots`` equals the CPU checker's ``map_slots`` entry for entry (ids outside the
  table, pads, rows past their length, slot rows outside the table);
* batched decode over a paged pool (pages of 64 positions from a shuffled free list) equals
  the unpaged batched decode byte for byte: the same rows in the same list order reach the
  same read plan, so the arithmetic is identical.
"""

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"


def test_map_slots_vs_oracle(oracle, lsa):
    from lsa_b200 import paged

    rng = np.random.default_rng(3)
    R, width, rows, cols = 37, 300, 5, 1000
    lists = rng.integers(-2, cols + 20, (R, width)).astype(np.int32)
    lengths = rng.integers(-1, width + 5, R).astype(np.int32)
    table = rng.integers(-1, 1 << 20, (rows, cols)).astype(np.int32)
    srows = rng.integers(-1, rows + 1, R).astype(np.int32)
    want = oracle.map_slots(lists, lengths, table, srows)
    t = lambda x: torch.from_numpy(x).to(DEV)
    got = paged.map_slots(t(lists), t(lengths), t(table), t(srows))
    assert np.array_equal(got.cpu().numpy(), want)


@pytest.mark.parametrize("top_p,top_k", [(8, 512), (64, 4096)])
def test_paged_batched_decode_equals_unpaged(lsa, top_p, top_k):
    from lsa_b200 import batched, paged
    from lsa_b200.index_space import index_keys, index_queries

    cfg = lsa.PortConfig(cluster_block_size=512, pool_size=4, bucket_size=64, bucket_cap=128, top_p=top_p,
                         top_k=top_k, window_size=64, sink_size=4)
    lengths = [9000, 4096, 300, 12345, 7001]
    B, Tmax, Hq, Hkv, D = len(lengths), max(lengths), 32, 8, 128
    g = torch.Generator(device=DEV)
    g.manual_seed(top_p)
    q = torch.randn(B, 1, Hq, D, generator=g, device=DEV).to(torch.bfloat16)
    k = torch.randn(B, Tmax, Hkv, D, generator=g, device=DEV).to(torch.bfloat16)
    v = torch.randn(B, Tmax, Hkv, D, generator=g, device=DEV).to(torch.bfloat16)
    iq = torch.cat([index_queries(q[b], Hkv) for b in range(B)])
    bb = batched.concat_buckets([lsa.build_buckets_gpu(index_keys(k[b, :L]), cfg) for b, L in enumerate(lengths)])
    pos = torch.tensor([L - 1 for L in lengths], dtype=torch.int32, device=DEV)
    want = batched.batched_decode(q, k, v, iq, pos, bb, cfg, D ** -0.5)
    cpu = torch.Generator()
    cpu.manual_seed(11)
    kv = paged.pack_paged(k, v, lengths, page=64, generator=cpu, spare_pages=7)
    lists, lens = batched.batched_select(iq, pos, bb, cfg)
    got = paged.paged_read(q, kv, lists, lens, torch.arange(B, dtype=torch.int32, device=DEV), D ** -0.5)
    assert torch.equal(got, want)
    slots = paged.map_slots(lists, lens, kv.slot_table, torch.arange(B, dtype=torch.int32, device=DEV))
    for b, L in enumerate(lengths):  # every listed slot holds the listed position's key row
        n = int(lens[b])
        assert torch.equal(kv.k[0, slots[b, :n].long()], k[b, lists[b, :n].long()])
