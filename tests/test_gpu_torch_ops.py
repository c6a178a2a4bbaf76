"""The torch.library operators (``torch.ops.lsa.*``, lsa_b200/_lsa_torch_ops.so) on the GPU:
byte-identical to the same C-ABI entry points called directly (same kernels, same plans), on
torch's current stream, and traceable into one graph by torch.compile (fullgraph, eager
backend: the ops are opaque graph nodes with Meta shapes)."""

import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _inputs(seed=3, Tk=4096, width=2116):
    g = torch.Generator(device=DEV)
    g.manual_seed(seed)
    q = torch.randn(1, 1, 32, 128, generator=g, device=DEV).bfloat16()
    k = torch.randn(1, Tk, 8, 128, generator=g, device=DEV).bfloat16()
    v = torch.randn(1, Tk, 8, 128, generator=g, device=DEV).bfloat16()
    ids = torch.randint(-1, Tk, (1, 1, width), generator=g, device=DEV, dtype=torch.int32)
    lengths = torch.tensor([[width - 7]], device=DEV, dtype=torch.int32)
    return q, k, v, ids, lengths


def test_sparse_read_op_equals_the_c_abi(lsa):
    from lsa_b200 import _lib

    q, k, v, ids, lengths = _inputs()
    got = _lib.torch_ops().sparse_read(q, k, v, ids, lengths, 128 ** -0.5)
    L = _lib.lib()
    s, sb, nc = ctypes.c_int64(), ctypes.c_int64(), ctypes.c_int64()
    assert L.lsa_sparse_read_plan(1, 1, 32, 8, 128, ids.shape[-1], 0, ctypes.byref(s), ctypes.byref(sb),
                                  ctypes.byref(nc)) == 0
    sc = torch.empty(max(sb.value, 256), dtype=torch.uint8, device=DEV)
    ct = torch.zeros(max(nc.value, 64), dtype=torch.int32, device=DEV)
    want = torch.empty_like(q)
    rc = L.lsa_sparse_read(_lib.ptr(q), _lib.ptr(k), _lib.ptr(v), _lib.BF16, _lib.ptr(ids), _lib.ptr(lengths), 1, 1,
                           4096, 32, 8, 128, ids.shape[-1], 128 ** -0.5, _lib.ptr(want), _lib.ptr(sc), sc.numel(),
                           _lib.ptr(ct), ct.numel(), 0, _lib.stream_of(q))
    assert rc == 0
    torch.cuda.synchronize()
    assert torch.equal(got, want)


def test_ops_run_on_the_current_stream(lsa):
    from lsa_b200 import _lib

    q, k, v, ids, lengths = _inputs(seed=4)
    ref = _lib.torch_ops().sparse_read(q, k, v, ids, lengths, 128 ** -0.5)
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        out = _lib.torch_ops().sparse_read(q, k, v, ids, lengths, 128 ** -0.5)
    torch.cuda.current_stream().wait_stream(side)
    assert torch.equal(out, ref)


def test_decode_traces_into_one_graph(lsa):
    """make_index_space -> flat_select(fused) -> lsa_read as torch ops under torch.compile
    (fullgraph): no graph break, and the compiled step returns what the eager step does."""
    from lsa_b200 import _lib

    ops = _lib.torch_ops()
    rng = np.random.default_rng(9)
    T = 2048
    q = torch.from_numpy(rng.standard_normal((1, T, 32, 128)).astype(np.float32)).bfloat16().to(DEV)
    k = torch.from_numpy(rng.standard_normal((1, T, 8, 128)).astype(np.float32)).bfloat16().to(DEV)
    v = torch.from_numpy(rng.standard_normal((1, T, 8, 128)).astype(np.float32)).bfloat16().to(DEV)
    cfg = lsa.PortConfig(cluster_block_size=512, pool_size=4, bucket_size=64, bucket_cap=128, top_p=32, top_k=512,
                         window_size=64, sink_size=4)
    _, ik = lsa.make_index_space(q, k)
    b = lsa.build_buckets_gpu(ik, cfg)
    pos = torch.tensor([T - 1], dtype=torch.int32, device=DEV)

    def step(qrow, klast):
        iq, _ = ops.regroup(qrow[0], klast)
        lists, lengths = ops.select_fused(iq, pos, b.centroids, b.members, 512, 8, 32, 64, 4, 512)
        return ops.sparse_read(qrow, k, v, lists[None], lengths[None], 128 ** -0.5)

    qrow, klast = q[:, -1:].contiguous(), k[0, -1:].contiguous()
    want = step(qrow, klast)
    got = torch.compile(step, backend="eager", fullgraph=True)(qrow, klast)
    assert torch.equal(got, want)
