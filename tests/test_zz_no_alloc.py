"""The no-allocation read entry point (lsa_sparse_read_noalloc) against the regular one.

lsa_sparse_read_noalloc exists for callers that cannot allocate device memory - a server
whose device memory is one arena owned by its own allocator, a plugin host that forbids
cudaMalloc once serving has started. Its scratch lives in fixed arrays inside the library
instead of caller buffers. This file is collected last (pytest orders files by name) so a
run that stops at the first failure has run every other test first; it passes alone in a
fresh process and after the rest.

Checks, through the C ABI: two calls in a row match lsa_sparse_read's output within the
bf16 read tolerance (2e-2) - the second call proves the shared counters were left (or
made) zero by the first; and a call whose plan exceeds the arrays is refused with
LSA_ERR_SIZE without launching.
"""

import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

LSA_ERR_SIZE = -5
TOL_BF16 = 2e-2


def _inputs(Tk=4096, Hq=32, Hkv=8, D=128, width=2116, seed=7):
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    q = torch.randn(1, 1, Hq, D, generator=g, device="cuda").bfloat16()
    k = torch.randn(1, Tk, Hkv, D, generator=g, device="cuda").bfloat16()
    v = torch.randn(1, Tk, Hkv, D, generator=g, device="cuda").bfloat16()
    ids = torch.randint(0, Tk, (1, width), generator=g, device="cuda", dtype=torch.int32)
    ids[0, 100:110] = -1
    lengths = torch.tensor([width - 5], device="cuda", dtype=torch.int32)
    return q, k, v, ids, lengths


def _noalloc(L, q, k, v, ids, lengths, out, scale):
    B, Tq, Hq, D = q.shape
    Tk, Hkv = k.shape[1], k.shape[2]
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    return L.lsa_sparse_read_noalloc(ctypes.c_void_p(q.data_ptr()), ctypes.c_void_p(k.data_ptr()),
                                     ctypes.c_void_p(v.data_ptr()), 2, ctypes.c_void_p(ids.data_ptr()),
                                     ctypes.c_void_p(lengths.data_ptr()), B, Tq, Tk, Hq, Hkv, D, ids.shape[-1], scale,
                                     ctypes.c_void_p(out.data_ptr()), 0, stream)


def test_noalloc_read_matches_regular_read_twice():
    from lsa_b200 import _lib
    from lsa_b200.read_kernel_tiled import sparse_read_auto

    L = _lib.lib()
    q, k, v, ids, lengths = _inputs()
    scale = 128 ** -0.5
    want = sparse_read_auto(q, k, v, ids[None], lengths[None], scale)
    for call in range(2):
        out = torch.full_like(q, float("nan"))
        rc = _noalloc(L, q, k, v, ids, lengths, out, scale)
        assert rc == 0, f"call {call}: status {rc}"
        torch.cuda.synchronize()
        err = float((out.float() - want.float()).abs().max())
        assert np.isfinite(err) and err <= TOL_BF16, f"call {call}: max abs {err}"


def test_noalloc_refuses_calls_beyond_its_arrays():
    from lsa_b200 import _lib

    L = _lib.lib()
    # 4096 rows x 8 KV heads x 64 forced splits x 4 heads x 128 dims of fp32 partials: far above 8 MiB
    q = torch.zeros(1, 4096, 32, 128, device="cuda", dtype=torch.bfloat16)
    k = torch.zeros(1, 64, 8, 128, device="cuda", dtype=torch.bfloat16)
    ids = torch.zeros(4096, 2048, device="cuda", dtype=torch.int32)
    lengths = torch.full((4096,), 2048, device="cuda", dtype=torch.int32)
    out = torch.zeros_like(q)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    rc = L.lsa_sparse_read_noalloc(ctypes.c_void_p(q.data_ptr()), ctypes.c_void_p(k.data_ptr()),
                                   ctypes.c_void_p(k.data_ptr()), 2, ctypes.c_void_p(ids.data_ptr()),
                                   ctypes.c_void_p(lengths.data_ptr()), 1, 4096, 64, 32, 8, 128, 2048, 0.1,
                                   ctypes.c_void_p(out.data_ptr()), 64, stream)
    assert rc == LSA_ERR_SIZE
    torch.cuda.synchronize()
    assert float(out.float().abs().max()) == 0.0, "a refused call launches nothing"
