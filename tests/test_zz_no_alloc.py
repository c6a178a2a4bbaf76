"""The no-allocation read entry point (lsa_sparse_read_noalloc) against the regular one.

lsa_sparse_read_noalloc exists for callers that cannot allocate device memory - a server
whose device memory is one arena owned by its own allocator, a plugin host that forbids
cudaMalloc once serving has started. Its scratch lives in fixed arrays inside the library
instead of caller buffers. This file is collected last (pytest orders files by name) so a
run that stops at the first failure has run every other test first; it passes alone in a
fresh process and after the rest.

Checks, through the C ABI:
* two calls in a row, on the decode row's shape and on a larger batch that takes the
  split kernel with scratch partials (ticket merge), match lsa_sparse_read's output and
  the CPU checker within the bf16 read tolerance (2e-2) - the second call reuses the
  arrays exactly as the first one left them (each call zeroes only the counters it uses);
* the optional status output receives 0 (no bounded wait expired);
* a call whose plan exceeds the arrays is refused with LSA_ERR_SIZE without launching.
"""

import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

LSA_ERR_SIZE = -5
TOL_BF16 = 2e-2


def _inputs(Tq=1, Tk=4096, Hq=32, Hkv=8, D=128, width=2116, seed=7):
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    q = torch.randn(1, Tq, Hq, D, generator=g, device="cuda").bfloat16()
    k = torch.randn(1, Tk, Hkv, D, generator=g, device="cuda").bfloat16()
    v = torch.randn(1, Tk, Hkv, D, generator=g, device="cuda").bfloat16()
    ids = torch.randint(0, Tk, (Tq, width), generator=g, device="cuda", dtype=torch.int32)
    ids[:, 100:110] = -1
    lengths = torch.full((Tq,), width - 5, device="cuda", dtype=torch.int32)
    return q, k, v, ids, lengths


def _noalloc(L, q, k, v, ids, lengths, out, scale, status=None, splits=0):
    B, Tq, Hq, D = q.shape
    Tk, Hkv = k.shape[1], k.shape[2]
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    st = None if status is None else ctypes.c_void_p(status.data_ptr())
    return L.lsa_sparse_read_noalloc(ctypes.c_void_p(q.data_ptr()), ctypes.c_void_p(k.data_ptr()),
                                     ctypes.c_void_p(v.data_ptr()), 2, ctypes.c_void_p(ids.data_ptr()),
                                     ctypes.c_void_p(lengths.data_ptr()), B, Tq, Tk, Hq, Hkv, D, ids.shape[-1], scale,
                                     ctypes.c_void_p(out.data_ptr()), splits, st, stream)


@pytest.mark.parametrize("Tq,splits", [(1, 0), (6, 24)])
def test_noalloc_read_matches_regular_read_twice(oracle, Tq, splits):
    from lsa_b200 import _lib
    from lsa_b200.read_kernel_tiled import _read

    L = _lib.lib()
    q, k, v, ids, lengths = _inputs(Tq=Tq)
    scale = 128 ** -0.5
    want = _read(q, k, v, ids[None], lengths[None], scale, splits=splits)
    ref = oracle.sparse_read(q.float().cpu().numpy(), k.float().cpu().numpy(), v.float().cpu().numpy(),
                             ids[None].cpu().numpy(), lengths[None].cpu().numpy(), scale)
    for call in range(2):
        out = torch.full_like(q, float("nan"))
        status = torch.full((1,), 12345, dtype=torch.int32, device="cuda")
        rc = _noalloc(L, q, k, v, ids, lengths, out, scale, status, splits)
        assert rc == 0, f"call {call}: status {rc}"
        torch.cuda.synchronize()
        assert int(status.item()) == 0, f"call {call}: device status {int(status.item())}"
        err = float((out.float() - want.float()).abs().max())
        assert np.isfinite(err) and err <= TOL_BF16, f"call {call}: max abs {err} vs lsa_sparse_read"
        err = float(np.abs(out.float().cpu().numpy() - ref).max())
        assert err <= TOL_BF16, f"call {call}: max abs {err} vs the CPU checker"


def test_noalloc_refuses_calls_beyond_its_arrays():
    from lsa_b200 import _lib

    L = _lib.lib()
    # 4096 rows x 8 KV heads x 64 forced splits x 4 heads x 128 dims of fp32 partials: far above 8 MiB
    q = torch.zeros(1, 4096, 32, 128, device="cuda", dtype=torch.bfloat16)
    k = torch.zeros(1, 64, 8, 128, device="cuda", dtype=torch.bfloat16)
    ids = torch.zeros(4096, 2048, device="cuda", dtype=torch.int32)
    lengths = torch.full((4096,), 2048, device="cuda", dtype=torch.int32)
    out = torch.zeros_like(q)
    rc = _noalloc(L, q, k, k, ids, lengths, out, 0.1, None, 64)
    assert rc == LSA_ERR_SIZE
    torch.cuda.synchronize()
    assert float(out.float().abs().max()) == 0.0, "a refused call launches nothing"
