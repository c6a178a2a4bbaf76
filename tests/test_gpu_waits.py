"""The kernels' bounded waits: the helper every mbarrier wait goes through returns at once
when the phase completes and gives up after its limit when nothing ever arrives, leaving
LSA_ERR_TIMEOUT in a status word the host reads; the context stays usable afterwards (a
read runs and is correct). No fault, trap or hang is involved: the failing wait is a
barrier nothing arrives on, with a 50 ms limit."""

import time

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _wait(arrive: int, limit_ns: int) -> int:
    from lsa_b200 import _lib

    status = torch.full((1,), 12345, dtype=torch.int32, device=DEV)
    rc = _lib.lib().lsa_wait_selftest(_lib.ptr(status), limit_ns, arrive, _lib.stream_of(status))
    assert rc == 0
    return int(status.item())


def test_wait_completes_when_the_phase_does(lsa):
    assert _wait(1, 50_000_000) == 0


def test_wait_gives_up_and_reports_timeout(lsa, oracle):
    from lsa_b200 import _lib

    t0 = time.perf_counter()
    assert _wait(0, 50_000_000) == _lib.ERR_TIMEOUT
    assert time.perf_counter() - t0 < 5.0
    # the context is intact: a read after the expired wait runs and matches the checker
    rng = np.random.default_rng(0)
    q = (rng.standard_normal((1, 1, 8, 64)) * 0.3).astype(np.float32)
    k = (rng.standard_normal((1, 256, 2, 64)) * 0.3).astype(np.float32)
    v = rng.standard_normal((1, 256, 2, 64)).astype(np.float32)
    ids = rng.integers(0, 256, (1, 1, 100)).astype(np.int32)
    ln = np.array([[100]], np.int32)
    want = oracle.sparse_read(q, k, v, ids, ln)
    t = lambda x: torch.from_numpy(x).to(DEV)
    got = lsa.read_kernel_tiled.sparse_read_auto(t(q), t(k), t(v), t(ids), t(ln), 64 ** -0.5)
    assert float(np.abs(got.cpu().numpy() - want).max()) <= 1e-5


def test_selftest_rejects_bad_limits(lsa):
    from lsa_b200 import _lib

    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    assert _lib.lib().lsa_wait_selftest(_lib.ptr(status), 0, 1, _lib.stream_of(status)) == _lib.ERR_ARG
    assert _lib.lib().lsa_wait_selftest(_lib.ptr(status), 3_000_000_000, 1, _lib.stream_of(status)) == _lib.ERR_ARG


def test_expired_wait_in_cached_counters_is_caught_and_reset(lsa, oracle):
    """A timeout word left in the per-stream counter cache (where the reads, selects and
    fused decode keep their tickets and status words) is found by check_status, which
    raises and zeroes the cache; the next read (checked mode) runs clean and is correct."""
    from lsa_b200 import _lib

    ct = _lib.counters(64, torch.device(DEV))
    view = ct[5:6]  # any word of the cache: the position of a status word depends on the call
    assert _lib.lib().lsa_wait_selftest(_lib.ptr(view), 20_000_000, 0, _lib.stream_of(view)) == 0
    with pytest.raises(RuntimeError, match="bounded device wait expired"):
        lsa.check_status(DEV)
    assert int(ct.abs().sum().item()) == 0
    rng = np.random.default_rng(1)
    q = (rng.standard_normal((1, 1, 32, 128)) * 0.3).astype(np.float32)
    k = (rng.standard_normal((1, 512, 8, 128)) * 0.3).astype(np.float32)
    v = rng.standard_normal((1, 512, 8, 128)).astype(np.float32)
    ids = rng.integers(0, 512, (1, 1, 300)).astype(np.int32)
    ln = np.array([[300]], np.int32)
    want = oracle.sparse_read(q, k, v, ids, ln)
    t = lambda x: torch.from_numpy(x).to(DEV)
    got = lsa.read_kernel_tiled.sparse_read_auto(t(q), t(k), t(v), t(ids), t(ln), 128 ** -0.5)
    assert float(np.abs(got.cpu().numpy() - want).max()) <= 1e-5
