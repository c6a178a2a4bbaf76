"""Host logic of the failure check (no GPU): lsa_b200.check_status finds a non-zero word in
any cached counter or status buffer, zeroes every such buffer and raises - a timeout when
a LSA_ERR_TIMEOUT word is among them - and passes once the buffers are back at zero. The
buffers here are CPU tensors planted in the cache; on a GPU the same words are written by
kernels whose bounded waits expired (tests/test_gpu_waits.py)."""

import pytest
import torch


@pytest.fixture()
def cache():
    from lsa_b200 import _lib

    saved = dict(_lib._ws.counters), dict(_lib._ws.status)
    _lib._ws.counters.clear()
    _lib._ws.status.clear()
    yield _lib
    _lib._ws.counters.clear()
    _lib._ws.status.clear()
    _lib._ws.counters.update(saved[0])
    _lib._ws.status.update(saved[1])


def test_timeout_word_raises_and_resets(cache):
    buf = torch.zeros(16, dtype=torch.int32)
    buf[9] = cache.ERR_TIMEOUT
    cache._ws.counters[("cpu", 0)] = buf
    with pytest.raises(RuntimeError, match="bounded device wait expired"):
        cache.check_status("cpu", "test")
    assert int(buf.abs().sum()) == 0
    cache.check_status("cpu", "test")  # recovered: the next check passes


def test_stale_ticket_raises_and_resets(cache):
    buf = torch.zeros(8, dtype=torch.int32)
    buf[2] = 3  # a ticket left counted
    st = torch.zeros(1, dtype=torch.int32)
    cache._ws.counters[("cpu", 1)] = buf
    cache._ws.status[("cpu", 1)] = st
    with pytest.raises(RuntimeError, match="not at rest"):
        cache.check_status("cpu")
    assert int(buf.abs().sum()) == 0


def test_checked_mode_is_off_unless_asked(cache, monkeypatch):
    buf = torch.zeros(4, dtype=torch.int32)
    buf[0] = cache.ERR_TIMEOUT
    cache._ws.counters[("cpu", 2)] = buf
    monkeypatch.setenv("LSA_CHECK_STATUS", "0")
    cache.after_call(torch.device("cpu"), "test")  # unchecked: no sync, no raise
    monkeypatch.setenv("LSA_CHECK_STATUS", "1")
    with pytest.raises(RuntimeError):
        cache.after_call(torch.device("cpu"), "test")
