"""An all-gather over peer memory for the sharded decode steps (``lsa_peer_all_gather``).

The sequence-sharded tree decode and the head-sharded batched decode exchange a few KB to a
few MB per step (candidate keys, partial outputs, read lists). NCCL's all-gather costs tens of
microseconds of latency for such sizes; here every rank stores its chunk straight into every
peer's memory over NVLink (CUDA IPC mappings of one arena per rank) and publishes an epoch
flag there, and each rank waits (bounded) for all flags before copying the gathered rows out -
two small kernels on the caller's stream, CUDA-graph safe.

``PeerGather(group)`` is a collective to construct (the ranks exchange their arena handles
with ``torch.distributed.all_gather_object``); afterwards it is a callable with the contract of
``seqshard.all_gather_fn``: ``x [...] -> [world, ...]``. Every rank must make the same
sequence of calls. A channel (flags + two receive buffers) is carved out of the arena per
message size the first time that size is gathered - the offsets follow from the call order
alone, so every rank lays its arena out alike without communicating.
"""

from __future__ import annotations

import ctypes

import torch

from . import _lib
from ._lib import check, lib, stream_of

_HANDLE_BYTES = 64  # cudaIpcMemHandle_t
_MAX_CHANNELS = 64


def _align(x: int, a: int = 256) -> int:
    return (x + a - 1) // a * a


class PeerGather:
    """All-gather over peer memory among the ranks of ``group`` (one GPU per rank)."""

    def __init__(self, group=None, arena_bytes: int = 32 << 20, device=None):
        import torch.distributed as dist

        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        if self.world > 8:
            raise ValueError(f"peer gather covers up to 8 ranks, got {self.world}")
        self.device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        L = lib()
        own = ctypes.c_void_p()
        handle = (ctypes.c_char * _HANDLE_BYTES)()
        with torch.cuda.device(self.device):
            check(L.lsa_peer_arena_alloc(arena_bytes, ctypes.byref(own), handle), "peer arena")
        self.arena_bytes = arena_bytes
        self._own = own.value
        handles: list = [None] * self.world
        dist.all_gather_object(handles, bytes(handle), group=group)
        bases = []
        self._opened = []
        with torch.cuda.device(self.device):
            for r, h in enumerate(handles):
                if r == self.rank:
                    bases.append(self._own)
                    continue
                p = ctypes.c_void_p()
                buf = (ctypes.c_char * _HANDLE_BYTES).from_buffer_copy(h)
                check(L.lsa_peer_arena_open(buf, ctypes.byref(p)), "peer arena open")
                bases.append(p.value)
                self._opened.append(p.value)
        self._bases = (ctypes.c_void_p * self.world)(*bases)
        # per channel: 4 uint32 control words (epoch, two tickets), zero at rest but the epoch
        self._ctrl = torch.zeros(_MAX_CHANNELS, 4, dtype=torch.int32, device=self.device)
        self._channels: dict = {}
        self._next = 0

    def _channel(self, nbytes: int):
        ch = self._channels.get(nbytes)
        if ch is None:
            if len(self._channels) == _MAX_CHANNELS:
                raise RuntimeError(f"peer gather: more than {_MAX_CHANNELS} message sizes")
            flag_off = self._next
            recv_off = _align(flag_off + 4 * self.world)
            end = _align(recv_off + 2 * self.world * nbytes)
            if end > self.arena_bytes:
                raise RuntimeError(f"peer gather: arena of {self.arena_bytes} bytes is full "
                                   f"(a {nbytes}-byte channel needs {end - self._next})")
            ch = (flag_off, recv_off, self._ctrl[len(self._channels)])
            self._channels[nbytes] = ch
            self._next = end
        return ch

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        if x.device != self.device:
            raise ValueError(f"peer gather lives on {self.device}, got a tensor on {x.device}")
        x = x.contiguous()
        flat = x.reshape(-1).view(torch.uint8)
        n = flat.numel()
        nbytes = _align(n, 16)
        if nbytes != n or flat.data_ptr() % 16:  # 16-byte pieces from a 16-byte aligned start
            padded = torch.zeros(nbytes, dtype=torch.uint8, device=x.device)
            padded[:n] = flat
            flat = padded
        flag_off, recv_off, ctrl = self._channel(nbytes)
        out = torch.empty(self.world, nbytes, dtype=torch.uint8, device=x.device)
        st = _lib.status_word(x.device)
        check(lib().lsa_peer_all_gather(ctypes.c_void_p(flat.data_ptr()), ctypes.c_void_p(out.data_ptr()), nbytes,
                                        self.rank, self.world, self._bases, flag_off, recv_off,
                                        ctypes.c_void_p(ctrl.data_ptr()), ctypes.c_void_p(st.data_ptr()),
                                        stream_of(x)), "peer gather")
        _lib.after_call(x.device, "peer gather")
        return out[:, :n].contiguous().view(x.dtype).view((self.world,) + tuple(x.shape)) if nbytes != n else \
            out.view(x.dtype).view((self.world,) + tuple(x.shape))

    def close(self) -> None:
        """Unmap the peers' arenas and free this rank's (after every rank's last gather)."""
        L = lib()
        for p in self._opened:
            L.lsa_peer_arena_close(ctypes.c_void_p(p))
        self._opened = []
        if self._own is not None:
            L.lsa_peer_arena_free(ctypes.c_void_p(self._own))
            self._own = None


__all__ = ["PeerGather"]
