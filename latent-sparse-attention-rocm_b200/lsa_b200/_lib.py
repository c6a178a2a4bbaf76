"""ctypes binding of ``liblsa_b200.so`` - the C-ABI every operator of this package calls.

There is no fallback: if the library is missing, or a tensor is not on a CUDA device,
the operators raise. Streams: every call launches on torch's current stream of the
tensors' device. Workspaces: scratch (any content) and counters (int32, zero at rest; the
kernels that use them leave them zero) are cached per (device, stream) and only grow.
"""

from __future__ import annotations

import ctypes
import os
import pathlib
import threading

import torch

LIB_PATH = pathlib.Path(__file__).resolve().parent / "liblsa_b200.so"

F32, F16, BF16 = 0, 1, 2
F32_AS_BF16 = 3  # selects' query code: fp32 storage read as its bf16 rounding
DTYPE_CODE = {torch.float32: F32, torch.float16: F16, torch.bfloat16: BF16}

OK, ERR_ARG, ERR_CUDA, ERR_TIMEOUT, ERR_SHORT, ERR_SIZE = 0, -1, -2, -3, -4, -5

_lib = None
_lock = threading.RLock()  # re-entrant: torch_ops() loads lib() first

_P = ctypes.c_void_p
_I = ctypes.c_int64
_INT = ctypes.c_int
_F = ctypes.c_float

# name -> (restype, argtypes); mirrors include/lsa_b200.h
SIGNATURES = {
    "lsa_bucket_scores": (_INT, [_P, _INT, _I, _I, _P, _INT, _I, _I, _P, _I, _P]),
    "lsa_visible_counts": (_INT, [_P, _I, _I, _I, _I, _P, _P]),
    "lsa_pack_keys": (_INT, [_P, _I, _I, _I, _P, _P, _I, _P]),
    "lsa_best_first_keys": (_INT, [_P, _I, _I, _I, _I, _P, _P, _I, _P]),
    "lsa_unpack_ids": (_INT, [_P, _I, _P, _P]),
    "lsa_select_topk_scores": (_INT, [_P, _I, _I, _I, _P, _I, _P, _I, _P]),
    "lsa_expand_in_order": (_INT, [_P, _I, _I, _I, _P, _I, _I, _P, _I, _I, _I, _P, _P, _P]),
    "lsa_expand_from_keys": (_INT, [_P, _I, _I, _I, _P, _I, _I, _P, _I, _I, _I, _P, _P, _P]),
    "lsa_select_fused_scratch": (_I, [_I, _I]),
    "lsa_peer_arena_alloc": (_INT, [_I, _P, _P]),
    "lsa_peer_arena_open": (_INT, [_P, _P]),
    "lsa_peer_arena_close": (_INT, [_P]),
    "lsa_peer_arena_free": (_INT, [_P]),
    "lsa_peer_all_gather": (_INT, [_P, _P, _I, _INT, _INT, _P, _I, _I, _P, _P, _P]),
    "lsa_select_fused_grouped": (_INT, [_P, _INT, _I, _I, _I, _I, _P, _INT, _I, _P, _I, _I, _P, _I, _I, _I, _I, _I,
                                        _P, _P, _P]),
    "lsa_select_fused": (_INT, [_P, _INT, _I, _I, _P, _INT, _I, _I, _P, _I, _I, _P, _I, _I, _I, _I, _I, _P, _P, _P,
                                _I, _P, _I, _I, _P]),
    "lsa_sparse_read_plan": (_INT, [_I, _I, _I, _I, _I, _I, _I, _P, _P, _P]),
    "lsa_sparse_read": (_INT, [_P, _P, _P, _INT, _P, _P, _I, _I, _I, _I, _I, _I, _I, _F, _P, _P, _I, _P, _I, _I,
                               _P]),
    "lsa_regroup": (_INT, [_P, _P, _INT, _I, _I, _I, _I, _P, _P, _P]),
    "lsa_regroup_project": (_INT, [_P, _P, _INT, _I, _I, _I, _I, _P, _I, _P, _P, _P]),
    "lsa_normalize_rows": (_INT, [_P, _I, _I, _P, _P, _P]),
    "lsa_build_buckets_workspace": (_I, [_I, _I, _I, _I]),
    "lsa_build_buckets": (_INT, [_P, _I, _I, _I, _I, _I, _I, _P, _P, _P, _P, _P, _P, _I, _P, _P]),
    "lsa_position_buckets": (_INT, [_P, _I, _I, _I, _I, _I, _P, _P, _P, _P, _P, _P, _P]),
    "lsa_pair_to_size_workspace": (_I, [_I, _I, _I]),
    "lsa_pair_to_size": (_INT, [_P, _I, _I, _I, _I, _P, _P, _P, _P, _I, _P, _P]),
    "lsa_sparse_read_noalloc": (_INT, [_P, _P, _P, _INT, _P, _P, _I, _I, _I, _I, _I, _I, _I, _F, _P, _I, _P, _P]),
    "lsa_positional_picks": (_INT, [_P, _I, _I, _I, _I, _I, _I, _I, _P, _P]),
    "lsa_select_batched_scratch": (_I, [_I, _I]),
    "lsa_select_batched": (_INT, [_P, _INT, _I, _I, _P, _INT, _I, _P, _P, _I, _P, _I, _I, _P, _I, _I, _I, _I, _I, _P,
                                  _P, _P, _I, _P, _I, _I, _P]),
    "lsa_decode_fused_plan": (_INT, [_I, _I, _I, _I, _I, _I, _P, _P]),
    "lsa_map_slots": (_INT, [_P, _P, _I, _I, _P, _I, _I, _I, _P, _P, _P]),
    "lsa_wait_selftest": (_INT, [_P, _I, _INT, _P]),
    "lsa_decode_fused": (_INT, [_P, _I, _I, _P, _I, _I, _P, _I, _P, _I, _I, _I, _I, _I, _I, _P, _P, _P, _INT, _I, _I,
                                _I, _I, _F, _P, _P, _P, _P, _I, _P, _I, _P]),
    "lsa_tile_queries": (_INT, [_P, _INT, _I, _I, _I, _I, _P, _P]),
    "lsa_tile_select_scratch": (_I, [_I, _I, _I, _I]),
    "lsa_tile_select": (_INT, [_P, _INT, _I, _I, _I, _P, _INT, _I, _I, _I, _I, _P, _I, _I, _I, _I, _P, _P, _P, _I,
                               _P, _I, _P]),
    "lsa_sparse_prefill": (_INT, [_P, _P, _P, _INT, _P, _P, _I, _I, _I, _I, _I, _I, _I, _I, _I, _F, _P, _P, _P]),
    "lsa_tree_select_keys": (_INT, [_P, _I, _I, _P, _I, _I, _I, _I, _P, _P, _P, _P, _I, _I, _I, _I, _I, _P, _P, _I,
                                    _P, _I, _P, _I, _P]),
    "lsa_sparse_read_partial": (_INT, [_P, _P, _P, _INT, _P, _P, _I, _I, _I, _I, _I, _I, _I, _F, _I, _P, _P, _P, _I,
                                       _P, _I, _I, _P]),
    "lsa_merge_partials": (_INT, [_P, _P, _I, _I, _I, _INT, _P, _P]),
    "lsa_tree_plan": (_INT, [_I, _I, _P, _I, _I, _I, _I, _I, _P, _P]),
    "lsa_tree_select": (_INT, [_P, _I, _I, _P, _I, _I, _I, _I, _P, _P, _P, _P, _I, _I, _I, _I, _I, _P, _P, _I, _P,
                               _I, _P]),
    "lsa_tree_select_lists": (_INT, [_P, _I, _I, _P, _I, _I, _I, _I, _P, _P, _P, _P, _I, _I, _I, _I, _I, _P, _I, _I,
                                     _I, _I, _I, _P, _P, _P, _P, _I, _P, _I, _P]),
}


def lib():
    """The loaded library; raises when it has not been built (no CPU fallback exists)."""
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not LIB_PATH.exists():
                    raise RuntimeError(
                        f"{LIB_PATH} is missing: the LSA kernels are CUDA-only; build them with "
                        "`python latent-sparse-attention-rocm_b200/build.py` (or __graft_entry__.build())"
                    )
                handle = ctypes.CDLL(str(LIB_PATH))
                for name, (res, args) in SIGNATURES.items():
                    fn = getattr(handle, name)
                    fn.restype = res
                    fn.argtypes = args
                _lib = handle
    return _lib


TORCH_OPS_PATH = pathlib.Path(__file__).resolve().parent / "_lsa_torch_ops.so"
_torch_ops_loaded = False


def torch_ops():
    """``torch.ops.lsa`` - the hot-path operators registered by ``_lsa_torch_ops.so`` (a C++
    torch.library over this C ABI, launching on at::cuda::getCurrentCUDAStream()). Raises when
    the library is missing: there is no fallback."""
    global _torch_ops_loaded
    if not _torch_ops_loaded:
        lib()  # the C-ABI library first (the ops library links against it), outside this lock
        with _lock:
            if not _torch_ops_loaded:
                if not TORCH_OPS_PATH.exists():
                    raise RuntimeError(f"{TORCH_OPS_PATH} is missing: build it with "
                                       "latent-sparse-attention-rocm_b200/build.py (needs liblsa_b200.so)")
                torch.ops.load_library(str(TORCH_OPS_PATH))
                _torch_ops_loaded = True
    return torch.ops.lsa


def exported_symbols() -> list[str]:
    return sorted(SIGNATURES)


def check(rc: int, what: str) -> None:
    if rc == OK:
        return
    if rc == ERR_ARG:
        raise ValueError(f"{what}: arguments rejected by the kernel entry point")
    if rc == ERR_TIMEOUT:
        raise RuntimeError(f"{what}: a bounded device wait expired")
    if rc == ERR_SIZE:
        raise ValueError(f"{what}: the call exceeds the fixed no-allocation scratch (8 MiB, 65536 counters)")
    if rc == ERR_SHORT:
        raise ValueError(f"{what}: a cluster block could not reach its bucket count under the cap")
    raise RuntimeError(f"{what}: CUDA launch failed (status {rc})")


def ptr(t: torch.Tensor | None):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def stream_of(t: torch.Tensor):
    return ctypes.c_void_p(torch.cuda.current_stream(t.device).cuda_stream)


def require_cuda(*tensors: torch.Tensor, what: str, exc=ValueError) -> None:
    for t in tensors:
        if t is not None and t.device.type != "cuda":
            raise exc(f"{what} is a CUDA kernel (B200, sm_100a), got device {t.device}")


class _Workspace:
    def __init__(self):
        self.scratch: dict = {}
        self.counters: dict = {}
        self.status: dict = {}


_ws = _Workspace()


def _key(device: torch.device):
    idx = device.index if device.index is not None else torch.cuda.current_device()
    return (idx, torch.cuda.current_stream(device).cuda_stream)


def scratch(nbytes: int, device: torch.device) -> torch.Tensor:
    """Cached scratch bytes (any content) for the current stream of ``device``."""
    key = _key(device)
    buf = _ws.scratch.get(key)
    if buf is None or buf.numel() < nbytes:
        buf = torch.empty(max(int(nbytes), 256), dtype=torch.uint8, device=device)
        _ws.scratch[key] = buf
    return buf


def status_word(device: torch.device) -> torch.Tensor:
    """A device int32 status word per (device, stream) that kernels set on a failed
    bounded wait (LSA_ERR_TIMEOUT); zero while nothing has gone wrong."""
    key = _key(device)
    buf = _ws.status.get(key)
    if buf is None:
        buf = torch.zeros(1, dtype=torch.int32, device=device)
        _ws.status[key] = buf
    return buf


def counters(n: int, device: torch.device) -> torch.Tensor:
    """Cached int32 counters, zero at rest, for the current stream of ``device``."""
    key = _key(device)
    buf = _ws.counters.get(key)
    if buf is None or buf.numel() < n:
        buf = torch.zeros(max(int(n), 64), dtype=torch.int32, device=device)
        _ws.counters[key] = buf
    return buf


def _on(buf: torch.Tensor, device) -> bool:
    if device is None:
        return True
    dev = torch.device(device)
    if buf.device.type != dev.type:
        return False
    if dev.type != "cuda":
        return True
    return buf.device.index == (dev.index if dev.index is not None else torch.cuda.current_device())


def check_status(device=None, what: str = "lsa") -> None:
    """Raise if any call since the last check left a failure behind, and recover.

    Every cached counter buffer is zero between calls (tickets of last-CTA merges, barrier
    words, the status word of a bounded wait); a kernel whose bounded wait expired writes
    LSA_ERR_TIMEOUT (-3) into its status word and may leave a ticket counted. So at a point
    where the device is idle, any non-zero word is a failure: this synchronises ``device``
    (all devices with cached buffers when None), zeroes every such buffer so the next call
    starts clean, and raises RuntimeError (timeout when a -3 word was found). Graph users
    call it after replays; with LSA_CHECK_STATUS=1 every entry point calls it after its
    launch (outside stream capture)."""
    cached = list(_ws.counters.values()) + list(_ws.status.values())
    if _torch_ops_loaded:  # the torch ops' own per-stream counters
        cached += list(torch.ops.lsa.workspace_counters())
    bufs = [b for b in cached if _on(b, device)]
    for d in {b.device for b in bufs if b.device.type == "cuda"}:
        torch.cuda.synchronize(d)
    timed_out, dirty = False, False
    for b in bufs:
        bad = b != 0
        if bool(bad.any()):
            dirty = True
            timed_out = timed_out or bool((b == ERR_TIMEOUT).any())
            b.zero_()
    if timed_out:
        raise RuntimeError(f"{what}: a bounded device wait expired (LSA_ERR_TIMEOUT); counters reset")
    if dirty:
        raise RuntimeError(f"{what}: device counters were not at rest after the call; counters reset")


def after_call(device: torch.device, what: str) -> None:
    """The checked mode (LSA_CHECK_STATUS=1, read per call): synchronise and raise on a
    failure word right after the launch - skipped while a CUDA graph is being captured."""
    if os.environ.get("LSA_CHECK_STATUS", "0") != "1":
        return
    if torch.cuda.is_current_stream_capturing():
        return
    check_status(device, what)
