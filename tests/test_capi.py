"""The C-ABI library loads and exports every symbol include/lsa_b200.h declares (CPU only).

No compute call is made here (there may be no GPU); the Python binding's signature table
must also cover exactly the header's entry points, and the header must compile as C.
"""

import pathlib
import re
import subprocess

import pytest

ROOT = pathlib.Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "lsa_b200.h"


def _declared():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"^(?:int|int64_t)\s+(lsa_\w+)\s*\(", text, flags=re.M)))


def test_header_declares_entry_points():
    names = _declared()
    assert "lsa_sparse_read" in names and "lsa_select_fused" in names and "lsa_build_buckets" in names
    assert len(names) >= 20


def test_library_exports_every_declared_symbol():
    from lsa_b200 import _lib

    undefined = subprocess.run(["nm", "-D", "--undefined-only", str(_lib.LIB_PATH)], capture_output=True, text=True)
    own = [ln for ln in undefined.stdout.splitlines() if "_ZN3lsa" in ln or " lsa_" in ln]
    assert not own, f"the library references its own symbols that it does not define: {own}"
    try:
        L = _lib.lib()
    except OSError as e:  # a machine without the CUDA runtime cannot dlopen it
        if "undefined symbol" in str(e):
            raise
        pytest.skip(f"CUDA runtime not loadable here: {e}")
    for name in _declared():
        assert hasattr(L, name), name
    out = subprocess.run(["nm", "-D", "--defined-only", str(_lib.LIB_PATH)], capture_output=True, text=True)
    exported = set(re.findall(r"\bT (lsa_\w+)", out.stdout))
    assert set(_declared()) <= exported


def test_binding_table_matches_header():
    from lsa_b200 import _lib

    assert sorted(_lib.SIGNATURES) == _declared()


def test_header_compiles_as_c(tmp_path):
    src = tmp_path / "use.c"
    src.write_text('#include "lsa_b200.h"\nint main(void) { return lsa_sparse_read == 0; }\n')
    res = subprocess.run(["gcc", "-fsyntax-only", "-I", str(ROOT / "include"), "-I", "/usr/local/cuda/include",
                          str(src)], capture_output=True, text=True)
    assert res.returncode == 0, res.stderr


def test_cpu_tensors_fail_loudly():
    import torch

    import lsa_b200

    with pytest.raises(ValueError):
        lsa_b200.select_fused.select_topk_scores(torch.zeros(2, 4), torch.zeros(2, dtype=torch.int32), 2)
    with pytest.raises(AssertionError):
        lsa_b200.read_kernel_tiled.sparse_read_auto(torch.zeros(1, 1, 2, 64), torch.zeros(1, 4, 2, 64),
                                                    torch.zeros(1, 4, 2, 64), torch.zeros(1, 1, 4, dtype=torch.int32),
                                                    torch.zeros(1, 1, dtype=torch.int32))
    with pytest.raises(ValueError):
        lsa_b200.build_buckets_gpu(torch.zeros(64, 8), lsa_b200.PortConfig())


def test_switch_validation_on_cpu(monkeypatch):
    import torch

    import lsa_b200

    monkeypatch.setenv("LSA_SELECT_IMPL", "bogus")
    with pytest.raises(ValueError, match="LSA_SELECT_IMPL"):
        lsa_b200.flat_select(torch.zeros(2, 8), torch.tensor([7, 7]), None, lsa_b200.PortConfig())


def test_dense_baseline_semantics_on_cpu():
    """tests/test_dense_read.py:46-104 - decode row == prefill's last row; chunks bottom-right."""
    import torch

    import lsa_b200

    torch.manual_seed(20261106)
    q = torch.randn(1, 64, 8, 64) * 0.2
    k = torch.randn(1, 64, 2, 64) * 0.2
    v = torch.randn(1, 64, 2, 64) * 0.2
    pre = lsa_b200.dense_read(q, k, v, 0.125)
    assert torch.allclose(lsa_b200.dense_read(q[:, -1:], k, v, 0.125), pre[:, -1:], atol=1e-5)
    assert torch.allclose(lsa_b200.dense_read(q[:, -7:], k, v, 0.125), pre[:, -7:], atol=1e-5)
    with pytest.raises(ValueError):
        lsa_b200.dense_read(q, k[:, :32], v[:, :32], 0.125)


def test_torch_ops_register_with_shapes():
    """The torch.library operators (lsa_b200/_lsa_torch_ops.so, over this C ABI) load on a
    machine without a GPU and give FX / torch.compile their output shapes (Meta kernels)."""
    import torch

    from lsa_b200 import _lib

    ops = _lib.torch_ops()
    m = dict(device="meta")
    q = torch.empty(2, 3, 32, 128, dtype=torch.bfloat16, **m)
    k = torch.empty(2, 4096, 8, 128, dtype=torch.bfloat16, **m)
    out = ops.sparse_read(q, k, k, torch.empty(2, 3, 2116, dtype=torch.int32, **m),
                          torch.empty(2, 3, dtype=torch.int32, **m), 0.1)
    assert out.shape == q.shape and out.dtype == q.dtype
    lists, lengths = ops.select_fused(torch.empty(5, 1024, **m), torch.empty(5, dtype=torch.int32, **m),
                                      torch.empty(512, 1024, dtype=torch.bfloat16, **m),
                                      torch.empty(512, 128, dtype=torch.int32, **m), 512, 8, 32, 64, 4, 2048)
    assert lists.shape == (5, 2116) and lengths.shape == (5,) and lists.dtype == torch.int32
    iq, ik = ops.regroup(torch.empty(7, 32, 128, **m), torch.empty(7, 8, 128, **m))
    assert iq.shape == ik.shape == (7, 1024) and iq.dtype == torch.float32


def test_torch_ops_load_first_in_a_fresh_process():
    """Loading the torch ops before anything else loads the C-ABI library (a fresh
    interpreter) returns: the ops loader takes the library first, under a re-entrant lock."""
    import subprocess
    import sys

    code = ("import sys; sys.path.insert(0, %r); from lsa_b200 import _lib; "
            "print(_lib.torch_ops().sparse_read)" % str(ROOT / "latent-sparse-attention-rocm_b200"))
    res = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=120)
    assert res.returncode == 0 and "lsa.sparse_read" in res.stdout, res.stderr[-2000:]


def test_tree_lists_refuses_missing_buffers_before_any_cuda_call():
    """lsa_tree_select_lists checks its expansion arguments first: a null member table or
    output, or a negative window, returns LSA_ERR_ARG (-1) without touching the GPU."""
    import ctypes

    from lsa_b200 import _lib

    try:
        L = _lib.lib()
    except OSError as e:
        pytest.skip(f"CUDA runtime not loadable here: {e}")
    one = (ctypes.c_int64 * 1)(1)
    ptrs = (ctypes.c_void_p * 1)(None)
    buf = ctypes.c_void_p(16)  # never dereferenced: the call returns before any use

    def call(members, lists, window):
        return L.lsa_tree_select_lists(buf, 1, 64, buf, 512, 8, 8, 1, ptrs, ptrs, one, buf, 4, 64, 3, 64, 32,
                                       members, 8, 64, window, 4, 2048, buf, lists, buf, buf, 1 << 20, buf, 2, None)

    assert call(None, buf, 64) == -1
    assert call(buf, None, 64) == -1
    assert call(buf, buf, -1) == -1
