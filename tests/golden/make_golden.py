"""Generate the read-kernel golden fixtures from the reference's OWN Triton kernels.

The reference's two sparse-read kernels (AIwork4me/latent-sparse-attention-rocm,
``src/lsa_rocm_lab/port/read_kernel.py:26-77`` and ``read_kernel_tiled.py:30-89``) import
only torch and triton, so they run here on the CPU under ``TRITON_INTERPRET=1``. This
script loads them by file path from a reference checkout (``--reference``), launches
the ``@triton.jit`` kernels directly with the wrappers' own launch arithmetic
(``read_kernel_tiled.py:109-135``; the wrappers assert CUDA tensors), and writes every
case's inputs and outputs to ``read_golden.npz``. The fixtures travel with the repo;
the reference checkout is needed only to regenerate them.

Cases mirror the reference's read tests (``tests/test_read_kernel_tiled.py``): GQA
and MQA mappings, -1 padding and boundary ids, duplicate ids counted per occurrence,
zero-length rows (tiled -> 0), ragged batches, a full causal row set, fp32 and bf16.

Usage: TRITON_INTERPRET=1 python tests/golden/make_golden.py --reference <checkout>
"""

import argparse
import importlib.util
import os
import pathlib
import sys

os.environ.setdefault("TRITON_INTERPRET", "1")

import numpy as np  # noqa: E402
import torch  # noqa: E402

HERE = pathlib.Path(__file__).resolve().parent


def _load(path: pathlib.Path, name: str):
    spec = importlib.util.spec_from_file_location(name, path)
    module = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(module)
    return module


def run_tiled(mod, q, k, v, ids, lengths, scale, tile_rows, chunk):
    """The launch of read_kernel_tiled.sparse_read_tiled (:109-135), minus the CUDA assert."""
    B, Tq, Hq, D = q.shape
    Tk, Hkv = k.shape[1], k.shape[2]
    width = ids.shape[-1]
    flat_ids = ids.reshape(-1, width).contiguous()
    flat_lengths = lengths.reshape(-1).contiguous().clamp_max(width)
    out = torch.empty_like(q)
    rows = B * Tq
    nq = -(-width // chunk) * chunk
    grid = (-(-rows // tile_rows) * Hq,)
    mod._sparse_read_tiled_kernel[grid](q, k, v, flat_ids, flat_lengths, out, scale, Tk, Tq, rows,
                                        HQ=Hq, HKV=Hkv, D=D, WIDTH=width, NQ=nq, TM=tile_rows, CN=chunk)
    return out


def run_v1(mod, q, k, v, ids, lengths, scale, block=64):
    """The launch of read_kernel.sparse_read (:103-119), minus the CUDA assert."""
    B, Tq, Hq, D = q.shape
    Tk, Hkv = k.shape[1], k.shape[2]
    width = ids.shape[-1]
    out = torch.empty_like(q)
    nq = -(-width // block) * block
    mod._sparse_read_kernel[(B * Tq * Hq,)](q, k, v, ids.reshape(-1, width).contiguous(),
                                            lengths.reshape(-1).contiguous(), out, scale, Tk,
                                            TQ=Tq, HQ=Hq, HKV=Hkv, D=D, WIDTH=width, NQ=nq, ID_BLOCK=block)
    return out


def cases():
    g = torch.Generator().manual_seed(20261106)

    def qkv(B, Tq, Tk, Hq, Hkv, D, dtype):
        q = (torch.randn(B, Tq, Hq, D, generator=g) * 0.2).to(dtype)
        k = (torch.randn(B, Tk, Hkv, D, generator=g) * 0.2).to(dtype)
        v = (torch.randn(B, Tk, Hkv, D, generator=g) * 0.2).to(dtype)
        return q, k, v

    out = []
    # GQA 8q/2kv, random ids incl. duplicates, full lengths (test_gqa_mqa_mapping shape, smaller)
    for hq, hkv in [(8, 2), (4, 1), (2, 2)]:
        q, k, v = qkv(1, 6, 48, hq, hkv, 64, torch.float32)
        ids = torch.randint(0, 48, (1, 6, 96), generator=g, dtype=torch.int32)
        lengths = torch.full((1, 6), 96, dtype=torch.int32)
        out.append((f"gqa_{hq}_{hkv}_fp32", q, k, v, ids, lengths))
    # batch + ragged lengths (test_batch_and_ragged_tile)
    q, k, v = qkv(3, 5, 13, 4, 2, 64, torch.float32)
    ids = torch.randint(0, 13, (3, 5, 40), generator=g, dtype=torch.int32)
    lengths = torch.randint(1, 41, (3, 5), generator=g, dtype=torch.int32)
    out.append(("batch_ragged_fp32", q, k, v, ids, lengths))
    # pad + boundary ids (test_pad_and_boundary_indices)
    q, k, v = qkv(1, 4, 64, 4, 2, 64, torch.float32)
    ids = torch.full((1, 4, 32), -1, dtype=torch.int32)
    ids[:, :, 0] = 0
    ids[:, :, 1] = 63
    lengths = torch.full((1, 4), 3, dtype=torch.int32)
    out.append(("pad_boundary_fp32", q, k, v, ids, lengths))
    # duplicates counted per occurrence (test_duplicate_ids_counted_per_occurrence)
    q, k, v = qkv(1, 2, 16, 8, 2, 64, torch.float32)
    ids = torch.full((1, 2, 8), -1, dtype=torch.int32)
    ids[:, 0, 0] = 5
    ids[:, 0, 1] = 5
    ids[:, 1, :3] = torch.tensor([3, 7, 3], dtype=torch.int32)
    lengths = torch.tensor([[2, 3]], dtype=torch.int32)
    out.append(("duplicates_fp32", q, k, v, ids, lengths))
    # mixed zero and real rows (test_mixed_zero_and_real_rows); tiled gives exact zeros
    q, k, v = qkv(1, 6, 24, 4, 2, 64, torch.float32)
    ids = torch.randint(0, 24, (1, 6, 16), generator=g, dtype=torch.int32)
    lengths = torch.full((1, 6), 16, dtype=torch.int32)
    lengths[0, 1::2] = 0
    out.append(("zero_rows_fp32", q, k, v, ids, lengths))
    # full causal lists (the D2 anchor shape), D = 128
    T = 20
    q, k, v = qkv(1, T, T, 4, 1, 128, torch.float32)
    row = torch.arange(T, dtype=torch.int32)
    ids = torch.where(row[None, :] <= row[:, None], row[None, :].expand(T, T), torch.tensor(-1, dtype=torch.int32))
    out.append(("causal_d128_fp32", q, k, v, ids.view(1, T, T).contiguous(), (row + 1).view(1, T).contiguous()))
    # bf16 decode-shaped row with a long list (test_decode_single_row, smaller)
    q, k, v = qkv(1, 1, 80, 8, 2, 64, torch.bfloat16)
    ids = torch.randint(0, 80, (1, 1, 300), generator=g, dtype=torch.int32)
    lengths = torch.full((1, 1), 300, dtype=torch.int32)
    out.append(("decode_bf16", q, k, v, ids, lengths))
    return out


def main() -> int:
    parser = argparse.ArgumentParser()
    parser.add_argument("--reference", required=True, help="path of a reference checkout")
    parser.add_argument("--out", default=str(HERE / "read_golden.npz"))
    args = parser.parse_args()
    port = pathlib.Path(args.reference) / "src" / "lsa_rocm_lab" / "port"
    tiled = _load(port / "read_kernel_tiled.py", "ref_read_kernel_tiled")
    v1 = _load(port / "read_kernel.py", "ref_read_kernel")
    blob = {}
    names = []
    for name, q, k, v, ids, lengths in cases():
        scale = q.shape[-1] ** -0.5
        t = run_tiled(tiled, q, k, v, ids, lengths, scale, tile_rows=4, chunk=32)
        t1 = run_tiled(tiled, q, k, v, ids, lengths, scale, tile_rows=1, chunk=64)
        base = run_v1(v1, q, k, v, ids, lengths, scale)
        names.append(name)
        blob[f"{name}/q"] = q.float().numpy()
        blob[f"{name}/k"] = k.float().numpy()
        blob[f"{name}/v"] = v.float().numpy()
        blob[f"{name}/dtype"] = np.array(str(q.dtype).split(".")[-1])
        blob[f"{name}/ids"] = ids.numpy()
        blob[f"{name}/lengths"] = lengths.numpy()
        blob[f"{name}/scale"] = np.array(scale, dtype=np.float64)
        blob[f"{name}/tiled_tm4_cn32"] = t.float().numpy()
        blob[f"{name}/tiled_tm1_cn64"] = t1.float().numpy()
        blob[f"{name}/v1"] = base.float().numpy()
        print(name, tuple(q.shape), "tiled-v1 max", float((t.float() - base.float()).abs().nan_to_num().max()))
    blob["cases"] = np.array(names)
    np.savez_compressed(args.out, **blob)
    print("wrote", args.out)
    return 0


if __name__ == "__main__":
    sys.exit(main())
