"""lsa_b200 - Latent Sparse Attention select + read for NVIDIA B200 (sm_100a).

A drop-in for the select/read operators of ``lsa_rocm_lab.port`` (AIwork4me/
latent-sparse-attention-rocm): ``pipeline``, ``select_fused``, ``read_kernel``,
``read_kernel_tiled`` and ``_tree`` keep the reference's names, arguments, outputs and
errors. Every operator runs hand-written CUDA kernels through the C-ABI library
``liblsa_b200.so`` (``include/lsa_b200.h``); there is no CPU path.
"""

from . import _lib, pipeline, prefill, read_kernel, read_kernel_tiled, select_fused  # noqa: F401
from ._lib import check_status  # noqa: F401
from .index_space import make_index_space  # noqa: F401
from .pipeline import (  # noqa: F401
    Buckets,
    Hierarchy,
    NodeLevel,
    PortConfig,
    best_first_keys,
    build_buckets_gpu,
    build_hierarchy_gpu,
    dense_read,
    flat_select,
    flat_select_reference,
    lsa_read,
    position_buckets,
    select_from_queries,
    tree_select,
    visible_counts,
)

__all__ = [
    "Buckets", "Hierarchy", "NodeLevel", "PortConfig", "best_first_keys", "build_buckets_gpu",
    "build_hierarchy_gpu", "dense_read", "flat_select", "flat_select_reference", "lsa_read",
    "make_index_space", "position_buckets", "select_from_queries", "tree_select", "visible_counts",
    "check_status",
]
