"""D-LSA projection maps: the index space through a learned or training-free linear map.

Reference: AIwork4me/latent-sparse-attention-rocm, ``docs/ROADMAP.md:41-43`` ("model-specific
distilled projections (D-LSA maps)"): the index space of a model is a per-layer linear map of
the regrouped queries and keys, trained upstream (``lsa.training.distillation``, absent) for one
frozen checkpoint and never transferable. This module holds what the selection path needs:

* the map format - per layer a matrix ``[d_out, Hkv * D]`` fp32 (one row per output dim),
  applied by ``lsa_regroup_project`` (``index_space.make_index_space(..., projection=W)``):
  index queries are projected group means, index keys projected key rows normalised after the
  projection; the buckets, selection and tree run unchanged in the d_out-wide space;
* ``pca_map`` - a training-free map (the reference's evaluation plan lists "training-free PCA"
  beside the distilled one): the top principal directions of a layer's index keys;
* ``ProjectionMaps`` - a model's maps, one per layer, saved and loaded as ``.npz`` (a distilled
  map trained elsewhere is loaded the same way).
Training a distilled map (a campaign over a real checkpoint and data) is not part of this path.
"""

from __future__ import annotations

import pathlib
from dataclasses import dataclass, field

import numpy as np
import torch


def pca_map(index_keys: torch.Tensor, d_out: int) -> torch.Tensor:
    """A training-free map [d_out, d]: the d_out leading eigenvectors of the keys' (uncentred)
    second moment, largest first - the projection that keeps the most of the keys' dot products.
    Computed in fp64 (a map is an input of the selection, built once per layer)."""
    x = index_keys.double()
    d = x.shape[1]
    if not 0 < d_out <= d or d_out % 8:
        raise ValueError(f"d_out must be a positive multiple of 8 not above {d}, got {d_out}")
    evals, evecs = torch.linalg.eigh(x.T @ x / max(x.shape[0], 1))
    order = torch.argsort(evals, descending=True)[:d_out]
    return evecs[:, order].T.contiguous().float()


@dataclass
class ProjectionMaps:
    """One projection map per layer ([d_out, Hkv * D] fp32 each)."""

    maps: list = field(default_factory=list)

    def __getitem__(self, layer: int) -> torch.Tensor:
        return self.maps[layer]

    def __len__(self) -> int:
        return len(self.maps)

    def to(self, device) -> "ProjectionMaps":
        return ProjectionMaps([m.to(device).float().contiguous() for m in self.maps])

    def save(self, path) -> None:
        np.savez(pathlib.Path(path), **{f"layer{i}": m.detach().float().cpu().numpy() for i, m in enumerate(self.maps)})

    @classmethod
    def load(cls, path, device="cpu") -> "ProjectionMaps":
        blob = np.load(pathlib.Path(path))
        n = len([k for k in blob.files if k.startswith("layer")])
        return cls([torch.from_numpy(blob[f"layer{i}"]).to(device).float().contiguous() for i in range(n)])

    @classmethod
    def pca(cls, per_layer_keys, d_out: int) -> "ProjectionMaps":
        """Training-free maps from each layer's index keys."""
        return cls([pca_map(k, d_out) for k in per_layer_keys])
