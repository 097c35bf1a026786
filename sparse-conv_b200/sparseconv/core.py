"""``SparseConvTensor``: the sparse voxel container of the reference (``core.py:19-77``),
with the same constructor, properties and conversions.

``indices`` is [M, 4] int32 (b, x, y, z); ``features`` is [M, C] and read-only (assign a
new tensor with ``replace_feature``); ``spatial_shape`` is a list of three ints.
"""
from __future__ import annotations

from typing import List, Union

import numpy as np
import torch
from torch.fx import ProxyableClassMeta


def scatter_nd(indices: torch.Tensor, src: torch.Tensor, shape: List[int]) -> torch.Tensor:
    """Scatter rows of ``src`` into a zero tensor of ``shape`` at ``indices`` (core.py:9-17)."""
    res = torch.zeros(*shape, dtype=src.dtype, device=src.device)
    ndim = indices.shape[-1]
    flat = indices.view(-1, ndim)
    res[tuple(flat[:, i] for i in range(ndim)) + (Ellipsis,)] = src.view(
        *(list(indices.shape[:-1]) + list(shape[ndim:])))
    return res


class SparseConvTensor(metaclass=ProxyableClassMeta):
    def __init__(self, features: torch.Tensor, indices: torch.Tensor,
                 spatial_shape: Union[List[int], np.ndarray], batch_size: int):
        self._features = features
        self.indices = indices
        self.spatial_shape = [int(v) for v in spatial_shape]
        self.batch_size = batch_size

    def __repr__(self) -> str:
        return f"SparseConvTensor[shape={self.features.shape}]"

    def replace_feature(self, feature: torch.Tensor) -> "SparseConvTensor":
        return SparseConvTensor(feature, self.indices, self.spatial_shape, self.batch_size)

    @property
    def features(self) -> torch.Tensor:
        return self._features

    @features.setter
    def features(self, val) -> None:
        raise ValueError(
            "Due to issues related to fx, you cannot set features directly."
            "Use 'x = x.replace_feature(new_feature)'"
            "to generate new SparseConvTensor instead.")

    @classmethod
    def from_dense(cls, x: torch.Tensor) -> "SparseConvTensor":
        """Channels-last dense [B, *spatial, C] -> sparse; a voxel is active iff any of
        its channels is non-zero. Indices come out sorted by (b, x, y, z).

        CUDA [B, W, H, D, C] float tensors go through the library's compaction kernels (one
        host synchronisation for the voxel count); other inputs use torch's ``to_sparse`` as
        the reference does (core.py:56-63)."""
        if x.is_cuda and x.dim() == 5 and x.dtype in (torch.float32, torch.float16, torch.bfloat16):
            from sparseconv import _native
            indices, features = _native.dense_to_sparse(x)
            return cls(features, indices, list(x.shape[1:4]), int(x.shape[0]))
        x_sp = x.to_sparse(x.ndim - 1)
        spatial_shape = x_sp.shape[1:-1]
        batch_size = x_sp.shape[0]
        indices = x_sp.indices().permute(1, 0).contiguous().int()
        features = x_sp.values()
        return cls(features, indices, spatial_shape, batch_size)

    def dense(self, channels_first: bool = True) -> torch.Tensor:
        """Zero-filled dense tensor, [B, C, *spatial] (channels_first) or [B, *spatial, C]
        (core.py:65-77); CUDA 3-D tensors are scattered by the library in the final layout."""
        if (self.features.is_cuda and len(self.spatial_shape) == 3 and self.features.dim() == 2
                and self.features.dtype in (torch.float32, torch.float16, torch.bfloat16)):
            from sparseconv import _native
            return _native.sparse_to_dense(self.features, self.indices.to(self.features.device),
                                           int(self.batch_size), self.spatial_shape, channels_first)
        output_shape = [self.batch_size] + list(self.spatial_shape) + [self.features.shape[1]]
        res = scatter_nd(self.indices.to(self.features.device).long(), self.features, output_shape)
        if not channels_first:
            return res
        ndim = len(self.spatial_shape)
        perm = list(range(0, ndim + 1))
        perm.insert(1, ndim + 1)
        return res.permute(*perm).contiguous()
