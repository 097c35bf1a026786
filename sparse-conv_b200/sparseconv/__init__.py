"""B200-native (sm_100a) submanifold 3D sparse convolution with the Python API of
Arktetra/sparse-conv: ``SparseConvTensor`` and
``sparseconv.ops.submanifold_conv3d.sparse_submanifold_conv3d``."""
from sparseconv.core import SparseConvTensor
from sparseconv._native import check_errors

__all__ = [
    "SparseConvTensor",
    "check_errors",
]
