"""Host-side behaviour of the Python front end (no GPU needed): the SparseConvTensor API
ported from the reference's tests/test_core.py, the op's argument handling, and the
no-CPU-fallback rule."""
import pytest
import torch

from sparseconv import SparseConvTensor
from sparseconv.ops.submanifold_conv3d import (Algorithm, SubMConv3dFunction,
                                               SubMConv3dNeighborCache,
                                               sparse_submanifold_conv3d)


class TestSparseConvTensor:
    # tests/test_core.py:6-17 of the reference
    def test_conversion_one(self):
        x = torch.zeros((1, 255, 255, 3))
        x_sp = SparseConvTensor.from_dense(x)
        x_d = x_sp.dense()
        assert (x_d.permute(0, 3, 2, 1) == x).all() == True  # noqa: E712

    def test_conversion_two(self):
        x = torch.zeros((1, 255, 255, 3))
        x_sp = SparseConvTensor.from_dense(x)
        x_d = x_sp.dense(channels_first=False)
        assert (x_d == x).all() == True  # noqa: E712

    def test_round_trip_nonzero_3d(self):
        g = torch.Generator().manual_seed(0)
        x = torch.zeros((2, 6, 5, 4, 3))
        mask = torch.rand((2, 6, 5, 4), generator=g) < 0.3
        x[mask] = torch.randn((int(mask.sum()), 3), generator=g)
        sp = SparseConvTensor.from_dense(x)
        assert sp.indices.dtype == torch.int32 and sp.indices.shape[1] == 4
        assert sp.spatial_shape == [6, 5, 4] and sp.batch_size == 2
        flat = ((sp.indices[:, 0] * 6 + sp.indices[:, 1]) * 5 + sp.indices[:, 2]) * 4 + sp.indices[:, 3]
        assert torch.all(flat[1:] > flat[:-1]), "indices sorted by (b, x, y, z)"
        assert torch.equal(sp.dense(channels_first=False), x)
        assert torch.equal(sp.dense(), x.permute(0, 4, 1, 2, 3))

    def test_features_read_only(self):
        sp = SparseConvTensor(torch.zeros(2, 3), torch.zeros(2, 4, dtype=torch.int32), [4, 4, 4], 1)
        with pytest.raises(ValueError):
            sp.features = torch.ones(2, 3)
        sp2 = sp.replace_feature(torch.ones(2, 3))
        assert torch.equal(sp2.features, torch.ones(2, 3)) and sp2.indices is sp.indices
        assert repr(sp) == "SparseConvTensor[shape=torch.Size([2, 3])]"


def test_algorithm_constants():
    assert Algorithm.EXPLICIT_GEMM == "explicit_gemm"
    assert Algorithm.IMPLICIT_GEMM == "implicit_gemm"
    assert Algorithm.IMPLICIT_GEMM_SPLITK == "implicit_gemm_splitk"
    assert Algorithm.MASKED_IMPLICIT_GEMM == "masked_implicit_gemm"
    assert Algorithm.MASKED_IMPLICIT_GEMM_SPLITK == "masked_implicit_gemm_splitk"


def test_neighbor_cache_item_access():
    c = SubMConv3dNeighborCache(neighbor_map=1)
    assert c["neighbor_map"] == 1
    c["masks"] = 2
    assert c.masks == 2


def test_cpu_tensors_have_no_fallback():
    feats = torch.randn(3, 3)
    coords = torch.tensor([[0, 0, 0, 0], [0, 1, 1, 1], [0, 2, 2, 2]], dtype=torch.int32)
    w = torch.randn(3, 3, 3, 3, 3)
    with pytest.raises(NotImplementedError, match="CPU version of hashmap"):
        sparse_submanifold_conv3d(feats, coords, torch.Size((1, 3, 5, 5, 5)), w)


def test_readme_positional_algorithm_is_not_taken_as_bias():
    """README.md:37-39 passes Algorithm.IMPLICIT_GEMM in the bias slot; the reference
    fails in addmm with a TypeError. Here it reaches the (CUDA-only) map build."""
    feats = torch.randn(3, 3)
    coords = torch.tensor([[0, 0, 0, 0], [0, 1, 1, 1], [0, 2, 2, 2]], dtype=torch.int32)
    w = torch.randn(3, 3, 3, 3, 3)
    with pytest.raises(NotImplementedError):
        sparse_submanifold_conv3d(feats, coords, torch.Size((1, 3, 5, 5, 5)), w, Algorithm.IMPLICIT_GEMM)


def test_compute_neighbor_cache_argument_checks():
    coords = torch.zeros((4, 4), dtype=torch.int32)
    with pytest.raises(AssertionError, match="contiguous"):
        SubMConv3dFunction._compute_neighbor_cache(coords.t(), (1, 1, 4, 4, 4), (3, 3, 3), (1, 1, 1))
    with pytest.raises(AssertionError, match="int32"):
        SubMConv3dFunction._compute_neighbor_cache(coords.long(), (1, 1, 4, 4, 4), (3, 3, 3), (1, 1, 1))
    with pytest.raises(ValueError, match="Unsupported Algorithm"):
        SubMConv3dFunction._compute_neighbor_cache(coords, (1, 1, 4, 4, 4), (3, 3, 3), (1, 1, 1), "nope")
