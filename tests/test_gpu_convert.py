"""SparseConvTensor.from_dense / .dense on the GPU (core.py:52-77): the library's compaction and
scatter kernels against torch's to_sparse (what the reference calls), bit for bit."""
import numpy as np
import pytest
import torch

from sparseconv import SparseConvTensor, _native

pytestmark = pytest.mark.gpu


def _dense(seed, B, W, H, D, C, p, dtype):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn((B, W, H, D, C), generator=g)
    keep = torch.rand((B, W, H, D), generator=g) < p
    part = torch.rand((B, W, H, D, C), generator=g) < 0.5     # some active voxels have zero channels
    x = torch.where(keep[..., None] & part, x, torch.zeros_like(x))
    if B * W * H * D > 3:
        x[0, 0, 0, 1, 0] = float("nan")                         # NaN counts as non-zero
        x[0, 0, 0, 2, :] = -0.0                                 # -0 does not
    return x.to(dtype)


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16])
@pytest.mark.parametrize("C", [1, 3, 8, 32, 64])
def test_from_dense_matches_torch_to_sparse(dtype, C):
    x = _dense(C, 2, 17, 9, 13, C, 0.1, dtype).cuda()
    st = SparseConvTensor.from_dense(x)
    ref = x.to_sparse(x.ndim - 1)
    ref_idx = ref.indices().permute(1, 0).contiguous().int()
    assert st.indices.dtype == torch.int32 and st.indices.shape == ref_idx.shape
    assert torch.equal(st.indices, ref_idx)
    assert torch.equal(st.features.view(torch.uint8) if dtype != torch.float32 else st.features.view(torch.int32),
                       ref.values().contiguous().view(torch.uint8) if dtype != torch.float32 else ref.values().contiguous().view(torch.int32))
    assert st.spatial_shape == [17, 9, 13] and st.batch_size == 2


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16])
@pytest.mark.parametrize("channels_first", [True, False])
def test_dense_round_trip(dtype, channels_first):
    x = _dense(5, 3, 12, 10, 8, 16, 0.2, dtype).nan_to_num(0.0).cuda()
    st = SparseConvTensor.from_dense(x)
    d = st.dense(channels_first=channels_first)
    ref = x.permute(0, 4, 1, 2, 3).contiguous() if channels_first else x
    assert d.shape == ref.shape and torch.equal(d, ref)


def test_empty_and_all_zero():
    x = torch.zeros((1, 4, 4, 4, 3), device="cuda")
    st = SparseConvTensor.from_dense(x)
    assert st.indices.shape == (0, 4) and st.features.shape == (0, 3)
    assert torch.equal(st.dense(), torch.zeros((1, 3, 4, 4, 4), device="cuda"))


def test_large_grid_count():
    x = _dense(9, 4, 128, 128, 128, 8, 0.02, torch.float16).cuda()
    idx, f = _native.dense_to_sparse(x)
    assert idx.shape[0] == int((x != 0).any(-1).sum().item())
    assert bool((idx[1:, 0].long() * 2 ** 21 + idx[1:, 1].long() * 2 ** 14 + idx[1:, 2].long() * 2 ** 7 + idx[1:, 3].long()
                 > idx[:-1, 0].long() * 2 ** 21 + idx[:-1, 1].long() * 2 ** 14 + idx[:-1, 2].long() * 2 ** 7 + idx[:-1, 3].long()).all())
