"""Split-K forward (``spconv_submanifold_conv_forward_splitk``, the ``*_SPLITK`` algorithms):
the heaviest tiles' active offsets run as two halves on different CTAs, whose fp32 partials the
second half to finish adds. Checked against the float64 oracle (same tolerances as the unsplit
kernel), against the unsplit kernel, and run to run: the two-term fp32 sum commutes, so repeated
launches give identical bits whichever half finishes last."""
import numpy as np
import pytest
import torch

import gpu_cases
from oracle import oracle
from sparseconv import _native
from sparseconv.ops.submanifold_conv3d import Algorithm, sparse_submanifold_conv3d

pytestmark = pytest.mark.gpu

TOL = {torch.float16: dict(rtol=1e-2, atol=1e-2), torch.bfloat16: dict(rtol=1e-2, atol=1e-2)}


def _inputs(seed, M, Ci, Co, V, dtype):
    g = torch.Generator().manual_seed(seed)
    feats = torch.randn((M, Ci), generator=g).to(dtype)
    weight = (torch.randn((Co, V, Ci), generator=g) / np.sqrt(V * Ci)).to(dtype)
    bias = torch.randn((Co,), generator=g).to(dtype)
    return feats.cuda(), weight.cuda(), bias.cuda()


def _case(name):
    if name == "mixed":
        coords, shape = gpu_cases.mixed_density_coords()
        return coords, shape, (3, 3, 3), (1, 1, 1)
    return gpu_cases.small_cases()[name]


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("ci,co", [(16, 16), (32, 32), (64, 64), (128, 128), (32, 128), (64, 16)])
@pytest.mark.parametrize("case", ["dense3", "mixed", "rand5"])
@pytest.mark.parametrize("with_masks", [True, False])
def test_splitk_matches_oracle_and_is_deterministic(dtype, ci, co, case, with_masks):
    coords, shape, ks, dil = _case(case)
    N, _C, W, H, D = shape
    nbr, masks, order = _native.build_neighbor_map(torch.from_numpy(coords).cuda(), N, W, H, D, ks, dil)
    if not with_masks:           # every offset active: all of the first tiles split
        masks, order = None, None
    feats, weight, bias = _inputs(ci * 5 + co, coords.shape[0], ci, co, nbr.shape[1], dtype)
    a = _native.conv_forward(feats, weight, bias, nbr, masks, order, split=True)
    b = _native.conv_forward(feats, weight, bias, nbr, masks, order, split=True)
    u = _native.conv_forward(feats, weight, bias, nbr, masks, order)
    torch.cuda.synchronize()
    _native.check_errors()
    assert torch.equal(a, b)                                     # run to run
    ref = oracle.conv_gather_f64(feats.double().cpu().numpy(), nbr.cpu().numpy().view(np.uint32),
                                 weight.double().cpu().numpy(), bias.double().cpu().numpy())
    np.testing.assert_allclose(a.float().cpu().numpy(), ref, **TOL[dtype])
    np.testing.assert_allclose(a.float().cpu().numpy(), u.float().cpu().numpy(), **TOL[dtype])


@pytest.mark.parametrize("algorithm", [Algorithm.IMPLICIT_GEMM_SPLITK, Algorithm.MASKED_IMPLICIT_GEMM_SPLITK])
def test_splitk_algorithms_full_cube(algorithm):
    w = gpu_cases.workload("cube")
    coords, feats, weight = torch.from_numpy(w.coords).cuda(), w.feats.cuda(), w.weight.cuda()
    out, cache = sparse_submanifold_conv3d(feats, coords, torch.Size(w.shape), weight, algorithm=algorithm)
    out2, _ = sparse_submanifold_conv3d(feats, coords, torch.Size(w.shape), weight,
                                        neighbor_cache=cache, algorithm=algorithm)
    torch.cuda.synchronize()
    assert torch.equal(out, out2)
    rows = np.sort(np.random.default_rng(1).choice(w.num_voxels, size=4096, replace=False))
    ref = oracle.conv_gather_f64(w.feats.double().numpy(), cache.neighbor_map.cpu().numpy()[rows],
                                 w.weight.double().numpy())
    np.testing.assert_allclose(out[torch.from_numpy(rows).cuda()].float().cpu().numpy(), ref, **TOL[w.dtype])


def test_splitk_workspace_size_and_validation():
    lib = _native.load_library()
    assert lib.spconv_conv_splitk_workspace_bytes(128 * 1000, 64) == 4096 + 256 * 2 * 128 * 64 * 4
    assert lib.spconv_conv_splitk_workspace_bytes(130, 32) == 4096 + 2 * 2 * 128 * 32 * 4
    coords, shape, ks, dil = gpu_cases.small_cases()["dense3"]
    N, _C, W, H, D = shape
    nbr, masks, order = _native.build_neighbor_map(torch.from_numpy(coords).cuda(), N, W, H, D, ks, dil)
    feats, weight, bias = _inputs(0, coords.shape[0], 32, 32, nbr.shape[1], torch.float16)
    out = torch.empty((coords.shape[0], 32), dtype=torch.float16, device="cuda")
    rc = lib.spconv_submanifold_conv_forward_splitk(
        feats.data_ptr(), 1, coords.shape[0], 32, weight.data_ptr(), None, 32, nbr.shape[1], nbr.data_ptr(),
        masks.data_ptr(), order.data_ptr(), None, 0, out.data_ptr(), None, None)
    assert rc == _native.SPCONV_ERR_ARG
    assert b"split-K workspace" in lib.spconv_last_error()
