"""Conv parity on the GPU, through the C ABI and the public API.

Tolerances (stated by the workload spec): fp16/bf16 outputs within rtol 1e-2 / atol 1e-2
of a float64 evaluation on the same (rounded) inputs; fp32 within 1e-4.
"""
import os

import numpy as np
import pytest
import torch

import gpu_cases
from oracle import oracle
from sparseconv import SparseConvTensor, _native
from sparseconv.ops.submanifold_conv3d import Algorithm, sparse_submanifold_conv3d

pytestmark = pytest.mark.gpu

TOL = {torch.float32: dict(rtol=1e-4, atol=1e-4),
       torch.float16: dict(rtol=1e-2, atol=1e-2),
       torch.bfloat16: dict(rtol=1e-2, atol=1e-2)}
GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def _inputs(seed, M, Ci, Co, V, dtype, with_bias):
    g = torch.Generator().manual_seed(seed)
    feats = torch.randn((M, Ci), generator=g).to(dtype)
    weight = (torch.randn((Co, V, Ci), generator=g) / np.sqrt(V * Ci)).to(dtype)
    bias = torch.randn((Co,), generator=g).to(dtype) if with_bias else None
    return feats, weight, bias


def _oracle(feats, nbr, weight, bias):
    return oracle.conv_gather_f64(feats.double().numpy(), nbr, weight.double().numpy(),
                                  None if bias is None else bias.double().numpy())


def _gpu_conv(feats, weight, bias, nbr_t, masks, order, kernel):
    out = _native.conv_forward(feats.cuda(), weight.cuda(), None if bias is None else bias.cuda(),
                               nbr_t, masks, order, kernel=kernel)
    torch.cuda.synchronize()
    return out.float().cpu().numpy()


KERNELS = {"simt": _native.KERNEL_SIMT, "tcgen05": _native.KERNEL_TCGEN05}


@pytest.mark.parametrize("kernel", ["simt", "tcgen05"])
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("ci,co", [(16, 16), (32, 32), (64, 64), (128, 128), (16, 64), (128, 32), (64, 16)])
@pytest.mark.parametrize("case", ["rand3", "dense3", "rand5"])
def test_conv_matches_f64_oracle(kernel, dtype, ci, co, case):
    coords, shape, ks, dil = gpu_cases.small_cases()[case]
    N, _C, W, H, D = shape
    nbr, masks, order = _native.build_neighbor_map(torch.from_numpy(coords).cuda(), N, W, H, D, ks, dil)
    V = nbr.shape[1]
    feats, weight, bias = _inputs(ci * 7 + co, coords.shape[0], ci, co, V, dtype, with_bias=True)
    got = _gpu_conv(feats, weight, bias, nbr, masks, order, KERNELS[kernel])
    ref = _oracle(feats, nbr.cpu().numpy().view(np.uint32), weight, bias)
    np.testing.assert_allclose(got, ref, **TOL[dtype])


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("ci,co", [(16, 16), (32, 32), (64, 64), (128, 128)])
def test_tcgen05_mixed_density(dtype, ci, co):
    """Tiles of dense blocks and of isolated voxels in one launch (whole index rows staged for
    the former, per-offset contexts for the latter)."""
    coords, shape = gpu_cases.mixed_density_coords()
    N, _C, W, H, D = shape
    nbr, masks, order = _native.build_neighbor_map(torch.from_numpy(coords).cuda(), N, W, H, D,
                                                   (3, 3, 3), (1, 1, 1))
    feats, weight, bias = _inputs(ci + 3 * co, coords.shape[0], ci, co, nbr.shape[1], dtype, with_bias=True)
    got = _gpu_conv(feats, weight, bias, nbr, masks, order, _native.KERNEL_TCGEN05)
    ref = _oracle(feats, nbr.cpu().numpy().view(np.uint32), weight, bias)
    np.testing.assert_allclose(got, ref, **TOL[dtype])


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16])
@pytest.mark.parametrize("ci,co", [(3, 3), (3, 8), (48, 24), (16, 16)])
@pytest.mark.parametrize("case", sorted(gpu_cases.small_cases()))
def test_simt_all_shapes(dtype, ci, co, case):
    coords, shape, ks, dil = gpu_cases.small_cases()[case]
    N, _C, W, H, D = shape
    nbr, masks, order = _native.build_neighbor_map(torch.from_numpy(coords).cuda(), N, W, H, D, ks, dil)
    feats, weight, bias = _inputs(ci + co, coords.shape[0], ci, co, nbr.shape[1], dtype, with_bias=(ci % 2 == 1))
    got = _gpu_conv(feats, weight, bias, nbr, None, None, _native.KERNEL_AUTO)
    ref = _oracle(feats, nbr.cpu().numpy().view(np.uint32), weight, bias)
    np.testing.assert_allclose(got, ref, **TOL[dtype])


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_tcgen05_without_masks_or_order(dtype):
    coords, shape, ks, dil = gpu_cases.small_cases()["dil2"]
    N, _C, W, H, D = shape
    nbr, masks, order = _native.build_neighbor_map(torch.from_numpy(coords).cuda(), N, W, H, D, ks, dil)
    feats, weight, bias = _inputs(1, coords.shape[0], 32, 64, nbr.shape[1], dtype, with_bias=False)
    a = _gpu_conv(feats, weight, bias, nbr, None, None, _native.KERNEL_TCGEN05)
    b = _gpu_conv(feats, weight, bias, nbr, masks, order, _native.KERNEL_TCGEN05)
    c = _gpu_conv(feats, weight, bias, nbr, masks, None, _native.KERNEL_TCGEN05)
    # results do not depend on the row order or on skipped all-missing offsets: bit-identical
    np.testing.assert_array_equal(a, b)
    np.testing.assert_array_equal(a, c)


def test_readme_toy_through_public_api():
    """README.md:12-39 call form (algorithm in the bias slot) on the reference's own toy
    fixture; compared with the reference EXPLICIT_GEMM output and the float64 conv3d."""
    g = np.load(os.path.join(GOLDEN, "readme_toy.npz"))
    dense = torch.from_numpy(g["dense"]).cuda()
    sp = SparseConvTensor.from_dense(dense)
    feats, coords = sp.features, sp.indices
    shape = torch.Size((sp.batch_size, feats.shape[-1], *sp.spatial_shape))
    weight = torch.from_numpy(g["weight"]).cuda()
    out, cache = sparse_submanifold_conv3d(feats, coords, shape, weight, Algorithm.IMPLICIT_GEMM)
    np.testing.assert_array_equal(cache.neighbor_map.cpu().numpy(), g["neighbor_map"])
    np.testing.assert_allclose(out.cpu().numpy(), g["conv3d_f64_out"], rtol=1e-4, atol=1e-4)
    np.testing.assert_allclose(out.cpu().numpy(), g["reference_explicit_out"], rtol=1e-4, atol=1e-4)


class TestSubMConv3dReference:
    """The reference's tests/test_submanifold_conv3d.py on CUDA (seeded here)."""
    B, Cin, W, H, D = 3, 3, 5, 5, 5
    Kw, Kh, Kd = 3, 3, 3
    Cout = 3

    def _setup(self):
        g = torch.Generator().manual_seed(1)
        dense = torch.zeros((self.B, self.W, self.H, self.D, self.Cin))
        for i in range(self.W):
            dense[:, i, i, i, :] = torch.randn((self.Cin,), generator=g)
        dense = dense.cuda()
        sp = SparseConvTensor.from_dense(dense)
        feats, coords = sp.features, sp.indices
        shape = torch.Size((sp.batch_size, feats.shape[-1], *sp.spatial_shape))
        weight = torch.randn((self.Cout, self.Kw, self.Kh, self.Kd, self.Cin), generator=g).cuda()
        mask = dense != 0
        conv3d = torch.nn.Conv3d(self.Cin, self.Cout, (3, 3, 3), padding=1, bias=False).cuda().double()
        conv3d.weight = torch.nn.Parameter(weight.double().permute(0, -1, 1, 2, 3))
        with torch.no_grad():
            ref = conv3d(dense.double().permute(0, -1, 1, 2, 3)).permute(0, 2, 3, 4, 1)[mask]
        return feats, coords, shape, weight, ref

    def test_explicit_gemm_no_bias(self):
        feats, coords, shape, weight, ref = self._setup()
        out, _ = sparse_submanifold_conv3d(feats, coords, shape, weight)
        assert torch.allclose(ref.float(), out.view(-1), rtol=1e-4, atol=1e-4)

    def test_implicit_gemm_no_bias(self):
        feats, coords, shape, weight, ref = self._setup()
        out, _ = sparse_submanifold_conv3d(feats, coords, shape, weight, algorithm=Algorithm.IMPLICIT_GEMM)
        assert torch.allclose(ref.float(), out.view(-1), rtol=1e-4, atol=1e-4)

    def test_all_algorithms_agree(self):
        feats, coords, shape, weight, ref = self._setup()
        outs = [sparse_submanifold_conv3d(feats, coords, shape, weight, algorithm=a)[0]
                for a in (Algorithm.EXPLICIT_GEMM, Algorithm.IMPLICIT_GEMM, Algorithm.IMPLICIT_GEMM_SPLITK,
                          Algorithm.MASKED_IMPLICIT_GEMM, Algorithm.MASKED_IMPLICIT_GEMM_SPLITK)]
        for o in outs[1:]:
            assert torch.equal(o, outs[0])
        with pytest.raises(ValueError):
            sparse_submanifold_conv3d(feats, coords, shape, weight, algorithm="bogus")

    def test_cache_reuse_and_bias(self):
        feats, coords, shape, weight, ref = self._setup()
        bias = torch.randn(self.Cout, device="cuda")
        out1, cache = sparse_submanifold_conv3d(feats, coords, shape, weight, bias)
        out2, cache2 = sparse_submanifold_conv3d(feats, coords, shape, weight, bias, neighbor_cache=cache)
        assert cache2 is cache
        assert torch.equal(out1, out2)
        assert torch.allclose(out1.view(-1), (ref.view(-1, 3) + bias.double()).float().view(-1), rtol=1e-4, atol=1e-4)


@pytest.mark.parametrize("name", ["cube", "lidar", "indoor", "wide3", "wide5"])
def test_full_size_configs(name):
    """Full-size workloads through the public API; the float64 oracle is evaluated on a
    seeded sample of 4096 output rows (the map itself is checked bit-exact elsewhere)."""
    w = gpu_cases.workload(name)
    coords = torch.from_numpy(w.coords).cuda()
    feats = w.feats.cuda()
    weight = w.weight.cuda()
    out, cache = sparse_submanifold_conv3d(feats, coords, torch.Size(w.shape), weight,
                                           algorithm=Algorithm.IMPLICIT_GEMM)
    torch.cuda.synchronize()
    rows = np.sort(np.random.default_rng(0).choice(w.num_voxels, size=min(4096, w.num_voxels), replace=False))
    nbr = cache.neighbor_map.cpu().numpy()[rows]
    ref = oracle.conv_gather_f64(w.feats.double().numpy(), nbr, w.weight.double().numpy())
    np.testing.assert_allclose(out[torch.from_numpy(rows).cuda()].float().cpu().numpy(), ref, **TOL[w.dtype])
    # size-independent property: the same map reused gives bit-identical features
    out2, _ = sparse_submanifold_conv3d(feats, coords, torch.Size(w.shape), weight,
                                        neighbor_cache=cache, algorithm=Algorithm.IMPLICIT_GEMM)
    assert torch.equal(out, out2)
