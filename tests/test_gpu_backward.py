"""Backward parity on the GPU: transposed map (bit-exact), weight / bias gradients and the
input gradient against the float64 backward oracle, and autograd through the public API.

Tolerances: 16-bit inputs within rtol 1e-2 and atol 1e-2 x max|reference| of the float64
evaluation on the same rounded inputs (the weight gradient sums over up to M voxels); fp32
within 1e-4 x max|reference|."""
import numpy as np
import pytest
import torch

import gpu_cases
from oracle import oracle
from sparseconv import _native
from sparseconv.ops.submanifold_conv3d import Algorithm, sparse_submanifold_conv3d

pytestmark = pytest.mark.gpu

RTOL = {torch.float32: 1e-4, torch.float16: 1e-2, torch.bfloat16: 1e-2}


def _close(got, ref, dtype, what):
    scale = max(1.0, float(np.abs(ref).max())) if ref.size else 1.0
    np.testing.assert_allclose(got, ref, rtol=RTOL[dtype], atol=RTOL[dtype] * scale, err_msg=what)


def _map(coords, shape, ks, dil):
    N, _C, W, H, D = shape
    return _native.build_neighbor_map(torch.from_numpy(coords).cuda(), N, W, H, D, ks, dil)


def _transpose_np(nbr):
    nb = nbr.view(np.int32)
    M, V = nb.shape
    out = np.full((M, V), -1, np.int32)
    i, v = np.nonzero(nb >= 0)
    out[nb[i, v], v] = i
    return out


CASES = sorted(gpu_cases.small_cases())


@pytest.mark.parametrize("case", CASES)
def test_transposed_map_bit_exact(case):
    coords, shape, ks, dil = gpu_cases.small_cases()[case]
    nbr, masks, order = _map(coords, shape, ks, dil)
    nbr_t, masks_t = _native.transpose_neighbor_map(nbr)
    ref = _transpose_np(nbr.cpu().numpy())
    np.testing.assert_array_equal(nbr_t.cpu().numpy(), ref)
    V = ref.shape[1]
    bits = np.zeros((ref.shape[0], (V + 31) // 32), np.uint64)
    for v in range(V):
        bits[:, v // 32] |= (ref[:, v] >= 0).astype(np.uint64) << np.uint64(v % 32)
    np.testing.assert_array_equal(masks_t.cpu().numpy().view(np.uint32).astype(np.uint64), bits)
    if all(k % 2 == 1 for k in ks):     # odd sizes: the transpose is the reference's flip
        np.testing.assert_array_equal(ref, nbr.cpu().numpy().view(np.int32)[:, ::-1])


def _grads(seed, coords, shape, ks, dil, ci, co, dtype):
    nbr, masks, order = _map(coords, shape, ks, dil)
    g = torch.Generator().manual_seed(seed)
    M, V = nbr.shape
    f = torch.randn((M, ci), generator=g).to(dtype)
    w = (torch.randn((co, V, ci), generator=g) / np.sqrt(V * ci)).to(dtype)
    go = torch.randn((M, co), generator=g).to(dtype)
    ref = oracle.conv_backward_f64(f.double().numpy(), nbr.cpu().numpy(), w.double().numpy(), go.double().numpy())
    return nbr, masks, order, f, w, go, ref


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16, torch.float32])
@pytest.mark.parametrize("ci,co", [(64, 64), (128, 128), (64, 128), (128, 64), (16, 16), (32, 32), (3, 8), (48, 24)])
@pytest.mark.parametrize("case", ["rand3", "dense3", "rand5", "even2"])
def test_weight_and_bias_grad(dtype, ci, co, case):
    coords, shape, ks, dil = gpu_cases.small_cases()[case]
    nbr, masks, order, f, w, go, (gf_ref, gw_ref, gb_ref) = _grads(ci + 7 * co, coords, shape, ks, dil, ci, co, dtype)
    gw, gb = _native.conv_weight_grad(f.cuda(), go.cuda(), nbr, order)
    torch.cuda.synchronize()
    _close(gw.cpu().numpy(), gw_ref, dtype, "grad_weight")
    _close(gb.cpu().numpy(), gb_ref, dtype, "grad_bias")


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("ci,co", [(64, 64), (128, 128)])
def test_weight_grad_mixed_density(dtype, ci, co):
    """Tiles with and without a neighbour at each offset (the skip path of the tensor-core
    weight-gradient kernel), without and with the voxel order."""
    coords, shape = gpu_cases.mixed_density_coords()
    nbr, masks, order, f, w, go, (_gf, gw_ref, _gb) = _grads(3, coords, shape, (3, 3, 3), (1, 1, 1), ci, co, dtype)
    for od in (order, None):
        gw, gb = _native.conv_weight_grad(f.cuda(), go.cuda(), nbr, od, with_bias=False)
        torch.cuda.synchronize()
        assert gb is None
        _close(gw.cpu().numpy(), gw_ref, dtype, "grad_weight")


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16, torch.float32])
@pytest.mark.parametrize("ci,co", [(32, 32), (64, 16), (3, 3)])
@pytest.mark.parametrize("case", ["rand3", "rand5", "even2", "aniso", "dil2", "single", "k1"])
def test_autograd_through_public_api(dtype, ci, co, case):
    coords, shape, ks, dil = gpu_cases.small_cases()[case]
    c = torch.from_numpy(coords).cuda()
    M = coords.shape[0]
    V = int(np.prod(ks))
    g = torch.Generator().manual_seed(ci * 3 + co)
    f = torch.randn((M, ci), generator=g).to(dtype)
    w = (torch.randn((co, *ks, ci), generator=g) / np.sqrt(V * ci)).to(dtype)
    b = torch.randn((co,), generator=g).to(dtype)
    r = torch.randn((M, co), generator=g).to(dtype)
    fd = f.cuda().requires_grad_(True)
    wd = w.cuda().requires_grad_(True)
    bd = b.cuda().requires_grad_(True)
    out, cache = sparse_submanifold_conv3d(fd, c, torch.Size(shape), wd, bd, dilation=dil,
                                           algorithm=Algorithm.IMPLICIT_GEMM)
    (out * r.cuda()).sum().backward()
    torch.cuda.synchronize()
    gf_ref, gw_ref, gb_ref = oracle.conv_backward_f64(
        f.double().numpy(), cache.neighbor_map.cpu().numpy(), w.double().numpy().reshape(co, V, ci),
        r.double().numpy())
    _close(fd.grad.float().cpu().numpy(), gf_ref, dtype, "grad_feats")
    _close(wd.grad.float().cpu().numpy().reshape(co, V, ci), gw_ref, dtype, "grad_weight")
    _close(bd.grad.float().cpu().numpy(), gb_ref, dtype, "grad_bias")
    assert fd.grad.dtype == dtype and wd.grad.dtype == dtype and bd.grad.dtype == dtype


def test_autograd_only_the_requested_gradients():
    coords, shape, ks, dil = gpu_cases.small_cases()["rand3"]
    c = torch.from_numpy(coords).cuda()
    f = torch.randn((coords.shape[0], 16), device="cuda", dtype=torch.float16)
    w = torch.randn((16, 3, 3, 3, 16), device="cuda", dtype=torch.float16, requires_grad=True)
    out, cache = sparse_submanifold_conv3d(f, c, torch.Size(shape), w, algorithm=Algorithm.IMPLICIT_GEMM)
    out.float().sum().backward()
    assert f.grad is None and w.grad is not None
    assert getattr(cache, "neighbor_map_t", None) is None     # odd kernel: never a transposed map


@pytest.mark.parametrize("name", ["cube", "lidar"])
def test_full_size_backward(name):
    """Full-size workloads: weight and bias gradients in full, the input gradient on a seeded
    sample of 4096 rows."""
    w_ = gpu_cases.workload(name)
    c = torch.from_numpy(w_.coords).cuda()
    f = w_.feats.cuda().requires_grad_(True)
    wt = w_.weight.cuda().requires_grad_(True)
    Co = int(w_.weight.shape[0])
    g = torch.Generator().manual_seed(1)
    r = torch.randn((w_.num_voxels, Co), generator=g).to(w_.dtype)
    out, cache = sparse_submanifold_conv3d(f, c, torch.Size(w_.shape), wt, algorithm=Algorithm.IMPLICIT_GEMM)
    (out * r.cuda()).sum().backward()
    torch.cuda.synchronize()
    V = int(np.prod(w_.kernel_size))
    Ci = int(w_.weight.shape[-1])
    gf_ref, gw_ref, _gb = oracle.conv_backward_f64(
        w_.feats.double().numpy(), cache.neighbor_map.cpu().numpy(),
        w_.weight.double().numpy().reshape(Co, V, Ci), r.double().numpy())
    _close(wt.grad.float().cpu().numpy().reshape(Co, V, Ci), gw_ref, w_.dtype, "grad_weight")
    rows = np.sort(np.random.default_rng(0).choice(w_.num_voxels, size=4096, replace=False))
    _close(f.grad.float().cpu().numpy()[rows], gf_ref[rows], w_.dtype, "grad_feats")


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16, torch.float32])
@pytest.mark.parametrize("ci,co", [(32, 32), (64, 64), (16, 128), (3, 8)])
@pytest.mark.parametrize("case", ["rand3", "dense3", "rand5", "dil2", "aniso", "even2", "k1"])
def test_backward_input_flip_and_transpose(dtype, ci, co, case):
    """The input gradient with the offsets reversed (odd kernel volumes) and over the built
    transposed map (any volume) agree with the oracle, with and without masks / order."""
    coords, shape, ks, dil = gpu_cases.small_cases()[case]
    nbr, masks, order, f, w, go, (gf_ref, _gw, _gb) = _grads(ci + co, coords, shape, ks, dil, ci, co, dtype)
    V = nbr.shape[1]
    nbr_t, masks_t = _native.transpose_neighbor_map(nbr)
    variants = [(masks, order, nbr_t, masks_t), (None, None, nbr_t, None)]
    if V % 2 == 1:
        variants += [(masks, order, None, None), (None, None, None, None)]
    for mk, od, nt, mt in variants:
        gf = _native.conv_backward_input(go.cuda(), w.cuda(), nbr, mk, od, nt, mt)
        torch.cuda.synchronize()
        _close(gf.float().cpu().numpy(), gf_ref, dtype, "grad_feats")
