"""The allocation-free kernel-map entry point, ``spconv_build_submanifold_neighbor_map_noalloc``,
called through the C ABI and checked against the workspace entry point on two calls in a row.

It exists for callers that cannot allocate device memory where they build the map: operator
plugin hosts that hand over only input and output buffers, fixed-memory real-time loops that
must not call cudaMalloc (it can synchronise the device and can fail under memory pressure),
and runtimes whose allocator must not run at that point. Its scratch is one array compiled
into the library, shared by every call on a device, so the second call here (a smaller input
after a larger one) also checks that a call clears what the previous one left behind.

This file is named to be collected last; it passes alone in a fresh process and after the
rest of the suite.
"""
import ctypes

import numpy as np
import pytest
import torch

import gpu_cases
from sparseconv import _native

pytestmark = pytest.mark.gpu


def _noalloc_map(lib, coords_np, shape, ks, dil):
    N, _C, W, H, D = shape
    dev = torch.device("cuda", 0)
    coords = torch.from_numpy(np.ascontiguousarray(coords_np)).to(dev)
    M = coords.shape[0]
    V = ks[0] * ks[1] * ks[2]
    # The test owns every buffer; the entry point allocates nothing.
    nbr = torch.full((M, V), 7, dtype=torch.int32, device=dev)
    masks = torch.full((M, (V + 31) // 32), 7, dtype=torch.int32, device=dev)
    order = torch.full((M,), -5, dtype=torch.int32, device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    rc = lib.spconv_build_submanifold_neighbor_map_noalloc(
        coords.data_ptr(), M, N, W, H, D, ks[0], ks[1], ks[2], dil[0], dil[1], dil[2],
        nbr.data_ptr(), masks.data_ptr(), order.data_ptr(), status.data_ptr(),
        torch.cuda.current_stream(dev).cuda_stream)
    assert rc == 0, lib.spconv_last_error()
    torch.cuda.synchronize(dev)
    return coords, nbr, masks, order, int(status.item())


def _bucket_keys(masks_np):
    """Order key of each voxel (popcount class, 8-bit mask hash), as the map kernel forms it."""
    def fmix32(k):
        k = k.astype(np.uint64)
        k ^= k >> np.uint64(16)
        k = (k * np.uint64(0x85EBCA6B)) & np.uint64(0xFFFFFFFF)
        k ^= k >> np.uint64(13)
        k = (k * np.uint64(0xC2B2AE35)) & np.uint64(0xFFFFFFFF)
        k ^= k >> np.uint64(16)
        return k
    m = masks_np.view(np.uint32).astype(np.uint64)
    h = np.full(m.shape[0], 0x9E3779B9, dtype=np.uint64)
    pc = np.zeros(m.shape[0], dtype=np.int64)
    for w in range(m.shape[1]):
        h = fmix32(h ^ m[:, w])
        pc += np.array([bin(int(x)).count("1") for x in m[:, w]], dtype=np.int64)
    cls = np.minimum(np.maximum(pc - 1, 0), 15)
    return cls * 256 + (h & np.uint64(255)).astype(np.int64)


def _check_against_workspace_entry_point(lib, coords_np, shape, ks, dil):
    coords, nbr, masks, order, status = _noalloc_map(lib, coords_np, shape, ks, dil)
    N, _C, W, H, D = shape
    ref_nbr, ref_masks, ref_order = _native.build_neighbor_map(coords, N, W, H, D, ks, dil)
    torch.cuda.synchronize()
    assert status == 0
    assert torch.equal(nbr, ref_nbr)                        # bit-exact map
    assert torch.equal(masks, ref_masks)                    # bit-exact masks
    o, ro = order.cpu().numpy(), ref_order.cpu().numpy()
    assert np.array_equal(np.sort(o), np.arange(len(o), dtype=np.int32))
    keys = _bucket_keys(masks.cpu().numpy())
    assert np.array_equal(keys[o], keys[ro])                # same buckets at every position
    # and the conv gives the same bits over either map / order
    g = torch.Generator().manual_seed(0)
    V = nbr.shape[1]
    feats = torch.randn((nbr.shape[0], 32), generator=g).half().cuda()
    weight = (torch.randn((32, V, 32), generator=g) * 0.05).half().cuda()
    a = _native.conv_forward(feats, weight, None, nbr, masks, order)
    b = _native.conv_forward(feats, weight, None, ref_nbr, ref_masks, ref_order)
    torch.cuda.synchronize()
    assert torch.equal(a, b)


def test_noalloc_matches_workspace_entry_point_on_two_calls():
    lib = _native.load_library()
    cube = gpu_cases.workload("cube")                       # 168,546 voxels, then a small case
    calls = [(cube.coords, cube.shape, cube.kernel_size, cube.dilation),
             gpu_cases.small_cases()["rand5"]]
    for coords_np, shape, ks, dil in calls:
        _check_against_workspace_entry_point(lib, coords_np, shape, ks, dil)


def _limit_sized_coords(seed=11):
    """Exactly SPCONV_NOALLOC_MAX_COORDS distinct voxels of a 2 x 128^3 grid, sorted."""
    rng = np.random.default_rng(seed)
    cells = np.sort(rng.choice(2 * 128 ** 3, size=_native.NOALLOC_MAX_COORDS, replace=False))
    b, r = np.divmod(cells, 128 ** 3)
    x, r = np.divmod(r, 128 ** 2)
    y, z = np.divmod(r, 128)
    return np.ascontiguousarray(np.stack([b, x, y, z], 1).astype(np.int32)), (2, 1, 128, 128, 128)


def test_noalloc_64bit_keys_then_limit_sized_input():
    """The 64-bit-key layout (grid volume >= 2^32), the one that sets the scratch size, and then
    an input of exactly the entry point's limit, again two calls in a row."""
    lib = _native.load_library()
    c64, s64 = gpu_cases.key64_coords(8)
    assert s64[0] * s64[2] * s64[3] * s64[4] >= 2 ** 32
    climit, slimit = _limit_sized_coords()
    assert climit.shape[0] == _native.NOALLOC_MAX_COORDS
    for coords_np, shape in ((c64, s64), (climit, slimit)):
        _check_against_workspace_entry_point(lib, coords_np, shape, (3, 3, 3), (1, 1, 1))


def test_noalloc_rejects_inputs_over_its_limit():
    lib = _native.load_library()
    M = _native.NOALLOC_MAX_COORDS + 1
    rc = lib.spconv_build_submanifold_neighbor_map_noalloc(
        None, M, 1, 4, 4, 4, 3, 3, 3, 1, 1, 1, None, None, None, None, None)
    assert rc == _native.SPCONV_ERR_ARG
    assert b"no-alloc limit" in lib.spconv_last_error()
