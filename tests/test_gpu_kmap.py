"""Kernel-map parity on the GPU: the library's map must equal the oracle's (and so the
reference's) bit for bit; masks and order must be consistent with it. Calls go through
the C ABI (``sparseconv._native``)."""
import numpy as np
import pytest
import torch

import gpu_cases
from oracle import oracle
from sparseconv import _native

pytestmark = pytest.mark.gpu


def gpu_map(coords, shape, ks, dil):
    N, _C, W, H, D = shape
    c = torch.from_numpy(np.ascontiguousarray(coords)).cuda()
    nbr, masks, order = _native.build_neighbor_map(c, N, W, H, D, ks, dil)
    torch.cuda.synchronize()
    return (nbr.cpu().numpy().view(np.uint32), masks.cpu().numpy().view(np.uint32),
            order.cpu().numpy())


def check_masks_and_order(nbr, masks, order, grid_cells=None):
    M, V = nbr.shape
    MW = (V + 31) // 32
    assert masks.shape == (M, MW)
    valid = nbr != 0xFFFFFFFF
    expect = np.zeros((M, MW), dtype=np.uint64)
    for v in range(V):
        expect[:, v // 32] |= valid[:, v].astype(np.uint64) << np.uint64(v % 32)
    np.testing.assert_array_equal(masks.astype(np.uint64), expect)
    assert np.array_equal(np.sort(order), np.arange(M, dtype=np.int32)), "order is a permutation"
    if M:
        cls = np.minimum(valid.sum(1) - 1, 15)[order]
        assert np.all(np.diff(cls) >= 0), "order groups voxels by neighbour-count class"
    if radix_order(M, grid_cells) and V <= RADIX_MAX_V:
        # large maps of small kernels: exactly the stable sort by (class, mask without centre)
        np.testing.assert_array_equal(order, np.argsort(order_keys(masks[:, 0], V), kind="stable"))


RADIX_MIN_VOXELS, RADIX_MAX_V = 1 << 19, 27
RADIX_SPARSE_MIN_VOXELS, RADIX_SPARSE_DENSITY = 1 << 17, 0.003


def radix_order(M, grid_cells):
    """The library's choice of the radix order (by size, and for sparse grids above 2^17)."""
    if M >= RADIX_MIN_VOXELS:
        return True
    return grid_cells is not None and M > RADIX_SPARSE_MIN_VOXELS and M <= RADIX_SPARSE_DENSITY * grid_cells


def order_keys(m, V):
    """min(popcount - 1, 15) above the top 20 bits of the mask without its centre bit."""
    m = m.astype(np.int64) & ((1 << V) - 1)
    c = V // 2
    comp = (m & ((1 << c) - 1)) | ((m >> (c + 1)) << c)
    drop = max(V - 1 - 20, 0)
    popc = np.zeros_like(m)
    for v in range(V):
        popc += (m >> v) & 1
    cls = np.clip(popc - 1, 0, 15)
    return (cls << (V - 1 - drop)) | (comp >> drop)


@pytest.mark.parametrize("name", sorted(gpu_cases.small_cases()))
def test_small_cases_bit_exact(name):
    coords, shape, ks, dil = gpu_cases.small_cases()[name]
    nbr, masks, order = gpu_map(coords, shape, ks, dil)
    np.testing.assert_array_equal(nbr, oracle.neighbor_map(coords, shape, ks, dil))
    check_masks_and_order(nbr, masks, order)


@pytest.mark.parametrize("batch", [1, 2])
def test_sparse_grid_radix_order(batch):
    """One or two indoor samples (250k / 500k voxels filling 0.19 % of the grid: the per-rank
    inputs of the benchmark's batch split at 8 and 4 ranks): bit-exact map and the radix order,
    exactly the stable sort of the keys."""
    from sparseconv import synthetic
    w = synthetic.make("indoor", seed=0, batch=batch)
    nbr, masks, order = gpu_map(w.coords, w.shape, w.kernel_size, w.dilation)
    np.testing.assert_array_equal(nbr, oracle.neighbor_map(w.coords, w.shape, w.kernel_size, w.dilation))
    cells = int(np.prod(w.shape[:1])) * int(np.prod(w.shape[2:]))
    assert radix_order(w.num_voxels, cells) == (w.num_voxels > RADIX_SPARSE_MIN_VOXELS)
    check_masks_and_order(nbr, masks, order, cells)


@pytest.mark.parametrize("name", ["cube", "lidar", "indoor", "wide3", "wide5"])
def test_full_size_configs_bit_exact(name):
    w = gpu_cases.workload(name)
    nbr, masks, order = gpu_map(w.coords, w.shape, w.kernel_size, w.dilation)
    ref = oracle.neighbor_map(w.coords, w.shape, w.kernel_size, w.dilation)
    np.testing.assert_array_equal(nbr, ref)
    check_masks_and_order(nbr, masks, order)


def test_readme_toy_known_answer():
    import os
    g = np.load(os.path.join(os.path.dirname(__file__), "golden", "readme_toy.npz"))
    nbr, masks, order = gpu_map(g["coords"], tuple(g["shape"]), (3, 3, 3), (1, 1, 1))
    np.testing.assert_array_equal(nbr, g["neighbor_map"])


def test_empty_input():
    nbr, masks, order = gpu_map(np.zeros((0, 4), np.int32), (1, 1, 4, 4, 4), (3, 3, 3), (1, 1, 1))
    assert nbr.shape == (0, 27) and order.shape == (0,)


def test_unsorted_input_matches_oracle():
    coords, shape, ks, dil = gpu_cases.small_cases()["rand3"]
    perm = np.random.default_rng(0).permutation(coords.shape[0])
    c = np.ascontiguousarray(coords[perm])
    nbr, masks, order = gpu_map(c, shape, ks, dil)
    np.testing.assert_array_equal(nbr, oracle.neighbor_map(c, shape, ks, dil))


def test_duplicate_coordinates_keep_highest_row():
    coords = np.array([[0, 1, 1, 1], [0, 1, 1, 2], [0, 1, 1, 1], [0, 3, 3, 3]], dtype=np.int32)
    _native.reset_status()
    nbr, _, _ = gpu_map(coords, (1, 1, 5, 5, 5), (3, 3, 3), (1, 1, 1))
    np.testing.assert_array_equal(nbr, oracle.neighbor_map(coords, (1, 1, 5, 5, 5), (3, 3, 3)))
    bits = _native.check_errors(torch.device("cuda", 0))
    assert bits & _native.STATUS_DUPLICATE
    _native.reset_status()


def test_duplicate_next_to_its_z_neighbour_uses_the_highest_row():
    """Sorted input whose z + 1 neighbour repeats: the adjacent row holds that coordinate but is
    not the highest row of it, so the map build must probe (its own record of the duplicate,
    kept in the call's workspace) rather than take the adjacent row. Repeated with the device
    status word already holding a duplicate from an earlier call and after a clean call."""
    dup = np.array([[0, 1, 1, 1], [0, 1, 1, 2], [0, 1, 1, 2], [0, 1, 2, 1]], dtype=np.int32)
    clean = np.array([[0, 1, 1, 1], [0, 1, 1, 2], [0, 1, 2, 1]], dtype=np.int32)
    shape = (1, 1, 5, 5, 5)
    _native.reset_status()
    for coords in (dup, dup, clean, dup):
        nbr, _, _ = gpu_map(coords, shape, (3, 3, 3), (1, 1, 1))
        np.testing.assert_array_equal(nbr, oracle.neighbor_map(coords, shape, (3, 3, 3)))
    assert _native.check_errors(torch.device("cuda", 0)) & _native.STATUS_DUPLICATE
    _native.reset_status()


def test_out_of_range_coordinates_raise():
    coords = torch.tensor([[0, 1, 1, 1], [0, 5, 1, 1]], dtype=torch.int32, device="cuda")
    _native.reset_status()
    _native.build_neighbor_map(coords, 1, 5, 5, 5, (3, 3, 3), (1, 1, 1))
    with pytest.raises(RuntimeError, match="outside the spatial shape"):
        _native.check_errors(torch.device("cuda", 0))
    _native.reset_status()


def test_repeated_builds_reuse_workspace():
    coords, shape, ks, dil = gpu_cases.small_cases()["rand5"]
    a = gpu_map(coords, shape, ks, dil)[0]
    b = gpu_map(coords, shape, ks, dil)[0]
    np.testing.assert_array_equal(a, b)


def test_non_default_stream():
    coords, shape, ks, dil = gpu_cases.small_cases()["dense3"]
    N, _C, W, H, D = shape
    s = torch.cuda.Stream()
    c = torch.from_numpy(coords).cuda()
    torch.cuda.synchronize()
    with torch.cuda.stream(s):
        nbr, masks, order = _native.build_neighbor_map(c, N, W, H, D, ks, dil)
    s.synchronize()
    np.testing.assert_array_equal(nbr.cpu().numpy().view(np.uint32),
                                  oracle.neighbor_map(coords, shape, ks, dil))


@pytest.mark.parametrize("name", ["rand3", "rand5", "aniso", "dense3"])
def test_hash_only_path_matches_bitmap_path(name):
    """Grids of <= 2^30 cells screen probes with an occupancy bitmap when the workspace has
    room for it; with a workspace too small for the bitmap the build probes the hash table
    alone. Both must give the oracle's map."""
    coords, shape, ks, dil = gpu_cases.small_cases()[name]
    N, _C, W, H, D = shape
    lib = _native.load_library()
    c = torch.from_numpy(coords).cuda()
    M, V = coords.shape[0], ks[0] * ks[1] * ks[2]
    full = _native.workspace_bytes(M, N, W, H, D)
    a256 = lambda x: (x + 255) // 256 * 256
    bitmap_bytes = a256((((N * W * H * D) + 31) // 32) * 4)
    # 3x3x3 kernels on grids of < 2^32 cells and <= 2^23 columns also get the sorted-input
    # path's column ranges and keys; leave them out too, so only the hash table remains.
    sorted_bytes = a256(N * W * H * 8) + a256(M * 4) if N * W * H * D < 2 ** 32 and N * W * H <= 2 ** 23 else 0
    ws = torch.empty((full - bitmap_bytes - sorted_bytes,), dtype=torch.uint8, device="cuda")
    nbr = torch.empty((M, V), dtype=torch.int32, device="cuda")
    masks = torch.empty((M, (V + 31) // 32), dtype=torch.int32, device="cuda")
    order = torch.empty((M,), dtype=torch.int32, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    rc = lib.spconv_build_submanifold_neighbor_map(
        c.data_ptr(), M, N, W, H, D, *ks, *dil, ws.data_ptr(), ws.numel(), nbr.data_ptr(),
        masks.data_ptr(), order.data_ptr(), status.data_ptr(), torch.cuda.current_stream().cuda_stream)
    assert rc == 0, lib.spconv_last_error()
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    np.testing.assert_array_equal(nbr.cpu().numpy().view(np.uint32), oracle.neighbor_map(coords, shape, ks, dil))


@pytest.mark.parametrize("ks,dil", [((3, 3, 3), (1, 1, 1)), ((2, 2, 2), (1, 1, 1)), ((3, 3, 1), (1, 1, 1)),
                                    ((1, 1, 1), (1, 1, 1)), ((3, 3, 3), (2, 2, 2)), ((5, 5, 1), (1, 1, 1))])
def test_radix_order_large_maps(ks, dil):
    """Maps of >= 2^19 voxels take the radix-sort order (1 to 4 digit passes by kernel size)."""
    rng = np.random.default_rng(11)
    B, R = 1, 128
    coords = np.ascontiguousarray(np.argwhere(rng.random((B, R, R, R)) < 0.3).astype(np.int32))
    assert coords.shape[0] >= RADIX_MIN_VOXELS
    nbr, masks, order = gpu_map(coords, (B, 1, R, R, R), ks, dil)
    check_masks_and_order(nbr, masks, order)


def _edge_coords(seed, B, W, H, D, p):
    """Random voxels plus every cell on the z = 0 and z = D - 1 faces of some columns, so that
    flat keys of neighbouring columns are adjacent (z = D - 1 of one column, z = 0 of the
    next): a z +- d neighbour must never be taken from the next or previous column."""
    rng = np.random.default_rng(seed)
    occ = rng.random((B, W, H, D)) < p
    occ[:, :, :, 0] |= rng.random((B, W, H)) < 0.5
    occ[:, :, :, D - 1] |= rng.random((B, W, H)) < 0.5
    occ[:, 0, :, :] |= rng.random((B, H, D)) < 0.3
    occ[:, W - 1, :, :] |= rng.random((B, H, D)) < 0.3
    return np.ascontiguousarray(np.argwhere(occ).astype(np.int32))


@pytest.mark.parametrize("dil", [(1, 1, 1), (2, 2, 2), (1, 2, 3), (3, 1, 2)])
def test_sorted_path_column_edges(dil):
    """Sorted 3x3x3 input takes the column path (binary searches inside each (b, x, y)
    column's row range): grid faces and adjacent-column keys, several dilations."""
    B, W, H, D = 2, 9, 7, 6
    coords = _edge_coords(21, B, W, H, D, 0.15)
    shape = (B, 1, W, H, D)
    nbr, masks, order = gpu_map(coords, shape, (3, 3, 3), dil)
    np.testing.assert_array_equal(nbr, oracle.neighbor_map(coords, shape, (3, 3, 3), dil))
    check_masks_and_order(nbr, masks, order)


@pytest.mark.parametrize("swap", ["adjacent", "far", "equal"])
def test_nearly_sorted_input_takes_the_hash_path(swap):
    """One out-of-order pair (or one repeated row) in otherwise sorted input: the device-side
    sortedness test sends the build to the hash path, whose map must still be the oracle's."""
    coords, shape, ks, dil = gpu_cases.small_cases()["dense3"]
    c = coords.copy()
    M = c.shape[0]
    if swap == "adjacent":
        c[[M // 2, M // 2 + 1]] = c[[M // 2 + 1, M // 2]]
    elif swap == "far":
        c[[5, M - 5]] = c[[M - 5, 5]]
    else:
        c[M // 3] = c[M // 3 - 1]
    _native.reset_status()
    nbr, masks, order = gpu_map(c, shape, ks, dil)
    np.testing.assert_array_equal(nbr, oracle.neighbor_map(c, shape, ks, dil))
    _native.reset_status()


def test_sorted_then_unsorted_reuse_one_workspace():
    """Alternating sorted and shuffled inputs through one workspace: each call clears what its
    path reads (column ranges every call, table and bitmap on the hash path)."""
    coords, shape, ks, dil = gpu_cases.small_cases()["rand3"]
    N, _C, W, H, D = shape
    perm = np.random.default_rng(5).permutation(coords.shape[0])
    shuffled = np.ascontiguousarray(coords[perm])
    M = coords.shape[0]
    ws = torch.empty((_native.workspace_bytes(M, N, W, H, D),), dtype=torch.uint8, device="cuda")
    for c in (coords, shuffled, coords, shuffled):
        t = torch.from_numpy(c).cuda()
        nbr, _m, _o = _native.build_neighbor_map(t, N, W, H, D, ks, dil, workspace=ws)
        torch.cuda.synchronize()
        np.testing.assert_array_equal(nbr.cpu().numpy().view(np.uint32), oracle.neighbor_map(c, shape, ks, dil))
