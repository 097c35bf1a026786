"""Writes ``tests/golden/readme_toy.npz``: the README toy run through the reference's OWN
Python code (``/root/reference/src/sparseconv``) on CPU.

The reference's map builder is CUDA-only, so its EXPLICIT_GEMM forward
(``ops/submanifold_conv3d.py:76-86``) is driven with a precomputed ``neighbor_cache``:
the known-answer map of the toy, derived by hand from ``neighbor_map.cu:145-176`` (voxel
(b,i,i,i) at row 5b+i has its own row at offset 13, row-1 at offset 0 (i>0) and row+1 at
offset 26 (i<4)). ``flex_gemm`` (an unused import of ``implicit_gemm.py:5-6``) and the
CUDA extension module are stubbed so the package imports without them.

Stored arrays: dense [3,5,5,5,3] float32 input, feats/coords from the reference's
``SparseConvTensor.from_dense``, weight [3,3,3,3,3], the known-answer map, the reference
EXPLICIT_GEMM output (float32), and the reference test's own oracle
(``tests/test_submanifold_conv3d.py:25-26``: ``nn.Conv3d`` with the permuted weight, here in
float64) read at the active voxels.

Run in a container that has the reference mounted:
    python tests/golden/make_golden.py
"""
import os
import sys
import types

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REF_SRC = "/root/reference/src"


def _import_reference():
    flex = types.ModuleType("flex_gemm")
    flex_ops = types.ModuleType("flex_gemm.ops")
    flex_spconv = types.ModuleType("flex_gemm.ops.spconv")
    flex_spconv.sparse_submanifold_conv3d = None
    flex.ops = flex_ops
    flex_ops.spconv = flex_spconv
    sys.modules.update({"flex_gemm": flex, "flex_gemm.ops": flex_ops,
                        "flex_gemm.ops.spconv": flex_spconv})
    sys.path.insert(0, REF_SRC)
    import sparseconv.kernels as kernels  # noqa: E402
    cuda_stub = types.ModuleType("sparseconv.kernels.cuda")
    sys.modules["sparseconv.kernels.cuda"] = cuda_stub
    kernels.cuda = cuda_stub
    from sparseconv.core import SparseConvTensor
    from sparseconv.ops import submanifold_conv3d as ops
    return SparseConvTensor, ops


def toy_map() -> np.ndarray:
    B, W, V = 3, 5, 27
    nbr = np.full((B * W, V), 0xFFFFFFFF, dtype=np.uint32)
    for b in range(B):
        for i in range(W):
            r = b * W + i
            nbr[r, 13] = r
            if i > 0:
                nbr[r, 0] = r - 1
            if i < W - 1:
                nbr[r, 26] = r + 1
    return nbr


def main():
    import torch
    SparseConvTensor, ops = _import_reference()
    g = torch.Generator().manual_seed(0)
    B, Cin, W, H, D = 3, 3, 5, 5, 5
    Cout = 3
    dense = torch.zeros((B, W, H, D, Cin))
    for i in range(W):
        dense[:, i, i, i, :] = torch.randn((Cin,), generator=g)
    weight = torch.randn((Cout, 3, 3, 3, Cin), generator=g)
    sp = SparseConvTensor.from_dense(dense)
    feats, coords = sp.features, sp.indices
    shape = torch.Size((sp.batch_size, feats.shape[-1], *sp.spatial_shape))
    nbr = toy_map()
    cache = ops.SubMConv3dNeighborCache(neighbor_map=torch.from_numpy(nbr))
    out, _ = ops.sparse_submanifold_conv3d(feats, coords, shape, weight, neighbor_cache=cache)
    conv = torch.nn.Conv3d(Cin, Cout, (3, 3, 3), padding=1, bias=False).double()
    conv.weight = torch.nn.Parameter(weight.double().permute(0, -1, 1, 2, 3))
    with torch.no_grad():
        ref_dense = conv(dense.double().permute(0, -1, 1, 2, 3)).permute(0, 2, 3, 4, 1)
    c = coords.long()
    conv_at_active = ref_dense[c[:, 0], c[:, 1], c[:, 2], c[:, 3]]
    path = os.path.join(HERE, "readme_toy.npz")
    np.savez_compressed(
        path, dense=dense.numpy(), feats=feats.numpy(), coords=coords.numpy(),
        shape=np.asarray(list(shape), dtype=np.int64), weight=weight.numpy(), neighbor_map=nbr,
        reference_explicit_out=out.detach().numpy(), conv3d_f64_out=conv_at_active.numpy())
    print("wrote", path, "M =", feats.shape[0])


if __name__ == "__main__":
    main()
