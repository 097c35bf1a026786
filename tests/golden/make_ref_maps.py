"""Writes golden kernel maps produced by the reference's OWN CUDA map builder.

Needs a CUDA device and ``oracle/_ref/sparseconv_ref_cuda.so`` (built from the reference's
sources by ``oracle/build_ref.py``). For each small case of ``tests/gpu_cases.py`` it
allocates the table exactly as the reference does (``ops/utils.py:3-16``: capacity
``int(2.0 * M)``, uint32 keys when N*W*H*D < 2^32 else uint64, filled with all-ones;
uint32 values) and calls ``hashmap_build_submanifold_conv_neighbor_map_cuda_naive``
(``neighbor_map.cu:179-237``). The table never fills (load 0.5), so the reference's
unbounded probe loops terminate.

    python tests/golden/make_ref_maps.py OUT.npz
"""
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "tests"))


def reference_map(mod, coords_np, shape, ks, dil):
    import torch
    N, _C, W, H, D = [int(s) for s in shape]
    coords = torch.from_numpy(np.ascontiguousarray(coords_np, dtype=np.int32)).cuda()
    M = coords.shape[0]
    cap = int(2.0 * M)
    if N * W * H * D < 2 ** 32:
        keys = torch.full((cap,), torch.iinfo(torch.uint32).max, dtype=torch.uint32, device="cuda")
    else:
        keys = torch.full((cap,), torch.iinfo(torch.uint64).max, dtype=torch.uint64, device="cuda")
    vals = torch.empty((cap,), dtype=torch.uint32, device="cuda")
    nbr = mod.hashmap_build_submanifold_conv_neighbor_map_cuda_naive(
        keys, vals, coords, W, H, D, int(ks[0]), int(ks[1]), int(ks[2]),
        int(dil[0]), int(dil[1]), int(dil[2]))
    torch.cuda.synchronize()
    return nbr.cpu().numpy().astype(np.uint32)


def main(out_path):
    import torch  # noqa: F401
    from oracle import build_ref
    import gpu_cases
    mod = build_ref.load()
    arrays = {}
    for name, (coords, shape, ks, dil) in sorted(gpu_cases.small_cases().items()):
        arrays[f"{name}__coords"] = coords
        arrays[f"{name}__shape"] = np.asarray(shape, dtype=np.int64)
        arrays[f"{name}__kernel"] = np.asarray(ks, dtype=np.int64)
        arrays[f"{name}__dilation"] = np.asarray(dil, dtype=np.int64)
        arrays[f"{name}__map"] = reference_map(mod, coords, shape, ks, dil)
        print(name, coords.shape[0], "voxels", flush=True)
    np.savez_compressed(out_path, **arrays)
    print("wrote", out_path)


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else os.path.join(ROOT, "tests", "golden", "ref_maps.npz"))
