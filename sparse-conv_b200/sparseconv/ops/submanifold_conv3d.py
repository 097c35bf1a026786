"""Submanifold 3D sparse convolution: the reference's operator interface
(``src/sparseconv/ops/submanifold_conv3d.py``) on the sm_100a CUDA library.

Same names, argument meanings and return values as the reference:

* ``Algorithm`` string constants (``ops:10-15``);
* ``SubMConv3dNeighborCache`` attribute bag with ``[]`` access (``ops:17-26``); the cache
  built here carries ``neighbor_map`` ([M, V] uint32, 0xFFFFFFFF = missing, bit-identical
  to the reference's map) plus ``masks`` and ``order`` that the conv kernels use;
* ``SubMConv3dFunction`` (``ops:28-206``) and ``sparse_submanifold_conv3d`` (``ops:208-236``),
  returning ``(out_feats [M, Co], neighbor_cache)``.

Differences, all deliberate:

* Every algorithm value runs the CUDA kernels (the tcgen05 kernel for fp16/bf16 with 16,
  32, 64 or 128 channels, the SIMT kernel otherwise). The reference's EXPLICIT_GEMM (torch
  im2col + mm) and the unimplemented ``*_SPLITK`` / ``MASKED_*`` slots (bare ``pass`` there,
  ``ops:94-99``) all produce the same result here.
* The README's positional call ``sparse_submanifold_conv3d(feats, coords, shape, weight,
  Algorithm.IMPLICIT_GEMM)`` passes the algorithm in the ``bias`` slot; the reference then
  fails inside ``addmm``. Here an ``Algorithm`` string in that slot is taken as the algorithm.
* CPU tensors raise: there is no CPU path.
* Bias is added in fp32 before the single rounding to the feature dtype (the reference's
  Triton kernel rounds first and adds the bias in the feature dtype).
* Out-of-range coordinates raise ``RuntimeError`` (the reference silently aliases keys).
"""
from __future__ import annotations

from typing import Optional, Tuple

import torch
from torch.autograd import Function

from sparseconv import _native


class Algorithm:
    EXPLICIT_GEMM = "explicit_gemm"
    IMPLICIT_GEMM = "implicit_gemm"
    IMPLICIT_GEMM_SPLITK = "implicit_gemm_splitk"
    MASKED_IMPLICIT_GEMM = "masked_implicit_gemm"
    MASKED_IMPLICIT_GEMM_SPLITK = "masked_implicit_gemm_splitk"


_ALGORITHMS = (
    Algorithm.EXPLICIT_GEMM,
    Algorithm.IMPLICIT_GEMM,
    Algorithm.IMPLICIT_GEMM_SPLITK,
    Algorithm.MASKED_IMPLICIT_GEMM,
    Algorithm.MASKED_IMPLICIT_GEMM_SPLITK,
)


class SubMConv3dNeighborCache:
    def __init__(self, **kwargs):
        for k, v in kwargs.items():
            setattr(self, k, v)

    def __getitem__(self, key):
        return getattr(self, key)

    def __setitem__(self, key, value):
        setattr(self, key, value)


def _cache_tensors(cache: SubMConv3dNeighborCache):
    nbr = cache.neighbor_map
    if nbr.dtype == torch.uint32:
        nbr = nbr.view(torch.int32)
    elif nbr.dtype == torch.int64:
        nbr = nbr.to(torch.int32)
    return nbr.contiguous(), getattr(cache, "masks", None), getattr(cache, "order", None)


class SubMConv3dFunction(Function):
    @staticmethod
    def _compute_neighbor_cache(
        coords: torch.Tensor,
        shape: torch.Size,
        kernel_size: Tuple[int, int, int],
        dilation: Tuple[int, int, int],
        algorithm: str = Algorithm.EXPLICIT_GEMM,
        hashmap_ratio: float = 2.0,
    ) -> SubMConv3dNeighborCache:
        """Build the kernel map of ``coords`` (ops:29-61).

        ``hashmap_ratio`` is accepted for signature compatibility; the table always has
        the next power of two >= 2M slots (load factor <= 0.5), which the library sizes.
        """
        assert coords.is_contiguous(), "Coords should be contiguous."
        assert coords.dtype == torch.int32, "Unsupported coords dtype. Expected int32."
        N, C, W, H, D = shape
        if algorithm not in _ALGORITHMS:
            raise ValueError(f"Unsupported Algorithm {algorithm}.")
        if not coords.is_cuda:
            raise NotImplementedError("CPU version of hashmap is not implemented.")
        nbr, masks, order = _native.build_neighbor_map(
            coords, int(N), int(W), int(H), int(D), kernel_size, dilation)
        return SubMConv3dNeighborCache(
            neighbor_map=nbr.view(torch.uint32),
            masks=masks,
            order=order,
            kernel_size=tuple(int(k) for k in kernel_size),
            dilation=tuple(int(d) for d in dilation),
        )

    @staticmethod
    def _sparse_submanifold_conv_forward(
        feats: torch.Tensor,
        neighbor_cache: SubMConv3dNeighborCache,
        weight: torch.Tensor,
        bias: Optional[torch.Tensor] = None,
        algorithm: str = Algorithm.EXPLICIT_GEMM,
    ) -> torch.Tensor:
        """Conv over a built map (ops:63-103); every algorithm runs the CUDA kernels."""
        assert feats.is_contiguous(), "Input features should be contiguous."
        if algorithm not in _ALGORITHMS:
            raise ValueError(f"Unsupported Algorithm {algorithm}.")
        Co, Kw, Kh, Kd, Ci = weight.shape
        nbr, masks, order = _cache_tensors(neighbor_cache)
        if nbr.shape[1] != Kw * Kh * Kd:
            raise ValueError(
                f"neighbor map has {nbr.shape[1]} offsets, weight has {Kw * Kh * Kd}")
        out = _native.conv_forward(feats, weight, bias, nbr, masks, order)
        _native.after_launch(out.device)
        return out

    @staticmethod
    def forward(
        ctx,
        feats: torch.Tensor,
        coords: torch.Tensor,
        shape: torch.Size,
        neighbor_cache: Optional[SubMConv3dNeighborCache],
        weight: torch.Tensor,
        bias: Optional[torch.Tensor] = None,
        dilation: Tuple[int, int, int] = (1, 1, 1),
        algorithm: str = Algorithm.EXPLICIT_GEMM,
    ) -> Tuple[torch.Tensor, SubMConv3dNeighborCache]:
        Co, Kw, Kh, Kd, Ci = weight.shape
        assert feats.shape[-1] == Ci, \
            f"Input channels ({feats.shape[-1]}) should match weight channels ({Ci})"
        if neighbor_cache is None:
            neighbor_cache = SubMConv3dFunction._compute_neighbor_cache(
                coords, shape, (Kw, Kh, Kd), dilation)
        output = SubMConv3dFunction._sparse_submanifold_conv_forward(
            feats, neighbor_cache, weight, bias, algorithm)
        ctx.save_for_backward(feats, weight, bias)
        ctx.neighbor_cache = neighbor_cache
        return output, neighbor_cache

    @staticmethod
    def backward(ctx, grad_output: torch.Tensor, _grad_cache=None):
        raise NotImplementedError(
            "sparseconv: the submanifold conv backward is not available in this build "
            "(the reference's backward is not functional either)")


def sparse_submanifold_conv3d(
    feats: torch.Tensor,
    coords: torch.Tensor,
    shape: torch.Size,
    weight: torch.Tensor,
    bias: Optional[torch.Tensor] = None,
    neighbor_cache: Optional[SubMConv3dNeighborCache] = None,
    dilation: Tuple[int, int, int] = (1, 1, 1),
    algorithm: str = Algorithm.EXPLICIT_GEMM,
) -> Tuple[torch.Tensor, SubMConv3dNeighborCache]:
    """Sparse submanifold convolution for 3D input (ops:208-236).

    Args:
        feats: [N, C] input features (fp32, fp16 or bf16), contiguous, on CUDA.
        coords: [N, 4] int32 (b, x, y, z) coordinates, contiguous, on CUDA.
        shape: NCWHD size of the input.
        weight: [Co, Kw, Kh, Kd, Ci] weights (cast to the feature dtype).
        bias: [Co] bias or None. An ``Algorithm`` string here is taken as ``algorithm``
            (the README's positional form).
        neighbor_cache: a cache returned by an earlier call on the same coordinates and
            kernel size, or None to build it.
        dilation: kernel dilation.
        algorithm: any ``Algorithm`` value; all run the CUDA kernels.

    Returns:
        (output [N, Co] in the feature dtype, neighbor_cache)
    """
    if isinstance(bias, str):
        algorithm, bias = bias, None
    return SubMConv3dFunction.apply(feats, coords, shape, neighbor_cache, weight, bias,
                                    tuple(dilation), algorithm)
