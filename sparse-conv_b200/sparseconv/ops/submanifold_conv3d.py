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
* The backward runs (the reference's autograd ``backward`` cannot be called, ``ops:186-206``):
  the input gradient uses the exact transposed map, which for even kernel sizes differs from
  the reference's flipped map (``ops:123-126``); for odd sizes they are the same.
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

        ``hashmap_ratio`` is accepted for signature compatibility; the library sizes the
        table itself (the next power of two >= 4M slots while that stays <= 64 MB, else >= 2M).
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
        """Conv over a built map (ops:63-103); every algorithm runs the CUDA kernels. The two
        split-K values (empty slots in the reference, ops:94-99) run the split-K variant, which
        spreads the heaviest tiles' offsets over two CTAs; the others run the unsplit kernel."""
        assert feats.is_contiguous(), "Input features should be contiguous."
        if algorithm not in _ALGORITHMS:
            raise ValueError(f"Unsupported Algorithm {algorithm}.")
        Co, Kw, Kh, Kd, Ci = weight.shape
        nbr, masks, order = _cache_tensors(neighbor_cache)
        if nbr.shape[1] != Kw * Kh * Kd:
            raise ValueError(
                f"neighbor map has {nbr.shape[1]} offsets, weight has {Kw * Kh * Kd}")
        split = algorithm in (Algorithm.IMPLICIT_GEMM_SPLITK, Algorithm.MASKED_IMPLICIT_GEMM_SPLITK)
        out = _native.conv_forward(feats, weight, bias, nbr, masks, order, split=split)
        _native.after_launch(out.device)
        return out

    @staticmethod
    def _sparse_submanifold_conv_backward(
        grad_output: torch.Tensor,
        feats: torch.Tensor,
        neighbor_cache: SubMConv3dNeighborCache,
        weight: torch.Tensor,
        bias: Optional[torch.Tensor] = None,
        algorithm: str = Algorithm.EXPLICIT_GEMM,
        needs: Tuple[bool, bool, bool] = None,
    ) -> Tuple[Optional[torch.Tensor], Optional[torch.Tensor], Optional[torch.Tensor]]:
        """(grad_feats, grad_weight, grad_bias) of the conv (ops:105-150); every algorithm runs
        the CUDA kernels.

        grad_feats is a forward conv of grad_output over the transposed map with the weight's
        channel axes swapped. For odd kernel sizes the transposed map is the reference's
        flipped map (ops:123-126) and the kernels read the forward map with the offsets
        reversed; for even sizes it is built (the exact transpose, where the flip is not) and
        cached on ``neighbor_cache`` as ``neighbor_map_t`` / ``masks_t``.
        grad_weight / grad_bias are accumulated in fp32 and returned in the parameters' dtypes.
        ``needs`` = which of (feats, weight, bias) want a gradient (default: requires_grad).
        """
        if algorithm not in _ALGORITHMS:
            raise ValueError(f"Unsupported Algorithm {algorithm}.")
        if needs is None:
            needs = (feats.requires_grad, weight.requires_grad,
                     bias is not None and bias.requires_grad)
        Co, Kw, Kh, Kd, Ci = weight.shape
        V = Kw * Kh * Kd
        nbr, masks, order = _cache_tensors(neighbor_cache)
        g = grad_output.to(feats.dtype).contiguous()
        grad_input = grad_weight = grad_bias = None
        if needs[0]:
            nbr_t = masks_t = None
            if V % 2 == 0:           # even sizes: the flipped map is not the transpose
                nbr_t = getattr(neighbor_cache, "neighbor_map_t", None)
                masks_t = getattr(neighbor_cache, "masks_t", None)
                if nbr_t is None:
                    nbr_t, masks_t = _native.transpose_neighbor_map(nbr)
                    neighbor_cache.neighbor_map_t, neighbor_cache.masks_t = nbr_t, masks_t
            grad_input = _native.conv_backward_input(g, weight, nbr, masks, order, nbr_t, masks_t)
        if needs[1] or (bias is not None and needs[2]):
            gw, gb = _native.conv_weight_grad(feats.contiguous(), g, nbr, order,
                                              with_bias=bias is not None and needs[2], masks=masks)
            if needs[1]:
                grad_weight = gw.view(Co, Kw, Kh, Kd, Ci).to(weight.dtype)
            if gb is not None:
                grad_bias = gb.to(bias.dtype)
        _native.after_launch(g.device)
        return grad_input, grad_weight, grad_bias

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
        ctx.algorithm = algorithm
        return output, neighbor_cache

    @staticmethod
    def backward(ctx, grad_output: torch.Tensor, _grad_cache=None):
        """Gradients for feats, weight and bias (ops:186-206, whose signature there cannot
        be called by autograd: it takes the cache's gradient as the algorithm)."""
        feats, weight, bias = ctx.saved_tensors
        needs = (ctx.needs_input_grad[0], ctx.needs_input_grad[4],
                 bias is not None and ctx.needs_input_grad[5])
        grad_input, grad_weight, grad_bias = SubMConv3dFunction._sparse_submanifold_conv_backward(
            grad_output, feats, ctx.neighbor_cache, weight, bias, ctx.algorithm, needs)
        return grad_input, None, None, None, grad_weight, grad_bias, None, None


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
