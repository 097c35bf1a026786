"""The backward oracle (CPU): the exact float64 gradients of the gather formula against
torch autograd and against the reference's EXPLICIT_GEMM backward formula
(ops/submanifold_conv3d.py:117-143)."""
import numpy as np
import pytest
import torch

from oracle import oracle


def _case(seed, B, R, p, ks, dil=(1, 1, 1), ci=5, co=4):
    rng = np.random.default_rng(seed)
    occ = rng.random((B, R, R, R)) < p
    coords = np.ascontiguousarray(np.argwhere(occ).astype(np.int32))
    shape = (B, ci, R, R, R)
    nbr = oracle.neighbor_map(coords, shape, ks, dil)
    V = int(np.prod(ks))
    f = rng.standard_normal((coords.shape[0], ci))
    w = rng.standard_normal((co, V, ci))
    g = rng.standard_normal((coords.shape[0], co))
    return nbr, f, w, g


def _autograd(nbr, f, w, g):
    """torch autograd of out[i] = sum_v f[nbr[i,v]] @ w[:, v, :]^T + b, in float64."""
    nb = torch.as_tensor(nbr.view(np.int32).astype(np.int64))
    ft = torch.tensor(f, requires_grad=True)
    wt = torch.tensor(w, requires_grad=True)
    bt = torch.zeros(w.shape[0], dtype=torch.float64, requires_grad=True)
    out = bt.expand(nb.shape[0], -1).clone()
    for v in range(nb.shape[1]):
        valid = nb[:, v] >= 0
        rows = torch.zeros((nb.shape[0], f.shape[1]), dtype=torch.float64)
        rows = torch.where(valid[:, None], ft[nb[:, v].clamp(min=0)], rows)
        out = out + rows @ wt[:, v, :].t()
    (out * torch.as_tensor(g)).sum().backward()
    return ft.grad.numpy(), wt.grad.numpy(), bt.grad.numpy()


@pytest.mark.parametrize("ks,dil", [((3, 3, 3), (1, 1, 1)), ((5, 5, 5), (1, 1, 1)), ((2, 2, 2), (1, 1, 1)),
                                    ((4, 3, 2), (1, 2, 3)), ((3, 3, 3), (2, 2, 2)), ((1, 1, 1), (1, 1, 1))])
def test_backward_oracle_is_the_gradient(ks, dil):
    nbr, f, w, g = _case(3, 2, 9, 0.25, ks, dil)
    for got, ref in zip(oracle.conv_backward_f64(f, nbr, w, g), _autograd(nbr, f, w, g)):
        np.testing.assert_allclose(got, ref, rtol=1e-12, atol=1e-12)


@pytest.mark.parametrize("ks,dil", [((3, 3, 3), (1, 1, 1)), ((5, 5, 5), (1, 1, 1)), ((3, 1, 3), (2, 1, 1))])
def test_reference_formula_agrees_for_odd_kernels(ks, dil):
    nbr, f, w, g = _case(5, 2, 9, 0.3, ks, dil)
    for got, ref in zip(oracle.explicit_gemm_backward_f64(f, nbr, w, g), oracle.conv_backward_f64(f, nbr, w, g)):
        np.testing.assert_allclose(got, ref, rtol=1e-12, atol=1e-12)


def test_reference_flip_is_not_the_transpose_for_even_kernels():
    nbr, f, w, g = _case(7, 1, 8, 0.4, (2, 2, 2))
    ref_gf = oracle.explicit_gemm_backward_f64(f, nbr, w, g)[0]
    exact_gf = oracle.conv_backward_f64(f, nbr, w, g)[0]
    assert not np.allclose(ref_gf, exact_gf)
    # the weight and bias gradients do not involve the flip
    for got, ref in zip(oracle.explicit_gemm_backward_f64(f, nbr, w, g)[1:], oracle.conv_backward_f64(f, nbr, w, g)[1:]):
        np.testing.assert_allclose(got, ref, rtol=1e-12, atol=1e-12)
