"""The bounded-wait path of the tensor-core conv kernel, exercised on the GPU without a fault.

Every pipeline wait inside ``conv_tc_kernel`` has a time limit (2 s by default). Lowering the
limit to 1 ns through the C ABI (``spconv_set_wait_limit_ns``) makes the first wait that is not
already satisfied give up: the kernel raises ``SPCONV_STATUS_WAIT_TIMEOUT``, waits (bounded) for
its own copies, weight loads and MMAs, frees its tensor memory and returns. The host then sees
the status bit as a ``RuntimeError``, and, with the default limit restored, the same conv on the
same context gives the correct result.
"""
import pytest
import torch

from sparseconv import _native, synthetic

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("name", ["cube", "toy_c64"])
def test_wait_timeout_is_reported_and_the_context_stays_usable(name):
    dev = torch.device("cuda", 0)
    if name == "cube":
        w = synthetic.make("cube", seed=0)
    else:       # C = 64: the eight-gatherer launch shape (one CTA per SM)
        w = synthetic.cube(seed=1, batch=1, res=64, p=0.05, channels=64)
    coords = torch.from_numpy(w.coords).to(dev)
    feats, weight = w.feats.to(dev), w.weight.to(dev)
    N, _C, W, H, D = w.shape
    nbr, masks, order = _native.build_neighbor_map(coords, N, W, H, D, w.kernel_size, w.dilation)
    ref = _native.conv_forward(feats, weight, None, nbr, masks, order, kernel=_native.KERNEL_TCGEN05)
    torch.cuda.synchronize()
    _native.check_errors(dev)

    prev = _native.set_wait_limit_ns(1)
    try:
        out = _native.conv_forward(feats, weight, None, nbr, masks, order, kernel=_native.KERNEL_TCGEN05)
        torch.cuda.synchronize()           # the launch returns: every wait is bounded
    finally:
        _native.set_wait_limit_ns(prev)
    with pytest.raises(RuntimeError, match="wait reached its time limit"):
        _native.check_errors(dev)
    del out

    again = _native.conv_forward(feats, weight, None, nbr, masks, order, kernel=_native.KERNEL_TCGEN05)
    torch.cuda.synchronize()
    assert _native.check_errors(dev) & _native.STATUS_WAIT_TIMEOUT == 0
    assert torch.equal(again, ref)
