"""Generic table bindings (the reference's hashmap_insert_cuda / hashmap_lookup_cuda,
hash.cu:8-146): against a dict, and against the reference's own insert / lookup run live (the
tables share their layout and slots, so each side reads the other's)."""
import os

import numpy as np
import pytest
import torch

from oracle import build_ref
from sparseconv import _native

pytestmark = pytest.mark.gpu


def _table(cap, kdt, vdt):
    return (torch.full((cap,), torch.iinfo(kdt).max, dtype=kdt, device="cuda"),
            torch.zeros((cap,), dtype=vdt, device="cuda"))


def _keys(seed, n, kdt):
    rng = np.random.default_rng(seed)
    hi = 2 ** 31 if kdt == torch.uint32 else 2 ** 62
    k = np.unique(rng.integers(0, hi, size=n * 2, dtype=np.int64))[:n]
    rng.shuffle(k)
    return k


@pytest.mark.parametrize("kdt", [torch.uint32, torch.uint64])
@pytest.mark.parametrize("vdt", [torch.uint32, torch.uint64])
def test_insert_lookup_matches_dict(kdt, vdt):
    n, cap = 50000, 100000
    k = _keys(1, n, kdt)
    v = np.arange(n, dtype=np.int64) * 7 + 3
    tk, tv = _table(cap, kdt, vdt)
    kt = torch.from_numpy(k).to(kdt).cuda() if kdt == torch.uint64 else torch.from_numpy(k.astype(np.uint32)).cuda()
    vt = torch.from_numpy(v.astype(np.uint64 if vdt == torch.uint64 else np.uint32)).cuda()
    _native.hashmap_insert(tk, tv, kt, vt)
    q = np.concatenate([k[::3], _keys(2, 1000, kdt)])
    qt = torch.from_numpy(q).to(kdt).cuda() if kdt == torch.uint64 else torch.from_numpy(q.astype(np.uint32)).cuda()
    got = _native.hashmap_lookup(tk, tv, qt).cpu().numpy().astype(np.uint64)
    d = dict(zip(k.tolist(), v.tolist()))
    miss = np.iinfo(np.uint64 if vdt == torch.uint64 else np.uint32).max
    ref = np.array([d.get(int(x), miss) for x in q], dtype=np.uint64)
    np.testing.assert_array_equal(got, ref)


def test_full_table_is_reported_not_spun():
    tk, tv = _table(64, torch.uint32, torch.uint32)
    _native.reset_status(torch.device("cuda"))
    with pytest.raises(RuntimeError):
        _native.hashmap_insert(tk, tv, torch.from_numpy(np.arange(100, dtype=np.uint32)).cuda(),
                               torch.from_numpy(np.arange(100, dtype=np.uint32)).cuda())
        torch.cuda.synchronize()
        _native.check_errors(torch.device("cuda"))
    _native.reset_status(torch.device("cuda"))


@pytest.fixture(scope="module")
def ref_module():
    if not os.path.exists(build_ref.OUT):
        pytest.skip("oracle/_ref was not built (reference sources absent where it was built)")
    return build_ref.load()


@pytest.mark.parametrize("kdt", [torch.uint32, torch.uint64])
def test_tables_interoperate_with_the_reference(ref_module, kdt):
    n, cap = 20000, 40000
    k = _keys(3, n, kdt)
    kt = torch.from_numpy(k).to(kdt).cuda() if kdt == torch.uint64 else torch.from_numpy(k.astype(np.uint32)).cuda()
    vt = torch.from_numpy((np.arange(n) + 11).astype(np.uint32)).cuda()
    # built here, read by the reference
    tk, tv = _table(cap, kdt, torch.uint32)
    _native.hashmap_insert(tk, tv, kt, vt)
    r1 = ref_module.hashmap_lookup_cuda(tk, tv, kt)
    # built by the reference, read here
    tk2, tv2 = _table(cap, kdt, torch.uint32)
    ref_module.hashmap_insert_cuda(tk2, tv2, kt, vt)
    r2 = _native.hashmap_lookup(tk2, tv2, kt)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(r1.cpu().numpy().astype(np.int64), vt.cpu().numpy().astype(np.int64))
    np.testing.assert_array_equal(r2.cpu().numpy().astype(np.int64), vt.cpu().numpy().astype(np.int64))
