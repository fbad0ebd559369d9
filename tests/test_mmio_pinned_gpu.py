"""pf_mmio_read_pinned / pf_mmio_read_cached_pinned: the Matrix Market reader
writing its CSR straight into page-locked host memory. The arrays must equal
the heap reader's bit for bit, be page-locked according to the CUDA runtime
(cudaPointerGetAttributes: host memory type), go through the host-buffer
multiply (pf_spmv_host_f64_i64) to the oracle's result, and be freed by
pf_free (the arrays' owner hands them back when the last view goes)."""
import os

import numpy as np
import pytest

from test_mmio import write_random_mtx

pytestmark = pytest.mark.gpu


def page_locked(ptr: int) -> bool:
    from cuda.bindings import runtime as rt
    err, attr = rt.cudaPointerGetAttributes(ptr)
    assert err == rt.cudaError_t.cudaSuccess
    return attr.type == rt.cudaMemoryType.cudaMemoryTypeHost


@pytest.mark.parametrize("symmetry", ["general", "symmetric"])
def test_pinned_reader_matches_and_multiplies(pf, oracle, tmp_path, symmetry):
    import torch
    torch.cuda.init()
    rng = np.random.default_rng(41)
    path = os.path.join(tmp_path, f"a_{symmetry}.mtx")
    write_random_mtx(path, rng, 3000, 3000, 40000, symmetry=symmetry)
    heap = pf.mmio_read(path)
    pin = pf.mmio_read(path, pinned=True)
    assert heap[:4] == pin[:4]
    for a, b in zip(heap[4:], pin[4:]):
        assert np.array_equal(a, b)
    _, n, _, _, rp, col, val = pin
    for arr in (rp, col, val):
        assert page_locked(arr.ctypes.data)
    assert not page_locked(heap[4].ctypes.data)
    x = np.random.default_rng(42).uniform(-1, 1, n)
    y = np.zeros(len(rp) - 1)
    h = pf.Handle()
    pf.spmv_host(h, rp, col, val, x, y)
    h.close()
    ref = oracle.serial(rp, col, val, x)
    a, comp = oracle.abs_comp(rp, col, val, x)
    ok, worst, nbad = oracle.tolerance_report(y, ref, a, 1e-12, y_comp=comp)
    assert ok, f"{nbad} rows out of tolerance (worst {worst:.3g})"
    del pin, rp, col, val    # pf_free on page-locked arrays


def test_pinned_cached_reader(pf, tmp_path):
    import torch
    torch.cuda.init()
    rng = np.random.default_rng(43)
    path = os.path.join(tmp_path, "b.mtx")
    cache = os.path.join(tmp_path, "b.csr")
    write_random_mtx(path, rng, 2000, 2500, 30000)
    first, hit1 = pf.mmio_read_cached(path, cache, pinned=True)
    again, hit2 = pf.mmio_read_cached(path, cache, pinned=True)
    assert (hit1, hit2) == (False, True)
    for a, b in zip(first[4:], again[4:]):
        assert np.array_equal(a, b)
        assert page_locked(b.ctypes.data)
