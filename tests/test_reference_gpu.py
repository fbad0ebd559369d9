"""The reference's own GPU path against this library's drop-in, same inputs.

oracle/_ref/libref_gpu.so is src/spmv_kernel/preFreeSpMV.cu compiled unmodified
for sm_100a (oracle/Makefile). Both entry points take the same host CSR
(include/PreFree.h:3-5) and overwrite y. With the harness's integer values
(i % 15, include/common.h:126-133) every partial sum is an exact integer, so
the reference's GPU result, this library's result and the CPU oracle must agree
bit for bit. The cases keep row 0 within the reference's first 512-non-zero
tile: a longer row 0 trips its start-row sentinel (start_row = 0 read as "no
row", src/spmv_kernel/preFreeSpMV.cu:431-432), after which its own output is
not a product of A and x.
"""
import numpy as np
import pytest

from csr_cases import case

pytestmark = pytest.mark.gpu


def mod15(k):
    return (np.arange(k) % 15).astype(np.float64)


@pytest.mark.parametrize("name", ["uniform16", "powerlaw", "empty_edges", "mixed_long",
                                  "unsorted"])
def test_reference_gpu_matches_dropin_bit_exact(pf, oracle, name):
    if not oracle.ref_gpu_available():
        pytest.skip("oracle/_ref/libref_gpu.so not built")
    rp, col, _, n = case(name, seed=41)
    m, nnz = len(rp) - 1, len(col)
    assert int(rp[1]) - int(rp[0]) <= 512, "row 0 must fit the reference's first tile"
    val = mod15(nnz)
    x = mod15(n)
    rp32 = rp.astype(np.int32)
    y_ref_gpu, t_ref, _ = oracle.ref_gpu_prefree(val, rp32, col, x, m, n)
    y = np.full(m, np.nan)
    t, _ = pf.preFreeSpMV(val, rp32, col, x, y, m, n, nnz)
    y_cpu = oracle.ref_serial(rp32, col, val, x)
    assert np.array_equal(y_ref_gpu, y_cpu), "reference GPU path differs from its CPU oracle"
    assert np.array_equal(y, y_cpu)
    assert t > 0 and t_ref > 0
