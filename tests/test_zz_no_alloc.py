"""pf_spmv_noalloc_f64_i32, the multiply for callers that cannot allocate
device memory (an application that has reserved the GPU's memory for itself,
or code that must not call cudaMalloc mid-run because it can synchronize the
device and fail under memory pressure).

Checked through the C ABI, on two calls in a row (the second call reuses the
built-in scratch the first one left behind), against both the regular entry
point pf_spmv_f64_i32 on the same inputs and the CPU oracle's spmv_serial,
with the fp64 tolerance used throughout the tests: per row
|y - y_ref| <= 1e-12 * sum_j |a_ij x_j| (scaled by |alpha| and |beta|). The
test buffers are allocated by torch, as the caller's own memory would be.

The refusal of more than the built-in 2048 slices cannot be reached on a
B200: the slice count is at most the SM count times the kernel's occupancy
(444 there).
"""
import ctypes as C

import numpy as np
import pytest

from csr_cases import case

pytestmark = pytest.mark.gpu

EPS = 1e-12


def noalloc(pf, m, n, nnz, d_rp, d_col, d_val, alpha, d_x, beta, y, stream):
    return pf.lib.pf_spmv_noalloc_f64_i32(m, n, nnz, d_rp.data_ptr(), d_col.data_ptr(),
                                          d_val.data_ptr(), alpha, d_x.data_ptr(), beta,
                                          y.data_ptr(), C.c_void_p(stream))


def check_rows(oracle, got, ref, scale, what):
    ok, worst, nbad = oracle.tolerance_report(got, ref, scale, EPS)
    assert ok, f"{what}: {nbad} rows out of tolerance (worst {worst:.3g})"


@pytest.mark.parametrize("name", ["powerlaw", "mixed_long", "row0_long", "empty_edges"])
def test_noalloc_matches_regular_entry_point(pf, oracle, name):
    import torch
    assert torch.cuda.is_available()
    rp, col, val, n = case(name, seed=31)
    x = np.random.default_rng(32).uniform(-1, 1, n)
    m, nnz = len(rp) - 1, len(col)
    d_rp = torch.from_numpy(rp.astype(np.int32)).cuda()
    d_col = torch.from_numpy(col).cuda()
    d_val = torch.from_numpy(val).cuda()
    d_x = torch.from_numpy(x).cuda()
    stream = torch.cuda.current_stream().cuda_stream

    h = pf.Handle()
    y_ref = torch.zeros(m, dtype=torch.float64, device="cuda")
    pf.spmv(h, m, n, nnz, d_rp, d_col, d_val, d_x, y_ref, 1.5, 0.0)
    torch.cuda.synchronize()
    assert h.device_error() == 0
    h.close()
    ref = y_ref.cpu().numpy()
    a, comp = oracle.abs_comp(rp, col, val, x)
    serial = 1.5 * oracle.serial(rp, col, val, x)

    for call in range(2):
        y = torch.full((m,), float("nan"), dtype=torch.float64, device="cuda")
        st = noalloc(pf, m, n, nnz, d_rp, d_col, d_val, 1.5, d_x, 0.0, y, stream)
        assert st == 0, pf.lib.pf_last_error()
        got = y.cpu().numpy()
        check_rows(oracle, got, ref, 1.5 * a, f"call {call} vs pf_spmv_f64_i32")
        ok, worst, nbad = oracle.tolerance_report(got, serial, 1.5 * a, EPS, y_comp=1.5 * comp)
        assert ok, f"call {call} vs spmv_serial: {nbad} rows out of tolerance (worst {worst:.3g})"


def test_noalloc_beta_and_empty_matrix(pf, oracle):
    import torch
    rp, col, val, n = case("powerlaw", seed=33)
    m, nnz = len(rp) - 1, len(col)
    x = np.random.default_rng(34).uniform(-1, 1, n)
    y0 = np.random.default_rng(35).uniform(-1, 1, m)
    args = [torch.from_numpy(a).cuda() for a in (rp.astype(np.int32), col, val, x)]
    stream = torch.cuda.current_stream().cuda_stream
    h = pf.Handle()
    y_ref = torch.from_numpy(y0.copy()).cuda()
    pf.spmv(h, m, n, nnz, *args, y_ref, 0.5, -2.0)
    torch.cuda.synchronize()
    h.close()
    a, _ = oracle.abs_comp(rp, col, val, x)
    scale = 0.5 * a + 2.0 * np.abs(y0)
    serial = 0.5 * oracle.serial(rp, col, val, x) - 2.0 * y0
    for call in range(2):
        y = torch.from_numpy(y0.copy()).cuda()
        st = noalloc(pf, m, n, nnz, *args[:3], 0.5, args[3], -2.0, y, stream)
        assert st == 0, pf.lib.pf_last_error()
        got = y.cpu().numpy()
        check_rows(oracle, got, y_ref.cpu().numpy(), scale, f"call {call} vs pf_spmv_f64_i32")
        check_rows(oracle, got, serial, scale, f"call {call} vs spmv_serial")
    # nnz = 0: y = beta * y, finished when the call returns
    z_rp = torch.zeros(5, dtype=torch.int32, device="cuda")
    yz = torch.ones(4, dtype=torch.float64, device="cuda")
    st = pf.lib.pf_spmv_noalloc_f64_i32(4, 3, 0, z_rp.data_ptr(), None, None, 1.0, None, 3.0,
                                        yz.data_ptr(), C.c_void_p(stream))
    assert st == 0 and yz.tolist() == [3.0] * 4


def test_noalloc_device_error_then_clean_call(pf, oracle):
    """A row_ptr whose last entry does not match nnz makes the kernel flag
    its error word and return before reading anything else: the call reports
    PF_ERR_DEVICE (3) and leaves y alone. The next correct call, on the same
    built-in scratch, is right again."""
    import torch
    rp, col, val, n = case("mixed_long", seed=36)
    m, nnz = len(rp) - 1, len(col)
    x = np.random.default_rng(37).uniform(-1, 1, n)
    d_rp, d_col, d_val, d_x = (torch.from_numpy(a).cuda() for a in (rp.astype(np.int32), col, val, x))
    stream = torch.cuda.current_stream().cuda_stream
    y = torch.full((m,), 7.0, dtype=torch.float64, device="cuda")
    st = noalloc(pf, m, n, nnz - 1, d_rp, d_col, d_val, 1.0, d_x, 0.0, y, stream)
    assert st == 3, pf.lib.pf_last_error()
    assert b"device error" in pf.lib.pf_last_error()
    assert (y == 7.0).all().item()
    a, comp = oracle.abs_comp(rp, col, val, x)
    serial = oracle.serial(rp, col, val, x)
    st = noalloc(pf, m, n, nnz, d_rp, d_col, d_val, 1.0, d_x, 0.0, y, stream)
    assert st == 0, pf.lib.pf_last_error()
    ok, worst, nbad = oracle.tolerance_report(y.cpu().numpy(), serial, a, EPS, y_comp=comp)
    assert ok, f"{nbad} rows out of tolerance after the failed call (worst {worst:.3g})"
