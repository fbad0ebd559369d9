"""pf_spmv_noalloc_f64_i32, the multiply for callers that cannot allocate
device memory (an application that has reserved the GPU's memory for itself,
or code that must not call cudaMalloc mid-run because it can synchronize the
device and fail under memory pressure).

Checked through the C ABI against the regular entry point pf_spmv_f64_i32 on
the same inputs, within the fp64 tolerance used throughout the tests
(|y - y_ref| <= 1e-12 * sum_j |a_ij x_j| per row), on two calls in a row: the
second call reuses the built-in scratch the first one left behind. The test
buffers are allocated by torch, as the caller's own memory would be.
"""
import ctypes as C

import numpy as np
import pytest

from csr_cases import case

pytestmark = pytest.mark.gpu


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
    a, _ = oracle.abs_comp(rp, col, val, x)

    for call in range(2):
        y = torch.full((m,), float("nan"), dtype=torch.float64, device="cuda")
        st = pf.lib.pf_spmv_noalloc_f64_i32(m, n, nnz, d_rp.data_ptr(), d_col.data_ptr(),
                                            d_val.data_ptr(), 1.5, d_x.data_ptr(), 0.0,
                                            y.data_ptr(), C.c_void_p(stream))
        assert st == 0, pf.lib.pf_last_error()
        got = y.cpu().numpy()
        ok, worst, nbad = oracle.tolerance_report(got, ref, 1.5 * a, 1e-12)
        assert ok, f"call {call}: {nbad} rows out of tolerance (worst {worst:.3g})"


def test_noalloc_beta_and_empty_matrix(pf):
    import torch
    rp, col, val, n = case("powerlaw", seed=33)
    m, nnz = len(rp) - 1, len(col)
    x = np.random.default_rng(34).uniform(-1, 1, n)
    y0 = np.random.default_rng(35).uniform(-1, 1, m)
    args = [torch.from_numpy(a).cuda() for a in (rp.astype(np.int32), col, val, x)]
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    h = pf.Handle()
    y_ref = torch.from_numpy(y0.copy()).cuda()
    pf.spmv(h, m, n, nnz, *args, y_ref, 0.5, -2.0)
    torch.cuda.synchronize()
    h.close()
    y = torch.from_numpy(y0.copy()).cuda()
    st = pf.lib.pf_spmv_noalloc_f64_i32(m, n, nnz, args[0].data_ptr(), args[1].data_ptr(),
                                        args[2].data_ptr(), 0.5, args[3].data_ptr(), -2.0,
                                        y.data_ptr(), stream)
    assert st == 0, pf.lib.pf_last_error()
    d = (y - y_ref).abs().max().item()
    assert d <= 1e-12 * (y_ref.abs().max().item() + 1)
    # nnz = 0: y = beta * y
    z_rp = torch.zeros(5, dtype=torch.int32, device="cuda")
    yz = torch.ones(4, dtype=torch.float64, device="cuda")
    st = pf.lib.pf_spmv_noalloc_f64_i32(4, 3, 0, z_rp.data_ptr(), None, None, 1.0, None, 3.0,
                                        yz.data_ptr(), stream)
    torch.cuda.synchronize()
    assert st == 0 and yz.tolist() == [3.0] * 4
