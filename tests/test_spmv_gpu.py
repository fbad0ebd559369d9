"""GPU parity of the CSR SpMV kernels against the CPU oracle, through the C ABI.

Tolerance (north star): per row |y - y_ref| <= eps * sum_j |a_ij x_j| with
eps = 1e-12 for fp64 and 1e-5 for fp32 (y_ref = the restated spmv_serial of
test/test_cdspmv.cpp:4-20, accumulated in double). With the reference
harness's integer values (i % 15, include/common.h:126-133) every partial sum
is an exact integer, so fp64 results must be bit-identical.
"""
import numpy as np
import pytest

from csr_cases import CASES, case, from_lengths

pytestmark = pytest.mark.gpu

EPS = {np.float64: 1e-12, np.float32: 1e-5}


@pytest.fixture(scope="module")
def torch_cuda():
    import torch
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    return torch


@pytest.fixture(scope="module")
def handle(pf, torch_cuda):
    h = pf.Handle()
    yield h
    h.close()


def to_dev(torch, a, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a))
    if dtype is not None:
        t = t.to(dtype)
    return t.cuda()


def run_gpu(pf, torch, h, rp, col, val, x, n, vdt, idt, alpha=1.0, beta=0.0, y0=None):
    m = len(rp) - 1
    tv = {np.float64: torch.float64, np.float32: torch.float32}[vdt]
    ti = {np.int32: torch.int32, np.int64: torch.int64}[idt]
    d_rp = to_dev(torch, rp.astype(idt))
    d_col = to_dev(torch, col.astype(np.int32)) if len(col) else torch.zeros(1, dtype=torch.int32, device="cuda")
    d_val = to_dev(torch, val.astype(vdt)) if len(val) else torch.zeros(1, dtype=tv, device="cuda")
    d_x = to_dev(torch, x.astype(vdt)) if len(x) else torch.zeros(1, dtype=tv, device="cuda")
    if y0 is None:
        d_y = torch.full((max(m, 1),), float("nan"), dtype=tv, device="cuda")
    else:
        d_y = to_dev(torch, y0.astype(vdt))
    nnz = int(rp[-1]) - int(rp[0])
    pf.spmv(h, m, n, nnz, d_rp, d_col, d_val, d_x, d_y, alpha, beta)
    torch.cuda.synchronize()
    assert h.device_error() == 0
    assert d_rp.dtype == ti
    return d_y[:m].cpu().numpy().astype(np.float64)


def check(oracle, y, rp, col, val, x, vdt, alpha=1.0, beta=0.0, y0=None):
    vq = val.astype(vdt)
    xq = x.astype(vdt)
    s = oracle.serial(rp, col, vq, xq)
    a, comp = oracle.abs_comp(rp, col, vq, xq)
    m = len(rp) - 1
    yb = np.zeros(m) if y0 is None else y0.astype(vdt).astype(np.float64)
    ref = alpha * s + beta * yb
    scale = abs(alpha) * a + abs(beta) * np.abs(yb)
    ok, worst, nbad = oracle.tolerance_report(y, ref, scale, EPS[vdt],
                                              y_comp=alpha * comp + beta * yb)
    assert ok, f"{nbad} rows out of tolerance (worst ratio {worst:.3g})"


VARIANTS = {"auto": 0, "nnzsplit": 1, "rowgroup": 2, "rowvec": 4, "nnzrow": 7}


@pytest.fixture
def variant_handle(handle, request):
    handle.set_variant(VARIANTS[request.param])
    yield handle
    handle.set_variant(0)
    handle.set_slice(0)


@pytest.mark.parametrize("variant_handle", list(VARIANTS), indirect=True)
@pytest.mark.parametrize("name", CASES)
@pytest.mark.parametrize("vdt", [np.float64, np.float32])
@pytest.mark.parametrize("idt", [np.int32, np.int64])
def test_cases_variants(pf, oracle, torch_cuda, variant_handle, name, vdt, idt):
    rp, col, val, n = case(name, seed=1)
    x = np.random.default_rng(2).uniform(-1, 1, n)
    y = run_gpu(pf, torch_cuda, variant_handle, rp, col, val, x, n, vdt, idt)
    check(oracle, y, rp, col, val, x, vdt)


@pytest.mark.parametrize("variant_handle", ["nnzsplit", "nnzrow"],
                         indirect=True)
@pytest.mark.parametrize("name", ["tiny", "row0_long", "empty_edges", "powerlaw", "mixed_long"])
@pytest.mark.parametrize("slice_nnz", [1, 3, 7, 64, 1000, 5000])
@pytest.mark.parametrize("idt", [np.int32, np.int64])
def test_small_slices_force_cut_rows(pf, oracle, torch_cuda, variant_handle, name, slice_nnz, idt):
    rp, col, val, n = case(name, seed=3)
    x = np.random.default_rng(4).uniform(-1, 1, n)
    variant_handle.set_slice(slice_nnz)
    y = run_gpu(pf, torch_cuda, variant_handle, rp, col, val, x, n, np.float64, idt)
    check(oracle, y, rp, col, val, x, np.float64)


@pytest.mark.parametrize("variant_handle", ["nnzsplit", "rowgroup", "rowvec", "nnzrow"],
                         indirect=True)
@pytest.mark.parametrize("offset", [1, 2, 3, 5])
def test_unaligned_array_starts(pf, oracle, torch_cuda, variant_handle, offset):
    """val/col/row_ptr that do not start on a 16-byte boundary (views into
    larger buffers): the bulk copies must round to 16-byte blocks correctly."""
    torch = torch_cuda
    rp, col, val, n = case("powerlaw", seed=21)
    x = np.random.default_rng(22).uniform(-1, 1, n)
    big_col = torch.zeros(len(col) + 8, dtype=torch.int32, device="cuda")
    big_val = torch.zeros(len(val) + 8, dtype=torch.float64, device="cuda")
    big_rp = torch.zeros(len(rp) + 8, dtype=torch.int32, device="cuda")
    d_col = big_col[offset:offset + len(col)]
    d_val = big_val[offset:offset + len(val)]
    d_rp = big_rp[offset:offset + len(rp)]
    d_col.copy_(torch.from_numpy(col))
    d_val.copy_(torch.from_numpy(val))
    d_rp.copy_(torch.from_numpy(rp.astype(np.int32)))
    d_y = torch.zeros(len(rp) - 1, dtype=torch.float64, device="cuda")
    variant_handle.set_slice(997)
    pf.spmv(variant_handle, len(rp) - 1, n, len(col), d_rp, d_col, d_val, to_dev(torch, x), d_y)
    torch.cuda.synchronize()
    assert variant_handle.device_error() == 0
    check(oracle, d_y.cpu().numpy(), rp, col, val, x, np.float64)


@pytest.mark.parametrize("alpha,beta", [(2.5, 0.0), (1.0, 1.0), (-0.75, 0.5), (0.0, 2.0)])
@pytest.mark.parametrize("vdt", [np.float64, np.float32])
@pytest.mark.parametrize("name", ["mixed_long", "long_rows"])
def test_alpha_beta(pf, oracle, torch_cuda, handle, alpha, beta, vdt, name):
    rp, col, val, n = case(name, seed=5)
    rng = np.random.default_rng(6)
    x = rng.uniform(-1, 1, n)
    y0 = rng.uniform(-1, 1, len(rp) - 1)
    y = run_gpu(pf, torch_cuda, handle, rp, col, val, x, n, vdt, np.int64, alpha, beta, y0)
    check(oracle, y, rp, col, val, x, vdt, alpha, beta, y0)


@pytest.mark.parametrize("name", ["powerlaw", "mixed_long", "row0_long", "long_rows"])
@pytest.mark.parametrize("slice_nnz", [0, 5, 300])
def test_integer_values_bit_exact(pf, oracle, torch_cuda, handle, name, slice_nnz):
    rp, col, _, n = case(name, seed=7)
    val = (np.arange(len(col)) % 15).astype(np.float64)
    x = (np.arange(n) % 15).astype(np.float64)
    handle.set_slice(slice_nnz)
    try:
        y = run_gpu(pf, torch_cuda, handle, rp, col, val, x, n, np.float64, np.int32)
    finally:
        handle.set_slice(0)
    ref = oracle.serial(rp, col, val, x)
    assert np.array_equal(y, ref)


def test_deterministic(pf, torch_cuda, handle):
    rp, col, val, n = case("powerlaw", seed=8)
    x = np.random.default_rng(9).uniform(-1, 1, n)
    y1 = run_gpu(pf, torch_cuda, handle, rp, col, val, x, n, np.float64, np.int32)
    y2 = run_gpu(pf, torch_cuda, handle, rp, col, val, x, n, np.float64, np.int32)
    assert np.array_equal(y1, y2)


def test_row_slice_view(pf, oracle, torch_cuda, handle):
    """row_ptr[0] != 0: a row slice addressed with absolute offsets."""
    torch = torch_cuda
    rp, col, val, n = case("powerlaw", seed=10)
    x = np.random.default_rng(11).uniform(-1, 1, n)
    r0, r1 = 1234, 15678
    d_rp = to_dev(torch, rp.astype(np.int64))
    d_col, d_val, d_x = to_dev(torch, col), to_dev(torch, val), to_dev(torch, x)
    d_y = torch.zeros(r1 - r0, dtype=torch.float64, device="cuda")
    nnz = int(rp[r1] - rp[r0])
    pf.spmv(handle, r1 - r0, n, nnz, d_rp[r0:], d_col, d_val, d_x, d_y)
    torch.cuda.synchronize()
    full = oracle.serial(rp, col, val, x)
    a, _ = oracle.abs_comp(rp, col, val, x)
    y = d_y.cpu().numpy()
    ok, worst, _ = oracle.tolerance_report(y, full[r0:r1], a[r0:r1], 1e-12)
    assert ok, worst


def test_host_buffer_call(pf, oracle, torch_cuda, handle):
    rp, col, val, n = case("mixed_long", seed=12)
    x = np.random.default_rng(13).uniform(-1, 1, n)
    y = np.zeros(len(rp) - 1)
    pf.spmv_host(handle, rp, col, val, x, y)
    check(oracle, y, rp, col, val, x, np.float64)
    # a row slice of the host CSR (absolute offsets)
    r0, r1 = 100, 5000
    ys = np.zeros(r1 - r0)
    pf.spmv_host(handle, rp[r0:r1 + 1], col, val, x, ys, m=r1 - r0, n=n)
    full = oracle.serial(rp, col, val, x)
    a, _ = oracle.abs_comp(rp, col, val, x)
    ok, worst, _ = oracle.tolerance_report(ys, full[r0:r1], a[r0:r1], 1e-12)
    assert ok, worst


@pytest.mark.parametrize("name", ["mixed_long", "powerlaw", "empty_edges", "row0_long",
                                  "empty_matrix"])
@pytest.mark.parametrize("vdt", [np.float64, np.float32])
@pytest.mark.parametrize("idt", [np.int32, np.int64])
def test_host_buffer_pipelined_chunks(pf, oracle, torch_cuda, handle, monkeypatch, name, vdt, idt):
    """The host-buffer call copies col/val in row chunks of about equal nnz and
    multiplies each chunk as it arrives. 4 KB chunks (16 at most) put chunk
    boundaries among empty and long rows; beta != 0, and a row slice of the
    host CSR whose first offset is not 0."""
    monkeypatch.setenv("PF_HOST_CHUNK_BYTES", "4096")
    rp, col, val, n = case(name, seed=31)
    rp = rp.astype(idt)
    rng = np.random.default_rng(32)
    x = rng.uniform(-1, 1, n).astype(vdt)
    val = val.astype(vdt)
    m = len(rp) - 1
    y0 = rng.uniform(-1, 1, m).astype(vdt)
    y = y0.copy()
    pf.spmv_host(handle, rp, col, val, x, y, alpha=0.75, beta=-0.5)
    check(oracle, y.astype(np.float64), rp, col, val, x, vdt, alpha=0.75, beta=-0.5, y0=y0)
    if m > 10:
        r0, r1 = m // 7, m - m // 5
        ys = np.zeros(r1 - r0, dtype=vdt)
        pf.spmv_host(handle, rp[r0:r1 + 1], col, val, x, ys, m=r1 - r0, n=n)
        full = oracle.serial(rp, col, val, x)
        a, _ = oracle.abs_comp(rp, col, val, x)
        ok, worst, _ = oracle.tolerance_report(ys.astype(np.float64), full[r0:r1], a[r0:r1],
                                               EPS[vdt])
        assert ok, worst


def test_prefree_entry_point(pf, oracle, torch_cuda, monkeypatch):
    """The reference's call shape: host arrays, int32 offsets, Y overwritten,
    timing outputs in ms (include/PreFree.h:3-5, preFreeSpMV.cu:563-662)."""
    monkeypatch.setenv("PF_PREFREE_WARMUP", "3")
    monkeypatch.setenv("PF_PREFREE_ITERS", "20")
    rp, col, _, n = case("row0_long", seed=14)
    val = (np.arange(len(col)) % 15).astype(np.float64)   # the harness's initVec
    x = (np.arange(n) % 15).astype(np.float64)
    m = len(rp) - 1
    y = np.full(m, 123.0)                                 # incoming Y is ignored
    rp32 = rp.astype(np.int32)
    t, p = pf.preFreeSpMV(val, rp32, col, x, y, m, n, len(col))
    assert t > 0 and p >= 0
    assert np.array_equal(y, oracle.serial(rp32, col, val, x))
    # fp32 and int64 overloads
    y32 = np.zeros(m, dtype=np.float32)
    pf.preFreeSpMV(val.astype(np.float32), rp32, col, x.astype(np.float32), y32, m, n, len(col))
    check(oracle, y32.astype(np.float64), rp, col, val, x, np.float32)
    y64 = np.zeros(m)
    pf.preFreeSpMV(val, rp.astype(np.int64), col, x, y64, m, n, len(col))
    assert np.array_equal(y64, y)


def test_bad_column_index_reported(pf, torch_cuda, handle):
    """An out-of-range column is skipped and flagged in the error word (no fault)."""
    torch = torch_cuda
    rp = np.array([0, 2, 3], dtype=np.int32)
    col = np.array([0, 7, 1], dtype=np.int32)      # 7 >= n
    val = np.ones(3)
    x = np.ones(2)
    d_y = torch.zeros(2, dtype=torch.float64, device="cuda")
    pf.spmv(handle, 2, 2, 3, to_dev(torch, rp), to_dev(torch, col), to_dev(torch, val),
            to_dev(torch, x), d_y)
    bits = handle.device_error(clear=True)
    assert bits & 2
    assert handle.device_error() == 0


def test_selector_choice(pf, torch_cuda):
    """The variant query reports what the selector runs: ROWVEC for regular
    rows (two lanes up to 16 non-zeros per row), NNZROW for power-law rows,
    for every value size."""
    torch = torch_cuda
    rng = np.random.default_rng(51)
    regular = from_lengths(rng, np.full(20000, 16), 20000)[0]
    skewed = np.zeros(20001, dtype=np.int64)
    np.cumsum(np.minimum(np.rint(rng.random(20000) ** (-1 / 1.1)), 5000).astype(np.int64),
              out=skewed[1:])
    h = pf.Handle()
    for rp, want in ((regular, ("rowvec", 2)), (skewed, ("nnzrow", 0))):
        d_rp = torch.from_numpy(rp.astype(np.int32)).cuda()
        for vb in (8, 4, 2):
            assert h.choice(len(rp) - 1, int(rp[-1]), d_rp, vb) == want
    h.set_variant(2)
    assert h.choice(len(regular) - 1, int(regular[-1]),
                    torch.from_numpy(regular).cuda(), 8)[0] == "rowgroup"
    h.close()
