"""SpMM (pf_spmm_*): Y = alpha*A*X + beta*Y for k dense columns, through the C
ABI, against the CPU oracle column by column (the reference's serial loop,
test/test_cdspmv.cpp:4-20, on column j of X), with the per-row tolerance used
throughout (|y - y_ref| <= eps * sum_j |a_ij x_j|, eps 1e-12 fp64 / 1e-5 fp32)
and bit-exact on the harness's integer values (i % 15)."""
import numpy as np
import pytest

from csr_cases import case

pytestmark = pytest.mark.gpu

EPS = {np.float64: 1e-12, np.float32: 1e-5}


def run_spmm(pf, torch, rp, col, val, X, k, vdt, idt, alpha=1.0, beta=0.0, Y0=None, ldx=None,
             ldy=None, offset=0):
    tv = {np.float64: torch.float64, np.float32: torch.float32}[vdt]
    m, n = len(rp) - 1, X.shape[0]
    d_rp = torch.from_numpy(rp.astype(idt)).cuda()
    # col/val as views `offset` elements into larger buffers (unaligned starts)
    big_col = torch.zeros(len(col) + 8, dtype=torch.int32, device="cuda")
    big_val = torch.zeros(len(val) + 8, dtype=tv, device="cuda")
    d_col = big_col[offset:offset + len(col)]
    d_val = big_val[offset:offset + len(val)]
    if len(col):
        d_col.copy_(torch.from_numpy(col.astype(np.int32)))
        d_val.copy_(torch.from_numpy(val.astype(vdt)))
    ldx = ldx or k
    ldy = ldy or k
    Xb = torch.zeros(max(n, 1), ldx, dtype=tv, device="cuda")
    Xb[:n, :k] = torch.from_numpy(X.astype(vdt))
    Yb = torch.full((max(m, 1), ldy), float("nan"), dtype=tv, device="cuda")
    if Y0 is not None:
        Yb[:m, :k] = torch.from_numpy(Y0.astype(vdt))
    h = pf.Handle()
    pf.spmm(h, m, n, len(col), d_rp, d_col, d_val, Xb[:, :k], Yb[:, :k], alpha, beta)
    torch.cuda.synchronize()
    assert h.device_error() == 0
    h.close()
    return Yb[:m, :k].cpu().numpy().astype(np.float64)


def check(oracle, Y, rp, col, val, X, vdt, alpha=1.0, beta=0.0, Y0=None):
    vq = val.astype(vdt)
    for j in range(X.shape[1]):
        xq = X[:, j].astype(vdt)
        s = oracle.serial(rp, col, vq, xq)
        a, comp = oracle.abs_comp(rp, col, vq, xq)
        y0 = np.zeros(len(rp) - 1) if Y0 is None else Y0[:, j].astype(vdt).astype(np.float64)
        ref = alpha * s + beta * y0
        scale = abs(alpha) * a + abs(beta) * np.abs(y0)
        ok, worst, nbad = oracle.tolerance_report(Y[:, j], ref, scale, EPS[vdt],
                                                  y_comp=alpha * comp + beta * y0)
        assert ok, f"column {j}: {nbad} rows out of tolerance (worst {worst:.3g})"


@pytest.mark.parametrize("name", ["tiny", "powerlaw", "mixed_long", "empty_edges", "uniform16",
                                  "row0_long", "unsorted"])
@pytest.mark.parametrize("k", [1, 3, 8, 11])
def test_spmm_cases(pf, oracle, name, k):
    import torch
    rp, col, val, n = case(name, seed=51)
    X = np.random.default_rng(52 + k).uniform(-1, 1, (n, k))
    Y = run_spmm(pf, torch, rp, col, val, X, k, np.float64, np.int32)
    check(oracle, Y, rp, col, val, X, np.float64)


@pytest.mark.parametrize("vdt", [np.float64, np.float32])
@pytest.mark.parametrize("idt", [np.int32, np.int64])
@pytest.mark.parametrize("offset", [0, 1, 3])
def test_spmm_types_strides_alpha_beta(pf, oracle, vdt, idt, offset):
    import torch
    rp, col, val, n = case("mixed_long", seed=53)
    k = 5
    rng = np.random.default_rng(54)
    X = rng.uniform(-1, 1, (n, k))
    Y0 = rng.uniform(-1, 1, (len(rp) - 1, k))
    Y = run_spmm(pf, torch, rp, col, val, X, k, vdt, idt, alpha=-0.5, beta=1.5, Y0=Y0,
                 ldx=7, ldy=9, offset=offset)
    check(oracle, Y, rp, col, val, X, vdt, alpha=-0.5, beta=1.5, Y0=Y0)


def test_spmm_mod15_bit_exact_and_spmv_agree(pf, oracle):
    """Integer values: every column equals the serial loop bit for bit, and
    column j equals the SpMV of column j."""
    import torch
    rp, col, _, n = case("powerlaw", seed=55)
    val = (np.arange(len(col)) % 15).astype(np.float64)
    k = 8
    X = (np.arange(n * k).reshape(n, k) % 15).astype(np.float64)
    Y = run_spmm(pf, torch, rp, col, val, X, k, np.float64, np.int32)
    for j in range(k):
        assert np.array_equal(Y[:, j], oracle.serial(rp, col, val, X[:, j]))


def test_spmm_empty_matrix_scales_y(pf):
    import torch
    rp = np.zeros(6, dtype=np.int32)
    Y0 = np.arange(15, dtype=np.float64).reshape(5, 3)
    Y = run_spmm(pf, torch, rp, np.zeros(0, np.int32), np.zeros(0), np.zeros((4, 3)), 3,
                 np.float64, np.int32, beta=2.0, Y0=Y0)
    assert np.array_equal(Y, 2.0 * Y0)


@pytest.mark.parametrize("vdt,k,ldx", [(np.float64, 11, 12), (np.float64, 8, 8),
                                       (np.float32, 6, 8), (np.float32, 13, 16)])
def test_spmm_vector_x_rows(pf, oracle, vdt, k, ldx):
    """X rows on 16-byte boundaries (16-byte X loads), with a last pass whose
    columns end inside a 16-byte piece."""
    import torch
    rp, col, val, n = case("powerlaw", seed=56)
    X = np.random.default_rng(57).uniform(-1, 1, (n, k))
    Y = run_spmm(pf, torch, rp, col, val, X, k, vdt, np.int32, ldx=ldx)
    check(oracle, Y, rp, col, val, X, vdt)
