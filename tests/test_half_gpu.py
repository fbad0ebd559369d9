"""16-bit values (pf_spmv_f16_* / pf_spmv_bf16_*): binary16 and bfloat16 val,
x and y, products and sums in double, y rounded once. The reference's intended
second value type (valT = half, include/common.h:43-46), whose build does not
compile (src/spmv_kernel/preFreeSpMV.cu:326), so the oracle is its serial loop
(test/test_cdspmv.cpp:4-20) on the 16-bit inputs widened exactly to double.

Tolerance per row: |y - y_ref| <= 2^-p * |y_ref| + 1e-12 * sum_j |a_ij x_j| +
t_min, the rounding of the one 16-bit output (p = 10 for binary16, 7 for
bfloat16: one unit in the last place) over the double sums' order effects;
t_min is binary16's smallest subnormal (0 for bfloat16)."""
import numpy as np
import pytest

from csr_cases import case

pytestmark = pytest.mark.gpu

VARIANTS = {"auto": 0, "nnzsplit": 1, "rowgroup": 2, "rowvec": 4, "nnzrow": 7}


def run_half(pf, torch, h, rp, col, val, x, n, tdt, idt, alpha=1.0, beta=0.0, y0=None):
    m = len(rp) - 1
    d_rp = torch.from_numpy(rp.astype(idt)).cuda()
    d_col = torch.from_numpy(col.astype(np.int32)).cuda() if len(col) else \
        torch.zeros(1, dtype=torch.int32, device="cuda")
    d_val = torch.from_numpy(val).to(tdt).cuda() if len(val) else torch.zeros(1, dtype=tdt, device="cuda")
    d_x = torch.from_numpy(x).to(tdt).cuda()
    d_y = torch.full((max(m, 1),), float("nan"), dtype=tdt, device="cuda") if y0 is None \
        else torch.from_numpy(y0).to(tdt).cuda()
    pf.spmv(h, m, n, len(col), d_rp, d_col, d_val, d_x, d_y, alpha, beta)
    torch.cuda.synchronize()
    assert h.device_error() == 0
    return (d_y[:m].double().cpu().numpy(), d_val.double().cpu().numpy()[:len(val)],
            d_x.double().cpu().numpy())


def check(oracle, y, rp, col, v64, x64, p, tmin, alpha=1.0, beta=0.0, y0=None):
    s = oracle.serial(rp, col, v64, x64)
    a, _ = oracle.abs_comp(rp, col, v64, x64)
    yb = np.zeros(len(rp) - 1) if y0 is None else y0
    ref = alpha * s + beta * yb
    tol = 2.0 ** -p * np.abs(ref) + 1e-12 * (abs(alpha) * a + abs(beta) * np.abs(yb)) + tmin
    bad = ~(np.abs(y - ref) <= tol)
    assert not bad.any(), f"{int(bad.sum())} rows out of tolerance"


@pytest.mark.parametrize("fmt", ["f16", "bf16"])
@pytest.mark.parametrize("variant", list(VARIANTS))
@pytest.mark.parametrize("name", ["tiny", "powerlaw", "mixed_long", "row0_long", "empty_edges",
                                  "uniform16", "long_rows"])
def test_half_cases_variants(pf, oracle, fmt, variant, name):
    import torch
    tdt = torch.float16 if fmt == "f16" else torch.bfloat16
    p, tmin = (10, 2.0 ** -24) if fmt == "f16" else (7, 0.0)
    rp, col, val, n = case(name, seed=61)
    x = np.random.default_rng(62).uniform(-1, 1, n)
    h = pf.Handle()
    h.set_variant(VARIANTS[variant])
    y, v64, x64 = run_half(pf, torch, h, rp, col, val, x, n, tdt, np.int32)
    h.close()
    check(oracle, y, rp, col, v64, x64, p, tmin)


@pytest.mark.parametrize("fmt", ["f16", "bf16"])
@pytest.mark.parametrize("idt", [np.int32, np.int64])
def test_half_alpha_beta_int64(pf, oracle, fmt, idt):
    import torch
    tdt = torch.float16 if fmt == "f16" else torch.bfloat16
    p, tmin = (10, 2.0 ** -24) if fmt == "f16" else (7, 0.0)
    rp, col, val, n = case("mixed_long", seed=63)
    rng = np.random.default_rng(64)
    x = rng.uniform(-1, 1, n)
    y0 = torch.from_numpy(rng.uniform(-1, 1, len(rp) - 1)).to(tdt).double().numpy()
    h = pf.Handle()
    y, v64, x64 = run_half(pf, torch, h, rp, col, val, x, n, tdt, idt, alpha=0.75, beta=-1.25, y0=y0)
    h.close()
    check(oracle, y, rp, col, v64, x64, p, tmin, alpha=0.75, beta=-1.25, y0=y0)


@pytest.mark.parametrize("fmt", ["f16", "bf16"])
@pytest.mark.parametrize("name", ["powerlaw", "mixed_long", "row0_long", "empty_edges"])
@pytest.mark.parametrize("slice_nnz", [1, 63, 319, 320, 640, 1000])
def test_half_nnzrow_cut_rows(pf, oracle, fmt, name, slice_nnz):
    """NNZROW walks 320-element tiles with 16-bit values: slices shorter and
    longer than a tile, ending on and off tile boundaries, cut every kind of
    row."""
    import torch
    tdt = torch.float16 if fmt == "f16" else torch.bfloat16
    p, tmin = (10, 2.0 ** -24) if fmt == "f16" else (7, 0.0)
    rp, col, val, n = case(name, seed=65)
    x = np.random.default_rng(66).uniform(-1, 1, n)
    h = pf.Handle()
    h.set_variant(VARIANTS["nnzrow"])
    h.set_slice(slice_nnz)
    y, v64, x64 = run_half(pf, torch, h, rp, col, val, x, n, tdt, np.int64)
    h.close()
    check(oracle, y, rp, col, v64, x64, p, tmin)
