"""The CPU oracle, pinned to the reference: the C restatement of spmv_serial
(test/test_cdspmv.cpp:4-20) must reproduce the golden outputs that the
reference's own compiled spmv_serial produced (tests/golden/make_golden.py),
bit for bit, and agree with the live reference build when it is present."""
import os

import numpy as np
import pytest

from csr_cases import CASES, case

HERE = os.path.dirname(os.path.abspath(__file__))
GOLD = os.path.join(HERE, "golden", "spmv_serial_golden.npz")


def golden_cases():
    g = np.load(GOLD)
    names = sorted({k.split("/")[0] for k in g.files})
    return g, names


def test_hand_checked_3x3(oracle):
    rp = np.array([0, 2, 3, 5], dtype=np.int32)
    col = np.array([0, 2, 1, 0, 2], dtype=np.int32)
    val = np.array([1., 2., 3., 4., 5.])
    y = oracle.serial(rp, col, val, np.array([1., 2., 3.]))
    assert y.tolist() == [7.0, 6.0, 19.0]


def test_restatement_matches_reference_golden(oracle):
    g, names = golden_cases()
    assert len(names) >= 5
    for nm in names:
        rp, col, val, x, y = (g[f"{nm}/{k}"] for k in ("row_ptr", "col", "val", "x", "y"))
        assert np.array_equal(oracle.serial(rp, col, val, x), y), nm
        # int64 offsets: same loop, same order -> same bits
        assert np.array_equal(oracle.serial(rp.astype(np.int64), col, val, x), y), nm


def test_y_accumulates_like_reference(oracle):
    """spmv_serial adds into Y (Y[i] = Y[i] + t); the harness passes zeros."""
    g, _ = golden_cases()
    rp, col, val, x, y = (g[f"powerlaw/{k}"] for k in ("row_ptr", "col", "val", "x", "y"))
    y0 = np.linspace(-1, 1, len(rp) - 1)
    got = oracle.serial(rp, col, val, x, y0=y0)
    assert np.array_equal(got, y0 + y)


@pytest.mark.skipif(not os.path.exists(os.path.join(os.path.dirname(HERE), "oracle", "_ref",
                                                    "libref.so")),
                    reason="reference build absent")
@pytest.mark.parametrize("name", CASES)
def test_restatement_matches_live_reference(oracle, name):
    rp, col, val, n = case(name, seed=11)
    x = np.random.default_rng(12).uniform(-1, 1, max(n, 1))
    a = oracle.serial(rp.astype(np.int32), col, val, x)
    b = oracle.ref_serial(rp.astype(np.int32), col, val, x)
    assert np.array_equal(a, b)


def test_fp32_inputs_widened(oracle):
    g, _ = golden_cases()
    rp, col, val, x = (g[f"powerlaw/{k}"] for k in ("row_ptr", "col", "val", "x"))
    y32 = oracle.serial(rp, col, val.astype(np.float32), x.astype(np.float32))
    ref = oracle.serial(rp, col, val.astype(np.float32).astype(np.float64),
                        x.astype(np.float32).astype(np.float64))
    assert np.array_equal(y32, ref)


def test_abs_sum_and_compensated_sum(oracle):
    rp = np.array([0, 3, 3, 5], dtype=np.int64)
    col = np.array([0, 1, 2, 0, 1], dtype=np.int32)
    val = np.array([1e16, 1.0, -1e16, 2.0, -3.0])
    x = np.ones(3)
    a, comp = oracle.abs_comp(rp, col, val, x)
    assert a.tolist() == [2e16 + 1.0, 0.0, 5.0]
    assert comp.tolist() == [1.0, 0.0, -1.0]          # exact, unlike the serial sum
    assert oracle.serial(rp, col, val, x)[0] == 0.0   # the serial sum loses the 1


def test_tolerance_report(oracle):
    y_ref = np.array([1.0, 2.0, 0.0])
    scale = np.array([1.0, 1.0, 0.0])
    ok, worst, nbad = oracle.tolerance_report(np.array([1.0 + 5e-13, 2.0, 0.0]), y_ref, scale, 1e-12)
    assert ok and nbad == 0 and worst == pytest.approx(0.5, rel=1e-3)
    ok, _, nbad = oracle.tolerance_report(np.array([1.0, 2.0, 1e-300]), y_ref, scale, 1e-12)
    assert not ok and nbad == 1                        # empty row must be exactly 0
    # a planted mistake in one row is caught
    ok, _, nbad = oracle.tolerance_report(np.array([1.0, 2.0 + 1e-9, 0.0]), y_ref, scale, 1e-12)
    assert not ok and nbad == 1


def read_coords(path):
    """Minimal independent parse of the golden .mtx files (test helper)."""
    with open(path) as f:
        lines = f.read().splitlines()
    banner = lines[0].lower().split()
    body = [l for l in lines[1:] if l.strip() and not l.lstrip().startswith("%")]
    m, n, z = map(int, body[0].split())
    ri, ci, vi = [], [], []
    for l in body[1:1 + z]:
        t = l.split()
        ri.append(int(t[0]) - 1)
        ci.append(int(t[1]) - 1)
        vi.append(1.0 if banner[3] == "pattern" else float(t[2]))
    sym = banner[4] in ("symmetric", "hermitian")
    return m, n, np.array(ri), np.array(ci), np.array(vi), sym


def test_coo_to_csr_restatement_matches_reference_golden(oracle):
    g = np.load(os.path.join(HERE, "golden", "mmio_golden.npz"))
    files = sorted({k.split("/")[0] for k in g.files})
    assert len(files) >= 6
    for fn in files:
        m, n, ri, ci, vi, sym = read_coords(os.path.join(HERE, "golden", "mtx", fn))
        rp, col, val = oracle.coo_to_csr(m, ri, ci, vi, sym)
        assert np.array_equal(rp, g[f"{fn}/row_ptr"]), fn
        assert np.array_equal(col, g[f"{fn}/col"]), fn
        assert np.array_equal(val, g[f"{fn}/val"]), fn
