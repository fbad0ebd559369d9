"""Generate the golden fixtures from the REFERENCE's own CPU code.

Run in a container that has the reference tree (oracle/_ref/libref.so built by
`make -C oracle`): the reference's spmv_serial (test/test_cdspmv.cpp:4-20)
computes y for a set of seeded CSR cases, and its mmio_allinone
(utilities/mmio.cpp:1547-1713) reads a set of Matrix Market files written
here. Inputs and outputs are saved as .npz next to this script; the tests pin
the C restatement in oracle/ and the library's own reader to them.

    python tests/golden/make_golden.py
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "tests"))

import oracle  # noqa: E402
from csr_cases import from_lengths  # noqa: E402


def spmv_cases():
    rng = np.random.default_rng(20241201)
    out = {}
    # hand-checked 3x3: [[1,0,2],[0,3,0],[4,0,5]] * [1,2,3] = [7, 6, 19]
    out["tiny3"] = (np.array([0, 2, 3, 5]), np.array([0, 2, 1, 0, 2]),
                    np.array([1., 2., 3., 4., 5.]), np.array([1., 2., 3.]))
    lens = np.concatenate([np.zeros(5), rng.integers(0, 12, 300), np.zeros(40),
                           [700], rng.integers(1, 5, 200), np.zeros(7)]).astype(np.int64)
    rp, col, val = from_lengths(rng, lens, 900)
    out["empty_rows_and_long_row"] = (rp, col, val, rng.uniform(-1, 1, 900))
    lens = np.full(400, 16)
    rp, col, _ = from_lengths(rng, lens, 400)
    val = (np.arange(len(col)) % 15).astype(np.float64)     # the harness's initVec
    out["mod15_uniform16"] = (rp, col, val, (np.arange(400) % 15).astype(np.float64))
    u = rng.random(2000)
    lens = np.minimum(np.rint(u ** (-1 / 1.1)), 1500).astype(np.int64)
    rp, col, val = from_lengths(rng, lens, 2500)
    out["powerlaw"] = (rp, col, val, rng.uniform(-1, 1, 2500))
    rp, col, val = from_lengths(rng, rng.integers(0, 30, 500), 700, sorted_cols=False)
    out["unsorted_cols"] = (rp, col, val, rng.normal(size=700))
    return out


MTX = {
    "general_real.mtx": "%%MatrixMarket matrix coordinate real general\n% comment\n4 5 6\n"
                        "1 1 1.5\n3 2 -2.25e-3\n1 5 7\n4 4 1e10\n2 3 0.5\n3 1 3.0\n",
    "symmetric_real.mtx": "%%MatrixMarket matrix coordinate real symmetric\n5 5 7\n"
                          "1 1 4\n2 1 -1\n3 2 -1\n4 1 2.5\n5 5 9\n5 3 -0.125\n3 3 8\n",
    "pattern_general.mtx": "%%MatrixMarket matrix coordinate pattern general\n3 3 4\n"
                           "1 2\n3 3\n2 1\n1 1\n",
    "integer_symmetric.mtx": "%%MatrixMarket matrix coordinate integer symmetric\n%c1\n%c2\n"
                             "4 4 5\n1 1 3\n2 1 -7\n4 2 11\n4 4 2\n3 1 5\n",
    "complex_general.mtx": "%%MatrixMarket matrix coordinate complex general\n2 3 3\n"
                           "1 1 1.5 2.0\n2 3 -4.0 0.5\n1 2 0.25 -1\n",
    "hermitian.mtx": "%%MatrixMarket matrix coordinate complex hermitian\n3 3 3\n"
                     "2 1 1.0 1.0\n3 3 2.0 0.0\n3 2 -1.0 3.0\n",
    "skew_symmetric.mtx": "%%MatrixMarket matrix coordinate real skew-symmetric\n3 3 2\n"
                          "2 1 1.5\n3 1 -2.0\n",
    "empty_rows.mtx": "%%MatrixMarket Matrix Coordinate Real General\n6 4 3\n"
                      "6 4 1.0\n2 1 2.0\n2 2 3.0\n",
}


def main():
    assert oracle.ref_available(), "needs oracle/_ref/libref.so (make -C oracle with the reference)"
    arrays = {}
    for name, (rp, col, val, x) in spmv_cases().items():
        rp32 = rp.astype(np.int32)
        y = oracle.ref_serial(rp32, col.astype(np.int32), val, x)
        arrays[f"{name}/row_ptr"] = rp32
        arrays[f"{name}/col"] = col.astype(np.int32)
        arrays[f"{name}/val"] = val
        arrays[f"{name}/x"] = x
        arrays[f"{name}/y"] = y
    np.savez_compressed(os.path.join(HERE, "spmv_serial_golden.npz"), **arrays)
    mdir = os.path.join(HERE, "mtx")
    os.makedirs(mdir, exist_ok=True)
    marr = {}
    for fname, text in MTX.items():
        p = os.path.join(mdir, fname)
        with open(p, "w") as f:
            f.write(text)
        m, n, z, sym, rp, col, val = oracle.ref_mmio(p)
        marr[f"{fname}/dims"] = np.array([m, n, z, int(sym)], dtype=np.int64)
        marr[f"{fname}/row_ptr"] = rp
        marr[f"{fname}/col"] = col
        marr[f"{fname}/val"] = val
    np.savez_compressed(os.path.join(HERE, "mmio_golden.npz"), **marr)
    print("wrote", len(arrays), "spmv arrays,", len(marr), "mmio arrays")


if __name__ == "__main__":
    main()
