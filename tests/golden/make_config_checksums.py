"""Checksums of the seeded benchmark configs 1-4 and of the REFERENCE's y.

Run in a container that has the reference tree (oracle/_ref/libref.so built by
`make -C oracle`): each config is generated at full size with the library's
seeded generator (seed 12345, the bench's), and the reference's own
spmv_serial (test/test_cdspmv.cpp:4-20) computes y = A*x. SHA-256 digests of
row_ptr, col, val, x and y are written to config_checksums.json next to this
script; tests/test_config_checksums.py pins the generator and the oracle's
restatement to them. Config 5 (2^31 non-zeros) is pinned on two slices of
2^16 rows (its head and rows from 2^25) over its full x. Config 3 is also checked with fp32 values and x (widened
to double for the reference's fp64 spmv_serial, which is how the fp32 oracle
works).

    python tests/golden/make_config_checksums.py
"""
import hashlib
import importlib
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "tests"))

import oracle  # noqa: E402
from csr_cases import gen_config_host  # noqa: E402

SEED = 12345
CASES = {"1": (1, np.float64), "2": (2, np.float64), "3": (3, np.float64),
         "3_f32": (3, np.float32), "4": (4, np.float64)}
# config 5 (2^31 non-zeros) as row slices over the full x: rows [r0, r0 + 2^16)
SLICES = {"5_head": (5, 0), "5_mid": (5, 1 << 25)}
SLICE_ROWS = 1 << 16


def sha(a: np.ndarray) -> str:
    """SHA-256 of an array's bytes (read in place, no copy)."""
    return hashlib.sha256(memoryview(np.ascontiguousarray(a)).cast("B")).hexdigest()


def main():
    assert oracle.ref_available(), "the reference build (oracle/_ref/libref.so) is needed"
    pf = importlib.import_module("prefree-public_b200")
    out = {"seed": SEED, "configs": {}}
    for name, (cfg, vdt) in CASES.items():
        spec = pf.GenSpec(cfg=cfg, seed=SEED)
        rp, col, val, x = gen_config_host(pf, spec)
        vq = val.astype(vdt, copy=False).astype(np.float64, copy=False)
        xq = x.astype(vdt, copy=False).astype(np.float64, copy=False)
        y = oracle.ref_serial(rp.astype(np.int32), col, vq, xq)
        out["configs"][name] = {
            "m": int(len(rp) - 1), "n": int(len(x)), "nnz": int(rp[-1]),
            "values": np.dtype(vdt).name,
            "sha256": {"row_ptr": sha(rp), "col": sha(col), "val": sha(vq), "x": sha(xq),
                       "y": sha(y)},
            "y_sum": float(y.sum()),
        }
        print(name, out["configs"][name]["nnz"], out["configs"][name]["y_sum"])
    out["slices"] = {}
    for name, (cfg, r0) in SLICES.items():
        spec = pf.GenSpec(cfg=cfg, seed=SEED)
        rp, col, val = pf.gen_rows_host(spec, r0, r0 + SLICE_ROWS)
        x = pf.gen_x_host(spec)
        y = oracle.ref_serial(rp.astype(np.int32), col, val, x)
        out["slices"][name] = {
            "r0": r0, "rows": SLICE_ROWS, "n": int(len(x)), "nnz": int(rp[-1]),
            "sha256": {"row_ptr": sha(rp), "col": sha(col), "val": sha(val), "x": sha(x),
                       "y": sha(y)},
            "y_sum": float(y.sum()),
        }
        print(name, out["slices"][name]["nnz"], out["slices"][name]["y_sum"])
    with open(os.path.join(HERE, "config_checksums.json"), "w") as f:
        json.dump(out, f, indent=1)


if __name__ == "__main__":
    main()
