"""The seeded benchmark configs 1-4 and their y, pinned to checksums made by
the reference's own spmv_serial (tests/golden/make_config_checksums.py).

Each config is regenerated at full size with the library's host generator;
SHA-256 digests of row_ptr, col, val and x pin the generator, and the digest
of y = A*x computed by the oracle's restatement of spmv_serial
(test/test_cdspmv.cpp:4-20) must equal the one the reference computed: the
same bits, not just within tolerance. Config 3 is also pinned with fp32
values and x; config 5 (2^31 non-zeros, int64 row_ptr) on two row slices
over its full x.
"""
import hashlib
import json
import os

import numpy as np
import pytest

from csr_cases import gen_config_host

HERE = os.path.dirname(os.path.abspath(__file__))
GOLD = json.load(open(os.path.join(HERE, "golden", "config_checksums.json")))
DTYPES = {"float64": np.float64, "float32": np.float32}


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(memoryview(np.ascontiguousarray(a)).cast("B")).hexdigest()


@pytest.mark.parametrize("name", sorted(GOLD["configs"]))
def test_config_and_reference_y_checksums(pf, oracle, name):
    g = GOLD["configs"][name]
    cfg = int(name.split("_")[0])
    vdt = DTYPES[g["values"]]
    rp, col, val, x = gen_config_host(pf, pf.GenSpec(cfg=cfg, seed=GOLD["seed"]))
    assert (len(rp) - 1, len(x), int(rp[-1])) == (g["m"], g["n"], g["nnz"])
    vq = val.astype(vdt, copy=False).astype(np.float64, copy=False)
    xq = x.astype(vdt, copy=False).astype(np.float64, copy=False)
    got = {"row_ptr": sha(rp), "col": sha(col), "val": sha(vq), "x": sha(xq)}
    for k, v in got.items():
        assert v == g["sha256"][k], f"{name}: generated {k} changed"
    y = oracle.serial(rp, col, vq, xq)
    assert sha(y) == g["sha256"]["y"], f"{name}: y differs from the reference's"


@pytest.mark.parametrize("name", sorted(GOLD.get("slices", {})))
def test_config5_slices_and_reference_y(pf, oracle, name):
    g = GOLD["slices"][name]
    spec = pf.GenSpec(cfg=5, seed=GOLD["seed"])
    rp, col, val = pf.gen_rows_host(spec, g["r0"], g["r0"] + g["rows"])
    x = pf.gen_x_host(spec)
    assert (len(x), int(rp[-1])) == (g["n"], g["nnz"])
    got = {"row_ptr": sha(rp), "col": sha(col), "val": sha(val), "x": sha(x)}
    for k, v in got.items():
        assert v == g["sha256"][k], f"{name}: generated {k} changed"
    y = oracle.serial(rp, col, val, x)
    assert sha(y) == g["sha256"]["y"], f"{name}: y differs from the reference's"
