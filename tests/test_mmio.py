"""pf_mmio_read (the library's Matrix Market reader) against the reference's
mmio_allinone (utilities/mmio.cpp:1547-1713): golden fixtures produced by the
reference build, plus the live reference when present."""
import os

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
MTX = os.path.join(HERE, "golden", "mtx")


def test_matches_reference_golden(pf):
    g = np.load(os.path.join(HERE, "golden", "mmio_golden.npz"))
    files = sorted({k.split("/")[0] for k in g.files})
    for fn in files:
        m, n, z, sym, rp, col, val = pf.mmio_read(os.path.join(MTX, fn))
        d = g[f"{fn}/dims"]
        assert (m, n, z, int(sym)) == tuple(int(v) for v in d), fn
        assert np.array_equal(rp, g[f"{fn}/row_ptr"].astype(np.int64)), fn
        assert np.array_equal(col, g[f"{fn}/col"]), fn
        assert np.array_equal(val, g[f"{fn}/val"]), fn


def write_random_mtx(path, rng, m, n, z, field="real", symmetry="general"):
    rows = rng.integers(1, m + 1, z)
    cols = rng.integers(1, n + 1, z)
    if symmetry == "symmetric":
        rows, cols = np.maximum(rows, cols), np.minimum(rows, cols)
    with open(path, "w") as f:
        f.write(f"%%MatrixMarket matrix coordinate {field} {symmetry}\n% generated\n{m} {n} {z}\n")
        for i, j in zip(rows, cols):
            if field == "pattern":
                f.write(f"{i} {j}\n")
            elif field == "integer":
                f.write(f"{i} {j} {int(rng.integers(-9, 10))}\n")
            else:
                f.write(f"{i} {j} {rng.normal():.17g}\n")


@pytest.mark.skipif(not os.path.exists(os.path.join(os.path.dirname(HERE), "oracle", "_ref",
                                                    "libref.so")),
                    reason="reference build absent")
@pytest.mark.parametrize("field,symmetry,size", [("real", "general", 20000),
                                                 ("real", "symmetric", 20000),
                                                 ("integer", "general", 3000),
                                                 ("pattern", "symmetric", 3000),
                                                 ("real", "general", 300000)])
def test_matches_live_reference(pf, oracle, tmp_path, field, symmetry, size):
    rng = np.random.default_rng(size)
    p = str(tmp_path / "a.mtx")
    write_random_mtx(p, rng, 500, 500, size, field, symmetry)   # 300k lines -> threaded parse
    ours = pf.mmio_read(p)
    ref = oracle.ref_mmio(p)
    assert ours[:4] == ref[:4]
    assert np.array_equal(ours[4], ref[4].astype(np.int64))
    assert np.array_equal(ours[5], ref[5])
    assert np.array_equal(ours[6], ref[6])


@pytest.mark.parametrize("text,status", [
    ("%%MatrixMarket matrix array real general\n2 2\n1\n2\n3\n4\n", 6),
    ("not a banner\n", 6),
    ("%%MatrixMarket matrix coordinate real general\n3 3 2\n1 1 1.0\n", 6),   # too few entries
    ("%%MatrixMarket matrix coordinate real general\n3 3 1\n4 1 1.0\n", 6),   # row out of range
    ("%%MatrixMarket matrix coordinate real symmetric\n3 2 1\n1 1 1.0\n", 6),  # symmetric, M != N
])
def test_rejects_bad_input(pf, tmp_path, text, status):
    p = tmp_path / "bad.mtx"
    p.write_text(text)
    with pytest.raises(pf.PfError) as e:
        pf.mmio_read(str(p))
    assert e.value.status == status
