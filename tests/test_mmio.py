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


REF_PRESENT = os.path.exists(os.path.join(os.path.dirname(HERE), "oracle", "_ref", "libref.so"))


@pytest.mark.skipif(not REF_PRESENT, reason="reference build absent")
@pytest.mark.parametrize("symmetry", ["general", "symmetric"])
def test_parallel_csr_build_matches_live_reference(pf, oracle, tmp_path, symmetry):
    """More than 2^20 entries: the CSR is built by several threads, each owning
    a range of rows. Many repeated coordinates (a 700 x 700 matrix), so the
    order of entries inside a row (file order, mirrors right after their
    entry) decides the result."""
    rng = np.random.default_rng(5)
    z = (1 << 20) + 12345
    rows = rng.integers(1, 701, z)
    cols = rng.integers(1, 701, z)
    if symmetry == "symmetric":
        rows, cols = np.maximum(rows, cols), np.minimum(rows, cols)
    vals = rng.standard_normal(z)
    p = str(tmp_path / "big.mtx")
    with open(p, "w") as f:
        f.write(f"%%MatrixMarket matrix coordinate real {symmetry}\n700 700 {z}\n")
        f.write("".join(f"{i} {j} {v:.17g}\n" for i, j, v in
                        zip(rows.tolist(), cols.tolist(), vals.tolist())))
    ours = pf.mmio_read(p)
    ref = oracle.ref_mmio(p)
    assert ours[:4] == ref[:4]
    assert np.array_equal(ours[4], ref[4].astype(np.int64))
    assert np.array_equal(ours[5], ref[5])
    assert np.array_equal(ours[6].view(np.uint64), ref[6].view(np.uint64))


@pytest.mark.skipif(not REF_PRESENT, reason="reference build absent")
def test_value_tokens_match_live_reference(pf, oracle, tmp_path):
    """Value spellings that take the strtod path (a leading '+', hex, out of
    range, inf/nan, subnormals) and ones that do not: the same bits as the
    reference's fscanf %lg."""
    toks = ["1.5", "+2.25", "-0.0", "1e400", "-1e400", "4.9e-324", "2.2250738585072011e-308",
            "0x1.8p1", "nan", "-inf", "INF", "1.0E+05", "0.1", "123456789012345678901234567890",
            "-7", "3.", ".5e-3", "1e-400"]
    lines = [f"{k + 1}\t {k % 3 + 1}   {t}  " for k, t in enumerate(toks)]
    lines.append(f"+{len(toks) + 1} +2 6.25")
    p = tmp_path / "tokens.mtx"
    p.write_text(f"%%MatrixMarket matrix coordinate real general\n{len(lines)} 3 {len(lines)}\n"
                 + "\n".join(lines) + "\n")
    ours = pf.mmio_read(str(p))
    ref = oracle.ref_mmio(str(p))
    assert ours[:4] == ref[:4]
    assert np.array_equal(ours[4], ref[4].astype(np.int64))
    assert np.array_equal(ours[5], ref[5])
    assert np.array_equal(ours[6].view(np.uint64), ref[6].view(np.uint64))


@pytest.mark.skipif(not REF_PRESENT, reason="reference build absent")
def test_crlf_and_blank_lines_match_live_reference(pf, oracle, tmp_path):
    """Windows line endings and blank lines between entries (fscanf skips
    both): the same CSR as the reference, bit for bit."""
    rng = np.random.default_rng(3)
    lines = ["%%MatrixMarket matrix coordinate real symmetric", "% comment", "50 50 300"]
    for k in range(300):
        i = int(rng.integers(1, 51))
        j = int(rng.integers(1, i + 1))
        lines.append(f"{i} {j} {rng.standard_normal():.17g}")
        if k % 50 == 7:
            lines.append("")
    p = tmp_path / "crlf.mtx"
    p.write_bytes(("\r\n".join(lines) + "\r\n").encode())
    ours = pf.mmio_read(str(p))
    ref = oracle.ref_mmio(str(p))
    assert ours[:4] == ref[:4]
    assert np.array_equal(ours[4], ref[4].astype(np.int64))
    assert np.array_equal(ours[5], ref[5])
    assert np.array_equal(ours[6].view(np.uint64), ref[6].view(np.uint64))


def test_returned_arrays_own_their_memory(pf, tmp_path):
    """The CSR arrays are the library's own buffers, handed over without a
    copy: views of them stay valid after the tuple is dropped, and each buffer
    goes back to the library once nothing views it."""
    import gc
    rng = np.random.default_rng(9)
    p = str(tmp_path / "own.mtx")
    write_random_mtx(p, rng, 300, 300, 5000)
    first = pf.mmio_read(p)
    expect = [a.copy() for a in first[4:]]
    views = [a[1:] for a in first[4:]]
    del first
    gc.collect()
    for _ in range(3):
        pf.mmio_read(p)  # allocations that would reuse freed buffers
    for v, e in zip(views, expect):
        assert np.array_equal(v, e[1:])
    del views
    gc.collect()


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
