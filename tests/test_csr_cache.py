"""Binary CSR cache of the Matrix Market loader (pf_csr_write / pf_csr_read /
pf_mmio_read_cached): a cached load returns exactly what pf_mmio_read parses
(the reference's mmio_allinone semantics, utilities/mmio.cpp:1547-1713), a
changed .mtx or a damaged cache is never trusted. CPU only."""
import os
import shutil

import numpy as np
import pytest

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "mtx")
NAMES = sorted(f for f in os.listdir(GOLDEN) if f.endswith(".mtx"))


def same(a, b):
    assert a[:4] == b[:4]
    for x, y in zip(a[4:], b[4:]):
        assert np.array_equal(x, y)


@pytest.mark.parametrize("name", NAMES)
def test_cached_equals_parse(pf, tmp_path, name):
    src = tmp_path / name
    shutil.copy(os.path.join(GOLDEN, name), src)
    cache = tmp_path / (name + ".csr")
    direct = pf.mmio_read(str(src))
    first, hit1 = pf.mmio_read_cached(str(src), str(cache))
    second, hit2 = pf.mmio_read_cached(str(src), str(cache))
    assert not hit1 and hit2
    same(first, direct)
    same(second, direct)
    same(pf.csr_read(str(cache)), direct)


def test_stale_cache_is_reparsed(pf, tmp_path):
    src = tmp_path / "a.mtx"
    cache = tmp_path / "a.csr"
    src.write_text("%%MatrixMarket matrix coordinate real general\n3 3 2\n1 1 1.5\n3 2 -2\n")
    (_, hit) = pf.mmio_read_cached(str(src), str(cache))
    assert not hit
    src.write_text("%%MatrixMarket matrix coordinate real general\n3 3 3\n1 1 1.5\n3 2 -2\n2 2 7\n")
    os.utime(src, ns=(os.stat(src).st_atime_ns, os.stat(src).st_mtime_ns + 10**9))
    csr, hit = pf.mmio_read_cached(str(src), str(cache))
    assert not hit and csr[2] == 3
    csr, hit = pf.mmio_read_cached(str(src), str(cache))
    assert hit and csr[2] == 3


@pytest.mark.parametrize("damage", ["magic", "truncate", "rowptr", "column"])
def test_damaged_cache_rejected(pf, tmp_path, damage):
    rp = np.array([0, 2, 2, 5], dtype=np.int64)
    col = np.array([0, 3, 1, 2, 3], dtype=np.int32)
    val = np.arange(5, dtype=np.float64)
    path = tmp_path / "m.csr"
    pf.csr_write(str(path), 3, 4, rp, col, val)
    same(pf.csr_read(str(path)), (3, 4, 5, False, rp, col, val))
    raw = bytearray(path.read_bytes())
    if damage == "magic":
        raw[0] ^= 0xFF
    elif damage == "truncate":
        raw = raw[:-3]
    elif damage == "rowptr":
        raw[64 + 8] = 9          # row_ptr[1] = 9 > row_ptr[2]
    else:
        raw[64 + 32 + 4] = 200  # col[1] = 200 >= n
    path.write_bytes(bytes(raw))
    with pytest.raises(pf.PfError):
        pf.csr_read(str(path))


def test_cache_of_empty_matrix(pf, tmp_path):
    path = tmp_path / "e.csr"
    pf.csr_write(str(path), 4, 4, np.zeros(5, dtype=np.int64), np.zeros(0, np.int32), np.zeros(0))
    m, n, z, _, rp, col, val = pf.csr_read(str(path))
    assert (m, n, z) == (4, 4, 0) and rp.tolist() == [0] * 5 and len(col) == 0
