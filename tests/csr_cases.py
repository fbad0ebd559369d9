"""Seeded CSR test matrices with the edge cases the reference's tiling meets
(empty rows, row 0 spanning many tiles, trailing empty rows, one huge row,
long runs of empty rows, nnz = 0)."""
import numpy as np


def from_lengths(rng, lens, n, sorted_cols=True, values="uniform"):
    lens = np.asarray(lens, dtype=np.int64)
    m = len(lens)
    rp = np.zeros(m + 1, dtype=np.int64)
    np.cumsum(lens, out=rp[1:])
    z = int(rp[-1])
    col = np.empty(z, dtype=np.int32)
    for r in range(m):
        k = int(lens[r])
        if k == 0:
            continue
        if k <= n:
            c = rng.choice(n, size=k, replace=False)
        else:
            c = rng.integers(0, n, size=k)
        if sorted_cols:
            c = np.sort(c)
        col[rp[r]:rp[r + 1]] = c
    if values == "mod15":
        val = (np.arange(z) % 15).astype(np.float64)
    else:
        val = rng.uniform(-1, 1, size=z)
    return rp, col, val


def case(name, seed=0):
    rng = np.random.default_rng(seed)
    if name == "tiny":
        rp = np.array([0, 2, 3, 5], dtype=np.int64)
        col = np.array([0, 2, 1, 0, 2], dtype=np.int32)
        val = np.array([1.0, 2.0, 3.0, 4.0, 5.0])
        return rp, col, val, 3
    if name == "empty_matrix":
        return np.zeros(7, dtype=np.int64), np.zeros(0, np.int32), np.zeros(0), 5
    if name == "one_long_row":
        return (*from_lengths(rng, [50000], 60000), 60000)
    if name == "row0_long":
        lens = np.concatenate([[20000], rng.integers(0, 20, size=3000)])
        return (*from_lengths(rng, lens, 5000), 5000)
    if name == "empty_edges":
        lens = np.concatenate([np.zeros(37), rng.integers(0, 40, size=2000), np.zeros(1500),
                               rng.integers(1, 9, size=500), np.zeros(23)])
        return (*from_lengths(rng, lens, 3000), 3000)
    if name == "powerlaw":
        u = rng.random(20000)
        lens = np.minimum(np.rint(u ** (-1 / 1.1)), 30000).astype(np.int64)
        return (*from_lengths(rng, lens, 40000), 40000)
    if name == "uniform16":
        return (*from_lengths(rng, np.full(5000, 16), 5000), 5000)
    if name == "mixed_long":
        lens = rng.integers(0, 6, size=8000)
        lens[[5, 700, 701, 4000, 7999]] = [9000, 4000, 12000, 2500, 7000]
        return (*from_lengths(rng, lens, 8000), 8000)
    if name == "long_rows":
        # rows of 128-600 non-zeros (the long-row ROWVEC path: every lane
        # walks two blocks or more), with empty, 1-7 and one 20000-long row
        lens = rng.integers(128, 600, size=2000)
        lens[[0, 3, 500, 501, 1200, 1999]] = [0, 1, 3, 7, 20000, 0]
        return (*from_lengths(rng, lens, 30000), 30000)
    if name == "unsorted":
        lens = rng.integers(0, 30, size=3000)
        return (*from_lengths(rng, lens, 2000, sorted_cols=False), 2000)
    raise KeyError(name)


CASES = ["tiny", "empty_matrix", "one_long_row", "row0_long", "empty_edges", "powerlaw",
         "uniform16", "mixed_long", "unsorted", "long_rows"]


def gen_config_host(pf, spec, threads=None):
    """A whole generated config on the host: (row_ptr int64, col, val, x).
    Row ranges are generated on several threads straight into the final
    arrays (the library call releases the GIL); the result equals one call
    over all rows."""
    import ctypes as C
    import os
    import threading
    threads = threads or os.cpu_count() or 1
    s = spec.resolved()
    m = s.m
    cuts = [m * k // threads for k in range(threads + 1)]
    offs = [pf.gen_count(spec, 0, c) for c in cuts]
    z = offs[-1]
    rp = np.empty(m + 1, dtype=np.int64)
    rp[0] = 0
    col = np.empty(max(z, 1), dtype=np.int32)
    val = np.empty(max(z, 1), dtype=np.float64)
    cs = s.c()
    err = []

    def work(k):
        r0, r1 = cuts[k], cuts[k + 1]
        lrp = np.empty(r1 - r0 + 1, dtype=np.int64)
        st = pf.lib.pf_gen_rows_host(C.byref(cs), r0, r1, lrp.ctypes.data,
                                     col.ctypes.data + 4 * offs[k], val.ctypes.data + 8 * offs[k])
        if st:
            err.append(st)
        rp[r0 + 1:r1 + 1] = lrp[1:] + offs[k]

    ts = [threading.Thread(target=work, args=(k,)) for k in range(threads)]
    for t in ts:
        t.start()
    for t in ts:
        t.join()
    assert not err, err
    return rp, col[:z], val[:z], pf.gen_x_host(spec)
