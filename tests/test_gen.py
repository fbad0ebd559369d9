"""Synthetic config generators (host side): the structure each benchmark
config promises, determinism, and the i % 15 mode."""
import numpy as np
import pytest


def rows_ok(rp, col, n):
    for r in range(len(rp) - 1):
        c = col[rp[r]:rp[r + 1]]
        assert np.all(np.diff(c) > 0), f"row {r} not strictly increasing"
        assert len(c) == 0 or (c[0] >= 0 and c[-1] < n)


@pytest.mark.parametrize("cfg", [1, 3, 4, 5])
def test_sorted_distinct_in_range(pf, cfg):
    spec = pf.GenSpec(cfg=cfg, seed=5).resolved()
    r0 = spec.m // 3
    rp, col, val = pf.gen_rows_host(spec, r0, r0 + 300)
    rows_ok(rp, col, spec.n)
    if cfg in (1, 4, 5):
        assert np.all(np.diff(rp) == spec.k)


def test_config_sizes(pf):
    want = {1: (100000, 100000, 16), 2: (2048 * 2048, 2048 * 2048, 5), 3: (4000000, 4000000, 200000),
            4: (50000, 50000, 2000), 5: (1 << 26, 1 << 26, 32)}
    for cfg, (m, n, k) in want.items():
        s = pf.GenSpec(cfg=cfg).resolved()
        assert (s.m, s.n, s.k) == (m, n, k)
    assert pf.gen_count(pf.GenSpec(cfg=2)) == 20963328          # 5-point stencil on 2048^2
    assert pf.gen_count(pf.GenSpec(cfg=5)) == 2 ** 31


def test_laplacian_rows(pf):
    spec = pf.GenSpec(cfg=2, m=16).resolved()                   # 4x4 grid
    rp, col, val = pf.gen_rows_host(spec)
    rows_ok(rp, col, 16)
    r = 5                                                        # interior point (1,1)
    assert col[rp[r]:rp[r + 1]].tolist() == [1, 4, 5, 6, 9]
    assert val[rp[r]:rp[r + 1]].tolist() == [-1, -1, 4, -1, -1]
    assert (rp[1] - rp[0]) == 3                                  # corner


def test_values_and_x_ranges(pf):
    spec = pf.GenSpec(cfg=1, seed=3).resolved()
    _, _, val = pf.gen_rows_host(spec, 0, 5000)
    assert val.min() >= -1 and val.max() < 1 and abs(val.mean()) < 0.05
    x = pf.gen_x_host(spec)
    assert x.min() >= -1 and x.max() < 1
    _, _, v4 = pf.gen_rows_host(pf.GenSpec(cfg=4, seed=3), 0, 50)    # Irwin-Hall(12) - 6
    assert abs(v4.mean()) < 0.05 and abs(v4.std() - 1) < 0.05


def test_mod15_mode_matches_harness(pf):
    spec = pf.GenSpec(cfg=3, seed=9, value_mode=1, m=5000).resolved()
    rp, col, val = pf.gen_rows_host(spec)
    assert np.array_equal(val, (np.arange(len(val)) % 15).astype(np.float64))
    # a later row range carries the global non-zero index
    rp2, _, val2 = pf.gen_rows_host(spec, 1000, 2000)
    assert np.array_equal(val2, val[rp[1000]:rp[2000]])
    assert np.array_equal(pf.gen_x_host(spec)[:30], np.arange(30) % 15)


def test_row_ranges_compose(pf):
    """Row r is a pure function of (seed, r): any split reproduces the whole."""
    spec = pf.GenSpec(cfg=3, seed=21, m=20000).resolved()
    rp, col, val = pf.gen_rows_host(spec)
    a = pf.gen_rows_host(spec, 0, 7000)
    b = pf.gen_rows_host(spec, 7000, 20000)
    assert np.array_equal(np.concatenate([a[1], b[1]]), col)
    assert np.array_equal(np.concatenate([a[2], b[2]]), val)
    assert np.array_equal(np.concatenate([a[0][:-1], b[0] + a[0][-1]]), rp)


@pytest.mark.slow
def test_powerlaw_mean_row_length(pf):
    spec = pf.GenSpec(cfg=3, seed=12345).resolved()
    z = pf.gen_count(spec)
    assert 7.5 < z / spec.m < 8.8                                # "mean ~ 8"
    lens = np.zeros(spec.m, dtype=np.int64)
    import ctypes as C
    pf._check(pf.lib.pf_gen_row_lengths_host(C.byref(spec.c()), 0, spec.m, lens.ctypes.data))
    assert lens.min() == 1 and lens.max() <= 200000
    assert (lens >= 4096).sum() > 100


def test_banded_fraction(pf):
    spec = pf.GenSpec(cfg=5, seed=4).resolved()
    r0 = 1 << 25
    rp, col, _ = pf.gen_rows_host(spec, r0, r0 + 2000)
    rows = np.repeat(np.arange(r0, r0 + 2000), 32)
    frac = np.mean(np.abs(col.astype(np.int64) - rows) <= 4096)
    assert 0.66 < frac < 0.74
