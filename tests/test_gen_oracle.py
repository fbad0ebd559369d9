"""The C restatement of the synthetic generators (oracle/gen_oracle.c) against
the library's host generator: every config, row slices away from the start
and both value modes give bit-identical row_ptr, col, val and x."""
import numpy as np
import pytest

CASES = [(1, 0), (2, 0), (3, 0), (4, 0), (5, 0), (1, 1), (3, 1), (5, 1)]


@pytest.mark.parametrize("cfg,value_mode", CASES)
def test_gen_oracle_matches_library(pf, oracle, cfg, value_mode):
    spec = pf.GenSpec(cfg=cfg, seed=12345, value_mode=value_mode).resolved()
    rows = {1: 3000, 2: 5000, 3: 3000, 4: 200, 5: 3000}[cfg]
    for r0 in (0, spec.m // 2, spec.m - rows):
        r1 = r0 + rows
        rp, col, val = pf.gen_rows_host(spec, r0, r1)
        orp, ocol, oval, ox = oracle.gen_config(cfg, seed=12345, value_mode=value_mode,
                                                m=spec.m, n=spec.n, r0=r0, r1=r1, threads=3)
        assert np.array_equal(rp, orp)
        assert np.array_equal(col, ocol)
        assert np.array_equal(val.view(np.uint64), oval.view(np.uint64))
    x = pf.gen_x_host(spec)
    assert np.array_equal(x.view(np.uint64), ox.view(np.uint64))


def test_gen_oracle_thread_split_invariant(oracle):
    """The same rows whatever the number of host threads."""
    a = oracle.gen_config(3, m=20000, n=20000, threads=1)
    b = oracle.gen_config(3, m=20000, n=20000, threads=7)
    for u, v in zip(a, b):
        assert np.array_equal(u, v)
