"""NNZROW at the edges of its tile walk, against the CPU oracle.

A tile is 224 non-zeros of a slice with fp64 values (7 per thread of a
one-warp CTA) and 320 with fp32 or 16-bit values (10 per thread); its rows
are taken in windows of 32 (one per thread), a row piece of more than 64
products goes to a warp, and the sum of the row left open at the tile's end
is carried to the next tile. These matrices put that walk at its edges: long
runs of one-non-zero rows (a tile of row ends: seven or ten windows), short
rows mixed with empty ones,
heavy tails (long pieces next to short ones), and slice lengths around and
at multiples of the tile, so that a slice's cut first row ends inside a tile
and cut rows span several slices. Tolerance as in the other parity tests;
with integer values every sum is exact and the results must be
bit-identical.
"""
import numpy as np
import pytest

from csr_cases import from_lengths

pytestmark = pytest.mark.gpu

EPS = {np.float64: 1e-12, np.float32: 1e-5}
NNZROW = 7


@pytest.fixture(scope="module")
def torch_cuda():
    import torch
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    return torch


@pytest.fixture
def ws_handle(pf, torch_cuda):
    h = pf.Handle()
    h.set_variant(NNZROW)
    yield h
    h.close()


def lengths(name, rng):
    if name == "unit_rows":
        # long stretches of one-non-zero rows, a few runs of 2-3, long rows between
        parts = []
        for _ in range(6):
            parts.append(np.ones(int(rng.integers(3000, 9000)), dtype=np.int64))
            parts.append(rng.integers(2, 4, size=int(rng.integers(200, 2000))))
            parts.append(rng.integers(300, 3000, size=3))
        return np.concatenate(parts)
    if name == "short_with_empty":
        # lengths 0-3: many empty rows between short ones
        return rng.choice([0, 1, 1, 2, 3], size=40000)
    if name == "short_no_empty":
        return rng.integers(1, 5, size=40000)
    if name == "powerlaw_unit":
        # most rows one non-zero, a heavy tail (the shape of config 3)
        u = rng.random(30000)
        return np.minimum(np.floor(u ** (-1 / 1.1)), 20000).astype(np.int64)
    raise KeyError(name)


NAMES = ["unit_rows", "short_with_empty", "short_no_empty", "powerlaw_unit"]


def run(pf, torch, h, rp, col, val, x, n, vdt, idt, alpha=1.0, beta=0.0, y0=None):
    m = len(rp) - 1
    tv = {np.float64: torch.float64, np.float32: torch.float32}[vdt]
    d_rp = torch.from_numpy(rp.astype(idt)).cuda()
    d_col = torch.from_numpy(col.astype(np.int32)).cuda()
    d_val = torch.from_numpy(val.astype(vdt)).cuda()
    d_x = torch.from_numpy(x.astype(vdt)).cuda()
    if y0 is None:
        d_y = torch.full((m,), float("nan"), dtype=tv, device="cuda")
    else:
        d_y = torch.from_numpy(y0.astype(vdt)).cuda()
    pf.spmv(h, m, n, len(col), d_rp, d_col, d_val, d_x, d_y, alpha, beta)
    torch.cuda.synchronize()
    assert h.device_error() == 0
    return d_y.cpu().numpy().astype(np.float64)


def check(oracle, y, rp, col, val, x, vdt, alpha=1.0, beta=0.0, y0=None):
    vq, xq = val.astype(vdt), x.astype(vdt)
    s = oracle.serial(rp, col, vq, xq)
    a, comp = oracle.abs_comp(rp, col, vq, xq)
    yb = np.zeros(len(rp) - 1) if y0 is None else y0.astype(vdt).astype(np.float64)
    ref = alpha * s + beta * yb
    scale = abs(alpha) * a + abs(beta) * np.abs(yb)
    ok, worst, nbad = oracle.tolerance_report(y, ref, scale, EPS[vdt],
                                              y_comp=alpha * comp + beta * yb)
    assert ok, f"{nbad} rows out of tolerance (worst ratio {worst:.3g})"


@pytest.mark.parametrize("name", NAMES)
@pytest.mark.parametrize("slice_nnz", [0, 1, 63, 223, 224, 256, 319, 320, 448, 511, 512, 640, 768, 1000, 4096])
@pytest.mark.parametrize("idt", [np.int32, np.int64])
@pytest.mark.parametrize("vdt", [np.float64, np.float32])
def test_tile_walk_slices(pf, oracle, torch_cuda, ws_handle, name, slice_nnz, idt, vdt):
    rng = np.random.default_rng(11)
    n = 50000
    rp, col, val = from_lengths(rng, lengths(name, rng), n)
    x = np.random.default_rng(12).uniform(-1, 1, n)
    ws_handle.set_slice(slice_nnz)
    y = run(pf, torch_cuda, ws_handle, rp, col, val, x, n, vdt, idt)
    check(oracle, y, rp, col, val, x, vdt)


@pytest.mark.parametrize("name", NAMES)
@pytest.mark.parametrize("vdt", [np.float64, np.float32])
@pytest.mark.parametrize("alpha,beta", [(1.0, 0.0), (-0.75, 0.5), (0.0, 2.0)])
def test_tile_walk_alpha_beta(pf, oracle, torch_cuda, ws_handle, name, vdt, alpha, beta):
    rng = np.random.default_rng(13)
    n = 50000
    rp, col, val = from_lengths(rng, lengths(name, rng), n)
    x = np.random.default_rng(14).uniform(-1, 1, n)
    y0 = np.random.default_rng(15).uniform(-1, 1, len(rp) - 1)
    ws_handle.set_slice(512)
    y = run(pf, torch_cuda, ws_handle, rp, col, val, x, n, vdt, np.int32, alpha, beta, y0)
    check(oracle, y, rp, col, val, x, vdt, alpha, beta, y0)


@pytest.mark.parametrize("name", NAMES)
@pytest.mark.parametrize("slice_nnz", [0, 768])
def test_tile_walk_integer_bit_exact(pf, oracle, torch_cuda, ws_handle, name, slice_nnz):
    """Integer values and x (the reference harness's i % 15 values): every
    partial sum is exact, so y must equal the serial sum bit for bit."""
    rng = np.random.default_rng(16)
    n = 50000
    rp, col, val = from_lengths(rng, lengths(name, rng), n, values="mod15")
    x = np.random.default_rng(17).integers(-7, 8, n).astype(np.float64)
    ws_handle.set_slice(slice_nnz)
    y = run(pf, torch_cuda, ws_handle, rp, col, val, x, n, np.float64, np.int64)
    ref = oracle.serial(rp, col, val, x)
    assert np.array_equal(y, ref)
