"""The benchmark configurations at full size on the GPU, checked against the
oracle: configs 1-4 row by row (the serial oracle runs in seconds at these
sizes), config 5 (2^31 non-zeros, int64 row_ptr) on seeded sampled rows plus
size-independent properties. Inputs come from the device generator, which is
itself checked against the host generator on sampled rows."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def torch_cuda():
    import torch
    assert torch.cuda.is_available()
    return torch


@pytest.fixture(scope="module")
def handle(pf, torch_cuda):
    h = pf.Handle()
    yield h
    h.close()


def gen_device(pf, torch, spec, vdt, idt):
    tv = torch.float64 if vdt == np.float64 else torch.float32
    ti = torch.int32 if idt == np.int32 else torch.int64
    rp, col, val = pf.gen_rows_device(spec, index_dtype=ti, value_dtype=tv)
    x = pf.gen_x_device(spec, value_dtype=tv)
    torch.cuda.synchronize()
    return rp, col, val, x


@pytest.mark.parametrize("cfg,vdt,idt", [
    (1, np.float64, np.int32),
    (2, np.float64, np.int32),
    (3, np.float64, np.int32),
    (3, np.float32, np.int32),
    (4, np.float64, np.int32),
    (4, np.float64, np.int64),
])
def test_config_parity(pf, oracle, torch_cuda, handle, cfg, vdt, idt):
    torch = torch_cuda
    spec = pf.GenSpec(cfg=cfg, seed=12345).resolved()
    rp, col, val, x = gen_device(pf, torch, spec, vdt, idt)
    m, n = spec.m, spec.n
    y = torch.empty(m, dtype=val.dtype, device="cuda")
    pf.spmv(handle, m, n, col.numel(), rp, col, val, x, y)
    torch.cuda.synchronize()
    assert handle.device_error() == 0
    h_rp, h_col, h_val, h_x = (t.cpu().numpy() for t in (rp, col, val, x))
    ref = oracle.serial(h_rp, h_col, h_val, h_x)
    a, comp = oracle.abs_comp(h_rp, h_col, h_val, h_x)
    eps = 1e-12 if vdt == np.float64 else 1e-5
    ok, worst, nbad = oracle.tolerance_report(y.cpu().numpy().astype(np.float64), ref, a, eps,
                                              y_comp=comp)
    assert ok, f"config {cfg}: {nbad} rows out of tolerance, worst {worst:.3g}"


@pytest.mark.parametrize("cfg", [1, 2, 3, 4])
def test_config_integer_mode_bit_exact(pf, oracle, torch_cuda, handle, cfg):
    torch = torch_cuda
    spec = pf.GenSpec(cfg=cfg, seed=777, value_mode=1).resolved()
    rp, col, val, x = gen_device(pf, torch, spec, np.float64, np.int32)
    y = torch.empty(spec.m, dtype=torch.float64, device="cuda")
    pf.spmv(handle, spec.m, spec.n, col.numel(), rp, col, val, x, y)
    h = [t.cpu().numpy() for t in (rp, col, val, x)]
    ref = oracle.serial(*h)
    assert np.array_equal(y.cpu().numpy(), ref)
    if oracle.ref_available():
        assert np.array_equal(oracle.ref_serial(*h), ref)


@pytest.mark.parametrize("cfg", [1, 2, 3, 4, 5])
def test_device_generator_matches_host(pf, torch_cuda, cfg):
    torch = torch_cuda
    spec = pf.GenSpec(cfg=cfg, seed=99).resolved()
    rng = np.random.default_rng(cfg)
    for r0 in [0, int(rng.integers(0, spec.m - 64)), spec.m - 64]:
        rp_d, col_d, val_d = pf.gen_rows_device(spec, r0, r0 + 64, index_dtype=torch.int64)
        rp_h, col_h, val_h = pf.gen_rows_host(spec, r0, r0 + 64)
        assert np.array_equal(rp_d.cpu().numpy(), rp_h)
        assert np.array_equal(col_d.cpu().numpy(), col_h)
        assert np.array_equal(val_d.cpu().numpy(), val_h)
    xd = pf.gen_x_device(spec, 1000, 3000).cpu().numpy()
    assert np.array_equal(xd, pf.gen_x_host(spec, 1000, 3000))


def test_config5_sampled_rows(pf, oracle, torch_cuda, handle):
    """Config 5 at full size: 2^26 rows, 2^31 non-zeros (int64 row_ptr)."""
    torch = torch_cuda
    spec = pf.GenSpec(cfg=5, seed=2024).resolved()
    rp, col, val, x = gen_device(pf, torch, spec, np.float64, np.int64)
    assert int(rp[-1]) == 2 ** 31
    y = torch.empty(spec.m, dtype=torch.float64, device="cuda")
    pf.spmv(handle, spec.m, spec.n, col.numel(), rp, col, val, x, y)
    y2 = torch.empty_like(y)
    pf.spmv(handle, spec.m, spec.n, col.numel(), rp, col, val, x, y2)
    torch.cuda.synchronize()
    assert handle.device_error() == 0
    assert torch.equal(y, y2)                      # deterministic
    rng = np.random.default_rng(5)
    rows = np.unique(np.concatenate([[0, 1, spec.m - 1], rng.integers(0, spec.m, 2000)]))
    hx = pf.gen_x_host(spec)
    yh = y.cpu().numpy()
    for r in rows:
        rph, colh, valh = pf.gen_rows_host(spec, int(r), int(r) + 1)
        ref = oracle.serial(rph, colh, valh, hx)
        a, _ = oracle.abs_comp(rph, colh, valh, hx)
        assert abs(yh[r] - ref[0]) <= 1e-12 * a[0], (r, yh[r], ref[0])
    # linearity: A(2x) = 2 A x exactly (scaling by 2 is exact)
    x2 = x * 2
    pf.spmv(handle, spec.m, spec.n, col.numel(), rp, col, val, x2, y2)
    torch.cuda.synchronize()
    assert torch.equal(y2, 2 * y)
