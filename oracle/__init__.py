"""CPU oracle for the CSR SpMV hot path — TEST INFRASTRUCTURE ONLY.

Loaded by tests/, ``__graft_entry__.smoke()`` and bench.py's cpu_baseline /
``--impl reference`` arm, as the checker or the timed CPU baseline; the
product (prefree-public_b200/) never imports it.

Three libraries:
  * ``liboracle.so`` — the C restatement in spmv_oracle.c of the reference's
    ``spmv_serial`` (test/test_cdspmv.cpp:4-20) with int32/int64 offsets and
    fp64/fp32 inputs, plus per-row |a*x| sums and a compensated sum; and, in
    gen_oracle.c, a separately written host copy of the synthetic config
    generators (inputs for the reference arm without the library under test,
    and a second implementation the library's generators are pinned to);
  * ``_ref/libref.so`` — the reference's own ``spmv_serial`` and
    ``mmio_allinone`` (utilities/mmio.cpp:1547-1713), compiled from the
    reference sources by oracle/Makefile;
  * ``_ref/libref_gpu.so`` — the reference's own GPU entry point
    ``preFreeSpMV`` with its kernel (src/spmv_kernel/preFreeSpMV.cu),
    compiled unmodified for sm_100a by oracle/Makefile: a second checker on
    inputs it handles correctly, and the B200 timing comparison.
The restatement is pinned to the reference build by tests/test_oracle.py
(bit-identical outputs) and by the golden fixtures in tests/golden/ that the
reference build produced (tests/golden/make_golden.py).
"""
from __future__ import annotations

import ctypes as C
import os
import threading

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_LIB = os.path.join(_HERE, "liboracle.so")
REF_LIB = os.path.join(_HERE, "_ref", "libref.so")
REF_GPU_LIB = os.path.join(_HERE, "_ref", "libref_gpu.so")
# include/PreFree.h:3-5 under -Dfp64: preFreeSpMV(double*, int*, int*, double*,
# double*, int, int, int, double*, double*), C++ linkage
REF_GPU_SYMBOL = "_Z11preFreeSpMVPdPiS0_S_S_iiiS_S_"

_vp, _i64, _i32 = C.c_void_p, C.c_int64, C.c_int32


def _load_oracle():
    lib = C.CDLL(ORACLE_LIB)
    for v in ("f64", "f32"):
        for i in ("i32", "i64"):
            f = getattr(lib, f"oracle_spmv_serial_{v}_{i}")
            f.argtypes = [_vp, _vp, _vp, _vp, _vp, _i64]
            f.restype = None
            g = getattr(lib, f"oracle_spmv_abs_comp_{v}_{i}")
            g.argtypes = [_vp, _vp, _vp, _vp, _vp, _vp, _i64]
            g.restype = None
    lib.oracle_coo_to_csr.argtypes = [_i64, _i64, _vp, _vp, _vp, C.c_int, _vp, _vp, _vp, _vp]
    lib.oracle_coo_to_csr.restype = _i64
    g = [C.c_int, C.c_int, C.c_uint64, _i64, _i64, _i64]
    lib.oracle_gen_count.argtypes = g + [_i64, _i64]
    lib.oracle_gen_count.restype = _i64
    lib.oracle_gen_rows.argtypes = g + [_i64, _i64, _vp, _vp, _vp]
    lib.oracle_gen_rows.restype = C.c_int
    lib.oracle_gen_x.argtypes = g + [_i64, _i64, _vp]
    lib.oracle_gen_x.restype = C.c_int
    lib.oracle_gen_resolve.argtypes = [C.c_int, C.POINTER(_i64), C.POINTER(_i64), C.POINTER(_i64)]
    lib.oracle_gen_resolve.restype = C.c_int
    return lib


lib = _load_oracle()
_ref = None


def ref_available() -> bool:
    return os.path.exists(REF_LIB)


def ref_lib():
    """The reference's own compiled CPU code (oracle/_ref/libref.so)."""
    global _ref
    if _ref is None:
        if not ref_available():
            raise FileNotFoundError(f"{REF_LIB} not built (make -C oracle with the reference tree)")
        r = C.CDLL(REF_LIB)
        r.ref_spmv_serial.argtypes = [_vp, _vp, _vp, _vp, _vp, C.c_int, C.c_int, C.c_int]
        r.ref_spmv_serial.restype = None
        r.ref_mmio_allinone.argtypes = [C.c_char_p, C.POINTER(C.c_int), C.POINTER(C.c_int),
                                        C.POINTER(C.c_int), C.POINTER(C.c_int),
                                        C.POINTER(_vp), C.POINTER(_vp), C.POINTER(_vp)]
        r.ref_mmio_allinone.restype = C.c_int
        r.ref_free.argtypes = [_vp]
        r.ref_free.restype = None
        _ref = r
    return _ref


_ref_gpu = None


def ref_gpu_available() -> bool:
    return os.path.exists(REF_GPU_LIB)


def ref_gpu_prefree(val, row_ptr, col, x, m: int, n: int):
    """The reference's own preFreeSpMV on the GPU (oracle/_ref/libref_gpu.so):
    host fp64 CSR with int32 indices in, y = A*x out, with the reference's own
    timings (ms per multiply over 4000 launches after 200 warm-ups, and ms of
    its start-row pre-pass). Returns (y, cdTime, cdPre). The reference copies
    row_ptr[0 .. m+1] (one entry past the CSR, src/spmv_kernel/preFreeSpMV.cu:580),
    so it is handed a copy with one padding entry."""
    global _ref_gpu
    if _ref_gpu is None:
        if not ref_gpu_available():
            raise FileNotFoundError(f"{REF_GPU_LIB} not built (make -C oracle with the reference tree)")
        r = C.CDLL(REF_GPU_LIB)
        f = getattr(r, REF_GPU_SYMBOL)
        f.argtypes = [_vp, _vp, _vp, _vp, _vp, C.c_int, C.c_int, C.c_int,
                      C.POINTER(C.c_double), C.POINTER(C.c_double)]
        f.restype = None
        _ref_gpu = f
    nnz = int(row_ptr[m]) - int(row_ptr[0])
    assert int(row_ptr[0]) == 0 and nnz < 2**31
    rp = np.empty(m + 2, dtype=np.int32)
    rp[:m + 1] = row_ptr
    rp[m + 1] = row_ptr[m]
    v = np.ascontiguousarray(val, dtype=np.float64)
    c = np.ascontiguousarray(col, dtype=np.int32)
    xx = np.ascontiguousarray(x, dtype=np.float64)
    y = np.zeros(max(m, 1), dtype=np.float64)
    t, pre = C.c_double(), C.c_double()
    _ref_gpu(_p(v), _p(rp), _p(c), _p(xx), _p(y), m, n, nnz, C.byref(t), C.byref(pre))
    return y[:m], t.value, pre.value


def _p(a: np.ndarray) -> int:
    return a.ctypes.data


def _tags(val: np.ndarray, row_ptr: np.ndarray) -> str:
    v = {np.dtype(np.float64): "f64", np.dtype(np.float32): "f32"}[val.dtype]
    i = {np.dtype(np.int32): "i32", np.dtype(np.int64): "i64"}[row_ptr.dtype]
    return f"{v}_{i}"


def serial(row_ptr, col, val, x, y0=None) -> np.ndarray:
    """Restated spmv_serial: y[i] = y0[i] + sum_j val*x[col] in storage order,
    accumulated in double. row_ptr may start at a non-zero offset (absolute
    indexing into col/val)."""
    row_ptr = np.ascontiguousarray(row_ptr)
    col = np.ascontiguousarray(col, dtype=np.int32)
    val = np.ascontiguousarray(val)
    x = np.ascontiguousarray(x, dtype=val.dtype)
    m = len(row_ptr) - 1
    y = np.zeros(m, dtype=np.float64) if y0 is None else np.array(y0, dtype=np.float64)
    if m > 0:
        getattr(lib, "oracle_spmv_serial_" + _tags(val, row_ptr))(
            _p(val), _p(row_ptr), _p(col), _p(x), _p(y), m)
    return y


def abs_comp(row_ptr, col, val, x):
    """Per-row (sum |val*x|, Neumaier-compensated sum)."""
    row_ptr = np.ascontiguousarray(row_ptr)
    col = np.ascontiguousarray(col, dtype=np.int32)
    val = np.ascontiguousarray(val)
    x = np.ascontiguousarray(x, dtype=val.dtype)
    m = len(row_ptr) - 1
    a = np.zeros(m, dtype=np.float64)
    s = np.zeros(m, dtype=np.float64)
    if m > 0:
        getattr(lib, "oracle_spmv_abs_comp_" + _tags(val, row_ptr))(
            _p(val), _p(row_ptr), _p(col), _p(x), _p(a), _p(s), m)
    return a, s


def ref_serial(row_ptr, col, val, x, y0=None) -> np.ndarray:
    """The reference's own spmv_serial (int32 offsets, fp64)."""
    r = ref_lib()
    row_ptr = np.ascontiguousarray(row_ptr, dtype=np.int32)
    col = np.ascontiguousarray(col, dtype=np.int32)
    val = np.ascontiguousarray(val, dtype=np.float64)
    x = np.ascontiguousarray(x, dtype=np.float64)
    m = len(row_ptr) - 1
    y = np.zeros(m, dtype=np.float64) if y0 is None else np.array(y0, dtype=np.float64)
    if m > 0:
        r.ref_spmv_serial(_p(val), _p(row_ptr), _p(col), _p(x), _p(y), m, len(x), len(val))
    return y


def ref_serial_rows(row_ptr32: np.ndarray, col: np.ndarray, val: np.ndarray,
                    x: np.ndarray, y: np.ndarray, r0: int, r1: int):
    """The reference's spmv_serial on rows [r0, r1): it indexes col/val with
    the absolute row_ptr values, so passing row_ptr + r0 and y + r0 runs the
    unmodified function on a row slice. ctypes releases the GIL, so several
    threads can run slices at once."""
    r = ref_lib()
    if r1 <= r0:
        return
    rp = row_ptr32.ctypes.data + 4 * r0
    yp = y.ctypes.data + 8 * r0
    r.ref_spmv_serial(_p(val), rp, _p(col), _p(x), yp, r1 - r0, len(x), len(val))


def ref_serial_threaded(row_ptr32, col, val, x, threads: int) -> np.ndarray:
    """spmv_serial of the reference over equal-nnz row slices on `threads`
    host threads (the reference function itself is single-threaded)."""
    m = len(row_ptr32) - 1
    y = np.zeros(m, dtype=np.float64)
    z = int(row_ptr32[m]) - int(row_ptr32[0])
    cuts = [0]
    for k in range(1, threads):
        cuts.append(int(np.searchsorted(row_ptr32, int(row_ptr32[0]) + z * k // threads)))
    cuts.append(m)
    ts = [threading.Thread(target=ref_serial_rows,
                           args=(row_ptr32, col, val, x, y, cuts[k], cuts[k + 1]))
          for k in range(threads)]
    for t in ts:
        t.start()
    for t in ts:
        t.join()
    return y


def ref_mmio(path: str):
    """The reference's mmio_allinone: (m, n, nnz, sym, row_ptr, col, val)."""
    r = ref_lib()
    m, n, z, s = C.c_int(), C.c_int(), C.c_int(), C.c_int()
    rp, ci, va = _vp(), _vp(), _vp()
    rc = r.ref_mmio_allinone(os.fsencode(path), C.byref(m), C.byref(n), C.byref(z), C.byref(s),
                             C.byref(rp), C.byref(ci), C.byref(va))
    if rc != 0:
        raise RuntimeError(f"mmio_allinone returned {rc}")
    try:
        row_ptr = np.ctypeslib.as_array(C.cast(rp, C.POINTER(C.c_int32)), (m.value + 1,)).copy()
        nz = max(z.value, 1)
        col = np.ctypeslib.as_array(C.cast(ci, C.POINTER(C.c_int32)), (nz,))[:z.value].copy()
        val = np.ctypeslib.as_array(C.cast(va, C.POINTER(C.c_double)), (nz,))[:z.value].copy()
    finally:
        r.ref_free(rp)
        r.ref_free(ci)
        r.ref_free(va)
    return m.value, n.value, z.value, bool(s.value), row_ptr, col, val


def coo_to_csr(m: int, ri, ci, vi, symmetric: bool):
    """Restated CSR construction of mmio_allinone from 0-based coordinates."""
    ri = np.ascontiguousarray(ri, dtype=np.int32)
    ci = np.ascontiguousarray(ci, dtype=np.int32)
    vi = np.ascontiguousarray(vi, dtype=np.float64)
    cap = max(1, 2 * len(ri))
    rp = np.zeros(m + 1, dtype=np.int64)
    col = np.zeros(cap, dtype=np.int32)
    val = np.zeros(cap, dtype=np.float64)
    cur = np.zeros(max(m, 1), dtype=np.int64)
    z = lib.oracle_coo_to_csr(m, len(ri), _p(ri), _p(ci), _p(vi), int(symmetric), _p(rp),
                              _p(col), _p(val), _p(cur))
    return rp, col[:z], val[:z]


def gen_resolve(cfg: int, m: int = 0, n: int = 0, k: int = 0):
    """(m, n, k) of a config with its defaults filled in."""
    mm, nn, kk = _i64(m), _i64(n), _i64(k)
    if lib.oracle_gen_resolve(cfg, C.byref(mm), C.byref(nn), C.byref(kk)):
        raise ValueError(f"bad config spec {cfg} m={m} n={n} k={k}")
    return mm.value, nn.value, kk.value


def gen_config(cfg: int, seed: int = 12345, value_mode: int = 0, m: int = 0, n: int = 0,
               k: int = 0, r0: int = 0, r1: int | None = None, threads: int | None = None):
    """Rows [r0, r1) of a synthetic config and its full x, from the C
    restatement of the generators: (row_ptr int64 from 0, col int32, val f64,
    x f64). Row ranges run on parallel host threads (ctypes releases the GIL)
    straight into the final arrays."""
    m, n, k = gen_resolve(cfg, m, n, k)
    r1 = m if r1 is None else r1
    threads = threads or os.cpu_count() or 1
    spec = (cfg, value_mode, seed, m, n, k)
    cuts = [r0 + (r1 - r0) * t // threads for t in range(threads + 1)]
    offs = [0] * (threads + 1)
    cnt = [0] * threads

    def count(t):
        cnt[t] = lib.oracle_gen_count(*spec, cuts[t], cuts[t + 1])

    _run_threads(count, threads)
    for t in range(threads):
        offs[t + 1] = offs[t] + cnt[t]
    z = offs[-1]
    rp = np.zeros(r1 - r0 + 1, dtype=np.int64)
    col = np.zeros(max(z, 1), dtype=np.int32)
    val = np.zeros(max(z, 1), dtype=np.float64)
    x = np.zeros(n, dtype=np.float64)
    xc = [n * t // threads for t in range(threads + 1)]
    rc = [0] * threads

    def fill(t):
        a, b = cuts[t], cuts[t + 1]
        lrp = np.zeros(b - a + 1, dtype=np.int64)
        rc[t] |= lib.oracle_gen_rows(*spec, a, b, _p(lrp), col.ctypes.data + 4 * offs[t],
                                     val.ctypes.data + 8 * offs[t])
        rp[a - r0 + 1:b - r0 + 1] = lrp[1:] + offs[t]
        rc[t] |= lib.oracle_gen_x(*spec, xc[t], xc[t + 1], x.ctypes.data + 8 * xc[t])

    _run_threads(fill, threads)
    if any(rc):
        raise RuntimeError("oracle generator failed")
    return rp, col[:z], val[:z], x


def _run_threads(fn, threads: int):
    ts = [threading.Thread(target=fn, args=(t,)) for t in range(threads)]
    for t in ts:
        t.start()
    for t in ts:
        t.join()


def tolerance_report(y, y_ref, abs_sum, eps: float, y_comp=None):
    """Per-row check |y - y_ref| <= eps * sum_j |a_ij x_j| (the north-star
    tolerance). Rows that fail against the serial sum are re-checked against
    the compensated sum when given (the serial sum itself can be off by more
    than eps on very long rows). Returns (ok, worst_ratio, n_bad)."""
    y = np.asarray(y, dtype=np.float64)
    err = np.abs(y - y_ref)
    bound = eps * abs_sum
    bad = err > bound
    if y_comp is not None and bad.any():
        bad &= np.abs(y - y_comp) > bound
    with np.errstate(divide="ignore", invalid="ignore"):
        ratio = np.where(bound > 0, err / np.where(bound > 0, bound, 1), np.where(err > 0, np.inf, 0))
    worst = float(ratio.max()) if len(ratio) else 0.0
    return (not bad.any()), worst, int(bad.sum())
