"""Python host mirror of the B200 CSR SpMV library (libprefree_b200.so).

Thin ctypes bindings over the C ABI declared in include/prefree_b200.h. There
is no CPU fallback: importing this module loads the CUDA library and fails
loudly if it has not been built (``make -C prefree-public_b200`` or
``__graft_entry__.build()``).

The reference's operator interface is ``preFreeSpMV(csrVal, csrRowPtr,
csrColInd, X_val, Y_val, rowA, colA, nnzA, &cdTime, &cdPre)``
(include/PreFree.h:3-5); :func:`preFreeSpMV` here takes the same arguments as
numpy host arrays, overwrites ``Y_val`` in place and returns
``(cdTime, cdPre)``.
"""
from __future__ import annotations

import ctypes as C
import os
from dataclasses import dataclass

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libprefree_b200.so")

PF_OK = 0
STATUS_NAMES = {0: "PF_OK", 1: "PF_ERR_INVALID", 2: "PF_ERR_CUDA", 3: "PF_ERR_DEVICE",
                4: "PF_ERR_UNSUPPORTED", 5: "PF_ERR_IO", 6: "PF_ERR_FORMAT"}
VARIANT_AUTO, VARIANT_NNZSPLIT, VARIANT_ROWGROUP, VARIANT_ROWVEC, VARIANT_NNZROW = 0, 1, 2, 4, 7
VARIANT_NAMES = {0: "auto", 1: "nnzsplit", 2: "rowgroup", 4: "rowvec", 7: "nnzrow"}

# every extern "C" symbol include/*.h declares (checked by the CPU tests)
EXPORTED = [
    "pf_last_error", "pf_version", "pf_launch_count",
    "pf_handle_create", "pf_handle_destroy", "pf_handle_set_variant",
    "pf_handle_set_slice", "pf_handle_device_error", "pf_handle_choice_i32",
    "pf_handle_choice_i64", "pf_handle_dist_wait",
    "pf_spmv_f64_i32", "pf_spmv_f64_i64", "pf_spmv_f32_i32", "pf_spmv_f32_i64",
    "pf_spmv_host_f64_i32", "pf_spmv_host_f64_i64", "pf_spmv_host_f32_i32",
    "pf_spmv_host_f32_i64",
    "pf_prefree_spmv_f64_i32", "pf_prefree_spmv_f64_i64", "pf_prefree_spmv_f32_i32",
    "pf_mmio_read", "pf_free", "pf_shard_bounds_i32", "pf_shard_bounds_i64",
    "pf_gen_resolve", "pf_gen_count", "pf_gen_row_lengths_host", "pf_gen_rows_host",
    "pf_gen_x_host", "pf_gen_rows_device", "pf_gen_x_device",
    "pf_spmv_noalloc_f64_i32", "pf_spmv_dist_f64_i64", "pf_spmv_dist_f64_i32",
    "pf_spmm_f64_i32", "pf_spmm_f64_i64", "pf_spmm_f32_i32", "pf_spmm_f32_i64",
    "pf_spmv_f16_i32", "pf_spmv_f16_i64", "pf_spmv_bf16_i32", "pf_spmv_bf16_i64",
    "pf_csr_write", "pf_csr_read", "pf_mmio_read_cached", "pf_mmio_read_pinned",
    "pf_mmio_read_cached_pinned",
]
# the C++ drop-in symbols of include/PreFree.h (mangled)
CXX_EXPORTED = [
    "_Z11preFreeSpMVPdPiS0_S_S_iiiS_S_",   # (double*, int*, int*, double*, double*, int, int, int, double*, double*)
    "_Z11preFreeSpMVPfPiS0_S_S_iiiPdS1_",  # float overload
    "_Z11preFreeSpMVPdPlPiS_S_lllS_S_",    # int64 overload
]


class PfError(RuntimeError):
    def __init__(self, status: int, msg: str):
        super().__init__(f"{STATUS_NAMES.get(status, status)}: {msg}")
        self.status = status


class pf_gen_spec(C.Structure):
    _fields_ = [("cfg", C.c_int), ("value_mode", C.c_int), ("seed", C.c_uint64),
                ("m", C.c_int64), ("n", C.c_int64), ("k", C.c_int64)]


def _load():
    if not os.path.exists(LIB_PATH):
        raise ImportError(
            f"{LIB_PATH} is missing: build it with `make -C prefree-public_b200` "
            "(there is no CPU fallback)")
    lib = C.CDLL(LIB_PATH)
    vp, i64, i32, dbl = C.c_void_p, C.c_int64, C.c_int32, C.c_double
    st = C.c_int
    lib.pf_last_error.restype = C.c_char_p
    lib.pf_version.restype = C.c_char_p
    lib.pf_launch_count.restype = C.c_uint64
    lib.pf_handle_create.argtypes = [C.POINTER(vp)]
    lib.pf_handle_destroy.argtypes = [vp]
    lib.pf_handle_set_variant.argtypes = [vp, C.c_int]
    lib.pf_handle_set_slice.argtypes = [vp, i64]
    lib.pf_handle_device_error.argtypes = [vp, C.POINTER(C.c_uint32), C.c_int]
    lib.pf_handle_dist_wait.argtypes = [vp, C.POINTER(C.c_uint64), C.POINTER(i64), C.c_int]
    lib.pf_handle_dist_wait.restype = st
    for name in ("pf_handle_choice_i32", "pf_handle_choice_i64"):
        getattr(lib, name).argtypes = [vp, i64, i64, vp, C.c_int, vp, C.POINTER(C.c_int),
                                       C.POINTER(C.c_int)]
        getattr(lib, name).restype = st
    for name in ("pf_spmv_f64_i32", "pf_spmv_f64_i64", "pf_spmv_f32_i32", "pf_spmv_f32_i64",
                 "pf_spmv_f16_i32", "pf_spmv_f16_i64", "pf_spmv_bf16_i32", "pf_spmv_bf16_i64",
                 "pf_spmv_host_f64_i32", "pf_spmv_host_f64_i64", "pf_spmv_host_f32_i32",
                 "pf_spmv_host_f32_i64"):
        f = getattr(lib, name)
        f.argtypes = [vp, i64, i64, i64, vp, vp, vp, dbl, vp, dbl, vp, vp]
        f.restype = st
    for name in ("pf_spmm_f64_i32", "pf_spmm_f64_i64", "pf_spmm_f32_i32", "pf_spmm_f32_i64"):
        f = getattr(lib, name)
        f.argtypes = [vp, i64, i64, i64, vp, vp, vp, C.c_int, dbl, vp, i64, dbl, vp, i64, vp]
        f.restype = st
    for name in ("pf_spmv_dist_f64_i64", "pf_spmv_dist_f64_i32"):
        f = getattr(lib, name)
        f.argtypes = [vp, i64, i64, i64, vp, vp, vp, vp, vp, C.c_int, C.c_int, vp, vp, i64, vp,
                      C.c_uint64, vp]
        f.restype = st
    lib.pf_spmv_noalloc_f64_i32.argtypes = [i64, i64, i64, vp, vp, vp, dbl, vp, dbl, vp, vp]
    lib.pf_spmv_noalloc_f64_i32.restype = st
    lib.pf_prefree_spmv_f64_i32.argtypes = [vp, vp, vp, vp, vp, i32, i32, i32,
                                            C.POINTER(dbl), C.POINTER(dbl)]
    lib.pf_prefree_spmv_f32_i32.argtypes = lib.pf_prefree_spmv_f64_i32.argtypes
    lib.pf_prefree_spmv_f64_i64.argtypes = [vp, vp, vp, vp, vp, i64, i64, i64,
                                            C.POINTER(dbl), C.POINTER(dbl)]
    lib.pf_mmio_read.argtypes = [C.c_char_p, C.POINTER(i64), C.POINTER(i64), C.POINTER(i64),
                                 C.POINTER(C.c_int), C.POINTER(vp), C.POINTER(vp),
                                 C.POINTER(vp)]
    csr_out = [C.POINTER(i64), C.POINTER(i64), C.POINTER(i64), C.POINTER(C.c_int),
               C.POINTER(vp), C.POINTER(vp), C.POINTER(vp)]
    lib.pf_csr_write.argtypes = [C.c_char_p, i64, i64, i64, C.c_int, vp, vp, vp]
    lib.pf_csr_read.argtypes = [C.c_char_p] + csr_out
    lib.pf_mmio_read_cached.argtypes = [C.c_char_p, C.c_char_p] + csr_out + [C.POINTER(C.c_int)]
    lib.pf_mmio_read_cached_pinned.argtypes = lib.pf_mmio_read_cached.argtypes
    lib.pf_mmio_read_pinned.argtypes = lib.pf_mmio_read.argtypes
    lib.pf_free.argtypes = [vp]
    lib.pf_free.restype = None
    lib.pf_shard_bounds_i32.argtypes = [vp, i64, C.c_int, vp]
    lib.pf_shard_bounds_i64.argtypes = [vp, i64, C.c_int, vp]
    sp = C.POINTER(pf_gen_spec)
    lib.pf_gen_resolve.argtypes = [sp]
    lib.pf_gen_count.argtypes = [sp, i64, i64, C.POINTER(i64)]
    lib.pf_gen_row_lengths_host.argtypes = [sp, i64, i64, vp]
    lib.pf_gen_rows_host.argtypes = [sp, i64, i64, vp, vp, vp]
    lib.pf_gen_x_host.argtypes = [sp, i64, i64, vp]
    lib.pf_gen_rows_device.argtypes = [sp, i64, i64, C.c_int, vp, vp, C.c_int, vp, vp]
    lib.pf_gen_x_device.argtypes = [sp, i64, i64, C.c_int, vp, vp]
    return lib


lib = _load()


def _check(status: int):
    if status != PF_OK:
        raise PfError(status, lib.pf_last_error().decode(errors="replace"))


def version() -> str:
    return lib.pf_version().decode()


def launch_count() -> int:
    """Kernels of this library launched since it was loaded (all devices)."""
    return int(lib.pf_launch_count())


def _ptr(a) -> int:
    """Raw address of a numpy array or torch tensor (None -> 0)."""
    if a is None:
        return 0
    if isinstance(a, np.ndarray):
        return a.ctypes.data
    return a.data_ptr()


# ---------------------------------------------------------------------------
# handles and the device-pointer core
# ---------------------------------------------------------------------------
class Handle:
    """Per-device scratch + error word (pf_handle). Create with the target CUDA
    device current; one handle per stream."""

    def __init__(self):
        h = C.c_void_p()
        _check(lib.pf_handle_create(C.byref(h)))
        self._h = h

    @property
    def ptr(self):
        return self._h

    def set_variant(self, v: int):
        _check(lib.pf_handle_set_variant(self._h, int(v)))

    def set_slice(self, nnz_per_cta: int):
        _check(lib.pf_handle_set_slice(self._h, int(nnz_per_cta)))

    def device_error(self, clear: bool = True) -> int:
        bits = C.c_uint32()
        _check(lib.pf_handle_device_error(self._h, C.byref(bits), int(clear)))
        return int(bits.value)

    def choice(self, m: int, nnz: int, row_ptr, value_bytes: int = 8, stream=None):
        """(variant name, lanes per row) this handle runs for the device
        CSR with this row_ptr (a torch tensor) and values of value_bytes
        bytes: the forced variant or the selector's cached choice."""
        import torch
        if stream is None:
            stream = torch.cuda.current_stream().cuda_stream
        elif hasattr(stream, "cuda_stream"):
            stream = stream.cuda_stream
        v, ln = C.c_int(), C.c_int()
        fn = lib.pf_handle_choice_i64 if row_ptr.element_size() == 8 else lib.pf_handle_choice_i32
        _check(fn(self._h, int(m), int(nnz), row_ptr.data_ptr(), int(value_bytes),
                  C.c_void_p(stream), C.byref(v), C.byref(ln)))
        return VARIANT_NAMES[v.value], int(ln.value)

    def dist_wait_ns(self, reset: bool = True) -> tuple[int, int]:
        """(nanoseconds the fused steps spent in their in-kernel step barrier,
        summed over CTAs and steps; CTAs of the last fused launch).
        Synchronizes the device."""
        v, g = C.c_uint64(), C.c_int64()
        _check(lib.pf_handle_dist_wait(self._h, C.byref(v), C.byref(g), int(reset)))
        return int(v.value), int(g.value)

    def close(self):
        if self._h:
            lib.pf_handle_destroy(self._h)
            self._h = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def _suffix(val_itemsize: int, idx_itemsize: int, val_dtype=None) -> str:
    if val_itemsize == 2:
        import torch
        v = "bf16" if val_dtype == torch.bfloat16 else "f16"
    else:
        v = {8: "f64", 4: "f32"}[val_itemsize]
    i = {4: "i32", 8: "i64"}[idx_itemsize]
    return f"{v}_{i}"


def spmv(handle: Handle, m: int, n: int, nnz: int, row_ptr, col, val, x, y,
         alpha: float = 1.0, beta: float = 0.0, stream=None):
    """y = alpha*A*x + beta*y on device tensors (torch CUDA tensors or raw
    integer addresses). Asynchronous on ``stream`` (torch stream, raw handle or
    None = torch's current stream)."""
    import torch
    if stream is None:
        stream = torch.cuda.current_stream().cuda_stream
    elif hasattr(stream, "cuda_stream"):
        stream = stream.cuda_stream
    vsz = val.element_size() if hasattr(val, "element_size") else 8
    isz = row_ptr.element_size() if hasattr(row_ptr, "element_size") else 4
    f = getattr(lib, "pf_spmv_" + _suffix(vsz, isz, getattr(val, "dtype", None)))
    _check(f(handle.ptr, int(m), int(n), int(nnz), _ptr(row_ptr), _ptr(col), _ptr(val),
             float(alpha), _ptr(x), float(beta), _ptr(y), C.c_void_p(stream)))


def spmm(handle: Handle, m: int, n: int, nnz: int, row_ptr, col, val, X, Y,
         alpha: float = 1.0, beta: float = 0.0, stream=None):
    """Y = alpha*A*X + beta*Y for k = X.shape[1] dense columns (torch CUDA
    tensors, X n x k and Y m x k, row-major with any row stride >= k)."""
    import torch
    if stream is None:
        stream = torch.cuda.current_stream().cuda_stream
    elif hasattr(stream, "cuda_stream"):
        stream = stream.cuda_stream
    k = int(X.shape[1])
    assert Y.shape[1] == k and X.stride(1) == 1 and Y.stride(1) == 1
    f = getattr(lib, "pf_spmm_" + _suffix(val.element_size(), row_ptr.element_size()))
    _check(f(handle.ptr, int(m), int(n), int(nnz), _ptr(row_ptr), _ptr(col), _ptr(val), k,
             float(alpha), _ptr(X), int(X.stride(0)), float(beta), _ptr(Y), int(Y.stride(0)),
             C.c_void_p(stream)))


def spmv_dist(handle: Handle, m: int, n: int, nnz: int, row_ptr, col, val, x, prev_slots,
              nranks: int, rank: int, out_ptrs_dev: int, slot_ptrs_dev: int, row_offset: int,
              stream=None, flag_ptrs_dev: int = 0, step: int = 0):
    """Fused multiply + all-gather step (see pf_spmv_dist_* in prefree_b200.h):
    this rank's rows of alpha*A*x go straight into every rank's next-x buffer
    (out_ptrs_dev: device array of nranks pointers), ||y||^2 into every rank's
    slot `rank` (slot_ptrs_dev); alpha = 1/sqrt(sum(prev_slots)). With
    flag_ptrs_dev the kernel also is the step barrier (step = 0, 1, ...)."""
    import torch
    if stream is None:
        stream = torch.cuda.current_stream().cuda_stream
    elif hasattr(stream, "cuda_stream"):
        stream = stream.cuda_stream
    f = lib.pf_spmv_dist_f64_i64 if row_ptr.element_size() == 8 else lib.pf_spmv_dist_f64_i32
    _check(f(handle.ptr, int(m), int(n), int(nnz), _ptr(row_ptr), _ptr(col), _ptr(val), _ptr(x),
             _ptr(prev_slots), int(nranks), int(rank), C.c_void_p(int(out_ptrs_dev)),
             C.c_void_p(int(slot_ptrs_dev)), int(row_offset),
             C.c_void_p(int(flag_ptrs_dev) or None), int(step), C.c_void_p(stream)))


def spmv_host(handle: Handle, row_ptr: np.ndarray, col: np.ndarray, val: np.ndarray,
              x: np.ndarray, y: np.ndarray, alpha: float = 1.0, beta: float = 0.0,
              stream: int = 0, m: int | None = None, n: int | None = None):
    """One multiply on host numpy arrays: copies in, multiplies, copies y out."""
    m = len(row_ptr) - 1 if m is None else m
    n = len(x) if n is None else n
    nnz = int(row_ptr[m]) - int(row_ptr[0])
    f = getattr(lib, "pf_spmv_host_" + _suffix(val.itemsize, row_ptr.itemsize))
    _check(f(handle.ptr, m, n, nnz, _ptr(row_ptr), _ptr(col), _ptr(val), float(alpha),
             _ptr(x), float(beta), _ptr(y), C.c_void_p(stream)))


def preFreeSpMV(csrVal: np.ndarray, csrRowPtr: np.ndarray, csrColInd: np.ndarray,
                X_val: np.ndarray, Y_val: np.ndarray, rowA: int, colA: int, nnzA: int):
    """The reference's entry point (include/PreFree.h:3-5) on numpy host arrays.
    Overwrites Y_val with A*X_val; returns (cdTime, cdPre) in ms."""
    t, p = C.c_double(), C.c_double()
    if csrRowPtr.dtype == np.int64:
        f = lib.pf_prefree_spmv_f64_i64
        assert csrVal.dtype == np.float64
    elif csrVal.dtype == np.float32:
        f = lib.pf_prefree_spmv_f32_i32
    else:
        f = lib.pf_prefree_spmv_f64_i32
    _check(f(_ptr(csrVal), _ptr(csrRowPtr), _ptr(csrColInd), _ptr(X_val), _ptr(Y_val),
             int(rowA), int(colA), int(nnzA), C.byref(t), C.byref(p)))
    return t.value, p.value


# ---------------------------------------------------------------------------
# Matrix Market input path and sharding
# ---------------------------------------------------------------------------
class _LibBuffer:
    """An array the library allocated (pf_mmio_read, pf_csr_read), exposed to
    numpy without a copy and handed back to pf_free when the last array that
    views it is gone."""

    def __init__(self, addr: int, n: int, typestr: str):
        self._addr = addr
        self.__array_interface__ = {"data": (addr, False), "shape": (n,),
                                    "typestr": typestr, "version": 3}

    def __del__(self):
        addr, self._addr = self._addr, None
        if addr:
            try:
                lib.pf_free(addr)
            except Exception:  # interpreter shutdown: the process frees it
                pass


def _owned_array(ptr: C.c_void_p, n: int, dtype) -> np.ndarray:
    addr = ptr.value
    if not addr or n == 0:
        if addr:
            lib.pf_free(addr)
        return np.empty(n, dtype=dtype)
    return np.asarray(_LibBuffer(addr, n, np.dtype(dtype).str))


def _take_csr(m, n, z, sym, rp, ci, va):
    """The CSR arrays a library call returned, as numpy arrays that own them
    (no copy: a copy of a large fresh array can cost seconds of page faults)."""
    bufs = [(rp, m.value + 1, np.int64), (ci, z.value, np.int32), (va, z.value, np.float64)]
    out = []
    try:
        for ptr, cnt, dt in bufs:
            out.append(_owned_array(ptr, cnt, dt))
            ptr.value = None
    finally:
        for ptr, _, _ in bufs:
            if ptr.value:
                lib.pf_free(ptr.value)
    row_ptr, col, val = out
    return m.value, n.value, z.value, bool(sym.value), row_ptr, col, val


def _csr_out():
    return (C.c_int64(), C.c_int64(), C.c_int64(), C.c_int(), C.c_void_p(), C.c_void_p(),
            C.c_void_p())


def mmio_read(path: str, pinned: bool = False):
    """Matrix Market -> CSR (mmio_allinone semantics). Returns
    (m, n, nnz, is_symmetric, row_ptr int64[m+1], col int32[nnz], val f64[nnz]).
    pinned: the arrays live in page-locked host memory (full-speed copies to
    the device, e.g. by spmv_host)."""
    o = _csr_out()
    f = lib.pf_mmio_read_pinned if pinned else lib.pf_mmio_read
    _check(f(os.fsencode(path), *[C.byref(v) for v in o]))
    return _take_csr(*o)


def csr_write(path: str, m: int, n: int, row_ptr, col, val, is_symmetric: bool = False):
    """Store a CSR (int64 row_ptr, int32 col, f64 val) in the binary cache format."""
    rp = np.ascontiguousarray(row_ptr, dtype=np.int64)
    ci = np.ascontiguousarray(col, dtype=np.int32)
    va = np.ascontiguousarray(val, dtype=np.float64)
    _check(lib.pf_csr_write(os.fsencode(path), int(m), int(n), len(ci), int(is_symmetric),
                            rp.ctypes.data, ci.ctypes.data, va.ctypes.data))


def csr_read(path: str):
    """Load a binary CSR cache file; same return value as mmio_read."""
    o = _csr_out()
    _check(lib.pf_csr_read(os.fsencode(path), *[C.byref(v) for v in o]))
    return _take_csr(*o)


def mmio_read_cached(mtx_path: str, cache_path: str, pinned: bool = False):
    """mmio_read through a binary cache: returns (csr tuple, from_cache)."""
    o = _csr_out()
    fc = C.c_int()
    f = lib.pf_mmio_read_cached_pinned if pinned else lib.pf_mmio_read_cached
    _check(f(os.fsencode(mtx_path), os.fsencode(cache_path), *[C.byref(v) for v in o],
             C.byref(fc)))
    return _take_csr(*o), bool(fc.value)


def shard_bounds(row_ptr: np.ndarray, parts: int) -> np.ndarray:
    """Equal-nnz row split: bounds[k] = first row at or after k*nnz/parts."""
    m = len(row_ptr) - 1
    out = np.zeros(parts + 1, dtype=np.int64)
    rp = np.ascontiguousarray(row_ptr)
    f = lib.pf_shard_bounds_i64 if rp.dtype == np.int64 else lib.pf_shard_bounds_i32
    _check(f(_ptr(rp), m, int(parts), _ptr(out)))
    return out


# ---------------------------------------------------------------------------
# synthetic inputs
# ---------------------------------------------------------------------------
@dataclass
class GenSpec:
    cfg: int
    seed: int = 12345
    value_mode: int = 0
    m: int = 0
    n: int = 0
    k: int = 0

    def c(self) -> pf_gen_spec:
        s = pf_gen_spec(self.cfg, self.value_mode, self.seed, self.m, self.n, self.k)
        _check(lib.pf_gen_resolve(C.byref(s)))
        return s

    def resolved(self) -> "GenSpec":
        s = self.c()
        return GenSpec(s.cfg, s.seed, s.value_mode, s.m, s.n, s.k)


def gen_count(spec: GenSpec, r0: int = 0, r1: int | None = None) -> int:
    s = spec.c()
    r1 = s.m if r1 is None else r1
    out = C.c_int64()
    _check(lib.pf_gen_count(C.byref(s), r0, r1, C.byref(out)))
    return out.value


def gen_rows_host(spec: GenSpec, r0: int = 0, r1: int | None = None):
    """Rows [r0, r1) on the host: (row_ptr int64 starting at 0, col int32, val f64)."""
    s = spec.c()
    r1 = s.m if r1 is None else r1
    z = gen_count(spec, r0, r1)
    rp = np.zeros(r1 - r0 + 1, dtype=np.int64)
    col = np.zeros(max(z, 1), dtype=np.int32)
    val = np.zeros(max(z, 1), dtype=np.float64)
    _check(lib.pf_gen_rows_host(C.byref(s), r0, r1, _ptr(rp), _ptr(col), _ptr(val)))
    return rp, col[:z], val[:z]


def gen_x_host(spec: GenSpec, c0: int = 0, c1: int | None = None) -> np.ndarray:
    s = spec.c()
    c1 = s.n if c1 is None else c1
    x = np.zeros(max(c1 - c0, 1), dtype=np.float64)
    _check(lib.pf_gen_x_host(C.byref(s), c0, c1, _ptr(x)))
    return x[:c1 - c0]


def gen_rows_device(spec: GenSpec, r0: int = 0, r1: int | None = None, index_dtype=None,
                    value_dtype=None, device=None):
    """Rows [r0, r1) generated on the current CUDA device: torch tensors
    (row_ptr rebased to 0, col int32, val)."""
    import torch
    index_dtype = index_dtype or torch.int32
    value_dtype = value_dtype or torch.float64
    s = spec.c()
    r1 = s.m if r1 is None else r1
    z = gen_count(spec, r0, r1)
    dev = device or torch.device("cuda", torch.cuda.current_device())
    rp = torch.empty(r1 - r0 + 1, dtype=index_dtype, device=dev)
    col = torch.empty(max(z, 1), dtype=torch.int32, device=dev)
    val = torch.empty(max(z, 1), dtype=value_dtype, device=dev)
    stream = torch.cuda.current_stream(dev).cuda_stream
    _check(lib.pf_gen_rows_device(C.byref(s), r0, r1, rp.element_size(), _ptr(rp), _ptr(col),
                                  val.element_size(), _ptr(val), C.c_void_p(stream)))
    return rp, col[:z], val[:z]


def gen_x_device(spec: GenSpec, c0: int = 0, c1: int | None = None, value_dtype=None,
                 device=None):
    import torch
    value_dtype = value_dtype or torch.float64
    s = spec.c()
    c1 = s.n if c1 is None else c1
    dev = device or torch.device("cuda", torch.cuda.current_device())
    x = torch.empty(max(c1 - c0, 1), dtype=value_dtype, device=dev)
    stream = torch.cuda.current_stream(dev).cuda_stream
    _check(lib.pf_gen_x_device(C.byref(s), c0, c1, x.element_size(), _ptr(x),
                               C.c_void_p(stream)))
    return x[:c1 - c0]


def compulsory_bytes(m: int, n: int, nnz: int, val_bytes: int, idx_bytes: int,
                     beta_nonzero: bool = False) -> int:
    """Algorithmic bytes of one multiply: nnz*(V+4) + (m+1)*R + n*V + m*V
    (+ m*V when y is read), the reference's data_origin1
    (test/test_cdspmv.cpp:305) generalised to the index/value widths."""
    b = nnz * (val_bytes + 4) + (m + 1) * idx_bytes + n * val_bytes + m * val_bytes
    if beta_nonzero:
        b += m * val_bytes
    return b
