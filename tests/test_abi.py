"""The C-ABI library: loads, exports every symbol include/*.h declares (and
the C++ drop-in symbols), and its host-only calls behave (no GPU needed)."""
import ctypes as C
import os
import re
import subprocess

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_c_functions():
    names = set()
    for h in ("prefree_b200.h",):
        text = open(os.path.join(ROOT, "include", h)).read()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        for m in re.finditer(r"\b(?:pf_status|void|const char \*|uint64_t)\s+(pf_\w+)\s*\(", text):
            names.add(m.group(1))
    return sorted(names)


def test_every_declared_symbol_is_exported(pf):
    out = subprocess.run(["nm", "-D", "--defined-only", pf.LIB_PATH], capture_output=True,
                         text=True, check=True).stdout
    exported = {l.split()[-1] for l in out.splitlines() if l.strip()}
    decl = declared_c_functions()
    assert len(decl) >= 25
    missing = [s for s in decl if s not in exported]
    assert not missing, missing
    for s in pf.CXX_EXPORTED:
        assert s in exported, s
    assert set(decl) <= set(pf.EXPORTED)


def test_cxx_symbol_demangles_to_reference_signature(pf):
    out = subprocess.run(["c++filt", "_Z11preFreeSpMVPdPiS0_S_S_iiiS_S_"], capture_output=True,
                         text=True).stdout.strip()
    assert out == "preFreeSpMV(double*, int*, int*, double*, double*, int, int, int, double*, double*)"


def test_version_and_errors(pf):
    assert "sm_100a" in pf.version()
    with pytest.raises(pf.PfError) as e:
        pf.mmio_read("/nonexistent/file.mtx")
    assert e.value.status == 5
    assert b"cannot open" in pf.lib.pf_last_error()


def test_handle_without_gpu_reports_error(pf):
    import torch
    if torch.cuda.is_available():
        pytest.skip("GPU present")
    h = C.c_void_p()
    st = pf.lib.pf_handle_create(C.byref(h))
    assert st == 2                        # PF_ERR_CUDA, no crash
    assert pf.lib.pf_last_error()


def test_null_and_bad_arguments(pf):
    # argument checks run before any CUDA call
    st = pf.lib.pf_spmv_f64_i32(None, 1, 1, 0, None, None, None, 1.0, None, 0.0, None, None)
    assert st == 1
    b = np.zeros(3, dtype=np.int64)
    assert pf.lib.pf_shard_bounds_i64(None, 2, 2, b.ctypes.data) == 1
    s = pf.pf_gen_spec(9, 0, 1, 0, 0, 0)
    assert pf.lib.pf_gen_resolve(C.byref(s)) == 1


def test_shard_bounds(pf):
    rp = np.array([0, 5, 5, 9, 20, 21, 30], dtype=np.int64)
    b = pf.shard_bounds(rp, 3)
    assert b[0] == 0 and b[-1] == 6 and np.all(np.diff(b) >= 0)
    # bounds[k] = first row starting at or after k*nnz/parts
    for k in range(1, 3):
        assert rp[b[k]] >= 30 * k // 3 and (b[k] == 0 or rp[b[k] - 1] < 30 * k // 3)
    assert np.array_equal(pf.shard_bounds(rp.astype(np.int32), 3), b)


def test_invalid_arguments_return_status_not_crash(pf):
    """Argument checks run on the host before any device work: a null handle,
    negative sizes or a bad variant return PF_ERR_INVALID (1) with a message,
    as the reference's callers would otherwise meet an exit() or a fault."""
    lib = pf.lib
    null = C.c_void_p()
    assert lib.pf_spmv_f64_i32(null, 4, 4, 0, None, None, None, 1.0, None, 0.0, None, None) == 1
    assert b"null handle" in lib.pf_last_error()
    assert lib.pf_spmv_f16_i64(null, 4, 4, 0, None, None, None, 1.0, None, 0.0, None, None) == 1
    assert lib.pf_spmm_f64_i32(null, 4, 4, 0, None, None, None, 2, 1.0, None, 2, 0.0, None, 2,
                               None) == 1
    assert lib.pf_handle_set_variant(null, 0) == 1
    v, ln = C.c_int(), C.c_int()
    assert lib.pf_handle_choice_i32(null, 4, 4, None, 8, None, C.byref(v), C.byref(ln)) == 1
    assert lib.pf_handle_choice_i64(null, 4, 4, None, 8, None, C.byref(v), C.byref(ln)) == 1
    assert lib.pf_spmv_dist_f64_i64(null, 4, 4, 4, None, None, None, None, None, 1, 0, None,
                                    None, 0, None, 0, None) == 1
    t, p = C.c_double(), C.c_double()
    assert lib.pf_prefree_spmv_f64_i32(None, None, None, None, None, -1, 4, 0,
                                       C.byref(t), C.byref(p)) == 1
    assert b"negative" in lib.pf_last_error()


def test_shard_bounds_equal_nnz(pf):
    rp = np.array([0, 3, 3, 10, 11, 20], dtype=np.int64)
    b = pf.shard_bounds(rp, 3)
    assert b[0] == 0 and b[-1] == 5 and list(b) == sorted(b)
    # every boundary is the first row whose start reaches k * nnz / parts
    for k in range(1, 3):
        assert b[k] == int(np.searchsorted(rp, k * 20 // 3))


def _build_and_run(tmp_path, pf, src_name, source, compiler, flags):
    src = tmp_path / src_name
    src.write_text(source)
    exe = tmp_path / (src_name + ".out")
    lib_dir = os.path.dirname(pf.LIB_PATH)
    cuda_lib = "/usr/local/cuda/lib64"
    cmd = [compiler, *flags, "-I", os.path.join(ROOT, "include"), str(src), pf.LIB_PATH,
           f"-Wl,-rpath,{lib_dir}", f"-Wl,-rpath-link,{cuda_lib}", "-o", str(exe)]
    subprocess.run(cmd, check=True, capture_output=True, text=True)
    return subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout


def test_c_header_compiles_as_c99_and_links(pf, tmp_path):
    """A C caller (or an FFI generator reading the header as C) sees every
    entry point: the header compiles as strict C99 with warnings as errors,
    each declared function links against the library, and a host-only call
    runs without a GPU."""
    names = declared_c_functions()
    body = ",\n  ".join(f"(fn){n}" for n in names)
    source = (
        "#include <stdio.h>\n#include \"prefree_b200.h\"\n"
        "typedef void (*fn)(void);\n"
        f"static const fn all[] = {{\n  {body}\n}};\n"
        "int main(void) {\n"
        "  printf(\"%s %u\\n\", pf_version(), (unsigned)(sizeof(all) / sizeof(all[0])));\n"
        "  return 0;\n}\n")
    out = _build_and_run(tmp_path, pf, "abi_c.c", source, "gcc",
                         ["-std=c99", "-Wall", "-Wextra", "-Werror", "-Wno-cast-function-type"])
    assert "sm_100a" in out
    assert out.split()[-1] == str(len(names))


def test_cxx_drop_in_header_links(pf, tmp_path):
    """The C++ harness's view: include/PreFree.h declares the reference's
    preFreeSpMV, which resolves against the library (same mangled name)."""
    source = (
        "#include <cstdio>\n#include \"PreFree.h\"\n#include \"prefree_b200.h\"\n"
        "int main() {\n"
        "  void (*f)(double *, int *, int *, double *, double *, int, int, int, double *,\n"
        "            double *) = &preFreeSpMV;\n"
        "  std::printf(\"%s %d\\n\", pf_version(), f != nullptr);\n"
        "  return 0;\n}\n")
    out = _build_and_run(tmp_path, pf, "abi_cxx.cpp", source, "g++",
                         ["-std=c++17", "-Wall", "-Wextra", "-Werror"])
    assert "sm_100a" in out and out.split()[-1] == "1"
