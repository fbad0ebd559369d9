"""The reference's own GPU path and this library's, timed on the same B200.

Run on a GPU machine (not collected by pytest):

    python tests/reference_gpu_timing.py [--configs 1,2,3,4] [--md OUT.md]

A third column times the vendor library on the same device arrays: cuSPARSE
CSR SpMV through torch's sparse CSR matmul (the comparison the reference's
harness runs, test/test_cdspmv.cpp:155-267), 200 warm-up + 4000 back-to-back
calls replayed from a CUDA graph, checked against the same oracle.

Both sides are the same drop-in call, preFreeSpMV (include/PreFree.h:3-5),
on the same host CSR (fp64 values, int32 indices; synthetic configs 1-4 from
the seeded generator): oracle/_ref/libref_gpu.so is the reference's
src/spmv_kernel/preFreeSpMV.cu compiled unmodified for sm_100a, and each side
reports its own cdTime, the mean of 4000 back-to-back launches after 200
warm-ups with L2 warm (src/spmv_kernel/preFreeSpMV.cu:604-650). Each result is
checked against the reference's CPU spmv_serial with the north-star tolerance
(per row |y - y_ref| <= 1e-12 * sum_j |a_ij x_j|). Config 5 does not fit the
reference's int nnz. Prints one JSON line per config and, with --md, a table.
"""
import argparse
import importlib
import json
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)


def cusparse_ms(torch, oracle, rp, col, val, x, y_cpu, a, comp, warm=200, iters=4000):
    """cuSPARSE CSR SpMV (torch sparse CSR x dense vector) on the device."""
    A = torch.sparse_csr_tensor(torch.from_numpy(rp.astype(np.int64)).cuda(),
                                torch.from_numpy(col.astype(np.int64)).cuda(),
                                torch.from_numpy(val).cuda(), size=(len(rp) - 1, len(x)))
    xv = torch.from_numpy(x).cuda().unsqueeze(1)
    y = torch.empty(len(rp) - 1, 1, dtype=torch.float64, device="cuda")
    for _ in range(3):
        torch.matmul(A, xv, out=y)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    g = None
    try:  # replayed from a graph when the library call can be captured
        s = torch.cuda.Stream()
        with torch.cuda.stream(s):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=s):
                for _ in range(100):
                    torch.matmul(A, xv, out=y)
        for _ in range(max(1, warm // 100)):
            g.replay()
        torch.cuda.synchronize()
        e0.record()
        for _ in range(iters // 100):
            g.replay()
        e1.record()
    except RuntimeError:
        g = None
        torch.cuda.synchronize()
        for _ in range(warm):
            torch.matmul(A, xv, out=y)
        e0.record()
        for _ in range(iters // 100 * 100):
            torch.matmul(A, xv, out=y)
        e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / (iters // 100 * 100)
    _, _, bad = oracle.tolerance_report(y.squeeze(1).cpu().numpy(), y_cpu, a, 1e-12, y_comp=comp)
    del g, A, xv, y
    torch.cuda.empty_cache()
    return ms, bad


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--configs", default="1,2,3,4")
    ap.add_argument("--seed", type=int, default=12345)
    ap.add_argument("--md", default=None)
    args = ap.parse_args()
    import torch
    import oracle
    pf = importlib.import_module("prefree-public_b200")
    rows = []
    for cfg in [int(c) for c in args.configs.split(",")]:
        spec = pf.GenSpec(cfg=cfg, seed=args.seed).resolved()
        d_rp, d_col, d_val = pf.gen_rows_device(spec, index_dtype=torch.int32)
        rp = d_rp.cpu().numpy()
        col = d_col.cpu().numpy()
        val = d_val.cpu().numpy()
        x = pf.gen_x_device(spec).cpu().numpy()
        del d_rp, d_col, d_val
        torch.cuda.empty_cache()
        m, n, nnz = spec.m, spec.n, len(col)
        y_cpu = oracle.ref_serial(rp, col, val, x)
        a, comp = oracle.abs_comp(rp, col, val, x)

        y = np.full(m, np.nan)
        t_ours, _ = pf.preFreeSpMV(val, rp, col, x, y, m, n, nnz)
        ok_ours, _, bad_ours = oracle.tolerance_report(y, y_cpu, a, 1e-12, y_comp=comp)
        y_ref, t_ref, t_pre = oracle.ref_gpu_prefree(val, rp, col, x, m, n)
        ok_ref, _, bad_ref = oracle.tolerance_report(y_ref, y_cpu, a, 1e-12, y_comp=comp)

        t_cs, bad_cs = cusparse_ms(torch, oracle, rp, col, val, x, y_cpu, a, comp)
        B = pf.compulsory_bytes(m, n, nnz, 8, 4)
        row = {"config": cfg, "m": m, "nnz": nnz, "alg_bytes": B,
               "ref_gpu_ms": t_ref, "ref_prepass_ms": t_pre, "ours_ms": t_ours,
               "speedup": t_ref / t_ours,
               "ref_gpu_GBps": B / t_ref / 1e6, "ours_GBps": B / t_ours / 1e6,
               "cusparse_ms": t_cs, "cusparse_rows_out_of_tol": int(bad_cs),
               "ref_gpu_rows_out_of_tol": int(bad_ref), "ours_rows_out_of_tol": int(bad_ours),
               "ours_ok": bool(ok_ours), "ref_ok": bool(ok_ref)}
        print(json.dumps(row), flush=True)
        rows.append(row)
    if args.md:
        with open(args.md, "w") as f:
            f.write("| config | nnz | reference GPU ms | + its pre-pass ms | ours ms | cuSPARSE ms "
                    "| ours vs reference | reference GB/s | ours GB/s | rows out of tolerance "
                    "(reference / ours / cuSPARSE) |\n|---|---|---|---|---|---|---|---|---|---|\n")
            for r in rows:
                f.write(f"| C{r['config']} | {r['nnz']:,} | {r['ref_gpu_ms']:.4f} | "
                        f"{r['ref_prepass_ms']:.4f} | {r['ours_ms']:.4f} | {r['cusparse_ms']:.4f} | "
                        f"{r['speedup']:.2f}x | {r['ref_gpu_GBps']:.0f} | {r['ours_GBps']:.0f} | "
                        f"{r['ref_gpu_rows_out_of_tol']} / {r['ours_rows_out_of_tol']} / "
                        f"{r['cusparse_rows_out_of_tol']} |\n")


if __name__ == "__main__":
    main()
