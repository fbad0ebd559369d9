"""Row-sharded iterated multiply on GPUs: the fused multiply + all-gather
(pf_spmv_dist_*: rows stored straight into every rank's next x, ||y||^2
reduced in the kernel) against the unfused path (pf_spmv + NCCL all-gather)
and against the CPU oracle's power iteration. The multi-GPU cases spawn one
NCCL rank per GPU and are skipped when fewer GPUs are visible."""
import os
import socket
import sys

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
STEPS = 5


def small_spec(pf, cfg=5):
    """Config 5 (banded + uniform, equal shards) or config 3 (power-law rows:
    equal-nnz shards of unequal row counts) at 2^15 rows."""
    return pf.GenSpec(cfg=cfg, seed=77, m=1 << 15, n=1 << 15)


def oracle_iterates(pf, oracle, spec, steps):
    rp, col, val = pf.gen_rows_host(spec)
    x = pf.gen_x_host(spec)
    norms = []
    alpha = 1.0 / np.sqrt(x @ x)
    for _ in range(steps):
        y = alpha * oracle.serial(rp, col, val, x)
        nsq = float(y @ y)
        norms.append(nsq)
        x, alpha = y, 1.0 / np.sqrt(nsq)
    return x, norms


def close(a, b, tol=1e-12):
    return np.abs(a - b).max() <= tol * np.abs(b).max()


def test_fused_one_gpu_matches_unfused_and_oracle(pf, oracle):
    import torch
    import importlib
    pfd = importlib.import_module("prefree-public_b200.dist")
    spec = small_spec(pf).resolved()
    rp, col, val = pf.gen_rows_device(spec, index_dtype=torch.int64)
    x0 = pf.gen_x_device(spec)
    bounds = np.array([0, spec.m])
    h = pf.Handle()
    fused = pfd.FusedPowerIteration(pf, h, rp, col, val, x0, bounds, 0, 1)
    nf = []
    for _ in range(STEPS):
        fused.step()
        nf.append(fused.norm_sq())
    y = torch.empty(spec.m, dtype=torch.float64, device="cuda")
    x = x0.clone()

    def local(xf, yl, alpha):
        pf.spmv(h, spec.m, spec.n, col.numel(), rp, col, val, xf, yl, alpha, 0.0)

    plain = pfd.PowerIteration(local, x, y, bounds, 0, 1)
    nu = [plain.step().norm_sq for _ in range(STEPS)]
    assert h.device_error() == 0
    xr, nr = oracle_iterates(pf, oracle, spec, STEPS)
    assert close(fused.x.cpu().numpy(), xr) and close(x.cpu().numpy(), xr)
    assert np.allclose(nf, nr, rtol=1e-12) and np.allclose(nu, nr, rtol=1e-12)
    # the fused kernel is deterministic
    again = pfd.FusedPowerIteration(pf, h, rp, col, val, x0, bounds, 0, 1)
    for _ in range(STEPS):
        again.step()
    assert torch.equal(again.x, fused.x)
    h.close()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, q, cfg=5, index_bits=64):
    sys.path.insert(0, ROOT)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world), NCCL_NVLS_ENABLE="0")
    import importlib
    from datetime import timedelta
    import torch
    import torch.distributed as dist
    try:
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
        pf = importlib.import_module("prefree-public_b200")
        pfd = importlib.import_module("prefree-public_b200.dist")
        spec = small_spec(pf, cfg).resolved()
        b = pfd.gen_bounds(pf, spec, world)
        r0, r1 = int(b[rank]), int(b[rank + 1])
        idt = torch.int64 if index_bits == 64 else torch.int32
        rp, col, val = pf.gen_rows_device(spec, r0, r1, index_dtype=idt, device=dev)
        x0 = pf.gen_x_device(spec, device=dev)
        h = pf.Handle()
        fused = pfd.FusedPowerIteration(pf, h, rp, col, val, x0, b, rank, world)
        nf = []
        for _ in range(STEPS):
            fused.step()
            nf.append(fused.norm_sq())
        x = x0.clone()
        y = torch.empty(r1 - r0, dtype=torch.float64, device=dev)

        def local(xf, yl, alpha):
            pf.spmv(h, r1 - r0, spec.n, col.numel(), rp, col, val, xf, yl, alpha, 0.0)

        plain = pfd.PowerIteration(local, x, y, b, rank, world)
        nu = [plain.step().norm_sq for _ in range(STEPS)]
        torch.cuda.synchronize()
        q.put((rank, "ok", fused.x.cpu().numpy(), x.cpu().numpy(), nf, nu, h.device_error()))
        del fused
        dist.barrier()
        dist.destroy_process_group()
    except Exception as e:  # noqa: BLE001
        q.put((rank, "error", repr(e), None, None, None, None))


@pytest.mark.parametrize("world,cfg,index_bits", [(2, 5, 64), (2, 3, 32), (4, 3, 32),
                                                  (4, 5, 64)])
def test_multi_gpu_fused_and_nccl_match_oracle(pf, oracle, world, cfg, index_bits):
    """world ranks, one per GPU (spawned NCCL processes, NVLS off): the fused
    step and the NCCL path both reproduce the CPU oracle's power iteration.
    Config 3 gives equal-nnz shards of unequal row counts (the NCCL path then
    all-gathers through broadcasts) and runs the int32 row_ptr kernels."""
    import torch
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_rank_main, args=(r, world, port, q, cfg, index_bits))
          for r in range(world)]
    [p.start() for p in ps]
    res = sorted([q.get(timeout=300) for _ in range(world)], key=lambda r: r[0])
    [p.join(timeout=60) for p in ps]
    for p in ps:
        if p.is_alive():
            p.kill()
    assert all(r[1] == "ok" for r in res), res
    xr, nr = oracle_iterates(pf, oracle, small_spec(pf, cfg), STEPS)
    for rank, _, xf, xu, nf, nu, err in res:
        assert err == 0
        assert close(xf, xr) and close(xu, xr), rank
        assert np.allclose(nf, nr, rtol=1e-12) and np.allclose(nu, nr, rtol=1e-12)
    for r in res[1:]:
        assert np.array_equal(res[0][2], r[2])       # every rank holds the same x


def test_step_barrier_times_out_without_peer(pf):
    """The fused step's in-kernel barrier waits for every rank's previous step
    with a bound: a step counter that nothing sets makes the kernel give up
    after ~1 s, flag PF_DEVERR_WAIT_TIMEOUT and still finish (announcing its
    own step). One GPU: the "second rank" is only memory here, no kernel of
    it runs, so nothing waits on this kernel."""
    import time
    import torch
    spec = small_spec(pf).resolved()
    rp, col, val = pf.gen_rows_device(spec, index_dtype=torch.int64)
    x = pf.gen_x_device(spec)
    m, n = spec.m, spec.n
    outs = [torch.zeros(n, dtype=torch.float64, device="cuda") for _ in range(2)]
    slots = [torch.zeros(64, dtype=torch.float64, device="cuda") for _ in range(2)]
    flags = [torch.zeros(64, dtype=torch.int64, device="cuda") for _ in range(2)]
    prev = torch.zeros(64, dtype=torch.float64, device="cuda")
    prev[0] = float(x.dot(x))
    ptrs = lambda ts: torch.tensor([t.data_ptr() for t in ts], dtype=torch.int64, device="cuda")
    out_p, slot_p, flag_p = ptrs(outs), ptrs(slots), ptrs(flags)
    h = pf.Handle()
    t0 = time.time()
    pf.spmv_dist(h, m, n, col.numel(), rp, col, val, x, prev, 2, 0, out_p.data_ptr(),
                 slot_p.data_ptr(), 0, flag_ptrs_dev=flag_p.data_ptr(), step=1)
    torch.cuda.synchronize()
    waited = time.time() - t0
    bits = h.device_error()
    # the barrier-wait diagnostic saw every CTA wait about the 1 s bound
    wait_ns, ctas = h.dist_wait_ns(reset=True)
    assert ctas > 0 and 0.5e9 < wait_ns / ctas < 30e9, (wait_ns, ctas)
    assert h.dist_wait_ns()[0] == 0  # reset
    h.close()
    assert bits & 1, f"expected the wait-timeout bit, got {bits:#x}"
    assert 0.5 < waited < 30
    # the step still ran and announced step 2 on both ranks' counters
    assert int(flags[0][0]) == 2 and int(flags[1][0]) == 2
    assert float(slots[0][0]) > 0 and float(slots[1][0]) == float(slots[0][0])
