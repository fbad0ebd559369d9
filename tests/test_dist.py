"""Row-sharded power iteration on world_size-2 gloo ranks (CPU): the same
PowerIteration code the GPU bench runs over NCCL, with the CPU oracle as the
local multiply. Also: a rank that fails mid-run makes the other rank's next
collective end with an error within the process-group timeout (no hang)."""
import os
import socket
import sys

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _spec(cfg):
    import importlib
    pf = importlib.import_module("prefree-public_b200")
    if cfg == 3:
        return pf, pf.GenSpec(cfg=3, seed=17, m=6000)
    return pf, pf.GenSpec(cfg=5, seed=17, m=4096, n=4096)


def reference_iterates(cfg, steps):
    sys.path.insert(0, ROOT)
    import oracle
    pf, spec = _spec(cfg)
    rp, col, val = pf.gen_rows_host(spec)
    x = pf.gen_x_host(spec)
    norms = []
    alpha = 1.0 / np.sqrt(x @ x)
    for _ in range(steps):
        y = alpha * oracle.serial(rp, col, val, x)
        nsq = float(y @ y)
        norms.append(nsq)
        x = y
        alpha = 1.0 / np.sqrt(nsq)
    return x, norms


def worker(rank, world, port, cfg, steps, out, fail_rank):
    sys.path.insert(0, ROOT)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    from datetime import timedelta
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=10))
    import importlib
    import oracle
    pfd = importlib.import_module("prefree-public_b200.dist")
    pf, spec = _spec(cfg)
    b = pfd.gen_bounds(pf, spec, world)
    r0, r1 = int(b[rank]), int(b[rank + 1])
    rp, col, val = pf.gen_rows_host(spec, r0, r1)
    x = torch.from_numpy(pf.gen_x_host(spec).copy())
    y = torch.zeros(r1 - r0, dtype=torch.float64)

    def local(xf, yl, alpha):
        yl.copy_(torch.from_numpy(alpha * oracle.serial(rp, col, val, xf.numpy())))

    it = pfd.PowerIteration(local, x, y, b, rank, world)
    norms = []
    try:
        for s in range(steps):
            if rank == fail_rank and s == 1:
                raise RuntimeError("planted failure on this rank")
            norms.append(it.step().norm_sq)
        out.put((rank, "ok", norms, x.numpy().copy(), [int(v) for v in b]))
    except Exception as e:  # noqa: BLE001
        out.put((rank, "error", repr(e), None, None))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:  # noqa: BLE001
            pass


def run(world, cfg, steps, fail_rank=-1):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    ps = [ctx.Process(target=worker, args=(r, world, port, cfg, steps, q, fail_rank))
          for r in range(world)]
    [p.start() for p in ps]
    res = [q.get(timeout=120) for _ in range(world)]
    [p.join(timeout=60) for p in ps]
    for p in ps:
        if p.is_alive():
            p.kill()
    return sorted(res, key=lambda r: r[0])


@pytest.mark.parametrize("cfg", [5, 3])
def test_two_rank_power_iteration_matches_single(cfg):
    steps = 4
    res = run(2, cfg, steps)
    assert all(r[1] == "ok" for r in res), res
    x_ref, n_ref = reference_iterates(cfg, steps)
    for rank, _, norms, x, b in res:
        # same serial loop per row; only ||y||^2 is summed in a different
        # order (per shard, then all-reduce), so agreement is to rounding
        scale = np.abs(x_ref).max()
        assert np.abs(x - x_ref).max() <= 1e-13 * scale
        assert np.allclose(norms, n_ref, rtol=1e-13)
    if cfg == 3:
        b = res[0][4]
        assert b[1] not in (0, b[2])                 # uneven rows, equal nnz


def test_failing_rank_surfaces_as_error_not_hang():
    res = run(2, 5, 3, fail_rank=1)
    assert res[1][1] == "error" and "planted" in res[1][2]
    assert res[0][1] == "error"                      # the survivor's collective failed
