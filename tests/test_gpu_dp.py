"""The fused data-parallel exchange (ffn_dp_reduce_apply: gradient sum across ranks, table SGD on
each rank's shard, broadcast of the updated table) against the NCCL path (all-reduce of the
gradient buffer, then the table pass), on 2 GPUs, in both forms: NVLink peer loads/stores ("p2p")
and NVSwitch multicast ("nvls": multimem.ld_reduce / multimem.st on symmetric memory; skipped
where the switch offers no multicast).

Each rank holds two identical contexts and trains both for 3 steps on its half of the batch: one
through NCCL + ffn_apply_updates, one through ffn_dp_reduce_apply + ffn_apply_updates(TABLE_APPLIED).
Contracts: the table and parameter updates of the two paths agree within rel-L2 1e-4 on every rank
(the one-step gradient tolerance: the two contexts' table gradients differ in the order of their
float atomic adds, and the cross-rank sums in summation order); both ranks end with the same
table; the gradient buffers are clear; the status word stays 0.  Needs 2 GPUs (skipped otherwise).
"""
import os
import socket
import sys
from pathlib import Path

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parents[1]


def _port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, mode, q):
    try:
        for p in (ROOT / "ffnerf-experimental_b200", ROOT / "tests"):
            sys.path.insert(0, str(p))
        import datetime
        import torch.distributed as dist
        import ffn_native as fn
        from _helpers import init_blob, init_occ, init_table, rays_toward_box, rel_l2, targets
        from ffn_config import make_geometry
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        torch.cuda.set_device(rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                                device_id=torch.device("cuda", rank))
        g = make_geometry(F=2, ND=1, NC=2, spr=64, G=64, log2_entries=14, rmax=512.0)
        blob, table, occ = init_blob(g, 4), init_table(g, 4), init_occ(g, 4)
        ctxs = []
        for prec in ("fp16", "fp16"):
            c = fn.Context(g, device=rank, mlp_precision=prec)
            c.tensor(fn.BUF_PARAMS).copy_(torch.from_numpy(blob))
            c.tensor(fn.BUF_TABLE).copy_(torch.from_numpy(table))
            c.tensor(fn.BUF_OCC_IN).copy_(torch.from_numpy(occ.view(np.int32)))
            c.tensor(fn.BUF_OCC_ST).copy_(torch.from_numpy(occ.view(np.int32)))
            ctxs.append(c)
        nccl_ctx, fused_ctx = ctxs
        mc = None
        if mode == "nvls":
            import torch.distributed._symmetric_memory as symm_mem
            bufs = []
            for bid in (fn.BUF_GRADS, fn.BUF_TABLE):
                t = symm_mem.empty(fused_ctx.tensor(bid).numel(), dtype=torch.float32, device=f"cuda:{rank}")
                bufs.append((t, symm_mem.rendezvous(t, dist.group.WORLD.group_name)))
            good = torch.tensor([int(all(int(getattr(h, "multicast_ptr", 0) or 0) != 0 for _, h in bufs))], device="cuda")
            dist.all_reduce(good, op=dist.ReduceOp.MIN)
            if int(good.item()) == 0:
                dist.barrier()
                dist.destroy_process_group()
                q.put((rank, "skip", "no multicast support"))
                return
            fused_ctx.bind_external(fn.BUF_GRADS, bufs[0][0])
            fused_ctx.bind_external(fn.BUF_TABLE, bufs[1][0])
            mc = (int(bufs[0][1].multicast_ptr), int(bufs[1][1].multicast_ptr))
        handles = fused_ctx.dp_ipc_handles()
        allh = [None] * world
        dist.all_gather_object(allh, handles)
        fused_ctx.dp_attach(rank, world, allh)
        if mc is not None:
            fused_ctx.dp_attach_multicast(*mc)
        n = 256
        half = n // world
        dev = torch.device("cuda", rank)
        for step in range(1, 4):
            rays = torch.from_numpy(rays_toward_box(n, 100 + step, radius=2.0, n_miss=2)[rank * half:(rank + 1) * half]).to(dev)
            tg = torch.from_numpy(targets(n, 100 + step)[rank * half:(rank + 1) * half]).to(dev)
            kw = dict(lr_f=2e-2, lr_t=1e-3, color_rel_lr=0.5, rng_u32=step * 977, ray_offset=rank * half)
            s = fn.make_step(**kw)
            out = torch.zeros((half, 4), device=dev)
            nccl_ctx.forward_backward(rays, tg, out, half, s)
            dist.all_reduce(nccl_ctx.tensor(fn.BUF_GRADS), op=dist.ReduceOp.SUM)
            nccl_ctx.apply_updates(s)
            out2 = torch.zeros((half, 4), device=dev)
            fused_ctx.forward_backward(rays, tg, out2, half, s)
            fused_ctx.dp_reduce_apply(s)
            fused_ctx.apply_updates(fn.make_step(**kw, table_applied=True))
            torch.cuda.synchronize()
        t_a = nccl_ctx.tensor(fn.BUF_TABLE).cpu().numpy()
        t_b = fused_ctx.tensor(fn.BUF_TABLE).cpu().numpy()
        p_a = nccl_ctx.tensor(fn.BUF_PARAMS).cpu().numpy()
        p_b = fused_ctx.tensor(fn.BUF_PARAMS).cpu().numpy()
        res = dict(table=rel_l2(t_b - table, t_a - table), params=rel_l2(p_b - blob, p_a - blob),
                   grads_clear=not fused_ctx.tensor(fn.BUF_GRADS).any().item(),
                   status=(nccl_ctx.status(), fused_ctx.status()), checksum=float(np.float64(t_b).sum()))
        sums = [None] * world
        dist.all_gather_object(sums, res["checksum"])
        res["same_table"] = len(set(sums)) == 1
        for c in ctxs:
            c.close()
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, "ok", res))
    except Exception as exc:
        import traceback
        q.put((rank, "err", f"{exc}\n{traceback.format_exc()}"))


@pytest.mark.parametrize("mode", ["p2p", "nvls"])
def test_fused_exchange_matches_nccl(mode):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, mode, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = {}
    try:
        for _ in range(2):
            rank, st, res = q.get(timeout=240)
            results[rank] = (st, res)
    finally:
        # In the NVLS form a worker's table and gradient buffer are bound to NVLink multicast objects:
        # such a rank is never ended from outside.  It ends by itself -- the exchange's waits are
        # bounded and the process group has a 60 s timeout -- and the parent only reports it.
        for p in procs:
            p.join(timeout=60 if mode == "p2p" else 180)
            if p.is_alive() and mode == "p2p":
                p.kill()
    stuck = [r for r, p in enumerate(procs) if p.is_alive()]
    assert not stuck, f"ranks {stuck} had not exited ({mode} form; left to end by themselves)"
    if any(st == "skip" for st, _ in results.values()):
        pytest.skip("the NVSwitch offers no multicast here")
    for rank, (st, res) in results.items():
        assert st == "ok", res
        assert res["table"] < 1e-4 and res["params"] < 1e-4, res
        assert res["grads_clear"] and res["same_table"] and res["status"] == (0, 0), res


def _timeout_worker(rank, world, port, q):
    """Both ranks stay alive; in the second exchange rank 1 withholds its call, so rank 0's waits
    for rank 1's flags run out (short limit), the kernel sets STATUS_DP_TIMEOUT and returns."""
    try:
        os.environ["NCCL_NVLS_ENABLE"] = "0"   # no NVLink multicast anywhere in this test
        for p in (ROOT / "ffnerf-experimental_b200", ROOT / "tests"):
            sys.path.insert(0, str(p))
        import datetime
        import time
        import torch.distributed as dist
        import ffn_native as fn
        from ffn_config import make_geometry
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        torch.cuda.set_device(rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                                device_id=torch.device("cuda", rank))
        g = make_geometry(F=2, ND=1, NC=2, spr=64, G=64, log2_entries=14, rmax=512.0)
        ctx = fn.Context(g, device=rank, mlp_precision="fp32")
        handles = ctx.dp_ipc_handles()
        allh = [None] * world
        dist.all_gather_object(allh, handles)
        ctx.dp_attach(rank, world, allh)
        ctx.dp_set_wait_limit(200_000)          # ~0.2 s per wait instead of ~16 s
        step = fn.make_step(lr_f=1e-2, lr_t=1e-3, rng_u32=1)
        ctx.dp_reduce_apply(step)               # every rank calls: completes
        torch.cuda.synchronize()
        st1 = ctx.status()
        dist.barrier()
        t0 = time.time()
        if rank == 0:
            ctx.dp_reduce_apply(step)           # rank 1 does not call this one
            torch.cuda.synchronize()
        elapsed = time.time() - t0
        st2 = ctx.status()
        dist.barrier()                          # rank 1 waits on the host until rank 0 is back
        ctx.close()
        dist.destroy_process_group()
        q.put((rank, "ok", dict(st1=st1, st2=st2, elapsed=elapsed)))
    except Exception as exc:
        import traceback
        q.put((rank, "err", f"{exc}\n{traceback.format_exc()}"))


def test_exchange_wait_runs_out():
    """The exchange's cross-rank waits are bounded: with a short limit, a rank whose peer withholds
    its call gets STATUS_DP_TIMEOUT within a second and both ranks tear down cleanly (peer form,
    NVLS off: no rank's memory is bound to a multicast object)."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import ffn_native as fn
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_timeout_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = {}
    try:
        for _ in range(2):
            rank, st, res = q.get(timeout=180)
            results[rank] = (st, res)
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    for rank, (st, res) in results.items():
        assert st == "ok", res
        assert res["st1"] == 0, res
    assert results[0][1]["st2"] & fn.STATUS_DP_TIMEOUT, results[0]
    assert results[0][1]["elapsed"] < 5.0, results[0]
    assert results[1][1]["st2"] == 0, results[1]
    assert all(p.exitcode == 0 for p in procs)
