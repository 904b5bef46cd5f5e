"""Data-parallel host logic on CPU: two `gloo` ranks (world size 2) in child processes.

  * sharding: each rank runs the CPU oracle on its contiguous half of a batch with its global
    ray offset; the all-reduced gradients equal the single-process gradients of the whole batch
    (rel-L2 1e-6: only the float summation order of the two halves differs) and the per-ray
    colours are bit-exact;
  * DataParallel.allreduce_grads sums the gradient buffer across ranks;
  * DataParallel.merge_occupancy takes the nibble-wise maximum of the ranks' proposal grids
    (byte expansion, MAX all-reduce, packing), with the byte conversion of the device replaced by
    a numpy double of ffn_occ_st_bytes;
  * Nerf falls back to the deferred table update once data parallelism is on.
"""
import os
import socket
import sys
from pathlib import Path

import numpy as np
import pytest

torch = pytest.importorskip("torch")
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parents[1]


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _paths():
    for p in (ROOT / "ffnerf-experimental_b200", ROOT / "oracle", ROOT / "tests"):
        if str(p) not in sys.path:
            sys.path.insert(0, str(p))


class _FakeNative:
    """CPU double of the parts of ffn_native.Context that DataParallel touches."""

    def __init__(self, grads, occ_st):
        self.device = "cpu"
        self._grads = grads
        self.occ_st = occ_st            # uint32 numpy [G^3]

    def tensor(self, buf_id):
        return self._grads

    def occ_st_bytes(self, buf, to_bytes, stream=None):
        if to_bytes:   # one byte per nibble, word-major, nibble 0 first
            w = self.occ_st[:, None] >> (4 * np.arange(8, dtype=np.uint32))[None, :]
            buf.copy_(torch.from_numpy((w & 0xF).astype(np.uint8).reshape(-1)))
        else:
            b = buf.numpy().reshape(-1, 8).astype(np.uint32)
            self.occ_st[:] = (b << (4 * np.arange(8, dtype=np.uint32))[None, :]).sum(1).astype(np.uint32)


def _worker(rank, world, port, q):
    try:
        _paths()
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world)
        import ffnerf_tools as ft
        from _helpers import init_blob, init_occ, init_table, rays_toward_box, targets
        from ffn_config import make_geometry
        from oracle import Oracle, OrcStep, make_orc_config

        # ---- sharded oracle step, gradients all-reduced over gloo
        g = make_geometry(F=2, ND=1, NC=2, spr=64, G=32, log2_entries=12, rmax=256.0)
        n = 64
        rays, tg = rays_toward_box(n, 5, radius=2.0, n_miss=4), targets(n, 5)
        blob, table, occ = init_blob(g, 5), init_table(g, 5), init_occ(g, 5)
        orc = Oracle()
        half = n // world
        sl = slice(rank * half, (rank + 1) * half)
        tgo, mgo = np.zeros(table.size, np.float32), np.zeros(blob.size, np.float32)
        out = np.zeros((half, 4), np.float32)
        orc.forward_backward(make_orc_config(g), OrcStep(1e-3, 1.0, 0.0, 77, 1, rank * half), blob, table.copy(),
                             occ.copy(), occ.copy(), rays[sl], tg[sl], out, tgo, mgo)
        grads = torch.from_numpy(np.concatenate([tgo, mgo]))
        nat = _FakeNative(grads, np.zeros(8, np.uint32))
        dp = ft.DataParallel()
        assert (dp.rank, dp.world) == (rank, world)

        class _N:
            native = nat
        dp.allreduce_grads(_N())
        outs = [torch.zeros(half, 4) for _ in range(world)]
        dist.all_gather(outs, torch.from_numpy(out))

        # ---- occupancy merge: nibble-wise max of the ranks' grids
        G = 4
        rng = np.random.default_rng(100 + rank)
        mine = rng.integers(0, 2 ** 32, G ** 3, dtype=np.uint64).astype(np.uint32)
        nat_o = _FakeNative(grads, mine.copy())

        class _M:
            native = nat_o
            occ = type("O", (), {"G_occ": G})()
            _occ_bytes = torch.empty(G ** 3 * 8, dtype=torch.uint8)
        m = _M()
        dp.merge_occupancy(m)
        all_grids = [torch.zeros(G ** 3, dtype=torch.int64) for _ in range(world)]
        dist.all_gather(all_grids, torch.from_numpy(mine.astype(np.int64)))
        if rank == 0:
            q.put(("ok", grads.numpy().copy(), torch.cat(outs).numpy(), nat_o.occ_st.copy(),
                   [a.numpy().astype(np.uint32) for a in all_grids]))
        dist.barrier()
        dist.destroy_process_group()
    except Exception as exc:  # report to the parent instead of hanging it
        import traceback
        q.put(("err", f"rank {rank}: {exc}\n{traceback.format_exc()}"))


def test_two_rank_shards_and_exchange():
    _paths()
    from _helpers import init_blob, init_occ, init_table, rays_toward_box, rel_l2, targets
    from ffn_config import make_geometry
    from oracle import Oracle, OrcStep, make_orc_config

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    try:
        res = q.get(timeout=180)
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    assert res[0] == "ok", res[1]
    _, grads, out_sh, merged, grids = res
    # single-process reference of the whole batch
    g = make_geometry(F=2, ND=1, NC=2, spr=64, G=32, log2_entries=12, rmax=256.0)
    n = 64
    rays, tg = rays_toward_box(n, 5, radius=2.0, n_miss=4), targets(n, 5)
    blob, table, occ = init_blob(g, 5), init_table(g, 5), init_occ(g, 5)
    tgo, mgo = np.zeros(table.size, np.float32), np.zeros(blob.size, np.float32)
    out = np.zeros((n, 4), np.float32)
    Oracle().forward_backward(make_orc_config(g), OrcStep(1e-3, 1.0, 0.0, 77, 1, 0), blob, table.copy(), occ.copy(),
                              occ.copy(), rays, tg, out, tgo, mgo)
    assert np.array_equal(out_sh, out)
    assert rel_l2(grads[:table.size], tgo) < 1e-6
    assert rel_l2(grads[table.size:], mgo) < 1e-6
    # nibble-wise max
    a, b = grids
    sh = 4 * np.arange(8, dtype=np.uint32)
    na, nb = (a[:, None] >> sh) & 0xF, (b[:, None] >> sh) & 0xF
    expect = (np.maximum(na, nb) << sh).sum(1).astype(np.uint32)
    assert np.array_equal(merged, expect)


def test_nerf_uses_deferred_updates_under_data_parallel(tmp_path):
    _paths()
    import ffnerf_tools as ft
    nerf = ft.Nerf(None, None, training_dir=tmp_path, model_id="dp", transfer_fmt="fp32", table_size_entries=16 << 10,
                   f_per_level=2, verbose=False)
    assert nerf.table_immediate
    nerf.dp = object()          # what enable_data_parallel installs
    assert not nerf.table_immediate
    nerf.dp = None
    nerf.table_optimizer = "adam"
    assert not nerf.table_immediate
    with pytest.raises(ValueError):
        ft.Nerf(None, None, training_dir=tmp_path, model_id="x", table_update="sometimes", verbose=False)
