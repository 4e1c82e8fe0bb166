"""Tensor-parallel sharding scheme on CPU with gloo ranks (world size 2).

The engine splits q/k/v and gate/up by output rows and o/down by input
columns at 128-column group boundaries, and sums the row-parallel partials
with one all-reduce per block. These tests run that scheme with the CPU
oracle's W4 Linear on each rank and check that the all-reduced result equals
the unsharded Linear, and that a rank that never joins makes the others fail
with a timeout error instead of hanging.
"""
import os
import socket
from datetime import timedelta

import numpy as np
import pytest
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _tp_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import torch

        import oracle
        n_out, k = 64, 512
        rng = np.random.default_rng(0)
        x = oracle.bf16_round(rng.normal(0, 1, (2, k)).astype(np.float32))
        qw, sw = oracle.synth_w4(3, 7, n_out, k, oracle.W4_BASE)
        full = oracle.linear_w4(x, qw, sw, bf=False)
        # column-parallel: rows [r*n/w, (r+1)*n/w) -> gather
        rows = n_out // world
        col = oracle.linear_w4(x, qw[rank * rows:(rank + 1) * rows], sw[rank * rows:(rank + 1) * rows], bf=False)
        parts = [torch.zeros(2, rows) for _ in range(world)]
        dist.all_gather(parts, torch.from_numpy(col))
        gathered = torch.cat(parts, dim=1).numpy()
        # row-parallel: columns [r*k/w, ...) -> all-reduce(sum)
        kc = k // world
        part = oracle.linear_w4(np.ascontiguousarray(x[:, rank * kc:(rank + 1) * kc]),
                                np.ascontiguousarray(qw[:, rank * kc // 2:(rank + 1) * kc // 2]),
                                np.ascontiguousarray(sw[:, rank * kc // 128:(rank + 1) * kc // 128]), bf=False)
        t = torch.from_numpy(part.copy())
        dist.all_reduce(t)
        q.put((rank, float(np.abs(gathered - full).max()), float(np.abs(t.numpy() - full).max()),
               float(np.abs(full).max())))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2])
def test_tp_sharding_reproduces_full_linear(oracle_lib, world):
    port = _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_tp_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, col_err, row_err, scale in res:
        assert col_err == 0.0  # column split is exact (same rows, same order)
        assert row_err <= 1e-5 * scale + 1e-6  # row split regroups the fp32 sum


def _absent_peer_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import torch
    if rank == 1:
        q.put((rank, "left"))  # this rank leaves before joining the group
        return
    try:
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=3))
        dist.all_reduce(torch.ones(4))
        q.put((rank, "no error"))
    except Exception as e:  # the missing rank surfaces as an error, not a hang
        q.put((rank, type(e).__name__))


def test_missing_rank_times_out_instead_of_hanging():
    port = _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_absent_peer_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in range(2))
    for p in procs:
        p.join(timeout=60)
    assert res[1] == "left"
    assert res[0] != "no error"


def _engine_plan_worker(rank, world, port, q):
    """One attention block and one MLP block of a small W4 layer, each rank
    holding the blocks the engine's own shard rule (am_debug_tp_shard) gives
    it; the row-parallel partials are summed with a gloo all-reduce."""
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import ctypes as C

        import torch

        import oracle
        from aethermind_b200 import _lib as L

        def plan(name, n, k):
            out = (C.c_int64 * 4)()
            L.check(L.lib().am_debug_tp_shard(name.encode(), n, k, rank, world, out), "am_debug_tp_shard")
            return tuple(out)

        def take(wq, n, k, name):
            q4, s4 = wq
            r0, nr, c0, nc = plan(name, n, k)
            return (np.ascontiguousarray(q4[r0:r0 + nr, c0 // 2:(c0 + nc) // 2]),
                    np.ascontiguousarray(s4[r0:r0 + nr, c0 // 128:(c0 + nc) // 128])), (c0, nc)

        H, nq, nkv, d, I, M = 256, 4, 2, 64, 512, 3
        rng = np.random.default_rng(0)
        x = oracle.bf16_round(rng.normal(0, 1, (M, H)).astype(np.float32))
        W = {n: oracle.synth_w4(5, i, *shp, oracle.W4_BASE) for i, (n, shp) in enumerate(
            {"wq": (nq * d, H), "wk": (nkv * d, H), "wv": (nkv * d, H), "wo": (H, nq * d),
             "wg": (I, H), "wu": (I, H), "wd": (H, I)}.items())}

        def block(Wq, Wk, Wv, Wo, nq_l, nkv_l, Wg, Wu, Wd):
            lin = lambda a, w: oracle.linear_w4(a, *w, bf=False)
            qh, kh, vh = lin(x, Wq), lin(x, Wk), lin(x, Wv)
            kp = np.ascontiguousarray(kh.reshape(M, nkv_l, d).transpose(1, 0, 2))
            vp = np.ascontiguousarray(vh.reshape(M, nkv_l, d).transpose(1, 0, 2))
            att = oracle.attention(qh, kp, vp, 0, nq_l, nkv_l, d)
            o = lin(att, Wo)
            act = oracle.silu_mul(lin(x, Wg), lin(x, Wu))
            return o, lin(act, Wd)

        full_o, full_d = block(W["wq"], W["wk"], W["wv"], W["wo"], nq, nkv, W["wg"], W["wu"], W["wd"])
        sh = {n: take(W[n], *{"wq": (nq * d, H), "wk": (nkv * d, H), "wv": (nkv * d, H), "wo": (H, nq * d),
                              "wg": (I, H), "wu": (I, H), "wd": (H, I)}[n], n)[0] for n in W}
        o, dn = block(sh["wq"], sh["wk"], sh["wv"], sh["wo"], nq // world, nkv // world, sh["wg"], sh["wu"], sh["wd"])
        to, td = torch.from_numpy(o.copy()), torch.from_numpy(dn.copy())
        dist.all_reduce(to)
        dist.all_reduce(td)
        q.put((rank, float(np.abs(to.numpy() - full_o).max()), float(np.abs(full_o).max()),
               float(np.abs(td.numpy() - full_d).max()), float(np.abs(full_d).max()),
               plan("wq", nq * d, H), plan("wo", H, nq * d), plan("attn_norm", 1, H)))
    finally:
        dist.destroy_process_group()


def test_engine_shard_plan_reproduces_full_layer(oracle_lib, built_lib):
    """The engine's sharding rule (the function that slices weights at model
    load, exposed as am_debug_tp_shard) run on 2 gloo ranks: q/k/v by heads,
    gate/up by intermediate rows, o/down by input columns; the all-reduced
    attention and MLP blocks equal the unsharded ones."""
    world = 2
    port = _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_engine_plan_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=180) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, eo, so, ed, sd, pq, po, pn in res:
        assert eo <= 1e-5 * so + 1e-6 and ed <= 1e-5 * sd + 1e-6, (eo, so, ed, sd)
        assert pq == (rank * 128, 128, 0, 256)   # q rows: this rank's two heads
        assert po == (0, 256, rank * 128, 128)   # o: this rank's input columns
        assert pn == (0, 1, 0, 256)              # norms replicated
