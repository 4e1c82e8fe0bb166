"""Tensor parallelism on 2 GPUs (skipped with fewer): greedy tokens of a
2-layer 8B-shaped W4 model under TP=2 -- with the one-shot all-reduce over
peer memory and with NCCL -- against the same model on one GPU. Near-ties
as in test_model_gpu (the TP sums round differently)."""
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _rank(rank, world, port, peer, out_dir):
    import dataclasses

    import torch
    import torch.distributed as dist

    from aethermind_b200 import session

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    obj = [session.nccl_unique_id() if rank == 0 else None]
    dist.broadcast_object_list(obj, src=0)
    rt = session.Runtime(rank, rank, world, obj[0])
    if peer:
        handles = [None] * world
        dist.all_gather_object(handles, rt.peer_handle())
        rt.open_peers(handles)
    cfg = dataclasses.replace(session.LLAMA_8B_W4, layers=2, max_seq=256, max_batch=2)
    m = session.Model(rt, cfg)
    m.init_synthetic(3)
    s = session.Session(m)
    prompt = np.random.default_rng(11).integers(0, cfg.vocab, 20).astype(np.uint32)
    got = s.generate(prompt, 12)
    p2 = np.stack([prompt, np.random.default_rng(12).integers(0, cfg.vocab, 20).astype(np.uint32)])
    got2 = s.generate(p2, 6)
    if rank == 0:
        np.save(os.path.join(out_dir, f"tp_{int(peer)}.npy"), got)
        np.save(os.path.join(out_dir, f"tp2_{int(peer)}.npy"), got2)
    dist.barrier()
    dist.destroy_process_group()


def _run(peer, port, tmp):
    import torch.multiprocessing as mp
    mp.start_processes(_rank, args=(2, port, peer, str(tmp)), nprocs=2, join=True, start_method="spawn")


@pytest.mark.parametrize("peer,fused", [(True, False), (True, True), (False, False)])
def test_tp2_matches_one_gpu(built_lib, oracle_lib, tmp_path, monkeypatch, peer, fused):
    """peer: decode all-reduces over peer memory (else NCCL); fused: the sum
    runs inside the o/down GEMV's epilogue (AmcuLinearArgs::peer_reduce)
    instead of a separate one-shot kernel."""
    monkeypatch.setenv("AMCU_TP_FUSED_ALLREDUCE", "1" if fused else "0")
    import dataclasses

    import torch

    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    from aethermind_b200 import session
    from tests.test_model_gpu import _compare

    _run(peer, 29611 + int(peer) + 2 * int(fused), tmp_path)
    got = np.load(tmp_path / f"tp_{int(peer)}.npy")
    got2 = np.load(tmp_path / f"tp2_{int(peer)}.npy")
    cfg = dataclasses.replace(session.LLAMA_8B_W4, layers=2, max_seq=256, max_batch=2)
    prompt = np.random.default_rng(11).integers(0, cfg.vocab, 20).astype(np.uint32)
    ref, gaps = oracle_lib.synthetic_oracle_model(cfg, seed=3).generate(prompt.astype(np.int64), 12)
    assert _compare(got.tolist(), ref.tolist(), gaps, 0.125) >= 6
    rt = session.Runtime(0)
    m = session.Model(rt, cfg)
    m.init_synthetic(3)
    one = session.Session(m).generate(prompt, 12)
    assert _compare(got.tolist(), one.tolist(), gaps, 0.125) >= 6
    assert _compare(got2[0].tolist()[:6], got.tolist()[:6], gaps, 0.125) >= 6
