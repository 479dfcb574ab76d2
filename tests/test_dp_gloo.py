"""Data-parallel semantics on CPU ranks (gloo, world size 2).

The B200 step shards a global batch across ranks, scales each rank's CE
backward by 1/(global tokens) and sums gradients with an allreduce: the
reference's weighted-microbatch accumulation (native/f32_parameter_internal.h:
150-159) with ranks in place of microbatches.  Here two gloo ranks run the
oracle on their halves and allreduce; the result must equal the single-rank
full-batch gradient within f32 summation-order tolerance, and the ranks'
updated weights must stay identical.  Also checks that a rank which fails
before the exchange surfaces as an error on the other rank (short timeout),
not a hang.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

SHAPE = dict(layers=1, d_model=32, heads=2, ffn=64, vocabulary=64, seq_len=16)
BATCH = 4


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, out_dir):
    import sys
    from pathlib import Path
    sys.path.insert(0, str(Path(__file__).resolve().parents[1]))
    from oracle import oracle as orc
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=__import__("datetime").timedelta(seconds=60))
    per = BATCH // world
    om = orc.LanguageModel(batch=per, **SHAPE)
    params = om.init(42)
    ids, targets = orc.synthetic_batch(5, BATCH, SHAPE["seq_len"], SHAPE["vocabulary"])
    mine = slice(rank * per, (rank + 1) * per)
    loss, grads = om.forward_backward(params, ids[mine], targets[mine],
                                      token_scale=float(BATCH * SHAPE["seq_len"]))
    g = torch.from_numpy(grads)
    dist.all_reduce(g)  # sum of per-rank numerators / global N
    m, v = np.zeros_like(params), np.zeros_like(params)
    om.adamw(params, g.numpy(), m, v, orc.adamw_options(1e-3, 0.9, 0.999, 1e-8, 0.01), 1)
    np.save(os.path.join(out_dir, f"grads{rank}.npy"), g.numpy())
    np.save(os.path.join(out_dir, f"params{rank}.npy"), params)
    lt = torch.tensor([loss])
    dist.all_reduce(lt)
    np.save(os.path.join(out_dir, f"loss{rank}.npy"), lt.numpy() / world)
    dist.destroy_process_group()


def test_two_rank_gradient_sum_equals_full_batch(tmp_path):
    from oracle import oracle as orc
    port = _free_port()
    mp.start_processes(_worker, args=(2, port, str(tmp_path)), nprocs=2, start_method="spawn")
    om = orc.LanguageModel(batch=BATCH, **SHAPE)
    params = om.init(42)
    ids, targets = orc.synthetic_batch(5, BATCH, SHAPE["seq_len"], SHAPE["vocabulary"])
    loss_full, grads_full = om.forward_backward(params, ids, targets)
    g0 = np.load(tmp_path / "grads0.npy")
    g1 = np.load(tmp_path / "grads1.npy")
    assert np.array_equal(g0, g1)
    for t, (a, b) in enumerate(zip(om.split(g0), om.split(grads_full))):
        err = np.abs(a.astype(np.float64) - b).max()
        assert err <= 1e-5 * max(np.abs(b).max(), 1e-30) + 1e-9, (t, err)
    assert np.array_equal(np.load(tmp_path / "params0.npy"), np.load(tmp_path / "params1.npy"))
    assert abs(float(np.load(tmp_path / "loss0.npy")[0]) - loss_full) <= 2e-6 * abs(loss_full)


def _dying_worker(rank, world, port, out_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=__import__("datetime").timedelta(seconds=5))
    if rank == 1:
        # leaves between steps, with no collective in flight
        os._exit(0)
    try:
        dist.all_reduce(torch.ones(4))
        outcome = "completed"
    except Exception as exc:  # gloo reports the lost peer or the timeout
        outcome = f"error:{type(exc).__name__}"
    with open(os.path.join(out_dir, "outcome.txt"), "w") as fh:
        fh.write(outcome)
    os._exit(0)


def test_lost_rank_surfaces_as_error_not_hang(tmp_path):
    port = _free_port()
    ctx = mp.start_processes(_dying_worker, args=(2, port, str(tmp_path)), nprocs=2,
                             start_method="spawn", join=False)
    for p in ctx.processes:
        p.join(timeout=60)
        assert not p.is_alive()
    assert (tmp_path / "outcome.txt").read_text().startswith("error:")
