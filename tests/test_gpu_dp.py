"""Data-parallel training on 2 GPUs: the NCCL gradient allreduce inside the
library (one process per GPU).

Each rank runs half of the tiny LM's batch with the CE weight of the global
token count; after the bucketed allreduce every rank must hold the full-batch
gradients (oracle, per-tensor normwise 5e-5), and after the AdamW step both
ranks' weights must be bit-identical.  Split-f16 runs a first (3xTF32,
scale-measuring) pass, then the split-f16 pass that is compared; its
operand-range flag rides the last gradient reduction, so both ranks take
the same decision.  Skips on hosts with fewer than 2 GPUs.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _loss_mask(R: int) -> np.ndarray:
    """The masked case's full-batch loss mask: rank 0's half selects no
    token at all, rank 1's about two thirds."""
    m = (np.arange(R) % 3 != 1).astype(np.uint8)
    m[:R // 2] = 0
    return m


def _rank(rank, world, port, out_dir, precision, masked):
    import sys
    from pathlib import Path
    sys.path.insert(0, str(Path(__file__).resolve().parents[1]))
    import torch.distributed as dist

    import eshkol_transformer_b200 as etb
    from oracle import oracle as orc
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=__import__("datetime").timedelta(seconds=120))
    s = etb.TINY
    per = s.batch // world
    shape = etb.ModelShape(s.layers, s.d_model, s.heads, s.ffn, s.vocabulary, s.seq_len, per)
    model = etb.LanguageModel(shape, precision=precision, global_tokens=s.batch * s.seq_len)
    model.init(4321)
    uid = [etb.nccl_unique_id() if rank == 0 else None]
    dist.broadcast_object_list(uid, src=0)
    model.enable_data_parallel(uid[0], rank, world)
    ids, targets = orc.synthetic_batch(31, s.batch, s.seq_len, s.vocabulary)
    mine = slice(rank * per, (rank + 1) * per)
    if masked:
        model.set_loss_mask(_loss_mask(s.batch * s.seq_len).reshape(s.batch, s.seq_len)[mine])
    model.forward_backward(ids[mine], targets[mine])
    if precision == etb.PRECISION_F16X3:
        model.forward_backward(ids[mine], targets[mine])
    np.save(os.path.join(out_dir, f"grads{rank}.npy"), model.read(1))
    model.step(ids[mine], targets[mine])
    model.step(ids[mine], targets[mine])
    np.save(os.path.join(out_dir, f"params{rank}.npy"), model.read(0))
    model.close()
    dist.barrier()
    dist.destroy_process_group()


# (precision, masked): PRECISION_TF32X3 = 0, PRECISION_F16X3 = 3; the masked
# case puts the loss-mask weight on the last bucket's all-reduce (rank 0
# selects no token, so its AdamW divides by rank 1's weight alone)
@pytest.mark.parametrize("precision,masked", [(0, False), (3, False), (0, True)])
def test_two_gpu_allreduce_matches_full_batch(tmp_path, precision, masked):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import eshkol_transformer_b200 as etb
    from oracle import oracle as orc
    mp.start_processes(_rank, args=(2, _free_port(), str(tmp_path), precision, masked), nprocs=2,
                       start_method="spawn")
    s = etb.TINY
    om = orc.LanguageModel(s.layers, s.d_model, s.heads, s.ffn, s.vocabulary, s.seq_len, s.batch)
    params = om.init(4321)
    ids, targets = orc.synthetic_batch(31, s.batch, s.seq_len, s.vocabulary)
    if masked:
        _, grads_ref = om.forward_backward_masked(params, ids, targets,
                                                  _loss_mask(s.batch * s.seq_len), 2.0 ** -9)
    else:
        _, grads_ref = om.forward_backward(params, ids, targets)
    g0, g1 = np.load(tmp_path / "grads0.npy"), np.load(tmp_path / "grads1.npy")
    assert np.array_equal(g0.view(np.uint32), g1.view(np.uint32))
    for t, (a, b) in enumerate(zip(om.split(g0), om.split(grads_ref))):
        err = np.abs(a.astype(np.float64) - b).max() / max(np.abs(b).max(), 1e-30)
        assert err <= 5e-5, (t, err)
    p0, p1 = np.load(tmp_path / "params0.npy"), np.load(tmp_path / "params1.npy")
    assert np.array_equal(p0.view(np.uint32), p1.view(np.uint32))
