"""Tensor parallelism on 2 GPUs: each rank loads its Megatron shard of a seeded
model (CudaTransformer(tp_rank, tp_size, nccl_comm)); after attn_output and
ffn_down the partial sums are joined either by ncclAllReduce (the default)
or, with WL_TP_PEER set, by the NVLink peer exchange (the GEMV pushes them to
every rank, the next RMSNorm adds them up).  Rank 0's logits for a prompt
and three teacher-forced decode steps must match the CPU oracle within the
model-level tolerance (max |d| <= 1e-2).  Skipped with fewer than two GPUs.
"""
import os
import socket

import numpy as np
import pytest
import torch

import oracle as O

pytestmark = pytest.mark.gpu

TOL = 1e-2


def _rank(rank, world, port, path, prompt, steps, q, mode):
    import torch.distributed as dist
    if mode == "peer":
        os.environ["WL_TP_PEER"] = "1"
    from woolly_b200.model import CudaTransformer, Session, nccl_communicator, nccl_destroy
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    comm = nccl_communicator(rank, world)
    m = CudaTransformer(path, device=rank, tp_rank=rank, tp_size=world, nccl_comm=comm,
                        max_sessions=2, max_context=64, max_batch=2, max_prefill=32)
    s = Session(m)
    out = [s.infer(prompt)]
    for t in steps:
        out.append(s.infer([t]))
    s.close()
    m.close()
    dist.barrier()
    nccl_destroy(comm)
    if rank == 0:
        q.put([np.asarray(o, dtype=np.float32) for o in out])
    dist.destroy_process_group()


def _free_port():
    with socket.socket() as sk:
        sk.bind(("127.0.0.1", 0))
        return sk.getsockname()[1]


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("name", ["gqa_q4_0", "mha_q4_1"])  # kv heads divisible by 2
@pytest.mark.parametrize("mode", ["peer", "nccl"])
def test_tp2_matches_oracle(tiny_models, name, mode):
    """mode "peer": decode-sized batches exchange partial sums through the
    GEMV's NVLink stores and the RMSNorm's reduce; "nccl": ncclAllReduce."""
    import torch.multiprocessing as mp
    path = tiny_models[name]
    rng = np.random.default_rng(7)
    om = O.Model(path)
    vocab = om.vocab
    prompt = rng.integers(0, min(vocab, 512), 9).tolist()
    steps = rng.integers(0, min(vocab, 512), 3).tolist()
    kv = om.new_kv(64)
    ref = [om.forward(kv, prompt, all_rows=True)]
    for t in steps:
        ref.append(om.forward(kv, [t], all_rows=True))
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, path, prompt, steps, q, mode)) for r in range(2)]
    for p in procs:
        p.start()
    got = q.get(timeout=300)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for g, r in zip(got, ref):
        g = g.reshape(r.shape)
        assert np.abs(g - r).max() <= TOL
        assert (g.argmax(-1) == r.argmax(-1)).mean() >= 0.99
