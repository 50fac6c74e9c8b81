"""Tensor-parallel partition logic on CPU: two gloo ranks run one decoder layer
of a seeded model on their Megatron shards (q/k/v and gate/up split by columns,
attn_output and ffn_down by rows, one all-reduce after each row-parallel
projection) and must reproduce the unsharded layer.  The shard boundaries are
the ones the CUDA loader uses (woolly_b200/csrc/model.cpp, Loader::add_mat
calls): q columns [r*H/T*hd, ...), k/v columns [r*KVH/T*hd, ...), ffn columns
[r*ff/T, ...), and the matching rows of attn_output / ffn_down.
"""
import os
import socket

import numpy as np
import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle as O

EPS = 1e-5


def _layer_weights(path):
    from woolly_b200.gguf import GGUFLoader
    g = GGUFLoader.from_path(path)
    out = {}
    for t in g.tensors():
        if t.name.startswith("blk.0."):
            raw = g.tensor_data(t.name)
            n = t.n_elements
            out[t.name[6:]] = O.dequantize(raw, t.ggml_type, n).reshape(t.shape if len(t.shape) == 2 else (n,))
    cfg = g.model_config()
    g.close()
    return out, cfg


def _layer(x, W, H, KVH, hd, ff, d, q_cols, kv_cols, f_cols, reduce):
    """Pre-norm decoder layer on rows x (positions 0..rows-1, no past) with the
    given column slices of q, k/v and ffn; `reduce` sums row-parallel partials."""
    rows = x.shape[0]
    xn = O.rms_norm(x, W["attn_norm.weight"], EPS)
    Wq = W["attn_q.weight"][:, q_cols]
    Wk = W["attn_k.weight"][:, kv_cols]
    Wv = W["attn_v.weight"][:, kv_cols]
    nq, nkv = Wq.shape[1], Wk.shape[1]
    q = O.matmul_b(xn, Wq, d, nq)
    k = O.matmul_b(xn, Wk, d, nkv)
    v = O.matmul_b(xn, Wv, d, nkv)
    att = O.attention(q, k, v, rows, 0, nq // hd, nkv // hd, hd)
    Wo = W["attn_output.weight"][q_cols, :]
    h = x + reduce(O.matmul_b(att, Wo, nq, d))
    hn = O.rms_norm(h, W["ffn_norm.weight"], EPS)
    Wg = W["ffn_gate.weight"][:, f_cols]
    Wu = W["ffn_up.weight"][:, f_cols]
    nf = Wg.shape[1]
    a = O.swiglu(O.matmul_b(hn, Wg, d, nf), O.matmul_b(hn, Wu, d, nf))
    Wd = W["ffn_down.weight"][f_cols, :]
    return h + reduce(O.matmul_b(a, Wd, nf, d))


def _rank(rank, world, port, path, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    import torch
    W, cfg = _layer_weights(path)
    d, H = cfg["hidden_size"], cfg["num_heads"]
    KVH = cfg["num_key_value_heads"] or H
    hd = d // H
    ff = cfg["intermediate_size"]
    x = np.random.default_rng(3).standard_normal((5, d)).astype(np.float32)
    qc, kc, fc = H // world * hd, KVH // world * hd, ff // world

    def allreduce(p):
        t = torch.from_numpy(np.ascontiguousarray(p))
        dist.all_reduce(t)
        return t.numpy()

    y = _layer(x, W, H, KVH, hd, ff, d, slice(rank * qc, (rank + 1) * qc),
               slice(rank * kc, (rank + 1) * kc), slice(rank * fc, (rank + 1) * fc), allreduce)
    if rank == 0:
        ref = _layer(x, W, H, KVH, hd, ff, d, slice(None), slice(None), slice(None), lambda p: p)
        q.put(float(np.abs(y - ref).max()))
    dist.barrier()
    dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("name", ["gqa_q4_0", "mha_q4_1"])
def test_tp2_layer_matches_unsharded(tiny_models, name):
    O.build()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, tiny_models[name], q)) for r in range(2)]
    for p in procs:
        p.start()
    err = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert err < 1e-4
