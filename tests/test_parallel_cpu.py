"""Multi-rank host logic on CPU with the gloo backend (world size 2).

* batch sharding partitions the batch exactly;
* the tensor-parallel plan (which heads / FFN columns a rank owns and how the
  reference's parameters are sliced) reproduces the unsharded forward when
  each rank computes its partial sums and an all-reduce completes them -- the
  same op sequence TensorParallelTransformer runs on GPUs with NCCL, executed
  here with the oracle's NumPy operations;
* a rank that dies before a collective makes the survivors' next collective
  fail with an error after the process group's timeout (no hang).
"""

import os
import socket
import sys
from datetime import timedelta

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle
from conftest import REPO


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _pkg():
    sys.path.insert(0, REPO)
    import torch_transformer_benchmark as T
    return T._pkg


def test_batch_shard_partitions():
    par = _pkg().parallel
    for B in (1, 7, 32, 10000):
        for world in (1, 2, 3, 8):
            parts = [par.batch_shard(B, r, world) for r in range(world)]
            assert parts[0].start == 0 and parts[-1].stop == B
            assert all(a.stop == b.start for a, b in zip(parts, parts[1:]))
            sizes = [p.stop - p.start for p in parts]
            assert max(sizes) - min(sizes) <= 1


def test_tp_plan_slices():
    par = _pkg().parallel
    sd = oracle.init_state_dict(1, 64, 256, 1)
    shards = [par.TensorParallelPlan(64, 4, 256, r, 2).shard_layer(sd, 0) for r in range(2)]
    assert shards[0]["w_qkv"].shape == (96, 64)
    assert shards[0]["w_o"].shape == (64, 32)
    assert shards[1]["w_in"].shape == (128, 64) and shards[1]["w_out"].shape == (64, 128)
    # the rank slices tile the full weights
    assert torch.equal(torch.cat([s["w_in"] for s in shards], 0), sd["layers.0.ffn_in.weight"])
    assert torch.equal(torch.cat([s["w_out"] for s in shards], 1), sd["layers.0.ffn_out.weight"])
    with pytest.raises(ValueError):
        par.TensorParallelPlan(64, 3, 256, 0, 2)


def _tp_worker(rank, world, port, L, out_q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        par = _pkg().parallel
        B, S, d, H, F = 2, 24, 64, 4, 256
        sd = oracle.init_state_dict(L, d, F, 5)
        x, _ = oracle.generate_random_case(B, S, d, 6)
        plan = par.TensorParallelPlan(d, H, F, rank, world)
        Hl, hd = plan.local_heads, plan.head_dim
        cur = x.numpy()
        for i in range(L):
            w = {k: v.numpy() for k, v in plan.shard_layer(sd, i).items()}
            n1 = oracle.layer_norm(cur, w["ln1_w"], w["ln1_b"])
            qkv = oracle.linear(n1, w["w_qkv"], w["b_qkv"])
            dl = Hl * hd
            split = lambda t: t.reshape(B, S, Hl, hd).transpose(0, 2, 1, 3)  # noqa: E731
            ctx = oracle.causal_attention(split(qkv[..., :dl]), split(qkv[..., dl:2 * dl]), split(qkv[..., 2 * dl:]))
            ctx = ctx.transpose(0, 2, 1, 3).reshape(B, S, dl)
            part = torch.from_numpy(np.ascontiguousarray(oracle.linear(ctx, w["w_o"], None)))
            dist.all_reduce(part)
            x1 = cur + part.numpy() + w["b_o"]
            hdn = oracle.gelu_erf(oracle.linear(oracle.layer_norm(x1, w["ln2_w"], w["ln2_b"]), w["w_in"], w["b_in"]))
            part = torch.from_numpy(np.ascontiguousarray(oracle.linear(hdn, w["w_out"], None)))
            dist.all_reduce(part)
            cur = x1 + part.numpy() + w["b_out"]
        y = oracle.layer_norm(cur, sd["final_norm.weight"].numpy(), sd["final_norm.bias"].numpy())
        ref = oracle.model_forward(oracle.params_from_state_dict(sd), oracle.OracleConfig(B, S, d, H, F, L, True),
                                   x.numpy())
        out_q.put((rank, float(np.abs(y - ref).max())))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("L", [1, 2])
def test_tensor_parallel_decomposition_gloo(L):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_tp_worker, args=(r, 2, port, L, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
        assert p.exitcode == 0
    res = dict(q.get(timeout=5) for _ in range(2))
    assert max(res.values()) < 1e-5, res


def _dying_worker(rank, world, port, out_q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=3))
    t = torch.ones(4)
    dist.all_reduce(t)  # both ranks take part in the first step
    if rank == 1:
        os._exit(0)  # rank 1 leaves between steps, with nothing in flight
    try:
        dist.all_reduce(t)
        out_q.put(("no-error", rank))
    except Exception as e:  # noqa: BLE001 - the point of the test
        out_q.put(("error", type(e).__name__))


def test_dead_rank_fails_next_collective_with_timeout():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_dying_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(60)
    kind, detail = q.get(timeout=5)
    assert kind == "error", detail
