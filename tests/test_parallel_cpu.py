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


def test_tp_schedule_orders_and_slots():
    """Every chunk passes A, B, F in that order; a per-chunk slot (i % 2) is rewritten
    only after the last reader of its previous chunk (A(i+2) after B(i), B(i+2) after F(i))."""
    par = _pkg().parallel
    for n in range(1, 9):
        sch = par.tp_schedule(n)
        pos = {st: i for i, st in enumerate(sch)}
        assert len(sch) == 3 * n and len(pos) == 3 * n
        for i in range(n):
            assert pos[("A", i)] < pos[("B", i)] < pos[("F", i)]
            if i + 2 < n:
                assert pos[("B", i)] < pos[("A", i + 2)]
                assert pos[("F", i)] < pos[("B", i + 2)]


@pytest.mark.parametrize("B,S,R", [(3, 300, 128), (5, 128, 300), (2, 256, 256), (1, 1000, 4096)])
def test_tp_chunks_cover_every_row_once(B, S, R):
    par = _pkg().parallel
    seen = np.zeros(B * S, dtype=int)
    last = 0
    for b0, nb, c0, c1 in par.tp_chunks(B, S, R):
        assert nb == 1 or (c0 == 0 and c1 == S)
        assert nb * (c1 - c0) <= max(R, S)
        r0 = b0 * S + c0
        assert r0 == last  # chunks are in row order, contiguous
        seen[r0:r0 + nb * (c1 - c0)] += 1
        last = r0 + nb * (c1 - c0)
    assert (seen == 1).all()


def _tp_chunked_worker(rank, world, port, out_q):
    """The chunked tensor-parallel forward's host logic (tp_chunks, tp_schedule, two
    slots, an all-reduce per partial issued asynchronously and waited for only by the
    stage that reads it), with the oracle's NumPy ops standing in for the kernels."""
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        par = _pkg().parallel
        B, S, d, H, F, R = 3, 40, 64, 4, 256, 16
        sd = oracle.init_state_dict(1, d, F, 8)
        x, _ = oracle.generate_random_case(B, S, d, 9)
        xf = x.numpy().reshape(B * S, d)
        plan = par.TensorParallelPlan(d, H, F, rank, world)
        Hl, hd = plan.local_heads, plan.head_dim
        dl = Hl * hd
        w = {k: v.numpy() for k, v in plan.shard_layer(sd, 0).items()}
        chunks = par.tp_chunks(B, S, R)
        kv = np.zeros((B * S, 2 * dl), dtype=np.float32)
        p1 = [torch.zeros(R, d) for _ in range(2)]
        p2 = [torch.zeros(R, d) for _ in range(2)]
        x1 = [np.zeros((R, d), dtype=np.float32) for _ in range(2)]
        work1, work2 = [None, None], [None, None]
        y = np.full((B * S, d), np.nan, dtype=np.float32)
        heads = lambda t: t.reshape(1, -1, Hl, hd).transpose(0, 2, 1, 3)  # noqa: E731
        for stage, i in par.tp_schedule(len(chunks)):
            b0, nb, c0, c1 = chunks[i]
            r0 = b0 * S + c0
            n_r = nb * (c1 - c0)
            sl = i % 2
            if stage == "A":
                n = oracle.layer_norm(xf[r0:r0 + n_r], w["ln1_w"], w["ln1_b"])
                q = oracle.linear(n, w["w_qkv"][:dl], w["b_qkv"][:dl])
                kv[r0:r0 + n_r] = oracle.linear(n, w["w_qkv"][dl:], w["b_qkv"][dl:])
                ctx = np.empty((n_r, dl), dtype=np.float32)
                for j in range(nb):
                    b = b0 + j
                    qj = q[j * (c1 - c0):(j + 1) * (c1 - c0)]
                    kj, vj = kv[b * S:b * S + c1, :dl], kv[b * S:b * S + c1, dl:]
                    o = oracle.causal_attention(heads(qj), heads(kj), heads(vj), q_offset=c0)
                    ctx[j * (c1 - c0):(j + 1) * (c1 - c0)] = o.transpose(0, 2, 1, 3).reshape(-1, dl)
                p1[sl][:n_r] = torch.from_numpy(oracle.linear(ctx, w["w_o"], None))
                work1[sl] = dist.all_reduce(p1[sl][:n_r], async_op=True)
            elif stage == "B":
                work1[sl].wait()
                x1[sl][:n_r] = xf[r0:r0 + n_r] + p1[sl][:n_r].numpy() + w["b_o"]
                hdn = oracle.gelu_erf(oracle.linear(oracle.layer_norm(x1[sl][:n_r], w["ln2_w"], w["ln2_b"]),
                                                    w["w_in"], w["b_in"]))
                p2[sl][:n_r] = torch.from_numpy(oracle.linear(hdn, w["w_out"], None))
                work2[sl] = dist.all_reduce(p2[sl][:n_r], async_op=True)
            else:
                work2[sl].wait()
                y[r0:r0 + n_r] = oracle.layer_norm(x1[sl][:n_r] + p2[sl][:n_r].numpy() + w["b_out"],
                                                   sd["final_norm.weight"].numpy(), sd["final_norm.bias"].numpy())
        ref = oracle.model_forward(oracle.params_from_state_dict(sd), oracle.OracleConfig(B, S, d, H, F, 1, True),
                                   x.numpy()).reshape(B * S, d)
        out_q.put((rank, float(np.abs(y - ref).max())))
    finally:
        dist.destroy_process_group()


def test_tensor_parallel_chunked_schedule_gloo():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_tp_chunked_worker, args=(r, 2, port, q)) for r in range(2)]
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
