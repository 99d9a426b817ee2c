"""Chunked forward, tensor parallelism and batch sharding on B200s.

Distributed cases run in spawned child processes (NCCL, 127.0.0.1
rendezvous, NVLS off, short process-group timeout) so the test process keeps
no communicator.  Two-rank cases need two GPUs and skip otherwise.
"""

import os
import socket
import sys
from datetime import timedelta

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

import oracle
from conftest import REPO

pytestmark = pytest.mark.gpu

ATOL, RTOL = 0.002, 0.02
DEV = "cuda"


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _model(tt, B, S, d, H, F, L, seed=1234):
    cfg = tt.TransformerConfig(B, S, d, H, F, L, True)
    torch.manual_seed(seed)
    return tt.UserOptimizedTransformer(cfg).to(DEV).eval()


@pytest.mark.parametrize("rows", [128, 192, 256])
def test_chunked_matches_chain(tt, rows):
    model = _model(tt, 3, 640, 256, 4, 1024, 1)
    x, _ = oracle.generate_random_case(3, 640, 256, 41)
    xd = x.to(DEV)
    with torch.inference_mode():
        model.force_strategy = "chain"
        y_chain = model(xd).clone()
        model.force_strategy = "chunked"
        model.chunk_rows = rows
        y_chunk = model(xd).clone()
    torch.cuda.synchronize()
    res = oracle.compare_outputs(y_chain.cpu(), y_chunk.cpu(), rtol=RTOL, atol=ATOL)
    assert res.passed, res
    assert res.max_abs_error < 5e-4


def test_chunked_two_layers_vs_oracle(tt):
    model = _model(tt, 2, 300, 128, 2, 512, 2, seed=9)
    model.force_strategy, model.chunk_rows = "chunked", 128
    x, _ = oracle.generate_random_case(2, 300, 128, 10)
    with torch.inference_mode():
        y = model(x.to(DEV)).cpu()
    ref = oracle.model_forward(oracle.params_from_state_dict(model.state_dict()),
                               oracle.OracleConfig(2, 300, 128, 2, 512, 2, True), x.numpy())
    assert oracle.compare_outputs(ref, y, rtol=RTOL, atol=ATOL).passed


def test_add_layernorm_and_f32_epilogue(pkg):
    rt = pkg.runtime
    g = torch.Generator().manual_seed(3)
    M, d = 777, 256
    a = torch.randn(M, d, generator=g).to(DEV)
    b = torch.randn(M, d, generator=g).to(DEV)
    bias = torch.randn(d, generator=g).to(DEV)
    gamma, beta = torch.randn(d, generator=g).to(DEV), torch.randn(d, generator=g).to(DEV)
    s = torch.empty(M, d, device=DEV)
    out = torch.empty(M, d, device=DEV)
    rt.add_layernorm(a, b, bias, s, gamma, beta, out)
    ref_s = a + b + bias
    ref = torch.nn.functional.layer_norm(ref_s, (d,), gamma, beta, 1e-5)
    torch.cuda.synchronize()
    assert torch.allclose(s, ref_s, atol=1e-6) and (out - ref).abs().max() < 1e-4
    # fp32 epilogue, exact-integer operands
    A = torch.randint(-2, 3, (300, 128), generator=g).half().to(DEV)
    W = torch.randint(-2, 3, (96, 128), generator=g).half().to(DEV)
    o = torch.empty(300, 96, device=DEV)
    rt.gemm(rt.EPI_BIAS_F32, A, W, None, o)
    torch.cuda.synchronize()
    assert torch.equal(o.double(), A.double() @ W.double().T)


def _tp_child(rank, world, port, mode, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    sys.path.insert(0, REPO)
    import torch.distributed as dist
    import torch_transformer_benchmark as T
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60), device_id=dev)
    try:
        par = T._pkg.parallel
        if mode == "tp_c5":
            # the C5 head shape (d=1024, 16 heads of 64), 1024-row query chunks over S=4096
            B, S, d, H, F, L = 2, 4096, 1024, 16, 4096, 1
        else:
            B, S, d, H, F, L = 4, 256, 256, 4, 1024, 2
        cfg = T.TransformerConfig(B, S, d, H, F, L, True)
        torch.manual_seed(1234)
        model = T.UserOptimizedTransformer(cfg).to(dev).eval()
        x, _ = oracle.generate_random_case(B, S, d, 77)
        if mode == "tp_c5":
            tpm = par.TensorParallelTransformer(model, rank, world, chunk_rows=1024)
            with torch.inference_mode():
                yd = tpm(x.to(dev))
                yd2 = tpm(x.to(dev))  # a second call reuses the buffers and weight slices
            torch.cuda.synchronize()
            same = bool(torch.equal(yd, yd2))
            # every TP rank holds the same (replicated) output
            cks = torch.tensor([float(yd.double().sum()), float((yd.double() ** 2).sum())], device=dev)
            allc = [torch.empty_like(cks) for _ in range(world)]
            dist.all_gather(allc, cks)
            same = same and all(torch.equal(allc[0], c) for c in allc)
            y = yd.cpu()
            params = oracle.params_from_state_dict(model.state_dict())
            ok, worst = same, 0.0
            for b, c0, c1 in ((0, 3072, 4096), (1, 0, 1024), (1, 2048, 2560)):
                ref = oracle.chunk_rows_forward(params, H, x[b].numpy(), c0, c1)
                res = oracle.compare_outputs(ref, y[b, c0:c1], rtol=RTOL, atol=ATOL)
                ok, worst = ok and res.passed, max(worst, res.max_abs_error)
            q.put((rank, ok, worst))
            return
        # key padding as the reference harness generates it (--padding-ratio), plus holes in
        # sequence 1 (the chunks' attention applies key bits)
        x, mask = oracle.generate_random_case(B, S, d, 77, padding_ratio=0.3)
        mask[1, 7] = False
        mask[1, 130:140] = False
        if mode == "tp":
            y = par.TensorParallelTransformer(model, rank, world, chunk_rows=128)(x.to(dev), mask.to(dev)).cpu()
        else:
            sl = par.batch_shard(B, rank, world)
            y = par.BatchShardedTransformer(model, rank, world)(x[sl].to(dev).contiguous(), gather=True, batch=B,
                                                               valid_token_mask=mask[sl].to(dev)).cpu()
        ref = oracle.model_forward(oracle.params_from_state_dict(model.state_dict()),
                                   oracle.OracleConfig(B, S, d, H, F, L, True), x.numpy(), mask.numpy())
        res = oracle.compare_outputs(ref, y, rtol=RTOL, atol=ATOL)
        q.put((rank, res.passed and bool(torch.all(y[~mask] == 0)), res.max_abs_error))
    finally:
        dist.destroy_process_group()


def _spawn(world, mode):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_tp_child, args=(r, world, port, mode, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(300)
    codes = [p.exitcode for p in procs]
    assert codes == [0] * world, codes
    res = [q.get(timeout=5) for _ in range(world)]
    assert all(r[1] for r in res), res


@pytest.mark.parametrize("mode", ["tp", "batch", "tp_c5"])
def test_single_rank_process_group(mode):
    _spawn(1, mode)


@pytest.mark.parametrize("mode", ["tp", "batch", "tp_c5"])
def test_two_ranks(mode):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    _spawn(2, mode)
