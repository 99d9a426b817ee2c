"""The fused small-model kernel (b200_block_fused_small_launch) against the oracle and the chain.

Shapes: BASELINE configs 1-3 (d=128, H=4, ffn=512, S=128), ragged S, several
sequences per persistent CTA (B > 148), and the reference's own official
matrix shape (L=4, ffn=d=128; run_eval.sh:44-58), which the fused kernel runs
with the residual kept on chip across layers.
"""

import numpy as np
import pytest
import torch

import oracle

pytestmark = pytest.mark.gpu

ATOL, RTOL = 0.002, 0.02
DEV = "cuda"

CASES = [  # B, S, ffn, L
    (4, 128, 512, 1),
    (64, 128, 512, 1),
    (3, 100, 512, 1),
    (2, 37, 256, 1),
    (300, 128, 512, 1),
    (64, 128, 128, 4),
    (5, 64, 384, 2),
]


@pytest.mark.parametrize("B,S,F,L", CASES, ids=[f"B{c[0]}_S{c[1]}_F{c[2]}_L{c[3]}" for c in CASES])
def test_fused_small_vs_oracle(tt, B, S, F, L):
    cfg = tt.TransformerConfig(B, S, 128, 4, F, L, True)
    torch.manual_seed(1234 + L)
    model = tt.UserOptimizedTransformer(cfg).to(DEV).eval()
    x, mask = oracle.generate_random_case(B, S, 128, 1234 + B)
    with torch.inference_mode():
        y = model(x.to(DEV), mask.to(DEV)).cpu()
    assert model.last_strategy == "fused_small"
    rt = tt._pkg.runtime
    assert rt.device_error(clear=True) == 0
    nb = min(B, 16)
    ref = oracle.model_forward(oracle.params_from_state_dict(model.state_dict()),
                               oracle.OracleConfig(nb, S, 128, 4, F, L, True), x[:nb].numpy())
    res = oracle.compare_outputs(ref, y[:nb], rtol=RTOL, atol=ATOL)
    print(f"B{B} S{S} F{F} L{L}: max_abs={res.max_abs_error:.3g}")
    assert res.passed, res
    if B > 16:  # the last sequences too (other persistent-CTA iterations)
        ref2 = oracle.model_forward(oracle.params_from_state_dict(model.state_dict()),
                                    oracle.OracleConfig(8, S, 128, 4, F, L, True), x[B - 8:].numpy())
        assert oracle.compare_outputs(ref2, y[B - 8:], rtol=RTOL, atol=ATOL).passed


def test_fused_equals_chain_within_tolerance(tt):
    cfg = tt.TransformerConfig(32, 128, 128, 4, 512, 1, True)
    torch.manual_seed(7)
    model = tt.UserOptimizedTransformer(cfg).to(DEV).eval()
    x, mask = oracle.generate_random_case(32, 128, 128, 8)
    xd, md = x.to(DEV), mask.to(DEV)
    with torch.inference_mode():
        model.force_strategy = "fused_small"
        y_f = model(xd, md).clone()
        model.force_strategy = "chain"
        y_c = model(xd, md).clone()
    torch.cuda.synchronize()
    assert oracle.compare_outputs(y_c.cpu(), y_f.cpu(), rtol=RTOL, atol=ATOL).passed


def test_fused_repeatable_and_graph_replay(tt):
    cfg = tt.TransformerConfig(64, 128, 128, 4, 512, 1, True)
    torch.manual_seed(11)
    model = tt.UserOptimizedTransformer(cfg).to(DEV).eval()
    x, mask = oracle.generate_random_case(64, 128, 128, 12)
    xd, md = x.to(DEV), mask.to(DEV)
    with torch.inference_mode():
        outs = [model(xd, md).clone() for _ in range(4)]  # eager, capture, replay, replay
    torch.cuda.synchronize()
    for o in outs[1:]:
        assert torch.equal(o, outs[0])


@pytest.mark.parametrize("B,S,F,L", [(4, 128, 512, 1), (3, 70, 256, 2)])
def test_fused_small_noncausal(tt, B, S, F, L):
    cfg = tt.TransformerConfig(B, S, 128, 4, F, L, False)
    torch.manual_seed(3)
    model = tt.UserOptimizedTransformer(cfg).to(DEV).eval()
    x, mask = oracle.generate_random_case(B, S, 128, 4, padding_ratio=0.3)
    for m in (None, mask):
        with torch.inference_mode():
            y = model(x.to(DEV), None if m is None else m.to(DEV)).cpu()
        assert model.last_strategy == "fused_small"
        ref = oracle.model_forward(oracle.params_from_state_dict(model.state_dict()),
                                   oracle.OracleConfig(B, S, 128, 4, F, L, False), x.numpy(),
                                   None if m is None else m.numpy())
        assert oracle.compare_outputs(ref, y, rtol=RTOL, atol=ATOL).passed


@pytest.mark.parametrize("mode", ["0", "1"])
def test_fused_single_and_row_split_in_subprocess(mode):
    """The one-CTA-per-sequence kernel and the row-split kernel (two CTAs per
    sequence, each finishing half of the query rows; B200_SMALL_ROWS forces the
    choice and is read once per process, hence the child process) against the
    oracle: ffn 128-512, ragged S, key padding, non-causal, more sequences than
    SMs, and a two-layer model (always the one-CTA kernel)."""
    import os
    import subprocess
    import sys
    code = r'''
import torch
import oracle
import torch_transformer_benchmark as tt
rt = tt._pkg.runtime
DEV = "cuda"
for (B, S, F, L, causal, pad) in ((4, 128, 512, 1, True, 0.0), (64, 128, 512, 1, True, 0.0),
                                  (3, 100, 512, 1, True, 0.0), (2, 37, 256, 1, True, 0.0),
                                  (5, 128, 128, 1, True, 0.25), (6, 120, 384, 1, True, 0.2),
                                  (3, 70, 512, 1, False, 0.3), (4, 128, 256, 1, False, 0.0),
                                  (300, 128, 512, 1, True, 0.0), (3, 128, 512, 2, True, 0.0)):
    cfg = tt.TransformerConfig(B, S, 128, 4, F, L, causal)
    torch.manual_seed(B * 7 + L + F)
    model = tt.UserOptimizedTransformer(cfg).to(DEV).eval()
    x, mask = oracle.generate_random_case(B, S, 128, B + S + F, padding_ratio=pad)
    m = mask if pad > 0 else None
    with torch.inference_mode():
        y = model(x.to(DEV), None if m is None else m.to(DEV)).cpu()
    assert model.last_strategy == "fused_small"
    assert rt.device_error(clear=True) == 0
    params = oracle.params_from_state_dict(model.state_dict())
    for lo, hi in ((0, min(B, 8)), (max(B - 4, 0), B)):
        ref = oracle.model_forward(params, oracle.OracleConfig(hi - lo, S, 128, 4, F, L, causal), x[lo:hi].numpy(),
                                   None if m is None else m[lo:hi].numpy())
        res = oracle.compare_outputs(ref, y[lo:hi], rtol=0.02, atol=0.002)
        assert res.passed, (B, S, F, L, causal, pad, res)
print("OK")
'''
    env = dict(os.environ, B200_SMALL_ROWS=mode)
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    r = subprocess.run([sys.executable, "-c", code], cwd=root, env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0 and "OK" in r.stdout, r.stdout[-3000:] + r.stderr[-3000:]


@pytest.mark.parametrize("mode", ["0", "1"])
def test_fused_one_and_two_heads_in_subprocess(mode):
    """d_model = 128 with 1 or 2 heads (head_dim 128 / 64: S = Q.K^T over 8 / 4
    K-steps, P.V into 4 / 2 32-column blocks per head) in the one-CTA and the
    row-split kernel against the oracle: the reference matrix's shapes (4 layers,
    ffn = d), ragged S with key padding, non-causal, ffn 512."""
    import os
    import subprocess
    import sys
    code = r'''
import torch
import oracle
import torch_transformer_benchmark as tt
rt = tt._pkg.runtime
DEV = "cuda"
for (B, S, H, F, L, causal, pad) in ((64, 128, 1, 128, 4, True, 0.0), (64, 128, 2, 128, 4, True, 0.0),
                                     (5, 100, 1, 512, 1, True, 0.25), (6, 128, 2, 256, 1, True, 0.0),
                                     (3, 77, 2, 384, 1, False, 0.3), (4, 128, 1, 128, 1, False, 0.0),
                                     (200, 128, 2, 512, 1, True, 0.0), (3, 64, 1, 256, 2, True, 0.0)):
    cfg = tt.TransformerConfig(B, S, 128, H, F, L, causal)
    torch.manual_seed(B * 11 + H + F + L)
    model = tt.UserOptimizedTransformer(cfg).to(DEV).eval()
    x, mask = oracle.generate_random_case(B, S, 128, B + S + F + H, padding_ratio=pad)
    m = mask if pad > 0 else None
    with torch.inference_mode():
        y = model(x.to(DEV), None if m is None else m.to(DEV)).cpu()
    assert model.last_strategy == "fused_small"
    assert rt.device_error(clear=True) == 0
    params = oracle.params_from_state_dict(model.state_dict())
    for lo, hi in ((0, min(B, 8)), (max(B - 4, 0), B)):
        ref = oracle.model_forward(params, oracle.OracleConfig(hi - lo, S, 128, H, F, L, causal), x[lo:hi].numpy(),
                                   None if m is None else m[lo:hi].numpy())
        res = oracle.compare_outputs(ref, y[lo:hi], rtol=0.02, atol=0.002)
        assert res.passed, (B, S, H, F, L, causal, pad, res)
print("OK")
'''
    env = dict(os.environ, B200_SMALL_ROWS=mode)
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    r = subprocess.run([sys.executable, "-c", code], cwd=root, env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0 and "OK" in r.stdout, r.stdout[-3000:] + r.stderr[-3000:]


TINY_CASES = [  # B, S, H, ffn, L, causal, padding ratio
    (64, 128, 4, 32, 4, True, 0.0),   # the reference's official matrix row 7
    (3, 100, 2, 64, 2, True, 0.0),
    (5, 128, 1, 128, 1, True, 0.25),
    (4, 77, 4, 96, 3, False, 0.3),
    (200, 128, 4, 32, 1, True, 0.0),
]


@pytest.mark.parametrize("B,S,H,F,L,causal,pad", TINY_CASES,
                         ids=[f"B{c[0]}_S{c[1]}_H{c[2]}_F{c[3]}_L{c[4]}_{'c' if c[5] else 'nc'}" for c in TINY_CASES])
def test_tiny_model_single_kernel_vs_oracle(tt, B, S, H, F, L, causal, pad):
    """d_model = 32 runs as one CUDA-core kernel (fused_tiny.cuh) for the whole model."""
    cfg = tt.TransformerConfig(B, S, 32, H, F, L, causal)
    torch.manual_seed(B + H + F + L)
    model = tt.UserOptimizedTransformer(cfg).to(DEV).eval()
    x, mask = oracle.generate_random_case(B, S, 32, B * 3 + S, padding_ratio=pad)
    m = mask if pad > 0 else None
    with torch.inference_mode():
        y = model(x.to(DEV), None if m is None else m.to(DEV)).cpu()
    assert model.last_strategy == "fused_small"
    assert tt._pkg.runtime.device_error(clear=True) == 0
    nb = min(B, 16)
    ref = oracle.model_forward(oracle.params_from_state_dict(model.state_dict()),
                               oracle.OracleConfig(nb, S, 32, H, F, L, causal), x[:nb].numpy(),
                               None if m is None else m[:nb].numpy())
    res = oracle.compare_outputs(ref, y[:nb], rtol=RTOL, atol=ATOL)
    print(f"tiny B{B} S{S} H{H} F{F} L{L}: max_abs={res.max_abs_error:.3g}")
    assert res.passed, res


@pytest.mark.parametrize("mode", ["0", "1"])
def test_tiny_single_cta_and_cluster_split_in_subprocess(mode):
    """d_model = 32 with one CTA per sequence and with a two-CTA cluster per
    sequence (each half finishing 64 query rows, K / V rows exchanged through
    distributed shared memory; B200_TINY_SPLIT forces the choice and is read once
    per process, hence the child process) against the oracle: 1, 2 and 4 heads,
    several layers (the exchange buffers alternate by layer), ragged S, key
    padding, non-causal, and more clusters than fit on the GPU at once."""
    import os
    import subprocess
    import sys
    code = r'''
import torch
import oracle
import torch_transformer_benchmark as tt
rt = tt._pkg.runtime
DEV = "cuda"
for (B, S, H, F, L, causal, pad) in ((64, 128, 4, 32, 4, True, 0.0), (3, 100, 2, 64, 3, True, 0.0),
                                     (5, 128, 1, 128, 2, True, 0.25), (4, 77, 4, 96, 3, False, 0.3),
                                     (2, 33, 4, 32, 5, True, 0.0), (160, 128, 4, 64, 2, True, 0.1)):
    cfg = tt.TransformerConfig(B, S, 32, H, F, L, causal)
    torch.manual_seed(B * 5 + H + F + L)
    model = tt.UserOptimizedTransformer(cfg).to(DEV).eval()
    x, mask = oracle.generate_random_case(B, S, 32, B + S + F + L, padding_ratio=pad)
    m = mask if pad > 0 else None
    with torch.inference_mode():
        y = model(x.to(DEV), None if m is None else m.to(DEV)).cpu()
    assert model.last_strategy == "fused_small"
    assert rt.device_error(clear=True) == 0
    params = oracle.params_from_state_dict(model.state_dict())
    for lo, hi in ((0, min(B, 8)), (max(B - 4, 0), B)):
        ref = oracle.model_forward(params, oracle.OracleConfig(hi - lo, S, 32, H, F, L, causal), x[lo:hi].numpy(),
                                   None if m is None else m[lo:hi].numpy())
        res = oracle.compare_outputs(ref, y[lo:hi], rtol=0.02, atol=0.002)
        assert res.passed, (B, S, H, F, L, causal, pad, res)
print("OK")
'''
    env = dict(os.environ, B200_TINY_SPLIT=mode)
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    r = subprocess.run([sys.executable, "-c", code], cwd=root, env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0 and "OK" in r.stdout, r.stdout[-3000:] + r.stderr[-3000:]
