"""BASELINE configuration 5 (and official-matrix row 14) at full shape on a B200: every output element checked.

B=32, S=100000, d=1024, H=16 (head_dim 64), ffn=4096, one causal layer (row 14:
two layers, ffn=1024).  The
module's forward over the whole batch is compared, element by element with the
reference harness's rule (atol 0.002 OR rtol 0.02, TTB:1821-1888), against an
fp32 forward assembled from exact batch slices -- one sequence at a time, as
the reference's own full-shape check does (experiments/g7_0_chunked_oversize.py:
588-660, check 8).  The fp32 forward is plain PyTorch on the same device with
TF32 off: LayerNorm / Linear / erf-GELU in fp32 and causal attention through
the memory-efficient fp32 kernel (the reference's fp32 chunked path uses that
kernel too, TTB:1502-1519), so no S x S score matrix is formed.  It is the
checker, not the thing measured.  Inputs are drawn on the device from a seeded
generator (13 GB; both sides read the same tensor).
"""

import pytest
import torch
import torch.nn.functional as F

import oracle

pytestmark = pytest.mark.gpu

ATOL, RTOL = 0.002, 0.02
DEV = "cuda"


def _fp32_block(model, x):
    """One sequence [S, d] through the fp32 model: pre-LN blocks, then the final norm (TTB:154-192)."""
    for L in model.layers:
        x = _fp32_layer(L, x)
    return F.layer_norm(x, (x.shape[1],), model.final_norm.weight, model.final_norm.bias, model.final_norm.eps)


def _fp32_layer(L, x):
    at = L.attention
    S, d = x.shape
    H, hd = at.num_heads, at.head_dim
    n1 = F.layer_norm(x, (d,), L.norm1.weight, L.norm1.bias, L.norm1.eps)
    split = lambda t: t.view(1, S, H, hd).transpose(1, 2)  # noqa: E731
    q = split(F.linear(n1, at.q_proj.weight, at.q_proj.bias))
    k = split(F.linear(n1, at.k_proj.weight, at.k_proj.bias))
    v = split(F.linear(n1, at.v_proj.weight, at.v_proj.bias))
    del n1
    from torch.nn.attention import SDPBackend, sdpa_kernel
    with sdpa_kernel(SDPBackend.EFFICIENT_ATTENTION):
        ctx = F.scaled_dot_product_attention(q, k, v, is_causal=True)
    del q, k, v
    ctx = ctx.transpose(1, 2).reshape(S, d)
    x1 = x + F.linear(ctx, at.out_proj.weight, at.out_proj.bias)
    del ctx
    h = F.gelu(F.linear(F.layer_norm(x1, (d,), L.norm2.weight, L.norm2.bias, L.norm2.eps),
                        L.ffn_in.weight, L.ffn_in.bias), approximate="none")
    x2 = x1 + F.linear(h, L.ffn_out.weight, L.ffn_out.bias)
    del h, x1
    return x2


# BASELINE configuration 5 (one layer, ffn 4096) and row 14 of the reference's official
# matrix (two layers, ffn 1024; README.md:59), both B=32 S=100000 d=1024 H=16
FULL = [("C5", 32, 100000, 1024, 16, 4096, 1), ("row14", 32, 100000, 1024, 16, 1024, 2)]


@pytest.mark.parametrize("name,B,S,d,H,Fd,L", FULL, ids=[f[0] for f in FULL])
def test_c5_full_shape_every_element(tt, name, B, S, d, H, Fd, L):
    free, _ = torch.cuda.mem_get_info()
    if free < 120 * (1 << 30):
        pytest.skip("needs ~120 GB of free device memory (a whole B200)")
    cfg = tt.TransformerConfig(B, S, d, H, Fd, L, True)
    torch.manual_seed(1234)
    model = tt.UserOptimizedTransformer(cfg).to(DEV).eval()
    gen = torch.Generator(device=DEV).manual_seed(1234 + 5)
    x = torch.randn(B, S, d, generator=gen, device=DEV)
    mask = torch.ones(B, S, dtype=torch.bool, device=DEV)
    with torch.inference_mode():
        y = model(x, mask)
    torch.cuda.synchronize()
    assert model.last_strategy == "chain"
    model._ws.clear()  # release the 72 GB workspace before the reference runs
    torch.cuda.empty_cache()
    tf32 = (torch.backends.cuda.matmul.allow_tf32, torch.backends.cudnn.allow_tf32)
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.backends.cudnn.allow_tf32 = False
    failed, worst, worst_rel = 0, 0.0, 0.0
    try:
        with torch.inference_mode():
            for b in range(B):
                ref = _fp32_block(model, x[b])
                diff = (y[b] - ref).abs()
                bad = ~((diff <= ATOL) | (diff <= RTOL * ref.abs()))
                failed += int(bad.sum())
                worst = max(worst, float(diff.max()))
                worst_rel = max(worst_rel, float((diff / ref.abs().clamp_min(1e-6)).max()))
                assert torch.isfinite(y[b]).all()
                del ref, diff, bad
    finally:
        torch.backends.cuda.matmul.allow_tf32, torch.backends.cudnn.allow_tf32 = tf32
    print(f"{name} full shape: {B * S * d} elements, failed {failed}, max_abs {worst:.3g}, max_rel {worst_rel:.3g}")
    assert failed == 0, (failed, worst)
    assert worst < ATOL


def test_c5_slice_matches_the_chunked_restatement(tt):
    """The same check on one query chunk against the NumPy oracle (oracle.chunk_rows_forward),
    which pins the fp32 torch checker above to the restatement of the reference."""
    B, S, d, H, Fd = 2, 20000, 1024, 16, 4096
    cfg = tt.TransformerConfig(B, S, d, H, Fd, 1, True)
    torch.manual_seed(1234)
    model = tt.UserOptimizedTransformer(cfg).to(DEV).eval()
    gen = torch.Generator(device=DEV).manual_seed(99)
    x = torch.randn(B, S, d, generator=gen, device=DEV)
    tf32 = (torch.backends.cuda.matmul.allow_tf32, torch.backends.cudnn.allow_tf32)
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.backends.cudnn.allow_tf32 = False
    try:
        with torch.inference_mode():
            y = model(x).cpu()
            ref_t = _fp32_block(model, x[1]).cpu()
    finally:
        torch.backends.cuda.matmul.allow_tf32, torch.backends.cudnn.allow_tf32 = tf32
    c0, c1 = S - 512, S
    ref_np = oracle.chunk_rows_forward(oracle.params_from_state_dict(model.state_dict()), H,
                                       x[1, :c1].cpu().numpy(), c0, c1)
    pin = oracle.compare_outputs(ref_np, ref_t[c0:c1].numpy(), rtol=5e-3, atol=5e-4)
    print(f"fp32 torch checker vs NumPy oracle: max_abs {pin.max_abs_error:.3g}")
    assert pin.passed, pin
    res = oracle.compare_outputs(ref_np, y[1, c0:c1], rtol=RTOL, atol=ATOL)
    assert res.passed, res
