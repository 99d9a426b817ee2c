"""The PyTorch op layer on a B200: opcheck (schema, fake impl, autograd
registration), values against torch fp32, and torch.compile(fullgraph=True)
tracing the ops the way the reference's reduce-overhead compile traced its
custom ops (torch_transformer_benchmark.py:292-327)."""

import math

import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.fixture(scope="module")
def ops(pkg):
    torch.backends.cuda.matmul.allow_tf32 = False
    return pkg.ops


def _rand(g, *shape, scale=1.0, dtype=torch.float32):
    return (torch.randn(*shape, generator=g) * scale).to(dtype).to(DEV)


def test_opcheck_linear_layernorm_attention(ops):
    g = torch.Generator().manual_seed(1)
    a = _rand(g, 256, 128, dtype=torch.float16)
    w = _rand(g, 384, 128, scale=1 / math.sqrt(128), dtype=torch.float16)
    b = _rand(g, 384)
    torch.library.opcheck(torch.ops.b200.linear.default, (a, w, b, ops.EPI_BIAS_F16))
    torch.library.opcheck(torch.ops.b200.linear_residual.default, (a, w, b, _rand(g, 256, 384)))
    x = _rand(g, 300, 128)
    torch.library.opcheck(torch.ops.b200.layernorm.default, (x, _rand(g, 128), _rand(g, 128), 1e-5, True))
    q = _rand(g, 2, 160, 128, dtype=torch.float16)
    torch.library.opcheck(torch.ops.b200.flash_causal.default, (q, q, q, 4, 0, False, None))


def test_linear_values(ops):
    g = torch.Generator().manual_seed(2)
    a = _rand(g, 300, 256, dtype=torch.float16)
    w = _rand(g, 512, 256, scale=1 / 16, dtype=torch.float16)
    b = _rand(g, 512)
    ref = a.float() @ w.float().T + b
    y = torch.ops.b200.linear(a, w, b, ops.EPI_BIAS_GELU_F16)
    assert (y.float() - torch.nn.functional.gelu(ref)).abs().max().item() < 2e-3
    r = _rand(g, 300, 512)
    y2 = torch.ops.b200.linear_residual(a, w, b, r)
    assert (y2 - (ref + r)).abs().max().item() < 1e-3
    out = r.clone()
    torch.ops.b200.gemm_out(a, w, b, ops.EPI_BIAS_RESID_F32, out)
    assert torch.equal(out, y2)
    w128 = _rand(g, 128, 256, scale=1 / 16, dtype=torch.float16)
    b128, r128 = _rand(g, 128), _rand(g, 300, 128)
    gam, bet = _rand(g, 128), _rand(g, 128)
    x1, n = torch.ops.b200.linear_residual_layernorm(a, w128, b128, r128, gam, bet, 1e-5)
    ref1 = r128 + a.float() @ w128.float().T + b128
    assert (x1 - ref1).abs().max().item() < 1e-3
    ref_n = torch.nn.functional.layer_norm(ref1, (128,), gam, bet, eps=1e-5)
    assert (n.float() - ref_n).abs().max().item() < 2e-2


def test_compiled_block_matches_eager(ops, pkg):
    """A pre-LN block written with the ops, compiled with fullgraph=True, equals the
    same function run eagerly (both run the library's kernels)."""
    import torch_transformer_benchmark as T
    cfg = T.TransformerConfig(2, 256, 256, 4, 1024, 1, True)
    torch.manual_seed(0)
    m = T.UserOptimizedTransformer(cfg).to(DEV).eval()
    m._ensure_packs(torch.device(DEV))
    pk = m._packs[0]
    lnf_w, lnf_b = m._lnf

    def block(x):
        B, S, d = x.shape
        x2 = x.reshape(B * S, d)
        n = torch.ops.b200.layernorm(x2, pk.ln1_w, pk.ln1_b, 1e-5, True)
        qkv = torch.ops.b200.linear(n, pk.w_qkv, pk.b_qkv, ops.EPI_BIAS_F16).view(B, S, 3 * d)
        ctx = torch.ops.b200.flash_causal(qkv[..., :d], qkv[..., d:2 * d], qkv[..., 2 * d:], 4, 0, False, None)
        x1 = torch.ops.b200.linear_residual(ctx.reshape(B * S, d), pk.w_o, pk.b_o, x2)
        h = torch.ops.b200.linear(torch.ops.b200.layernorm(x1, pk.ln2_w, pk.ln2_b, 1e-5, True), pk.w_in, pk.b_in,
                                  ops.EPI_BIAS_GELU_F16)
        x2n = torch.ops.b200.linear_residual(h, pk.w_out, pk.b_out, x1)
        return torch.ops.b200.layernorm(x2n, lnf_w, lnf_b, 1e-5, False).view(B, S, d)

    x = torch.randn(2, 256, 256, device=DEV)
    with torch.inference_mode():
        eager = block(x)
        compiled = torch.compile(block, fullgraph=True)(x)
        model_y = m(x)
    torch.cuda.synchronize()
    assert torch.equal(eager, compiled)
    # the module's own chain computes the same block (same kernels, same order of additions)
    assert (eager - model_y).abs().max().item() < 2e-3


def test_block_megakernel_op_matches_model(ops, pkg):
    import torch_transformer_benchmark as T
    cfg = T.TransformerConfig(8, 128, 128, 4, 512, 2, True)
    torch.manual_seed(3)
    m = T.UserOptimizedTransformer(cfg).to(DEV).eval()
    m.force_strategy = "fused_small"
    m._ensure_packs(torch.device(DEV))
    st = m._stack
    x = torch.randn(8, 128, 128, device=DEV)
    with torch.inference_mode():
        y_model = m(x)
        y_op = torch.ops.b200.block_megakernel(x, st["ln1_w"], st["ln1_b"], st["w_qkv"], st["b_qkv"], st["w_o"],
                                               st["b_o"], st["ln2_w"], st["ln2_b"], st["w_in"], st["b_in"],
                                               st["w_out"], st["b_out"], m._lnf[0], m._lnf[1], 4, 1e-5, True, None)
    torch.cuda.synchronize()
    assert torch.equal(y_model, y_op)


def test_kv_write_chunks_equal_full_projection(ops):
    """K|V of three chunks written at their cache rows equal the whole projection;
    rows outside the written range are untouched."""
    g = torch.Generator().manual_seed(5)
    d, S = 128, 700
    a = _rand(g, S, d, dtype=torch.float16)
    w = _rand(g, 2 * d, d, scale=1 / math.sqrt(d), dtype=torch.float16)
    b = _rand(g, 2 * d)
    cache = torch.full((S + 50, 2 * d), 7.0, dtype=torch.float16, device=DEV)
    for r0, r1 in ((0, 256), (256, 512), (512, S)):
        torch.ops.b200.kv_write(a[r0:r1], w, b, cache, r0)
    torch.library.opcheck(torch.ops.b200.kv_write.default, (a[:64], w, b, cache.clone(), 10))
    ref = a.float() @ w.float().T + b
    torch.cuda.synchronize()
    assert (cache[:S].float() - ref).abs().max().item() < 2e-3
    assert bool((cache[S:] == 7.0).all())
