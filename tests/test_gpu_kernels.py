"""Kernel-level checks on a B200, through the C ABI.

The patterns follow the reference's kernel probes
(experiments/g4_7_ffn_gelu_correctness.py:100-150): exact-integer operands
(every fp32 partial sum exact, so the GEMM must be bit-exact), a one-hot index
sweep (catches transposed / swizzled indexing), and seeded random operands
against a torch fp32 reference of the same op (TF32 off).
"""

import math

import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = "cuda"


@pytest.fixture(scope="module")
def rt(pkg):
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.backends.cudnn.allow_tf32 = False
    r = pkg.runtime
    r.lib()
    assert r.device_error(clear=True) == 0
    yield r
    assert r.device_error(clear=True) == 0


def _ints(shape, lo, hi, gen):
    return torch.randint(lo, hi + 1, shape, generator=gen).to(torch.float16).to(DEV)


GEMM_SHAPES = [(256, 384, 128), (300, 96, 520), (1000, 512, 64), (8192, 3072, 1024), (129, 4096, 1024)]


@pytest.mark.parametrize("M,N,K", GEMM_SHAPES)
def test_gemm_exact_integer_f16(rt, M, N, K):
    g = torch.Generator().manual_seed(M * 7 + N)
    a = _ints((M, K), -1, 1, g)
    w = _ints((N, K), -1, 1, g)
    bias = torch.randint(-4, 5, (N,), generator=g).float().to(DEV)
    out = torch.empty(M, N, dtype=torch.float16, device=DEV)
    rt.gemm(rt.EPI_BIAS_F16, a, w, bias, out)
    ref = (a.double() @ w.double().T + bias.double())
    assert ref.abs().max() <= 2048  # exactly representable in fp16
    torch.cuda.synchronize()
    assert torch.equal(out.double(), ref)


@pytest.mark.parametrize("M,N,K", GEMM_SHAPES[:4])
def test_gemm_exact_integer_resid_f32(rt, M, N, K):
    g = torch.Generator().manual_seed(M + N * 3)
    a = _ints((M, K), -2, 2, g)
    w = _ints((N, K), -2, 2, g)
    bias = torch.randint(-4, 5, (N,), generator=g).float().to(DEV)
    resid = torch.randint(-100, 101, (M, N), generator=g).float().to(DEV)
    out = torch.empty(M, N, dtype=torch.float32, device=DEV)
    rt.gemm(rt.EPI_BIAS_RESID_F32, a, w, bias, out, resid=resid)
    ref = a.double() @ w.double().T + bias.double() + resid.double()
    torch.cuda.synchronize()
    assert torch.equal(out.double(), ref)
    # in place: out aliases resid
    rt.gemm(rt.EPI_BIAS_RESID_F32, a, w, bias, resid, resid=resid)
    torch.cuda.synchronize()
    assert torch.equal(resid.double(), ref)


@pytest.mark.parametrize("M,N,K", [(300, 96, 520), (1000, 512, 64), (256, 4096, 128)])
def test_gemm_exact_integer_f32_into_column_slice(rt, M, N, K):
    """EPI_BIAS_F32 into columns [32, 32+N) of a wider buffer: exact values in
    the slice (the TMA store box clips at M and N), nothing written outside."""
    g = torch.Generator().manual_seed(M + 11 * N)
    a = _ints((M, K), -2, 2, g)
    w = _ints((N, K), -2, 2, g)
    bias = torch.randint(-4, 5, (N,), generator=g).float().to(DEV)
    wide = torch.full((M, N + 96), 7.0, dtype=torch.float32, device=DEV)
    out = wide[:, 32:32 + N]
    rt.gemm(rt.EPI_BIAS_F32, a, w, bias, out)
    ref = a.double() @ w.double().T + bias.double()
    torch.cuda.synchronize()
    assert torch.equal(out.double(), ref)
    assert (wide[:, :32] == 7.0).all() and (wide[:, 32 + N:] == 7.0).all()


def test_gemm_f16_into_column_slice(rt):
    M, N, K = 777, 160, 256
    g = torch.Generator().manual_seed(3)
    a = _ints((M, K), -1, 1, g)
    w = _ints((N, K), -1, 1, g)
    wide = torch.full((M, 3 * N), -3.0, dtype=torch.float16, device=DEV)
    out = wide[:, N:2 * N]
    rt.gemm(rt.EPI_BIAS_F16, a, w, None, out)
    torch.cuda.synchronize()
    assert torch.equal(out.double(), a.double() @ w.double().T)
    assert (wide[:, :N] == -3.0).all() and (wide[:, 2 * N:] == -3.0).all()


@pytest.mark.parametrize("M,N,K", [(512, 256, 128), (384, 128, 1024)])
def test_gemm_one_hot_index_sweep(rt, M, N, K):
    g = torch.Generator().manual_seed(5)
    a = torch.zeros(M, K, dtype=torch.float16)
    a[torch.arange(M), (torch.arange(M) * 7) % K] = 1
    a = a.to(DEV)
    w = torch.randn(N, K, generator=g).to(torch.float16).to(DEV)
    out = torch.empty(M, N, dtype=torch.float16, device=DEV)
    rt.gemm(rt.EPI_BIAS_F16, a, w, None, out)
    ref = w.T[(torch.arange(M) * 7) % K]
    torch.cuda.synchronize()
    assert torch.equal(out, ref)


def test_gemm_gelu_matches_torch(rt):
    M, N, K = 2048, 512, 128
    g = torch.Generator().manual_seed(9)
    a = torch.randn(M, K, generator=g).to(torch.float16).to(DEV)
    w = (torch.randn(N, K, generator=g) / math.sqrt(K)).to(torch.float16).to(DEV)
    bias = torch.randn(N, generator=g).to(DEV)
    out = torch.empty(M, N, dtype=torch.float16, device=DEV)
    rt.gemm(rt.EPI_BIAS_GELU_F16, a, w, bias, out)
    ref = torch.nn.functional.gelu(a.float() @ w.float().T + bias, approximate="none")
    torch.cuda.synchronize()
    err = (out.float() - ref).abs()
    # fp16 output rounding (half an ulp) plus fp32 summation-order differences
    assert (err <= 1e-3 + 1e-3 * ref.abs()).all(), err.max().item()


@pytest.mark.parametrize("M,N,K", [(4096, 384, 128), (1000, 1024, 4096)])
def test_gemm_random_vs_torch_fp32(rt, M, N, K):
    g = torch.Generator().manual_seed(M)
    a = torch.randn(M, K, generator=g).to(torch.float16).to(DEV)
    w = (torch.randn(N, K, generator=g) / math.sqrt(K)).to(torch.float16).to(DEV)
    bias = torch.randn(N, generator=g).to(DEV)
    resid = torch.randn(M, N, generator=g).to(DEV)
    out = torch.empty(M, N, dtype=torch.float32, device=DEV)
    rt.gemm(rt.EPI_BIAS_RESID_F32, a, w, bias, out, resid=resid)
    ref = a.float() @ w.float().T + bias + resid
    torch.cuda.synchronize()
    assert (out - ref).abs().max().item() < 1e-4 * math.sqrt(K)


@pytest.mark.parametrize("d", [64, 96, 128, 1024])
@pytest.mark.parametrize("f16", [True, False])
def test_layernorm_vs_torch(rt, d, f16):
    g = torch.Generator().manual_seed(d)
    rows = 1531
    x = (torch.randn(rows, d, generator=g) * 3 + 1).to(DEV)
    gamma = torch.randn(d, generator=g).to(DEV)
    beta = torch.randn(d, generator=g).to(DEV)
    out = torch.empty(rows, d, dtype=torch.float16 if f16 else torch.float32, device=DEV)
    rt.layernorm(x, gamma, beta, out, eps=1e-5)
    ref = torch.nn.functional.layer_norm(x, (d,), gamma, beta, eps=1e-5)
    torch.cuda.synchronize()
    tol = 2e-3 if f16 else 2e-5
    assert ((out.float() - ref).abs() <= tol * (1 + ref.abs())).all()


@pytest.mark.parametrize("d", [96, 1024])
def test_layernorm_residual_copy(rt, d):
    """norm1 with the residual copy: out as without it, residual_out == x exactly."""
    g = torch.Generator().manual_seed(d + 1)
    rows = 1000
    x = (torch.randn(rows, d, generator=g) * 2).to(DEV)
    gamma = torch.randn(d, generator=g).to(DEV)
    beta = torch.randn(d, generator=g).to(DEV)
    out = torch.empty(rows, d, dtype=torch.float16, device=DEV)
    out_plain = torch.empty_like(out)
    res = torch.full((rows, d), float("nan"), device=DEV)
    rt.layernorm(x, gamma, beta, out, eps=1e-5, residual_out=res)
    rt.layernorm(x, gamma, beta, out_plain, eps=1e-5)
    torch.cuda.synchronize()
    assert torch.equal(res, x)
    assert torch.equal(out, out_plain)


def _attn_ref(q, k, v, q_offset):
    # q [B,H,Sq,hd], k/v [B,H,Sk,hd] fp32
    hd = q.shape[-1]
    s = (q @ k.transpose(-1, -2)) * hd ** -0.5
    Sq, Sk = q.shape[-2], k.shape[-2]
    qpos = q_offset + torch.arange(Sq, device=q.device)[:, None]
    kpos = torch.arange(Sk, device=q.device)[None, :]
    s = s.masked_fill(kpos > qpos, float("-inf"))
    return torch.softmax(s, dim=-1) @ v


ATTN_CASES = [  # B, H, S, hd
    (2, 4, 128, 32), (3, 2, 100, 32), (2, 4, 384, 64), (1, 2, 300, 128), (2, 4, 128, 256), (1, 2, 200, 256),
    (2, 4, 1024, 32),
    (1, 2, 2304, 64), (2, 2, 2100, 32),  # long rows; two query tiles per CTA only when forced (below)
    (2, 4, 128, 8), (3, 16, 100, 8), (2, 8, 300, 16), (1, 4, 1000, 8),  # head_dim 8 / 16: CUDA-core kernel
]


@pytest.mark.parametrize("B,H,S,hd", ATTN_CASES)
def test_flash_causal_vs_torch(rt, B, H, S, hd):
    g = torch.Generator().manual_seed(B * 1000 + S + hd)
    d = H * hd
    qkv = (torch.randn(B * S, 3 * d, generator=g)).to(torch.float16).to(DEV)
    out = torch.full((B * S, d), float("nan"), dtype=torch.float16, device=DEV)
    rt.flash_causal(qkv, qkv, qkv, out, batch=B, heads=H, head_dim=hd, q_len=S, kv_len=S, k_col0=d, v_col0=2 * d)
    t = qkv.float().view(B, S, 3, H, hd).permute(2, 0, 3, 1, 4)
    ref = _attn_ref(t[0], t[1], t[2], 0).permute(0, 2, 1, 3).reshape(B * S, d)
    torch.cuda.synchronize()
    err = (out.float() - ref).abs().max().item()
    assert err < 4e-3, err


@pytest.mark.parametrize("hd,chunk,S", [(64, 256, 640), (32, 128, 640), (64, 192, 640), (256, 128, 640),
                                        (64, 2048, 4352), (32, 2176, 4352), (8, 192, 640), (16, 256, 700)])
def test_flash_prefix_chunks_equal_full(rt, hd, chunk, S):
    """Query chunks [c0:c1) over the K/V prefix [0:c1) (q_offset=c0) reproduce
    full causal attention row for row -- the chunked forward's identity."""
    B, H = 2, 2
    d = H * hd
    g = torch.Generator().manual_seed(hd + chunk)
    q = torch.randn(B * S, d, generator=g).to(torch.float16).to(DEV)
    kv = torch.randn(B * S, 2 * d, generator=g).to(torch.float16).to(DEV)
    full = torch.empty(B * S, d, dtype=torch.float16, device=DEV)
    rt.flash_causal(q, kv, kv, full, batch=B, heads=H, head_dim=hd, q_len=S, kv_len=S, k_col0=0, v_col0=d)
    parts = torch.empty_like(full)
    for c0 in range(0, S, chunk):
        c1 = min(S, c0 + chunk)
        rt.flash_causal(q, kv, kv, parts, batch=B, heads=H, head_dim=hd, q_len=c1 - c0, q_offset=c0, kv_len=c1,
                        q_seq_rows=S, kv_seq_rows=S, q_row0=c0, k_col0=0, v_col0=d, out_seq_rows=S, out_row0=c0)
    t = q.float().view(B, S, H, hd).transpose(1, 2)
    kk = kv.float().view(B, S, 2, H, hd).permute(2, 0, 3, 1, 4)
    ref = _attn_ref(t, kk[0], kk[1], 0).transpose(1, 2).reshape(B * S, d)
    torch.cuda.synchronize()
    assert (full.float() - ref).abs().max().item() < 4e-3
    assert (parts.float() - ref).abs().max().item() < 4e-3


# (B, H, S, hd): more (query tile, head, sequence) items than the persistent one-tile
# kernel has CTAs (two per SM for head_dim <= 64, one for 128 / 256), so every CTA runs
# several items back to back with the next item's Q, K/V and first S issued early
PERSISTENT_CASES = [(24, 4, 1000, 32), (40, 4, 384, 64), (48, 4, 300, 128), (40, 4, 200, 256), (12, 2, 1900, 32)]


@pytest.mark.parametrize("B,H,S,hd", PERSISTENT_CASES)
@pytest.mark.parametrize("mode", ["causal", "noncausal_holes", "prefix_lens"])
def test_flash_persistent_many_items_vs_torch(rt, B, H, S, hd, mode):
    g = torch.Generator().manual_seed(B * 7 + S + hd)
    d = H * hd
    nqt = -(-S // 128)
    assert B * H * nqt > 2 * torch.cuda.get_device_properties(0).multi_processor_count or hd >= 128
    qkv = torch.randn(B * S, 3 * d, generator=g).to(torch.float16).to(DEV)
    t = qkv.float().view(B, S, 3, H, hd).permute(2, 0, 3, 1, 4)
    out = torch.full((B * S, d), float("nan"), dtype=torch.float16, device=DEV)
    valid = torch.ones(B, S, dtype=torch.bool)
    kw = {}
    q_offset = 0
    if mode == "noncausal_holes":
        for b in range(B):  # sequences alternate between holes and a plain padded tail
            if b % 2:
                valid[b, torch.randperm(S, generator=g)[: S // 5]] = False
            else:
                valid[b, S - 13 * (b + 1):] = False
            valid[b, 0] = True
    elif mode == "prefix_lens":
        for b in range(B):
            valid[b, S - 17 * (b % 5 + 1):] = False
    if mode != "causal":
        m = valid.to(DEV)
        lens = torch.zeros(B, dtype=torch.int32, device=DEV)
        holes = torch.zeros(B, dtype=torch.int32, device=DEV)
        bits = torch.zeros(B, rt.mask_key_words(S), dtype=torch.int32, device=DEV)
        rt.mask_prepare(m, lens, holes, bits)
        kw = dict(kv_lens=lens, key_holes=holes, key_bits=bits)
    if mode == "prefix_lens":  # queries [q_offset, S) over the whole K/V prefix
        q_offset = S // 3 + 3
    qn = S - q_offset
    rt.flash_causal(qkv, qkv, qkv, out, batch=B, heads=H, head_dim=hd, q_len=qn, q_offset=q_offset, kv_len=S,
                    q_seq_rows=S, kv_seq_rows=S, q_row0=q_offset, k_col0=d, v_col0=2 * d, out_seq_rows=S,
                    out_row0=q_offset, non_causal=(mode == "noncausal_holes"), **kw)
    s_ = (t[0] @ t[1].transpose(-1, -2)) * hd ** -0.5
    if mode != "noncausal_holes":
        causal = torch.arange(S, device=DEV)[None, :] > torch.arange(S, device=DEV)[:, None]
        s_ = s_.masked_fill(causal, float("-inf"))
    s_ = s_.masked_fill(~valid.to(DEV)[:, None, None, :], float("-inf"))
    ref = (torch.softmax(s_, -1) @ t[2]).permute(0, 2, 1, 3)[:, q_offset:]
    got = out.float().view(B, S, H, hd)[:, q_offset:]
    torch.cuda.synchronize()
    assert torch.isfinite(got).all()
    err = (got - ref).abs().max().item()
    assert err < 4e-3, err
    assert rt.device_error(clear=True) == 0


def test_launch_rejects_unsupported_shapes(rt):
    a = torch.zeros(64, 40, dtype=torch.float16, device=DEV)
    w = torch.zeros(48, 40, dtype=torch.float16, device=DEV)
    out = torch.zeros(64, 48, dtype=torch.float16, device=DEV)
    with pytest.raises(rt.B200Error, match="granule"):
        rt.gemm(rt.EPI_BIAS_F16, a, w, None, out)
    qkv = torch.zeros(128, 3 * 96, dtype=torch.float16, device=DEV)
    o = torch.zeros(128, 96, dtype=torch.float16, device=DEV)
    with pytest.raises(rt.B200Error, match="head_dim"):
        rt.flash_causal(qkv, qkv, qkv, o, batch=1, heads=2, head_dim=48, q_len=128, kv_len=128)


@pytest.mark.parametrize("B,H,S,hd", [(2, 2, 200, 64), (2, 4, 128, 32), (1, 2, 2200, 64), (2, 2, 300, 256),
                                      (2, 16, 128, 8), (2, 4, 300, 16)])
def test_flash_noncausal_with_key_lengths_vs_torch(rt, B, H, S, hd):
    """Full attention with per-sequence valid key counts (key padding)."""
    g = torch.Generator().manual_seed(S + hd)
    d = H * hd
    qkv = torch.randn(B * S, 3 * d, generator=g).to(torch.float16).to(DEV)
    lens = torch.tensor([S - 37 * (i + 1) for i in range(B)], dtype=torch.int32)
    out = torch.empty(B * S, d, dtype=torch.float16, device=DEV)
    rt.flash_causal(qkv, qkv, qkv, out, batch=B, heads=H, head_dim=hd, q_len=S, kv_len=S, k_col0=d, v_col0=2 * d,
                    non_causal=True, kv_lens=lens.to(DEV))
    t = qkv.float().view(B, S, 3, H, hd).permute(2, 0, 3, 1, 4)
    s_ = (t[0] @ t[1].transpose(-1, -2)) * hd ** -0.5
    keymask = torch.arange(S, device=DEV)[None, :] >= lens.to(DEV)[:, None].long()
    s_ = s_.masked_fill(keymask[:, None, None, :], float("-inf"))
    ref = (torch.softmax(s_, -1) @ t[2]).permute(0, 2, 1, 3).reshape(B * S, d)
    torch.cuda.synchronize()
    assert (out.float() - ref).abs().max().item() < 4e-3


@pytest.mark.parametrize("mode", ["0", "1"])
def test_gemm_both_kernels_exact_in_subprocess(mode):
    """The one-SM and the CTA-pair GEMM (B200_GEMM_PAIR forces the choice; it is
    read once per process, hence the child process) give exact integer results,
    fp16 and in-place residual epilogues, on aligned and ragged shapes."""
    import os
    import subprocess
    import sys
    code = r'''
import torch, sys
import torch_transformer_benchmark as T
rt = T._pkg.runtime
dev = "cuda"
for (M, N, K) in ((256, 256, 64), (512, 768, 256), (300, 96, 520), (777, 1280, 4096), (4096, 2048, 1024)):
    g = torch.Generator().manual_seed(M + N + K)
    a = torch.randint(-1, 2, (M, K), generator=g).half().to(dev)
    w = torch.randint(-1, 2, (N, K), generator=g).half().to(dev)
    bias = torch.randint(-4, 5, (N,), generator=g).float().to(dev)
    out = torch.empty(M, N, dtype=torch.float16, device=dev)
    rt.gemm(rt.EPI_BIAS_F16, a, w, bias, out)
    ref = a.double() @ w.double().T + bias.double()
    resid = torch.randint(-100, 101, (M, N), generator=g).float().to(dev)
    ref2 = ref + resid.double()
    rt.gemm(rt.EPI_BIAS_RESID_F32, a, w, bias, resid, resid=resid)
    torch.cuda.synchronize()
    assert torch.equal(out.double(), ref), (M, N, K)
    assert torch.equal(resid.double(), ref2), (M, N, K)
assert rt.device_error(clear=True) == 0
print("OK")
'''
    env = dict(os.environ, B200_GEMM_PAIR=mode)
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    r = subprocess.run([sys.executable, "-c", code], cwd=root, env=env, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0 and "OK" in r.stdout, r.stdout + r.stderr


@pytest.mark.parametrize("tiles", ["1", "2"])
def test_flash_both_kernels_in_subprocess(tiles):
    """The one- and the two-query-tile attention kernel (B200_ATTN_TILES forces
    the choice for head_dim 32/64; read once per process) against torch fp32 on
    shapes where the second query tile of a CTA is empty (S=300, S=384), where
    both tiles need the same number of key tiles (non-causal) and where the
    second needs one more (causal), with and without a prefix offset."""
    import os
    import subprocess
    import sys
    code = r'''
import torch
import torch_transformer_benchmark as T
rt = T._pkg.runtime
dev = "cuda"
def ref_attn(q, k, v, q_offset, causal, lens=None):
    hd = q.shape[-1]
    s = (q @ k.transpose(-1, -2)) * hd ** -0.5
    Sq, Sk = q.shape[-2], k.shape[-2]
    if causal:
        qpos = q_offset + torch.arange(Sq, device=dev)[:, None]
        s = s.masked_fill(torch.arange(Sk, device=dev)[None, :] > qpos, float("-inf"))
    if lens is not None:
        km = torch.arange(Sk, device=dev)[None, :] >= lens[:, None].long()
        s = s.masked_fill(km[:, None, None, :], float("-inf"))
    return torch.softmax(s, -1) @ v
worst = 0.0
for (B, H, S, hd) in ((2, 2, 300, 64), (1, 2, 384, 32), (2, 2, 640, 64), (1, 3, 1000, 32), (1, 2, 1536, 64)):
    d = H * hd
    g = torch.Generator().manual_seed(S * 3 + hd)
    qkv = torch.randn(B * S, 3 * d, generator=g).half().to(dev)
    t = qkv.float().view(B, S, 3, H, hd).permute(2, 0, 3, 1, 4)
    out = torch.full((B * S, d), float("nan"), dtype=torch.float16, device=dev)
    rt.flash_causal(qkv, qkv, qkv, out, batch=B, heads=H, head_dim=hd, q_len=S, kv_len=S, k_col0=d, v_col0=2 * d)
    ref = ref_attn(t[0], t[1], t[2], 0, True).permute(0, 2, 1, 3).reshape(B * S, d)
    worst = max(worst, (out.float() - ref).abs().max().item())
    lens = torch.tensor([S - 29 * (i + 1) for i in range(B)], dtype=torch.int32, device=dev)
    rt.flash_causal(qkv, qkv, qkv, out, batch=B, heads=H, head_dim=hd, q_len=S, kv_len=S, k_col0=d, v_col0=2 * d,
                    non_causal=True, kv_lens=lens)
    ref = ref_attn(t[0], t[1], t[2], 0, False, lens).permute(0, 2, 1, 3).reshape(B * S, d)
    worst = max(worst, (out.float() - ref).abs().max().item())
    c0 = S // 3  # queries [c0, S) over keys [0, S): prefix offset c0
    part = torch.full((B * S, d), float("nan"), dtype=torch.float16, device=dev)
    rt.flash_causal(qkv, qkv, qkv, part, batch=B, heads=H, head_dim=hd, q_len=S - c0, q_offset=c0, kv_len=S,
                    q_seq_rows=S, kv_seq_rows=S, q_row0=c0, k_col0=d, v_col0=2 * d, out_seq_rows=S, out_row0=c0)
    ref = ref_attn(t[0], t[1], t[2], 0, True).permute(0, 2, 1, 3)
    got = part.float().view(B, S, H, hd)[:, c0:]
    worst = max(worst, (got - ref[:, c0:]).abs().max().item())
torch.cuda.synchronize()
assert worst < 4e-3, worst
assert rt.device_error(clear=True) == 0
print("OK", worst)
'''
    env = dict(os.environ, B200_ATTN_TILES=tiles)
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    r = subprocess.run([sys.executable, "-c", code], cwd=root, env=env, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0 and "OK" in r.stdout, r.stdout + r.stderr


@pytest.mark.parametrize("M,K", [(1000, 128), (300, 512), (65536, 128)])
@pytest.mark.parametrize("f16", [True, False])
def test_gemm_residual_layernorm_vs_torch(rt, M, K, f16):
    """The residual projection with the LayerNorm in its epilogue (N = 128):
    v = res + a.w^T + bias, ln_out = LN(v)*gamma + beta; fp16 output also writes
    v back into res, fp32 output leaves res alone."""
    N = 128
    g = torch.Generator().manual_seed(M + K + int(f16))
    a = torch.randn(M, K, generator=g).to(torch.float16).to(DEV)
    w = (torch.randn(N, K, generator=g) / math.sqrt(K)).to(torch.float16).to(DEV)
    bias = torch.randn(N, generator=g).to(DEV)
    res0 = torch.randn(M, N, generator=g).to(DEV)
    gamma = (1 + 0.1 * torch.randn(N, generator=g)).to(DEV)
    beta = (0.1 * torch.randn(N, generator=g)).to(DEV)
    res = res0.clone()
    out = torch.full((M, N), float("nan"), dtype=torch.float16 if f16 else torch.float32, device=DEV)
    rt.gemm_residual_layernorm(a, w, bias, res, gamma, beta, out, eps=1e-5)
    v = res0 + a.float() @ w.float().T + bias
    ref = torch.nn.functional.layer_norm(v, (N,), gamma, beta, eps=1e-5)
    torch.cuda.synchronize()
    tol = 3e-3 if f16 else 2e-4
    assert (out.float() - ref).abs().max().item() < tol
    if f16:
        assert (res - v).abs().max().item() < 1e-4 * math.sqrt(K)
    else:
        assert torch.equal(res, res0)


def test_gemm_residual_layernorm_rejects_wide_rows(rt):
    a = torch.zeros(128, 64, dtype=torch.float16, device=DEV)
    w = torch.zeros(256, 64, dtype=torch.float16, device=DEV)
    res = torch.zeros(128, 256, device=DEV)
    g = torch.ones(256, device=DEV)
    out = torch.empty(128, 256, dtype=torch.float16, device=DEV)
    with pytest.raises(rt.B200Error):
        rt.gemm_residual_layernorm(a, w, None, res, g, g, out)
