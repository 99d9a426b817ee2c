"""The no-allocation entry point, b200_block_forward_noalloc, on a B200 (collected last).

Some callers cannot allocate device memory -- a plugin host whose memory
belongs to another allocator's pool and that hands out no workspace, a
foreign-language caller with no CUDA allocator, a loop that cannot pay for
cudaMalloc's implicit synchronisation -- so the library offers the block
forward with its intermediates in a static 32 MiB device buffer instead of a
caller-provided workspace.  This file checks, through the C ABI, that two
calls in a row agree with b200_block_forward (which takes a workspace): both
run the same kernels on the same inputs, so the outputs must be bit-identical
(stricter than the harness's atol 0.002 / rtol 0.02, which is checked too), and
that a problem larger than the buffer is refused before anything is launched.
It must pass alone in a fresh process and after the rest of the suite.
"""

import ctypes

import pytest
import torch

import oracle

pytestmark = pytest.mark.gpu

ATOL, RTOL = 0.002, 0.02
DEV = "cuda"


def _block_args(rt, model, x, y):
    cfg = model.config
    pk = model._packs[0]
    lnf_w, lnf_b = model._lnf
    B, S, d = x.shape
    a = rt.BlockArgs()
    a.batch, a.seq_len, a.d_model, a.num_heads, a.ffn_dim = B, S, d, cfg.num_heads, cfg.ffn_dim
    a.x, a.y = x.data_ptr(), y.data_ptr()
    a.ln1_w, a.ln1_b = pk.ln1_w.data_ptr(), pk.ln1_b.data_ptr()
    a.w_qkv, a.b_qkv = pk.w_qkv.data_ptr(), pk.b_qkv.data_ptr()
    a.w_o, a.b_o = pk.w_o.data_ptr(), pk.b_o.data_ptr()
    a.ln2_w, a.ln2_b = pk.ln2_w.data_ptr(), pk.ln2_b.data_ptr()
    a.w_in, a.b_in = pk.w_in.data_ptr(), pk.b_in.data_ptr()
    a.w_out, a.b_out = pk.w_out.data_ptr(), pk.b_out.data_ptr()
    a.lnf_w, a.lnf_b = lnf_w.data_ptr(), lnf_b.data_ptr()
    a.eps = 1e-5
    return a


def test_noalloc_matches_workspace_entry_point(tt):
    rt = tt._pkg.runtime
    lib = rt.lib()
    assert rt.device_error(clear=True) == 0
    B, S, d, H, F = 64, 128, 128, 4, 512  # 22 MiB of scratch, within the 32 MiB buffer
    cfg = tt.TransformerConfig(B, S, d, H, F, 1, True)
    torch.manual_seed(1234)
    model = tt.UserOptimizedTransformer(cfg).to(DEV).eval()
    model._ensure_packs(torch.device(DEV, torch.cuda.current_device()))
    need = rt.block_workspace_bytes(B * S, d, F)
    assert need <= rt.NOALLOC_SCRATCH_BYTES
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    for call in range(2):  # two calls in a row, different inputs
        x, _ = oracle.generate_random_case(B, S, d, 2024 + call)
        x = x.to(DEV)
        y_ws = torch.full_like(x, float("nan"))
        y_na = torch.full_like(x, float("nan"))
        ws = torch.empty(need, dtype=torch.uint8, device=DEV)
        a = _block_args(rt, model, x, y_ws)
        a.workspace, a.workspace_bytes = ws.data_ptr(), ws.numel()
        assert lib.b200_block_forward(ctypes.byref(a), stream) == 0
        b = _block_args(rt, model, x, y_na)  # workspace left NULL: ignored by the no-allocation entry point
        assert lib.b200_block_forward_noalloc(ctypes.byref(b), stream) == 0
        torch.cuda.synchronize()
        assert torch.isfinite(y_na).all()
        res = oracle.compare_outputs(y_ws.cpu(), y_na.cpu(), rtol=RTOL, atol=ATOL)
        assert res.passed, (call, res)
        assert torch.equal(y_ws, y_na), (call, (y_ws - y_na).abs().max().item())
    assert rt.device_error(clear=True) == 0


def test_noalloc_refuses_problems_beyond_its_buffer(tt):
    rt = tt._pkg.runtime
    lib = rt.lib()
    a = rt.BlockArgs()
    a.batch, a.seq_len, a.d_model, a.num_heads, a.ffn_dim = 1024, 128, 128, 4, 512  # 352 MiB of scratch
    assert rt.block_workspace_bytes(1024 * 128, 128, 512) > rt.NOALLOC_SCRATCH_BYTES
    rc = lib.b200_block_forward_noalloc(ctypes.byref(a), None)
    assert rc == -13
    assert "32 MiB" in rt.status_str(rc)
