"""The C ABI library loads on a machine without a GPU and exports every declared symbol."""

import os
import re

import pytest
import torch

from conftest import REPO

HEADER = os.path.join(REPO, "include", "b200_block.h")


def declared_functions():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(b200_[a-z0-9_]+)\s*\(", src)))


def test_header_declares_entry_points():
    names = declared_functions()
    for n in ("b200_gemm_launch", "b200_flash_causal_launch", "b200_layernorm_launch", "b200_block_forward",
              "b200_block_workspace_bytes", "b200_status_str", "b200_device_error", "b200_abi_version"):
        assert n in names


def test_library_exports_every_declared_symbol(pkg):
    lib = pkg.runtime.lib()
    for n in declared_functions():
        assert hasattr(lib, n), n
    bound = {e[0] for e in pkg.runtime.EXPORTS}
    assert set(declared_functions()) <= bound


def test_abi_version_and_status_strings(pkg):
    rt = pkg.runtime
    assert rt.lib().b200_abi_version() == 2
    assert rt.status_str(0) == "ok"
    assert "head_dim" in rt.status_str(-6)
    assert rt.status_str(12345) == "unknown status"


def test_workspace_bytes(pkg):
    rt = pkg.runtime
    M, d, F = 8192, 128, 512
    need = rt.block_workspace_bytes(M, d, F)
    assert need >= M * (2 * d + 6 * d + 2 * d + 4 * d + 2 * F)
    assert rt.block_workspace_bytes(0, d, F) == 0


def test_arg_checks_do_not_touch_device(pkg):
    """Invalid arguments are rejected before any CUDA call (safe without a GPU)."""
    rt = pkg.runtime
    lib = rt.lib()
    assert lib.b200_gemm_launch(0, None, 0, None, 0, None, None, 0, None, 0, 1, 32, 8, None) == -9
    assert lib.b200_gemm_launch(7, 16, 8, 16, 8, None, None, 0, 16, 32, 1, 32, 8, None) == -1
    assert lib.b200_gemm_launch(0, 16, 8, 16, 8, None, None, 0, 16, 32, 1, 30, 8, None) == -2
    a = rt.AttnArgs()
    a.q = a.k = a.v = a.out = 256
    a.ld_q = a.ld_k = a.ld_v = a.ld_out = 96
    a.q_rows = a.kv_rows = 128
    a.batch, a.heads, a.head_dim = 1, 2, 48
    a.q_len = a.kv_len = 128
    assert lib.b200_flash_causal_launch(a, None) == -6
    a.head_dim, a.q_offset = 32, 5
    assert lib.b200_flash_causal_launch(a, None) == -9


def test_fused_small_arg_checks_do_not_touch_device(pkg):
    """The whole-model launcher rejects unsupported shapes, aliasing and
    misalignment before any CUDA call: d_model 128 takes 1, 2 or 4 heads (3 and
    16 are refused), ffn a multiple of 128 up to 512, seq_len <= 128."""
    rt = pkg.runtime
    lib = rt.lib()

    def args(**kw):
        a = rt.FusedSmallArgs()
        a.batch, a.seq_len, a.d_model, a.num_heads, a.ffn_dim, a.num_layers = 2, 128, 128, 4, 512, 1
        for name in ("ln1_w", "ln1_b", "w_qkv", "b_qkv", "w_o", "b_o", "ln2_w", "ln2_b", "w_in", "b_in", "w_out",
                     "b_out", "lnf_w", "lnf_b"):
            setattr(a, name, 4096)
        a.x, a.y, a.eps = 256, 512, 1e-5
        for k, v in kw.items():
            setattr(a, k, v)
        return a

    for heads in (3, 16):
        assert lib.b200_block_fused_small_launch(args(num_heads=heads), None) == -1
    assert lib.b200_block_fused_small_launch(args(ffn_dim=96), None) == -1
    assert lib.b200_block_fused_small_launch(args(ffn_dim=640), None) == -1
    assert lib.b200_block_fused_small_launch(args(seq_len=129), None) == -1
    assert lib.b200_block_fused_small_launch(args(y=256), None) == -9      # y aliases x
    assert lib.b200_block_fused_small_launch(args(w_in=4100), None) == -5  # weights 16-byte aligned
    assert lib.b200_block_fused_small_launch(args(b_o=4100), None) == -5   # vectors arrive by bulk copy
    assert lib.b200_block_fused_small_launch(args(lnf_w=None), None) == -9


def test_model_state_dict_matches_reference_layout(tt):
    import oracle
    cfg = tt.TransformerConfig(2, 16, 64, 2, 256, 2, True)
    torch.manual_seed(99)
    m = tt.UserOptimizedTransformer(cfg)
    ref = oracle.init_state_dict(2, 64, 256, 99)
    sd = m.state_dict()
    assert list(sd.keys()) == list(ref.keys())
    assert all(torch.equal(sd[k], ref[k]) for k in ref)
    m.load_state_dict(ref, strict=True)


def test_config_validation(tt):
    with pytest.raises(ValueError):
        tt.TransformerConfig(1, 1, 10, 3, 4, 1, True).validate()
    with pytest.raises(ValueError):
        tt.TransformerConfig(0, 1, 8, 2, 4, 1, True).validate()


def test_cpu_tensor_raises_no_fallback(tt):
    cfg = tt.TransformerConfig(1, 8, 64, 2, 256, 1, True)
    m = tt.UserOptimizedTransformer(cfg)
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        m(torch.randn(1, 8, 64))


def test_model_built_under_inference_mode_has_param_key():
    """A model constructed inside torch.inference_mode (inference tensors, no
    version counter) must still produce its weight-pack key."""
    import torch
    import torch_transformer_benchmark as T
    with torch.inference_mode():
        m = T.UserOptimizedTransformer(T.TransformerConfig(1, 8, 64, 2, 128, 1, True))
        k1 = m._param_key(torch.device("cpu"))
        k2 = m._param_key(torch.device("cpu"))
    assert k1 == k2
