"""The PyTorch op layer (torch.ops.b200.*) without a GPU: registration, fake
implementations (what torch.compile traces with) and CPU rejection (no
fallback)."""

import pytest
import torch


def test_ops_registered(pkg):
    for name in ("gemm_out", "linear", "linear_residual", "linear_residual_layernorm", "kv_write", "layernorm",
                 "flash_causal", "block_megakernel"):
        assert hasattr(torch.ops.b200, name), name


def test_fake_shapes(pkg):
    from torch._subclasses.fake_tensor import FakeTensorMode
    ops = pkg.ops
    with FakeTensorMode():
        a = torch.empty(300, 128, dtype=torch.float16, device="cuda")
        w = torch.empty(384, 128, dtype=torch.float16, device="cuda")
        assert torch.ops.b200.linear(a, w, None, ops.EPI_BIAS_GELU_F16).shape == (300, 384)
        assert torch.ops.b200.linear(a, w, None, ops.EPI_BIAS_F32).dtype == torch.float32
        r = torch.empty(300, 384, dtype=torch.float32, device="cuda")
        assert torch.ops.b200.linear_residual(a, w, None, r).shape == (300, 384)
        x = torch.empty(7, 128, dtype=torch.float32, device="cuda")
        g = torch.empty(128, device="cuda")
        assert torch.ops.b200.layernorm(x, g, g, 1e-5, True).dtype == torch.float16
        q = torch.empty(2, 96, 256, dtype=torch.float16, device="cuda")
        o = torch.ops.b200.flash_causal(q, q, q, 4, 0, False, None)
        assert o.shape == (2, 96, 256) and o.dtype == torch.float16


def test_kv_write_fake_checks_the_cache_rows(pkg):
    from torch._subclasses.fake_tensor import FakeTensorMode
    with FakeTensorMode():
        a = torch.empty(64, 128, dtype=torch.float16, device="cuda")
        w = torch.empty(256, 128, dtype=torch.float16, device="cuda")
        cache = torch.empty(1000, 256, dtype=torch.float16, device="cuda")
        assert torch.ops.b200.kv_write(a, w, None, cache, 936) is None
        with pytest.raises(ValueError):
            torch.ops.b200.kv_write(a, w, None, cache, 937)  # past the end of the cache
        with pytest.raises(ValueError):
            torch.ops.b200.kv_write(a, w, None, cache[:, :128], 0)  # columns do not match w_kv


def test_residual_epilogue_rejected_by_functional_linear(pkg):
    from torch._subclasses.fake_tensor import FakeTensorMode
    with FakeTensorMode():
        a = torch.empty(8, 32, dtype=torch.float16, device="cuda")
        with pytest.raises(ValueError):
            torch.ops.b200.linear(a, a, None, pkg.ops.EPI_BIAS_RESID_F32)


def test_cpu_tensors_rejected(pkg):
    a = torch.zeros(4, 32, dtype=torch.float16)
    with pytest.raises(NotImplementedError):
        torch.ops.b200.linear(a, a, None, 0)
