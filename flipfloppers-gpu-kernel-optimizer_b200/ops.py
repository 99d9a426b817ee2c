"""PyTorch op layer over the C ABI: ``torch.ops.b200.*``.

The reference exposed its native GEMM to PyTorch as ``torch.library.custom_op``
ops with registered fake implementations, so that ``torch.compile`` could trace
them and capture them into CUDA graphs, plus an out-parameter variant because
allocations inside captured ops do not survive at large sizes
(torch_transformer_benchmark.py:292-327, 497-586).  These are the B200
library's equivalents:

* ``b200::gemm_out(a, w, bias, epilogue, out)`` -- in place into ``out``; for
  ``EPI_BIAS_RESID_F32`` ``out`` holds the residual on entry (the chain's
  residual stream) and receives ``out + a.w^T + bias``;
* ``b200::linear(a, w, bias, epilogue)`` -- functional GEMM (fp16 out for the
  bias / bias+GELU epilogues, fp32 for ``EPI_BIAS_F32``);
* ``b200::linear_residual(a, w, bias, resid)`` -- functional ``resid + a.w^T + bias``;
* ``b200::linear_residual_layernorm(a, w, bias, resid, gamma, beta, eps)`` --
  ``x1 = resid + a.w^T + bias`` and its LayerNorm (fp16) from one kernel (N = 128);
* ``b200::kv_write(a, w_kv, b_kv, kv_cache, row0)`` -- the chunked forward's
  K/V cache update fused into the projection: the K|V projection of a chunk's
  normalised rows written in place into cache rows ``[row0, row0 + rows)``;
* ``b200::layernorm(x, gamma, beta, eps, out_f16)``;
* ``b200::flash_causal(q, k, v, heads, q_offset, non_causal, kv_lens)`` on
  ``[B, S, H*hd]`` fp16 tensors (prefix-causal when ``q_offset > 0``: query i
  sits at key position ``q_offset + i``);
* ``b200::block_megakernel(x, <stacked layer weights>, ...)`` -- the whole
  small-model forward in one kernel (``k_block_small``).

Every op runs the library's kernels; CPU tensors are rejected (the ops are
registered for CUDA only), there is no fallback.
"""

from __future__ import annotations

from typing import Optional

import torch
from torch import Tensor

from . import runtime as rt

EPI_BIAS_F16 = rt.EPI_BIAS_F16
EPI_BIAS_GELU_F16 = rt.EPI_BIAS_GELU_F16
EPI_BIAS_RESID_F32 = rt.EPI_BIAS_RESID_F32
EPI_BIAS_F32 = rt.EPI_BIAS_F32


# ------------------------------------------------------------------ GEMM
@torch.library.custom_op("b200::gemm_out", mutates_args=("out",), device_types="cuda")
def gemm_out(a: Tensor, w: Tensor, bias: Optional[Tensor], epilogue: int, out: Tensor) -> None:
    resid = out if int(epilogue) == EPI_BIAS_RESID_F32 else None
    rt.gemm(int(epilogue), a, w, bias, out, resid=resid)


@gemm_out.register_fake
def _gemm_out_fake(a, w, bias, epilogue, out) -> None:
    return None


def _linear_out_dtype(epilogue: int) -> torch.dtype:
    if epilogue in (EPI_BIAS_F16, EPI_BIAS_GELU_F16):
        return torch.float16
    if epilogue == EPI_BIAS_F32:
        return torch.float32
    raise ValueError("b200::linear takes EPI_BIAS_F16, EPI_BIAS_GELU_F16 or EPI_BIAS_F32 "
                     "(the residual epilogue is b200::linear_residual / b200::gemm_out)")


@torch.library.custom_op("b200::linear", mutates_args=(), device_types="cuda")
def linear(a: Tensor, w: Tensor, bias: Optional[Tensor], epilogue: int) -> Tensor:
    out = torch.empty(a.shape[0], w.shape[0], dtype=_linear_out_dtype(int(epilogue)), device=a.device)
    rt.gemm(int(epilogue), a, w, bias, out)
    return out


@linear.register_fake
def _linear_fake(a, w, bias, epilogue):
    return a.new_empty((a.shape[0], w.shape[0]), dtype=_linear_out_dtype(int(epilogue)))


@torch.library.custom_op("b200::linear_residual", mutates_args=(), device_types="cuda")
def linear_residual(a: Tensor, w: Tensor, bias: Optional[Tensor], resid: Tensor) -> Tensor:
    out = resid.clone()
    rt.gemm(EPI_BIAS_RESID_F32, a, w, bias, out, resid=out)
    return out


@linear_residual.register_fake
def _linear_residual_fake(a, w, bias, resid):
    return resid.new_empty((a.shape[0], w.shape[0]), dtype=torch.float32)


@torch.library.custom_op("b200::linear_residual_layernorm", mutates_args=(), device_types="cuda")
def linear_residual_layernorm(a: Tensor, w: Tensor, bias: Optional[Tensor], resid: Tensor, gamma: Tensor,
                              beta: Tensor, eps: float) -> tuple[Tensor, Tensor]:
    """x1 = resid + a.w^T + bias and LayerNorm(x1)*gamma + beta (fp16) in one kernel (N = 128)."""
    x1 = resid.clone()
    n = torch.empty(x1.shape, dtype=torch.float16, device=x1.device)
    rt.gemm_residual_layernorm(a, w, bias, x1, gamma, beta, n, eps=eps)
    return x1, n


@linear_residual_layernorm.register_fake
def _linear_residual_layernorm_fake(a, w, bias, resid, gamma, beta, eps):
    shape = (a.shape[0], w.shape[0])
    return resid.new_empty(shape, dtype=torch.float32), resid.new_empty(shape, dtype=torch.float16)


# ------------------------------------------------------------------ K/V cache
def _check_kv_write(a: Tensor, w_kv: Tensor, kv_cache: Tensor, row0: int) -> None:
    if kv_cache.dim() != 2 or kv_cache.dtype != torch.float16 or kv_cache.shape[1] != w_kv.shape[0]:
        raise ValueError("b200::kv_write: kv_cache must be fp16 [tokens, n] with n = w_kv.shape[0] (K | V columns)")
    if a.dim() != 2 or a.shape[1] != w_kv.shape[1]:
        raise ValueError("b200::kv_write: a must be [rows, d] with d = w_kv.shape[1]")
    if row0 < 0 or row0 + a.shape[0] > kv_cache.shape[0]:
        raise ValueError(f"b200::kv_write: rows [{row0}, {row0 + a.shape[0]}) outside the cache's {kv_cache.shape[0]}")


@torch.library.custom_op("b200::kv_write", mutates_args=("kv_cache",), device_types="cuda")
def kv_write(a: Tensor, w_kv: Tensor, b_kv: Optional[Tensor], kv_cache: Tensor, row0: int) -> None:
    """kv_cache[row0 + i] = a[i] . w_kv^T + b_kv (fp16), for the rows of one query chunk.

    The reference's chunked forward projects each chunk's K and V and stores them
    into a preallocated fp16 cache that later chunks attend over (TTB:1463-1500);
    here the projection's epilogue writes the cache rows directly, as the
    library's own chunked forward does."""
    _check_kv_write(a, w_kv, kv_cache, row0)
    rows = a.shape[0]
    rt.gemm(EPI_BIAS_F16, a, w_kv, b_kv, kv_cache[row0:row0 + rows])


@kv_write.register_fake
def _kv_write_fake(a, w_kv, b_kv, kv_cache, row0) -> None:
    _check_kv_write(a, w_kv, kv_cache, row0)
    return None


# ------------------------------------------------------------------ LayerNorm
@torch.library.custom_op("b200::layernorm", mutates_args=(), device_types="cuda")
def layernorm(x: Tensor, gamma: Tensor, beta: Tensor, eps: float, out_f16: bool) -> Tensor:
    out = torch.empty(x.shape, dtype=torch.float16 if out_f16 else torch.float32, device=x.device)
    rt.layernorm(x, gamma, beta, out, eps=eps)
    return out


@layernorm.register_fake
def _layernorm_fake(x, gamma, beta, eps, out_f16):
    return x.new_empty(x.shape, dtype=torch.float16 if out_f16 else torch.float32)


# ------------------------------------------------------------------ attention
@torch.library.custom_op("b200::flash_causal", mutates_args=(), device_types="cuda")
def flash_causal(q: Tensor, k: Tensor, v: Tensor, heads: int, q_offset: int, non_causal: bool,
                 kv_lens: Optional[Tensor]) -> Tensor:
    B, Sq, d = q.shape
    Skv = k.shape[1]
    if k.shape != v.shape or k.shape[0] != B or k.shape[2] != d or d % heads:
        raise ValueError("b200::flash_causal: q [B,Sq,H*hd], k and v [B,Skv,H*hd]")
    q2, k2, v2 = (t.reshape(-1, d) for t in (q.contiguous(), k.contiguous(), v.contiguous()))
    out = torch.empty(B * Sq, d, dtype=torch.float16, device=q.device)
    rt.flash_causal(q2, k2, v2, out, batch=B, heads=heads, head_dim=d // heads, q_len=Sq, q_offset=q_offset,
                    kv_len=Skv, q_seq_rows=Sq, kv_seq_rows=Skv, out_seq_rows=Sq, non_causal=non_causal,
                    kv_lens=kv_lens)
    return out.view(B, Sq, d)


@flash_causal.register_fake
def _flash_causal_fake(q, k, v, heads, q_offset, non_causal, kv_lens):
    return q.new_empty(q.shape, dtype=torch.float16)


# ------------------------------------------------------------------ whole small model
@torch.library.custom_op("b200::block_megakernel", mutates_args=(), device_types="cuda")
def block_megakernel(x: Tensor, ln1_w: Tensor, ln1_b: Tensor, w_qkv: Tensor, b_qkv: Tensor, w_o: Tensor,
                     b_o: Tensor, ln2_w: Tensor, ln2_b: Tensor, w_in: Tensor, b_in: Tensor, w_out: Tensor,
                     b_out: Tensor, lnf_w: Tensor, lnf_b: Tensor, num_heads: int, eps: float, causal: bool,
                     row_valid: Optional[Tensor]) -> Tensor:
    """Layer weights concatenated over the L layers along dim 0: ln1_*/ln2_*/b_o/b_out
    [L*d], b_qkv [L*3d], b_in [L*F] (fp32); w_qkv [L*3d, d], w_o [L*d, d], w_in [L*F, d],
    w_out [L*d, F] (fp16); lnf_* [d]."""
    B, S, d = x.shape
    L = ln1_w.numel() // d
    if L <= 0 or ln1_w.numel() != L * d or w_in.shape[0] % L:
        raise ValueError("b200::block_megakernel: weights must be L layers concatenated along dim 0")
    xc = x.contiguous()  # kept alive until the launch below
    y = torch.empty_like(xc)
    a = rt.FusedSmallArgs()
    a.batch, a.seq_len, a.d_model, a.num_heads = B, S, d, num_heads
    a.ffn_dim, a.num_layers = w_in.shape[0] // L, L
    a.x, a.y = xc.data_ptr(), y.data_ptr()
    for name, t in (("ln1_w", ln1_w), ("ln1_b", ln1_b), ("w_qkv", w_qkv), ("b_qkv", b_qkv), ("w_o", w_o),
                    ("b_o", b_o), ("ln2_w", ln2_w), ("ln2_b", ln2_b), ("w_in", w_in), ("b_in", b_in),
                    ("w_out", w_out), ("b_out", b_out), ("lnf_w", lnf_w), ("lnf_b", lnf_b)):
        setattr(a, name, t.data_ptr())
    a.eps = float(eps)
    a.row_valid = None if row_valid is None else row_valid.data_ptr()
    a.non_causal = 0 if causal else 1
    rt.fused_small(a)
    return y


@block_megakernel.register_fake
def _block_megakernel_fake(x, ln1_w, ln1_b, w_qkv, b_qkv, w_o, b_o, ln2_w, ln2_b, w_in, b_in, w_out, b_out, lnf_w,
                           lnf_b, num_heads, eps, causal, row_valid):
    return torch.empty_like(x)
