"""ctypes binding of libb200block.so (the C ABI declared in include/b200_block.h).

This is the Python-side equivalent of the reference's extension loader and
custom-op layer (torch_transformer_benchmark.py:262-327, 443-586): it loads the
native library once, and each wrapper passes raw device pointers, sizes and the
caller's current CUDA stream.  Unlike the reference (which returned ``None``
from a failed build and silently fell back to ``F.linear``, TTB:467-469,
502-506) a missing library or a non-zero status raises: there is no fallback.
"""

from __future__ import annotations

import ctypes
import os
import threading
from typing import Optional

import torch

from . import build as _build

LIB_PATH = _build.LIB_PATH

B200_OK = 0
EPI_BIAS_F16 = 0
EPI_BIAS_GELU_F16 = 1
EPI_BIAS_RESID_F32 = 2
EPI_BIAS_F32 = 3

_lib = None
_lock = threading.Lock()

_c_ll = ctypes.c_longlong
_vp = ctypes.c_void_p


class B200Error(RuntimeError):
    """A launcher in libb200block.so returned a non-zero status."""

    def __init__(self, what: str, status: int):
        self.status = status
        try:
            detail = lib().b200_last_error_detail().decode()
        except Exception:  # noqa: BLE001
            detail = ""
        super().__init__(f"{what}: {status_str(status)} (status {status})" + (f" [{detail}]" if detail else ""))


class AttnArgs(ctypes.Structure):
    _fields_ = [
        ("q", _vp), ("k", _vp), ("v", _vp),
        ("ld_q", _c_ll), ("ld_k", _c_ll), ("ld_v", _c_ll),
        ("q_rows", _c_ll), ("kv_rows", _c_ll),
        ("batch", ctypes.c_int), ("heads", ctypes.c_int), ("head_dim", ctypes.c_int),
        ("q_len", ctypes.c_int), ("q_offset", ctypes.c_int), ("kv_len", ctypes.c_int),
        ("q_seq_rows", ctypes.c_int), ("kv_seq_rows", ctypes.c_int),
        ("q_row0", ctypes.c_int), ("kv_row0", ctypes.c_int),
        ("q_col0", ctypes.c_int), ("k_col0", ctypes.c_int), ("v_col0", ctypes.c_int),
        ("out", _vp), ("ld_out", _c_ll), ("out_seq_rows", ctypes.c_int), ("out_row0", ctypes.c_int),
        ("non_causal", ctypes.c_int), ("kv_lens", _vp),
        ("key_bits", _vp), ("key_words", ctypes.c_int), ("key_holes", _vp),
    ]


class BlockArgs(ctypes.Structure):
    _fields_ = [
        ("batch", ctypes.c_int), ("seq_len", ctypes.c_int), ("d_model", ctypes.c_int),
        ("num_heads", ctypes.c_int), ("ffn_dim", ctypes.c_int),
        ("x", _vp), ("y", _vp),
        ("ln1_w", _vp), ("ln1_b", _vp),
        ("w_qkv", _vp), ("b_qkv", _vp),
        ("w_o", _vp), ("b_o", _vp),
        ("ln2_w", _vp), ("ln2_b", _vp),
        ("w_in", _vp), ("b_in", _vp),
        ("w_out", _vp), ("b_out", _vp),
        ("lnf_w", _vp), ("lnf_b", _vp),
        ("eps", ctypes.c_float),
        ("workspace", _vp), ("workspace_bytes", ctypes.c_size_t),
        ("non_causal", ctypes.c_int), ("kv_lens", _vp),
        ("key_bits", _vp), ("key_words", ctypes.c_int), ("key_holes", _vp),
    ]


class FusedSmallArgs(ctypes.Structure):
    _fields_ = [
        ("batch", ctypes.c_int), ("seq_len", ctypes.c_int), ("d_model", ctypes.c_int),
        ("num_heads", ctypes.c_int), ("ffn_dim", ctypes.c_int), ("num_layers", ctypes.c_int),
        ("x", _vp), ("y", _vp),
        ("ln1_w", _vp), ("ln1_b", _vp),
        ("w_qkv", _vp), ("b_qkv", _vp),
        ("w_o", _vp), ("b_o", _vp),
        ("ln2_w", _vp), ("ln2_b", _vp),
        ("w_in", _vp), ("b_in", _vp),
        ("w_out", _vp), ("b_out", _vp),
        ("lnf_w", _vp), ("lnf_b", _vp),
        ("eps", ctypes.c_float),
        ("row_valid", _vp),
        ("non_causal", ctypes.c_int),
    ]


# (name, restype, argtypes) of every exported symbol; include/b200_block.h is the source of truth.
EXPORTS = [
    ("b200_abi_version", ctypes.c_int, []),
    ("b200_status_str", ctypes.c_char_p, [ctypes.c_int]),
    ("b200_last_error_detail", ctypes.c_char_p, []),
    ("b200_device_error", ctypes.c_int, [ctypes.c_int]),
    ("b200_layernorm_launch", ctypes.c_int,
     [_vp, _c_ll, _vp, _vp, _vp, _c_ll, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_float, _vp]),
    ("b200_layernorm_residual_launch", ctypes.c_int,
     [_vp, _c_ll, _vp, _vp, _vp, _c_ll, ctypes.c_int, _vp, _c_ll, ctypes.c_int, ctypes.c_int, ctypes.c_float, _vp]),
    ("b200_add_layernorm_launch", ctypes.c_int,
     [_vp, _vp, _vp, _vp, _vp, _vp, _vp, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_float, _vp]),
    ("b200_zero_masked_rows", ctypes.c_int, [_vp, _vp, _c_ll, ctypes.c_int, _vp]),
    ("b200_mask_key_words", ctypes.c_int, [ctypes.c_int]),
    ("b200_mask_prepare", ctypes.c_int, [_vp, ctypes.c_int, ctypes.c_int, _vp, _vp, _vp, _vp]),
    ("b200_gemm_launch", ctypes.c_int,
     [ctypes.c_int, _vp, _c_ll, _vp, _c_ll, _vp, _vp, _c_ll, _vp, _c_ll, ctypes.c_int, ctypes.c_int, ctypes.c_int, _vp]),
    ("b200_gemm_residual_layernorm_launch", ctypes.c_int,
     [_vp, _c_ll, _vp, _c_ll, _vp, _vp, _c_ll, _vp, _vp, ctypes.c_float, _vp, _c_ll, ctypes.c_int, ctypes.c_int,
      ctypes.c_int, ctypes.c_int, _vp]),
    ("b200_flash_causal_launch", ctypes.c_int, [ctypes.POINTER(AttnArgs), _vp]),
    ("b200_block_workspace_bytes", ctypes.c_size_t, [_c_ll, ctypes.c_int, ctypes.c_int]),
    ("b200_block_forward", ctypes.c_int, [ctypes.POINTER(BlockArgs), _vp]),
    ("b200_block_forward_noalloc", ctypes.c_int, [ctypes.POINTER(BlockArgs), _vp]),
    ("b200_block_fused_small_launch", ctypes.c_int, [ctypes.POINTER(FusedSmallArgs), _vp]),
    ("b200_block_chunked_workspace_bytes", ctypes.c_size_t, [_c_ll, ctypes.c_int, ctypes.c_int, ctypes.c_int]),
    ("b200_block_forward_chunked", ctypes.c_int, [ctypes.POINTER(BlockArgs), ctypes.c_int, _vp]),
]


def lib():
    """Load libb200block.so once (raises if it has not been built)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise RuntimeError(
                    f"{LIB_PATH} is missing: build it with `python {_build.__file__}` "
                    "(there is no non-CUDA implementation to fall back to)")
            handle = ctypes.CDLL(LIB_PATH)
            for name, res, args in EXPORTS:
                fn = getattr(handle, name)
                fn.restype = res
                fn.argtypes = args
            _lib = handle
    return _lib


def status_str(status: int) -> str:
    try:
        return lib().b200_status_str(int(status)).decode()
    except Exception:  # noqa: BLE001 - only used while formatting an error
        return "unknown status"


def check(status: int, what: str) -> None:
    if status != B200_OK:
        raise B200Error(what, status)


def device_error(clear: bool = True) -> int:
    """First device-side failure code since the last clear (0 = none). Synchronises."""
    return int(lib().b200_device_error(1 if clear else 0))


def _p(t: Optional[torch.Tensor]):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _stream(stream=None):
    s = torch.cuda.current_stream() if stream is None else stream
    return ctypes.c_void_p(s.cuda_stream)


def _require_cuda(*ts):
    for t in ts:
        if t is not None and not t.is_cuda:
            raise RuntimeError("libb200block kernels take CUDA tensors only (no CPU fallback)")


def layernorm(x: torch.Tensor, gamma: torch.Tensor, beta: torch.Tensor, out: torch.Tensor,
              eps: float = 1e-5, stream=None, residual_out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """out = LayerNorm(x) * gamma + beta over the last dim; out fp16 or fp32.

    With ``residual_out`` (fp32, x's shape) x is also copied there: the residual
    stream a following ``gemm(EPI_BIAS_RESID_F32, ..., out=r, resid=r)`` adds onto."""
    _require_cuda(x, gamma, beta, out, residual_out)
    d = x.shape[-1]
    rows = x.numel() // d
    if x.dtype != torch.float32 or out.dtype not in (torch.float16, torch.float32):
        raise TypeError("layernorm: x must be fp32, out fp16 or fp32")
    ldx = x.stride(-2) if x.dim() > 1 else d
    ldo = out.stride(-2) if out.dim() > 1 else d
    if residual_out is None:
        rc = lib().b200_layernorm_launch(_p(x), ldx, _p(gamma), _p(beta), _p(out), ldo,
                                         int(out.dtype == torch.float16), rows, d, float(eps), _stream(stream))
        check(rc, "b200_layernorm_launch")
    else:
        if residual_out.dtype != torch.float32:
            raise TypeError("layernorm: residual_out must be fp32")
        rc = lib().b200_layernorm_residual_launch(
            _p(x), ldx, _p(gamma), _p(beta), _p(out), ldo, int(out.dtype == torch.float16), _p(residual_out),
            residual_out.stride(-2) if residual_out.dim() > 1 else d, rows, d, float(eps), _stream(stream))
        check(rc, "b200_layernorm_residual_launch")
    return out


def add_layernorm(a: torch.Tensor, b: torch.Tensor, bias: Optional[torch.Tensor], sum_out: torch.Tensor,
                  gamma: torch.Tensor, beta: torch.Tensor, out: torch.Tensor, eps: float = 1e-5,
                  stream=None) -> torch.Tensor:
    """sum_out = a + b + bias; out = LayerNorm(sum_out) * gamma + beta (fp16 or fp32 out)."""
    _require_cuda(a, b, bias, sum_out, gamma, beta, out)
    d = a.shape[-1]
    rows = a.numel() // d
    rc = lib().b200_add_layernorm_launch(_p(a), _p(b), _p(bias), _p(sum_out), _p(gamma), _p(beta), _p(out),
                                         int(out.dtype == torch.float16), rows, d, float(eps), _stream(stream))
    check(rc, "b200_add_layernorm_launch")
    return out


def zero_masked_rows(y: torch.Tensor, row_valid: torch.Tensor, stream=None) -> torch.Tensor:
    """Zero the rows of y (fp32 [..., d]) whose flag in row_valid (bool/uint8, one per row) is 0."""
    _require_cuda(y, row_valid)
    d = y.shape[-1]
    rc = lib().b200_zero_masked_rows(_p(y), _p(row_valid), y.numel() // d, d, _stream(stream))
    check(rc, "b200_zero_masked_rows")
    return y


def mask_key_words(seq_len: int) -> int:
    """32-bit words per sequence of the packed key mask (one 16-byte group per 128 keys)."""
    return int(lib().b200_mask_key_words(int(seq_len)))


def mask_prepare(mask: torch.Tensor, kv_lens: torch.Tensor, key_holes: Optional[torch.Tensor] = None,
                 key_bits: Optional[torch.Tensor] = None, stream=None) -> None:
    """From ``mask`` ([B, S] bool/uint8 on the device, contiguous), on the device: kv_lens[b] =
    one past the last valid token, key_holes[b] = 1 if the mask is not prefix-valid, and for such
    a sequence key_bits[b, :] the mask as bits (int32 [B, mask_key_words(S)])."""
    _require_cuda(mask, kv_lens, key_holes, key_bits)
    B, S = mask.shape
    if kv_lens.dtype != torch.int32 or kv_lens.numel() < B:
        raise TypeError("mask_prepare: kv_lens must be int32 with one entry per sequence")
    if (key_holes is None) != (key_bits is None):
        raise ValueError("mask_prepare: key_holes and key_bits go together")
    if key_bits is not None and key_bits.numel() < B * mask_key_words(S):
        raise ValueError("mask_prepare: key_bits too small")
    check(lib().b200_mask_prepare(_p(mask), B, S, _p(kv_lens), _p(key_holes), _p(key_bits), _stream(stream)),
          "b200_mask_prepare")


def gemm(epilogue: int, a: torch.Tensor, w: torch.Tensor, bias: Optional[torch.Tensor], out: torch.Tensor,
         resid: Optional[torch.Tensor] = None, stream=None) -> torch.Tensor:
    """out = epilogue(a @ w.T + bias [+ resid]); a [M,K] fp16, w [N,K] fp16, bias fp32."""
    _require_cuda(a, w, bias, out, resid)
    if a.dtype != torch.float16 or w.dtype != torch.float16:
        raise TypeError("gemm: operands must be fp16")
    M, K = a.shape
    N = w.shape[0]
    rc = lib().b200_gemm_launch(int(epilogue), _p(a), a.stride(0), _p(w), w.stride(0), _p(bias), _p(resid),
                                resid.stride(0) if resid is not None else 0, _p(out), out.stride(0),
                                M, N, K, _stream(stream))
    check(rc, "b200_gemm_launch")
    return out


def gemm_residual_layernorm(a: torch.Tensor, w: torch.Tensor, bias: Optional[torch.Tensor], res: torch.Tensor,
                            gamma: torch.Tensor, beta: torch.Tensor, ln_out: torch.Tensor, eps: float = 1e-5,
                            stream=None) -> torch.Tensor:
    """v = res + a @ w.T + bias; ln_out = LayerNorm(v)*gamma + beta (fp16: res = v as well;
    fp32: res unchanged).  N = w.shape[0] must be 128."""
    _require_cuda(a, w, bias, res, gamma, beta, ln_out)
    if a.dtype != torch.float16 or w.dtype != torch.float16 or res.dtype != torch.float32:
        raise TypeError("gemm_residual_layernorm: fp16 operands, fp32 residual")
    if ln_out.dtype not in (torch.float16, torch.float32):
        raise TypeError("gemm_residual_layernorm: ln_out fp16 or fp32")
    M, K = a.shape
    N = w.shape[0]
    rc = lib().b200_gemm_residual_layernorm_launch(
        _p(a), a.stride(0), _p(w), w.stride(0), _p(bias), _p(res), res.stride(0), _p(gamma), _p(beta), float(eps),
        _p(ln_out), ln_out.stride(0), int(ln_out.dtype == torch.float16), M, N, K, _stream(stream))
    check(rc, "b200_gemm_residual_layernorm_launch")
    return ln_out


def flash_causal(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, out: torch.Tensor, *, batch: int, heads: int,
                 head_dim: int, q_len: int, kv_len: int, q_offset: int = 0, q_seq_rows: int = None,
                 kv_seq_rows: int = None, q_col0: int = 0, k_col0: int = 0, v_col0: int = 0, q_row0: int = 0,
                 kv_row0: int = 0, out_seq_rows: int = None, out_row0: int = 0, non_causal: bool = False,
                 kv_lens: Optional[torch.Tensor] = None, key_holes: Optional[torch.Tensor] = None,
                 key_bits: Optional[torch.Tensor] = None, stream=None) -> torch.Tensor:
    """Prefix-causal (or full) attention over 2-D fp16 tensors (see B200AttnArgs); key_holes /
    key_bits ([batch] / [batch, words] int32, from mask_prepare) mask keys of sequences whose
    key-padding mask is not prefix-valid."""
    _require_cuda(q, k, v, out)
    a = AttnArgs()
    a.q, a.k, a.v = q.data_ptr(), k.data_ptr(), v.data_ptr()
    a.ld_q, a.ld_k, a.ld_v = q.stride(0), k.stride(0), v.stride(0)
    a.q_rows, a.kv_rows = q.shape[0], k.shape[0]
    a.batch, a.heads, a.head_dim = batch, heads, head_dim
    a.q_len, a.q_offset, a.kv_len = q_len, q_offset, kv_len
    a.q_seq_rows = q_len if q_seq_rows is None else q_seq_rows
    a.kv_seq_rows = kv_len if kv_seq_rows is None else kv_seq_rows
    a.q_row0, a.kv_row0 = q_row0, kv_row0
    a.q_col0, a.k_col0, a.v_col0 = q_col0, k_col0, v_col0
    a.out, a.ld_out = out.data_ptr(), out.stride(0)
    a.out_seq_rows = q_len if out_seq_rows is None else out_seq_rows
    a.out_row0 = out_row0
    a.non_causal = int(bool(non_causal))
    a.kv_lens = None if kv_lens is None else kv_lens.data_ptr()
    if key_bits is not None:
        a.key_bits, a.key_words, a.key_holes = key_bits.data_ptr(), key_bits.shape[-1], key_holes.data_ptr()
    check(lib().b200_flash_causal_launch(ctypes.byref(a), _stream(stream)), "b200_flash_causal_launch")
    return out


def block_workspace_bytes(tokens: int, d_model: int, ffn_dim: int) -> int:
    return int(lib().b200_block_workspace_bytes(int(tokens), int(d_model), int(ffn_dim)))


def block_forward(args: BlockArgs, stream=None) -> None:
    check(lib().b200_block_forward(ctypes.byref(args), _stream(stream)), "b200_block_forward")


def chunked_workspace_bytes(tokens: int, chunk_rows: int, d_model: int, ffn_dim: int) -> int:
    return int(lib().b200_block_chunked_workspace_bytes(int(tokens), int(chunk_rows), int(d_model), int(ffn_dim)))


def block_forward_chunked(args: BlockArgs, chunk_rows: int, stream=None) -> None:
    check(lib().b200_block_forward_chunked(ctypes.byref(args), int(chunk_rows), _stream(stream)),
          "b200_block_forward_chunked")


def fused_small(args: FusedSmallArgs, stream=None) -> None:
    check(lib().b200_block_fused_small_launch(ctypes.byref(args), _stream(stream)), "b200_block_fused_small_launch")


# Size of the static scratch buffer behind b200_block_forward_noalloc (B200_NOALLOC_SCRATCH_BYTES).
NOALLOC_SCRATCH_BYTES = 32 * 1024 * 1024


def block_forward_noalloc(args: BlockArgs, stream=None) -> None:
    """b200_block_forward without a workspace: for callers that cannot allocate device
    memory (the library's static 32 MiB buffer holds the intermediates; calls that
    overlap on the GPU race on it).  args.workspace is ignored."""
    check(lib().b200_block_forward_noalloc(ctypes.byref(args), _stream(stream)), "b200_block_forward_noalloc")
