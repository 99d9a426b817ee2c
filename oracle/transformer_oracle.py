"""NumPy restatement of the reference's fp32 transformer forward (TEST INFRASTRUCTURE).

Only tests, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg use
this module.  It restates, operation by operation, the frozen PyTorch module of
yeoshuyi/Flipfloppers-GPU-Kernel-Optimizer ("TTB" = torch_transformer_benchmark.py):

* ``TransformerConfig`` shape record ...................... TTB:49-76
* ``BaselineSelfAttention.forward`` ....................... TTB:105-142
  - q/k/v projections and head split ....................... TTB:97-115
  - ``scores = q @ k^T * head_dim**-0.5`` ................... TTB:90, 117
  - causal ``triu(1)`` mask to -inf ......................... TTB:119-123
  - key-padding mask to -inf ................................ TTB:125-128
  - fp32 softmax, ``probs @ v``, head merge ................. TTB:131-137
  - out_proj, zero padded query rows ........................ TTB:138-141
* ``BaselineTransformerBlock.forward`` (pre-LN) ........... TTB:154-165
  ``x = x + attn(norm1(x)); x = x + ffn_out(gelu_erf(ffn_in(norm2(x))))``
* ``BaselineTransformer.forward`` (layers + final_norm) ... TTB:182-192

Arithmetic is float32 by default (``dtype=np.float64`` gives an fp64 oracle for
error budgeting).  Matrix products go through NumPy's BLAS; the reference goes
through ATen's.  Both are fp32 with different summation orders, which is why
the golden test allows ~1e-5, not bit equality.

Parameters are a dict keyed exactly like the reference's ``state_dict``
(``layers.{i}.norm1.weight``, ``layers.{i}.attention.q_proj.weight`` ...).
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Dict, Iterable, Optional

import numpy as np
from scipy.special import erf as _erf

LN_EPS = 1e-5  # nn.LayerNorm default eps (TTB:148, 150, 178)


@dataclass(frozen=True)
class OracleConfig:
    """Shape record; same fields and checks as TTB:49-76."""

    batch_size: int
    seq_len: int
    d_model: int
    num_heads: int
    ffn_dim: int
    num_layers: int
    causal: bool

    def validate(self) -> None:
        for name in ("batch_size", "seq_len", "d_model", "num_heads", "ffn_dim", "num_layers"):
            if getattr(self, name) <= 0:
                raise ValueError(f"{name} must be positive")
        if self.d_model % self.num_heads != 0:
            raise ValueError("d_model must be divisible by num_heads")


def layer_norm(x: np.ndarray, weight: Optional[np.ndarray], bias: Optional[np.ndarray],
               eps: float = LN_EPS) -> np.ndarray:
    """nn.LayerNorm over the last dim: biased variance, ``(x-mu)/sqrt(var+eps)*g+b``."""
    dt = x.dtype
    mu = x.mean(axis=-1, keepdims=True, dtype=dt)
    xc = x - mu
    var = (xc * xc).mean(axis=-1, keepdims=True, dtype=dt)
    y = xc / np.sqrt(var + dt.type(eps))
    if weight is not None:
        y = y * weight.astype(dt)
    if bias is not None:
        y = y + bias.astype(dt)
    return y.astype(dt, copy=False)


def linear(x: np.ndarray, weight: np.ndarray, bias: Optional[np.ndarray]) -> np.ndarray:
    """nn.Linear: ``x @ W^T + b`` with W stored ``[out, in]``."""
    dt = x.dtype
    y = x @ weight.astype(dt).T
    if bias is not None:
        y = y + bias.astype(dt)
    return y


def gelu_erf(x: np.ndarray) -> np.ndarray:
    """Exact GELU, ``F.gelu(approximate="none")`` (TTB:161): ``x/2*(1+erf(x/sqrt2))``."""
    dt = x.dtype
    return (dt.type(0.5) * x * (dt.type(1.0) + _erf(x * dt.type(1.0 / np.sqrt(2.0))))).astype(dt, copy=False)


def _softmax_lastdim(s: np.ndarray) -> np.ndarray:
    m = s.max(axis=-1, keepdims=True)
    with np.errstate(invalid="ignore"):
        e = np.exp(s - m)
        return e / e.sum(axis=-1, keepdims=True)


def causal_attention(q: np.ndarray, k: np.ndarray, v: np.ndarray, causal: bool = True,
                     key_valid: Optional[np.ndarray] = None, q_offset: int = 0) -> np.ndarray:
    """Attention core of TTB:117-132 on head-split tensors.

    q: [B, H, Sq, hd]; k, v: [B, H, Sk, hd].  Query row i sits at absolute
    position ``q_offset + i`` and (when ``causal``) sees keys ``0..q_offset+i``
    -- with ``q_offset=0, Sq=Sk`` this is exactly the reference's ``triu(1)``
    mask; with ``q_offset>0`` it is the prefix-causal (bottom-right aligned)
    mask of the reference's chunked path (TTB:1491-1500).
    ``key_valid``: [B, Sk] bool, False keys are masked (TTB:125-128).
    Returns [B, H, Sq, hd].
    """
    dt = q.dtype
    hd = q.shape[-1]
    scale = dt.type(hd ** -0.5)
    scores = np.matmul(q, np.swapaxes(k, -1, -2)) * scale
    Sq, Sk = q.shape[-2], k.shape[-2]
    if causal:
        qpos = q_offset + np.arange(Sq)[:, None]
        kpos = np.arange(Sk)[None, :]
        scores = np.where(kpos > qpos, dt.type(-np.inf), scores)
    if key_valid is not None:
        scores = np.where(key_valid[:, None, None, :], scores, dt.type(-np.inf))
    probs = _softmax_lastdim(scores.astype(np.float32 if dt == np.float32 else dt)).astype(dt)
    return np.matmul(probs, v)


def _split_heads(x: np.ndarray, H: int) -> np.ndarray:
    B, S, d = x.shape
    return x.reshape(B, S, H, d // H).transpose(0, 2, 1, 3)


def _merge_heads(x: np.ndarray) -> np.ndarray:
    B, H, S, hd = x.shape
    return x.transpose(0, 2, 1, 3).reshape(B, S, H * hd)


def _p(params: Dict[str, np.ndarray], name: str, dt) -> np.ndarray:
    return np.asarray(params[name], dtype=dt)


def block_forward(params: Dict[str, np.ndarray], layer: int, x: np.ndarray, num_heads: int,
                  causal: bool = True, valid_token_mask: Optional[np.ndarray] = None) -> np.ndarray:
    """One pre-LN block, TTB:154-165 with the attention of TTB:105-142."""
    dt = x.dtype
    pre = f"layers.{layer}."
    g = lambda n: _p(params, pre + n, dt)  # noqa: E731
    n1 = layer_norm(x, g("norm1.weight"), g("norm1.bias"))
    q = _split_heads(linear(n1, g("attention.q_proj.weight"), g("attention.q_proj.bias")), num_heads)
    k = _split_heads(linear(n1, g("attention.k_proj.weight"), g("attention.k_proj.bias")), num_heads)
    v = _split_heads(linear(n1, g("attention.v_proj.weight"), g("attention.v_proj.bias")), num_heads)
    ctx = _merge_heads(causal_attention(q, k, v, causal=causal, key_valid=valid_token_mask))
    attn_out = linear(ctx, g("attention.out_proj.weight"), g("attention.out_proj.bias"))
    if valid_token_mask is not None:
        attn_out = np.where(valid_token_mask[..., None], attn_out, dt.type(0))
    x = x + attn_out
    n2 = layer_norm(x, g("norm2.weight"), g("norm2.bias"))
    hdn = gelu_erf(linear(n2, g("ffn_in.weight"), g("ffn_in.bias")))
    x = x + linear(hdn, g("ffn_out.weight"), g("ffn_out.bias"))
    if valid_token_mask is not None:
        x = np.where(valid_token_mask[..., None], x, dt.type(0))
    return x


def model_forward(params: Dict[str, np.ndarray], cfg: OracleConfig, x: np.ndarray,
                  valid_token_mask: Optional[np.ndarray] = None,
                  dtype=np.float32) -> np.ndarray:
    """Whole model, TTB:182-192: the layer loop, then ``final_norm``."""
    x = np.asarray(x, dtype=dtype)
    for i in range(cfg.num_layers):
        x = block_forward(params, i, x, cfg.num_heads, cfg.causal, valid_token_mask)
    x = layer_norm(x, _p(params, "final_norm.weight", dtype), _p(params, "final_norm.bias", dtype))
    if valid_token_mask is not None:
        x = np.where(valid_token_mask[..., None], x, x.dtype.type(0))
    return x


def sampled_rows_forward(params: Dict[str, np.ndarray], num_heads: int, x_seq: np.ndarray,
                         rows: Iterable[int], dtype=np.float32,
                         key_block: int = 8192) -> np.ndarray:
    """Exact single-layer causal output for selected rows of ONE sequence.

    For a causal, unpadded, one-layer model, output row ``t`` depends only on
    ``x[0..t]`` (TTB:119-123 masks every later key), so it can be computed
    without the full ``[S, S]`` score matrix: LN1 and the K/V projections over
    the prefix ``0..max(rows)`` (in ``key_block`` row blocks), then, per
    sampled row, its query, a softmax over its prefix, and the row-wise tail of
    the block (out_proj, residual, LN2, FFN, residual, final_norm) -- the same
    operations as :func:`model_forward`, restricted to the needed rows.  Used
    for the S=100000 configuration, whose score tensor cannot be materialised.

    x_seq: [S, d] one sequence.  Returns [len(set(rows)), d], rows in ascending order.
    """
    rows = np.asarray(sorted(set(int(r) for r in rows)), dtype=np.int64)
    x_seq = np.asarray(x_seq)
    d = x_seq.shape[-1]
    H = num_heads
    hd = d // H
    dt = np.dtype(dtype)
    g = lambda n: _p(params, "layers.0." + n, dt)  # noqa: E731
    T = int(rows.max()) + 1
    wk, bk = g("attention.k_proj.weight"), g("attention.k_proj.bias")
    wv, bv = g("attention.v_proj.weight"), g("attention.v_proj.bias")
    kk = np.empty((T, d), dtype=dt)
    vv = np.empty((T, d), dtype=dt)
    for c0 in range(0, T, key_block):
        c1 = min(T, c0 + key_block)
        n1 = layer_norm(x_seq[c0:c1].astype(dt), g("norm1.weight"), g("norm1.bias"))
        kk[c0:c1] = linear(n1, wk, bk)
        vv[c0:c1] = linear(n1, wv, bv)
    xr = x_seq[rows].astype(dt)
    n1r = layer_norm(xr, g("norm1.weight"), g("norm1.bias"))
    qr = linear(n1r, g("attention.q_proj.weight"), g("attention.q_proj.bias"))
    ctx = np.empty((len(rows), d), dtype=dt)
    scale = dt.type(hd ** -0.5)
    for i, t in enumerate(rows):
        for h in range(H):
            sl = slice(h * hd, (h + 1) * hd)
            s = (kk[: t + 1, sl] @ qr[i, sl]) * scale
            p = _softmax_lastdim(s.astype(np.float32 if dt == np.float32 else dt)).astype(dt)
            ctx[i, sl] = p @ vv[: t + 1, sl]
    x1 = xr + linear(ctx, g("attention.out_proj.weight"), g("attention.out_proj.bias"))
    n2 = layer_norm(x1, g("norm2.weight"), g("norm2.bias"))
    x2 = x1 + linear(gelu_erf(linear(n2, g("ffn_in.weight"), g("ffn_in.bias"))),
                     g("ffn_out.weight"), g("ffn_out.bias"))
    return layer_norm(x2, _p(params, "final_norm.weight", dt), _p(params, "final_norm.bias", dt))


def prefix_kv(params: Dict[str, np.ndarray], x_seq: np.ndarray, c1: int, dtype=np.float32) -> tuple:
    """K and V ([c1, d] each) of the first ``c1`` rows of one sequence: LN1, then the
    k/v projections (TTB:110-112) -- the K/V cache of the reference's chunked forward."""
    dt = np.dtype(dtype)
    g = lambda n: _p(params, "layers.0." + n, dt)  # noqa: E731
    n1p = layer_norm(np.asarray(x_seq)[:c1].astype(dt), g("norm1.weight"), g("norm1.bias"))
    return (linear(n1p, g("attention.k_proj.weight"), g("attention.k_proj.bias")),
            linear(n1p, g("attention.v_proj.weight"), g("attention.v_proj.bias")))


def chunk_rows_forward(params: Dict[str, np.ndarray], num_heads: int, x_seq: np.ndarray, c0: int, c1: int,
                       kv: Optional[tuple] = None, dtype=np.float32) -> np.ndarray:
    """Exact one-layer causal output for the query chunk ``[c0, c1)`` of ONE sequence.

    The body of the reference's sequence-chunked forward (TTB:1378-1609) for one
    chunk, in fp32 and with the rows of the chunk processed together: LN1 and the
    K/V projections over the prefix ``0..c1`` (or ``kv = (K, V)`` already
    computed, ``[>= c1, d]``), the chunk's queries, a bottom-right-aligned causal
    softmax over the prefix (query ``c0 + i`` sees keys ``0..c0 + i``,
    TTB:1491-1500), then out_proj, residual, LN2, FFN, residual and final_norm
    -- the same operations as :func:`model_forward` restricted to the chunk's rows.
    x_seq: [S, d].  Returns [c1 - c0, d]."""
    x_seq = np.asarray(x_seq)
    d = x_seq.shape[-1]
    H = num_heads
    hd = d // H
    dt = np.dtype(dtype)
    g = lambda n: _p(params, "layers.0." + n, dt)  # noqa: E731
    kk, vv = prefix_kv(params, x_seq, c1, dt) if kv is None else kv
    xr = x_seq[c0:c1].astype(dt)
    n1r = layer_norm(xr, g("norm1.weight"), g("norm1.bias"))
    q = linear(n1r, g("attention.q_proj.weight"), g("attention.q_proj.bias"))
    scale = dt.type(hd ** -0.5)
    masked = np.arange(c1)[None, :] > (c0 + np.arange(c1 - c0))[:, None]
    ctx = np.empty((c1 - c0, d), dtype=dt)
    for h in range(H):
        sl = slice(h * hd, (h + 1) * hd)
        s = (q[:, sl] @ kk[:c1, sl].T) * scale
        s = np.where(masked, dt.type(-np.inf), s)
        ctx[:, sl] = _softmax_lastdim(s.astype(np.float32 if dt == np.float32 else dt)).astype(dt) @ vv[:c1, sl]
    x1 = xr + linear(ctx, g("attention.out_proj.weight"), g("attention.out_proj.bias"))
    n2 = layer_norm(x1, g("norm2.weight"), g("norm2.bias"))
    x2 = x1 + linear(gelu_erf(linear(n2, g("ffn_in.weight"), g("ffn_in.bias"))),
                     g("ffn_out.weight"), g("ffn_out.bias"))
    return layer_norm(x2, _p(params, "final_norm.weight", dt), _p(params, "final_norm.bias", dt))
