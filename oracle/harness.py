"""Harness-side helpers restated from the reference (TEST INFRASTRUCTURE).

* :func:`generate_random_case` -- TTB:1766-1804 (seeded ``torch.Generator`` on
  a named device, ``randn(B,S,d) * input_scale``, prefix-valid padding mask).
  Inputs are always generated on the CPU generator so that the CPU oracle and
  the GPU run see the same ``x`` (CPU and CUDA generators give different
  streams for one seed).
* :func:`compare_outputs` -- TTB:1821-1888: an element passes when
  ``|opt-ref| <= atol OR |opt-ref| <= rtol*|ref|`` (stricter than
  ``torch.isclose``), non-finite values fail.
* :func:`generate_chunked_input` -- per-(batch, sequence-chunk) seeding for the
  S=100000 configuration, so any slice can be regenerated on its own
  (the reference learned one generator stream cannot be replayed for a slice,
  experiments/g7_0_chunked_oversize.py:613-619).

"TTB" = torch_transformer_benchmark.py of yeoshuyi/Flipfloppers-GPU-Kernel-Optimizer.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Dict, List, Tuple

import numpy as np
import torch


def generate_random_case(batch_size: int, seq_len: int, d_model: int, seed: int,
                         padding_ratio: float = 0.0, input_scale: float = 1.0,
                         dtype=torch.float32) -> Tuple[torch.Tensor, torch.Tensor]:
    """CPU restatement of TTB:1766-1804; returns ``(x, valid_token_mask)`` on CPU."""
    gen = torch.Generator(device="cpu")
    gen.manual_seed(seed)
    x = torch.randn(batch_size, seq_len, d_model, generator=gen, dtype=dtype)
    x = x * input_scale
    if padding_ratio <= 0:
        return x, torch.ones(batch_size, seq_len, dtype=torch.bool)
    min_valid = max(1, int(round(seq_len * (1.0 - padding_ratio))))
    lengths = torch.randint(low=min_valid, high=seq_len + 1, size=(batch_size,), generator=gen)
    valid = torch.arange(seq_len)[None, :] < lengths[:, None]
    x = x.masked_fill(~valid[..., None], 0)
    return x, valid


def generate_chunked_input(batch_size: int, seq_len: int, d_model: int, seed: int,
                           chunk: int = 8192, batches=None, rows: int = None,
                           out: torch.Tensor = None) -> torch.Tensor:
    """x ~ N(0,1) fp32 built per (b, chunk) from ``seed + 1_000_003*b + chunk_index``.

    ``batches`` selects which batch elements to build (default all); ``rows``
    truncates each sequence to its first ``rows`` positions (the CPU oracle
    only needs a prefix).  ``out`` may be a preallocated (pinned) CPU tensor.
    """
    batches = list(range(batch_size)) if batches is None else list(batches)
    rows = seq_len if rows is None else min(rows, seq_len)
    if out is None:
        out = torch.empty(len(batches), rows, d_model, dtype=torch.float32)
    gen = torch.Generator(device="cpu")
    for i, b in enumerate(batches):
        for ci, c0 in enumerate(range(0, rows, chunk)):
            c1 = min(rows, c0 + chunk)
            gen.manual_seed(seed + 1_000_003 * b + ci)
            # draw the full chunk so that a truncated prefix reproduces the same values
            full = torch.randn(min(chunk, seq_len - c0), d_model, generator=gen)
            out[i, c0:c1] = full[: c1 - c0]
    return out


def params_from_state_dict(sd) -> Dict[str, np.ndarray]:
    """state_dict (torch tensors) -> dict of float32 NumPy arrays, same keys."""
    return {k: v.detach().to("cpu", torch.float32).numpy() for k, v in sd.items()}


@dataclass
class AccuracyResult:
    passed: bool
    total_elements: int
    failed_elements: int
    max_abs_error: float
    max_relative_error: float
    mean_abs_error: float
    failed_feature_dims: List[int]
    worst_index: Tuple[int, ...]
    reference_at_worst: float
    optimized_at_worst: float


def compare_outputs(reference, optimized, rtol: float = 0.02, atol: float = 0.002) -> AccuracyResult:
    """The reference harness's element-wise gate (TTB:1821-1888)."""
    ref = torch.as_tensor(np.asarray(reference) if not torch.is_tensor(reference) else reference)
    opt = torch.as_tensor(np.asarray(optimized) if not torch.is_tensor(optimized) else optimized)
    if tuple(ref.shape) != tuple(opt.shape):
        raise AssertionError(f"shape mismatch: baseline={tuple(ref.shape)}, optimized={tuple(opt.shape)}")
    ref = ref.detach().to("cpu", torch.float64)
    opt = opt.detach().to("cpu", torch.float64)
    finite = torch.isfinite(ref) & torch.isfinite(opt)
    err = (opt - ref).abs()
    passed_mask = finite & ((err <= atol) | (err <= rtol * ref.abs()))
    failed_mask = ~passed_mask
    failed = int(failed_mask.sum().item())
    err_f = torch.where(torch.isfinite(err), err, torch.full_like(err, float("inf")))
    flat_worst = int(err_f.reshape(-1).argmax().item()) if err.numel() else 0
    worst = []
    rem = flat_worst
    for size in reversed(ref.shape):
        worst.append(rem % size)
        rem //= size
    worst_index = tuple(reversed(worst))
    rel = err / ref.abs().clamp_min(1e-12)
    if ref.ndim >= 2:
        failed_dims = torch.nonzero(failed_mask.any(dim=tuple(range(ref.ndim - 1))), as_tuple=False).flatten().tolist()
    else:
        failed_dims = torch.nonzero(failed_mask, as_tuple=False).flatten().tolist()
    return AccuracyResult(
        passed=failed == 0,
        total_elements=ref.numel(),
        failed_elements=failed,
        max_abs_error=float(err_f.max().item()) if err.numel() else 0.0,
        max_relative_error=float(rel.max().item()) if err.numel() else 0.0,
        mean_abs_error=float(err.mean().item()) if err.numel() else 0.0,
        failed_feature_dims=failed_dims,
        worst_index=worst_index,
        reference_at_worst=float(ref[worst_index].item()) if err.numel() else 0.0,
        optimized_at_worst=float(opt[worst_index].item()) if err.numel() else 0.0,
    )


def init_state_dict(num_layers: int, d_model: int, ffn_dim: int, seed: int) -> Dict[str, torch.Tensor]:
    """Parameters drawn exactly as ``torch.manual_seed(seed); BaselineTransformer(cfg)``.

    The reference constructs, per layer, norm1 (no RNG), q/k/v/out_proj
    Linears (TTB:92-95), norm2, ffn_in, ffn_out (TTB:148-152); final_norm last
    (TTB:180).  nn.Linear draws its weight then its bias, so creating the same
    Linears in the same order reproduces the reference's weights bit for bit.
    """
    import torch.nn as nn

    torch.manual_seed(seed)
    sd: Dict[str, torch.Tensor] = {}
    for i in range(num_layers):
        p = f"layers.{i}."
        n1 = nn.LayerNorm(d_model)
        lins = {}
        for name in ("q_proj", "k_proj", "v_proj", "out_proj"):
            lins[name] = nn.Linear(d_model, d_model)
        n2 = nn.LayerNorm(d_model)
        fi = nn.Linear(d_model, ffn_dim)
        fo = nn.Linear(ffn_dim, d_model)
        sd[p + "norm1.weight"], sd[p + "norm1.bias"] = n1.weight.data, n1.bias.data
        for name, lin in lins.items():
            sd[p + f"attention.{name}.weight"] = lin.weight.data
            sd[p + f"attention.{name}.bias"] = lin.bias.data
        sd[p + "norm2.weight"], sd[p + "norm2.bias"] = n2.weight.data, n2.bias.data
        sd[p + "ffn_in.weight"], sd[p + "ffn_in.bias"] = fi.weight.data, fi.bias.data
        sd[p + "ffn_out.weight"], sd[p + "ffn_out.bias"] = fo.weight.data, fo.bias.data
    fn = nn.LayerNorm(d_model)
    sd["final_norm.weight"], sd["final_norm.bias"] = fn.weight.data, fn.bias.data
    return sd


def fingerprint(sd) -> Dict[str, Tuple[float, float]]:
    """Per-tensor (sum, sum of squares) in float64 -- pins weight generation."""
    out = {}
    for k, v in sd.items():
        a = v.detach().to("cpu", torch.float64)
        out[k] = (float(a.sum().item()), float((a * a).sum().item()))
    return out
