"""Multi-GPU execution: one process per GPU, ``torch.distributed`` for the plumbing.

The reference has no distributed code (its long-context path is single-GPU
sequence chunking, TTB:1378-1609); this module adds the two partitionings the
block admits:

* **batch sharding** (:class:`BatchShardedTransformer`): sequences are
  independent (attention is per sequence, LayerNorm and the FFN per token), so
  each rank runs the whole model on a contiguous slice of the batch.  No
  collective on the data path; outputs are gathered only when asked.
* **tensor parallelism** (:class:`TensorParallelTransformer`): heads are split
  across the ranks of a TP group -- QKV column-parallel, attention on local
  heads, out_proj row-parallel -- then ffn_in column-parallel and ffn_out
  row-parallel.  Each row-parallel GEMM yields an fp32 partial ``[M, d]`` that
  one NCCL all-reduce (sum) completes; bias, residual and the next LayerNorm
  run once, after it, in one fused kernel.

:class:`TensorParallelPlan` is the pure host-side part (which heads / FFN
columns a rank owns, how the reference's ``state_dict`` tensors are sliced);
it is shared by the GPU executor and the CPU (gloo) tests.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Dict, List, Optional

import torch
import torch.distributed as dist

from . import runtime as rt


def batch_shard(batch: int, rank: int, world: int) -> slice:
    """Contiguous shard of ``batch`` sequences for ``rank`` (sizes differ by at most one)."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError("invalid rank/world")
    base, extra = divmod(batch, world)
    start = rank * base + min(rank, extra)
    return slice(start, start + base + (1 if rank < extra else 0))


class BatchShardedTransformer:
    """Runs ``model`` on this rank's batch shard; ``gather=True`` all-gathers the outputs."""

    def __init__(self, model, rank: int, world: int, group=None):
        self.model, self.rank, self.world, self.group = model, rank, world, group

    def local_slice(self, batch: int) -> slice:
        return batch_shard(batch, self.rank, self.world)

    def __call__(self, x_local: torch.Tensor, gather: bool = False, batch: Optional[int] = None) -> torch.Tensor:
        y = self.model(x_local)
        if not gather or self.world == 1:
            return y
        batch = batch if batch is not None else x_local.shape[0] * self.world
        sizes = [batch_shard(batch, r, self.world).stop - batch_shard(batch, r, self.world).start
                 for r in range(self.world)]
        parts = [torch.empty((n,) + tuple(y.shape[1:]), dtype=y.dtype, device=y.device) for n in sizes]
        dist.all_gather(parts, y.contiguous(), group=self.group)
        return torch.cat(parts, 0)


@dataclass
class TensorParallelPlan:
    """Which heads and FFN columns TP rank ``tp_rank`` of ``tp_size`` owns."""

    d_model: int
    num_heads: int
    ffn_dim: int
    tp_rank: int
    tp_size: int

    def __post_init__(self):
        if self.num_heads % self.tp_size or self.ffn_dim % self.tp_size:
            raise ValueError(f"num_heads ({self.num_heads}) and ffn_dim ({self.ffn_dim}) must divide by tp_size "
                             f"({self.tp_size})")
        if not 0 <= self.tp_rank < self.tp_size:
            raise ValueError("invalid tp_rank")

    @property
    def head_dim(self) -> int:
        return self.d_model // self.num_heads

    @property
    def local_heads(self) -> int:
        return self.num_heads // self.tp_size

    @property
    def head_cols(self) -> slice:
        """Columns of q/k/v (and rows of the context) this rank owns."""
        w = self.local_heads * self.head_dim
        return slice(self.tp_rank * w, (self.tp_rank + 1) * w)

    @property
    def ffn_cols(self) -> slice:
        w = self.ffn_dim // self.tp_size
        return slice(self.tp_rank * w, (self.tp_rank + 1) * w)

    def shard_layer(self, sd: Dict[str, torch.Tensor], layer: int) -> Dict[str, torch.Tensor]:
        """Slices of one layer's parameters (reference state_dict names) for this rank.

        w_qkv [3*dl, d]  rows q[hc] | k[hc] | v[hc]          (column-parallel)
        w_o   [d, dl]    out_proj.weight[:, hc]               (row-parallel)
        w_in  [fl, d]    ffn_in.weight[fc]                    (column-parallel)
        w_out [d, fl]    ffn_out.weight[:, fc]                (row-parallel)
        b_o / b_out and the LayerNorm parameters are full (applied after the reduce).
        """
        p = f"layers.{layer}."
        hc, fc = self.head_cols, self.ffn_cols
        g = lambda n: sd[p + n]  # noqa: E731
        return {
            "ln1_w": g("norm1.weight"), "ln1_b": g("norm1.bias"),
            "w_qkv": torch.cat([g("attention.q_proj.weight")[hc], g("attention.k_proj.weight")[hc],
                                g("attention.v_proj.weight")[hc]], 0),
            "b_qkv": torch.cat([g("attention.q_proj.bias")[hc], g("attention.k_proj.bias")[hc],
                                g("attention.v_proj.bias")[hc]], 0),
            "w_o": g("attention.out_proj.weight")[:, hc], "b_o": g("attention.out_proj.bias"),
            "ln2_w": g("norm2.weight"), "ln2_b": g("norm2.bias"),
            "w_in": g("ffn_in.weight")[fc], "b_in": g("ffn_in.bias")[fc],
            "w_out": g("ffn_out.weight")[:, fc], "b_out": g("ffn_out.bias"),
        }


class TensorParallelTransformer:
    """Causal model with heads / FFN columns split across a TP process group (NCCL).

    Per layer on each rank (M = B*S tokens, dl = d/tp, fl = ffn/tp):
      LN1(x) -> n [M,d] f16 ; QKV GEMM (local rows) -> [M,3dl] ; flash attention
      on the local heads -> ctx [M,dl] ; out_proj partial ctx.W_o[:,hc]^T -> [M,d]
      f32 ; all_reduce(sum) ; x1 = x + partial + b_o and n = LN2(x1) (one fused
      kernel) ; ffn_in local + GELU -> [M,fl] ; ffn_out partial -> [M,d] f32 ;
      all_reduce(sum) ; x2 = x1 + partial + b_out, then final LayerNorm.
    Every rank holds the full activations x, x1 (replicated); weights are
    sharded, so each rank streams 1/tp of them.
    """

    def __init__(self, model, tp_rank: int, tp_size: int, group=None):
        cfg = model.config
        self.model = model
        self.group = group
        self.plan = TensorParallelPlan(cfg.d_model, cfg.num_heads, cfg.ffn_dim, tp_rank, tp_size)
        self._weights: Optional[List[Dict[str, torch.Tensor]]] = None
        self._key = None

    def _ensure_weights(self, device):
        key = (device, tuple((id(p), p._version) for p in self.model.parameters()))
        if key == self._key:
            return
        sd = self.model.state_dict()
        out = []
        for i in range(self.model.config.num_layers):
            sh = self.plan.shard_layer(sd, i)
            out.append({k: (v.detach().to(device, torch.float16) if k.startswith("w_") else
                            v.detach().to(device, torch.float32)).contiguous() for k, v in sh.items()})
        self._weights = out
        self._lnf = (self.model.final_norm.weight.detach().to(device, torch.float32).contiguous(),
                     self.model.final_norm.bias.detach().to(device, torch.float32).contiguous())
        self._key = key

    @torch.no_grad()
    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        if not x.is_cuda:
            raise RuntimeError("TensorParallelTransformer runs on CUDA devices only")
        cfg, pl = self.model.config, self.plan
        B, S, d = x.shape
        M = B * S
        dev = x.device
        self._ensure_weights(dev)
        dl, fl, hd, Hl = d // pl.tp_size, cfg.ffn_dim // pl.tp_size, pl.head_dim, pl.local_heads
        eps = float(self.model.layers[0].norm1.eps)
        xf = x.reshape(M, d).to(torch.float32).contiguous()
        n = torch.empty(M, d, dtype=torch.float16, device=dev)
        qkv = torch.empty(M, 3 * dl, dtype=torch.float16, device=dev)
        ctx = torch.empty(M, dl, dtype=torch.float16, device=dev)
        part = torch.empty(M, d, dtype=torch.float32, device=dev)
        x1 = torch.empty(M, d, dtype=torch.float32, device=dev)
        h = torch.empty(M, fl, dtype=torch.float16, device=dev)
        nl = len(self._weights)
        y = torch.empty(M, d, dtype=torch.float32, device=dev)
        cur = xf
        rt.layernorm(cur, self._weights[0]["ln1_w"], self._weights[0]["ln1_b"], n, eps)
        for i, w in enumerate(self._weights):
            rt.gemm(rt.EPI_BIAS_F16, n, w["w_qkv"], w["b_qkv"], qkv)
            rt.flash_causal(qkv, qkv, qkv, ctx, batch=B, heads=Hl, head_dim=hd, q_len=S, kv_len=S,
                            q_col0=0, k_col0=dl, v_col0=2 * dl, non_causal=not cfg.causal)
            rt.gemm(rt.EPI_BIAS_F32, ctx, w["w_o"], None, part)
            dist.all_reduce(part, op=dist.ReduceOp.SUM, group=self.group)
            # x1 = x + partial + b_o ; n = LN2(x1)
            rt.add_layernorm(cur, part, w["b_o"], x1, w["ln2_w"], w["ln2_b"], n, eps)
            rt.gemm(rt.EPI_BIAS_GELU_F16, n, w["w_in"], w["b_in"], h)
            rt.gemm(rt.EPI_BIAS_F32, h, w["w_out"], None, part)
            dist.all_reduce(part, op=dist.ReduceOp.SUM, group=self.group)
            if i == nl - 1:
                # x2 = x1 + partial + b_out ; y = final_norm(x2)
                rt.add_layernorm(x1, part, w["b_out"], x1, self._lnf[0], self._lnf[1], y, eps)
            else:
                # x2 = x1 + partial + b_out becomes the next layer's input; n = its LN1(x2)
                nxt = torch.empty(M, d, dtype=torch.float32, device=dev)
                nw = self._weights[i + 1]
                rt.add_layernorm(x1, part, w["b_out"], nxt, nw["ln1_w"], nw["ln1_b"], n, eps)
                cur = nxt
        return y.reshape(B, S, d)
