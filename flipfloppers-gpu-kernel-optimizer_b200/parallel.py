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
  row-parallel.  Each row-parallel GEMM yields an fp32 partial that one NCCL
  all-reduce (sum) completes; bias, residual and the next LayerNorm run once,
  after it, in one fused kernel.  The block runs over query chunks of each
  sequence with a K/V cache of the local heads, as the reference's
  sequence-chunked forward does (TTB:1378-1609), and each chunk's two
  all-reduces run on a side stream while the compute stream works on the next
  chunks (:func:`tp_schedule`).

:class:`TensorParallelPlan` is the pure host-side part (which heads / FFN
columns a rank owns, how the reference's ``state_dict`` tensors are sliced);
it is shared by the GPU executor and the CPU (gloo) tests.
"""

from __future__ import annotations

import os
from dataclasses import dataclass
from typing import Dict, List, Optional, Tuple

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

    def __call__(self, x_local: torch.Tensor, gather: bool = False, batch: Optional[int] = None,
                 valid_token_mask: Optional[torch.Tensor] = None) -> torch.Tensor:
        """``x_local`` / ``valid_token_mask``: this rank's batch slice (the mask as in the module's forward)."""
        y = self.model(x_local, valid_token_mask)
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




def tp_schedule(n_chunks: int) -> List[Tuple[str, int]]:
    """Order of the compute stream's stages over the chunks of one layer.

    ``("A", i)``: chunk i's LN1, Q and K/V projections (K/V into the cache),
    attention on the local heads and the out_proj partial; its all-reduce is
    then queued on the communication stream.
    ``("B", i)``: after that all-reduce, residual + bias + LN2 in one kernel, ffn_in
    + GELU, the ffn_out partial; its all-reduce is queued.
    ``("F", i)``: after that all-reduce, residual + bias + final LN (or the next
    layer's input).
    Pipelined two deep -- A(i), B(i-1), F(i-2) -- so that chunk i's compute runs
    while chunk i-1's and i-2's all-reduces are in flight.  Every rank issues the
    collectives in this same order.  Per-chunk buffers alternate between two
    slots (i % 2): a slot is rewritten by A(i+2) / B(i+2) only after B(i) / F(i),
    the last readers of chunk i's partial sums, are on the compute stream."""
    out: List[Tuple[str, int]] = []
    for i in range(n_chunks + 2):
        if i < n_chunks:
            out.append(("A", i))
        if 0 <= i - 1 < n_chunks:
            out.append(("B", i - 1))
        if 0 <= i - 2 < n_chunks:
            out.append(("F", i - 2))
    return out


def tp_chunks(batch: int, seq_len: int, chunk_rows: int) -> List[Tuple[int, int, int, int]]:
    """Query chunks ``(b0, nb, c0, c1)``: sequences ``b0 .. b0+nb-1``, query rows ``[c0, c1)``
    of each.  Sequences longer than ``chunk_rows`` are cut into prefix chunks (nb = 1,
    attention over keys ``[0, c1)``); shorter ones are grouped whole, several per chunk.
    The chunk's rows are contiguous in the ``[batch*seq_len, d]`` layout."""
    if chunk_rows <= 0:
        raise ValueError("chunk_rows must be positive")
    out = []
    if seq_len >= chunk_rows:
        for b in range(batch):
            for c0 in range(0, seq_len, chunk_rows):
                out.append((b, 1, c0, min(seq_len, c0 + chunk_rows)))
    else:
        g = max(1, chunk_rows // seq_len)
        for b0 in range(0, batch, g):
            out.append((b0, min(g, batch - b0), 0, seq_len))
    return out


class TensorParallelTransformer:
    """Causal model with heads / FFN columns split across a TP process group (NCCL).

    Per layer and query chunk (R rows, dl = d/tp, fl = ffn/tp), on each rank:
      A: n = LN1(x) [R,d] f16 ; q = n.Wq[hc]^T [R,dl] ; K|V rows = n.Wkv[hc]^T into the
         cache [M, 2dl] ; ctx = prefix-causal attention of the local heads [R,dl] ;
         p1 = ctx.W_o[:,hc]^T [R,d] f32 ; all_reduce(p1) on the side stream
      B: x1 = x + p1 + b_o and n = LN2(x1) (one kernel) ; h = gelu(n.W_in[fc]^T + b_in[fc])
         [R,fl] ; p2 = h.W_out[:,fc]^T [R,d] f32 ; all_reduce(p2) on the side stream
      F: y = LN_f(x1 + p2 + b_out) (one kernel; for a layer before the last, its output)
    in the order of :func:`tp_schedule`.  Every rank holds the full activations of its
    sequences (x, x1 and y are replicated across the TP group); weights and the K/V
    cache are sharded, so each rank streams 1/tp of them.  Weights are sliced once and
    again only when a parameter changes (the module's own parameter key); buffers are
    allocated once per shape.  ``comm_ms()`` reports the time the all-reduces of the
    last call spent on the side stream when built with ``profile_comm=True``.
    """

    def __init__(self, model, tp_rank: int, tp_size: int, group=None, chunk_rows: int = 32768,
                 profile_comm: bool = False):
        cfg = model.config
        if not cfg.causal:
            raise ValueError("the chunked tensor-parallel forward is causal (prefix chunks)")
        self.model = model
        self.group = group
        self.plan = TensorParallelPlan(cfg.d_model, cfg.num_heads, cfg.ffn_dim, tp_rank, tp_size)
        dl = cfg.d_model // tp_size
        if dl % 32 or (cfg.ffn_dim // tp_size) % 32:
            raise ValueError("d_model / tp and ffn_dim / tp must be multiples of 32 (GEMM granule)")
        self.chunk_rows = int(chunk_rows)
        self.profile_comm = profile_comm
        self._weights: Optional[List[Dict[str, torch.Tensor]]] = None
        self._key = None
        self._bufs: Dict[tuple, Dict[str, object]] = {}
        self._comm: Dict[int, torch.cuda.Stream] = {}
        self._comm_events: List[Tuple[torch.cuda.Event, torch.cuda.Event]] = []

    def _ensure_weights(self, device):
        key = self.model._param_key(device)
        if key == self._key:
            return
        sd = self.model.state_dict()
        out = []
        with torch.no_grad():
            for i in range(self.model.config.num_layers):
                sh = self.plan.shard_layer(sd, i)
                out.append({k: (v.detach().to(device, torch.float16) if k.startswith("w_") else
                                v.detach().to(device, torch.float32)).contiguous() for k, v in sh.items()})
            self._lnf = (self.model.final_norm.weight.detach().to(device, torch.float32).contiguous(),
                         self.model.final_norm.bias.detach().to(device, torch.float32).contiguous())
        self._weights = out
        self._key = key

    def _buffers(self, B: int, S: int, device) -> Dict[str, object]:
        key = (B, S, device.index)
        bufs = self._bufs.get(key)
        if bufs is not None:
            return bufs
        cfg, pl = self.model.config, self.plan
        d = cfg.d_model
        dl, fl = d // pl.tp_size, cfg.ffn_dim // pl.tp_size
        chunks = tp_chunks(B, S, self.chunk_rows)
        R = max(nb * (c1 - c0) for _, nb, c0, c1 in chunks)
        e = lambda *shape, dt=torch.float16: torch.empty(*shape, dtype=dt, device=device)  # noqa: E731
        bufs = {
            "chunks": chunks,
            "kv": e(B * S, 2 * dl),
            "n": e(R, d), "q": e(R, dl), "ctx": e(R, dl), "n2": e(R, d), "h": e(R, fl),
            "p1": [e(R, d, dt=torch.float32) for _ in range(2)],
            "x1": [e(R, d, dt=torch.float32) for _ in range(2)],
            "p2": [e(R, d, dt=torch.float32) for _ in range(2)],
            "scratch": e(R, d),
            "xmid": e(B * S, d, dt=torch.float32) if cfg.num_layers > 1 else None,
            "ev": {k: [torch.cuda.Event() for _ in range(2)] for k in ("a", "b", "c1", "c2")},
        }
        self._bufs[key] = bufs
        return bufs

    def _comm_stream(self, device) -> torch.cuda.Stream:
        """The side stream of the all-reduces, at the highest priority: as the attention
        kernel's CTAs (one per SM) retire, the block scheduler places NCCL's blocks first
        instead of the next compute CTAs, so a chunk's reduce is not starved by the next
        chunk's compute (B200_TP_COMM_PRIORITY=0 gives it normal priority)."""
        s = self._comm.get(device.index)
        if s is None:
            hi = os.environ.get("B200_TP_COMM_PRIORITY", "1") != "0"
            s = torch.cuda.Stream(device=device, priority=-1 if hi else 0)
            self._comm[device.index] = s
        return s

    def _all_reduce(self, t: torch.Tensor, after: torch.cuda.Event, done: torch.cuda.Event, comm) -> None:
        comm.wait_event(after)
        with torch.cuda.stream(comm):
            if self.profile_comm:
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record(comm)
            dist.all_reduce(t, op=dist.ReduceOp.SUM, group=self.group)
            if self.profile_comm:
                b.record(comm)
                self._comm_events.append((a, b))
        done.record(comm)

    def comm_ms(self) -> float:
        """Side-stream time (ms) of the last call's all-reduces (needs profile_comm; synchronises)."""
        torch.cuda.synchronize()
        return sum(a.elapsed_time(b) for a, b in self._comm_events)

    @torch.no_grad()
    def __call__(self, x: torch.Tensor, valid_token_mask: Optional[torch.Tensor] = None,
                 out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """y = model(x, valid_token_mask) with the work split over the TP group.  A key-padding
        mask is turned into key counts, hole flags and key bits on the device
        (``b200_mask_prepare``), which every chunk's attention applies; padded rows of the
        output are zeroed at the end."""
        if not x.is_cuda:
            raise RuntimeError("TensorParallelTransformer runs on CUDA devices only (no CPU fallback)")
        cfg, pl = self.model.config, self.plan
        B, S, d = x.shape
        dev = x.device
        mask = self.model._mask_bytes(valid_token_mask, B, S, dev)
        keys = None
        if mask is not None:
            keys = self.model._mask_buffers(B, S, dev)
            rt.mask_prepare(mask, *keys)
        self._ensure_weights(dev)
        bufs = self._buffers(B, S, dev)
        comm = self._comm_stream(dev)
        cur = torch.cuda.current_stream(dev)
        comm.wait_stream(cur)  # the input (and last call's readers) are ordered before this call
        self._comm_events = []
        dl, fl, hd, Hl = d // pl.tp_size, cfg.ffn_dim // pl.tp_size, pl.head_dim, pl.local_heads
        eps = float(self.model.layers[0].norm1.eps)
        xf = x.reshape(B * S, d)
        if xf.dtype != torch.float32 or not xf.is_contiguous():
            xf = xf.to(torch.float32).contiguous()
        if out is not None and (out.dtype != torch.float32 or not out.is_contiguous() or out.numel() != B * S * d
                                or out.device != dev):
            raise ValueError("out must be a contiguous float32 tensor of x's shape on x's device")
        y = torch.empty(B * S, d, dtype=torch.float32, device=dev) if out is None else out.view(B * S, d)
        chunks = bufs["chunks"]
        ev = bufs["ev"]
        kv = bufs["kv"]
        nl = len(self._weights)
        for li, w in enumerate(self._weights):
            last = li == nl - 1
            src = xf if li == 0 else bufs["xmid"]
            dst = y if last else bufs["xmid"]  # in place for middle layers: a chunk's rows are
            #                                    rewritten by F only after A and B have read them
            wq, bq = w["w_qkv"][:dl], w["b_qkv"][:dl]
            wkv, bkv = w["w_qkv"][dl:], w["b_qkv"][dl:]

            def rows_of(i):
                b0, nb, c0, c1 = chunks[i]
                r0 = b0 * S + c0
                return r0, r0 + nb * (c1 - c0)

            for stage, i in tp_schedule(len(chunks)):
                b0, nb, c0, c1 = chunks[i]
                r0, r1 = rows_of(i)
                R = r1 - r0
                sl = i % 2
                if stage == "A":
                    n, q, ctx, p1 = bufs["n"][:R], bufs["q"][:R], bufs["ctx"][:R], bufs["p1"][sl][:R]
                    rt.layernorm(src[r0:r1], w["ln1_w"], w["ln1_b"], n, eps)
                    rt.gemm(rt.EPI_BIAS_F16, n, wq, bq, q)
                    rt.gemm(rt.EPI_BIAS_F16, n, wkv, bkv, kv[r0:r1])
                    # keys of the chunk's sequences up to its last row; the cache ends there, so the
                    # key tile that straddles it reads zeros instead of rows not written yet
                    kvv = kv[: r1]
                    qlen = c1 - c0
                    mk = {} if keys is None else dict(key_holes=keys[1][b0:b0 + nb], key_bits=keys[2][b0:b0 + nb])
                    rt.flash_causal(q, kvv, kvv, ctx, batch=nb, heads=Hl, head_dim=hd, q_len=qlen,
                                    kv_len=c1, q_offset=c0, q_seq_rows=qlen, kv_seq_rows=S, q_col0=0,
                                    k_col0=0, v_col0=dl, kv_row0=b0 * S, out_seq_rows=qlen, **mk)
                    rt.gemm(rt.EPI_BIAS_F32, ctx, w["w_o"], None, p1)
                    ev["a"][sl].record(cur)
                    self._all_reduce(bufs["p1"][sl][:R], ev["a"][sl], ev["c1"][sl], comm)
                elif stage == "B":
                    cur.wait_event(ev["c1"][sl])
                    n2, h, x1, p2 = bufs["n2"][:R], bufs["h"][:R], bufs["x1"][sl][:R], bufs["p2"][sl][:R]
                    rt.add_layernorm(src[r0:r1], bufs["p1"][sl][:R], w["b_o"], x1, w["ln2_w"], w["ln2_b"], n2, eps)
                    rt.gemm(rt.EPI_BIAS_GELU_F16, n2, w["w_in"], w["b_in"], h)
                    rt.gemm(rt.EPI_BIAS_F32, h, w["w_out"], None, p2)
                    ev["b"][sl].record(cur)
                    self._all_reduce(p2, ev["b"][sl], ev["c2"][sl], comm)
                else:
                    cur.wait_event(ev["c2"][sl])
                    x1, p2 = bufs["x1"][sl][:R], bufs["p2"][sl][:R]
                    if last:
                        rt.add_layernorm(x1, p2, w["b_out"], x1, self._lnf[0], self._lnf[1], dst[r0:r1], eps)
                    else:  # the next layer's input; the LayerNorm output goes to a scratch buffer
                        rt.add_layernorm(x1, p2, w["b_out"], dst[r0:r1], w["ln2_w"], w["ln2_b"],
                                         bufs["scratch"][:R], eps)
        if mask is not None:
            rt.zero_masked_rows(y, mask)
        return y.reshape(B, S, d)
