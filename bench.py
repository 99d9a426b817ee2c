#!/usr/bin/env python3
"""Benchmark of the causal transformer-block forward on B200 (one JSON line).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference] [--config C2]
    torchrun --nproc-per-node N bench.py --gpus N ...     (N > 1: one process per GPU)

Workload (default): BASELINE configuration 5 (``configs[4]``), the largest
configuration that fits one B200 -- causal pre-LN block, B=32, S=100000,
d=1024, H=16 (head_dim 64), ffn=4096, L=1, fp32 in/out, seeded default init,
x ~ N(0,1) drawn on the device (13 GB).  N>1: the 32 sequences are split
across the ranks (batch sharding, no collective on the data path; strong
scaling, the global batch stays 32); timing is the max over ranks.
``--config C2|C3|C4a|C4b`` measure the other BASELINE configurations (B per
rank fixed: weak scaling), ``--config M7|M11`` two rows of the reference's
official matrix.

``value``: tokens/s of the whole job with x resident in HBM (CUDA events on
the launching stream around each step, L2 flushed between steps by a 256 MiB
write, barrier + synchronize around the timed loop).  ``e2e``: the same
metric through the public API (``UserOptimizedTransformer.__call__``) with
the pinned host->device copy of x and the device->host copy of y inside each
timed step.  ``roofline``: the dominant kernel, timed with CUDA events in an
eager profiling pass over the same workload.  ``cpu_baseline``: the NumPy
restatement of the reference module (oracle/) on the host cores.

``--impl reference`` times the reference's algorithm on the CPU (the oracle
port, all host threads; the reference's own code is Python and does not
travel to the GPU box) on the same config and prints the same line with
``"impl": "reference"``.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)

METRIC = "block forward latency (ms) & tokens/s per shape at 1/2/4/8 B200; % of tensor/HBM roofline"
CONFIGS = {
    # name: (B, S, d, H, ffn, L) -- B per rank (weak scaling) except C5
    "C2": (64, 128, 128, 4, 512, 1),
    "C3": (10000, 128, 128, 4, 512, 1),
    "C4a": (64, 1024, 128, 4, 512, 1),
    "C4b": (64, 128, 1024, 4, 4096, 1),
    "C5": (32, 100000, 1024, 16, 4096, 1),
    # rows 7 and 11 of the reference's official matrix (run_eval.sh:44-58: 4 layers,
    # ffn = d): optional workloads for the d=32 kernel and head_dim-8 attention
    "M7": (64, 128, 32, 4, 32, 4),
    "M11": (64, 128, 128, 16, 128, 4),
    # row 14 (README.md:59: two layers, ffn 1024 at S=100000; the reference's harness cannot
    # score it -- its fp32 baseline runs out of memory -- and times it with a separate probe)
    "M14": (32, 100000, 1024, 16, 1024, 2),
}
# C5 / M14 keep the global batch (B=32) fixed and split it across the ranks (strong scaling)
STRONG = {"C5", "M14"}
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=None, help="timed steps (default 10 for C5, else 200)")
    ap.add_argument("--warmup", type=int, default=None, help="warm-up steps (default 3 for C5, else 20)")
    ap.add_argument("--impl", choices=("b200", "reference"), default="b200")
    ap.add_argument("--config", choices=sorted(CONFIGS), default="C5")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--tp", type=int, default=1,
                    help="tensor-parallel group size (C5): heads / FFN columns split over TP ranks with an NCCL "
                         "all-reduce per row-parallel projection; the remaining factor of --gpus splits the batch")
    ap.add_argument("--chunk-rows", type=int, default=32768, help="query rows per chunk of the tensor-parallel forward")
    a = ap.parse_args()
    if a.steps is None:
        a.steps = 10 if a.config in STRONG else 200
    if a.warmup is None:
        a.warmup = 3 if a.config in STRONG else 20
    return a


def rank_batch(cfg_name, rank, world):
    B = CONFIGS[cfg_name][0]
    if cfg_name in STRONG:
        base, extra = divmod(B, world)
        return base + (1 if rank < extra else 0)
    return B


# bounded CPU sample of the multi-GB configuration (one sequence): the K/V prefix of
# C5_PREFIXES[-1] rows and one query chunk of C5_CHUNK rows ending at each prefix
C5_CHUNK = 512
C5_PREFIXES = (4096, 16384)

# ~20 ms of device-side spinning queued ahead of the timed steps
QUEUE_PREFILL_CYCLES = 40_000_000


def flushes(cfg_name):
    """Flush L2 between steps unless one step's input alone is several times the 126 MB L2."""
    B, S, d = CONFIGS[cfg_name][:3]
    return B * S * d * 4 < (512 << 20)


def workload_name(cfg_name):
    B, S, d, H, F, L = CONFIGS[cfg_name]
    per = "" if cfg_name in STRONG else "/rank"
    return f"{cfg_name}: causal pre-LN block B={B}{per} S={S} d={d} H={H} ffn={F} L={L}"


def config_dict(cfg_name, n):
    B, S, d, H, F, L = CONFIGS[cfg_name]
    strong = cfg_name in STRONG
    return {"workload": workload_name(cfg_name), "batch_per_rank": (B + n - 1) // n if strong else B,
            "global_batch": B if strong else B * n, "seq_len": S,
            "d_model": d, "heads": H, "head_dim": d // H, "ffn_dim": F, "layers": L, "causal": True,
            "parallelism": f"batch-sharded x{n} (no data-path collective)" if n > 1 else "single GPU",
            "l2": ("flushed between timed steps (256 MiB write)" if flushes(cfg_name)
                   else "inputs larger than L2 (no flush)"), "seed": 1234}


def load_peaks():
    p = os.path.join(REPO, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            d = json.load(f)
        return {"hbm_gbs": float(d["hbm_gbs"]), "bf16_tflops": float(d["bf16_tflops"]), "src": "measured"}
    except Exception:  # noqa: BLE001
        return dict(FALLBACK_PEAKS, src="fallback")


# ---------------------------------------------------------------- algorithmic work per kernel
def stage_work(B, S, d, H, F):
    """(flops, bytes) per launch of each chain stage, counted once (causal pairs only)."""
    M = B * S
    return {
        "ln1": (8 * M * d, M * d * 4 + M * d * 2 + 8 * d),
        "qkv": (2 * M * d * 3 * d, M * d * 2 + 3 * d * d * 2 + M * 3 * d * 2 + 12 * d),
        "attn": (2 * B * d * S * (S + 1), M * 3 * d * 2 + M * d * 2),
        "out_proj": (2 * M * d * d, M * d * 2 + d * d * 2 + M * d * 4 * 2 + 4 * d),
        "ln2": (8 * M * d, M * d * 4 + M * d * 2 + 8 * d),
        "ffn_in": (2 * M * d * F, M * d * 2 + F * d * 2 + M * F * 2 + 4 * F),
        "ffn_out": (2 * M * F * d, M * F * 2 + F * d * 2 + M * d * 4 * 2 + 4 * d),
        "ln_f": (8 * M * d, M * d * 4 * 2 + 8 * d),
        # residual projections with the following LayerNorm in the epilogue (d == 128)
        "out_proj_ln2": (2 * M * d * d + 8 * M * d, M * d * 2 + d * d * 2 + M * d * 4 * 2 + M * d * 2 + 12 * d),
        "ffn_out_lnf": (2 * M * F * d + 8 * M * d, M * F * 2 + F * d * 2 + M * d * 4 * 2 + 12 * d),
    }


def block_work(B, S, d, H, F):
    M = B * S
    flops = 2 * M * d * (3 * d + d) + 4 * M * d * F + 2 * B * d * S * (S + 1)  # = 24*M*d^2 + attn at F=4d
    byts = 8 * M * d + 2 * (4 * d * d + 2 * d * F)
    return flops, byts


# ---------------------------------------------------------------- clocks
class ClockSampler:
    def __init__(self, index):
        self.index = index
        self.proc = None
        self.lines = []

    def start(self):
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={q}", "--format=csv,noheader,nounits",
                                          "-lms", "100", "-i", str(self.index)],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            threading.Thread(target=self._read, daemon=True).start()
        except Exception:  # noqa: BLE001
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def median_mhz(self):
        """Median SM clock of the samples taken so far (None without samples)."""
        sm = []
        for ln in list(self.lines):
            parts = [p.strip() for p in ln.split(",")]
            try:
                sm.append(float(parts[1]))
            except (IndexError, ValueError):
                continue
        return statistics.median(sm) if sm else None

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:  # noqa: BLE001
            self.proc.kill()
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for nm, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


# ---------------------------------------------------------------- CPU baseline (oracle port)
def _host_cores():
    try:
        from threadpoolctl import threadpool_info
        return int(max([i.get("num_threads", 1) for i in threadpool_info()] or [os.cpu_count() or 1]))
    except Exception:  # noqa: BLE001
        return os.cpu_count() or 1


def cpu_chunked_step(cfg_name, params, x_seq):
    """One bounded CPU sample of the multi-GB configuration, extrapolated to a full forward.

    A full CPU forward of C5 is infeasible (hours), so one step times the NumPy
    restatement of the reference's chunked forward (oracle.prefix_kv and
    oracle.chunk_rows_forward, TTB:1378-1609) on one sequence: the K/V prefix of
    P2 rows, and one C5_CHUNK-row query chunk ending at P1 and at P2.  A chunk's
    cost is a + b * prefix (projections and FFN of its rows, attention over its
    prefix), so the two chunks fix a and b; a sequence is S / R chunks at
    prefixes R, 2R, .. S plus the K/V projection of S rows, and the forward is B
    sequences.  Returns (estimated seconds per forward, wall seconds of the
    sample, output rows [P2 - R, P2) of the sequence)."""
    import oracle
    B, S, d, H, F, L = CONFIGS[cfg_name]
    P1, P2 = C5_PREFIXES
    R = C5_CHUNK
    w0 = time.perf_counter()
    kv = oracle.prefix_kv(params, x_seq, P2)
    t_kv = time.perf_counter() - w0
    t0 = time.perf_counter()
    oracle.chunk_rows_forward(params, H, x_seq, P1 - R, P1, kv=kv)
    t1 = time.perf_counter() - t0
    t0 = time.perf_counter()
    y2 = oracle.chunk_rows_forward(params, H, x_seq, P2 - R, P2, kv=kv)
    t2 = time.perf_counter() - t0
    wall = time.perf_counter() - w0
    b = max((t2 - t1) / (P2 - P1), 0.0)
    a = max(t1 - b * P1, 0.0)
    n = -(-S // R)
    per_seq = t_kv * S / P2 + n * a + b * R * n * (n + 1) / 2
    return B * per_seq, wall, y2


def cpu_chunked_estimate(cfg_name, x_seq=None, steps=1):
    """cpu_baseline of the multi-GB configuration: the median of ``steps`` samples."""
    import oracle
    B, S, d, H, F, L = CONFIGS[cfg_name]
    params = oracle.params_from_state_dict(oracle.init_state_dict(1, d, F, 1234))
    if x_seq is None:
        x_seq = oracle.generate_chunked_input(1, S, d, seed=1234, rows=C5_PREFIXES[-1])[0].numpy()
    ests, walls, y = [], [], None
    for _ in range(steps):
        est, wall, y = cpu_chunked_step(cfg_name, params, x_seq)
        ests.append(est)
        walls.append(wall)
    est = statistics.median(ests)
    P1, P2 = C5_PREFIXES
    base = {"value": B * S / est, "unit": "tokens/s", "cores": _host_cores(), "kind": "port",
            "sample": f"ESTIMATE: NumPy fp32 restatement of the reference's chunked forward (oracle.chunk_rows_forward) "
                      f"on one sequence -- K/V of a {P2}-row prefix and {C5_CHUNK}-row query chunks ending at {P1} and "
                      f"{P2} ({statistics.median(walls):.2f} s per sample), chunk cost linear in its prefix, "
                      f"extrapolated to B={B} x S={S}: {est / 60:.1f} min per forward"}
    return base, est, statistics.median(walls), y


def cpu_sample_batch(cfg_name):
    """Sequences in the CPU leg's bounded sample of the workload (the first ones of the timed input)."""
    B, S = CONFIGS[cfg_name][:2]
    return B if B * S <= 16384 else max(1, 16384 // S)


def cpu_forward_rate(cfg_name, budget_s=12.0, min_reps=1):
    """tokens/s of the NumPy restatement of the reference module on this host (all BLAS threads)."""
    import numpy as np
    import oracle
    cores = _host_cores()
    B, S, d, H, F, L = CONFIGS[cfg_name]
    Bs = cpu_sample_batch(cfg_name)
    params = oracle.params_from_state_dict(oracle.init_state_dict(L, d, F, 1234))
    x, _ = oracle.generate_random_case(Bs, S, d, 1234 + 100000)
    xn = x.numpy()
    cfg = oracle.OracleConfig(Bs, S, d, H, F, L, True)
    oracle.model_forward(params, cfg, xn[:1])  # warm BLAS
    times = []
    y_ref = None
    t_end = time.perf_counter() + budget_s
    while len(times) < min_reps or time.perf_counter() < t_end:
        t0 = time.perf_counter()
        y_ref = oracle.model_forward(params, cfg, xn)
        times.append(time.perf_counter() - t0)
        if len(times) >= 50:
            break
    med = statistics.median(times)
    return {"value": Bs * S / med, "unit": "tokens/s", "cores": int(cores), "kind": "port",
            "sample": f"{len(times)} forwards of B={Bs} x S={S} (NumPy fp32 restatement of the reference "
                      f"module, oracle/), median {med * 1e3:.1f} ms"}, med, Bs, y_ref


def run_reference(args, rank, world):
    if rank != 0:
        return 0
    B, S, d, H, F, L = CONFIGS[args.config]
    import numpy as np
    import oracle
    if args.config in STRONG and L != 1:
        print(json.dumps({"impl": "reference", "unavailable": "the CPU estimate restates one layer (chunk_rows_forward); "
                                                              f"{args.config} has {L}"}), flush=True)
        return 0
    if args.config in STRONG:
        # every step is one bounded sample (about a second or two of CPU work), extrapolated
        import oracle
        params = oracle.params_from_state_dict(oracle.init_state_dict(1, d, F, 1234))
        x_seq = oracle.generate_chunked_input(1, S, d, seed=1234, rows=C5_PREFIXES[-1])[0].numpy()
        for _ in range(args.warmup):
            cpu_chunked_step(args.config, params, x_seq)
        ests, walls = [], []
        for _ in range(args.steps):
            est, wall, _ = cpu_chunked_step(args.config, params, x_seq)
            ests.append(est)
            walls.append(wall)
        est = statistics.median(ests)
        tok = B * S / est
        P1, P2 = C5_PREFIXES
        base = {"value": tok, "unit": "tokens/s", "cores": _host_cores(), "kind": "port",
                "sample": f"ESTIMATE per step: NumPy fp32 restatement of the reference's chunked forward on one "
                          f"sequence (K/V of a {P2}-row prefix, {C5_CHUNK}-row query chunks ending at {P1} and {P2}), "
                          f"extrapolated to B={B} x S={S}; value = tokens/s of the median step's estimate "
                          f"({est / 60:.1f} min per forward); ms_per_step = wall time of one sample"}
        line = {"impl": "reference", "metric": METRIC, "value": tok, "unit": "tokens/s",
                "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
                "ms_per_step": statistics.median(walls) * 1e3, "estimated_ms_per_forward": est * 1e3,
                "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
                "data": "synthetic (seeded N(0,1) input, seeded default init)", "config": config_dict(args.config, 1),
                "cpu_baseline": base,
                "e2e": {"value": tok, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
        print(json.dumps(line), flush=True)
        return 0
    base, med, Bs, _ = cpu_forward_rate(args.config, budget_s=0.0, min_reps=1)
    params = oracle.params_from_state_dict(oracle.init_state_dict(L, d, F, 1234))
    x, _ = oracle.generate_random_case(Bs, S, d, 1234 + 100000)
    xn = x.numpy()
    cfg = oracle.OracleConfig(Bs, S, d, H, F, L, True)
    for _ in range(args.warmup):
        oracle.model_forward(params, cfg, xn)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        oracle.model_forward(params, cfg, xn)
    el = time.perf_counter() - t0
    tok = Bs * S * args.steps / el
    base.update(value=tok, sample=f"{args.steps} timed forwards of B={Bs} x S={S} per step "
                                   f"(NumPy fp32 restatement of the reference module)")
    line = {"impl": "reference", "metric": METRIC, "value": tok, "unit": "tokens/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": el * 1e3 / args.steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded N(0,1) input, seeded default init)",
            "config": config_dict(args.config, 1), "cpu_baseline": base,
            "e2e": {"value": tok, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------------- GPU arm
def main():
    args = parse()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        return run_reference(args, rank, world)

    import torch
    import torch.distributed as dist
    import torch_transformer_benchmark as T

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)

    if args.tp > 1:
        return run_tp(args, rank, world, dev)
    _, S, d, H, F, L = CONFIGS[args.config]
    B = rank_batch(args.config, rank, world)
    cfg = T.TransformerConfig(B, S, d, H, F, L, True)
    torch.manual_seed(1234)
    model = T.UserOptimizedTransformer(cfg).to(dev).eval()
    if B * S * d * 4 <= (1 << 30):
        gen = torch.Generator(device="cpu").manual_seed(1234 + 100000 + 7919 * rank)
        x_host = torch.randn(B, S, d, generator=gen).pin_memory()
        x = x_host.to(dev)
    else:  # multi-GB inputs: draw on the device, keep a pinned host copy for the end-to-end leg
        gen = torch.Generator(device=dev).manual_seed(1234 + 100000 + 7919 * rank)
        x = torch.randn(B, S, d, generator=gen, device=dev)
        x_host = torch.empty(B, S, d).pin_memory()
        x_host.copy_(x)
    y_host = torch.empty(B, S, d).pin_memory()
    mask = torch.ones(B, S, dtype=torch.bool, device=dev)
    flush = torch.empty((256 << 20) if flushes(args.config) else 16, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream()
    tokens_rank = B * S

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(v):
        if world == 1:
            return v
        t = torch.tensor([v], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    clk = ClockSampler(torch.cuda.current_device() if "CUDA_VISIBLE_DEVICES" not in os.environ else
                       int(os.environ["CUDA_VISIBLE_DEVICES"].split(",")[local]))
    clk.start()
    with torch.inference_mode():
        # keep each warm-up output alive across the next call, as the timed loop does: the
        # output then alternates between two blocks and both CUDA graphs (one per output
        # address) are captured here, not inside the timed region
        y_w = None
        for _ in range(max(args.warmup, 3)):
            y_w = model(x, mask)
        del y_w
        torch.cuda.synchronize()
        # ---- device-resident timed region
        starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
        ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
        barrier()
        torch.cuda.synchronize()
        # keep the GPU busy while the host enqueues every timed step, so no
        # host-side enqueue latency (Python call overhead) falls between an
        # event pair: the events then bracket device work only
        torch.cuda._sleep(QUEUE_PREFILL_CYCLES)
        y_last = None
        for i in range(args.steps):
            flush.zero_()
            starts[i].record(stream)
            y_last = model(x, mask)
            ends[i].record(stream)
        torch.cuda.synchronize()
        barrier()
        ms_rank = sum(a.elapsed_time(b) for a, b in zip(starts, ends))
        ms_total = max_over_ranks(ms_rank)
        strong = args.config in STRONG
        # the device path's output of the timed input, kept to check the end-to-end leg's
        # downloads against (all of it, or for the multi-GB configuration a set of rows of
        # every sequence)
        pos = torch.tensor(sorted({0, 1, S // 3, S // 2, S - 2, S - 1}), device=dev)
        y_dev_ref = y_last.index_select(1, pos).cpu() if strong else y_last.cpu()
        # ---- dominant-kernel roofline (rank 0; one sequence of the multi-GB configuration)
        roof = None
        if rank == 0:
            xp = x[:1].contiguous() if strong else x
            roof = roofline_pass(model, xp, mask, flush if flushes(args.config) else None, cfg,
                                 steps=3 if strong else max(20, min(args.steps, 200)), cfg_name=args.config,
                                 clock_mhz=clk.median_mhz())
            del xp
        # GPU outputs compared with the oracle in the CPU leg (rank 0, one GPU)
        y_check = None
        cpu_leg = rank == 0 and world == 1 and not args.no_cpu_baseline and not (strong and L != 1)
        if cpu_leg:
            if strong:  # one query chunk of sequence 0, from the timed forward's output
                y_check = y_last[0, C5_PREFIXES[-1] - C5_CHUNK:C5_PREFIXES[-1]].float().cpu()
            else:
                y_check = y_last[:cpu_sample_batch(args.config)].float().cpu()
        del y_last
        e2e_serial_ms = None
        if strong:
            del x  # make room for the two pipeline slots
            torch.cuda.empty_cache()
        else:
            # ---- end to end through the public API, serial: pinned H2D of x, forward, D2H of y per step
            e_st = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
            e_en = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
            xd = torch.empty_like(x)
            y_w = None
            for _ in range(3):  # capture this loop's graphs (new input address) before timing it
                xd.copy_(x_host, non_blocking=True)
                y_w = model(xd, mask)
                y_host.copy_(y_w, non_blocking=True)
            del y_w
            barrier()
            torch.cuda.synchronize()
            for i in range(args.steps):
                flush.zero_()
                e_st[i].record(stream)
                xd.copy_(x_host, non_blocking=True)
                y = model(xd, mask)
                y_host.copy_(y, non_blocking=True)
                e_en[i].record(stream)
            torch.cuda.synchronize()
            barrier()
            e2e_serial_ms = max_over_ranks(sum(a.elapsed_time(b) for a, b in zip(e_st, e_en)))
            del xd
        # ---- end to end, pipelined (UserOptimizedTransformer.forward_host): every step still
        # uploads its x and downloads its y, but step i's download, step i+1's forward and
        # step i+2's upload overlap; L2 flushed before every forward
        y_hosts = [y_host, torch.empty(B, S, d).pin_memory()]
        for i in range(2 if strong else 4):
            model.forward_host(x_host, out=y_hosts[i % 2], wait=False, flush=flush)
        model.synchronize_host()
        t0 = torch.cuda.Event(enable_timing=True)
        t1 = torch.cuda.Event(enable_timing=True)
        barrier()
        torch.cuda.synchronize()
        t0.record(stream)
        model.host_pipe_wait(t0, (B, S, d))  # the first upload starts inside the timed region
        for i in range(args.steps):
            model.forward_host(x_host, out=y_hosts[i % 2], wait=False, flush=flush)
        stream.wait_event(model.host_done_event((B, S, d)))
        t1.record(stream)
        torch.cuda.synchronize()
        barrier()
        e2e_ms = max_over_ranks(t0.elapsed_time(t1))
        y_e2e = y_hosts[(args.steps - 1) % 2]
        ok_e2e = bool(torch.equal(y_e2e.index_select(1, pos.cpu()) if strong else y_e2e, y_dev_ref))
    clocks = clk.stop()

    tokens_all = (CONFIGS[args.config][0] * S) if args.config in STRONG else world * tokens_rank
    value = tokens_all * args.steps / (ms_total / 1e3)
    e2e_value = tokens_all * args.steps / (e2e_ms / 1e3)
    launches_per_step = kernels_per_forward(model, B, S)

    cpu = None
    accuracy = None
    if cpu_leg:
        import oracle
        if strong:
            P2 = C5_PREFIXES[-1]
            cpu, _, _, y_ref = cpu_chunked_estimate(args.config, x_seq=x_host[0, :P2].numpy())
            acc = oracle.compare_outputs(y_ref, y_check.numpy())
            sample = (f"rows {P2 - C5_CHUNK}..{P2 - 1} of sequence 0 of the timed forward "
                      f"(exact chunked restatement, oracle.chunk_rows_forward)")
        else:
            cpu, _, Bs, y_ref = cpu_forward_rate(args.config)
            acc = oracle.compare_outputs(y_ref, y_check.numpy())
            sample = f"sequences 0..{Bs - 1} of the timed input"
        accuracy = {"max_abs": acc.max_abs_error, "max_rel": acc.max_relative_error, "failed": acc.failed_elements,
                    "total": acc.total_elements, "rule": "atol 0.002 OR rtol 0.02 (reference harness)",
                    "vs": "oracle/ (NumPy fp32 restatement of the reference module)", "sample": sample,
                    "gelu": oracle.gelu_as_max_error()}
    if rank == 0:
        line = {"metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": ms_total / args.steps, "higher_is_better": True,
                "scaling": "strong" if args.config in STRONG else "weak", "vs_baseline": None,
                "dtype": "f16 operands / f32 accumulate, f32 in-out",
                "data": "synthetic (seeded N(0,1) input, seeded default init)",
                "config": config_dict(args.config, world), "strategy": model.last_strategy,
                "e2e": {"value": e2e_value, "unit": "tokens/s", "ms_per_step": e2e_ms / args.steps,
                        "h2d_bytes_per_step": x_host.numel() * 4, "d2h_bytes_per_step": y_host.numel() * 4,
                        "api": "UserOptimizedTransformer.forward_host (pinned host in/out, upload/forward/"
                               "download overlapped across steps, L2 flushed before each forward)",
                        "outputs_match_device_path": bool(ok_e2e),
                        "outputs_checked": ("rows " + ",".join(str(int(v)) for v in pos.tolist()) +
                                            " of every sequence" if strong else "all") +
                                           " of the last download vs the device path's output (bitwise)",
                        "serial": None if e2e_serial_ms is None else {
                            "value": tokens_all * args.steps / (e2e_serial_ms / 1e3),
                            "ms_per_step": e2e_serial_ms / args.steps,
                            "api": "UserOptimizedTransformer.__call__ with H2D/D2H on one stream"}},
                "roofline": roof, "cpu_baseline": cpu, "accuracy": accuracy, "clocks": clocks,
                "gpu_launches": launches_per_step * args.steps}
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def run_tp(args, rank, world, dev):
    """Tensor-parallel (x batch-sharded) forward of a strong-scaling configuration.

    Ranks [g*tp, (g+1)*tp) form TP group g; the global batch is split over the
    world/tp groups.  Each rank runs parallel.TensorParallelTransformer (query
    chunks, K/V cache of its heads, two NCCL all-reduces per chunk on a side
    stream).  value = tokens of the whole job / max-over-ranks device time."""
    import torch
    import torch.distributed as dist
    import torch_transformer_benchmark as T
    par = T._pkg.parallel
    tp = args.tp
    if world % tp or args.config not in STRONG:
        raise SystemExit("--tp needs --gpus divisible by it and a strong-scaling config (C5)")
    dp = world // tp
    g, tp_rank = rank // tp, rank % tp
    groups = [dist.new_group(list(range(k * tp, (k + 1) * tp))) for k in range(dp)]
    Bg, S, d, H, F, L = CONFIGS[args.config]
    sl = par.batch_shard(Bg, g, dp)
    B = sl.stop - sl.start
    cfg = T.TransformerConfig(B, S, d, H, F, L, True)
    torch.manual_seed(1234)
    model = T.UserOptimizedTransformer(cfg).to(dev).eval()
    tpm = par.TensorParallelTransformer(model, tp_rank, tp, group=groups[g], chunk_rows=args.chunk_rows,
                                        profile_comm=True)
    # every rank of a TP group holds its group's input (replicated activations)
    gen = torch.Generator(device=dev).manual_seed(1234 + 100000 + 7919 * g)
    x = torch.randn(B, S, d, generator=gen, device=dev)
    y = torch.empty_like(x)
    stream = torch.cuda.current_stream()

    def max_over_ranks(v):
        t = torch.tensor([v], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    clk = ClockSampler(torch.cuda.current_device() if "CUDA_VISIBLE_DEVICES" not in os.environ else
                       int(os.environ["CUDA_VISIBLE_DEVICES"].split(",")[int(os.environ.get("LOCAL_RANK", "0"))]))
    clk.start()
    comm_ms = []
    with torch.inference_mode():
        for _ in range(max(args.warmup, 3)):
            tpm(x, out=y)
        torch.cuda.synchronize()
        starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
        ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
        dist.barrier()
        torch.cuda.synchronize()
        torch.cuda._sleep(QUEUE_PREFILL_CYCLES)
        for i in range(args.steps):
            starts[i].record(stream)
            tpm(x, out=y)
            ends[i].record(stream)
            comm_ms.append(tpm.comm_ms() if i == args.steps - 1 else None)
        torch.cuda.synchronize()
        dist.barrier()
        step_ms = [a.elapsed_time(b) for a, b in zip(starts, ends)]
        ms_total = max_over_ranks(sum(step_ms))
        ar_ms = max_over_ranks(comm_ms[-1])
        last_ms = max_over_ranks(step_ms[-1])
        # accuracy of one query chunk of the group's first sequence (rank 0, CPU restatement)
        accuracy = None
        y_rows = None
        P2 = C5_PREFIXES[-1]
        if rank == 0 and not args.no_cpu_baseline:
            y_rows = y[0, P2 - C5_CHUNK:P2].float().cpu()
            x_seq = x[0, :P2].float().cpu().numpy()
    clocks = clk.stop()
    if rank == 0 and y_rows is not None:
        import oracle
        params = oracle.params_from_state_dict(model.state_dict())
        ref = oracle.chunk_rows_forward(params, H, x_seq, P2 - C5_CHUNK, P2)
        acc = oracle.compare_outputs(ref, y_rows.numpy())
        accuracy = {"max_abs": acc.max_abs_error, "max_rel": acc.max_relative_error, "failed": acc.failed_elements,
                    "total": acc.total_elements, "rule": "atol 0.002 OR rtol 0.02 (reference harness)",
                    "sample": f"rows {P2 - C5_CHUNK}..{P2 - 1} of the first sequence of TP group 0 "
                              f"(exact chunked restatement, oracle.chunk_rows_forward)"}
    if rank == 0:
        chunks = len(par.tp_chunks(B, S, args.chunk_rows))
        value = Bg * S * args.steps / (ms_total / 1e3)
        line = {"metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": ms_total / args.steps, "higher_is_better": True,
                "scaling": "strong", "vs_baseline": None, "dtype": "f16 operands / f32 accumulate, f32 in-out",
                "data": "synthetic (seeded N(0,1) input, seeded default init)",
                "config": dict(config_dict(args.config, world),
                               parallelism=f"tp{tp} x dp{dp} (heads / FFN columns over {tp} ranks, NCCL all-reduce "
                                           f"after out_proj and ffn_out per {args.chunk_rows}-row query chunk; "
                                           f"batch over {dp} groups)"),
                "strategy": "tensor-parallel chunked",
                "tp": {"size": tp, "dp": dp, "chunk_rows": args.chunk_rows, "chunks_per_rank": chunks,
                       "allreduce_bytes_per_step_per_rank": 2 * B * S * d * 4 * L,
                       "allreduce_stream_ms_last_step": ar_ms, "step_ms_last_step": last_ms,
                       "allreduce_busy_share": ar_ms / last_ms if last_ms else None,
                       "note": "all-reduce time = CUDA events around each NCCL call on the side stream (max over "
                               "ranks); it overlaps the compute stream, so the share is busy time, not exposed time"},
                "e2e": None, "roofline": None, "cpu_baseline": None, "accuracy": accuracy, "clocks": clocks,
                "gpu_launches": (9 * chunks * L) * args.steps}
        print(json.dumps(line), flush=True)
    dist.barrier()
    del groups
    dist.destroy_process_group()
    return 0


def kernels_per_forward(model, B, S, masked=True):
    """Launches of the library's kernels per forward (the host code of
    b200_block_forward / b200_block_forward_chunked, counted per layer)."""
    cfg = model.config
    strat, nl, d = model.last_strategy, cfg.num_layers, cfg.d_model
    mask = 2 if masked else 0  # b200_mask_prepare + b200_zero_masked_rows
    if strat == "fused_small":
        return 1  # the whole model in one kernel; it reads the mask itself
    fuse = d == 128  # residual GEMM + following LayerNorm in one kernel
    # LN1, QKV, attention, out_proj (+LN2), ffn_in, ffn_out (+final LN)
    mid = 6 if fuse else 7          # a layer without the final norm
    last = 6 if fuse else 8         # the last layer (final norm)
    per_model = mid * (nl - 1) + last
    if strat == "chunked":          # per chunk: Q and K|V are two GEMMs
        rows = model._chunk_plan[(B, S, torch_device_index(model))]
        chunks = B * (-(-S // rows))
        per_model = chunks * ((mid + 1) * (nl - 1) + last + 1)
    return per_model + mask


def torch_device_index(model):
    import torch
    return torch.cuda.current_device()


def measured_traffic(cfg_name, kernel):
    """DRAM bytes per launch of `kernel` at `cfg_name` from the committed ncu summaries
    (profiles/traffic.json), or (None, None) when no capture covers it."""
    try:
        with open(os.path.join(REPO, "profiles", "traffic.json")) as f:
            t = json.load(f).get(cfg_name)
    except (OSError, ValueError):
        return None, None
    if not t or t.get("kernel") != kernel:
        return None, None
    return int(t["bytes"]), "profiles/" + t["source"]


def roofline_pass(model, x, mask, flush, cfg, steps, cfg_name=None, clock_mhz=None):
    """Dominant-kernel roofline: per-stage CUDA-event timing of an eager pass on the same inputs."""
    import torch
    peaks = load_peaks()
    B, S, d = x.shape
    H, F = cfg.num_heads, cfg.ffn_dim
    timing = model.profile_stages(x, steps=steps, flush=flush)
    if not timing:
        return None
    work = stage_work(B, S, d, H, F)
    name = max(timing, key=timing.get)
    if name == "fused_small":
        fl, by = block_work(B, S, d, H, F)
        fl *= cfg.num_layers
    else:
        fl, by = work[name]
    ms = timing[name]
    t_tensor = fl / (peaks["bf16_tflops"] * 1e12)
    t_hbm = by / (peaks["hbm_gbs"] * 1e9)
    if t_tensor >= t_hbm:
        ach = fl / (ms * 1e-3) / 1e12
        out = {"bound": "tensor", "achieved": ach, "peak": peaks["bf16_tflops"], "unit": "TFLOP/s"}
    else:
        ach = by / (ms * 1e-3) / 1e9
        out = {"bound": "hbm", "achieved": ach, "peak": peaks["hbm_gbs"], "unit": "GB/s"}
    traffic, traffic_src = measured_traffic(cfg_name, name)
    if name == "attn":
        # the exponentials: one exp2 per causal score (B*H*S(S+1)/2) against the SFU's 16 per
        # clock per SM -- for head_dim 64 the unit that binds before the tensor pipe
        import torch
        exps = B * H * S * (S + 1) / 2
        sms = torch.cuda.get_device_properties(x.device).multi_processor_count
        clk_hz = clock_mhz * 1e6 if clock_mhz else 1.965e9
        peak = 16 * sms * clk_hz
        out["sfu"] = {"exp2_per_s": exps / (ms * 1e-3), "peak_exp2_per_s": peak,
                      "frac": exps / (ms * 1e-3) / peak, "clock_mhz": clk_hz / 1e6,
                      "note": "16 exp2 per clock per SM at the median SM clock sampled during the timed region"}
    out.update(frac=out["achieved"] / out["peak"], traffic=traffic, traffic_src=traffic_src, kernel=name,
               ms_per_launch=ms,
               peak_src=f"{peaks['src']} (MEASURED_PEAKS.json burst)" if peaks["src"] == "measured" else "fallback",
               stage_ms=timing, algorithmic={"flops": fl, "bytes": by})
    return out


if __name__ == "__main__":
    raise SystemExit(main())
