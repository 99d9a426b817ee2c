"""The shape arbiter and its memory gate, on the CPU (no device memory is touched).

The reference routes a causal shape to its sequence-chunked forward only when
its byte model says the compiled path would not fit (``_would_oom_causal``,
TTB:1036-1116), and checks that the gate never fires on a scored row of its
matrix (experiments/g7_0_chunked_oversize.py:19-22, check 2).  Here the gate is
``_would_oom`` (the chain's workspace against a fraction of free HBM) and these
tests pin, with the free memory of a B200 stood in for the device query:

* every BASELINE configuration and every row of the reference's official matrix
  takes the single kernel or the chain -- never the chunked path -- on one B200;
* the chunked path is chosen only when the budget is lowered, with the largest
  query chunk (a multiple of 128, at most 16384) whose workspace fits.
The GPU side (an auto-routed chunked forward bit-identical to a forced one) is
in tests/test_gpu_parity.py.
"""

import pytest
import torch

B200_FREE = 178 * (1 << 30)  # free HBM of a B200 with nothing else resident (183,359 MiB total)

# BASELINE.json configs (L=1, ffn=4d) and the reference's official matrix rows (L=4, ffn=d;
# row 14: L=2, ffn=1024), with the strategy each must take on one B200
SHAPES = [
    ("C1", 4, 128, 128, 4, 512, 1, "fused_small"),
    ("C2", 64, 128, 128, 4, 512, 1, "fused_small"),
    ("C3", 10000, 128, 128, 4, 512, 1, "fused_small"),
    ("C4a", 64, 1024, 128, 4, 512, 1, "chain"),
    ("C4b", 64, 128, 1024, 4, 4096, 1, "chain"),
    ("C5", 32, 100000, 1024, 16, 4096, 1, "chain"),
    ("row1", 64, 128, 128, 4, 128, 4, "fused_small"),
    ("row2", 1, 128, 128, 4, 128, 4, "fused_small"),
    ("row3", 4, 128, 128, 4, 128, 4, "fused_small"),
    ("row4", 16, 128, 128, 4, 128, 4, "fused_small"),
    ("row5", 128, 128, 128, 4, 128, 4, "fused_small"),
    ("row6", 10000, 128, 128, 4, 128, 4, "fused_small"),
    ("row7", 64, 128, 32, 4, 32, 4, "fused_small"),
    ("row8", 64, 128, 1024, 4, 1024, 4, "chain"),
    ("row9", 64, 128, 128, 1, 128, 4, "fused_small"),
    ("row10", 64, 128, 128, 2, 128, 4, "fused_small"),
    ("row11", 64, 128, 128, 16, 128, 4, "chain"),
    ("row12", 64, 32, 128, 4, 128, 4, "fused_small"),
    ("row13", 64, 1024, 128, 4, 128, 4, "chain"),
    ("row14", 32, 100000, 1024, 16, 1024, 2, "chain"),
]


def _model(tt, B, S, d, H, F, L, budget):
    cfg = tt.TransformerConfig(B, S, d, H, F, L, True)
    m = tt.UserOptimizedTransformer(cfg)
    m._memory_budget = lambda device: int(budget)  # stands in for 0.6 x torch.cuda.mem_get_info
    return m


@pytest.mark.parametrize("name,B,S,d,H,F,L,want", SHAPES, ids=[s[0] for s in SHAPES])
def test_gate_never_fires_on_a_scored_shape(tt, name, B, S, d, H, F, L, want):
    m = _model(tt, B, S, d, H, F, L, 0.6 * B200_FREE)
    dev = torch.device("cuda", 0)
    assert not m._would_oom(B, S, dev)
    assert m._strategy(B, S, dev) == want


def test_gate_routes_to_chunks_when_the_budget_is_lowered(tt, pkg):
    rt = pkg.runtime
    B, S, d, H, F = 32, 100000, 1024, 16, 4096
    dev = torch.device("cuda", 0)
    need = rt.block_workspace_bytes(B * S, d, F)
    m = _model(tt, B, S, d, H, F, 1, need - 1)  # one byte short of the chain's workspace
    assert m._would_oom(B, S, dev)
    assert m._strategy(B, S, dev) == "chunked"
    rows = m._chunk_plan[(B, S, 0)]
    assert rows == 16384  # the K/V cache plus a 16384-row chunk fit easily
    assert rt.chunked_workspace_bytes(B * S, rows, d, F) <= need - 1
    # a tighter budget: the largest multiple of 128 whose workspace fits
    kv = rt.chunked_workspace_bytes(B * S, 128, d, F)
    budget = kv + (rt.chunked_workspace_bytes(B * S, 1024, d, F) - kv) // 2
    m2 = _model(tt, B, S, d, H, F, 1, budget)
    assert m2._strategy(B, S, dev) == "chunked"
    r2 = m2._chunk_plan[(B, S, 0)]
    assert r2 % 128 == 0 and 128 <= r2 < 1024
    assert rt.chunked_workspace_bytes(B * S, r2, d, F) <= budget < rt.chunked_workspace_bytes(B * S, r2 + 128, d, F)


def test_gate_decision_is_cached_per_shape(tt):
    m = _model(tt, 64, 1024, 128, 4, 512, 1, 0.6 * B200_FREE)
    dev = torch.device("cuda", 0)
    assert m._strategy(64, 1024, dev) == "chain"
    m._memory_budget = lambda device: 0  # the decision is made once per shape, eagerly
    assert m._strategy(64, 1024, dev) == "chain"
    assert m._strategy(32, 1024, dev) == "chunked"  # a new shape sees the new budget


def test_non_causal_never_chunks(tt):
    cfg = tt.TransformerConfig(2, 4096, 256, 4, 1024, 1, False)
    m = tt.UserOptimizedTransformer(cfg)
    m._memory_budget = lambda device: 0
    assert m._strategy(2, 4096, torch.device("cuda", 0)) == "chain"


@pytest.mark.parametrize("shape,groups", [((32, 100000, 1024), 4), ((16, 100000, 1024), 4), ((8, 100000, 1024), 2),
                                          ((4, 100000, 1024), 1), ((64, 128, 128), 1), ((10000, 128, 128), 1),
                                          ((3, 300000, 1024), 1), ((12, 100000, 1024), 3)])
def test_forward_host_batch_groups(tt, shape, groups):
    """``forward_host`` splits inputs of several GB into batch groups of about 2 GiB of x
    (the group count a divisor of B): whole, equal, contiguous, in-order ranges covering the
    batch once; small inputs stay one group."""
    g = tt.UserOptimizedTransformer._host_groups(shape)
    assert len(g) == groups
    B = shape[0]
    assert g[0][0] == 0 and g[-1][1] == B
    assert all(a[1] == b[0] for a, b in zip(g, g[1:]))
    assert len({b1 - b0 for b0, b1 in g}) == 1
