"""Key-padding masks on a B200: the mask is read on the device on every call.

The reference masks padded keys in attention and zeroes padded rows after each
block and after the final norm (TTB:125-128, 140-141, 163-164, 190-191); its
``_mask_is_all_ones`` caches one property of a mask by ``data_ptr``
(TTB:1011-1025).  Here nothing about a mask's contents is cached on the host:
these tests change the mask behind the same address -- an in-place edit, and a
new mask allocated where a freed one was -- and require the forward to follow,
on the single-kernel path, the kernel chain and the chunked chain, including the
CUDA-graph replay path.  Masks of any shape are exact: the single kernel tests
each key's flag; the chain's attention applies packed key bits to sequences
whose mask is not prefix-valid (a valid token after a padded one).
"""

import numpy as np
import pytest
import torch

import oracle

pytestmark = pytest.mark.gpu

ATOL, RTOL = 0.002, 0.02
DEV = "cuda"


@pytest.fixture(scope="module", autouse=True)
def _clean_device_errors(pkg):
    rt = pkg.runtime
    rt.lib()
    assert rt.device_error(clear=True) == 0
    yield
    assert rt.device_error(clear=True) == 0


def _model(tt, B, S, d, H, F, L, causal=True, strategy=None, chunk_rows=None, seed=77):
    cfg = tt.TransformerConfig(B, S, d, H, F, L, causal)
    torch.manual_seed(seed)
    m = tt.UserOptimizedTransformer(cfg).to(DEV).eval()
    m.force_strategy = strategy
    m.chunk_rows = chunk_rows
    return m


def _oracle(model, x, mask):
    c = model.config
    return oracle.model_forward(oracle.params_from_state_dict(model.state_dict()),
                                oracle.OracleConfig(c.batch_size, c.seq_len, c.d_model, c.num_heads, c.ffn_dim,
                                                    c.num_layers, c.causal),
                                x.numpy(), None if mask is None else mask.cpu().numpy())


def _check(model, x, y, mask):
    ref = _oracle(model, x, mask)
    res = oracle.compare_outputs(ref, y, rtol=RTOL, atol=ATOL)
    assert res.passed, res
    if mask is not None:
        assert torch.all(y[~mask.cpu()] == 0)


def _prefix_mask(B, S, lens):
    return torch.arange(S)[None, :] < torch.tensor(lens)[:, None]


STRATEGIES = [
    # (id, B, S, d, H, F, L, strategy, chunk_rows)
    ("fused_small", 6, 128, 128, 4, 512, 2, None, None),
    ("chain", 4, 192, 256, 4, 1024, 1, "chain", None),
    ("chunked", 3, 384, 256, 4, 512, 1, "chunked", 128),
]


@pytest.mark.parametrize("sid,B,S,d,H,F,L,strategy,chunk_rows", STRATEGIES, ids=[s[0] for s in STRATEGIES])
def test_mask_edited_in_place_and_at_a_reused_address(tt, sid, B, S, d, H, F, L, strategy, chunk_rows):
    """All-ones mask (enough calls to reach CUDA-graph replay), then the SAME mask tensor
    edited in place into a padded prefix mask, then a different padded mask allocated at
    the freed mask's address: every forward matches the oracle for the mask it was given,
    with padded rows exactly 0."""
    model = _model(tt, B, S, d, H, F, L, strategy=strategy, chunk_rows=chunk_rows)
    x, _ = oracle.generate_random_case(B, S, d, 4242)
    xd = x.to(DEV)
    mask = torch.ones(B, S, dtype=torch.bool, device=DEV)
    with torch.inference_mode():
        for _ in range(3):  # eager first call, graph capture, graph replay
            y = model(xd, mask).cpu()
        assert model.last_strategy == sid
        _check(model, x, y, None)
        ptr = mask.data_ptr()
        # in place: the same tensor, the same address, new contents
        lens1 = [S - 1 - 37 * i for i in range(B)]
        mask[:] = _prefix_mask(B, S, lens1).to(DEV)
        assert mask.data_ptr() == ptr
        y1 = model(xd, mask).cpu()
        _check(model, x, y1, _prefix_mask(B, S, lens1))
        y1b = model(xd, mask).cpu()  # and again, through the replay path
        assert torch.equal(y1, y1b)
        # a new mask where the old one was
        del mask
        lens2 = [max(1, S // 2 - 11 * i) for i in range(B)]
        m2 = torch.empty(B, S, dtype=torch.bool, device=DEV)
        m2.copy_(_prefix_mask(B, S, lens2))
        assert m2.data_ptr() == ptr, "the caching allocator did not hand the freed block back"
        y2 = model(xd, m2).cpu()
        _check(model, x, y2, _prefix_mask(B, S, lens2))
        # back to all ones, in place
        m2.fill_(True)
        y3 = model(xd, m2).cpu()
        assert torch.equal(y3, y)


def _holey_mask(B, S):
    g = torch.Generator().manual_seed(5)
    m = torch.rand(B, S, generator=g) > 0.3
    m[0, 0] = False       # a causal row that sees no valid key at all
    m[1, :] = True
    m[1, S // 3] = False  # one hole
    return m


@pytest.mark.parametrize("causal", [True, False], ids=["causal", "noncausal"])
@pytest.mark.parametrize("d,H,F", [(128, 4, 512), (128, 2, 256), (32, 4, 32)], ids=["d128h4", "d128h2", "d32"])
def test_masks_with_holes_on_the_single_kernel(tt, causal, d, H, F):
    """The single-kernel path masks each key by its own flag, so any mask works -- including
    a row whose visible keys are all padded (its context is zero, and two layers keep the
    valid rows finite)."""
    B, S, L = 4, 128, 2
    model = _model(tt, B, S, d, H, F, L, causal=causal)
    x, _ = oracle.generate_random_case(B, S, d, 99)
    m = _holey_mask(B, S)
    with torch.inference_mode():
        y = model(x.to(DEV), m.to(DEV)).cpu()
    assert model.last_strategy == "fused_small"
    assert torch.isfinite(y).all()
    _check(model, x, y, m)


HOLES = [
    # (id, B, S, d, H, F, L, causal, strategy, chunk_rows)
    ("chain", 3, 256, 256, 4, 1024, 1, True, "chain", None),
    ("chunked", 3, 256, 256, 4, 1024, 1, True, "chunked", 128),
    ("chain_unaligned", 3, 250, 256, 4, 1024, 1, True, "chain", None),  # masks off the 16-byte grid
    ("chain_noncausal", 3, 256, 256, 4, 1024, 1, False, "chain", None),
    ("chain_2layers", 3, 200, 256, 4, 512, 2, True, "chain", None),
    ("chain_hd8", 2, 160, 128, 16, 512, 1, True, None, None),            # head_dim 8: CUDA-core attention
    ("chain_hd64_long", 2, 1100, 256, 4, 512, 1, True, "chain", None),  # 9 query tiles per sequence
]


@pytest.mark.parametrize("sid,B,S,d,H,F,L,causal,strategy,chunk_rows", HOLES, ids=[h[0] for h in HOLES])
def test_masks_with_holes_on_the_chain(tt, pkg, sid, B, S, d, H, F, L, causal, strategy, chunk_rows):
    """The chain's attention applies packed key bits to sequences whose mask is not
    prefix-valid, so any mask matches the reference -- including a causal row whose
    visible keys are all padded (key 0 padded), which gets a zero context and keeps later
    layers finite; padded rows are 0 and no device error is recorded."""
    rt = pkg.runtime
    model = _model(tt, B, S, d, H, F, L, causal=causal, strategy=strategy, chunk_rows=chunk_rows)
    x, _ = oracle.generate_random_case(B, S, d, 7)
    m = _prefix_mask(B, S, [S] + [S - 40 * i for i in range(1, B)])
    m[0, 0] = False            # sequence 0: padded first token (row 0 sees no valid key under causal attention)
    m[0, S // 3:S // 3 + 5] = False
    m[1, 50] = False           # sequence 1: one hole inside its valid prefix
    assert rt.device_error(clear=True) == 0
    with torch.inference_mode():
        y = model(x.to(DEV), m.to(DEV)).cpu()
    assert model.last_strategy in ("chain", "chunked")
    assert rt.device_error(clear=True) == 0
    assert torch.isfinite(y).all()
    _check(model, x, y, m)


@pytest.mark.parametrize("causal", [True, False], ids=["causal", "noncausal"])
def test_masks_with_holes_on_the_two_tile_kernel_in_subprocess(causal):
    """The same masks through the two-query-tile attention kernel (k_flash_causal2), which the
    library picks by itself only for head_dim-64 grids of many waves; B200_ATTN_TILES=2 (read
    once per process, hence the child) forces it here at a size the oracle checks quickly."""
    import os
    import subprocess
    import sys
    code = r'''
import sys, torch
import oracle
import torch_transformer_benchmark as tt
causal = sys.argv[1] == "1"
B, S, d, H, F, L = 2, 1100, 256, 4, 512, 1
cfg = tt.TransformerConfig(B, S, d, H, F, L, causal)
torch.manual_seed(77)
model = tt.UserOptimizedTransformer(cfg).to("cuda").eval()
model.force_strategy = "chain"
x, _ = oracle.generate_random_case(B, S, d, 7)
m = torch.ones(B, S, dtype=torch.bool)
m[1, S - 40:] = False
m[0, 0] = False
m[0, S // 3:S // 3 + 5] = False
m[1, 50] = False
with torch.inference_mode():
    y = model(x.to("cuda"), m.to("cuda")).cpu()
rt = tt._pkg.runtime
assert rt.device_error(clear=True) == 0
ref = oracle.model_forward(oracle.params_from_state_dict(model.state_dict()),
                           oracle.OracleConfig(B, S, d, H, F, L, causal), x.numpy(), m.numpy())
res = oracle.compare_outputs(ref, y, rtol=0.02, atol=0.002)
assert res.passed, res
assert torch.all(y[~m] == 0) and torch.isfinite(y).all()
print("OK", res.max_abs_error)
'''
    env = dict(os.environ, B200_ATTN_TILES="2")
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    r = subprocess.run([sys.executable, "-c", code, "1" if causal else "0"], cwd=root, env=env,
                       capture_output=True, text=True, timeout=600)
    assert r.returncode == 0 and "OK" in r.stdout, r.stdout + r.stderr


def test_mask_is_never_cached_on_the_host(tt):
    """The module keeps no per-mask state: no attribute holds a mask verdict, and the
    reference's helper name answers from the tensor itself."""
    model = _model(tt, 2, 64, 128, 4, 512, 1)
    m = torch.ones(2, 64, dtype=torch.bool, device=DEV)
    assert model._mask_is_all_ones(m)
    m[0, -1] = False
    assert not model._mask_is_all_ones(m)
    assert not hasattr(model, "_mask_cache")
