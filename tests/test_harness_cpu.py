"""Host-side logic that needs no GPU: the compare rule, seeded inputs, attention identities."""

import numpy as np
import pytest
import torch

import oracle


def test_compare_outputs_or_rule():
    ref = torch.tensor([1.0, 100.0, 0.0, 1.0])
    opt = torch.tensor([1.0019, 101.9, 0.0021, float("nan")])
    r = oracle.compare_outputs(ref, opt, rtol=0.02, atol=0.002)
    # 1: abs ok; 2: rel ok (1.9 <= 2.0); 3: abs 0.0021 > atol and rel fails; 4: nan fails
    assert r.failed_elements == 2
    assert not r.passed
    assert oracle.compare_outputs(ref[:2], opt[:2]).passed


def test_compare_outputs_shape_mismatch():
    with pytest.raises(AssertionError):
        oracle.compare_outputs(torch.zeros(2, 3), torch.zeros(3, 2))


def test_chunked_input_slices_regenerate():
    full = oracle.generate_chunked_input(3, 50, 8, seed=7, chunk=16)
    part = oracle.generate_chunked_input(3, 50, 8, seed=7, chunk=16, batches=[2], rows=21)
    assert torch.equal(full[2, :21], part[0])
    assert not torch.equal(full[0], full[1])


@pytest.mark.parametrize("chunk", [32, 48, 128])
def test_prefix_causal_chunks_equal_full_attention(chunk):
    """The identity the chunked path rests on (the reference's check at
    experiments/g7_0_chunked_oversize.py:149-179): attention of query chunk
    [c0:c1) over keys [0:c1) with prefix offset c0 equals rows [c0:c1) of full
    causal attention."""
    rng = np.random.default_rng(11)
    B, H, S, hd = 2, 3, 128, 16
    q, k, v = (rng.standard_normal((B, H, S, hd)).astype(np.float32) for _ in range(3))
    full = oracle.causal_attention(q, k, v)
    parts = [oracle.causal_attention(q[:, :, c0:c0 + chunk], k[:, :, :c0 + chunk], v[:, :, :c0 + chunk],
                                     q_offset=c0) for c0 in range(0, S, chunk)]
    got = np.concatenate(parts, axis=2)
    assert np.abs(got - full).max() < 1e-5


def test_batch_independence_of_oracle():
    """A forward is batch-independent: a batch slice equals the slice of the batch."""
    sd = oracle.params_from_state_dict(oracle.init_state_dict(1, 64, 256, 3))
    x, _ = oracle.generate_random_case(4, 40, 64, seed=5)
    cfg = oracle.OracleConfig(4, 40, 64, 2, 256, 1, True)
    y = oracle.model_forward(sd, cfg, x.numpy())
    y2 = oracle.model_forward(sd, oracle.OracleConfig(2, 40, 64, 2, 256, 1, True), x[1:3].numpy())
    assert np.abs(y[1:3] - y2).max() < 1e-6


@pytest.mark.parametrize("L", [1, 2])
def test_prefix_padding_only_zeroes_padded_rows(L):
    """The padding design argument, on the oracle: with causal attention and a
    prefix-valid mask, the reference's masked forward equals the unmasked forward
    on valid rows and is 0 on padded rows (so the kernels only mask the output)."""
    B, S, d, H, F = 4, 48, 64, 2, 256
    sd = oracle.params_from_state_dict(oracle.init_state_dict(L, d, F, 8))
    x, mask = oracle.generate_random_case(B, S, d, 9, padding_ratio=0.6)
    cfg = oracle.OracleConfig(B, S, d, H, F, L, True)
    masked = oracle.model_forward(sd, cfg, x.numpy(), mask.numpy())
    plain = oracle.model_forward(sd, cfg, x.numpy())
    m = mask.numpy()
    assert np.abs(masked[m] - plain[m]).max() < 1e-5
    assert np.all(masked[~m] == 0)
