"""The oracle against the reference's own outputs (golden vectors, CPU only)."""

import json

import numpy as np
import pytest
import torch

import oracle
from conftest import golden_cases, load_golden

CASES = golden_cases()


@pytest.mark.parametrize("case", CASES, ids=[c["name"] for c in CASES])
def test_input_regenerates_from_seed(case):
    g = load_golden(case["name"])
    x, mask = oracle.generate_random_case(case["B"], case["S"], case["d"], case["x_seed"], case["padding_ratio"])
    assert float(x.double().sum()) == float(g["x_sum"])
    assert float(x.double().abs().sum()) == float(g["x_abs_sum"])
    np.testing.assert_array_equal(x.reshape(-1)[:64].numpy(), g["x_head"])
    np.testing.assert_array_equal(mask.numpy(), g["mask"])


@pytest.mark.parametrize("case", CASES, ids=[c["name"] for c in CASES])
def test_weight_init_matches_reference(case):
    g = load_golden(case["name"])
    fp = oracle.fingerprint(oracle.init_state_dict(case["L"], case["d"], case["ffn"], case["seed"]))
    ref = json.loads(str(g["fingerprint"]))
    assert set(fp) == set(ref)
    for k in ref:
        assert fp[k][0] == ref[k][0] and fp[k][1] == ref[k][1], k


@pytest.mark.parametrize("case", CASES, ids=[c["name"] for c in CASES])
@pytest.mark.parametrize("dtype", [np.float32, np.float64])
def test_oracle_matches_reference_output(case, dtype):
    g = load_golden(case["name"])
    x, mask = oracle.generate_random_case(case["B"], case["S"], case["d"], case["x_seed"], case["padding_ratio"])
    sd = oracle.init_state_dict(case["L"], case["d"], case["ffn"], case["seed"])
    cfg = oracle.OracleConfig(case["B"], case["S"], case["d"], case["H"], case["ffn"], case["L"],
                              case.get("causal", True))
    m = mask.numpy() if case["padding_ratio"] > 0 else None
    y = oracle.model_forward(oracle.params_from_state_dict(sd), cfg, x.numpy(), m, dtype=dtype)
    err = np.abs(y.astype(np.float64) - g["y"].astype(np.float64)).max()
    assert err < 1e-5, err
    res = oracle.compare_outputs(g["y"], y, rtol=0.0, atol=1e-5)
    assert res.passed


@pytest.mark.parametrize("name", ["c1", "ragged", "h16"])  # causal cases only
def test_sampled_rows_match_reference(name):
    case = next(c for c in CASES if c["name"] == name)
    g = load_golden(name)
    x, _ = oracle.generate_random_case(case["B"], case["S"], case["d"], case["x_seed"])
    sd = oracle.params_from_state_dict(oracle.init_state_dict(1, case["d"], case["ffn"], case["seed"]))
    rows = [0, 1, case["S"] // 2, case["S"] - 1]
    for b in range(case["B"]):
        ys = oracle.sampled_rows_forward(sd, case["H"], x[b].numpy(), rows, key_block=37)
        assert np.abs(ys - g["y"][b, rows]).max() < 1e-5
