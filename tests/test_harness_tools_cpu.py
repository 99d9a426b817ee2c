"""Harness-integrity tooling (harness_tools.py): frozen-symbol verification,
the sentinel splice, the static validity gate and the bench-line check.

The reference guards its drop-in file with tools/verify_baseline.py,
tools/sync_entrypoint.py and tools/check_validity.py; these tests pin the same
behaviours on synthetic harnesses, and on the reference's own harness where it
is present (the build container only; the test skips elsewhere).
"""

import copy
import json
import os
import subprocess
import sys
import textwrap

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(REPO, "flipfloppers-gpu-kernel-optimizer_b200")
sys.path.insert(0, PKG)
import harness_tools as ht  # noqa: E402

# a checkout of the reference, named like tests/golden/make_golden.py does (REFERENCE_DIR)
REFERENCE_HARNESS = os.path.join(os.environ.get("REFERENCE_DIR", ""), "torch_transformer_benchmark.py")

# a miniature harness with every frozen symbol, a stub user class and the tolerance flags
CANON = textwrap.dedent('''
    import argparse


    class TransformerConfig:
        pass


    class BaselineSelfAttention:
        pass


    class BaselineTransformerBlock:
        pass


    class BaselineTransformer:
        pass


    class UserOptimizedTransformer(BaselineTransformer):
        """stub"""

        def forward(self, x, valid_token_mask=None):
            raise NotImplementedError


    def copy_model_weights(src, dst):
        dst.load_state_dict(src.state_dict(), strict=True)

    ''') + "".join(f"\n\ndef {n}():\n    return {i}\n" for i, n in enumerate(ht.FROZEN_SYMBOLS)
                   if n not in ("TransformerConfig", "BaselineSelfAttention", "BaselineTransformerBlock",
                                "BaselineTransformer", "copy_model_weights", "parse_args")) + textwrap.dedent('''


    def parse_args():
        ap = argparse.ArgumentParser()
        ap.add_argument("--atol", type=float, default=0.002)
        ap.add_argument("--rtol", type=float, default=0.02)
        return ap.parse_args([])
    ''')


def test_verify_passes_on_identical_and_formatting_changes():
    assert ht.verify_frozen(CANON, CANON) == []
    reformatted = CANON.replace("def percentile():", "# a comment\ndef percentile():")
    assert ht.verify_frozen(reformatted, CANON) == []


def test_verify_flags_changed_symbol_and_tolerance():
    changed = CANON.replace("return ap.parse_args([])", "return ap.parse_args(['--atol', '1'])")
    assert any("parse_args: differs" in p for p in ht.verify_frozen(changed, CANON))
    loose = CANON.replace("default=0.002", "default=0.01")
    probs = ht.verify_frozen(loose, loose)
    assert any("--atol default is 0.01" in p for p in probs)
    missing = CANON.replace("def compare_outputs():", "def compare_outputs_renamed():")
    assert any("compare_outputs: missing" in p for p in ht.verify_frozen(missing, CANON))


def test_splice_replaces_stub_and_is_idempotent():
    out = ht.splice(CANON, "/some/root")
    assert "raise NotImplementedError" not in out
    assert ht.BEGIN_MODEL in out and ht.END_MODEL in out and "'/some/root'" in out
    assert ht.splice(out, "/some/root") == out          # re-splicing a spliced file changes nothing
    assert ht.verify_frozen(out, CANON) == []           # the harness half is untouched
    assert "UserOptimizedTransformer" not in ht.top_level_defs(out)  # a binding now, not a class


def test_splice_replaces_sentinel_blocks():
    canon = CANON.replace('class UserOptimizedTransformer(BaselineTransformer):\n    """stub"""\n\n'
                          '    def forward(self, x, valid_token_mask=None):\n        raise NotImplementedError\n',
                          "# >>> BEGIN user helpers >>>\nHELPER = 1\n# <<< END user helpers <<<\n\n"
                          "# >>> BEGIN user model >>>\nclass UserOptimizedTransformer:\n    pass\n"
                          "# <<< END user model <<<\n")
    assert "BEGIN user helpers" in canon
    out = ht.splice(canon, "/r")
    assert "HELPER = 1" not in out and out.count(ht.BEGIN_MODEL) == 1
    assert ht.splice(out, "/r") == out
    with pytest.raises(ValueError):
        ht.splice(canon.replace("# <<< END user model <<<\n", ""), "/r")


def test_splice_cli_check(tmp_path):
    canon = tmp_path / "canon.py"
    canon.write_text(CANON)
    out = tmp_path / "ttb.py"
    tool = os.path.join(PKG, "harness_tools.py")
    r = subprocess.run([sys.executable, tool, "splice", str(canon), str(out), "--check"], capture_output=True, text=True)
    assert r.returncode == 1
    assert subprocess.run([sys.executable, tool, "splice", str(canon), str(out)]).returncode == 0
    r = subprocess.run([sys.executable, tool, "splice", str(canon), str(out), "--check"], capture_output=True, text=True)
    assert r.returncode == 0 and "PASS" in r.stdout
    out.write_text(out.read_text() + "\nx = 1\n")
    assert subprocess.run([sys.executable, tool, "splice", str(canon), str(out), "--check"],
                          capture_output=True).returncode == 1


@pytest.mark.skipif(not os.environ.get("REFERENCE_DIR") or not os.path.exists(REFERENCE_HARNESS),
                    reason="reference harness not present (set REFERENCE_DIR to a checkout)")
def test_splice_of_the_reference_harness_builds_the_library_model(tmp_path):
    """The reference's own harness, spliced: frozen symbols unchanged, and its
    UserOptimizedTransformer is this library's, loading the baseline's weights strictly."""
    with open(REFERENCE_HARNESS) as f:
        canon = f.read()
    out = ht.splice(canon, REPO)
    assert ht.verify_frozen(out, canon) == []
    path = tmp_path / "ttb_spliced.py"
    path.write_text(out)
    code = textwrap.dedent(f'''
        import sys, torch
        sys.path.insert(0, {str(tmp_path)!r})
        import ttb_spliced as T
        cfg = T.TransformerConfig(batch_size=2, seq_len=16, d_model=128, num_heads=4, ffn_dim=512,
                                  num_layers=1, causal=True)
        torch.manual_seed(0)
        base = T.BaselineTransformer(cfg)
        opt = T.UserOptimizedTransformer(cfg)
        T.copy_model_weights(base, opt)
        print(type(opt).__module__)
    ''')
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    assert r.stdout.strip().endswith("ffgko_b200.model")


def test_gate_passes_on_the_library():
    assert ht.gate_paths([PKG]) == []


@pytest.mark.parametrize("src,needle", [
    ("import oracle\n", "CPU oracle"),
    ("from oracle.transformer_oracle import model_forward\n", "CPU oracle"),
    ("import importlib\nm = importlib.import_module('oracle')\n", "dynamically"),
    ("import torch.nn.functional as F\ndef f(x, w):\n    return F.linear(x, w)\n", "F.linear"),
    ("import torch\ndef f(q, k, v):\n    return torch.nn.functional.scaled_dot_product_attention(q, k, v)\n",
     "scaled_dot_product_attention"),
    ("def f(a, b):\n    return a @ b\n", "@"),
    ("def f(s):\n    return s.softmax(-1)\n", ".softmax"),
    ("import torch\nclass M(torch.nn.Module):\n    def __init__(self):\n        self.register_buffer('c', None)\n",
     "register_buffer"),
    ("import torch\np = torch.nn.Parameter(torch.zeros(1))\n", "Parameter"),
    ("_cache = {}\n", "module-level mutable '_cache'"),
    ("def f(y):\n    y.detach_()\n", "detach_"),
])
def test_gate_flags(src, needle):
    probs = ht.gate_source(src, "m.py")
    assert probs and any(needle in p for p in probs), probs


def test_gate_allows_constants_and_mask_caches():
    assert ht.gate_source("EXPORTS = [1, 2]\n_mask_cache = {}\nLIMITS = {'a': 1}\n") == []


def _good_line():
    return {"metric": "m", "value": 3.0e8, "unit": "tokens/s", "warmup": 10, "steps": 100, "higher_is_better": True,
            "roofline": {"frac": 0.08}, "gpu_launches": 100, "accuracy": {"failed": 0, "total": 10},
            "e2e": {"value": 7.0e7}, "clocks": {"reasons": []}}


def test_bench_check():
    assert ht.check_bench_line(_good_line()) == []
    assert ht.check_bench_line({"impl": "reference", "unavailable": "why"}) == []
    for mutate, needle in ((lambda d: d["roofline"].update(frac=3.0), "far above"),
                           (lambda d: d.pop("gpu_launches"), "gpu_launches"),
                           (lambda d: d["accuracy"].update(failed=5), "outside the tolerance"),
                           (lambda d: d["e2e"].update(value=9e8), "e2e"),
                           (lambda d: d.update(warmup=1), "warmup"),
                           (lambda d: d["clocks"].update(reasons=["hw_slowdown"]), "throttling"),
                           (lambda d: d.update(value=0), "value")):
        d = copy.deepcopy(_good_line())
        mutate(d)
        probs = ht.check_bench_line(d)
        assert any(needle in p for p in probs), (needle, probs)


def test_bench_cli(tmp_path):
    f = tmp_path / "b.json"
    f.write_text("noise\n" + json.dumps(_good_line()) + "\n")
    tool = os.path.join(PKG, "harness_tools.py")
    assert subprocess.run([sys.executable, tool, "bench", str(f)], capture_output=True).returncode == 0
    bad = _good_line()
    bad["roofline"]["frac"] = 2.0
    f.write_text(json.dumps(bad) + "\n")
    assert subprocess.run([sys.executable, tool, "bench", str(f)], capture_output=True).returncode == 1
