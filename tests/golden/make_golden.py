"""Generate the golden vectors that pin the oracle (run in the build container only).

It imports the reference's own ``torch_transformer_benchmark`` (the frozen fp32
``BaselineTransformer`` and ``generate_random_case``, TTB:49-192 and
TTB:1766-1804 of yeoshuyi/Flipfloppers-GPU-Kernel-Optimizer) from a checkout
given by ``--reference`` (default: the ``REFERENCE_DIR`` environment variable),
builds each case exactly as the reference harness does
(``torch.manual_seed(seed)`` then the model; ``x`` from the CPU generator at
``seed + trial``), runs the reference forward in fp32 on the CPU and writes:

* ``golden_<case>.npz``: ``y`` (reference output, fp32), the padding mask,
  checksums of ``x`` and the per-parameter (sum, sum of squares) fingerprints;
* ``golden_index.json``: the case list with shapes and seeds.

``x`` itself is not stored: the tests regenerate it from the seed with the
CPU generator and check it against the stored checksums.  Nothing at test or
bench time reads the reference checkout.

    REFERENCE_DIR=/path/to/reference python tests/golden/make_golden.py
"""

from __future__ import annotations

import argparse
import importlib.util
import json
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))

# (name, B, S, d, H, ffn, L, padding_ratio, seed, trial[, causal])
CASES = [
    ("c1", 4, 128, 128, 4, 512, 1, 0.0, 1234, 0),        # BASELINE config 1, trial 0
    ("c1_t1", 4, 128, 128, 4, 512, 1, 0.0, 1234, 1),     # trial 1 (seed 1235)
    ("ragged", 2, 100, 128, 4, 512, 1, 0.0, 1234, 0),     # S not a multiple of 128
    ("hd64", 2, 64, 256, 4, 1024, 1, 0.0, 1234, 0),       # head_dim 64
    ("h16", 1, 96, 1024, 16, 4096, 1, 0.0, 1234, 0),      # d=1024, H=16 (config-5 head shape)
    ("hd256", 2, 32, 1024, 4, 4096, 1, 0.0, 1234, 0),     # head_dim 256 (config 4b head shape)
    ("pad_l2", 3, 48, 64, 2, 256, 2, 0.3, 1234, 1),       # padding mask + two layers
    ("nc_c1", 4, 128, 128, 4, 512, 1, 0.0, 1234, 0, False),   # non-causal (harness default without --causal)
    ("nc_pad", 3, 100, 256, 4, 1024, 2, 0.4, 1234, 2, False),  # non-causal + padding + two layers
]


def load_reference(ref_dir: str):
    path = os.path.join(ref_dir, "torch_transformer_benchmark.py")
    spec = importlib.util.spec_from_file_location("_ref_ttb", path)
    mod = importlib.util.module_from_spec(spec)
    sys.modules["_ref_ttb"] = mod
    spec.loader.exec_module(mod)
    return mod


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("REFERENCE_DIR", ""))
    ap.add_argument("--out", default=HERE)
    args = ap.parse_args()
    if not args.reference:
        raise SystemExit("give --reference or REFERENCE_DIR")
    ref = load_reference(args.reference)
    torch.set_num_threads(os.cpu_count() or 1)
    index = []
    for case in CASES:
        name, B, S, d, H, F, L, pad, seed, trial = case[:10]
        causal = case[10] if len(case) > 10 else True
        cfg = ref.TransformerConfig(batch_size=B, seq_len=S, d_model=d, num_heads=H,
                                    ffn_dim=F, num_layers=L, causal=causal)
        cfg.validate()
        torch.manual_seed(seed)
        base = ref.BaselineTransformer(cfg).eval()
        x, mask = ref.generate_random_case(cfg, torch.device("cpu"), torch.float32,
                                           seed + trial, pad, 1.0)
        with torch.inference_mode():
            y = base(x, mask)
        fp = {k: [float(v.double().sum()), float((v.double() ** 2).sum())]
              for k, v in base.state_dict().items()}
        np.savez_compressed(
            os.path.join(args.out, f"golden_{name}.npz"),
            y=y.numpy().astype(np.float32),
            mask=mask.numpy(),
            x_sum=np.float64(x.double().sum()),
            x_abs_sum=np.float64(x.double().abs().sum()),
            x_head=x.reshape(-1)[:64].numpy().astype(np.float32),
            fingerprint=json.dumps(fp),
        )
        index.append(dict(name=name, B=B, S=S, d=d, H=H, ffn=F, L=L, padding_ratio=pad,
                          seed=seed, trial=trial, x_seed=seed + trial, causal=causal,
                          torch=torch.__version__))
        print(f"{name}: y max|.|={float(y.abs().max()):.4f}")
    with open(os.path.join(args.out, "golden_index.json"), "w") as f:
        json.dump(index, f, indent=1)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
