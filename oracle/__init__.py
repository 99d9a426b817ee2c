"""CPU oracle for the causal transformer-block forward (TEST INFRASTRUCTURE).

This package is the checker, never the product.  Only ``tests/``,
``__graft_entry__.smoke()`` and the CPU-baseline leg of ``bench.py`` may import
it.  The product path (``torch_transformer_benchmark.UserOptimizedTransformer``
and the CUDA library under ``flipfloppers-gpu-kernel-optimizer_b200/``) never
calls into it and has no CPU fallback.

Parity is pinned: ``tests/golden/make_golden.py`` imported the reference's own
fp32 ``BaselineTransformer`` (torch_transformer_benchmark.py:49-192 of
yeoshuyi/Flipfloppers-GPU-Kernel-Optimizer) in the build container, ran it on
seeded inputs and committed inputs, outputs and weight fingerprints under
``tests/golden/``; ``tests/test_oracle_golden.py`` checks this restatement
against those vectors.
"""

from .transformer_oracle import (  # noqa: F401
    OracleConfig,
    block_forward,
    causal_attention,
    chunk_rows_forward,
    gelu_erf,
    layer_norm,
    linear,
    model_forward,
    prefix_kv,
    sampled_rows_forward,
)
from .kernel_gelu import gelu_as_f32, gelu_as_max_error  # noqa: F401
from .harness import (  # noqa: F401
    AccuracyResult,
    compare_outputs,
    generate_random_case,
    generate_chunked_input,
    params_from_state_dict,
    init_state_dict,
    fingerprint,
)
