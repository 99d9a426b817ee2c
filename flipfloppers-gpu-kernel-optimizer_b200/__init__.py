"""B200-native (sm_100a) causal transformer-block forward.

Package layout (imported as ``ffgko_b200`` through ``load_package()`` in the
repository root's ``torch_transformer_benchmark.py``, because the directory
name is not a Python identifier):

* ``csrc/``   -- hand-written CUDA: tcgen05/TMA GEMM, flash causal attention,
  LayerNorm, and the C ABI (``include/b200_block.h``) in one translation unit;
* ``build.py`` -- nvcc recipe producing ``lib/libb200block.so`` in-tree;
* ``runtime.py`` -- ctypes binding of the C ABI;
* ``ops.py`` -- the PyTorch op layer (``torch.ops.b200.*`` custom ops with fake
  implementations, for torch.compile and graph capture);
* ``model.py`` -- the drop-in ``UserOptimizedTransformer`` and its arbiter;
* ``parallel.py`` -- one-process-per-GPU batch sharding and tensor parallelism.
"""

from . import build, ops, parallel, runtime  # noqa: F401
from .model import TransformerConfig, UserOptimizedTransformer  # noqa: F401
