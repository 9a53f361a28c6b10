"""B200-native per-symbol model-and-code loop of altxs (LTCB text compressor).

Host-side Python over a C-ABI CUDA library (``libaltxs_b200.so``, sm_100a):
mixed-bit GEMV/GEMM, sliding-window decode step, integer-CDF range coder and
test-time LoRA.  Entry points mirroring the reference live in
``altxs_b200.incremental``; the device coder in ``altxs_b200.gpu_ac``.
"""

from .config import ModelConfig, c1_config, c3_config  # noqa: F401

__version__ = "0.1.0"
