"""comp_b200: B200-native (sm_100a) backend for COMP's quantized decode path.

The four ops of COMP (`quant_q8_0`, `quant_q8_K`, `q4_0_gemv`, `tq2_0_gemv`) on KURN's split layout, as hand-written
CUDA kernels behind a C-ABI library (include/comp_b200.h), with COMP's host API (`comp_b200.host`), its spec/CLI
routing (`comp_b200.spec`, `comp_b200.cli`, `comp_b200.kurn_ext`) and a row-sharded multi-GPU layer
(`comp_b200.dist`).
"""

__version__ = "0.1.0"
