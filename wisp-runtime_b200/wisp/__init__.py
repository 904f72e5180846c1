"""wisp (B200 build): the WiSP Runtime decode hot path on hand-written sm_100a CUDA kernels.

Drop-in for the reference package of the same name (imronpuji/wisp-runtime 0.1.0): the modules keep the
reference's names and signatures (quant, kernels, store, cache_core, cache, moe, graphdec, model);
every kernel behind them lives in libwisp_b200.so (C ABI: include/wisp_b200.h).
"""

__version__ = "0.1.0+b200"
