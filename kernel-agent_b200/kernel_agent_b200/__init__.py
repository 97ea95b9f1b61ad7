"""B200-native (sm_100a) implementation of kernel-agent's low-precision hot path.

``kernel_agent_b200.kernels.quant`` mirrors ``kernel_agent.kernels.quant`` (quantisers and
scaled linears), ``kernel_agent_b200.kernels.compare`` mirrors ``kernel_agent.kernels.compare``
(the evaluator's comparator) and ``kernel_agent_b200.kernels.scale_guard`` its scale-rule
guard; ``kernel_agent_b200.kernels.blockwise`` and ``.attention`` add the blockwise-FP8 and
FP8-attention APIs in the same style. Every numeric loop runs in ``libkab.so`` (CUDA for
sm_100a, C ABI in ``include/kab.h``); CPU tensors are refused.
"""

__version__ = "0.1.0"
