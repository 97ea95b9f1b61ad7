"""The GPU drop-ins of ``kernel_agent.kernels.{quant,compare,scale_guard}`` and the new
blockwise-FP8 and FP8-attention APIs."""
