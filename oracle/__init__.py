"""CPU oracle of kernel-agent's low-precision path: TEST INFRASTRUCTURE ONLY.

A numpy restatement of the reference's arithmetic (``src/kernel_agent/kernels/quant.py``,
``src/kernel_agent/kernels/compare.py``, ``docs/research-scripts/fp8-sm120/fp8lib.py``),
each function citing the reference file:line it follows. It is pinned by the golden
vectors under ``tests/golden/`` (outputs of the reference itself, made by
``tests/golden/make_golden.py``) and by the known answers of the reference's own tests.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py`` (its CPU-baseline and
``--impl reference`` arms) import this package, and only as the checker or as the timed
CPU baseline. The product path (``kernel_agent_b200``) never imports it: it runs the CUDA
library or raises.

Conventions: floating-point inputs are numpy ``float32`` arrays holding the values of the
reference's tensors (bf16 inputs are exactly representable); fp32 arithmetic is done in
``float32`` one operation at a time, as torch does on the CPU; bf16 outputs are returned as
``uint16`` bit patterns, e4m3 / e8m0 / packed e2m1 as ``uint8`` bytes.
"""
