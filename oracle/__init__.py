"""CPU oracle for NanoInfer's per-token decoder elementwise path.

TEST INFRASTRUCTURE ONLY. This package restates, on the CPU, the reference
algorithms that the CUDA kernels in ``nano_vllm_multimodal_b200`` replace. It
is the checker, never the thing measured or shipped: only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline / reference arm may
import it. The product path never routes through it.

Pinning: ``tests/golden/make_golden.py`` ran the reference's own modules
(``nanovllm.layers.*``, ``nanovllm.models.qwen3_vl``, the PyTorch paged-KV
backend) on seeded inputs and committed their outputs as fixtures;
``tests/test_oracle_golden.py`` checks every function here against those
fixtures bit-for-bit, and against the known-answer vectors of the reference's
own test-suite.
"""

from oracle.ops import *  # noqa: F401,F403
