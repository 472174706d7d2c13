"""B200-native position-shifted KV reuse: store gather, RoPE re-rotation, paged scatter.

Modules mirror the reference package ``marathon`` for this path:
``shift_kernels`` (tables, single-layer scatter, batched launcher),
``shift_store`` (session store and load/save planning) and
``vllm_shift_connector`` (the vLLM KV-connector hooks).  The native work is in
``libmarathon_shift.so`` (``csrc/``, C ABI in ``include/marathon_shift.h``).
"""

__version__ = "0.1.0"

from . import torch_ops  # noqa: E402,F401  registers torch.ops.marathon.*
