"""xllms_b200 — B200-native (sm_100a) paged decode attention for xLLMs.

The product is the native code under csrc/ (kernels + C ABI, built into
_lib/libxpa.so, and the backend plugin _lib/libxllm_cuda_backend.so). This
package binds it for Python callers and carries the seeded workloads and the
KV-head sharding used by the tests and the benchmark.
"""
from . import _native  # noqa: F401
from .operator_api import (  # noqa: F401
    CudaBackendPlugin,
    NxtPagedAttentionInput,
    PagedAttentionError,
    device_status,
    kernel_path,
    make_input,
    nxt_paged_attention,
    nxt_paged_attention_flash,
    nxt_paged_attention_v2,
    paged_attention,
    workspace_size,
)

__all__ = [
    "paged_attention",
    "nxt_paged_attention",
    "nxt_paged_attention_v2",
    "nxt_paged_attention_flash",
    "CudaBackendPlugin",
    "NxtPagedAttentionInput",
    "PagedAttentionError",
    "make_input",
    "kernel_path",
    "workspace_size",
    "device_status",
]
