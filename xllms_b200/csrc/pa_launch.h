// pa_launch.h — host-side launchers of the kernels in pa_kernels.cu.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include "pa_device.cuh"

namespace xpa {

// CUDA-core kernel for every supported shape (fp16/fp32, head size <= 256).
cudaError_t launch_generic(const Params& p, int dtype_size, cudaStream_t st);

// TMA + tensor-core kernel; requires fast_path_shape_ok() and tensor maps
// describing the K and V pools as {d, slot, kv head, page} with a 64 x 16 box
// and 128-byte swizzle.
// kv_fmt: 0 = K/V in the query's dtype, kKvE4M3 / kKvE5M2 / kKvInt8 = one-byte cache.
bool fast_path_shape_ok(int head_size, int group, int block_size, int dtype_size, int kv_fmt = 0);
cudaError_t launch_fast(const CUtensorMap& tk, const CUtensorMap& tv, const Params& p,
                        cudaStream_t st);

// Merges split-context partials; a no-op per row whose sequence has one partition.
cudaError_t launch_reduce(const Params& p, int dtype_size, cudaStream_t st);

// KV append ("reshape and cache") of new tokens into the paged pools.
cudaError_t launch_append(const AppendParams& a, int dtype_size, cudaStream_t st);

// End-of-step barrier of the fused head gather (one warp; bounded waits).
cudaError_t launch_peer_barrier(void* const* flags, int world, int rank, unsigned long long step,
                                int* status, unsigned long long budget_ns, cudaStream_t st);

}  // namespace xpa
