// pa_noalloc.cu — nxt_paged_attention_noalloc: paged decode attention that
// allocates no device memory.
//
// Who needs it: a serving engine that reserves almost all of HBM for its KV
// page pool before the first decode step has nothing left for a library's
// cudaMalloc, and hosts that route every device allocation through their own
// pool do not let a library allocate behind their back. cudaMalloc/cudaFree
// also synchronise the device, which stalls a decode loop. The regular entry
// points need device memory for split-context partials (a per-stream
// workspace they allocate, or one the caller passes); this one takes the
// partials from a fixed array compiled into the library instead.
//
// The array: g_noalloc_scratch below, NXT_PA_NOALLOC_SCRATCH_BYTES (32 MiB).
// Every GPU that loads this library module holds it until the process exits.
// Host code only ever passes its device address, which cudaGetSymbolAddress
// returns per device (in host code the name g_noalloc_scratch is a host-side
// stand-in, not a device address).
#include <climits>
#include <mutex>

#include "operator_api.h"
#include "pa_host.h"
#include "pa_launch.h"

namespace {

static __device__ __align__(256) unsigned char g_noalloc_scratch[NXT_PA_NOALLOC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;

std::mutex g_mu;
void* g_scratch_addr[kMaxDevices];  // device address of the array, per device

// Set-up, once per device, with that device current: look up the array's
// device address. May load this module onto the device, so a caller should
// make its first call on each device before any stream capture. The address
// is kept until the process exits; a cudaDeviceReset unloads the module and
// leaves it stale, so the entry point is not for use across a reset.
int scratch_address(int dev, void** out) {
  if (dev < 0 || dev >= kMaxDevices) return NXT_PA_EINVAL;
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_scratch_addr[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || p == nullptr)
      return NXT_PA_ECUDA;
    g_scratch_addr[dev] = p;
  }
  *out = g_scratch_addr[dev];
  return NXT_PA_OK;
}

}  // namespace

extern "C" int nxt_paged_attention_noalloc(
    void* out, const void* query, const void* key_cache, const void* value_cache,
    const int* block_tables, const int* seq_lens, int num_seqs, int num_heads, int head_size,
    int num_kv_heads, float scale, int max_num_blocks_per_seq, int block_size, int dtype_size,
    int64_t kv_block_stride, int64_t kv_head_stride, int64_t num_blocks, int* device_status,
    nxt_stream_t stream) {
  using namespace xpa::host;
  const int B = num_seqs, Hq = num_heads, D = head_size, Hkv = num_kv_heads;
  int rc = check_args(out, query, key_cache, value_cache, block_tables, seq_lens, B, Hq, D, Hkv,
                      max_num_blocks_per_seq, block_size, dtype_size, kv_block_stride,
                      kv_head_stride);
  if (rc != NXT_PA_OK || B == 0) return rc;

  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return NXT_PA_ECUDA;
  const Plan pl = make_plan(B, Hq, D, Hkv, max_num_blocks_per_seq, sm_count_of(dev));
  if ((long long)B * Hkv * pl.max_parts > INT_MAX || (long long)B * Hq > INT_MAX)
    return NXT_PA_EINVAL;
  if (pl.ws_bytes > (size_t)NXT_PA_NOALLOC_SCRATCH_BYTES) return NXT_PA_ESCRATCH;

  // Every partial the reduce reads is written earlier in the same call, so
  // nothing in the array has to start at zero.
  void* scratch = nullptr;
  if (pl.ws_bytes > 0) {
    rc = scratch_address(dev, &scratch);
    if (rc != NXT_PA_OK) return rc;
  }

  xpa::Params p{};
  p.out = out;
  p.q = query;
  p.k = key_cache;
  p.v = value_cache;
  p.block_tables = block_tables;
  p.seq_lens = seq_lens;
  p.part_o = static_cast<float*>(scratch);
  p.part_ml = scratch ? reinterpret_cast<float*>(
                            static_cast<char*>(scratch) +
                            part_ml_offset_bytes((long long)B * Hq * pl.max_parts, D))
                      : nullptr;
  p.status = device_status;
  p.kv_block_stride = kv_block_stride;
  p.kv_head_stride = kv_head_stride;
  p.num_blocks = num_blocks;
  p.timeout_ns = wait_budget_ns();
  p.B = B;
  p.Hq = Hq;
  p.Hkv = Hkv;
  p.D = D;
  p.GS = Hq / Hkv;
  p.max_blocks = max_num_blocks_per_seq;
  p.block_size = block_size;
  p.part_pages = pl.part_pages;
  p.max_parts = pl.max_parts;
  p.slots = pl.max_parts;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.vec8 = (D % 8 == 0 && (reinterpret_cast<uintptr_t>(out) & 15u) == 0) ? 1 : 0;

  cudaStream_t st = static_cast<cudaStream_t>(stream);
  CUtensorMap tk, tv;
  const bool fast =
      xpa::fast_path_shape_ok(D, p.GS, block_size, dtype_size) &&
      fast_layout_ok(key_cache, value_cache, D, Hkv, kv_block_stride, kv_head_stride) &&
      (reinterpret_cast<uintptr_t>(query) & 3u) == 0 &&
      encode_pool(&tk, key_cache, D, Hkv, num_blocks, kv_block_stride, kv_head_stride) &&
      encode_pool(&tv, value_cache, D, Hkv, num_blocks, kv_block_stride, kv_head_stride);
  cudaError_t e = fast ? xpa::launch_fast(tk, tv, p, st) : xpa::launch_generic(p, dtype_size, st);
  if (e != cudaSuccess) return NXT_PA_ECUDA;
  if (pl.max_parts > 1 && xpa::launch_reduce(p, dtype_size, st) != cudaSuccess)
    return NXT_PA_ECUDA;
  return NXT_PA_OK;
}
