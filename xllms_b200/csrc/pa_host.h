// pa_host.h — host-side planning helpers shared by the C-ABI entry points
// (pa_api.cu) and the allocation-free entry point (pa_noalloc.cu).
#pragma once

#include <cuda.h>
#include <stddef.h>

namespace xpa {
namespace host {

int ceil_div(long long a, long long b);

// SM count of device `dev` (cached; 148 when the query fails).
int sm_count_of(int dev);

// Bound on every pipeline wait of kernels launched by this host thread
// (nxt_paged_attention_set_wait_budget_ns; 1 s by default).
unsigned long long wait_budget_ns();

// Split-context partials of one call, in one workspace: part_o
// [rows][slots][D] fp32 from byte 0, then part_ml [rows][slots][2] fp32 from
// the next kPartAlign-byte boundary (rows = B * Hq). The merge reads (m, l)
// as 8-byte pairs, which an odd rows * slots * D would otherwise misalign,
// and part_o rows as 16-byte vectors, so the workspace itself must start on a
// 16-byte boundary.
constexpr size_t kPartAlign = 256;
inline size_t part_ml_offset_bytes(long long row_slots, int D) {
  const size_t o = (size_t)row_slots * (size_t)D * sizeof(float);
  return (o + kPartAlign - 1) / kPartAlign * kPartAlign;
}
inline size_t partial_bytes(long long row_slots, int D) {
  return part_ml_offset_bytes(row_slots, D) + (size_t)row_slots * 2 * sizeof(float);
}
inline bool workspace_aligned(const void* ws) {
  return (reinterpret_cast<size_t>(ws) & 15u) == 0;
}

// Context partitioning of one call and the split-context partial bytes it needs.
struct Plan {
  int part_pages = 32;
  int max_parts = 1;
  size_t ws_bytes = 0;
};
// kv_es: bytes per K / V element (1 for fp8 pools, whose partitions keep
// shrinking until the grid holds 24 CTAs per SM instead of 12).
Plan make_plan(int B, int Hq, int D, int Hkv, int max_blocks, int nsm, int kv_es = 2);

// Tensor map of one pool for the TMA path; false when it cannot be encoded.
// es: bytes per K / V element (2 = fp16, 1 = fp8).
bool encode_pool(CUtensorMap* m, const void* base, int D, int Hkv, long long num_blocks,
                 long long kbs, long long khs, int es = 2);

// Pool alignment and stride order the TMA path needs.
bool fast_layout_ok(const void* k, const void* v, int D, int Hkv, long long kbs, long long khs,
                    int es = 2);

// NXT_PA_OK or NXT_PA_EINVAL for the argument set of one call.
int check_args(const void* out, const void* q, const void* k, const void* v, const int* bt,
               const int* sl, int B, int Hq, int D, int Hkv, int max_blocks, int bs, int ds,
               long long kbs, long long khs);

}  // namespace host
}  // namespace xpa
