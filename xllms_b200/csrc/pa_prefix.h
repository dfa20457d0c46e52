// pa_prefix.h — shared-prefix (cascade) attention kernel launcher.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include "pa_device.cuh"

namespace xpa {

// Prefix groups on the device: group g's members are
// members[offsets[g] .. offsets[g+1]); they share the first prefix_pages[m]
// pages of their block-table rows (the same count for every member).
struct PrefixGroups {
  const int* offsets;  // [num_groups + 1]
  const int* members;  // [offsets[num_groups]]
  int num_groups;
  int max_group_size;  // members of the largest group
  int max_chunks;      // ceil(longest prefix / prefix_chunk)
  int max_qblocks;     // set by launch_prefix: ceil(largest group * GS / rows per CTA)
  int rows;            // set by launch_prefix: query rows per CTA
};

// fp16, page size 16, head size 64/128/256 (the TMA path's shapes). Head
// sizes 64 and 128 with a 16-byte aligned query run on the tcgen05 kernel
// (128 query rows per CTA), 256 on the mma.sync kernel (64 rows per CTA).
// Whether launch_prefix takes the tcgen05 kernel for these parameters.
bool prefix_tc_ok(const Params& p);

// The tcgen05 kernel is persistent with at most max_ctas CTAs (one per SM).
cudaError_t launch_prefix(const CUtensorMap& tk, const CUtensorMap& tv, const Params& p,
                          const PrefixGroups& pg, int max_ctas, cudaStream_t st);

}  // namespace xpa
