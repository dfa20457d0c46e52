// pa_tables.cu — block-table builder: one decode step's kernel inputs from
// the scheduler's page lists.
//
// The reference stops at the scheduler (src/core/scheduler.c:278-440 picks
// the requests of a step; src/core/memory_manager.c:207-273 hands out pages;
// src/core/prefix_sharing.c:211-265 matches radix prefixes) and never builds
// the device arrays the attention operator reads. This file does: from host
// CSR page lists it produces, in one caller-owned device buffer,
//   block tables [B][max_blocks] int32 (-1 past a sequence's pages),
//   seq_lens [B], the slot of each sequence's newest token (int64, the KV
//   append's slot_mapping), and the prefix groups of the cascade call
//   (sequences sharing a radix node with >= 1 whole shared page).
// The host packs every input into one pinned image (one H2D copy); a
// grid-stride kernel expands the CSR lists into the padded table rows with
// coalesced stores.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <cstring>
#include <map>
#include <vector>

#include "operator_api.h"

namespace {

constexpr size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

// Device layout of the builder's buffer (byte offsets).
struct Layout {
  size_t seq_lens, prefix_pages, group_offsets, members, page_offsets, page_ids, image_end;
  size_t slots, tables, total;
};

Layout layout_of(long long B, long long max_blocks, long long total_pages) {
  Layout L{};
  size_t o = 0;
  L.seq_lens = o;
  o += (size_t)B * 4;
  L.prefix_pages = o;
  o += (size_t)B * 4;
  L.group_offsets = o;
  o += (size_t)(B + 1) * 4;
  L.members = o;
  o += (size_t)B * 4;
  L.page_offsets = o;
  o += (size_t)(B + 1) * 4;
  L.page_ids = o;
  o += (size_t)total_pages * 4;
  L.image_end = o;
  L.slots = align_up(o, 16);
  L.tables = align_up(L.slots + (size_t)B * 8, 16);
  L.total = L.tables + (size_t)B * max_blocks * 4;
  return L;
}

__global__ void __launch_bounds__(256)
    build_tables_kernel(int* __restrict__ tables, long long* __restrict__ slots,
                        const int* __restrict__ page_offsets, const int* __restrict__ page_ids,
                        const int* __restrict__ seq_lens, int B, int max_blocks, int block_size) {
  const long long n = (long long)B * max_blocks;
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
    const int b = (int)(i / max_blocks), j = (int)(i - (long long)b * max_blocks);
    const int off = __ldg(page_offsets + b), np = __ldg(page_offsets + b + 1) - off;
    tables[i] = j < np ? __ldg(page_ids + off + j) : -1;
  }
  for (long long b = (long long)blockIdx.x * blockDim.x + threadIdx.x; b < B; b += stride) {
    const int L = __ldg(seq_lens + b);
    long long slot = -1;
    if (L > 0) {
      const int page = __ldg(page_ids + __ldg(page_offsets + b) + (L - 1) / block_size);
      slot = (long long)page * block_size + (L - 1) % block_size;
    }
    slots[b] = slot;
  }
}

}  // namespace

extern "C" {

size_t nxt_block_tables_layout(int num_seqs, int max_blocks_per_seq, int total_pages,
                               size_t offsets[NXT_BT_NUM_ARRAYS]) {
  if (num_seqs < 0 || max_blocks_per_seq < 0 || total_pages < 0) return 0;
  const Layout L = layout_of(num_seqs, max_blocks_per_seq, total_pages);
  if (offsets) {
    offsets[NXT_BT_TABLES] = L.tables;
    offsets[NXT_BT_SEQ_LENS] = L.seq_lens;
    offsets[NXT_BT_SLOTS] = L.slots;
    offsets[NXT_BT_PREFIX_PAGES] = L.prefix_pages;
    offsets[NXT_BT_GROUP_OFFSETS] = L.group_offsets;
    offsets[NXT_BT_GROUP_MEMBERS] = L.members;
  }
  return L.total;
}

size_t nxt_block_tables_staging_size(int num_seqs, int total_pages) {
  if (num_seqs < 0 || total_pages < 0) return 0;
  return layout_of(num_seqs, 0, total_pages).image_end;
}

int nxt_build_block_tables(const int* page_offsets, const int* page_ids, const int* seq_lens,
                           const int* prefix_node, const int* prefix_pages, int num_seqs,
                           int max_blocks_per_seq, int block_size, void* device_buffer,
                           size_t device_bytes, void* host_staging, size_t staging_bytes,
                           int* num_groups, int* max_group_size, int* max_prefix_pages,
                           nxt_stream_t stream) {
  if (num_seqs < 0 || max_blocks_per_seq < 0 || block_size <= 0) return NXT_PA_EINVAL;
  if (num_groups) *num_groups = 0;
  if (max_group_size) *max_group_size = 0;
  if (max_prefix_pages) *max_prefix_pages = 0;
  if (num_seqs == 0) return NXT_PA_OK;
  if (!page_offsets || !seq_lens || !device_buffer) return NXT_PA_EINVAL;
  if ((prefix_node == nullptr) != (prefix_pages == nullptr)) return NXT_PA_EINVAL;
  const int B = num_seqs;
  if (page_offsets[0] != 0) return NXT_PA_EINVAL;
  for (int b = 0; b < B; ++b) {
    const long long np = (long long)page_offsets[b + 1] - page_offsets[b];
    if (np < 0 || np > max_blocks_per_seq) return NXT_PA_EINVAL;
    if (seq_lens[b] < 0 || (long long)seq_lens[b] > np * block_size) return NXT_PA_EINVAL;
  }
  const int total = page_offsets[B];
  if (total > 0 && !page_ids) return NXT_PA_EINVAL;
  const Layout L = layout_of(B, max_blocks_per_seq, total);
  if (device_bytes < L.total || (reinterpret_cast<uintptr_t>(device_buffer) & 15u)) {
    return NXT_PA_EWORKSPACE;
  }

  // Host image of [seq_lens | prefix_pages | group_offsets | members |
  // page_offsets | page_ids], copied to the device in one transfer.
  std::vector<uint8_t> own;
  uint8_t* img;
  if (host_staging) {
    if (staging_bytes < L.image_end) return NXT_PA_EWORKSPACE;
    img = static_cast<uint8_t*>(host_staging);
  } else {
    own.resize(L.image_end);
    img = own.data();
  }
  int* i_seq = reinterpret_cast<int*>(img + L.seq_lens);
  int* i_pp = reinterpret_cast<int*>(img + L.prefix_pages);
  int* i_go = reinterpret_cast<int*>(img + L.group_offsets);
  int* i_mem = reinterpret_cast<int*>(img + L.members);
  std::memcpy(i_seq, seq_lens, (size_t)B * 4);
  std::memcpy(img + L.page_offsets, page_offsets, (size_t)(B + 1) * 4);
  if (total) std::memcpy(img + L.page_ids, page_ids, (size_t)total * 4);
  std::memset(i_pp, 0, (size_t)B * 4);

  // Prefix groups: sequences with the same radix node and >= 1 whole shared
  // page; every member must carry the same count and the same page ids.
  int G = 0, max_size = 0, max_pages = 0, nmem = 0;
  i_go[0] = 0;
  if (prefix_node) {
    std::map<int, std::vector<int>> by_node;
    for (int b = 0; b < B; ++b)
      if (prefix_node[b] >= 0 && prefix_pages[b] > 0) by_node[prefix_node[b]].push_back(b);
    for (auto& kv : by_node) {
      const std::vector<int>& m = kv.second;
      if (m.size() < 2) continue;  // a group of one shares nothing
      const int P = prefix_pages[m[0]];
      for (int b : m) {
        if (prefix_pages[b] != P) return NXT_PA_EINVAL;
        if ((long long)P * block_size > seq_lens[b]) return NXT_PA_EINVAL;
        for (int j = 0; j < P; ++j)
          if (page_ids[page_offsets[b] + j] != page_ids[page_offsets[m[0]] + j])
            return NXT_PA_EINVAL;
      }
      for (int b : m) {
        i_pp[b] = P;
        i_mem[nmem++] = b;
      }
      i_go[++G] = nmem;
      max_size = std::max(max_size, (int)m.size());
      max_pages = std::max(max_pages, P);
    }
  }
  for (int g = G + 1; g <= B; ++g) i_go[g] = nmem;
  for (int k = nmem; k < B; ++k) i_mem[k] = 0;

  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  uint8_t* dev = static_cast<uint8_t*>(device_buffer);
  if (cudaMemcpyAsync(dev, img, L.image_end, cudaMemcpyHostToDevice, st) != cudaSuccess)
    return NXT_PA_ECUDA;
  const long long work = (long long)B * std::max(max_blocks_per_seq, 1);
  int dev_id = 0, sms = 148;
  if (cudaGetDevice(&dev_id) == cudaSuccess)
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev_id);
  const long long grid = std::min<long long>((work + 255) / 256, (long long)sms * 8);
  build_tables_kernel<<<(unsigned)std::max<long long>(grid, 1), 256, 0, st>>>(
      reinterpret_cast<int*>(dev + L.tables), reinterpret_cast<long long*>(dev + L.slots),
      reinterpret_cast<const int*>(dev + L.page_offsets),
      reinterpret_cast<const int*>(dev + L.page_ids), reinterpret_cast<const int*>(dev + L.seq_lens),
      B, max_blocks_per_seq, block_size);
  if (cudaGetLastError() != cudaSuccess) return NXT_PA_ECUDA;
  // a pageable image must outlive the copy
  if (!host_staging && cudaStreamSynchronize(st) != cudaSuccess) return NXT_PA_ECUDA;
  if (num_groups) *num_groups = G;
  if (max_group_size) *max_group_size = max_size;
  if (max_prefix_pages) *max_prefix_pages = max_pages;
  return NXT_PA_OK;
}

}  // extern "C"
