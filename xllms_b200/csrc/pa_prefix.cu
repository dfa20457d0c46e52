// pa_prefix.cu — shared-prefix ("cascade") attention for prefix groups.
//
// A prefix group is a set of sequences whose block-table rows begin with the
// same P pages (a radix-tree prefix shared by all of them). Instead of every
// member re-reading those pages for its own GS query heads, one CTA takes a
// block of 64 query rows — (member, head) pairs of the group, for one KV head
// — and runs them against the shared pages as a dense tile, flash-attention
// style: per 16-token page
//   S (64 rows x 16 tokens) = Q (64 x D) . K_page^T          [mma.sync]
//   online softmax per row, O (64 x D) += P (64 x 16) . V_page [mma.sync]
// with pages streamed by TMA through a shared-memory ring that all four
// consumer warps read (each warp owns 16 rows). P is split into fp16 hi + lo
// so PV keeps fp32-level accuracy. Each CTA covers one chunk of prefix_chunk
// prefix pages and writes, for each of its rows, the partial (m, l, o) into
// slot `chunk` of that row; the decode kernel covers the pages after the
// prefix (slots after the prefix chunks) and pa_reduce_kernel merges all of
// them by log-sum-exp.
#include <climits>

#include "pa_device.cuh"
#include "pa_prefix.h"
#include "pa_tcgen05.cuh"

namespace xpa {

namespace {

constexpr uint64_t kPrefixDrainNs = 1000000000ull;
// Largest chunk (pages) one prefix CTA takes; the host keeps chunks within it.
constexpr int kMaxPrefixChunk = 512;

template <int D, int STAGES>
struct PrefixCfg {
  static constexpr int kTile = 16 * D * 2;
  static constexpr int kStage = 2 * kTile;
  static constexpr int kKSteps = D / 16;
  static constexpr int kBoxes = D / 64;
  static constexpr int kNT = D / 8;  // n-tiles of the output (8 dims each)
  static constexpr int kRows = 64;   // query rows per CTA (16 per consumer warp)
  static constexpr int kWarps = 4;
  static constexpr int kSmem = 1024 + STAGES * kStage + STAGES * 16 + STAGES * 4;
};

// Grid index -> (group, kv head, query block, chunk) with chunk fastest.
struct PrefixItem {
  int g, kvh, qb, chunk;
  int first;       // first member: its block-table row supplies the pages
  int members;     // members of the group
  int rows;        // members * GS query rows
  int L;           // the first member's context length (bounds the prefix tokens)
  int page_begin, page_end;
};

__device__ __forceinline__ bool decode_prefix_item(const Params& p, const PrefixGroups& pg,
                                                   int idx, PrefixItem& it) {
  it.chunk = idx % pg.max_chunks;
  int r = idx / pg.max_chunks;
  it.qb = r % pg.max_qblocks;
  r /= pg.max_qblocks;
  it.kvh = r % p.Hkv;
  it.g = r / p.Hkv;
  const int off0 = __ldg(pg.offsets + it.g), off1 = __ldg(pg.offsets + it.g + 1);
  it.members = off1 - off0;
  it.rows = it.members * p.GS;
  if (it.members <= 0 || it.qb * pg.rows >= it.rows) return false;
  it.first = __ldg(pg.members + off0);
  int L = __ldg(p.seq_lens + it.first);
  const long long cap = (long long)p.max_blocks * p.block_size;
  L = L < 0 ? 0 : ((long long)L > cap ? (int)cap : L);
  it.L = L;
  const int npages = (L + p.block_size - 1) / p.block_size;
  const int P = prefix_of(p, it.first, npages);
  it.page_begin = it.chunk * p.prefix_chunk;
  it.page_end = min(P, it.page_begin + p.prefix_chunk);
  return it.page_begin < it.page_end;
}

template <int D, int STAGES>
__global__ void __launch_bounds__(160)
    pa_prefix_kernel(const __grid_constant__ CUtensorMap tmK,
                     const __grid_constant__ CUtensorMap tmV, const Params p,
                     const PrefixGroups pg) {
  using C = PrefixCfg<D, STAGES>;
  pdl_launch_dependents();  // the suffix kernel runs alongside
  PrefixItem it;
  if (!decode_prefix_item(p, pg, blockIdx.x, it)) return;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const uint32_t sbase = smem_u32(smem);
  const uint32_t bar_full = smem_u32(smem + STAGES * C::kStage);
  const uint32_t bar_empty = bar_full + 8 * STAGES;
  int* meta = reinterpret_cast<int*>(smem + STAGES * C::kStage + STAGES * 16);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
#pragma unroll
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(bar_full + 8 * s, 1);
      mbar_init(bar_empty + 8 * s, C::kWarps);  // every consumer warp reads every page
    }
    fence_mbar_init();
  }
  __syncthreads();
  const int np = it.page_end - it.page_begin;
  const uint64_t budget = p.timeout_ns;

  if (warp == C::kWarps) {
    // ── producer: the shared pages, from the first member's block-table row
    if (lane == 0) {
      tmap_prefetch(&tmK);
      tmap_prefetch(&tmV);
    }
    const int* bt_row = p.block_tables + (long long)it.first * p.max_blocks;
    int ent = -1, ok = 1, issued = 0;
    for (int j = 0; j < np; ++j) {
      if ((j & 31) == 0) {
        const int idx = it.page_begin + j + lane;
        ent = idx < it.page_end ? __ldg(bt_row + idx) : -1;
      }
      const int phys = __shfl_sync(0xffffffffu, ent, j & 31);
      if (lane == 0) {
        const int s = j % STAGES;
        if (j >= STAGES && !mbar_wait(bar_empty + 8 * s, ((j / STAGES) + 1) & 1, budget)) {
          raise_status(p, kDevTimeout);
          ok = 0;
        } else {
          const bool valid = phys >= 0 && (p.num_blocks <= 0 || phys < p.num_blocks);
          meta[s] = valid ? 1 : 0;
          if (valid) {
            const uint32_t full = bar_full + 8 * s;
            mbar_arrive_expect_tx(full, C::kStage);
            const uint32_t tk = sbase + s * C::kStage, tv = tk + C::kTile;
#pragma unroll
            for (int x = 0; x < C::kBoxes; ++x) {
              tma_load_4d(tk + x * 2048, &tmK, x * 64, 0, it.kvh, phys, full);
              tma_load_4d(tv + x * 2048, &tmV, x * 64, 0, it.kvh, phys, full);
            }
          } else {
            raise_status(p, kDevBadPage);
            mbar_arrive(bar_full + 8 * s);
          }
          issued = j + 1;
        }
      }
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) break;
    }
    if (!ok && lane == 0) {
      for (int j = issued > STAGES ? issued - STAGES : 0; j < issued; ++j)
        (void)mbar_wait(bar_full + 8 * (j % STAGES), (j / STAGES) & 1, kPrefixDrainNs);
    }
    return;
  }

  // ── consumers: warp w owns rows qb*64 + 16w + [0, 16)
  const int g = lane >> 2, c = lane & 3;
  const int GS = p.GS;
  const int row_base = it.qb * C::kRows + warp * 16;
  long long qrow[2];   // global (b * Hq + hq) of rows g and g + 8
  bool live[2];
#pragma unroll
  for (int k = 0; k < 2; ++k) {
    const int r = row_base + g + 8 * k;
    live[k] = r < it.rows;
    qrow[k] = -1;
    if (live[k]) {
      const int member = __ldg(pg.members + __ldg(pg.offsets + it.g) + r / GS);
      qrow[k] = (long long)member * p.Hq + (long long)it.kvh * GS + r % GS;
    }
  }
  // Q as the A operand (m = rows, k = d): a0/a2 from row g, a1/a3 from row g+8.
  uint32_t qa[C::kKSteps][4];
  const __half* Q = static_cast<const __half*>(p.q);
#pragma unroll
  for (int ks = 0; ks < C::kKSteps; ++ks) {
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      if (live[k]) {
        const __half* src = Q + qrow[k] * D + ks * 16 + 2 * c;
        qa[ks][k] = __ldg(reinterpret_cast<const unsigned int*>(src));
        qa[ks][2 + k] = __ldg(reinterpret_cast<const unsigned int*>(src + 8));
      } else {
        qa[ks][k] = qa[ks][2 + k] = 0u;
      }
    }
  }
  float o[C::kNT][4];
#pragma unroll
  for (int nt = 0; nt < C::kNT; ++nt) o[nt][0] = o[nt][1] = o[nt][2] = o[nt][3] = 0.f;
  float mrun[2] = {-INFINITY, -INFINITY}, lrun[2] = {0.f, 0.f};
  const float sl2 = p.scale_log2;
  const int mi = lane >> 3, r8 = lane & 7;

  for (int j = 0; j < np; ++j) {
    const int s = j % STAGES;
    if (!mbar_wait(bar_full + 8 * s, (j / STAGES) & 1, budget)) {
      raise_status(p, kDevTimeout);
      break;
    }
    if (meta[s]) {
      const uint32_t tk = sbase + s * C::kStage, tv = tk + C::kTile;
      // S = Q . K^T: K rows are tokens; ldmatrix gives (tok 0-7 | 8-15) x (d lo | hi).
      float sc[2][4];
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) sc[nt][0] = sc[nt][1] = sc[nt][2] = sc[nt][3] = 0.f;
#pragma unroll
      for (int ks = 0; ks < C::kKSteps; ++ks) {
        uint32_t b0, b1, b2, b3;
        ldsm_x4(tk + tile_off(r8 + ((mi >> 1) << 3), 2 * ks + (mi & 1)), b0, b1, b2, b3);
        mma_f16_16816(sc[0], qa[ks][0], qa[ks][1], qa[ks][2], qa[ks][3], b0, b1);
        mma_f16_16816(sc[1], qa[ks][0], qa[ks][1], qa[ks][2], qa[ks][3], b2, b3);
      }
      // Online softmax per row (rows g: regs 0,1; g+8: regs 2,3); all 16
      // tokens of a prefix page are valid.
      float mx[2];
      mx[0] = fmaxf(fmaxf(sc[0][0], sc[0][1]), fmaxf(sc[1][0], sc[1][1])) * sl2;
      mx[1] = fmaxf(fmaxf(sc[0][2], sc[0][3]), fmaxf(sc[1][2], sc[1][3])) * sl2;
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        mx[k] = fmaxf(mx[k], __shfl_xor_sync(0xffffffffu, mx[k], 1));
        mx[k] = fmaxf(mx[k], __shfl_xor_sync(0xffffffffu, mx[k], 2));
      }
      float al[2], pp[2][4];
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        const float mn = fmaxf(mrun[k], mx[k]);
        al[k] = ex2(mrun[k] - mn);
        mrun[k] = mn;
      }
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) {
        pp[nt][0] = ex2(sc[nt][0] * sl2 - mrun[0]);
        pp[nt][1] = ex2(sc[nt][1] * sl2 - mrun[0]);
        pp[nt][2] = ex2(sc[nt][2] * sl2 - mrun[1]);
        pp[nt][3] = ex2(sc[nt][3] * sl2 - mrun[1]);
      }
      lrun[0] = fmaf(lrun[0], al[0], pp[0][0] + pp[0][1] + pp[1][0] + pp[1][1]);
      lrun[1] = fmaf(lrun[1], al[1], pp[0][2] + pp[0][3] + pp[1][2] + pp[1][3]);
#pragma unroll
      for (int nt = 0; nt < C::kNT; ++nt) {
        o[nt][0] *= al[0];
        o[nt][1] *= al[0];
        o[nt][2] *= al[1];
        o[nt][3] *= al[1];
      }
      // P as the A operand of PV (m = rows, k = tokens): the S accumulators
      // already sit in that layout; split into fp16 hi + lo.
      uint32_t ph[4], pl[4];
      {
        const float v[4][2] = {{pp[0][0], pp[0][1]}, {pp[0][2], pp[0][3]},
                               {pp[1][0], pp[1][1]}, {pp[1][2], pp[1][3]}};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          ph[i] = pack_half2(v[i][0], v[i][1]);
          const float2 f = unpack_half2(ph[i]);
          pl[i] = pack_half2(v[i][0] - f.x, v[i][1] - f.y);
        }
      }
      // O += P . V: V rows are tokens; transposed loads give the B operand
      // (k = tokens, n = d) for two 8-dim n-tiles per ldmatrix.x4.
#pragma unroll
      for (int jt = 0; jt < D / 16; ++jt) {
        uint32_t b0, b1, b2, b3;
        ldsm_x4_trans(tv + tile_off(r8 + ((mi & 1) << 3), 2 * jt + (mi >> 1)), b0, b1, b2, b3);
        mma_f16_16816(o[2 * jt], ph[0], ph[1], ph[2], ph[3], b0, b1);
        mma_f16_16816(o[2 * jt], pl[0], pl[1], pl[2], pl[3], b0, b1);
        mma_f16_16816(o[2 * jt + 1], ph[0], ph[1], ph[2], ph[3], b2, b3);
        mma_f16_16816(o[2 * jt + 1], pl[0], pl[1], pl[2], pl[3], b2, b3);
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(bar_empty + 8 * s);
  }

  // ── partial (m, l, o) of rows g and g+8 into slot `chunk`
#pragma unroll
  for (int k = 0; k < 2; ++k) {
    lrun[k] += __shfl_xor_sync(0xffffffffu, lrun[k], 1);
    lrun[k] += __shfl_xor_sync(0xffffffffu, lrun[k], 2);
  }
#pragma unroll
  for (int k = 0; k < 2; ++k) {
    if (!live[k]) continue;
    const long long pr = qrow[k] * p.slots + it.chunk;
    float* dst = p.part_o + pr * D;
#pragma unroll
    for (int nt = 0; nt < C::kNT; ++nt) {
      float2 v2 = make_float2(o[nt][2 * k], o[nt][2 * k + 1]);
      *reinterpret_cast<float2*>(dst + nt * 8 + 2 * c) = v2;
    }
    if (c == 0) {
      p.part_ml[2 * pr] = mrun[k];
      p.part_ml[2 * pr + 1] = lrun[k];
    }
  }
}

// ════════════════════════════════════════════════════════════════════════
// tcgen05 version (head size 64 or 128), persistent: CTA c takes the items
// (group, KV head, block of 128 query rows, chunk) c, c + grid, c + 2 grid,
// ... For each item, per S block of 4 pages (64 tokens):
//   S (128 x 64, fp32 in TMEM)  = Q (128 x D, smem) . K_blk^T     [tcgen05.mma]
//   softmax: S rows -> registers (tcgen05.ld), P = 2^(s - m) split into
//     fp16 hi + lo, written to shared memory in the MMA's operand layout
//   O (128 x D, fp32 in TMEM)  += P_hi . V_blk + P_lo . V_blk       [tcgen05.mma]
// Warp roles: warps 0 and 2 (lane 0) stream K and V pages by TMA into a
// STAGES-deep ring; warp 1 owns the TMEM allocation and its lane 0 issues
// every MMA; warp 3 decodes the CTA's items into a table at start; warps
// 4..11 run the softmax: row i (TMEM lane i) belongs to the two warps of
// lane quadrant i / 32, one taking tokens 0..31 of each block, the other
// 32..63, exchanging their row maxima through shared memory. S is double
// buffered so QK of block j+1 runs while the softmax works on block j; ring
// slots, S and P buffers and their barrier phases run on across items.
// The running max m is raised only when a row's block max exceeds it by more
// than 8 (log2 units); then O's row is rescaled in TMEM once PV of the
// previous block has completed. P stays <= 2^8, exact enough in fp16 hi+lo.
// An item's partial (m, l, O) leaves through the P buffers (idle by then)
// so each output row is written by one warp in 16-byte pieces.
// Every wait is bounded; on expiry the kernel raises the timeout bit, drains
// its copies and MMAs and frees TMEM before returning.
// ════════════════════════════════════════════════════════════════════════
constexpr int kTcMaxItems = 64;  // items per CTA (the host sizes the grid)

struct TcItem {
  int kvh, qb, chunk, first, rows, L, page_begin, page_end, off0, pad;
};

template <int D, int STAGES>
struct TcCfg {
  static constexpr int kThreads = 384;
  static constexpr int kRows = 128;
  static constexpr int kBlkPages = 4;
  static constexpr int kBlkTok = 64;
  static constexpr int kBoxes = D / 64;                 // 64-element blocks of d
  static constexpr int kRegion = kBlkPages * 2048;      // one d-block of a block's K (or V)
  static constexpr int kKV = kBoxes * kRegion;
  static constexpr int kStage = 2 * kKV;
  static constexpr int kQ = kBoxes * kRows * 128;       // Q: [d-block][128 rows x 128 B]
  static constexpr int kP = kRows * 128;                // P hi (or lo): 128 rows x 64 tokens
  static constexpr int kPBuf = 2 * kP;
  static constexpr int kORow = D * 4;                   // O staging row (chunks XOR-swizzled)
  static constexpr int kOffStage = kQ;
  static constexpr int kOffP = kQ + STAGES * kStage;
  static constexpr int kOffBar = kOffP + 2 * kPBuf;
  static constexpr int kNumBars = 2 * STAGES + 10;
  static constexpr int kOffTmem = kOffBar + kNumBars * 8;
  static constexpr int kOffMeta = kOffTmem + 16;        // per stage: valid-page mask, token limit
  // row exchange between a quadrant's two warps: block maxima [2 buffers][2
  // halves][128 rows], then the item's l [2 halves][128 rows]
  static constexpr int kOffX = kOffMeta + STAGES * 8;
  static constexpr int kOffItems = kOffX + 6 * kRows * 4;
  static constexpr int kSmem = 1024 + kOffItems + kTcMaxItems * (int)sizeof(TcItem) + 16;
  static constexpr int kColO = 2 * kBlkTok;             // S buffers at columns [0, 128)
  static constexpr int kTmemCols = 256;
  static_assert(kColO + D <= kTmemCols, "TMEM columns");
  static_assert(kRows * kORow <= 2 * kPBuf, "O staging fits in the P buffers");
};

// Exact split of p (|p| <= 2^8) into fp16 hi + lo: hi keeps p's sign,
// exponent and top 10 mantissa bits (exact in fp16 for normal values), lo
// is the rest (exact in fp32, rounded once to fp16).
__device__ __forceinline__ void split_hi_lo(float a, float b, uint32_t& hi, uint32_t& lo) {
  const float ah = __uint_as_float(__float_as_uint(a) & 0xFFFFE000u);
  const float bh = __uint_as_float(__float_as_uint(b) & 0xFFFFE000u);
  hi = pack_half2(ah, bh);
  lo = pack_half2(a - ah, b - bh);
}

template <int D, int STAGES>
__global__ void __launch_bounds__(384, 1)
    pa_prefix_tc_kernel(const __grid_constant__ CUtensorMap tmK,
                        const __grid_constant__ CUtensorMap tmV, const Params p,
                        const PrefixGroups pg) {
  using C = TcCfg<D, STAGES>;
  pdl_launch_dependents();  // the suffix kernel runs beside this one
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    tmap_prefetch(&tmK);
    tmap_prefetch(&tmV);
  }
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const uint32_t sb = smem_u32(smem);
  const uint32_t sQ = sb, sStage = sb + C::kOffStage, sP = sb + C::kOffP;
  const uint32_t bars = sb + C::kOffBar;
  const uint32_t bar_full = bars, bar_empty = bars + 8 * STAGES;
  const uint32_t bar_sfull = bars + 16 * STAGES, bar_sfree = bar_sfull + 16;
  const uint32_t bar_pfull = bar_sfree + 16, bar_pv = bar_pfull + 16;
  const uint32_t bar_done = bar_pv + 16, bar_q = bar_done + 8;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::kOffTmem);
  int* s_meta = reinterpret_cast<int*>(smem + C::kOffMeta);
  float* s_x = reinterpret_cast<float*>(smem + C::kOffX);
  TcItem* s_items = reinterpret_cast<TcItem*>(smem + C::kOffItems);
  int* s_nitems = reinterpret_cast<int*>(smem + C::kOffItems + kTcMaxItems * sizeof(TcItem));

  if (threadIdx.x == 0) {
#pragma unroll
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(bar_full + 8 * s, 2);  // the K and the V producer
      mbar_init(bar_empty + 8 * s, 1);
    }
#pragma unroll
    for (int b = 0; b < 2; ++b) {
      mbar_init(bar_sfull + 8 * b, 1);
      mbar_init(bar_sfree + 8 * b, 8);  // one arrival per softmax warp
      mbar_init(bar_pfull + 8 * b, 8);
      mbar_init(bar_pv + 8 * b, 1);
    }
    mbar_init(bar_done, 1);
    mbar_init(bar_q, 8);  // an item's Q tile: one arrival per softmax warp
    fence_mbar_init();
  }
  if (warp == 1) {
    tc::tmem_alloc(smem_u32(tmem_slot), C::kTmemCols);
    tc::tmem_relinquish();
  }
  if (warp == 3) {
    // this CTA's items; an empty one keeps page_begin == page_end
    const long long total = (long long)pg.num_groups * p.Hkv * pg.max_qblocks * pg.max_chunks;
    const long long mine = total > blockIdx.x ? (total - blockIdx.x + gridDim.x - 1) / gridDim.x : 0;
    const int n = (int)(mine < kTcMaxItems ? mine : kTcMaxItems);
    for (int k = lane; k < n; k += 32) {
      PrefixItem it;
      TcItem ti{};
      if (decode_prefix_item(p, pg, (int)(blockIdx.x + (long long)k * gridDim.x), it)) {
        ti.kvh = it.kvh;
        ti.qb = it.qb;
        ti.chunk = it.chunk;
        ti.first = it.first;
        ti.rows = it.rows;
        ti.L = it.L;
        ti.page_begin = it.page_begin;
        ti.page_end = it.page_end;
        ti.off0 = __ldg(pg.offsets + it.g);
      }
      s_items[k] = ti;
    }
    if (lane == 0) *s_nitems = n;
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = *tmem_slot;
  const uint64_t budget = p.timeout_ns;
  const int nitems = *s_nitems;

  if (warp == 0 || warp == 2) {
    // ── producers: K (warp 0) and V (warp 2) of each block's 4 pages into
    // ring slot (block count) % STAGES; the K producer also records the
    // block's valid-page mask and token limit for the softmax
    const bool isv = warp == 2;
    const CUtensorMap* tm = isv ? &tmV : &tmK;
    int jg = 0, issued = 0;
    bool ok = true;
    for (int k = 0; ok && k < nitems; ++k) {
      const TcItem ti = s_items[k];
      const int np = ti.page_end - ti.page_begin;
      const int nb = (np + C::kBlkPages - 1) / C::kBlkPages;
      const int* bt_row = p.block_tables + (long long)ti.first * p.max_blocks;
      int ent = -1;
      for (int j = 0; j < nb; ++j) {
        if ((j & 7) == 0) {  // lanes fetch the entries of the next 8 blocks
          const int idx = j * C::kBlkPages + lane;
          ent = -1;
          if (idx < np) {
            ent = __ldg(bt_row + ti.page_begin + idx);
            if (ent < 0 || (p.num_blocks > 0 && ent >= p.num_blocks)) {
              if (!isv) raise_status(p, kDevBadPage);
              ent = -1;
            }
          }
        }
        int phys[C::kBlkPages];
#pragma unroll
        for (int pi = 0; pi < C::kBlkPages; ++pi)
          phys[pi] = __shfl_sync(0xffffffffu, ent, (j & 7) * C::kBlkPages + pi);
        const int jj = jg + j, s = jj % STAGES;
        if (lane == 0) {
          if (jj >= STAGES && !mbar_wait(bar_empty + 8 * s, ((jj / STAGES) + 1) & 1, budget)) {
            raise_status(p, kDevTimeout);
            ok = false;
          } else {
            if (!isv) {
              int vmask = 0;
#pragma unroll
              for (int pi = 0; pi < C::kBlkPages; ++pi) vmask |= (phys[pi] >= 0 ? 1 : 0) << pi;
              s_meta[2 * s] = vmask;
              s_meta[2 * s + 1] = ti.L - (ti.page_begin + j * C::kBlkPages) * 16;
            }
            const uint32_t full = bar_full + 8 * s;
            mbar_arrive_expect_tx(full, C::kKV);
            const uint32_t dst = sStage + s * C::kStage + (isv ? C::kKV : 0);
            // pages past the chunk and invalid entries read as zeros (the
            // box lies wholly outside the pool); the softmax masks them
#pragma unroll
            for (int pi = 0; pi < C::kBlkPages; ++pi)
#pragma unroll
              for (int x = 0; x < C::kBoxes; ++x)
                tma_load_4d(dst + x * C::kRegion + pi * 2048, tm, x * 64, 0, ti.kvh, phys[pi],
                            full);
            issued = jj + 1;
          }
        }
        ok = __shfl_sync(0xffffffffu, ok, 0);
        if (!ok) break;
      }
      jg += nb;
    }
    if (!ok && lane == 0) {
      for (int j = issued > STAGES ? issued - STAGES : 0; j < issued; ++j)
        (void)mbar_wait(bar_full + 8 * (j % STAGES), (j / STAGES) & 1, kPrefixDrainNs);
    }
  } else if (warp == 1) {
    // ── MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc_s = tc::idesc_f16_f32(128, C::kBlkTok, false);
      constexpr uint32_t idesc_o = tc::idesc_f16_f32(128, D, true);
      // O (+)= P_i . V_i for global block i; `first` starts the item's O
      auto issue_pv = [&](int i, bool first) -> bool {
        const int s = i % STAGES, b = i & 1;
        if (!mbar_wait(bar_pfull + 8 * b, (i >> 1) & 1, budget)) return false;
        tc::fence_after_sync();
        const uint32_t vst = sStage + s * C::kStage + C::kKV;
        const uint32_t ph = sP + b * C::kPBuf, pl = ph + C::kP;
#pragma unroll
        for (int ks = 0; ks < C::kBlkTok / 16; ++ks) {
          const uint64_t bd = tc::sw128_desc(vst + ks * 2048, C::kRegion, 1024);
          tc::mma_f16_ss(tmem + C::kColO, tc::sw128_desc(ph + ks * 32, 16, 1024), bd, idesc_o,
                         (first && ks == 0) ? 0u : 1u);
          tc::mma_f16_ss(tmem + C::kColO, tc::sw128_desc(pl + ks * 32, 16, 1024), bd, idesc_o,
                         1u);
        }
        tc::commit(bar_empty + 8 * s);
        tc::commit(bar_pv + 8 * b);
        return true;
      };
      int jg = 0, nq = 0;
      bool ok = true;
      for (int k = 0; ok && k < nitems; ++k) {
        const TcItem ti = s_items[k];
        const int np = ti.page_end - ti.page_begin;
        if (np <= 0) continue;
        const int nb = (np + C::kBlkPages - 1) / C::kBlkPages;
        ok = mbar_wait(bar_q, nq & 1, budget);  // this item's Q tile
        ++nq;
        for (int j = 0; ok && j < nb; ++j) {
          const int jj = jg + j, s = jj % STAGES, b = jj & 1;
          if (!mbar_wait(bar_full + 8 * s, (jj / STAGES) & 1, budget) ||
              (jj >= 2 && !mbar_wait(bar_sfree + 8 * b, ((jj >> 1) - 1) & 1, budget))) {
            ok = false;
            break;
          }
          tc::fence_after_sync();
          const uint32_t kst = sStage + s * C::kStage;
#pragma unroll
          for (int ks = 0; ks < D / 16; ++ks) {
            const int x = ks >> 2, kk = ks & 3;
            tc::mma_f16_ss(tmem + b * C::kBlkTok,
                           tc::sw128_desc(sQ + x * (C::kRows * 128) + kk * 32, 16, 1024),
                           tc::sw128_desc(kst + x * C::kRegion + kk * 32, 16, 1024), idesc_s,
                           ks > 0 ? 1u : 0u);
          }
          tc::commit(bar_sfull + 8 * b);
          if (j >= 1 && !issue_pv(jj - 1, j == 1)) ok = false;
        }
        if (ok) ok = issue_pv(jg + nb - 1, nb == 1);
        jg += nb;
      }
      if (!ok) raise_status(p, kDevTimeout);
      tc::commit(bar_done);  // arrives once every MMA above has completed
      (void)mbar_wait(bar_done, 0, kPrefixDrainNs);
    }
    __syncwarp();
  } else if (warp >= 4) {
    // ── softmax: row r (TMEM lane r) = (member r / GS, head r % GS) of the
    // item's KV head; half h takes tokens [32h, 32h + 32) of each block.
    constexpr int kHalf = D / 16;  // 16-byte Q chunks per half row
    const int q4 = warp & 3, h = (warp - 4) >> 2;
    const int r = q4 * 32 + lane;
    const uint32_t trow = tmem + ((uint32_t)(q4 * 32) << 16);
    const float sl2 = p.scale_log2;
    uint8_t* stage = smem + C::kOffP;  // O staging (the P buffers)
    // Q rows of the next item with work, loaded ahead into registers
    auto next_item = [&](int k) {
      while (k < nitems && s_items[k].page_end <= s_items[k].page_begin) ++k;
      return k;
    };
    uint4 qv[kHalf];
    long long pr_next = -1;
    auto load_q = [&](int k) {
      pr_next = -1;
#pragma unroll
      for (int i = 0; i < kHalf; ++i) qv[i] = make_uint4(0u, 0u, 0u, 0u);
      if (k >= nitems) return;
      const TcItem ti = s_items[k];
      const int grow = ti.qb * C::kRows + r;
      if (grow >= ti.rows) return;
      const int member = __ldg(pg.members + ti.off0 + grow / p.GS);
      const long long qrow = (long long)member * p.Hq + (long long)ti.kvh * p.GS + grow % p.GS;
      pr_next = qrow * p.slots + ti.chunk;
      const uint4* src =
          reinterpret_cast<const uint4*>(static_cast<const __half*>(p.q) + qrow * D) + h * kHalf;
#pragma unroll
      for (int i = 0; i < kHalf; ++i) qv[i] = __ldg(src + i);
    };
    int k = next_item(0);
    load_q(k);
    int jg = 0;
    // The two warps of a quadrant meet at the same named barriers in every
    // case, so a wait that expires in one of them leaves it skipping work,
    // not barriers.
    bool ok = true;
    while (k < nitems) {
      const TcItem ti = s_items[k];
      const int np = ti.page_end - ti.page_begin;
      const int nb = (np + C::kBlkPages - 1) / C::kBlkPages;
      const long long pr = pr_next;
      // Q tile, K-major with 128-byte swizzle (16-byte chunk c of row r at
      // chunk c ^ (r % 8)); the previous item's MMAs have all completed
#pragma unroll
      for (int i = 0; i < kHalf; ++i) {
        const int cg = h * kHalf + i, x = cg >> 3, c = cg & 7;
        const uint32_t dst = sQ + x * (C::kRows * 128) + r * 128 + ((c ^ (r & 7)) << 4);
        asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(dst), "r"(qv[i].x),
                     "r"(qv[i].y), "r"(qv[i].z), "r"(qv[i].w)
                     : "memory");
      }
      fence_proxy_async_smem();  // Q's generic stores before the tensor cores read them
      __syncwarp();
      if (lane == 0) mbar_arrive(bar_q);
      const int k_next = next_item(k + 1);
      load_q(k_next);  // in flight during this item

      float m_used = -INFINITY, l = 0.f;
      for (int j = 0; j < nb; ++j) {
        const int jj = jg + j, b = jj & 1, s = jj % STAGES;
        if (ok) ok = __all_sync(0xffffffffu, mbar_wait(bar_sfull + 8 * b, (jj >> 1) & 1, budget));
        // the block's page mask and token limit (full(s) completed before
        // S did, so this wait only orders the producer's record)
        if (ok) ok = __all_sync(0xffffffffu, mbar_wait(bar_full + 8 * s, (jj / STAGES) & 1, budget));
        uint32_t sr[32];
        int vmask = 0, lim = 0;
        if (ok) {
          vmask = s_meta[2 * s];
          lim = s_meta[2 * s + 1] - 32 * h;
          tc::fence_after_sync();
          tc::tmem_ld32(trow + b * C::kBlkTok + 32 * h, sr);
          tc::tmem_wait_ld();
          tc::fence_before_sync();
          __syncwarp();
          if (lane == 0) mbar_arrive(bar_sfree + 8 * b);
        } else {
#pragma unroll
          for (int t = 0; t < 32; ++t) sr[t] = 0u;
        }
        const bool v0 = (vmask >> (2 * h)) & 1, v1 = (vmask >> (2 * h + 1)) & 1;
        // A block whose 32 tokens of this half are all valid (the usual
        // case inside a prefix) keeps its raw scores: no masking selects,
        // the scale applied once to the maximum (a positive scale keeps the
        // order) and folded into one FFMA before each ex2 below. The flag is
        // the same for the whole warp.
        const bool raw = v0 && v1 && lim >= 32 && sl2 > 0.f;
        float sv[32];
        if (raw) {
#pragma unroll
          for (int t = 0; t < 32; ++t) sv[t] = __uint_as_float(sr[t]);
        } else {
#pragma unroll
          for (int t = 0; t < 32; ++t) {
            const bool valid = (t < 16 ? v0 : v1) && t < lim;
            sv[t] = valid ? __uint_as_float(sr[t]) * sl2 : -INFINITY;
          }
        }
        float mx4[4];
#pragma unroll
        for (int q = 0; q < 4; ++q)
          mx4[q] = fmaxf(fmaxf(fmaxf(sv[q], sv[q + 4]), fmaxf(sv[q + 8], sv[q + 12])),
                         fmaxf(fmaxf(sv[q + 16], sv[q + 20]), fmaxf(sv[q + 24], sv[q + 28])));
        float mx = fmaxf(fmaxf(mx4[0], mx4[1]), fmaxf(mx4[2], mx4[3]));
        if (raw) mx *= sl2;
        // combine with the other half of the row
        s_x[(b * 2 + h) * C::kRows + r] = mx;
        named_bar_sync(1 + q4, 64);
        mx = fmaxf(mx, s_x[(b * 2 + (h ^ 1)) * C::kRows + r]);
        if (!ok) continue;
        const bool raise = mx > m_used + 8.f;
        const float alpha = raise ? ex2(m_used - mx) : 1.f;
        if (raise) {
          l *= alpha;
          m_used = mx;
        }
        if (__any_sync(0xffffffffu, raise) && j > 0) {
          // rescale this half's O columns once PV of block jj-1 has completed
          ok = __all_sync(0xffffffffu,
                          mbar_wait(bar_pv + 8 * ((jj - 1) & 1), ((jj - 1) >> 1) & 1, budget));
          if (!ok) continue;
          tc::fence_after_sync();
#pragma unroll 1
          for (int c0 = h * (D / 2); c0 < (h + 1) * (D / 2); c0 += 32) {
            uint32_t o[32];
            tc::tmem_ld32(trow + C::kColO + c0, o);
            tc::tmem_wait_ld();
#pragma unroll
            for (int q = 0; q < 32; ++q) o[q] = __float_as_uint(__uint_as_float(o[q]) * alpha);
            tc::tmem_st32(trow + C::kColO + c0, o);
          }
          tc::tmem_wait_st();
        }
        // P buffer b was last read by PV of block jj-2 (or the staging of a
        // previous item's O, finished before that item ended)
        if (jj >= 2) {
          ok = __all_sync(0xffffffffu, mbar_wait(bar_pv + 8 * b, ((jj - 2) >> 1) & 1, budget));
          if (!ok) continue;
        }
        const float mu = m_used == -INFINITY ? 0.f : m_used;  // all masked so far: P = 0
        // raw scores: 2^(s * scale_log2 - mu) as one FFMA + ex2
        const float ka = raw ? sl2 : 1.f;
        const uint32_t ph = sP + b * C::kPBuf + r * 128, pl = ph + C::kP;
        float ls[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint32_t hi[4], lo[4];
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const int t = c * 8 + 2 * q;
            const float p0 = ex2(fmaf(sv[t], ka, -mu)), p1 = ex2(fmaf(sv[t + 1], ka, -mu));
            ls[q] += p0 + p1;
            split_hi_lo(p0, p1, hi[q], lo[q]);
          }
          const uint32_t off = (uint32_t)(((4 * h + c) ^ (r & 7)) << 4);
          asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(ph + off), "r"(hi[0]),
                       "r"(hi[1]), "r"(hi[2]), "r"(hi[3])
                       : "memory");
          asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(pl + off), "r"(lo[0]),
                       "r"(lo[1]), "r"(lo[2]), "r"(lo[3])
                       : "memory");
        }
        l += (ls[0] + ls[1]) + (ls[2] + ls[3]);
        fence_proxy_async_smem();  // P's generic stores before the tensor cores read them
        tc::fence_before_sync();
        __syncwarp();
        if (lane == 0) mbar_arrive(bar_pfull + 8 * b);
      }
      const int jl = jg + nb - 1;  // the item's last block
      if (ok)
        ok = __all_sync(0xffffffffu, mbar_wait(bar_pv + 8 * (jl & 1), (jl >> 1) & 1, budget));
      // ── the item's partial (m, l, o)
      s_x[(4 + h) * C::kRows + r] = l;  // the row's l is the sum of its halves'
      named_bar_sync(1 + q4, 64);
      const float ltot = l + s_x[(4 + (h ^ 1)) * C::kRows + r];
      // every P buffer read has completed (PV of the last two blocks): stage
      // O row r (16-byte chunk c at chunk c ^ (r % 8)) there
      named_bar_sync(5, 256);
      if (ok) {
        tc::fence_after_sync();
#pragma unroll 1
        for (int c0 = h * (D / 2); c0 < (h + 1) * (D / 2); c0 += 32) {
          uint32_t o[32];
          tc::tmem_ld32(trow + C::kColO + c0, o);
          tc::tmem_wait_ld();
#pragma unroll
          for (int q = 0; q < 32; q += 4) {
            const int c = (c0 + q) >> 2;
            *reinterpret_cast<uint4*>(stage + r * C::kORow + ((c ^ (r & 7)) << 4)) =
                make_uint4(o[q], o[q + 1], o[q + 2], o[q + 3]);
          }
        }
        tc::fence_before_sync();
      }
      named_bar_sync(1 + q4, 64);  // both halves of the quadrant's rows staged
      // this warp writes 16 of the quadrant's 32 rows
      for (int rr = 16 * h; rr < 16 * h + 16; ++rr) {
        const long long prr = __shfl_sync(0xffffffffu, pr, rr);
        if (prr < 0) continue;
        const int row = q4 * 32 + rr;
        const uint8_t* srow = stage + row * C::kORow;
        float* dst = p.part_o + prr * D;
        for (int c = lane; c < D / 4; c += 32) {
          uint4 v = *reinterpret_cast<const uint4*>(srow + ((c ^ (row & 7)) << 4));
          if (!ok) v = make_uint4(0u, 0u, 0u, 0u);
          if (p.vec8) {
            *reinterpret_cast<uint4*>(dst + 4 * c) = v;
          } else {
            dst[4 * c] = __uint_as_float(v.x);
            dst[4 * c + 1] = __uint_as_float(v.y);
            dst[4 * c + 2] = __uint_as_float(v.z);
            dst[4 * c + 3] = __uint_as_float(v.w);
          }
        }
      }
      if (h == 0 && pr >= 0) {
        const bool valid = ok && m_used != -INFINITY;
        p.part_ml[2 * pr] = valid ? m_used : -INFINITY;
        p.part_ml[2 * pr + 1] = valid ? ltot : 0.f;
      }
      named_bar_sync(5, 256);  // staging read out before the P buffers are reused
      jg += nb;
      k = k_next;
    }
    if (!ok) raise_status(p, kDevTimeout);
  }
  // ── teardown: every role has drained its copies and MMAs
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 1) {
    tc::fence_after_sync();
    tc::tmem_dealloc(tmem, C::kTmemCols);
  }
}

}  // namespace

bool prefix_tc_ok(const Params& p) {
  return (p.D == 64 || p.D == 128) && (reinterpret_cast<uintptr_t>(p.q) & 15u) == 0 &&
         p.prefix_chunk <= kMaxPrefixChunk;
}

cudaError_t launch_prefix(const CUtensorMap& tk, const CUtensorMap& tv, const Params& p,
                          const PrefixGroups& pg_in, int max_ctas, cudaStream_t st) {
  constexpr int STAGES = 4;
  const bool tc = prefix_tc_ok(p);
  PrefixGroups pg = pg_in;
  pg.rows = tc ? 128 : 64;
  pg.max_qblocks = (int)(((long long)pg.max_group_size * p.GS + pg.rows - 1) / pg.rows);
  const long long items = (long long)pg.num_groups * p.Hkv * pg.max_qblocks * pg.max_chunks;
  if (items <= 0) return cudaSuccess;
  if (items > INT_MAX) return cudaErrorInvalidValue;
  auto run = [&](auto kern, int smem, int threads, long long grid) -> cudaError_t {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    kern<<<(unsigned)grid, threads, smem, st>>>(tk, tv, p, pg);
    return cudaGetLastError();
  };
  if (tc) {
    // persistent: at most max_ctas CTAs (one per SM), each with at most
    // kTcMaxItems items
    long long grid = items < max_ctas ? items : max_ctas;
    const long long need = (items + kTcMaxItems - 1) / kTcMaxItems;
    if (grid < need) grid = need;
    if (p.D == 64)
      return run(pa_prefix_tc_kernel<64, 3>, TcCfg<64, 3>::kSmem, TcCfg<64, 3>::kThreads, grid);
    return run(pa_prefix_tc_kernel<128, 3>, TcCfg<128, 3>::kSmem, TcCfg<128, 3>::kThreads, grid);
  }
  switch (p.D) {
    case 64: return run(pa_prefix_kernel<64, STAGES>, PrefixCfg<64, STAGES>::kSmem, 160, items);
    case 128: return run(pa_prefix_kernel<128, STAGES>, PrefixCfg<128, STAGES>::kSmem, 160, items);
    case 256: return run(pa_prefix_kernel<256, 2>, PrefixCfg<256, 2>::kSmem, 160, items);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace xpa
