// pa_kernels.cu — paged decode attention kernels for sm_100a.
//
// Work decomposition (all kernels): one CTA per item = (sequence b, KV head
// kvh, context partition part). A partition is `part_pages` consecutive pages
// of the sequence's block-table row. A sequence that fits in one partition is
// finished in place (normalised output written directly); longer ones write
// per-partition partials (running max m, sum l, unnormalised o) that
// pa_reduce_kernel merges by log-sum-exp, launched as a programmatic
// dependent of the attention kernel so its launch overlaps that kernel's tail.
// Scores are kept in the exp2 domain (scale * log2 e folded into the score),
// which is the same softmax.
//
// Reference semantics followed: GQA mapping kv = h / (Hq/Hkv)
// (examples/text_gen.c:1285), max-subtracted softmax and o = sum w*v
// (examples/text_gen.c:1288-1309), paged indexing
// phys*kv_block_stride + kvh*kv_head_stride + slot*D + d
// (operators/page_attention_v2.cu:143-146), zero row for seq_len 0
// (operators/page_attention.cu:157).
#include <utility>

#include "pa_device.cuh"
#include "pa_launch.h"

namespace xpa {

// ════════════════════════════════════════════════════════════════════════
// Generic path: CUDA cores, any head size <= 256, fp16 or fp32, any page size.
// Each of the 4 warps walks every 4th token of the item; lanes split the head
// dimension (DPL dims per lane) and each token's K row is used for HG query
// heads of the group at once, so K/V are read once per HG heads.
// ════════════════════════════════════════════════════════════════════════
// K/V element idx of a pool: T, or a one-byte code (KVF = kKvE4M3 / kKvE5M2 /
// kKvInt8).
template <typename T, int KVF>
__device__ __forceinline__ float kv_load(const void* base, long long idx) {
  if constexpr (KVF == 0)
    return to_float(static_cast<const T*>(base)[idx]);
  else
    return fp8_to_float<KVF>(static_cast<const uint8_t*>(base)[idx]);
}

template <typename T, int DPL, int HG, int KVF>
__global__ void __launch_bounds__(128) pa_generic_kernel(const Params p) {
  constexpr int NW = 4;
  constexpr int DMAX = DPL * 32;
  __shared__ float sm_o[NW][HG][DMAX + 1];
  __shared__ float sm_m[NW][HG];
  __shared__ float sm_l[NW][HG];

  pdl_launch_dependents();
  if (p.wait_first) pdl_wait_primary();
  Item it;
  const ItemKind kind = decode_item(p, blockIdx.x, it);
  if (kind == kItemNone) return;
  const int D = p.D, GS = p.GS;
  if (kind == kItemZero) {
    const long long row0 = (long long)it.b * p.Hq + (long long)it.kvh * GS;
    for (int e = threadIdx.x; e < GS * D; e += blockDim.x) store_out<T>(p, row0 + e / D, e % D, 0.f);
    return;
  }

  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  if (p.after_append) pdl_wait_primary();  // appended tokens are read like any other
  const T* Q = static_cast<const T*>(p.q);
  const float vs = KVF ? p.v_scale : 1.f;  // k_scale is in scale_log2
  const int* bt_row = p.block_tables + (long long)it.b * p.max_blocks;
  const int t_begin = it.page_begin * p.block_size;
  const int t_end = min(it.L, it.page_end * p.block_size);

  for (int hg0 = 0; hg0 < GS; hg0 += HG) {
    const int nh = min(HG, GS - hg0);
    float q[HG][DPL], o[HG][DPL], m[HG], l[HG];
#pragma unroll
    for (int j = 0; j < HG; ++j) {
      const long long qrow = ((long long)it.b * p.Hq + (long long)it.kvh * GS + hg0 + j) * D;
#pragma unroll
      for (int i = 0; i < DPL; ++i) {
        const int d = lane + 32 * i;
        q[j][i] = (j < nh && d < D) ? to_float(Q[qrow + d]) : 0.f;
        o[j][i] = 0.f;
      }
      m[j] = -INFINITY;
      l[j] = 0.f;
    }

    // Tokens w, w + NW, ... of the item, U at a time: the K / V loads of U
    // tokens are in flight together and their U dot products reduce in
    // independent butterflies, instead of one HBM round trip per token.
    constexpr int U = DPL <= 4 ? 4 : 2;
    for (int t0 = t_begin + w; t0 < t_end; t0 += NW * U) {
      float kf[U][DPL], vf[U][DPL];
      bool ok[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int t = t0 + u * NW;
        ok[u] = false;
        if (t < t_end) {
          const int phys = __ldg(bt_row + t / p.block_size);
          if (phys < 0 || (p.num_blocks > 0 && phys >= p.num_blocks)) {
            if (lane == 0 && hg0 == 0) raise_status(p, kDevBadPage);
          } else {
            ok[u] = true;
          }
          const long long base = (long long)(ok[u] ? phys : 0) * p.kv_block_stride +
                                 (long long)it.kvh * p.kv_head_stride +
                                 (long long)(t % p.block_size) * D;
#pragma unroll
          for (int i = 0; i < DPL; ++i) {
            const int d = lane + 32 * i;
            kf[u][i] = (ok[u] && d < D) ? kv_load<T, KVF>(p.k, base + d) : 0.f;
            vf[u][i] = (ok[u] && d < D) ? kv_load<T, KVF>(p.v, base + d) * vs : 0.f;
          }
        } else {
#pragma unroll
          for (int i = 0; i < DPL; ++i) kf[u][i] = vf[u][i] = 0.f;
        }
      }
#pragma unroll
      for (int j = 0; j < HG; ++j) {
        float dot[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
          dot[u] = 0.f;
#pragma unroll
          for (int i = 0; i < DPL; ++i) dot[u] = fmaf(q[j][i], kf[u][i], dot[u]);
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1)
#pragma unroll
          for (int u = 0; u < U; ++u) dot[u] += __shfl_xor_sync(0xffffffffu, dot[u], off);
#pragma unroll
        for (int u = 0; u < U; ++u) {
          if (!ok[u]) continue;  // the same for every lane
          const float sv = dot[u] * p.scale_log2;
          const float mn = fmaxf(m[j], sv);
          const float alpha = ex2(m[j] - mn);
          const float pj = ex2(sv - mn);
          l[j] = fmaf(l[j], alpha, pj);
#pragma unroll
          for (int i = 0; i < DPL; ++i) o[j][i] = fmaf(o[j][i], alpha, pj * vf[u][i]);
          m[j] = mn;
        }
      }
    }

#pragma unroll
    for (int j = 0; j < HG; ++j) {
#pragma unroll
      for (int i = 0; i < DPL; ++i) sm_o[w][j][lane + 32 * i] = o[j][i];
      if (lane == 0) {
        sm_m[w][j] = m[j];
        sm_l[w][j] = l[j];
      }
    }
    __syncthreads();

    for (int e = threadIdx.x; e < nh * D; e += blockDim.x) {
      const int j = e / D, d = e - j * D;
      float M = -INFINITY;
#pragma unroll
      for (int ww = 0; ww < NW; ++ww) M = fmaxf(M, sm_m[ww][j]);
      float num = 0.f, den = 0.f;
      if (M != -INFINITY) {
#pragma unroll
        for (int ww = 0; ww < NW; ++ww) {
          const float wt = ex2(sm_m[ww][j] - M);
          den = fmaf(wt, sm_l[ww][j], den);
          num = fmaf(wt, sm_o[ww][j][d], num);
        }
      }
      const long long row = (long long)it.b * p.Hq + (long long)it.kvh * GS + hg0 + j;
      if (it.direct) {
        store_out<T>(p, row, d, den > 0.f ? num / den : 0.f);
      } else {
        const long long pr = row * p.slots + it.slot0 + it.part;
        p.part_o[pr * D + d] = num;
        if (d == 0) {
          p.part_ml[2 * pr] = M;
          p.part_ml[2 * pr + 1] = den;
        }
      }
    }
    __syncthreads();
  }
}

// ════════════════════════════════════════════════════════════════════════
// Fast path: fp16, page size 16, head size D in {64, 128, 256}.
//
// Warp specialisation: warp NWC is the producer; one lane streams the
// item's pages through a STAGES-deep ring with TMA (one 16 x 64 box per 64
// dims of K and of V, 128-byte swizzle, completion on the stage's mbarrier).
// Warps 0..NWC-1 consume pages round-robin. Per page a consumer computes
//   S^T (16 tokens x 8 heads) = K_page (16 x D) . Q^T (D x 8)      [mma.sync]
// runs the online softmax on the fragments, transposes P with movmatrix and
//   O^T (D x 8 heads) += V_page^T (D x 16) . P^T (16 x 8)           [mma.sync]
// with P split as fp16 hi + lo so the PV product carries fp32-level accuracy.
// Each page of a KV head is read from HBM exactly once for all GS query heads.
// ════════════════════════════════════════════════════════════════════════

// Bound on the producer's wait for its own in-flight copies after a timeout.
constexpr uint64_t kDrainBudgetNs = 1000000000ull;

// One-byte pages: PV reads V's A fragments from registers loaded straight
// from the ring stage (transposed 16-bit ldmatrix over the byte rows) before
// the softmax, so the stage goes back to its producer at once and no fp16 V
// tile is needed. 0 widens V into a per-warp fp16 tile instead (measured
// slower on B200); a build may choose either for tuning sweeps.
#ifndef XPA_KV8_DIRECT_V
#define XPA_KV8_DIRECT_V 1
#endif

template <int D, int NT, int STAGES, int NWC, int KVF>
struct FastCfg {
  static constexpr int kElem = KVF ? 1 : 2;      // bytes per K / V element
  static constexpr int kTile = 16 * D * kElem;   // bytes of one K (or V) page
  static constexpr int kStage = 2 * kTile;       // K + V
  static constexpr int kKSteps = D / 16;
  static constexpr int kBoxes = D * kElem / 128; // 128-byte-wide TMA boxes per row
  static constexpr int kBoxElems = 128 / kElem;
  static constexpr int kRing = STAGES * kStage;
  static constexpr bool kDirectV = KVF != 0 && XPA_KV8_DIRECT_V;
  // one-byte caches without direct V: each consumer warp widens its V page
  // to an fp16 tile here
  static constexpr int kV16 = (KVF && !kDirectV) ? NWC * 16 * D * 2 : 0;
  static constexpr int kMerge = NWC * NT * 8 * (D + 4) * 4 + NWC * NT * 8 * 8;
  static constexpr int kBarOff = kRing + kV16 > kMerge ? kRing + kV16 : kMerge;
  static constexpr int kSmem = 1024 + kBarOff + STAGES * 16 + STAGES * 4;
  static constexpr int kThreads = (NWC + 1) * 32;
};

template <int D, int NT, int STAGES, int NWC, int KVF>
__device__ __forceinline__ void tma_mma_body(const CUtensorMap& tmK, const CUtensorMap& tmV,
                                             const Params& p) {
  using C = FastCfg<D, NT, STAGES, NWC, KVF>;
  // Page j goes to stage j % STAGES and to consumer warp j % NWC. The parity
  // waits below are only sound when every stage always belongs to the same
  // warp: otherwise a warp could test a stage one phase early, see the parity
  // of the previous (completed) phase and arrive on the barrier out of turn.
  static_assert(STAGES % NWC == 0, "ring stages must be a multiple of the consumer warps");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  int* meta = reinterpret_cast<int*>(smem + C::kBarOff + STAGES * 16);

  pdl_launch_dependents();
  if (p.wait_first) pdl_wait_primary();
  Item it;
  const ItemKind kind = decode_item(p, blockIdx.x, it);
  if (kind == kItemNone) return;
  const int GS = p.GS;
  if (kind == kItemZero) {
    const long long row0 = (long long)it.b * p.Hq + (long long)it.kvh * GS;
    for (int e = threadIdx.x; e < GS * D; e += blockDim.x)
      store_out<__half>(p, row0 + e / D, e % D, 0.f);
    return;
  }

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t sbase = smem_u32(smem);
  const uint32_t bar_full = smem_u32(smem + C::kBarOff);
  const uint32_t bar_empty = bar_full + 8 * STAGES;
  if (threadIdx.x == 0) {
#pragma unroll
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(bar_full + 8 * s, 1);
      mbar_init(bar_empty + 8 * s, 1);
    }
    fence_mbar_init();
  }
  __syncthreads();

  const int np = it.page_end - it.page_begin;
  const uint64_t budget = p.timeout_ns;

  if (warp == NWC) {
    // ── producers: lane k < NWC feeds consumer warp k, i.e. the pages
    // j = k, k + NWC, ... and their ring stages (STAGES % NWC == 0 gives each
    // stage one owner), so a consumer that frees its stages late holds up
    // only its own next page.
    if (lane == 0) {
      tmap_prefetch(&tmK);
      tmap_prefetch(&tmV);
    }
    if (lane < NWC) {
      const int* bt_row = p.block_tables + (long long)it.b * p.max_blocks;
      bool ok = true;
      int last = -1;  // this lane's last issued page
      const int last_page = (it.L + 15) / 16 - 1;  // holds an appended token
      for (int j0 = lane; ok && j0 < np; j0 += 8 * NWC) {
        int ent[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          const int jj = j0 + u * NWC;
          ent[u] = jj < np ? __ldg(bt_row + it.page_begin + jj) : -1;
        }
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          const int jj = j0 + u * NWC;
          if (jj >= np) break;
          const int s = jj % STAGES;
          const int phys = ent[u];
          // Only the page an append kernel wrote into must wait for that kernel.
          if (p.after_append && it.page_begin + jj == last_page) pdl_wait_primary();
          if (jj >= STAGES && !mbar_wait(bar_empty + 8 * s, ((jj / STAGES) + 1) & 1, budget)) {
            raise_status(p, kDevTimeout);
            ok = false;
            break;
          }
          const bool valid = phys >= 0 && (p.num_blocks <= 0 || phys < p.num_blocks);
          meta[s] = valid ? 1 : 0;
          if (valid) {
            const uint32_t full = bar_full + 8 * s;
            mbar_arrive_expect_tx(full, C::kStage);
            const uint32_t tk = sbase + s * C::kStage, tv = tk + C::kTile;
#pragma unroll
            for (int x = 0; x < C::kBoxes; ++x) {
              tma_load_4d(tk + x * 2048, &tmK, x * C::kBoxElems, 0, it.kvh, phys, full);
              tma_load_4d(tv + x * 2048, &tmV, x * C::kBoxElems, 0, it.kvh, phys, full);
            }
          } else {
            raise_status(p, kDevBadPage);
            mbar_arrive(bar_full + 8 * s);
          }
          last = jj;
        }
      }
      if (!ok) {
        // Let this lane's copies in flight land before the CTA can retire.
        // The drain has its own bound, independent of the pipeline budget.
        for (int jj = last; jj >= 0 && jj > last - STAGES; jj -= NWC)
          (void)mbar_wait(bar_full + 8 * (jj % STAGES), (jj / STAGES) & 1, kDrainBudgetNs);
      }
    }
    return;
  }

  // ── consumers ──────────────────────────────────────────────────────
  const int g = lane >> 2, c = lane & 3;
  const __half* qrow =
      static_cast<const __half*>(p.q) + ((long long)it.b * p.Hq + (long long)it.kvh * GS) * D;
  // Q^T as the B operand (k = d, n = head): lane (g, c) holds
  // Q[head g][16ks + 2c, +1] and Q[head g][16ks + 8 + 2c, +1]. With an fp8
  // cache the k index of a step is permuted, the same way for K and Q, so
  // that lane c's four K elements are four consecutive bytes: k (2c, 2c+1,
  // 2c+8, 2c+9) <-> d 16ks + 4c + (0, 1, 2, 3).
  uint32_t qf[NT][C::kKSteps][2];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    const int head = nt * 8 + g;
#pragma unroll
    for (int ks = 0; ks < C::kKSteps; ++ks) {
      if (head < GS && KVF) {
        const uint2 q4 =
            __ldg(reinterpret_cast<const uint2*>(qrow + head * D + ks * 16 + 4 * c));
        qf[nt][ks][0] = q4.x;
        qf[nt][ks][1] = q4.y;
      } else if (head < GS) {
        const __half* qp = qrow + head * D + ks * 16 + 2 * c;
        qf[nt][ks][0] = __ldg(reinterpret_cast<const unsigned int*>(qp));
        qf[nt][ks][1] = __ldg(reinterpret_cast<const unsigned int*>(qp + 8));
      } else {
        qf[nt][ks][0] = 0u;
        qf[nt][ks][1] = 0u;
      }
    }
  }

  float o[NT][C::kKSteps][4];
  float mrun[NT][2], lrun[NT][2];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
    for (int mt = 0; mt < C::kKSteps; ++mt)
#pragma unroll
      for (int r = 0; r < 4; ++r) o[nt][mt][r] = 0.f;
    mrun[nt][0] = mrun[nt][1] = -INFINITY;
    lrun[nt][0] = lrun[nt][1] = 0.f;
  }

  const float sl2 = p.scale_log2;
  const int tok_begin = it.page_begin * 16;
  const int mi = lane >> 3, r8 = lane & 7;
  for (int j = warp; j < np; j += NWC) {
    const int s = j % STAGES;
    if (!mbar_wait(bar_full + 8 * s, (j / STAGES) & 1, budget)) {
      raise_status(p, kDevTimeout);
      break;
    }
    if (meta[s]) {
      const uint32_t tk = sbase + s * C::kStage, tv = tk + C::kTile;
      const int ntok = min(16, it.L - (tok_begin + j * 16));

      // S^T = K . Q^T. A operand rows = tokens: matrices (tok 0-7 | 8-15) x
      // (d lo | hi) -> a0..a3.
      float sc[NT][4];
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) sc[nt][0] = sc[nt][1] = sc[nt][2] = sc[nt][3] = 0.f;
      if constexpr (KVF != 0) {
        // fp8 rows of 128 bytes, 16-byte chunk ks % 8 of box ks / 8 (chunk
        // index XOR row % 8); lane (g, c) reads 4 bytes of tokens g, g + 8.
        // All loads first, then two independent accumulation chains.
        uint32_t kw[C::kKSteps][2];
#pragma unroll
        for (int ks = 0; ks < C::kKSteps; ++ks) {
          const uint32_t off = (uint32_t)((ks >> 3) * 2048 + (((ks & 7) ^ g) << 4) + 4 * c);
          asm volatile("ld.shared.u32 %0, [%1];" : "=r"(kw[ks][0]) : "r"(tk + off + g * 128));
          asm volatile("ld.shared.u32 %0, [%1];" : "=r"(kw[ks][1]) : "r"(tk + off + (g + 8) * 128));
        }
        float sc2[NT][4];
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) sc2[nt][0] = sc2[nt][1] = sc2[nt][2] = sc2[nt][3] = 0.f;
#pragma unroll
        for (int ks = 0; ks < C::kKSteps; ++ks) {
          uint32_t a0, a1, a2, a3;
          kv8x4_to_h2x2<KVF>(kw[ks][0], a0, a2);
          kv8x4_to_h2x2<KVF>(kw[ks][1], a1, a3);
#pragma unroll
          for (int nt = 0; nt < NT; ++nt)
            mma_f16_16816((ks & 1) ? sc2[nt] : sc[nt], a0, a1, a2, a3, qf[nt][ks][0],
                          qf[nt][ks][1]);
        }
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
          for (int r = 0; r < 4; ++r) sc[nt][r] += sc2[nt][r];
      } else {
#pragma unroll
        for (int ks = 0; ks < C::kKSteps; ++ks) {
          uint32_t a0, a1, a2, a3;
          ldsm_x4(tk + tile_off(r8 + ((mi & 1) << 3), 2 * ks + (mi >> 1)), a0, a1, a2, a3);
#pragma unroll
          for (int nt = 0; nt < NT; ++nt)
            mma_f16_16816(sc[nt], a0, a1, a2, a3, qf[nt][ks][0], qf[nt][ks][1]);
        }
      }

      // One-byte cache: V's PV fragments come straight from the stage into
      // registers (direct V, the default), or the V page is widened into this
      // warp's fp16 tile (rows >= ntok as zeros) in the layout the fp16 PV
      // loads expect. Either way the ring stage is then free for the producer.
      uint32_t vsrc = tv;
      // direct V: vr[x][h] holds, for d-block x (16 d) and tokens 8h..8h+7,
      // lane (g, c)'s bytes V[8h + 2c][16x + 2g, +1], V[8h + 2c + 1][16x + 2g, +1]
      uint32_t vr[C::kDirectV ? C::kKSteps : 1][2];
      if constexpr (C::kDirectV) {
        const int t = ((mi & 1) << 3) + r8;  // lanes 8q..8q+7: rows of matrix q
#pragma unroll
        for (int x = 0; x < C::kKSteps; x += 2) {
          const int db = x + (mi >> 1);
          ldsm_x4_trans(tv + (db >> 3) * 2048 + t * 128 + (((db & 7) ^ (t & 7)) << 4), vr[x][0],
                        vr[x][1], vr[x + 1][0], vr[x + 1][1]);
        }
        if (ntok < 16) {  // slots past the sequence end: zero bytes (decode to 0)
          const uint32_t m0 = (2 * c < ntok ? 0xffffu : 0u) | (2 * c + 1 < ntok ? 0xffff0000u : 0u);
          const uint32_t m1 =
              (2 * c + 8 < ntok ? 0xffffu : 0u) | (2 * c + 9 < ntok ? 0xffff0000u : 0u);
#pragma unroll
          for (int x = 0; x < C::kKSteps; ++x) {
            vr[x][0] &= m0;
            vr[x][1] &= m1;
          }
        }
        __syncwarp();  // every lane's ring loads precede the release
        if (lane == 0) mbar_arrive(bar_empty + 8 * s);
      } else if constexpr (KVF != 0) {
        vsrc = sbase + C::kRing + warp * (16 * D * 2);
        constexpr int CH8 = D / 16;  // 16-byte fp8 chunks per row
        // lanes of one 8-lane store phase take 8 rows of one chunk column:
        // distinct swizzled 16-byte slots, no bank conflicts. Every load is
        // issued before the first conversion.
        constexpr int ITER = 16 * CH8 / 32;
        uint4 wv[ITER];
#pragma unroll
        for (int i = 0; i < ITER; ++i) {
          const int qi = lane + 32 * i, row = qi & 15, c8 = qi >> 4;
          asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
                       : "=r"(wv[i].x), "=r"(wv[i].y), "=r"(wv[i].z), "=r"(wv[i].w)
                       : "r"(tv + (c8 >> 3) * 2048 + row * 128 + (((c8 & 7) ^ (row & 7)) << 4)));
          if (row >= ntok) wv[i] = make_uint4(0u, 0u, 0u, 0u);
        }
#pragma unroll
        for (int i = 0; i < ITER; ++i) {
          const int qi = lane + 32 * i, row = qi & 15, c8 = qi >> 4;
          const uint4 w = wv[i];
          uint32_t h0, h1, h2, h3, h4, h5, h6, h7;
          kv8x4_to_h2x2<KVF>(w.x, h0, h1);
          kv8x4_to_h2x2<KVF>(w.y, h2, h3);
          kv8x4_to_h2x2<KVF>(w.z, h4, h5);
          kv8x4_to_h2x2<KVF>(w.w, h6, h7);
          const int chunk = 2 * c8;  // 8-element fp16 chunk of d = 16 c8
          asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(vsrc + tile_off(row, chunk)),
                       "r"(h0), "r"(h1), "r"(h2), "r"(h3)
                       : "memory");
          asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(vsrc + tile_off(row, chunk + 1)),
                       "r"(h4), "r"(h5), "r"(h6), "r"(h7)
                       : "memory");
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(bar_empty + 8 * s);
      }

      if (KVF == 0 && ntok < 16) {
        // Last page of the sequence: slots >= ntok hold whatever the pool
        // holds; clear them in V so 0 * (inf or NaN) cannot enter PV.
        const int nclr = (16 - ntok) * C::kBoxes * 8;
        for (int idx = lane; idx < nclr; idx += 32) {
          const int row = ntok + idx / (C::kBoxes * 8);
          const int rem = idx % (C::kBoxes * 8);
          const uint32_t addr = tv + (rem >> 3) * 2048 + row * 128 + (rem & 7) * 16;
          asm volatile("st.shared.v4.u32 [%0], {%1, %1, %1, %1};" ::"r"(addr), "r"(0u) : "memory");
        }
        __syncwarp();
      }

      // Online softmax. Lane (g, c): tokens g, g+8; heads 2c, 2c+1 of tile nt.
      const bool v0 = g < ntok, v1 = g + 8 < ntok;
      uint32_t pb[NT][2], pl[NT][2];
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        const float x0 = v0 ? sc[nt][0] * sl2 : -INFINITY;
        const float x1 = v0 ? sc[nt][1] * sl2 : -INFINITY;
        const float x2 = v1 ? sc[nt][2] * sl2 : -INFINITY;
        const float x3 = v1 ? sc[nt][3] * sl2 : -INFINITY;
        float mx0 = fmaxf(x0, x2), mx1 = fmaxf(x1, x3);
#pragma unroll
        for (int off = 4; off < 32; off <<= 1) {
          mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, off));
          mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, off));
        }
        const float mn0 = fmaxf(mrun[nt][0], mx0), mn1 = fmaxf(mrun[nt][1], mx1);
        // A running max that did not move gives alpha = 2^0 = 1 exactly, so
        // when no lane's max moved the O rescale is skipped (bit-identical).
        const bool moved = __any_sync(0xffffffffu, mn0 != mrun[nt][0] || mn1 != mrun[nt][1]);
        const float al0 = ex2(mrun[nt][0] - mn0), al1 = ex2(mrun[nt][1] - mn1);
        const float p0 = ex2(x0 - mn0), p1 = ex2(x1 - mn1);
        const float p2 = ex2(x2 - mn0), p3 = ex2(x3 - mn1);
        lrun[nt][0] = fmaf(lrun[nt][0], al0, p0 + p2);
        lrun[nt][1] = fmaf(lrun[nt][1], al1, p1 + p3);
        mrun[nt][0] = mn0;
        mrun[nt][1] = mn1;
        if (moved) {
#pragma unroll
          for (int mt = 0; mt < C::kKSteps; ++mt) {
            o[nt][mt][0] *= al0;
            o[nt][mt][1] *= al1;
            o[nt][mt][2] *= al0;
            o[nt][mt][3] *= al1;
          }
        }
        // P^T as the B operand (k = token, n = head): transpose the
        // (token x head) accumulator pairs with movmatrix.
        const uint32_t h01 = pack_half2(p0, p1), h23 = pack_half2(p2, p3);
        const float2 f01 = unpack_half2(h01), f23 = unpack_half2(h23);
        pb[nt][0] = movmatrix_trans(h01);
        pb[nt][1] = movmatrix_trans(h23);
        pl[nt][0] = movmatrix_trans(pack_half2(p0 - f01.x, p1 - f01.y));
        pl[nt][1] = movmatrix_trans(pack_half2(p2 - f23.x, p3 - f23.y));
      }

      // O^T += V^T . P^T. A operand rows = d: transposed loads of matrices
      // (tok 0-7 | 8-15) x (d lo | hi) -> a0 (d lo, tok lo), a1 (d hi, tok lo),
      // a2 (d lo, tok hi), a3 (d hi, tok hi).
#pragma unroll
      for (int mt = 0; mt < C::kKSteps; ++mt) {
        uint32_t a0, a1, a2, a3;
        if constexpr (C::kDirectV) {
          // A rows of m-tile mt: g -> d = 16 mt + 2g, g + 8 -> d = 16 mt + 2g + 1
          kv8x4_to_h2_even_odd<KVF>(vr[mt][0], a0, a1);
          kv8x4_to_h2_even_odd<KVF>(vr[mt][1], a2, a3);
        } else {
          ldsm_x4_trans(vsrc + tile_off(r8 + ((mi >> 1) << 3), 2 * mt + (mi & 1)), a0, a1, a2,
                        a3);
        }
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          mma_f16_16816(o[nt][mt], a0, a1, a2, a3, pb[nt][0], pb[nt][1]);
          mma_f16_16816(o[nt][mt], a0, a1, a2, a3, pl[nt][0], pl[nt][1]);
        }
      }
      if (KVF == 0 && ntok < 16) fence_proxy_async_smem();
      __syncwarp();  // this warp's fp16 V tile is rewritten for its next page
      if (KVF == 0 && lane == 0) mbar_arrive(bar_empty + 8 * s);
    } else {
      __syncwarp();
      if (lane == 0) mbar_arrive(bar_empty + 8 * s);
    }
  }

  // ── merge the consumer warps' states ─────────────────────────────────
#pragma unroll
  for (int nt = 0; nt < NT; ++nt)
#pragma unroll
    for (int k = 0; k < 2; ++k)
#pragma unroll
      for (int off = 4; off < 32; off <<= 1)
        lrun[nt][k] += __shfl_xor_sync(0xffffffffu, lrun[nt][k], off);

  named_bar_sync(1, NWC * 32);  // every consumer is done with the ring
  constexpr int RS = D + 4;     // padded row: conflict-free stores below
  float* sm_o = reinterpret_cast<float*>(smem);  // [NWC][GS][RS]
  float* sm_ml = sm_o + NWC * GS * RS;           // [NWC][GS][2]
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const int head = nt * 8 + 2 * c + k;
      if (head < GS) {
        float* row = sm_o + (warp * GS + head) * RS;
#pragma unroll
        for (int mt = 0; mt < C::kKSteps; ++mt) {
          if constexpr (C::kDirectV) {  // O^T rows are d = 16 mt + 2g, + 1
            row[mt * 16 + 2 * g] = o[nt][mt][k];
            row[mt * 16 + 2 * g + 1] = o[nt][mt][2 + k];
          } else {
            row[mt * 16 + g] = o[nt][mt][k];
            row[mt * 16 + g + 8] = o[nt][mt][2 + k];
          }
        }
        if (g == 0) {
          sm_ml[(warp * GS + head) * 2] = mrun[nt][k];
          sm_ml[(warp * GS + head) * 2 + 1] = lrun[nt][k];
        }
      }
    }
  }
  named_bar_sync(1, NWC * 32);

  // Each thread merges 8 consecutive d of one head (RS keeps rows 16-byte
  // aligned, so the shared-memory reads are two float4 loads per warp state).
  const long long row0 = (long long)it.b * p.Hq + (long long)it.kvh * GS;
  constexpr int CH = D / 8;
  for (int e = threadIdx.x; e < GS * CH; e += NWC * 32) {
    const int head = e / CH, d0 = (e - head * CH) * 8;
    float M = -INFINITY;
#pragma unroll
    for (int ww = 0; ww < NWC; ++ww) M = fmaxf(M, sm_ml[(ww * GS + head) * 2]);
    float num[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    float den = 0.f;
    if (M != -INFINITY) {
#pragma unroll
      for (int ww = 0; ww < NWC; ++ww) {
        const float wt = ex2(sm_ml[(ww * GS + head) * 2] - M);
        den = fmaf(wt, sm_ml[(ww * GS + head) * 2 + 1], den);
        const float4* src = reinterpret_cast<const float4*>(sm_o + (ww * GS + head) * RS + d0);
        const float4 a = src[0], b = src[1];
        num[0] = fmaf(wt, a.x, num[0]);
        num[1] = fmaf(wt, a.y, num[1]);
        num[2] = fmaf(wt, a.z, num[2]);
        num[3] = fmaf(wt, a.w, num[3]);
        num[4] = fmaf(wt, b.x, num[4]);
        num[5] = fmaf(wt, b.y, num[5]);
        num[6] = fmaf(wt, b.z, num[6]);
        num[7] = fmaf(wt, b.w, num[7]);
      }
    }
    if constexpr (KVF != 0) {
#pragma unroll
      for (int k = 0; k < 8; ++k) num[k] *= p.v_scale;
    }
    if (it.direct) {
#pragma unroll
      for (int k = 0; k < 8; ++k) num[k] = den > 0.f ? num[k] / den : 0.f;
      if (p.vec8) {
        store_out8<__half>(p, row0 + head, d0, num);
      } else {
#pragma unroll
        for (int k = 0; k < 8; ++k) store_out<__half>(p, row0 + head, d0 + k, num[k]);
      }
    } else {
      const long long pr = (row0 + head) * p.slots + it.slot0 + it.part;
      float* dst = p.part_o + pr * D + d0;
#pragma unroll
      for (int k = 0; k < 8; ++k) dst[k] = num[k];
      if (d0 == 0) {
        p.part_ml[2 * pr] = M;
        p.part_ml[2 * pr + 1] = den;
      }
    }
  }
}

// Resident CTAs per SM the register allocation must allow, for D <= 128 with
// one 8-head tile: 6 for fp16 pages (the shared-memory limit of the 4-page
// ring), 4 for one-byte pages (3 consumer warps, 128 registers, 50 KB of ring
// each). The wider variants (D = 256, 16 heads per KV head) keep their
// registers instead: a bound would spill them.
#ifndef XPA_FP16_MIN_CTAS
#define XPA_FP16_MIN_CTAS 6
#endif
#ifndef XPA_FP8_MIN_CTAS
#define XPA_FP8_MIN_CTAS 4
#endif
#ifndef XPA_INT8_MIN_CTAS
#define XPA_INT8_MIN_CTAS XPA_FP8_MIN_CTAS
#endif
template <int D, int NT, int STAGES, int NWC, int KVF>
__global__ void __launch_bounds__((NWC + 1) * 32,
                                  (D <= 128 && NT == 1)
                                      ? (KVF == kKvInt8 ? XPA_INT8_MIN_CTAS
                                                        : KVF ? XPA_FP8_MIN_CTAS : XPA_FP16_MIN_CTAS)
                                      : 1)
    pa_tma_mma_kernel(const __grid_constant__ CUtensorMap tmK,
                      const __grid_constant__ CUtensorMap tmV, const Params p) {
  tma_mma_body<D, NT, STAGES, NWC, KVF>(tmK, tmV, p);
  // Beside a running shared-prefix grid: this grid may not complete before
  // that one has (the merge after it reads both grids' partials).
  if (p.join_primary && blockIdx.x == 0) pdl_wait_primary();
}

// ════════════════════════════════════════════════════════════════════════
// Log-sum-exp reduce of split-context partials (and shared-prefix chunks):
//   M = max_p m_p,  w_p = 2^(m_p - M),  out = sum_p w_p o_p / sum_p w_p l_p
// One warp per (b, q head) row, 4 rows per CTA (merge_row_warp).
// ════════════════════════════════════════════════════════════════════════
template <typename T>
__global__ void __launch_bounds__(128) pa_reduce_kernel(const Params p) {
  __shared__ float sw[4][32];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long long row = (long long)blockIdx.x * 4 + warp;
  int nslots = 0;
  bool direct = true;
  if (row < (long long)p.B * p.Hq) {
    const int b = (int)(row / p.Hq);
    int L = __ldg(p.seq_lens + b);
    const long long lim = (long long)p.max_blocks * p.block_size;
    L = L < 0 ? 0 : ((long long)L > lim ? (int)lim : L);
    const int npages = (L + p.block_size - 1) / p.block_size;
    const int P = prefix_of(p, b, npages);
    const int nparts = (npages - P + p.part_pages - 1) / p.part_pages;
    nslots = (P > 0 ? (P + p.prefix_chunk - 1) / p.prefix_chunk : 0) + nparts;
    // written directly by the attention kernel (zero rows always are)
    direct = P == 0 && (nparts == 0 || (nparts == 1 && !p.merge_all));
  }
  pdl_launch_dependents();  // the gather barrier (if any) may be scheduled now
  // Every CTA waits for the attention grid, also those with nothing to merge:
  // this grid must not complete before the attention kernel has (later work
  // on the stream is ordered after this grid, not after that kernel).
  pdl_wait_primary();
  if (direct) return;
  merge_row_warp<T>(p, row, nslots, lane, sw[warp]);
}

// ════════════════════════════════════════════════════════════════════════
// The same merge for rows with many partials (long contexts split into tens
// of partitions): one CTA of four warps per (b, q head) row. Warp w
// accumulates slots w, w + 4, ... (each lane 4 consecutive elements, four
// slots' loads in flight), so a row's partials are read by four warps at
// once instead of one; the four partial sums meet in shared memory.
// ════════════════════════════════════════════════════════════════════════
template <typename T>
__global__ void __launch_bounds__(128) pa_reduce_wide_kernel(const Params p) {
  constexpr int NW = 4;
  __shared__ float s_num[NW][256];
  __shared__ float s_den[NW];
  __shared__ float s_max[NW];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long long row = blockIdx.x;
  const int b = (int)(row / p.Hq);
  int L = __ldg(p.seq_lens + b);
  const long long lim = (long long)p.max_blocks * p.block_size;
  L = L < 0 ? 0 : ((long long)L > lim ? (int)lim : L);
  const int npages = (L + p.block_size - 1) / p.block_size;
  const int P = prefix_of(p, b, npages);
  const int nparts = (npages - P + p.part_pages - 1) / p.part_pages;
  const int nslots = (P > 0 ? (P + p.prefix_chunk - 1) / p.prefix_chunk : 0) + nparts;
  const bool direct = P == 0 && (nparts == 0 || (nparts == 1 && !p.merge_all));
  pdl_launch_dependents();  // the gather barrier (if any) may be scheduled now
  pdl_wait_primary();       // every CTA: this grid must not complete before the attention grid
  if (direct) return;

  const float2* ml = reinterpret_cast<const float2*>(p.part_ml) + row * p.slots;
  float mx = -INFINITY;
  for (int i = threadIdx.x; i < nslots; i += NW * 32) mx = fmaxf(mx, __ldcg(&ml[i].x));
  mx = warp_max(mx);
  if (lane == 0) s_max[warp] = mx;
  __syncthreads();
  const float M = fmaxf(fmaxf(s_max[0], s_max[1]), fmaxf(s_max[2], s_max[3]));
  auto weight = [M](float m) { return (M == -INFINITY || m == -INFINITY) ? 0.f : ex2(m - M); };

  const float* po = p.part_o + row * p.slots * p.D;
  float den = 0.f;
  const bool vec = (p.D & 3) == 0;  // part_o rows are 16-byte aligned when D % 4 == 0
  for (int base = 0; base < p.D; base += vec ? 128 : 32) {
    const int d0 = base + (vec ? lane * 4 : lane);
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    float dsum = 0.f;
    int i = warp;
    for (; i + 3 * NW < nslots; i += 4 * NW) {
      float2 m4[4];
      float4 x4[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        m4[u] = __ldcg(ml + i + u * NW);
        if (d0 < p.D) {
          const float* src = po + (long long)(i + u * NW) * p.D + d0;
          x4[u] = vec ? __ldcg(reinterpret_cast<const float4*>(src))
                      : make_float4(__ldcg(src), 0.f, 0.f, 0.f);
        } else {
          x4[u] = make_float4(0.f, 0.f, 0.f, 0.f);
        }
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const float w = weight(m4[u].x);
        dsum = fmaf(w, m4[u].y, dsum);
        acc.x = fmaf(w, x4[u].x, acc.x);
        acc.y = fmaf(w, x4[u].y, acc.y);
        acc.z = fmaf(w, x4[u].z, acc.z);
        acc.w = fmaf(w, x4[u].w, acc.w);
      }
    }
    for (; i < nslots; i += NW) {
      const float2 m = __ldcg(ml + i);
      const float w = weight(m.x);
      dsum = fmaf(w, m.y, dsum);
      if (d0 < p.D) {
        const float* src = po + (long long)i * p.D + d0;
        const float4 x = vec ? __ldcg(reinterpret_cast<const float4*>(src))
                             : make_float4(__ldcg(src), 0.f, 0.f, 0.f);
        acc.x = fmaf(w, x.x, acc.x);
        acc.y = fmaf(w, x.y, acc.y);
        acc.z = fmaf(w, x.z, acc.z);
        acc.w = fmaf(w, x.w, acc.w);
      }
    }
    if (base == 0) den = dsum;  // every pass sums the same weights
    if (d0 < p.D) {
      if (vec) {
        s_num[warp][d0] = acc.x;
        s_num[warp][d0 + 1] = acc.y;
        s_num[warp][d0 + 2] = acc.z;
        s_num[warp][d0 + 3] = acc.w;
      } else {
        s_num[warp][d0] = acc.x;
      }
    }
  }
  if (lane == 0) s_den[warp] = den;
  __syncthreads();
  const float tot = s_den[0] + s_den[1] + s_den[2] + s_den[3];
  auto final = [&](int d) {
    const float num = s_num[0][d] + s_num[1][d] + s_num[2][d] + s_num[3][d];
    return tot > 0.f ? num / tot : 0.f;
  };
  if (p.vec8) {
    // 8 consecutive elements per thread: one 16-byte store per destination
    for (int d0 = threadIdx.x * 8; d0 < p.D; d0 += NW * 32 * 8) {
      float v8[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) v8[k] = final(d0 + k);
      store_out8<T>(p, row, d0, v8);
    }
  } else {
    for (int d = threadIdx.x; d < p.D; d += NW * 32) store_out<T>(p, row, d, final(d));
  }
}

// ════════════════════════════════════════════════════════════════════════
// Fused head gather: end-of-step barrier across the ranks' GPUs. Lane r
// stores `step` into rank r's flag slot for this rank (release, system
// scope), then waits until rank r's own signal for `step` has arrived in this
// rank's flag array (acquire, system scope). Each wait is bounded; on expiry
// the kernel raises NXT_PA_DEV_TIMEOUT and returns. One warp, one launch per
// GPU; the ranks' barrier kernels run on different GPUs.
// ════════════════════════════════════════════════════════════════════════
struct PeerFlags {
  unsigned long long* flags[kMaxPeers];  // rank r's flag array [world]
};

__global__ void __launch_bounds__(32) pa_peer_barrier_kernel(PeerFlags f, unsigned long long step,
                                                             int rank, int world, int* status,
                                                             unsigned long long budget_ns) {
  const int r = threadIdx.x;
  // The next call's attention grid may become resident while this one waits
  // (it waits for this grid itself before it reads anything).
  pdl_launch_dependents();
  // Launched as a programmatic dependent: wait until the kernels that stored
  // this rank's rows (attention, then merge) have completed; their writes,
  // peer writes included, are flushed by then.
  pdl_wait_primary();
  if (r >= world) return;
  __threadfence_system();
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(f.flags[r] + rank), "l"(step)
               : "memory");
  const unsigned long long* mine = f.flags[rank] + r;
  const uint64_t t0 = globaltimer_ns();
  for (;;) {
    unsigned long long v;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(mine) : "memory");
    if (v >= step) break;
    if (globaltimer_ns() - t0 >= budget_ns) {
      if (status) atomicOr(status, kDevTimeout);
      break;
    }
    __nanosleep(64);
  }
}

// ════════════════════════════════════════════════════════════════════════
// KV append ("reshape and cache"): token t's K and V rows ([Hkv][D] each)
// go to page slot_mapping[t] / block_size, slot slot_mapping[t] % block_size
// of the paged pools; a negative slot skips the token. One warp per
// (token, KV head), 16-byte copies when every row is 16-byte aligned. It
// triggers its dependents at start, so an attention grid launched after it
// as a programmatic dependent starts streaming at once.
// ════════════════════════════════════════════════════════════════════════
template <typename T>
__global__ void __launch_bounds__(128) pa_append_kernel(AppendParams a) {
  pdl_launch_dependents();
  const long long w = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (w >= (long long)a.num_tokens * a.Hkv) return;
  const int t = (int)(w / a.Hkv), h = (int)(w % a.Hkv);
  const long long slot = a.slots[t];
  if (slot < 0) return;
  const long long page = slot / a.block_size, s = slot % a.block_size;
  const long long dst = page * a.kv_block_stride + (long long)h * a.kv_head_stride + s * a.D;
  const long long src = (long long)t * a.token_stride + (long long)h * a.D;
  const T* k = static_cast<const T*>(a.key) + src;
  const T* v = static_cast<const T*>(a.value) + src;
  T* kc = static_cast<T*>(a.key_cache) + dst;
  T* vc = static_cast<T*>(a.value_cache) + dst;
  if (a.vec16) {
    constexpr int E = 16 / sizeof(T);
    for (int i = lane; i < a.D / E; i += 32) {
      reinterpret_cast<uint4*>(kc)[i] = __ldg(reinterpret_cast<const uint4*>(k) + i);
      reinterpret_cast<uint4*>(vc)[i] = __ldg(reinterpret_cast<const uint4*>(v) + i);
    }
  } else {
    for (int i = lane; i < a.D; i += 32) {
      kc[i] = k[i];
      vc[i] = v[i];
    }
  }
}

// KV append into a one-byte cache: fp16 rows in, encode(x / scale) bytes out
// (round to nearest even, saturating), 8 elements per lane and step when
// every row is 16-byte (source) / 8-byte (cache) aligned.
template <int KVF>
__global__ void __launch_bounds__(128) pa_append_fp8_kernel(AppendParams a) {
  pdl_launch_dependents();
  const long long w = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (w >= (long long)a.num_tokens * a.Hkv) return;
  const int t = (int)(w / a.Hkv), h = (int)(w % a.Hkv);
  const long long slot = a.slots[t];
  if (slot < 0) return;
  const long long page = slot / a.block_size, s = slot % a.block_size;
  const long long dst = page * a.kv_block_stride + (long long)h * a.kv_head_stride + s * a.D;
  const long long src = (long long)t * a.token_stride + (long long)h * a.D;
  const __half* k = static_cast<const __half*>(a.key) + src;
  const __half* v = static_cast<const __half*>(a.value) + src;
  uint8_t* kc = static_cast<uint8_t*>(a.key_cache) + dst;
  uint8_t* vc = static_cast<uint8_t*>(a.value_cache) + dst;
  const float ks = a.k_scale, vs = a.v_scale;
  auto q8 = [&](uint4 x, float sc) {  // 8 fp16 -> 8 fp8 bytes
    const __half2* h2 = reinterpret_cast<const __half2*>(&x);
    uint32_t b[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = __half22float2(h2[i]);
      b[i] = float2_to_fp8x2<KVF>(f.x / sc, f.y / sc);
    }
    return make_uint2(b[0] | (b[1] << 16), b[2] | (b[3] << 16));
  };
  if (a.vec16) {
    for (int i = lane; i < a.D / 8; i += 32) {
      reinterpret_cast<uint2*>(kc)[i] = q8(__ldg(reinterpret_cast<const uint4*>(k) + i), ks);
      reinterpret_cast<uint2*>(vc)[i] = q8(__ldg(reinterpret_cast<const uint4*>(v) + i), vs);
    }
  } else {
    for (int i = lane; i < a.D; i += 32) {
      kc[i] = (uint8_t)(float2_to_fp8x2<KVF>(__half2float(k[i]) / ks, 0.f) & 0xffu);
      vc[i] = (uint8_t)(float2_to_fp8x2<KVF>(__half2float(v[i]) / vs, 0.f) & 0xffu);
    }
  }
}

// ════════════════════════════════════════════════════════════════════════
// Launchers
// ════════════════════════════════════════════════════════════════════════
namespace {

// Launches `kern` on `st`; as a programmatic dependent of the previous
// launch on the stream when `pdl` is set.
template <typename... KArgs, typename... Args>
cudaError_t launch_ex(void (*kern)(KArgs...), unsigned grid, unsigned block, size_t smem,
                      cudaStream_t st, bool pdl, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(block);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

template <typename T, int DPL, int HG>
cudaError_t launch_generic_t(const Params& p, cudaStream_t st) {
  const long long grid = (long long)p.B * p.Hkv * p.max_parts;
  const bool pdl = p.after_append != 0 || p.wait_first != 0;
  if constexpr (sizeof(T) == 2) {  // fp8 caches pair with fp16 queries
    if (p.kv_fmt == kKvE4M3)
      return launch_ex(pa_generic_kernel<T, DPL, HG, kKvE4M3>, (unsigned)grid, 128, 0, st, pdl, p);
    if (p.kv_fmt == kKvE5M2)
      return launch_ex(pa_generic_kernel<T, DPL, HG, kKvE5M2>, (unsigned)grid, 128, 0, st, pdl, p);
    if (p.kv_fmt == kKvInt8)
      return launch_ex(pa_generic_kernel<T, DPL, HG, kKvInt8>, (unsigned)grid, 128, 0, st, pdl, p);
  }
  return launch_ex(pa_generic_kernel<T, DPL, HG, 0>, (unsigned)grid, 128, 0, st, pdl, p);
}

template <typename T, int DPL>
cudaError_t launch_generic_dpl(const Params& p, cudaStream_t st) {
  // Heads per pass: enough to cover the group, with HG*DPL <= 32 registers
  // of accumulator per lane.
  constexpr int HGMAX = 32 / DPL;
  int hg = 1;
  while (hg < p.GS && hg < HGMAX) hg <<= 1;
  switch (hg) {
    case 1: return launch_generic_t<T, DPL, 1>(p, st);
    case 2: return launch_generic_t<T, DPL, 2>(p, st);
    case 4: return launch_generic_t<T, DPL, 4>(p, st);
    case 8: return launch_generic_t<T, DPL, (HGMAX >= 8 ? 8 : HGMAX)>(p, st);
    default: return launch_generic_t<T, DPL, (HGMAX >= 16 ? 16 : HGMAX)>(p, st);
  }
}

template <typename T>
cudaError_t launch_generic_typed(const Params& p, cudaStream_t st) {
  if (p.D <= 32) return launch_generic_dpl<T, 1>(p, st);
  if (p.D <= 64) return launch_generic_dpl<T, 2>(p, st);
  if (p.D <= 128) return launch_generic_dpl<T, 4>(p, st);
  return launch_generic_dpl<T, 8>(p, st);
}

// Ring depth of the TMA pipeline (pages in flight per CTA) and consumer warps
// per CTA. Measured on B200 at config 2: a 4-page ring with 2 consumer warps
// (~35 KB of shared memory, 6 CTAs per SM) streams faster than deeper rings
// with more warps per CTA; more resident CTAs hide page latency better than a
// deeper ring per CTA. A build may override either for tuning sweeps.
#ifndef XPA_RING_PAGES
#define XPA_RING_PAGES 4
#endif
#ifndef XPA_CONSUMER_WARPS
#define XPA_CONSUMER_WARPS 2
#endif

// One-byte caches: pages are half the bytes, so the SM needs twice the page
// rate. With V read straight into registers (no fp16 V tiles), 3 consumer
// warps sharing a 12-page ring, 4 CTAs per SM, measured fastest on B200.
#ifndef XPA_FP8_RING_PAGES
#define XPA_FP8_RING_PAGES 12
#endif
#ifndef XPA_FP8_CONSUMER_WARPS
#define XPA_FP8_CONSUMER_WARPS 3
#endif
// int8 caches: the same page rate as fp8, more conversion work per page.
#ifndef XPA_INT8_RING_PAGES
#define XPA_INT8_RING_PAGES XPA_FP8_RING_PAGES
#endif
#ifndef XPA_INT8_CONSUMER_WARPS
#define XPA_INT8_CONSUMER_WARPS XPA_FP8_CONSUMER_WARPS
#endif

template <int D, int NT, int KVF>
cudaError_t launch_fast_t(const CUtensorMap& tk, const CUtensorMap& tv, const Params& p,
                          cudaStream_t st) {
  constexpr int RING =
      KVF == kKvInt8 ? XPA_INT8_RING_PAGES : KVF ? XPA_FP8_RING_PAGES : XPA_RING_PAGES;
  constexpr int NWC = KVF == kKvInt8 ? XPA_INT8_CONSUMER_WARPS
                                     : KVF ? XPA_FP8_CONSUMER_WARPS : XPA_CONSUMER_WARPS;
  // D = 256 pages are twice as large: half the ring, still a multiple of NWC
  constexpr int HALF = RING / 2 > NWC ? RING / 2 : NWC;
  constexpr int STAGES = (D == 256) ? (HALF + NWC - 1) / NWC * NWC : RING;
  using C = FastCfg<D, NT, STAGES, NWC, KVF>;
  auto kern = pa_tma_mma_kernel<D, NT, STAGES, NWC, KVF>;
  // The attribute is per function and device; setting it every call costs
  // a driver call only.
  cudaError_t e =
      cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmem);
  if (e != cudaSuccess) return e;
  // all of the SM's unified L1 / shared storage as shared memory: the
  // resident-CTA count, not L1 hits, keeps the page stream going
  e = cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout,
                           (int)cudaSharedmemCarveoutMaxShared);
  if (e != cudaSuccess) return e;
  const long long grid = (long long)p.B * p.Hkv * p.max_parts;
  return launch_ex(kern, (unsigned)grid, C::kThreads, C::kSmem, st,
                   p.after_append != 0 || p.join_primary != 0 || p.wait_first != 0, tk, tv,
                   p);
}

template <int D, int NT>
cudaError_t launch_fast_kv(const CUtensorMap& tk, const CUtensorMap& tv, const Params& p,
                           cudaStream_t st) {
  if (p.kv_fmt == kKvE4M3) return launch_fast_t<D, NT, kKvE4M3>(tk, tv, p, st);
  if (p.kv_fmt == kKvE5M2) return launch_fast_t<D, NT, kKvE5M2>(tk, tv, p, st);
  if (p.kv_fmt == kKvInt8) return launch_fast_t<D, NT, kKvInt8>(tk, tv, p, st);
  return launch_fast_t<D, NT, 0>(tk, tv, p, st);
}

}  // namespace

cudaError_t launch_generic(const Params& p, int dtype_size, cudaStream_t st) {
  return dtype_size == 4 ? launch_generic_typed<float>(p, st)
                         : launch_generic_typed<__half>(p, st);
}

bool fast_path_shape_ok(int head_size, int group, int block_size, int dtype_size, int kv_fmt) {
  if (dtype_size != 2 || block_size != 16) return false;
  if (head_size != 64 && head_size != 128 && head_size != 256) return false;
  if (kv_fmt != 0 && head_size == 64) return false;  // 1-byte rows narrower than a 128-byte box
  if (group < 1 || group > 16) return false;
  if (group > 8 && head_size == 256) return false;  // accumulator registers
  return true;
}

cudaError_t launch_fast(const CUtensorMap& tk, const CUtensorMap& tv, const Params& p,
                        cudaStream_t st) {
  const bool two = p.GS > 8;
  switch (p.D) {
    case 64:
      if (p.kv_fmt) return cudaErrorInvalidValue;
      return two ? launch_fast_t<64, 2, 0>(tk, tv, p, st) : launch_fast_t<64, 1, 0>(tk, tv, p, st);
    case 128:
      return two ? launch_fast_kv<128, 2>(tk, tv, p, st) : launch_fast_kv<128, 1>(tk, tv, p, st);
    case 256: return launch_fast_kv<256, 1>(tk, tv, p, st);
    default: return cudaErrorInvalidValue;
  }
}

// Rows with more partial slots than this are merged by four warps each.
#ifndef XPA_WIDE_MERGE_SLOTS
#define XPA_WIDE_MERGE_SLOTS 16
#endif

cudaError_t launch_reduce(const Params& p, int dtype_size, cudaStream_t st) {
  const long long rows = (long long)p.B * p.Hq;
  const bool wide = p.slots > XPA_WIDE_MERGE_SLOTS;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(wide ? rows : (rows + 3) / 4));
  cfg.blockDim = dim3(128);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (wide) {
    if (dtype_size == 4) return cudaLaunchKernelEx(&cfg, pa_reduce_wide_kernel<float>, p);
    return cudaLaunchKernelEx(&cfg, pa_reduce_wide_kernel<__half>, p);
  }
  if (dtype_size == 4) return cudaLaunchKernelEx(&cfg, pa_reduce_kernel<float>, p);
  return cudaLaunchKernelEx(&cfg, pa_reduce_kernel<__half>, p);
}

cudaError_t launch_append(const AppendParams& a, int dtype_size, cudaStream_t st) {
  const long long warps = (long long)a.num_tokens * a.Hkv;
  const unsigned grid = (unsigned)((warps * 32 + 127) / 128);
  if (grid == 0) return cudaSuccess;
  if (a.kv_fmt == kKvE4M3)
    pa_append_fp8_kernel<kKvE4M3><<<grid, 128, 0, st>>>(a);
  else if (a.kv_fmt == kKvE5M2)
    pa_append_fp8_kernel<kKvE5M2><<<grid, 128, 0, st>>>(a);
  else if (a.kv_fmt == kKvInt8)
    pa_append_fp8_kernel<kKvInt8><<<grid, 128, 0, st>>>(a);
  else if (dtype_size == 4)
    pa_append_kernel<float><<<grid, 128, 0, st>>>(a);
  else
    pa_append_kernel<__half><<<grid, 128, 0, st>>>(a);
  return cudaGetLastError();
}

cudaError_t launch_peer_barrier(void* const* flags, int world, int rank, unsigned long long step,
                                int* status, unsigned long long budget_ns, cudaStream_t st) {
  PeerFlags f{};
  for (int r = 0; r < world && r < kMaxPeers; ++r)
    f.flags[r] = static_cast<unsigned long long*>(flags[r]);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(1);
  cfg.blockDim = dim3(32);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, pa_peer_barrier_kernel, f, step, rank, world, status, budget_ns);
}

}  // namespace xpa
