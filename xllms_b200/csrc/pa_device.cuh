// pa_device.cuh — sm_100a device primitives and the shared kernel parameter
// block for paged decode attention. Inline PTX only; no library kernels.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace xpa {

// Device status bits; the same values as NXT_PA_DEV_* in operator_api.h.
constexpr int kDevTimeout = 0x1;
constexpr int kDevBadPage = 0x2;
constexpr int kDevSeqClamped = 0x4;

constexpr int kMaxPeers = 8;

// Everything a launch needs besides the tensor maps. Strides are in elements.
struct Params {
  void* out;              // [B][Hq][D]
  const void* q;          // [B][Hq][D]
  const void* k;          // paged pool
  const void* v;          // paged pool
  const int* block_tables;  // [B][max_blocks]
  const int* seq_lens;      // [B]
  float* part_o;   // [B][Hq][max_parts][D] unnormalised partial outputs
  float* part_ml;  // [B][Hq][max_parts][2] (max in log2 units, sum of exp2)
  int* status;     // device status word (NXT_PA_DEV_* bits), may be null
  long long kv_block_stride;
  long long kv_head_stride;
  long long num_blocks;  // <= 0: unknown, no upper bound check
  unsigned long long timeout_ns;  // bound on every pipeline wait (not on the drain)
  int B, Hq, Hkv, D, GS;
  int max_blocks, block_size;
  int part_pages, max_parts;
  float scale_log2;  // scale * log2(e): scores live in the exp2 domain
  // Fused head gather (KV-head sharding over GPUs): when npeers > 0 every
  // output row (b, h) of this rank is stored into each peers[r] at element
  // peer_off + (b * Hq_total + head_offset + h) * D, and `out` is unused.
  int npeers, Hq_total, head_offset;
  long long peer_off;
  void* peers[kMaxPeers];
  // 1 when D % 8 == 0 and out / peer buffers and the partial workspace are
  // 16-byte aligned: rows are then stored 8 elements (16 or 32 bytes) at a time.
  int vec8;
  // 1 when this grid was launched as a programmatic dependent of the KV
  // append kernel: a sequence's last page may only be read after
  // griddepcontrol.wait (the appended token lives there).
  int after_append;
};

// KV append: token t's rows key/value[t*token_stride + h*D + d] go to the
// pool slot slots[t] (page slot/block_size, slot slot%block_size).
struct AppendParams {
  const void* key;
  const void* value;
  void* key_cache;
  void* value_cache;
  const long long* slots;
  long long kv_block_stride, kv_head_stride, token_stride;
  int num_tokens, Hkv, D, block_size;
  int vec16;  // every row 16-byte aligned: copy 16 bytes per lane
};

// One unit of work: context partition `part` of (sequence b, KV head kvh).
struct Item {
  int b, kvh, part;
  int L;            // clamped context length of sequence b
  int page_begin;   // first page of this partition
  int page_end;     // one past its last page
  int nparts;       // partitions of sequence b (0 when L == 0)
};

enum ItemKind { kItemNone = 0, kItemZero = 1, kItemWork = 2 };

__device__ __forceinline__ void raise_status(const Params& p, int bits) {
  if (p.status) atomicOr(p.status, bits);
}

// Grid index -> item. Index order is (b, kvh, part) with part fastest, so the
// CTAs of one sequence are dispatched together.
__device__ __forceinline__ ItemKind decode_item(const Params& p, int idx, Item& it) {
  it.part = idx % p.max_parts;
  const int rest = idx / p.max_parts;
  it.kvh = rest % p.Hkv;
  it.b = rest / p.Hkv;
  int L = __ldg(p.seq_lens + it.b);
  const long long cap = (long long)p.max_blocks * p.block_size;
  if (L < 0 || (long long)L > cap) {
    if (it.part == 0 && it.kvh == 0 && threadIdx.x == 0) raise_status(p, kDevSeqClamped);
    L = L < 0 ? 0 : (int)cap;
  }
  it.L = L;
  const int npages = (L + p.block_size - 1) / p.block_size;
  it.nparts = (npages + p.part_pages - 1) / p.part_pages;
  if (it.nparts == 0) return it.part == 0 ? kItemZero : kItemNone;
  if (it.part >= it.nparts) return kItemNone;
  it.page_begin = it.part * p.part_pages;
  it.page_end = min(npages, it.page_begin + p.part_pages);
  return kItemWork;
}

__device__ __forceinline__ uint32_t smem_u32(const void* ptr) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(ptr));
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// 2^x via the PTX approximate instruction (ex2.approx, ftz): 2^-inf = +0.
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// ── mbarrier ────────────────────────────────────────────────────────────
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ uint32_t mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred P;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 P, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, P;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok;
}

__device__ __forceinline__ uint32_t mbar_test_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred P;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 P, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, P;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok;
}

// Waits for the phase with the given parity to complete, for at most
// budget_ns of %globaltimer time. Returns false when the budget ran out.
// The first probe does not block (test_wait), and the budget is checked
// before the first blocking probe (try_wait may suspend the thread in
// hardware) and then before every XPA_WAIT_CHECK_EVERY-th one, so a zero
// budget gives up as soon as the phase is found incomplete.
#ifndef XPA_WAIT_CHECK_EVERY
#define XPA_WAIT_CHECK_EVERY 8
#endif
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, uint64_t budget_ns) {
  if (mbar_test_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t it = 0;; ++it) {
    if (it % XPA_WAIT_CHECK_EVERY == 0 && globaltimer_ns() - t0 >= budget_ns) return false;
    if (mbar_try_wait(bar, parity)) return true;
  }
}

// Orders this thread's generic-proxy shared-memory writes before later
// async-proxy (TMA) accesses of the same bytes.
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void named_bar_sync(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// ── programmatic dependent launch ───────────────────────────────────────
// Lets a kernel launched after this one with programmatic stream
// serialisation start once every CTA of this grid has issued the trigger.
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
// Waits until the preceding grid has completed and its memory is visible
// (a no-op when the launch did not use programmatic serialisation).
__device__ __forceinline__ void pdl_wait_primary() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}

// ── TMA (tensor, tiled, no multicast) ───────────────────────────────────
__device__ __forceinline__ void tmap_prefetch(const CUtensorMap* tm) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(tm)) : "memory");
}

__device__ __forceinline__ void tma_load_4d(uint32_t dst, const CUtensorMap* tm, int c0, int c1,
                                            int c2, int c3, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4, %5}], [%6];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(tm)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(bar)
      : "memory");
}

// ── warp-level tensor-core fragments ────────────────────────────────────
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                        uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ void ldsm_x4_trans(uint32_t addr, uint32_t& r0, uint32_t& r1,
                                              uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

// D += A(16x16, row) * B(16x8, col), fp16 inputs, fp32 accumulate.
__device__ __forceinline__ void mma_f16_16816(float (&d)[4], uint32_t a0, uint32_t a1,
                                              uint32_t a2, uint32_t a3, uint32_t b0,
                                              uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7},"
      " {%8, %9}, {%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Transposes an 8x8 b16 matrix held one 32-bit pair per lane.
__device__ __forceinline__ uint32_t movmatrix_trans(uint32_t x) {
  uint32_t y;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(y) : "r"(x));
  return y;
}

__device__ __forceinline__ uint32_t pack_half2(float lo, float hi) {
  __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

__device__ __forceinline__ float2 unpack_half2(uint32_t u) {
  __half2 h = *reinterpret_cast<__half2*>(&u);
  return __half22float2(h);
}

template <typename T>
__device__ __forceinline__ float to_float(T x);
template <>
__device__ __forceinline__ float to_float<float>(float x) { return x; }
template <>
__device__ __forceinline__ float to_float<__half>(__half x) { return __half2float(x); }

template <typename T>
__device__ __forceinline__ T from_float(float x);
template <>
__device__ __forceinline__ float from_float<float>(float x) { return x; }
template <>
__device__ __forceinline__ __half from_float<__half>(float x) { return __float2half_rn(x); }


// Stores element d of output row `row` (= b * Hq + h, this launch's heads):
// into `out`, or, with the fused head gather, into every rank's buffer. The
// peer stores need no fence here: the gather barrier that publishes them runs
// only after these grids have completed, and completion flushes their writes,
// peer writes included (the guarantee CUDA's event-ordered P2P model uses).
template <typename T>
__device__ __forceinline__ void store_out(const Params& p, long long row, int d, float v) {
  const T x = from_float<T>(v);
  if (p.npeers == 0) {
    static_cast<T*>(p.out)[row * p.D + d] = x;
    return;
  }
  const long long b = row / p.Hq, h = row - b * p.Hq;
  const long long off = p.peer_off + (b * p.Hq_total + p.head_offset + h) * p.D + d;
#pragma unroll
  for (int r = 0; r < kMaxPeers; ++r)
    if (r < p.npeers) static_cast<T*>(p.peers[r])[off] = x;
}

// Stores elements d0 .. d0+7 of output row `row` with one 16-byte store (fp16)
// or two (fp32) per destination. Requires Params::vec8.
template <typename T>
__device__ __forceinline__ void store_out8(const Params& p, long long row, int d0,
                                           const float (&v)[8]) {
  long long off;
  if (p.npeers == 0) {
    off = row * p.D + d0;
  } else {
    const long long b = row / p.Hq, h = row - b * p.Hq;
    off = p.peer_off + (b * p.Hq_total + p.head_offset + h) * p.D + d0;
  }
  if constexpr (sizeof(T) == 2) {
    uint4 u;
    u.x = pack_half2(v[0], v[1]);
    u.y = pack_half2(v[2], v[3]);
    u.z = pack_half2(v[4], v[5]);
    u.w = pack_half2(v[6], v[7]);
    if (p.npeers == 0) {
      *reinterpret_cast<uint4*>(static_cast<__half*>(p.out) + off) = u;
      return;
    }
#pragma unroll
    for (int r = 0; r < kMaxPeers; ++r)
      if (r < p.npeers) *reinterpret_cast<uint4*>(static_cast<__half*>(p.peers[r]) + off) = u;
  } else {
    const float4 a = make_float4(v[0], v[1], v[2], v[3]), c = make_float4(v[4], v[5], v[6], v[7]);
    if (p.npeers == 0) {
      float4* dst = reinterpret_cast<float4*>(static_cast<float*>(p.out) + off);
      dst[0] = a;
      dst[1] = c;
      return;
    }
#pragma unroll
    for (int r = 0; r < kMaxPeers; ++r)
      if (r < p.npeers) {
        float4* dst = reinterpret_cast<float4*>(static_cast<float*>(p.peers[r]) + off);
        dst[0] = a;
        dst[1] = c;
      }
  }
}

// ── split-context merge ─────────────────────────────────────────────────
struct CtaSync {
  __device__ __forceinline__ void operator()() const { __syncthreads(); }
};

// Log-sum-exp merge of the partials of one (b, q head) row into out:
//   M = max_p m_p,  w_p = 2^(m_p - M),  out = sum_p w_p o_p / sum_p w_p l_p.
// Run by `nthr` threads (index tid) that synchronise with sync(); `sm` is
// shared scratch of cap + 34 floats (weights of the first `cap` partitions,
// the rest recomputed). Partials were written by other CTAs of the same
// launch, so they are read through L2 (ld.global.cg).
template <typename T, typename Sync>
__device__ __forceinline__ void merge_row(const Params& p, long long row, int nparts, int tid,
                                          int nthr, float* sm, int cap, Sync sync) {
  float* red = sm + cap;
  const float* ml = p.part_ml + row * p.max_parts * 2;
  const int lane = tid & 31, wid = tid >> 5, nw = (nthr + 31) >> 5;
  float mx = -INFINITY;
  for (int i = tid; i < nparts; i += nthr) mx = fmaxf(mx, __ldcg(ml + 2 * i));
  mx = warp_max(mx);
  if (lane == 0) red[wid] = mx;
  sync();
  float M = -INFINITY;
  for (int w = 0; w < nw; ++w) M = fmaxf(M, red[w]);
  float den = 0.f;
  for (int i = tid; i < nparts; i += nthr) {
    const float mp = __ldcg(ml + 2 * i);
    const float wt = (M == -INFINITY || mp == -INFINITY) ? 0.f : ex2(mp - M);
    if (i < cap) sm[i] = wt;
    den = fmaf(wt, __ldcg(ml + 2 * i + 1), den);
  }
  den = warp_sum(den);
  sync();  // every thread has read M from red[]
  if (lane == 0) red[wid] = den;
  sync();
  float tot = 0.f;
  for (int w = 0; w < nw; ++w) tot += red[w];
  const float* po = p.part_o + row * p.max_parts * p.D;
  if (p.vec8) {
    for (int c = tid; c < p.D / 8; c += nthr) {
      float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      for (int i = 0; i < nparts; ++i) {
        float wt;
        if (i < cap) {
          wt = sm[i];
        } else {
          const float mp = __ldcg(ml + 2 * i);
          wt = (M == -INFINITY || mp == -INFINITY) ? 0.f : ex2(mp - M);
        }
        const float4* src = reinterpret_cast<const float4*>(po + (long long)i * p.D + c * 8);
        const float4 a = __ldcg(src), b = __ldcg(src + 1);
        acc[0] = fmaf(wt, a.x, acc[0]);
        acc[1] = fmaf(wt, a.y, acc[1]);
        acc[2] = fmaf(wt, a.z, acc[2]);
        acc[3] = fmaf(wt, a.w, acc[3]);
        acc[4] = fmaf(wt, b.x, acc[4]);
        acc[5] = fmaf(wt, b.y, acc[5]);
        acc[6] = fmaf(wt, b.z, acc[6]);
        acc[7] = fmaf(wt, b.w, acc[7]);
      }
#pragma unroll
      for (int k = 0; k < 8; ++k) acc[k] = tot > 0.f ? acc[k] / tot : 0.f;
      store_out8<T>(p, row, c * 8, acc);
    }
  } else {
    for (int d = tid; d < p.D; d += nthr) {
      float acc = 0.f;
      for (int i = 0; i < nparts; ++i) {
        float wt;
        if (i < cap) {
          wt = sm[i];
        } else {
          const float mp = __ldcg(ml + 2 * i);
          wt = (M == -INFINITY || mp == -INFINITY) ? 0.f : ex2(mp - M);
        }
        acc = fmaf(wt, __ldcg(po + (long long)i * p.D + d), acc);
      }
      store_out<T>(p, row, d, tot > 0.f ? acc / tot : 0.f);
    }
  }
  sync();  // sm and red are reused by the next row
}

// Merges the partials of the GS query heads (rows row0 .. row0+GS-1) of one
// (sequence, KV head) at once: every
// (head, partition) max and sum is staged in shared memory in one pass, the
// weights of all heads are formed in parallel, and each output element then
// needs nparts independent loads. Falls back to merge_row per head when the
// staging does not fit in `cap` floats.
template <typename T, typename Sync>
__device__ __forceinline__ void merge_group(const Params& p, long long row0, int np, int tid,
                                            int nthr, float* sm, int cap, Sync sync) {
  const int GS = p.GS, D = p.D;
  if (2 * GS * np + GS > cap) {
    for (int h = 0; h < GS; ++h) merge_row<T>(p, row0 + h, np, tid, nthr, sm, cap, sync);
    return;
  }
  float* sw = sm;                // [GS][np]: maxima, then weights
  float* sl = sm + GS * np;      // [GS][np]: sums
  float* sinv = sl + GS * np;    // [GS]: 1 / merged sum
  for (int e = tid; e < GS * np; e += nthr) {
    const int h = e / np, i = e - h * np;
    const float* ml = p.part_ml + ((row0 + h) * p.max_parts + i) * 2;
    sw[e] = __ldcg(ml);
    sl[e] = __ldcg(ml + 1);
  }
  sync();
  for (int h = tid; h < GS; h += nthr) {
    float M = -INFINITY;
    for (int i = 0; i < np; ++i) M = fmaxf(M, sw[h * np + i]);
    float den = 0.f;
    for (int i = 0; i < np; ++i) {
      const float m = sw[h * np + i];
      const float wt = (M == -INFINITY || m == -INFINITY) ? 0.f : ex2(m - M);
      sw[h * np + i] = wt;
      den = fmaf(wt, sl[h * np + i], den);
    }
    sinv[h] = den > 0.f ? 1.f / den : 0.f;
  }
  sync();
  for (int e = tid; e < GS * D; e += nthr) {
    const int h = e / D, d = e - h * D;
    const float* po = p.part_o + (row0 + h) * p.max_parts * D + d;
    const float* w = sw + h * np;
    float acc = 0.f;
#pragma unroll 4
    for (int i = 0; i < np; ++i) acc = fmaf(w[i], __ldcg(po + (long long)i * D), acc);
    store_out<T>(p, row0 + h, d, acc * sinv[h]);
  }
}

}  // namespace xpa
