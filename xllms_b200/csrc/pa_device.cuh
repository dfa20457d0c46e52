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
  float* part_o;   // [B][Hq][slots][D] unnormalised partial outputs
  float* part_ml;  // [B][Hq][slots][2] (max in log2 units, sum of exp2)
  int* status;     // device status word (NXT_PA_DEV_* bits), may be null
  long long kv_block_stride;
  long long kv_head_stride;
  long long num_blocks;  // <= 0: unknown, no upper bound check
  unsigned long long timeout_ns;  // bound on every pipeline wait (not on the drain)
  int B, Hq, Hkv, D, GS;
  int max_blocks, block_size;
  int part_pages, max_parts;
  int slots;         // partial slots per (b, q head) row: max_parts (+ prefix chunks)
  // Shared-prefix (cascade) calls: the first prefix_pages[b] pages of sequence
  // b are covered by its prefix group's partials (slots [0, ceil(P/pp)));
  // this launch's partitions then start after them. Null: no prefix.
  const int* prefix_pages;
  int prefix_chunk;  // pages per prefix partial slot (cascade calls)
  float scale_log2;  // scale * log2(e): scores live in the exp2 domain
  // Fused head gather (KV-head sharding over GPUs): when npeers > 0 every
  // output row (b, h) of this rank is stored into each peers[r] at element
  // peer_off + (b * Hq_total + head_offset + h) * D, and `out` is unused.
  int npeers, Hq_total, head_offset;
  long long peer_off;
  void* peers[kMaxPeers];
  // Multicast address of the peers' buffers (same element offsets), or null:
  // with vec8, each 16-byte row chunk is then one multimem store that
  // NVSwitch replicates into every peer's buffer.
  void* mc;
  // 1 when D % 8 == 0 and out / peer buffers and the partial workspace are
  // 16-byte aligned: rows are then stored 8 elements (16 or 32 bytes) at a time.
  int vec8;
  // 1 when this grid was launched as a programmatic dependent of the KV
  // append kernel: a sequence's last page may only be read after
  // griddepcontrol.wait (the appended token lives there).
  int after_append;
  int join_primary;  // CTA 0 waits for the preceding grid before it exits
  // 1: no row is written by the attention kernel; rows of single-partition
  // sequences leave a one-slot partial and the merge writes every row (the
  // fused head gather keeps peer stores out of the attention kernel this way)
  int merge_all;
  // 1: this grid was launched as a programmatic dependent of whatever kernel
  // precedes the call on the stream, so that its CTAs are resident before
  // that kernel ends; every CTA waits for it (griddepcontrol.wait) before it
  // reads anything. Only the launch latency is hidden, no work overlaps.
  int wait_first;
  // Quantised KV cache: 0 = K/V in the query's dtype; kKvE4M3 / kKvE5M2 /
  // kKvInt8 = one byte per element holding encode(x / scale). k_scale is folded into
  // scale_log2; v_scale multiplies V (generic path) or O (fast path).
  int kv_fmt;
  float v_scale;
};

constexpr int kKvE4M3 = 1;
constexpr int kKvE5M2 = 2;
constexpr int kKvInt8 = 3;  // two's-complement int8, decode(c) = c

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
  // one-byte cache (kKvE4M3 / kKvE5M2 / kKvInt8): the fp16 rows are stored
  // as encode(x / k_scale) and encode(x / v_scale), rounded to nearest even
  // and saturated at the format's largest finite value. 0: bit copy.
  int kv_fmt;
  float k_scale, v_scale;
};

// One unit of work: context partition `part` of (sequence b, KV head kvh).
struct Item {
  int b, kvh, part;
  int L;            // clamped context length of sequence b
  int page_begin;   // first page of this partition
  int page_end;     // one past its last page
  int nparts;       // partitions of sequence b after its prefix (0 when none)
  int slot0;        // partial slot of partition 0 (= prefix chunks before it)
  int direct;       // the item is the whole sequence: write the output itself
};

enum ItemKind { kItemNone = 0, kItemZero = 1, kItemWork = 2 };

__device__ __forceinline__ void raise_status(const Params& p, int bits) {
  if (p.status) atomicOr(p.status, bits);
}

// Pages of sequence b (of npages) covered by its shared-prefix partials.
__device__ __forceinline__ int prefix_of(const Params& p, int b, int npages) {
  if (!p.prefix_pages) return 0;
  const int P = __ldg(p.prefix_pages + b);
  return P < 0 ? 0 : (P > npages ? npages : P);
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
  const int P = prefix_of(p, it.b, npages);
  it.nparts = (npages - P + p.part_pages - 1) / p.part_pages;
  it.slot0 = P > 0 ? (P + p.prefix_chunk - 1) / p.prefix_chunk : 0;
  it.direct = (P == 0 && it.nparts == 1 && !p.merge_all) ? 1 : 0;
  if (it.nparts == 0) return (it.part == 0 && npages == 0) ? kItemZero : kItemNone;
  if (it.part >= it.nparts) return kItemNone;
  it.page_begin = P + it.part * p.part_pages;
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

// Shared-memory byte offset of the 16-byte chunk `chunk` (along d) of token
// row `tok` in a page tile written by TMA with 128-byte swizzle: the tile is
// D/64 boxes of 16 rows x 128 bytes, and within each 1024-byte group the
// chunk index is XORed with the row index mod 8.
__device__ __forceinline__ uint32_t tile_off(int tok, int chunk) {
  return (uint32_t)((chunk >> 3) * 2048 + tok * 128 + (((chunk & 7) ^ (tok & 7)) << 4));
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

// Two one-byte codes (low byte first) -> fp16x2 (low half first); exact,
// since every E4M3, E5M2 and int8 value is an fp16 value. int8: the byte
// biased by 128 (c ^ 0x80 = c + 128 in 0..255) sits under the fp16 exponent
// of 1024, where the spacing is 1, giving 1024 + 128 + c; subtracting 1152
// is exact.
template <int FMT>
__device__ __forceinline__ uint32_t fp8x2_to_h2(uint32_t two) {
  uint32_t r;
  if constexpr (FMT == kKvInt8) {
    const uint32_t biased = __byte_perm(two ^ 0x8080u, 0x64646464u, 0x5140);
    const __half2 h = __hsub2(*reinterpret_cast<const __half2*>(&biased),
                              __halves2half2(__ushort_as_half(0x6480), __ushort_as_half(0x6480)));
    r = *reinterpret_cast<const uint32_t*>(&h);
    return r;
  }
  const unsigned short v = (unsigned short)(two & 0xffffu);
  if constexpr (FMT == kKvE4M3)
    asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(r) : "h"(v));
  else
    asm("cvt.rn.f16x2.e5m2x2 %0, %1;" : "=r"(r) : "h"(v));
  return r;
}
// Four one-byte codes (byte 0 lowest) -> two fp16x2: lo = bytes 0, 1 and
// hi = bytes 2, 3. int8 biases the whole word with one XOR.
template <int FMT>
__device__ __forceinline__ void kv8x4_to_h2x2(uint32_t w, uint32_t& lo, uint32_t& hi) {
  if constexpr (FMT == kKvInt8) {
    const uint32_t x = w ^ 0x80808080u;
    const uint32_t b0 = __byte_perm(x, 0x64646464u, 0x5140);
    const uint32_t b1 = __byte_perm(x, 0x64646464u, 0x7362);
    const __half2 off = __halves2half2(__ushort_as_half(0x6480), __ushort_as_half(0x6480));
    const __half2 h0 = __hsub2(*reinterpret_cast<const __half2*>(&b0), off);
    const __half2 h1 = __hsub2(*reinterpret_cast<const __half2*>(&b1), off);
    lo = *reinterpret_cast<const uint32_t*>(&h0);
    hi = *reinterpret_cast<const uint32_t*>(&h1);
  } else {
    lo = fp8x2_to_h2<FMT>(w);
    hi = fp8x2_to_h2<FMT>(w >> 16);
  }
}
// Four one-byte codes -> the fp16x2 pairs (byte 0, byte 2) and (byte 1,
// byte 3), low half first.
template <int FMT>
__device__ __forceinline__ void kv8x4_to_h2_even_odd(uint32_t w, uint32_t& even, uint32_t& odd) {
  if constexpr (FMT == kKvInt8) {
    const uint32_t x = w ^ 0x80808080u;
    const uint32_t b0 = __byte_perm(x, 0x64646464u, 0x4240);
    const uint32_t b1 = __byte_perm(x, 0x64646464u, 0x4341);
    const __half2 off = __halves2half2(__ushort_as_half(0x6480), __ushort_as_half(0x6480));
    const __half2 h0 = __hsub2(*reinterpret_cast<const __half2*>(&b0), off);
    const __half2 h1 = __hsub2(*reinterpret_cast<const __half2*>(&b1), off);
    even = *reinterpret_cast<const uint32_t*>(&h0);
    odd = *reinterpret_cast<const uint32_t*>(&h1);
  } else {
    const uint32_t t = __byte_perm(w, 0u, 0x3120);  // bytes 0, 2 | 1, 3
    even = fp8x2_to_h2<FMT>(t);
    odd = fp8x2_to_h2<FMT>(t >> 16);
  }
}
template <int FMT>
__device__ __forceinline__ float fp8_to_float(uint8_t b) {
  if constexpr (FMT == kKvInt8) return (float)(signed char)b;
  const uint32_t h2 = fp8x2_to_h2<FMT>(b);
  return __half2float(__ushort_as_half((unsigned short)(h2 & 0xffffu)));
}
// (a, b) -> two one-byte codes, a in the low byte; round to nearest even,
// saturating at the largest finite value (fp8: NaN stays NaN; int8: the
// range is [-128, 127] and NaN gives 0).
template <int FMT>
__device__ __forceinline__ uint32_t float2_to_fp8x2(float a, float b) {
  if constexpr (FMT == kKvInt8) {
    const int ia = min(max(__float2int_rn(a), -128), 127);
    const int ib = min(max(__float2int_rn(b), -128), 127);
    return ((uint32_t)ia & 0xffu) | (((uint32_t)ib & 0xffu) << 8);
  }
  unsigned short r;
  // the first source operand lands in the upper byte
  if constexpr (FMT == kKvE4M3)
    asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(b), "f"(a));
  else
    asm("cvt.rn.satfinite.e5m2x2.f32 %0, %1, %2;" : "=h"(r) : "f"(b), "f"(a));
  return r;
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

// One 16-byte store through a multicast address: NVSwitch writes it into
// every buffer bound to the multicast object (relaxed, system scope; the
// gather barrier's release / acquire orders it for the readers).
__device__ __forceinline__ void multimem_st16(void* mc_addr, uint4 u) {
  asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(mc_addr),
               "r"(u.x), "r"(u.y), "r"(u.z), "r"(u.w)
               : "memory");
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
    if (p.mc) {
      multimem_st16(static_cast<__half*>(p.mc) + off, u);
      return;
    }
#pragma unroll
    for (int r = 0; r < kMaxPeers; ++r)
      if (r < p.npeers) *reinterpret_cast<uint4*>(static_cast<__half*>(p.peers[r]) + off) = u;
  } else {
    const float4 a = make_float4(v[0], v[1], v[2], v[3]), c = make_float4(v[4], v[5], v[6], v[7]);
    if (p.npeers > 0 && p.mc) {
      float* dst = static_cast<float*>(p.mc) + off;
      multimem_st16(dst, make_uint4(__float_as_uint(a.x), __float_as_uint(a.y),
                                    __float_as_uint(a.z), __float_as_uint(a.w)));
      multimem_st16(dst + 4, make_uint4(__float_as_uint(c.x), __float_as_uint(c.y),
                                        __float_as_uint(c.z), __float_as_uint(c.w)));
      return;
    }
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
// Log-sum-exp merge of the partials (slots) of one (b, q head) row into out,
// by one warp:
//   M = max_i m_i,  w_i = 2^(m_i - M),  out = sum_i w_i o_i / sum_i w_i l_i.
// Lane i holds slot i's (m, l) (slots past 32 are re-read from L2); the
// weights of the first 32 slots go to the warp's 32 floats of shared memory
// `sw`. Each lane then accumulates 4 consecutive output elements (1 without
// vec8) over the slots, four slots' loads in flight at a time; with vec8 the
// even lane of each pair stores the pair's 8 elements in one 16-byte store. Partials were
// written by other CTAs, so they are read through L2 (ld.global.cg).
template <typename T>
__device__ __forceinline__ void merge_row_warp(const Params& p, long long row, int nslots,
                                               int lane, float* sw) {
  const float2* ml = reinterpret_cast<const float2*>(p.part_ml) + row * p.slots;
  const float2 mine = lane < nslots ? __ldcg(ml + lane) : make_float2(-INFINITY, 0.f);
  float mx = mine.x;
  for (int i = lane + 32; i < nslots; i += 32) mx = fmaxf(mx, __ldcg(&ml[i].x));
  const float M = warp_max(mx);
  auto weight = [M](float m) { return (M == -INFINITY || m == -INFINITY) ? 0.f : ex2(m - M); };
  const float wm = weight(mine.x);
  sw[lane] = wm;
  float den = wm * mine.y;
  for (int i = lane + 32; i < nslots; i += 32) {
    const float2 x = __ldcg(ml + i);
    den = fmaf(weight(x.x), x.y, den);
  }
  const float tot = warp_sum(den);  // also orders sw[] for the whole warp
  __syncwarp();
  auto wt = [&](int i) { return i < 32 ? sw[i] : weight(__ldcg(&ml[i].x)); };
  const float* po = p.part_o + row * p.slots * p.D;
  if (p.vec8) {
    // Every lane runs every 128-element pass (lanes past D load nothing), so
    // the pair shuffles below have the whole warp.
    for (int base = 0; base < p.D; base += 128) {
      const int d0 = base + lane * 4;
      const bool act = d0 < p.D;
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
      if (act) {
        int i = 0;
        for (; i + 4 <= nslots; i += 4) {
          float4 x[4];
#pragma unroll
          for (int u = 0; u < 4; ++u)
            x[u] = __ldcg(reinterpret_cast<const float4*>(po + (long long)(i + u) * p.D + d0));
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const float w = wt(i + u);
            acc.x = fmaf(w, x[u].x, acc.x);
            acc.y = fmaf(w, x[u].y, acc.y);
            acc.z = fmaf(w, x[u].z, acc.z);
            acc.w = fmaf(w, x[u].w, acc.w);
          }
        }
        for (; i < nslots; ++i) {
          const float4 x = __ldcg(reinterpret_cast<const float4*>(po + (long long)i * p.D + d0));
          const float w = wt(i);
          acc.x = fmaf(w, x.x, acc.x);
          acc.y = fmaf(w, x.y, acc.y);
          acc.z = fmaf(w, x.z, acc.z);
          acc.w = fmaf(w, x.w, acc.w);
        }
        if (tot > 0.f) {
          acc.x /= tot;
          acc.y /= tot;
          acc.z /= tot;
          acc.w /= tot;
        } else {
          acc = make_float4(0.f, 0.f, 0.f, 0.f);
        }
      }
      // even lanes take their odd neighbour's 4 elements and store 8 at once
      // (16-byte stores: half the transactions, which counts most for the
      // peer stores of the fused head gather); D % 8 == 0 keeps pairs whole
      const float4 nb = make_float4(__shfl_down_sync(0xffffffffu, acc.x, 1),
                                    __shfl_down_sync(0xffffffffu, acc.y, 1),
                                    __shfl_down_sync(0xffffffffu, acc.z, 1),
                                    __shfl_down_sync(0xffffffffu, acc.w, 1));
      if (act && (lane & 1) == 0) {
        const float v8[8] = {acc.x, acc.y, acc.z, acc.w, nb.x, nb.y, nb.z, nb.w};
        store_out8<T>(p, row, d0, v8);
      }
    }
  } else {
    for (int d = lane; d < p.D; d += 32) {
      float acc = 0.f;
#pragma unroll 4
      for (int i = 0; i < nslots; ++i) acc = fmaf(wt(i), __ldcg(po + (long long)i * p.D + d), acc);
      store_out<T>(p, row, d, tot > 0.f ? acc / tot : 0.f);
    }
  }
}

}  // namespace xpa
