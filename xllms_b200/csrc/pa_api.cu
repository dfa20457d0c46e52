// pa_api.cu — the C ABI of libxpa.so (include/operator_api.h): argument
// checks, launch planning, tensor-map encoding, library-owned workspaces and
// status words, and the drop-in entry points.
#include <cudaTypedefs.h>

#include <climits>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <map>
#include <algorithm>
#include <cmath>
#include <mutex>
#include <thread>
#include <functional>
#include <utility>

#include "operator_api.h"
#include "pa_host.h"
#include "pa_launch.h"
#include "pa_prefix.h"

static_assert(NXT_KV_FP8_E4M3 == xpa::kKvE4M3 && NXT_KV_FP8_E5M2 == xpa::kKvE5M2 &&
                  NXT_KV_INT8 == xpa::kKvInt8,
              "one-byte KV format codes");

namespace {

thread_local int g_last_error = NXT_PA_OK;
thread_local cudaEvent_t g_prof_before = nullptr;  // one-shot timing events
thread_local cudaEvent_t g_prof_after = nullptr;
thread_local cudaEvent_t g_prof_merged = nullptr;

constexpr unsigned long long kWaitBudgetNs = 1000000000ull;  // 1 s per pipeline wait
thread_local unsigned long long g_wait_budget_ns = kWaitBudgetNs;
constexpr int kMaxDevices = 64;

std::mutex g_mu;

struct DeviceState {
  bool probed = false;
  int sm_count = 0;
  int* status = nullptr;  // library status word
};
DeviceState g_dev[kMaxDevices];

// Map key of a stream. The per-thread default stream has one handle for
// every host thread but is a different stream in each, so it is told apart
// by the thread.
uintptr_t stream_key(cudaStream_t st) {
  if (st == cudaStreamPerThread)
    return (static_cast<uintptr_t>(std::hash<std::thread::id>{}(std::this_thread::get_id()))
            << 4) | 0xfu;
  return reinterpret_cast<uintptr_t>(st);
}

struct Workspace {
  void* ptr = nullptr;  // split-context partials
  size_t bytes = 0;
};
// Keyed by (device, stream) so calls on different streams never share partials.
std::map<std::pair<int, uintptr_t>, Workspace> g_ws;

int map_cuda(cudaError_t e) { return e == cudaSuccess ? NXT_PA_OK : NXT_PA_ECUDA; }

}  // namespace

namespace xpa {
namespace host {

int ceil_div(long long a, long long b) { return (int)((a + b - 1) / b); }

unsigned long long wait_budget_ns() { return g_wait_budget_ns; }

}  // namespace host
}  // namespace xpa

namespace {

// Per-device facts; status word allocated on first use. Caller holds g_mu.
int device_state_locked(int dev, DeviceState** out) {
  if (dev < 0 || dev >= kMaxDevices) return NXT_PA_EINVAL;
  DeviceState& d = g_dev[dev];
  if (!d.probed) {
    int sms = 0;
    cudaError_t e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return NXT_PA_ECUDA;
    d.sm_count = sms;
    d.probed = true;
  }
  if (!d.status) {
    void* p = nullptr;
    if (cudaMalloc(&p, 256) != cudaSuccess) return NXT_PA_ENOMEM;
    if (cudaMemset(p, 0, 256) != cudaSuccess) {
      cudaFree(p);
      return NXT_PA_ECUDA;
    }
    d.status = static_cast<int*>(p);
  }
  *out = &d;
  return NXT_PA_OK;
}

}  // namespace

namespace xpa {
namespace host {

int sm_count_of(int dev) {
  std::lock_guard<std::mutex> lk(g_mu);
  if (dev < 0 || dev >= kMaxDevices) return 148;
  DeviceState& d = g_dev[dev];
  if (!d.probed) {
    int sms = 0;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
      return 148;
    d.sm_count = sms;
    d.probed = true;
  }
  return d.sm_count;
}

// Sharded calls on several GPUs: 1 = every output row is stored (to every
// peer) by the merge kernel, 0 = single-partition rows by the attention kernel.
#ifndef XPA_SHARD_MERGE_ALL
#define XPA_SHARD_MERGE_ALL 1
#endif

// 1: the first attention kernel of a plain call is launched as a
// programmatic dependent of the stream's previous kernel and waits for it
// before reading anything (hides its launch latency); 0: an ordinary launch.
#ifndef XPA_EARLY_LAUNCH
#define XPA_EARLY_LAUNCH 1
#endif

// Partition size: XPA_PART_PAGES by default, halved (down to 4 pages) while
// the grid would hold fewer than XPA_MIN_ITEMS_PER_SM items per SM, and
// doubled while a row would have more than 8192 partitions.
// Default partition length in pages (128 pages = 2048 tokens at page size 16);
// a build may override it with -DXPA_PART_PAGES=n for tuning sweeps.
#ifndef XPA_PART_PAGES
#define XPA_PART_PAGES 128
#endif

// Items per SM before partitions stop shrinking: 24 (four per resident
// fp16 CTA). A CTA streams a 128-page item in ~140 us when every slot is
// busy, so with few, long items per slot the grid's last items run on a
// half-idle GPU. Measured on B200 over five seeded config-2 batches:
// 128-page partitions (the old floor of 12 items per SM) gave 0.91-1.01 of
// the copy peak, 64-page ones 0.99-1.00, on 1 GPU and on an 8-GPU shard.
#ifndef XPA_MIN_ITEMS_PER_SM
#define XPA_MIN_ITEMS_PER_SM 24
#endif
// fp8 pages stream in half the time, so the grid needs more CTAs per SM
// before partitions stop shrinking.
#ifndef XPA_FP8_MIN_ITEMS_PER_SM
#define XPA_FP8_MIN_ITEMS_PER_SM 24
#endif
Plan make_plan(int B, int Hq, int D, int Hkv, int max_blocks, int nsm, int kv_es) {
  Plan pl;
  const long long mb = max_blocks > 0 ? max_blocks : 1;
  int pp = XPA_PART_PAGES;
  const long long min_items =
      (long long)(kv_es == 1 ? XPA_FP8_MIN_ITEMS_PER_SM : XPA_MIN_ITEMS_PER_SM) * nsm;
  while (pp > 4 && (long long)B * Hkv * ceil_div(mb, pp) < min_items) pp >>= 1;
  while (ceil_div(mb, pp) > 8192) pp <<= 1;
  pl.part_pages = pp;
  pl.max_parts = ceil_div(mb, pp);
  if (pl.max_parts > 1) pl.ws_bytes = partial_bytes((long long)B * Hq * pl.max_parts, D);
  return pl;
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static std::once_flag once;
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  });
  return fn;
}

// One pool (K or V) as a 4-D fp16 tensor {d, slot, kv head, page}, boxed
// 64 x 16 x 1 x 1 with 128-byte swizzle. An unknown pool size uses the
// largest page coordinate TMA accepts.
bool encode_pool(CUtensorMap* m, const void* base, int D, int Hkv, long long num_blocks,
                 long long kbs, long long khs, int es) {
  auto fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[4] = {(cuuint64_t)D, 16u, (cuuint64_t)Hkv,
                        (cuuint64_t)(num_blocks > 0 ? num_blocks : (long long)INT_MAX)};
  cuuint64_t strides[3] = {(cuuint64_t)D * es, (cuuint64_t)khs * es, (cuuint64_t)kbs * es};
  // one box row = 128 bytes (64 fp16 or 128 fp8 elements), the 128-byte swizzle span
  cuuint32_t box[4] = {(cuuint32_t)(128 / es), 16u, 1u, 1u};
  cuuint32_t estr[4] = {1u, 1u, 1u, 1u};
  const CUtensorMapDataType dt =
      es == 1 ? CU_TENSOR_MAP_DATA_TYPE_UINT8 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  auto encode = [&] {
    return fn(m, dt, 4, const_cast<void*>(base), dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  };
  CUresult r = encode();
  if (r != CUDA_SUCCESS) {
    // A host thread whose first CUDA call this is has no current context
    // yet, and the driver call fails without one: bind the current device's
    // primary context (what the runtime's own first call would do) and
    // encode again, so that such a call still takes the TMA path.
    int dev = 0;
    if (cudaGetDevice(&dev) == cudaSuccess && cudaSetDevice(dev) == cudaSuccess) r = encode();
  }
  return r == CUDA_SUCCESS;
}

bool fast_layout_ok(const void* k, const void* v, int D, int Hkv, long long kbs, long long khs,
                    int es) {
  const uintptr_t a = reinterpret_cast<uintptr_t>(k), b = reinterpret_cast<uintptr_t>(v);
  if ((a | b) & 15u) return false;
  if ((kbs * es) % 16 || (khs * es) % 16) return false;
  if (khs < 16LL * D) return false;             // a page's slots are contiguous rows
  if (Hkv > 1 && kbs < khs * Hkv && khs != 0) {
    // Non-standard order (heads outermost): tensor-map strides may then not
    // be increasing; leave such pools to the generic kernel.
    return false;
  }
  return true;
}

int check_args(const void* out, const void* q, const void* k, const void* v, const int* bt,
               const int* sl, int B, int Hq, int D, int Hkv, int max_blocks, int bs, int ds,
               long long kbs, long long khs) {
  if (B < 0) return NXT_PA_EINVAL;
  if (B == 0) return NXT_PA_OK;
  if (!out || !q || !k || !v || !bt || !sl) return NXT_PA_EINVAL;
  if (Hq <= 0 || Hkv <= 0 || Hq % Hkv) return NXT_PA_EINVAL;
  if (D <= 0 || D > 256) return NXT_PA_EINVAL;
  if (ds != 2 && ds != 4) return NXT_PA_EINVAL;
  if (bs <= 0 || max_blocks < 0) return NXT_PA_EINVAL;
  if (kbs < 0 || khs < 0) return NXT_PA_EINVAL;
  return NXT_PA_OK;
}

}  // namespace host
}  // namespace xpa

using namespace xpa::host;

namespace {

// Shared-prefix groups of a cascade call (device arrays, host sizes).
struct PrefixArgs {
  const int* prefix_pages;
  const int* offsets;
  const int* members;
  int num_groups, max_group_size, max_prefix_pages;
};

#ifndef XPA_PREFIX_CTA_SCALE
#define XPA_PREFIX_CTA_SCALE 2.0
#endif
// CTAs of the persistent shared-prefix kernel, which runs beside the suffix
// kernel: enough that its estimated work (S blocks of 64 tokens x 128 rows at
// ~1.2 us each on one SM) ends within the suffix kernel's estimated HBM time
// (half the non-prefix pages of every sequence at 6 TB/s), at least 8.
int prefix_ctas(int B, int Hq, int D, int Hkv, int max_blocks, int num_groups,
                int max_group_size, int max_prefix_pages, int sm_count) {
  const double blocks = (double)num_groups * Hkv * ceil_div((long long)max_group_size * (Hq / Hkv), 128) *
                        ceil_div(max_prefix_pages, 4);
  const double work_us = blocks * 1.2;
  const double suffix_pages = std::max(1.0, 0.5 * (max_blocks - max_prefix_pages));
  const double suffix_us =
      std::max(1.0, (double)B * Hkv * suffix_pages * (16.0 * D * 2 * 2) / 6.0e6);
  const int n = (int)std::ceil(XPA_PREFIX_CTA_SCALE * work_us / suffix_us);
  return std::min(sm_count, std::max(8, n));
}

// Pages per prefix partial slot. The floor, which the workspace query sizes
// for: short chunks (at most 64, each within the prefix kernel's 512 pages),
// so the prefix kernel has items enough. Given the items one chunk index
// yields (`items_per_chunk`: groups x KV heads x 128-row query blocks) and the
// prefix grid (`ctas`), a call then takes chunks twice as long while the grid
// keeps at least one item per CTA: fewer partial slots for the merge to read
// (config 4 on B200: 16-page chunks 0.1177 ms, 32: 0.1118, 64: 0.1105,
// 128: 0.1089).
#ifndef XPA_PREFIX_CHUNK_PAGES
#define XPA_PREFIX_CHUNK_PAGES 16
#endif
int prefix_chunk_pages(int max_prefix_pages, long long items_per_chunk = 0, int ctas = 0) {
  int cp = XPA_PREFIX_CHUNK_PAGES;
  while (ceil_div(max_prefix_pages, cp) > 64 && cp < 512) cp <<= 1;
  while (items_per_chunk > 0 && cp < 512 && cp < max_prefix_pages &&
         items_per_chunk * ceil_div(max_prefix_pages, 2 * cp) >= ctas)
    cp <<= 1;
  return cp;
}

// Quantised KV cache of a one-byte (fp8 / int8) call.
struct KvQuant {
  int fmt;  // xpa::kKvE4M3, xpa::kKvE5M2 or xpa::kKvInt8
  float k_scale, v_scale;
};

int run(void* out, const void* q, const void* k, const void* v, const int* bt, const int* sl,
        int B, int Hq, int D, int Hkv, float scale, int max_blocks, int bs, int ds,
        long long kbs, long long khs, long long num_blocks, void* ws, size_t ws_bytes,
        int* dev_status, cudaStream_t st, const NxtPaShard* shard = nullptr,
        uint64_t step = 0, bool after_append = false, const PrefixArgs* pre = nullptr,
        const KvQuant* kvq = nullptr) {
  if (shard) {
    if (shard->world_size < 1 || shard->world_size > NXT_PA_MAX_PEERS || shard->rank < 0 ||
        shard->rank >= shard->world_size || step == 0 || shard->head_offset < 0 ||
        (long long)shard->head_offset + Hq > shard->total_heads)
      return NXT_PA_EINVAL;
    for (int r = 0; r < shard->world_size; ++r)
      if (!shard->peer_out[r] || !shard->peer_flags[r]) return NXT_PA_EINVAL;
    if (reinterpret_cast<uintptr_t>(shard->mc_out) & 15u) return NXT_PA_EINVAL;
    out = shard->peer_out[shard->rank];
  }
  int rc = check_args(out, q, k, v, bt, sl, B, Hq, D, Hkv, max_blocks, bs, ds, kbs, khs);
  if (rc != NXT_PA_OK || B == 0) return rc;
  if (ws && !workspace_aligned(ws)) return NXT_PA_EINVAL;
  const int kv_fmt = kvq ? kvq->fmt : 0;
  const int kv_es = kvq ? 1 : ds;
  if (kvq) {
    if ((kvq->fmt != xpa::kKvE4M3 && kvq->fmt != xpa::kKvE5M2 && kvq->fmt != xpa::kKvInt8) ||
        ds != 2 ||
        !(kvq->k_scale > 0.f) || !(kvq->v_scale > 0.f) || !std::isfinite(kvq->k_scale) ||
        !std::isfinite(kvq->v_scale))
      return NXT_PA_EINVAL;
    pre = nullptr;  // the shared-prefix kernels read fp16 caches only
  }

  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return NXT_PA_ECUDA;
  const int sms = sm_count_of(dev);
  Plan pl = make_plan(B, Hq, D, Hkv, max_blocks, sms, kv_es);
  // A cascade call needs the TMA path's shapes; others run without the prefix
  // information, which gives the same result.
  CUtensorMap tk, tv;
  const bool fast = xpa::fast_path_shape_ok(D, Hq / Hkv, bs, ds, kv_fmt) &&
                    fast_layout_ok(k, v, D, Hkv, kbs, khs, kv_es) &&
                    (reinterpret_cast<uintptr_t>(q) & (kv_fmt ? 7u : 3u)) == 0 &&
                    encode_pool(&tk, k, D, Hkv, num_blocks, kbs, khs, kv_es) &&
                    encode_pool(&tv, v, D, Hkv, num_blocks, kbs, khs, kv_es);
  if (pre && (!fast || pre->num_groups <= 0 || pre->max_prefix_pages <= 0 ||
              pre->max_group_size <= 0))
    pre = nullptr;
  int slots = pl.max_parts, pchunk = 1, pchunks = 0;
  if (pre) {
    if (!pre->prefix_pages || !pre->offsets || !pre->members) return NXT_PA_EINVAL;
    // longer chunks only for the tcgen05 prefix kernel (head sizes 64, 128)
    const long long items_per_chunk =
        (D == 64 || D == 128)
            ? (long long)pre->num_groups * Hkv *
                  ceil_div((long long)pre->max_group_size * (Hq / Hkv), 128)
            : 0;
    pchunk = prefix_chunk_pages(pre->max_prefix_pages, items_per_chunk,
                                prefix_ctas(B, Hq, D, Hkv, max_blocks, pre->num_groups,
                                            pre->max_group_size, pre->max_prefix_pages, sms));
    pchunks = ceil_div(pre->max_prefix_pages, pchunk);
    slots = pl.max_parts + pchunks;
    pl.ws_bytes = partial_bytes((long long)B * Hq * slots, D);
  }
  // Sharded calls over several GPUs store every row through the merge, so
  // the attention kernel's CTAs never wait on stores to peers' memory.
  const bool merge_all = shard && shard->world_size > 1 && XPA_SHARD_MERGE_ALL;
  if (merge_all && pl.ws_bytes == 0) pl.ws_bytes = partial_bytes((long long)B * Hq * slots, D);
  if ((long long)B * Hkv * pl.max_parts > INT_MAX || (long long)B * Hq > INT_MAX)
    return NXT_PA_EINVAL;

  int* status = dev_status;
  void* part = ws;
  // A library-owned workspace stays locked until this call's kernels are
  // enqueued: another host thread on the same stream could otherwise grow
  // (free) it between the lookup and the launches. Nothing below takes g_mu.
  std::unique_lock<std::mutex> lk(g_mu);
  if (!status) {
    DeviceState* d = nullptr;
    rc = device_state_locked(dev, &d);
    if (rc != NXT_PA_OK) return rc;
    status = d->status;
  }
  if (pl.ws_bytes > 0) {
    if (ws) {
      if (ws_bytes < pl.ws_bytes) return NXT_PA_EWORKSPACE;
    } else {
      Workspace& w = g_ws[{dev, stream_key(st)}];
      if (w.bytes < pl.ws_bytes) {
        if (w.ptr) cudaFree(w.ptr);  // synchronises: no kernel still reads it
        w.ptr = nullptr;
        w.bytes = 0;
        if (cudaMalloc(&w.ptr, pl.ws_bytes) != cudaSuccess) return NXT_PA_ENOMEM;
        w.bytes = pl.ws_bytes;
      }
      part = w.ptr;
    }
  }
  if (part == ws) lk.unlock();  // caller-owned (or no) workspace

  xpa::Params p{};
  p.out = out;
  p.q = q;
  p.k = k;
  p.v = v;
  p.block_tables = bt;
  p.seq_lens = sl;
  p.part_o = static_cast<float*>(part);
  p.part_ml = part ? reinterpret_cast<float*>(static_cast<char*>(part) +
                                              part_ml_offset_bytes((long long)B * Hq * slots, D))
                   : nullptr;
  p.status = status;
  p.kv_block_stride = kbs;
  p.kv_head_stride = khs;
  p.num_blocks = num_blocks;
  p.timeout_ns = g_wait_budget_ns;
  p.B = B;
  p.Hq = Hq;
  p.Hkv = Hkv;
  p.D = D;
  p.GS = Hq / Hkv;
  p.max_blocks = max_blocks;
  p.block_size = bs;
  p.part_pages = pl.part_pages;
  p.max_parts = pl.max_parts;
  p.slots = slots;
  p.prefix_pages = pre ? pre->prefix_pages : nullptr;
  p.prefix_chunk = pchunk;
  p.scale_log2 = scale * (kvq ? kvq->k_scale : 1.f) * 1.4426950408889634f;
  p.kv_fmt = kv_fmt;
  p.v_scale = kvq ? kvq->v_scale : 1.f;
  p.after_append = after_append ? 1 : 0;
  p.merge_all = merge_all ? 1 : 0;
  // The first kernel of a plain call (not after an append, not a cascade)
  // becomes resident while the stream's previous kernel finishes.
  p.wait_first = (!pre && !after_append && XPA_EARLY_LAUNCH) ? 1 : 0;
  {
    auto a16 = [](const void* x) { return (reinterpret_cast<uintptr_t>(x) & 15u) == 0; };
    bool ok = D % 8 == 0 && a16(part);
    if (shard) {
      for (int r = 0; r < shard->world_size; ++r) ok = ok && a16(shard->peer_out[r]);
    } else {
      ok = ok && a16(out);
    }
    p.vec8 = ok ? 1 : 0;
  }
  if (shard) {
    p.npeers = shard->world_size;
    p.Hq_total = shard->total_heads;
    p.head_offset = shard->head_offset;
    p.peer_off = (long long)(step & 1) * B * shard->total_heads * D;
    for (int r = 0; r < shard->world_size; ++r) p.peers[r] = shard->peer_out[r];
    p.mc = shard->world_size > 1 ? shard->mc_out : nullptr;
  }

  cudaEvent_t ev_a = g_prof_before, ev_b = g_prof_after, ev_c = g_prof_merged;
  g_prof_before = g_prof_after = g_prof_merged = nullptr;
  if (ev_a && cudaEventRecord(ev_a, st) != cudaSuccess) return NXT_PA_ECUDA;
  cudaError_t e;
  if (pre) {
    xpa::PrefixGroups pg{};
    pg.offsets = pre->offsets;
    pg.members = pre->members;
    pg.num_groups = pre->num_groups;
    pg.max_group_size = pre->max_group_size;
    pg.max_chunks = pchunks;
    if (xpa::prefix_tc_ok(p)) {
      // The persistent tcgen05 prefix kernel (compute-bound, one CTA per SM)
      // takes a few SMs; the suffix kernel, launched as its programmatic
      // dependent, starts at once and streams HBM on the others. CTA 0 of
      // the suffix kernel waits for the prefix grid before exiting, so the
      // merge (dependent of the suffix kernel) sees both.
      const int ctas = prefix_ctas(B, Hq, D, Hkv, max_blocks, pre->num_groups,
                                   pre->max_group_size, pre->max_prefix_pages, sms);
      e = xpa::launch_prefix(tk, tv, p, pg, ctas, st);
      if (e != cudaSuccess) return map_cuda(e);
      xpa::Params ps = p;
      ps.join_primary = 1;
      e = xpa::launch_fast(tk, tv, ps, st);
      if (e != cudaSuccess) return map_cuda(e);
    } else {
      e = xpa::launch_prefix(tk, tv, p, pg, sms, st);
      if (e != cudaSuccess) return map_cuda(e);
      e = xpa::launch_fast(tk, tv, p, st);
      if (e != cudaSuccess) return map_cuda(e);
    }
  } else {
    e = fast ? xpa::launch_fast(tk, tv, p, st) : xpa::launch_generic(p, ds, st);
    if (e != cudaSuccess) return map_cuda(e);
  }
  if (ev_b && cudaEventRecord(ev_b, st) != cudaSuccess) return NXT_PA_ECUDA;
  if (pl.max_parts > 1 || pre || merge_all) {
    e = xpa::launch_reduce(p, ds, st);
    if (e != cudaSuccess) return map_cuda(e);
  }
  if (ev_c && cudaEventRecord(ev_c, st) != cudaSuccess) return NXT_PA_ECUDA;
  if (shard) {
    e = xpa::launch_peer_barrier(reinterpret_cast<void* const*>(shard->peer_flags),
                                 shard->world_size, shard->rank, step, status, g_wait_budget_ns,
                                 st);
    if (e != cudaSuccess) return map_cuda(e);
  }
  return NXT_PA_OK;
}

void dropin(void* out, const void* q, const void* k, const void* v, const int* bt, const int* sl,
            int B, int Hq, int D, int Hkv, float scale, int max_blocks, int bs, int ds, int kbs,
            int khs, nxt_stream_t stream) {
  g_last_error = run(out, q, k, v, bt, sl, B, Hq, D, Hkv, scale, max_blocks, bs, ds, kbs, khs,
                     -1, nullptr, 0, nullptr, static_cast<cudaStream_t>(stream));
}

}  // namespace

extern "C" {

void nxt_paged_attention(void* out, const void* query, const void* key_cache,
                         const void* value_cache, const int* block_tables, const int* seq_lens,
                         int num_seqs, int num_heads, int head_size, int num_kv_heads,
                         float scale, int max_num_blocks_per_seq, int block_size, int dtype_size,
                         int kv_block_stride, int kv_head_stride, nxt_stream_t stream) {
  dropin(out, query, key_cache, value_cache, block_tables, seq_lens, num_seqs, num_heads,
         head_size, num_kv_heads, scale, max_num_blocks_per_seq, block_size, dtype_size,
         kv_block_stride, kv_head_stride, stream);
}

void nxt_paged_attention_v2(void* out, const void* query, const void* key_cache,
                            const void* value_cache, const int* block_tables,
                            const int* seq_lens, int num_seqs, int num_heads, int head_size,
                            int num_kv_heads, float scale, int max_num_blocks_per_seq,
                            int block_size, int dtype_size, int kv_block_stride,
                            int kv_head_stride, nxt_stream_t stream) {
  dropin(out, query, key_cache, value_cache, block_tables, seq_lens, num_seqs, num_heads,
         head_size, num_kv_heads, scale, max_num_blocks_per_seq, block_size, dtype_size,
         kv_block_stride, kv_head_stride, stream);
}

void nxt_paged_attention_flash(void* out, const void* query, const void* key_cache,
                               const void* value_cache, const int* block_tables,
                               const int* seq_lens, int num_seqs, int num_heads, int head_size,
                               int num_kv_heads, float scale, int max_num_blocks_per_seq,
                               int block_size, int dtype_size, int kv_block_stride,
                               int kv_head_stride, nxt_stream_t stream) {
  dropin(out, query, key_cache, value_cache, block_tables, seq_lens, num_seqs, num_heads,
         head_size, num_kv_heads, scale, max_num_blocks_per_seq, block_size, dtype_size,
         kv_block_stride, kv_head_stride, stream);
}

int nxt_paged_attention_last_error(void) { return g_last_error; }

const char* nxt_paged_attention_strerror(int code) {
  switch (code) {
    case NXT_PA_OK: return "ok";
    case NXT_PA_EINVAL: return "unsupported or inconsistent arguments";
    case NXT_PA_ENOMEM: return "workspace allocation failed";
    case NXT_PA_EWORKSPACE: return "workspace smaller than required";
    case NXT_PA_ECUDA: return "CUDA call failed";
    case NXT_PA_ESCRATCH: return "request needs more split-context scratch than the no-alloc array holds";
    default: return "unknown status";
  }
}

int nxt_paged_attention_ex(void* out, const void* query, const void* key_cache,
                           const void* value_cache, const int* block_tables, const int* seq_lens,
                           int num_seqs, int num_heads, int head_size, int num_kv_heads,
                           float scale, int max_num_blocks_per_seq, int block_size,
                           int dtype_size, int64_t kv_block_stride, int64_t kv_head_stride,
                           int64_t num_blocks, void* workspace, size_t workspace_bytes,
                           int* device_status, nxt_stream_t stream) {
  return run(out, query, key_cache, value_cache, block_tables, seq_lens, num_seqs, num_heads,
             head_size, num_kv_heads, scale, max_num_blocks_per_seq, block_size, dtype_size,
             kv_block_stride, kv_head_stride, num_blocks, workspace, workspace_bytes,
             device_status, static_cast<cudaStream_t>(stream));
}

size_t nxt_paged_attention_workspace_size(int num_seqs, int num_heads, int head_size,
                                          int num_kv_heads, int max_num_blocks_per_seq,
                                          int block_size, int dtype_size) {
  (void)block_size;
  (void)dtype_size;
  if (num_seqs <= 0 || num_heads <= 0 || num_kv_heads <= 0 || head_size <= 0) return 0;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) dev = -1;
  return make_plan(num_seqs, num_heads, head_size, num_kv_heads, max_num_blocks_per_seq,
                   sm_count_of(dev))
      .ws_bytes;
}

size_t nxt_paged_attention_fp8_workspace_size(int num_seqs, int num_heads, int head_size,
                                              int num_kv_heads, int max_num_blocks_per_seq,
                                              int block_size) {
  (void)block_size;
  if (num_seqs <= 0 || num_heads <= 0 || num_kv_heads <= 0 || head_size <= 0) return 0;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) dev = -1;
  return make_plan(num_seqs, num_heads, head_size, num_kv_heads, max_num_blocks_per_seq,
                   sm_count_of(dev), 1)
      .ws_bytes;
}

int nxt_paged_attention_path(const void* key_cache, const void* value_cache, int num_heads,
                             int head_size, int num_kv_heads, int block_size, int dtype_size,
                             int64_t kv_block_stride, int64_t kv_head_stride) {
  if (num_heads <= 0 || num_kv_heads <= 0 || num_heads % num_kv_heads || head_size <= 0 ||
      head_size > 256 || (dtype_size != 2 && dtype_size != 4) || block_size <= 0)
    return NXT_PA_PATH_NONE;
  CUtensorMap tk, tv;
  if (xpa::fast_path_shape_ok(head_size, num_heads / num_kv_heads, block_size, dtype_size) &&
      fast_layout_ok(key_cache, value_cache, head_size, num_kv_heads, kv_block_stride,
                     kv_head_stride) &&
      encode_pool(&tk, key_cache, head_size, num_kv_heads, -1, kv_block_stride,
                  kv_head_stride) &&
      encode_pool(&tv, value_cache, head_size, num_kv_heads, -1, kv_block_stride,
                  kv_head_stride))
    return NXT_PA_PATH_TMA_MMA;
  return NXT_PA_PATH_GENERIC;
}

int nxt_paged_attention_device_status(int clear) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return NXT_PA_ECUDA;
  int* st = nullptr;
  {
    std::lock_guard<std::mutex> lk(g_mu);
    DeviceState* d = nullptr;
    int rc = device_state_locked(dev, &d);
    if (rc != NXT_PA_OK) return rc;
    st = d->status;
  }
  if (cudaDeviceSynchronize() != cudaSuccess) return NXT_PA_ECUDA;
  int v = 0;
  if (cudaMemcpy(&v, st, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess) return NXT_PA_ECUDA;
  if (clear && cudaMemset(st, 0, sizeof(int)) != cudaSuccess) return NXT_PA_ECUDA;
  if (clear && cudaDeviceSynchronize() != cudaSuccess) return NXT_PA_ECUDA;
  return v;
}

int nxt_paged_attention_release_workspaces(void) {
  std::lock_guard<std::mutex> lk(g_mu);
  int prev = 0;
  const bool have_prev = cudaGetDevice(&prev) == cudaSuccess;
  int rc = NXT_PA_OK;
  for (auto& kv : g_ws) {
    if (!kv.second.ptr) continue;
    if (cudaSetDevice(kv.first.first) != cudaSuccess || cudaFree(kv.second.ptr) != cudaSuccess)
      rc = NXT_PA_ECUDA;
  }
  g_ws.clear();
  for (int dev = 0; dev < kMaxDevices; ++dev) {
    if (!g_dev[dev].status) continue;
    if (cudaSetDevice(dev) != cudaSuccess || cudaFree(g_dev[dev].status) != cudaSuccess)
      rc = NXT_PA_ECUDA;
    g_dev[dev].status = nullptr;
  }
  if (have_prev) cudaSetDevice(prev);
  return rc;
}

int nxt_paged_attention_prefix_ex(void* out, const void* query, const void* key_cache,
                                  const void* value_cache, const int* block_tables,
                                  const int* seq_lens, const int* prefix_pages,
                                  const int* group_offsets, const int* group_members,
                                  int num_groups, int max_group_size, int max_prefix_pages,
                                  int num_seqs, int num_heads, int head_size, int num_kv_heads,
                                  float scale, int max_num_blocks_per_seq, int block_size,
                                  int dtype_size, int64_t kv_block_stride, int64_t kv_head_stride,
                                  int64_t num_blocks, void* workspace, size_t workspace_bytes,
                                  int* device_status, nxt_stream_t stream) {
  if (num_groups < 0 || max_group_size < 0 || max_prefix_pages < 0) return NXT_PA_EINVAL;
  PrefixArgs pre{prefix_pages, group_offsets, group_members, num_groups, max_group_size,
                 max_prefix_pages};
  return run(out, query, key_cache, value_cache, block_tables, seq_lens, num_seqs, num_heads,
             head_size, num_kv_heads, scale, max_num_blocks_per_seq, block_size, dtype_size,
             kv_block_stride, kv_head_stride, num_blocks, workspace, workspace_bytes,
             device_status, static_cast<cudaStream_t>(stream), nullptr, 0, false, &pre);
}

size_t nxt_paged_attention_prefix_workspace_size(int num_seqs, int num_heads, int head_size,
                                                 int num_kv_heads, int max_num_blocks_per_seq,
                                                 int block_size, int max_prefix_pages) {
  (void)block_size;
  if (num_seqs <= 0 || num_heads <= 0 || num_kv_heads <= 0 || head_size <= 0) return 0;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) dev = -1;
  const Plan pl = make_plan(num_seqs, num_heads, head_size, num_kv_heads, max_num_blocks_per_seq,
                            sm_count_of(dev));
  const int pchunks =
      max_prefix_pages > 0 ? ceil_div(max_prefix_pages, prefix_chunk_pages(max_prefix_pages)) : 0;
  return partial_bytes((long long)num_seqs * num_heads * (pl.max_parts + pchunks), head_size);
}

int nxt_paged_attention_fp8_ex(void* out, const void* query, const void* key_cache,
                               const void* value_cache, const int* block_tables,
                               const int* seq_lens, int num_seqs, int num_heads, int head_size,
                               int num_kv_heads, float scale, int max_num_blocks_per_seq,
                               int block_size, int kv_format, float k_scale, float v_scale,
                               int64_t kv_block_stride, int64_t kv_head_stride,
                               int64_t num_blocks, void* workspace, size_t workspace_bytes,
                               int* device_status, nxt_stream_t stream) {
  const KvQuant kq{kv_format, k_scale, v_scale};
  return run(out, query, key_cache, value_cache, block_tables, seq_lens, num_seqs, num_heads,
             head_size, num_kv_heads, scale, max_num_blocks_per_seq, block_size, 2,
             kv_block_stride, kv_head_stride, num_blocks, workspace, workspace_bytes,
             device_status, static_cast<cudaStream_t>(stream), nullptr, 0, false, nullptr, &kq);
}

int nxt_reshape_and_cache_fp8(const void* key, const void* value, void* key_cache,
                              void* value_cache, const int64_t* slot_mapping, int num_tokens,
                              int num_kv_heads, int head_size, int block_size, int kv_format,
                              float k_scale, float v_scale, int64_t kv_block_stride,
                              int64_t kv_head_stride, int64_t token_stride, nxt_stream_t stream) {
  if (num_tokens < 0) return NXT_PA_EINVAL;
  if (num_tokens == 0) return NXT_PA_OK;
  if (!key || !value || !key_cache || !value_cache || !slot_mapping) return NXT_PA_EINVAL;
  if ((kv_format != xpa::kKvE4M3 && kv_format != xpa::kKvE5M2 && kv_format != xpa::kKvInt8) ||
      !(k_scale > 0.f) ||
      !(v_scale > 0.f) || !std::isfinite(k_scale) || !std::isfinite(v_scale))
    return NXT_PA_EINVAL;
  if (num_kv_heads <= 0 || head_size <= 0 || head_size > 256 || block_size <= 0 ||
      kv_block_stride < 0 || kv_head_stride < 0 ||
      token_stride < (int64_t)num_kv_heads * head_size)
    return NXT_PA_EINVAL;
  xpa::AppendParams a{};
  a.key = key;
  a.value = value;
  a.key_cache = key_cache;
  a.value_cache = value_cache;
  a.slots = reinterpret_cast<const long long*>(slot_mapping);
  a.kv_block_stride = kv_block_stride;
  a.kv_head_stride = kv_head_stride;
  a.token_stride = token_stride;
  a.num_tokens = num_tokens;
  a.Hkv = num_kv_heads;
  a.D = head_size;
  a.block_size = block_size;
  a.kv_fmt = kv_format;
  a.k_scale = k_scale;
  a.v_scale = v_scale;
  auto al = [](const void* x, unsigned m) { return (reinterpret_cast<uintptr_t>(x) & m) == 0; };
  // 8 fp16 in (16 bytes), 8 fp8 out (8 bytes) per lane step
  a.vec16 = (head_size % 8 == 0 && kv_block_stride % 8 == 0 && kv_head_stride % 8 == 0 &&
             (token_stride * 2) % 16 == 0 && al(key, 15u) && al(value, 15u) &&
             al(key_cache, 7u) && al(value_cache, 7u))
                ? 1
                : 0;
  return map_cuda(xpa::launch_append(a, 2, static_cast<cudaStream_t>(stream)));
}

int nxt_paged_attention_fp8_append_ex(void* out, const void* query, void* key_cache,
                                      void* value_cache, const int* block_tables,
                                      const int* seq_lens, const void* new_key,
                                      const void* new_value, const int64_t* slot_mapping,
                                      int num_seqs, int num_heads, int head_size,
                                      int num_kv_heads, float scale, int max_num_blocks_per_seq,
                                      int block_size, int kv_format, float k_scale,
                                      float v_scale, int64_t kv_block_stride,
                                      int64_t kv_head_stride, int64_t num_blocks,
                                      int* device_status, nxt_stream_t stream) {
  int rc = check_args(out, query, key_cache, value_cache, block_tables, seq_lens, num_seqs,
                      num_heads, head_size, num_kv_heads, max_num_blocks_per_seq, block_size, 2,
                      kv_block_stride, kv_head_stride);
  if (rc != NXT_PA_OK || num_seqs == 0) return rc;
  // format and scales are checked here, before anything is launched
  rc = nxt_reshape_and_cache_fp8(new_key, new_value, key_cache, value_cache, slot_mapping,
                                 num_seqs, num_kv_heads, head_size, block_size, kv_format,
                                 k_scale, v_scale, kv_block_stride, kv_head_stride,
                                 (int64_t)num_kv_heads * head_size, stream);
  if (rc != NXT_PA_OK) return rc;
  const KvQuant kq{kv_format, k_scale, v_scale};
  return run(out, query, key_cache, value_cache, block_tables, seq_lens, num_seqs, num_heads,
             head_size, num_kv_heads, scale, max_num_blocks_per_seq, block_size, 2,
             kv_block_stride, kv_head_stride, num_blocks, nullptr, 0, device_status,
             static_cast<cudaStream_t>(stream), nullptr, 0, true, nullptr, &kq);
}

int nxt_reshape_and_cache(const void* key, const void* value, void* key_cache, void* value_cache,
                          const int64_t* slot_mapping, int num_tokens, int num_kv_heads,
                          int head_size, int block_size, int dtype_size, int64_t kv_block_stride,
                          int64_t kv_head_stride, int64_t token_stride, nxt_stream_t stream) {
  if (num_tokens < 0) return NXT_PA_EINVAL;
  if (num_tokens == 0) return NXT_PA_OK;
  if (!key || !value || !key_cache || !value_cache || !slot_mapping) return NXT_PA_EINVAL;
  if (num_kv_heads <= 0 || head_size <= 0 || head_size > 256 || block_size <= 0 ||
      (dtype_size != 2 && dtype_size != 4) || kv_block_stride < 0 || kv_head_stride < 0 ||
      token_stride < (int64_t)num_kv_heads * head_size)
    return NXT_PA_EINVAL;
  xpa::AppendParams a{};
  a.key = key;
  a.value = value;
  a.key_cache = key_cache;
  a.value_cache = value_cache;
  a.slots = reinterpret_cast<const long long*>(slot_mapping);
  a.kv_block_stride = kv_block_stride;
  a.kv_head_stride = kv_head_stride;
  a.token_stride = token_stride;
  a.num_tokens = num_tokens;
  a.Hkv = num_kv_heads;
  a.D = head_size;
  a.block_size = block_size;
  auto a16 = [](const void* x) { return (reinterpret_cast<uintptr_t>(x) & 15u) == 0; };
  const int64_t es = dtype_size;
  a.vec16 = ((head_size * es) % 16 == 0 && (kv_block_stride * es) % 16 == 0 &&
             (kv_head_stride * es) % 16 == 0 && (token_stride * es) % 16 == 0 && a16(key) &&
             a16(value) && a16(key_cache) && a16(value_cache))
                ? 1
                : 0;
  return map_cuda(xpa::launch_append(a, dtype_size, static_cast<cudaStream_t>(stream)));
}

int nxt_paged_attention_append_ex(void* out, const void* query, void* key_cache,
                                  void* value_cache, const int* block_tables, const int* seq_lens,
                                  const void* new_key, const void* new_value,
                                  const int64_t* slot_mapping, int num_seqs, int num_heads,
                                  int head_size, int num_kv_heads, float scale,
                                  int max_num_blocks_per_seq, int block_size, int dtype_size,
                                  int64_t kv_block_stride, int64_t kv_head_stride,
                                  int64_t num_blocks, int* device_status, nxt_stream_t stream) {
  int rc = check_args(out, query, key_cache, value_cache, block_tables, seq_lens, num_seqs,
                      num_heads, head_size, num_kv_heads, max_num_blocks_per_seq, block_size,
                      dtype_size, kv_block_stride, kv_head_stride);
  if (rc != NXT_PA_OK || num_seqs == 0) return rc;
  rc = nxt_reshape_and_cache(new_key, new_value, key_cache, value_cache, slot_mapping, num_seqs,
                             num_kv_heads, head_size, block_size, dtype_size, kv_block_stride,
                             kv_head_stride, (int64_t)num_kv_heads * head_size, stream);
  if (rc != NXT_PA_OK) return rc;
  return run(out, query, key_cache, value_cache, block_tables, seq_lens, num_seqs, num_heads,
             head_size, num_kv_heads, scale, max_num_blocks_per_seq, block_size, dtype_size,
             kv_block_stride, kv_head_stride, num_blocks, nullptr, 0, device_status,
             static_cast<cudaStream_t>(stream), nullptr, 0, true);
}

int nxt_pa_peer_alloc(size_t bytes, void** dev_ptr, void* ipc_handle) {
  if (!dev_ptr || !ipc_handle || bytes == 0) return NXT_PA_EINVAL;
  static_assert(sizeof(cudaIpcMemHandle_t) == NXT_PA_IPC_HANDLE_BYTES, "IPC handle size");
  void* ptr = nullptr;
  if (cudaMalloc(&ptr, bytes) != cudaSuccess) return NXT_PA_ENOMEM;
  cudaIpcMemHandle_t h;
  if (cudaMemset(ptr, 0, bytes) != cudaSuccess || cudaDeviceSynchronize() != cudaSuccess ||
      cudaIpcGetMemHandle(&h, ptr) != cudaSuccess) {
    cudaFree(ptr);
    return NXT_PA_ECUDA;
  }
  std::memcpy(ipc_handle, &h, sizeof(h));
  *dev_ptr = ptr;
  return NXT_PA_OK;
}

int nxt_pa_peer_open(const void* ipc_handle, void** dev_ptr) {
  if (!dev_ptr || !ipc_handle) return NXT_PA_EINVAL;
  cudaIpcMemHandle_t h;
  std::memcpy(&h, ipc_handle, sizeof(h));
  void* ptr = nullptr;
  if (cudaIpcOpenMemHandle(&ptr, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess)
    return NXT_PA_ECUDA;
  *dev_ptr = ptr;
  return NXT_PA_OK;
}

int nxt_pa_peer_close(void* dev_ptr) {
  return cudaIpcCloseMemHandle(dev_ptr) == cudaSuccess ? NXT_PA_OK : NXT_PA_ECUDA;
}

int nxt_pa_peer_free(void* dev_ptr) {
  return cudaFree(dev_ptr) == cudaSuccess ? NXT_PA_OK : NXT_PA_ECUDA;
}

int nxt_paged_attention_sharded(const NxtPaShard* shard, uint64_t step, const void* query,
                                const void* key_cache, const void* value_cache,
                                const int* block_tables, const int* seq_lens, int num_seqs,
                                int num_heads, int head_size, int num_kv_heads, float scale,
                                int max_num_blocks_per_seq, int block_size, int dtype_size,
                                int64_t kv_block_stride, int64_t kv_head_stride,
                                int64_t num_blocks, int* device_status, nxt_stream_t stream) {
  if (!shard) return NXT_PA_EINVAL;
  return run(nullptr, query, key_cache, value_cache, block_tables, seq_lens, num_seqs, num_heads,
             head_size, num_kv_heads, scale, max_num_blocks_per_seq, block_size, dtype_size,
             kv_block_stride, kv_head_stride, num_blocks, nullptr, 0, device_status,
             static_cast<cudaStream_t>(stream), shard, step);
}

int nxt_paged_attention_fp8_sharded(const NxtPaShard* shard, uint64_t step, const void* query,
                                    const void* key_cache, const void* value_cache,
                                    const int* block_tables, const int* seq_lens, int num_seqs,
                                    int num_heads, int head_size, int num_kv_heads, float scale,
                                    int max_num_blocks_per_seq, int block_size, int kv_format,
                                    float k_scale, float v_scale, int64_t kv_block_stride,
                                    int64_t kv_head_stride, int64_t num_blocks,
                                    int* device_status, nxt_stream_t stream) {
  if (!shard) return NXT_PA_EINVAL;
  const KvQuant kq{kv_format, k_scale, v_scale};
  return run(nullptr, query, key_cache, value_cache, block_tables, seq_lens, num_seqs, num_heads,
             head_size, num_kv_heads, scale, max_num_blocks_per_seq, block_size, 2,
             kv_block_stride, kv_head_stride, num_blocks, nullptr, 0, device_status,
             static_cast<cudaStream_t>(stream), shard, step, false, nullptr, &kq);
}

uint64_t nxt_paged_attention_set_wait_budget_ns(uint64_t budget_ns) {
  const uint64_t prev = g_wait_budget_ns;
  g_wait_budget_ns = budget_ns;
  return prev;
}

int nxt_paged_attention_profile_next(void* before, void* after) {
  g_prof_before = static_cast<cudaEvent_t>(before);
  g_prof_after = static_cast<cudaEvent_t>(after);
  g_prof_merged = nullptr;
  return NXT_PA_OK;
}

int nxt_paged_attention_profile_next_ex(void* before, void* after_attention, void* after_merge) {
  g_prof_before = static_cast<cudaEvent_t>(before);
  g_prof_after = static_cast<cudaEvent_t>(after_attention);
  g_prof_merged = static_cast<cudaEvent_t>(after_merge);
  return NXT_PA_OK;
}

int nxt_paged_attention_device_info(int* device_id, int* sm_count, char* name, int name_len) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return NXT_PA_ECUDA;
  cudaDeviceProp prop;
  if (cudaGetDeviceProperties(&prop, dev) != cudaSuccess) return NXT_PA_ECUDA;
  if (device_id) *device_id = dev;
  if (sm_count) *sm_count = prop.multiProcessorCount;
  if (name && name_len > 0) {
    std::strncpy(name, prop.name, (size_t)name_len - 1);
    name[name_len - 1] = '\0';
  }
  return NXT_PA_OK;
}

}  // extern "C"
