// pa_act.cu — gated and element-wise activation kernels (the reference's
// operators/activation_kernels.cu operator set: nxt_silu_and_mul,
// nxt_mul_and_silu, nxt_gelu_and_mul, nxt_gelu_tanh_and_mul,
// nxt_gelu_elementwise, nxt_silu_elementwise; include/operator_api.h:121-150).
//
// Semantics kept from the reference (operators/activation_kernels.cu:25-135):
//   gated ops read row t of `input` as [gate (d) | up (d)] and write row t of
//   `out` (d); the activation is evaluated in fp32 with expf / erff / tanhf,
//   rounded to the storage type, and the product with the other half is taken
//   in the storage type (fp16 multiply for dtype_size 2);
//   silu(x) = x / (1 + exp(-x)), gelu(x) = x/2 (1 + erf(x / sqrt 2)),
//   gelu_tanh(x) = x/2 (1 + tanh(sqrt(2/pi) (x + 0.044715 x^3))).
// B200 layout: the ops are HBM-bound streams (fp16: 6 bytes per output
// element for the gated ops), so each thread moves 16-byte vectors (8 fp16 or
// 4 fp32 elements) in a grid-stride loop over (row, vector) pairs with the
// grid sized to the SM count; shapes without 16-byte alignment take a scalar
// loop. The reference launches one CTA per token with min(d, 1024) threads.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "operator_api.h"

namespace {

enum Op : int {
  kSiluMul = NXT_ACT_SILU_AND_MUL,
  kMulSilu = NXT_ACT_MUL_AND_SILU,
  kGeluMul = NXT_ACT_GELU_AND_MUL,
  kGeluTanhMul = NXT_ACT_GELU_TANH_AND_MUL,
  kGelu = NXT_ACT_GELU,
  kSilu = NXT_ACT_SILU,
};

__host__ __device__ constexpr bool gated(int op) { return op <= kGeluTanhMul; }

thread_local int g_act_last_error = NXT_PA_OK;

// fp32 activations, written as the reference evaluates them (operation order
// included, so that fp32 rounding agrees).
__device__ __forceinline__ float silu_f(float x) { return x / (1.0f + expf(-x)); }
__device__ __forceinline__ float gelu_f(float f) {
  constexpr float kInvSqrt2 = 0.70710678118654752440f;
  return f * 0.5f * (1.0f + erff(f * kInvSqrt2));
}
__device__ __forceinline__ float gelu_tanh_f(float f) {
  constexpr float kBeta = (float)(1.41421356237309504880 * 1.12837916709551257390 * 0.5);
  constexpr float kKappa = 0.044715f;
  const float cube = f * f * f;
  const float inner = kBeta * (f + kKappa * cube);
  return 0.5f * f * (1.0f + tanhf(inner));
}

template <int OP>
__device__ __forceinline__ float act_f(float x) {
  if constexpr (OP == kSiluMul || OP == kMulSilu || OP == kSilu) return silu_f(x);
  if constexpr (OP == kGeluMul || OP == kGelu) return gelu_f(x);
  return gelu_tanh_f(x);
}

// One output element from (gate, up) (or from x for the element-wise ops).
template <int OP>
__device__ __forceinline__ float apply(float g, float u) {
  if constexpr (OP == kMulSilu) return g * act_f<OP>(u);
  if constexpr (gated(OP)) return act_f<OP>(g) * u;
  return act_f<OP>(g);
}
template <int OP>
__device__ __forceinline__ __half apply(__half g, __half u) {
  if constexpr (OP == kMulSilu) return __hmul(g, __float2half_rn(act_f<OP>(__half2float(u))));
  if constexpr (gated(OP)) return __hmul(__float2half_rn(act_f<OP>(__half2float(g))), u);
  return __float2half_rn(act_f<OP>(__half2float(g)));
}

template <typename T>
struct Vec;  // 16 bytes of T
template <>
struct Vec<__half> {
  static constexpr int N = 8;
};
template <>
struct Vec<float> {
  static constexpr int N = 4;
};

// 16-byte path: d % N == 0 and 16-byte aligned rows. Thread i takes vectors
// i, i + S, i + 2S, ... (S = threads in the grid), two per step so that four
// (gated) or two loads are in flight; its (row, column) advances by S's
// quotient and remainder, with no division in the loop.
template <typename T, int OP>
__global__ void __launch_bounds__(256) act_vec_kernel(T* __restrict__ out,
                                                      const T* __restrict__ in, long long rows,
                                                      int d) {
  constexpr int N = Vec<T>::N;
  union U {
    uint4 v;
    T e[N];
  };
  const int per_row = d / N;
  const long long in_row = gated(OP) ? 2LL * d : d;
  const long long S = (long long)gridDim.x * blockDim.x;
  const long long s_rows = S / per_row;
  const int s_cols = (int)(S - s_rows * per_row);
  const long long i0 = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  long long r = i0 / per_row;
  int c = (int)(i0 - r * per_row);
  auto advance = [&](long long& rr, int& cc) {
    rr += s_rows;
    cc += s_cols;
    if (cc >= per_row) {
      cc -= per_row;
      ++rr;
    }
  };
  while (r < rows) {
    long long r1 = r;
    int c1 = c;
    advance(r1, c1);
    const bool two = r1 < rows;
    U g0, u0, g1, u1, o;
    const T* s0 = in + r * in_row + (long long)c * N;
    const T* s1 = in + r1 * in_row + (long long)c1 * N;
    g0.v = __ldg(reinterpret_cast<const uint4*>(s0));
    if constexpr (gated(OP)) u0.v = __ldg(reinterpret_cast<const uint4*>(s0 + d));
    if (two) {
      g1.v = __ldg(reinterpret_cast<const uint4*>(s1));
      if constexpr (gated(OP)) u1.v = __ldg(reinterpret_cast<const uint4*>(s1 + d));
    }
#pragma unroll
    for (int k = 0; k < N; ++k) o.e[k] = apply<OP>(g0.e[k], gated(OP) ? u0.e[k] : g0.e[k]);
    *reinterpret_cast<uint4*>(out + r * d + (long long)c * N) = o.v;
    if (two) {
#pragma unroll
      for (int k = 0; k < N; ++k) o.e[k] = apply<OP>(g1.e[k], gated(OP) ? u1.e[k] : g1.e[k]);
      *reinterpret_cast<uint4*>(out + r1 * d + (long long)c1 * N) = o.v;
    }
    r = r1;
    c = c1;
    advance(r, c);
  }
}

// Any shape: one element per thread and step.
template <typename T, int OP>
__global__ void __launch_bounds__(256) act_scalar_kernel(T* __restrict__ out,
                                                         const T* __restrict__ in,
                                                         long long rows, int d) {
  const long long total = rows * d;
  const long long in_row = gated(OP) ? 2LL * d : d;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const long long r = i / d;
    const int c = (int)(i - r * d);
    const T g = in[r * in_row + c];
    const T u = gated(OP) ? in[r * in_row + d + c] : g;
    out[r * d + c] = apply<OP>(g, u);
  }
}

int sm_count() {
  static thread_local int dev_cached = -1, sms_cached = 148;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  if (dev != dev_cached) {
    int sms = 0;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess && sms > 0)
      sms_cached = sms;
    dev_cached = dev;
  }
  return sms_cached;
}

template <typename T, int OP>
cudaError_t launch_t(void* out, const void* in, long long rows, int d, cudaStream_t st) {
  constexpr int N = Vec<T>::N;
  const bool vec = d % N == 0 && (reinterpret_cast<uintptr_t>(out) & 15u) == 0 &&
                   (reinterpret_cast<uintptr_t>(in) & 15u) == 0;
  const long long work = vec ? rows * (d / N) : rows * d;
  const long long cap = (long long)sm_count() * 8;  // 8 CTAs of 256 threads per SM
  long long grid = (work + 255) / 256;
  if (grid > cap) grid = cap;
  if (grid < 1) grid = 1;
  if (vec)
    act_vec_kernel<T, OP><<<(unsigned)grid, 256, 0, st>>>(static_cast<T*>(out),
                                                           static_cast<const T*>(in), rows, d);
  else
    act_scalar_kernel<T, OP><<<(unsigned)grid, 256, 0, st>>>(static_cast<T*>(out),
                                                              static_cast<const T*>(in), rows, d);
  return cudaGetLastError();
}

template <int OP>
cudaError_t launch_op(void* out, const void* in, long long rows, int d, int ds, cudaStream_t st) {
  return ds == 2 ? launch_t<__half, OP>(out, in, rows, d, st)
                 : launch_t<float, OP>(out, in, rows, d, st);
}

int run(int op, void* out, const void* in, int num_tokens, int d, int dtype_size,
        nxt_stream_t stream) {
  if (op < kSiluMul || op > kSilu) return NXT_PA_EINVAL;
  if (num_tokens < 0 || d <= 0 || (dtype_size != 2 && dtype_size != 4)) return NXT_PA_EINVAL;
  if (num_tokens == 0) return NXT_PA_OK;
  if (!out || !in) return NXT_PA_EINVAL;
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e;
  switch (op) {
    case kSiluMul: e = launch_op<kSiluMul>(out, in, num_tokens, d, dtype_size, st); break;
    case kMulSilu: e = launch_op<kMulSilu>(out, in, num_tokens, d, dtype_size, st); break;
    case kGeluMul: e = launch_op<kGeluMul>(out, in, num_tokens, d, dtype_size, st); break;
    case kGeluTanhMul: e = launch_op<kGeluTanhMul>(out, in, num_tokens, d, dtype_size, st); break;
    case kGelu: e = launch_op<kGelu>(out, in, num_tokens, d, dtype_size, st); break;
    default: e = launch_op<kSilu>(out, in, num_tokens, d, dtype_size, st); break;
  }
  return e == cudaSuccess ? NXT_PA_OK : NXT_PA_ECUDA;
}

}  // namespace

extern "C" {

int nxt_activation_ex(int op, void* out, const void* input, int num_tokens, int d,
                      int dtype_size, nxt_stream_t stream) {
  return run(op, out, input, num_tokens, d, dtype_size, stream);
}

int nxt_activation_last_error(void) { return g_act_last_error; }

void nxt_silu_and_mul(void* out, const void* input, int num_tokens, int d, int dtype_size,
                      nxt_stream_t stream) {
  g_act_last_error = run(kSiluMul, out, input, num_tokens, d, dtype_size, stream);
}
void nxt_mul_and_silu(void* out, const void* input, int num_tokens, int d, int dtype_size,
                      nxt_stream_t stream) {
  g_act_last_error = run(kMulSilu, out, input, num_tokens, d, dtype_size, stream);
}
void nxt_gelu_and_mul(void* out, const void* input, int num_tokens, int d, int dtype_size,
                      nxt_stream_t stream) {
  g_act_last_error = run(kGeluMul, out, input, num_tokens, d, dtype_size, stream);
}
void nxt_gelu_tanh_and_mul(void* out, const void* input, int num_tokens, int d,
                           int dtype_size, nxt_stream_t stream) {
  g_act_last_error = run(kGeluTanhMul, out, input, num_tokens, d, dtype_size, stream);
}
void nxt_gelu_elementwise(void* out, const void* input, int num_tokens, int d, int dtype_size,
                          nxt_stream_t stream) {
  g_act_last_error = run(kGelu, out, input, num_tokens, d, dtype_size, stream);
}
void nxt_silu_elementwise(void* out, const void* input, int num_tokens, int d, int dtype_size,
                          nxt_stream_t stream) {
  g_act_last_error = run(kSilu, out, input, num_tokens, d, dtype_size, stream);
}

}  // extern "C"
