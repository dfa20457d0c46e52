/*
 * ref_act_shim.cu — exposes the reference's own activation kernels.
 *
 * TEST INFRASTRUCTURE ONLY. The reference defines its activation launchers
 * (operators/activation_kernels.cu:139-239) with a cudaStream_t parameter
 * while its header declares them extern "C" with nxt_stream_t, so the
 * definitions get C++ linkage under other names. This shim compiles that
 * source file in place (its path comes from oracle/Makefile; nothing is
 * copied) and adds one C entry point that forwards to the reference
 * launchers unchanged. Tests compare xllms_b200's kernels with these on the
 * GPU.
 */
#include REF_ACT_CU

extern "C" int ref_activation(int op, void* out, const void* input, int num_tokens, int d,
                              int dtype_size, void* stream) {
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  switch (op) {
    case 0: nxt_silu_and_mul(out, input, num_tokens, d, dtype_size, st); break;
    case 1: nxt_mul_and_silu(out, input, num_tokens, d, dtype_size, st); break;
    case 2: nxt_gelu_and_mul(out, input, num_tokens, d, dtype_size, st); break;
    case 3: nxt_gelu_tanh_and_mul(out, input, num_tokens, d, dtype_size, st); break;
    case 4: nxt_gelu_elementwise(out, input, num_tokens, d, dtype_size, st); break;
    case 5: nxt_silu_elementwise(out, input, num_tokens, d, dtype_size, st); break;
    default: return -1;
  }
  return cudaGetLastError() == cudaSuccess ? 0 : -1;
}
