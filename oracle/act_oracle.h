/*
 * act_oracle.h — CPU restatement of xLLMs' gated / element-wise activations.
 *
 * TEST INFRASTRUCTURE ONLY (the checker for xllms_b200/csrc/pa_act.cu; only
 * tests/ may load it). Semantics (operators/activation_kernels.cu:25-135 of
 * the xLLMs project):
 *   gated ops: row t of `input` is [gate (d) | up (d)], row t of `out` is d;
 *     op 0 silu(gate)*up, 1 gate*silu(up), 2 gelu(gate)*up, 3 gelu_tanh(gate)*up;
 *   element-wise ops: 4 gelu(x), 5 silu(x);
 *   the activation is evaluated in binary32 (expf / erff / tanhf), rounded to
 *   the storage type, and the product is taken in the storage type (for
 *   binary16: the exact binary32 product of two halves rounded to binary16).
 * libm's expf / erff / tanhf may differ from CUDA's by an ulp or two, so
 * results agree with the GPU to a tolerance, not bit for bit.
 */
#ifndef XPA_ACT_ORACLE_H_
#define XPA_ACT_ORACLE_H_

#ifdef __cplusplus
extern "C" {
#endif

/* Returns 0, or -1 on an invalid argument. dtype_size 2 = binary16, 4 = binary32. */
int act_oracle(int op, void *out, const void *input, int num_tokens, int d, int dtype_size);

#ifdef __cplusplus
}
#endif
#endif /* XPA_ACT_ORACLE_H_ */
