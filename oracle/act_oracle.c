/*
 * act_oracle.c — CPU restatement of the reference's activation operators.
 * TEST INFRASTRUCTURE ONLY; see act_oracle.h for the semantics followed
 * (operators/activation_kernels.cu:25-135 of the xLLMs project).
 */
#include "act_oracle.h"

#include <math.h>
#include <stdint.h>

#include "pa_oracle.h"

static float silu_f(float x) { return x / (1.0f + expf(-x)); }

static float gelu_f(float f) { return f * 0.5f * (1.0f + erff(f * 0.70710678118654752440f)); }

static float gelu_tanh_f(float f) {
    const float beta = (float)(1.41421356237309504880 * 1.12837916709551257390 * 0.5);
    const float kappa = 0.044715f;
    const float cube = f * f * f;
    const float inner = beta * (f + kappa * cube);
    return 0.5f * f * (1.0f + tanhf(inner));
}

static float act_f(int op, float x) {
    switch (op) {
    case 0: case 1: case 5: return silu_f(x);
    case 2: case 4: return gelu_f(x);
    default: return gelu_tanh_f(x);
    }
}

/* storage-type rounding: identity for binary32, round-to-nearest-even binary16 */
static float round_to(float x, int dtype_size) {
    return dtype_size == 4 ? x : pa_half_to_float(pa_float_to_half(x));
}

static float load(const void *p, int64_t i, int dtype_size) {
    return dtype_size == 4 ? ((const float *)p)[i] : pa_half_to_float(((const uint16_t *)p)[i]);
}

static void store(void *p, int64_t i, float v, int dtype_size) {
    if (dtype_size == 4)
        ((float *)p)[i] = v;
    else
        ((uint16_t *)p)[i] = pa_float_to_half(v);
}

int act_oracle(int op, void *out, const void *input, int num_tokens, int d, int dtype_size) {
    if (op < 0 || op > 5 || num_tokens < 0 || d <= 0 || (dtype_size != 2 && dtype_size != 4))
        return -1;
    const int gated = op <= 3;
    const int64_t in_row = gated ? 2 * (int64_t)d : d;
    for (int64_t t = 0; t < num_tokens; ++t) {
        for (int64_t c = 0; c < d; ++c) {
            const float g = load(input, t * in_row + c, dtype_size);
            float v;
            if (!gated) {
                v = act_f(op, g);
            } else {
                const float u = load(input, t * in_row + d + c, dtype_size);
                if (op == 1)
                    v = g * round_to(act_f(op, u), dtype_size);
                else
                    v = round_to(act_f(op, g), dtype_size) * u;
            }
            store(out, t * d + c, v, dtype_size); /* rounds the product for binary16 */
        }
    }
    return 0;
}
