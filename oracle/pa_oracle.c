/*
 * pa_oracle.c — CPU restatement of xLLMs paged decode attention.
 *
 * TEST INFRASTRUCTURE ONLY: the checker for the CUDA kernels, never part of
 * the product path. The semantics and the reference lines they follow are
 * listed in pa_oracle.h. Parity of this file with the reference's own CPU
 * attention (examples/run_gpt2.c:46-83, compiled from the reference sources
 * by oracle/Makefile into oracle/_ref/) is checked by tests/test_oracle.py and
 * pinned by the fixtures under tests/golden/.
 */
#include "pa_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

/* IEEE 754 binary16 -> binary32, from the format definition: 1 sign bit,
 * 5 exponent bits (bias 15), 10 fraction bits; exponent 0 is subnormal
 * (fraction * 2^-24), exponent 31 is inf/NaN. Exact. */
float pa_half_to_float(uint16_t h) {
    const int sign = (h >> 15) & 1;
    const int e = (h >> 10) & 0x1f;
    const int f = h & 0x3ff;
    float v;
    if (e == 0) {
        v = ldexpf((float)f, -24);
    } else if (e == 31) {
        v = f ? NAN : INFINITY;
    } else {
        v = ldexpf((float)(f | 0x400), e - 25);
    }
    return sign ? -v : v;
}

/* binary32 -> binary16 with round-to-nearest-even. */
uint16_t pa_float_to_half(float x) {
    uint32_t u;
    memcpy(&u, &x, sizeof(u));
    const uint16_t sign = (uint16_t)((u >> 16) & 0x8000u);
    const uint32_t a = u & 0x7fffffffu;
    if (a >= 0x7f800000u) /* inf or NaN */
        return sign | 0x7c00u | (a > 0x7f800000u ? 0x200u : 0u);
    if (a >= 0x47800000u) /* >= 2^16: overflows to inf */
        return sign | 0x7c00u;
    if (a < 0x38800000u) { /* below 2^-14: half subnormal, units of 2^-24 */
        float mag;
        memcpy(&mag, &a, sizeof(mag));
        /* mag * 2^24 is exact; nearbyintf rounds half-to-even in the
         * default rounding mode. A result of 1024 is the smallest normal. */
        return sign | (uint16_t)nearbyintf(mag * 16777216.0f);
    }
    const uint32_t e = (a >> 23) - 127 + 15; /* 1..30 */
    const uint32_t m = a & 0x7fffffu;
    uint32_t h = (e << 10) | (m >> 13);
    const uint32_t rem = m & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h++; /* carries into exponent */
    return sign | (uint16_t)h;
}

/* ── one-byte codecs (OCP 8-bit floating point: E4M3 without infinities,
 * bias 7, max 448, 0x7F / 0xFF NaN; E5M2, bias 15, max 57344, IEEE-style
 * inf/NaN; two's-complement int8) ── */
static float fp8_decode_one(uint8_t c, int fmt) {
    if (fmt == PA_KV_INT8) return (float)(int8_t)c;
    const int sign = c >> 7;
    const int M = fmt == PA_FP8_E4M3 ? 3 : 2, bias = fmt == PA_FP8_E4M3 ? 7 : 15;
    const int e = (c & 0x7f) >> M, m = c & ((1 << M) - 1);
    float v;
    if (fmt == PA_FP8_E4M3 && (c & 0x7f) == 0x7f) {
        v = NAN;
    } else if (fmt == PA_FP8_E5M2 && e == 31) {
        v = m ? NAN : INFINITY;
    } else if (e == 0) {
        v = ldexpf((float)m, 1 - bias - M); /* subnormal */
    } else {
        v = ldexpf((float)((1 << M) + m), e - bias - M);
    }
    return sign ? -v : v;
}

/* Round to nearest even, saturating finite values (and infinities) at the
 * largest finite magnitude; NaN stays NaN. */
static uint8_t fp8_encode_one(float x, int fmt) {
    if (fmt == PA_KV_INT8) {
        /* nearbyintf rounds half to even in the default rounding mode */
        if (isnan(x)) return 0;
        const float r = nearbyintf(x);
        const int i = r > 127.0f ? 127 : (r < -128.0f ? -128 : (int)r);
        return (uint8_t)(int8_t)i;
    }
    const int M = fmt == PA_FP8_E4M3 ? 3 : 2, bias = fmt == PA_FP8_E4M3 ? 7 : 15;
    const uint8_t max_code = fmt == PA_FP8_E4M3 ? 0x7e : 0x7b;
    const uint8_t nan_code = 0x7f;
    uint8_t sign = signbit(x) ? 0x80 : 0;
    if (isnan(x)) return sign | nan_code;
    if (isinf(x)) return sign | max_code;
    const float a = fabsf(x);
    const float min_normal = ldexpf(1.0f, 1 - bias);
    uint32_t code;
    if (a < min_normal) {
        code = (uint32_t)nearbyintf(ldexpf(a, bias - 1 + M)); /* units of the subnormal step */
    } else {
        int e2;
        const float fr = frexpf(a, &e2);                   /* a = fr * 2^e2, fr in [0.5, 1) */
        const int e = e2 - 1;                               /* a = (2 fr) 2^e */
        const float mant = ldexpf(2.0f * fr - 1.0f, M);     /* exact */
        uint32_t m = (uint32_t)nearbyintf(mant);
        int eb = e + bias;
        if (m == (1u << M)) { m = 0; eb++; }
        if (eb > 31) eb = 31;
        code = ((uint32_t)eb << M) | m;
    }
    if (code > max_code) code = max_code;
    return sign | (uint8_t)code;
}

void pa_fp8_decode(float *out, const uint8_t *in, int64_t n, int fmt) {
    for (int64_t i = 0; i < n; i++) out[i] = fp8_decode_one(in[i], fmt);
}

void pa_fp8_encode(uint8_t *out, const float *in, int64_t n, int fmt) {
    for (int64_t i = 0; i < n; i++) out[i] = fp8_encode_one(in[i], fmt);
}

static inline float load_f(const void *base, int64_t idx, int dtype_size) {
    if (dtype_size == 4) return ((const float *)base)[idx];
    return pa_half_to_float(((const uint16_t *)base)[idx]);
}

typedef struct {
    const void *q, *k, *v;
    const int *bt, *sl;
    int B, H, D, Hkv, max_blocks, bs, ds;
    float scale;
    int64_t kbs, khs, num_blocks;
} pa_args;

static int check_args(const pa_args *a) {
    if (a->B < 0 || a->H <= 0 || a->D <= 0 || a->Hkv <= 0) return -1;
    if (a->H % a->Hkv != 0) return -1;
    if (a->bs <= 0 || a->max_blocks < 0) return -1;
    if (a->ds != 2 && a->ds != 4) return -1;
    if (a->B > 0 && (!a->q || !a->k || !a->v || !a->bt || !a->sl)) return -1;
    return 0;
}

/* Number of tokens of seq b the attention covers: seq_len clamped to the
 * block-table row (a longer seq_len would index past the row). */
static inline int seq_tokens(const pa_args *a, int b) {
    int L = a->sl[b];
    if (L < 0) L = 0;
    const int64_t cap = (int64_t)a->max_blocks * a->bs;
    if ((int64_t)L > cap) L = (int)cap;
    return L;
}

/* Physical page of token t of seq b, or -1 if the page is masked. */
static inline int64_t page_of(const pa_args *a, int b, int t) {
    const int phys = a->bt[(int64_t)b * a->max_blocks + t / a->bs];
    if (phys < 0) return -1;
    if (a->num_blocks > 0 && phys >= a->num_blocks) return -1;
    return phys;
}

static inline int64_t kv_index(const pa_args *a, int64_t phys, int kh, int slot) {
    return phys * a->kbs + (int64_t)kh * a->khs + (int64_t)slot * a->D;
}

/* One (seq, q head) row, fp32 accumulation, following examples/text_gen.c:1284-1309:
 * scores = dot*scale, running max, expf(s - max), w = e / sum, o += w * v. */
static void attend_row_f32(const pa_args *a, int b, int h, float *o, float *scores) {
    const int D = a->D;
    const int kh = h / (a->H / a->Hkv);
    const int L = seq_tokens(a, b);
    const int64_t qoff = ((int64_t)b * a->H + h) * D;
    memset(o, 0, (size_t)D * sizeof(float));

    float max_val = -INFINITY;
    for (int t = 0; t < L; t++) {
        const int64_t phys = page_of(a, b, t);
        if (phys < 0) { scores[t] = -INFINITY; continue; }
        const int64_t ko = kv_index(a, phys, kh, t % a->bs);
        float dot = 0.0f;
        for (int d = 0; d < D; d++)
            dot += load_f(a->q, qoff + d, a->ds) * load_f(a->k, ko + d, a->ds);
        scores[t] = dot * a->scale;
        if (scores[t] > max_val) max_val = scores[t];
    }
    if (max_val == -INFINITY) return; /* no valid token: zero row */
    float sum_exp = 0.0f;
    for (int t = 0; t < L; t++) {
        scores[t] = (scores[t] == -INFINITY) ? 0.0f : expf(scores[t] - max_val);
        sum_exp += scores[t];
    }
    for (int t = 0; t < L; t++) {
        if (scores[t] == 0.0f) continue;
        const int64_t phys = page_of(a, b, t);
        const int64_t vo = kv_index(a, phys, kh, t % a->bs);
        const float w = scores[t] / sum_exp;
        for (int d = 0; d < D; d++) o[d] += w * load_f(a->v, vo + d, a->ds);
    }
}

static int max_len(const pa_args *a) {
    int m = 1;
    for (int b = 0; b < a->B; b++) {
        const int L = seq_tokens(a, b);
        if (L > m) m = L;
    }
    return m;
}

#define PA_ARGS_INIT                                                         \
    pa_args a = {query, key_cache, value_cache, block_tables, seq_lens,       \
                 num_seqs, num_heads, head_size, num_kv_heads,                \
                 max_num_blocks_per_seq, block_size, dtype_size, scale,       \
                 kv_block_stride, kv_head_stride, num_blocks}

int pa_oracle_f32(float *out, const void *query, const void *key_cache,
                  const void *value_cache, const int *block_tables,
                  const int *seq_lens, int num_seqs, int num_heads,
                  int head_size, int num_kv_heads, float scale,
                  int max_num_blocks_per_seq, int block_size, int dtype_size,
                  int64_t kv_block_stride, int64_t kv_head_stride,
                  int64_t num_blocks) {
    PA_ARGS_INIT;
    if (check_args(&a) || (num_seqs > 0 && !out)) return -1;
    float *scores = (float *)malloc((size_t)max_len(&a) * sizeof(float));
    if (!scores) return -1;
    for (int b = 0; b < num_seqs; b++)
        for (int h = 0; h < num_heads; h++)
            attend_row_f32(&a, b, h, out + ((int64_t)b * num_heads + h) * head_size, scores);
    free(scores);
    return 0;
}

int pa_oracle_f32_omp(float *out, const void *query, const void *key_cache,
                      const void *value_cache, const int *block_tables,
                      const int *seq_lens, int num_seqs, int num_heads,
                      int head_size, int num_kv_heads, float scale,
                      int max_num_blocks_per_seq, int block_size,
                      int dtype_size, int64_t kv_block_stride,
                      int64_t kv_head_stride, int64_t num_blocks,
                      int nthreads) {
    PA_ARGS_INIT;
    if (check_args(&a) || (num_seqs > 0 && !out)) return -1;
    const int ml = max_len(&a);
    const int64_t rows = (int64_t)num_seqs * num_heads;
    int failed = 0;
#ifdef _OPENMP
    if (nthreads <= 0) nthreads = omp_get_max_threads();
#pragma omp parallel num_threads(nthreads) reduction(| : failed)
#else
    (void)nthreads;
#endif
    {
        float *scores = (float *)malloc((size_t)ml * sizeof(float));
        if (!scores) {
            failed = 1;
        } else {
#ifdef _OPENMP
#pragma omp for schedule(dynamic, 1)
#endif
            for (int64_t r = 0; r < rows; r++)
                attend_row_f32(&a, (int)(r / num_heads), (int)(r % num_heads),
                               out + r * head_size, scores);
            free(scores);
        }
    }
    return failed ? -1 : 0;
}

int pa_oracle_f64(double *out, const void *query, const void *key_cache,
                  const void *value_cache, const int *block_tables,
                  const int *seq_lens, int num_seqs, int num_heads,
                  int head_size, int num_kv_heads, float scale,
                  int max_num_blocks_per_seq, int block_size, int dtype_size,
                  int64_t kv_block_stride, int64_t kv_head_stride,
                  int64_t num_blocks) {
    PA_ARGS_INIT;
    if (check_args(&a) || (num_seqs > 0 && !out)) return -1;
    double *scores = (double *)malloc((size_t)max_len(&a) * sizeof(double));
    if (!scores) return -1;
    const int D = head_size;
    for (int b = 0; b < num_seqs; b++) {
        const int L = seq_tokens(&a, b);
        for (int h = 0; h < num_heads; h++) {
            const int kh = h / (num_heads / num_kv_heads);
            const int64_t qoff = ((int64_t)b * num_heads + h) * D;
            double *o = out + qoff;
            for (int d = 0; d < D; d++) o[d] = 0.0;
            double mx = -INFINITY;
            for (int t = 0; t < L; t++) {
                const int64_t phys = page_of(&a, b, t);
                if (phys < 0) { scores[t] = -INFINITY; continue; }
                const int64_t ko = kv_index(&a, phys, kh, t % block_size);
                double dot = 0.0;
                for (int d = 0; d < D; d++)
                    dot += (double)load_f(query, qoff + d, dtype_size) *
                           (double)load_f(key_cache, ko + d, dtype_size);
                scores[t] = dot * (double)scale;
                if (scores[t] > mx) mx = scores[t];
            }
            if (mx == -INFINITY) continue;
            double sum = 0.0;
            for (int t = 0; t < L; t++) {
                scores[t] = (scores[t] == -INFINITY) ? 0.0 : exp(scores[t] - mx);
                sum += scores[t];
            }
            for (int t = 0; t < L; t++) {
                if (scores[t] == 0.0) continue;
                const int64_t vo = kv_index(&a, page_of(&a, b, t), kh, t % block_size);
                const double w = scores[t] / sum;
                for (int d = 0; d < D; d++) o[d] += w * (double)load_f(value_cache, vo + d, dtype_size);
            }
        }
    }
    free(scores);
    return 0;
}

int pa_oracle_split_partials(float *m, float *l, float *o,
                             const void *query, const void *key_cache,
                             const void *value_cache, const int *block_tables,
                             const int *seq_lens, int num_seqs, int num_heads,
                             int head_size, int num_kv_heads, float scale,
                             int max_num_blocks_per_seq, int block_size,
                             int dtype_size, int64_t kv_block_stride,
                             int64_t kv_head_stride, int64_t num_blocks,
                             int part_pages, int max_parts) {
    PA_ARGS_INIT;
    if (check_args(&a) || part_pages <= 0 || max_parts <= 0) return -1;
    const int D = head_size;
    const int part_tok = part_pages * block_size;
    float *s = (float *)malloc((size_t)part_tok * sizeof(float));
    if (!s) return -1;
    int longest = 0;
    for (int b = 0; b < num_seqs; b++) {
        const int L = seq_tokens(&a, b);
        const int nparts = (L + part_tok - 1) / part_tok;
        if (nparts > longest) longest = nparts;
        for (int h = 0; h < num_heads; h++) {
            const int kh = h / (num_heads / num_kv_heads);
            const int64_t qoff = ((int64_t)b * num_heads + h) * D;
            for (int p = 0; p < max_parts; p++) {
                const int64_t ix = ((int64_t)b * num_heads + h) * max_parts + p;
                float *op = o + ix * D;
                for (int d = 0; d < D; d++) op[d] = 0.0f;
                m[ix] = -INFINITY;
                l[ix] = 0.0f;
                if (p >= nparts) continue;
                const int t0 = p * part_tok;
                const int t1 = (t0 + part_tok < L) ? t0 + part_tok : L;
                float mx = -INFINITY;
                for (int t = t0; t < t1; t++) {
                    const int64_t phys = page_of(&a, b, t);
                    if (phys < 0) { s[t - t0] = -INFINITY; continue; }
                    const int64_t ko = kv_index(&a, phys, kh, t % block_size);
                    float dot = 0.0f;
                    for (int d = 0; d < D; d++)
                        dot += load_f(query, qoff + d, dtype_size) * load_f(key_cache, ko + d, dtype_size);
                    s[t - t0] = dot * scale;
                    if (s[t - t0] > mx) mx = s[t - t0];
                }
                if (mx == -INFINITY) continue;
                float sum = 0.0f;
                for (int t = t0; t < t1; t++) {
                    if (s[t - t0] == -INFINITY) continue;
                    const float e = expf(s[t - t0] - mx);
                    sum += e;
                    const int64_t vo = kv_index(&a, page_of(&a, b, t), kh, t % block_size);
                    for (int d = 0; d < D; d++) op[d] += e * load_f(value_cache, vo + d, dtype_size);
                }
                m[ix] = mx;
                l[ix] = sum;
            }
        }
    }
    free(s);
    return longest;
}

void pa_oracle_merge_partials(float *out, const float *m, const float *l,
                              const float *o, const int *seq_lens,
                              int num_seqs, int num_heads, int head_size,
                              int block_size, int part_pages, int max_parts) {
    const int part_tok = part_pages * block_size;
    for (int b = 0; b < num_seqs; b++) {
        int L = seq_lens[b] < 0 ? 0 : seq_lens[b];
        int nparts = (L + part_tok - 1) / part_tok;
        if (nparts > max_parts) nparts = max_parts;
        for (int h = 0; h < num_heads; h++) {
            float *dst = out + ((int64_t)b * num_heads + h) * head_size;
            const int64_t base = ((int64_t)b * num_heads + h) * max_parts;
            float M = -INFINITY;
            for (int p = 0; p < nparts; p++)
                if (m[base + p] > M) M = m[base + p];
            for (int d = 0; d < head_size; d++) dst[d] = 0.0f;
            if (M == -INFINITY) continue;
            float denom = 0.0f;
            for (int p = 0; p < nparts; p++) {
                if (m[base + p] == -INFINITY) continue;
                const float w = expf(m[base + p] - M);
                denom += w * l[base + p];
                for (int d = 0; d < head_size; d++)
                    dst[d] += w * o[(base + p) * head_size + d];
            }
            for (int d = 0; d < head_size; d++) dst[d] /= denom;
        }
    }
}

/* SplitMix64 output function (Vigna's published finaliser) over a packed
 * (page, slot, kv head) key. */
uint64_t pa_gather_mix(uint64_t phys, uint64_t slot, uint64_t kv_head) {
    uint64_t z = (phys << 24) ^ (slot << 12) ^ kv_head;
    z += 0x9e3779b97f4a7c15ull;
    z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
    z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
    return z ^ (z >> 31);
}

int pa_oracle_gather_checksum(uint64_t *out, const int *block_tables,
                              const int *seq_lens, int num_seqs, int num_heads,
                              int num_kv_heads, int max_num_blocks_per_seq,
                              int block_size, int64_t num_blocks) {
    if (num_seqs < 0 || num_heads <= 0 || num_kv_heads <= 0 ||
        num_heads % num_kv_heads || block_size <= 0)
        return -1;
    pa_args a;
    memset(&a, 0, sizeof(a));
    a.bt = block_tables;
    a.sl = seq_lens;
    a.B = num_seqs;
    a.H = num_heads;
    a.Hkv = num_kv_heads;
    a.max_blocks = max_num_blocks_per_seq;
    a.bs = block_size;
    a.num_blocks = num_blocks;
    for (int b = 0; b < num_seqs; b++) {
        const int L = seq_tokens(&a, b);
        for (int h = 0; h < num_heads; h++) {
            const int kh = h / (num_heads / num_kv_heads);
            uint64_t acc = 0;
            for (int t = 0; t < L; t++) {
                const int64_t phys = page_of(&a, b, t);
                if (phys < 0) continue;
                acc += pa_gather_mix((uint64_t)phys, (uint64_t)(t % block_size), (uint64_t)kh);
            }
            out[(int64_t)b * num_heads + h] = acc;
        }
    }
    return 0;
}

void pa_oracle_reshape_and_cache(const void *key, const void *value, void *key_cache,
                                 void *value_cache, const int64_t *slots, int num_tokens,
                                 int num_kv_heads, int head_size, int block_size,
                                 int elem_size, int64_t kv_block_stride,
                                 int64_t kv_head_stride, int64_t token_stride) {
    const size_t row = (size_t)head_size * (size_t)elem_size;
    for (int t = 0; t < num_tokens; t++) {
        const int64_t slot = slots[t];
        if (slot < 0) continue;
        const int64_t page = slot / block_size, s = slot % block_size;
        for (int h = 0; h < num_kv_heads; h++) {
            const int64_t dst = page * kv_block_stride + (int64_t)h * kv_head_stride + s * head_size;
            const int64_t src = (int64_t)t * token_stride + (int64_t)h * head_size;
            memcpy((char *)key_cache + dst * elem_size, (const char *)key + src * elem_size, row);
            memcpy((char *)value_cache + dst * elem_size, (const char *)value + src * elem_size, row);
        }
    }
}
