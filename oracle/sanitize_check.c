/*
 * sanitize_check.c — runs the repository's host C code under AddressSanitizer
 * and UndefinedBehaviorSanitizer (oracle/Makefile target `sanitize`).
 *
 * TEST INFRASTRUCTURE ONLY. Covered:
 *   - the CPU oracle (pa_oracle.c, act_oracle.c): fp32 / fp64 / OpenMP
 *     attention over fp16 and fp32 pools with GQA, edge lengths (0, 1, 15,
 *     16, 17, 33), masked pages (negative and >= num_blocks), the split /
 *     merge restatement, KV append, one-byte formats, the gather checksum
 *     and every activation;
 *   - the reference's own CPU attention (examples/run_gpt2.c via
 *     ref_shim.c) when the build was given the reference sources
 *     (-DWITH_REF);
 *   - the backend plugin's C logic (xllms_b200/csrc/cuda_backend.c) with the
 *     three libxpa.so functions it calls replaced by stand-ins below: its
 *     NULL contracts, init / run / fini and the descriptor fields it forwards.
 * Exit status 0 and "sanitize ok" on success; a sanitizer report aborts.
 */
#include <math.h>
#include <stddef.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "act_oracle.h"
#include "pa_oracle.h"
#include "cuda_backend.h"
#include "xllm_backend_abi.h"

#define CHECK(c)                                                   \
    do {                                                           \
        if (!(c)) {                                                \
            fprintf(stderr, "check failed: %s (line %d)\n", #c, __LINE__); \
            exit(1);                                               \
        }                                                          \
    } while (0)

static uint64_t rng_state = 0x9E3779B97F4A7C15ull;
static uint64_t next_u64(void) { /* splitmix64 */
    uint64_t z = (rng_state += 0x9E3779B97F4A7C15ull);
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}
static float next_unit(void) { return (float)((next_u64() >> 40) * (1.0 / 16777216.0)) * 2.f - 1.f; }

/* ── oracle ───────────────────────────────────────────────────────────── */
static void check_attention(int dtype_size) {
    enum { B = 7, HQ = 8, HKV = 2, D = 40, BS = 16, MB = 3, NB = 24 };
    const int lens[B] = {0, 1, 15, 16, 17, 33, 48};
    int bt[B * MB];
    for (int i = 0; i < B * MB; i++) bt[i] = (int)(next_u64() % NB);
    bt[5 * MB + 1] = -1;      /* a masked page (negative) */
    bt[6 * MB + 2] = NB + 3;  /* a masked page (>= num_blocks) */
    const int64_t khs = (int64_t)BS * D, kbs = HKV * khs;
    const size_t n_q = (size_t)B * HQ * D, n_kv = (size_t)NB * kbs;
    void *q = malloc(n_q * dtype_size), *k = malloc(n_kv * dtype_size), *v = malloc(n_kv * dtype_size);
    CHECK(q && k && v);
    for (size_t i = 0; i < n_q; i++) {
        const float x = next_unit();
        if (dtype_size == 2) ((uint16_t *)q)[i] = pa_float_to_half(x); else ((float *)q)[i] = x;
    }
    for (size_t i = 0; i < n_kv; i++) {
        const float a = next_unit(), c = next_unit();
        if (dtype_size == 2) {
            ((uint16_t *)k)[i] = pa_float_to_half(a);
            ((uint16_t *)v)[i] = pa_float_to_half(c);
        } else {
            ((float *)k)[i] = a;
            ((float *)v)[i] = c;
        }
    }
    float *o32 = malloc(n_q * sizeof(float)), *omp = malloc(n_q * sizeof(float));
    float *merged = malloc(n_q * sizeof(float));
    double *o64 = malloc(n_q * sizeof(double));
    CHECK(o32 && omp && merged && o64);
    const float scale = 1.f / sqrtf((float)D);
    CHECK(pa_oracle_f32(o32, q, k, v, bt, lens, B, HQ, D, HKV, scale, MB, BS, dtype_size, kbs,
                        khs, NB) == 0);
    CHECK(pa_oracle_f64(o64, q, k, v, bt, lens, B, HQ, D, HKV, scale, MB, BS, dtype_size, kbs,
                        khs, NB) == 0);
    CHECK(pa_oracle_f32_omp(omp, q, k, v, bt, lens, B, HQ, D, HKV, scale, MB, BS, dtype_size,
                            kbs, khs, NB, 2) == 0);
    for (size_t i = 0; i < n_q; i++) {
        CHECK(fabs((double)o32[i] - o64[i]) < 1e-4);
        CHECK(o32[i] == omp[i]);
    }
    for (int d = 0; d < HQ * D; d++) CHECK(o32[d] == 0.f); /* seq_len 0: zero rows */

    /* split partitions of one page each, then the log-sum-exp merge */
    const int parts = MB;
    float *m = malloc((size_t)B * HQ * parts * sizeof(float));
    float *l = malloc((size_t)B * HQ * parts * sizeof(float));
    float *o = malloc((size_t)B * HQ * parts * D * sizeof(float));
    CHECK(m && l && o);
    CHECK(pa_oracle_split_partials(m, l, o, q, k, v, bt, lens, B, HQ, D, HKV, scale, MB, BS,
                                   dtype_size, kbs, khs, NB, 1, parts) >= 1);
    pa_oracle_merge_partials(merged, m, l, o, lens, B, HQ, D, BS, 1, parts);
    for (size_t i = 0; i < n_q; i++) CHECK(fabs((double)merged[i] - o64[i]) < 1e-4);

    uint64_t sums[B * HQ];
    CHECK(pa_oracle_gather_checksum(sums, bt, lens, B, HQ, HKV, MB, BS, NB) == 0);
    CHECK(sums[0] == 0);

    /* KV append into fresh pools: a bit copy, negative slots skipped */
    enum { T = 5 };
    const int64_t slots[T] = {0, 17, -1, 5 * BS + 3, NB * BS - 1};
    void *kc = calloc(n_kv, dtype_size), *vc = calloc(n_kv, dtype_size);
    CHECK(kc && vc);
    pa_oracle_reshape_and_cache(k, v, kc, vc, slots, T, HKV, D, BS, dtype_size, kbs, khs,
                                (int64_t)HKV * D);
    CHECK(memcmp(kc, k, (size_t)D * dtype_size) == 0);

    free(kc); free(vc); free(m); free(l); free(o);
    free(q); free(k); free(v); free(o32); free(omp); free(merged); free(o64);
}

static void check_one_byte(void) {
    enum { N = 1024 };
    float x[N], back[N];
    uint8_t c[N];
    for (int i = 0; i < N; i++) x[i] = next_unit() * 300.f;
    x[0] = NAN;
    x[1] = INFINITY;
    x[2] = -1e30f;
    for (int fmt = PA_FP8_E4M3; fmt <= PA_KV_INT8; fmt++) {
        pa_fp8_encode(c, x, N, fmt);
        pa_fp8_decode(back, c, N, fmt);
        for (int i = 3; i < N; i++) CHECK(isfinite(back[i]));
    }
}

static void check_activations(void) {
    enum { TOK = 3, DIM = 37 };
    for (int ds = 2; ds <= 4; ds += 2) {
        void *in = malloc((size_t)TOK * 2 * DIM * ds), *out = malloc((size_t)TOK * 2 * DIM * ds);
        CHECK(in && out);
        for (int i = 0; i < TOK * 2 * DIM; i++) {
            const float x = next_unit() * 4.f;
            if (ds == 2) ((uint16_t *)in)[i] = pa_float_to_half(x); else ((float *)in)[i] = x;
        }
        for (int op = 0; op <= 5; op++) CHECK(act_oracle(op, out, in, TOK, DIM, ds) == 0);
        CHECK(act_oracle(6, out, in, TOK, DIM, ds) == -1);
        free(in);
        free(out);
    }
}

/* ── the reference's CPU attention (examples/run_gpt2.c via ref_shim.c) ── */
#ifdef WITH_REF
void ref_run_gpt2_batch(const float *query, const float *key_cache, const float *value_cache,
                        const int *page_tables, const int *seq_lens, int num_seqs,
                        int max_tokens, int num_heads, int head_dim, int page_size,
                        float *output, int nthreads);
static void check_reference(void) {
    enum { B = 3, H = 4, D = 16, PS = 16, MAXT = 40, PAGES = 8 };
    const int lens[B] = {1, 17, 40};
    int pt[B * MAXT];
    for (int i = 0; i < B * MAXT; i++) pt[i] = (int)(next_u64() % PAGES);
    const size_t n_kv = (size_t)PAGES * PS * H * D;
    float *k = malloc(n_kv * sizeof(float)), *v = malloc(n_kv * sizeof(float));
    float q[B * H * D], out[B * H * D];
    CHECK(k && v);
    for (size_t i = 0; i < n_kv; i++) {
        k[i] = next_unit();
        v[i] = next_unit();
    }
    for (int i = 0; i < B * H * D; i++) q[i] = next_unit();
    ref_run_gpt2_batch(q, k, v, pt, lens, B, MAXT, H, D, PS, out, 2);
    for (int i = 0; i < B * H * D; i++) CHECK(isfinite(out[i]));
    free(k);
    free(v);
}
#endif

/* ── the backend plugin, its libxpa.so calls replaced ─────────────────── */
static NxtPagedAttentionInput g_seen;
static void *g_seen_out;
static int g_calls;

int nxt_paged_attention_device_info(int *device_id, int *sm_count, char *name, int name_len) {
    if (device_id) *device_id = 0;
    if (sm_count) *sm_count = 148;
    if (name && name_len > 0) snprintf(name, (size_t)name_len, "%s", "stand-in device");
    return NXT_PA_OK;
}

void nxt_paged_attention(void *out, const void *query, const void *key_cache,
                         const void *value_cache, const int *block_tables, const int *seq_lens,
                         int num_seqs, int num_heads, int head_size, int num_kv_heads,
                         float scale, int max_num_blocks_per_seq, int block_size,
                         int dtype_size, int kv_block_stride, int kv_head_stride,
                         nxt_stream_t stream) {
    g_calls++;
    g_seen_out = out;
    g_seen.query = query;
    g_seen.key_cache = key_cache;
    g_seen.value_cache = value_cache;
    g_seen.block_tables = block_tables;
    g_seen.seq_lens = seq_lens;
    g_seen.num_seqs = num_seqs;
    g_seen.num_heads = num_heads;
    g_seen.head_size = head_size;
    g_seen.num_kv_heads = num_kv_heads;
    g_seen.scale = scale;
    g_seen.max_num_blocks_per_seq = max_num_blocks_per_seq;
    g_seen.block_size = block_size;
    g_seen.dtype_size = dtype_size;
    g_seen.kv_block_stride = kv_block_stride;
    g_seen.kv_head_stride = kv_head_stride;
    g_seen.stream = stream;
}

int nxt_paged_attention_last_error(void) { return NXT_PA_OK; }

static int g_releases;
int nxt_paged_attention_release_workspaces(void) {
    g_releases++;
    return NXT_PA_OK;
}

static void check_plugin(void) {
    CHECK(nxt_backend_init(NULL) == -1);
    CHECK(nxt_backend_run(NULL, NULL, NULL) == -1);
    CHECK(nxt_backend_fini(NULL) == -1);
    NxtBackend be;
    memset(&be, 0, sizeof(be));
    int dummy = 0;
    CHECK(nxt_backend_run(&be, &dummy, &dummy) == -1); /* not initialised */
    CHECK(nxt_backend_init(&be) == 0);
    CHECK(be.state == NXT_BACKEND_STATE_READY && be.backend_state != NULL);
    CHECK(nxt_backend_run(&be, NULL, &dummy) == -1);
    CHECK(nxt_backend_run(&be, &dummy, NULL) == -1);
    CHECK(g_calls == 0);
    NxtPagedAttentionInput in;
    memset(&in, 0, sizeof(in));
    in.query = &dummy;
    in.num_seqs = 3;
    in.num_heads = 32;
    in.head_size = 128;
    in.num_kv_heads = 8;
    in.scale = 0.125f;
    in.max_num_blocks_per_seq = 9;
    in.block_size = 16;
    in.dtype_size = 2;
    in.kv_block_stride = 8 * 16 * 128;
    in.kv_head_stride = 16 * 128;
    float out_buf[4];
    CHECK(nxt_backend_run(&be, &in, out_buf) == 0);
    CHECK(g_calls == 1 && g_seen_out == out_buf && g_seen.query == &dummy);
    CHECK(memcmp(&g_seen.num_seqs, &in.num_seqs,
                 offsetof(NxtPagedAttentionInput, stream) -
                     offsetof(NxtPagedAttentionInput, num_seqs)) == 0);
    CHECK(nxt_backend_fini(&be) == 0);
    CHECK(be.state == NXT_BACKEND_STATE_UNINITIALIZED && be.backend_state == NULL);
    CHECK(g_releases == 1); /* fini hands the library's workspaces back */
}

int main(void) {
    check_attention(2);
    check_attention(4);
    check_one_byte();
    check_activations();
#ifdef WITH_REF
    check_reference();
#endif
    check_plugin();
    printf("sanitize ok%s\n",
#ifdef WITH_REF
           " (with the reference's CPU attention)"
#else
           ""
#endif
    );
    return 0;
}
