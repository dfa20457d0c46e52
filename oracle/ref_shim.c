/*
 * ref_shim.c — exposes the reference's own CPU paged attention.
 *
 * TEST INFRASTRUCTURE ONLY. The reference keeps its only paged CPU attention
 * as a file-static function inside an example program
 * (examples/run_gpt2.c:46-83, `static void paged_attention(...)`). This shim
 * compiles that source file in place (its path comes from the build recipe,
 * oracle/Makefile; nothing is copied) with its `main` renamed, and adds
 * non-static entry points so tests and the bench's reference arm can call it.
 *
 * The reference function's contract (run_gpt2.c:46-83):
 *   - MHA, fp32, one page-table entry per token (page_table[t]), slot t % page_size;
 *   - cache layout [page][slot][num_heads][head_dim];
 *   - scale fixed at 1/sqrt(head_dim); softmax without max subtraction.
 */
#define main xllm_reference_run_gpt2_main
#include REF_RUN_GPT2_C
#undef main

#ifdef _OPENMP
#include <omp.h>
#endif

/* One sequence: forwards to the reference function unchanged. */
void ref_run_gpt2_paged_attention(const float *query, const float *key_cache,
                                  const float *value_cache, const int *page_table,
                                  int seq_len, int num_heads, int head_dim,
                                  int page_size, float *output) {
    paged_attention(query, key_cache, value_cache, page_table, seq_len,
                    num_heads, head_dim, page_size, output);
}

/* A batch of sequences, one reference call per sequence, spread over
 * nthreads OpenMP threads (<= 0: all). query/output are [num_seqs][num_heads][head_dim];
 * page_tables is [num_seqs][max_tokens]. */
void ref_run_gpt2_batch(const float *query, const float *key_cache,
                        const float *value_cache, const int *page_tables,
                        const int *seq_lens, int num_seqs, int max_tokens,
                        int num_heads, int head_dim, int page_size,
                        float *output, int nthreads) {
#ifdef _OPENMP
    if (nthreads <= 0) nthreads = omp_get_max_threads();
#pragma omp parallel for schedule(dynamic, 1) num_threads(nthreads)
#else
    (void)nthreads;
#endif
    for (int b = 0; b < num_seqs; b++) {
        const long long row = (long long)b * num_heads * head_dim;
        paged_attention(query + row, key_cache, value_cache,
                        page_tables + (long long)b * max_tokens, seq_lens[b],
                        num_heads, head_dim, page_size, output + row);
    }
}

int ref_run_gpt2_max_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}
