/*
 * pa_oracle.h — CPU restatement of xLLMs paged decode attention.
 *
 * TEST INFRASTRUCTURE ONLY. This library is the checker for the CUDA
 * kernels in xllms_b200/csrc; only tests/, __graft_entry__.smoke() and the
 * cpu_baseline / reference legs of bench.py may load it. The product path
 * never calls it.
 *
 * Semantics followed (reference file:line, paths within the xLLMs project):
 *   - argument meaning and layout: include/operator_api.h:35-72
 *       q, out            [num_seqs][num_heads][head_size]
 *       key/value cache   element (phys, kvh, slot, d) at
 *                         phys*kv_block_stride + kvh*kv_head_stride + slot*head_size + d
 *                         (operators/page_attention.cu:112-115, page_attention_v2.cu:143-146)
 *       token t of seq b  page block_tables[b*max_blocks + t/block_size], slot t%block_size
 *   - GQA head mapping    kv head = q head / (num_heads/num_kv_heads)  (examples/text_gen.c:1285)
 *   - softmax             scores = scale*dot, max-subtracted expf, w = e/sum, o += w*v
 *                         (examples/text_gen.c:1288-1309)
 *   - empty sequence      seq_len == 0 gives an all-zero row (inv_sum = 0,
 *                         operators/page_attention.cu:157)
 *   - dtype_size          2 = IEEE binary16, 4 = binary32, for q, k, v and out alike
 *                         (backends/cuda_backend.h:43)
 *
 * Pages whose block-table entry is negative, or >= num_blocks when num_blocks
 * is known (> 0), are masked: their tokens take no part in the softmax. The
 * reference has no defined behaviour for such entries (its CPU code indexes
 * out of bounds; its V1 kernel stops the page loop).
 */
#ifndef XPA_ORACLE_H_
#define XPA_ORACLE_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

float    pa_half_to_float(uint16_t h);
uint16_t pa_float_to_half(float f);

/* fp32 accumulation, output fp32 [num_seqs][num_heads][head_size].
 * Returns 0, or -1 on an invalid argument. */
int pa_oracle_f32(float *out, const void *query, const void *key_cache,
                  const void *value_cache, const int *block_tables,
                  const int *seq_lens, int num_seqs, int num_heads,
                  int head_size, int num_kv_heads, float scale,
                  int max_num_blocks_per_seq, int block_size, int dtype_size,
                  int64_t kv_block_stride, int64_t kv_head_stride,
                  int64_t num_blocks);

/* Same, with fp64 accumulation and fp64 output: bounds the fp32 oracle's own error. */
int pa_oracle_f64(double *out, const void *query, const void *key_cache,
                  const void *value_cache, const int *block_tables,
                  const int *seq_lens, int num_seqs, int num_heads,
                  int head_size, int num_kv_heads, float scale,
                  int max_num_blocks_per_seq, int block_size, int dtype_size,
                  int64_t kv_block_stride, int64_t kv_head_stride,
                  int64_t num_blocks);

/* pa_oracle_f32 spread over (seq, head) pairs with OpenMP; nthreads <= 0 uses all. */
int pa_oracle_f32_omp(float *out, const void *query, const void *key_cache,
                      const void *value_cache, const int *block_tables,
                      const int *seq_lens, int num_seqs, int num_heads,
                      int head_size, int num_kv_heads, float scale,
                      int max_num_blocks_per_seq, int block_size,
                      int dtype_size, int64_t kv_block_stride,
                      int64_t kv_head_stride, int64_t num_blocks,
                      int nthreads);

/* Split-context restatement: partition p of seq b covers pages
 * [p*part_pages, (p+1)*part_pages). Per (b, h, p) it writes the running max m
 * (natural-log domain, of scale*dot), the sum l of exp(s - m) and the
 * unnormalised o = sum exp(s - m) * v. Layout: m, l [B][H][max_parts],
 * o [B][H][max_parts][D]. Partitions with no valid token get m = -INF, l = 0,
 * o = 0. Returns the number of partitions of the longest sequence. */
int pa_oracle_split_partials(float *m, float *l, float *o,
                             const void *query, const void *key_cache,
                             const void *value_cache, const int *block_tables,
                             const int *seq_lens, int num_seqs, int num_heads,
                             int head_size, int num_kv_heads, float scale,
                             int max_num_blocks_per_seq, int block_size,
                             int dtype_size, int64_t kv_block_stride,
                             int64_t kv_head_stride, int64_t num_blocks,
                             int part_pages, int max_parts);

/* Log-sum-exp merge of the partials above into out [B][H][D]. */
void pa_oracle_merge_partials(float *out, const float *m, const float *l,
                              const float *o, const int *seq_lens,
                              int num_seqs, int num_heads, int head_size,
                              int block_size, int part_pages, int max_parts);

/* KV append restated: token t's rows (t*token_stride + h*head_size + d) are
 * copied to page slots[t]/block_size, slot slots[t]%block_size of the pools
 * (negative slot: skipped). elem_size bytes per element (bit copy). The
 * reference has no paged writer; its decode loop copies each new token into
 * a contiguous cache (examples/text_gen.c:1274-1278). */
void pa_oracle_reshape_and_cache(const void *key, const void *value, void *key_cache,
                                 void *value_cache, const int64_t *slots, int num_tokens,
                                 int num_kv_heads, int head_size, int block_size,
                                 int elem_size, int64_t kv_block_stride,
                                 int64_t kv_head_stride, int64_t token_stride);

/* One-byte formats of a quantised KV cache (fmt): 1 = fp8 E4M3 (no
 * infinities, max 448, 0x7F NaN), 2 = fp8 E5M2 (max 57344), 3 = int8
 * (two's complement). decode is exact; encode rounds to nearest even and
 * saturates at the largest finite value (as the PTX cvt.rn.satfinite
 * conversions do); NaN stays NaN in fp8 and encodes as 0 in int8 (as a
 * float-to-integer conversion does). A quantised cache holds
 * encode(x / scale) and reads back as decode(c) * scale. */
#define PA_FP8_E4M3 1
#define PA_FP8_E5M2 2
#define PA_KV_INT8 3
void pa_fp8_decode(float *out, const uint8_t *in, int64_t n, int fmt);
void pa_fp8_encode(uint8_t *out, const float *in, int64_t n, int fmt);

/* Index-logic checksum: for every (seq, q head), the wrapping 64-bit sum of
 * pa_gather_mix(phys, slot, kv_head) over every token the attention reads. */
uint64_t pa_gather_mix(uint64_t phys, uint64_t slot, uint64_t kv_head);
int pa_oracle_gather_checksum(uint64_t *out, const int *block_tables,
                              const int *seq_lens, int num_seqs, int num_heads,
                              int num_kv_heads, int max_num_blocks_per_seq,
                              int block_size, int64_t num_blocks);

#ifdef __cplusplus
}
#endif
#endif /* XPA_ORACLE_H_ */
