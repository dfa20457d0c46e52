/*
 * operator_api.h — paged decode attention, C ABI of libxpa.so.
 *
 * Drop-in for the xLLMs operator header (include/operator_api.h of the xLLMs
 * project): the three attention entry points keep their names, argument order,
 * argument meaning and `void` return, and all of them have C linkage. Behind
 * them sit hand-written sm_100a kernels (xllms_b200/csrc). Additions are
 * marked "extension" and have no counterpart in the reference header.
 *
 * Layout contract (identical to the reference):
 *   out, query   [num_seqs][num_heads][head_size], element type by dtype_size
 *   key_cache,   element (page, kv_head, slot, d) at
 *   value_cache    page*kv_block_stride + kv_head*kv_head_stride + slot*head_size + d
 *   block_tables [num_seqs][max_num_blocks_per_seq] int32 physical page ids;
 *                token t of sequence b lives in page block_tables[b][t / block_size]
 *                at slot t % block_size
 *   seq_lens     [num_seqs] int32 context lengths
 *   query head h reads KV head h / (num_heads / num_kv_heads)
 *   dtype_size   2 = fp16, 4 = fp32, for query, caches and out alike
 * All pointers are device pointers; every call is asynchronous on `stream`
 * (NULL = the legacy default stream) and the caller synchronises.
 *
 * Behaviour the reference leaves undefined, defined here:
 *   - block_size is honoured (the reference kernels hard-code 16);
 *   - a block-table entry < 0 (or >= num_blocks when the _ex call gives it)
 *     masks that page's tokens out of the softmax and raises
 *     NXT_PA_DEV_BAD_PAGE in the device status word;
 *   - seq_len is clamped to [0, max_num_blocks_per_seq*block_size]
 *     (NXT_PA_DEV_SEQ_CLAMPED when clamping happened);
 *   - seq_len == 0 writes an all-zero output row (as the reference's inv_sum = 0);
 *   - an unsupported shape or dtype launches nothing and records NXT_PA_EINVAL
 *     (read it with nxt_paged_attention_last_error) instead of silently falling
 *     back to another head size.
 */
#ifndef XPA_OPERATOR_API_H_
#define XPA_OPERATOR_API_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Opaque stream handle: a cudaStream_t cast to void* (reference operator_api.h:29). */
typedef void *nxt_stream_t;

/* Replaces nxt_paged_attention (reference include/operator_api.h:63-72,
 * operators/page_attention.cu:170). Supported: dtype_size 2 or 4, any
 * head_size in 1..256, any num_heads that is a multiple of num_kv_heads. */
void nxt_paged_attention(
    void *out, const void *query,
    const void *key_cache, const void *value_cache,
    const int *block_tables, const int *seq_lens,
    int num_seqs, int num_heads, int head_size,
    int num_kv_heads, float scale,
    int max_num_blocks_per_seq,
    int block_size, int dtype_size,
    int kv_block_stride, int kv_head_stride,
    nxt_stream_t stream);

/* Replaces nxt_paged_attention_v2 (reference include/operator_api.h:84-93,
 * operators/page_attention_v2.cu:262). Same computation and kernels as above. */
void nxt_paged_attention_v2(
    void *out, const void *query,
    const void *key_cache, const void *value_cache,
    const int *block_tables, const int *seq_lens,
    int num_seqs, int num_heads, int head_size,
    int num_kv_heads, float scale,
    int max_num_blocks_per_seq,
    int block_size, int dtype_size,
    int kv_block_stride, int kv_head_stride,
    nxt_stream_t stream);

/* Replaces nxt_paged_attention_flash (reference include/operator_api.h:106-115,
 * operators/flashinfer_adapter.cu:329, built there only with USE_FLASHINFER;
 * always exported here). Same computation and kernels as above. */
void nxt_paged_attention_flash(
    void *out, const void *query,
    const void *key_cache, const void *value_cache,
    const int *block_tables, const int *seq_lens,
    int num_seqs, int num_heads, int head_size,
    int num_kv_heads, float scale,
    int max_num_blocks_per_seq,
    int block_size, int dtype_size,
    int kv_block_stride, int kv_head_stride,
    nxt_stream_t stream);

/* ── extension: status codes ──────────────────────────────────────────── */
#define NXT_PA_OK              0
#define NXT_PA_EINVAL        (-22) /* unsupported or inconsistent arguments   */
#define NXT_PA_ENOMEM        (-12) /* workspace allocation failed             */
#define NXT_PA_EWORKSPACE    (-28) /* caller workspace smaller than required  */
#define NXT_PA_ECUDA         (-5)  /* a CUDA runtime/driver call failed       */

/* Device status word bits (set by the kernels, read by
 * nxt_paged_attention_device_status). */
#define NXT_PA_DEV_TIMEOUT     0x1 /* a bounded pipeline wait expired          */
#define NXT_PA_DEV_BAD_PAGE    0x2 /* a block-table entry was masked           */
#define NXT_PA_DEV_SEQ_CLAMPED 0x4 /* a seq_len was outside [0, max_blocks*block_size] */

/* Kernel paths (nxt_paged_attention_path). */
#define NXT_PA_PATH_NONE       0
#define NXT_PA_PATH_TMA_MMA    1 /* fp16, block_size 16, head_size 64/128/256 */
#define NXT_PA_PATH_GENERIC    2 /* every other supported shape               */

/* extension — status of the last drop-in call (nxt_paged_attention{,_v2,_flash})
 * made by the calling host thread: NXT_PA_OK or a negative code. */
int nxt_paged_attention_last_error(void);

/* extension — human-readable text for a status code. */
const char *nxt_paged_attention_strerror(int code);

/* extension — status-returning form of the calls above.
 *   num_blocks        pages in each cache pool; > 0 lets the kernels mask
 *                     entries >= num_blocks, <= 0 means unknown.
 *   workspace         device memory for split-context partials, at least
 *                     nxt_paged_attention_workspace_size(...) bytes and
 *                     starting on a 16-byte boundary (NXT_PA_EINVAL
 *                     otherwise), or NULL to use the library's per-(device,
 *                     stream) workspace, which is allocated on first use and
 *                     grown as needed. The same rule holds for every _ex call
 *                     that takes a workspace.
 *   device_status     device int the kernels OR their NXT_PA_DEV_* bits into,
 *                     or NULL for the library's per-device status word.
 * Returns NXT_PA_OK once the kernels are enqueued, else a negative code.
 * Partials of one call live in the workspace until the call's kernels finish,
 * so concurrent calls need distinct workspaces. A call whose sequences span
 * more than one partition launches two kernels (attention, then the merge). */
int nxt_paged_attention_ex(
    void *out, const void *query,
    const void *key_cache, const void *value_cache,
    const int *block_tables, const int *seq_lens,
    int num_seqs, int num_heads, int head_size,
    int num_kv_heads, float scale,
    int max_num_blocks_per_seq,
    int block_size, int dtype_size,
    int64_t kv_block_stride, int64_t kv_head_stride,
    int64_t num_blocks,
    void *workspace, size_t workspace_bytes,
    int *device_status,
    nxt_stream_t stream);

/* extension — bytes of workspace a call with these arguments needs (0 when
 * no sequence can span more than one context partition). */
size_t nxt_paged_attention_workspace_size(
    int num_seqs, int num_heads, int head_size, int num_kv_heads,
    int max_num_blocks_per_seq, int block_size, int dtype_size);

/* extension — kernel path a call with these arguments takes (NXT_PA_PATH_*),
 * NXT_PA_PATH_NONE when the arguments are unsupported. Pointer alignment is
 * checked too, so pass the real cache pointers. */
int nxt_paged_attention_path(
    const void *key_cache, const void *value_cache,
    int num_heads, int head_size, int num_kv_heads,
    int block_size, int dtype_size,
    int64_t kv_block_stride, int64_t kv_head_stride);

/* extension — reads (and with clear != 0 resets) the current device's library
 * status word. Synchronises the device. Returns the NXT_PA_DEV_* bits, or a
 * negative code. */
int nxt_paged_attention_device_status(int clear);

/* extension — frees the library-owned workspaces and status words of every
 * device. Synchronises each device that has one. */
int nxt_paged_attention_release_workspaces(void);

/* extension, no counterpart in the reference — paged decode attention that
 * allocates no device memory, for callers that cannot allocate: a serving
 * engine that has reserved nearly all of HBM for its KV page pool, or a host
 * that routes every device allocation through its own pool, has no room for
 * (or forbids) a library's cudaMalloc, and cudaMalloc/cudaFree synchronise
 * the device mid decode loop. Same arguments and results as
 * nxt_paged_attention_ex without the workspace: split-context partials live
 * in one fixed array of NXT_PA_NOALLOC_SCRATCH_BYTES compiled into the
 * library, which every GPU that loads it holds until the process exits.
 *   - Limit: a call needing more partial storage than the array
 *     (nxt_paged_attention_workspace_size(...) > NXT_PA_NOALLOC_SCRATCH_BYTES)
 *     returns NXT_PA_ESCRATCH and launches nothing.
 *   - The first call on each device looks up the array's device address
 *     (set-up); make that first call before any stream capture. The address
 *     is kept for the life of the process: after cudaDeviceReset on a device
 *     (which unloads the library's module there) this entry point must not
 *     be called on that device again.
 *   - Its kernels' pipeline waits follow nxt_paged_attention_set_wait_budget_ns
 *     like every other call from the same host thread.
 *   - Every call shares the one array and leaves its partials there; calls
 *     whose kernels overlap on the GPU (other streams, other host threads on
 *     the same device) race on it. Nothing in it needs clearing between calls.
 *   - device_status: a caller-owned device int for NXT_PA_DEV_* bits, or NULL. */
#define NXT_PA_NOALLOC_SCRATCH_BYTES (32u << 20)
#define NXT_PA_ESCRATCH      (-27) /* request exceeds the fixed no-alloc scratch */
int nxt_paged_attention_noalloc(
    void *out, const void *query,
    const void *key_cache, const void *value_cache,
    const int *block_tables, const int *seq_lens,
    int num_seqs, int num_heads, int head_size,
    int num_kv_heads, float scale,
    int max_num_blocks_per_seq,
    int block_size, int dtype_size,
    int64_t kv_block_stride, int64_t kv_head_stride,
    int64_t num_blocks,
    int *device_status,
    nxt_stream_t stream);

/* extension — failure-detection testing: sets the bound on every pipeline
 * wait inside the kernels launched by later calls from this host thread
 * (default 1 s; each wait gives up after that much %globaltimer time, raises
 * NXT_PA_DEV_TIMEOUT and the kernel winds down, letting its own in-flight
 * copies land under a separate 1 s bound). Returns the previous budget. A
 * tiny budget makes the waits run out on purpose without faulting the GPU. */
uint64_t nxt_paged_attention_set_wait_budget_ns(uint64_t budget_ns);

/* ── extension: KV append (no paged writer exists in the
 * reference, whose decode loop memcpy's each token into a contiguous cache,
 * examples/text_gen.c:1274-1278) ──────────────────────────────────────
 * Writes token t's key and value rows (key/value[t*token_stride + h*head_size
 * + d], h < num_kv_heads) into the paged pools at page slot_mapping[t] /
 * block_size, slot slot_mapping[t] % block_size; a negative slot skips the
 * token. Bit-exact copy. */
int nxt_reshape_and_cache(
    const void *key, const void *value,
    void *key_cache, void *value_cache,
    const int64_t *slot_mapping, int num_tokens,
    int num_kv_heads, int head_size, int block_size, int dtype_size,
    int64_t kv_block_stride, int64_t kv_head_stride, int64_t token_stride,
    nxt_stream_t stream);

/* Decode step with the append fused in: writes new_key/new_value
 * ([num_seqs][num_kv_heads][head_size], one new token per sequence) at
 * slot_mapping[b], then runs nxt_paged_attention_ex over seq_lens (which
 * already count the new token). The attention grid is launched as a
 * programmatic dependent of the append: only the load of each sequence's
 * last page waits for the append, every other page streams meanwhile. */
int nxt_paged_attention_append_ex(
    void *out, const void *query,
    void *key_cache, void *value_cache,
    const int *block_tables, const int *seq_lens,
    const void *new_key, const void *new_value, const int64_t *slot_mapping,
    int num_seqs, int num_heads, int head_size,
    int num_kv_heads, float scale,
    int max_num_blocks_per_seq,
    int block_size, int dtype_size,
    int64_t kv_block_stride, int64_t kv_head_stride,
    int64_t num_blocks,
    int *device_status,
    nxt_stream_t stream);

/* ── extension: one-byte KV cache (reference operators/cache.py:16-24 lists
 * "fp8", "fp8_e4m3", "fp8_e5m2" and "int8" cache dtypes; no kernel there
 * reads them) ──
 * The pools hold one byte per element, encode(x / k_scale) for K and
 * encode(x / v_scale) for V; attention reads decode(byte) * scale. Query and
 * output are fp16; strides are in elements (= bytes). Head sizes 128 and 256
 * with page size 16 take the TMA + tensor-core path; every other shape the
 * CUDA-core kernel. Results are those of nxt_paged_attention_ex over the
 * dequantised cache. A caller-owned workspace needs
 * nxt_paged_attention_fp8_workspace_size bytes. */
#define NXT_KV_FP8_E4M3 1 /* 4 exponent bits, no infinities, max 448   */
#define NXT_KV_FP8_E5M2 2 /* 5 exponent bits, max 57344                 */
#define NXT_KV_INT8     3 /* two's-complement int8, -128 .. 127          */

int nxt_paged_attention_fp8_ex(
    void *out, const void *query,
    const void *key_cache, const void *value_cache,
    const int *block_tables, const int *seq_lens,
    int num_seqs, int num_heads, int head_size,
    int num_kv_heads, float scale,
    int max_num_blocks_per_seq, int block_size,
    int kv_format, float k_scale, float v_scale,
    int64_t kv_block_stride, int64_t kv_head_stride,
    int64_t num_blocks,
    void *workspace, size_t workspace_bytes,
    int *device_status,
    nxt_stream_t stream);

/* Workspace bytes a nxt_paged_attention_fp8_ex call with these sizes needs
 * (fp8 pools may take shorter context partitions than fp16 ones). */
size_t nxt_paged_attention_fp8_workspace_size(int num_seqs, int num_heads, int head_size,
                                              int num_kv_heads, int max_num_blocks_per_seq,
                                              int block_size);

/* KV append into one-byte pools: fp16 key/value rows ([num_tokens]
 * [num_kv_heads][head_size] at token_stride) are stored at slot_mapping[t]
 * as encode(x / scale), rounded to nearest even and saturated at the
 * format's largest finite value (fp8: NaN stays NaN; int8: NaN gives 0). */
int nxt_reshape_and_cache_fp8(
    const void *key, const void *value,
    void *key_cache, void *value_cache,
    const int64_t *slot_mapping, int num_tokens,
    int num_kv_heads, int head_size, int block_size,
    int kv_format, float k_scale, float v_scale,
    int64_t kv_block_stride, int64_t kv_head_stride, int64_t token_stride,
    nxt_stream_t stream);

/* Decode step on one-byte pools with the quantising append fused in:
 * new_key/new_value (fp16 [num_seqs][num_kv_heads][head_size], one new token
 * per sequence) are stored at slot_mapping[b] as nxt_reshape_and_cache_fp8
 * stores them, then nxt_paged_attention_fp8_ex runs over seq_lens (which
 * already count the new token) with the library's own workspace. The
 * attention grid is a programmatic dependent of the append: only the load of
 * each sequence's last page waits for it. */
int nxt_paged_attention_fp8_append_ex(
    void *out, const void *query,
    void *key_cache, void *value_cache,
    const int *block_tables, const int *seq_lens,
    const void *new_key, const void *new_value, const int64_t *slot_mapping,
    int num_seqs, int num_heads, int head_size,
    int num_kv_heads, float scale,
    int max_num_blocks_per_seq, int block_size,
    int kv_format, float k_scale, float v_scale,
    int64_t kv_block_stride, int64_t kv_head_stride,
    int64_t num_blocks,
    int *device_status,
    nxt_stream_t stream);

/* ── extension: block-table builder ─────────────────────────────────────
 * The glue between a continuous-batching scheduler and these kernels (the
 * reference's scheduler, src/core/scheduler.c:278-440, stops at the list of
 * scheduled requests). Host inputs, CSR over the step's sequences:
 *   page_offsets [num_seqs + 1], page_ids [page_offsets[num_seqs]]: each
 *     sequence's physical pages in token order;
 *   seq_lens [num_seqs]: context tokens, the newest one included;
 *   prefix_node / prefix_pages [num_seqs] (both NULL, or both given): the
 *     radix-tree node of a sequence's longest shared prefix (-1: none) and
 *     the whole pages it covers.
 * Outputs, in one caller-owned device buffer (16-byte aligned, at least
 * nxt_block_tables_layout bytes; offsets from the same call):
 *   NXT_BT_TABLES        int32 [num_seqs][max_blocks], -1 past a sequence's pages
 *   NXT_BT_SEQ_LENS      int32 [num_seqs]
 *   NXT_BT_SLOTS         int64 [num_seqs], page * block_size + slot of the
 *                        newest token (the KV append's slot_mapping; -1 when
 *                        seq_len is 0)
 *   NXT_BT_PREFIX_PAGES, NXT_BT_GROUP_OFFSETS, NXT_BT_GROUP_MEMBERS: the
 *     prefix groups of nxt_paged_attention_prefix_ex — sequences sharing a
 *     node with >= 1 whole page, groups of two or more; *num_groups,
 *     *max_group_size and *max_prefix_pages receive its host bounds.
 * The host packs the inputs into host_staging (pinned, at least
 * nxt_block_tables_staging_size bytes; NULL: a temporary, and the call
 * synchronises the stream) and issues one host-to-device copy and one
 * kernel. EINVAL: a row longer than max_blocks, seq_len beyond its pages, a
 * group whose members differ in shared page count or ids. */
#define NXT_BT_TABLES        0
#define NXT_BT_SEQ_LENS      1
#define NXT_BT_SLOTS         2
#define NXT_BT_PREFIX_PAGES  3
#define NXT_BT_GROUP_OFFSETS 4
#define NXT_BT_GROUP_MEMBERS 5
#define NXT_BT_NUM_ARRAYS    6

size_t nxt_block_tables_layout(int num_seqs, int max_blocks_per_seq, int total_pages,
                               size_t offsets[NXT_BT_NUM_ARRAYS]);
size_t nxt_block_tables_staging_size(int num_seqs, int total_pages);
int nxt_build_block_tables(
    const int *page_offsets, const int *page_ids, const int *seq_lens,
    const int *prefix_node, const int *prefix_pages,
    int num_seqs, int max_blocks_per_seq, int block_size,
    void *device_buffer, size_t device_bytes,
    void *host_staging, size_t staging_bytes,
    int *num_groups, int *max_group_size, int *max_prefix_pages,
    nxt_stream_t stream);

/* ═══════════════════════════════════════════════════════════════════════
 * Activation + gating kernels (reference include/operator_api.h:121-150,
 * operators/activation_kernels.cu). Row t of `input` is [gate (d) | up (d)]
 * for the gated ops and d wide for the element-wise ones; `out` rows are d.
 * dtype_size 2 = fp16, 4 = fp32, for input and out alike. The activation is
 * computed in fp32 (expf / erff / tanhf), rounded to the storage type, and
 * multiplied by the other half in the storage type, as in the reference.
 * The drop-in entry points return nothing (like the reference) and record
 * their status for nxt_activation_last_error.
 * ═══════════════════════════════════════════════════════════════════════ */

/** out = silu(gate) * up   (gate = first half of input) */
void nxt_silu_and_mul(void *out, const void *input, int num_tokens, int d, int dtype_size,
                      nxt_stream_t stream);
/** out = gate * silu(up)   (up = second half of input) */
void nxt_mul_and_silu(void *out, const void *input, int num_tokens, int d, int dtype_size,
                      nxt_stream_t stream);
/** out = gelu(gate) * up */
void nxt_gelu_and_mul(void *out, const void *input, int num_tokens, int d, int dtype_size,
                      nxt_stream_t stream);
/** out = gelu_tanh(gate) * up */
void nxt_gelu_tanh_and_mul(void *out, const void *input, int num_tokens, int d, int dtype_size,
                           nxt_stream_t stream);
/** out = GELU(input)  (element-wise) */
void nxt_gelu_elementwise(void *out, const void *input, int num_tokens, int d, int dtype_size,
                          nxt_stream_t stream);
/** out = SiLU(input)  (element-wise) */
void nxt_silu_elementwise(void *out, const void *input, int num_tokens, int d, int dtype_size,
                          nxt_stream_t stream);

#define NXT_ACT_SILU_AND_MUL      0
#define NXT_ACT_MUL_AND_SILU      1
#define NXT_ACT_GELU_AND_MUL      2
#define NXT_ACT_GELU_TANH_AND_MUL 3
#define NXT_ACT_GELU              4
#define NXT_ACT_SILU              5

/* extension — any of the six ops by code, returning NXT_PA_OK or a negative
 * code (EINVAL: unknown op, d <= 0, num_tokens < 0, dtype, NULL pointer). */
int nxt_activation_ex(int op, void *out, const void *input, int num_tokens, int d,
                      int dtype_size, nxt_stream_t stream);

/* extension — status of the calling thread's last drop-in activation call. */
int nxt_activation_last_error(void);

/* ── extension: shared-prefix (cascade) decode attention ────────────────
 * For batches whose sequences share radix-tree prefixes (config 4): prefix
 * group g lists its member sequences group_members[group_offsets[g] ..
 * group_offsets[g+1]); every member b has prefix_pages[b] = P_g and the same
 * first P_g block-table entries; sequences in no group have prefix_pages 0.
 * A sequence is in at most one group and its seq_len covers its prefix.
 * Results are those of nxt_paged_attention_ex on the same inputs; the shared
 * pages are read once per group and KV head and multiplied with all members'
 * queries as one tensor-core tile, the private pages as usual. Shapes the TMA
 * path does not take run the plain path. max_group_size / max_prefix_pages
 * bound the device arrays' contents (host values). For head sizes 64 and 128
 * the shared-prefix kernel (persistent, on a few SMs) and the private-page
 * kernel run at the same time on `stream` (programmatic dependent launch). */
int nxt_paged_attention_prefix_ex(
    void *out, const void *query,
    const void *key_cache, const void *value_cache,
    const int *block_tables, const int *seq_lens,
    const int *prefix_pages, const int *group_offsets, const int *group_members,
    int num_groups, int max_group_size, int max_prefix_pages,
    int num_seqs, int num_heads, int head_size,
    int num_kv_heads, float scale,
    int max_num_blocks_per_seq,
    int block_size, int dtype_size,
    int64_t kv_block_stride, int64_t kv_head_stride,
    int64_t num_blocks,
    void *workspace, size_t workspace_bytes,
    int *device_status,
    nxt_stream_t stream);

/* Workspace bytes that suffice for a nxt_paged_attention_prefix_ex call with
 * these sizes: an upper bound, sized for the shortest prefix chunks (a call
 * may take longer chunks, hence fewer partial slots, when its groups give the
 * prefix kernel items enough). */
size_t nxt_paged_attention_prefix_workspace_size(
    int num_seqs, int num_heads, int head_size, int num_kv_heads,
    int max_num_blocks_per_seq, int block_size, int max_prefix_pages);

/* ── extension: KV-head sharding with the output all-gather fused in ────
 * For P GPUs of one box, one process or thread per GPU. Rank r owns KV
 * heads [r*Hkv/P, (r+1)*Hkv/P) with their query heads (head_offset =
 * r*Hq/P), its own page pools and block tables. Every rank allocates one
 * gather buffer (nxt_pa_peer_alloc: 2 halves of [num_seqs][total_heads]
 * [head_size] elements, then world_size uint64 flags), shares its IPC handle
 * with the others (any host-side channel) and opens theirs (nxt_pa_peer_open).
 * nxt_paged_attention_sharded then writes this rank's output heads directly
 * into every rank's buffer over NVLink (no collective library) and ends with
 * a bounded cross-GPU barrier: when its stream
 * reaches the end of step s, half (s & 1) of this rank's buffer holds the
 * whole [num_seqs][total_heads][head_size] output of step s from all ranks.
 * Consume that half before enqueueing step s + 2 on the same stream. A peer
 * that does not arrive within the wait budget raises NXT_PA_DEV_TIMEOUT.
 *
 * Rows are stored with one 16-byte store per peer, or, when mc_out is set,
 * with one multimem store (NVLS) whose copies NVSwitch writes into every
 * rank's buffer: mc_out is the multicast address of the gather buffers (a
 * CUDA multicast object with every rank's buffer bound at the same offset,
 * e.g. from torch symmetric memory), 16-byte aligned; NULL for peer stores.
 * Only stores use it; nothing is ever loaded through it. */
#define NXT_PA_MAX_PEERS 8
#define NXT_PA_IPC_HANDLE_BYTES 64

typedef struct {
    int       world_size;                    /* P, 1..NXT_PA_MAX_PEERS        */
    int       rank;                          /* this GPU's rank               */
    int       total_heads;                   /* query heads over all ranks    */
    int       head_offset;                   /* first query head of this rank */
    void     *peer_out[NXT_PA_MAX_PEERS];    /* rank r's gather buffer (opened) */
    uint64_t *peer_flags[NXT_PA_MAX_PEERS];  /* rank r's flag array (opened)  */
    void     *mc_out;                        /* multicast address of the gather
                                                buffers, or NULL              */
} NxtPaShard;

/* Allocates `bytes` of zero-filled device memory on the current device and
 * writes its IPC handle (NXT_PA_IPC_HANDLE_BYTES) to `ipc_handle`. */
int nxt_pa_peer_alloc(size_t bytes, void **dev_ptr, void *ipc_handle);
/* Maps another process's buffer (from its IPC handle) on the current device. */
int nxt_pa_peer_open(const void *ipc_handle, void **dev_ptr);
/* Unmaps a buffer opened with nxt_pa_peer_open. */
int nxt_pa_peer_close(void *dev_ptr);
/* Frees a buffer from nxt_pa_peer_alloc (after every peer has closed it). */
int nxt_pa_peer_free(void *dev_ptr);

/* Sharded decode attention for step `step` (1, 2, 3, ...): the arguments of
 * nxt_paged_attention_ex for this rank's heads (num_heads, num_kv_heads are
 * this rank's counts), without `out` and the workspace. */
int nxt_paged_attention_sharded(
    const NxtPaShard *shard, uint64_t step,
    const void *query,
    const void *key_cache, const void *value_cache,
    const int *block_tables, const int *seq_lens,
    int num_seqs, int num_heads, int head_size,
    int num_kv_heads, float scale,
    int max_num_blocks_per_seq,
    int block_size, int dtype_size,
    int64_t kv_block_stride, int64_t kv_head_stride,
    int64_t num_blocks,
    int *device_status,
    nxt_stream_t stream);

/* The same over one-byte pools: this rank's K/V pools as for
 * nxt_paged_attention_fp8_ex (kv_format, k_scale, v_scale); query and the
 * gathered output are fp16, so the gather buffers are sized with 2-byte
 * elements. */
int nxt_paged_attention_fp8_sharded(
    const NxtPaShard *shard, uint64_t step,
    const void *query,
    const void *key_cache, const void *value_cache,
    const int *block_tables, const int *seq_lens,
    int num_seqs, int num_heads, int head_size,
    int num_kv_heads, float scale,
    int max_num_blocks_per_seq, int block_size,
    int kv_format, float k_scale, float v_scale,
    int64_t kv_block_stride, int64_t kv_head_stride,
    int64_t num_blocks,
    int *device_status,
    nxt_stream_t stream);

/* extension — instrumentation for timing the attention kernel alone. The next
 * call made by this host thread records `before` on its stream immediately
 * before the main attention kernel (before the shared-prefix kernel of a
 * cascade call) and `after` immediately after it (ahead of the split-context
 * reduce). Both are cudaEvent_t values cast to void*; the
 * request is consumed by that one call. NULL, NULL cancels a pending request. */
int nxt_paged_attention_profile_next(void *before, void *after);

/* extension — as nxt_paged_attention_profile_next, plus `after_merge`,
 * recorded after the split-context reduce (after the attention kernel when the
 * call launches no reduce) and ahead of the fused head gather's end-of-step
 * barrier of a sharded call. An event recorded after the call returns then
 * closes the barrier's share. Any of the three may be NULL. The events sit
 * between kernels that otherwise overlap by programmatic dependent launch, so
 * the three shares add up to a little more than an unprofiled call. */
int nxt_paged_attention_profile_next_ex(void *before, void *after_attention,
                                        void *after_merge);

/* extension — the calling thread's current CUDA device: its ordinal, SM count
 * and name (name_len bytes at most, NUL-terminated). Used by the backend
 * plugin's init. Returns NXT_PA_OK, or NXT_PA_ECUDA when no device is usable. */
int nxt_paged_attention_device_info(int *device_id, int *sm_count,
                                    char *name, int name_len);

#ifdef __cplusplus
}
#endif

#endif /* XPA_OPERATOR_API_H_ */
