/*
 * cuda_backend.h — the dlopen'd CUDA backend plugin, libxllm_cuda_backend.so.
 *
 * Drop-in for the xLLMs plugin (backends/cuda_backend.h and
 * backends/cuda_backend.c of the xLLMs project). The xLLMs backend manager
 * dlopen()s the library and looks up the three entry points below by name
 * (src/core/backend_manager.c:283-285), so names, signatures, return codes and
 * the input descriptor's layout are kept as they are there. The run entry
 * point forwards to the B200 kernels of libxpa.so (operator_api.h).
 */
#ifndef XPA_CUDA_BACKEND_H_
#define XPA_CUDA_BACKEND_H_

#include "operator_api.h"

#ifdef __cplusplus
extern "C" {
#endif

/* Opaque here; its layout is in xllm_backend_abi.h. */
typedef struct NxtBackend NxtBackend;

/* Paged-attention input descriptor, field for field the reference's
 * NxtPagedAttentionInput (backends/cuda_backend.h:29-46). Pointers are device
 * pointers; `stream` is a cudaStream_t cast to void*. The output tensor
 * [num_seqs][num_heads][head_size] is passed separately as `output`. */
typedef struct {
    const void   *query;
    const void   *key_cache;
    const void   *value_cache;
    const int    *block_tables;
    const int    *seq_lens;
    int           num_seqs;
    int           num_heads;
    int           head_size;
    int           num_kv_heads;
    float         scale;
    int           max_num_blocks_per_seq;
    int           block_size;
    int           dtype_size;
    int           kv_block_stride;
    int           kv_head_stride;
    nxt_stream_t  stream;
} NxtPagedAttentionInput;

/* Replaces nxt_backend_init (reference backends/cuda_backend.c:35-67):
 * -1 on NULL or when no CUDA device is current; otherwise allocates the
 * plugin state, sets backend->state = NXT_BACKEND_STATE_READY, returns 0. */
int nxt_backend_init(NxtBackend *backend);

/* Replaces nxt_backend_run (reference backends/cuda_backend.c:71-104):
 * -1 on a NULL backend, backend state, input or output; otherwise enqueues
 * paged decode attention for the NxtPagedAttentionInput at `input` into the
 * device tensor `output`. Returns 0 when the kernels were enqueued and -1
 * when the operator rejected the arguments or a launch failed (the reference
 * returns 0 after its launch in every case). */
int nxt_backend_run(NxtBackend *backend, void *input, void *output);

/* Replaces nxt_backend_fini (reference backends/cuda_backend.c:108-120):
 * -1 on NULL; frees the plugin state and the workspaces and status words
 * libxpa.so allocated on first use (nxt_paged_attention_release_workspaces,
 * which synchronises each device that holds one), sets state UNINITIALIZED,
 * returns 0 (-1 if a CUDA call of that release failed). A later call of any
 * entry point allocates them again. The reference process holds one CUDA
 * backend, so its fini is the end of the library's use. */
int nxt_backend_fini(NxtBackend *backend);

#ifdef __cplusplus
}
#endif

#endif /* XPA_CUDA_BACKEND_H_ */
