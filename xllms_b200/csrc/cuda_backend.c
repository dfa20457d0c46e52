/*
 * cuda_backend.c — libxllm_cuda_backend.so, the dlopen'd backend plugin.
 *
 * Exports the three entry points the xLLMs backend manager resolves by name
 * (src/core/backend_manager.c:283-285) with the reference plugin's contract
 * (backends/cuda_backend.c:35-120); the run entry point forwards the
 * NxtPagedAttentionInput descriptor to libxpa.so's paged decode attention.
 * Plain C11; all CUDA work happens inside libxpa.so.
 */
#include <stdio.h>
#include <stdlib.h>

#include "cuda_backend.h"
#include "xllm_backend_abi.h"

typedef struct {
    int  device_id;
    int  sm_count;
    char model_name[256];
} CudaBackendState;

int nxt_backend_init(NxtBackend *backend) {
    if (!backend) return -1;
    CudaBackendState *state = (CudaBackendState *)calloc(1, sizeof(CudaBackendState));
    if (!state) return -1;
    if (nxt_paged_attention_device_info(&state->device_id, &state->sm_count,
                                        state->model_name,
                                        (int)sizeof(state->model_name)) != NXT_PA_OK) {
        fprintf(stderr, "[xpa cuda_backend] no usable CUDA device\n");
        free(state);
        return -1;
    }
    backend->backend_state = state;
    backend->state = NXT_BACKEND_STATE_READY;
    return 0;
}

int nxt_backend_run(NxtBackend *backend, void *input, void *output) {
    if (!backend || !backend->backend_state) return -1;
    if (!input || !output) return -1;
    const NxtPagedAttentionInput *pa = (const NxtPagedAttentionInput *)input;
    nxt_paged_attention(output, pa->query, pa->key_cache, pa->value_cache,
                        pa->block_tables, pa->seq_lens, pa->num_seqs,
                        pa->num_heads, pa->head_size, pa->num_kv_heads,
                        pa->scale, pa->max_num_blocks_per_seq, pa->block_size,
                        pa->dtype_size, pa->kv_block_stride,
                        pa->kv_head_stride, pa->stream);
    return nxt_paged_attention_last_error() == NXT_PA_OK ? 0 : -1;
}

int nxt_backend_fini(NxtBackend *backend) {
    if (!backend) return -1;
    free(backend->backend_state);
    backend->backend_state = NULL;
    backend->state = NXT_BACKEND_STATE_UNINITIALIZED;
    /* the split-context workspaces and status words the attention calls
     * allocated lazily go with the backend */
    return nxt_paged_attention_release_workspaces() == NXT_PA_OK ? 0 : -1;
}
