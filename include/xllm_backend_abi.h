/*
 * xllm_backend_abi.h — the NxtBackend handle the xLLMs backend manager passes
 * to a plugin.
 *
 * The manager owns this struct and the plugin writes `state` and
 * `backend_state` in place, so the layout must match the reference's
 * include/backend.h:128-151 (NxtBackendAPI: eight function pointers;
 * NxtBackend: name, so_path, dl_handle, api, state, priority, model_count,
 * models, backend_state). On x86-64: state at byte 88, backend_state at 112,
 * the offsets the reference's tests/mock_cuda_backend.c:22-37 pins.
 * This header declares no functions.
 */
#ifndef XPA_XLLM_BACKEND_ABI_H_
#define XPA_XLLM_BACKEND_ABI_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
    NXT_BACKEND_STATE_UNINITIALIZED = 0,
    NXT_BACKEND_STATE_INITIALIZING  = 1,
    NXT_BACKEND_STATE_READY         = 2,
    NXT_BACKEND_STATE_ERROR         = 3,
    NXT_BACKEND_STATE_UNLOADING     = 4,
} NxtBackendState;

struct NxtBackend;

/* Eight entry points the manager resolves with dlsym; only the first three
 * are exported by this plugin. */
typedef struct {
    int (*backend_init)(struct NxtBackend *);
    int (*backend_run)(struct NxtBackend *, void *, void *);
    int (*backend_fini)(struct NxtBackend *);
    void *model_init;
    void *model_fini;
    void *instance_init;
    void *instance_fini;
    void *instance_exec;
} NxtBackendAPIABI;

struct NxtBackend {
    char            *name;
    char            *so_path;
    void            *dl_handle;
    NxtBackendAPIABI api;
    NxtBackendState  state;
    int32_t          priority;
    uint32_t         model_count;
    void            *models;
    void            *backend_state;
};

#ifdef __cplusplus
}
#endif

#endif /* XPA_XLLM_BACKEND_ABI_H_ */
