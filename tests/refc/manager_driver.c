/*
 * manager_driver.c — drives this repository's backend plugin through the
 * xLLMs backend manager itself (src/core/backend_manager.c, compiled in
 * place from the reference sources by tests/refc/Makefile), with the
 * reference's own headers (include/backend.h, backends/cuda_backend.h).
 *
 *   manager_driver discover
 *       nxt_backend_manager_init -> nxt_backend_discover (search order of
 *       backend_manager.c:131-180: XLLM_CUDA_BACKEND_PATH, XLLM_BACKEND_DIR,
 *       ...) -> nxt_backend_load (dlopen + dlsym of the three entry points +
 *       backend_init, :264-317) -> the manager's NULL / unknown-name
 *       contracts of nxt_backend_run (:339-344) -> nxt_backend_unload ->
 *       nxt_backend_manager_fini. Prints "loaded=<n> ready=<0|1>".
 *
 *   manager_driver run <problem.bin> <out.bin>
 *       the same load, then one paged decode attention call the way a
 *       manager caller makes it: device buffers from cudaMalloc, an
 *       NxtPagedAttentionInput descriptor, nxt_backend_run("cuda", &in, out).
 *       problem.bin: 10 int32 (num_seqs, num_heads, head_size, num_kv_heads,
 *       max_blocks, block_size, dtype_size, kv_block_stride, kv_head_stride,
 *       num_blocks), one float32 scale, then query, key pool, value pool
 *       (dtype_size-byte elements), block tables and seq_lens (int32).
 *       out.bin receives [num_seqs][num_heads][head_size] elements.
 */
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <cuda_runtime_api.h>

#include "backend.h"

/* The plugin's descriptor type. backends/cuda_backend.h also declares the
 * plugin-side nxt_backend_run, whose name the manager's public function
 * takes; the reference's plugin source resolves the clash the same way. */
#define nxt_backend_run nxt_plugin_backend_run
#define nxt_backend_init nxt_plugin_backend_init
#define nxt_backend_fini nxt_plugin_backend_fini
#include "cuda_backend.h"
#undef nxt_backend_run
#undef nxt_backend_init
#undef nxt_backend_fini

static int load_cuda_backend(void) {
    if (nxt_backend_manager_init(NULL) != 0) return -1;
    return nxt_backend_discover();
}

static int cmd_discover(void) {
    const int loaded = load_cuda_backend();
    NxtBackend *b = nxt_backend_find("cuda");
    const int ready = b && b->state == NXT_BACKEND_STATE_READY;
    int dummy = 0;
    /* the manager's own contracts: unknown backend name, NULL name */
    if (nxt_backend_run("no-such-backend", &dummy, &dummy) != -1) return 10;
    if (loaded > 0) {
        /* the plugin's NULL contract, reached through the manager */
        if (nxt_backend_run("cuda", NULL, &dummy) != -1) return 11;
        if (nxt_backend_run("cuda", &dummy, NULL) != -1) return 12;
        if (nxt_backend_unload("cuda") != 0) return 13;
        if (nxt_backend_find("cuda") != NULL) return 14;
    }
    printf("loaded=%d ready=%d\n", loaded, ready);
    nxt_backend_manager_fini();
    return 0;
}

static void *read_all(const char *path, size_t *len) {
    FILE *f = fopen(path, "rb");
    if (!f) return NULL;
    fseek(f, 0, SEEK_END);
    const long n = ftell(f);
    fseek(f, 0, SEEK_SET);
    void *buf = n > 0 ? malloc((size_t)n) : NULL;
    if (buf && fread(buf, 1, (size_t)n, f) != (size_t)n) {
        free(buf);
        buf = NULL;
    }
    fclose(f);
    *len = buf ? (size_t)n : 0;
    return buf;
}

static void *to_device(const unsigned char *src, size_t bytes) {
    void *d = NULL;
    if (cudaMalloc(&d, bytes ? bytes : 1) != cudaSuccess) return NULL;
    if (bytes && cudaMemcpy(d, src, bytes, cudaMemcpyHostToDevice) != cudaSuccess) {
        cudaFree(d);
        return NULL;
    }
    return d;
}

static int cmd_run(const char *in_path, const char *out_path) {
    size_t len = 0;
    unsigned char *buf = read_all(in_path, &len);
    if (!buf || len < 11 * 4) return 20;
    int hdr[10];
    float scale;
    memcpy(hdr, buf, sizeof(hdr));
    memcpy(&scale, buf + 40, 4);
    const int B = hdr[0], Hq = hdr[1], D = hdr[2], Hkv = hdr[3], mb = hdr[4], bs = hdr[5];
    const int ds = hdr[6], kbs = hdr[7], khs = hdr[8], nb = hdr[9];
    const size_t q_bytes = (size_t)B * Hq * D * ds;
    const size_t pool_bytes = (size_t)nb * kbs * ds;
    const size_t bt_bytes = (size_t)B * mb * 4, sl_bytes = (size_t)B * 4;
    if (len != 44 + q_bytes + 2 * pool_bytes + bt_bytes + sl_bytes) return 21;
    const unsigned char *p = buf + 44;
    void *d_q = to_device(p, q_bytes);
    p += q_bytes;
    void *d_k = to_device(p, pool_bytes);
    p += pool_bytes;
    void *d_v = to_device(p, pool_bytes);
    p += pool_bytes;
    void *d_bt = to_device(p, bt_bytes);
    p += bt_bytes;
    void *d_sl = to_device(p, sl_bytes);
    void *d_out = NULL;
    if (!d_q || !d_k || !d_v || !d_bt || !d_sl || cudaMalloc(&d_out, q_bytes) != cudaSuccess)
        return 22;
    cudaMemset(d_out, 0, q_bytes);

    if (load_cuda_backend() != 1) return 23;
    NxtPagedAttentionInput in;
    memset(&in, 0, sizeof(in));
    in.query = d_q;
    in.key_cache = d_k;
    in.value_cache = d_v;
    in.block_tables = (const int *)d_bt;
    in.seq_lens = (const int *)d_sl;
    in.num_seqs = B;
    in.num_heads = Hq;
    in.head_size = D;
    in.num_kv_heads = Hkv;
    in.scale = scale;
    in.max_num_blocks_per_seq = mb;
    in.block_size = bs;
    in.dtype_size = ds;
    in.kv_block_stride = kbs;
    in.kv_head_stride = khs;
    in.stream = NULL;
    const int rc = nxt_backend_run("cuda", &in, d_out);
    if (rc != 0) return 24;
    if (cudaDeviceSynchronize() != cudaSuccess) return 25;
    unsigned char *out = malloc(q_bytes ? q_bytes : 1);
    if (!out || cudaMemcpy(out, d_out, q_bytes, cudaMemcpyDeviceToHost) != cudaSuccess) return 26;
    FILE *f = fopen(out_path, "wb");
    if (!f || fwrite(out, 1, q_bytes, f) != q_bytes) return 27;
    fclose(f);
    nxt_backend_unload("cuda");
    nxt_backend_manager_fini();
    cudaFree(d_q);
    cudaFree(d_k);
    cudaFree(d_v);
    cudaFree(d_bt);
    cudaFree(d_sl);
    cudaFree(d_out);
    free(out);
    free(buf);
    printf("ok\n");
    return 0;
}

int main(int argc, char **argv) {
    if (argc >= 2 && strcmp(argv[1], "discover") == 0) return cmd_discover();
    if (argc >= 4 && strcmp(argv[1], "run") == 0) return cmd_run(argv[2], argv[3]);
    fprintf(stderr, "usage: manager_driver discover | run <problem.bin> <out.bin>\n");
    return 2;
}
