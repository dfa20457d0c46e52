/*
 * Stand-in for the build configuration header the xLLMs CMake build
 * generates from cmake/xllm_config.h.in. It carries the two settings
 * src/core/backend_manager.c reads: the build-time plugin directory (step 3
 * of its search order; pointed nowhere here, so the tests exercise the
 * XLLM_CUDA_BACKEND_PATH / XLLM_BACKEND_DIR steps) and the plugin's file
 * name, which this repository's plugin keeps.
 */
#ifndef XLLM_CONFIG_H
#define XLLM_CONFIG_H
#define XLLM_BACKEND_INSTALL_DIR "/nonexistent/xllm-backends"
#define XLLM_CUDA_BACKEND_SO "libxllm_cuda_backend.so"
#endif
