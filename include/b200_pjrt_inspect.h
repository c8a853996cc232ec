/*
 * b200_pjrt_inspect.h — diagnostics exported by libb200_pjrt.so beside
 * GetPjrtApi().  No GPU is needed: these run the compile pipeline (parse,
 * pattern match, fusion plan, CUDA C generation) and return text.
 *
 * The reference has no counterpart entry point; its equivalent is the
 * MLX_PJRT_DEBUG / MLX_DUMP_MLIR logging of src/jax_mlx_pjrt.cpp:232-236 and
 * :887-892, which prints the parsed graph and pattern matches at compile time.
 */
#ifndef B200_PJRT_INSPECT_H_
#define B200_PJRT_INSPECT_H_
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Compile `mlir` (StableHLO text) without a device.  what: 0 = optimized graph
 * (after call inlining, SDPA/LayerNorm matching), 1 = execution plan (slots and
 * steps), 2 = generated CUDA C, 3 = also NVRTC-compile the CUDA C for sm_100a
 * and return "ok <cubin bytes>".  Returns 0 and a malloc'd string in *out, or
 * the PJRT error code and the message in *out.  Free *out with
 * b200_pjrt_free(). */
__attribute__((visibility("default"))) int b200_pjrt_inspect(const char* mlir, size_t len,
                                                             int what, char** out);
__attribute__((visibility("default"))) void b200_pjrt_free(char* p);

/* The cudaStream_t on which the plugin runs every transfer and launch for
 * `device` (a PJRT_Device* of this plugin), or NULL if the device is not
 * addressable.  For profiling and event timing only: work enqueued on it by the
 * caller is ordered with the plugin's work. */
__attribute__((visibility("default"))) void* b200_pjrt_device_stream(void* device);

/* With B200_TIMING=1 in the environment, every Execute records CUDA events on
 * the first device's stream around its launch sequence (after host-side
 * preparation).  This returns how many executions were recorded since the last
 * call and writes up to `max` of their device times in milliseconds to `ms`
 * (waiting for them to finish), then forgets them.  The reference's
 * counterpart is its MLX_TIMING print of ExecuteGraph time
 * (src/jax_mlx_pjrt.cpp:246-250, :9340-9351). */
__attribute__((visibility("default"))) int b200_pjrt_execute_times(void* loaded_executable,
                                                                  double* ms, int max);

#ifdef __cplusplus
}
#endif
#endif /* B200_PJRT_INSPECT_H_ */
