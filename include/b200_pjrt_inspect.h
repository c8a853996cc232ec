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
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Compile `mlir` (StableHLO text) without a device.  what: 0 = optimized graph
 * (after call inlining, SDPA/LayerNorm matching), 1 = execution plan (slots and
 * steps), 2 = generated CUDA C, 3 = also NVRTC-compile the CUDA C for sm_100a
 * and return "ok <cubin bytes>", 4 = the key each compile unit's cubin is filed
 * under (one per line; a serialized executable carries its cubins by these).  Returns 0 and a malloc'd string in *out, or
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

/* How many of its generated kernels (the CUDA C of fused loops, rows,
 * reductions, gathers and scatters) the plugin has launched in this process.
 * The hand-written kernels an Execute calls are counted by libb200_kernels.so's
 * b200_kernel_launches(); the two together are every kernel an Execute starts.
 * The reference has no counterpart. */
__attribute__((visibility("default"))) uint64_t b200_pjrt_kernel_launches(void);

/* With B200_TIMING=1 in the environment, every Execute records CUDA events on
 * the first device's stream around its launch sequence (after host-side
 * preparation).  This returns how many executions were recorded since the last
 * call and writes up to `max` of their device times in milliseconds to `ms`
 * (waiting for them to finish), then forgets them.  The reference's
 * counterpart is its MLX_TIMING print of ExecuteGraph time
 * (src/jax_mlx_pjrt.cpp:246-250, :9340-9351). */
__attribute__((visibility("default"))) int b200_pjrt_execute_times(void* loaded_executable,
                                                                  double* ms, int max);

/* The key-value exchange that Execute performs for the NCCL unique id of a
 * multi-process run (one process per GPU), without a device: rank 0 puts
 * `value` under `key` through put_callback, any other rank gets `key` through
 * get_callback, with the PJRT_KeyValue*Callback_Args the plugin builds for
 * PJRT_Client_Create's kv_get_callback / kv_put_callback (callback_error set,
 * timeout from B200_KV_TIMEOUT_MS, default 120000).  Lets a deployment check
 * its KV-store wiring and its error path before the first collective.  Returns
 * 0 with the value written or read in *out (*out_len bytes, NUL-terminated;
 * may hold zero bytes), or the PJRT error code with the message in *out: a
 * callback's error object (made through callback_error) keeps its code.  Free
 * *out with b200_pjrt_free().  The reference (single device) has no
 * counterpart; jaxlib's distributed client supplies the callbacks. */
__attribute__((visibility("default"))) int b200_pjrt_kv_exchange(
    void* get_callback, void* get_user_arg, void* put_callback, void* put_user_arg, int rank,
    const char* key, size_t key_len, const char* value, size_t value_len, char** out,
    size_t* out_len);

#ifdef __cplusplus
}
#endif
#endif /* B200_PJRT_INSPECT_H_ */
