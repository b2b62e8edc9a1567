/* Allocation-free entry point of the split-KV paged decode attention kernel.
 *
 * This declaration has no counterpart in the reference (thebloodlust/VRAMancer):
 * it exists for callers of this library that cannot allocate GPU memory themselves
 * — code that runs inside a host framework owning every device allocation (a
 * custom allocator or memory-pool arena that forbids stray cudaMalloc), code that
 * must not perturb a memory budget measured up front, or plain C callers that load
 * the shared library without any tensor framework.  Such callers still pass their
 * own inputs and outputs; the split-KV partial results the kernel needs in between
 * live in a fixed, statically sized device array compiled into the library.
 *
 * Limits and behaviour:
 *   - scratch is VRM_NOALLOC_SCRATCH_BYTES (8 MiB) plus VRM_NOALLOC_MAX_GROUPS
 *     counters; every GPU that loads the library holds them until the process exits;
 *   - a request whose split partials need more scratch than that is rejected with a
 *     non-zero return code and a message from vrm_noalloc_last_error(); with
 *     num_splits <= 0 the split count is chosen automatically and lowered until it
 *     fits (one split needs no scratch at all); an explicit num_splits above 128 is
 *     rejected the same way;
 *   - the first call on a device (vrm_noalloc_setup(), or else the first decode
 *     call) resolves the scratch address on that device (with it current); make that
 *     first call before any stream capture;
 *   - errors that the kernel's bounded waits and bounds checks detect go to a static
 *     error word of this entry point, read with vrm_noalloc_read_and_clear_errors();
 *   - all calls share the one scratch array and it keeps the last call's contents:
 *     calls that overlap on the GPU (different streams, or threads without ordering)
 *     race with each other and must be serialised by the caller;
 *   - the function performs no cudaMalloc / cudaFree and calls no allocating
 *     library routine.
 */
#ifndef VRM_NOALLOC_H_
#define VRM_NOALLOC_H_

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#define VRM_NOALLOC_SCRATCH_BYTES (8u << 20)
#define VRM_NOALLOC_MAX_GROUPS 8192

#ifdef __cplusplus
extern "C" {
#endif

/* One decode token per sequence over the paged KV pool
 * cache[pages, num_layers, 2, num_kv_heads, 16, head_dim] (bf16, or fp8 e4m3 with
 * kv_scale[num_layers, 2, num_kv_heads] fp32).  q / out: bf16 rows of `batch`
 * sequences, head h of row b at base + b*ld + h*head_dim.  Returns 0 on success. */
int vrm_paged_attention_decode_noalloc(const void* q, int64_t ld_q, const void* kv_cache, int cache_is_fp8,
                                       int num_layers, int layer, int num_kv_heads, int head_dim,
                                       int num_q_heads, const int* block_tables, int block_table_stride,
                                       const int* context_lens, const float* kv_scale, float sm_scale,
                                       void* out, int64_t ld_out, int batch, int max_pages, int num_splits,
                                       cudaStream_t stream);

/* Resolves the scratch of the current device ahead of the first decode call (for
 * example before a stream capture).  Returns 0 on success. */
int vrm_noalloc_setup(void);

/* Synchronises the current device, stores the error bits the allocation-free calls
 * reported since the last read into *flags (0 = none) and clears them.  Returns 0
 * on success. */
int vrm_noalloc_read_and_clear_errors(uint32_t* flags);

/* Device allocations the library's host services have made so far in this process
 * (a check for callers and tests that the calls above add none). */
uint64_t vrm_host_device_allocations(void);

/* Message of the last failed call on this thread ("" if none). */
const char* vrm_noalloc_last_error(void);

/* Scratch capacity in bytes. */
size_t vrm_noalloc_scratch_capacity(void);

#ifdef __cplusplus
}
#endif

#endif /* VRM_NOALLOC_H_ */
