// Allocation-free C entry point of the paged split-KV decode attention.
//
// There is no counterpart of this entry point in kapsl-runtime; it exists for
// embedders that must not allocate device memory on the call path:
//   * hosts whose device-memory budget is fixed up front (a serving process that
//     has reserved the HBM for weights + KV pages and may not grow afterwards),
//   * real-time loops where a cudaMalloc/cudaFree (which can synchronise the
//     device) or a caching allocator's growth would stall the step,
//   * callers without PyTorch (plain C/C++ runtimes linking the extension's
//     shared object) that have no allocator to hand scratch buffers from.
// The split-KV partial results live in a fixed static __device__ array
// (KAPSL_NOALLOC_SCRATCH_BYTES per device) instead of caller-provided buffers.
//
// Rules for callers:
//   * Call kapsl_decode_attention_noalloc_setup() once per device, with that
//     device current, before the first launch.  If it is not called, the first
//     launch on a device performs the set-up itself; that first call should then
//     happen before any stream capture begins.
//   * B * Hq * nsplit must be <= KAPSL_NOALLOC_MAX_PARTIAL_ROWS when nsplit > 1;
//     larger requests are rejected with KAPSL_NOALLOC_ERR_TOO_LARGE and launch
//     nothing.
//   * The scratch array is shared by every call on a device: two calls whose
//     executions overlap (different streams, or different host threads without
//     ordering) race on it and produce wrong results.  Serialise them.
//   * Nothing in the scratch has to start at zero: every split writes its own
//     partial rows before the combine pass reads them.  The `err` word, when
//     given, must start at zero; the kernel sets it to 1 if a KV page load does
//     not arrive within its bounded wait.  With err == NULL a static per-device
//     word (zero when the module loads) is used instead; read it, and reset it
//     to zero, with kapsl_noalloc_read_and_clear_error() on the current device.
//
// Layouts match the tensor API: q [B, >= Hq*128] bf16 (row stride q_stride
// elements), k/v cache [num_blocks, Hkv, 16, 128] bf16 contiguous,
// block_tables [B, max_blocks] int32, ctx_lens [B] int32,
// out [B, >= Hq*128] bf16 (row stride out_stride elements).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#define KAPSL_NOALLOC_SCRATCH_BYTES (16u << 20)
// one partial row = 128 fp32 outputs + 1 fp32 log-sum-exp
#define KAPSL_NOALLOC_MAX_PARTIAL_ROWS (KAPSL_NOALLOC_SCRATCH_BYTES / (129u * 4u))

#define KAPSL_NOALLOC_OK 0
#define KAPSL_NOALLOC_ERR_TOO_LARGE 1   // B * Hq * nsplit exceeds the static scratch
#define KAPSL_NOALLOC_ERR_ARGS 2        // bad shape / alignment / GQA group
#define KAPSL_NOALLOC_ERR_SETUP 3       // cudaGetSymbolAddress failed
#define KAPSL_NOALLOC_ERR_LAUNCH 4      // CUDA reported an error at launch

#ifdef __cplusplus
extern "C" {
#endif

// Resolves the static scratch address for the current device.  Returns
// KAPSL_NOALLOC_OK or KAPSL_NOALLOC_ERR_SETUP.
int kapsl_decode_attention_noalloc_setup(void);

// Launches decode attention (and, for nsplit > 1, the split combine) on
// `stream`.  Returns a KAPSL_NOALLOC_* code; on error nothing was launched
// unless the code is KAPSL_NOALLOC_ERR_LAUNCH.
int kapsl_decode_attention_noalloc(const void* q, int64_t q_stride, const void* k_cache, const void* v_cache,
                                   int64_t num_blocks, const int32_t* block_tables, int max_blocks,
                                   const int32_t* ctx_lens, void* out, int64_t out_stride, int B, int Hq, int Hkv,
                                   int nsplit, float scale, int* err, cudaStream_t stream);

// Human-readable text of the last error on the calling thread ("" if none).
const char* kapsl_noalloc_last_error(void);

// Stores the current device's fallback error word (the one launches with
// err == NULL write) into *out and resets it to zero.  The copies are
// synchronous and use no device allocation; synchronise the stream of the
// launches it should cover first (a non-blocking stream is not ordered with
// these copies).  Returns a KAPSL_NOALLOC_* code.
int kapsl_noalloc_read_and_clear_error(int* out);

#ifdef __cplusplus
}
#endif
