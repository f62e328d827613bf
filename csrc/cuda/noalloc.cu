// Allocation-free C entry point of the split-KV decode attention: the partial
// outputs and log-sum-exps go to a static __device__ array instead of buffers
// the caller allocates.  Declared (with the caller rules) in kapsl_noalloc.h.
// The kernels are the same ones the tensor API launches (attention.cu).
#include <cstdio>
#include <cstring>
#include <exception>
#include <mutex>

#include "common.cuh"
#include "kapsl_noalloc.h"
#include "kernels.h"

namespace {

constexpr int kMaxDevices = 64;
constexpr unsigned kScratchFloats = KAPSL_NOALLOC_SCRATCH_BYTES / 4u;

// Partial rows: [rows][128] outputs, then [rows] log-sum-exps.  Needs no
// initial value (each split writes all of its rows before the combine reads).
__device__ __align__(256) float g_noalloc_scratch[kScratchFloats];
// Fallback error word for callers that pass err == NULL (zero at module load).
__device__ int g_noalloc_err;

struct DeviceSlots {
  float* scratch = nullptr;
  int* err = nullptr;
};
DeviceSlots g_slots[kMaxDevices];
std::mutex g_mu;
thread_local char g_last_error[256] = {0};

int fail(int code, const char* what) {
  std::snprintf(g_last_error, sizeof(g_last_error), "%s", what);
  return code;
}

int setup_current(DeviceSlots** out) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess || dev < 0 || dev >= kMaxDevices)
    return fail(KAPSL_NOALLOC_ERR_SETUP, "decode_attention_noalloc: no current CUDA device");
  std::lock_guard<std::mutex> lk(g_mu);
  DeviceSlots& s = g_slots[dev];
  if (s.scratch == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) {
      std::snprintf(g_last_error, sizeof(g_last_error),
                    "decode_attention_noalloc: cudaGetSymbolAddress(scratch) failed on device %d: %s", dev,
                    cudaGetErrorString(e));
      return KAPSL_NOALLOC_ERR_SETUP;
    }
    void* q = nullptr;
    e = cudaGetSymbolAddress(&q, g_noalloc_err);
    if (e != cudaSuccess) {
      std::snprintf(g_last_error, sizeof(g_last_error),
                    "decode_attention_noalloc: cudaGetSymbolAddress(err) failed on device %d: %s", dev,
                    cudaGetErrorString(e));
      return KAPSL_NOALLOC_ERR_SETUP;
    }
    s.scratch = static_cast<float*>(p);
    s.err = static_cast<int*>(q);
  }
  *out = &s;
  return KAPSL_NOALLOC_OK;
}

}  // namespace

extern "C" int kapsl_decode_attention_noalloc_setup(void) {
  DeviceSlots* s = nullptr;
  return setup_current(&s);
}

extern "C" const char* kapsl_noalloc_last_error(void) { return g_last_error; }

extern "C" int kapsl_noalloc_read_and_clear_error(int* out) {
  if (out == nullptr) return fail(KAPSL_NOALLOC_ERR_ARGS, "noalloc_read_and_clear_error: out is NULL");
  DeviceSlots* s = nullptr;
  int rc = setup_current(&s);
  if (rc != KAPSL_NOALLOC_OK) return rc;
  // Synchronous symbol copies on the legacy default stream; the caller has
  // synchronised the stream of the launches this read covers.
  int v = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, g_noalloc_err, sizeof(int));
  if (e == cudaSuccess) {
    const int zero = 0;
    e = cudaMemcpyToSymbol(g_noalloc_err, &zero, sizeof(int));
  }
  if (e != cudaSuccess) {
    std::snprintf(g_last_error, sizeof(g_last_error), "noalloc_read_and_clear_error: %s", cudaGetErrorString(e));
    return KAPSL_NOALLOC_ERR_LAUNCH;
  }
  *out = v;
  return KAPSL_NOALLOC_OK;
}

extern "C" int kapsl_decode_attention_noalloc(const void* q, int64_t q_stride, const void* k_cache,
                                              const void* v_cache, int64_t num_blocks, const int32_t* block_tables,
                                              int max_blocks, const int32_t* ctx_lens, void* out,
                                              int64_t out_stride, int B, int Hq, int Hkv, int nsplit, float scale,
                                              int* err, cudaStream_t stream) {
  g_last_error[0] = 0;
  if (B < 0 || Hq <= 0 || Hkv <= 0 || nsplit < 1 || nsplit > 64 || num_blocks <= 0 || max_blocks <= 0)
    return fail(KAPSL_NOALLOC_ERR_ARGS, "decode_attention_noalloc: bad sizes (need B>=0, Hq,Hkv>0, 1<=nsplit<=64)");
  if (Hq % Hkv != 0 || Hq / Hkv > 16)
    return fail(KAPSL_NOALLOC_ERR_ARGS, "decode_attention_noalloc: Hq must be a multiple of Hkv, group <= 16");
  if (!q || !k_cache || !v_cache || !block_tables || !ctx_lens || !out)
    return fail(KAPSL_NOALLOC_ERR_ARGS, "decode_attention_noalloc: null pointer argument");
  if ((reinterpret_cast<uintptr_t>(q) & 3) || (reinterpret_cast<uintptr_t>(out) & 3) || (q_stride & 1) ||
      (out_stride & 1) || q_stride < (int64_t)Hq * 128 || out_stride < (int64_t)Hq * 128)
    return fail(KAPSL_NOALLOC_ERR_ARGS,
                "decode_attention_noalloc: q/out must be 4-byte aligned with even row strides >= Hq*128");
  if ((reinterpret_cast<uintptr_t>(k_cache) & 15) || (reinterpret_cast<uintptr_t>(v_cache) & 15))
    return fail(KAPSL_NOALLOC_ERR_ARGS, "decode_attention_noalloc: KV caches must be 16-byte aligned");
  const uint64_t rows = (uint64_t)B * (uint64_t)Hq * (uint64_t)nsplit;
  if (nsplit > 1 && rows > KAPSL_NOALLOC_MAX_PARTIAL_ROWS) {
    std::snprintf(g_last_error, sizeof(g_last_error),
                  "decode_attention_noalloc: B*Hq*nsplit = %llu partial rows exceed the static scratch limit of %u "
                  "(%u bytes); lower nsplit or the batch",
                  (unsigned long long)rows, (unsigned)KAPSL_NOALLOC_MAX_PARTIAL_ROWS,
                  (unsigned)KAPSL_NOALLOC_SCRATCH_BYTES);
    return KAPSL_NOALLOC_ERR_TOO_LARGE;
  }
  DeviceSlots* s = nullptr;
  int rc = setup_current(&s);
  if (rc != KAPSL_NOALLOC_OK) return rc;
  if (B == 0) return KAPSL_NOALLOC_OK;
  float* part_o = s->scratch;
  float* part_lse = s->scratch + rows * 128;
  try {
    const uint64_t cache_rows = (uint64_t)num_blocks * (uint64_t)Hkv * 16u;
    CUtensorMap tk = kapsl::make_tmap_2d_bf16(k_cache, cache_rows, 128, 128, 16, 64, true);
    CUtensorMap tv = kapsl::make_tmap_2d_bf16(v_cache, cache_rows, 128, 128, 16, 64, true);
    kapsl::launch_decode_attention(tk, tv, static_cast<const __nv_bfloat16*>(q), q_stride, block_tables, max_blocks,
                                   ctx_lens, static_cast<__nv_bfloat16*>(out), out_stride, part_o, part_lse, B, Hq,
                                   Hkv, nsplit, scale, err ? err : s->err, stream);
  } catch (const std::exception& ex) {
    return fail(KAPSL_NOALLOC_ERR_LAUNCH, ex.what());
  }
  return KAPSL_NOALLOC_OK;
}
