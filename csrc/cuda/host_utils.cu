// Host-side helpers shared by all kernels: launch accounting and TMA
// descriptor encoding.
#include <atomic>
#include <cstdlib>
#include <mutex>
#include <string>

#include "common.cuh"

namespace kapsl {

static std::atomic<uint64_t> g_launches{0};

uint64_t launch_count() { return g_launches.load(std::memory_order_relaxed); }
void note_launch(uint64_t n) { g_launches.fetch_add(n, std::memory_order_relaxed); }

bool pdl_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("KAPSL_PDL");
    return v == nullptr || std::string(v) != "0";
  }();
  return on;
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn get_encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q);
    if (e == cudaSuccess && q == cudaDriverEntryPointSuccess) fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  if (!fn) throw std::runtime_error("cuTensorMapEncodeTiled is unavailable from the CUDA driver");
  return fn;
}

CUtensorMap make_tmap_2d_bf16(const void* base, uint64_t rows, uint64_t cols, uint64_t pitch_elems,
                              uint32_t box_rows, uint32_t box_cols, bool swizzle128) {
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0)
    throw std::runtime_error("TMA base address must be 16-byte aligned");
  if ((pitch_elems * 2) % 16 != 0) throw std::runtime_error("TMA row pitch must be a multiple of 16 bytes");
  if ((box_cols * 2) % 16 != 0) throw std::runtime_error("TMA box inner extent must be a multiple of 16 bytes");
  if (swizzle128 && box_cols * 2 > 128) throw std::runtime_error("128B swizzle needs a box of <=128 bytes inner");
  CUtensorMap m;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {pitch_elems * 2};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = get_encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims,
                               strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                               swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) throw std::runtime_error("cuTensorMapEncodeTiled failed: " + std::to_string((int)r));
  return m;
}

// 3-D bf16 tensor map: dims innermost first, strides of dims 1 and 2 in bytes.
CUtensorMap make_tmap_3d_bf16(const void* base, const uint64_t (&dims)[3], const uint64_t (&strides_bytes)[2],
                              const uint32_t (&box)[3], bool swizzle128) {
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0) throw std::runtime_error("TMA base address must be 16-byte aligned");
  if (strides_bytes[0] % 16 != 0 || strides_bytes[1] % 16 != 0)
    throw std::runtime_error("TMA strides must be multiples of 16 bytes");
  if ((box[0] * 2) % 16 != 0 || (swizzle128 && box[0] * 2 > 128) || box[1] > 256 || box[2] > 256)
    throw std::runtime_error("TMA 3-D box out of range");
  CUtensorMap m;
  cuuint64_t d[3] = {dims[0], dims[1], dims[2]};
  cuuint64_t st[2] = {strides_bytes[0], strides_bytes[1]};
  cuuint32_t b[3] = {box[0], box[1], box[2]};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = get_encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), d, st, b, estr,
                               CU_TENSOR_MAP_INTERLEAVE_NONE,
                               swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) throw std::runtime_error("cuTensorMapEncodeTiled (3-D) failed: " + std::to_string((int)r));
  return m;
}

// 2-D byte tensor map without swizzle (packed quantized blocks).
CUtensorMap make_tmap_2d_u8(const void* base, uint64_t rows, uint64_t cols_bytes, uint64_t pitch_bytes,
                            uint32_t box_rows, uint32_t box_cols) {
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0) throw std::runtime_error("TMA base address must be 16-byte aligned");
  if (pitch_bytes % 16 != 0) throw std::runtime_error("TMA row pitch must be a multiple of 16 bytes");
  if (box_cols % 16 != 0 || box_cols > 256 || box_rows > 256) throw std::runtime_error("TMA byte box out of range");
  CUtensorMap m;
  cuuint64_t dims[2] = {cols_bytes, rows};
  cuuint64_t strides[1] = {pitch_bytes};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = get_encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box,
                               estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) throw std::runtime_error("cuTensorMapEncodeTiled (u8) failed: " + std::to_string((int)r));
  return m;
}

}  // namespace kapsl
