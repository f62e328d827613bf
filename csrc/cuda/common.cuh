// Shared device helpers for the sm_100a kernels of kapsl_sdk_b200.
//
// Everything here is plain CUDA / inline PTX written for Blackwell (sm_100a):
// mbarrier + TMA (cp.async.bulk.tensor) helpers, warp reductions and the
// host-side launch counter that the benchmark reports as `gpu_launches`.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>
#include <stdexcept>
#include <string>
#include <utility>

namespace kapsl {

// ---------------------------------------------------------------- host side
uint64_t launch_count();
void note_launch(uint64_t n = 1);

#define KAPSL_CHECK_CUDA(expr)                                                   \
  do {                                                                           \
    cudaError_t _e = (expr);                                                     \
    if (_e != cudaSuccess)                                                       \
      throw std::runtime_error(std::string("CUDA error: ") +                     \
                               cudaGetErrorString(_e) + " at " + __FILE__ +      \
                               ":" + std::to_string(__LINE__));                  \
  } while (0)

#define KAPSL_LAUNCH_CHECK() KAPSL_CHECK_CUDA(cudaGetLastError())

// Raises the dynamic shared-memory limit of `kern` to `smem` bytes on the
// CURRENT device the first time a launch there needs it.  The attribute is
// per device, so `done` (a static owned by the launch site) keeps one bit per
// device ordinal: a process that drives several GPUs sets it on each of them.
// Two threads racing on the same device both call cudaFuncSetAttribute, which
// is idempotent; the bit is published with release order.
template <typename Kernel>
inline void ensure_smem_attr(std::atomic<uint64_t>& done, Kernel* kern, size_t smem) {
  int dev = 0;
  KAPSL_CHECK_CUDA(cudaGetDevice(&dev));
  const uint64_t bit = dev < 64 ? (1ull << dev) : 0ull;
  if (bit != 0 && (done.load(std::memory_order_acquire) & bit)) return;
  KAPSL_CHECK_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  if (bit != 0) done.fetch_or(bit, std::memory_order_acq_rel);
}

// Programmatic dependent launch.  Every kernel of this library starts with
// griddep_entry(): it lets the next kernel in the stream begin launching (its
// CTAs get scheduled and reach their own entry while this grid runs) and then
// waits until the previous grid has completed and its memory is visible.
// Because every kernel waits first, a grid never completes before its
// predecessor, so "previous grid done" implies "every earlier grid done".
// launch_k() issues a kernel with the attribute that allows the early launch
// (KAPSL_PDL=0 turns it off: plain stream order).
bool pdl_enabled();

template <typename... KArgs, typename... Args>
inline void launch_k(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  KAPSL_CHECK_CUDA(cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...));
}

// 2-D bf16 tensor map (row-major, `rows` x `cols`, row pitch `pitch_elems`),
// box = box_rows x box_cols, 128-byte swizzle.  Encoded through the driver
// entry point so the extension does not link libcuda directly.
CUtensorMap make_tmap_2d_bf16(const void* base, uint64_t rows, uint64_t cols,
                              uint64_t pitch_elems, uint32_t box_rows,
                              uint32_t box_cols, bool swizzle128 = true);
// 2-D uint8 tensor map without swizzle: rows x cols_bytes, row pitch in bytes.
CUtensorMap make_tmap_2d_u8(const void* base, uint64_t rows, uint64_t cols_bytes, uint64_t pitch_bytes,
                            uint32_t box_rows, uint32_t box_cols);

// --------------------------------------------------------------- device side
#ifdef __CUDACC__
__device__ __forceinline__ void griddep_entry() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");
}
// Entry of a kernel that does not let the next one launch early (it launches when
// this grid completes): waits for the previous grid only.  The sampler uses it:
// with the early trigger, back-to-back 256 x 152064 samplings measured 4x slower
// (339 us against 85 us); the dependents' waiting CTAs are not worth it there.
__device__ __forceinline__ void griddep_wait_only() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_min(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fminf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---- mbarrier --------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}
__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
// Bounded wait: polls the barrier and gives up after `timeout_ns` of wall time
// (read from %globaltimer), so a missing arrival turns into an error status
// for the host instead of a hung GPU.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity,
                                                  uint64_t timeout_ns = 2000000000ull) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  while (true) {
#pragma unroll 1
    for (int i = 0; i < 64; ++i)
      if (mbar_try_wait(bar, parity)) return true;
    if (globaltimer_ns() - t0 > timeout_ns) return false;
  }
}

// ---- cross-GPU flags (symmetric memory) --------------------------------------
__device__ __forceinline__ void st_release_sys(int64_t* p, int64_t v) {
  asm volatile("st.release.sys.global.b64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ int64_t ld_acquire_sys(const int64_t* p) {
  int64_t v;
  asm volatile("ld.acquire.sys.global.b64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ int64_t ld_relaxed_sys(const int64_t* p) {
  int64_t v;
  asm volatile("ld.relaxed.sys.global.b64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
// Waits until flags_site[p] >= epoch for every p < world; false after timeout_ns.
// The flags are polled with relaxed loads and one acquire fence follows the last
// one (fence-based acquire: later loads see what the peers released before their
// flag stores), which measured half the round trip of polling with ld.acquire.
__device__ __forceinline__ bool wait_flags(const int64_t* flags_site, int world, int64_t epoch,
                                           uint64_t timeout_ns) {
  const uint64_t t0 = globaltimer_ns();
  for (int p = 0; p < world; ++p) {
    while (ld_relaxed_sys(flags_site + p) < epoch) {
      if (globaltimer_ns() - t0 > timeout_ns) return false;
    }
  }
  asm volatile("fence.acq_rel.sys;" ::: "memory");
  return true;
}

// Same contract as mbar_wait_bounded, but the thread asks to be suspended
// inside try_wait (suspend-time hint) instead of spinning, so warps that wait
// for long stretches do not take issue slots from the warps doing the work.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t* bar, uint32_t parity, uint32_t hint_ns) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(hint_ns)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ bool mbar_wait_sleep(uint64_t* bar, uint32_t parity,
                                                uint64_t timeout_ns = 2000000000ull) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  while (true) {
    if (mbar_try_wait_sleep(bar, parity, 100000u)) return true;
    if (globaltimer_ns() - t0 > timeout_ns) return false;
  }
}

// ---- TMA -------------------------------------------------------------------
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* m) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(m)) : "memory");
}
// 2-D tiled load into this CTA's shared memory.  x = innermost (column) coordinate in elements.
__device__ __forceinline__ void tma_load_2d(void* smem_dst, const CUtensorMap* m, uint64_t* bar,
                                            int32_t x, int32_t y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}
__device__ __forceinline__ void tma_load_2d_hint(void* smem_dst, const CUtensorMap* m,
                                                 uint64_t* bar, int32_t x, int32_t y,
                                                 uint64_t hint) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%3, %4}], [%2], %5;" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(smem_u32(bar)), "r"(x), "r"(y), "l"(hint)
      : "memory");
}

// 1-D bulk copy (no tensor map) of `bytes` contiguous bytes into this CTA's
// shared memory; both addresses 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_load(void* smem_dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// ---- warp-level mma (m16n8k16 bf16) used by the attention kernels ----------
__device__ __forceinline__ void mma_bf16_16816(float (&d)[4], const uint32_t (&a)[4],
                                               const uint32_t (&b)[2]) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}
__device__ __forceinline__ void ldmatrix_x4(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void ldmatrix_x4_trans(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

// Byte offset of 16-byte chunk `chunk` (0..7) of row `row` inside a tile
// written by TMA with 128-byte swizzle (rows of 128 bytes, 1024-byte atoms).
__device__ __forceinline__ uint32_t sw128_offset(uint32_t row, uint32_t chunk) {
  return row * 128u + ((chunk ^ (row & 7u)) << 4);
}

#endif  // __CUDACC__

}  // namespace kapsl
