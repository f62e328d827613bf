// Issue-cost probe of the tcgen05 GEMM mainloop (a diagnostic behind
// `kernel_bench gemm_issue`): how many cycles the MMA thread spends per 64-wide
// k slice of a 256 x 256 (cta_group::2) tile under each piece of the pipeline
// protocol, read with clock64 on the issuing thread of CTA pair 0.
//
//   mode 0  MMAs only (4 per slice, accumulating into one TMEM accumulator)
//   mode 1  + one tcgen05.commit per stage (to a barrier nobody waits on)
//   mode 2  + one wait per stage on an mbarrier whose phase already completed
//   mode 3  the producer/consumer ring without loads (the producer only arrives)
//   mode 4  the ring with TMA loads walking A [M, K] and B [N, K] like the GEMM
//
// ksub 64-wide slices form one ring stage; `units` tiles per CTA pair alternate
// between two accumulators; `width` is the MMA's N (192 and 128 in modes 0..2).  The operand values do not matter for timing.
// Every wait is bounded (1 s); a run-out sets err[0] = 40 and ends the loops.
// A second kernel times back-to-back cta_group::1 MMAs (M = 128, K = 16) of width
// N on one accumulator.
#include "common.cuh"
#include "kernels.h"
#include "tcgen05.cuh"

namespace kapsl {
namespace probe {

using namespace tc;

__device__ __forceinline__ uint32_t cta_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ void tma_2sm(void* dst, const CUtensorMap* m, uint64_t* bar, int x, int y) {
  const uint32_t mb = smem_u32(bar) & 0xFEFFFFFFu;  // transaction bytes land on CTA 0's barrier
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(mb), "r"(x), "r"(y)
      : "memory");
}
__device__ __forceinline__ void mma_2sm(uint32_t d, uint64_t a, uint64_t b, uint32_t id, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d),
      "l"(a), "l"(b), "r"(id), "r"(acc)
      : "memory");
}
__device__ __forceinline__ void commit_2sm(uint64_t* bar) {
  const uint16_t mask = 0x3;
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
          smem_u32(bar)),
      "h"(mask)
      : "memory");
}
__device__ __forceinline__ void commit_1sm(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

constexpr int kStagesMax = 6;
constexpr int kSlice = 128 * 64 * 2 + 128 * 64 * 2;  // this CTA's A half + B half of one slice (32 KiB)

// BN: MMA width (256, 192 or 128); the stage layout stays the 256-wide one, so
// narrower widths read part of each B half (timing only).
template <int KSUB, int BN>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(128, 1)
    issue_probe_kernel(const __grid_constant__ CUtensorMap ta, const __grid_constant__ CUtensorMap tb, int mode,
                       int stages, int units, int kblocks, int m_tiles, int n_tiles, long long* cycles, int* err) {
  griddep_wait_only();
  constexpr int SB = KSUB * kSlice;
  constexpr uint32_t IDESC = idesc_bf16<256, BN>();
  extern __shared__ __align__(1024) uint8_t raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(raw) + 1023) & ~uintptr_t(1023));
  __shared__ __align__(8) uint64_t full[kStagesMax], empty[kStagesMax], done, spare, ready;
  __shared__ uint32_t tbase_sh;
  __shared__ int abort_sh;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cta_rank();
  const int cl = blockIdx.x >> 1;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStagesMax; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(&done, 1);
    mbar_init(&spare, 1);
    mbar_init(&ready, 1);
    mbar_arrive(&ready);  // phase 0 complete: a wait on parity 0 returns at once
    abort_sh = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tbase_sh)),
                 "r"(512)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  cluster_sync();
  tc_fence_after();
  const uint32_t tb0 = tbase_sh;
  auto fail = [&]() {
    abort_sh = 1;
    atomicExch(err, 40);
  };
  if (warp == 0 && lane == 0 && mode >= 3) {
    int stage = 0;
    uint32_t ph = 0;
    for (int u = 0; u < units && !*(volatile int*)&abort_sh; ++u) {
      const int unit = cl + u * (int)(gridDim.x >> 1);
      const int mt = unit % m_tiles, nt = (unit / m_tiles) % n_tiles;
      for (int kb = 0; kb < kblocks; ++kb) {
        if (!mbar_wait_bounded(&empty[stage], ph ^ 1, 1000000000ull)) {
          fail();
          break;
        }
        uint8_t* sa = smem + stage * SB;
        if (mode == 3) {
          if (rank == 0) mbar_arrive(&full[stage]);
        } else {
          if (rank == 0) mbar_arrive_expect_tx(&full[stage], 2 * SB);
#pragma unroll
          for (int j = 0; j < KSUB; ++j) {
            const int kx = (kb * KSUB + j) * 64;
            tma_2sm(sa + j * kSlice, &ta, &full[stage], kx, mt * 256 + (int)rank * 128);
            tma_2sm(sa + j * kSlice + 128 * 64 * 2, &tb, &full[stage], kx, nt * 256 + (int)rank * 128);
          }
        }
        if (++stage == stages) {
          stage = 0;
          ph ^= 1;
        }
      }
    }
  } else if (warp == 1 && lane == 0 && rank == 0) {
    const long long t0 = clock64();
    int stage = 0;
    uint32_t ph = 0;
    for (int u = 0; u < units && !*(volatile int*)&abort_sh; ++u) {
      const uint32_t d = tb0 + (uint32_t)((u & 1) * 256);
      for (int kb = 0; kb < kblocks; ++kb) {
        if (mode >= 3) {
          if (!mbar_wait_bounded(&full[stage], ph, 1000000000ull)) {
            fail();
            break;
          }
          tc_fence_after();
        } else if (mode == 2) {
          if (!mbar_wait_bounded(&ready, 0, 1000000000ull)) {
            fail();
            break;
          }
          tc_fence_after();
        }
#pragma unroll
        for (int j = 0; j < KSUB; ++j) {
          const uint32_t sa = smem_u32(smem + stage * SB + j * kSlice), sb = sa + 128 * 64 * 2;
#pragma unroll
          for (int k = 0; k < 4; ++k)
            mma_2sm(d, smem_desc_sw128(sa + k * 32), smem_desc_sw128(sb + k * 32), IDESC,
                    (kb > 0 || j > 0 || k > 0) ? 1u : 0u);
        }
        if (mode >= 3) commit_2sm(&empty[stage]);
        else if (mode == 1) commit_2sm(&spare);
        if (++stage == stages) {
          stage = 0;
          ph ^= 1;
        }
      }
    }
    commit_2sm(&done);
    if (!mbar_wait_bounded(&done, 0, 1000000000ull)) fail();
    const long long t1 = clock64();
    if (cl == 0) cycles[0] = (t1 - t0) / ((long long)units * kblocks * KSUB);
  }
  if (rank == 1 && warp == 1 && lane == 0 && !mbar_wait_bounded(&done, 0, 1000000000ull)) fail();
  tc_fence_before();
  __syncthreads();
  cluster_sync();
  tc_fence_after();
  if (warp == 1) asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tb0), "r"(512) : "memory");
}

template <int N>
__global__ void __launch_bounds__(128, 1) mma_rate_kernel(int iters, long long* cycles, int* err) {
  griddep_wait_only();
  constexpr uint32_t IDESC = idesc_bf16<128, N>();
  extern __shared__ __align__(1024) uint8_t raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(raw) + 1023) & ~uintptr_t(1023));
  __shared__ __align__(8) uint64_t done;
  __shared__ uint32_t tb_sh;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    mbar_init(&done, 1);
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(&tb_sh, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tb = tb_sh;
  if (warp == 1 && lane == 0) {
    const uint32_t sa = smem_u32(smem), sb = sa + 128 * 128;
    const long long t0 = clock64();
    for (int i = 0; i < iters; ++i) {
#pragma unroll
      for (int k = 0; k < 4; ++k)
        mma_bf16(tb, smem_desc_sw128(sa + k * 32), smem_desc_sw128(sb + k * 32), IDESC, (i > 0 || k > 0) ? 1u : 0u);
    }
    commit_1sm(&done);
    if (!mbar_wait_bounded(&done, 0, 1000000000ull)) atomicExch(err, 40);
    const long long t1 = clock64();
    if (blockIdx.x == 0) cycles[0] = (t1 - t0) / (4LL * iters);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tb, 512);
}

}  // namespace probe

void launch_gemm_issue_probe(const __nv_bfloat16* A, const __nv_bfloat16* B, int M, int N, int K, int mode, int ksub,
                             int stages, int units, int width, long long* cycles, int* err, cudaStream_t st) {
  using namespace probe;
  if (ksub != 1 && ksub != 2) throw std::runtime_error("gemm_issue_probe: ksub must be 1 or 2");
  if (width != 256 && ((width != 192 && width != 128) || ksub != 1 || mode > 2))
    throw std::runtime_error("gemm_issue_probe: widths 192 and 128 only without the ring (mode 0..2, ksub 1)");
  if (stages < 2 || stages > kStagesMax || stages * ksub * kSlice + 1024 > 232448)
    throw std::runtime_error("gemm_issue_probe: stages do not fit shared memory");
  if (M % 256 != 0 || N % 256 != 0 || K % (64 * ksub) != 0 || mode < 0 || mode > 4 || units < 1)
    throw std::runtime_error("gemm_issue_probe: M, N multiples of 256, K of 64 * ksub, mode 0..4");
  const int sms = gemm_num_sms() & ~1;
  CUtensorMap ta = make_tmap_2d_bf16(A, M, K, K, 128, 64);
  CUtensorMap tb = make_tmap_2d_bf16(B, N, K, K, 128, 64);
  const size_t smem = (size_t)stages * ksub * kSlice + 1024;
  const int kblocks = K / (64 * ksub);
  auto go = [&](auto kern) {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    launch_k(kern, sms, 128, smem, st, ta, tb, mode, stages, units, kblocks, M / 256, N / 256, cycles, err);
  };
  if (ksub == 2) go(issue_probe_kernel<2, 256>);
  else if (width == 192) go(issue_probe_kernel<1, 192>);
  else if (width == 128) go(issue_probe_kernel<1, 128>);
  else go(issue_probe_kernel<1, 256>);
  KAPSL_LAUNCH_CHECK();
  note_launch();
}

void launch_mma_rate_probe(int n, int iters, long long* cycles, int* err, cudaStream_t st) {
  using namespace probe;
  const size_t smem = 120 * 1024;  // one CTA per SM (TMEM allocation of 512 columns)
  const int sms = gemm_num_sms();
  auto go = [&](auto kern) {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    launch_k(kern, sms, 128, smem, st, iters, cycles, err);
  };
  switch (n) {
    case 64: go(mma_rate_kernel<64>); break;
    case 128: go(mma_rate_kernel<128>); break;
    case 256: go(mma_rate_kernel<256>); break;
    default: throw std::runtime_error("mma_rate_probe: N must be 64, 128 or 256");
  }
  KAPSL_LAUNCH_CHECK();
  note_launch();
}

}  // namespace kapsl
