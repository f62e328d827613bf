// Persistent bf16 GEMM on the 5th-generation tensor cores (tcgen05 + TMEM).
//
//   C[M, N] = epilogue( A[M, K] . B[N, K]^T )        A, B: bf16, K contiguous
//
// Warp roles (192 threads, one CTA per SM, persistent over output tiles):
//   warp 0      TMA producer: one elected thread streams 128x64 A and BNx64 B
//               tiles (128-byte swizzle) into a STAGES-deep smem ring.
//   warp 1      MMA issuer: allocates TMEM, one thread issues
//               tcgen05.mma.cta_group::1.kind::f16 (M=128, N=BN, K=16) from
//               smem descriptors and commits to mbarriers.
//   warps 2..5  epilogue: tcgen05.ld 32x32b rows out of TMEM (two accumulator
//               buffers so tile i's epilogue overlaps tile i+1's mainloop),
//               apply the fused op and store.
//
// Fused epilogues: plain, +bias[N], +residual[M,N] (may alias C), SwiGLU over
// an interleaved gate/up weight (per BN-column tile: first BN/2 columns gate,
// last BN/2 up) writing C[M, N/2].  Split-K writes fp32 partials that
// `splitk_reduce_kernel` sums and finishes with the same epilogue.
//
// Operand tiles are loaded per CTA (each CTA reads its own tiles from local
// HBM); EPI 5 stores rows into peer GPUs' receive buffers (tensor parallel).
#include "common.cuh"
#include "kernels.h"
#include "tcgen05.cuh"

namespace kapsl {

using bf16 = __nv_bfloat16;

namespace gemm {

constexpr int BM = 128;
constexpr int BK = 64;
constexpr int kThreads = 192;
// scatter-epilogue staging per epilogue warp: 32 rows x 64 bf16 columns, rows padded
// to 144 bytes so the per-lane row writes and the row-piece reads spread over banks
constexpr int kScatterRow = 144;
constexpr int kScatterStage = 32 * kScatterRow;
// 64-wide k slices per ring stage of the 2-SM kernel.  The MMA thread pays about
// 100 cycles per stage for its full-barrier wait that the tensor pipe does not hide
// (measured: 256 x 256 x 64 per pair takes ~620 cycles with one slice per stage and
// ~525 with two, against 512 of MMA issue), so a stage carries two slices and the
// wait is paid once per 8 MMAs.
constexpr int KSUB2 = 2;

using namespace tc;

template <int BN>
__host__ __device__ constexpr uint32_t instr_desc_bf16() {
  return idesc_bf16<BM, BN>();
}

__device__ __forceinline__ float silu(float x) { return x / (1.f + __expf(-x)); }

struct EpiArgs {
  void* out;           // bf16 or fp32
  int64_t ldc;         // elements
  const bf16* bias;    // [N] or null
  const bf16* res;     // [M, N] or null
  int64_t ldr;
  float* partial;      // split-K fp32 partials [splits, M, N]
  // EPI 5 (tensor-parallel scatter): row r belongs to rank r / rows_per_rank and
  // is stored into that rank's receive slot [my_rank] over NVLink.
  __nv_bfloat16* peers[8];
  int rows_per_rank;
  int my_rank;
  // Grouped (MoE) mode: [0] = number of valid 128-row M tiles, [1 + i] = the
  // expert (row block of B, N rows each) that M tile i multiplies with.
  const int* group_mtiles;
};

__device__ __forceinline__ __nv_bfloat16* scatter_dst(const EpiArgs& ep, int row, int col) {
  const int owner = row / ep.rows_per_rank;
  const int local = row - owner * ep.rows_per_rank;
  return ep.peers[owner] + ((int64_t)ep.my_rank * ep.rows_per_rank + local) * ep.ldc + col;
}

// Store 32 consecutive columns (c0..c0+31) of one row.
template <bool OUT_F32>
__device__ __forceinline__ void store_row32(void* out, int64_t ldc, int row, int c0, int ncols_valid,
                                            const float (&v)[32]) {
  if (OUT_F32) {
    float* dst = reinterpret_cast<float*>(out) + (int64_t)row * ldc + c0;
    if (ncols_valid >= 32) {
#pragma unroll
      for (int i = 0; i < 8; ++i)
        reinterpret_cast<float4*>(dst)[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
    } else {
      for (int i = 0; i < ncols_valid; ++i) dst[i] = v[i];
    }
  } else {
    bf16* dst = reinterpret_cast<bf16*>(out) + (int64_t)row * ldc + c0;
    if (ncols_valid >= 32) {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        uint4 u;
        u.x = pack_bf16(v[8 * i + 0], v[8 * i + 1]);
        u.y = pack_bf16(v[8 * i + 2], v[8 * i + 3]);
        u.z = pack_bf16(v[8 * i + 4], v[8 * i + 5]);
        u.w = pack_bf16(v[8 * i + 6], v[8 * i + 7]);
        reinterpret_cast<uint4*>(dst)[i] = u;
      }
    } else {
      for (int i = 0; i < ncols_valid; ++i) dst[i] = __float2bfloat16(v[i]);
    }
  }
}

__device__ __forceinline__ void load_bf16x32(const bf16* src, int nvalid, float (&v)[32]) {
  if (nvalid >= 32) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      uint4 u = reinterpret_cast<const uint4*>(src)[i];
      const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        float2 f = __bfloat1622float2(h[j]);
        v[8 * i + 2 * j] = f.x;
        v[8 * i + 2 * j + 1] = f.y;
      }
    }
  } else {
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = (i < nvalid) ? __bfloat162float(src[i]) : 0.f;
  }
}

// EPI: 0 plain, 1 bias, 2 residual, 3 swiglu (interleaved), 4 split-K partial (fp32, raw)
// GROUPED: A rows are expert-sorted segments padded to BM; M tile i uses the B
// rows of expert ep.group_mtiles[1 + i] (B holds the experts stacked, N rows each).
template <int BN, int STAGES, int EPI, bool OUT_F32, bool GROUPED = false>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b, int M,
                int N, int K, int splits, EpiArgs ep, int* __restrict__ err) {
  griddep_entry();
  constexpr int A_BYTES = BM * BK * 2;
  constexpr int B_BYTES = BN * BK * 2;
  constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  constexpr uint32_t TMEM_COLS = (2 * BN <= 32) ? 32 : (2 * BN <= 64) ? 64 : (2 * BN <= 128) ? 128 : (2 * BN <= 256) ? 256 : 512;
  constexpr uint32_t IDESC = instr_desc_bf16<BN>();

  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ __align__(8) uint64_t full_bar[STAGES];
  __shared__ __align__(8) uint64_t empty_bar[STAGES];
  __shared__ __align__(8) uint64_t tfull_bar[2];
  __shared__ __align__(8) uint64_t tempty_bar[2];
  __shared__ uint32_t tmem_base_sh;
  __shared__ int abort_sh;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m_tiles = GROUPED ? min(*ep.group_mtiles, (M + BM - 1) / BM) : (M + BM - 1) / BM;
  const int n_tiles = (N + BN - 1) / BN;
  const int k_blocks_total = (K + BK - 1) / BK;
  const int k_per_split = (k_blocks_total + splits - 1) / splits;
  const int num_units = m_tiles * n_tiles * splits;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull_bar[a], 1);
      mbar_init(&tempty_bar[a], 4);
    }
    abort_sh = 0;
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(&tmem_base_sh, TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = tmem_base_sh;

  // unit -> (m tile, n tile, split); m fastest so co-resident CTAs share B tiles in L2.
  auto decode_unit = [&](int u, int& mt, int& nt, int& sp) {
    sp = u % splits;
    const int t = u / splits;
    mt = t % m_tiles;
    nt = t / m_tiles;
  };

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&tmap_a);
      tma_prefetch_desc(&tmap_b);
      int stage = 0;
      uint32_t phase = 0;
      int issued_unwaited = 0;
      for (int u = blockIdx.x; u < num_units && !*(volatile int*)&abort_sh; u += gridDim.x) {
        int mt, nt, sp;
        decode_unit(u, mt, nt, sp);
        const int kb0 = sp * k_per_split;
        const int kb1 = min(k_blocks_total, kb0 + k_per_split);
        const int brow = GROUPED ? ep.group_mtiles[1 + mt] * N + nt * BN : nt * BN;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait_bounded(&empty_bar[stage], phase ^ 1)) {
            abort_sh = 1;
            atomicExch(err, 10);
            break;
          }
          uint8_t* sa = smem + (size_t)stage * STAGE_BYTES;
          uint8_t* sb = sa + A_BYTES;
          mbar_arrive_expect_tx(&full_bar[stage], STAGE_BYTES);
          tma_load_2d(sa, &tmap_a, &full_bar[stage], kb * BK, mt * BM);
          tma_load_2d(sb, &tmap_b, &full_bar[stage], kb * BK, brow);
          ++issued_unwaited;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      (void)issued_unwaited;
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int it = 0;
      for (int u = blockIdx.x; u < num_units && !*(volatile int*)&abort_sh; u += gridDim.x, ++it) {
        int mt, nt, sp;
        decode_unit(u, mt, nt, sp);
        const int kb0 = sp * k_per_split;
        const int kb1 = min(k_blocks_total, kb0 + k_per_split);
        const int acc = it & 1;
        const uint32_t acc_phase = (uint32_t)((it >> 1) & 1);
        if (!mbar_wait_bounded(&tempty_bar[acc], acc_phase ^ 1)) {
          abort_sh = 1;
          atomicExch(err, 11);
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(acc * BN);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait_bounded(&full_bar[stage], phase)) {
            abort_sh = 1;
            atomicExch(err, 12);
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + (size_t)stage * STAGE_BYTES);
          const uint32_t sb = sa + A_BYTES;
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            const uint64_t ad = smem_desc_sw128(sa + k * 32);
            const uint64_t bd = smem_desc_sw128(sb + k * 32);
            mma_bf16(d_tmem, ad, bd, IDESC, (kb > kb0 || k > 0) ? 1u : 0u);
          }
          mma_commit(&empty_bar[stage]);  // frees the smem stage once these MMAs retire
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (*(volatile int*)&abort_sh) break;
        mma_commit(&tfull_bar[acc]);  // accumulator ready for the epilogue
      }
    }
    __syncwarp();
  } else {
    // epilogue warps 2..5 -> TMEM lane quadrant warp % 4
    const int quad = warp & 3;
    int it = 0;
    for (int u = blockIdx.x; u < num_units; u += gridDim.x, ++it) {
      int mt, nt, sp;
      decode_unit(u, mt, nt, sp);
      const int acc = it & 1;
      const uint32_t acc_phase = (uint32_t)((it >> 1) & 1);
      const bool got = mbar_wait_bounded(&tfull_bar[acc], acc_phase);
      if (!__all_sync(0xffffffffu, got)) {
        if (lane == 0) {
          abort_sh = 1;
          atomicExch(err, 13);
        }
        break;
      }
      tc_fence_after();
      const int row = mt * BM + quad * 32 + lane;
      const uint32_t tbase = tmem_base + ((uint32_t)(quad * 32) << 16) + (uint32_t)(acc * BN);
      if (EPI == 3) {
        // SwiGLU over interleaved [gate(BN/2) | up(BN/2)] columns of this tile.
        constexpr int HALF = BN / 2;
        const int out_c0 = nt * HALF;
#pragma unroll 1
        for (int c = 0; c < HALF; c += 32) {
          float g[32], v[32];
          tmem_ld32(tbase + c, g);
          tmem_ld32(tbase + HALF + c, v);
          if (row < M) {
#pragma unroll
            for (int i = 0; i < 32; ++i) v[i] = silu(g[i]) * v[i];
            const int nvalid = min(32, N / 2 - (out_c0 + c));
            if (nvalid > 0) store_row32<OUT_F32>(ep.out, ep.ldc, row, out_c0 + c, nvalid, v);
          }
        }
      } else {
#pragma unroll 1
        for (int c = 0; c < BN; c += 32) {
          float v[32];
          tmem_ld32(tbase + c, v);
          const int col = nt * BN + c;
          const int nvalid = min(32, N - col);
          if (row < M && nvalid > 0) {
            if (EPI == 4) {
              float* dst = ep.partial + ((int64_t)sp * M + row) * N + col;
              if (nvalid >= 32) {
#pragma unroll
                for (int i = 0; i < 8; ++i)
                  reinterpret_cast<float4*>(dst)[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
              } else {
                for (int i = 0; i < nvalid; ++i) dst[i] = v[i];
              }
            } else {
              if (EPI == 1) {
                float bb[32];
                load_bf16x32(ep.bias + col, nvalid, bb);
#pragma unroll
                for (int i = 0; i < 32; ++i) v[i] += bb[i];
              } else if (EPI == 2) {
                float rr[32];
                load_bf16x32(ep.res + (int64_t)row * ep.ldr + col, nvalid, rr);
#pragma unroll
                for (int i = 0; i < 32; ++i) v[i] += rr[i];
              }
              if (EPI == 5)
                store_row32<false>(scatter_dst(ep, row, col), 0, 0, 0, nvalid, v);
              else
                store_row32<OUT_F32>(ep.out, ep.ldc, row, col, nvalid, v);
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty_bar[acc]);
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem_base, TMEM_COLS);
}

// ============================================================ 2-SM variant
// A CTA pair (cluster of 2) computes a 256 x 256 tile with
// tcgen05.mma.cta_group::2 (M = 256, N = 256, K = 16): CTA r TMA-loads rows
// [r*128, r*128+128) of the A tile and rows [r*128, r*128+128) of the B tile
// (half of N) into its own shared memory, signalling the leader's barrier.
// The leader (rank 0) issues the MMAs; each CTA's TMEM receives its 128 rows
// x 256 columns of the accumulator.  MMA completion is signalled to the
// barriers of both CTAs by one tcgen05.commit; epilogue warps of both CTAs
// release an accumulator by arriving on the leader's barrier.  Per CTA and
// k-block this moves 32 KiB of operands for 2 x 128 x 256 x 64 MACs (the 1-SM
// 128 x 256 tile moves 48 KiB for half of that).  Every operand copy is a plain
// per-CTA TMA load of this GPU's memory.
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ uint32_t mapa_shared(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}
__device__ __forceinline__ void mbar_arrive_remote(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
__device__ __forceinline__ void tma_load_2d_2sm(void* smem_dst, const CUtensorMap* m, uint64_t* bar, int32_t x,
                                                int32_t y) {
  // mbarrier address with the peer bit cleared: transaction bytes land on CTA 0's barrier
  const uint32_t mbar = smem_u32(bar) & 0xFEFFFFFFu;
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(mbar), "r"(x), "r"(y)
      : "memory");
}
__device__ __forceinline__ void mma_bf16_2sm(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                             uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void mma_commit_2sm_mc(uint64_t* bar) {
  const uint16_t mask = 0x3;
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
          smem_u32(bar)),
      "h"(mask)
      : "memory");
}

template <int BN, int STAGES, int EPI, bool OUT_F32>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    gemm2sm_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b, int M,
                   int N, int K, EpiArgs ep, int* __restrict__ err) {
  griddep_entry();
  static_assert(BN % 32 == 0 && BN >= 64 && BN <= 256, "2-SM tile width");
  constexpr int A_HALF = 128 * BK * 2;       // 16 KiB: this CTA's 128 rows of the A tile
  constexpr int B_HALF = (BN / 2) * BK * 2;  // this CTA's BN/2 rows of the B tile
  constexpr int HALF_BYTES = A_HALF;
  constexpr int ATOM_BYTES = A_HALF + B_HALF;  // one 64-wide k slice of both operands
  constexpr int STAGE_BYTES = KSUB2 * ATOM_BYTES;
  static_assert(ATOM_BYTES % 1024 == 0, "k slices stay 1 KiB aligned (128-byte swizzle atoms)");
  constexpr uint32_t TMEM_COLS = 512;        // two accumulators at columns 0 and 256
  constexpr uint32_t IDESC = idesc_bf16<256, BN>();

  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ __align__(8) uint64_t full_bar[STAGES];
  __shared__ __align__(8) uint64_t empty_bar[STAGES];
  __shared__ __align__(8) uint64_t tfull_bar[2];
  __shared__ __align__(8) uint64_t tempty_bar[2];
  __shared__ uint32_t tmem_base_sh;
  __shared__ int abort_sh;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int cluster = blockIdx.x >> 1;
  const int nclusters = gridDim.x >> 1;
  const int m_tiles = (M + 255) / 256;
  const int n_tiles = (N + BN - 1) / BN;
  const int kslices = (K + BK - 1) / BK;
  const int kblocks = (kslices + KSUB2 - 1) / KSUB2;  // stages per tile; the last may hold one slice
  const int units = m_tiles * n_tiles;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull_bar[a], 1);
      mbar_init(&tempty_bar[a], 8);  // 4 epilogue warps x 2 CTAs
    }
    abort_sh = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_base_sh)),
                 "r"(TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  cluster_sync_all();  // barriers of both CTAs initialised before any remote use
  tc_fence_after();
  const uint32_t tmem_base = tmem_base_sh;

  // Tile order: groups of G m-tiles, m fastest inside a group.  Up to 16 m-tiles
  // (4096 rows) one group holds them all, so each weight tile is streamed from HBM
  // once with every m-tile of a wave reusing it from L2; above that, groups of 8
  // keep a wave's operand footprint near-square (8192^3: ~69 MB of A and B per
  // wave instead of all of A, 128 MB, per wave).
  const int group_m = m_tiles > 16 ? 8 : m_tiles;
  auto decode = [&](int u, int& mt, int& nt) {
    const int g = u / (group_m * n_tiles), r = u % (group_m * n_tiles);
    const int m0 = g * group_m;
    const int gm = min(group_m, m_tiles - m0);
    mt = m0 + r % gm;
    nt = r / gm;
  };

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&tmap_a);
      tma_prefetch_desc(&tmap_b);
      int stage = 0;
      uint32_t phase = 0;
      for (int u = cluster; u < units && !*(volatile int*)&abort_sh; u += nclusters) {
        int mt, nt;
        decode(u, mt, nt);
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!mbar_wait_bounded(&empty_bar[stage], phase ^ 1)) {
            abort_sh = 1;
            atomicExch(err, 20);
            break;
          }
          uint8_t* sa = smem + (size_t)stage * STAGE_BYTES;
          const int nsl = min(KSUB2, kslices - kb * KSUB2);
          if (leader) mbar_arrive_expect_tx(&full_bar[stage], 2 * nsl * ATOM_BYTES);
          for (int j = 0; j < nsl; ++j) {
            const int kx = (kb * KSUB2 + j) * BK;
            tma_load_2d_2sm(sa + j * ATOM_BYTES, &tmap_a, &full_bar[stage], kx, mt * 256 + (int)rank * 128);
            tma_load_2d_2sm(sa + j * ATOM_BYTES + HALF_BYTES, &tmap_b, &full_bar[stage], kx,
                            nt * BN + (int)rank * (BN / 2));
          }
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    if (leader && lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int it = 0;
      for (int u = cluster; u < units && !*(volatile int*)&abort_sh; u += nclusters, ++it) {
        const int acc = it & 1;
        const uint32_t acc_phase = (uint32_t)((it >> 1) & 1);
        if (!mbar_wait_bounded(&tempty_bar[acc], acc_phase ^ 1)) {
          abort_sh = 1;
          atomicExch(err, 21);
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(acc * 256);
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!mbar_wait_bounded(&full_bar[stage], phase)) {
            abort_sh = 1;
            atomicExch(err, 22);
            break;
          }
          tc_fence_after();
          const int nsl = min(KSUB2, kslices - kb * KSUB2);
#pragma unroll
          for (int j = 0; j < KSUB2; ++j) {
            if (j < nsl) {
              const uint32_t sa = smem_u32(smem + (size_t)stage * STAGE_BYTES + j * ATOM_BYTES);
              const uint32_t sb = sa + HALF_BYTES;
#pragma unroll
              for (int k = 0; k < BK / 16; ++k)
                mma_bf16_2sm(d_tmem, smem_desc_sw128(sa + k * 32), smem_desc_sw128(sb + k * 32), IDESC,
                             (kb > 0 || j > 0 || k > 0) ? 1u : 0u);
            }
          }
          mma_commit_2sm_mc(&empty_bar[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (*(volatile int*)&abort_sh) break;
        mma_commit_2sm_mc(&tfull_bar[acc]);
      }
    }
    __syncwarp();
  } else {
    const int quad = warp & 3;
    const uint32_t leader_tempty0 = mapa_shared(smem_u32(&tempty_bar[0]), 0);
    const uint32_t leader_tempty1 = mapa_shared(smem_u32(&tempty_bar[1]), 0);
    int it = 0;
    for (int u = cluster; u < units; u += nclusters, ++it) {
      int mt, nt;
      decode(u, mt, nt);
      const int acc = it & 1;
      const uint32_t acc_phase = (uint32_t)((it >> 1) & 1);
      const bool got = mbar_wait_bounded(&tfull_bar[acc], acc_phase);
      if (!__all_sync(0xffffffffu, got)) {
        if (lane == 0) {
          abort_sh = 1;
          atomicExch(err, 23);
        }
        break;
      }
      tc_fence_after();
      const int row = mt * 256 + (int)rank * 128 + quad * 32 + lane;
      const uint32_t tbase = tmem_base + ((uint32_t)(quad * 32) << 16) + (uint32_t)(acc * 256);
      if (EPI == 3) {
        constexpr int HALF = BN / 2;
        const int out_c0 = nt * HALF;
#pragma unroll 1
        for (int c = 0; c < HALF; c += 32) {
          float g[32], v[32];
          tmem_ld32(tbase + c, g);
          tmem_ld32(tbase + HALF + c, v);
          if (row < M) {
#pragma unroll
            for (int i = 0; i < 32; ++i) v[i] = silu(g[i]) * v[i];
            const int nvalid = min(32, N / 2 - (out_c0 + c));
            if (nvalid > 0) store_row32<OUT_F32>(ep.out, ep.ldc, row, out_c0 + c, nvalid, v);
          }
        }
      } else if (EPI == 5) {
        // Tensor-parallel scatter: each 64-column slab of this warp's 32 rows goes
        // through shared memory (one 128-byte row per lane), then 8 rounds of 4 rows
        // x 8 lanes store 128-byte contiguous row pieces into the owner rank's
        // receive slot over NVLink (a lane-per-row store would send 16-byte pieces).
        uint8_t* stg = smem + (size_t)STAGES * STAGE_BYTES + (size_t)quad * kScatterStage;
        const int row0 = mt * 256 + (int)rank * 128 + quad * 32;
#pragma unroll 1
        for (int c = 0; c < BN; c += 64) {
          float v0[32], v1[32];
          tmem_ld32(tbase + c, v0);
          tmem_ld32(tbase + c + 32, v1);
          uint4* mine = reinterpret_cast<uint4*>(stg + lane * kScatterRow);
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            mine[q] = make_uint4(pack_bf16(v0[8 * q], v0[8 * q + 1]), pack_bf16(v0[8 * q + 2], v0[8 * q + 3]),
                                 pack_bf16(v0[8 * q + 4], v0[8 * q + 5]), pack_bf16(v0[8 * q + 6], v0[8 * q + 7]));
            mine[4 + q] = make_uint4(pack_bf16(v1[8 * q], v1[8 * q + 1]), pack_bf16(v1[8 * q + 2], v1[8 * q + 3]),
                                     pack_bf16(v1[8 * q + 4], v1[8 * q + 5]), pack_bf16(v1[8 * q + 6], v1[8 * q + 7]));
          }
          __syncwarp();
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            const int rr = 4 * k + (lane >> 3), seg = lane & 7;
            const int grow = row0 + rr, gcol = nt * BN + c + seg * 8;
            if (grow < M && gcol < N)
              *reinterpret_cast<uint4*>(scatter_dst(ep, grow, gcol)) =
                  *reinterpret_cast<const uint4*>(stg + rr * kScatterRow + seg * 16);
          }
          __syncwarp();
        }
      } else {
#pragma unroll 1
        for (int c = 0; c < BN; c += 32) {
          float v[32];
          tmem_ld32(tbase + c, v);
          const int col = nt * BN + c;
          const int nvalid = min(32, N - col);
          if (row < M && nvalid > 0) {
            if (EPI == 1) {
              float bb[32];
              load_bf16x32(ep.bias + col, nvalid, bb);
#pragma unroll
              for (int i = 0; i < 32; ++i) v[i] += bb[i];
            } else if (EPI == 2) {
              float rr[32];
              load_bf16x32(ep.res + (int64_t)row * ep.ldr + col, nvalid, rr);
#pragma unroll
              for (int i = 0; i < 32; ++i) v[i] += rr[i];
            }
            store_row32<OUT_F32>(ep.out, ep.ldc, row, col, nvalid, v);
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_remote(acc ? leader_tempty1 : leader_tempty0);
    }
  }
  if (EPI == 5) __threadfence_system();  // remote rows are performed before the grid completes
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // no CTA leaves while its peer may still signal it
  tc_fence_after();
  if (warp == 1) asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(TMEM_COLS) : "memory");
}

// Stages of the 2-SM kernel for a tile width: as many KSUB2-slice stages as fit next
// to the 1 KiB alignment pad (and the scatter epilogue's staging) under the 227 KiB
// dynamic shared-memory limit, at most four (three for 256-wide tiles).
constexpr int gemm2_fit(int bn, int epi) {
  return (232448 - 1024 - 512 - (epi == 5 ? 4 * kScatterStage : 0)) / (KSUB2 * (128 + bn / 2) * BK * 2);
}
constexpr int gemm2_stages(int bn, int epi = 0) { return gemm2_fit(bn, epi) < 4 ? gemm2_fit(bn, epi) : 4; }

template <int BN, int STAGES, int EPI, bool F32>
void launch_2sm(const CUtensorMap& ta, const CUtensorMap& tb, int M, int N, int K, const EpiArgs& ep, int grid,
                int* err, cudaStream_t st) {
  auto kern = gemm2sm_kernel<BN, STAGES, EPI, F32>;
  constexpr size_t smem = (size_t)STAGES * KSUB2 * (128 + BN / 2) * BK * 2 + 1024 + (EPI == 5 ? 4 * kScatterStage : 0);
  static std::atomic<uint64_t> attr_devs{0};
  ensure_smem_attr(attr_devs, kern, smem);
  launch_k(kern, grid, kThreads, smem, st, ta, tb, M, N, K, ep, err);
  KAPSL_LAUNCH_CHECK();
  note_launch();
}

// Sum split-K partials and apply the epilogue.
template <int EPI, bool OUT_F32>
__global__ void splitk_reduce_kernel(const float* __restrict__ partial, int splits, int M, int N, EpiArgs ep) {
  griddep_entry();
  const int64_t idx = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) * 4;
  const int64_t total = (int64_t)M * N;
  if (idx >= total) return;
  float4 acc = reinterpret_cast<const float4*>(partial + idx)[0];
  for (int s = 1; s < splits; ++s) {
    float4 p = reinterpret_cast<const float4*>(partial + (int64_t)s * total + idx)[0];
    acc.x += p.x;
    acc.y += p.y;
    acc.z += p.z;
    acc.w += p.w;
  }
  const int row = (int)(idx / N);
  const int col = (int)(idx % N);
  if (ep.group_mtiles != nullptr && row >= *ep.group_mtiles * BM) return;  // grouped: padding M tiles
  float v[4] = {acc.x, acc.y, acc.z, acc.w};
  if (EPI == 3) {
    // interleaved gate/up: tile width 256 -> halves of 128
    const int tile = col / 256, within = col % 256;
    if (within >= 128) return;  // threads on the "up" half do nothing
    float u[4];
    const float4 pu = reinterpret_cast<const float4*>(partial + idx + 128)[0];
    u[0] = pu.x;
    u[1] = pu.y;
    u[2] = pu.z;
    u[3] = pu.w;
    for (int s = 1; s < splits; ++s) {
      float4 p = reinterpret_cast<const float4*>(partial + (int64_t)s * total + idx + 128)[0];
      u[0] += p.x;
      u[1] += p.y;
      u[2] += p.z;
      u[3] += p.w;
    }
    const int oc = tile * 128 + within;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float o = silu(v[i]) * u[i];
      if (OUT_F32)
        reinterpret_cast<float*>(ep.out)[(int64_t)row * ep.ldc + oc + i] = o;
      else
        reinterpret_cast<bf16*>(ep.out)[(int64_t)row * ep.ldc + oc + i] = __float2bfloat16(o);
    }
    return;
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    if (EPI == 1) v[i] += __bfloat162float(ep.bias[col + i]);
    if (EPI == 2) v[i] += __bfloat162float(ep.res[(int64_t)row * ep.ldr + col + i]);
    if (OUT_F32)
      reinterpret_cast<float*>(ep.out)[(int64_t)row * ep.ldc + col + i] = v[i];
    else
      reinterpret_cast<bf16*>(ep.out)[(int64_t)row * ep.ldc + col + i] = __float2bfloat16(v[i]);
  }
}

template <int BN, int STAGES>
constexpr size_t smem_bytes() {
  return (size_t)STAGES * (BM * BK * 2 + BN * BK * 2) + 1024;
}

template <int BN, int STAGES, int EPI, bool F32, bool GROUPED = false>
void launch_cfg(const CUtensorMap& ta, const CUtensorMap& tb, int M, int N, int K, int splits, const EpiArgs& ep,
                int grid, int* err, cudaStream_t st) {
  auto kern = gemm_kernel<BN, STAGES, EPI, F32, GROUPED>;
  constexpr size_t smem = smem_bytes<BN, STAGES>();
  static std::atomic<uint64_t> attr_devs{0};
  ensure_smem_attr(attr_devs, kern, smem);
  launch_k(kern, grid, kThreads, smem, st, ta, tb, M, N, K, splits, ep, err);
  KAPSL_LAUNCH_CHECK();
  note_launch();
}

}  // namespace gemm

int gemm_num_sms() {
  static int n[16] = {0};
  int dev;
  KAPSL_CHECK_CUDA(cudaGetDevice(&dev));
  if (dev < 16 && n[dev] == 0) KAPSL_CHECK_CUDA(cudaDeviceGetAttribute(&n[dev], cudaDevAttrMultiProcessorCount, dev));
  return dev < 16 ? n[dev] : 148;
}

// Tensor-parallel row-parallel GEMM: every output row is stored into the
// receive buffer of the rank that owns it (peers[owner], slot my_rank) —
// the reduce-scatter's transfer happens inside the epilogue, tile by tile.
void launch_gemm_scatter(const bf16* A, int64_t lda, const bf16* B, int64_t ldb, bf16* const* peers, int world,
                         int my_rank, int rows_per_rank, int64_t ld_recv, int M, int N, int K, int* err,
                         cudaStream_t st) {
  using namespace gemm;
  if (M == 0 || N == 0) return;
  if (K % 8 != 0 || lda % 8 != 0 || ldb % 8 != 0 || ld_recv % 8 != 0)
    throw std::runtime_error("gemm_scatter: K and leading dims must be multiples of 8");
  if (world < 1 || world > 8 || rows_per_rank * world < M) throw std::runtime_error("gemm_scatter: bad row split");
  EpiArgs ep{nullptr, ld_recv, nullptr, nullptr, 0, nullptr};
  for (int i = 0; i < world; ++i) ep.peers[i] = peers[i];
  ep.rows_per_rank = rows_per_rank;
  ep.my_rank = my_rank;
  const int sms = gemm_num_sms();
  const int units2 = ((M + 255) / 256) * ((N + 255) / 256);
  if (M >= 256 && units2 * 4 >= (sms / 2) * 3) {
    CUtensorMap ta = make_tmap_2d_bf16(A, M, K, lda, 128, BK);
    CUtensorMap tb = make_tmap_2d_bf16(B, N, K, ldb, 128, BK);
    launch_2sm<256, gemm2_stages(256, 5), 5, false>(ta, tb, M, N, K, ep, 2 * std::min(units2, sms / 2), err, st);
    return;
  }
  const int m_tiles = (M + BM - 1) / BM;
  const bool narrow = m_tiles * ((N + 255) / 256) < sms && N % 128 == 0;
  const int bn = narrow ? 128 : 256;
  CUtensorMap ta = make_tmap_2d_bf16(A, M, K, lda, BM, BK);
  CUtensorMap tb = make_tmap_2d_bf16(B, N, K, ldb, bn, BK);
  const int units = m_tiles * ((N + bn - 1) / bn);
  if (narrow)
    launch_cfg<128, 6, 5, false>(ta, tb, M, N, K, 1, ep, std::min(units, sms), err, st);
  else
    launch_cfg<256, 4, 5, false>(ta, tb, M, N, K, 1, ep, std::min(units, sms), err, st);
}

// Chooses tile width and split-K so that the grid covers the SMs.
int launch_gemm(const bf16* A, int64_t lda, const bf16* B, int64_t ldb, void* C, int64_t ldc, bool out_f32, int M,
                int N, int K, int epi, const bf16* bias, const bf16* res, int64_t ldr, float* workspace,
                size_t workspace_bytes, int* err, cudaStream_t st, int force_bn, int force_splits, bool defer_splitk) {
  using namespace gemm;
  if (M == 0 || N == 0) return 1;
  if (defer_splitk && (epi != 0 || out_f32)) throw std::runtime_error("gemm: deferred split-K needs the plain bf16 epilogue");
  if (K % 8 != 0 || lda % 8 != 0 || ldb % 8 != 0) throw std::runtime_error("gemm: K and leading dims must be multiples of 8");
  if (ldc % 8 != 0) throw std::runtime_error("gemm: ldc must be a multiple of 8");
  if (epi == 3 && N % 256 != 0) throw std::runtime_error("gemm: SwiGLU epilogue needs N % 256 == 0");
  const int sms = gemm_num_sms();
  {
    // 2-SM tiles (256 rows x BN) when 256x256 tiles fill at least 3/4 of the CTA pairs.
    // force_bn > 256 forces them with BN = force_bn - 256 (512: 256-wide tiles).
    // BN is picked by a wave model: time ~ waves, where a wave is one tile per CTA
    // pair.  A tile's time does not depend on its width: a cta_group::2 MMA of
    // M = 256, K = 16 measured ~128 cycles for N = 128, 192 and 256 alike, so the
    // widest tile wins every tie and a narrower one only when it saves a wave.
    const int nclusters = sms / 2;
    const int m2 = (M + 255) / 256;
    const int units256 = m2 * ((N + 255) / 256);
    const bool use2 = force_bn > 256 || (force_bn == 0 && force_splits == 0 && M >= 256 && units256 * 4 >= nclusters * 3);
    if (use2) {
      int bn2 = force_bn > 256 ? force_bn - 256 : 256;
      if (force_bn == 0 && epi != 3) {
        long best = -1;
        for (int cand : {256, 224, 192, 128}) {
          const int units = m2 * ((N + cand - 1) / cand);
          const long cost = (long)((units + nclusters - 1) / nclusters);
          if (best < 0 || cost < best) {
            best = cost;
            bn2 = cand;
          }
        }
      }
      if (bn2 != 256 && bn2 != 224 && bn2 != 192 && bn2 != 128) throw std::runtime_error("gemm: 2-SM tile width");
      if (epi == 3 && (bn2 != 256 || N % 256 != 0)) throw std::runtime_error("gemm: SwiGLU epilogue needs 256-wide tiles");
      CUtensorMap ta = make_tmap_2d_bf16(A, M, K, lda, 128, BK);
      CUtensorMap tb = make_tmap_2d_bf16(B, N, K, ldb, bn2 / 2, BK);
      EpiArgs ep{C, ldc, bias, res, ldr, workspace};
      const int units2 = m2 * ((N + bn2 - 1) / bn2);
      const int grid = 2 * std::min(units2, nclusters);
#define KAPSL_GEMM2_DISPATCH(BNV)                                                                        \
  {                                                                                                     \
    constexpr int ST = gemm2_stages(BNV);                                                               \
    switch (epi) {                                                                                      \
      case 0: out_f32 ? launch_2sm<BNV, ST, 0, true>(ta, tb, M, N, K, ep, grid, err, st)                 \
                      : launch_2sm<BNV, ST, 0, false>(ta, tb, M, N, K, ep, grid, err, st); break;        \
      case 1: launch_2sm<BNV, ST, 1, false>(ta, tb, M, N, K, ep, grid, err, st); break;                   \
      case 2: launch_2sm<BNV, ST, 2, false>(ta, tb, M, N, K, ep, grid, err, st); break;                   \
      default: throw std::runtime_error("gemm: bad epilogue");                                          \
    }                                                                                                   \
  }
      switch (bn2) {
        case 256:
          if (epi == 3) {
            launch_2sm<256, gemm2_stages(256), 3, false>(ta, tb, M, N, K, ep, grid, err, st);
          } else {
            KAPSL_GEMM2_DISPATCH(256)
          }
          break;
        case 224: KAPSL_GEMM2_DISPATCH(224) break;
        case 192: KAPSL_GEMM2_DISPATCH(192) break;
        default: KAPSL_GEMM2_DISPATCH(128) break;
      }
#undef KAPSL_GEMM2_DISPATCH
      return 1;
    }
  }
  const int m_tiles = (M + BM - 1) / BM;
  const int kblocks = (K + BK - 1) / BK;
  // Small-M GEMMs stream the weights: every SM must take part, but no unit may
  // spill into a second wave, so splits = floor(SMs / tiles).
  auto split_for = [&](int tiles) {
    if (tiles >= sms / 2 || kblocks < 8) return 1;
    int s = std::min(std::min(kblocks / 4, 16), sms / tiles);
    if (s < 1) s = 1;
    if (s > 1 && (size_t)s * M * N * sizeof(float) > workspace_bytes) s = 1;
    return s;
  };
  int bn = force_bn ? force_bn : 256;
  if (!force_bn && epi != 3 && N % 128 == 0) {
    // Narrow tiles when they keep more SMs streaming (ties go to the narrow tile,
    // whose 6-stage ring keeps more bytes in flight per SM).
    const int t256 = m_tiles * ((N + 255) / 256), t128 = m_tiles * (N / 128);
    if (t256 < sms) {
      const int u256 = t256 * split_for(t256), u128 = t128 * split_for(t128);
      auto eff = [&](int u) { return (double)u / (double)(((u + sms - 1) / sms) * sms); };
      bn = eff(u128) >= eff(u256) ? 128 : 256;
    }
  }
  if (epi == 3) bn = 256;
  const int n_tiles = (N + bn - 1) / bn;
  int splits = force_splits > 0 ? force_splits : split_for(m_tiles * n_tiles);
  if (splits > kblocks) splits = kblocks;
  if (splits > 1) {  // no empty split: every split gets ceil(kblocks / splits) blocks but the last
    const int kps = (kblocks + splits - 1) / splits;
    splits = (kblocks + kps - 1) / kps;
  }
  if (splits > 1 && (workspace == nullptr || (size_t)splits * M * N * sizeof(float) > workspace_bytes))
    throw std::runtime_error("gemm: split-K needs a larger workspace");
  if (splits > 1 && N % 4 != 0) throw std::runtime_error("gemm: split-K needs N % 4 == 0");
  CUtensorMap ta = make_tmap_2d_bf16(A, M, K, lda, BM, BK);
  CUtensorMap tb = make_tmap_2d_bf16(B, N, K, ldb, bn, BK);
  EpiArgs ep{C, ldc, bias, res, ldr, workspace};
  const int units = m_tiles * n_tiles * splits;
  const int grid = std::min(units, sms);
  const int kepi = splits > 1 ? 4 : epi;
#define KAPSL_GEMM_DISPATCH(BNV, ST)                                                    \
  switch (kepi) {                                                                      \
    case 0: out_f32 ? launch_cfg<BNV, ST, 0, true>(ta, tb, M, N, K, splits, ep, grid, err, st)   \
                    : launch_cfg<BNV, ST, 0, false>(ta, tb, M, N, K, splits, ep, grid, err, st); break; \
    case 1: launch_cfg<BNV, ST, 1, false>(ta, tb, M, N, K, splits, ep, grid, err, st); break;     \
    case 2: launch_cfg<BNV, ST, 2, false>(ta, tb, M, N, K, splits, ep, grid, err, st); break;     \
    case 3: launch_cfg<BNV, ST, 3, false>(ta, tb, M, N, K, splits, ep, grid, err, st); break;     \
    case 4: launch_cfg<BNV, ST, 4, true>(ta, tb, M, N, K, splits, ep, grid, err, st); break;      \
    default: throw std::runtime_error("gemm: bad epilogue");                            \
  }
  if (bn == 256) {
    KAPSL_GEMM_DISPATCH(256, 4)
  } else {
    KAPSL_GEMM_DISPATCH(128, 6)
  }
#undef KAPSL_GEMM_DISPATCH
  if (splits > 1 && defer_splitk) return splits;  // the consumer sums the partials
  if (splits > 1) {
    const int64_t total = (int64_t)M * N / 4;
    const int blocks = (int)((total + 255) / 256);
    switch (epi) {
      case 0: out_f32 ? launch_k(splitk_reduce_kernel<0, true>, blocks, 256, 0, st, workspace, splits, M, N, ep)
                      : launch_k(splitk_reduce_kernel<0, false>, blocks, 256, 0, st, workspace, splits, M, N, ep); break;
      case 1: launch_k(splitk_reduce_kernel<1, false>, blocks, 256, 0, st, workspace, splits, M, N, ep); break;
      case 2: launch_k(splitk_reduce_kernel<2, false>, blocks, 256, 0, st, workspace, splits, M, N, ep); break;
      case 3: launch_k(splitk_reduce_kernel<3, false>, blocks, 256, 0, st, workspace, splits, M, N, ep); break;
    }
    KAPSL_LAUNCH_CHECK();
    note_launch();
  }
  return splits;
}


// Grouped (MoE expert) GEMM: C[rows, N] = A[rows, K] x B[g]^T per 128-row M tile,
// where the expert g of M tile i is mtiles[1 + i] and mtiles[0] is the number of
// valid M tiles (both written on the device by the routing kernels, so the
// launch needs no host synchronisation).  B is [num_groups * N, K].
// epi 0: plain bf16 store; epi 3: SwiGLU over interleaved gate/up (C is [rows, N/2]).
void launch_grouped_gemm(const bf16* A, int64_t lda, const bf16* B, int64_t ldb, bf16* C, int64_t ldc, int rows,
                         int N, int K, int num_groups, const int* mtiles, int epi, int bn, int splits,
                         float* workspace, size_t workspace_bytes, int* err, cudaStream_t st) {
  using namespace gemm;
  if (rows == 0 || N == 0) return;
  if (rows % BM != 0) throw std::runtime_error("grouped gemm: rows must be a multiple of 128");
  if (K % 8 != 0 || lda % 8 != 0 || ldb % 8 != 0 || ldc % 8 != 0)
    throw std::runtime_error("grouped gemm: K and leading dims must be multiples of 8");
  if (epi != 0 && epi != 3) throw std::runtime_error("grouped gemm: epilogue must be 0 (plain) or 3 (SwiGLU)");
  if (epi == 3 && N % 256 != 0) throw std::runtime_error("grouped gemm: SwiGLU needs N % 256 == 0");
  if (N % 128 != 0) throw std::runtime_error("grouped gemm: N must be a multiple of 128");
  const int sms = gemm_num_sms();
  if (bn == 0) bn = (epi == 3 || (rows / BM) * (N / 256) >= sms) ? 256 : 128;
  if (epi == 3) bn = 256;
  if (bn != 128 && bn != 256) throw std::runtime_error("grouped gemm: tile width must be 128 or 256");
  const int kblocks = (K + BK - 1) / BK;
  if (splits < 1) splits = 1;
  if (splits > kblocks) splits = kblocks;
  if (splits > 1) {  // no empty split: every split gets ceil(kblocks / splits) blocks but the last
    const int kps = (kblocks + splits - 1) / splits;
    splits = (kblocks + kps - 1) / kps;
  }
  if (splits > 1 && (workspace == nullptr || (size_t)splits * rows * N * sizeof(float) > workspace_bytes))
    throw std::runtime_error("grouped gemm: split-K needs a larger workspace");
  CUtensorMap ta = make_tmap_2d_bf16(A, rows, K, lda, BM, BK);
  CUtensorMap tb = make_tmap_2d_bf16(B, (uint64_t)num_groups * N, K, ldb, bn, BK);
  EpiArgs ep{C, ldc, nullptr, nullptr, 0, workspace};
  ep.group_mtiles = mtiles;
  const int units = (rows / BM) * (N / bn) * splits;  // upper bound; the kernel reads the valid count
  const int grid = std::min(units, sms);
  const int kepi = splits > 1 ? 4 : epi;
  if (bn == 256) {
    switch (kepi) {
      case 0: launch_cfg<256, 4, 0, false, true>(ta, tb, rows, N, K, splits, ep, grid, err, st); break;
      case 3: launch_cfg<256, 4, 3, false, true>(ta, tb, rows, N, K, splits, ep, grid, err, st); break;
      case 4: launch_cfg<256, 4, 4, true, true>(ta, tb, rows, N, K, splits, ep, grid, err, st); break;
    }
  } else {
    switch (kepi) {
      case 0: launch_cfg<128, 6, 0, false, true>(ta, tb, rows, N, K, splits, ep, grid, err, st); break;
      case 4: launch_cfg<128, 6, 4, true, true>(ta, tb, rows, N, K, splits, ep, grid, err, st); break;
      default: throw std::runtime_error("grouped gemm: bad epilogue");
    }
  }
  if (splits > 1) {
    const int64_t total = (int64_t)rows * N / 4;
    const int blocks = (int)((total + 255) / 256);
    if (epi == 3)
      launch_k(splitk_reduce_kernel<3, false>, blocks, 256, 0, st, workspace, splits, rows, N, ep);
    else
      launch_k(splitk_reduce_kernel<0, false>, blocks, 256, 0, st, workspace, splits, rows, N, ep);
    KAPSL_LAUNCH_CHECK();
    note_launch();
  }
}

}  // namespace kapsl
