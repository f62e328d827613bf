// GGUF Q4_K weights on the 5th-generation tensor cores, dequantized inside the
// GEMM mainloop.
//
//   Y[M, N] = X[M, K] . W[N, K]^T        X bf16 (activations), W Q4_K (weights)
//
// Q4_K super-block (256 weights along K, 144 bytes): fp16 d, fp16 dmin,
// 12 bytes of 6-bit sub-block scales/mins (8 sub-blocks of 32), 128 bytes of
// 4-bit quants (64-weight groups: low nibbles = first 32, high = next 32);
// w = d * sc[j] * q - dmin * m[j]   (ggml's block_q4_K, ggml-quants.c).
//
// The product is computed transposed, D[n, t] = W[n, :] . X[t, :], so that the
// weights are the MMA's A operand and can live in tensor memory:
//   warp 0       TMA: raw Q4_K rows (128 weight rows x 144 B per super-block)
//   warp 2       TMA: X tiles (TT tokens x 64, 128-byte swizzle); two producers so
//                the weight prefetch never waits behind the activation ring
//   warp 1       MMA: tcgen05.mma.kind::f16 with A read from TMEM (128 x 16),
//                B = the X tile from smem, D (128 x TT fp32) in TMEM
//   warps 3..10  dequant: each thread owns one weight row (its TMEM lane) and
//                one nibble half of every super-block; nibbles -> bf16 pairs with
//                a byte permute + exponent-bias trick, scaled with bf16x2 FMAs,
//                written to TMEM with tcgen05.st (no smem round trip).  The TMEM
//                A ring holds whole super-blocks (4 k-blocks = 128 columns), so
//                the dequant/MMA hand-off happens once per 256 weights.
//   warps 11..14 epilogue: tcgen05.ld of D rows, stores Y[t, n] (coalesced over
//                n across the warp), optional residual add or split-K partials
// Waiting warps sleep in try_wait (suspend hint) instead of spinning.
// The raw weights cross HBM once at 4.5 bits per weight; for small M the
// kernel streams them at memory speed, for large M the MMAs (N = TT = 256)
// amortise the dequant over 256 tokens.
#include <cstdlib>
#include <type_traits>

#include "common.cuh"
#include "kernels.h"
#include "tcgen05.cuh"

namespace kapsl {
namespace q4k {

using namespace tc;
using bf16 = __nv_bfloat16;

constexpr int WT = 128;     // weight rows per tile (MMA M)
constexpr int BK = 64;      // k per k-block
constexpr int QK = 256;     // weights per super-block
constexpr int QB = 144;     // bytes per super-block
constexpr int RAW_BYTES = WT * QB;  // 18432
constexpr int kDequantWarps = 8;
constexpr int kEpiWarps = 4;
constexpr int kDqWarp0 = 3;  // warps: 0 raw TMA, 1 MMA, 2 X TMA, 3..10 dequant, 11..14 epilogue
constexpr int kThreads = 32 * (kDqWarp0 + kDequantWarps + kEpiWarps);  // 480

template <int TT>
struct Cfg {
  static constexpr int NACC = TT <= 128 ? 2 : 1;
  static constexpr int NX = TT <= 64 ? 8 : (TT <= 128 ? 6 : 4);
  static constexpr int NRAW = TT <= 128 ? 6 : 5;  // raw super-block stages (18 KiB each)
  static constexpr int X_BYTES = TT * BK * 2;
  static constexpr int A_COL0 = NACC * TT;
  // TMEM A slots of one super-block each (4 k-blocks x 32 columns), filling
  // the 512 columns that the accumulators leave free.
  static constexpr int NA = (512 - A_COL0) / 128;
  static constexpr uint32_t TMEM_COLS = 512;
  static constexpr size_t SMEM = (size_t)NRAW * RAW_BYTES + (size_t)NX * X_BYTES + 1024;
};

struct Q4Args {
  bf16* out;          // Y [M, ldc]
  int64_t ldc;
  const bf16* res;    // residual [M, ldr] (EPI 2) or null
  int64_t ldr;
  float* partial;     // split-K fp32 partials [splits, M, N]
  // Tile-contiguous weights (null: row-major through the tensor map): the
  // 128 rows x 144 bytes of weight tile nt, super-block sb start at
  // tiled + (nt * nsb + sb) * RAW_BYTES, one bulk copy per super-block.
  const uint8_t* tiled;
  int M, N, K, splits;
  int spin;           // 1: waits spin on try_wait; 0: waits suspend in try_wait (KAPSL_Q4K_SPIN)
};

// Bounded mbarrier wait: spinning, or suspended in try_wait between polls.
__device__ __forceinline__ bool q4_wait(int spin, uint64_t* bar, uint32_t parity) {
  return spin ? mbar_wait_bounded(bar, parity) : mbar_wait_sleep(bar, parity);
}

__device__ __forceinline__ float half_bits_to_float(uint32_t h) {
  return __half2float(__ushort_as_half((unsigned short)h));
}

// 6-bit scale and min of sub-block j from the 12 packed bytes (ggml get_scale_min_k4).
__device__ __forceinline__ void scale_min(const uint8_t* q, int j, int& sc, int& m) {
  if (j < 4) {
    sc = q[j] & 63;
    m = q[j + 4] & 63;
  } else {
    sc = (q[j + 4] & 0xF) | ((q[j - 4] >> 6) << 4);
    m = (q[j + 4] >> 4) | ((q[j] >> 6) << 4);
  }
}

// Two low nibbles (bytes b0, b1 of `word` picked by the byte-permute selector)
// -> bf16x2 (q0 * ds - dm, q1 * ds - dm).  128 + q is built exactly in the bf16
// exponent/mantissa bits (mantissa ulp at 128 is 1), 128 is subtracted exactly
// and one bf16x2 FMA applies the sub-block scale and min.  High nibbles are
// shifted down by 4 before the call.
__device__ __forceinline__ uint32_t dq_pair(uint32_t word, uint32_t sel, __nv_bfloat162 ds, __nv_bfloat162 ndm) {
  const uint32_t t = __byte_perm(word, 0u, sel);
  const uint32_t v = (t & 0x000F000Fu) | 0x43004300u;
  __nv_bfloat162 b = *reinterpret_cast<const __nv_bfloat162*>(&v);
  b = __hsub2(b, __floats2bfloat162_rn(128.f, 128.f));
  b = __hfma2(b, ds, ndm);
  return *reinterpret_cast<uint32_t*>(&b);
}

// scale_min on the 12 bytes held as three words; `lo` = (j < 4), known at
// compile time in the unrolled callers so the word indices stay static.
__device__ __forceinline__ uint32_t byte_of(const uint32_t (&w)[3], int k) {
  return (w[k >> 2] >> (8 * (k & 3))) & 0xFFu;
}
__device__ __forceinline__ void scale_min_w(const uint32_t (&q)[3], int j, bool lo, int& sc, int& m) {
  if (lo) {
    sc = (int)(byte_of(q, j) & 63);
    m = (int)(byte_of(q, j + 4) & 63);
  } else {
    sc = (int)((byte_of(q, j + 4) & 0xF) | ((byte_of(q, j - 4) >> 6) << 4));
    m = (int)((byte_of(q, j + 4) >> 4) | ((byte_of(q, j) >> 6) << 4));
  }
}

template <int TT, int EPI>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_q4k_kernel(const __grid_constant__ CUtensorMap tmap_w, const __grid_constant__ CUtensorMap tmap_x, Q4Args a,
                    int* __restrict__ err) {
  griddep_entry();
  using C = Cfg<TT>;
  constexpr uint32_t IDESC = idesc_bf16<WT, TT>();
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* xring = smem;                                  // NX x X_BYTES (1024-aligned, swizzled)
  uint8_t* rawring = smem + (size_t)C::NX * C::X_BYTES;   // NRAW x RAW_BYTES
  __shared__ __align__(8) uint64_t raw_full[C::NRAW], raw_empty[C::NRAW];
  __shared__ __align__(8) uint64_t x_full[C::NX], x_empty[C::NX];
  __shared__ __align__(8) uint64_t a_full[C::NA], a_empty[C::NA];
  __shared__ __align__(8) uint64_t acc_full[C::NACC], acc_empty[C::NACC];
  __shared__ uint32_t tmem_base_sh;
  __shared__ int abort_sh;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_tiles = (a.N + WT - 1) / WT;
  const int t_tiles = (a.M + TT - 1) / TT;
  const int nsb = a.K / QK;
  const int sb_per_split = (nsb + a.splits - 1) / a.splits;
  const int num_units = n_tiles * t_tiles * a.splits;

  if (threadIdx.x == 0) {
    for (int i = 0; i < C::NRAW; ++i) {
      mbar_init(&raw_full[i], 1);
      mbar_init(&raw_empty[i], kDequantWarps);
    }
    for (int i = 0; i < C::NX; ++i) {
      mbar_init(&x_full[i], 1);
      mbar_init(&x_empty[i], 1);
    }
    for (int i = 0; i < C::NA; ++i) {
      mbar_init(&a_full[i], kDequantWarps);
      mbar_init(&a_empty[i], 1);
    }
    for (int i = 0; i < C::NACC; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], kEpiWarps);
    }
    abort_sh = 0;
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(&tmem_base_sh, C::TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = tmem_base_sh;

  // unit -> (token tile fastest, weight tile, split): consecutive CTAs share a weight tile
  auto decode_unit = [&](int u, int& tt, int& nt, int& sp) {
    tt = u % t_tiles;
    const int r = u / t_tiles;
    nt = r % n_tiles;
    sp = r / n_tiles;
  };
  // Each unit walks its super-blocks from a unit-dependent offset, so the CTAs
  // do not all read the same X tile (the same L2 lines) at the same moment.
  auto rot_sb = [](int u, int sb0, int sb1, int sb) {
    const int cnt = sb1 - sb0;
    return sb0 + (sb - sb0 + (u * 7) % cnt) % cnt;
  };
  auto fail = [&](int code) {
    abort_sh = 1;
    atomicExch(err, code);
  };

  if (warp == 0) {
    // ------------------------------------------------------------ raw Q4_K producer
    if (lane == 0) {
      tma_prefetch_desc(&tmap_w);
      int rs = 0;
      uint32_t rph = 0;
      for (int u = blockIdx.x; u < num_units && !*(volatile int*)&abort_sh; u += gridDim.x) {
        int tt, nt, sp;
        decode_unit(u, tt, nt, sp);
        const int sb0 = sp * sb_per_split, sb1 = min(nsb, sb0 + sb_per_split);
        for (int sb = sb0; sb < sb1; ++sb) {
          if (!q4_wait(a.spin, &raw_empty[rs], rph ^ 1)) { fail(60); break; }
          mbar_arrive_expect_tx(&raw_full[rs], RAW_BYTES);
          const int sbr = rot_sb(u, sb0, sb1, sb);
          if (a.tiled)
            bulk_load(rawring + (size_t)rs * RAW_BYTES, a.tiled + ((size_t)nt * nsb + sbr) * RAW_BYTES, RAW_BYTES,
                      &raw_full[rs]);
          else
            tma_load_2d(rawring + (size_t)rs * RAW_BYTES, &tmap_w, &raw_full[rs], sbr * QB, nt * WT);
          if (++rs == C::NRAW) { rs = 0; rph ^= 1; }
        }
      }
    }
    __syncwarp();
  } else if (warp == 2) {
    // ------------------------------------------------------------ X (activation) producer
    if (lane == 0) {
      tma_prefetch_desc(&tmap_x);
      int xs = 0;
      uint32_t xph = 0;
      for (int u = blockIdx.x; u < num_units && !*(volatile int*)&abort_sh; u += gridDim.x) {
        int tt, nt, sp;
        decode_unit(u, tt, nt, sp);
        const int sb0 = sp * sb_per_split, sb1 = min(nsb, sb0 + sb_per_split);
        for (int kb = sb0 * 4; kb < sb1 * 4; ++kb) {
          if (!q4_wait(a.spin, &x_empty[xs], xph ^ 1)) { fail(61); break; }
          mbar_arrive_expect_tx(&x_full[xs], C::X_BYTES);
          tma_load_2d(xring + (size_t)xs * C::X_BYTES, &tmap_x, &x_full[xs],
                      (rot_sb(u, sb0, sb1, kb >> 2) * 4 + (kb & 3)) * BK, tt * TT);
          if (++xs == C::NX) { xs = 0; xph ^= 1; }
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      int xs = 0, as = 0;
      uint32_t xph = 0, aph = 0;
      int it = 0;
      for (int u = blockIdx.x; u < num_units && !*(volatile int*)&abort_sh; u += gridDim.x, ++it) {
        int tt, nt, sp;
        decode_unit(u, tt, nt, sp);
        const int sb0 = sp * sb_per_split, sb1 = min(nsb, sb0 + sb_per_split);
        const int acc = C::NACC == 2 ? (it & 1) : 0;
        const uint32_t acc_ph = C::NACC == 2 ? (uint32_t)((it >> 1) & 1) : (uint32_t)(it & 1);
        if (!q4_wait(a.spin, &acc_empty[acc], acc_ph ^ 1)) { fail(62); break; }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(acc * TT);
        bool first = true, ok = true;
        for (int sb = sb0; sb < sb1 && ok; ++sb) {
          if (!q4_wait(a.spin, &a_full[as], aph)) { fail(63); ok = false; break; }
          const uint32_t a_tmem = tmem_base + (uint32_t)(C::A_COL0 + as * 128);
          for (int i = 0; i < QK / BK; ++i) {
            if (!q4_wait(a.spin, &x_full[xs], xph)) { fail(63); ok = false; break; }
            tc_fence_after();
            const uint32_t xa = smem_u32(xring + (size_t)xs * C::X_BYTES);
#pragma unroll
            for (int k = 0; k < BK / 16; ++k) {
              mma_bf16_tmem_a(d_tmem, a_tmem + i * 32 + k * 8, smem_desc_sw128(xa + k * 32), IDESC,
                              first ? 0u : 1u);
              first = false;
            }
            mma_commit(&x_empty[xs]);
            if (++xs == C::NX) { xs = 0; xph ^= 1; }
          }
          if (!ok) break;
          mma_commit(&a_empty[as]);
          if (++as == C::NA) { as = 0; aph ^= 1; }
        }
        if (!ok || *(volatile int*)&abort_sh) break;
        mma_commit(&acc_full[acc]);
      }
    }
    __syncwarp();
  } else if (warp < kDqWarp0 + kDequantWarps) {
    // ------------------------------------------------------------ dequant
    const int dw = warp - kDqWarp0;
    const int quad = warp & 3;        // TMEM lane quadrant this warp may access
    const int row = quad * 32 + lane; // weight row inside the tile
    const uint32_t lane_base = tmem_base + ((uint32_t)(quad * 32) << 16) + (uint32_t)C::A_COL0;
    // HALF 0: low nibbles (first sub-block of each 64-group), 1: high nibbles.
    auto run = [&](auto half_c) {
      constexpr int HALF = decltype(half_c)::value;
      int rs = 0, as = 0;
      uint32_t rph = 0, aph = 0;
      for (int u = blockIdx.x; u < num_units; u += gridDim.x) {
        int tt, nt, sp;
        decode_unit(u, tt, nt, sp);
        const int sb0 = sp * sb_per_split, sb1 = min(nsb, sb0 + sb_per_split);
        bool stop = false;
        for (int sb = sb0; sb < sb1; ++sb) {
          const bool got = q4_wait(a.spin, &raw_full[rs], rph);
          if (!__all_sync(0xffffffffu, got)) {
            if (lane == 0) fail(64);
            stop = true;
            break;
          }
          const uint8_t* blk = rawring + (size_t)rs * RAW_BYTES + (size_t)row * QB;
          const uint4 hdr = *reinterpret_cast<const uint4*>(blk);
          const float d = half_bits_to_float(hdr.x & 0xFFFFu);
          const float dmin = half_bits_to_float(hdr.x >> 16);
          const uint32_t scw[3] = {hdr.y, hdr.z, hdr.w};
          uint4 qv[4][2];
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            qv[i][0] = *reinterpret_cast<const uint4*>(blk + 16 + 32 * i);
            qv[i][1] = *reinterpret_cast<const uint4*>(blk + 32 + 32 * i);
          }
          __syncwarp();
          if (lane == 0) mbar_arrive(&raw_empty[rs]);  // the stage's bytes are in registers
          if (++rs == C::NRAW) { rs = 0; rph ^= 1; }
          const bool free_slot = q4_wait(a.spin, &a_empty[as], aph ^ 1);
          if (!__all_sync(0xffffffffu, free_slot)) {
            if (lane == 0) fail(65);
            stop = true;
            break;
          }
          tc_fence_after();
          // four k-blocks: 32 weights (16 packed columns) each, four stores, one wait
#pragma unroll
          for (int i = 0; i < QK / BK; ++i) {
            int sc, mn;
            scale_min_w(scw, 2 * i + HALF, i < 2, sc, mn);
            const float dsf = d * (float)sc;
            const float dmf = dmin * (float)mn;
            const __nv_bfloat162 ds = __floats2bfloat162_rn(dsf, dsf);
            const __nv_bfloat162 ndm = __floats2bfloat162_rn(-dmf, -dmf);
            const uint32_t w[8] = {qv[i][0].x >> (4 * HALF), qv[i][0].y >> (4 * HALF), qv[i][0].z >> (4 * HALF),
                                   qv[i][0].w >> (4 * HALF), qv[i][1].x >> (4 * HALF), qv[i][1].y >> (4 * HALF),
                                   qv[i][1].z >> (4 * HALF), qv[i][1].w >> (4 * HALF)};
            uint32_t r[16];  // column c = weights (2c, 2c + 1) of this sub-block
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              r[2 * j] = dq_pair(w[j], 0x4140u, ds, ndm);
              r[2 * j + 1] = dq_pair(w[j], 0x4342u, ds, ndm);
            }
            tmem_st16(lane_base + (uint32_t)(as * 128 + i * 32 + HALF * 16), r);
          }
          tmem_wait_st();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&a_full[as]);
          if (++as == C::NA) { as = 0; aph ^= 1; }
        }
        if (stop || *(volatile int*)&abort_sh) break;
      }
    };
    if (dw >= 4)
      run(std::integral_constant<int, 1>{});
    else
      run(std::integral_constant<int, 0>{});
  } else {
    // ------------------------------------------------------------ epilogue
    const int quad = warp & 3;
    int it = 0;
    for (int u = blockIdx.x; u < num_units; u += gridDim.x, ++it) {
      int tt, nt, sp;
      decode_unit(u, tt, nt, sp);
      const int acc = C::NACC == 2 ? (it & 1) : 0;
      const uint32_t acc_ph = C::NACC == 2 ? (uint32_t)((it >> 1) & 1) : (uint32_t)(it & 1);
      const bool got = q4_wait(a.spin, &acc_full[acc], acc_ph);
      if (!__all_sync(0xffffffffu, got)) {
        if (lane == 0) fail(66);
        break;
      }
      tc_fence_after();
      const int n = nt * WT + quad * 32 + lane;
      const uint32_t tbase = tmem_base + ((uint32_t)(quad * 32) << 16) + (uint32_t)(acc * TT);
#pragma unroll 1
      for (int c = 0; c < TT; c += 32) {
        float v[32];
        tmem_ld32(tbase + c, v);
        const int t0 = tt * TT + c;
        if (n < a.N) {
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const int t = t0 + j;
            if (t >= a.M) continue;
            if (EPI == 4) {
              a.partial[((int64_t)sp * a.M + t) * a.N + n] = v[j];
            } else {
              float o = v[j];
              if (EPI == 2) o += __bfloat162float(a.res[(int64_t)t * a.ldr + n]);
              a.out[(int64_t)t * a.ldc + n] = __float2bfloat16(o);
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[acc]);
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem_base, C::TMEM_COLS);
}

// Sum split-K partials [splits, M, N] -> bf16 Y (+ residual).
__global__ void q4k_reduce_kernel(const float* __restrict__ partial, int splits, int M, int N, bf16* __restrict__ out,
                                  int64_t ldc, const bf16* __restrict__ res, int64_t ldr) {
  griddep_entry();
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (int64_t)M * N) return;
  float acc = 0.f;
  for (int s = 0; s < splits; ++s) acc += partial[(int64_t)s * M * N + i];
  const int t = (int)(i / N), n = (int)(i % N);
  if (res) acc += __bfloat162float(res[(int64_t)t * ldr + n]);
  out[(int64_t)t * ldc + n] = __float2bfloat16(acc);
}

// ------------------------------------------------------------------ quantize
// One warp per super-block, lane = position inside each 32-weight sub-block.
// Same rounding steps as the Python reference quantizer (loaders.gguf.quantize_q4_k).
__global__ void q4k_quantize_kernel(const bf16* __restrict__ x, int64_t nblocks, uint8_t* __restrict__ out) {
  griddep_entry();
  const int64_t b = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (b >= nblocks) return;
  const bf16* xb = x + b * QK;
  float v[8], scales[8], mins[8];
  float smax = 0.f, mmax = 0.f;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    v[j] = __bfloat162float(xb[j * 32 + lane]);
    const float lo = fminf(warp_min(v[j]), 0.f);
    const float hi = warp_max(v[j]);
    mins[j] = -lo;
    scales[j] = (hi - lo) / 15.f;
    smax = j == 0 ? scales[j] : fmaxf(smax, scales[j]);
    mmax = j == 0 ? mins[j] : fmaxf(mmax, mins[j]);
  }
  const float d = smax / 63.f, dmin = mmax / 63.f;
  const __half d16 = __float2half_rn(d), dm16 = __float2half_rn(dmin);
  const float d16f = __half2float(d16), dm16f = __half2float(dm16);
  const float dq = d16f > 0.f ? d16f : 1.f, dmq = dm16f > 0.f ? dm16f : 1.f;
  int sc[8], mn[8];
  uint32_t q[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    sc[j] = (int)fminf(fmaxf(rintf(scales[j] / dq), 0.f), 63.f);
    mn[j] = (int)fminf(fmaxf(rintf(mins[j] / dmq), 0.f), 63.f);
    const float es = d16f * (float)sc[j];
    const float em = dm16f * (float)mn[j];
    float qq = es > 0.f ? rintf((v[j] + em) / es) : 0.f;
    q[j] = (uint32_t)fminf(fmaxf(qq, 0.f), 15.f);
  }
  uint8_t* o = out + b * QB;
  if (lane == 0) {
    const unsigned short db = __half_as_ushort(d16), mb = __half_as_ushort(dm16);
    o[0] = db & 0xFF;
    o[1] = db >> 8;
    o[2] = mb & 0xFF;
    o[3] = mb >> 8;
    for (int j = 0; j < 4; ++j) {
      o[4 + j] = (uint8_t)((sc[j] & 63) | ((sc[j + 4] >> 4) << 6));
      o[8 + j] = (uint8_t)((mn[j] & 63) | ((mn[j + 4] >> 4) << 6));
      o[12 + j] = (uint8_t)((sc[j + 4] & 0xF) | ((mn[j + 4] & 0xF) << 4));
    }
  }
#pragma unroll
  for (int c = 0; c < 4; ++c) o[16 + 32 * c + lane] = (uint8_t)(q[2 * c] | (q[2 * c + 1] << 4));
}

// Dequantize to bf16 (fp32 math), one thread per 32-weight sub-block row segment.
__global__ void q4k_dequant_kernel(const uint8_t* __restrict__ raw, int64_t nblocks, bf16* __restrict__ out) {
  griddep_entry();
  const int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;  // one per (block, sub-block)
  if (g >= nblocks * 8) return;
  const int64_t b = g >> 3;
  const int j = (int)(g & 7);
  const uint8_t* blk = raw + b * QB;
  const float d = half_bits_to_float(blk[0] | (blk[1] << 8));
  const float dmin = half_bits_to_float(blk[2] | (blk[3] << 8));
  int sc, mn;
  scale_min(blk + 4, j, sc, mn);
  const float ds = __fmul_rn(d, (float)sc), dm = __fmul_rn(dmin, (float)mn);
  const uint8_t* qs = blk + 16 + 32 * (j >> 1);
  bf16* o = out + b * QK + j * 32;
  for (int l = 0; l < 32; ++l) {
    const int qv = (j & 1) ? (qs[l] >> 4) : (qs[l] & 0xF);
    o[l] = __float2bfloat16(__fsub_rn(__fmul_rn(ds, (float)qv), dm));
  }
}

// Whole-matrix dequant for large-M products (the bf16 tcgen05 GEMM then runs at
// its full rate; the fused kernel re-dequantizes every weight tile once per
// 256-token tile).  One warp per (weight row, super-block): lane l makes weights
// 8l..8l+7 from 8 consecutive quant bytes (low nibbles for the first 32 of each
// 64-weight group, high for the next 32) and stores them as one 16-byte piece, so a
// warp writes the 512-byte row segment in one coalesced store.  Same arithmetic
// as q4k_dequant_kernel (d*sc and dmin*m rounded to fp32, then q*ds - dm, no
// contraction), so both produce the same bf16 bits.  `tiled`: blocks in the GEMM's
// tile-major order [n/128][k/256][128][144].  `half` > 0 writes gate/up rows
// interleaved in 128-row blocks for the SwiGLU epilogue (row r of the first half
// to 256*(r/128) + r%128, row half + r to 256*(r/128) + 128 + r%128).
__global__ void q4k_dequant_rows_kernel(const uint8_t* __restrict__ raw, int n, int k, int tiled, int half,
                                        bf16* __restrict__ out, int64_t ldo) {
  griddep_entry();
  const int nsb = k / QK;
  const int64_t wid = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (wid >= (int64_t)n * nsb) return;
  const int row = (int)(wid / nsb), sb = (int)(wid % nsb);
  const uint8_t* blk = tiled ? raw + (((int64_t)(row >> 7) * nsb + sb) * 128 + (row & 127)) * QB
                             : raw + ((int64_t)row * nsb + sb) * QB;
  const int j = lane >> 2;  // sub-block of weights 8l..8l+7
  const float d = half_bits_to_float(blk[0] | (blk[1] << 8));
  const float dmin = half_bits_to_float(blk[2] | (blk[3] << 8));
  int sc, mn;
  scale_min(blk + 4, j, sc, mn);
  const float ds = __fmul_rn(d, (float)sc), dm = __fmul_rn(dmin, (float)mn);
  const int g = lane >> 3, m8 = lane & 7;
  const uint2 q = *reinterpret_cast<const uint2*>(blk + 16 + 32 * g + 8 * (m8 & 3));
  const int shift = (m8 & 4) ? 4 : 0;
  uint32_t w[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint32_t word = i < 2 ? q.x : q.y;
    const int b0 = (2 * i) & 3;
    const int q0 = (word >> (8 * b0 + shift)) & 0xF, q1 = (word >> (8 * (b0 + 1) + shift)) & 0xF;
    const bf16 v0 = __float2bfloat16(__fsub_rn(__fmul_rn(ds, (float)q0), dm));
    const bf16 v1 = __float2bfloat16(__fsub_rn(__fmul_rn(ds, (float)q1), dm));
    w[i] = (uint32_t)__bfloat16_as_ushort(v0) | ((uint32_t)__bfloat16_as_ushort(v1) << 16);
  }
  int orow = row;
  if (half > 0) orow = row < half ? 256 * (row >> 7) + (row & 127) : 256 * ((row - half) >> 7) + 128 + ((row - half) & 127);
  *reinterpret_cast<uint4*>(out + (int64_t)orow * ldo + (int64_t)sb * QK + 8 * lane) = make_uint4(w[0], w[1], w[2], w[3]);
}

template <int TT, int EPI>
void launch_cfg(const CUtensorMap& tw, const CUtensorMap& tx, const Q4Args& a, int grid, int* err, cudaStream_t st) {
  auto kern = gemm_q4k_kernel<TT, EPI>;
  constexpr size_t smem = Cfg<TT>::SMEM;
  static std::atomic<uint64_t> attr_devs{0};
  ensure_smem_attr(attr_devs, kern, smem);
  launch_k(kern, grid, kThreads, smem, st, tw, tx, a, err);
  KAPSL_LAUNCH_CHECK();
  note_launch();
}

}  // namespace q4k

void launch_gemm_q4k(const __nv_bfloat16* X, int64_t ldx, const uint8_t* Wq, int64_t w_pitch, __nv_bfloat16* Y,
                     int64_t ldy, int M, int N, int K, const __nv_bfloat16* res, int64_t ldr, float* workspace,
                     size_t workspace_bytes, int force_splits, bool tiled, int* err, cudaStream_t st) {
  using namespace q4k;
  if (M == 0 || N == 0) return;
  if (K % QK != 0) throw std::runtime_error("gemm_q4k: K must be a multiple of 256");
  if (w_pitch != (int64_t)(K / QK) * QB) throw std::runtime_error("gemm_q4k: weight rows must be packed Q4_K blocks");
  if (ldx % 8 != 0) throw std::runtime_error("gemm_q4k: ldx must be a multiple of 8");
  const int sms = gemm_num_sms();
  const int TT = M <= 64 ? 64 : (M <= 128 ? 128 : 256);
  const int n_tiles = (N + WT - 1) / WT, t_tiles = (M + TT - 1) / TT;
  const int nsb = K / QK;
  const int tiles = n_tiles * t_tiles;
  int splits = force_splits > 0 ? force_splits : 1;
  if (force_splits <= 0 && tiles < sms / 2) splits = std::max(1, std::min(std::min(sms / tiles, nsb / 2), 16));
  if (splits > nsb) splits = nsb;
  if (splits > 1) {
    const int sps = (nsb + splits - 1) / splits;
    splits = (nsb + sps - 1) / sps;
  }
  if (splits > 1 && (workspace == nullptr || (size_t)splits * M * N * sizeof(float) > workspace_bytes))
    splits = 1;
  if (tiled && (N % WT != 0 || (reinterpret_cast<uintptr_t>(Wq) & 15) != 0))
    throw std::runtime_error("gemm_q4k: tile-contiguous weights need N % 128 == 0 and a 16-byte aligned base");
  CUtensorMap tw = make_tmap_2d_u8(Wq, N, (uint64_t)w_pitch, (uint64_t)w_pitch, WT, QB);
  CUtensorMap tx = make_tmap_2d_bf16(X, M, K, ldx, TT, BK);
  static const int spin = [] {
    const char* v = std::getenv("KAPSL_Q4K_SPIN");
    return (v != nullptr && v[0] == '1') ? 1 : 0;
  }();
  Q4Args a{Y, ldy, res, ldr, workspace, tiled ? Wq : nullptr, M, N, K, splits, spin};
  const int grid = std::min(tiles * splits, sms);
  const int epi = splits > 1 ? 4 : (res ? 2 : 0);
#define KAPSL_Q4_DISPATCH(TTV)                                            \
  switch (epi) {                                                          \
    case 0: launch_cfg<TTV, 0>(tw, tx, a, grid, err, st); break;          \
    case 2: launch_cfg<TTV, 2>(tw, tx, a, grid, err, st); break;          \
    default: launch_cfg<TTV, 4>(tw, tx, a, grid, err, st); break;         \
  }
  if (TT == 64) {
    KAPSL_Q4_DISPATCH(64)
  } else if (TT == 128) {
    KAPSL_Q4_DISPATCH(128)
  } else {
    KAPSL_Q4_DISPATCH(256)
  }
#undef KAPSL_Q4_DISPATCH
  if (splits > 1) {
    const int64_t total = (int64_t)M * N;
    launch_k(q4k_reduce_kernel, (unsigned)((total + 255) / 256), 256, 0, st, workspace, splits, M, N, Y, ldy, res, ldr);
    KAPSL_LAUNCH_CHECK();
    note_launch();
  }
}

void launch_q4k_quantize(const __nv_bfloat16* x, int64_t n, uint8_t* out, cudaStream_t st) {
  if (n % q4k::QK != 0) throw std::runtime_error("q4k_quantize: size must be a multiple of 256");
  const int64_t nb = n / q4k::QK;
  if (nb == 0) return;
  launch_k(q4k::q4k_quantize_kernel, (unsigned)((nb * 32 + 255) / 256), 256, 0, st, x, nb, out);
  KAPSL_LAUNCH_CHECK();
  note_launch();
}

void launch_q4k_dequant_rows(const uint8_t* raw, int n, int k, bool tiled, int half, __nv_bfloat16* out, int64_t ldo,
                             cudaStream_t st) {
  if (k % q4k::QK != 0 || (tiled && n % 128 != 0) || ldo % 8 != 0)
    throw std::runtime_error("q4k_dequant_rows: k % 256, n % 128 (tiled) and ldo % 8 must be 0");
  if (half > 0 && (half % 128 != 0 || 2 * half != n)) throw std::runtime_error("q4k_dequant_rows: bad gate/up split");
  const int64_t warps = (int64_t)n * (k / q4k::QK);
  if (warps == 0) return;
  launch_k(q4k::q4k_dequant_rows_kernel, (unsigned)((warps + 7) / 8), 256, 0, st, raw, n, k, tiled ? 1 : 0, half, out,
           ldo);
  KAPSL_LAUNCH_CHECK();
  note_launch();
}

void launch_q4k_dequant(const uint8_t* raw, int64_t n, __nv_bfloat16* out, cudaStream_t st) {
  if (n % q4k::QK != 0) throw std::runtime_error("q4k_dequant: size must be a multiple of 256");
  const int64_t nb = n / q4k::QK;
  if (nb == 0) return;
  launch_k(q4k::q4k_dequant_kernel, (unsigned)((nb * 8 + 255) / 256), 256, 0, st, raw, nb, out);
  KAPSL_LAUNCH_CHECK();
  note_launch();
}

}  // namespace kapsl
