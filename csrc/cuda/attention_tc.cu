// Chunked-prefill attention on the 5th-generation tensor cores (tcgen05 + TMEM).
//
// One CTA per (query work item, KV head).  A work item is up to floor(128 / g)
// query tokens of one sequence's prefill chunk, g = Hq / Hkv; their g query
// heads that share the KV head are packed into the 128 MMA rows (row r ->
// token r / g, head r % g), so each K/V tile is fetched once for the whole
// head group.  Per 128-key tile:
//
//   S = Q K^T      tcgen05.mma  (Q and K tiles K-major, 128B swizzle)  -> TMEM S[j % 2]
//   softmax        8 warps, one row per thread, two passes over S in TMEM;
//                  P (bf16) written to shared memory in the K-major layout
//   O_j = P V      tcgen05.mma  (P K-major, V used MN-major)            -> TMEM O
//   o = o * c + O_j in registers (each warpgroup keeps 64 of the 128 columns)
//
// Warp roles: warp 0 issues TMA loads (Q once, K/V into a 2-stage ring),
// warp 1 allocates TMEM and issues the MMAs (one elected thread), warps 2-9
// run the softmax, the rescaled accumulation and the epilogue.  S is double
// buffered in TMEM so the next tile's Q K^T runs while this tile's softmax
// runs.  Every wait is bounded (2 s); a timeout sets err and the CTA leaves.
//
// Checked against the fp32 attention oracle on three head layouts and serves
// chunked prefill by default (the mma.sync kernel in attention.cu remains
// selectable); 228-282 TFLOP/s on 2048- and 8192-token chunks, limited by the
// serial schedule between the two MMAs of a tile rather than the tensor cores.
#include "common.cuh"
#include "tcgen05.cuh"

namespace kapsl {
using namespace tc;

namespace {

constexpr int kD = 128;        // head dim
constexpr int kRows = 128;     // MMA rows per CTA
constexpr int kKeys = 128;     // keys per tile
constexpr int kPage = 16;      // tokens per KV page
constexpr uint32_t kHalfBytes = kRows * 64 * 2;  // 128 rows x 64 bf16 = 16 KiB
constexpr uint32_t kTileBytes = 2 * kHalfBytes;  // 32 KiB
constexpr int kSoftWarps = 8;
constexpr int kThreads = (2 + kSoftWarps) * 32;
constexpr uint32_t kTmemCols = 512;  // S0 [0,128) S1 [128,256) O [256,384)

struct alignas(1024) TcSmem {
  uint8_t q[kTileBytes];
  uint8_t k[2][kTileBytes];
  uint8_t v[2][kTileBytes];
  uint8_t p[kTileBytes];
  uint64_t q_full, kv_full[2], kv_empty[2], s_full[2], s_free[2], p_full, o_full;
  uint32_t tmem_base;
  int abort_flag;
};

// MN-major operand with 128-byte swizzle: 64-element rows of 128 B along MN,
// 8 rows (8 K indices) per 1 KiB atom; `lbo` steps between 64-wide MN groups,
// `sbo` between 8-row K groups.
__device__ __forceinline__ uint64_t smem_desc_sw128_mn(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFF);
  d |= (uint64_t)((lbo >> 4) & 0x3FFF) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFF) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}

__device__ __forceinline__ void tma_load_3d(void* smem_dst, const CUtensorMap* m, uint64_t* bar, int32_t x,
                                            int32_t y, int32_t z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z)
      : "memory");
}

__device__ __forceinline__ bool wait_or_abort(TcSmem& s, uint64_t* bar, uint32_t parity, int* err, int code) {
  if (mbar_wait_sleep(bar, parity)) return true;
  if (err) atomicCAS(err, 0, code);
  s.abort_flag = 1;
  return false;
}

}  // namespace

// q_map: 3-D (D, Hq, T) over q [T, Hq * D]; k_map / v_map: 2-D (D, blocks * Hkv * 16) over a
// layer's caches [blocks, Hkv, 16, D].  work: [nwork, 2] = (prefill sequence, first token in the
// chunk); seq_info: [S, 4] = (first q row, chunk tokens n, context length after the chunk,
// block-table row).  out: [T, Hq * D].
__global__ void __launch_bounds__(kThreads, 1)
    prefill_attn_tc_kernel(const __grid_constant__ CUtensorMap q_map, const __grid_constant__ CUtensorMap k_map,
                           const __grid_constant__ CUtensorMap v_map, const int32_t* __restrict__ work,
                           const int32_t* __restrict__ seq_info, const int32_t* __restrict__ block_tables,
                           int max_blocks, int Hq, int Hkv, float scale_log2, __nv_bfloat16* __restrict__ out,
                           int64_t out_stride, int* err) {
  griddep_entry();
  extern __shared__ uint8_t smem_raw[];
  TcSmem& s = *reinterpret_cast<TcSmem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int g = Hq / Hkv;
  const int tpc = kRows / g;  // tokens per CTA
  const int kvh = blockIdx.y;
  const int sj = work[2 * blockIdx.x], t0 = work[2 * blockIdx.x + 1];
  const int row0 = seq_info[4 * sj], n = seq_info[4 * sj + 1], ctx = seq_info[4 * sj + 2];
  const int bt_row = seq_info[4 * sj + 3];
  const int ntok = min(tpc, n - t0);
  const int q_last = ctx - n + t0 + ntok - 1;  // position of the last valid query
  const int ntiles = (q_last + kKeys) / kKeys;
  const int32_t* bt = block_tables + (int64_t)bt_row * max_blocks;
  const int npages = (ctx + kPage - 1) / kPage;

  if (threadIdx.x == 0) {
    s.abort_flag = 0;
    mbar_init(&s.q_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s.kv_full[i], 1);
      mbar_init(&s.kv_empty[i], 1);
      mbar_init(&s.s_full[i], 1);
      mbar_init(&s.s_free[i], kSoftWarps * 32);
    }
    mbar_init(&s.p_full, kSoftWarps * 32);
    mbar_init(&s.o_full, 1);
    fence_barrier_init();
  }
  // rows of the Q tile that no token fills stay zero (their scores are finite)
  for (uint32_t i = threadIdx.x; i < kTileBytes / 16; i += kThreads) {
    const uint32_t half = i / (kHalfBytes / 16), rem = i % (kHalfBytes / 16);
    if (rem * 16 / 128 >= (uint32_t)(g * tpc)) reinterpret_cast<uint4*>(s.q + half * kHalfBytes)[rem] = make_uint4(0, 0, 0, 0);
  }
  if (warp == 1) tmem_alloc(&s.tmem_base, kTmemCols);
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s.tmem_base;

  if (warp == 0) {
    // ---------------------------------------------------------------- TMA producer
    if (lane == 0) {
      mbar_arrive_expect_tx(&s.q_full, 2u * (uint32_t)(g * tpc) * 128u);
      for (int h = 0; h < 2; ++h) tma_load_3d(s.q + h * kHalfBytes, &q_map, &s.q_full, h * 64, kvh * g, row0 + t0);
      for (int j = 0; j < ntiles && !s.abort_flag; ++j) {
        const int st = j & 1;
        if (j >= 2 && !wait_or_abort(s, &s.kv_empty[st], ((j >> 1) - 1) & 1, err, 71)) break;
        mbar_arrive_expect_tx(&s.kv_full[st], 2u * kTileBytes);
        for (int pg = 0; pg < kKeys / kPage; ++pg) {
          const int page = j * (kKeys / kPage) + pg;
          const int blk = bt[page < npages ? page : 0];
          const int y = (blk * Hkv + kvh) * kPage;
          for (int h = 0; h < 2; ++h) {
            tma_load_2d(s.k[st] + h * kHalfBytes + pg * kPage * 128, &k_map, &s.kv_full[st], h * 64, y);
            tma_load_2d(s.v[st] + h * kHalfBytes + pg * kPage * 128, &v_map, &s.kv_full[st], h * 64, y);
          }
        }
      }
    }
  } else if (warp == 1) {
    // ----------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      const uint32_t idesc_s = idesc_bf16<kRows, kKeys>();
      const uint32_t idesc_o = idesc_bf16<kRows, kD>() | (1u << 16);  // B (V) MN-major
      const uint32_t q_addr = smem_u32(s.q), p_addr = smem_u32(s.p);
      auto issue_s = [&](int j) -> bool {
        const int st = j & 1;
        if (!wait_or_abort(s, &s.kv_full[st], (j >> 1) & 1, err, 72)) return false;
        if (j >= 2 && !wait_or_abort(s, &s.s_free[st], ((j >> 1) - 1) & 1, err, 73)) return false;
        tc_fence_after();
        const uint32_t k_addr = smem_u32(s.k[st]);
        for (int kk = 0; kk < kD / 16; ++kk) {
          const uint32_t off = (kk >> 2) * kHalfBytes + (kk & 3) * 32;
          mma_bf16(tmem + st * kKeys, smem_desc_sw128(q_addr + off), smem_desc_sw128(k_addr + off), idesc_s,
                   kk > 0);
        }
        mma_commit(&s.s_full[st]);
        return true;
      };
      bool ok = wait_or_abort(s, &s.q_full, 0, err, 74) && issue_s(0);
      for (int j = 0; ok && j < ntiles; ++j) {
        if (j + 1 < ntiles && !issue_s(j + 1)) break;
        if (!wait_or_abort(s, &s.p_full, j & 1, err, 75)) break;
        tc_fence_after();
        const uint32_t v_addr = smem_u32(s.v[j & 1]);
        for (int kk = 0; kk < kKeys / 16; ++kk) {
          const uint64_t a = smem_desc_sw128(p_addr + (kk >> 2) * kHalfBytes + (kk & 3) * 32);
          const uint64_t b = smem_desc_sw128_mn(v_addr + kk * 16 * 128, kHalfBytes, 1024);
          mma_bf16(tmem + 2 * kKeys, a, b, idesc_o, kk > 0);
        }
        mma_commit(&s.o_full);
        mma_commit(&s.kv_empty[j & 1]);
      }
    }
  } else {
    // ------------------------------------------- softmax, accumulation, epilogue
    const int quad = warp & 3;                 // TMEM lane quadrant of this warp
    const int half = (warp - 2) / 4;           // 0: O columns 0-63 and P keys 0-63; 1: the rest
    const int r = quad * 32 + lane;            // MMA row
    const int tok = r / g, head = r % g;
    const int qpos = ctx - n + t0 + tok;
    const uint32_t lane_off = (uint32_t)(quad * 32) << 16;
    float o[64];
#pragma unroll
    for (int i = 0; i < 64; ++i) o[i] = 0.f;
    float m = -INFINITY, l = 0.f, corr_prev = 0.f;
    bool ok = true;
    for (int j = 0; j < ntiles; ++j) {
      const int st = j & 1;
      if (!wait_or_abort(s, &s.s_full[st], (j >> 1) & 1, err, 76)) { ok = false; break; }
      tc_fence_after();
      const uint32_t s_tmem = tmem + lane_off + st * kKeys;
      // pass 1: row max of the scaled, masked scores
      float mx = -INFINITY;
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        float v[32];
        tmem_ld32(s_tmem + c * 32, v);
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const int kpos = j * kKeys + c * 32 + i;
          const float x = (kpos > qpos || kpos >= ctx) ? -INFINITY : v[i] * scale_log2;
          mx = fmaxf(mx, x);
        }
      }
      const float m_new = fmaxf(m, mx);
      const float corr = exp2f(m - m_new);  // 0 on the first tile (m = -inf)
      // the previous tile's P.V is done: fold it into o (it also frees P)
      if (j > 0) {
        if (!wait_or_abort(s, &s.o_full, (j - 1) & 1, err, 77)) { ok = false; break; }
        tc_fence_after();
        const uint32_t o_tmem = tmem + lane_off + 2 * kKeys + half * 64;
        float ov[32];
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          tmem_ld32(o_tmem + c * 32, ov);
#pragma unroll
          for (int i = 0; i < 32; ++i) o[c * 32 + i] = o[c * 32 + i] * corr_prev + ov[i];
        }
      }
      // pass 2: probabilities, row sum, this warpgroup's half of P
      float sum = 0.f;
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        float v[32];
        tmem_ld32(s_tmem + c * 32, v);
        uint32_t packed[16];
#pragma unroll
        for (int i = 0; i < 32; i += 2) {
          const int kpos = j * kKeys + c * 32 + i;
          const float x0 = (kpos > qpos || kpos >= ctx) ? -INFINITY : v[i] * scale_log2;
          const float x1 = (kpos + 1 > qpos || kpos + 1 >= ctx) ? -INFINITY : v[i + 1] * scale_log2;
          const float p0 = exp2f(x0 - m_new), p1 = exp2f(x1 - m_new);
          sum += p0 + p1;
          packed[i / 2] = pack_bf16(p0, p1);
        }
        if ((c >> 1) == half) {  // keys [64 * half, 64 * half + 64): row r, 16-byte chunks 4 * (c & 1) ..
          uint8_t* prow = s.p + half * kHalfBytes;
#pragma unroll
          for (int q4 = 0; q4 < 4; ++q4) {
            const uint32_t chunk = (c & 1) * 4 + q4;
            *reinterpret_cast<uint4*>(prow + sw128_offset(r, chunk)) =
                make_uint4(packed[4 * q4], packed[4 * q4 + 1], packed[4 * q4 + 2], packed[4 * q4 + 3]);
          }
        }
      }
      l = l * corr + sum;
      m = m_new;
      corr_prev = corr;
      fence_proxy_async_smem();  // P written by threads, read by tcgen05.mma
      tc_fence_before();
      mbar_arrive(&s.p_full);
      mbar_arrive(&s.s_free[st]);
    }
    if (ok && ntiles > 0 && wait_or_abort(s, &s.o_full, (ntiles - 1) & 1, err, 78)) {
      tc_fence_after();
      const uint32_t o_tmem = tmem + lane_off + 2 * kKeys + half * 64;
      float ov[32];
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        tmem_ld32(o_tmem + c * 32, ov);
#pragma unroll
        for (int i = 0; i < 32; ++i) o[c * 32 + i] = o[c * 32 + i] * corr_prev + ov[i];
      }
      if (tok < ntok) {
        const float inv = l > 0.f ? 1.f / l : 0.f;
        __nv_bfloat16* dst = out + (int64_t)(row0 + t0 + tok) * out_stride + (int64_t)(kvh * g + head) * kD + half * 64;
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          uint4 w;
          w.x = pack_bf16(o[8 * c + 0] * inv, o[8 * c + 1] * inv);
          w.y = pack_bf16(o[8 * c + 2] * inv, o[8 * c + 3] * inv);
          w.z = pack_bf16(o[8 * c + 4] * inv, o[8 * c + 5] * inv);
          w.w = pack_bf16(o[8 * c + 6] * inv, o[8 * c + 7] * inv);
          *reinterpret_cast<uint4*>(dst + 8 * c) = w;
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

size_t prefill_attn_tc_smem_bytes() { return sizeof(TcSmem) + 1024; }

// Work items for the tensor-core kernel: tiles of floor(128 / g) tokens per prefill sequence.
int prefill_attn_tc_tokens_per_cta(int Hq, int Hkv) { return kRows / (Hq / Hkv); }

void launch_prefill_attention_tc(const CUtensorMap& q_map, const CUtensorMap& k_map, const CUtensorMap& v_map,
                                 const int32_t* work, int nwork, const int32_t* seq_info,
                                 const int32_t* block_tables, int max_blocks, int Hq, int Hkv, float scale,
                                 __nv_bfloat16* out, int64_t out_stride, int* err, cudaStream_t st) {
  if (Hq % Hkv != 0 || Hq / Hkv > kRows) throw std::runtime_error("prefill attention (tc): bad head grouping");
  if (nwork <= 0) return;
  const size_t smem = prefill_attn_tc_smem_bytes();
  static std::atomic<uint64_t> attr_devs{0};
  ensure_smem_attr(attr_devs, prefill_attn_tc_kernel, smem);
  const float scale_log2 = scale * 1.4426950408889634f;
  launch_k(prefill_attn_tc_kernel, dim3(nwork, Hkv), kThreads, smem, st, q_map, k_map, v_map, work, seq_info,
                                                                   block_tables, max_blocks, Hq, Hkv, scale_log2,
                                                                   out, out_stride, err);
  KAPSL_LAUNCH_CHECK();
  note_launch();
}

}  // namespace kapsl
