// Paged attention for sm_100a over a block table (block size 16, head_dim 128).
//
// KV cache layout (per layer): [num_blocks, Hkv, 16, 128] bf16 for K and for V.
// One (block, kv-head) page is a contiguous 4 KiB row group, loaded by TMA as two
// 16x64 boxes with 128-byte swizzle, so the ldmatrix fragment reads are bank-
// conflict free.  Softmax runs in the log2 domain in fp32.
//
//  * decode: split-KV flash decoding.  One CTA per (split, kv head, sequence);
//    all query heads of the GQA group share each K/V page (rows of the MMA A
//    operand are the group's heads), 4 warps stream disjoint pages through
//    per-warp TMA pipelines and merge at the end.  Splits are merged by
//    `combine_kernel` through an fp32 scratch buffer.
//  * prefill (chunked): one CTA per (64-query tile, q head); causal mask with
//    the chunk's offset into the existing context, K/V tiles of 64 tokens
//    (4 pages) through a 3-stage TMA pipeline shared by 4 warps.
//
// Reference counterparts: CpuAttention::flash_attention_v2 and
// paged_attention_v1 (crates/kapsl-kernels/src/attention/mod.rs:8-99), which
// have no block table; the reference engine instead gathers paged KV into
// contiguous arrays on the host every step (crates/kapsl-llm/src/kv_cache.rs:1543-1617).
#include "common.cuh"
#include "kernels.h"

namespace kapsl {

using bf16 = __nv_bfloat16;

static constexpr int kD = 128;
static constexpr int kBS = 16;
static constexpr float kLog2e = 1.4426950408889634f;

// smem bytes of one K (or V) page: two 16x64 swizzled halves.
static constexpr int kPageBytes = kBS * kD * 2;  // 4096

__device__ __forceinline__ float fast_exp2(float x) { return exp2f(x); }

// Address (shared space) of the 16-byte chunk `chunk` (0..15, i.e. dims
// chunk*8..chunk*8+7) of token row `tok` (0..15) in a page.
__device__ __forceinline__ uint32_t page_chunk_addr(uint32_t page_base, int tok, int chunk) {
  return page_base + (uint32_t)(chunk >> 3) * 2048u + sw128_offset(tok, chunk & 7);
}

// =========================================================== decode kernel
template <int NWARPS, int STAGES>
__global__ void __launch_bounds__(NWARPS * 32)
    decode_attn_kernel(const __grid_constant__ CUtensorMap tmap_k, const __grid_constant__ CUtensorMap tmap_v,
                       const bf16* __restrict__ q, int64_t q_stride, const int32_t* __restrict__ block_tables,
                       int max_blocks, const int32_t* __restrict__ ctx_lens, bf16* __restrict__ out,
                       int64_t out_stride, float* __restrict__ part_o, float* __restrict__ part_lse, int Hq,
                       int Hkv, float scale_log2, int* __restrict__ err) {
  griddep_entry();
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // 1024-byte align the dynamic smem base (required by the 128B swizzle).
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ __align__(8) uint64_t full_bar[NWARPS][STAGES];
  __shared__ float m_sh[NWARPS][16];
  __shared__ float l_sh[NWARPS][16];

  const int split = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
  const int nsplit = gridDim.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int group = Hq / Hkv;
  const int ctx = ctx_lens[b];
  const int nblk = (ctx + kBS - 1) / kBS;
  const int per_split = (nblk + nsplit - 1) / nsplit;
  const int blk_begin = split * per_split;
  const int blk_end = min(nblk, blk_begin + per_split);
  const int32_t* bt = block_tables + (int64_t)b * max_blocks;

  uint8_t* wsm = smem + (size_t)warp * STAGES * 2 * kPageBytes;
  if (lane == 0) {
    for (int s = 0; s < STAGES; ++s) mbar_init(&full_bar[warp][s], 1);
    fence_barrier_init();
  }
  __syncwarp();

  // Blocks handled by this warp: blk_begin + warp + i*NWARPS.
  const int my_first = blk_begin + warp;
  const int n_local = (blk_end > my_first) ? (blk_end - my_first + NWARPS - 1) / NWARPS : 0;

  auto issue = [&](int i) {
    const int s = i % STAGES;
    const int j = my_first + i * NWARPS;
    const int phys = bt[j];
    const int row = (phys * Hkv + kvh) * kBS;
    uint8_t* kdst = wsm + (size_t)s * 2 * kPageBytes;
    uint8_t* vdst = kdst + kPageBytes;
    mbar_arrive_expect_tx(&full_bar[warp][s], 2 * kPageBytes);
    tma_load_2d(kdst, &tmap_k, &full_bar[warp][s], 0, row);
    tma_load_2d(kdst + 2048, &tmap_k, &full_bar[warp][s], 64, row);
    tma_load_2d(vdst, &tmap_v, &full_bar[warp][s], 0, row);
    tma_load_2d(vdst + 2048, &tmap_v, &full_bar[warp][s], 64, row);
  };
  if (lane == 0) {
    for (int i = 0; i < STAGES && i < n_local; ++i) issue(i);
  }

  // Q fragments (A operand, rows = heads of the group, 16 rows max).
  const int r0 = lane >> 2;       // row (head) r0 and r0 + 8
  const int cq = (lane & 3) * 2;  // k offset inside a 16-wide k step
  uint32_t qa[8][4];
  {
    const int qh = kvh * group;
    const bf16* q0 = q + (int64_t)b * q_stride + (int64_t)(qh + r0) * kD;
    const bf16* q1 = q + (int64_t)b * q_stride + (int64_t)(qh + r0 + 8) * kD;
    const bool v0 = r0 < group, v1 = (r0 + 8) < group;
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
      qa[ks][0] = v0 ? *reinterpret_cast<const uint32_t*>(q0 + ks * 16 + cq) : 0u;
      qa[ks][1] = v1 ? *reinterpret_cast<const uint32_t*>(q1 + ks * 16 + cq) : 0u;
      qa[ks][2] = v0 ? *reinterpret_cast<const uint32_t*>(q0 + ks * 16 + cq + 8) : 0u;
      qa[ks][3] = v1 ? *reinterpret_cast<const uint32_t*>(q1 + ks * 16 + cq + 8) : 0u;
    }
  }

  float o[16][4];
#pragma unroll
  for (int i = 0; i < 16; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m_r[2] = {-INFINITY, -INFINITY};
  float l_r[2] = {0.f, 0.f};
  bool ok = true;

  for (int i = 0; i < n_local; ++i) {
    const int s = i % STAGES;
    const uint32_t parity = (uint32_t)((i / STAGES) & 1);
    const bool got = mbar_wait_bounded(&full_bar[warp][s], parity);
    if (!__all_sync(0xffffffffu, got)) {  // warp-uniform exit on timeout
      ok = false;
      break;
    }
    const int j = my_first + i * NWARPS;
    const int valid = min(kBS, ctx - j * kBS);
    const uint32_t kbase = smem_u32(wsm + (size_t)s * 2 * kPageBytes);
    const uint32_t vbase = kbase + kPageBytes;

    // S = Q K^T  (rows: heads, cols: 16 tokens as two n-tiles)
    float sc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
      uint32_t kb[4];
      const int mat = lane >> 3;
      const int tok = ((mat >> 1) << 3) + (lane & 7);
      const int chunk = ks * 2 + (mat & 1);
      ldmatrix_x4(kb, page_chunk_addr(kbase, tok, chunk));
      const uint32_t b0[2] = {kb[0], kb[1]};
      const uint32_t b1[2] = {kb[2], kb[3]};
      mma_bf16_16816(sc[0], qa[ks], b0);
      mma_bf16_16816(sc[1], qa[ks], b1);
    }
    // scale, mask, online softmax
    float mx[2] = {m_r[0], m_r[1]};
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int tok = nt * 8 + cq + (e & 1);
        float v = sc[nt][e] * scale_log2;
        if (tok >= valid) v = -INFINITY;
        sc[nt][e] = v;
        mx[e >> 1] = fmaxf(mx[e >> 1], v);
      }
    }
#pragma unroll
    for (int rr = 0; rr < 2; ++rr) {
      mx[rr] = fmaxf(mx[rr], __shfl_xor_sync(0xffffffffu, mx[rr], 1));
      mx[rr] = fmaxf(mx[rr], __shfl_xor_sync(0xffffffffu, mx[rr], 2));
    }
    float alpha[2];
#pragma unroll
    for (int rr = 0; rr < 2; ++rr) {
      alpha[rr] = (m_r[rr] == -INFINITY) ? 0.f : fast_exp2(m_r[rr] - mx[rr]);
      m_r[rr] = mx[rr];
      l_r[rr] *= alpha[rr];
    }
    float p[2][4];
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float mm = m_r[e >> 1];
        p[nt][e] = (mm == -INFINITY) ? 0.f : fast_exp2(sc[nt][e] - mm);
        l_r[e >> 1] += p[nt][e];
      }
#pragma unroll
    for (int nt = 0; nt < 16; ++nt) {
      o[nt][0] *= alpha[0];
      o[nt][1] *= alpha[0];
      o[nt][2] *= alpha[1];
      o[nt][3] *= alpha[1];
    }
    uint32_t pa[4];
    pa[0] = pack_bf16(p[0][0], p[0][1]);
    pa[1] = pack_bf16(p[0][2], p[0][3]);
    pa[2] = pack_bf16(p[1][0], p[1][1]);
    pa[3] = pack_bf16(p[1][2], p[1][3]);
    // O += P V
#pragma unroll
    for (int c = 0; c < 16; c += 2) {
      uint32_t vb[4];
      const int mat = lane >> 3;
      const int tok = ((mat & 1) << 3) + (lane & 7);
      const int chunk = c + (mat >> 1);
      ldmatrix_x4_trans(vb, page_chunk_addr(vbase, tok, chunk));
      const uint32_t b0[2] = {vb[0], vb[1]};
      const uint32_t b1[2] = {vb[2], vb[3]};
      mma_bf16_16816(o[c], pa, b0);
      mma_bf16_16816(o[c + 1], pa, b1);
    }
    __syncwarp();
    if (lane == 0 && i + STAGES < n_local) issue(i + STAGES);
  }
  if (!ok && lane == 0) atomicExch(err, 1);

  // quad-reduce the row sums
#pragma unroll
  for (int rr = 0; rr < 2; ++rr) {
    l_r[rr] += __shfl_xor_sync(0xffffffffu, l_r[rr], 1);
    l_r[rr] += __shfl_xor_sync(0xffffffffu, l_r[rr], 2);
  }
  __syncthreads();  // every warp is done with its pages: reuse them for the merge
  float* osh = reinterpret_cast<float*>(wsm);  // [16][128] fp32 = 8 KiB per warp
#pragma unroll
  for (int nt = 0; nt < 16; ++nt) {
    const int d = nt * 8 + cq;
    osh[r0 * kD + d] = o[nt][0];
    osh[r0 * kD + d + 1] = o[nt][1];
    osh[(r0 + 8) * kD + d] = o[nt][2];
    osh[(r0 + 8) * kD + d + 1] = o[nt][3];
  }
  if ((lane & 3) == 0) {
    m_sh[warp][r0] = m_r[0];
    m_sh[warp][r0 + 8] = m_r[1];
    l_sh[warp][r0] = l_r[0];
    l_sh[warp][r0 + 8] = l_r[1];
  }
  __syncthreads();
  const int qh0 = kvh * group;
  for (int idx = threadIdx.x; idx < group * kD; idx += NWARPS * 32) {
    const int g = idx / kD, d = idx % kD;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < NWARPS; ++w) M = fmaxf(M, m_sh[w][g]);
    float L = 0.f, acc = 0.f;
    if (M != -INFINITY) {
#pragma unroll
      for (int w = 0; w < NWARPS; ++w) {
        const float f = (m_sh[w][g] == -INFINITY) ? 0.f : fast_exp2(m_sh[w][g] - M);
        L += l_sh[w][g] * f;
        acc += reinterpret_cast<float*>(smem + (size_t)w * STAGES * 2 * kPageBytes)[g * kD + d] * f;
      }
    }
    const int head = qh0 + g;
    if (nsplit == 1) {
      out[(int64_t)b * out_stride + (int64_t)head * kD + d] = __float2bfloat16(L > 0.f ? acc / L : 0.f);
    } else {
      const int64_t pidx = (((int64_t)b * Hq + head) * nsplit + split);
      part_o[pidx * kD + d] = L > 0.f ? acc / L : 0.f;
      if (d == 0) part_lse[pidx] = (L > 0.f) ? (M + log2f(L)) : -INFINITY;
    }
  }
}

__global__ void combine_kernel(const float* __restrict__ part_o, const float* __restrict__ part_lse,
                               bf16* __restrict__ out, int64_t out_stride, int Hq, int nsplit) {
  griddep_entry();
  const int head = blockIdx.x, b = blockIdx.y, d = threadIdx.x;
  const int64_t base = ((int64_t)b * Hq + head) * nsplit;
  float M = -INFINITY;
  for (int s = 0; s < nsplit; ++s) M = fmaxf(M, part_lse[base + s]);
  float L = 0.f, acc = 0.f;
  if (M != -INFINITY) {
    for (int s = 0; s < nsplit; ++s) {
      const float lse = part_lse[base + s];
      const float w = (lse == -INFINITY) ? 0.f : exp2f(lse - M);
      L += w;
      acc += w * part_o[(base + s) * kD + d];
    }
  }
  out[(int64_t)b * out_stride + (int64_t)head * kD + d] = __float2bfloat16(L > 0.f ? acc / L : 0.f);
}

static constexpr int kDecWarps = 4;
static constexpr int kDecStages = 3;

size_t decode_attn_smem_bytes() { return (size_t)kDecWarps * kDecStages * 2 * kPageBytes + 1024; }

int decode_attn_num_splits(int B, int Hkv, int max_ctx, int num_sms) {
  const int ctas = B * Hkv;
  const int target = 2 * num_sms;
  if (ctas >= target) return 1;
  int s = (target + ctas - 1) / ctas;
  const int max_by_len = max(1, (max_ctx + 255) / 256);  // keep >= 256 tokens per split
  s = min(s, max_by_len);
  return max(1, min(s, 64));
}

void launch_decode_attention(const CUtensorMap& tk, const CUtensorMap& tv, const bf16* q, int64_t q_stride,
                             const int32_t* block_tables, int max_blocks, const int32_t* ctx_lens, bf16* out,
                             int64_t out_stride, float* part_o, float* part_lse, int B, int Hq, int Hkv,
                             int nsplit, float scale, int* err, cudaStream_t st) {
  if (B == 0) return;
  if (Hq % Hkv != 0 || Hq / Hkv > 16) throw std::runtime_error("decode attention: GQA group must be <= 16");
  if (nsplit > 1 && (part_o == nullptr || part_lse == nullptr))
    throw std::runtime_error("decode attention: split-KV needs scratch buffers");
  auto kern = decode_attn_kernel<kDecWarps, kDecStages>;
  const size_t smem = decode_attn_smem_bytes();
  static std::atomic<uint64_t> attr_devs{0};
  ensure_smem_attr(attr_devs, kern, smem);
  dim3 grid(nsplit, Hkv, B);
  launch_k(kern, grid, kDecWarps * 32, smem, st, tk, tv, q, q_stride, block_tables, max_blocks, ctx_lens, out,
                                           out_stride, part_o, part_lse, Hq, Hkv, scale * kLog2e, err);
  KAPSL_LAUNCH_CHECK();
  note_launch();
  if (nsplit > 1) {
    launch_k(combine_kernel, dim3(Hq, B), kD, 0, st, part_o, part_lse, out, out_stride, Hq, nsplit);
    KAPSL_LAUNCH_CHECK();
    note_launch();
  }
}

// ========================================================== prefill kernel
// work[i] = {seq index, first query row of the tile (relative to the seq)}.
// seq_info[s] = {q_start (row in q), q_len, ctx_len (KV length incl. chunk), bt_row}.
template <int STAGES>
__global__ void __launch_bounds__(128)
    prefill_attn_kernel(const __grid_constant__ CUtensorMap tmap_k, const __grid_constant__ CUtensorMap tmap_v,
                        const bf16* __restrict__ q, int64_t q_stride, const int32_t* __restrict__ work,
                        const int32_t* __restrict__ seq_info, const int32_t* __restrict__ block_tables,
                        int max_blocks, bf16* __restrict__ out, int64_t out_stride, int Hq, int Hkv,
                        float scale_log2, int* __restrict__ err) {
  griddep_entry();
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ __align__(8) uint64_t full_bar[STAGES];
  __shared__ int abort_sh;
  constexpr int kTile = 64;                      // KV tokens per stage (4 pages)
  constexpr int kStageBytes = 2 * 4 * kPageBytes;  // K and V, 4 pages each

  const int head = blockIdx.y;
  const int seq = work[blockIdx.x * 2 + 0];
  const int qt0 = work[blockIdx.x * 2 + 1];
  const int q_start = seq_info[seq * 4 + 0];
  const int q_len = seq_info[seq * 4 + 1];
  const int ctx = seq_info[seq * 4 + 2];
  const int bt_row = seq_info[seq * 4 + 3];
  const int32_t* bt = block_tables + (int64_t)bt_row * max_blocks;
  const int kvh = head / (Hq / Hkv);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nblk = (ctx + kBS - 1) / kBS;
  const int pos0 = ctx - q_len;  // position of the chunk's first token
  const int q_hi = min(q_len, qt0 + 64);
  const int kv_end = pos0 + q_hi;  // exclusive
  const int ntiles = (kv_end + kTile - 1) / kTile;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) mbar_init(&full_bar[s], 1);
    abort_sh = 0;
    fence_barrier_init();
  }
  __syncthreads();

  auto issue = [&](int t) {
    const int s = t % STAGES;
    uint8_t* kdst = smem + (size_t)s * kStageBytes;
    uint8_t* vdst = kdst + 4 * kPageBytes;
    mbar_arrive_expect_tx(&full_bar[s], kStageBytes);
#pragma unroll
    for (int pg = 0; pg < 4; ++pg) {
      const int j = t * 4 + pg;
      const int phys = (j < nblk) ? bt[j] : bt[0];
      const int row = (phys * Hkv + kvh) * kBS;
      tma_load_2d(kdst + pg * kPageBytes, &tmap_k, &full_bar[s], 0, row);
      tma_load_2d(kdst + pg * kPageBytes + 2048, &tmap_k, &full_bar[s], 64, row);
      tma_load_2d(vdst + pg * kPageBytes, &tmap_v, &full_bar[s], 0, row);
      tma_load_2d(vdst + pg * kPageBytes + 2048, &tmap_v, &full_bar[s], 64, row);
    }
  };
  if (threadIdx.x == 0)
    for (int t = 0; t < STAGES && t < ntiles; ++t) issue(t);

  const int r0 = lane >> 2, cq = (lane & 3) * 2;
  const int qrow0 = qt0 + warp * 16 + r0;  // query index within the sequence
  const int qrow1 = qrow0 + 8;
  uint32_t qa[8][4];
  {
    const bool v0 = qrow0 < q_len, v1 = qrow1 < q_len;
    const bf16* q0 = q + (int64_t)(q_start + (v0 ? qrow0 : 0)) * q_stride + (int64_t)head * kD;
    const bf16* q1 = q + (int64_t)(q_start + (v1 ? qrow1 : 0)) * q_stride + (int64_t)head * kD;
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
      qa[ks][0] = v0 ? *reinterpret_cast<const uint32_t*>(q0 + ks * 16 + cq) : 0u;
      qa[ks][1] = v1 ? *reinterpret_cast<const uint32_t*>(q1 + ks * 16 + cq) : 0u;
      qa[ks][2] = v0 ? *reinterpret_cast<const uint32_t*>(q0 + ks * 16 + cq + 8) : 0u;
      qa[ks][3] = v1 ? *reinterpret_cast<const uint32_t*>(q1 + ks * 16 + cq + 8) : 0u;
    }
  }
  const int qpos[2] = {pos0 + qrow0, pos0 + qrow1};
  const int warp_max_pos = pos0 + min(q_len - 1, qt0 + warp * 16 + 15);

  float o[16][4];
#pragma unroll
  for (int i = 0; i < 16; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m_r[2] = {-INFINITY, -INFINITY};
  float l_r[2] = {0.f, 0.f};
  bool ok = true;

  for (int t = 0; t < ntiles; ++t) {
    const int s = t % STAGES;
    const bool got = mbar_wait_bounded(&full_bar[s], (uint32_t)((t / STAGES) & 1));
    if (!got) abort_sh = 1;
    const int kv0 = t * kTile;
    if (got && kv0 <= warp_max_pos) {  // warp-uniform skip of fully-masked tiles
      const uint32_t kbase = smem_u32(smem + (size_t)s * kStageBytes);
      const uint32_t vbase = kbase + 4 * kPageBytes;
      float sc[8][4];
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) sc[nt][0] = sc[nt][1] = sc[nt][2] = sc[nt][3] = 0.f;
#pragma unroll
      for (int ks = 0; ks < 8; ++ks) {
#pragma unroll
        for (int np = 0; np < 4; ++np) {  // pairs of n-tiles = 16 tokens = one page
          uint32_t kb[4];
          const int mat = lane >> 3;
          const int tok = ((mat >> 1) << 3) + (lane & 7);
          const int chunk = ks * 2 + (mat & 1);
          ldmatrix_x4(kb, page_chunk_addr(kbase + np * kPageBytes, tok, chunk));
          const uint32_t b0[2] = {kb[0], kb[1]};
          const uint32_t b1[2] = {kb[2], kb[3]};
          mma_bf16_16816(sc[np * 2], qa[ks], b0);
          mma_bf16_16816(sc[np * 2 + 1], qa[ks], b1);
        }
      }
      float mx[2] = {m_r[0], m_r[1]};
#pragma unroll
      for (int nt = 0; nt < 8; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int kpos = kv0 + nt * 8 + cq + (e & 1);
          float v = sc[nt][e] * scale_log2;
          if (kpos > qpos[e >> 1] || kpos >= ctx) v = -INFINITY;
          sc[nt][e] = v;
          mx[e >> 1] = fmaxf(mx[e >> 1], v);
        }
#pragma unroll
      for (int rr = 0; rr < 2; ++rr) {
        mx[rr] = fmaxf(mx[rr], __shfl_xor_sync(0xffffffffu, mx[rr], 1));
        mx[rr] = fmaxf(mx[rr], __shfl_xor_sync(0xffffffffu, mx[rr], 2));
      }
      float alpha[2];
#pragma unroll
      for (int rr = 0; rr < 2; ++rr) {
        alpha[rr] = (m_r[rr] == -INFINITY) ? 0.f : fast_exp2(m_r[rr] - mx[rr]);
        m_r[rr] = mx[rr];
        l_r[rr] *= alpha[rr];
      }
#pragma unroll
      for (int nt = 0; nt < 16; ++nt) {
        o[nt][0] *= alpha[0];
        o[nt][1] *= alpha[0];
        o[nt][2] *= alpha[1];
        o[nt][3] *= alpha[1];
      }
      uint32_t pa[4][4];
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) {
        float pv[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float mm = m_r[e >> 1];
          pv[e] = (mm == -INFINITY) ? 0.f : fast_exp2(sc[nt][e] - mm);
          l_r[e >> 1] += pv[e];
        }
        const int kk = nt >> 1, hi = nt & 1;
        pa[kk][hi * 2 + 0] = pack_bf16(pv[0], pv[1]);
        pa[kk][hi * 2 + 1] = pack_bf16(pv[2], pv[3]);
      }
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {  // 16 tokens (one page) per k-step
        const uint32_t pb = vbase + kk * kPageBytes;
#pragma unroll
        for (int c = 0; c < 16; c += 2) {
          uint32_t vb[4];
          const int mat = lane >> 3;
          const int tok = ((mat & 1) << 3) + (lane & 7);
          const int chunk = c + (mat >> 1);
          ldmatrix_x4_trans(vb, page_chunk_addr(pb, tok, chunk));
          const uint32_t b0[2] = {vb[0], vb[1]};
          const uint32_t b1[2] = {vb[2], vb[3]};
          mma_bf16_16816(o[c], pa[kk], b0);
          mma_bf16_16816(o[c + 1], pa[kk], b1);
        }
      }
    }
    __syncthreads();
    if (abort_sh) {  // uniform: every thread reads the flag after the barrier
      ok = false;
      break;
    }
    if (threadIdx.x == 0 && t + STAGES < ntiles) issue(t + STAGES);
  }
  if (!ok && threadIdx.x == 0) atomicExch(err, 2);
#pragma unroll
  for (int rr = 0; rr < 2; ++rr) {
    l_r[rr] += __shfl_xor_sync(0xffffffffu, l_r[rr], 1);
    l_r[rr] += __shfl_xor_sync(0xffffffffu, l_r[rr], 2);
  }
  const float inv0 = l_r[0] > 0.f ? 1.f / l_r[0] : 0.f;
  const float inv1 = l_r[1] > 0.f ? 1.f / l_r[1] : 0.f;
  if (qrow0 < q_len) {
    bf16* dst = out + (int64_t)(q_start + qrow0) * out_stride + (int64_t)head * kD;
#pragma unroll
    for (int nt = 0; nt < 16; ++nt)
      *reinterpret_cast<uint32_t*>(dst + nt * 8 + cq) = pack_bf16(o[nt][0] * inv0, o[nt][1] * inv0);
  }
  if (qrow1 < q_len) {
    bf16* dst = out + (int64_t)(q_start + qrow1) * out_stride + (int64_t)head * kD;
#pragma unroll
    for (int nt = 0; nt < 16; ++nt)
      *reinterpret_cast<uint32_t*>(dst + nt * 8 + cq) = pack_bf16(o[nt][2] * inv1, o[nt][3] * inv1);
  }
}

static constexpr int kPreStages = 3;
size_t prefill_attn_smem_bytes() { return (size_t)kPreStages * 2 * 4 * kPageBytes + 1024; }

void launch_prefill_attention(const CUtensorMap& tk, const CUtensorMap& tv, const bf16* q, int64_t q_stride,
                              const int32_t* work, int num_work, const int32_t* seq_info,
                              const int32_t* block_tables, int max_blocks, bf16* out, int64_t out_stride, int Hq,
                              int Hkv, float scale, int* err, cudaStream_t st) {
  if (num_work == 0) return;
  if (Hq % Hkv != 0) throw std::runtime_error("prefill attention: Hq must be a multiple of Hkv");
  auto kern = prefill_attn_kernel<kPreStages>;
  const size_t smem = prefill_attn_smem_bytes();
  static std::atomic<uint64_t> attr_devs{0};
  ensure_smem_attr(attr_devs, kern, smem);
  launch_k(kern, dim3(num_work, Hq), 128, smem, st, tk, tv, q, q_stride, work, seq_info, block_tables, max_blocks, out,
                                              out_stride, Hq, Hkv, scale * kLog2e, err);
  KAPSL_LAUNCH_CHECK();
  note_launch();
}

}  // namespace kapsl
