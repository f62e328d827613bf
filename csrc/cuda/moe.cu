// Mixture-of-experts routing, token permutation and combine (sm_100a).
//
// Expert-parallel layout: the hidden state is replicated on every rank (the
// attention block is tensor-parallel and ends with a reduce + all-gather), so
// the all-to-all *dispatch* needs no transfer: every rank routes all tokens
// identically and gathers, from its own copy, the rows bound for its local
// experts.  The grouped expert GEMMs (gemm_sm100.cu, grouped mode) run over
// those rows.  The *combine* is one kernel per layer that, for the tokens this
// rank owns, pulls each token's top-k expert rows straight from the owning
// ranks' output buffers over NVLink (P2P loads), applies the routing weights,
// adds the residual and pushes the finished rows into every rank's residual
// stream (all-gather).  Per token, only the k expert rows cross NVLink, not
// a dense all-reduce of world partial sums.
//
// Flag barriers are the ones of the tensor-parallel reduction (same flag words
// and epoch counter, bounded waits that record an error code).
#include "common.cuh"
#include "kernels.h"

namespace kapsl {

using bf16 = __nv_bfloat16;

// ------------------------------------------------------------------ routing
// One CTA per token: warp w computes the logits of experts w, w + 8, ... (fp32
// dot products over d, four independent 16-byte loads in flight per lane);
// warp 0 then takes the top-k (ties -> lower expert id) and the softmax
// weights over all experts at the chosen ids, renormalised over the k chosen
// ones when `renorm` (Mixtral).  E <= 64.
constexpr int kRouteWarps = 8;

__global__ void __launch_bounds__(kRouteWarps * 32) moe_route_kernel(const bf16* __restrict__ x, int64_t x_stride,
                                                                     const bf16* __restrict__ wr, int T, int d, int E,
                                                                     int K, int renorm, int32_t* __restrict__ ids,
                                                                     float* __restrict__ wts) {
  griddep_entry();
  __shared__ float logit_sh[64];
  const int t = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const bf16* xr = x + (int64_t)t * x_stride;
  for (int e = warp; e < E; e += kRouteWarps) {
    const bf16* w = wr + (int64_t)e * d;
    float acc = 0.f;
    int c = lane * 8;
    for (; c + 3 * 256 < d; c += 4 * 256) {
      uint4 xv[4], wv[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        xv[u] = *reinterpret_cast<const uint4*>(xr + c + u * 256);
        wv[u] = *reinterpret_cast<const uint4*>(w + c + u * 256);
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const __nv_bfloat162* xp = reinterpret_cast<const __nv_bfloat162*>(&xv[u]);
        const __nv_bfloat162* wp = reinterpret_cast<const __nv_bfloat162*>(&wv[u]);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 a = __bfloat1622float2(xp[j]);
          const float2 b = __bfloat1622float2(wp[j]);
          acc = fmaf(a.x, b.x, acc);
          acc = fmaf(a.y, b.y, acc);
        }
      }
    }
    for (; c < d; c += 256) {
      const uint4 xv = *reinterpret_cast<const uint4*>(xr + c);
      const uint4 wv = *reinterpret_cast<const uint4*>(w + c);
      const __nv_bfloat162* xp = reinterpret_cast<const __nv_bfloat162*>(&xv);
      const __nv_bfloat162* wp = reinterpret_cast<const __nv_bfloat162*>(&wv);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 a = __bfloat1622float2(xp[j]);
        const float2 b = __bfloat1622float2(wp[j]);
        acc = fmaf(a.x, b.x, acc);
        acc = fmaf(a.y, b.y, acc);
      }
    }
    acc = warp_sum(acc);
    if (lane == 0) logit_sh[e] = acc;
  }
  __syncthreads();
  if (warp != 0) return;
  float lg[2];
  lg[0] = lane < E ? logit_sh[lane] : -INFINITY;  // lane owns experts lane and lane + 32
  lg[1] = lane + 32 < E ? logit_sh[lane + 32] : -INFINITY;
  const float mx = warp_max(fmaxf(lg[0], lg[1]));
  float se = 0.f;
  if (lane < E) se += __expf(lg[0] - mx);
  if (lane + 32 < E) se += __expf(lg[1] - mx);
  se = warp_sum(se);
  float sel_sum = 0.f;
  float my_p = 0.f;
  int my_e = 0;
  for (int k = 0; k < K; ++k) {
    float bv = lg[0];
    int be = lane;
    if (lg[1] > bv) {
      bv = lg[1];
      be = lane + 32;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oe = __shfl_xor_sync(0xffffffffu, be, o);
      if (ov > bv || (ov == bv && oe < be)) {
        bv = ov;
        be = oe;
      }
    }
    const float p = __expf(bv - mx) / se;
    if (lane == k) {
      my_p = p;
      my_e = be;
    }
    sel_sum += p;
    if ((be & 31) == lane) lg[be >> 5] = -INFINITY;
  }
  if (lane < K) {
    ids[(int64_t)t * K + lane] = my_e;
    wts[(int64_t)t * K + lane] = renorm ? my_p / sel_sum : my_p;
  }
}

// -------------------------------------------------------------- permutation
// One CTA.  Stable counting sort of the T*K assignments by expert:
//   seg[e]    start row of expert e's segment (segments padded to BM = 128 rows)
//   seg[E]    total rows
//   pos[a]    row of assignment a in the expert-sorted order
//   mtiles    [0] = number of 128-row tiles of the local experts [e_lo, e_lo+el),
//             [1 + i] = local expert index of tile i
//   src[r]    token of local row r (r relative to seg[e_lo]); -1 on padding rows
constexpr int kPermThreads = 1024;
constexpr int kMaxExperts = 64;

__global__ void __launch_bounds__(kPermThreads) moe_permute_kernel(const int32_t* __restrict__ ids, int n_assign,
                                                                   int K, int E, int e_lo, int el, int max_rows,
                                                                   int32_t* __restrict__ seg, int32_t* __restrict__ pos,
                                                                   int32_t* __restrict__ mtiles,
                                                                   int32_t* __restrict__ src, int* __restrict__ err) {
  griddep_entry();
  __shared__ int warp_cnt[kPermThreads / 32][kMaxExperts];
  __shared__ int run_cnt[kMaxExperts];
  __shared__ int seg_sh[kMaxExperts + 1];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  constexpr int NW = kPermThreads / 32;
  for (int e = tid; e < E; e += kPermThreads) run_cnt[e] = 0;
  __syncthreads();
  for (int base = 0; base < n_assign; base += kPermThreads) {
    for (int i = tid; i < NW * E; i += kPermThreads) warp_cnt[i / E][i % E] = 0;
    __syncthreads();
    const int a = base + tid;
    const int e = a < n_assign ? ids[a] : -1;
    const unsigned peers = __match_any_sync(0xffffffffu, e);
    const int rank_in_warp = __popc(peers & ((1u << lane) - 1u));
    if (e >= 0 && rank_in_warp == 0) warp_cnt[warp][e] = __popc(peers);
    __syncthreads();
    // exclusive scan over warps, per expert (thread e)
    if (tid < E) {
      int acc = run_cnt[tid];
      for (int w = 0; w < NW; ++w) {
        const int c = warp_cnt[w][tid];
        warp_cnt[w][tid] = acc;
        acc += c;
      }
      run_cnt[tid] = acc;
    }
    __syncthreads();
    if (e >= 0) pos[a] = warp_cnt[warp][e] + rank_in_warp;  // rank inside the expert
    __syncthreads();
  }
  if (tid == 0) {
    int acc = 0;
    for (int e = 0; e < E; ++e) {
      seg_sh[e] = acc;
      acc += (run_cnt[e] + 127) / 128 * 128;
    }
    seg_sh[E] = acc;
  }
  __syncthreads();
  for (int e = tid; e <= E; e += kPermThreads) seg[e] = seg_sh[e];
  const int local0 = seg_sh[e_lo];
  const int local_rows = seg_sh[e_lo + el] - local0;
  if (local_rows > max_rows) {  // cannot happen when max_rows is sized by the host bound
    if (tid == 0) {
      atomicExch(err, 40);
      mtiles[0] = 0;
    }
    return;
  }
  for (int r = tid; r < local_rows; r += kPermThreads) src[r] = -1;
  __syncthreads();
  for (int a = tid; a < n_assign; a += kPermThreads) {
    const int e = ids[a];
    const int p = seg_sh[e] + pos[a];
    pos[a] = p;
    if (e >= e_lo && e < e_lo + el) src[p - local0] = a / K;
  }
  if (tid < el) {
    const int e = e_lo + tid;
    const int t0 = (seg_sh[e] - local0) / 128, nt = (seg_sh[e + 1] - seg_sh[e]) / 128;
    for (int i = 0; i < nt; ++i) mtiles[1 + t0 + i] = tid;
  }
  if (tid == 0) mtiles[0] = local_rows / 128;
}

// Copies token rows into the expert-sorted buffer (zeros on padding rows).
__global__ void __launch_bounds__(256) moe_gather_kernel(const bf16* __restrict__ x, int64_t x_stride,
                                                         const int32_t* __restrict__ src,
                                                         const int32_t* __restrict__ mtiles, bf16* __restrict__ xs,
                                                         int64_t xs_stride, int d) {
  griddep_entry();
  const int rows = mtiles[0] * 128;
  const int chunks = d / 8;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < (int64_t)rows * chunks;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int r = (int)(i / chunks), c = (int)(i % chunks) * 8;
    const int t = src[r];
    uint4 v = make_uint4(0, 0, 0, 0);
    if (t >= 0) v = *reinterpret_cast<const uint4*>(x + (int64_t)t * x_stride + c);
    *reinterpret_cast<uint4*>(xs + (int64_t)r * xs_stride + c) = v;
  }
}

// ------------------------------------------------------------------ combine
struct MoECombineArgs {
  const bf16* y[8];     // per rank: expert outputs in local expert-sorted rows [rows][ld_y]
  bf16* hidden[8];      // per rank: residual stream [rows_pad][ld_h]
  int64_t* flags[8];    // per rank flag words (world > 1)
  const int32_t* ids;   // [T, K]
  const float* wts;     // [T, K]
  const int32_t* pos;   // [T, K] global expert-sorted row
  const int32_t* seg;   // [E + 1]
  int T, K, el, cols;
  int64_t ld_y, ld_h;
  int world, rank, rows_per_rank;
  int64_t* epoch_ctr;
  uint64_t timeout_ns;  // limit of the peer-flag waits
  int* err;
};

template <int WORLD>
__global__ void __launch_bounds__(256) moe_combine_kernel(MoECombineArgs a) {
  griddep_entry();
  __shared__ int64_t epoch_sh;
  __shared__ int ok_sh;
  if (WORLD > 1) {
    if (threadIdx.x == 0) {
      epoch_sh = a.epoch_ctr[0] + 1;
      ok_sh = 1;
      if (blockIdx.x == 0) {
        __threadfence_system();
        for (int p = 0; p < WORLD; ++p) st_release_sys(a.flags[p] + 0 * 8 + a.rank, epoch_sh);
      }
      if (!wait_flags(a.flags[a.rank] + 0 * 8, WORLD, epoch_sh, a.timeout_ns)) {
        ok_sh = 0;
        atomicExch(a.err, 41);
      }
    }
    __syncthreads();
  }
  if (WORLD == 1 || ok_sh) {
    const int t0 = WORLD > 1 ? a.rank * a.rows_per_rank : 0;
    const int nrows = WORLD > 1 ? max(0, min(a.rows_per_rank, a.T - t0)) : a.T;
    const int chunks = a.cols / 8;
    bf16* own_h = a.hidden[0];
#pragma unroll
    for (int p = 1; p < WORLD; ++p)
      if (p == a.rank) own_h = a.hidden[p];
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < (int64_t)nrows * chunks;
         i += (int64_t)gridDim.x * blockDim.x) {
      const int t = t0 + (int)(i / chunks);
      const int c = (int)(i % chunks) * 8;
      float acc[8];
      {
        const uint4 hv = *reinterpret_cast<const uint4*>(own_h + (int64_t)t * a.ld_h + c);
        const __nv_bfloat162* hp = reinterpret_cast<const __nv_bfloat162*>(&hv);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 f = __bfloat1622float2(hp[j]);
          acc[2 * j] = f.x;
          acc[2 * j + 1] = f.y;
        }
      }
      for (int k = 0; k < a.K; ++k) {
        const int e = a.ids[(int64_t)t * a.K + k];
        const float w = a.wts[(int64_t)t * a.K + k];
        const int owner = e / a.el;
        if (WORLD == 1 && owner != a.rank) continue;  // local-only combine (NCCL reduction follows)
        const int row = a.pos[(int64_t)t * a.K + k] - a.seg[owner * a.el];
        const bf16* yb = a.y[0];
#pragma unroll
        for (int p = 1; p < WORLD; ++p)
          if (p == owner) yb = a.y[p];
        const uint4 yv = *reinterpret_cast<const uint4*>(yb + (int64_t)row * a.ld_y + c);
        const __nv_bfloat162* yp = reinterpret_cast<const __nv_bfloat162*>(&yv);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 f = __bfloat1622float2(yp[j]);
          acc[2 * j] = fmaf(w, f.x, acc[2 * j]);
          acc[2 * j + 1] = fmaf(w, f.y, acc[2 * j + 1]);
        }
      }
      uint4 o;
      o.x = pack_bf16(acc[0], acc[1]);
      o.y = pack_bf16(acc[2], acc[3]);
      o.z = pack_bf16(acc[4], acc[5]);
      o.w = pack_bf16(acc[6], acc[7]);
#pragma unroll
      for (int p = 0; p < WORLD; ++p) *reinterpret_cast<uint4*>(a.hidden[p] + (int64_t)t * a.ld_h + c) = o;
    }
  }
  if (WORLD > 1) {
    __syncthreads();
    if (threadIdx.x == 0) {
      __threadfence_system();
      const int64_t done = atomicAdd(reinterpret_cast<unsigned long long*>(&a.epoch_ctr[1]), 1ull);
      if (done == gridDim.x - 1) {
        for (int p = 0; p < WORLD; ++p) st_release_sys(a.flags[p] + 1 * 8 + a.rank, epoch_sh);
        if (!wait_flags(a.flags[a.rank] + 1 * 8, WORLD, epoch_sh, a.timeout_ns)) atomicExch(a.err, 42);
        a.epoch_ctr[1] = 0;
        a.epoch_ctr[0] = epoch_sh;
        __threadfence();
      }
    }
  }
}

// ------------------------------------------------------------------ launchers
void launch_moe_route(const bf16* x, int64_t x_stride, const bf16* wr, int T, int d, int E, int K, bool renorm,
                      int32_t* ids, float* wts, cudaStream_t st) {
  if (T == 0) return;
  if (E > kMaxExperts || K > 8 || K > E) throw std::runtime_error("moe_route: need E <= 64 and K <= min(8, E)");
  if (d % 8 != 0 || x_stride % 8 != 0) throw std::runtime_error("moe_route: d and stride must be multiples of 8");
  launch_k(moe_route_kernel, T, kRouteWarps * 32, 0, st, x, x_stride, wr, T, d, E, K, renorm ? 1 : 0, ids, wts);
  KAPSL_LAUNCH_CHECK();
  note_launch();
}

void launch_moe_permute(const int32_t* ids, int T, int K, int E, int e_lo, int el, int max_rows, int32_t* seg,
                        int32_t* pos, int32_t* mtiles, int32_t* src, int* err, cudaStream_t st) {
  if (E > kMaxExperts) throw std::runtime_error("moe_permute: at most 64 experts");
  if (e_lo < 0 || el < 1 || e_lo + el > E) throw std::runtime_error("moe_permute: bad local expert range");
  launch_k(moe_permute_kernel, 1, kPermThreads, 0, st, ids, T * K, K, E, e_lo, el, max_rows, seg, pos, mtiles, src, err);
  KAPSL_LAUNCH_CHECK();
  note_launch();
}

void launch_moe_gather(const bf16* x, int64_t x_stride, const int32_t* src, const int32_t* mtiles, bf16* xs,
                       int64_t xs_stride, int d, int max_rows, int num_sms, cudaStream_t st) {
  if (d % 8 != 0 || x_stride % 8 != 0 || xs_stride % 8 != 0)
    throw std::runtime_error("moe_gather: d and strides must be multiples of 8");
  const int64_t work = (int64_t)max_rows * (d / 8);
  const int grid = (int)std::max<int64_t>(1, std::min<int64_t>((work + 255) / 256, 4LL * num_sms));
  launch_k(moe_gather_kernel, grid, 256, 0, st, x, x_stride, src, mtiles, xs, xs_stride, d);
  KAPSL_LAUNCH_CHECK();
  note_launch();
}

void launch_moe_combine(const bf16* const* y, bf16* const* hidden, int64_t* const* flags, int world, int rank,
                        const int32_t* ids, const float* wts, const int32_t* pos, const int32_t* seg, int T, int K,
                        int el, int cols, int64_t ld_y, int64_t ld_h, int rows_per_rank, int64_t* epoch_ctr,
                        int* err, int num_sms, uint64_t timeout_ns, cudaStream_t st) {
  if (T == 0) return;
  if (cols % 8 != 0 || ld_y % 8 != 0 || ld_h % 8 != 0) throw std::runtime_error("moe_combine: cols % 8 != 0");
  MoECombineArgs a{};
  for (int p = 0; p < world; ++p) {
    a.y[p] = y[p];
    a.hidden[p] = hidden[p];
    a.flags[p] = flags ? flags[p] : nullptr;
  }
  a.ids = ids;
  a.wts = wts;
  a.pos = pos;
  a.seg = seg;
  a.T = T;
  a.K = K;
  a.el = el;
  a.cols = cols;
  a.ld_y = ld_y;
  a.ld_h = ld_h;
  a.world = world;
  a.rank = rank;
  a.rows_per_rank = rows_per_rank;
  a.epoch_ctr = epoch_ctr;
  a.timeout_ns = timeout_ns;
  a.err = err;
  const int rows = world > 1 ? rows_per_rank : T;
  const int64_t work = (int64_t)rows * (cols / 8);
  const int grid = (int)std::max<int64_t>(1, std::min<int64_t>((work + 255) / 256, 4LL * num_sms));
  switch (world) {
    case 1: launch_k(moe_combine_kernel<1>, grid, 256, 0, st, a); break;
    case 2: launch_k(moe_combine_kernel<2>, grid, 256, 0, st, a); break;
    case 4: launch_k(moe_combine_kernel<4>, grid, 256, 0, st, a); break;
    case 8: launch_k(moe_combine_kernel<8>, grid, 256, 0, st, a); break;
    default: throw std::runtime_error("moe_combine: world size must be 1, 2, 4 or 8");
  }
  KAPSL_LAUNCH_CHECK();
  note_launch();
}

}  // namespace kapsl
