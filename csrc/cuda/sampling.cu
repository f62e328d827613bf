// GPU token sampler with the reference sampler's semantics
// (crates/kapsl-llm/src/engine.rs:5842-5927 and the repetition penalty at
// engine.rs:3104-3123):
//   * repetition penalty applied once per occurrence of an id in
//     prompt + output (l > 0 ? l / p : l * p);
//   * temperature <= 0: argmax (last index wins ties, like Iterator::max_by);
//   * otherwise scale by 1/T, keep the top_k largest (top_k == 0: the whole
//     vocabulary), sort descending, top-p cut over the softmax of those
//     candidates, renormalise, draw with the per-sequence LCG
//     x = x * 6364136223846793005 + 1, u = (x >> 32) / u32::MAX.
//
// Kernels
//   sample_select_kernel   one CTA per row.  Sparse penalty: each sequence slot
//       keeps the list of ids that occurred (first-seen order) next to the
//       per-id counts, so only those logits are touched.  Top-k (k <= 1024):
//       a 12-bit radix histogram of the order-preserving float keys finds the
//       bin holding the k-th largest value; a second pass (the row is then in
//       L2) gathers every element at or above that bin into shared memory
//       (further 12/8-bit levels only when the boundary bin is too large),
//       and a bitonic sort orders them (value desc, index asc).  One HBM read
//       of the row in the common case.  With one rank the kernel finishes the
//       row (top-p, draw).  Under vocab-parallel tensor parallelism every rank
//       holds a slice of the logits: the kernel stores its sorted candidates
//       straight into every peer's candidate buffer (NVLink P2P stores) and
//       the last CTA raises this rank's flag in every peer.
//   sample_merge_kernel    (vocab-parallel) waits, bounded, for every rank's
//       flag, merges the ranks' candidate lists (global top-k of the union of
//       per-slice top-k lists is exact), then top-p and draw.  Every rank
//       draws the same token with the same LCG state.
//   sample_full_kernel     rows with T > 0 and top_k == 0 or > 1024: the
//       whole vocabulary in the reference's order.  The row is sorted in a
//       per-CTA global scratch (bitonic: shared-memory tiles + global passes),
//       then the f32 sums and the cumulative top-p walk run in the
//       reference's sequential order, so seeded streams reproduce it.
#include "common.cuh"
#include "kernels.h"

namespace kapsl {

static constexpr int kSampThreads = 1024;
// The select kernel runs 512 threads with two CTAs per SM (64 registers a thread, no
// spills), so one wave holds 296 rows.
static constexpr int kSelectThreads = 512;
static constexpr int kMaxTopK = 1024;   // largest top_k of the fast path
static constexpr int kCandCap = 2048;   // candidates gathered into shared memory
static constexpr int kHistBins = 4096;  // 12-bit digits

__device__ __forceinline__ uint32_t float_key(float f) {
  uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

__device__ __forceinline__ float apply_penalty(float l, int c, float p) {
  for (int i = 0; i < c; ++i) l = (l > 0.f) ? (l / p) : (l * p);
  return l;
}

// (value desc, index asc): true when (a, ia) sorts before (b, ib)
__device__ __forceinline__ bool cand_before(float a, int ia, float b, int ib) {
  return (a > b) || (a == b && ia < ib);
}

// Bitonic sort of n entries (padded to a power of two by the caller) of
// (val, idx) in shared memory, descending by value, ascending index on ties.
__device__ void bitonic_desc(float* val, int* idx, int npow) {
  const int tid = threadIdx.x;
  for (int size = 2; size <= npow; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int i = tid; i < npow; i += blockDim.x) {
        const int j = i ^ stride;
        if (j > i) {
          const bool desc = ((i & size) == 0);
          const float a = val[i], b = val[j];
          const int ia = idx[i], ib = idx[j];
          const bool a_first = cand_before(a, ia, b, ib);
          if (desc ? !a_first : a_first) {
            val[i] = b;
            val[j] = a;
            idx[i] = ib;
            idx[j] = ia;
          }
        }
      }
      __syncthreads();
    }
  }
}

// Top-p cut and LCG draw over n candidates sorted descending by scaled value
// (thread 0 only; sequential f32 sums in the reference's order).
__device__ int finish_draw(const float* val, const int* idx, int n, float top_p, uint64_t* rng_slot) {
  int cutoff = n;
  const float tp = fminf(fmaxf(top_p, 0.f), 1.f);
  const float mx = val[0];
  if (tp < 1.f && n > 1) {
    float sum = 0.f;
    for (int i = 0; i < n; ++i) sum += expf(val[i] - mx);
    float cum = 0.f;
    for (int i = 0; i < n; ++i) {
      cum += expf(val[i] - mx) / sum;
      if (cum >= tp) {
        cutoff = i + 1;
        break;
      }
    }
  }
  float sum = 0.f;
  for (int i = 0; i < cutoff; ++i) sum += expf(val[i] - mx);
  uint64_t x = *rng_slot;
  x = x * 6364136223846793005ull + 1ull;
  *rng_slot = x;
  const float u = __uint2float_rn((uint32_t)(x >> 32)) / 4294967295.0f;
  float draw = u * sum;
  int chosen = idx[0];
  for (int i = 0; i < cutoff; ++i) {
    const float e = expf(val[i] - mx);
    if (draw <= e) {
      chosen = idx[i];
      break;
    }
    draw -= e;
  }
  return chosen;
}

struct SampleArgs {
  float* logits;            // [B, >= Vl] fp32 (this rank's vocabulary slice), rewritten by the penalty
  int64_t stride;
  int B;
  int Vl;                   // columns of this slice
  int v0;                   // global id of column 0
  int Vtot;                 // real vocabulary size (ids >= Vtot are padding and never chosen)
  const float* temperature;
  const int32_t* top_k;
  const float* top_p;
  const float* rep_penalty;  // or null
  const int32_t* counts;     // [S, Vtot] occurrence counts, or null (no penalty)
  const int32_t* occ;        // [S, occ_cap] ids that occurred, or null (dense penalty scan)
  const int32_t* occ_n;      // [S]
  int occ_cap;
  const int32_t* slots;      // row -> slot (null: slot = row)
  uint64_t* rng;             // [S] LCG states
  int32_t* out;              // [B] sampled tokens
  // vocabulary-parallel candidate exchange (world > 1)
  int world;
  int rank;
  int b_cap;                 // rows per (parity, rank) block of the candidate buffers
  float2* cand[8];           // peers' candidate buffers [2][world][b_cap][kMaxTopK] (x = value, y = id bits)
  int64_t* flags[8];         // peers' flag words; this kernel uses site 2 ([2 * 8 + rank])
  int64_t* ctr;              // local [0] epoch, [1] finished-CTA count
  int64_t timeout_ns;
  int* err;
};

__device__ __forceinline__ int row_k(const SampleArgs& a, int row) {
  int k = a.top_k[row];
  if (k <= 0 || k > a.Vtot) k = a.Vtot;
  return k;
}

// rows the fast path does not sample: T > 0 with k > kMaxTopK
__device__ __forceinline__ bool needs_full(const SampleArgs& a, int row) {
  return a.temperature[row] > 0.f && row_k(a, row) > kMaxTopK;
}

__device__ void apply_row_penalty(const SampleArgs& a, float* lg, int row, int slot) {
  const float pen = a.rep_penalty ? a.rep_penalty[row] : 1.f;
  if (a.counts == nullptr || slot < 0 || pen == 1.f) return;
  const int32_t* cnt = a.counts + (int64_t)slot * a.Vtot;
  const int n = a.occ ? a.occ_n[slot] : -1;
  if (n >= 0 && n <= a.occ_cap) {
    const int32_t* ids = a.occ + (int64_t)slot * a.occ_cap;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
      const int id = ids[i];
      const int v = id - a.v0;
      if (v >= 0 && v < a.Vl && id < a.Vtot) lg[v] = apply_penalty(lg[v], cnt[id], pen);
    }
  } else {  // no occurrence list (or it overflowed): scan the slot's counts
    for (int v = threadIdx.x; v < a.Vl; v += blockDim.x) {
      const int id = a.v0 + v;
      if (id >= a.Vtot) break;
      const int c = cnt[id];
      if (c > 0) lg[v] = apply_penalty(lg[v], c, pen);
    }
  }
}

struct SelectSmem {
  uint32_t hist[kHistBins];
  float val[kCandCap];
  int idx[kCandCap];
  uint32_t wsum[32];
  int misc[8];
};

// Greedy: argmax of the slice, last index wins ties; thread 0 gets the result.
__device__ void slice_argmax(const SampleArgs& a, const float* lg, SelectSmem& sm, float* best_v, int* best_i) {
  const int tid = threadIdx.x;
  float best = -INFINITY;
  int bi = -1;
  const int vend = min(a.Vl, a.Vtot - a.v0);
  // float4 loads, four in flight per thread; a thread visits its elements in
  // increasing index order, so ">=" keeps the last of equal maxima
  const int vend4 = (reinterpret_cast<uintptr_t>(lg) & 15) == 0 ? (vend & ~3) : 0;
  const int step = (int)blockDim.x * 16;
  for (int base = 0; base < vend4; base += step) {
    float4 q[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int v = base + (u * (int)blockDim.x + tid) * 4;
      if (v < vend4) q[u] = *reinterpret_cast<const float4*>(lg + v);
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int v = base + (u * (int)blockDim.x + tid) * 4;
      if (v >= vend4) continue;
      const float e[4] = {q[u].x, q[u].y, q[u].z, q[u].w};
#pragma unroll
      for (int j = 0; j < 4; ++j)
        if (bi < 0 || e[j] >= best) {
          best = e[j];
          bi = v + j;
        }
    }
  }
  for (int v = vend4 + tid; v < vend; v += blockDim.x) {
    const float l = lg[v];
    if (bi < 0 || l >= best) {
      best = l;
      bi = v;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, best, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (oi >= 0 && (bi < 0 || ov > best || (ov == best && oi > bi))) {
      best = ov;
      bi = oi;
    }
  }
  if ((tid & 31) == 0) {
    sm.val[tid >> 5] = best;
    sm.idx[tid >> 5] = bi;
  }
  __syncthreads();
  if (tid == 0) {
    float b = -INFINITY;
    int i = -1;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w)
      if (sm.idx[w] >= 0 && (i < 0 || sm.val[w] > b || (sm.val[w] == b && sm.idx[w] > i))) {
        b = sm.val[w];
        i = sm.idx[w];
      }
    *best_v = b;
    *best_i = i < 0 ? 0 : a.v0 + i;
  }
  __syncthreads();
}

static constexpr int kSample = 4096;  // strided sample that places the one-pass threshold
static constexpr int kSamplePer = kSample / kSelectThreads;
static constexpr int kGatherVec = 4;  // float4 loads per thread in flight in the one-pass gather

__device__ __forceinline__ float key_float(uint32_t k) {
  return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}

// One-pass top-k candidates: a strided sample of the slice places a threshold t
// expected to let ~3k + 64 elements through (the largest 16-bit key prefix that
// at least r sample values reach, found by a bisection of block-wide counts; no
// sort); one pass then gathers every element >= t.  Returns the number gathered
// when it holds the top k (k <= count <= kCandCap), otherwise -1 and the caller
// takes the exact radix path.
__device__ int slice_gather_sampled(const SampleArgs& a, const float* lg, int k, int vend, SelectSmem& sm) {
  const int tid = threadIdx.x, lane = tid & 31;
  if (vend < 2 * kSample || k > 256 || blockDim.x != kSelectThreads) return -1;
  const int stride = vend / kSample;
  const int warp = tid >> 5, nwarps = kSelectThreads / 32;
  uint32_t sk[kSamplePer];
#pragma unroll
  for (int j = 0; j < kSamplePer; ++j) sk[j] = float_key(lg[(int64_t)(tid + j * kSelectThreads) * stride]);
  const int want = 3 * k + 64;
  int r = (int)(((int64_t)want * kSample + vend - 1) / vend);
  r = min(max(r, 2), kSample);
  uint32_t t = 0;
#pragma unroll 1
  for (int bit = 31; bit >= 16; --bit) {
    const uint32_t c = t | (1u << bit);
    int mine = 0;
#pragma unroll
    for (int j = 0; j < kSamplePer; ++j) mine += sk[j] >= c;
    mine = __reduce_add_sync(0xffffffffu, mine);
    if (lane == 0) sm.wsum[warp] = (uint32_t)mine;
    __syncthreads();
    int n = 0;
#pragma unroll
    for (int w = 0; w < nwarps; ++w) n += (int)sm.wsum[w];
    __syncthreads();
    if (n >= r) t = c;
  }
  const float t_thr = (t == 0) ? -INFINITY : key_float(t);
  if (tid == 0) sm.misc[3] = 0;
  __syncthreads();
  // One pass, kGatherVec float4 loads per thread in flight: each thread counts its
  // elements >= t, a warp scan places them, one shared atomic per warp reserves room.
  const bool vec_ok = (reinterpret_cast<uintptr_t>(lg) & 15) == 0;
  const int vend4 = vec_ok ? (vend & ~3) : 0;
  const int step = (int)blockDim.x * 4 * kGatherVec;
  for (int base = 0; base < vend4; base += step) {
    float4 q[kGatherVec];
#pragma unroll
    for (int u = 0; u < kGatherVec; ++u) {
      const int v = base + (u * (int)blockDim.x + tid) * 4;
      q[u] = v < vend4 ? *reinterpret_cast<const float4*>(lg + v) : make_float4(-INFINITY, -INFINITY, -INFINITY,
                                                                                  -INFINITY);
    }
    int cnt = 0;
#pragma unroll
    for (int u = 0; u < kGatherVec; ++u)
      if (base + (u * (int)blockDim.x + tid) * 4 < vend4)
        cnt += (q[u].x >= t_thr) + (q[u].y >= t_thr) + (q[u].z >= t_thr) + (q[u].w >= t_thr);
    int incl = cnt;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += y;
    }
    int wbase = 0;
    if (lane == 31 && incl > 0) wbase = atomicAdd(&sm.misc[3], incl);
    wbase = __shfl_sync(0xffffffffu, wbase, 31);
    int p = wbase + incl - cnt;
    if (cnt > 0) {
#pragma unroll
      for (int u = 0; u < kGatherVec; ++u) {
        const int v = base + (u * (int)blockDim.x + tid) * 4;
        if (v >= vend4) continue;
        const float e[4] = {q[u].x, q[u].y, q[u].z, q[u].w};
#pragma unroll
        for (int j = 0; j < 4; ++j)
          if (e[j] >= t_thr) {
            if (p < kCandCap) {
              sm.val[p] = e[j];
              sm.idx[p] = a.v0 + v + j;
            }
            ++p;
          }
      }
    }
  }
  for (int v = vend4 + tid; v < vend; v += blockDim.x) {  // tail (or an unaligned slice)
    const float l = lg[v];
    if (l >= t_thr) {
      const int p = atomicAdd(&sm.misc[3], 1);
      if (p < kCandCap) {
        sm.val[p] = l;
        sm.idx[p] = a.v0 + v;
      }
    }
  }
  __syncthreads();
  const int n = sm.misc[3];
  if (n < k || n > kCandCap) return -1;
  int npow = 1;
  while (npow < n) npow <<= 1;
  for (int i = n + tid; i < npow; i += blockDim.x) {
    sm.val[i] = -INFINITY;
    sm.idx[i] = 0x7fffffff;
  }
  __syncthreads();
  bitonic_desc(sm.val, sm.idx, npow);
  return n;
}

// Finds the top-k (k <= kMaxTopK) of the slice: on return sm.val/sm.idx[0..k)
// hold them sorted (raw value desc, global id asc) and the function returns k
// (fewer when the slice is shorter).
__device__ int slice_topk(const SampleArgs& a, const float* lg, int k, SelectSmem& sm) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int vend = min(a.Vl, a.Vtot - a.v0);
  if (k > vend) k = vend;
  if (k <= 0) return 0;
  if (slice_gather_sampled(a, lg, k, vend, sm) >= 0) return k;
  __syncthreads();
  uint32_t prefix = 0, mask = 0;
  int need = k;   // rank of the boundary element inside the current prefix group
  int shift = 20, bits = 12;
  bool degenerate = false;
  for (int level = 0;; ++level) {
    const int nbins = 1 << bits;
    const uint32_t dmask = (uint32_t)nbins - 1u;
    for (int i = tid; i < nbins; i += blockDim.x) sm.hist[i] = 0;
    __syncthreads();
    for (int base = 0; base < vend; base += blockDim.x) {
      const int v = base + tid;
      bool hit = false;
      uint32_t digit = 0;
      if (v < vend) {
        const uint32_t key = float_key(lg[v]);
        hit = (key & mask) == prefix;
        digit = (key >> shift) & dmask;
      }
      const unsigned hits = __ballot_sync(0xffffffffu, hit);
      if (hit) {
        const unsigned same = __match_any_sync(hits, digit);
        if (lane == __ffs(same) - 1) atomicAdd(&sm.hist[digit], (uint32_t)__popc(same));
      }
    }
    __syncthreads();
    // suffix scan from the top bin: thread t owns `per` consecutive bins counted from the top
    const int per = nbins / (int)blockDim.x > 0 ? nbins / (int)blockDim.x : 1;
    const int owned = (tid * per < nbins) ? per : 0;
    uint32_t mine = 0;
    for (int j = 0; j < owned; ++j) mine += sm.hist[nbins - 1 - (tid * per + j)];
    uint32_t incl = mine;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t t = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += t;
    }
    if (lane == 31) sm.wsum[warp] = incl;
    __syncthreads();
    if (warp == 0) {
      uint32_t w = lane < (int)(blockDim.x >> 5) ? sm.wsum[lane] : 0u;
      uint32_t wi = w;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const uint32_t t = __shfl_up_sync(0xffffffffu, wi, o);
        if (lane >= o) wi += t;
      }
      sm.wsum[lane] = wi - w;  // exclusive prefix of the warps
    }
    __syncthreads();
    const uint32_t excl = sm.wsum[warp] + incl - mine;
    if (owned && excl < (uint32_t)need && excl + mine >= (uint32_t)need) {
      uint32_t above = excl;
      for (int j = 0; j < owned; ++j) {
        const int b = nbins - 1 - (tid * per + j);
        const uint32_t h = sm.hist[b];
        if (above + h >= (uint32_t)need) {
          sm.misc[0] = b;
          sm.misc[1] = (int)above;  // elements of the group strictly above bin b
          sm.misc[2] = (int)h;
          break;
        }
        above += h;
      }
    }
    __syncthreads();
    const int b = sm.misc[0], above = sm.misc[1], hb = sm.misc[2];
    prefix |= (uint32_t)b << shift;
    mask |= dmask << shift;
    const int n_ge = (k - need) + above + hb;  // elements at or above the boundary prefix
    __syncthreads();
    if (n_ge <= kCandCap) break;
    need -= above;
    if (shift == 0) {  // every bit used: the boundary elements all share one key
      degenerate = true;
      break;
    }
    if (shift == 20) {
      shift = 8;
      bits = 12;
    } else {
      shift = 0;
      bits = 8;
    }
  }
  // gather the candidates
  if (tid == 0) sm.misc[3] = 0;
  __syncthreads();
  if (!degenerate) {
    for (int base = 0; base < vend; base += blockDim.x) {
      const int v = base + tid;
      bool take = false;
      float l = 0.f;
      if (v < vend) {
        l = lg[v];
        take = (float_key(l) & mask) >= prefix;
      }
      const unsigned m = __ballot_sync(0xffffffffu, take);
      int wbase = 0;
      if (lane == 0 && m) wbase = atomicAdd(&sm.misc[3], __popc(m));
      wbase = __shfl_sync(0xffffffffu, wbase, 0);
      if (take) {
        const int p = wbase + __popc(m & ((1u << lane) - 1u));
        sm.val[p] = l;
        sm.idx[p] = a.v0 + v;
      }
    }
  } else {
    // strictly greater keys first (fewer than k of them), then equal keys in index order
    const int take_eq = need;
    for (int base = 0; base < vend; base += blockDim.x) {
      const int v = base + tid;
      bool take = false;
      float l = 0.f;
      if (v < vend) {
        l = lg[v];
        take = float_key(l) > prefix;
      }
      const unsigned m = __ballot_sync(0xffffffffu, take);
      int wbase = 0;
      if (lane == 0 && m) wbase = atomicAdd(&sm.misc[3], __popc(m));
      wbase = __shfl_sync(0xffffffffu, wbase, 0);
      if (take) {
        const int p = wbase + __popc(m & ((1u << lane) - 1u));
        sm.val[p] = l;
        sm.idx[p] = a.v0 + v;
      }
    }
    __syncthreads();
    int taken = 0;  // block-uniform
    for (int base = 0; base < vend && taken < take_eq; base += blockDim.x) {
      const int v = base + tid;
      const bool eq = v < vend && float_key(lg[v]) == prefix;
      const unsigned m = __ballot_sync(0xffffffffu, eq);
      if (lane == 0) sm.wsum[warp] = __popc(m);
      __syncthreads();
      int before = 0, total = 0;
      for (int w = 0; w < (int)(blockDim.x >> 5); ++w) {
        if (w < warp) before += sm.wsum[w];
        total += sm.wsum[w];
      }
      const int rank_in = taken + before + __popc(m & ((1u << lane) - 1u));
      const int base_out = sm.misc[3];
      if (eq && rank_in < take_eq) {
        sm.val[base_out + rank_in] = lg[v];
        sm.idx[base_out + rank_in] = a.v0 + v;
      }
      taken += total;
      __syncthreads();
    }
    if (tid == 0) sm.misc[3] += min(taken, take_eq);
  }
  __syncthreads();
  const int n = sm.misc[3];
  int npow = 1;
  while (npow < n) npow <<= 1;
  for (int i = n + tid; i < npow; i += blockDim.x) {
    sm.val[i] = -INFINITY;
    sm.idx[i] = 0x7fffffff;
  }
  __syncthreads();
  bitonic_desc(sm.val, sm.idx, npow);
  return k;
}

template <bool FINISH>
__global__ void __launch_bounds__(kSelectThreads, 2) sample_select_kernel(SampleArgs a) {
  griddep_wait_only();
  __shared__ SelectSmem sm;
  __shared__ int64_t epoch_sh;
  const int row = blockIdx.x;
  const int tid = threadIdx.x;
  if (!FINISH && tid == 0) epoch_sh = a.ctr[0] + 1;
  __syncthreads();
  float* lg = a.logits + (int64_t)row * a.stride;
  const int slot = a.slots ? a.slots[row] : row;
  const float T = a.temperature[row];
  int nc = 0;
  if (!needs_full(a, row)) {
    apply_row_penalty(a, lg, row, slot);
    __syncthreads();
    if (T <= 0.f) {
      __shared__ float gv;
      __shared__ int gi;
      slice_argmax(a, lg, sm, &gv, &gi);
      if (tid == 0) {
        sm.val[0] = gv;
        sm.idx[0] = gi;
      }
      nc = 1;
    } else {
      nc = slice_topk(a, lg, min(row_k(a, row), kMaxTopK), sm);
      for (int i = tid; i < nc; i += blockDim.x) sm.val[i] = sm.val[i] / T;  // the reference divides: l / T
    }
    __syncthreads();
    if (FINISH && tid == 0) {
      uint64_t* rs = a.rng + slot;
      a.out[row] = (T <= 0.f) ? sm.idx[0] : finish_draw(sm.val, sm.idx, nc, a.top_p[row], rs);
    }
  }
  if (!FINISH) {
    // push this slice's candidates into every rank's buffer (P2P stores over NVLink)
    const int64_t epoch = epoch_sh;
    const int parity = a.flags[a.rank] != nullptr ? (int)(epoch & 1) : 0;
    for (int p = 0; p < a.world; ++p) {
      if (a.cand[p] == nullptr) continue;  // NCCL mode: only the own buffer; an all-gather follows
      float2* dst = a.cand[p] + (((int64_t)parity * a.world + a.rank) * a.b_cap + row) * kMaxTopK;
      for (int i = tid; i < nc; i += blockDim.x) dst[i] = make_float2(sm.val[i], __int_as_float(sm.idx[i]));
    }
    __threadfence_system();
    __syncthreads();
    if (tid == 0) {
      const unsigned long long done = atomicAdd(reinterpret_cast<unsigned long long*>(&a.ctr[1]), 1ull);
      if (done == gridDim.x - 1) {
        for (int p = 0; p < a.world; ++p)
          if (a.flags[p] != nullptr) st_release_sys(a.flags[p] + 2 * 8 + a.rank, epoch);
        a.ctr[1] = 0;
        a.ctr[0] = epoch;
        __threadfence();
      }
    }
  }
}

// Vocabulary-parallel merge: every rank's sorted slice candidates of a row ->
// the global top-k -> top-p -> draw.  Candidate buffers and flags as above.
__global__ void __launch_bounds__(kSampThreads) sample_merge_kernel(SampleArgs a) {
  griddep_entry();
  extern __shared__ __align__(16) unsigned char dyn[];
  float* val = reinterpret_cast<float*>(dyn);
  int* idx = reinterpret_cast<int*>(val + a.world * kMaxTopK);
  __shared__ int ok_sh;
  const int row = blockIdx.x;
  const int tid = threadIdx.x;
  const int64_t epoch = a.ctr[0];  // raised by this rank's select kernel (same stream)
  if (tid == 0) {
    ok_sh = 1;
    if (a.flags[a.rank] != nullptr && !wait_flags(a.flags[a.rank] + 2 * 8, a.world, epoch, (uint64_t)a.timeout_ns)) {
      ok_sh = 0;
      atomicExch(a.err, 50);
    }
  }
  __syncthreads();
  if (!ok_sh || needs_full(a, row)) return;
  const int parity = a.flags[a.rank] != nullptr ? (int)(epoch & 1) : 0;
  const float T = a.temperature[row];
  const int slot = a.slots ? a.slots[row] : row;
  const int vslice = a.Vl;
  int kr = (T <= 0.f) ? 1 : min(min(row_k(a, row), kMaxTopK), vslice);
  const float2* mine = reinterpret_cast<const float2*>(a.cand[a.rank]);
  if (T <= 0.f) {  // greedy: max value, last (largest) id wins ties
    if (tid == 0) {
      float b = -INFINITY;
      int bi = -1;
      for (int p = 0; p < a.world; ++p) {
        const float2 c = mine[(((int64_t)parity * a.world + p) * a.b_cap + row) * kMaxTopK];
        const int ci = __float_as_int(c.y);
        if (bi < 0 || c.x > b || (c.x == b && ci > bi)) {
          b = c.x;
          bi = ci;
        }
      }
      a.out[row] = bi < 0 ? 0 : bi;
    }
    return;
  }
  // ranks whose slice lies past the vocabulary end hold fewer (or no) candidates
  const int n = a.world * kr;
  for (int i = tid; i < n; i += blockDim.x) {
    const int p = i / kr, j = i % kr;
    const int valid = min(kr, max(0, a.Vtot - p * vslice));
    if (j < valid) {
      const float2 c = mine[(((int64_t)parity * a.world + p) * a.b_cap + row) * kMaxTopK + j];
      val[i] = c.x;
      idx[i] = __float_as_int(c.y);
    } else {
      val[i] = -INFINITY;
      idx[i] = 0x7fffffff;
    }
  }
  int npow = 1;
  while (npow < n) npow <<= 1;
  for (int i = n + tid; i < npow; i += blockDim.x) {
    val[i] = -INFINITY;
    idx[i] = 0x7fffffff;
  }
  __syncthreads();
  bitonic_desc(val, idx, npow);
  if (tid == 0) {
    const int k = min(row_k(a, row), kMaxTopK);
    a.out[row] = finish_draw(val, idx, min(k, n), a.top_p[row], a.rng + slot);
  }
}

// ------------------------------------------------------------ whole vocabulary
// One CTA per flagged row (grid-stride over rows).  Scratch per CTA:
// keys [npow] u64 = (~float_key(scaled) << 32) | id (ascending = value desc,
// id asc) and e [npow] f32.
static constexpr int kFullTile = 4096;

__device__ __forceinline__ void cas_u64(unsigned long long* k, int i, int j, bool asc) {
  const unsigned long long x = k[i], y = k[j];
  if ((x > y) == asc) {
    k[i] = y;
    k[j] = x;
  }
}

__global__ void __launch_bounds__(kSampThreads) sample_full_kernel(SampleArgs a, unsigned long long* scratch,
                                                                   int npow) {
  griddep_entry();
  __shared__ unsigned long long tile[kFullTile];
  __shared__ float s_red[32];
  __shared__ int s_i[4];
  const int tid = threadIdx.x;
  unsigned long long* keys = scratch + (int64_t)blockIdx.x * npow * 2;  // keys, then e / prefix sums
  float* e = reinterpret_cast<float*>(keys + npow);
  for (int row = 0; row < a.B; ++row) {
    if (!needs_full(a, row)) continue;
    // rows are spread over the CTAs by their rank among the flagged rows
    __syncthreads();
    if (tid == 0) {
      int r = 0;
      for (int q = 0; q < row; ++q) r += needs_full(a, q) ? 1 : 0;
      s_i[0] = r;
    }
    __syncthreads();
    if (s_i[0] % gridDim.x != blockIdx.x) continue;
    float* lg = a.logits + (int64_t)row * a.stride;
    const int slot = a.slots ? a.slots[row] : row;
    const float T = a.temperature[row];
    const int V = min(a.Vl, a.Vtot);
    apply_row_penalty(a, lg, row, slot);
    __syncthreads();
    for (int i = tid; i < npow; i += blockDim.x) {
      unsigned long long k = ~0ull;
      if (i < V) k = ((unsigned long long)(~float_key(lg[i] / T)) << 32) | (unsigned)i;
      keys[i] = k;
    }
    __syncthreads();
    // bitonic sort ascending.  Pairs closer than kFullTile lie in one aligned
    // tile: those stages run in shared memory (all sizes up to the tile in one
    // load, then the tail of every larger size); wider strides run in place.
    const int tile_n = min(kFullTile, npow);
    for (int t0 = 0; t0 < npow; t0 += tile_n) {
      for (int i = tid; i < tile_n; i += blockDim.x) tile[i] = keys[t0 + i];
      __syncthreads();
      for (int size = 2; size <= tile_n; size <<= 1)
        for (int s2 = size >> 1; s2 > 0; s2 >>= 1) {
          for (int i = tid; i < tile_n; i += blockDim.x) {
            const int j = i ^ s2;
            if (j > i) cas_u64(tile, i, j, ((t0 + i) & size) == 0);
          }
          __syncthreads();
        }
      for (int i = tid; i < tile_n; i += blockDim.x) keys[t0 + i] = tile[i];
      __syncthreads();
    }
    for (int size = tile_n * 2; size <= npow; size <<= 1) {
      for (int stride = size >> 1; stride >= tile_n; stride >>= 1) {
        for (int i = tid; i < npow; i += blockDim.x) {
          const int j = i ^ stride;
          if (j > i) cas_u64(keys, i, j, (i & size) == 0);
        }
        __syncthreads();
      }
      for (int t0 = 0; t0 < npow; t0 += tile_n) {
        for (int i = tid; i < tile_n; i += blockDim.x) tile[i] = keys[t0 + i];
        __syncthreads();
        for (int s2 = tile_n >> 1; s2 > 0; s2 >>= 1) {
          for (int i = tid; i < tile_n; i += blockDim.x) {
            const int j = i ^ s2;
            if (j > i) cas_u64(tile, i, j, ((t0 + i) & size) == 0);
          }
          __syncthreads();
        }
        for (int i = tid; i < tile_n; i += blockDim.x) keys[t0 + i] = tile[i];
        __syncthreads();
      }
    }
    // scaled values back from the sorted keys; e[i] = exp(l_i - max) in sorted order
    if (tid == 0) {
      const uint32_t kk = ~(uint32_t)(keys[0] >> 32);
      const uint32_t u = (kk & 0x80000000u) ? (kk & 0x7fffffffu) : ~kk;
      s_red[0] = __uint_as_float(u);
    }
    __syncthreads();
    const float top = s_red[0];
    for (int i = tid; i < V; i += blockDim.x) {
      const uint32_t kk = ~(uint32_t)(keys[i] >> 32);
      const uint32_t u = (kk & 0x80000000u) ? (kk & 0x7fffffffu) : ~kk;
      e[i] = expf(__uint_as_float(u) - top);
    }
    __syncthreads();
    if (tid == 0) {
      const float tp = fminf(fmaxf(a.top_p[row], 0.f), 1.f);
      int cutoff = V;
      float sum_all = 0.f;
      for (int i = 0; i < V; ++i) sum_all += e[i];
      float sum_cut = sum_all;
      if (tp < 1.f && V > 1) {
        float cum = 0.f, run = 0.f;
        for (int i = 0; i < V; ++i) {
          run += e[i];
          cum += e[i] / sum_all;
          if (cum >= tp) {
            cutoff = i + 1;
            break;
          }
        }
        sum_cut = run;  // the same sequential sum over the kept prefix
      }
      uint64_t* rs = a.rng + slot;
      uint64_t x = *rs;
      x = x * 6364136223846793005ull + 1ull;
      *rs = x;
      const float u = __uint2float_rn((uint32_t)(x >> 32)) / 4294967295.0f;
      float draw = u * sum_cut;
      int chosen = (int)(keys[0] & 0xffffffffu);
      for (int i = 0; i < cutoff; ++i) {
        if (draw <= e[i]) {
          chosen = (int)(keys[i] & 0xffffffffu);
          break;
        }
        draw -= e[i];
      }
      a.out[row] = a.v0 + chosen;
    }
    __syncthreads();
  }
}

static void fill_args(SampleArgs& s, const SampleLaunch& l) {
  s.logits = l.logits;
  s.stride = l.stride;
  s.B = l.B;
  s.Vl = l.Vl;
  s.v0 = l.v0;
  s.Vtot = l.Vtot;
  s.temperature = l.temperature;
  s.top_k = l.top_k;
  s.top_p = l.top_p;
  s.rep_penalty = l.rep_penalty;
  s.counts = l.counts;
  s.occ = l.occ;
  s.occ_n = l.occ_n;
  s.occ_cap = l.occ_cap;
  s.slots = l.slots;
  s.rng = l.rng;
  s.out = l.out;
  s.world = l.world;
  s.rank = l.rank;
  s.b_cap = l.b_cap;
  for (int i = 0; i < 8; ++i) {
    s.cand[i] = i < l.world ? reinterpret_cast<float2*>(l.cand[i]) : nullptr;
    s.flags[i] = i < l.world ? l.flags[i] : nullptr;
  }
  s.ctr = l.ctr;
  s.timeout_ns = l.timeout_ns;
  s.err = l.err;
}

size_t sample_full_scratch_bytes(int V, int ctas) {
  int npow = 1;
  while (npow < V) npow <<= 1;
  return (size_t)ctas * npow * 16;
}

void launch_sample_merge(const SampleLaunch& l, cudaStream_t st) {
  if (l.B == 0) return;
  if (l.world < 2 || l.world > 8 || l.B > l.b_cap) throw std::runtime_error("sample: bad vocab-parallel merge");
  SampleArgs a{};
  fill_args(a, l);
  const size_t smem = (size_t)l.world * kMaxTopK * 8;
  static std::atomic<uint64_t> attr_devs{0};
  ensure_smem_attr(attr_devs, sample_merge_kernel, (size_t)8 * kMaxTopK * 8);  // the largest group's need
  launch_k(sample_merge_kernel, l.B, kSampThreads, smem, st, a);
  KAPSL_LAUNCH_CHECK();
  note_launch();
}

// world == 1: select + finish in one kernel.  world > 1 with peer flags:
// select (pushes candidates to every rank) + merge.  world > 1 without flags
// (NCCL): select only; the caller all-gathers the candidates and calls
// launch_sample_merge.
void launch_sample(const SampleLaunch& l, cudaStream_t st) {
  if (l.B == 0) return;
  SampleArgs a{};
  fill_args(a, l);
  if (l.world <= 1) {
    launch_k(sample_select_kernel<true>, l.B, kSelectThreads, 0, st, a);
    KAPSL_LAUNCH_CHECK();
    note_launch();
  } else {
    if (l.world > 8 || l.B > l.b_cap || l.ctr == nullptr || l.cand[l.rank] == nullptr)
      throw std::runtime_error("sample: vocab-parallel buffers missing or too small");
    launch_k(sample_select_kernel<false>, l.B, kSelectThreads, 0, st, a);
    KAPSL_LAUNCH_CHECK();
    note_launch();
    if (l.flags[l.rank] != nullptr) launch_sample_merge(l, st);
  }
  if (l.full_scratch != nullptr && l.full_ctas > 0) {
    if (l.world > 1) throw std::runtime_error("sample: whole-vocabulary rows need the full logits");
    int npow = 1;
    while (npow < l.Vl) npow <<= 1;
    launch_k(sample_full_kernel, l.full_ctas, kSampThreads, 0, st, a, reinterpret_cast<unsigned long long*>(l.full_scratch),
                                                             npow);
    KAPSL_LAUNCH_CHECK();
    note_launch();
  }
}

// counts[row, ids[i]] += 1 for each i (row = rows[i]); the first occurrence of
// an id in a row also appends it to the row's occurrence list.  Used when a
// sequence is admitted (its prompt) and after every step (its new token).
__global__ void count_tokens_kernel(int32_t* __restrict__ counts, int V, const int32_t* __restrict__ rows,
                                    const int32_t* __restrict__ ids, int n, int32_t* __restrict__ occ,
                                    int32_t* __restrict__ occ_n, int occ_cap) {
  griddep_entry();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const int r = rows[i];
  const int id = ids[i];
  if (r >= 0 && id >= 0 && id < V) {
    const int old = atomicAdd(&counts[(int64_t)r * V + id], 1);
    if (old == 0 && occ != nullptr) {
      const int p = atomicAdd(&occ_n[r], 1);
      if (p < occ_cap) occ[(int64_t)r * occ_cap + p] = id;
    }
  }
}

void launch_count_tokens(int32_t* counts, int V, const int32_t* rows, const int32_t* ids, int n, int32_t* occ,
                         int32_t* occ_n, int occ_cap, cudaStream_t st) {
  if (n == 0) return;
  launch_k(count_tokens_kernel, (n + 255) / 256, 256, 0, st, counts, V, rows, ids, n, occ, occ_n, occ_cap);
  KAPSL_LAUNCH_CHECK();
  note_launch();
}

}  // namespace kapsl
