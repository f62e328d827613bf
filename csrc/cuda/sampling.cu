// GPU token sampler with the reference sampler's semantics
// (crates/kapsl-llm/src/engine.rs:5842-5927 and the repetition penalty at
// engine.rs:3104-3123):
//   * repetition penalty applied once per occurrence of an id in
//     prompt + output (l > 0 ? l / p : l * p), occurrences kept as per-slot
//     counts on the device;
//   * temperature <= 0: argmax (last index wins ties, like Iterator::max_by);
//   * otherwise scale by 1/T, keep the top_k largest (radix select over the
//     float keys, 11/11/10-bit digits), sort descending, top-p cut over the
//     softmax of those candidates, renormalise, draw with the per-sequence LCG
//     x = x * 6364136223846793005 + 1, u = (x >> 32) / u32::MAX.
// One CTA of 1024 threads per row; the LCG state lives on the device.
#include "common.cuh"
#include "kernels.h"

namespace kapsl {

static constexpr int kSampThreads = 1024;
static constexpr int kMaxTopK = 1024;

__device__ __forceinline__ uint32_t float_key(float f) {
  uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

__device__ __forceinline__ float apply_penalty(float l, int c, float p) {
  for (int i = 0; i < c; ++i) l = (l > 0.f) ? (l / p) : (l * p);
  return l;
}

__global__ void __launch_bounds__(kSampThreads)
    sample_kernel(float* __restrict__ logits, int64_t stride, int V, const float* __restrict__ temperature,
                  const int32_t* __restrict__ top_k, const float* __restrict__ top_p,
                  const float* __restrict__ rep_penalty, const int32_t* __restrict__ counts,
                  const int32_t* __restrict__ slots, uint64_t* __restrict__ rng, int32_t* __restrict__ out) {
  const int row = blockIdx.x;
  const int tid = threadIdx.x;
  float* lg = logits + (int64_t)row * stride;
  const float T = temperature[row];
  const float pen = rep_penalty ? rep_penalty[row] : 1.f;
  // per-sequence state (LCG, occurrence counts) lives in row `slot` of the tables
  const int slot = slots ? slots[row] : row;
  const int32_t* cnt = (counts && slot >= 0) ? counts + (int64_t)slot * V : nullptr;
  const bool use_pen = cnt && pen != 1.f;

  __shared__ float s_val[kMaxTopK];
  __shared__ int s_idx[kMaxTopK];
  __shared__ uint32_t s_hist[32 * 256];  // one 256-bin histogram per warp
  __shared__ uint32_t s_tot[256];
  __shared__ float s_redv[32];
  __shared__ int s_redi[32];
  __shared__ int s_misc[4];

  if (T <= 0.f) {  // greedy
    float best = -INFINITY;
    int bi = -1;
    for (int v = tid; v < V; v += kSampThreads) {
      float l = lg[v];
      if (use_pen) l = apply_penalty(l, cnt[v], pen);
      if (bi < 0 || l > best || (l == best && v > bi)) {
        best = l;
        bi = v;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      float ov = __shfl_xor_sync(0xffffffffu, best, o);
      int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (oi >= 0 && (bi < 0 || ov > best || (ov == best && oi > bi))) {
        best = ov;
        bi = oi;
      }
    }
    if ((tid & 31) == 0) {
      s_redv[tid >> 5] = best;
      s_redi[tid >> 5] = bi;
    }
    __syncthreads();
    if (tid == 0) {
      float b = -INFINITY;
      int i = -1;
      for (int w = 0; w < kSampThreads / 32; ++w)
        if (s_redi[w] >= 0 && (i < 0 || s_redv[w] > b || (s_redv[w] == b && s_redi[w] > i))) {
          b = s_redv[w];
          i = s_redi[w];
        }
      out[row] = i < 0 ? 0 : i;
    }
    return;
  }

  // Pass 0: the repetition penalty touches only ids that occurred; they are
  // rewritten in place (the row is scratch).  Temperature scaling preserves
  // the order, so it is applied to the surviving candidates only.
  if (use_pen) {
    for (int v = tid; v < V; v += kSampThreads) {
      const int c = cnt[v];
      if (c > 0) lg[v] = apply_penalty(lg[v], c, pen);
    }
  }
  int k = top_k[row];
  if (k <= 0 || k > V) k = V;
  if (k > kMaxTopK) k = kMaxTopK;  // candidates beyond 1024 are not kept
  __syncthreads();

  // Radix select of the k-th largest key: four 8-bit digits, one private
  // histogram per warp, lanes with equal digits combined before the atomic.
  uint32_t prefix = 0, mask = 0;
  int remaining = k;
  const int warp = tid >> 5, lane = tid & 31;
  uint32_t* whist = s_hist + warp * 256;
  for (int pass = 0; pass < 4; ++pass) {
    const int shift = 24 - 8 * pass;
    for (int i = tid; i < 32 * 256; i += kSampThreads) s_hist[i] = 0;
    __syncthreads();
    for (int base = 0; base < V; base += kSampThreads) {
      const int v = base + tid;
      bool hit = false;
      uint32_t digit = 0;
      if (v < V) {
        const uint32_t key = float_key(lg[v]);
        hit = (key & mask) == prefix;
        digit = (key >> shift) & 0xFFu;
      }
      const unsigned hits = __ballot_sync(0xffffffffu, hit);
      if (hit) {
        const unsigned same = __match_any_sync(hits, digit);
        if (lane == __ffs(same) - 1) atomicAdd(&whist[digit], (uint32_t)__popc(same));
      }
    }
    __syncthreads();
    if (tid < 256) {  // fold the per-warp histograms into warp 0's
      uint32_t t = 0;
      for (int w = 0; w < 32; ++w) t += s_hist[w * 256 + tid];
      s_tot[tid] = t;
    }
    __syncthreads();
    if (tid == 0) {
      int above = 0, d = 255;
      for (; d > 0; --d) {
        if (above + (int)s_tot[d] >= remaining) break;
        above += s_tot[d];
      }
      s_misc[0] = d;
      s_misc[1] = remaining - above;
    }
    __syncthreads();
    prefix |= ((uint32_t)s_misc[0]) << shift;
    mask |= 0xFFu << shift;
    remaining = s_misc[1];
    __syncthreads();
  }
  const uint32_t thr = prefix;  // key of the k-th largest value
  if (tid == 0) {
    s_misc[2] = 0;  // candidates strictly above the threshold
    s_misc[3] = 0;  // candidates equal to it
  }
  __syncthreads();
  const int n_above = k - remaining;
  for (int v = tid; v < V; v += kSampThreads) {
    const float raw = lg[v];
    const uint32_t key = float_key(raw);
    const float l = raw / T;
    if (key > thr) {
      int p = atomicAdd(&s_misc[2], 1);
      if (p < kMaxTopK) {
        s_val[p] = l;
        s_idx[p] = v;
      }
    } else if (key == thr) {
      int p = atomicAdd(&s_misc[3], 1);
      if (p < remaining && n_above + p < kMaxTopK) {
        s_val[n_above + p] = l;
        s_idx[n_above + p] = v;
      }
    }
  }
  __syncthreads();
  // pad to a power of two and bitonic-sort descending (ties: lower index first)
  int n = k;
  int npow = 1;
  while (npow < n) npow <<= 1;
  for (int i = n + tid; i < npow; i += kSampThreads) {
    s_val[i] = -INFINITY;
    s_idx[i] = 0x7fffffff;
  }
  __syncthreads();
  for (int size = 2; size <= npow; size <<= 1) {
    for (int stride2 = size >> 1; stride2 > 0; stride2 >>= 1) {
      for (int i = tid; i < npow; i += kSampThreads) {
        const int j = i ^ stride2;
        if (j > i) {
          const bool desc = ((i & size) == 0);
          const float a = s_val[i], b = s_val[j];
          const int ia = s_idx[i], ib = s_idx[j];
          // "a before b" in descending order with ascending index tie-break
          const bool a_first = (a > b) || (a == b && ia < ib);
          if (desc ? !a_first : a_first) {
            s_val[i] = b;
            s_val[j] = a;
            s_idx[i] = ib;
            s_idx[j] = ia;
          }
        }
      }
      __syncthreads();
    }
  }
  if (tid == 0) {
    int cutoff = n;
    const float tp = fminf(fmaxf(top_p[row], 0.f), 1.f);
    const float mx = s_val[0];
    if (tp < 1.f && n > 1) {
      float sum = 0.f;
      for (int i = 0; i < n; ++i) sum += expf(s_val[i] - mx);
      float cum = 0.f;
      for (int i = 0; i < n; ++i) {
        cum += expf(s_val[i] - mx) / sum;
        if (cum >= tp) {
          cutoff = i + 1;
          break;
        }
      }
    }
    float sum = 0.f;
    for (int i = 0; i < cutoff; ++i) sum += expf(s_val[i] - mx);
    uint64_t x = rng[slot];
    x = x * 6364136223846793005ull + 1ull;
    rng[slot] = x;
    const float u = __uint2float_rn((uint32_t)(x >> 32)) / 4294967295.0f;
    float draw = u * sum;
    int chosen = s_idx[0];
    for (int i = 0; i < cutoff; ++i) {
      const float e = expf(s_val[i] - mx);
      if (draw <= e) {
        chosen = s_idx[i];
        break;
      }
      draw -= e;
    }
    out[row] = chosen;
  }
}

void launch_sample(float* logits, int64_t stride, int B, int V, const float* temperature, const int32_t* top_k,
                   const float* top_p, const float* rep_penalty, const int32_t* counts, const int32_t* slots,
                   uint64_t* rng, int32_t* out, cudaStream_t st) {
  if (B == 0) return;
  sample_kernel<<<B, kSampThreads, 0, st>>>(logits, stride, V, temperature, top_k, top_p, rep_penalty, counts,
                                            slots, rng, out);
  KAPSL_LAUNCH_CHECK();
  note_launch();
}

// counts[row, ids[i]] += 1 for each i (row = rows[i]); used when a sequence is
// admitted (its prompt) and after every step (its new token).
__global__ void count_tokens_kernel(int32_t* __restrict__ counts, int V, const int32_t* __restrict__ rows,
                                    const int32_t* __restrict__ ids, int n) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const int r = rows[i];
  const int id = ids[i];
  if (r >= 0 && id >= 0 && id < V) atomicAdd(&counts[(int64_t)r * V + id], 1);
}

void launch_count_tokens(int32_t* counts, int V, const int32_t* rows, const int32_t* ids, int n, cudaStream_t st) {
  if (n == 0) return;
  count_tokens_kernel<<<(n + 255) / 256, 256, 0, st>>>(counts, V, rows, ids, n);
  KAPSL_LAUNCH_CHECK();
  note_launch();
}

}  // namespace kapsl
