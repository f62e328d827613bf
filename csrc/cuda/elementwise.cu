// Memory-bound transformer ops for sm_100a: RMSNorm (optionally fused with the
// residual add), RoPE fused with the paged-KV write, SwiGLU and the embedding
// gather.  All use 16-byte vector accesses and fp32 math.
//
// Reference counterparts: the only CPU kernels the reference ships are
// `CpuMlp::fused_swiglu` (crates/kapsl-kernels/src/mlp/mod.rs:13-49) and the
// attention in crates/kapsl-kernels/src/attention/mod.rs; RMSNorm/RoPE/KV
// writes happen inside ONNX Runtime graphs (crates/kapsl-llm/src/engine.rs:3567)
// and host KV packing (crates/kapsl-llm/src/kv_cache.rs:1423-1499).
#include <algorithm>

#include "common.cuh"
#include "kernels.h"

namespace kapsl {

using bf16 = __nv_bfloat16;

struct alignas(16) Vec8 {
  __nv_bfloat162 h[4];
};

// ------------------------------------------------------------------ RMSNorm
template <int NPT>
__global__ void __launch_bounds__(1024) rmsnorm_kernel(bf16* __restrict__ out, int64_t out_stride,
                                                       const bf16* __restrict__ x, int64_t x_stride,
                                                       bf16* __restrict__ residual, int64_t res_stride,
                                                       const bf16* __restrict__ w, int H, float eps) {
  griddep_entry();
  const int row = blockIdx.x;
  const int chunks = H >> 3;
  const Vec8* xr = reinterpret_cast<const Vec8*>(x + row * x_stride);
  Vec8* rr = residual ? reinterpret_cast<Vec8*>(residual + row * res_stride) : nullptr;
  float v[NPT][8];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < NPT; ++i) {
    int c = threadIdx.x + i * blockDim.x;
    if (c < chunks) {
      Vec8 a = xr[c];
      if (rr) {
        Vec8 b = rr[c];
        Vec8 s;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          float2 fa = __bfloat1622float2(a.h[j]);
          float2 fb = __bfloat1622float2(b.h[j]);
          v[i][2 * j] = fa.x + fb.x;
          v[i][2 * j + 1] = fa.y + fb.y;
          s.h[j] = __floats2bfloat162_rn(v[i][2 * j], v[i][2 * j + 1]);
        }
        rr[c] = s;
      } else {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          float2 fa = __bfloat1622float2(a.h[j]);
          v[i][2 * j] = fa.x;
          v[i][2 * j + 1] = fa.y;
        }
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) ss += v[i][j] * v[i][j];
    }
  }
  __shared__ float red[32];
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = (threadIdx.x < (blockDim.x >> 5)) ? red[threadIdx.x] : 0.f;
    t = warp_sum(t);
    if (threadIdx.x == 0) red[0] = t;
  }
  __syncthreads();
  const float inv = rsqrtf(red[0] / (float)H + eps);
  const Vec8* wr = reinterpret_cast<const Vec8*>(w);
  Vec8* orow = reinterpret_cast<Vec8*>(out + row * out_stride);
#pragma unroll
  for (int i = 0; i < NPT; ++i) {
    int c = threadIdx.x + i * blockDim.x;
    if (c < chunks) {
      Vec8 ww = wr[c];
      Vec8 o;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        float2 fw = __bfloat1622float2(ww.h[j]);
        o.h[j] = __floats2bfloat162_rn(v[i][2 * j] * inv * fw.x, v[i][2 * j + 1] * inv * fw.y);
      }
      orow[c] = o;
    }
  }
}

void launch_rmsnorm(bf16* out, int64_t out_stride, const bf16* x, int64_t x_stride, bf16* residual,
                    int64_t res_stride, const bf16* w, int rows, int H, float eps, cudaStream_t st) {
  if (rows == 0) return;
  if (H % 8 != 0) throw std::runtime_error("rmsnorm: hidden size must be a multiple of 8");
  int chunks = H / 8;
  int threads = ((chunks + 31) / 32) * 32;
  int npt = 1;
  while (threads > 1024) {
    npt *= 2;
    threads = (((chunks + npt - 1) / npt + 31) / 32) * 32;
  }
  switch (npt) {
    case 1: launch_k(rmsnorm_kernel<1>, rows, threads, 0, st, out, out_stride, x, x_stride, residual, res_stride, w, H, eps); break;
    case 2: launch_k(rmsnorm_kernel<2>, rows, threads, 0, st, out, out_stride, x, x_stride, residual, res_stride, w, H, eps); break;
    case 4: launch_k(rmsnorm_kernel<4>, rows, threads, 0, st, out, out_stride, x, x_stride, residual, res_stride, w, H, eps); break;
    default: throw std::runtime_error("rmsnorm: hidden size too large");
  }
  KAPSL_LAUNCH_CHECK();
  note_launch();
}

// ------------------------------------------------- RoPE + paged KV write
// qkv: [T, (Hq + 2*Hkv) * D] (row pitch `qkv_stride` elements).  Q and K are
// rotated in place (NeoX "rotate half" convention: pairs (i, i + D/2)); the
// rotated K and the V rows are written to the paged caches laid out as
// [num_blocks, Hkv, block_size, D].  Tokens with slot < 0 skip the cache write.
__global__ void rope_kv_write_kernel(bf16* __restrict__ qkv, int64_t qkv_stride,
                                     const int32_t* __restrict__ positions,
                                     const int64_t* __restrict__ slots,
                                     const float* __restrict__ cos_sin,  // [max_pos, D]
                                     bf16* __restrict__ k_cache, bf16* __restrict__ v_cache, int Hq,
                                     int Hkv, int D, int block_size) {
  griddep_entry();
  const int t = blockIdx.x;
  const int half = D >> 1;
  const int pos = positions[t];
  const int64_t slot = slots ? slots[t] : -1;
  bf16* row = qkv + t * qkv_stride;
  const float* cs = cos_sin + (int64_t)pos * D;
  const int pairs2 = half >> 1;  // bf16x2 pairs per head half
  const int nrot = (Hq + Hkv) * pairs2;
  int64_t blk = 0, off = 0;
  if (slot >= 0) {
    blk = slot / block_size;
    off = slot % block_size;
  }
  for (int idx = threadIdx.x; idx < nrot; idx += blockDim.x) {
    const int h = idx / pairs2;
    const int i = (idx % pairs2) * 2;
    bf16* base = row + h * D;
    float2 x1 = __bfloat1622float2(*reinterpret_cast<__nv_bfloat162*>(base + i));
    float2 x2 = __bfloat1622float2(*reinterpret_cast<__nv_bfloat162*>(base + i + half));
    float c0 = cs[i], c1 = cs[i + 1], s0 = cs[half + i], s1 = cs[half + i + 1];
    __nv_bfloat162 y1 = __floats2bfloat162_rn(x1.x * c0 - x2.x * s0, x1.y * c1 - x2.y * s1);
    __nv_bfloat162 y2 = __floats2bfloat162_rn(x2.x * c0 + x1.x * s0, x2.y * c1 + x1.y * s1);
    *reinterpret_cast<__nv_bfloat162*>(base + i) = y1;
    *reinterpret_cast<__nv_bfloat162*>(base + i + half) = y2;
    if (h >= Hq && slot >= 0) {
      const int kh = h - Hq;
      bf16* dst = k_cache + ((blk * Hkv + kh) * block_size + off) * D;
      *reinterpret_cast<__nv_bfloat162*>(dst + i) = y1;
      *reinterpret_cast<__nv_bfloat162*>(dst + i + half) = y2;
    }
  }
  if (slot >= 0) {
    const int vchunks = Hkv * (D >> 3);
    const bf16* vsrc = row + (Hq + Hkv) * D;
    for (int idx = threadIdx.x; idx < vchunks; idx += blockDim.x) {
      const int kh = idx / (D >> 3);
      const int c = idx % (D >> 3);
      bf16* dst = v_cache + ((blk * Hkv + kh) * block_size + off) * D;
      reinterpret_cast<Vec8*>(dst)[c] = reinterpret_cast<const Vec8*>(vsrc + kh * D)[c];
    }
  }
}

void launch_rope_kv_write(bf16* qkv, int64_t qkv_stride, const int32_t* positions, const int64_t* slots,
                          const float* cos_sin, bf16* k_cache, bf16* v_cache, int T, int Hq, int Hkv, int D,
                          int block_size, cudaStream_t st) {
  if (T == 0) return;
  if (D % 8 != 0) throw std::runtime_error("rope: head_dim must be a multiple of 8");
  launch_k(rope_kv_write_kernel, T, 256, 0, st, qkv, qkv_stride, positions, slots, cos_sin, k_cache, v_cache, Hq,
                                          Hkv, D, block_size);
  KAPSL_LAUNCH_CHECK();
  note_launch();
}

// ------------------------------------------------------------------ SwiGLU
// x: [T, 2F] = [gate | up]; out: [T, F] = silu(gate) * up.
__global__ void silu_mul_kernel(bf16* __restrict__ out, const bf16* __restrict__ x, int F) {
  griddep_entry();
  const int t = blockIdx.y;
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c * 8 >= F) return;
  const Vec8 g = reinterpret_cast<const Vec8*>(x + (int64_t)t * 2 * F)[c];
  const Vec8 u = reinterpret_cast<const Vec8*>(x + (int64_t)t * 2 * F + F)[c];
  Vec8 o;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    float2 fg = __bfloat1622float2(g.h[j]);
    float2 fu = __bfloat1622float2(u.h[j]);
    float a = fg.x / (1.f + __expf(-fg.x)) * fu.x;
    float b = fg.y / (1.f + __expf(-fg.y)) * fu.y;
    o.h[j] = __floats2bfloat162_rn(a, b);
  }
  reinterpret_cast<Vec8*>(out + (int64_t)t * F)[c] = o;
}

void launch_silu_mul(bf16* out, const bf16* x, int T, int F, cudaStream_t st) {
  if (T == 0) return;
  if (F % 8 != 0) throw std::runtime_error("silu_mul: width must be a multiple of 8");
  dim3 grid((F / 8 + 127) / 128, T);
  launch_k(silu_mul_kernel, grid, 128, 0, st, out, x, F);
  KAPSL_LAUNCH_CHECK();
  note_launch();
}

// --------------------------------------------------------------- embedding
// Rows t < n_src whose src_rows[t] >= 0 take their token from prev_tokens
// (the previous step's sampler output, still on the device) instead of ids[t]:
// the host schedules and launches step k+1 before it has read step k's tokens.
__global__ void embedding_kernel(bf16* __restrict__ out, const bf16* __restrict__ table,
                                 const int32_t* __restrict__ ids, int H, int64_t vocab_start,
                                 int64_t vocab_rows, const int32_t* __restrict__ src_rows,
                                 const int32_t* __restrict__ prev_tokens, int n_src) {
  griddep_entry();
  const int t = blockIdx.x;
  int32_t tok = ids[t];
  if (t < n_src) {
    const int32_t r = src_rows[t];
    if (r >= 0) tok = prev_tokens[r];
  }
  const int64_t id = (int64_t)tok - vocab_start;
  Vec8* o = reinterpret_cast<Vec8*>(out + (int64_t)t * H);
  const bool in_range = id >= 0 && id < vocab_rows;
  const Vec8* src = reinterpret_cast<const Vec8*>(table + (in_range ? id : 0) * H);
  for (int c = threadIdx.x; c < H / 8; c += blockDim.x) {
    if (in_range) {
      o[c] = src[c];
    } else {
      Vec8 z;
#pragma unroll
      for (int j = 0; j < 4; ++j) z.h[j] = __floats2bfloat162_rn(0.f, 0.f);
      o[c] = z;
    }
  }
}

void launch_embedding(bf16* out, const bf16* table, const int32_t* ids, int T, int H, int64_t vocab_start,
                      int64_t vocab_rows, const int32_t* src_rows, const int32_t* prev_tokens, int n_src,
                      cudaStream_t st) {
  if (T == 0) return;
  if (H % 8 != 0) throw std::runtime_error("embedding: hidden size must be a multiple of 8");
  if (n_src > 0 && (src_rows == nullptr || prev_tokens == nullptr))
    throw std::runtime_error("embedding: src_rows and prev_tokens are needed together");
  launch_k(embedding_kernel, T, 256, 0, st, out, table, ids, H, vocab_start, vocab_rows, src_rows, prev_tokens,
                                      std::min(n_src, T));
  KAPSL_LAUNCH_CHECK();
  note_launch();
}

}  // namespace kapsl
