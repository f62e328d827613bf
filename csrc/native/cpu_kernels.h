// fp32 CPU kernels of the CPU backend (threads over rows / heads, inner loops
// written for the compiler's vectoriser).  Matrix products stay with the BLAS that
// PyTorch links; everything between them runs here.
#pragma once
#include <cstdint>

namespace kapsl {
namespace cpu {

// out[t] = x[t] * rsqrt(mean(x[t]^2) + eps) * w      (out may alias x)
void rmsnorm(const float* x, const float* w, float* out, int64_t rows, int64_t d, float eps);

// Rotate-half RoPE in place on x [T, H, D]; cos_sin [max_pos, D] holds cos in
// the first half and sin in the second.
void rope(float* x, const int64_t* pos, const float* cos_sin, int64_t T, int64_t H, int64_t D);

// Write K/V rows [T, Hkv, D] into paged caches [blocks, Hkv, bs, D] at flat
// slots (block * bs + offset); slots < 0 are skipped.
void kv_write(const float* k, const float* v, const int64_t* slots, float* k_cache, float* v_cache, int64_t T,
              int64_t Hkv, int64_t bs, int64_t D);

// Causal attention over paged KV for a batch of sequences.  Sequence s owns
// query rows [row0[s], row0[s] + nq[s]) whose KV length is ctx[s] (the queries
// are the last nq[s] positions); its pages are block_tables[s * max_blocks ...].
// D <= 512.
void paged_attention(const float* q, const float* k_cache, const float* v_cache, const int64_t* row0,
                     const int64_t* nq, const int64_t* ctx, const int32_t* block_tables, int64_t max_blocks,
                     int64_t num_seqs, int64_t Hq, int64_t Hkv, int64_t bs, int64_t D, float scale, float* out);

// out[t, j] = silu(x[t, j]) * x[t, F + j]
void silu_mul(const float* x, float* out, int64_t T, int64_t F);

// GGUF Q4_K weights kept quantized: w holds N rows of K / 256 blocks of 144
// bytes (f16 d, f16 dmin, 12 bytes of 6-bit scale/min pairs, 128 bytes of
// 4-bit quants; v = d * sc * q - dmin * m).
// y[t, n] = sum_k x[t, k] * w[n, k]            (x [T, K], y [T, N] fp32)
void q4k_matmul(const float* x, const uint8_t* w, float* y, int64_t T, int64_t N, int64_t K);
// The same product with the activations quantized to int8 per 256-value
// block (scale = max|x| / 127, round to nearest) and integer dot products of
// the 4-bit quants with them (AVX2 u8 x s8 multiply-adds), scaled per 32-value
// sub-block:  y = dx * (d * sum_j sc_j * sum(q * xq) - dmin * sum_j m_j * sum(xq)).
// This is the arithmetic llama.cpp's CPU path uses for Q4_K (8-bit
// activation blocks); the error against q4k_matmul is that of rounding x to
// 8 bits.
void q4k_matmul_q8(const float* x, const uint8_t* w, float* y, int64_t T, int64_t N, int64_t K);
// out[(n - n0), k] = w[n, k] for rows n0 <= n < n1 (fp32)
void q4k_dequant_rows(const uint8_t* w, float* out, int64_t n0, int64_t n1, int64_t K);

// GGUF Q6_K rows (210-byte blocks of 256: 128 bytes of low 4 bits, 64 bytes of
// high 2 bits, 16 int8 scales, f16 d; v = d * scale[v / 16] * (q - 32)).
// The product with int8 activation blocks, as for Q4_K:
//   y = dx * d * (sum_g scale_g * sum(q * xq) - 32 * sum_g scale_g * sum_g(xq)).
void q6k_matmul_q8(const float* x, const uint8_t* w, float* y, int64_t T, int64_t N, int64_t K);
void q6k_dequant_rows(const uint8_t* w, float* out, int64_t n0, int64_t n1, int64_t K);

// GGUF Q8_0 rows (34-byte blocks of 32: f16 d, 32 int8; v = d * q), K a
// multiple of 256: y = dx * sum_b d_b * sum(q_b * xq_b) with int8 activation
// blocks of 256 as above (every int8 code, -128 included, is handled).
void q80_matmul_q8(const float* x, const uint8_t* w, float* y, int64_t T, int64_t N, int64_t K);
void q80_dequant_rows(const uint8_t* w, float* out, int64_t n0, int64_t n1, int64_t K);

}  // namespace cpu
}  // namespace kapsl
