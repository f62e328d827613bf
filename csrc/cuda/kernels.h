// Launchers of the sm_100a kernels (raw pointers + stream).  The torch
// bindings in bindings.cpp validate tensors and call these.
#pragma once
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <cstddef>
#include <string>

namespace kapsl {

void launch_rmsnorm(__nv_bfloat16* out, int64_t out_stride, const __nv_bfloat16* x, int64_t x_stride,
                    __nv_bfloat16* residual, int64_t res_stride, const __nv_bfloat16* w, int rows, int H, float eps,
                    cudaStream_t st);

void launch_rope_kv_write(__nv_bfloat16* qkv, int64_t qkv_stride, const int32_t* positions, const int64_t* slots,
                          const float* cos_sin, __nv_bfloat16* k_cache, __nv_bfloat16* v_cache, int T, int Hq,
                          int Hkv, int D, int block_size, cudaStream_t st);

void launch_silu_mul(__nv_bfloat16* out, const __nv_bfloat16* x, int T, int F, cudaStream_t st);

// rows t < n_src with src_rows[t] >= 0 read their token id from prev_tokens[src_rows[t]]
void launch_embedding(__nv_bfloat16* out, const __nv_bfloat16* table, const int32_t* ids, int T, int H,
                      int64_t vocab_start, int64_t vocab_rows, const int32_t* src_rows, const int32_t* prev_tokens,
                      int n_src, cudaStream_t st);

size_t decode_attn_smem_bytes();
int decode_attn_num_splits(int B, int Hkv, int max_ctx, int num_sms);
void launch_decode_attention(const CUtensorMap& tk, const CUtensorMap& tv, const __nv_bfloat16* q, int64_t q_stride,
                             const int32_t* block_tables, int max_blocks, const int32_t* ctx_lens,
                             __nv_bfloat16* out, int64_t out_stride, float* part_o, float* part_lse, int B, int Hq,
                             int Hkv, int nsplit, float scale, int* err, cudaStream_t st);

size_t prefill_attn_smem_bytes();
void launch_prefill_attention(const CUtensorMap& tk, const CUtensorMap& tv, const __nv_bfloat16* q,
                              int64_t q_stride, const int32_t* work, int num_work, const int32_t* seq_info,
                              const int32_t* block_tables, int max_blocks, __nv_bfloat16* out, int64_t out_stride,
                              int Hq, int Hkv, float scale, int* err, cudaStream_t st);

// tcgen05 prefill attention (attention_tc.cu): work items of prefill_attn_tc_tokens_per_cta tokens
int prefill_attn_tc_tokens_per_cta(int Hq, int Hkv);
size_t prefill_attn_tc_smem_bytes();
void launch_prefill_attention_tc(const CUtensorMap& q_map, const CUtensorMap& k_map, const CUtensorMap& v_map,
                                 const int32_t* work, int nwork, const int32_t* seq_info,
                                 const int32_t* block_tables, int max_blocks, int Hq, int Hkv, float scale,
                                 __nv_bfloat16* out, int64_t out_stride, int* err, cudaStream_t st);
CUtensorMap make_tmap_3d_bf16(const void* base, const uint64_t (&dims)[3], const uint64_t (&strides_bytes)[2],
                              const uint32_t (&box)[3], bool swizzle128);

// Sampler launch (sampling.cu).  world > 1: vocabulary-parallel (this rank's
// logits are columns [v0, v0 + Vl) of the vocabulary); cand / flags are the
// ranks' symmetric candidate buffers and flag words (cand[p] == null for
// p != rank when an NCCL all-gather moves the candidates instead).
struct SampleLaunch {
  float* logits = nullptr;
  int64_t stride = 0;
  int B = 0;
  int Vl = 0;
  int v0 = 0;
  int Vtot = 0;
  const float* temperature = nullptr;
  const int32_t* top_k = nullptr;
  const float* top_p = nullptr;
  const float* rep_penalty = nullptr;
  const int32_t* counts = nullptr;
  const int32_t* occ = nullptr;
  const int32_t* occ_n = nullptr;
  int occ_cap = 0;
  const int32_t* slots = nullptr;
  uint64_t* rng = nullptr;
  int32_t* out = nullptr;
  int world = 1;
  int rank = 0;
  int b_cap = 0;
  void* cand[8] = {nullptr};
  int64_t* flags[8] = {nullptr};
  int64_t* ctr = nullptr;
  int64_t timeout_ns = 0;
  int* err = nullptr;
  void* full_scratch = nullptr;  // whole-vocabulary rows: sample_full_scratch_bytes(Vl, full_ctas)
  int full_ctas = 0;
};
void launch_sample(const SampleLaunch& l, cudaStream_t st);
size_t sample_full_scratch_bytes(int V, int ctas);
// the vocabulary-parallel merge step alone (after an NCCL all-gather of the candidates)
void launch_sample_merge(const SampleLaunch& l, cudaStream_t st);
void launch_count_tokens(int32_t* counts, int V, const int32_t* rows, const int32_t* ids, int n, int32_t* occ,
                         int32_t* occ_n, int occ_cap, cudaStream_t st);

int gemm_num_sms();
// Mainloop issue-cost probes (diagnostics): cycles per 64-wide k slice of the 2-SM
// MMA thread under protocol mode 0..4, and cycles per cta_group::1 MMA of width n.
void launch_gemm_issue_probe(const __nv_bfloat16* A, const __nv_bfloat16* B, int M, int N, int K, int mode, int ksub,
                             int stages, int units, int width, long long* cycles, int* err, cudaStream_t st);
void launch_mma_rate_probe(int n, int iters, long long* cycles, int* err, cudaStream_t st);
// epi: 0 plain, 1 +bias, 2 +residual, 3 SwiGLU over interleaved gate/up (N % 256 == 0, C is [M, N/2]).
// Returns the number of K splits used.  defer_splitk (plain epilogue only): when the GEMM splits K,
// the fp32 partials stay in the workspace ([splits][M][N]) for the consumer to sum, and no reduce
// kernel runs (C is not written); with one split C is written as usual.
int launch_gemm(const __nv_bfloat16* A, int64_t lda, const __nv_bfloat16* B, int64_t ldb, void* C, int64_t ldc,
                bool out_f32, int M, int N, int K, int epi, const __nv_bfloat16* bias, const __nv_bfloat16* res,
                int64_t ldr, float* workspace, size_t workspace_bytes, int* err, cudaStream_t st, int force_bn,
                int force_splits, bool defer_splitk = false);

// grouped (MoE expert) GEMM; mtiles = [valid 128-row tiles, expert of tile 0, ...] on the device
void launch_grouped_gemm(const __nv_bfloat16* A, int64_t lda, const __nv_bfloat16* B, int64_t ldb, __nv_bfloat16* C,
                         int64_t ldc, int rows, int N, int K, int num_groups, const int* mtiles, int epi, int bn,
                         int splits, float* workspace, size_t workspace_bytes, int* err, cudaStream_t st);

// GGUF Q4_K weights (gemm_q4k.cu): Y = X . dequant(Wq)^T (+ res); Wq rows are packed 144-byte blocks,
// or (tiled) [N/128][K/256][128 rows][144 B] so each weight tile's super-block is contiguous
void launch_gemm_q4k(const __nv_bfloat16* X, int64_t ldx, const uint8_t* Wq, int64_t w_pitch, __nv_bfloat16* Y,
                     int64_t ldy, int M, int N, int K, const __nv_bfloat16* res, int64_t ldr, float* workspace,
                     size_t workspace_bytes, int force_splits, bool tiled, int* err, cudaStream_t st);
void launch_q4k_quantize(const __nv_bfloat16* x, int64_t n, uint8_t* out, cudaStream_t st);
void launch_q4k_dequant(const uint8_t* raw, int64_t n, __nv_bfloat16* out, cudaStream_t st);
// Q4_K weight matrix [n, k] (row-major or tile-major blocks) -> bf16 rows of pitch
// ldo; half > 0 interleaves the two row halves in 128-row blocks (SwiGLU layout).
void launch_q4k_dequant_rows(const uint8_t* raw, int n, int k, bool tiled, int half, __nv_bfloat16* out, int64_t ldo,
                             cudaStream_t st);

// mixture of experts (moe.cu)
void launch_moe_route(const __nv_bfloat16* x, int64_t x_stride, const __nv_bfloat16* wr, int T, int d, int E, int K,
                      bool renorm, int32_t* ids, float* wts, cudaStream_t st);
void launch_moe_permute(const int32_t* ids, int T, int K, int E, int e_lo, int el, int max_rows, int32_t* seg,
                        int32_t* pos, int32_t* mtiles, int32_t* src, int* err, cudaStream_t st);
void launch_moe_gather(const __nv_bfloat16* x, int64_t x_stride, const int32_t* src, const int32_t* mtiles,
                       __nv_bfloat16* xs, int64_t xs_stride, int d, int max_rows, int num_sms, cudaStream_t st);
void launch_moe_combine(const __nv_bfloat16* const* y, __nv_bfloat16* const* hidden, int64_t* const* flags, int world,
                        int rank, const int32_t* ids, const float* wts, const int32_t* pos, const int32_t* seg, int T,
                        int K, int el, int cols, int64_t ld_y, int64_t ld_h, int rows_per_rank, int64_t* epoch_ctr,
                        int* err, int num_sms, uint64_t timeout_ns, cudaStream_t st);

// disaggregated prefill/decode: push KV blocks into a peer pool (kv_connector.cu)
void launch_kv_push(const void* src_pool, void* dst_pool, const int32_t* src_ids, const int32_t* dst_ids, int nblocks,
                    int planes, int64_t src_blocks_per_plane, int64_t dst_blocks_per_plane, int64_t block_bytes,
                    int num_sms, cudaStream_t st);

// tensor parallel over NVLink peer memory (tp_comm.cu / gemm_sm100.cu)
void launch_gemm_scatter(const __nv_bfloat16* A, int64_t lda, const __nv_bfloat16* B, int64_t ldb,
                         __nv_bfloat16* const* peers, int world, int my_rank, int rows_per_rank, int64_t ld_recv,
                         int M, int N, int K, int* err, cudaStream_t st);
void launch_tp_reduce_ag(__nv_bfloat16* const* recv, __nv_bfloat16* const* hidden, int64_t* const* flags, int world,
                         int rank, int rows_per_rank, int rows_total, int cols, int64_t ld, int64_t* epoch_ctr,
                         int* err, int num_sms, uint64_t timeout_ns, cudaStream_t st);
void launch_tp_pull_reduce_ag(__nv_bfloat16* const* partial, __nv_bfloat16* const* hidden, int64_t* const* flags,
                              int world, int rank, int rows_per_rank, int rows_total, int cols, int64_t ld,
                              int64_t* epoch_ctr, int* err, int num_sms, uint64_t timeout_ns, cudaStream_t st);
// row-parallel reduction + residual (rows owned by this rank) + RMSNorm + all-gather of the normed rows
void launch_tp_reduce_norm_ag(const __nv_bfloat16* const* partial, __nv_bfloat16* const* xout,
                              int64_t* const* flags, __nv_bfloat16* h, const __nv_bfloat16* w, float eps, int world,
                              int rank, int rows_per_rank, int rows_total, int cols, int64_t ld, int64_t* epoch_ctr,
                              int* err, int num_sms, uint64_t timeout_ns, cudaStream_t st);
void launch_flag_pingpong(int64_t* my_flag, int64_t* peer_flag, void* peer_data, int payload_bytes, int rank,
                          int iters, int mode, int64_t base, uint64_t timeout_ns, int64_t* out_ns, int* err,
                          cudaStream_t st);
// row-parallel reduction + residual + RMSNorm with flag-carrying 8-byte lines (one-shot / two-shot)
size_t tp_ll_slot_bytes(int world, int cap, int cols, bool two);
void launch_tp_ll_norm(const __nv_bfloat16* own, const float* ws, int splits, void* const* slot, void* const* gslot,
                       __nv_bfloat16* h, __nv_bfloat16* xout, const __nv_bfloat16* w, float eps, int world, int rank,
                       int rows_per_rank, int rows_total, int cols, int64_t ld, int cap, bool two, int64_t* epoch_ctr,
                       int* err, int num_sms, uint64_t timeout_ns, cudaStream_t st);
void launch_p2p_copy(void* dst, const void* src, int64_t bytes, int ctas_per_sm, cudaStream_t st);
void* symm_alloc(size_t bytes);
void symm_free(void* p);
std::string symm_handle(void* p);
void* symm_open(const std::string& handle);
void symm_close(void* p);

}  // namespace kapsl
