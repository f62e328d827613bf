// Python bindings of the sm_100a kernels (module kapsl_sdk_b200._cuda).
// Every entry point validates device, dtype, shape and strides, then launches
// on the current torch CUDA stream, so all of them are CUDA-graph capturable.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "common.cuh"
#include "kernels.h"

namespace {

using torch::Tensor;

#define CHECK_CUDA_T(x, name) TORCH_CHECK((x).is_cuda(), name " must be a CUDA tensor")
#define CHECK_DT(x, dt, name) TORCH_CHECK((x).scalar_type() == (dt), name " has the wrong dtype")

inline __nv_bfloat16* bf(const Tensor& t) { return reinterpret_cast<__nv_bfloat16*>(t.data_ptr()); }
inline cudaStream_t cur_stream() { return at::cuda::getCurrentCUDAStream().stream(); }

void rmsnorm(Tensor out, Tensor x, Tensor w, double eps, c10::optional<Tensor> residual) {
  CHECK_CUDA_T(x, "x");
  CHECK_DT(x, at::kBFloat16, "x");
  CHECK_DT(out, at::kBFloat16, "out");
  CHECK_DT(w, at::kBFloat16, "weight");
  TORCH_CHECK(x.dim() == 2 && out.dim() == 2 && x.stride(1) == 1 && out.stride(1) == 1, "rmsnorm: 2-D row-major");
  const int H = (int)x.size(1);
  TORCH_CHECK(w.numel() == H && out.size(1) == H && out.size(0) == x.size(0), "rmsnorm: shape mismatch");
  __nv_bfloat16* r = nullptr;
  int64_t rs = 0;
  if (residual.has_value()) {
    CHECK_DT(*residual, at::kBFloat16, "residual");
    TORCH_CHECK(residual->size(0) == x.size(0) && residual->size(1) == H && residual->stride(1) == 1,
                "rmsnorm: residual shape");
    r = bf(*residual);
    rs = residual->stride(0);
  }
  const c10::cuda::CUDAGuard g(x.device());
  kapsl::launch_rmsnorm(bf(out), out.stride(0), bf(x), x.stride(0), r, rs, bf(w), (int)x.size(0), H, (float)eps,
                        cur_stream());
}

void rope_kv_write(Tensor qkv, Tensor positions, c10::optional<Tensor> slots, Tensor cos_sin, Tensor k_cache,
                   Tensor v_cache, int64_t Hq, int64_t Hkv, int64_t D) {
  CHECK_DT(qkv, at::kBFloat16, "qkv");
  CHECK_DT(positions, at::kInt, "positions");
  CHECK_DT(cos_sin, at::kFloat, "cos_sin");
  TORCH_CHECK(qkv.dim() == 2 && qkv.stride(1) == 1 && qkv.size(1) >= (Hq + 2 * Hkv) * D, "rope: qkv layout");
  TORCH_CHECK(cos_sin.dim() == 2 && cos_sin.size(1) == D && cos_sin.is_contiguous(), "rope: cos_sin [max_pos, D]");
  TORCH_CHECK(k_cache.dim() == 4 && k_cache.size(1) == Hkv && k_cache.size(3) == D && k_cache.is_contiguous(),
              "rope: k_cache [blocks, Hkv, BS, D]");
  TORCH_CHECK(v_cache.sizes() == k_cache.sizes() && v_cache.is_contiguous(), "rope: v_cache layout");
  const int64_t* sp = nullptr;
  if (slots.has_value()) {
    CHECK_DT(*slots, at::kLong, "slots");
    TORCH_CHECK(slots->numel() >= qkv.size(0), "rope: slots too short");
    sp = slots->data_ptr<int64_t>();
  }
  TORCH_CHECK(positions.numel() >= qkv.size(0), "rope: positions too short");
  const c10::cuda::CUDAGuard g(qkv.device());
  kapsl::launch_rope_kv_write(bf(qkv), qkv.stride(0), positions.data_ptr<int32_t>(), sp, cos_sin.data_ptr<float>(),
                              bf(k_cache), bf(v_cache), (int)qkv.size(0), (int)Hq, (int)Hkv, (int)D,
                              (int)k_cache.size(2), cur_stream());
}

void silu_mul(Tensor out, Tensor x) {
  CHECK_DT(x, at::kBFloat16, "x");
  TORCH_CHECK(x.is_contiguous() && out.is_contiguous() && x.size(1) == 2 * out.size(1) && x.size(0) == out.size(0),
              "silu_mul: x [T, 2F], out [T, F]");
  const c10::cuda::CUDAGuard g(x.device());
  kapsl::launch_silu_mul(bf(out), bf(x), (int)x.size(0), (int)out.size(1), cur_stream());
}

void embedding(Tensor out, Tensor table, Tensor ids, int64_t vocab_start, c10::optional<Tensor> src_rows,
               c10::optional<Tensor> prev_tokens) {
  CHECK_DT(table, at::kBFloat16, "table");
  CHECK_DT(ids, at::kInt, "ids");
  TORCH_CHECK(table.is_contiguous() && out.is_contiguous() && out.size(1) == table.size(1), "embedding: layout");
  TORCH_CHECK(out.size(0) <= ids.numel(), "embedding: ids too short");
  TORCH_CHECK(src_rows.has_value() == prev_tokens.has_value(), "embedding: src_rows and prev_tokens go together");
  const int32_t* src = nullptr;
  const int32_t* prev = nullptr;
  int n_src = 0;
  if (src_rows.has_value()) {
    CHECK_DT((*src_rows), at::kInt, "src_rows");
    CHECK_DT((*prev_tokens), at::kInt, "prev_tokens");
    TORCH_CHECK(src_rows->is_contiguous() && prev_tokens->is_contiguous(), "embedding: src/prev layout");
    src = src_rows->data_ptr<int32_t>();
    prev = prev_tokens->data_ptr<int32_t>();
    n_src = (int)src_rows->numel();
  }
  const c10::cuda::CUDAGuard g(table.device());
  kapsl::launch_embedding(bf(out), bf(table), ids.data_ptr<int32_t>(), (int)out.size(0), (int)table.size(1),
                          vocab_start, table.size(0), src, prev, n_src, cur_stream());
}

CUtensorMap cache_map(const Tensor& cache) {
  TORCH_CHECK(cache.dim() == 4 && cache.is_contiguous() && cache.size(2) == 16 && cache.size(3) == 128,
              "attention: cache must be [blocks, Hkv, 16, 128] contiguous");
  CHECK_DT(cache, at::kBFloat16, "cache");
  const uint64_t rows = (uint64_t)cache.size(0) * cache.size(1) * 16;
  return kapsl::make_tmap_2d_bf16(cache.data_ptr(), rows, 128, 128, 16, 64, true);
}

int64_t decode_num_splits(int64_t B, int64_t Hkv, int64_t max_ctx) {
  return kapsl::decode_attn_num_splits((int)B, (int)Hkv, (int)max_ctx, kapsl::gemm_num_sms());
}

void decode_attention(Tensor q, Tensor k_cache, Tensor v_cache, Tensor block_tables, Tensor ctx_lens, Tensor out,
                      int64_t Hq, int64_t Hkv, double scale, int64_t nsplit, c10::optional<Tensor> part_o,
                      c10::optional<Tensor> part_lse, Tensor err) {
  CHECK_DT(q, at::kBFloat16, "q");
  CHECK_DT(out, at::kBFloat16, "out");
  CHECK_DT(block_tables, at::kInt, "block_tables");
  CHECK_DT(ctx_lens, at::kInt, "ctx_lens");
  CHECK_DT(err, at::kInt, "err");
  TORCH_CHECK(q.dim() == 2 && q.stride(1) == 1 && q.size(1) >= Hq * 128, "decode: q [B, >=Hq*128]");
  TORCH_CHECK(out.dim() == 2 && out.stride(1) == 1 && out.size(1) >= Hq * 128, "decode: out [B, >=Hq*128]");
  TORCH_CHECK(block_tables.dim() == 2 && block_tables.is_contiguous(), "decode: block_tables [B, max_blocks]");
  const int B = (int)q.size(0);
  TORCH_CHECK(block_tables.size(0) >= B && ctx_lens.numel() >= B && out.size(0) >= B, "decode: batch mismatch");
  TORCH_CHECK(k_cache.size(1) == Hkv, "decode: Hkv mismatch");
  float* po = nullptr;
  float* pl = nullptr;
  if (nsplit > 1) {
    TORCH_CHECK(part_o.has_value() && part_lse.has_value(), "decode: split-KV needs scratch");
    TORCH_CHECK(part_o->numel() >= (int64_t)B * Hq * nsplit * 128 && part_lse->numel() >= (int64_t)B * Hq * nsplit,
                "decode: scratch too small");
    po = part_o->data_ptr<float>();
    pl = part_lse->data_ptr<float>();
  }
  const c10::cuda::CUDAGuard g(q.device());
  CUtensorMap tk = cache_map(k_cache), tv = cache_map(v_cache);
  kapsl::launch_decode_attention(tk, tv, bf(q), q.stride(0), block_tables.data_ptr<int32_t>(),
                                 (int)block_tables.size(1), ctx_lens.data_ptr<int32_t>(), bf(out), out.stride(0), po,
                                 pl, B, (int)Hq, (int)Hkv, (int)nsplit, (float)scale, err.data_ptr<int>(),
                                 cur_stream());
}

void prefill_attention(Tensor q, Tensor k_cache, Tensor v_cache, Tensor work, Tensor seq_info, Tensor block_tables,
                       Tensor out, int64_t Hq, int64_t Hkv, double scale, Tensor err) {
  CHECK_DT(q, at::kBFloat16, "q");
  CHECK_DT(work, at::kInt, "work");
  CHECK_DT(seq_info, at::kInt, "seq_info");
  CHECK_DT(block_tables, at::kInt, "block_tables");
  TORCH_CHECK(q.dim() == 2 && q.stride(1) == 1 && q.size(1) >= Hq * 128, "prefill: q [T, >=Hq*128]");
  TORCH_CHECK(out.dim() == 2 && out.stride(1) == 1, "prefill: out row-major");
  TORCH_CHECK(work.dim() == 2 && work.size(1) == 2 && work.is_contiguous(), "prefill: work [n, 2]");
  TORCH_CHECK(seq_info.dim() == 2 && seq_info.size(1) == 4 && seq_info.is_contiguous(), "prefill: seq_info [S, 4]");
  const c10::cuda::CUDAGuard g(q.device());
  CUtensorMap tk = cache_map(k_cache), tv = cache_map(v_cache);
  kapsl::launch_prefill_attention(tk, tv, bf(q), q.stride(0), work.data_ptr<int32_t>(), (int)work.size(0),
                                  seq_info.data_ptr<int32_t>(), block_tables.data_ptr<int32_t>(),
                                  (int)block_tables.size(1), bf(out), out.stride(0), (int)Hq, (int)Hkv, (float)scale,
                                  err.data_ptr<int>(), cur_stream());
}

// tcgen05 version of prefill_attention; work items hold prefill_attn_tc_tokens(Hq, Hkv) tokens.
void prefill_attention_tc(Tensor q, Tensor k_cache, Tensor v_cache, Tensor work, Tensor seq_info,
                          Tensor block_tables, Tensor out, int64_t Hq, int64_t Hkv, double scale, Tensor err) {
  CHECK_DT(q, at::kBFloat16, "q");
  CHECK_DT(work, at::kInt, "work");
  CHECK_DT(seq_info, at::kInt, "seq_info");
  CHECK_DT(block_tables, at::kInt, "block_tables");
  TORCH_CHECK(q.dim() == 2 && q.stride(1) == 1 && q.size(1) >= Hq * 128, "prefill (tc): q [T, >=Hq*128]");
  TORCH_CHECK(out.dim() == 2 && out.stride(1) == 1, "prefill (tc): out row-major");
  TORCH_CHECK(work.dim() == 2 && work.size(1) == 2 && work.is_contiguous(), "prefill (tc): work [n, 2]");
  TORCH_CHECK(seq_info.dim() == 2 && seq_info.size(1) == 4 && seq_info.is_contiguous(), "prefill (tc): seq_info");
  const c10::cuda::CUDAGuard g(q.device());
  const int gq = (int)(Hq / Hkv);
  const int tpc = kapsl::prefill_attn_tc_tokens_per_cta((int)Hq, (int)Hkv);
  const uint64_t dims[3] = {128, (uint64_t)Hq, (uint64_t)q.size(0)};
  const uint64_t strides[2] = {256, (uint64_t)q.stride(0) * 2};
  const uint32_t box[3] = {64, (uint32_t)gq, (uint32_t)tpc};
  CUtensorMap tq = kapsl::make_tmap_3d_bf16(q.data_ptr(), dims, strides, box, true);
  CUtensorMap tk = cache_map(k_cache), tv = cache_map(v_cache);
  kapsl::launch_prefill_attention_tc(tq, tk, tv, work.data_ptr<int32_t>(), (int)work.size(0),
                                     seq_info.data_ptr<int32_t>(), block_tables.data_ptr<int32_t>(),
                                     (int)block_tables.size(1), (int)Hq, (int)Hkv, (float)scale, bf(out),
                                     out.stride(0), err.data_ptr<int>(), cur_stream());
}

int64_t prefill_attn_tc_tokens(int64_t Hq, int64_t Hkv) {
  return kapsl::prefill_attn_tc_tokens_per_cta((int)Hq, (int)Hkv);
}

// rng and counts are per-sequence tables indexed by slots[row] (row itself when slots is None).
kapsl::SampleLaunch sample_args(Tensor logits, Tensor temperature, Tensor top_k, Tensor top_p,
                                c10::optional<Tensor> rep_penalty, c10::optional<Tensor> counts,
                                c10::optional<Tensor> slots, Tensor rng, Tensor out, c10::optional<Tensor> occ,
                                c10::optional<Tensor> occ_n, int64_t vocab_start, int64_t vocab_size,
                                const std::vector<int64_t>& cand_ptrs, const std::vector<int64_t>& flag_ptrs,
                                int64_t rank, int64_t b_cap, c10::optional<Tensor> ctr, int64_t timeout_ns,
                                Tensor err) {
  CHECK_DT(logits, at::kFloat, "logits");
  TORCH_CHECK(logits.dim() == 2 && logits.stride(1) == 1, "sample: logits [B, V]");
  CHECK_DT(rng, at::kLong, "rng");
  CHECK_DT(out, at::kInt, "out");
  CHECK_DT(err, at::kInt, "err");
  const int B = (int)logits.size(0);
  TORCH_CHECK(temperature.numel() >= B && top_k.numel() >= B && top_p.numel() >= B && out.numel() >= B,
              "sample: per-row parameter arrays too short");
  TORCH_CHECK(slots.has_value() || rng.numel() >= B, "sample: rng table too short");
  kapsl::SampleLaunch l;
  l.logits = logits.data_ptr<float>();
  l.stride = logits.stride(0);
  l.B = B;
  l.Vl = (int)logits.size(1);
  l.v0 = (int)vocab_start;
  l.Vtot = vocab_size > 0 ? (int)vocab_size : (int)logits.size(1);
  TORCH_CHECK(l.v0 >= 0 && l.v0 < l.Vtot, "sample: vocab_start outside the vocabulary");
  l.temperature = temperature.data_ptr<float>();
  l.top_k = top_k.data_ptr<int32_t>();
  l.top_p = top_p.data_ptr<float>();
  l.rep_penalty = rep_penalty.has_value() ? rep_penalty->data_ptr<float>() : nullptr;
  if (counts.has_value()) {
    CHECK_DT(*counts, at::kInt, "counts");
    TORCH_CHECK(counts->size(-1) == l.Vtot, "sample: counts width must equal the vocabulary");
    l.counts = counts->data_ptr<int32_t>();
  }
  if (occ.has_value()) {
    TORCH_CHECK(occ_n.has_value(), "sample: occ needs occ_n");
    CHECK_DT(*occ, at::kInt, "occ");
    CHECK_DT(*occ_n, at::kInt, "occ_n");
    l.occ = occ->data_ptr<int32_t>();
    l.occ_n = occ_n->data_ptr<int32_t>();
    l.occ_cap = (int)occ->size(-1);
  }
  if (slots.has_value()) {
    CHECK_DT(*slots, at::kInt, "slots");
    TORCH_CHECK(slots->numel() >= B, "sample: slots too short");
    l.slots = slots->data_ptr<int32_t>();
  }
  l.rng = reinterpret_cast<uint64_t*>(rng.data_ptr<int64_t>());
  l.out = out.data_ptr<int32_t>();
  l.err = err.data_ptr<int>();
  l.world = cand_ptrs.empty() ? 1 : (int)cand_ptrs.size();
  TORCH_CHECK(l.world <= 8, "sample: at most 8 ranks");
  TORCH_CHECK(flag_ptrs.empty() || flag_ptrs.size() == cand_ptrs.size(), "sample: one flag word set per rank");
  l.rank = (int)rank;
  l.b_cap = (int)b_cap;
  for (int i = 0; i < l.world && !cand_ptrs.empty(); ++i) {
    l.cand[i] = reinterpret_cast<void*>(cand_ptrs[i]);
    l.flags[i] = flag_ptrs.empty() ? nullptr : reinterpret_cast<int64_t*>(flag_ptrs[i]);
  }
  if (l.world > 1) {
    TORCH_CHECK(ctr.has_value(), "sample: vocab-parallel sampling needs its counter tensor");
    CHECK_DT(*ctr, at::kLong, "ctr");
    l.ctr = ctr->data_ptr<int64_t>();
  }
  l.timeout_ns = timeout_ns;
  return l;
}

void sample(Tensor logits, Tensor temperature, Tensor top_k, Tensor top_p, c10::optional<Tensor> rep_penalty,
            c10::optional<Tensor> counts, c10::optional<Tensor> slots, Tensor rng, Tensor out,
            c10::optional<Tensor> occ, c10::optional<Tensor> occ_n, int64_t vocab_start, int64_t vocab_size,
            c10::optional<Tensor> full_scratch, int64_t full_ctas, std::vector<int64_t> cand_ptrs,
            std::vector<int64_t> flag_ptrs, int64_t rank, int64_t b_cap, c10::optional<Tensor> ctr,
            int64_t timeout_ns, Tensor err) {
  kapsl::SampleLaunch l = sample_args(logits, temperature, top_k, top_p, rep_penalty, counts, slots, rng, out, occ,
                                      occ_n, vocab_start, vocab_size, cand_ptrs, flag_ptrs, rank, b_cap, ctr,
                                      timeout_ns, err);
  if (full_scratch.has_value() && full_ctas > 0) {
    TORCH_CHECK((size_t)full_scratch->nbytes() >= kapsl::sample_full_scratch_bytes(l.Vl, (int)full_ctas),
                "sample: whole-vocabulary scratch too small");
    l.full_scratch = full_scratch->data_ptr();
    l.full_ctas = (int)full_ctas;
  }
  const c10::cuda::CUDAGuard g(logits.device());
  kapsl::launch_sample(l, cur_stream());
}

void sample_merge(Tensor logits, Tensor temperature, Tensor top_k, Tensor top_p, c10::optional<Tensor> slots,
                  Tensor rng, Tensor out, int64_t vocab_size, std::vector<int64_t> cand_ptrs, int64_t rank,
                  int64_t b_cap, Tensor ctr, Tensor err) {
  kapsl::SampleLaunch l = sample_args(logits, temperature, top_k, top_p, c10::nullopt, c10::nullopt, slots, rng,
                                      out, c10::nullopt, c10::nullopt, 0, vocab_size, cand_ptrs, {}, rank, b_cap,
                                      ctr, 0, err);
  const c10::cuda::CUDAGuard g(logits.device());
  kapsl::launch_sample_merge(l, cur_stream());
}

int64_t sample_full_scratch_bytes(int64_t V, int64_t ctas) {
  return (int64_t)kapsl::sample_full_scratch_bytes((int)V, (int)ctas);
}

void count_tokens(Tensor counts, Tensor rows, Tensor ids, c10::optional<Tensor> occ, c10::optional<Tensor> occ_n) {
  CHECK_DT(counts, at::kInt, "counts");
  CHECK_DT(rows, at::kInt, "rows");
  CHECK_DT(ids, at::kInt, "ids");
  TORCH_CHECK(rows.numel() == ids.numel(), "count_tokens: rows/ids length");
  TORCH_CHECK(occ.has_value() == occ_n.has_value(), "count_tokens: occ and occ_n go together");
  int32_t* o = nullptr;
  int32_t* on = nullptr;
  int cap = 0;
  if (occ.has_value()) {
    CHECK_DT(*occ, at::kInt, "occ");
    CHECK_DT(*occ_n, at::kInt, "occ_n");
    o = occ->data_ptr<int32_t>();
    on = occ_n->data_ptr<int32_t>();
    cap = (int)occ->size(-1);
  }
  const c10::cuda::CUDAGuard g(counts.device());
  kapsl::launch_count_tokens(counts.data_ptr<int32_t>(), (int)counts.size(-1), rows.data_ptr<int32_t>(),
                             ids.data_ptr<int32_t>(), (int)ids.numel(), o, on, cap, cur_stream());
}

void gemm(Tensor A, Tensor B, Tensor C, int64_t epi, c10::optional<Tensor> bias, c10::optional<Tensor> res,
          c10::optional<Tensor> workspace, Tensor err, int64_t force_bn, int64_t force_splits) {
  CHECK_DT(A, at::kBFloat16, "A");
  CHECK_DT(B, at::kBFloat16, "B");
  TORCH_CHECK(A.dim() == 2 && B.dim() == 2 && C.dim() == 2, "gemm: 2-D operands");
  TORCH_CHECK(A.stride(1) == 1 && B.stride(1) == 1 && C.stride(1) == 1, "gemm: K-contiguous A/B, row-major C");
  const int64_t M = A.size(0), K = A.size(1), N = B.size(0);
  TORCH_CHECK(B.size(1) == K, "gemm: K mismatch");
  const bool f32 = C.scalar_type() == at::kFloat;
  TORCH_CHECK(f32 || C.scalar_type() == at::kBFloat16, "gemm: C must be bf16 or fp32");
  TORCH_CHECK(C.size(0) == M && C.size(1) == (epi == 3 ? N / 2 : N), "gemm: C shape");
  TORCH_CHECK(!(f32 && epi != 0), "gemm: fp32 output only with the plain epilogue");
  const __nv_bfloat16* bp = nullptr;
  const __nv_bfloat16* rp = nullptr;
  int64_t ldr = 0;
  if (epi == 1) {
    TORCH_CHECK(bias.has_value() && bias->numel() == N, "gemm: bias [N] required");
    bp = bf(*bias);
  }
  if (epi == 2) {
    TORCH_CHECK(res.has_value() && res->size(0) == M && res->size(1) == N && res->stride(1) == 1,
                "gemm: residual [M, N] required");
    rp = bf(*res);
    ldr = res->stride(0);
  }
  float* ws = nullptr;
  size_t wsb = 0;
  if (workspace.has_value()) {
    CHECK_DT(*workspace, at::kFloat, "workspace");
    ws = workspace->data_ptr<float>();
    wsb = workspace->numel() * sizeof(float);
  }
  const c10::cuda::CUDAGuard g(A.device());
  kapsl::launch_gemm(bf(A), A.stride(0), bf(B), B.stride(0), C.data_ptr(), C.stride(0), f32, (int)M, (int)N, (int)K,
                     (int)epi, bp, rp, ldr, ws, wsb, err.data_ptr<int>(), cur_stream(), (int)force_bn,
                     (int)force_splits);
}

// Plain bf16 GEMM whose split-K partials (if it splits K) stay in the workspace for the
// consumer; returns the number of splits (1: C was written).
int64_t gemm_deferred(Tensor A, Tensor B, Tensor C, Tensor workspace, Tensor err) {
  CHECK_DT(A, at::kBFloat16, "A");
  CHECK_DT(B, at::kBFloat16, "B");
  CHECK_DT(C, at::kBFloat16, "C");
  CHECK_DT(workspace, at::kFloat, "workspace");
  TORCH_CHECK(A.dim() == 2 && B.dim() == 2 && C.dim() == 2 && A.stride(1) == 1 && B.stride(1) == 1 &&
                  C.stride(1) == 1 && B.size(1) == A.size(1) && C.size(0) == A.size(0) && C.size(1) == B.size(0),
              "gemm_deferred: A [M, K], B [N, K], C [M, N]");
  const c10::cuda::CUDAGuard g(A.device());
  return kapsl::launch_gemm(bf(A), A.stride(0), bf(B), B.stride(0), C.data_ptr(), C.stride(0), false, (int)A.size(0),
                            (int)B.size(0), (int)A.size(1), 0, nullptr, nullptr, 0, workspace.data_ptr<float>(),
                            workspace.numel() * sizeof(float), err.data_ptr<int>(), cur_stream(), 0, 0, true);
}

// ---- tensor parallel over NVLink peer memory
template <class T>
std::vector<T*> as_ptrs(const std::vector<int64_t>& v) {
  std::vector<T*> out;
  for (int64_t x : v) out.push_back(reinterpret_cast<T*>(x));
  return out;
}

void gemm_scatter(Tensor A, Tensor B, std::vector<int64_t> peers, int64_t my_rank, int64_t rows_per_rank,
                  int64_t ld_recv, Tensor err) {
  CHECK_DT(A, at::kBFloat16, "A");
  CHECK_DT(B, at::kBFloat16, "B");
  TORCH_CHECK(A.dim() == 2 && B.dim() == 2 && A.stride(1) == 1 && B.stride(1) == 1 && A.size(1) == B.size(1),
              "gemm_scatter: A [M, K], B [N, K]");
  TORCH_CHECK(ld_recv >= B.size(0), "gemm_scatter: receive rows narrower than N");
  const c10::cuda::CUDAGuard g(A.device());
  auto p = as_ptrs<__nv_bfloat16>(peers);
  kapsl::launch_gemm_scatter(bf(A), A.stride(0), bf(B), B.stride(0), p.data(), (int)p.size(), (int)my_rank,
                             (int)rows_per_rank, ld_recv, (int)A.size(0), (int)B.size(0), (int)A.size(1),
                             err.data_ptr<int>(), cur_stream());
}

void tp_reduce_ag(std::vector<int64_t> recv, std::vector<int64_t> hidden, std::vector<int64_t> flags, int64_t rank,
                  int64_t rows_per_rank, int64_t rows_total, int64_t cols, int64_t ld, Tensor epoch_ctr, Tensor err,
                  int64_t timeout_ns) {
  TORCH_CHECK(timeout_ns > 0, "tp_reduce_ag: timeout_ns must be positive");
  TORCH_CHECK(recv.size() == hidden.size() && recv.size() == flags.size(), "tp_reduce_ag: pointer tables differ");
  CHECK_DT(epoch_ctr, at::kLong, "epoch_ctr");
  const c10::cuda::CUDAGuard g(epoch_ctr.device());
  auto r = as_ptrs<__nv_bfloat16>(recv);
  auto h = as_ptrs<__nv_bfloat16>(hidden);
  auto f = as_ptrs<int64_t>(flags);
  kapsl::launch_tp_reduce_ag(r.data(), h.data(), f.data(), (int)r.size(), (int)rank, (int)rows_per_rank,
                             (int)rows_total, (int)cols, ld, epoch_ctr.data_ptr<int64_t>(), err.data_ptr<int>(),
                             kapsl::gemm_num_sms(), (uint64_t)timeout_ns, cur_stream());
}

void tp_pull_reduce_ag(std::vector<int64_t> partial, std::vector<int64_t> hidden, std::vector<int64_t> flags,
                       int64_t rank, int64_t rows_per_rank, int64_t rows_total, int64_t cols, int64_t ld,
                       Tensor epoch_ctr, Tensor err, int64_t timeout_ns) {
  TORCH_CHECK(timeout_ns > 0, "tp_pull_reduce_ag: timeout_ns must be positive");
  TORCH_CHECK(partial.size() == hidden.size() && partial.size() == flags.size(), "tp_pull_reduce_ag: tables differ");
  CHECK_DT(epoch_ctr, at::kLong, "epoch_ctr");
  const c10::cuda::CUDAGuard g(epoch_ctr.device());
  auto r = as_ptrs<__nv_bfloat16>(partial);
  auto h = as_ptrs<__nv_bfloat16>(hidden);
  auto f = as_ptrs<int64_t>(flags);
  kapsl::launch_tp_pull_reduce_ag(r.data(), h.data(), f.data(), (int)r.size(), (int)rank, (int)rows_per_rank,
                                  (int)rows_total, (int)cols, ld, epoch_ctr.data_ptr<int64_t>(), err.data_ptr<int>(),
                                  kapsl::gemm_num_sms(), (uint64_t)timeout_ns, cur_stream());
}

void tp_reduce_norm_ag(std::vector<int64_t> partial, std::vector<int64_t> xout, std::vector<int64_t> flags, Tensor h,
                       Tensor w, double eps, int64_t rank, int64_t rows_per_rank, int64_t rows_total, int64_t ld,
                       Tensor epoch_ctr, Tensor err, int64_t timeout_ns) {
  TORCH_CHECK(partial.size() == xout.size() && partial.size() == flags.size(), "tp_reduce_norm_ag: tables differ");
  TORCH_CHECK(timeout_ns > 0, "tp_reduce_norm_ag: timeout_ns must be positive");
  CHECK_DT(h, at::kBFloat16, "h");
  CHECK_DT(w, at::kBFloat16, "w");
  CHECK_DT(epoch_ctr, at::kLong, "epoch_ctr");
  TORCH_CHECK(h.dim() == 2 && h.stride(1) == 1 && h.stride(0) == ld && w.numel() == h.size(1) && w.is_contiguous(),
              "tp_reduce_norm_ag: h [rows, cols] with row stride ld, w [cols]");
  const c10::cuda::CUDAGuard g(h.device());
  auto pp = as_ptrs<const __nv_bfloat16>(partial);
  auto xp = as_ptrs<__nv_bfloat16>(xout);
  auto fp = as_ptrs<int64_t>(flags);
  kapsl::launch_tp_reduce_norm_ag(pp.data(), xp.data(), fp.data(), bf(h), reinterpret_cast<const __nv_bfloat16*>(
                                      w.data_ptr()), (float)eps, (int)pp.size(), (int)rank, (int)rows_per_rank,
                                  (int)rows_total, (int)h.size(1), ld, epoch_ctr.data_ptr<int64_t>(),
                                  err.data_ptr<int>(), kapsl::gemm_num_sms(), (uint64_t)timeout_ns, cur_stream());
}

void flag_pingpong(int64_t my_flag, int64_t peer_flag, int64_t peer_data, int64_t payload_bytes, int64_t rank,
                   int64_t iters, int64_t mode, int64_t base, int64_t timeout_ns, Tensor out_ns, Tensor err) {
  TORCH_CHECK(my_flag % 8 == 0 && peer_flag % 8 == 0 && peer_data % 16 == 0 && payload_bytes % 16 == 0,
              "flag_pingpong: aligned flags and payload");
  CHECK_DT(out_ns, at::kLong, "out_ns");
  kapsl::launch_flag_pingpong(reinterpret_cast<int64_t*>(my_flag), reinterpret_cast<int64_t*>(peer_flag),
                              reinterpret_cast<void*>(peer_data), (int)payload_bytes, (int)rank, (int)iters,
                              (int)mode, base, (uint64_t)timeout_ns, out_ns.data_ptr<int64_t>(), err.data_ptr<int>(),
                              cur_stream());
}

void tp_ll_norm(Tensor own, std::vector<int64_t> slot, std::vector<int64_t> gslot, Tensor h, Tensor xout, Tensor w,
                double eps, int64_t rank, int64_t rows_per_rank, int64_t rows_total, int64_t cap, bool two,
                Tensor epoch_ctr, Tensor err, int64_t timeout_ns, c10::optional<Tensor> ws, int64_t splits) {
  const float* wsp = nullptr;
  if (splits > 1) {
    TORCH_CHECK(ws.has_value() && ws->scalar_type() == at::kFloat &&
                    ws->numel() >= splits * rows_total * h.size(1),
                "tp_ll_norm: split-K partials need the fp32 workspace [splits, rows, cols]");
    wsp = ws->data_ptr<float>();
  }
  TORCH_CHECK(timeout_ns > 0, "tp_ll_norm: timeout_ns must be positive");
  TORCH_CHECK(!two || gslot.size() == slot.size(), "tp_ll_norm: gather slot table");
  CHECK_DT(own, at::kBFloat16, "own");
  CHECK_DT(h, at::kBFloat16, "h");
  CHECK_DT(xout, at::kBFloat16, "xout");
  CHECK_DT(w, at::kBFloat16, "w");
  CHECK_DT(epoch_ctr, at::kLong, "epoch_ctr");
  CHECK_DT(err, at::kInt, "err");
  const int64_t ld = h.stride(0);
  TORCH_CHECK(h.dim() == 2 && h.stride(1) == 1 && w.numel() == h.size(1) && w.is_contiguous() &&
                  own.stride(0) == ld && xout.stride(0) == ld && own.stride(1) == 1 && xout.stride(1) == 1 &&
                  own.size(0) >= rows_total && xout.size(0) >= rows_total && h.size(0) >= rows_total,
              "tp_ll_norm: own / h / xout [rows, cols] with one row stride, w [cols]");
  for (auto p : slot) TORCH_CHECK(p % 16 == 0, "tp_ll_norm: slots must be 16-byte aligned");
  for (auto p : gslot) TORCH_CHECK(p % 16 == 0, "tp_ll_norm: slots must be 16-byte aligned");
  const c10::cuda::CUDAGuard g(h.device());
  std::vector<void*> sp, gp;
  for (auto p : slot) sp.push_back(reinterpret_cast<void*>(p));
  for (auto p : gslot) gp.push_back(reinterpret_cast<void*>(p));
  kapsl::launch_tp_ll_norm(bf(own), wsp, (int)splits, sp.data(), two ? gp.data() : nullptr, bf(h), bf(xout),
                           reinterpret_cast<const __nv_bfloat16*>(w.data_ptr()), (float)eps, (int)sp.size(), (int)rank,
                           (int)rows_per_rank, (int)rows_total, (int)h.size(1), ld, (int)cap, two,
                           epoch_ctr.data_ptr<int64_t>(), err.data_ptr<int>(), kapsl::gemm_num_sms(),
                           (uint64_t)timeout_ns, cur_stream());
}

void p2p_copy(int64_t dst, int64_t src, int64_t bytes, int64_t ctas_per_sm) {
  TORCH_CHECK(bytes % 16 == 0 && dst % 16 == 0 && src % 16 == 0, "p2p_copy: 16-byte aligned sizes and addresses");
  kapsl::launch_p2p_copy(reinterpret_cast<void*>(dst), reinterpret_cast<const void*>(src), bytes, (int)ctas_per_sm,
                         cur_stream());
}

int64_t symm_alloc(int64_t bytes) { return reinterpret_cast<int64_t>(kapsl::symm_alloc((size_t)bytes)); }
void symm_free(int64_t p) { kapsl::symm_free(reinterpret_cast<void*>(p)); }
py::bytes symm_handle(int64_t p) { return py::bytes(kapsl::symm_handle(reinterpret_cast<void*>(p))); }
int64_t symm_open(py::bytes h) { return reinterpret_cast<int64_t>(kapsl::symm_open(std::string(h))); }
void symm_close(int64_t p) { kapsl::symm_close(reinterpret_cast<void*>(p)); }

// A tensor view over raw device memory (symmetric buffers); no ownership.
void grouped_gemm(Tensor A, Tensor B, Tensor C, int64_t N, int64_t num_groups, Tensor mtiles, int64_t epi,
                  int64_t bn, int64_t splits, c10::optional<Tensor> workspace, Tensor err) {
  CHECK_DT(A, at::kBFloat16, "A");
  CHECK_DT(B, at::kBFloat16, "B");
  CHECK_DT(C, at::kBFloat16, "C");
  CHECK_DT(mtiles, at::kInt, "mtiles");
  TORCH_CHECK(A.dim() == 2 && A.stride(1) == 1 && B.dim() == 2 && B.stride(1) == 1 && C.dim() == 2 &&
                  C.stride(1) == 1, "grouped_gemm: row-major 2-D operands");
  TORCH_CHECK(B.size(0) == N * num_groups && B.size(1) == A.size(1), "grouped_gemm: B must be [groups*N, K]");
  const int64_t rows = A.size(0);
  TORCH_CHECK(C.size(0) >= rows && C.size(1) >= (epi == 3 ? N / 2 : N), "grouped_gemm: C too small");
  TORCH_CHECK(mtiles.numel() >= 1 + rows / 128, "grouped_gemm: tile table too short");
  float* ws = nullptr;
  size_t wsb = 0;
  if (workspace.has_value()) {
    CHECK_DT(*workspace, at::kFloat, "workspace");
    ws = workspace->data_ptr<float>();
    wsb = workspace->numel() * sizeof(float);
  }
  const c10::cuda::CUDAGuard g(A.device());
  kapsl::launch_grouped_gemm(bf(A), A.stride(0), bf(B), B.stride(0), bf(C), C.stride(0), (int)rows, (int)N,
                             (int)A.size(1), (int)num_groups, mtiles.data_ptr<int>(), (int)epi, (int)bn, (int)splits,
                             ws, wsb, err.data_ptr<int>(), cur_stream());
}

// Y[M, N] = X[M, K] . dequant(Wq[N, K/256 * 144 bytes])^T (+ residual)
void gemm_q4k(Tensor X, Tensor Wq, Tensor Y, int64_t K, c10::optional<Tensor> res, c10::optional<Tensor> workspace,
              int64_t force_splits, bool tiled, Tensor err) {
  CHECK_DT(X, at::kBFloat16, "X");
  CHECK_DT(Y, at::kBFloat16, "Y");
  TORCH_CHECK(Wq.scalar_type() == at::kByte && Wq.dim() == 2 && Wq.is_contiguous(), "gemm_q4k: Wq uint8 [N, bytes]");
  TORCH_CHECK(X.dim() == 2 && X.stride(1) == 1 && X.size(1) == K && Y.dim() == 2 && Y.stride(1) == 1,
              "gemm_q4k: X [M, K], Y [M, N] row-major");
  const int64_t M = X.size(0), N = Wq.size(0);
  TORCH_CHECK(Y.size(0) >= M && Y.size(1) >= N, "gemm_q4k: Y too small");
  const __nv_bfloat16* rp = nullptr;
  int64_t ldr = 0;
  if (res.has_value()) {
    CHECK_DT(*res, at::kBFloat16, "res");
    TORCH_CHECK(res->stride(1) == 1 && res->size(0) >= M && res->size(1) >= N, "gemm_q4k: residual shape");
    rp = bf(*res);
    ldr = res->stride(0);
  }
  float* ws = nullptr;
  size_t wsb = 0;
  if (workspace.has_value()) {
    CHECK_DT(*workspace, at::kFloat, "workspace");
    ws = workspace->data_ptr<float>();
    wsb = workspace->numel() * sizeof(float);
  }
  const c10::cuda::CUDAGuard g(X.device());
  kapsl::launch_gemm_q4k(bf(X), X.stride(0), Wq.data_ptr<uint8_t>(), Wq.size(1), bf(Y), Y.stride(0), (int)M, (int)N,
                         (int)K, rp, ldr, ws, wsb, (int)force_splits, tiled, err.data_ptr<int>(), cur_stream());
}

void q4k_quantize(Tensor x, Tensor out) {
  CHECK_DT(x, at::kBFloat16, "x");
  TORCH_CHECK(x.is_contiguous() && out.is_contiguous() && out.scalar_type() == at::kByte, "q4k_quantize: layout");
  TORCH_CHECK(out.numel() * 256 == x.numel() * 144, "q4k_quantize: output must hold numel/256 * 144 bytes");
  const c10::cuda::CUDAGuard g(x.device());
  kapsl::launch_q4k_quantize(bf(x), x.numel(), out.data_ptr<uint8_t>(), cur_stream());
}

void q4k_dequant(Tensor raw, Tensor out) {
  CHECK_DT(out, at::kBFloat16, "out");
  TORCH_CHECK(raw.is_contiguous() && out.is_contiguous() && raw.scalar_type() == at::kByte, "q4k_dequant: layout");
  TORCH_CHECK(raw.numel() * 256 == out.numel() * 144, "q4k_dequant: sizes");
  const c10::cuda::CUDAGuard g(raw.device());
  kapsl::launch_q4k_dequant(raw.data_ptr<uint8_t>(), out.numel(), bf(out), cur_stream());
}

void gemm_issue_probe(Tensor A, Tensor B, int64_t mode, int64_t ksub, int64_t stages, int64_t units, int64_t width,
                      Tensor cycles, Tensor err) {
  CHECK_DT(A, at::kBFloat16, "A");
  CHECK_DT(B, at::kBFloat16, "B");
  TORCH_CHECK(A.is_contiguous() && B.is_contiguous() && A.size(1) == B.size(1), "gemm_issue_probe: A [M, K], B [N, K]");
  TORCH_CHECK(cycles.scalar_type() == at::kLong && err.scalar_type() == at::kInt, "gemm_issue_probe: int64 cycles, int32 err");
  const c10::cuda::CUDAGuard g(A.device());
  kapsl::launch_gemm_issue_probe(bf(A), bf(B), (int)A.size(0), (int)B.size(0), (int)A.size(1), (int)mode, (int)ksub,
                                 (int)stages, (int)units, (int)width,
                                 reinterpret_cast<long long*>(cycles.data_ptr<int64_t>()),
                                 err.data_ptr<int>(), cur_stream());
}

void mma_rate_probe(int64_t n, int64_t iters, Tensor cycles, Tensor err) {
  TORCH_CHECK(cycles.scalar_type() == at::kLong && err.scalar_type() == at::kInt && cycles.is_cuda(),
              "mma_rate_probe: int64 cycles, int32 err");
  const c10::cuda::CUDAGuard g(cycles.device());
  kapsl::launch_mma_rate_probe((int)n, (int)iters, reinterpret_cast<long long*>(cycles.data_ptr<int64_t>()),
                               err.data_ptr<int>(), cur_stream());
}

void q4k_dequant_rows(Tensor raw, int64_t n, int64_t k, bool tiled, int64_t half, Tensor out) {
  CHECK_DT(out, at::kBFloat16, "out");
  TORCH_CHECK(raw.is_contiguous() && raw.scalar_type() == at::kByte && raw.numel() * 256 == n * k * 144,
              "q4k_dequant_rows: raw must hold n * k / 256 blocks");
  TORCH_CHECK(out.dim() == 2 && out.stride(1) == 1 && out.size(0) >= n && out.size(1) >= k, "q4k_dequant_rows: out");
  const c10::cuda::CUDAGuard g(raw.device());
  kapsl::launch_q4k_dequant_rows(raw.data_ptr<uint8_t>(), (int)n, (int)k, tiled, (int)half, bf(out), out.stride(0),
                                 cur_stream());
}

void moe_route(Tensor x, Tensor wr, int64_t K, bool renorm, Tensor ids, Tensor wts) {
  CHECK_DT(x, at::kBFloat16, "x");
  CHECK_DT(wr, at::kBFloat16, "w_router");
  CHECK_DT(ids, at::kInt, "ids");
  CHECK_DT(wts, at::kFloat, "weights");
  TORCH_CHECK(x.dim() == 2 && x.stride(1) == 1 && wr.is_contiguous() && wr.size(1) == x.size(1), "moe_route: shapes");
  const int T = (int)x.size(0);
  TORCH_CHECK(ids.numel() >= T * K && wts.numel() >= T * K, "moe_route: outputs too small");
  const c10::cuda::CUDAGuard g(x.device());
  kapsl::launch_moe_route(bf(x), x.stride(0), bf(wr), T, (int)x.size(1), (int)wr.size(0), (int)K, renorm,
                          ids.data_ptr<int32_t>(), wts.data_ptr<float>(), cur_stream());
}

void moe_permute(Tensor ids, int64_t T, int64_t K, int64_t E, int64_t e_lo, int64_t el, int64_t max_rows, Tensor seg,
                 Tensor pos, Tensor mtiles, Tensor src, Tensor err) {
  for (auto* t : {&ids, &seg, &pos, &mtiles, &src}) CHECK_DT(*t, at::kInt, "moe_permute int32");
  TORCH_CHECK(ids.numel() >= T * K && pos.numel() >= T * K && seg.numel() >= E + 1, "moe_permute: sizes");
  TORCH_CHECK(mtiles.numel() >= 1 + max_rows / 128 && src.numel() >= max_rows, "moe_permute: tables too short");
  const c10::cuda::CUDAGuard g(ids.device());
  kapsl::launch_moe_permute(ids.data_ptr<int32_t>(), (int)T, (int)K, (int)E, (int)e_lo, (int)el, (int)max_rows,
                            seg.data_ptr<int32_t>(), pos.data_ptr<int32_t>(), mtiles.data_ptr<int32_t>(),
                            src.data_ptr<int32_t>(), err.data_ptr<int>(), cur_stream());
}

void moe_gather(Tensor x, Tensor src, Tensor mtiles, Tensor xs) {
  CHECK_DT(x, at::kBFloat16, "x");
  CHECK_DT(xs, at::kBFloat16, "xs");
  TORCH_CHECK(x.stride(1) == 1 && xs.stride(1) == 1 && xs.size(1) == x.size(1), "moe_gather: shapes");
  const c10::cuda::CUDAGuard g(x.device());
  kapsl::launch_moe_gather(bf(x), x.stride(0), src.data_ptr<int32_t>(), mtiles.data_ptr<int32_t>(), bf(xs),
                           xs.stride(0), (int)x.size(1), (int)xs.size(0), kapsl::gemm_num_sms(), cur_stream());
}

// y / hidden / flags: per-rank device addresses (world = len(y)); flags empty when world == 1.
void moe_combine(std::vector<int64_t> y, std::vector<int64_t> hidden, std::vector<int64_t> flags, int64_t rank,
                 Tensor ids, Tensor wts, Tensor pos, Tensor seg, int64_t T, int64_t K, int64_t el, int64_t cols,
                 int64_t ld_y, int64_t ld_h, int64_t rows_per_rank, c10::optional<Tensor> epoch_ctr, Tensor err,
                 int64_t timeout_ns) {
  const int world = (int)y.size();
  TORCH_CHECK(hidden.size() == y.size() && (world == 1 || flags.size() == y.size()), "moe_combine: tables differ");
  TORCH_CHECK(world == 1 || epoch_ctr.has_value(), "moe_combine: epoch counter needed for world > 1");
  const c10::cuda::CUDAGuard g(ids.device());
  auto yp = as_ptrs<const __nv_bfloat16>(y);
  auto hp = as_ptrs<__nv_bfloat16>(hidden);
  auto fp = as_ptrs<int64_t>(flags);
  kapsl::launch_moe_combine(yp.data(), hp.data(), world > 1 ? fp.data() : nullptr, world, (int)rank,
                            ids.data_ptr<int32_t>(), wts.data_ptr<float>(), pos.data_ptr<int32_t>(),
                            seg.data_ptr<int32_t>(), (int)T, (int)K, (int)el, (int)cols, ld_y, ld_h,
                            (int)rows_per_rank, epoch_ctr.has_value() ? epoch_ctr->data_ptr<int64_t>() : nullptr,
                            err.data_ptr<int>(), kapsl::gemm_num_sms(), (uint64_t)timeout_ns, cur_stream());
}

// Copy blocks src_ids[i] -> dst_ids[i] of every plane (layer x K/V) from the local
// pool `src` into the pool at `dst_ptr` (typically a peer GPU's pool mapped by CUDA IPC).
void kv_push(Tensor src, int64_t dst_ptr, Tensor src_ids, Tensor dst_ids, int64_t planes, int64_t dst_blocks_per_plane) {
  CHECK_DT(src_ids, at::kInt, "src_ids");
  CHECK_DT(dst_ids, at::kInt, "dst_ids");
  TORCH_CHECK(src.is_contiguous() && src.dim() >= 3, "kv_push: src pool [layers, 2, blocks, ...] contiguous");
  TORCH_CHECK(src_ids.numel() == dst_ids.numel(), "kv_push: id lists differ in length");
  const int64_t src_blocks = src.size(2);
  const int64_t block_bytes = src.numel() / (src.size(0) * src.size(1) * src_blocks) * src.element_size();
  TORCH_CHECK(planes == src.size(0) * src.size(1), "kv_push: plane count mismatch");
  const c10::cuda::CUDAGuard g(src.device());
  kapsl::launch_kv_push(src.data_ptr(), reinterpret_cast<void*>(dst_ptr), src_ids.data_ptr<int32_t>(),
                        dst_ids.data_ptr<int32_t>(), (int)src_ids.numel(), (int)planes, src_blocks,
                        dst_blocks_per_plane, block_bytes, kapsl::gemm_num_sms(), cur_stream());
}

// Block gather/scatter between any two device-accessible pools (this GPU's
// memory, a peer's through CUDA IPC, or pinned host memory through unified
// addressing): planes x blocks of block_bytes each, src_ids[i] -> dst_ids[i].
// Used for KV swap-out to and swap-in from host memory in one launch.
void kv_copy_blocks(int64_t src_ptr, int64_t dst_ptr, Tensor src_ids, Tensor dst_ids, int64_t planes,
                    int64_t src_blocks_per_plane, int64_t dst_blocks_per_plane, int64_t block_bytes) {
  CHECK_DT(src_ids, at::kInt, "src_ids");
  CHECK_DT(dst_ids, at::kInt, "dst_ids");
  TORCH_CHECK(src_ids.is_cuda() && dst_ids.is_cuda(), "kv_copy_blocks: id lists on the GPU");
  TORCH_CHECK(src_ids.numel() == dst_ids.numel(), "kv_copy_blocks: id lists differ in length");
  const c10::cuda::CUDAGuard g(src_ids.device());
  kapsl::launch_kv_push(reinterpret_cast<const void*>(src_ptr), reinterpret_cast<void*>(dst_ptr),
                        src_ids.data_ptr<int32_t>(), dst_ids.data_ptr<int32_t>(), (int)src_ids.numel(), (int)planes,
                        src_blocks_per_plane, dst_blocks_per_plane, block_bytes, kapsl::gemm_num_sms(), cur_stream());
}

// Asynchronous copy on the current stream (copy engine) between device addresses,
// either of which may be a peer GPU's memory mapped by CUDA IPC.
void copy_async(int64_t dst_ptr, int64_t src_ptr, int64_t bytes) {
  KAPSL_CHECK_CUDA(cudaMemcpyAsync(reinterpret_cast<void*>(dst_ptr), reinterpret_cast<const void*>(src_ptr),
                                   (size_t)bytes, cudaMemcpyDeviceToDevice, cur_stream()));
}

Tensor tensor_from_ptr(int64_t ptr, std::vector<int64_t> shape, std::string dtype, int64_t device) {
  at::ScalarType st;
  if (dtype == "bfloat16") st = at::kBFloat16;
  else if (dtype == "float32") st = at::kFloat;
  else if (dtype == "int64") st = at::kLong;
  else if (dtype == "int32") st = at::kInt;
  else TORCH_CHECK(false, "tensor_from_ptr: unsupported dtype ", dtype);
  auto opts = torch::TensorOptions().dtype(st).device(torch::kCUDA, device);
  return torch::from_blob(reinterpret_cast<void*>(ptr), shape, opts);
}

int64_t launch_count() { return (int64_t)kapsl::launch_count(); }
int64_t num_sms() { return kapsl::gemm_num_sms(); }

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "kapsl_sdk_b200 sm_100a kernels";
  m.def("rmsnorm", &rmsnorm, "RMSNorm (optionally residual += x first)", py::arg("out"), py::arg("x"),
        py::arg("weight"), py::arg("eps"), py::arg("residual") = py::none());
  m.def("rope_kv_write", &rope_kv_write, "RoPE on q/k in place + paged KV write");
  m.def("silu_mul", &silu_mul, "SwiGLU: out = silu(x[:, :F]) * x[:, F:]");
  m.def("embedding", &embedding, "embedding gather (rows outside the shard are zero)", py::arg("out"),
        py::arg("table"), py::arg("ids"), py::arg("vocab_start"), py::arg("src_rows") = py::none(),
        py::arg("prev_tokens") = py::none());
  m.def("decode_num_splits", &decode_num_splits);
  m.def("decode_attention", &decode_attention, "paged split-KV decode attention");
  m.def("prefill_attention", &prefill_attention, "paged chunked-prefill attention");
  m.def("sample", &sample, "top-k/top-p/temperature/penalty sampler with per-row LCG (vocab-parallel capable)");
  m.def("sample_merge", &sample_merge, "vocab-parallel sampler: merge all-gathered candidates, top-p, draw");
  m.def("sample_full_scratch_bytes", &sample_full_scratch_bytes);
  m.def("count_tokens", &count_tokens, "counts[rows[i], ids[i]] += 1 (+ first-occurrence lists)",
        py::arg("counts"), py::arg("rows"), py::arg("ids"), py::arg("occ") = py::none(),
        py::arg("occ_n") = py::none());
  m.def("gemm", &gemm, "tcgen05 GEMM C = epi(A @ B^T)");
  m.def("gemm_scatter", &gemm_scatter, "row-parallel GEMM storing rows into owner ranks' receive buffers");
  m.def("tp_reduce_ag", &tp_reduce_ag, "barrier + reduce own rows + residual + all-gather push + barrier");
  m.def("gemm_q4k", &gemm_q4k, "GEMM with GGUF Q4_K weights dequantized into TMEM inside the mainloop");
  m.def("q4k_quantize", &q4k_quantize, "bf16 -> GGUF Q4_K blocks");
  m.def("q4k_dequant", &q4k_dequant, "GGUF Q4_K blocks -> bf16");
  m.def("gemm_issue_probe", &gemm_issue_probe, "cycles per k slice of the 2-SM MMA thread (diagnostic)");
  m.def("mma_rate_probe", &mma_rate_probe, "cycles per cta_group::1 MMA of width n (diagnostic)");
  m.def("q4k_dequant_rows", &q4k_dequant_rows, "GGUF Q4_K weight matrix -> bf16 rows (tile-major input, SwiGLU layout)");
  m.def("grouped_gemm", &grouped_gemm, "grouped (per-expert) tcgen05 GEMM driven by a device tile table");
  m.def("moe_route", &moe_route, "router logits + top-k + softmax weights");
  m.def("moe_permute", &moe_permute, "stable expert sort of the top-k assignments (padded segments)");
  m.def("moe_gather", &moe_gather, "gather token rows into the expert-sorted buffer");
  m.def("moe_combine", &moe_combine, "weighted top-k combine + residual (+ peer pull and all-gather)");
  m.def("prefill_attention_tc", &prefill_attention_tc,
        "tcgen05 chunked-prefill attention (work items of prefill_attn_tc_tokens tokens)");
  m.def("prefill_attn_tc_tokens", &prefill_attn_tc_tokens, "query tokens per CTA of prefill_attention_tc");
  m.def("kv_push", &kv_push, "KV connector: copy pool blocks into a (peer) pool over NVLink");
  m.def("kv_copy_blocks", &kv_copy_blocks, "KV block gather/scatter between device-accessible pools (host swap)");
  m.def("copy_async", &copy_async, "cudaMemcpyAsync on the current stream (copy-engine baseline)");
  m.def("tp_pull_reduce_ag", &tp_pull_reduce_ag, "barrier + pull peers' partial rows + residual + all-gather push");
  m.def("tp_reduce_norm_ag", &tp_reduce_norm_ag,
        "barrier + pull peers' partial rows + residual (own rows) + RMSNorm + all-gather of the normed rows");
  m.def("flag_pingpong", &flag_pingpong, "NVLink flag round-trip latency probe (two ranks)");
  m.def("gemm_deferred", &gemm_deferred, "plain GEMM leaving split-K partials in the workspace; returns splits");
  m.def("tp_ll_norm", &tp_ll_norm,
        "one-shot row reduction + residual + RMSNorm with flag-carrying 8-byte lines (few rows)");
  m.def("tp_ll_slot_bytes", &kapsl::tp_ll_slot_bytes);
  m.def("p2p_copy", &p2p_copy, "16-byte vector copy between (possibly peer-mapped) device addresses");
  m.def("symm_alloc", &symm_alloc);
  m.def("symm_free", &symm_free);
  m.def("symm_handle", &symm_handle);
  m.def("symm_open", &symm_open);
  m.def("symm_close", &symm_close);
  m.def("tensor_from_ptr", &tensor_from_ptr);
  m.def("launch_count", &launch_count, "kernels launched through this library so far");
  m.def("num_sms", &num_sms);
}
