// fp32 CPU kernels of the CPU backend (see cpu_kernels.h).  In the Python
// module they run on OpenMP from PyTorch's libgomp, so the worker team that
// serves torch's GEMMs also serves these kernels; built without OpenMP (the
// standalone sanitizer build) they use a small persistent thread pool.
//
// Reference counterpart: crates/kapsl-kernels/src/attention/mod.rs:8-99 (naive
// f32 attention without a block table) and src/mlp/mod.rs:7-49 (SwiGLU); the
// reference runs everything else inside ONNX Runtime.  Here attention reads
// the paged KV cache directly through the block table with an online
// softmax (one pass over the keys), parallel over (query row, head).
#include "cpu_kernels.h"

#include <algorithm>
#include <cmath>
#include <cstring>
#include <condition_variable>
#include <functional>
#include <mutex>
#include <thread>
#include <vector>

#ifdef _OPENMP
#include <omp.h>
#endif

#ifdef __AVX2__
#include <immintrin.h>
#endif

namespace kapsl {
namespace cpu {

namespace {

#ifdef _OPENMP
// Items [0, n) in static contiguous chunks over at most one thread per `grain` items.
template <class F>
void parallel_for(int64_t n, int64_t grain, F&& body) {
  const int64_t parts = std::min<int64_t>(omp_get_max_threads(), std::max<int64_t>(1, n / std::max<int64_t>(grain, 1)));
  if (parts <= 1) {
    for (int64_t i = 0; i < n; ++i) body(i);
    return;
  }
  // the full team every time (a changing team size makes libgomp rebuild it);
  // threads past `parts` have no range
#pragma omp parallel
  {
    const int64_t id = omp_get_thread_num();
    if (id < parts) {
      const int64_t b = n * id / parts, e = n * (id + 1) / parts;
      for (int64_t i = b; i < e; ++i) body(i);
    }
  }
}
#else

// Persistent worker threads; parallel_for splits [0, n) into one contiguous
// range per thread (the calling thread takes the first).  Small ranges run
// inline.  (`#pragma omp simd` still vectorises the inner loops.)
class Pool {
 public:
  static Pool& get() {
    static Pool p;
    return p;
  }
  void run(int64_t n, int64_t min_per_thread, const std::function<void(int64_t, int64_t)>& fn) {
    const int64_t want = std::min<int64_t>((int64_t)workers_.size() + 1, std::max<int64_t>(1, n / min_per_thread));
    if (want <= 1) {
      fn(0, n);
      return;
    }
    std::unique_lock<std::mutex> call(call_mu_);  // one parallel region at a time
    {
      std::lock_guard<std::mutex> lk(mu_);
      fn_ = &fn;
      n_ = n;
      parts_ = want;
      pending_ = (int)want - 1;
      ++gen_;
    }
    cv_.notify_all();
    fn(0, chunk(0));
    std::unique_lock<std::mutex> lk(mu_);
    done_cv_.wait(lk, [&] { return pending_ == 0; });
  }

 private:
  Pool() {
    const unsigned hc = std::max(1u, std::thread::hardware_concurrency());
    for (unsigned i = 1; i < hc; ++i) workers_.emplace_back([this, i] { loop((int)i); });
  }
  ~Pool() {
    {
      std::lock_guard<std::mutex> lk(mu_);
      stop_ = true;
    }
    cv_.notify_all();
    for (auto& t : workers_) t.join();
  }
  int64_t chunk(int64_t part) const { return std::min(n_, (n_ * (part + 1) + parts_ - 1) / parts_); }
  void loop(int id) {
    uint64_t seen = 0;
    while (true) {
      const std::function<void(int64_t, int64_t)>* fn;
      int64_t b, e;
      {
        std::unique_lock<std::mutex> lk(mu_);
        cv_.wait(lk, [&] { return stop_ || gen_ != seen; });
        if (stop_) return;
        seen = gen_;
        if (id >= parts_) continue;
        fn = fn_;
        b = (n_ * id + parts_ - 1) / parts_;
        e = std::min(n_, (n_ * (id + 1) + parts_ - 1) / parts_);
      }
      if (b < e) (*fn)(b, e);
      std::lock_guard<std::mutex> lk(mu_);
      if (--pending_ == 0) done_cv_.notify_one();
    }
  }
  std::vector<std::thread> workers_;
  std::mutex mu_, call_mu_;
  std::condition_variable cv_, done_cv_;
  const std::function<void(int64_t, int64_t)>* fn_ = nullptr;
  int64_t n_ = 0, parts_ = 1;
  int pending_ = 0;
  uint64_t gen_ = 0;
  bool stop_ = false;
};

template <class F>
void parallel_for(int64_t n, int64_t min_per_thread, F&& body) {
  const std::function<void(int64_t, int64_t)> fn = [&](int64_t b, int64_t e) {
    for (int64_t i = b; i < e; ++i) body(i);
  };
  Pool::get().run(n, min_per_thread, fn);
}
#endif

}  // namespace

void rmsnorm(const float* x, const float* w, float* out, int64_t rows, int64_t d, float eps) {
  parallel_for(rows, 4, [&](int64_t r) {
    const float* xr = x + r * d;
    float* o = out + r * d;
    double ss = 0.0;
#pragma omp simd reduction(+ : ss)
    for (int64_t i = 0; i < d; ++i) ss += (double)xr[i] * xr[i];
    const float inv = 1.0f / std::sqrt((float)(ss / (double)d) + eps);
#pragma omp simd
    for (int64_t i = 0; i < d; ++i) o[i] = xr[i] * inv * w[i];
  });
}

void rope(float* x, const int64_t* pos, const float* cos_sin, int64_t T, int64_t H, int64_t D) {
  const int64_t half = D / 2;
  parallel_for(T * H, 16, [&](int64_t th) {
    {
      const int64_t t = th / H, h = th % H;
      const float* c = cos_sin + pos[t] * D;
      const float* s = c + half;
      float* v = x + (t * H + h) * D;
#pragma omp simd
      for (int64_t i = 0; i < half; ++i) {
        const float a = v[i], b = v[i + half];
        v[i] = a * c[i] - b * s[i];
        v[i + half] = b * c[i] + a * s[i];
      }
    }
  });
}

void kv_write(const float* k, const float* v, const int64_t* slots, float* k_cache, float* v_cache, int64_t T,
              int64_t Hkv, int64_t bs, int64_t D) {
  parallel_for(T * Hkv, 64, [&](int64_t th) {
    {
      const int64_t t = th / Hkv, h = th % Hkv;
      const int64_t slot = slots[t];
      if (slot < 0) return;
      const int64_t blk = slot / bs, off = slot % bs;
      const int64_t dst = ((blk * Hkv + h) * bs + off) * D;
      std::copy(k + (t * Hkv + h) * D, k + (t * Hkv + h + 1) * D, k_cache + dst);
      std::copy(v + (t * Hkv + h) * D, v + (t * Hkv + h + 1) * D, v_cache + dst);
    }
  });
}

void paged_attention(const float* q, const float* k_cache, const float* v_cache, const int64_t* row0,
                     const int64_t* nq, const int64_t* ctx, const int32_t* block_tables, int64_t max_blocks,
                     int64_t num_seqs, int64_t Hq, int64_t Hkv, int64_t bs, int64_t D, float scale, float* out) {
  // work items: (sequence, query index, head)
  std::vector<int64_t> seq_of_row, qi_of_row;
  for (int64_t s = 0; s < num_seqs; ++s)
    for (int64_t i = 0; i < nq[s]; ++i) {
      seq_of_row.push_back(s);
      qi_of_row.push_back(i);
    }
  const int64_t rows = (int64_t)seq_of_row.size();
  const int64_t group = Hq / Hkv;
  parallel_for(rows * Hq, 1, [&](int64_t rh) {
    const int64_t r = rh / Hq, h = rh % Hq;
    float acc[512];  // D <= 512
    const int64_t s = seq_of_row[r], i = qi_of_row[r];
    const int64_t row = row0[s] + i;
    const int64_t limit = ctx[s] - nq[s] + i + 1;  // keys [0, limit) are visible
    const int64_t kvh = h / group;
    const float* qv = q + (row * Hq + h) * D;
    const int32_t* bt = block_tables + s * max_blocks;
    float m = -INFINITY, l = 0.f;
    std::fill(acc, acc + D, 0.f);
    for (int64_t j = 0; j < limit; ++j) {
      const int64_t base = (((int64_t)bt[j / bs] * Hkv + kvh) * bs + j % bs) * D;
      const float* kv = k_cache + base;
      float dot = 0.f;
#pragma omp simd reduction(+ : dot)
      for (int64_t e = 0; e < D; ++e) dot += qv[e] * kv[e];
      const float sc = dot * scale;
      const float mn = std::max(m, sc);
      const float corr = std::exp(m - mn);  // exp(-inf) = 0 on the first key
      const float p = std::exp(sc - mn);
      l = l * corr + p;
      const float* vv = v_cache + base;
#pragma omp simd
      for (int64_t e = 0; e < D; ++e) acc[e] = acc[e] * corr + p * vv[e];
      m = mn;
    }
    float* o = out + (row * Hq + h) * D;
    const float inv = l > 0.f ? 1.f / l : 0.f;
#pragma omp simd
    for (int64_t e = 0; e < D; ++e) o[e] = acc[e] * inv;
  });
}

void silu_mul(const float* x, float* out, int64_t T, int64_t F) {
  // chunks of up to 1024 features of one row; a thread per 16 chunks at least
  const int64_t per_row = (F + 1023) / 1024;
  parallel_for(T * per_row, 16, [&](int64_t c) {
    const int64_t t = c / per_row, j0 = (c % per_row) * 1024, j1 = std::min<int64_t>(F, j0 + 1024);
    const float* g = x + t * 2 * F;
    const float* u = g + F;
    float* o = out + t * F;
#pragma omp simd
    for (int64_t j = j0; j < j1; ++j) o[j] = g[j] / (1.f + std::exp(-g[j])) * u[j];
  });
}

// ------------------------------------------------------------------ Q4_K
namespace {

constexpr int64_t kQK = 256, kQ4KBytes = 144;

// IEEE half -> float (exact; subnormals, infinities and NaN included).
inline float half_to_float(uint16_t h) {
  const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  uint32_t exp = (h >> 10) & 0x1Fu, man = h & 0x3FFu;
  uint32_t bits;
  if (exp == 0) {
    if (man == 0) {
      bits = sign;
    } else {  // subnormal: normalise
      int e = -1;
      do {
        ++e;
        man <<= 1;
      } while (!(man & 0x400u));
      bits = sign | ((uint32_t)(127 - 15 - e) << 23) | ((man & 0x3FFu) << 13);
    }
  } else if (exp == 31) {
    bits = sign | 0x7F800000u | (man << 13);
  } else {
    bits = sign | ((exp + 127 - 15) << 23) | (man << 13);
  }
  float f;
  std::memcpy(&f, &bits, 4);
  return f;
}

// Dequantize one 256-value block into out[0..255].
inline void q4k_block(const uint8_t* b, float* out) {
  uint16_t dh, mh;
  std::memcpy(&dh, b, 2);
  std::memcpy(&mh, b + 2, 2);
  const float d = half_to_float(dh), dmin = half_to_float(mh);
  const uint8_t* sc = b + 4;
  const uint8_t* qs = b + 16;
  for (int j = 0; j < 8; ++j) {
    uint8_t s, m;
    if (j < 4) {
      s = sc[j] & 63;
      m = sc[j + 4] & 63;
    } else {
      s = (sc[j + 4] & 0xF) | ((sc[j - 4] >> 6) << 4);
      m = (sc[j + 4] >> 4) | ((sc[j] >> 6) << 4);
    }
    const float ds = d * s, mm = dmin * m;
    const uint8_t* q = qs + (j / 2) * 32;
    const int shift = (j & 1) * 4;
    float* o = out + j * 32;
#pragma omp simd
    for (int i = 0; i < 32; ++i) o[i] = ds * (float)((q[i] >> shift) & 0xF) - mm;
  }
}

}  // namespace

namespace {

// 6-bit scale and min of sub-block j (0..7) of a Q4_K block's 12 scale bytes
inline void q4k_scale_min(const uint8_t* sc, int j, int* s, int* m) {
  if (j < 4) {
    *s = sc[j] & 63;
    *m = sc[j + 4] & 63;
  } else {
    *s = (sc[j + 4] & 0xF) | ((sc[j - 4] >> 6) << 4);
    *m = (sc[j + 4] >> 4) | ((sc[j] >> 6) << 4);
  }
}

// sum_j s[j] * (q_j . xq_j) over the 8 sub-blocks of one block; q_j are the low
// (even j) or high (odd j) nibbles of qs[(j / 2) * 32 .. + 32]
inline int32_t q4k_dot_q8(const uint8_t* qs, const int8_t* xq, const int* s) {
#ifdef __AVX2__
  const __m256i lo4 = _mm256_set1_epi8(0x0F);
  __m256i acc = _mm256_setzero_si256();
  for (int p = 0; p < 4; ++p) {
    const __m256i q = _mm256_loadu_si256((const __m256i*)(qs + p * 32));
    const __m256i ql = _mm256_and_si256(q, lo4), qh = _mm256_and_si256(_mm256_srli_epi16(q, 4), lo4);
    const __m256i xl = _mm256_loadu_si256((const __m256i*)(xq + p * 64));
    const __m256i xh = _mm256_loadu_si256((const __m256i*)(xq + p * 64 + 32));
    // u8 x s8 -> pairwise s16 (|.| <= 2 * 15 * 127), then x scale with pairwise s32 sums
    acc = _mm256_add_epi32(acc, _mm256_madd_epi16(_mm256_maddubs_epi16(ql, xl), _mm256_set1_epi16((short)s[2 * p])));
    acc = _mm256_add_epi32(acc,
                           _mm256_madd_epi16(_mm256_maddubs_epi16(qh, xh), _mm256_set1_epi16((short)s[2 * p + 1])));
  }
  const __m128i h = _mm_add_epi32(_mm256_castsi256_si128(acc), _mm256_extracti128_si256(acc, 1));
  const __m128i h2 = _mm_add_epi32(h, _mm_shuffle_epi32(h, 0x4E));
  return _mm_cvtsi128_si32(_mm_add_epi32(h2, _mm_shuffle_epi32(h2, 0xB1)));
#else
  int32_t total = 0;
  for (int j = 0; j < 8; ++j) {
    const uint8_t* q = qs + (j / 2) * 32;
    const int shift = (j & 1) * 4;
    int32_t d = 0;
    for (int i = 0; i < 32; ++i) d += ((q[i] >> shift) & 0xF) * xq[j * 32 + i];
    total += s[j] * d;
  }
  return total;
#endif
}

}  // namespace

namespace {

constexpr int64_t kQ6KBytes = 210;

// the 6-bit quants of one Q6_K block in value order (0..63)
inline void q6k_unpack(const uint8_t* b, uint8_t* q) {
  for (int h = 0; h < 2; ++h) {
    const uint8_t* L = b + h * 64;
    const uint8_t* H = b + 128 + h * 32;
    uint8_t* o = q + h * 128;
    for (int i = 0; i < 32; ++i) {
      o[i] = (uint8_t)((L[i] & 0xF) | ((H[i] & 3) << 4));
      o[32 + i] = (uint8_t)((L[32 + i] & 0xF) | (((H[i] >> 2) & 3) << 4));
      o[64 + i] = (uint8_t)((L[i] >> 4) | (((H[i] >> 4) & 3) << 4));
      o[96 + i] = (uint8_t)((L[32 + i] >> 4) | (((H[i] >> 6) & 3) << 4));
    }
  }
}

// sum_g scale_g * (q_g . xq_g) over the 16 groups of 16 values of one block
// (blk: the packed block; q: its unpacked quants, used without AVX2)
inline int32_t q6k_dot_q8(const uint8_t* blk, const uint8_t* q, const int8_t* xq, const int8_t* sc) {
#ifdef __AVX2__
  (void)q;
  const __m256i m4 = _mm256_set1_epi8(0x0F), m2 = _mm256_set1_epi8(0x03);
  __m256i acc = _mm256_setzero_si256();
  for (int h = 0; h < 2; ++h) {
    const __m256i L0 = _mm256_loadu_si256((const __m256i*)(blk + h * 64));
    const __m256i L1 = _mm256_loadu_si256((const __m256i*)(blk + h * 64 + 32));
    const __m256i H = _mm256_loadu_si256((const __m256i*)(blk + 128 + h * 32));
    // the four 32-value chunks of this half, in value order
    const __m256i qv[4] = {
        _mm256_or_si256(_mm256_and_si256(L0, m4), _mm256_slli_epi16(_mm256_and_si256(H, m2), 4)),
        _mm256_or_si256(_mm256_and_si256(L1, m4),
                        _mm256_slli_epi16(_mm256_and_si256(_mm256_srli_epi16(H, 2), m2), 4)),
        _mm256_or_si256(_mm256_and_si256(_mm256_srli_epi16(L0, 4), m4),
                        _mm256_slli_epi16(_mm256_and_si256(_mm256_srli_epi16(H, 4), m2), 4)),
        _mm256_or_si256(_mm256_and_si256(_mm256_srli_epi16(L1, 4), m4),
                        _mm256_slli_epi16(_mm256_and_si256(_mm256_srli_epi16(H, 6), m2), 4))};
    for (int j = 0; j < 4; ++j) {
      const int c = h * 4 + j;  // values 32c .. 32c + 31 = groups 2c, 2c + 1
      const __m256i xv = _mm256_loadu_si256((const __m256i*)(xq + c * 32));
      // pairwise u8 x s8 (|.| <= 2 * 63 * 127); lanes 0-7 hold group 2c, 8-15 group 2c + 1
      const __m256i p = _mm256_maddubs_epi16(qv[j], xv);
      const __m256i s = _mm256_set_m128i(_mm_set1_epi16(sc[2 * c + 1]), _mm_set1_epi16(sc[2 * c]));
      acc = _mm256_add_epi32(acc, _mm256_madd_epi16(p, s));
    }
  }
  const __m128i hs = _mm_add_epi32(_mm256_castsi256_si128(acc), _mm256_extracti128_si256(acc, 1));
  const __m128i h2 = _mm_add_epi32(hs, _mm_shuffle_epi32(hs, 0x4E));
  return _mm_cvtsi128_si32(_mm_add_epi32(h2, _mm_shuffle_epi32(h2, 0xB1)));
#else
  (void)blk;
  int32_t total = 0;
  for (int g = 0; g < 16; ++g) {
    int32_t d = 0;
    for (int i = 0; i < 16; ++i) d += q[g * 16 + i] * xq[g * 16 + i];
    total += sc[g] * d;
  }
  return total;
#endif
}

#ifdef __AVX2__
constexpr bool kUnpackForDot = false;
#else
constexpr bool kUnpackForDot = true;
#endif

// int8 activation blocks of 256 values: scale = max|x| / 127 and per-group sums
// (group = `group` values)
void quantize_rows_q8(const float* x, int64_t T, int64_t K, int group, std::vector<int8_t>& xq,
                      std::vector<float>& dx, std::vector<int32_t>& gsum) {
  const int64_t nb = K / kQK, ng = kQK / group;
  xq.resize((size_t)(T * K));
  dx.resize((size_t)(T * nb));
  gsum.resize((size_t)(T * nb * ng));
  parallel_for(T * nb, 4, [&](int64_t tb) {
    const float* xr = x + tb * kQK;
    float amax = 0.f;
    for (int i = 0; i < kQK; ++i) amax = std::max(amax, std::fabs(xr[i]));
    const float inv = amax > 0.f ? 127.f / amax : 0.f;
    dx[tb] = amax / 127.f;
    int8_t* q = xq.data() + tb * kQK;
    for (int64_t g = 0; g < ng; ++g) {
      int32_t sum = 0;
      for (int i = 0; i < group; ++i) {
        const int v = (int)std::nearbyint(xr[g * group + i] * inv);
        q[g * group + i] = (int8_t)std::max(-127, std::min(127, v));
        sum += q[g * group + i];
      }
      gsum[tb * ng + g] = sum;
    }
  });
}

}  // namespace

void q4k_matmul_q8(const float* x, const uint8_t* w, float* y, int64_t T, int64_t N, int64_t K) {
  const int64_t nb = K / kQK;
  std::vector<int8_t> xq;
  std::vector<float> dx;
  std::vector<int32_t> bsum;  // per 32 values
  quantize_rows_q8(x, T, K, 32, xq, dx, bsum);
  parallel_for(N, 16, [&](int64_t n) {
    const uint8_t* row = w + n * nb * kQ4KBytes;
    float acc[16];
    for (int64_t t0 = 0; t0 < T; t0 += 16) {
      const int64_t tn = std::min<int64_t>(16, T - t0);
      for (int64_t t = 0; t < tn; ++t) acc[t] = 0.f;
      for (int64_t b = 0; b < nb; ++b) {
        const uint8_t* blk = row + b * kQ4KBytes;
        uint16_t dh, mh;
        std::memcpy(&dh, blk, 2);
        std::memcpy(&mh, blk + 2, 2);
        const float d = half_to_float(dh), dmin = half_to_float(mh);
        int s[8], m[8];
        for (int j = 0; j < 8; ++j) q4k_scale_min(blk + 4, j, &s[j], &m[j]);
        for (int64_t t = 0; t < tn; ++t) {
          const int64_t tb = (t0 + t) * nb + b;
          const int32_t dot = q4k_dot_q8(blk + 16, xq.data() + tb * kQK, s);
          int32_t msum = 0;
          for (int j = 0; j < 8; ++j) msum += m[j] * bsum[tb * 8 + j];
          acc[t] += dx[tb] * (d * (float)dot - dmin * (float)msum);
        }
      }
      for (int64_t t = 0; t < tn; ++t) y[(t0 + t) * N + n] = acc[t];
    }
  });
}

void q6k_matmul_q8(const float* x, const uint8_t* w, float* y, int64_t T, int64_t N, int64_t K) {
  const int64_t nb = K / kQK;
  std::vector<int8_t> xq;
  std::vector<float> dx;
  std::vector<int32_t> gsum;  // per 16 values
  quantize_rows_q8(x, T, K, 16, xq, dx, gsum);
  parallel_for(N, 16, [&](int64_t n) {
    const uint8_t* row = w + n * nb * kQ6KBytes;
    alignas(32) uint8_t q[kQK];
    float acc[16];
    for (int64_t t0 = 0; t0 < T; t0 += 16) {
      const int64_t tn = std::min<int64_t>(16, T - t0);
      for (int64_t t = 0; t < tn; ++t) acc[t] = 0.f;
      for (int64_t b = 0; b < nb; ++b) {
        const uint8_t* blk = row + b * kQ6KBytes;
        if (kUnpackForDot) q6k_unpack(blk, q);
        const int8_t* sc = (const int8_t*)(blk + 192);
        uint16_t dh;
        std::memcpy(&dh, blk + 208, 2);
        const float d = half_to_float(dh);
        for (int64_t t = 0; t < tn; ++t) {
          const int64_t tb = (t0 + t) * nb + b;
          const int32_t dot = q6k_dot_q8(blk, q, xq.data() + tb * kQK, sc);
          int32_t off = 0;
          for (int g = 0; g < 16; ++g) off += sc[g] * gsum[tb * 16 + g];
          acc[t] += dx[tb] * d * (float)(dot - 32 * off);
        }
      }
      for (int64_t t = 0; t < tn; ++t) y[(t0 + t) * N + n] = acc[t];
    }
  });
}

void q6k_dequant_rows(const uint8_t* w, float* out, int64_t n0, int64_t n1, int64_t K) {
  const int64_t nb = K / kQK;
  parallel_for(n1 - n0, 8, [&](int64_t r) {
    const uint8_t* row = w + (n0 + r) * nb * kQ6KBytes;
    uint8_t q[kQK];
    for (int64_t b = 0; b < nb; ++b) {
      const uint8_t* blk = row + b * kQ6KBytes;
      q6k_unpack(blk, q);
      const int8_t* sc = (const int8_t*)(blk + 192);
      uint16_t dh;
      std::memcpy(&dh, blk + 208, 2);
      const float d = half_to_float(dh);
      float* o = out + r * K + b * kQK;
      for (int v = 0; v < kQK; ++v) o[v] = d * (float)sc[v / 16] * (float)((int)q[v] - 32);
    }
  });
}

namespace {

// q_b . xq_b for one 32-value Q8_0 block: s8 x s8 as |q| (u8, 128 for -128)
// times sign(xq, q) (xq is never -128, so negating it cannot overflow)
inline int32_t q80_dot_q8(const int8_t* q, const int8_t* xq) {
#ifdef __AVX2__
  const __m256i qv = _mm256_loadu_si256((const __m256i*)q);
  const __m256i xv = _mm256_loadu_si256((const __m256i*)xq);
  const __m256i p = _mm256_maddubs_epi16(_mm256_abs_epi8(qv), _mm256_sign_epi8(xv, qv));  // |.| <= 2 * 128 * 127
  const __m256i s = _mm256_madd_epi16(p, _mm256_set1_epi16(1));
  const __m128i h = _mm_add_epi32(_mm256_castsi256_si128(s), _mm256_extracti128_si256(s, 1));
  const __m128i h2 = _mm_add_epi32(h, _mm_shuffle_epi32(h, 0x4E));
  return _mm_cvtsi128_si32(_mm_add_epi32(h2, _mm_shuffle_epi32(h2, 0xB1)));
#else
  int32_t d = 0;
  for (int i = 0; i < 32; ++i) d += q[i] * xq[i];
  return d;
#endif
}

constexpr int64_t kQ80Bytes = 34;

}  // namespace

void q80_matmul_q8(const float* x, const uint8_t* w, float* y, int64_t T, int64_t N, int64_t K) {
  const int64_t nb = K / 32;
  std::vector<int8_t> xq;
  std::vector<float> dx;
  std::vector<int32_t> gsum;
  quantize_rows_q8(x, T, K, 32, xq, dx, gsum);
  parallel_for(N, 16, [&](int64_t n) {
    const uint8_t* row = w + n * nb * kQ80Bytes;
    float acc[16];
    for (int64_t t0 = 0; t0 < T; t0 += 16) {
      const int64_t tn = std::min<int64_t>(16, T - t0);
      for (int64_t t = 0; t < tn; ++t) acc[t] = 0.f;
      for (int64_t b8 = 0; b8 < nb / 8; ++b8) {  // one 256-value activation block = 8 weight blocks
        float d[8];
        for (int j = 0; j < 8; ++j) {
          uint16_t dh;
          std::memcpy(&dh, row + (b8 * 8 + j) * kQ80Bytes, 2);
          d[j] = half_to_float(dh);
        }
        for (int64_t t = 0; t < tn; ++t) {
          const int64_t tb = (t0 + t) * (K / kQK) + b8;
          const int8_t* xb = xq.data() + tb * kQK;
          float s = 0.f;
          for (int j = 0; j < 8; ++j)
            s += d[j] * (float)q80_dot_q8((const int8_t*)(row + (b8 * 8 + j) * kQ80Bytes + 2), xb + j * 32);
          acc[t] += dx[tb] * s;
        }
      }
      for (int64_t t = 0; t < tn; ++t) y[(t0 + t) * N + n] = acc[t];
    }
  });
}

void q80_dequant_rows(const uint8_t* w, float* out, int64_t n0, int64_t n1, int64_t K) {
  const int64_t nb = K / 32;
  parallel_for(n1 - n0, 8, [&](int64_t r) {
    const uint8_t* row = w + (n0 + r) * nb * kQ80Bytes;
    for (int64_t b = 0; b < nb; ++b) {
      uint16_t dh;
      std::memcpy(&dh, row + b * kQ80Bytes, 2);
      const float d = half_to_float(dh);
      const int8_t* q = (const int8_t*)(row + b * kQ80Bytes + 2);
      for (int i = 0; i < 32; ++i) out[r * K + b * 32 + i] = d * (float)q[i];
    }
  });
}

void q4k_dequant_rows(const uint8_t* w, float* out, int64_t n0, int64_t n1, int64_t K) {
  const int64_t nb = K / kQK;
  parallel_for(n1 - n0, 8, [&](int64_t r) {
    const uint8_t* row = w + (n0 + r) * nb * kQ4KBytes;
    for (int64_t b = 0; b < nb; ++b) q4k_block(row + b * kQ4KBytes, out + r * K + b * kQK);
  });
}

void q4k_matmul(const float* x, const uint8_t* w, float* y, int64_t T, int64_t N, int64_t K) {
  const int64_t nb = K / kQK;
  parallel_for(N, 16, [&](int64_t n) {
    float buf[kQK];
    float acc[16];
    const uint8_t* row = w + n * nb * kQ4KBytes;
    for (int64_t t0 = 0; t0 < T; t0 += 16) {  // up to 16 activation rows share each dequantized block
      const int64_t tn = std::min<int64_t>(16, T - t0);
      for (int64_t t = 0; t < tn; ++t) acc[t] = 0.f;
      for (int64_t b = 0; b < nb; ++b) {
        q4k_block(row + b * kQ4KBytes, buf);
        for (int64_t t = 0; t < tn; ++t) {
          const float* xr = x + (t0 + t) * K + b * kQK;
          float s = 0.f;
#pragma omp simd reduction(+ : s)
          for (int i = 0; i < kQK; ++i) s += xr[i] * buf[i];
          acc[t] += s;
        }
      }
      for (int64_t t = 0; t < tn; ++t) y[(t0 + t) * N + n] = acc[t];
    }
  });
}

}  // namespace cpu
}  // namespace kapsl
