// Tensor-parallel communication over NVLink peer memory (CUDA IPC mappings).
//
//  * symmetric buffers: each rank cudaMalloc's a region, exports its IPC handle,
//    and maps every peer's region; kernels get a table of peer base pointers.
//  * row-parallel reduction, fused with the residual add and the all-gather:
//      GEMM epilogue (gemm_sm100.cu, EPI_SCATTER) stores each partial tile row
//      into the receive slot [my_rank] of the rank that owns the row;
//      tp_reduce_ag_kernel then, on each rank:
//        1. barrier 1 ("my partials are out") with every peer,
//        2. sums the world_size partials of its own rows in fp32, adds the
//           residual, writes bf16 rows into its residual stream and pushes the
//           same rows into every peer's residual stream (all-gather),
//        3. barrier 2 ("my rows are out"), done by the last CTA to finish,
//      so when the kernel completes every rank holds the full reduced hidden
//      state.  Data crosses NVLink once in each direction (reduce-scatter +
//      all-gather volume, no extra HBM round trip for the partials).
//  * barriers: per-rank int64 flag words in symmetric memory, written with
//    st.release.sys into the peers and polled with ld.acquire.sys; every wait is
//    bounded by %globaltimer and records an error code instead of hanging.
//    Epochs live in device memory, so the kernels can be captured in CUDA graphs.
#include "common.cuh"
#include "kernels.h"

namespace kapsl {

using bf16 = __nv_bfloat16;

// flags layout per rank: [2 sites][8 peers] int64, then [2] epoch/done counters
struct TPArgs {
  bf16* recv[8];       // peer receive buffers: [world][rows_per_rank][ld] bf16 partials
  bf16* hidden[8];     // peer residual streams [rows_pad][ld] bf16
  int64_t* flags[8];   // peer flag words
  int world;
  int rank;
  int rows_per_rank;
  int rows_total;      // real rows (T)
  int cols;
  int64_t ld;
  int64_t* epoch_ctr;  // local: [0] epoch, [1] finished-CTA counter
  uint64_t timeout_ns; // limit of every wait on a peer flag; past it the kernel records an error and returns
  int* err;
};

__global__ void __launch_bounds__(256) tp_reduce_ag_kernel(TPArgs a) {
  griddep_entry();
  __shared__ int64_t epoch_sh;
  __shared__ int ok_sh;
  if (threadIdx.x == 0) {
    epoch_sh = a.epoch_ctr[0] + 1;
    ok_sh = 1;
    if (blockIdx.x == 0) {
      __threadfence_system();  // the previous kernel's peer stores are performed
      for (int p = 0; p < a.world; ++p) st_release_sys(a.flags[p] + 0 * 8 + a.rank, epoch_sh);
    }
    if (!wait_flags(a.flags[a.rank] + 0 * 8, a.world, epoch_sh, a.timeout_ns)) {
      ok_sh = 0;
      atomicExch(a.err, 30);
    }
  }
  __syncthreads();
  const int64_t epoch = epoch_sh;
  if (ok_sh) {
    // rows owned by this rank, 8 columns (16 B) per thread-iteration
    const int r0 = a.rank * a.rows_per_rank;
    const int nrows = max(0, min(a.rows_per_rank, a.rows_total - r0));
    const int chunks = a.cols / 8;
    const int64_t total = (int64_t)nrows * chunks;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
      const int lr = (int)(i / chunks), c = (int)(i % chunks);
      float acc[8];
      {
        const uint4 h = *reinterpret_cast<const uint4*>(a.hidden[a.rank] + (int64_t)(r0 + lr) * a.ld + c * 8);
        const __nv_bfloat162* hp = reinterpret_cast<const __nv_bfloat162*>(&h);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          float2 f = __bfloat1622float2(hp[j]);
          acc[2 * j] = f.x;
          acc[2 * j + 1] = f.y;
        }
      }
      const bf16* mine = a.recv[a.rank];
      for (int p = 0; p < a.world; ++p) {
        const uint4 v = *reinterpret_cast<const uint4*>(mine + ((int64_t)p * a.rows_per_rank + lr) * a.ld + c * 8);
        const __nv_bfloat162* vp = reinterpret_cast<const __nv_bfloat162*>(&v);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          float2 f = __bfloat1622float2(vp[j]);
          acc[2 * j] += f.x;
          acc[2 * j + 1] += f.y;
        }
      }
      uint4 o;
      o.x = pack_bf16(acc[0], acc[1]);
      o.y = pack_bf16(acc[2], acc[3]);
      o.z = pack_bf16(acc[4], acc[5]);
      o.w = pack_bf16(acc[6], acc[7]);
      for (int p = 0; p < a.world; ++p)  // local copy first (p == rank) is just another destination
        *reinterpret_cast<uint4*>(a.hidden[(a.rank + p) % a.world] + (int64_t)(r0 + lr) * a.ld + c * 8) = o;
    }
  }
  // last CTA to finish: barrier 2 (every rank's rows are out), then bump the epoch
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    const int64_t done = atomicAdd(reinterpret_cast<unsigned long long*>(&a.epoch_ctr[1]), 1ull);
    if (done == gridDim.x - 1) {
      for (int p = 0; p < a.world; ++p) st_release_sys(a.flags[p] + 1 * 8 + a.rank, epoch);
      if (!wait_flags(a.flags[a.rank] + 1 * 8, a.world, epoch, a.timeout_ns)) atomicExch(a.err, 31);
      a.epoch_ctr[1] = 0;
      a.epoch_ctr[0] = epoch;
      __threadfence();
    }
  }
}

// Pull variant: every rank's GEMM wrote its full partial [T, cols] into its own
// symmetric buffer (plain epilogue, local HBM bandwidth).  After barrier 1 each
// rank reads the partials of its own rows from all peers with P2P loads (many
// CTAs x 2 chunks in flight per thread), adds the residual, and pushes the
// reduced rows to every peer; barrier 2 as above.
template <int WORLD>
__global__ void __launch_bounds__(256) tp_pull_reduce_ag_kernel(TPArgs a) {
  griddep_entry();
  __shared__ int64_t epoch_sh;
  __shared__ int ok_sh;
  if (threadIdx.x == 0) {
    epoch_sh = a.epoch_ctr[0] + 1;
    ok_sh = 1;
    if (blockIdx.x == 0) {
      a.epoch_ctr[2] = (int64_t)globaltimer_ns();  // phase stamps for profiling
      __threadfence_system();
      for (int p = 0; p < a.world; ++p) st_release_sys(a.flags[p] + 0 * 8 + a.rank, epoch_sh);
    }
    if (!wait_flags(a.flags[a.rank] + 0 * 8, a.world, epoch_sh, a.timeout_ns)) {
      ok_sh = 0;
      atomicExch(a.err, 32);
    }
    if (blockIdx.x == 0) a.epoch_ctr[3] = (int64_t)globaltimer_ns();
  }
  __syncthreads();
  const int64_t epoch = epoch_sh;
  if (ok_sh) {
    const int r0 = a.rank * a.rows_per_rank;
    const int nrows = max(0, min(a.rows_per_rank, a.rows_total - r0));
    const int chunks = a.cols / 8;
    const int64_t total = (int64_t)nrows * chunks;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    const bf16* own_hidden = a.hidden[0];
#pragma unroll
    for (int p = 1; p < WORLD; ++p)
      if (p == a.rank) own_hidden = a.hidden[p];
    for (int64_t i0 = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i0 < total; i0 += 2 * stride) {
      uint4 v[2][WORLD];
      uint4 hres[2];
      int64_t off[2];
      bool live[2];
#pragma unroll
      for (int u = 0; u < 2; ++u) {  // issue all loads of two chunks before any use
        const int64_t i = i0 + u * stride;
        live[u] = i < total;
        const int64_t idx = live[u] ? i : i0;
        const int lr = (int)(idx / chunks), c = (int)(idx % chunks);
        off[u] = (int64_t)(r0 + lr) * a.ld + c * 8;
        hres[u] = *reinterpret_cast<const uint4*>(own_hidden + off[u]);
#pragma unroll
        for (int p = 0; p < WORLD; ++p) v[u][p] = *reinterpret_cast<const uint4*>(a.recv[p] + off[u]);
      }
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        if (!live[u]) continue;
        float acc[8];
        const __nv_bfloat162* hp = reinterpret_cast<const __nv_bfloat162*>(&hres[u]);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          float2 f = __bfloat1622float2(hp[j]);
          acc[2 * j] = f.x;
          acc[2 * j + 1] = f.y;
        }
#pragma unroll
        for (int p = 0; p < WORLD; ++p) {
          const __nv_bfloat162* vp = reinterpret_cast<const __nv_bfloat162*>(&v[u][p]);
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            float2 f = __bfloat1622float2(vp[j]);
            acc[2 * j] += f.x;
            acc[2 * j + 1] += f.y;
          }
        }
        uint4 o;
        o.x = pack_bf16(acc[0], acc[1]);
        o.y = pack_bf16(acc[2], acc[3]);
        o.z = pack_bf16(acc[4], acc[5]);
        o.w = pack_bf16(acc[6], acc[7]);
#pragma unroll
        for (int p = 0; p < WORLD; ++p) *reinterpret_cast<uint4*>(a.hidden[p] + off[u]) = o;
      }
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    const int64_t done = atomicAdd(reinterpret_cast<unsigned long long*>(&a.epoch_ctr[1]), 1ull);
    if (done == gridDim.x - 1) {
      a.epoch_ctr[4] = (int64_t)globaltimer_ns();
      for (int p = 0; p < a.world; ++p) st_release_sys(a.flags[p] + 1 * 8 + a.rank, epoch);
      if (!wait_flags(a.flags[a.rank] + 1 * 8, a.world, epoch, a.timeout_ns)) atomicExch(a.err, 33);
      a.epoch_ctr[5] = (int64_t)globaltimer_ns();
      // running sums over calls: barrier-1 wait (CTA 0), data phase (until the
      // last CTA retires), barrier-2 wait, number of calls
      a.epoch_ctr[8] += a.epoch_ctr[3] - a.epoch_ctr[2];
      a.epoch_ctr[9] += a.epoch_ctr[4] - a.epoch_ctr[3];
      a.epoch_ctr[10] += a.epoch_ctr[5] - a.epoch_ctr[4];
      a.epoch_ctr[11] += 1;
      a.epoch_ctr[1] = 0;
      a.epoch_ctr[0] = epoch;
      __threadfence();
    }
  }
}

// Pull reduction fused with the residual add, the next RMSNorm and the
// all-gather of the normed rows.  The residual stream is sharded by rows: this
// rank keeps (and updates) only the rows it owns; what every rank needs in
// full is the next GEMM's input x = rmsnorm(h) * w.  One CTA per owned row:
//   pass 1  h_row += sum over ranks of their partial rows (P2P loads), rounded
//           to bf16 and stored back; sum of squares of the rounded values
//   pass 2  x_row = h_row * rsqrt(mean + eps) * w, stored into every rank's x
// between the usual two flag barriers (partials out / x rows out).
struct TPNormArgs {
  const bf16* partial[8];  // peers' partial sums [rows_pad][ld] (their GEMM outputs)
  bf16* xout[8];           // peers' normed-input buffers [rows_pad][ld]
  int64_t* flags[8];
  bf16* h;                 // local residual stream (rows owned by this rank are kept current)
  const bf16* w;           // RMSNorm weight [cols]
  float eps;
  int world, rank, rows_per_rank, rows_total, cols;
  int64_t ld;
  int64_t* epoch_ctr;
  uint64_t timeout_ns;
  int* err;
};

static constexpr int kNormThreads = 256;
static constexpr int kNormMaxChunks = 4;  // 16-byte chunks per thread: cols <= 8 * 256 * 4 = 8192

template <int WORLD>
__global__ void __launch_bounds__(kNormThreads) tp_reduce_norm_ag_kernel(TPNormArgs a) {
  griddep_entry();
  __shared__ int64_t epoch_sh;
  __shared__ int ok_sh;
  __shared__ float red[kNormThreads / 32];
  if (threadIdx.x == 0) {
    epoch_sh = a.epoch_ctr[0] + 1;
    ok_sh = 1;
    if (blockIdx.x == 0) {
      a.epoch_ctr[2] = (int64_t)globaltimer_ns();
      __threadfence_system();
      for (int p = 0; p < WORLD; ++p) st_release_sys(a.flags[p] + 0 * 8 + a.rank, epoch_sh);
    }
    if (!wait_flags(a.flags[a.rank] + 0 * 8, WORLD, epoch_sh, a.timeout_ns)) {
      ok_sh = 0;
      atomicExch(a.err, 34);
    }
    if (blockIdx.x == 0) a.epoch_ctr[3] = (int64_t)globaltimer_ns();
  }
  __syncthreads();
  const int64_t epoch = epoch_sh;
  if (ok_sh) {
    const int r0 = a.rank * a.rows_per_rank;
    const int nrows = max(0, min(a.rows_per_rank, a.rows_total - r0));
    const int chunks = a.cols / 8;
    const int tid = threadIdx.x;
    for (int lr = blockIdx.x; lr < nrows; lr += gridDim.x) {
      const int64_t base = (int64_t)(r0 + lr) * a.ld;
      uint4 hb[kNormMaxChunks];
      float ss = 0.f;
#pragma unroll
      for (int j0 = 0; j0 < kNormMaxChunks; j0 += 2) {
        uint4 v[2][WORLD];
        uint4 hr[2];
#pragma unroll
        for (int u = 0; u < 2; ++u) {  // every load of two chunks in flight before any use
          const int c = tid + (j0 + u) * kNormThreads;
          if (c < chunks) {
            hr[u] = *reinterpret_cast<const uint4*>(a.h + base + c * 8);
#pragma unroll
            for (int p = 0; p < WORLD; ++p) v[u][p] = *reinterpret_cast<const uint4*>(a.partial[p] + base + c * 8);
          }
        }
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          const int c = tid + (j0 + u) * kNormThreads;
          if (c >= chunks) continue;
          float acc[8];
          const __nv_bfloat162* hp = reinterpret_cast<const __nv_bfloat162*>(&hr[u]);
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const float2 f = __bfloat1622float2(hp[j]);
            acc[2 * j] = f.x;
            acc[2 * j + 1] = f.y;
          }
#pragma unroll
          for (int p = 0; p < WORLD; ++p) {
            const __nv_bfloat162* vp = reinterpret_cast<const __nv_bfloat162*>(&v[u][p]);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const float2 f = __bfloat1622float2(vp[j]);
              acc[2 * j] += f.x;
              acc[2 * j + 1] += f.y;
            }
          }
          uint4 o;
          o.x = pack_bf16(acc[0], acc[1]);
          o.y = pack_bf16(acc[2], acc[3]);
          o.z = pack_bf16(acc[4], acc[5]);
          o.w = pack_bf16(acc[6], acc[7]);
          *reinterpret_cast<uint4*>(a.h + base + c * 8) = o;
          hb[j0 + u] = o;
          const __nv_bfloat162* op = reinterpret_cast<const __nv_bfloat162*>(&o);
#pragma unroll
          for (int j = 0; j < 4; ++j) {  // the norm sees the rounded residual, as a separate pass would
            const float2 f = __bfloat1622float2(op[j]);
            ss += f.x * f.x + f.y * f.y;
          }
        }
      }
      ss = warp_sum(ss);
      if ((tid & 31) == 0) red[tid >> 5] = ss;
      __syncthreads();
      float tot = 0.f;
#pragma unroll
      for (int i = 0; i < kNormThreads / 32; ++i) tot += red[i];
      const float inv = rsqrtf(tot / (float)a.cols + a.eps);
#pragma unroll
      for (int j = 0; j < kNormMaxChunks; ++j) {
        const int c = tid + j * kNormThreads;
        if (c >= chunks) continue;
        const uint4 wv = *reinterpret_cast<const uint4*>(a.w + c * 8);
        const __nv_bfloat162* wp = reinterpret_cast<const __nv_bfloat162*>(&wv);
        const __nv_bfloat162* hp = reinterpret_cast<const __nv_bfloat162*>(&hb[j]);
        uint4 o;
        uint32_t* ow = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float2 hv = __bfloat1622float2(hp[q]);
          const float2 fw = __bfloat1622float2(wp[q]);
          ow[q] = pack_bf16(hv.x * inv * fw.x, hv.y * inv * fw.y);
        }
#pragma unroll
        for (int p = 0; p < WORLD; ++p) *reinterpret_cast<uint4*>(a.xout[p] + base + c * 8) = o;
      }
      __syncthreads();  // red[] is reused by the next row
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    const int64_t done = atomicAdd(reinterpret_cast<unsigned long long*>(&a.epoch_ctr[1]), 1ull);
    if (done == gridDim.x - 1) {
      a.epoch_ctr[4] = (int64_t)globaltimer_ns();
      for (int p = 0; p < WORLD; ++p) st_release_sys(a.flags[p] + 1 * 8 + a.rank, epoch);
      if (!wait_flags(a.flags[a.rank] + 1 * 8, WORLD, epoch, a.timeout_ns)) atomicExch(a.err, 35);
      a.epoch_ctr[5] = (int64_t)globaltimer_ns();
      a.epoch_ctr[8] += a.epoch_ctr[3] - a.epoch_ctr[2];
      a.epoch_ctr[9] += a.epoch_ctr[4] - a.epoch_ctr[3];
      a.epoch_ctr[10] += a.epoch_ctr[5] - a.epoch_ctr[4];
      a.epoch_ctr[11] += 1;
      a.epoch_ctr[1] = 0;
      a.epoch_ctr[0] = epoch;
      __threadfence();
    }
  }
}

void launch_tp_reduce_norm_ag(const bf16* const* partial, bf16* const* xout, int64_t* const* flags, bf16* h,
                              const bf16* w, float eps, int world, int rank, int rows_per_rank, int rows_total,
                              int cols, int64_t ld, int64_t* epoch_ctr, int* err, int num_sms, uint64_t timeout_ns,
                              cudaStream_t st) {
  if (world > 8) throw std::runtime_error("tp: at most 8 ranks");
  if (cols % 8 != 0 || ld % 8 != 0) throw std::runtime_error("tp: columns must be a multiple of 8");
  if (cols / 8 > kNormThreads * kNormMaxChunks) throw std::runtime_error("tp: hidden size above 8192");
  TPNormArgs a{};
  for (int i = 0; i < world; ++i) {
    a.partial[i] = partial[i];
    a.xout[i] = xout[i];
    a.flags[i] = flags[i];
  }
  a.h = h;
  a.w = w;
  a.eps = eps;
  a.world = world;
  a.rank = rank;
  a.rows_per_rank = rows_per_rank;
  a.rows_total = rows_total;
  a.cols = cols;
  a.ld = ld;
  a.epoch_ctr = epoch_ctr;
  a.timeout_ns = timeout_ns;
  a.err = err;
  int grid = std::min(rows_per_rank, num_sms * 4);
  if (grid < 1) grid = 1;
  switch (world) {
    case 2: launch_k(tp_reduce_norm_ag_kernel<2>, grid, kNormThreads, 0, st, a); break;
    case 4: launch_k(tp_reduce_norm_ag_kernel<4>, grid, kNormThreads, 0, st, a); break;
    case 8: launch_k(tp_reduce_norm_ag_kernel<8>, grid, kNormThreads, 0, st, a); break;
    default: throw std::runtime_error("tp: fused norm reduction needs world size 2, 4 or 8");
  }
  KAPSL_LAUNCH_CHECK();
  note_launch();
}

__device__ __forceinline__ void add_bf16x8(float (&acc)[8], const uint4& v) {
  const __nv_bfloat162* vp = reinterpret_cast<const __nv_bfloat162*>(&v);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float2 f = __bfloat1622float2(vp[j]);
    acc[2 * j] += f.x;
    acc[2 * j + 1] += f.y;
  }
}

// Low-latency variants for decode-sized row counts: the data carries its own
// flag.  Every 16-byte store holds two 8-byte lines {4 bytes of data, 4 bytes of
// the call's epoch}; a reader polls the lines themselves until both flags equal
// the epoch, so there is no fence and no separate flag word.  An aligned 8-byte
// line is never seen half written.  Slots are double-buffered by epoch parity (a
// stale line carries epoch - 2, never the current value).  Twice the bytes of a
// plain copy, so these are for few rows.  CTA b of every rank handles rows
// r = b, b + G, ... (the same G everywhere) and waits only for CTA b of peers.
//  one-shot (TWO = false): push this rank's partial rows to every peer's slot
//    [parity][my rank]; reduce + norm every row of CTA b from the polled lines.
//    Reuse: a rank reaches call e+2 only after reading every peer's lines of
//    call e+1, which those peers stored after finishing their reads of call e.
//  two-shot (TWO = true): push the partial rows another rank owns into its
//    reduce slot [parity][my rank]; reduce + norm the owned rows of CTA b, store
//    them locally and push them as lines into every peer's gather slot
//    [parity][row]; copy the other owners' normed rows of CTA b out of the
//    local gather slot.  Reuse: a rank reaches call e+2 after receiving every
//    owner's normed rows of call e+1, produced after those owners read call e.
struct TPLLArgs {
  const bf16* own;      // this rank's partial [rows][ld] (when splits == 0)
  const float* ws;      // or the GEMM's fp32 split-K partials [splits][rows][cols], summed here
  int splits;
  uint4* slot[8];       // peers' reduce slots [2][W][cap][cols / 4] (16 B = two lines = 4 values)
  uint4* gslot[8];      // two-shot: peers' gather slots [2][W * cap][cols / 4]
  bf16* h;              // residual stream (one-shot: every row; two-shot: owned rows kept current)
  bf16* xout;           // local normed-input buffer
  const bf16* w;
  float eps;
  int rank, rows_total, rows_per_rank, cols, cap;
  int64_t ld;
  int64_t* epoch_ctr;
  uint64_t timeout_ns;
  int* err;
};

__device__ __forceinline__ void st_volatile_v4(uint4* p, const uint4& v) {
  asm volatile("st.volatile.global.v4.u32 [%0], {%1, %2, %3, %4};" ::"l"(p), "r"(v.x), "r"(v.y), "r"(v.z),
               "r"(v.w)
               : "memory");
}
__device__ __forceinline__ uint4 ld_volatile_v4(const uint4* p) {
  uint4 v;
  asm volatile("ld.volatile.global.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p)
               : "memory");
  return v;
}
__device__ __forceinline__ void ll_store(uint4* dst, const uint4& v, uint32_t fl) {
  st_volatile_v4(dst, make_uint4(v.x, fl, v.y, fl));
  st_volatile_v4(dst + 1, make_uint4(v.z, fl, v.w, fl));
}
// Polls the two lines pairs at src until they carry flag fl; false (and error 38)
// once the call has waited longer than timeout_ns.
__device__ __forceinline__ bool ll_load(const uint4* src, uint32_t fl, uint64_t t0, uint64_t timeout_ns,
                                        bool ok, int* err, uint4& out) {
  uint4 l0 = ld_volatile_v4(src), l1 = ld_volatile_v4(src + 1);
  int spins = 0;
  while (ok && (l0.y != fl || l0.w != fl || l1.y != fl || l1.w != fl)) {
    if (++spins == 64) {
      spins = 0;
      if (globaltimer_ns() - t0 > timeout_ns) {
        ok = false;
        atomicExch(err, 38);
      }
    }
    l0 = ld_volatile_v4(src);
    l1 = ld_volatile_v4(src + 1);
  }
  out = make_uint4(l0.x, l0.z, l1.x, l1.z);
  return ok;
}

// 16-byte chunk c (8 columns) of this rank's partial row r: the bf16 GEMM output, or
// the sum of the split-K partials in split order rounded to bf16 (the arithmetic of
// the split-K reduce kernel, so every reduction variant sees the same values).
__device__ __forceinline__ uint4 own_chunk(const TPLLArgs& a, int r, int c) {
  if (a.splits == 0) return *reinterpret_cast<const uint4*>(a.own + (int64_t)r * a.ld + c * 8);
  const int64_t sstride = (int64_t)a.rows_total * a.cols;
  const float* p = a.ws + (int64_t)r * a.cols + c * 8;
  float4 lo = reinterpret_cast<const float4*>(p)[0], hi = reinterpret_cast<const float4*>(p)[1];
  for (int sp = 1; sp < a.splits; ++sp) {
    const float4 l2 = reinterpret_cast<const float4*>(p + sp * sstride)[0];
    const float4 h2 = reinterpret_cast<const float4*>(p + sp * sstride)[1];
    lo.x += l2.x; lo.y += l2.y; lo.z += l2.z; lo.w += l2.w;
    hi.x += h2.x; hi.y += h2.y; hi.z += h2.z; hi.w += h2.w;
  }
  return make_uint4(pack_bf16(lo.x, lo.y), pack_bf16(lo.z, lo.w), pack_bf16(hi.x, hi.y), pack_bf16(hi.z, hi.w));
}

template <int WORLD, bool TWO>
__global__ void __launch_bounds__(kNormThreads) tp_ll_norm_kernel(TPLLArgs a) {
  griddep_entry();
  __shared__ int64_t epoch_sh;
  __shared__ float red[kNormThreads / 32];
  const int tid = threadIdx.x, b = blockIdx.x, G = gridDim.x;
  if (tid == 0) {
    epoch_sh = a.epoch_ctr[0] + 1;
    if (b == 0) a.epoch_ctr[2] = (int64_t)globaltimer_ns();
  }
  __syncthreads();
  const int64_t epoch = epoch_sh;
  const uint32_t fl = (uint32_t)epoch;
  const int par = (int)(epoch & 1);
  const int chunks = a.cols / 8;  // 16-byte chunks of bf16 = two line pairs each
  const int lines = a.cols / 4;   // uint4 per row in a slot
  const int rpr = a.rows_per_rank;
  // phase 1: push this rank's partial rows of CTA b
  for (int r = b; r < a.rows_total; r += G) {
    const int owner = TWO ? r / rpr : -1;
    if (TWO && owner == a.rank) continue;
    for (int c = tid; c < chunks; c += kNormThreads) {
      const uint4 v = own_chunk(a, r, c);
      if (TWO) {
        ll_store(a.slot[owner] + (((int64_t)par * WORLD + a.rank) * a.cap + (r - owner * rpr)) * lines + 2 * c, v, fl);
      } else {
#pragma unroll
        for (int q = 1; q < WORLD; ++q) {
          const int p = (a.rank + q) % WORLD;
          ll_store(a.slot[p] + (((int64_t)par * WORLD + a.rank) * a.cap + r) * lines + 2 * c, v, fl);
        }
      }
    }
  }
  if (tid == 0 && b == 0) a.epoch_ctr[3] = (int64_t)globaltimer_ns();
  // phase 2: reduce + norm the rows of CTA b (two-shot: the owned ones)
  bool ok = true;
  const uint64_t t0 = globaltimer_ns();
  int r = b;
  if (TWO) {
    const int r0 = a.rank * rpr;
    r = r0 + ((b - r0 % G) % G + G) % G;
  }
  const int rend = TWO ? min(a.rows_total, (a.rank + 1) * rpr) : a.rows_total;
  for (; r < rend; r += G) {
    const int64_t base = (int64_t)r * a.ld;
    const int lr = TWO ? r - a.rank * rpr : r;
    uint4 hb[kNormMaxChunks];
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < kNormMaxChunks; ++j) {
      const int c = tid + j * kNormThreads;
      if (c >= chunks) continue;
      uint4 v[WORLD];
#pragma unroll
      for (int p = 0; p < WORLD; ++p) {
        if (p == a.rank) {
          v[p] = own_chunk(a, r, c);
        } else {
          const uint4* src = a.slot[a.rank] + (((int64_t)par * WORLD + p) * a.cap + lr) * lines + 2 * c;
          ok = ll_load(src, fl, t0, a.timeout_ns, ok, a.err, v[p]);
        }
      }
      const uint4 hr = *reinterpret_cast<const uint4*>(a.h + base + c * 8);
      float acc[8];
      const __nv_bfloat162* hp = reinterpret_cast<const __nv_bfloat162*>(&hr);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float2 f = __bfloat1622float2(hp[q]);
        acc[2 * q] = f.x;
        acc[2 * q + 1] = f.y;
      }
#pragma unroll
      for (int p = 0; p < WORLD; ++p) add_bf16x8(acc, v[p]);
      uint4 o;
      o.x = pack_bf16(acc[0], acc[1]);
      o.y = pack_bf16(acc[2], acc[3]);
      o.z = pack_bf16(acc[4], acc[5]);
      o.w = pack_bf16(acc[6], acc[7]);
      *reinterpret_cast<uint4*>(a.h + base + c * 8) = o;
      hb[j] = o;
      const __nv_bfloat162* op = reinterpret_cast<const __nv_bfloat162*>(&o);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float2 f = __bfloat1622float2(op[q]);
        ss += f.x * f.x + f.y * f.y;
      }
    }
    ss = warp_sum(ss);
    if ((tid & 31) == 0) red[tid >> 5] = ss;
    __syncthreads();
    float tot = 0.f;
#pragma unroll
    for (int i = 0; i < kNormThreads / 32; ++i) tot += red[i];
    const float inv = rsqrtf(tot / (float)a.cols + a.eps);
#pragma unroll
    for (int j = 0; j < kNormMaxChunks; ++j) {
      const int c = tid + j * kNormThreads;
      if (c >= chunks) continue;
      const uint4 wv = *reinterpret_cast<const uint4*>(a.w + c * 8);
      const __nv_bfloat162* wp = reinterpret_cast<const __nv_bfloat162*>(&wv);
      const __nv_bfloat162* hp = reinterpret_cast<const __nv_bfloat162*>(&hb[j]);
      uint4 o;
      uint32_t* ow = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float2 hv = __bfloat1622float2(hp[q]);
        const float2 fw = __bfloat1622float2(wp[q]);
        ow[q] = pack_bf16(hv.x * inv * fw.x, hv.y * inv * fw.y);
      }
      *reinterpret_cast<uint4*>(a.xout + base + c * 8) = o;
      if (TWO) {
#pragma unroll
        for (int q = 1; q < WORLD; ++q) {
          const int p = (a.rank + q) % WORLD;
          ll_store(a.gslot[p] + ((int64_t)par * WORLD * a.cap + r) * lines + 2 * c, o, fl);
        }
      }
    }
    __syncthreads();
  }
  if (tid == 0 && b == 0) a.epoch_ctr[4] = (int64_t)globaltimer_ns();
  // phase 3 (two-shot): the other owners' normed rows of CTA b, out of the local gather slot
  if (TWO) {
    for (int rr = b; rr < a.rows_total; rr += G) {
      if (rr / rpr == a.rank) continue;
      for (int c = tid; c < chunks; c += kNormThreads) {
        uint4 v;
        ok = ll_load(a.gslot[a.rank] + ((int64_t)par * WORLD * a.cap + rr) * lines + 2 * c, fl, t0, a.timeout_ns, ok,
                     a.err, v);
        *reinterpret_cast<uint4*>(a.xout + (int64_t)rr * a.ld + c * 8) = v;
      }
    }
  }
  __syncthreads();
  if (tid == 0) {
    if (b == 0) {  // running sums: push phase, reduce phase, gather phase, calls
      const int64_t t5 = (int64_t)globaltimer_ns();
      a.epoch_ctr[8] += a.epoch_ctr[3] - a.epoch_ctr[2];
      a.epoch_ctr[9] += a.epoch_ctr[4] - a.epoch_ctr[3];
      a.epoch_ctr[10] += t5 - a.epoch_ctr[4];
      a.epoch_ctr[11] += 1;
    }
    __threadfence();
    const int64_t done = atomicAdd(reinterpret_cast<unsigned long long*>(&a.epoch_ctr[1]), 1ull);
    if (done == G - 1) {
      a.epoch_ctr[1] = 0;
      a.epoch_ctr[0] = epoch;
      __threadfence();
    }
  }
}

// bytes of one rank's LL region: reduce slots then gather slots (two-shot only)
size_t tp_ll_slot_bytes(int world, int cap, int cols, bool two) {
  const size_t red = (size_t)2 * world * cap * (size_t)cols * 4;
  return two ? 2 * red : red;
}

void launch_tp_ll_norm(const bf16* own, const float* ws, int splits, void* const* slot, void* const* gslot, bf16* h,
                       bf16* xout, const bf16* w, float eps, int world, int rank, int rows_per_rank, int rows_total,
                       int cols, int64_t ld, int cap, bool two, int64_t* epoch_ctr, int* err, int num_sms,
                       uint64_t timeout_ns, cudaStream_t st) {
  if (world != 2 && world != 4 && world != 8) throw std::runtime_error("tp: LL reduction needs world size 2, 4 or 8");
  if (cols % 8 != 0 || ld % 8 != 0) throw std::runtime_error("tp: columns must be a multiple of 8");
  if (cols / 8 > kNormThreads * kNormMaxChunks) throw std::runtime_error("tp: hidden size above 8192");
  if (!two && rows_total > cap) throw std::runtime_error("tp: LL rows exceed the slot capacity");
  if (two && (rows_per_rank > cap || (int64_t)rows_per_rank * world < rows_total))
    throw std::runtime_error("tp: LL two-shot rows per rank exceed the slot capacity");
  if (rows_total <= 0) return;
  if (splits > 1 && ws == nullptr) throw std::runtime_error("tp: split-K partials without a workspace");
  TPLLArgs a{};
  a.own = own;
  a.ws = ws;
  a.splits = splits > 1 ? splits : 0;
  for (int i = 0; i < world; ++i) {
    a.slot[i] = reinterpret_cast<uint4*>(slot[i]);
    a.gslot[i] = two ? reinterpret_cast<uint4*>(gslot[i]) : nullptr;
  }
  a.h = h;
  a.xout = xout;
  a.w = w;
  a.eps = eps;
  a.rank = rank;
  a.rows_total = rows_total;
  a.rows_per_rank = rows_per_rank;
  a.cols = cols;
  a.cap = cap;
  a.ld = ld;
  a.epoch_ctr = epoch_ctr;
  a.timeout_ns = timeout_ns;
  a.err = err;
  // every CTA resident (CTA b waits for CTA b of the peers): at most one per SM
  const int grid = std::max(1, std::min(rows_total, num_sms));
#define KAPSL_LL_LAUNCH(W)                                                                                  \
  two ? launch_k(tp_ll_norm_kernel<W, true>, grid, kNormThreads, 0, st, a)                                 \
      : launch_k(tp_ll_norm_kernel<W, false>, grid, kNormThreads, 0, st, a)
  switch (world) {
    case 2: KAPSL_LL_LAUNCH(2); break;
    case 4: KAPSL_LL_LAUNCH(4); break;
    default: KAPSL_LL_LAUNCH(8); break;
  }
#undef KAPSL_LL_LAUNCH
  KAPSL_LAUNCH_CHECK();
  note_launch();
}

void launch_tp_pull_reduce_ag(bf16* const* partial, bf16* const* hidden, int64_t* const* flags, int world, int rank,
                              int rows_per_rank, int rows_total, int cols, int64_t ld, int64_t* epoch_ctr, int* err,
                              int num_sms, uint64_t timeout_ns, cudaStream_t st) {
  if (world > 8) throw std::runtime_error("tp: at most 8 ranks");
  if (cols % 8 != 0 || ld % 8 != 0) throw std::runtime_error("tp: columns must be a multiple of 8");
  TPArgs a{};
  for (int i = 0; i < world; ++i) {
    a.recv[i] = partial[i];
    a.hidden[i] = hidden[i];
    a.flags[i] = flags[i];
  }
  a.world = world;
  a.rank = rank;
  a.rows_per_rank = rows_per_rank;
  a.rows_total = rows_total;
  a.cols = cols;
  a.ld = ld;
  a.epoch_ctr = epoch_ctr;
  a.timeout_ns = timeout_ns;
  a.err = err;
  const int64_t work = (int64_t)rows_per_rank * (cols / 8);
  // at most 4 CTAs of 256 threads per SM: every CTA is resident, so the barrier cannot deadlock
  int grid = (int)std::min<int64_t>((work + 511) / 512, (int64_t)num_sms * 4);
  if (grid < 1) grid = 1;
  switch (world) {
    case 1: launch_k(tp_pull_reduce_ag_kernel<1>, grid, 256, 0, st, a); break;
    case 2: launch_k(tp_pull_reduce_ag_kernel<2>, grid, 256, 0, st, a); break;
    case 4: launch_k(tp_pull_reduce_ag_kernel<4>, grid, 256, 0, st, a); break;
    case 8: launch_k(tp_pull_reduce_ag_kernel<8>, grid, 256, 0, st, a); break;
    default: throw std::runtime_error("tp: world size must be 1, 2, 4 or 8");
  }
  KAPSL_LAUNCH_CHECK();
  note_launch();
}

void launch_tp_reduce_ag(bf16* const* recv, bf16* const* hidden, int64_t* const* flags, int world, int rank,
                         int rows_per_rank, int rows_total, int cols, int64_t ld, int64_t* epoch_ctr, int* err,
                         int num_sms, uint64_t timeout_ns, cudaStream_t st) {
  if (world > 8) throw std::runtime_error("tp: at most 8 ranks");
  if (cols % 8 != 0 || ld % 8 != 0) throw std::runtime_error("tp: columns must be a multiple of 8");
  TPArgs a{};
  for (int i = 0; i < world; ++i) {
    a.recv[i] = recv[i];
    a.hidden[i] = hidden[i];
    a.flags[i] = flags[i];
  }
  a.world = world;
  a.rank = rank;
  a.rows_per_rank = rows_per_rank;
  a.rows_total = rows_total;
  a.cols = cols;
  a.ld = ld;
  a.epoch_ctr = epoch_ctr;
  a.timeout_ns = timeout_ns;
  a.err = err;
  const int64_t work = (int64_t)rows_per_rank * (cols / 8);
  int grid = (int)std::min<int64_t>((work + 255) / 256, (int64_t)num_sms);  // all CTAs co-resident
  if (grid < 1) grid = 1;
  launch_k(tp_reduce_ag_kernel, grid, 256, 0, st, a);
  KAPSL_LAUNCH_CHECK();
  note_launch();
}

// ------------------------------------------------ NVLink flag latency probe
// Two ranks bounce a counter through each other's flag word `iters` times (one
// thread per GPU); out_ns[0] = mean round trip.  mode 0: st.release.sys store,
// ld.acquire.sys poll; mode 1: st.relaxed.sys store, ld.relaxed.sys poll;
// mode 2: like 0, but before each store the thread writes `payload` bytes into
// the peer's buffer (16-byte stores) and issues fence.sc.sys (data-then-flag).
__device__ __forceinline__ void st_relaxed_sys(int64_t* p, int64_t v) {
  asm volatile("st.relaxed.sys.global.b64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__global__ void flag_pingpong_kernel(int64_t* my_flag, int64_t* peer_flag, uint4* peer_data, int payload16,
                                     int rank, int iters, int mode, int64_t base, uint64_t timeout_ns,
                                     int64_t* out_ns, int* err) {
  griddep_entry();
  __shared__ int ok_sh;
  if (threadIdx.x == 0) ok_sh = 1;
  __syncthreads();
  const uint64_t t0 = globaltimer_ns();
  for (int i = 1; i <= iters; ++i) {
    const int64_t v = base + i;
    for (int turn = 0; turn < 2; ++turn) {
      const bool send = (turn == 0) == (rank == 0);
      if (send) {
        if (mode == 2) {
          for (int j = threadIdx.x; j < payload16; j += blockDim.x) peer_data[j] = make_uint4(i, i, i, i);
          __syncthreads();
        }
        if (threadIdx.x == 0) {
          if (mode == 1) {
            st_relaxed_sys(peer_flag, v);
          } else {
            if (mode == 2) __threadfence_system();
            st_release_sys(peer_flag, v);
          }
        }
      } else if (threadIdx.x == 0) {
        const uint64_t w0 = globaltimer_ns();
        while ((mode == 1 ? ld_relaxed_sys(my_flag) : ld_acquire_sys(my_flag)) < v) {
          if (globaltimer_ns() - w0 > timeout_ns) {
            atomicExch(err, 39);
            ok_sh = 0;
            break;
          }
        }
      }
      __syncthreads();
      if (!ok_sh) {
        if (threadIdx.x == 0) out_ns[0] = -1;
        return;
      }
    }
  }
  if (threadIdx.x == 0) out_ns[0] = (int64_t)((globaltimer_ns() - t0) / (uint64_t)iters);
}

void launch_flag_pingpong(int64_t* my_flag, int64_t* peer_flag, void* peer_data, int payload_bytes, int rank,
                          int iters, int mode, int64_t base, uint64_t timeout_ns, int64_t* out_ns, int* err,
                          cudaStream_t st) {
  launch_k(flag_pingpong_kernel, 1, 256, 0, st, my_flag, peer_flag, reinterpret_cast<uint4*>(peer_data),
           payload_bytes / 16, rank, iters, mode, base, timeout_ns, out_ns, err);
  KAPSL_LAUNCH_CHECK();
  note_launch();
}

// ------------------------------------------------ NVLink bandwidth probe
// dst[i] = src[i] in 16-byte vectors, UNROLL vectors in flight per thread; with
// one side in a peer's memory this measures SM-driven NVLink reads or writes.
template <int UNROLL>
__global__ void __launch_bounds__(256) p2p_copy_kernel(uint4* __restrict__ dst, const uint4* __restrict__ src,
                                                      int64_t n) {
  griddep_entry();
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride * UNROLL) {
    uint4 v[UNROLL];
#pragma unroll
    for (int u = 0; u < UNROLL; ++u)
      if (i + u * stride < n) v[u] = src[i + u * stride];
#pragma unroll
    for (int u = 0; u < UNROLL; ++u)
      if (i + u * stride < n) dst[i + u * stride] = v[u];
  }
}

void launch_p2p_copy(void* dst, const void* src, int64_t bytes, int ctas_per_sm, cudaStream_t st) {
  const int64_t n = bytes / 16;
  const int grid = gemm_num_sms() * ctas_per_sm;
  launch_k(p2p_copy_kernel<4>, grid, 256, 0, st, reinterpret_cast<uint4*>(dst), reinterpret_cast<const uint4*>(src), n);
  KAPSL_LAUNCH_CHECK();
  note_launch();
}

// ------------------------------------------------------- symmetric memory
void* symm_alloc(size_t bytes) {
  void* p = nullptr;
  KAPSL_CHECK_CUDA(cudaMalloc(&p, bytes));
  KAPSL_CHECK_CUDA(cudaMemset(p, 0, bytes));
  return p;
}
void symm_free(void* p) {
  if (p) cudaFree(p);
}
std::string symm_handle(void* p) {
  cudaIpcMemHandle_t h;
  KAPSL_CHECK_CUDA(cudaIpcGetMemHandle(&h, p));
  return std::string(reinterpret_cast<const char*>(&h), sizeof(h));
}
void* symm_open(const std::string& handle) {
  if (handle.size() != sizeof(cudaIpcMemHandle_t)) throw std::runtime_error("bad IPC handle size");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle.data(), sizeof(h));
  void* p = nullptr;
  KAPSL_CHECK_CUDA(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess));
  return p;
}
void symm_close(void* p) {
  if (p) cudaIpcCloseMemHandle(p);
}

}  // namespace kapsl
