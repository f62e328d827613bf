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
