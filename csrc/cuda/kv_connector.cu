// KV connector for disaggregated prefill/decode: copies finished KV blocks of
// the prefill GPU's paged pool straight into the decode GPU's paged pool.
//
// Both pools use the layout [planes = layers * 2 (K, V)][num_blocks][block_elems]
// with block_elems = kv_heads * block_size * head_dim (bf16).  The decode pool
// is mapped into the prefill process with CUDA IPC; each thread moves 16-byte
// vectors with a local load and a peer store over NVLink, so the transfer is
// one kernel for every layer of every block of the request (no staging copy,
// no host round trip), and the block ids on the decode side are the ones its
// scheduler allocated.  A system-scope fence at the end makes the stores
// visible to the decode GPU once the kernel has completed.
#include "common.cuh"
#include "kernels.h"

namespace kapsl {

__global__ void __launch_bounds__(256) kv_push_kernel(const uint4* __restrict__ src, uint4* __restrict__ dst,
                                                      const int32_t* __restrict__ src_ids,
                                                      const int32_t* __restrict__ dst_ids, int nblocks, int planes,
                                                      int64_t src_plane_vecs, int64_t dst_plane_vecs,
                                                      int block_vecs) {
  griddep_entry();
  const int64_t total = (int64_t)planes * nblocks * block_vecs;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i0 = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i0 < total; i0 += 4 * stride) {
    uint4 v[4];
    int64_t d[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {  // four independent 16-byte loads in flight
      const int64_t i = i0 + u * stride;
      d[u] = -1;
      if (i < total) {
        const int e = (int)(i % block_vecs);
        const int64_t r = i / block_vecs;
        const int b = (int)(r % nblocks);
        const int p = (int)(r / nblocks);
        v[u] = src[p * src_plane_vecs + (int64_t)src_ids[b] * block_vecs + e];
        d[u] = p * dst_plane_vecs + (int64_t)dst_ids[b] * block_vecs + e;
      }
    }
#pragma unroll
    for (int u = 0; u < 4; ++u)
      if (d[u] >= 0) dst[d[u]] = v[u];
  }
  __threadfence_system();
}

void launch_kv_push(const void* src_pool, void* dst_pool, const int32_t* src_ids, const int32_t* dst_ids, int nblocks,
                    int planes, int64_t src_blocks_per_plane, int64_t dst_blocks_per_plane, int64_t block_bytes,
                    int num_sms, cudaStream_t st) {
  if (nblocks <= 0) return;
  if (block_bytes % 16 != 0 || (reinterpret_cast<uintptr_t>(src_pool) & 15) || (reinterpret_cast<uintptr_t>(dst_pool) & 15))
    throw std::runtime_error("kv_push: pools must be 16-byte aligned with 16-byte multiple blocks");
  const int block_vecs = (int)(block_bytes / 16);
  const int64_t total = (int64_t)planes * nblocks * block_vecs;
  const int grid = (int)std::max<int64_t>(1, std::min<int64_t>((total + 1023) / 1024, 4LL * num_sms));
  launch_k(kv_push_kernel, grid, 256, 0, st, static_cast<const uint4*>(src_pool), static_cast<uint4*>(dst_pool), src_ids,
                                       dst_ids, nblocks, planes, src_blocks_per_plane * block_vecs,
                                       dst_blocks_per_plane * block_vecs, block_vecs);
  KAPSL_LAUNCH_CHECK();
  note_launch();
}

}  // namespace kapsl
