// Stream compaction (union over heads -> stable active-first permutation +
// count), block gather / pack, sum-of-squares block energy, and the
// exchange index of the sequence-parallel path.
//
// Reference semantics (j-arndt/orthocache v0.3.0):
//   compaction.stream_compact        src/orthocache/compaction.py:28-100
//   alltoallv.stream_compact         src/orthocache/alltoallv.py:44-75
//   alltoallv.pack_active_blocks     alltoallv.py:150-212
//   alltoallv.compute_offsets        alltoallv.py:113-145
//   distributed_attention (index)    src/orthocache/distributed_attention.py:179-191
//   compute_block_energy_jax         src/orthocache/spectral_energy.py:21-35
//
// The reference computes the permutation with a stable argsort of the
// negated mask.  Here one CTA per batch row scans the mask in 1024-block
// tiles: a warp ballot + popc gives each block's rank among the active (or
// inactive) blocks of its tile, a scan over the 32 warp totals gives the tile
// prefix, and the running totals carry across tiles.  Active block j lands at
// (#active blocks before j); inactive block j at count + (#inactive before j).
// That is exactly the stable argsort order, with O(nb) work and no sort.
#include "oc_common.cuh"

namespace oc {
namespace {

constexpr int kScanThreads = 1024;

// Block-wide exclusive scan of a 0/1 flag; returns the prefix for this
// thread and writes the tile total to *total.
__device__ __forceinline__ int tile_scan(bool flag, int* s_warp, int* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const unsigned bal = __ballot_sync(0xffffffffu, flag);
  const int in_warp = __popc(bal & ((1u << lane) - 1u));
  if (lane == 0) s_warp[warp] = __popc(bal);
  __syncthreads();
  if (warp == 0) {
    const int v = s_warp[lane];
    int x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, x, o);
      if (lane >= o) x += y;
    }
    s_warp[lane] = x - v;  // exclusive
    if (lane == 31) s_warp[32] = x;
  }
  __syncthreads();
  const int pre = s_warp[warp] + in_warp;
  *total = s_warp[32];
  __syncthreads();
  return pre;
}

__global__ void __launch_bounds__(kScanThreads)
compact_kernel(const uint8_t* __restrict__ keep, int nb, int heads,
               int32_t* __restrict__ perm, int32_t* __restrict__ count) {
  __shared__ int s_warp[33];
  pdl_trigger();
  pdl_wait();  // keep comes from the scorer
  const int b = blockIdx.x;
  const uint8_t* kb = keep + (size_t)b * nb * heads;
  int32_t* pb = perm + (size_t)b * nb;

  if (nb <= kScanThreads) {  // one tile: count and scatter from the same scan
    const int j = threadIdx.x;
    bool act = false;
    if (j < nb)
      for (int h = 0; h < heads; ++h) act |= kb[(size_t)j * heads + h] != 0;
    int tot;
    const int pre = tile_scan(act, s_warp, &tot);
    if (j < nb) pb[act ? pre : tot + (j - pre)] = j;
    if (threadIdx.x == 0) count[b] = tot;
    return;
  }
  // Pass 1: number of active blocks.
  int n_active = 0;
  for (int t0 = 0; t0 < nb; t0 += kScanThreads) {
    const int j = t0 + threadIdx.x;
    bool act = false;
    if (j < nb)
      for (int h = 0; h < heads; ++h) act |= kb[(size_t)j * heads + h] != 0;
    int tot;
    tile_scan(act, s_warp, &tot);
    n_active += tot;
  }
  // Pass 2: scatter.
  int run_a = 0, run_i = 0;
  for (int t0 = 0; t0 < nb; t0 += kScanThreads) {
    const int j = t0 + threadIdx.x;
    bool act = false;
    if (j < nb)
      for (int h = 0; h < heads; ++h) act |= kb[(size_t)j * heads + h] != 0;
    int tot;
    const int pre = tile_scan(act, s_warp, &tot);
    const int valid = min(kScanThreads, nb - t0);
    if (j < nb) {
      const int tile_pos = threadIdx.x;  // position in tile; inactive rank = pos - active rank
      pb[act ? run_a + pre : n_active + run_i + (tile_pos - pre)] = j;
    }
    run_a += tot;
    run_i += valid - tot;
  }
  if (threadIdx.x == 0) count[b] = n_active;
}

// dst[b, i] = src[b, perm[b, i]] for i < count[b]; zero the tail if asked.
// One CTA per (destination block, batch) pair, 16-byte vectors.
__global__ void __launch_bounds__(256)
gather_blocks_kernel(const uint4* __restrict__ src, int nb_src, int64_t vec_per_block,
                     const int32_t* __restrict__ perm, int perm_stride,
                     const int32_t* __restrict__ count, uint4* __restrict__ dst, int nb_dst,
                     int zero_tail, int32_t* __restrict__ err) {
  const int i = blockIdx.x;
  const int b = blockIdx.y;
  const int n = count ? count[b] : nb_dst;
  uint4* d = dst + ((size_t)b * nb_dst + i) * vec_per_block;
  if (i >= n) {
    if (zero_tail)
      for (int64_t t = threadIdx.x; t < vec_per_block; t += blockDim.x) d[t] = make_uint4(0, 0, 0, 0);
    return;
  }
  const int sblk = perm[(size_t)b * perm_stride + i];
  if (sblk < 0 || sblk >= nb_src) {  // bad index: record it and skip the copy
    if (threadIdx.x == 0 && err) atomicExch(err, 1);
    return;
  }
  const uint4* s = src + ((size_t)b * nb_src + sblk) * vec_per_block;
  for (int64_t t = threadIdx.x; t < vec_per_block; t += blockDim.x) d[t] = s[t];
}

template <typename T>
__global__ void __launch_bounds__(256)
block_energy_kernel(const T* __restrict__ keys, int S, int H, int D, int bs, float* __restrict__ out) {
  __shared__ float s_red[8];
  const int nb = S / bs;
  const int h = blockIdx.x % H;
  const int j = (blockIdx.x / H) % nb;
  const int b = blockIdx.x / (H * nb);
  const T* base = keys + (((size_t)b * S + (size_t)j * bs) * H + h) * D;
  float acc = 0.f;
  for (int64_t e = threadIdx.x; e < (int64_t)bs * D; e += blockDim.x) {
    const int t = (int)(e / D), c = (int)(e % D);
    const float x = to_f32<T>(base[(size_t)t * H * D + c]);
    acc = fmaf(x, x, acc);
  }
  acc = warp_sum(acc);
  if ((threadIdx.x & 31) == 0) s_red[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x == 0) {
    float s = 0.f;
    for (int w = 0; w < 8; ++w) s += s_red[w];
    out[blockIdx.x] = s;
  }
}

// Valid slots of the gathered exchange buffer first (distributed_attention.py:182-191).
__global__ void __launch_bounds__(kScanThreads)
exchange_index_kernel(const int32_t* __restrict__ counts, int P, int slots,
                      int32_t* __restrict__ order, int32_t* __restrict__ total,
                      int32_t* __restrict__ offsets) {
  __shared__ int s_warp[33];
  const int n = P * slots;
  int n_valid = 0;
  for (int t0 = 0; t0 < n; t0 += kScanThreads) {
    const int jj = t0 + threadIdx.x;
    const bool v = jj < n && (jj % slots) < counts[jj / slots];
    int tot;
    tile_scan(v, s_warp, &tot);
    n_valid += tot;
  }
  int run_a = 0, run_i = 0;
  for (int t0 = 0; t0 < n; t0 += kScanThreads) {
    const int jj = t0 + threadIdx.x;
    const bool v = jj < n && (jj % slots) < counts[jj / slots];
    int tot;
    const int pre = tile_scan(v, s_warp, &tot);
    if (jj < n) order[v ? run_a + pre : n_valid + run_i + ((int)threadIdx.x - pre)] = jj;
    run_a += tot;
    run_i += min(kScanThreads, n - t0) - tot;
  }
  if (threadIdx.x == 0) {
    *total = n_valid;
    if (offsets) {
      int acc = 0;
      for (int p = 0; p < P; ++p) { offsets[p] = acc; acc += counts[p]; }
    }
  }
}

// dst[b, perm[b, i]] = src[b, i] for i < count[b] (the rest of dst was zeroed).
__global__ void __launch_bounds__(256)
scatter_blocks_kernel(const uint4* __restrict__ src, int nb_src, int64_t vec_per_block,
                      const int32_t* __restrict__ perm, int perm_stride,
                      const int32_t* __restrict__ count, uint4* __restrict__ dst, int nb_dst) {
  const int i = blockIdx.x;
  const int b = blockIdx.y;
  const int n = count ? count[b] : nb_src;
  if (i >= n) return;
  const int dblk = perm[(size_t)b * perm_stride + i];
  if (dblk < 0 || dblk >= nb_dst) return;
  const uint4* s = src + ((size_t)b * nb_src + i) * vec_per_block;
  uint4* d = dst + ((size_t)b * nb_dst + dblk) * vec_per_block;
  for (int64_t t = threadIdx.x; t < vec_per_block; t += blockDim.x) d[t] = s[t];
}

// Round each count up to the next of 1, 2, 4, ..., 512 (a count above 512 is
// kept), then clamp to cap; 0 stays 0 (indirect_attention.py:20-26, 150-157).
__global__ void bucket_count_kernel(const int32_t* __restrict__ in, int n, int cap, int32_t* __restrict__ out) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const int c = in[i];
  int b = c;
  if (c > 0 && c <= 512) {
    b = 1;
    while (b < c) b <<= 1;
  }
  out[i] = min(b, cap);
}

// keep = (bound_max >= tau) && (zeta <= zeta_max)  (spectral_energy.py:196, 231-234)
__global__ void apply_gates_kernel(const float* __restrict__ bmax, const float* __restrict__ zeta, int64_t n,
                                   const float* __restrict__ tau_dev, float tau, float zeta_max,
                                   uint8_t* __restrict__ keep) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const float t = tau_dev ? *tau_dev : tau;
  const bool g1 = bmax ? (bmax[i] >= t) : true;
  const bool g2 = zeta ? (zeta[i] <= zeta_max) : true;
  keep[i] = (g1 && g2) ? 1 : 0;
}

}  // namespace
}  // namespace oc

using namespace oc;

extern "C" int oc_scatter_blocks(const void* src, int dtype, int batch, int nb_src, int64_t block_elems,
                                 const int32_t* perm, int perm_stride, const int32_t* count,
                                 void* dst, int nb_dst, oc_stream_t stream) {
  OC_REQUIRE(src && dst && perm, OC_ERR_NULL, "oc_scatter_blocks: null pointer");
  OC_REQUIRE(dtype == OC_F32 || dtype == OC_BF16, OC_ERR_DTYPE, "oc_scatter_blocks: dtype %d", dtype);
  const int64_t esz = dtype == OC_F32 ? 4 : 2;
  OC_REQUIRE(batch >= 1 && nb_src >= 0 && nb_dst >= 0 && block_elems > 0 && perm_stride >= nb_src,
             OC_ERR_SHAPE, "oc_scatter_blocks: bad shape");
  OC_REQUIRE((block_elems * esz) % 16 == 0, OC_ERR_ALIGN, "oc_scatter_blocks: block bytes not a multiple of 16");
  OC_REQUIRE(aligned16(src) && aligned16(dst), OC_ERR_ALIGN, "oc_scatter_blocks: pointers not 16-byte aligned");
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const size_t bytes = (size_t)batch * nb_dst * block_elems * esz;
  if (bytes) {
    cudaError_t e = cudaMemsetAsync(dst, 0, bytes, st);
    if (e != cudaSuccess) return set_error(OC_ERR_CUDA, "oc_scatter_blocks: %s", cudaGetErrorString(e));
  }
  if (nb_src == 0) return OC_OK;
  dim3 grid(nb_src, batch);
  scatter_blocks_kernel<<<grid, 256, 0, st>>>((const uint4*)src, nb_src, block_elems * esz / 16, perm,
                                              perm_stride, count, (uint4*)dst, nb_dst);
  return check_launch("scatter_blocks_kernel");
}

extern "C" int oc_bucket_count(const int32_t* count, int n, int cap, int32_t* out, oc_stream_t stream) {
  OC_REQUIRE(count && out, OC_ERR_NULL, "oc_bucket_count: null pointer");
  OC_REQUIRE(n >= 0 && cap >= 0, OC_ERR_SHAPE, "oc_bucket_count: bad shape");
  if (n == 0) return OC_OK;
  bucket_count_kernel<<<(n + 255) / 256, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(count, n, cap, out);
  return check_launch("bucket_count_kernel");
}

extern "C" int oc_apply_gates(const float* bound_max, const float* zeta, int64_t cells, const float* tau_dev,
                              float tau, float zeta_max, uint8_t* keep, oc_stream_t stream) {
  OC_REQUIRE(keep, OC_ERR_NULL, "oc_apply_gates: keep is NULL");
  OC_REQUIRE(cells >= 0, OC_ERR_SHAPE, "oc_apply_gates: cells < 0");
  if (cells == 0) return OC_OK;
  apply_gates_kernel<<<(unsigned)((cells + 255) / 256), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      bound_max, zeta, cells, tau_dev, tau, zeta_max, keep);
  return check_launch("apply_gates_kernel");
}

extern "C" int oc_stream_compact(const uint8_t* keep, int batch, int num_blocks, int heads,
                                 int32_t* perm, int32_t* count, oc_stream_t stream) {
  OC_REQUIRE(keep && perm && count, OC_ERR_NULL, "oc_stream_compact: null pointer");
  OC_REQUIRE(batch >= 1 && num_blocks >= 0 && heads >= 1, OC_ERR_SHAPE,
             "oc_stream_compact: batch %d, num_blocks %d, heads %d", batch, num_blocks, heads);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const cudaError_t e = launch_pdl(compact_kernel, dim3(batch), dim3(kScanThreads), 0, st, keep, num_blocks, heads,
                                   perm, count);
  if (e != cudaSuccess) return set_error(OC_ERR_CUDA, "compact_kernel: %s", cudaGetErrorString(e));
  return check_launch("compact_kernel");
}

extern "C" int oc_gather_blocks(const void* src, int dtype, int batch, int nb_src, int64_t block_elems,
                                const int32_t* perm, int perm_stride, const int32_t* count,
                                void* dst, int nb_dst, int zero_tail, oc_stream_t stream) {
  OC_REQUIRE(src && dst && perm, OC_ERR_NULL, "oc_gather_blocks: null pointer");
  OC_REQUIRE(dtype == OC_F32 || dtype == OC_BF16, OC_ERR_DTYPE, "oc_gather_blocks: dtype %d", dtype);
  const int64_t esz = dtype == OC_F32 ? 4 : 2;
  OC_REQUIRE(batch >= 1 && nb_src >= 0 && nb_dst >= 0 && block_elems > 0 && perm_stride >= nb_dst,
             OC_ERR_SHAPE, "oc_gather_blocks: bad shape");
  OC_REQUIRE((block_elems * esz) % 16 == 0, OC_ERR_ALIGN,
             "oc_gather_blocks: block bytes %lld not a multiple of 16", (long long)(block_elems * esz));
  OC_REQUIRE(aligned16(src) && aligned16(dst), OC_ERR_ALIGN, "oc_gather_blocks: pointers not 16-byte aligned");
  if (nb_dst == 0) return OC_OK;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  dim3 grid(nb_dst, batch);
  gather_blocks_kernel<<<grid, 256, 0, st>>>((const uint4*)src, nb_src, block_elems * esz / 16, perm,
                                             perm_stride, count, (uint4*)dst, nb_dst, zero_tail, nullptr);
  return check_launch("gather_blocks_kernel");
}

extern "C" int oc_block_energy(const void* keys, int dtype, int batch, int seq_len, int heads,
                               int head_dim, int block_size, float* energy, oc_stream_t stream) {
  OC_REQUIRE(keys && energy, OC_ERR_NULL, "oc_block_energy: null pointer");
  OC_REQUIRE(batch >= 1 && heads >= 1 && head_dim >= 1 && block_size >= 1 && seq_len % block_size == 0,
             OC_ERR_SHAPE, "oc_block_energy: bad shape");
  const int64_t ncta = (int64_t)batch * (seq_len / block_size) * heads;
  if (ncta == 0) return OC_OK;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (dtype == OC_F32)
    block_energy_kernel<float><<<(unsigned)ncta, 256, 0, st>>>((const float*)keys, seq_len, heads, head_dim,
                                                                block_size, energy);
  else if (dtype == OC_BF16)
    block_energy_kernel<__nv_bfloat16><<<(unsigned)ncta, 256, 0, st>>>(
        (const __nv_bfloat16*)keys, seq_len, heads, head_dim, block_size, energy);
  else
    return set_error(OC_ERR_DTYPE, "oc_block_energy: dtype %d", dtype);
  return check_launch("block_energy_kernel");
}

extern "C" int oc_exchange_index(const int32_t* all_counts, int num_devices, int slots,
                                 int32_t* order, int32_t* total, int32_t* offsets, oc_stream_t stream) {
  OC_REQUIRE(all_counts && order && total, OC_ERR_NULL, "oc_exchange_index: null pointer");
  OC_REQUIRE(num_devices >= 1 && slots >= 0, OC_ERR_SHAPE, "oc_exchange_index: bad shape");
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  exchange_index_kernel<<<1, kScanThreads, 0, st>>>(all_counts, num_devices, slots, order, total, offsets);
  return check_launch("exchange_index_kernel");
}

// ---------------------------------------------------------------------------
// Paged KV: index lists of logical blocks -> lists of pool pages.
// phys[b][i] = table[b][idx[b][i]] for i < min(count[b], max_blocks), -1
// elsewhere or for a logical index outside the table (the attention kernels
// skip negative entries).
// ---------------------------------------------------------------------------
namespace oc {
namespace {
__global__ void page_lists_kernel(const int32_t* __restrict__ table, int table_stride, int nlogical,
                                  const int32_t* __restrict__ idx, int idx_stride, const int32_t* __restrict__ count,
                                  int count_stride, int max_blocks, int num_pages, int32_t* __restrict__ phys) {
  const int b = blockIdx.y;
  const int n = min(max(count[(size_t)b * count_stride], 0), max_blocks);
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < max_blocks; i += gridDim.x * blockDim.x) {
    int p = -1;
    if (i < n) {
      const int j = idx[(size_t)b * idx_stride + i];
      if (j >= 0 && j < nlogical) {
        p = table[(size_t)b * table_stride + j];
        if (p < 0 || p >= num_pages) p = -1;
      }
    }
    phys[(size_t)b * max_blocks + i] = p;
  }
}
}  // namespace

int compose_page_lists(const int32_t* table, int table_stride, int nlogical, const int32_t* idx, int idx_stride,
                       const int32_t* count, int count_stride, int batch, int max_blocks, int num_pages,
                       int32_t* phys, cudaStream_t st) {
  if (max_blocks == 0) return OC_OK;
  dim3 grid((max_blocks + 255) / 256, batch);
  page_lists_kernel<<<grid, 256, 0, st>>>(table, table_stride, nlogical, idx, idx_stride, count, count_stride,
                                          max_blocks, num_pages, phys);
  return check_launch("page_lists_kernel");
}
}  // namespace oc
