// Bulk-tensor (TMA) loads and mbarriers for sm_100a, in inline PTX, plus the
// host-side tensor-map encoder (driver entry point fetched through the
// runtime, so the library needs no link against libcuda).
//
// Every wait is bounded: after g_wait_limit_ns of %globaltimer time a wait gives
// up and reports failure, and the kernel records an error status instead of
// spinning forever.
#pragma once

#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace oc {

constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s, the default

// The limit in force, one copy per translation unit (set from the host by
// oc_set_wait_limit_ns through set_wait_limit_here of every unit).
static __device__ unsigned long long g_wait_limit_ns = kWaitLimitNs;
static inline int set_wait_limit_here(unsigned long long ns) {
  return (int)cudaMemcpyToSymbol(g_wait_limit_ns, &ns, sizeof(ns));
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

// Plain arrival (release semantics at CTA scope).
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Wait for the phase with the given parity; false once the wait limit
// (g_wait_limit_ns, 2 s by default) has passed.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  const uint64_t limit = g_wait_limit_ns;
  while (!mbar_try_wait(bar, parity))
    if (globaltimer_ns() - t0 > limit) return false;
  return true;
}

// 2-D tiled bulk tensor load (no multicast) into shared memory; completion
// is signalled as transaction bytes on `bar`.  x is the innermost (column)
// coordinate in elements and must be 16-byte aligned in bytes.
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
      ::"r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

// 4-D tiled bulk tensor load (no multicast); x innermost, same rules as 2-D.
__device__ __forceinline__ void tma_load_4d(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y, int z,
                                            int w) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5}], "
      "[%6];"
      ::"r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(w),
        "r"(smem_u32(bar))
      : "memory");
}

// Untiled bulk copy global -> shared (no multicast); both addresses 16-byte
// aligned, bytes a multiple of 16; completion as transaction bytes on bar.
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
               ::"r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}

// Host: encode a row-major 2-D tensor map (cols innermost).  Returns 0 or a
// CUresult code.
// swizzle128: 16-byte chunk c of box row r lands at chunk c ^ (r % 8) within
// each 1024-byte group of 8 rows (needs box_cols * elem_bytes == 128).
int encode_map_2d(CUtensorMap* map, const void* base, CUtensorMapDataType dt, int elem_bytes, uint64_t cols,
                  uint64_t rows, uint32_t box_cols, uint32_t box_rows, bool swizzle128 = false);

// Host: a process-wide cache of encoded tensor maps keyed by four words
// (kind, base address, shape digest); see oc_common.cu.
bool map_cache_get(const uint64_t key[4], CUtensorMap* out);
void map_cache_put(const uint64_t key[4], const CUtensorMap& map);

// Host: encode a 3-D tensor map (dims[0] innermost, byte strides of dims 1
// and 2).  Returns 0 or a CUresult.
int encode_map_3d(CUtensorMap* map, const void* base, CUtensorMapDataType dt, const uint64_t dims[3],
                  const uint64_t strides[2], const uint32_t box[3], bool swizzle128);

// Host: encode a 4-D tensor map; dims[0] is innermost (contiguous), strides
// are the byte strides of dims 1..3 in any order of size (a box is laid out
// in shared memory dim 0 fastest, then 1, 2, 3).  Returns 0 or a CUresult.
int encode_map_4d(CUtensorMap* map, const void* base, CUtensorMapDataType dt, const uint64_t dims[4],
                  const uint64_t strides[3], const uint32_t box[4], bool swizzle128);

}  // namespace oc
