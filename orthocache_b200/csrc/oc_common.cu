// Error state, status strings and small host utilities shared by all entry points.
#include "oc_common.cuh"
#include "oc_tma.cuh"

#include <atomic>
#include <cstring>
#include <mutex>

#include <stdarg.h>
#include <stdio.h>

namespace oc {

static thread_local char g_msg[512] = "";

int set_error(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_msg, sizeof(g_msg), fmt, ap);
  va_end(ap);
  return code;
}

int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess)
    return set_error(OC_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
  return OC_OK;
}

int device_sm_count() {
  static std::atomic<int> cache[kMaxCachedDevices] = {};
  int dev = 0, n = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  if (dev >= 0 && dev < kMaxCachedDevices && (n = cache[dev].load(std::memory_order_relaxed)) > 0) return n;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) return 148;
  if (dev >= 0 && dev < kMaxCachedDevices) cache[dev].store(n, std::memory_order_relaxed);
  return n;
}

bool first_on_device(std::atomic<uint64_t>& done) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxCachedDevices) return true;
  const uint64_t bit = 1ull << dev;
  if (done.load(std::memory_order_acquire) & bit) return false;
  done.fetch_or(bit, std::memory_order_acq_rel);
  return true;
}

// Encoded tensor maps by (kind, base address, shape): encoding goes through
// the driver and costs microseconds per map, and decode loops pass the same
// few buffers every call.  A map depends only on the address and the shape,
// so an entry stays valid whatever happens to the memory behind it.
namespace {
struct MapEntry {
  uint64_t key[4];
  CUtensorMap map;
  bool used;
};
constexpr int kMapCache = 64;
MapEntry g_maps[kMapCache];
int g_map_next = 0;
std::mutex g_map_mu;
}  // namespace

bool map_cache_get(const uint64_t key[4], CUtensorMap* out) {
  std::lock_guard<std::mutex> lock(g_map_mu);
  for (int i = 0; i < kMapCache; ++i)
    if (g_maps[i].used && !memcmp(g_maps[i].key, key, sizeof(g_maps[i].key))) {
      *out = g_maps[i].map;
      return true;
    }
  return false;
}

void map_cache_put(const uint64_t key[4], const CUtensorMap& map) {
  std::lock_guard<std::mutex> lock(g_map_mu);
  MapEntry& e = g_maps[g_map_next];
  g_map_next = (g_map_next + 1) % kMapCache;
  memcpy(e.key, key, sizeof(e.key));
  e.map = map;
  e.used = true;
}

}  // namespace oc

extern "C" {

int oc_version(void) { return 100; /* 0.1.0 */ }

const char* oc_status_string(int s) {
  switch (s) {
    case OC_OK: return "ok";
    case OC_ERR_NULL: return "null pointer";
    case OC_ERR_SHAPE: return "bad shape";
    case OC_ERR_ALIGN: return "misaligned pointer";
    case OC_ERR_CAPACITY: return "capacity exceeded";
    case OC_ERR_DTYPE: return "unsupported dtype";
    case OC_ERR_CUDA: return "CUDA error";
    case OC_ERR_UNSUPPORTED: return "unsupported";
    case OC_ERR_COMM: return "NCCL error";
    default: return "unknown status";
  }
}

const char* oc_last_error(void) { return oc::g_msg; }

int oc_stratified_bucket(int nb, int gmax) {
  if (nb <= 0) return oc::set_error(OC_ERR_SHAPE, "nb_per_device must be > 0");
  // Buckets of build_stratified: nb/4, nb/2, 3nb/4, nb (each at least 1),
  // deduplicated; the first that holds the global max count is chosen.
  int b[4] = {nb / 4 > 1 ? nb / 4 : 1, nb / 2 > 1 ? nb / 2 : 1,
              (3 * nb) / 4 > 1 ? (3 * nb) / 4 : 1, nb};
  for (int i = 0; i < 3; ++i)
    if (gmax <= b[i]) return b[i];
  return b[3];
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Tensor-map encoding through the driver entry point.
// ---------------------------------------------------------------------------
#include "oc_tma.cuh"

namespace oc {

static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

int encode_map_3d(CUtensorMap* map, const void* base, CUtensorMapDataType dt, const uint64_t dims[3],
                  const uint64_t strides[2], const uint32_t box[3], bool swizzle128) {
  auto fn = encode_fn();
  if (!fn) return -1;
  cuuint64_t d[3] = {dims[0], dims[1], dims[2]};
  cuuint64_t s[2] = {strides[0], strides[1]};
  cuuint32_t b[3] = {box[0], box[1], box[2]};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(map, dt, 3, const_cast<void*>(base), d, s, b, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return (int)r;
}

int encode_map_2d(CUtensorMap* map, const void* base, CUtensorMapDataType dt, int elem_bytes, uint64_t cols,
                  uint64_t rows, uint32_t box_cols, uint32_t box_rows, bool swizzle128) {
  auto fn = encode_fn();
  if (!fn) return -1;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {cols * (uint64_t)elem_bytes};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return (int)r;
}

int encode_map_4d(CUtensorMap* map, const void* base, CUtensorMapDataType dt, const uint64_t dims[4],
                  const uint64_t strides[3], const uint32_t box[4], bool swizzle128) {
  auto fn = encode_fn();
  if (!fn) return -1;
  cuuint64_t d[4] = {dims[0], dims[1], dims[2], dims[3]};
  cuuint64_t s[3] = {strides[0], strides[1], strides[2]};
  cuuint32_t b[4] = {box[0], box[1], box[2], box[3]};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = fn(map, dt, 4, const_cast<void*>(base), d, s, b, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return (int)r;
}

}  // namespace oc

extern "C" int oc_set_wait_limit_ns(uint64_t ns) {
  OC_REQUIRE(ns >= 1000 && ns <= 60000000000ull, OC_ERR_SHAPE, "oc_set_wait_limit_ns: %llu ns outside [1 us, 60 s]",
             (unsigned long long)ns);
  int e = oc::wait_limit_score(ns);
  if (!e) e = oc::wait_limit_attn(ns);
  if (!e) e = oc::wait_limit_prefill(ns);
  if (e) return oc::set_error(OC_ERR_CUDA, "oc_set_wait_limit_ns: %s", cudaGetErrorString((cudaError_t)e));
  return OC_OK;
}

extern "C" int oc_device_status(int reset) {
  int s1 = 0, s2 = 0;
  int rc = oc::score_status(&s1, reset);
  if (rc) return rc;
  rc = oc::attn_status(&s2, reset);
  if (rc) return rc;
  int s3 = 0;
  rc = oc::prefill_status(&s3, reset);
  if (rc) return rc;
  return s1 | (s2 << 1) | (s3 << 2);
}
