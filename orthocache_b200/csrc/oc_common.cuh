// Shared helpers for the OrthoCache sm_100a kernels: error reporting,
// element conversion and 16-byte vector access.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>
#include <stddef.h>
#include <atomic>
#include <utility>

#include "../../include/orthocache_b200.h"

namespace oc {

// ---------------------------------------------------------------------------
// Error state.  Every entry point validates its arguments on the host before
// any launch, returns an OC_ERR_* code and leaves a message retrievable with
// oc_last_error() (thread-local, so concurrent callers do not clobber it).
// ---------------------------------------------------------------------------
int set_error(int code, const char* fmt, ...);
int check_launch(const char* what);
int device_sm_count();  // cached per device
constexpr int kMaxCachedDevices = 64;
// True the first time it is called for the current device (per `done`
// mask): per-device set-up such as cudaFuncSetAttribute runs once.
bool first_on_device(std::atomic<uint64_t>& done);
// Device-side error status of the pipelined kernels (a bounded wait gave up):
// copies it to *status (0 = none) and clears it if reset.  Synchronous.
int score_status(int* status, int reset);
int score_status_meta(int* status, int reset);  // the metadata form of the fused layer (oc_score_meta.cu)
int attn_status(int* status, int reset);
int prefill_status(int* status, int reset);
// Set the bounded-wait limit of the kernels of each translation unit.
int wait_limit_score(unsigned long long ns);
int wait_limit_score_meta(unsigned long long ns);
int wait_limit_attn(unsigned long long ns);
int wait_limit_prefill(unsigned long long ns);

// Fused decode layer (score, compact, attend and merge in one persistent
// kernel; oc_score.cu).  decode_fused_bytes: workspace it needs; it must be
// zero-filled before the first call, after which calls keep its epoch and
// counter sets consistent.  decode_fused returns OC_ERR_UNSUPPORTED, without launching, for
// shapes it does not cover (head_dim != 128, more than 8 query rows per KV
// head, batch * kv_heads above the grid, workspace too small).  With pm, pl,
// po non-null it writes the layer's (m, l, o) partials (the format of
// oc_partial_attention) instead of out.
size_t decode_fused_bytes(int batch, int seq_len, int kv_heads);
// Cross-GPU exchange of the fused layer's per-shard partials by peer stores:
// every rank's exchange region is mapped into every other rank's address
// space; bases[p] is rank p's region (this rank's own at [rank]), a device
// array of P pointers.  Region layout: uint64 words [2][P][NG][kXchgBlock]
// (parity of the call, source rank, group (b, h): m[8] | l[8] | o[8][128]),
// each word = the float's bits (low half) | the call number + 1 (high half),
// so a reader knows a word is this call's by looking at it: no separate flag.
struct PeerXchg {
  char* const* bases;
  int P, rank;
};
constexpr int kXchgBlock = 8 * (128 + 2);
size_t xchg_region_bytes(int P, int NG);
int decode_fused(const void* q, const void* k, const void* v, int batch, int q_len, int q_heads, int kv_heads,
                 int head_dim, int seq_len, float tau, float zeta_max, uint8_t* keep, int32_t* perm, int32_t* count,
                 void* out, int out_dtype, float* pm, float* pl, float* po, void* ws, size_t ws_bytes,
                 cudaStream_t st, const PeerXchg* px = nullptr, const float* meta_dc = nullptr,
                 const float* meta_eac = nullptr, const float* meta_zeta = nullptr);
// The same layer with the block decisions from write-time metadata (dc,
// e_ac, zeta of oc_block_metadata); decode_fused forwards to it when the
// metadata pointers are given.
int decode_fused_meta(const void* q, const void* k, const void* v, int batch, int q_len, int q_heads, int kv_heads,
                      int head_dim, int seq_len, float tau, float zeta_max, uint8_t* keep, int32_t* perm,
                      int32_t* count, void* out, int out_dtype, float* pm, float* pl, float* po, void* ws,
                      size_t ws_bytes, cudaStream_t st, const PeerXchg* px, const float* meta_dc,
                      const float* meta_eac, const float* meta_zeta);

// Paged KV: phys (batch, max_blocks) = block_table[b][idx[b][i]] for the
// first min(count[b], max_blocks) entries, -1 elsewhere (oc_compact.cu).
int compose_page_lists(const int32_t* table, int table_stride, int nlogical, const int32_t* idx, int idx_stride,
                       const int32_t* count, int count_stride, int batch, int max_blocks, int num_pages,
                       int32_t* phys, cudaStream_t st);

#define OC_REQUIRE(cond, code, ...)                                   \
  do {                                                                \
    if (!(cond)) return ::oc::set_error((code), __VA_ARGS__);         \
  } while (0)

// ---------------------------------------------------------------------------
// Element types.  Keys, values and queries arrive as float32 or bfloat16; all
// arithmetic is float32.
// ---------------------------------------------------------------------------
template <typename T> struct Elem;
template <> struct Elem<float> {
  static constexpr int kVec = 4;  // elements per 16-byte vector
  static constexpr int kCode = OC_F32;
};
template <> struct Elem<__nv_bfloat16> {
  static constexpr int kVec = 8;
  static constexpr int kCode = OC_BF16;
};

// bfloat16 is the upper half of an IEEE float32: widening is a shift.
__device__ __forceinline__ float bf16lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16hi(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }

// Read-only, L1-bypassing 16-byte load for data streamed once.
__device__ __forceinline__ uint4 ldg_stream(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

// Unpack one 16-byte vector into float32 lanes.
template <typename T> __device__ __forceinline__ void unpack16(const uint4& v, float* out);
template <> __device__ __forceinline__ void unpack16<float>(const uint4& v, float* out) {
  out[0] = __uint_as_float(v.x); out[1] = __uint_as_float(v.y);
  out[2] = __uint_as_float(v.z); out[3] = __uint_as_float(v.w);
}
template <> __device__ __forceinline__ void unpack16<__nv_bfloat16>(const uint4& v, float* out) {
  out[0] = bf16lo(v.x); out[1] = bf16hi(v.x);
  out[2] = bf16lo(v.y); out[3] = bf16hi(v.y);
  out[4] = bf16lo(v.z); out[5] = bf16hi(v.z);
  out[6] = bf16lo(v.w); out[7] = bf16hi(v.w);
}

template <typename T> __device__ __forceinline__ float to_f32(T x);
template <> __device__ __forceinline__ float to_f32<float>(float x) { return x; }
template <> __device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 x) {
  return __bfloat162float(x);
}

template <typename T> __device__ __forceinline__ T from_f32(float x);
template <> __device__ __forceinline__ float from_f32<float>(float x) { return x; }
template <> __device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float x) {
  return __float2bfloat16_rn(x);
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Programmatic dependent launch.  A kernel launched with launch_pdl may
// start while the kernel before it on the stream is still running; it must
// call pdl_wait() before touching memory that earlier kernels write (or read
// and this kernel overwrites).  pdl_trigger() lets the next kernel start
// early; without it the next kernel starts when this one ends.  Both are
// no-ops for a kernel launched the ordinary way.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                       Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

}  // namespace oc
