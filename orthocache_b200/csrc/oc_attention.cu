// Indirect block attention over the retained blocks (decode / short query),
// split across CTAs by (retained block, 128-token chunk, kv head) with a
// log-sum-exp merge; and the one-call decode step (score -> compact -> attend).
//
// Reference semantics (j-arndt/orthocache v0.3.0):
//   indirect_attention.indirect_attention     src/orthocache/indirect_attention.py:127-170
//   adaptive_attention._multihead_loop        src/orthocache/adaptive_attention.py:90-120
//   distributed_attention._online_softmax_indirect_attention
//                                             src/orthocache/distributed_attention.py:78-128
//   pipeline.orthocache_forward (compact)     src/orthocache/pipeline.py:33-157
//
// The reference walks the retained blocks one after the other with an online
// softmax (running max m, sum l, output o).  The same algebra is split here:
// each work item (one chunk of one retained block for one kv head and a tile
// of query rows) produces its own (m, l, o) in a workspace, and a merge
// kernel combines them in log-sum-exp form, o / l.  Work items are taken by a
// persistent grid, so evicted blocks cost nothing and the number of retained
// blocks (device-side count) never leaves the GPU.
//
// Logits are kept in log2 units: s = (q.k) * log2(e) / sqrt(D), p = 2^(s - m).
#include "oc_common.cuh"
#include "oc_tma.cuh"
#include "oc_mma.cuh"

#include <math.h>

#include <mutex>

namespace oc {
namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kMaxChunk = 128;  // tokens per work item
constexpr float kLog2e = 1.4426950408889634f;

struct AttnArgs {
  const void* q;
  const void* k;
  const void* v;
  const int32_t* idx;
  const int32_t* count;
  int idx_stride, idx_hstride;      // list of (b, h) starts at b*idx_stride + h*idx_hstride
  int cnt_stride, cnt_hstride;      // its length is count[b*cnt_stride + h*cnt_hstride]
  int B, Sq, Hq, Hkv, G, D, S, bs;
  int kv_rows;      // token rows of K / V per batch row (S; 0 for a page pool shared by the batch)
  int nblk;         // block indices below this are valid (S / bs; the pool's pages)
  int R;            // query rows per kv head = Sq * G
  int n_rt;         // row tiles
  int chunk;        // tokens per item
  int chunks;       // items per block
  int max_items;    // max_blocks * chunks
  float scale_log2; // log2(e) / sqrt(D)
  float* ws_m;      // [B][max_items][Hkv][R]
  float* ws_l;
  float* ws_o;      // [B][max_items][Hkv][R][D]
  int run_grid;     // > 0: stream kernel on this many CTAs (partials only at run starts)
  int rt_tile;      // query rows per row tile
  void* out;        // final output (mode 0), bf16 if out_bf16
  int out_bf16;
  float *pm, *pl, *po;  // mode 1: (m, l, o) per output row
  const uint8_t* keep;  // non-null: build the union lists from this (B, S / bs, Hkv) mask in the kernel
  int32_t* perm_out;    // ... and CTA 0 writes the permutation here (count goes to `count`)
  int mode;
};

__device__ __forceinline__ int list_len(const AttnArgs& a, int b, int h) {
  const int n = a.count[(size_t)b * a.cnt_stride + (size_t)h * a.cnt_hstride];
  return max(0, min(n, a.max_items / a.chunks));
}

// Work item w -> (b, item, h, rt); false when past the end.  Items are
// ordered by (batch, item, head, row tile) for union lists (consecutive CTAs
// read the same token rows of neighbouring heads) and by (batch, head, item,
// row tile) for per-head lists.
__device__ __forceinline__ bool decode_item(const AttnArgs& a, int w, int& b, int& item, int& h, int& rt) {
  if (a.idx_hstride == 0 && a.cnt_hstride == 0) {
    const int per_item = a.Hkv * a.n_rt;
    for (b = 0; b < a.B; ++b) {
      const int n = list_len(a, b, 0) * a.chunks * per_item;
      if (w < n) {
        item = w / per_item;
        const int rem = w - item * per_item;
        h = rem / a.n_rt;
        rt = rem - h * a.n_rt;
        return true;
      }
      w -= n;
    }
    return false;
  }
  for (b = 0; b < a.B; ++b)
    for (h = 0; h < a.Hkv; ++h) {
      const int n = list_len(a, b, h) * a.chunks * a.n_rt;
      if (w < n) {
        item = w / a.n_rt;
        rt = w - item * a.n_rt;
        return true;
      }
      w -= n;
    }
  return false;
}

template <typename T, int D, int RT>
__global__ void __launch_bounds__(kThreads, 2)
attn_partial_kernel(AttnArgs a) {
  constexpr int VEC = Elem<T>::kVec;
  constexpr int LPR = D / VEC;           // lanes per key row (one 16-byte vector each)
  constexpr int RPW = 32 / LPR;          // rows per warp instruction
  constexpr int ROWS_PER_WARP = kMaxChunk / kWarps;
  constexpr int ITERS = ROWS_PER_WARP / RPW;
  static_assert(32 % LPR == 0 && ROWS_PER_WARP % RPW == 0, "mapping");

  __shared__ float s_p[RT][kMaxChunk];
  __shared__ float s_m[RT];
  __shared__ float s_l[RT];
  __shared__ float s_o[kWarps][RT][D];

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int sub = lane / LPR;            // which row of the warp instruction
  const int vl = lane % LPR;             // which 16-byte vector of the row
  const int d0 = vl * VEC;

  for (int w = blockIdx.x;; w += gridDim.x) {
    int b, item, h, rt;
    if (!decode_item(a, w, b, item, h, rt)) break;
    const int slot = item / a.chunks;
    const int c = item - slot * a.chunks;
    const int blk = a.idx[(size_t)b * a.idx_stride + (size_t)h * a.idx_hstride + slot];
    const int tok0 = blk * a.bs + c * a.chunk;
    const int r0 = rt * RT;
    const int nr = min(RT, a.R - r0);
    if (blk < 0 || blk >= a.nblk) {
      // Out-of-range index: this item contributes nothing (no memory access).
      const size_t part = (((size_t)b * a.max_items + item) * a.Hkv + h) * a.R + r0;
      for (int x = tid; x < nr * D; x += kThreads) a.ws_o[part * D + x] = 0.f;
      if (tid < nr) { a.ws_m[part + tid] = -INFINITY; a.ws_l[part + tid] = 0.f; }
      continue;
    }

    // Query rows of this tile in registers (this thread's VEC dims).
    float qv[RT][VEC];
    const T* qb = reinterpret_cast<const T*>(a.q) + (size_t)b * a.Sq * a.Hq * D;
#pragma unroll
    for (int r = 0; r < RT; ++r) {
      if (r < nr) {
        const int row = r0 + r, s = row / a.G, g = row - s * a.G;
        const T* qr = qb + ((size_t)s * a.Hq + (size_t)h * a.G + g) * D + d0;
        uint4 raw = *reinterpret_cast<const uint4*>(qr);
        unpack16<T>(raw, qv[r]);
#pragma unroll
        for (int e = 0; e < VEC; ++e) qv[r][e] *= a.scale_log2;
      } else {
#pragma unroll
        for (int e = 0; e < VEC; ++e) qv[r][e] = 0.f;
      }
    }

    const size_t tok_stride = (size_t)a.Hkv * D;
    const T* kbase = reinterpret_cast<const T*>(a.k) +
                     (((size_t)b * a.kv_rows + tok0) * a.Hkv + h) * D + d0;
    const T* vbase = reinterpret_cast<const T*>(a.v) +
                     (((size_t)b * a.kv_rows + tok0) * a.Hkv + h) * D + d0;
    const int trow0 = warp * ROWS_PER_WARP + sub;

    // ---- logits: s[r][t] = q_r . k_t (scaled) ----
    uint4 kr[ITERS];
#pragma unroll
    for (int i = 0; i < ITERS; ++i) {
      const int t = trow0 + i * RPW;
      kr[i] = t < a.chunk ? ldg_stream(kbase + (size_t)t * tok_stride) : make_uint4(0, 0, 0, 0);
    }
    // V of the same rows is requested now, so its latency hides behind the softmax.
    uint4 vr[ITERS];
#pragma unroll
    for (int i = 0; i < ITERS; ++i) {
      const int t = trow0 + i * RPW;
      vr[i] = t < a.chunk ? ldg_stream(vbase + (size_t)t * tok_stride) : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int i = 0; i < ITERS; ++i) {
      const int t = trow0 + i * RPW;
      float kf[VEC];
      unpack16<T>(kr[i], kf);
#pragma unroll
      for (int r = 0; r < RT; ++r) {
        float acc = 0.f;
#pragma unroll
        for (int e = 0; e < VEC; ++e) acc = fmaf(qv[r][e], kf[e], acc);
#pragma unroll
        for (int o = LPR / 2; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
        if (vl == 0 && t < a.chunk) s_p[r][t] = acc;
      }
    }
    __syncthreads();

    // ---- softmax statistics per row (one warp per row) ----
    for (int r = warp; r < RT; r += kWarps) {
      float m = -INFINITY;
      for (int t = lane; t < a.chunk; t += 32) m = fmaxf(m, s_p[r][t]);
      m = warp_max(m);
      float l = 0.f;
      for (int t = lane; t < a.chunk; t += 32) {
        const float p = exp2f(s_p[r][t] - m);
        s_p[r][t] = p;
        l += p;
      }
      l = warp_sum(l);
      if (lane == 0) { s_m[r] = m; s_l[r] = l; }
    }
    __syncthreads();

    // ---- o[r][d] = sum_t p[r][t] v[t][d] ----
    float acc[RT][VEC];
#pragma unroll
    for (int r = 0; r < RT; ++r)
#pragma unroll
      for (int e = 0; e < VEC; ++e) acc[r][e] = 0.f;
#pragma unroll
    for (int i = 0; i < ITERS; ++i) {
      const int t = trow0 + i * RPW;
      if (t < a.chunk) {
        float vf[VEC];
        unpack16<T>(vr[i], vf);
#pragma unroll
        for (int r = 0; r < RT; ++r) {
          const float p = s_p[r][t];
#pragma unroll
          for (int e = 0; e < VEC; ++e) acc[r][e] = fmaf(p, vf[e], acc[r][e]);
        }
      }
    }
    // lanes with the same vl but different sub hold the same dims
#pragma unroll
    for (int r = 0; r < RT; ++r)
#pragma unroll
      for (int e = 0; e < VEC; ++e) {
        float x = acc[r][e];
#pragma unroll
        for (int o = LPR; o < 32; o <<= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
        acc[r][e] = x;
      }
    if (sub == 0) {
#pragma unroll
      for (int r = 0; r < RT; ++r)
#pragma unroll
        for (int e = 0; e < VEC; ++e) s_o[warp][r][d0 + e] = acc[r][e];
    }
    __syncthreads();
    const size_t part = (((size_t)b * a.max_items + item) * a.Hkv + h) * a.R + r0;
    for (int x = tid; x < nr * D; x += kThreads) {
      const int r = x / D, d = x - r * D;
      float s = 0.f;
#pragma unroll
      for (int ww = 0; ww < kWarps; ++ww) s += s_o[ww][r][d];
      a.ws_o[(part + r) * D + d] = s;
    }
    if (tid < nr) {
      a.ws_m[part + tid] = s_m[tid];
      a.ws_l[part + tid] = s_l[tid];
    }
    __syncthreads();  // shared buffers are reused by the next item
  }
}


// ---------------------------------------------------------------------------
// bfloat16 path.  Work items are ordered (batch, kv head, row tile, index
// slot, chunk) and every CTA of the persistent grid takes one contiguous range
// of them, so a CTA walks long runs of items that share (batch, head, row
// tile).  The K and V rows of each item (CH = 8192 / D tokens) stream through
// a ring of kVStages shared-memory stages by 2-D tensor loads.  All 16 warps
// consume every stage in order (a stage is refilled by the last warp done
// with it, counted in shared memory), so no warp ever waits on a stage whose
// previous phase is still pending.  Warp w takes tokens w*TPW .. w*TPW+TPW-1
// of each item and keeps its own online-softmax state (running max m, sum l
// and output o, lanes holding D/32 output channels) across the items of a
// run; logits are reduced across lanes by a transpose-reduce.  At the end of
// a run (uniform across the CTA) the 16 warp states are combined through
// shared memory into one (m, l, o) partial, written at the run's first item;
// the other items of the run get m = -inf and are skipped by the merge.
// ---------------------------------------------------------------------------
typedef unsigned long long f32x2;  // packed float32 pair (sm_100a f32x2 arithmetic)
__device__ __forceinline__ f32x2 pack2(float lo, float hi) {
  f32x2 r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ void unpack2(f32x2 v, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ f32x2 fma2(f32x2 a, f32x2 b, f32x2 c) {
  f32x2 d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ f32x2 fmul2(f32x2 a, f32x2 b) {
  f32x2 d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}

constexpr int kVThreads = 512;
constexpr int kVWarps = kVThreads / 32;
constexpr int kVStages = 5;
constexpr int kVStageBytes = 32768;  // K + V of one item: 2 * CH * D * 2 with CH * D = 8192

__device__ int g_attn_status = 0;

// Work items of the (batch, kv head) lists: list i = (b = i / Hkv, h = i %
// Hkv) holds list_len x chunks x row tiles items.  The stream kernels keep an
// exclusive prefix of these counts in shared memory, pre[0 .. B*Hkv] (the
// last entry is the total), built by the whole CTA in one round of
// independent loads; locating an item is then a binary search instead of a
// walk over every list before it.
constexpr int kMaxLists = 1024;  // B * Hkv of the stream kernels (the host checks)

template <int NT>
__device__ __forceinline__ void build_list_prefix(const AttnArgs& a, int* pre, int* s_warp) {
  constexpr int NW = NT / 32;
  constexpr int kPer = (kMaxLists + NT - 1) / NT;
  const int NL = a.B * a.Hkv;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int i0 = tid * kPer;
  int len[kPer];
  int v = 0;
#pragma unroll
  for (int u = 0; u < kPer; ++u) {
    const int i = i0 + u;
    len[u] = i < NL ? list_len(a, i / a.Hkv, i % a.Hkv) * a.chunks * a.n_rt : 0;
    v += len[u];
  }
  int x = v;  // inclusive scan over the warp
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) s_warp[warp] = x;
  __syncthreads();
  int run = x - v;
#pragma unroll
  for (int w = 0; w < NW; ++w)
    if (w < warp) run += s_warp[w];
#pragma unroll
  for (int u = 0; u < kPer; ++u) {
    const int i = i0 + u;
    if (i < NL) pre[i] = run;
    run += len[u];
  }
  if (tid == NT - 1) pre[NL] = run;
  __syncthreads();
}

// Item w (< pre[NL]) of the (batch, head, row tile, slot, chunk) order.
struct ItemIter {
  const int* pre;
  int NL, li, b, h, rt, item, n;  // n: items of one row tile of list li; b == B marks the end
  __device__ void start(const AttnArgs& a, const int* p, int w) {
    pre = p;
    NL = a.B * a.Hkv;
    if (w >= pre[NL]) { li = NL; b = a.B; h = rt = item = 0; n = 1; return; }
    int lo = 0, hi = NL;  // pre[lo] <= w < pre[hi]; ends on the non-empty list holding w
    while (hi - lo > 1) {
      const int mid = (lo + hi) >> 1;
      if (pre[mid] <= w) lo = mid;
      else hi = mid;
    }
    li = lo;
    b = li / a.Hkv;
    h = li - b * a.Hkv;
    n = (pre[li + 1] - pre[li]) / a.n_rt;
    const int local = w - pre[li];
    rt = local / n;
    item = local - rt * n;
  }
  __device__ void next(const AttnArgs& a) {
    if (b >= a.B) return;
    if (++item < n) return;
    item = 0;
    if (++rt < a.n_rt) return;
    rt = 0;
    do {
      if (++li >= NL) { b = a.B; n = 1; return; }
      n = (pre[li + 1] - pre[li]) / a.n_rt;
    } while (n == 0);
    b = li / a.Hkv;
    h = li - b * a.Hkv;
  }
};

template <int NV>
__device__ __forceinline__ float transpose_reduce(float (&v)[NV], int lane) {
  // After the halving steps lane holds the sum of value index lane >> (5 - log2 NV)
  // over its group; the remaining offsets sum across the group.
  int c = NV;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    if (c > 1) {
      const bool up = (lane & o) != 0;
#pragma unroll
      for (int i = 0; i < NV / 2; ++i) {
        if (i < c / 2) {
          const float send = up ? v[i] : v[i + c / 2];
          const float keep = up ? v[i + c / 2] : v[i];
          v[i] = keep + __shfl_xor_sync(0xffffffffu, send, o);
        }
      }
      c >>= 1;
    } else {
      v[0] += __shfl_xor_sync(0xffffffffu, v[0], o);
    }
  }
  return v[0];
}

// Block indices of a CTA's first kBlkCache items, loaded by one warp in a
// single round of independent loads, so that no stage refill waits on a
// global load.
constexpr int kBlkCache = 64;

__device__ __forceinline__ void fill_blk_cache(const AttnArgs& a, const int* pre, int beg, int n_mine, int* s_blk,
                                               int lane) {
  const int n = min(n_mine, kBlkCache);
  for (int i = lane; i < n; i += 32) {
    ItemIter p;
    p.start(a, pre, beg + i);
    s_blk[i] = a.idx[(size_t)p.b * a.idx_stride + (size_t)p.h * a.idx_hstride + p.item / a.chunks];
  }
}

__device__ __forceinline__ void prefetch_tensormap(const CUtensorMap* m) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(m)) : "memory");
}

template <int D, int RT>
__global__ void __launch_bounds__(kVThreads, 1)
attn_stream_kernel(const __grid_constant__ CUtensorMap kmap, const __grid_constant__ CUtensorMap vmap, AttnArgs a) {
  constexpr int CH = 8192 / D;           // tokens per item
  constexpr int TPW = CH / kVWarps;      // tokens per warp per item
  constexpr int DPL = D / 32;            // output channels per lane
  constexpr int NV = TPW * RT;           // logits per warp per item (one per lane after reduction)
  constexpr int LOGNV = NV == 1 ? 0 : NV == 2 ? 1 : NV == 4 ? 2 : NV == 8 ? 3 : NV == 16 ? 4 : 5;
  constexpr int SH = 5 - LOGNV;          // lane = (value index << SH) | group position
  static_assert(NV <= 32 && (NV & (NV - 1)) == 0 && TPW * kVWarps == CH, "tile mapping");
  constexpr int KB = CH * D * 2;         // bytes of the K (or V) half of a stage
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  __shared__ __align__(8) uint64_t full[kVStages];
  __shared__ int s_rel[kVStages];
  __shared__ volatile int s_abort;
  __shared__ int s_blk[kBlkCache];
  __shared__ int s_sblk[kVStages];  // block index of the item in each stage (set when it is issued)
  __shared__ float s_wm[kVWarps][RT], s_wl[kVWarps][RT];
  __shared__ float s_wo[kVWarps][RT][D];
  __shared__ int s_pre[kMaxLists + 1];
  __shared__ int s_scan[kVWarps];

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (tid == 0) {
    for (int i = 0; i < kVStages; ++i) { mbar_init(&full[i], 1); s_rel[i] = 0; }
    fence_mbar_init();
    s_abort = 0;
    prefetch_tensormap(&kmap);
    prefetch_tensormap(&vmap);
  }
  // Launched as a programmatic dependent of the compaction: the lists and
  // counts (and everything else) are read only after it has finished.
  pdl_wait();
  build_list_prefix<kVThreads>(a, s_pre, s_scan);
  const int N = s_pre[a.B * a.Hkv];
  const int per = (N + gridDim.x - 1) / gridDim.x;
  const int beg = min(N, (int)blockIdx.x * per), end = min(N, beg + per);
  const int n_mine = end - beg;

  // Loads item position `pos` (the CTA's k-th item) into stage k % kVStages.
  auto issue = [&](int k, const ItemIter& pos) {
    const int slot = pos.item / a.chunks, c = pos.item - slot * a.chunks;
    const int blk = k < kBlkCache ? s_blk[k] : a.idx[(size_t)pos.b * a.idx_stride + (size_t)pos.h * a.idx_hstride + slot];
    // An out-of-range index is never dereferenced: block 0 is loaded instead
    // and the item is skipped.
    const int y = (blk < 0 || blk >= a.nblk) ? pos.b * a.kv_rows : pos.b * a.kv_rows + blk * a.bs + c * CH;
    uint8_t* dst = smem + (size_t)(k % kVStages) * kVStageBytes;
    uint64_t* bar = &full[k % kVStages];
    s_sblk[k % kVStages] = blk;  // published to the consumers by the arrive below
    mbar_expect_tx(bar, 2 * KB);
    tma_load_2d(dst, &kmap, bar, pos.h * D, y);
    tma_load_2d(dst + KB, &vmap, bar, pos.h * D, y);
  };

  if (warp == 0) {
    fill_blk_cache(a, s_pre, beg, n_mine, s_blk, lane);
    __syncwarp();
  }
  if (tid == 0) {
    ItemIter pre;
    pre.start(a, s_pre, beg);
    for (int k = 0; k < kVStages && k < n_mine; ++k) {
      issue(k, pre);
      pre.next(a);
    }
  }
  __syncthreads();
  // The merge kernel may now be scheduled (it waits for this grid to finish).
  pdl_trigger();

  // Per-warp online-softmax state of the current run.
  float m_run[RT];
  f32x2 o2[RT][DPL / 2];  // output channels in packed pairs
  float l_acc = 0.f;  // this lane's (token, row) share of l
  float qv[RT][DPL];
  int cur_b = -1, cur_h = -1, cur_rt = -1, run_first = 0;
  // Position of the item being consumed, and of the item kVStages ahead
  // (the one a stage released now is refilled with).
  ItemIter cur, ahead;
  cur.start(a, s_pre, beg);
  ahead.start(a, s_pre, beg);
  for (int i = 0; i < kVStages; ++i) ahead.next(a);
  const int my_v = lane >> SH;            // value index this lane ends up holding
  const int my_t = my_v / RT, my_r = my_v % RT;

  // End of a run (CTA-uniform): combine the 16 warp states into one partial
  // and publish it at the run's first item; the merge kernel combines the
  // runs of each (batch, head, row tile) segment.
  auto flush_run = [&]() {
    const int r0 = cur_rt * RT;
    const int nr = min(RT, a.R - r0);
    float l_sum = l_acc;
#pragma unroll
    for (int off = 1 << SH; off < 32; off <<= 1)  // lanes of the same row differ in the token bits
      if ((off >> SH) >= RT) l_sum += __shfl_xor_sync(0xffffffffu, l_sum, off);
    if ((lane & ((1 << SH) - 1)) == 0 && my_t == 0) {
#pragma unroll
      for (int r = 0; r < RT; ++r)
        if (r == my_r) { s_wl[warp][r] = l_sum; s_wm[warp][r] = m_run[r]; }
    }
#pragma unroll
    for (int r = 0; r < RT; ++r)
#pragma unroll
      for (int e = 0; e < DPL; e += 2) unpack2(o2[r][e / 2], s_wo[warp][r][lane * DPL + e], s_wo[warp][r][lane * DPL + e + 1]);
    __syncthreads();
    const size_t stride = (size_t)a.Hkv * a.R;
    const size_t p0 = ((size_t)cur_b * a.max_items * a.Hkv + cur_h) * a.R + r0;  // item 0, row r0
    for (int x = tid; x < nr * D; x += kVThreads) {
      const int r = x / D, d = x - r * D;
      float M = -INFINITY;
      for (int w = 0; w < kVWarps; ++w) M = fmaxf(M, s_wm[w][r]);
      float L = 0.f, O = 0.f;
      if (M != -INFINITY)
        for (int w = 0; w < kVWarps; ++w) {
          const float f = exp2f(s_wm[w][r] - M);
          L = fmaf(s_wl[w][r], f, L);
          O = fmaf(s_wo[w][r][d], f, O);
        }
      const size_t pr = p0 + (size_t)run_first * stride + r;
      a.ws_o[pr * D + d] = O;
      if (d == 0) { a.ws_m[pr] = M; a.ws_l[pr] = L; }
    }
    __syncthreads();
  };

  for (int k = 0; k < n_mine; ++k) {
    const int b = cur.b, h = cur.h, rt = cur.rt, item = cur.item;
    cur.next(a);
    const bool new_run = b != cur_b || h != cur_h || rt != cur_rt;
    if (new_run && cur_b >= 0) flush_run();
    if (new_run) {
      cur_b = b; cur_h = h; cur_rt = rt; run_first = item;
      const int r0 = rt * RT;
      const int nr = min(RT, a.R - r0);
      const __nv_bfloat16* qb = reinterpret_cast<const __nv_bfloat16*>(a.q) + (size_t)b * a.Sq * a.Hq * D;
#pragma unroll
      for (int r = 0; r < RT; ++r) {
        m_run[r] = -INFINITY;
#pragma unroll
        for (int e = 0; e < DPL; ++e) qv[r][e] = 0.f;
#pragma unroll
        for (int e = 0; e < DPL / 2; ++e) o2[r][e] = pack2(0.f, 0.f);
        if (r < nr) {
          const int row = r0 + r, s = row / a.G, g = row - s * a.G;
          const __nv_bfloat16* qr = qb + ((size_t)s * a.Hq + (size_t)h * a.G + g) * D + lane * DPL;
#pragma unroll
          for (int e = 0; e < DPL; ++e) qv[r][e] = __bfloat162float(qr[e]) * a.scale_log2;
        }
      }
      l_acc = 0.f;
    }

    const int stage = k % kVStages;
    if (!s_abort && !mbar_wait(&full[stage], (k / kVStages) & 1)) {
      s_abort = 1;
      if (lane == 0) atomicExch(&g_attn_status, 1);
    }
    const int blk = s_sblk[stage];
    const bool valid = !s_abort && blk >= 0 && blk < a.nblk;
    const uint8_t* ks = smem + (size_t)stage * kVStageBytes;
    const uint8_t* vs = ks + KB;
    // K and V rows of this warp's tokens into registers, then release the stage.
    float kf[TPW][DPL], vf[TPW][DPL];
#pragma unroll
    for (int t = 0; t < TPW; ++t) {
      const uint8_t* kr = ks + (size_t)(warp * TPW + t) * (D * 2) + lane * DPL * 2;
      const uint8_t* vr = vs + (size_t)(warp * TPW + t) * (D * 2) + lane * DPL * 2;
      if constexpr (DPL == 8) {
        const uint4 kw = *reinterpret_cast<const uint4*>(kr), vw = *reinterpret_cast<const uint4*>(vr);
        unpack16<__nv_bfloat16>(kw, kf[t]);
        unpack16<__nv_bfloat16>(vw, vf[t]);
      } else if constexpr (DPL == 4) {
        const uint2 kw = *reinterpret_cast<const uint2*>(kr), vw = *reinterpret_cast<const uint2*>(vr);
        kf[t][0] = bf16lo(kw.x); kf[t][1] = bf16hi(kw.x); kf[t][2] = bf16lo(kw.y); kf[t][3] = bf16hi(kw.y);
        vf[t][0] = bf16lo(vw.x); vf[t][1] = bf16hi(vw.x); vf[t][2] = bf16lo(vw.y); vf[t][3] = bf16hi(vw.y);
      } else {
        const uint32_t kw = *reinterpret_cast<const uint32_t*>(kr), vw = *reinterpret_cast<const uint32_t*>(vr);
        kf[t][0] = bf16lo(kw); kf[t][1] = bf16hi(kw);
        vf[t][0] = bf16lo(vw); vf[t][1] = bf16hi(vw);
      }
    }
    __threadfence_block();
    __syncwarp();
    if (lane == 0 && atomicAdd(&s_rel[stage], 1) == kVWarps - 1) {
      s_rel[stage] = 0;
      if (k + kVStages < n_mine && !s_abort) {
        fence_proxy_async();
        issue(k + kVStages, ahead);
      }
    }
    ahead.next(a);
    if (!valid) continue;

    // logits of (token t, row r): partial dots over this lane's channels, reduced across lanes
    float lv[NV];
#pragma unroll
    for (int t = 0; t < TPW; ++t)
#pragma unroll
      for (int r = 0; r < RT; ++r) {
        f32x2 acc = fmul2(pack2(qv[r][0], qv[r][1]), pack2(kf[t][0], kf[t][1]));
#pragma unroll
        for (int e = 2; e < DPL; e += 2) acc = fma2(pack2(qv[r][e], qv[r][e + 1]), pack2(kf[t][e], kf[t][e + 1]), acc);
        float lo, hi;
        unpack2(acc, lo, hi);
        lv[t * RT + r] = lo + hi;
      }
    const float s = transpose_reduce<NV>(lv, lane);  // logit of (my_t, my_r)
    // row max over this warp's tokens: lanes of the same row differ in the token bits
    float mx = s;
#pragma unroll
    for (int off = 1 << SH; off < 32; off <<= 1)
      if ((off >> SH) >= RT) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
    float alpha[RT];
#pragma unroll
    for (int r = 0; r < RT; ++r) {
      const float mr = __shfl_sync(0xffffffffu, mx, r << SH);
      const float mn = fmaxf(m_run[r], mr);
      alpha[r] = exp2f(m_run[r] - mn);  // 0 on the first item (m_run = -inf)
      m_run[r] = mn;
    }
    float m_mine = 0.f, a_mine = 0.f;  // register-only selection of this lane's row
#pragma unroll
    for (int r = 0; r < RT; ++r)
      if (r == my_r) { m_mine = m_run[r]; a_mine = alpha[r]; }
    const float p = exp2f(s - m_mine);
    l_acc = fmaf(l_acc, a_mine, p);
#pragma unroll
    for (int r = 0; r < RT; ++r) {
      const f32x2 al = pack2(alpha[r], alpha[r]);
#pragma unroll
      for (int e = 0; e < DPL; e += 2) o2[r][e / 2] = fmul2(o2[r][e / 2], al);
    }
#pragma unroll
    for (int t = 0; t < TPW; ++t)
#pragma unroll
      for (int r = 0; r < RT; ++r) {
        const float ptr = __shfl_sync(0xffffffffu, p, (t * RT + r) << SH);
        const f32x2 pp = pack2(ptr, ptr);
#pragma unroll
        for (int e = 0; e < DPL; e += 2) o2[r][e / 2] = fma2(pp, pack2(vf[t][e], vf[t][e + 1]), o2[r][e / 2]);
      }
  }
  if (cur_b >= 0) flush_run();
}

template <int D>
int launch_attn_stream(const AttnArgs& a, int rt, cudaStream_t st) {
  constexpr int CH = 8192 / D;
  CUtensorMap km, vm;
  const uint64_t cols = (uint64_t)a.Hkv * D, rows = a.kv_rows ? (uint64_t)a.B * a.kv_rows : (uint64_t)a.nblk * a.bs;
  int rc = encode_map_2d(&km, a.k, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, cols, rows, D, CH);
  if (!rc) rc = encode_map_2d(&vm, a.v, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, cols, rows, D, CH);
  if (rc) return set_error(OC_ERR_CUDA, "attention: tensor map encode failed (%d)", rc);
  const int smem = kVStages * kVStageBytes + 1024;
  const int grid = device_sm_count();
#define OC_ASTREAM(RTV)                                                                                   \
  do {                                                                                                    \
    cudaFuncSetAttribute(attn_stream_kernel<D, RTV>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem); \
    e = launch_pdl(attn_stream_kernel<D, RTV>, dim3(grid), dim3(kVThreads), smem, st, km, vm, a);      \
  } while (0)
  cudaError_t e = cudaSuccess;
  if (rt == 1) OC_ASTREAM(1);
  else if (rt == 2) OC_ASTREAM(2);
  else if constexpr (D <= 128) {
    if (rt == 4) OC_ASTREAM(4);
    else return set_error(OC_ERR_SHAPE, "attention: row tile %d", rt);
  } else
    return set_error(OC_ERR_SHAPE, "attention: row tile %d", rt);
#undef OC_ASTREAM
  if (e != cudaSuccess) return set_error(OC_ERR_CUDA, "attn_stream_kernel: %s", cudaGetErrorString(e));
  return check_launch("attn_stream_kernel");
}

// ---------------------------------------------------------------------------
// bfloat16 path on tensor cores (D = 64 or 128).  Same item order, contiguous
// per-CTA ranges, TMA stage ring and run partials as the CUDA-core
// stream kernel above, but each warp owns 16 tokens of every item and does
// both products with warp-level MMA (m16n8k16, bf16 inputs, fp32
// accumulation): S = Q K^T with the query rows of the tile as M (padded to
// 16), then O += P V with P taken straight from the S accumulators.  K and V
// arrive as 128-byte swizzled boxes of 64 channels, so every ldmatrix of a
// stage is free of bank conflicts.
// ---------------------------------------------------------------------------
constexpr int kMStages = 3;
constexpr int kMStageBytes = 32768;  // K + V of one item

#ifdef OC_TIMING
__device__ unsigned long long g_tstamp[4096][8];
#define OC_STAMP(i) do { if (threadIdx.x == 0 && blockIdx.x < 4096) g_tstamp[blockIdx.x][i] = globaltimer_ns(); } while (0)
#else
#define OC_STAMP(i) do {} while (0)
#endif


// Union lists from the scorer's keep mask (the compaction of
// compaction.py:28-100 folded into the attention prologue): every CTA
// derives the active-first list of each batch row in shared memory with a
// ballot scan (active block j goes to the number of active blocks before
// it), then reads its work from there.  CTA 0 also writes the complete
// stable permutation (inactive blocks after the active ones, in order) and
// the counts.  On return a.idx / a.count point at the shared-memory lists.
template <int NT>
__device__ void lists_from_keep(AttnArgs& a, int* s_list, int* s_cnt, int* s_scan) {
  constexpr int NWP = NT / 32;
  const int nb = a.S / a.bs, H = a.Hkv;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const bool writer = blockIdx.x == 0;
  for (int pass = 0; pass < (writer ? 2 : 1); ++pass) {
    for (int b = 0; b < a.B; ++b) {
      int base = 0;
      for (int j0 = 0; j0 < nb; j0 += NT) {
        const int j = j0 + tid;
        bool act = false;
        if (j < nb) {
          const uint8_t* kp = a.keep + ((size_t)b * nb + j) * H;
          if (H == 8 && (reinterpret_cast<uintptr_t>(kp) & 7) == 0) {
            act = *reinterpret_cast<const unsigned long long*>(kp) != 0ull;  // one load per block
          } else {
            for (int h = 0; h < H; ++h) act |= kp[h] != 0;
          }
        }
        const unsigned bal = __ballot_sync(0xffffffffu, act);
        if (lane == 0) s_scan[warp] = __popc(bal);
        __syncthreads();
        int before = 0, tot = 0;
#pragma unroll
        for (int w = 0; w < NWP; ++w) {
          const int v = s_scan[w];
          before += w < warp ? v : 0;
          tot += v;
        }
        const int rank = base + before + __popc(bal & ((1u << lane) - 1u));  // active blocks before j
        if (pass == 0 && act) s_list[b * nb + rank] = j;
        if (pass == 1 && j < nb) a.perm_out[(size_t)b * nb + (act ? rank : s_cnt[b] + j - rank)] = j;
        __syncthreads();
        base += tot;
      }
      if (pass == 0 && tid == 0) s_cnt[b] = base;
      if (pass == 1 && tid == 0) const_cast<int32_t*>(a.count)[b] = base;
    }
    __syncthreads();
  }
  a.idx = s_list;
  a.count = s_cnt;
  a.idx_stride = nb;
  a.idx_hstride = 0;
  a.cnt_stride = 1;
  a.cnt_hstride = 0;
}

// Warps of the tensor-core stream kernel: (8192 / D) / 16 token groups of 16
// tokens, times the output-channel slices of at most 128 channels (two at
// D = 256: both warps of a token group compute its logits, each accumulates
// half of the output channels).
template <int D>
constexpr int mma_threads() {
  return 32 * ((8192 / D) / 16) * (D > 128 ? D / 128 : 1);
}

template <int D, int RT>
__global__ void __launch_bounds__(mma_threads<D>(), 2)
attn_mma_kernel(const __grid_constant__ CUtensorMap kmap, const __grid_constant__ CUtensorMap vmap, AttnArgs a_in) {
  constexpr int CH = 8192 / D;           // tokens per item
  constexpr int NTG = CH / 16;           // token groups of 16
  constexpr int CS = D > 128 ? D / 128 : 1;  // output-channel slices
  constexpr int DO = D / CS;             // output channels per warp
  constexpr int NW = NTG * CS;           // warps
  constexpr int NT = 32 * NW;
  constexpr int KS = D / 16;             // k-steps of S = Q K^T
  constexpr int NO = DO / 8;             // n-tiles of this warp's O
  constexpr int KB = CH * D * 2;         // bytes of the K (or V) half of a stage
  static_assert(NT == mma_threads<D>(), "warp layout");
  static_assert(RT == 4 || RT == 8, "row tile");
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  __shared__ __align__(8) uint64_t full[kMStages];
  __shared__ int s_rel[kMStages];
  __shared__ volatile int s_abort;
  __shared__ int s_blk[kBlkCache];
  __shared__ float s_wm[NW][RT], s_wl[NW][RT];
  __shared__ float s_wo[NW][RT][DO];
  __shared__ int s_pre[kMaxLists + 1];
  __shared__ int s_wsum[NW];

  OC_STAMP(0);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int tg = warp % NTG, cs = warp / NTG;  // token group, output-channel slice
  const int g = lane >> 2, c = lane & 3;  // MMA fragment coordinates
  if (tid == 0) {
    for (int i = 0; i < kMStages; ++i) { mbar_init(&full[i], 1); s_rel[i] = 0; }
    fence_mbar_init();
    s_abort = 0;
    prefetch_tensormap(&kmap);
    prefetch_tensormap(&vmap);
  }
  // Launched as a programmatic dependent of the compaction: the lists and
  // counts (and everything else) are read only after it has finished.
  pdl_wait();
  OC_STAMP(5);
  AttnArgs a = a_in;
  if (a.keep) {
    __shared__ int s_scan[NW];
    int* s_list = reinterpret_cast<int*>(smem + (size_t)kMStages * kMStageBytes);
    lists_from_keep<NT>(a, s_list, s_list + a.B * (a.S / a.bs), s_scan);
  }
  build_list_prefix<NT>(a, s_pre, s_wsum);
  const int N = s_pre[a.B * a.Hkv];
  const int per = (N + gridDim.x - 1) / gridDim.x;
  const int beg = min(N, (int)blockIdx.x * per), end = min(N, beg + per);
  const int n_mine = end - beg;
  OC_STAMP(6);

  auto issue = [&](int k, const ItemIter& pos) {
    const int slot = pos.item / a.chunks, cc = pos.item - slot * a.chunks;
    const int blk = k < kBlkCache ? s_blk[k] : a.idx[(size_t)pos.b * a.idx_stride + (size_t)pos.h * a.idx_hstride + slot];
    const int y = (blk < 0 || blk >= a.nblk) ? pos.b * a.kv_rows : pos.b * a.kv_rows + blk * a.bs + cc * CH;
    uint8_t* dst = smem + (size_t)(k % kMStages) * kMStageBytes;
    uint64_t* bar = &full[k % kMStages];
    mbar_expect_tx(bar, 2 * KB);
#pragma unroll
    for (int jb = 0; jb < D / 64; ++jb) {
      tma_load_2d(dst + jb * (CH * 128), &kmap, bar, pos.h * D + jb * 64, y);
      tma_load_2d(dst + KB + jb * (CH * 128), &vmap, bar, pos.h * D + jb * 64, y);
    }
  };

  if (warp == 0) {
    fill_blk_cache(a, s_pre, beg, n_mine, s_blk, lane);
    OC_STAMP(7);
    __syncwarp();
  }
  if (tid == 0) {
    ItemIter pre;
    pre.start(a, s_pre, beg);
    for (int k = 0; k < kMStages && k < n_mine; ++k) {
      issue(k, pre);
      pre.next(a);
    }
  }
  __syncthreads();
  // The merge kernel may now be scheduled (it waits for this grid to finish).
  pdl_trigger();

  // per-warp online-softmax state of the run: rows g and g + 8 of the tile
  float m_run[2], l_acc[2];
  float o[NO][4];
  uint32_t qa[KS][4];
  int cur_b = -1, cur_h = -1, cur_rt = -1, run_first = 0;
  ItemIter cur, ahead;
  cur.start(a, s_pre, beg);
  ahead.start(a, s_pre, beg);
  for (int i = 0; i < kMStages; ++i) ahead.next(a);
  OC_STAMP(1);

  // End of a run (CTA-uniform): combine the warp states into one partial and
  // publish it at the run's first item.
  auto flush_run = [&]() {
    const int r0 = cur_rt * RT;
    const int nr = min(RT, a.R - r0);
#pragma unroll
    for (int hf = 0; hf < 2; ++hf) {
      float l = l_acc[hf];
      l += __shfl_xor_sync(0xffffffffu, l, 1);
      l += __shfl_xor_sync(0xffffffffu, l, 2);
      const int row = g + 8 * hf;
      if (row < RT) {
        if (c == 0) { s_wl[warp][row] = l; s_wm[warp][row] = m_run[hf]; }
#pragma unroll
        for (int nt = 0; nt < NO; ++nt) {
          s_wo[warp][row][8 * nt + 2 * c] = o[nt][2 * hf];
          s_wo[warp][row][8 * nt + 2 * c + 1] = o[nt][2 * hf + 1];
        }
      }
    }
    __syncthreads();
    const size_t stride = (size_t)a.Hkv * a.R;
    const size_t p0 = ((size_t)cur_b * a.max_items * a.Hkv + cur_h) * a.R + r0;  // item 0, row r0
    for (int x = tid; x < nr * D; x += NT) {
      // channel d of row r: the token groups' states of its slice (the
      // slices of a token group hold the same m and l)
      const int r = x / D, d = x - r * D, w0 = (d / DO) * NTG, dl = d % DO;
      float M = -INFINITY;
      for (int t = 0; t < NTG; ++t) M = fmaxf(M, s_wm[w0 + t][r]);
      float L = 0.f, O = 0.f;
      if (M != -INFINITY)
        for (int t = 0; t < NTG; ++t) {
          const float f = exp2f(s_wm[w0 + t][r] - M);
          L = fmaf(s_wl[w0 + t][r], f, L);
          O = fmaf(s_wo[w0 + t][r][dl], f, O);
        }
      const size_t pr = p0 + (size_t)run_first * stride + r;
      a.ws_o[pr * D + d] = O;
      if (d == 0) { a.ws_m[pr] = M; a.ws_l[pr] = L; }
    }
    __syncthreads();
  };

  for (int k = 0; k < n_mine; ++k) {
    const int b = cur.b, h = cur.h, rt = cur.rt, item = cur.item;
    cur.next(a);
    const bool new_run = b != cur_b || h != cur_h || rt != cur_rt;
    if (new_run && cur_b >= 0) flush_run();
    if (new_run) {
      cur_b = b; cur_h = h; cur_rt = rt; run_first = item;
      const int r0 = rt * RT;
      const __nv_bfloat16* qb = reinterpret_cast<const __nv_bfloat16*>(a.q) + (size_t)b * a.Sq * a.Hq * D;
      // A fragments of Q (rows g and g + 8 of the tile; rows past the tile are zero)
      const uint32_t* qrow[2] = {nullptr, nullptr};
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {
        const int rr = g + 8 * hf;
        const int row = r0 + rr;
        if (rr < RT && row < a.R) {
          const int s = row / a.G, gq = row - s * a.G;
          qrow[hf] = reinterpret_cast<const uint32_t*>(qb + ((size_t)s * a.Hq + (size_t)h * a.G + gq) * D);
        }
      }
#pragma unroll
      for (int ks = 0; ks < KS; ++ks) {
        qa[ks][0] = qrow[0] ? qrow[0][8 * ks + c] : 0u;      // row g,     channels 16ks + 2c, +1
        qa[ks][1] = qrow[1] ? qrow[1][8 * ks + c] : 0u;      // row g + 8
        qa[ks][2] = qrow[0] ? qrow[0][8 * ks + 4 + c] : 0u;  // row g,     channels 16ks + 8 + 2c, +1
        qa[ks][3] = qrow[1] ? qrow[1][8 * ks + 4 + c] : 0u;
      }
      m_run[0] = m_run[1] = -INFINITY;
      l_acc[0] = l_acc[1] = 0.f;
#pragma unroll
      for (int nt = 0; nt < NO; ++nt) o[nt][0] = o[nt][1] = o[nt][2] = o[nt][3] = 0.f;
    }

    const int stage = k % kMStages;
    if (!s_abort && !mbar_wait(&full[stage], (k / kMStages) & 1)) {
      s_abort = 1;
      if (lane == 0) atomicExch(&g_attn_status, 1);
    }
    if (k == 0) OC_STAMP(2);
    const int slot = item / a.chunks;
    const int blk = a.idx[(size_t)b * a.idx_stride + (size_t)h * a.idx_hstride + slot];
    const bool valid = !s_abort && blk >= 0 && blk < a.nblk;
    const uint32_t ks_base = smem_u32(smem + (size_t)stage * kMStageBytes);
    const uint32_t vs_base = ks_base + KB;
    float sa[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
    const int mm = lane >> 3, rr = lane & 7;
    uint32_t vb[NO / 2][4];
    if constexpr (CS == 1) {
      // All fragments of this warp's 16 tokens, then the stage is released.
      uint32_t kb[KS][4];
#pragma unroll
      for (int ks = 0; ks < KS; ++ks)  // matrices: (tokens 0-7 | 8-15) x (channels 16ks..+8 | +8..+16)
        ldsm_x4(kb[ks], ks_base + swz<CH>(16 * tg + 8 * (mm >> 1) + rr, 2 * ks + (mm & 1)));
#pragma unroll
      for (int np2 = 0; np2 < NO / 2; ++np2)  // matrices: (tokens 0-7 | 8-15) x (channel tiles 2np2 | 2np2+1)
        ldsm_x4_t(vb[np2], vs_base + swz<CH>(16 * tg + 8 * (mm & 1) + rr, 2 * np2 + (mm >> 1)));
      __syncwarp();
      if (lane == 0 && atomicAdd(&s_rel[stage], 1) == NW - 1) {
        s_rel[stage] = 0;
        if (k + kMStages < n_mine && !s_abort) {
          fence_proxy_async();
          issue(k + kMStages, ahead);
        }
      }
      ahead.next(a);
      if (!valid) continue;
      // S = Q K^T for the two 8-token tiles (rows g, g+8; tokens 2c, 2c+1)
#pragma unroll
      for (int ks = 0; ks < KS; ++ks) {
        mma_bf16_16816(sa[0], qa[ks], kb[ks][0], kb[ks][1]);
        mma_bf16_16816(sa[1], qa[ks], kb[ks][2], kb[ks][3]);
      }
    } else {
      // Wide heads: the logits k-step by k-step (K fragments are not all
      // held at once), then this slice's V fragments, then the release.
#pragma unroll
      for (int ks = 0; ks < KS; ++ks) {
        uint32_t kb[4];
        ldsm_x4(kb, ks_base + swz<CH>(16 * tg + 8 * (mm >> 1) + rr, 2 * ks + (mm & 1)));
        mma_bf16_16816(sa[0], qa[ks], kb[0], kb[1]);
        mma_bf16_16816(sa[1], qa[ks], kb[2], kb[3]);
      }
#pragma unroll
      for (int np2 = 0; np2 < NO / 2; ++np2)
        ldsm_x4_t(vb[np2], vs_base + swz<CH>(16 * tg + 8 * (mm & 1) + rr, cs * NO + 2 * np2 + (mm >> 1)));
      __syncwarp();
      if (lane == 0 && atomicAdd(&s_rel[stage], 1) == NW - 1) {
        s_rel[stage] = 0;
        if (k + kMStages < n_mine && !s_abort) {
          fence_proxy_async();
          issue(k + kMStages, ahead);
        }
      }
      ahead.next(a);
      if (!valid) continue;
    }
    // online softmax in log2 units
#pragma unroll
    for (int j = 0; j < 2; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) sa[j][e] *= a.scale_log2;
    float alpha[2];
#pragma unroll
    for (int hf = 0; hf < 2; ++hf) {
      float mx = fmaxf(fmaxf(sa[0][2 * hf], sa[0][2 * hf + 1]), fmaxf(sa[1][2 * hf], sa[1][2 * hf + 1]));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
      const float mn = fmaxf(m_run[hf], mx);
      alpha[hf] = exp2f(m_run[hf] - mn);
      m_run[hf] = mn;
      float ls = 0.f;
#pragma unroll
      for (int j = 0; j < 2; ++j)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const float p = exp2f(sa[j][2 * hf + e] - mn);
          sa[j][2 * hf + e] = p;
          ls += p;
        }
      l_acc[hf] = fmaf(l_acc[hf], alpha[hf], ls);
    }
    const uint32_t pa[4] = {pack_bf16x2(sa[0][0], sa[0][1]), pack_bf16x2(sa[0][2], sa[0][3]),
                            pack_bf16x2(sa[1][0], sa[1][1]), pack_bf16x2(sa[1][2], sa[1][3])};
#pragma unroll
    for (int nt = 0; nt < NO; ++nt) {
      o[nt][0] *= alpha[0]; o[nt][1] *= alpha[0];
      o[nt][2] *= alpha[1]; o[nt][3] *= alpha[1];
    }
    // O += P V over the warp's 16 tokens
#pragma unroll
    for (int np2 = 0; np2 < NO / 2; ++np2) {
      mma_bf16_16816(o[2 * np2], pa, vb[np2][0], vb[np2][1]);
      mma_bf16_16816(o[2 * np2 + 1], pa, vb[np2][2], vb[np2][3]);
    }
  }
  OC_STAMP(4);
  if (cur_b >= 0) flush_run();
  OC_STAMP(3);
}

// Shared memory for lists built from a keep mask (B rows of nb blocks + B counts).
constexpr int kKeepListMax = 1024;  // B * nb at most (4 KB)
int keep_list_bytes(int B, int nb) { return ((B * nb + B) * 4 + 15) / 16 * 16; }

template <int D>
int launch_attn_mma(const AttnArgs& a, int rt, cudaStream_t st) {
  constexpr int CH = 8192 / D;
  constexpr int NT = mma_threads<D>();
  CUtensorMap km, vm;
  const uint64_t cols = (uint64_t)a.Hkv * D, rows = a.kv_rows ? (uint64_t)a.B * a.kv_rows : (uint64_t)a.nblk * a.bs;
  int rc = encode_map_2d(&km, a.k, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, cols, rows, 64, CH, true);
  if (!rc) rc = encode_map_2d(&vm, a.v, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, cols, rows, 64, CH, true);
  if (rc) return set_error(OC_ERR_CUDA, "attention: tensor map encode failed (%d)", rc);
  // keep mode: the union lists and counts follow the stage ring
  const int smem = kMStages * kMStageBytes + 1024 + (a.keep ? keep_list_bytes(a.B, a.S / a.bs) : 0);
  const int grid = a.run_grid;
#define OC_AMMA(RTV)                                                                                   \
  do {                                                                                                 \
    cudaFuncSetAttribute(attn_mma_kernel<D, RTV>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem); \
    e = launch_pdl(attn_mma_kernel<D, RTV>, dim3(grid), dim3(NT), smem, st, km, vm, a);               \
  } while (0)
  cudaError_t e = cudaSuccess;
  if (rt <= 4) OC_AMMA(4);
  else OC_AMMA(8);
#undef OC_AMMA
  if (e != cudaSuccess) return set_error(OC_ERR_CUDA, "attn_mma_kernel: %s", cudaGetErrorString(e));
  return check_launch("attn_mma_kernel");
}

// Combine the partials of one (batch, kv head, row): M = max m_i,
// L = sum l_i 2^(m_i - M), O = sum o_i 2^(m_i - M).  mode 0 writes O / L in
// the output dtype at the reference's (Sq, Hq, D) position (zeros when the
// batch row has no retained block); mode 1 writes (M, L, O) float32 for a
// later cross-shard merge.  kMergeThreads threads: NQ = kMergeThreads / D
// groups of D channels, group q taking the partials j = q (mod NQ), so the
// output loads of a row go out in few rounds; the groups are summed in
// shared memory at the end.  The code is kept small: it runs once per row
// and its instructions are fetched cold.
constexpr int kMergeThreads = 512;

template <typename TO>
__global__ void __launch_bounds__(kMergeThreads)
attn_merge_kernel(AttnArgs a, TO* out, float* pm, float* pl, float* po, int mode) {
  __shared__ float s_w[kMergeThreads];            // weights 2^(m_j - M) of the current chunk
  __shared__ float s_red[kMergeThreads / 32];
  __shared__ float s_o[kMergeThreads];            // per-group sums
  pdl_trigger();  // the next kernel may stage its prologue meanwhile
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int NQ = kMergeThreads / a.D;
  const int d = tid % a.D, q = tid / a.D;
  const int r = blockIdx.x % a.R;
  const int h = (blockIdx.x / a.R) % a.Hkv;
  const int b = blockIdx.x / (a.R * a.Hkv);
  const int n = list_len(a, b, h) * a.chunks;
  const int s = r / a.G, g = r - s * a.G;
  const size_t orow = ((size_t)b * a.Sq + s) * a.Hq + (size_t)h * a.G + g;
  const size_t stride = (size_t)a.Hkv * a.R;
  const size_t p0 = ((size_t)b * a.max_items * a.Hkv + h) * a.R + r;

  // Items holding a partial.  Dense layout: every item.  Stream kernel: the
  // first item of each CTA run -- local index 0 of this (batch, head, row
  // tile) list and every CTA boundary c * per that falls inside it.
  int np = n, s0 = 0, per = 1, c1 = 0;
  if (a.run_grid > 0 && n > 0) {
    // Items of all lists and of the lists before (b, h): one load per
    // thread, summed over the CTA.
    __shared__ int s_tb[2][kMergeThreads / 32];
    const int me = b * a.Hkv + h;
    int total = 0, before = 0;
    for (int i = tid; i < a.B * a.Hkv; i += kMergeThreads) {
      const int len = list_len(a, i / a.Hkv, i % a.Hkv) * a.chunks * a.n_rt;
      total += len;
      if (i < me) before += len;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      total += __shfl_xor_sync(0xffffffffu, total, o);
      before += __shfl_xor_sync(0xffffffffu, before, o);
    }
    if (lane == 0) { s_tb[0][warp] = total; s_tb[1][warp] = before; }
    __syncthreads();
    total = before = 0;
    for (int w = 0; w < kMergeThreads / 32; ++w) { total += s_tb[0][w]; before += s_tb[1][w]; }
    per = (total + a.run_grid - 1) / a.run_grid;
    s0 = before + (r / a.rt_tile) * n;
    c1 = s0 / per + 1;                                   // first CTA boundary after s0
    const int last = (s0 + n - 1) / per;                 // last CTA touching the list
    np = 1 + max(0, last - c1 + 1);
  }
  auto prow = [&](int j) -> size_t {
    return p0 + (size_t)((a.run_grid > 0 && j > 0) ? (c1 + j - 1) * per - s0 : j) * stride;
  };
  // Launched as a programmatic dependent of the stream kernel: wait for it to
  // finish (and its partials to be visible).  A no-op for a plain launch.
  pdl_wait();

  // M over all partials
  float mj = -INFINITY, lj = 0.f;  // this thread's partial of the first chunk
  if (tid < np) { mj = a.ws_m[prow(tid)]; lj = a.ws_l[prow(tid)]; }
  float M = mj;
  for (int j = tid + kMergeThreads; j < np; j += kMergeThreads) M = fmaxf(M, a.ws_m[prow(j)]);
  M = warp_max(M);
  if (lane == 0) s_red[warp] = M;
  __syncthreads();
  M = s_red[0];
  for (int w = 1; w < kMergeThreads / 32; ++w) M = fmaxf(M, s_red[w]);
  __syncthreads();

  float L = 0.f, O = 0.f;
  for (int c0 = 0; c0 < np; c0 += kMergeThreads) {
    const int j = c0 + tid;
    float w = 0.f;
    if (j < np) {
      const float m = c0 == 0 ? mj : a.ws_m[prow(j)];
      const float l = c0 == 0 ? lj : a.ws_l[prow(j)];
      if (m != -INFINITY) {
        w = exp2f(m - M);
        L = fmaf(l, w, L);
      }
    }
    s_w[tid] = w;
    __syncthreads();
    // Every listed partial holds a written output row (zeros when its max is
    // -inf), so the loads are unconditional.
    const int cn = min(kMergeThreads, np - c0);
#pragma unroll 8
    for (int u = q; u < cn; u += NQ) O = fmaf(s_w[u], a.ws_o[prow(c0 + u) * a.D + d], O);
    __syncthreads();
  }
  s_o[tid] = O;
  L = warp_sum(L);
  if (lane == 0) s_red[warp] = L;
  __syncthreads();
  if (q == 0) {
    for (int qq = 1; qq < NQ; ++qq) O += s_o[qq * a.D + d];
    L = 0.f;
    for (int w = 0; w < kMergeThreads / 32; ++w) L += s_red[w];
    if (mode == 0) {
      out[orow * a.D + d] = from_f32<TO>(L > 0.f ? O / L : 0.f);
    } else {
      po[orow * a.D + d] = L > 0.f ? O : 0.f;
      if (d == 0) { pm[orow] = M; pl[orow] = L; }
    }
  }
}

// Cross-shard merge of (m, l, o) triples (P parts of `rows` rows).
template <typename TO>
__global__ void __launch_bounds__(128)
merge_parts_kernel(const float* m, const float* l, const float* o, int P, int rows, int D, TO* out,
                   size_t ml_stride, size_t o_stride) {
  // part p's m and l at p * ml_stride, its o at p * o_stride (floats)
  const int r = blockIdx.x;
  float M = -INFINITY;
  for (int p = 0; p < P; ++p) M = fmaxf(M, m[(size_t)p * ml_stride + r]);
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    float L = 0.f, O = 0.f;
    if (M != -INFINITY) {
      for (int p = 0; p < P; ++p) {
        const float mp = m[(size_t)p * ml_stride + r];
        if (mp == -INFINITY) continue;
        const float f = exp2f(mp - M);
        L = fmaf(l[(size_t)p * ml_stride + r], f, L);
        O = fmaf(o[(size_t)p * o_stride + (size_t)r * D + d], f, O);
      }
    }
    out[(size_t)r * D + d] = from_f32<TO>(L > 0.f ? O / L : 0.f);
  }
}

// Rows of (batch, kv head) pairs whose index list is empty get the mean of
// all value rows of that head: the reference's predicated attention masks
// every logit of such a head with -1e9, and its softmax is then uniform over
// all tokens (sparse_attention.py:49-57).
template <typename T, typename TO>
__global__ void __launch_bounds__(256)
empty_heads_mean_kernel(const T* __restrict__ v, const int32_t* __restrict__ count, int cnt_stride,
                        int cnt_hstride, int Sq, int Hq, int Hkv, int D, int S, TO* __restrict__ out) {
  __shared__ float s_acc[256];
  const int h = blockIdx.x % Hkv, b = blockIdx.x / Hkv;
  if (count[(size_t)b * cnt_stride + (size_t)h * cnt_hstride] != 0) return;
  const int G = Hq / Hkv;
  const int lanes_per_d = 256 / D;  // D in {64, 128, 256}
  const int d = threadIdx.x % D, part = threadIdx.x / D;
  float acc = 0.f;
  for (int t = part; t < S; t += lanes_per_d)
    acc += to_f32<T>(v[(((size_t)b * S + t) * Hkv + h) * D + d]);
  s_acc[threadIdx.x] = acc;
  __syncthreads();
  if (part == 0) {
    for (int p2 = 1; p2 < lanes_per_d; ++p2) acc += s_acc[p2 * D + d];
    const float mean = acc / (float)S;
    for (int sq = 0; sq < Sq; ++sq)
      for (int g = 0; g < G; ++g)
        out[(((size_t)b * Sq + sq) * Hq + (size_t)h * G + g) * D + d] = from_f32<TO>(mean);
  }
}

inline size_t align256(size_t x) { return (x + 255) & ~(size_t)255; }

// Row-tile size: query rows handled per work item (8 at most; 4 at D = 256 so
// the per-warp reduction buffer stays within static shared memory).
int pick_rt(int R, int D) {
  const int rt = R <= 1 ? 1 : R <= 2 ? 2 : R <= 4 ? 4 : 8;
  return D == 256 && rt > 4 ? 4 : rt;
}

// Tokens per work item: CH = 8192 / D (a K + V chunk of 32 KB in bfloat16),
// or 64 when the block size is not a multiple of CH.
int chunk_for(int bs, int D) { return bs % (8192 / D) == 0 ? 8192 / D : 64; }

// bfloat16 inputs stream through the bulk-tensor path when the chunk fits.
// Stream kernels: bfloat16, whole items per block, and at most kMaxLists
// (batch, kv head) lists (their prefix lives in shared memory).
bool use_tma_path(int dtype, int bs, int D, int64_t lists) {
  return dtype == OC_BF16 && bs % (8192 / D) == 0 && lists <= kMaxLists;
}

size_t attn_ws_bytes(int B, int Sq, int Hq, int Hkv, int D, int bs, int max_blocks) {
  const int G = Hq / Hkv;
  const size_t R = (size_t)Sq * G;
  const size_t items = (size_t)max_blocks * (bs / chunk_for(bs, D));
  const size_t parts = (size_t)B * items * Hkv * R;
  return 2 * align256(parts * sizeof(float)) + align256(parts * D * sizeof(float));
}

int validate_attn(const void* q, const void* k, const void* v, int dtype, const int32_t* idx,
                  int idx_stride, int idx_hstride, const int32_t* count, int B, int Sq, int Hq, int Hkv, int D,
                  int S, int bs, int max_blocks) {
  OC_REQUIRE(q && k && v && idx && count, OC_ERR_NULL, "attention: null pointer");
  OC_REQUIRE(dtype == OC_F32 || dtype == OC_BF16, OC_ERR_DTYPE, "attention: dtype %d", dtype);
  OC_REQUIRE(D == 64 || D == 128 || D == 256, OC_ERR_SHAPE, "attention: head_dim %d not in {64,128,256}", D);
  OC_REQUIRE(B >= 1 && Sq >= 1 && Hkv >= 1 && Hq >= Hkv && Hq % Hkv == 0, OC_ERR_SHAPE,
             "attention: batch %d, q_len %d, q_heads %d, kv_heads %d", B, Sq, Hq, Hkv);
  OC_REQUIRE(bs >= 64 && bs % 64 == 0 && S % bs == 0, OC_ERR_SHAPE,
             "attention: block_size %d must be a multiple of 64 dividing seq_len %d", bs, S);
  OC_REQUIRE(max_blocks >= 0 && max_blocks <= S / bs, OC_ERR_SHAPE,
             "attention: max_blocks %d > nb %d", max_blocks, S / bs);
  OC_REQUIRE(idx_stride >= 0 && idx_hstride >= 0, OC_ERR_SHAPE, "attention: negative index stride");
  OC_REQUIRE(aligned16(q) && aligned16(k) && aligned16(v), OC_ERR_ALIGN, "attention: q/k/v not 16-byte aligned");
  return OC_OK;
}

template <typename T, int D>
int launch_partials_d(const AttnArgs& a, int rt, int grid, cudaStream_t st) {
  if constexpr (Elem<T>::kVec * 32 < D) {
    return set_error(OC_ERR_UNSUPPORTED, "attention: float32 inputs support head_dim <= 128");
  } else {
  switch (rt) {
    case 1: attn_partial_kernel<T, D, 1><<<grid, kThreads, 0, st>>>(a); break;
    case 2: attn_partial_kernel<T, D, 2><<<grid, kThreads, 0, st>>>(a); break;
    case 4: attn_partial_kernel<T, D, 4><<<grid, kThreads, 0, st>>>(a); break;
    default:
      if constexpr (D == 256) attn_partial_kernel<T, D, 4><<<grid, kThreads, 0, st>>>(a);
      else attn_partial_kernel<T, D, 8><<<grid, kThreads, 0, st>>>(a);
      break;
  }
  return check_launch("attn_partial_kernel");
  }
}

template <typename T>
int launch_partials(const AttnArgs& a, int rt, int grid, cudaStream_t st) {
  switch (a.D) {
    case 64: return launch_partials_d<T, 64>(a, rt, grid, st);
    case 128: return launch_partials_d<T, 128>(a, rt, grid, st);
    default: return launch_partials_d<T, 256>(a, rt, grid, st);
  }
}

// Enqueue the partial + merge kernels.  mode 0: final output; mode 1: (m,l,o).
int run_attention(const void* q, const void* k, const void* v, int dtype, const int32_t* idx,
                  int idx_stride, int idx_hstride, const int32_t* count, int cnt_stride, int cnt_hstride,
                  int B, int Sq, int Hq, int Hkv, int D,
                  int S, int bs, int max_blocks, void* out, int out_dtype, float* pm, float* pl,
                  float* po, void* ws, size_t ws_bytes, int mode, cudaStream_t st,
                  const uint8_t* keep = nullptr, int32_t* perm_out = nullptr, int pool_pages = 0) {
  int rc = validate_attn(q, k, v, dtype, idx, idx_stride, idx_hstride, count, B, Sq, Hq, Hkv, D, S, bs,
                         max_blocks);
  if (rc) return rc;
  const size_t need = attn_ws_bytes(B, Sq, Hq, Hkv, D, bs, max_blocks);
  OC_REQUIRE(ws || need == 0, OC_ERR_NULL, "attention: workspace is NULL");
  OC_REQUIRE(ws_bytes >= need, OC_ERR_CAPACITY, "attention: workspace %zu bytes < %zu needed", ws_bytes, need);
  OC_REQUIRE(mode == 1 || out_dtype == OC_F32 || out_dtype == OC_BF16, OC_ERR_DTYPE,
             "attention: out_dtype %d", out_dtype);
  AttnArgs a;
  a.q = q; a.k = k; a.v = v; a.idx = idx; a.count = count;
  a.idx_stride = idx_stride; a.idx_hstride = idx_hstride;
  a.cnt_stride = cnt_stride; a.cnt_hstride = cnt_hstride;
  a.B = B; a.Sq = Sq; a.Hq = Hq; a.Hkv = Hkv; a.G = Hq / Hkv; a.D = D; a.S = S; a.bs = bs;
  // pool_pages > 0: k / v are a pool of pool_pages blocks shared by the
  // batch, and the index lists hold pool pages
  a.kv_rows = pool_pages > 0 ? 0 : S;
  a.nblk = pool_pages > 0 ? pool_pages : S / bs;
  a.R = Sq * a.G;
  const bool tma = use_tma_path(dtype, bs, D, (int64_t)B * Hkv);
  const bool mma = tma && (D == 64 || D == 128 || D == 256);  // tensor-core stream kernel
  int rt = pick_rt(a.R, D);
  if (tma && rt * D > 512) rt = 512 / D;
  if (tma && rt > 4) rt = 4;
  if (mma) rt = a.R <= 4 ? 4 : 8;
  a.n_rt = (a.R + rt - 1) / rt;
  a.chunk = chunk_for(bs, D);
  a.chunks = bs / a.chunk;
  a.max_items = max_blocks * a.chunks;
  a.scale_log2 = kLog2e / sqrtf((float)D);
  // Stream kernels: persistent grid; two CTAs per SM for the tensor-core one
  // (its 4 warps per CTA leave the SM latency-bound otherwise).
  a.run_grid = tma ? device_sm_count() * (mma ? 2 : 1) : 0;
  a.rt_tile = rt;
  const size_t parts = (size_t)B * a.max_items * Hkv * a.R;
  char* w = static_cast<char*>(ws);
  a.ws_m = reinterpret_cast<float*>(w);
  a.ws_l = reinterpret_cast<float*>(w + align256(parts * sizeof(float)));
  a.ws_o = reinterpret_cast<float*>(w + 2 * align256(parts * sizeof(float)));
  a.out = out;
  a.out_bf16 = out_dtype == OC_BF16;
  a.pm = pm; a.pl = pl; a.po = po;
  a.mode = mode;
  a.keep = keep;
  a.perm_out = perm_out;
  const int64_t rows = (int64_t)B * Hkv * a.R;
  OC_REQUIRE(rows < (1ll << 31), OC_ERR_CAPACITY, "attention: too many rows");

  const bool stream_path = tma && max_blocks > 0;
  if (stream_path) {
    rc = mma ? (D == 64    ? launch_attn_mma<64>(a, rt, st)
                : D == 128 ? launch_attn_mma<128>(a, rt, st)
                           : launch_attn_mma<256>(a, rt, st))
             : launch_attn_stream<256>(a, rt, st);
    if (rc) return rc;
  } else if (max_blocks > 0) {
    const int grid = device_sm_count() * 2;
    rc = dtype == OC_F32 ? launch_partials<float>(a, rt, grid, st)
                           : launch_partials<__nv_bfloat16>(a, rt, grid, st);
    if (rc) return rc;
  }
  // After a stream kernel the merge is a programmatic dependent launch: its
  // CTAs become resident while the stream kernel drains and wait for it with
  // griddepcontrol.wait before reading the run partials.
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.gridDim = dim3((unsigned)rows);
  cfg.blockDim = dim3(kMergeThreads);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = stream_path ? 1 : 0;
  cudaError_t e;
  if (mode == 0) {
    if (out_dtype == OC_F32)
      e = cudaLaunchKernelEx(&cfg, attn_merge_kernel<float>, a, (float*)out, (float*)nullptr, (float*)nullptr,
                             (float*)nullptr, 0);
    else
      e = cudaLaunchKernelEx(&cfg, attn_merge_kernel<__nv_bfloat16>, a, (__nv_bfloat16*)out, (float*)nullptr,
                             (float*)nullptr, (float*)nullptr, 0);
  } else {
    e = cudaLaunchKernelEx(&cfg, attn_merge_kernel<float>, a, (float*)nullptr, pm, pl, po, 1);
  }
  if (e != cudaSuccess) return set_error(OC_ERR_CUDA, "attn_merge_kernel: %s", cudaGetErrorString(e));
  return check_launch("attn_merge_kernel");
}

}  // namespace
}  // namespace oc

using namespace oc;

extern "C" size_t oc_indirect_attention_workspace_bytes(int batch, int q_len, int q_heads, int kv_heads,
                                                        int head_dim, int block_size, int max_blocks) {
  if (batch < 1 || q_len < 1 || kv_heads < 1 || q_heads % kv_heads || block_size < 64 || block_size % 64 ||
      (head_dim != 64 && head_dim != 128 && head_dim != 256) || max_blocks < 0)
    return 0;
  return attn_ws_bytes(batch, q_len, q_heads, kv_heads, head_dim, block_size, max_blocks);
}

extern "C" int oc_indirect_attention(const void* q, const void* k, const void* v, int dtype,
                                     const int32_t* idx, int idx_stride, int idx_head_stride,
                                     const int32_t* count, int count_stride, int count_head_stride,
                                     int batch, int q_len, int q_heads, int kv_heads, int head_dim,
                                     int seq_len, int block_size, int max_blocks,
                                     void* out, int out_dtype,
                                     void* workspace, size_t workspace_bytes, oc_stream_t stream) {
  OC_REQUIRE(out, OC_ERR_NULL, "oc_indirect_attention: out is NULL");
  return run_attention(q, k, v, dtype, idx, idx_stride, idx_head_stride, count, count_stride,
                       count_head_stride, batch, q_len, q_heads, kv_heads, head_dim,
                       seq_len, block_size, max_blocks, out, out_dtype, nullptr, nullptr, nullptr, workspace,
                       workspace_bytes, 0, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" size_t oc_indirect_attention_paged_workspace_bytes(int batch, int q_len, int q_heads, int kv_heads,
                                                              int head_dim, int block_size, int max_blocks) {
  const size_t attn = oc_indirect_attention_workspace_bytes(batch, q_len, q_heads, kv_heads, head_dim, block_size,
                                                            max_blocks);
  if (!attn && max_blocks > 0) return 0;
  return align256((size_t)batch * max_blocks * sizeof(int32_t)) + attn;
}

extern "C" int oc_indirect_attention_paged(const void* q, const void* k_pool, const void* v_pool, int dtype,
                                           const int32_t* block_table, int table_stride, const int32_t* idx,
                                           int idx_stride, const int32_t* count, int count_stride, int batch,
                                           int q_len, int q_heads, int kv_heads, int head_dim, int num_pages,
                                           int block_size, int max_blocks, void* out, int out_dtype,
                                           void* workspace, size_t workspace_bytes, oc_stream_t stream) {
  OC_REQUIRE(out && block_table && idx && count, OC_ERR_NULL, "oc_indirect_attention_paged: NULL pointer");
  OC_REQUIRE(num_pages >= 1 && table_stride >= 1 && max_blocks >= 0 && max_blocks <= table_stride, OC_ERR_SHAPE,
             "oc_indirect_attention_paged: num_pages %d, table_stride %d, max_blocks %d", num_pages, table_stride,
             max_blocks);
  OC_REQUIRE(idx_stride >= 0 && count_stride >= 0 && batch >= 1, OC_ERR_SHAPE, "oc_indirect_attention_paged: bad strides");
  const size_t need = oc_indirect_attention_paged_workspace_bytes(batch, q_len, q_heads, kv_heads, head_dim,
                                                                  block_size, max_blocks);
  OC_REQUIRE(need && workspace && workspace_bytes >= need, OC_ERR_CAPACITY,
             "oc_indirect_attention_paged: workspace %zu < %zu bytes", workspace_bytes, need);
  OC_REQUIRE((int64_t)num_pages * block_size < INT32_MAX, OC_ERR_SHAPE, "oc_indirect_attention_paged: pool too large");
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  int32_t* phys = static_cast<int32_t*>(workspace);
  const size_t lists = align256((size_t)batch * max_blocks * sizeof(int32_t));
  int rc = compose_page_lists(block_table, table_stride, table_stride, idx, idx_stride, count, count_stride, batch,
                              max_blocks, num_pages, phys, st);
  if (rc) return rc;
  return run_attention(q, k_pool, v_pool, dtype, phys, max_blocks, 0, count, count_stride, 0, batch, q_len, q_heads,
                       kv_heads, head_dim, table_stride * block_size, block_size, max_blocks, out, out_dtype, nullptr,
                       nullptr, nullptr, static_cast<char*>(workspace) + lists, workspace_bytes - lists, 0, st,
                       nullptr, nullptr, num_pages);
}

extern "C" int oc_partial_attention(const void* q, const void* k, const void* v, int dtype,
                                    const int32_t* idx, int idx_stride, int idx_head_stride,
                                    const int32_t* count, int count_stride, int count_head_stride,
                                    int batch, int q_len, int q_heads, int kv_heads, int head_dim,
                                    int seq_len, int block_size, int max_blocks,
                                    float* m, float* l, float* o,
                                    void* workspace, size_t workspace_bytes, oc_stream_t stream) {
  OC_REQUIRE(m && l && o, OC_ERR_NULL, "oc_partial_attention: m/l/o is NULL");
  return run_attention(q, k, v, dtype, idx, idx_stride, idx_head_stride, count, count_stride,
                       count_head_stride, batch, q_len, q_heads, kv_heads, head_dim,
                       seq_len, block_size, max_blocks, nullptr, OC_F32, m, l, o, workspace, workspace_bytes, 1,
                       reinterpret_cast<cudaStream_t>(stream));
}

namespace {
int merge_parts(const float* m, const float* l, const float* o, int parts, int rows, int head_dim, void* out,
                int out_dtype, size_t ml_stride, size_t o_stride, oc_stream_t stream) {
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (out_dtype == OC_F32)
    merge_parts_kernel<float><<<rows, 128, 0, st>>>(m, l, o, parts, rows, head_dim, (float*)out, ml_stride,
                                                    o_stride);
  else if (out_dtype == OC_BF16)
    merge_parts_kernel<__nv_bfloat16><<<rows, 128, 0, st>>>(m, l, o, parts, rows, head_dim,
                                                             (__nv_bfloat16*)out, ml_stride, o_stride);
  else
    return set_error(OC_ERR_DTYPE, "oc_merge_partials: out_dtype %d", out_dtype);
  return check_launch("merge_parts_kernel");
}
}  // namespace

extern "C" int oc_merge_partials(const float* m, const float* l, const float* o, int parts, int rows,
                                 int head_dim, void* out, int out_dtype, oc_stream_t stream) {
  OC_REQUIRE(m && l && o && out, OC_ERR_NULL, "oc_merge_partials: null pointer");
  OC_REQUIRE(parts >= 1 && rows >= 0 && head_dim >= 1, OC_ERR_SHAPE, "oc_merge_partials: bad shape");
  if (rows == 0) return OC_OK;
  return merge_parts(m, l, o, parts, rows, head_dim, out, out_dtype, (size_t)rows, (size_t)rows * head_dim,
                     stream);
}

extern "C" int oc_merge_partials_packed(const float* packed, int parts, int rows, int head_dim, void* out,
                                        int out_dtype, oc_stream_t stream) {
  OC_REQUIRE(packed && out, OC_ERR_NULL, "oc_merge_partials_packed: null pointer");
  OC_REQUIRE(parts >= 1 && rows >= 0 && head_dim >= 1, OC_ERR_SHAPE, "oc_merge_partials_packed: bad shape");
  if (rows == 0) return OC_OK;
  const size_t part = (size_t)rows * (head_dim + 2);
  return merge_parts(packed, packed + rows, packed + 2 * (size_t)rows, parts, rows, head_dim, out, out_dtype, part,
                     part, stream);
}

extern "C" size_t oc_decode_step_workspace_bytes(int batch, int q_len, int q_heads, int kv_heads,
                                                 int head_dim, int seq_len) {
  if (seq_len % 512 || seq_len < 512 || batch < 1 || kv_heads < 1 || q_len < 1 || q_heads % kv_heads ||
      (head_dim != 64 && head_dim != 128 && head_dim != 256))
    return 0;
  // The fused layer's region first (its counters stay zero between calls),
  // then the scratch of the separate score / attention path.
  return oc::decode_fused_bytes(batch, seq_len, kv_heads) +
         oc_indirect_attention_workspace_bytes(batch, q_len, q_heads, kv_heads, head_dim, 512, seq_len / 512);
}

extern "C" int oc_decode_step(const void* q, const void* k, const void* v, int dtype,
                              int batch, int q_len, int q_heads, int kv_heads, int head_dim, int seq_len,
                              float tau, float zeta_max,
                              uint8_t* keep, int32_t* perm, int32_t* count,
                              void* out, int out_dtype,
                              void* workspace, size_t workspace_bytes, oc_stream_t stream) {
  OC_REQUIRE(keep && perm && count && out, OC_ERR_NULL, "oc_decode_step: null output pointer");
  OC_REQUIRE(seq_len % 512 == 0, OC_ERR_SHAPE, "oc_decode_step: seq_len %d not a multiple of 512", seq_len);
  OC_REQUIRE(batch >= 1 && kv_heads >= 1, OC_ERR_SHAPE, "oc_decode_step: batch/kv_heads < 1");
  const int nb = seq_len / 512;
  const size_t fused_bytes = oc::decode_fused_bytes(batch, seq_len, kv_heads);
  OC_REQUIRE(workspace && workspace_bytes >= fused_bytes, OC_ERR_CAPACITY,
             "oc_decode_step: workspace of %zu bytes, need at least %zu", workspace_bytes, fused_bytes);
  if (dtype == OC_BF16 && seq_len > 0) {
    // One persistent kernel for the whole layer where the shape allows it.
    const int frc = oc::decode_fused(q, k, v, batch, q_len, q_heads, kv_heads, head_dim, seq_len, tau, zeta_max,
                                     keep, perm, count, out, out_dtype, nullptr, nullptr, nullptr, workspace,
                                     fused_bytes, reinterpret_cast<cudaStream_t>(stream));
    if (frc != OC_ERR_UNSUPPORTED) return frc;
  }
  workspace = static_cast<uint8_t*>(workspace) + fused_bytes;
  workspace_bytes -= fused_bytes;
  int rc = oc_score_blocks(k, q, dtype, batch, seq_len, kv_heads, head_dim, q_len, q_heads, 1, 64, 64, 256,
                           256, 512, tau, zeta_max, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr,
                           keep, 0, stream);
  if (rc) return rc;
  if (dtype == OC_BF16 && (head_dim == 64 || head_dim == 128) && batch * nb <= kKeepListMax) {
    // The compaction runs inside the tensor-core attention kernel.
    OC_REQUIRE(out, OC_ERR_NULL, "oc_decode_step: out is NULL");
    return run_attention(q, k, v, dtype, perm, nb, 0, count, 1, 0, batch, q_len, q_heads, kv_heads, head_dim,
                         seq_len, 512, nb, out, out_dtype, nullptr, nullptr, nullptr, workspace, workspace_bytes, 0,
                         reinterpret_cast<cudaStream_t>(stream), keep, perm);
  }
  rc = oc_stream_compact(keep, batch, nb, kv_heads, perm, count, stream);
  if (rc) return rc;
  return oc_indirect_attention(q, k, v, dtype, perm, nb, 0, count, 1, 0, batch, q_len, q_heads, kv_heads, head_dim,
                               seq_len, 512, nb, out, out_dtype, workspace, workspace_bytes, stream);
}

extern "C" int oc_decode_step_from_metadata(const void* q, const void* k, const void* v, int dtype,
                                            const float* dc, const float* e_ac, const float* zeta,
                                            int batch, int q_len, int q_heads, int kv_heads, int head_dim,
                                            int seq_len, float tau, float zeta_max,
                                            uint8_t* keep, int32_t* perm, int32_t* count,
                                            void* out, int out_dtype,
                                            void* workspace, size_t workspace_bytes, oc_stream_t stream) {
  OC_REQUIRE(keep && perm && count && out, OC_ERR_NULL, "oc_decode_step_from_metadata: null output pointer");
  OC_REQUIRE(dc && e_ac && zeta, OC_ERR_NULL, "oc_decode_step_from_metadata: null metadata pointer");
  OC_REQUIRE(seq_len >= 0 && seq_len % 512 == 0, OC_ERR_SHAPE,
             "oc_decode_step_from_metadata: seq_len %d not a non-negative multiple of 512", seq_len);
  OC_REQUIRE(batch >= 1 && kv_heads >= 1, OC_ERR_SHAPE, "oc_decode_step_from_metadata: batch/kv_heads < 1");
  OC_REQUIRE(head_dim == 64 || head_dim == 128 || head_dim == 256, OC_ERR_SHAPE,
             "oc_decode_step_from_metadata: head_dim %d not in {64,128,256}", head_dim);
  OC_REQUIRE(q_len >= 1 && q_heads >= kv_heads && q_heads % kv_heads == 0, OC_ERR_SHAPE,
             "oc_decode_step_from_metadata: q_heads %d must be a positive multiple of kv_heads %d (q_len %d)",
             q_heads, kv_heads, q_len);
  const int nb = seq_len / 512;
  const size_t fused_bytes = oc::decode_fused_bytes(batch, seq_len, kv_heads);
  OC_REQUIRE(workspace && workspace_bytes >= fused_bytes, OC_ERR_CAPACITY,
             "oc_decode_step_from_metadata: workspace of %zu bytes, need at least %zu", workspace_bytes,
             fused_bytes);
  if (dtype == OC_BF16 && seq_len > 0) {
    // One persistent kernel: decisions from the metadata, then attention.
    const int frc = oc::decode_fused(q, k, v, batch, q_len, q_heads, kv_heads, head_dim, seq_len, tau, zeta_max,
                                     keep, perm, count, out, out_dtype, nullptr, nullptr, nullptr, workspace,
                                     fused_bytes, reinterpret_cast<cudaStream_t>(stream), nullptr, dc, e_ac, zeta);
    if (frc != OC_ERR_UNSUPPORTED) return frc;
  }
  workspace = static_cast<uint8_t*>(workspace) + fused_bytes;
  workspace_bytes -= fused_bytes;
  int rc = oc_score_from_metadata(dc, e_ac, zeta, q, dtype, batch, nb, kv_heads, head_dim, q_len, q_heads, tau,
                                  zeta_max, nullptr, nullptr, keep, stream);
  if (rc) return rc;
  rc = oc_stream_compact(keep, batch, nb, kv_heads, perm, count, stream);
  if (rc) return rc;
  return oc_indirect_attention(q, k, v, dtype, perm, nb, 0, count, 1, 0, batch, q_len, q_heads, kv_heads, head_dim,
                               seq_len, 512, nb, out, out_dtype, workspace, workspace_bytes, stream);
}

extern "C" int oc_decode_step_partial(const void* q, const void* k, const void* v, int dtype,
                                      int batch, int q_len, int q_heads, int kv_heads, int head_dim, int seq_len,
                                      float tau, float zeta_max,
                                      uint8_t* keep, int32_t* perm, int32_t* count,
                                      float* m, float* l, float* o,
                                      void* workspace, size_t workspace_bytes, oc_stream_t stream) {
  OC_REQUIRE(keep && perm && count && m && l && o, OC_ERR_NULL, "oc_decode_step_partial: null output pointer");
  OC_REQUIRE(seq_len % 512 == 0, OC_ERR_SHAPE, "oc_decode_step_partial: seq_len %d not a multiple of 512",
             seq_len);
  OC_REQUIRE(batch >= 1 && kv_heads >= 1, OC_ERR_SHAPE, "oc_decode_step_partial: batch/kv_heads < 1");
  const int nb = seq_len / 512;
  const size_t fused_bytes = oc::decode_fused_bytes(batch, seq_len, kv_heads);
  OC_REQUIRE(workspace && workspace_bytes >= fused_bytes, OC_ERR_CAPACITY,
             "oc_decode_step_partial: workspace of %zu bytes, need at least %zu", workspace_bytes, fused_bytes);
  if (dtype == OC_BF16 && seq_len > 0) {
    const int frc = oc::decode_fused(q, k, v, batch, q_len, q_heads, kv_heads, head_dim, seq_len, tau, zeta_max,
                                     keep, perm, count, nullptr, OC_F32, m, l, o, workspace, fused_bytes,
                                     reinterpret_cast<cudaStream_t>(stream));
    if (frc != OC_ERR_UNSUPPORTED) return frc;
  }
  workspace = static_cast<uint8_t*>(workspace) + fused_bytes;
  workspace_bytes -= fused_bytes;
  int rc = oc_score_blocks(k, q, dtype, batch, seq_len, kv_heads, head_dim, q_len, q_heads, 1, 64, 64, 256,
                           256, 512, tau, zeta_max, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr,
                           keep, 0, stream);
  if (rc) return rc;
  rc = oc_stream_compact(keep, batch, nb, kv_heads, perm, count, stream);
  if (rc) return rc;
  return oc_partial_attention(q, k, v, dtype, perm, nb, 0, count, 1, 0, batch, q_len, q_heads, kv_heads, head_dim,
                              seq_len, 512, nb, m, l, o, workspace, workspace_bytes, stream);
}

extern "C" int oc_empty_heads_mean(const void* v, int dtype, const int32_t* count, int count_stride,
                                   int count_head_stride, int batch, int q_len, int q_heads, int kv_heads,
                                   int head_dim, int seq_len, void* out, int out_dtype, oc_stream_t stream) {
  OC_REQUIRE(v && count && out, OC_ERR_NULL, "oc_empty_heads_mean: null pointer");
  OC_REQUIRE(head_dim == 64 || head_dim == 128 || head_dim == 256, OC_ERR_SHAPE, "oc_empty_heads_mean: head_dim");
  OC_REQUIRE(batch >= 1 && kv_heads >= 1 && q_heads % kv_heads == 0 && seq_len >= 1, OC_ERR_SHAPE,
             "oc_empty_heads_mean: bad shape");
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const int grid = batch * kv_heads;
#define OC_EHM(T, TO) empty_heads_mean_kernel<T, TO><<<grid, 256, 0, st>>>((const T*)v, count, count_stride, \
      count_head_stride, q_len, q_heads, kv_heads, head_dim, seq_len, (TO*)out)
  if (dtype == OC_F32 && out_dtype == OC_F32) OC_EHM(float, float);
  else if (dtype == OC_F32 && out_dtype == OC_BF16) OC_EHM(float, __nv_bfloat16);
  else if (dtype == OC_BF16 && out_dtype == OC_F32) OC_EHM(__nv_bfloat16, float);
  else if (dtype == OC_BF16 && out_dtype == OC_BF16) OC_EHM(__nv_bfloat16, __nv_bfloat16);
  else return set_error(OC_ERR_DTYPE, "oc_empty_heads_mean: dtype %d / %d", dtype, out_dtype);
#undef OC_EHM
  return check_launch("empty_heads_mean_kernel");
}

namespace oc {
int wait_limit_attn(unsigned long long ns) { return set_wait_limit_here(ns); }
int attn_status(int* status, int reset) {
  cudaError_t e = cudaMemcpyFromSymbol(status, g_attn_status, sizeof(int));
  if (e != cudaSuccess) return set_error(OC_ERR_CUDA, "oc_device_status: %s", cudaGetErrorString(e));
  if (reset) {
    const int zero = 0;
    e = cudaMemcpyToSymbol(g_attn_status, &zero, sizeof(int));
    if (e != cudaSuccess) return set_error(OC_ERR_CUDA, "oc_device_status: %s", cudaGetErrorString(e));
  }
  return OC_OK;
}
}  // namespace oc

// ---------------------------------------------------------------------------
// Indirect attention without any allocation (no counterpart in the reference).
//
// Some callers cannot allocate device memory at the point where they run the
// attention: code inside a custom memory pool or a framework that forbids
// allocations during a decode step, an FFI host that has no CUDA allocator of
// its own, or a process whose allocator is already exhausted.  For them this
// entry point takes its scratch (the per-chunk (m, l, o) partials of the
// split-KV attention) from a file-scope device array that exists on every GPU
// that loads this library, for the life of the process.
// ---------------------------------------------------------------------------
namespace oc {
namespace {

constexpr size_t kNoAllocScratchBytes = 32u << 20;  // 32 MiB per device
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

constexpr int kMaxDevices = 64;
void* g_noalloc_ptr[kMaxDevices] = {};
std::mutex g_noalloc_mu;

// Device address of the scratch array on the current device.  Host code may
// not use the symbol itself: on the host it names a stand-in, not GPU memory.
int noalloc_scratch(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return set_error(OC_ERR_CUDA, "oc_indirect_attention_noalloc: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices)
    return set_error(OC_ERR_UNSUPPORTED, "oc_indirect_attention_noalloc: device %d >= %d", dev, kMaxDevices);
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (!g_noalloc_ptr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || !p)
      return set_error(OC_ERR_CUDA, "oc_indirect_attention_noalloc: cudaGetSymbolAddress: %s",
                       cudaGetErrorString(e));
    g_noalloc_ptr[dev] = p;
  }
  *out = g_noalloc_ptr[dev];
  return OC_OK;
}

}  // namespace
}  // namespace oc

extern "C" size_t oc_indirect_attention_noalloc_max_scratch_bytes(void) { return oc::kNoAllocScratchBytes; }

extern "C" int oc_indirect_attention_noalloc(const void* q, const void* k, const void* v, int dtype,
                                             const int32_t* idx, int idx_stride, int idx_head_stride,
                                             const int32_t* count, int count_stride, int count_head_stride,
                                             int batch, int q_len, int q_heads, int kv_heads, int head_dim,
                                             int seq_len, int block_size, int max_blocks,
                                             void* out, int out_dtype, oc_stream_t stream) {
  OC_REQUIRE(out, OC_ERR_NULL, "oc_indirect_attention_noalloc: out is NULL");
  OC_REQUIRE(batch >= 1 && q_len >= 1 && kv_heads >= 1 && q_heads >= kv_heads && q_heads % kv_heads == 0 &&
                 block_size >= 64 && block_size % 64 == 0 && max_blocks >= 0 &&
                 (head_dim == 64 || head_dim == 128 || head_dim == 256),
             OC_ERR_SHAPE, "oc_indirect_attention_noalloc: bad shape (head_dim must be 64, 128 or 256)");
  const size_t need = oc::attn_ws_bytes(batch, q_len, q_heads, kv_heads, head_dim, block_size, max_blocks);
  OC_REQUIRE(need <= oc::kNoAllocScratchBytes, OC_ERR_CAPACITY,
             "oc_indirect_attention_noalloc: this shape needs %zu bytes of scratch, above the fixed %zu-byte "
             "limit; use oc_indirect_attention with a caller-provided workspace",
             need, oc::kNoAllocScratchBytes);
  void* scratch = nullptr;
  int rc = oc::noalloc_scratch(&scratch);
  if (rc) return rc;
  // Every partial the merge reads is written first by the partial kernel of
  // the same call, so the scratch needs no clearing between calls.
  return oc::run_attention(q, k, v, dtype, idx, idx_stride, idx_head_stride, count, count_stride,
                           count_head_stride, batch, q_len, q_heads, kv_heads, head_dim, seq_len, block_size,
                           max_blocks, out, out_dtype, nullptr, nullptr, nullptr, scratch, oc::kNoAllocScratchBytes,
                           0, reinterpret_cast<cudaStream_t>(stream));
}

#ifdef OC_TIMING
extern "C" int oc_probe_read_stamps(unsigned long long* host, int n) {
  return (int)cudaMemcpyFromSymbol(host, oc::g_tstamp, sizeof(unsigned long long) * 8 * n);
}
#endif
