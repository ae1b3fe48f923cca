// Block scorer: Walsh–Hadamard spectral bands, ζ, query-aware logit bound and
// the two-gate keep mask, in one pass over the keys; plus the stand-alone
// 512-point FWHT.
//
// Reference semantics (j-arndt/orthocache v0.3.0):
//   fwht_512                     src/orthocache/fwht.py:4-65
//   _run_fwht_on_blocks          src/orthocache/spectral_energy.py:38-66
//   compute_spectral_bands       spectral_energy.py:69-106
//   compute_spectral_decay_ratio spectral_energy.py:109-138
//   compute_query_aware_bounds   spectral_energy.py:141-177
//   compute_query_aware_mask     spectral_energy.py:180-196
//   compute_multiband_mask       spectral_energy.py:199-234
//
// Two scorers share one epilogue:
//
//  * Partial-transform scorer (mode 1; default when every band edge is 0, 1 or
//    a multiple of 64).  Write the token index of a 512-block as
//    i = 64*i_hi + i_lo and the coefficient index as k = 64*k_hi + k_lo.  The
//    natural-order WHT factors as  c[k] = sum_{i_lo} (-1)^{k_lo.i_lo} y[k_hi,i_lo]
//    with  y[k_hi, i_lo] = sum_{i_hi} (-1)^{k_hi.i_hi} x[64 i_hi + i_lo]  — the
//    last three butterfly stages (h = 64, 128, 256) applied first.  By
//    Parseval over the 64-point inner transform, the energy of coefficient
//    group k_hi (indices 64 k_hi .. 64 k_hi + 63) is sum_{i_lo} y[k_hi,i_lo]^2 / 8
//    after the reference's 1/sqrt(512) normalisation, and the energy of
//    indices 1..63 is the centred sum  sum (y[0,i_lo] - mean)^2 / 8 (two-pass,
//    so no cancellation against a large DC term).  DC = sum_{i_lo} y[0,i_lo]
//    / sqrt(512).  Every band of the reference (1-63, 64-255, 256-511) is a
//    union of these groups, so the band energies need 3 butterfly stages per
//    element instead of 9; the results equal the reference's up to float32
//    summation order.
//
//  * Full-butterfly scorer (mode 2; any bands).  All 9 stages in the
//    reference's order in shared memory, coefficient by coefficient, then band
//    sums of coef^2.  Coefficients are bit-identical to fwht_512.
//
// One CTA scores one (batch, block, kv-head) tile of 512 x D keys.
#include "oc_common.cuh"
#include "oc_tma.cuh"
#include "oc_mma.cuh"
#include "oc_tcgen05.cuh"

#include <math.h>
#include <algorithm>
#include <type_traits>

namespace oc {
namespace {

constexpr int kBlock = 512;
constexpr int kThreads = 256;
constexpr float kNorm = 22.627416997969522f;  // fwht.py:61, rounded to float32

struct Bands {
  int lo[3], hi[3];  // low, mid, high: [lo, hi) in natural coefficient order
};

struct ScoreArgs {
  const void* keys;
  const void* q;
  int S, H, D, nb;
  int Sq, Hq, G;
  Bands bands;
  float tau, zeta_max;
  float* dc;
  float* e_low;
  float* e_mid;
  float* e_high;
  float* zeta;
  float* bound_max;
  float* bounds;  // (B, Sq, nb, Hq) or null
  float* e_ac;    // (B, nb, H) energy of coefficients 1..511, or null
  uint8_t* keep;
};

// ---------------------------------------------------------------------------
// Epilogue shared by both scorers.  Inputs in shared memory: dc_coef[D]
// (normalised WHT coefficient 0 per column) and band[4] = {E_low, E_mid,
// E_high, E_AC}.  Computes the bound over the Sq*G query rows of this KV head
// (spectral_energy.py:150-177), its max (:195), ζ (:138) and the keep bit
// (:196, :231-234).
// ---------------------------------------------------------------------------
// Synchronisation of a 256-thread group: the whole CTA, or one named barrier.
struct CtaSync {
  __device__ void operator()() const { __syncthreads(); }
};
struct GroupSync {
  int id;  // named barrier 1 or 2
  __device__ void operator()() const { asm volatile("bar.sync %0, 256;" ::"r"(id) : "memory"); }
};

template <typename T, typename Sync = CtaSync>
__device__ void score_epilogue(const ScoreArgs& a, int b, int j, int h,
                               const float* dc_coef, const float* band, float* red,
                               int tid = threadIdx.x, Sync sync = Sync()) {
  const int lane = tid & 31, warp = tid >> 5;
  const int D = a.D;
  const size_t cell = ((size_t)b * a.nb + j) * a.H + h;
  if (a.dc)
    for (int c = tid; c < D; c += kThreads) a.dc[cell * D + c] = dc_coef[c];

  float bmax = -INFINITY;
  if (a.q) {
    const float e_ac = band[3];
    const float sqrt_d = sqrtf((float)D);
    const float resid_scale = sqrtf(e_ac);
    const int rows = a.Sq * a.G;
    const T* qb = reinterpret_cast<const T*>(a.q) + (size_t)b * a.Sq * a.Hq * D;
    for (int r = warp; r < rows; r += kThreads / 32) {
      const int s = r / a.G, g = r - s * a.G;
      const T* qr = qb + ((size_t)s * a.Hq + (size_t)h * a.G + g) * D;
      float dot = 0.f, nrm = 0.f;
      for (int c = lane; c < D; c += 32) {
        const float qv = to_f32<T>(qr[c]);
        const float mean = dc_coef[c] / kNorm;  // block mean = DC / sqrt(512)  (:166)
        dot = fmaf(qv, mean, dot);
        nrm = fmaf(qv, qv, nrm);
      }
      dot = warp_sum(dot);
      nrm = warp_sum(nrm);
      const float align = dot / sqrt_d;                        // (:169)
      const float resid = (sqrtf(nrm) * resid_scale) / sqrt_d;  // (:172-175)
      const float bound = align + resid;
      if (a.bounds && lane == 0)
        a.bounds[(((size_t)b * a.Sq + s) * a.nb + j) * a.Hq + (size_t)h * a.G + g] = bound;
      bmax = fmaxf(bmax, bound);
    }
    if (lane == 0) red[warp] = bmax;
    sync();
    bmax = red[0];
#pragma unroll
    for (int w = 1; w < kThreads / 32; ++w) bmax = fmaxf(bmax, red[w]);
    sync();  // red is reused by the caller
  }
  if (tid == 0) {
    const float z = band[2] / (band[0] + 1e-6f);  // (:138)
    if (a.e_low) a.e_low[cell] = band[0];
    if (a.e_mid) a.e_mid[cell] = band[1];
    if (a.e_high) a.e_high[cell] = band[2];
    if (a.zeta) a.zeta[cell] = z;
    if (a.e_ac) a.e_ac[cell] = band[3];
    if (a.q && a.bound_max) a.bound_max[cell] = bmax;
    if (a.keep) {
      const bool gate1 = a.q ? (bmax >= a.tau) : true;
      a.keep[cell] = (gate1 && (z <= a.zeta_max)) ? 1 : 0;
    }
  }
}

// Energy of band [lo, hi) from the 8 coefficient-group energies of the
// partial transform (grp[0] excludes the DC coefficient) and the DC energy.
__device__ __forceinline__ float band_from_groups(int lo, int hi, const float* grp, float e_dc) {
  float e = 0.f;
  if (lo == 0 && hi >= 1) e += e_dc;
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const int glo = k == 0 ? 1 : 64 * k;
    if (lo <= glo && hi >= 64 * (k + 1)) e += grp[k];
  }
  return e;
}

// ---------------------------------------------------------------------------
// Partial-transform scorer.
// Thread t owns column group cg = t % CG (VEC consecutive columns, one 16-byte
// vector) and the inner token offsets i_lo = t / CG + n * (256 / CG).  For
// each i_lo it loads the 8 tokens i_lo + 64 * i_hi, runs the butterfly
// stages h = 64, 128, 256 across them and accumulates the squared results
// per coefficient group.
// ---------------------------------------------------------------------------
template <typename T, int D>
__global__ void __launch_bounds__(kThreads)
score_partial_kernel(ScoreArgs a) {
  constexpr int VEC = Elem<T>::kVec;
  constexpr int CG = D / VEC;
  constexpr int STEP = kThreads / CG;  // i_lo stride between a thread's items
  constexpr int ITEMS = 64 / STEP;
  static_assert(kThreads % CG == 0 && 64 % STEP == 0, "tile mapping");

  __shared__ float s_part[STEP][D];  // per-thread-row column sums of y0
  __shared__ float s_dc[D];
  __shared__ float s_mean[D];
  __shared__ float s_grp[kThreads / 32][8];
  __shared__ float s_band[4];
  __shared__ float s_red[kThreads / 32];

  const int tid = threadIdx.x;
  const int h = blockIdx.x % a.H;
  const int j = (blockIdx.x / a.H) % a.nb;
  const int b = blockIdx.x / (a.H * a.nb);
  const int cg = tid % CG;
  const int row0 = tid / CG;

  const T* base = reinterpret_cast<const T*>(a.keys) +
                  (((size_t)b * a.S + (size_t)j * kBlock) * a.H + h) * D + cg * VEC;
  const size_t tok_stride = (size_t)a.H * D;  // elements between consecutive tokens

  float y0[ITEMS][VEC];
  float grp[8];
#pragma unroll
  for (int k = 0; k < 8; ++k) grp[k] = 0.f;
  float colsum[VEC];
#pragma unroll
  for (int v = 0; v < VEC; ++v) colsum[v] = 0.f;

  // Software pipeline: the 8 loads of item it+1 are in flight while item it
  // is transformed.
  uint4 raw[8], nxt[8];
#pragma unroll
  for (int ih = 0; ih < 8; ++ih) raw[ih] = ldg_stream(base + (size_t)(ih * 64 + row0) * tok_stride);
#pragma unroll
  for (int it = 0; it < ITEMS; ++it) {
    if (it + 1 < ITEMS) {
      const int ilo_n = row0 + (it + 1) * STEP;
#pragma unroll
      for (int ih = 0; ih < 8; ++ih) nxt[ih] = ldg_stream(base + (size_t)(ih * 64 + ilo_n) * tok_stride);
    }
    {
      float x[8][VEC];
#pragma unroll
      for (int ih = 0; ih < 8; ++ih) unpack16<T>(raw[ih], x[ih]);
#pragma unroll
      for (int v = 0; v < VEC; ++v) {
        // stage h = 64 (token bit 6)
        float a0 = x[0][v] + x[1][v], a1 = x[0][v] - x[1][v];
        float a2 = x[2][v] + x[3][v], a3 = x[2][v] - x[3][v];
        float a4 = x[4][v] + x[5][v], a5 = x[4][v] - x[5][v];
        float a6 = x[6][v] + x[7][v], a7 = x[6][v] - x[7][v];
        // stage h = 128 (bit 7)
        float b0 = a0 + a2, b2 = a0 - a2, b1 = a1 + a3, b3 = a1 - a3;
        float b4 = a4 + a6, b6 = a4 - a6, b5 = a5 + a7, b7 = a5 - a7;
        // stage h = 256 (bit 8)
        float c0 = b0 + b4, c4 = b0 - b4, c1 = b1 + b5, c5 = b1 - b5;
        float c2 = b2 + b6, c6 = b2 - b6, c3 = b3 + b7, c7 = b3 - b7;
        y0[it][v] = c0;
        colsum[v] += c0;
        grp[1] = fmaf(c1, c1, grp[1]);
        grp[2] = fmaf(c2, c2, grp[2]);
        grp[3] = fmaf(c3, c3, grp[3]);
        grp[4] = fmaf(c4, c4, grp[4]);
        grp[5] = fmaf(c5, c5, grp[5]);
        grp[6] = fmaf(c6, c6, grp[6]);
        grp[7] = fmaf(c7, c7, grp[7]);
      }
    }
    if (it + 1 < ITEMS) {
#pragma unroll
      for (int ih = 0; ih < 8; ++ih) raw[ih] = nxt[ih];
    }
  }

  // Column sums of y0 over the 64 inner offsets -> DC (deterministic order).
#pragma unroll
  for (int v = 0; v < VEC; ++v) s_part[row0][cg * VEC + v] = colsum[v];
  __syncthreads();
  for (int c = tid; c < D; c += kThreads) {
    float s = 0.f;
    for (int r = 0; r < STEP; ++r) s += s_part[r][c];
    s_mean[c] = s * (1.0f / 64.0f);
    s_dc[c] = s / kNorm;
  }
  __syncthreads();

  // Second pass: centred energy of group 0 (coefficients 1..63).
  float g0 = 0.f;
#pragma unroll
  for (int it = 0; it < ITEMS; ++it)
#pragma unroll
    for (int v = 0; v < VEC; ++v) {
      const float d = y0[it][v] - s_mean[cg * VEC + v];
      g0 = fmaf(d, d, g0);
    }
  grp[0] = g0;

  const int lane = tid & 31, warp = tid >> 5;
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const float s = warp_sum(grp[k]);
    if (lane == 0) s_grp[warp][k] = s;
  }
  __syncthreads();
  if (tid == 0) {
    float g[8];
    for (int k = 0; k < 8; ++k) {
      float s = 0.f;
      for (int w = 0; w < kThreads / 32; ++w) s += s_grp[w][k];
      g[k] = s * 0.125f;  // (64 / 512) Parseval factor of the inner transform
    }
    float e_dc = 0.f;
    for (int c = 0; c < D; ++c) e_dc = fmaf(s_dc[c], s_dc[c], e_dc);
    float e_ac = 0.f;
    for (int k = 0; k < 8; ++k) e_ac += g[k];
    s_band[0] = band_from_groups(a.bands.lo[0], a.bands.hi[0], g, e_dc);
    s_band[1] = band_from_groups(a.bands.lo[1], a.bands.hi[1], g, e_dc);
    s_band[2] = band_from_groups(a.bands.lo[2], a.bands.hi[2], g, e_dc);
    s_band[3] = e_ac;
  }
  __syncthreads();
  score_epilogue<T>(a, b, j, h, s_dc, s_band, s_red);
}


// ---------------------------------------------------------------------------
// Partial-transform scorer, bfloat16 keys, bulk-tensor pipeline.
//
// Persistent grid, one CTA per SM.  The unit of work is a slab of 512 tokens
// x 64 channels of one (batch, block, kv head) tile (64 KB); a tile of D
// channels is D / 64 consecutive slabs.  Thread 0 keeps kStages slabs in
// flight with 4-D tensor loads (one box per half of the inner offsets) into
// a ring of shared-memory stages, each completed on its own mbarrier.
//
// With token i = 64 i_hi + i_lo, the natural-order transform factors as
// H512 = H8 (x) H64, and coefficient group q (indices 64q .. 64q+63) holds
// the 64-point transform of z_q(i_lo) = sum_i_hi H8[q][i_hi] x(64 i_hi + i_lo).
// By Parseval its energy is (64 / 512) sum_i_lo z_q^2, except group 0, whose
// coefficient 0 (the DC) is split off: (64 / 512) sum (z_0 - mean z_0)^2.
// The 8-point transforms run on the tensor cores: each warp takes one
// 8-channel chunk and 32 inner offsets of a slab, loads them as transposed
// 8x8 matrices (ldmatrix) and multiplies by diag(H8, H8) (m16n8k16, fp32
// accumulation; sums of eight bfloat16 values are exact in fp32), then
// squares and sums the results in registers.  The stage is refilled with
// the slab kStages ahead as soon as the last warp holds its operands.
// Band sums and the DC column sums accumulate across the slabs of a tile; the
// tile's epilogue (bound, ζ, keep) runs after its last slab.
// ---------------------------------------------------------------------------
// Packed float32x2 arithmetic (sm_100a): one instruction for two lanes of math.
typedef unsigned long long f32x2;
__device__ __forceinline__ f32x2 pack2(float lo, float hi) {
  f32x2 r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ void unpack2(f32x2 v, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ f32x2 add2(f32x2 a, f32x2 b) {
  f32x2 d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ f32x2 sub2(f32x2 a, f32x2 b) {
  f32x2 d;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ f32x2 fma2(f32x2 a, f32x2 b, f32x2 c) {
  f32x2 d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}

// ldmatrix of four transposed 8x8 bf16 matrices: lane (g, c) receives
// M[2c][g], M[2c + 1][g] of each matrix (row addresses from lanes 8m .. 8m+7).
__device__ __forceinline__ void ldsm_x4_trans(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr)
               : "memory");
}

// D = diag(H8, H8) B + C on the tensor cores (m16n8k16, bf16 in, fp32 out):
// A fragment a0 = a3 = hA, a1 = a2 = 0; C = (c0, c1) on both row halves.
__device__ __forceinline__ void mma_h8(float (&d)[4], uint32_t hA, uint32_t b0, uint32_t b1, float c0, float c1) {
  const uint32_t zero = 0;
  asm("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%10, %11, %12, %13};"
      : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
      : "r"(hA), "r"(zero), "r"(zero), "r"(hA), "r"(b0), "r"(b1), "f"(c0), "f"(c1), "f"(c0), "f"(c1));
}

// Sum each of v[0..7] over the warp; lanes 4r .. 4r+3 return the sum of v[r]
// (halving exchanges, 9 shuffles instead of 40).
__device__ __forceinline__ float transpose_sum8(float (&v)[8], int lane) {
#pragma unroll
  for (int o = 16, c = 8; o >= 4; o >>= 1, c >>= 1) {
    const bool up = (lane & o) != 0;
#pragma unroll
    for (int i = 0; i < 4; ++i)
      if (i < c / 2) {
        const float send = up ? v[i] : v[i + c / 2];
        const float keep = up ? v[i + c / 2] : v[i];
        v[i] = keep + __shfl_xor_sync(0xffffffffu, send, o);
      }
  }
  v[0] += __shfl_xor_sync(0xffffffffu, v[0], 2);
  v[0] += __shfl_xor_sync(0xffffffffu, v[0], 1);
  return v[0];
}

constexpr int kStages = 3;
constexpr int kScoreThreads = 512;  // compute warps
constexpr int kEpiWarps = 4;        // epilogue warps (and tile buffers)
constexpr int kQCacheBytes = 16384;  // queries staged in shared memory up to this size  // 16 warps consume every stage in order
constexpr int kSlabC = 64;                                  // channels per slab
constexpr int kSlabB = kBlock * kSlabC * 2;                 // bytes per slab (bf16)

__device__ int g_score_status = 0;

#ifdef OC_TIMING
// Diagnostic build only: per-CTA time stamps of the pipelined scorer.
__device__ unsigned long long g_sstamp[1024][24];
#define OC_SSTAMP(i, v) do { if (blockIdx.x < 1024) g_sstamp[blockIdx.x][i] = (v); } while (0)
#else
#define OC_SSTAMP(i, v) do {} while (0)
#endif

// ---------------------------------------------------------------------------
// Fused decode layer (score -> compact -> attend -> merge in one launch).
//
// The scorer kernel below, instantiated with FUSED = true, goes on from the
// keep mask to the attention of pipeline.orthocache_forward(mode='compact')
// (src/orthocache/pipeline.py:100-149): the union compaction of
// compaction.py:65,76-82 and the online-softmax attention over the retained
// blocks of adaptive_attention.py:46-76 / distributed_attention.py:95-128.
//
//  * Block decisions.  When the epilogue of tile (b, j, h) has its keep bit,
//    it adds (1 + keep << 16) to blk_state[b, j].  The epilogue that brings
//    the head count to H decides block j: if any head kept it, j is appended
//    to queue[b] (slot = tail[b]++), then decided[b]++.  Blocks therefore
//    enter the queue while the rest of the keys are still being scored.
//  * Attention work.  CTA x serves group (b, h) = x mod (B * Hkv); its
//    producer warp claims units (queue slot, 128-token chunk) from
//    grp_ctr[group], waits (bounded) until the slot is published, and loads
//    the chunk's K and V (64 KB) into the stage ring the scorer used.  The
//    16 compute warps run QK^T and PV with m16n8k16 MMAs (warp = 16 tokens x
//    64 value channels) and keep one online-softmax state per warp for the
//    CTA's whole run, so each CTA emits one (m, l, o) partial per group row.
//  * Merge.  The last CTA of a group to finish combines the group's
//    partials in log-sum-exp form and writes the output rows.  The epilogue
//    that completes a batch row's decisions writes that row's stable
//    active-first permutation and count from blk_state, long before the
//    attention ends.
//  * Counters.  The workspace holds an epoch and two counter sets; a call
//    uses set (epoch & 1), CTA 0 clears the other set for the next call, and
//    the last row decision advances the epoch.  No CTA waits for the grid to
//    finish, so the kernel ends with the last group merge.
// ---------------------------------------------------------------------------
constexpr int kFusedChunk = 128;           // tokens per attention unit
constexpr int kFusedMaxRows = 8;           // query rows per KV head (Sq * G)
constexpr int kFusedMaxGrid = 256;
constexpr int kMergeRound = 20;            // partials per load round of a group merge
constexpr int kFusedThreads = kScoreThreads + kEpiWarps * 32;

struct FusedArgs {
  int* epoch;       // calls so far; counter set (epoch & 1) serves this call
  int* sets;        // two counter sets of set_ints ints (FusedSet layout)
  int set_ints;
  float* part_m;    // (NG, cpg, kFusedMaxRows)
  float* part_l;
  float* part_o;    // (NG, cpg, kFusedMaxRows, D)
  void* out;        // (B, Sq, Hq, D)
  int out_bf16;
  float* pm;        // non-null: write the layer's (m, l, o) per output row
  float* pl;        //   instead of out (log2 units, as oc_partial_attention)
  float* po;
  int32_t* perm;    // (B, nb)
  int32_t* count;   // (B)
  int B, NG, cpg, R;
  float scale_log2;
  PeerXchg px;      // px.P > 0: merge this shard's partial with every rank's by peer stores
};

// One call's counters.  A call uses set (epoch & 1); CTA 0 zeroes the other
// set when it starts (the call before, its last user, has completed), so the
// set is zero when the next call picks it up.
struct FusedSet {
  int* blk_state;    // (B * nb): heads decided | heads kept << 16
  int* queue;        // (B * nb): 1 + block index, in decision order
  int* row;          // (B) blocks decided | blocks kept (queue tail) << 16
  int* decided_all;  // (1) batch rows fully decided
  int* grp_ctr;      // (NG) next unit of group (b, h)
  int* grp_done;     // (NG) CTAs of the group that published their partial
};
__host__ __device__ __forceinline__ int fused_set_ints(int B, int nb, int NG) { return 2 * B * nb + B + 1 + 2 * NG; }
__device__ __forceinline__ FusedSet fused_set(const FusedArgs& f, int nb, int which) {
  FusedSet t;
  int* c = f.sets + (size_t)which * f.set_ints;
  t.blk_state = c; c += (size_t)f.B * nb;
  t.queue = c; c += (size_t)f.B * nb;
  t.row = c; c += f.B;
  t.decided_all = c; c += 1;
  t.grp_ctr = c; c += f.NG;
  t.grp_done = c;
  return t;
}

__device__ __forceinline__ void st_release(int* p, int v) {
  asm volatile("st.release.gpu.global.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ int atom_add_acq_rel(int* p, int v) {
  int old;
  asm volatile("atom.add.acq_rel.gpu.global.s32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
  return old;
}
__device__ __forceinline__ int ld_relaxed(const int* p) {
  int v;
  asm volatile("ld.relaxed.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ int ld_acquire(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Fused: every warp calls this once, with all 32 lanes, when it has no work
// left.  The CTA's last warp counts the CTA out of the grid; the grid's last
// CTA writes the permutation and counts and zeroes the state.
// Stable active-first permutation and count of batch row b from the final
// block states (compaction.py:76-82: active blocks ascending, then the others
// ascending); one warp, 256 blocks per sweep with their states loaded at once.
__device__ __forceinline__ void fused_write_perm(const int* st, int nb, int32_t* perm, int32_t* count, int lane) {
  int n_act = 0;
  for (int pass = 0; pass < 2; ++pass) {
    int base = pass == 0 ? 0 : n_act;
    for (int j0 = 0; j0 < nb; j0 += 256) {
      int v[8];
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        const int j = j0 + 32 * c + lane;
        v[c] = j < nb ? __ldcg(st + j) : -1;
      }
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        const bool take = v[c] >= 0 && ((v[c] >> 16) > 0) == (pass == 0);
        const unsigned m = __ballot_sync(0xffffffffu, take);
        if (take) perm[base + __popc(m & ((1u << lane) - 1u))] = j0 + 32 * c + lane;
        base += __popc(m);
      }
    }
    if (pass == 0) {
      n_act = base;
      if (lane == 0) *count = n_act;
    }
  }
}

// Words of the cross-GPU exchange: one aligned 8-byte store / load each
// (single-copy atomic), relaxed at system scope (a volatile store is one);
// a word is this call's when its high half is the call number + 1 (slots
// alternate by parity, so a stale word holds an older number).  The store
// is a volatile access rather than inline assembly with a memory clobber:
// the clobber would also pin the single-GPU merge loop's loads in place.
__device__ __forceinline__ void xchg_put(uint64_t* p, uint64_t v) { *reinterpret_cast<volatile uint64_t*>(p) = v; }
__device__ __forceinline__ uint64_t xchg_get(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// The cross-GPU half of the fused layer's group merge (FusedArgs::px): kept
// out of line so that the single-GPU kernel's register allocation does not
// pay for it.  The calling CTA has stored this shard's partial of the group
// into every rank's slot; each thread here waits (bounded) for the words of
// its output element from every rank and merges the P partials: out on
// every rank.
struct PeerMergeArgs {
  PeerXchg px;
  int NG, R, G, Sq, Hq, out_bf16;
  void* out;
};

__device__ __noinline__ void fused_peer_merge(const PeerMergeArgs pa, int grp, int bq, int hq, int seq, int tid,
                                              volatile int* abort_flag) {
  constexpr int D = 128;
  const PeerXchg& px = pa.px;
  const int par = seq & 1;
  const uint32_t want = (uint32_t)(seq + 1);
  const uint64_t* base = reinterpret_cast<const uint64_t*>(px.bases[px.rank]);
  const uint64_t t0 = globaltimer_ns();
  bool ok = true;
  // a word of this call (bounded wait); false if the limit passed
  auto get = [&](const uint64_t* p, float& v) {
    uint64_t w = xchg_get(p);
    while ((uint32_t)(w >> 32) != want) {
      if (globaltimer_ns() - t0 > g_wait_limit_ns) return false;
      __nanosleep(32);
      w = xchg_get(p);
    }
    v = __uint_as_float((uint32_t)w);
    return true;
  };
  for (int x = tid; x < pa.R * D && ok; x += kScoreThreads) {
    const int r = x / D, d = x - r * D;
    float M = -INFINITY, L = 0.f, O = 0.f;
    for (int src = 0; src < px.P && ok; ++src) {
      const uint64_t* blk = base + ((size_t)(par * px.P + src) * pa.NG + grp) * kXchgBlock;
      float m, l, o;
      ok = get(blk + r, m) && get(blk + 8 + r, l) && get(blk + 16 + r * D + d, o);
      if (!ok || m == -INFINITY) continue;
      const float mc = fmaxf(M, m);
      const float sa = exp2f(M - mc), sb = exp2f(m - mc);
      L = L * sa + l * sb;
      O = O * sa + o * sb;
      M = mc;
    }
    if (!ok) break;
    const int s = r / pa.G, gq = r - s * pa.G;
    const size_t orow = ((size_t)bq * pa.Sq + s) * pa.Hq + (size_t)hq * pa.G + gq;
    const float y = L > 0.f ? O / L : 0.f;
    if (pa.out_bf16) reinterpret_cast<__nv_bfloat16*>(pa.out)[orow * D + d] = __float2bfloat16_rn(y);
    else reinterpret_cast<float*>(pa.out)[orow * D + d] = y;
  }
  if (!ok) {
    *abort_flag = 1;
    atomicExch(&g_score_status, 1);
  }
  if (tid == 0) OC_SSTAMP(22, globaltimer_ns());
}

// Keep decision of tile `tile` of this CTA from write-time metadata
// (warp-collective, the result on every lane): the bound of the key path's
// epilogue (block mean = DC / sqrt(512), residual sqrt(|q|^2) sqrt(E_AC))
// and the two gates, with a.dc / a.e_ac / a.zeta the stored metadata.
template <int D>
__device__ __forceinline__ int meta_keep(const ScoreArgs& a, int tile, bool q_cached, const __nv_bfloat16* s_q,
                                         const float* s_qn, int lane) {
  const int rows = a.Sq * a.G;
  const __nv_bfloat16* qb = q_cached ? s_q : reinterpret_cast<const __nv_bfloat16*>(a.q);
  const int t = blockIdx.x + tile * gridDim.x;
  const int h = t % a.H;
  const int j = (t / a.H) % a.nb;
  const int b = t / (a.H * a.nb);
  const size_t cell = ((size_t)b * a.nb + j) * a.H + h;
  const float resid_scale = sqrtf(__ldg(a.e_ac + cell));
  const float z = __ldg(a.zeta + cell);
  const float* dcp = a.dc + cell * D;
  float dv[8], nv[8];
#pragma unroll
  for (int r = 0; r < 8; ++r) dv[r] = nv[r] = 0.f;
#pragma unroll
  for (int c = lane; c < D; c += 32) {
    const float mean = __ldg(dcp + c) / kNorm;
#pragma unroll
    for (int r = 0; r < 8; ++r)
      if (r < rows) {
        const int s = r / a.G, gq = r - s * a.G;
        const size_t qrow = ((size_t)b * a.Sq + s) * a.Hq + (size_t)h * a.G + gq;
        const float qv = __bfloat162float(qb[qrow * D + c]);
        dv[r] = fmaf(qv, mean, dv[r]);
        nv[r] = fmaf(qv, qv, nv[r]);  // squared norms on the same loads (uncached queries)
      }
  }
  const float dot = transpose_sum8(dv, lane);
  const float nrm_lanes = q_cached ? 0.f : transpose_sum8(nv, lane);
  const int r = lane >> 2;
  float bound = -INFINITY;
  if (r < rows) {
    const int s = r / a.G, gq = r - s * a.G;
    const size_t qrow = ((size_t)b * a.Sq + s) * a.Hq + (size_t)h * a.G + gq;
    float nrm = 0.f;
    nrm = q_cached ? s_qn[qrow] : nrm_lanes;
    const float sqrt_d = sqrtf((float)D);
    bound = dot / sqrt_d + (sqrtf(nrm) * resid_scale) / sqrt_d;
  }
  const float bmax = warp_max(bound);
  return (bmax >= a.tau && z <= a.zeta_max) ? 1 : 0;
}

// META (with FUSED): the block decisions come from write-time metadata
// instead of a pass over the keys, and ScoreArgs::dc / e_ac / zeta are those
// INPUTS (per cell (b, j, h): D DC coefficients, E_AC, zeta); the compute
// warps go straight to the attention phase.
template <int D, bool FUSED, bool META = false>
__global__ void __launch_bounds__(kFusedThreads, 1)
score_tma_kernel(const __grid_constant__ CUtensorMap kmap, const __grid_constant__ CUtensorMap amap_k,
                 const __grid_constant__ CUtensorMap amap_v, ScoreArgs a, int n_tiles, FusedArgs f) {
  constexpr int PARTS = D / kSlabC;
  constexpr int kW = kScoreThreads / 32;  // 16 warps
  constexpr int NE = kEpiWarps;           // epilogue warps
  constexpr int NBUF = NE;                // tile buffers, one per epilogue warp
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // 128-byte swizzled stages must start on a 1024-byte boundary.
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  __shared__ __align__(8) uint64_t full[kStages];
  __shared__ __align__(8) uint64_t empty[kStages];  // fused: stage free for the producer
  __shared__ int s_desc[kStages];            // fused: unit in a stage (block * 4 + chunk), -1 = end
  __shared__ int s_set;                      // fused: counter set of this call
  __shared__ int s_seq;                      // fused: calls before this one (the epoch)
  __shared__ __align__(8) uint64_t setbar;   // fused: s_set is known (after the previous kernel)
  __shared__ int s_merge;                    // fused: this CTA merges its group
  __shared__ int s_rel[kStages];             // warps done with a stage
  __shared__ __align__(8) uint64_t tfull[NBUF], tempty[NBUF];  // tile buffer hand-over
  __shared__ float s_grp[NBUF][kW][8];       // per-warp coefficient-group energies
  __shared__ float s_mu[NBUF][2][D];         // per-channel means of y0 over each half of the inner offsets
  __shared__ float s_dcw[NBUF][D];           // DC coefficients of the tile in buffer tb
  __shared__ float s_qn[kQCacheBytes / (2 * 64)];  // squared norms of the staged query rows
  __shared__ volatile int s_abort;
  constexpr int kMetaPre = 32 * NE;          // META: tiles whose decisions the compute warps make
  __shared__ int s_kpre[META ? kMetaPre : 1];
  __shared__ __align__(8) uint64_t kpbar;    // META: s_kpre is filled
#ifdef OC_TIMING
  __shared__ unsigned long long s_tarr[kStages];
  __shared__ unsigned long long s_trel;
  if (threadIdx.x == 0) s_trel = 0;
#endif

  const int tid = threadIdx.x;
  if (tid == 0) OC_SSTAMP(0, globaltimer_ns());
  const int lane = tid & 31, warp = tid >> 5;
  const int ch = warp & 7;    // channels 8ch .. 8ch+7 of a slab (one 16-byte chunk)
  const int hb = warp >> 3;   // inner offsets 32hb .. 32hb+31 (one box of the stage)
  const int g = lane >> 2, c4 = lane & 3;  // MMA fragment coordinates
  // A = diag(H8, H8) in bfloat16, H8[q][i] = (-1)^popcount(q & i):
  // a0 = a3 = (H8[g][2c4], H8[g][2c4 + 1]), a1 = a2 = 0.
  const uint32_t hA = ((__popc(g & (2 * c4)) & 1) ? 0xBF80u : 0x3F80u) |
                      (((__popc(g & (2 * c4 + 1)) & 1) ? 0xBF80u : 0x3F80u) << 16);
  const int my_tiles = n_tiles > (int)blockIdx.x ? (n_tiles - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
  const int n_units = META ? 0 : my_tiles * PARTS;  // key slabs this CTA streams for scoring
  // Queries staged in shared memory when they fit (decode), so the tile
  // epilogue never waits on global memory.
  const size_t q_elems = a.q ? (size_t)(n_tiles / (a.H * a.nb)) * a.Sq * a.Hq * D : 0;
  const bool q_cached = a.q && q_elems * 2 <= (size_t)kQCacheBytes;
  __nv_bfloat16* s_q = reinterpret_cast<__nv_bfloat16*>(smem + (size_t)kStages * kSlabB);

  auto issue = [&](int k) {
    const int t = blockIdx.x + (k / PARTS) * gridDim.x;
    const int part = k % PARTS;
    const int h = t % a.H;
    const int j = (t / a.H) % a.nb;
    const int b = t / (a.H * a.nb);
    uint8_t* dst = smem + (size_t)(k % kStages) * kSlabB;
    uint64_t* bar = &full[k % kStages];
    mbar_expect_tx(bar, kSlabB);
    const int col = h * D + part * kSlabC, blk = b * a.nb + j;
    tma_load_4d(dst, &kmap, bar, col, 0, 0, blk);                 // inner offsets 0..31
    tma_load_4d(dst + kSlabB / 2, &kmap, bar, col, 0, 32, blk);   // inner offsets 32..63
  };

  if (tid == 0) {
    for (int i = 0; i < kStages; ++i) { mbar_init(&full[i], 1); mbar_init(&empty[i], 1); s_rel[i] = 0; }
    for (int i = 0; i < NBUF; ++i) { mbar_init(&tfull[i], kW); mbar_init(&tempty[i], 1); }
    mbar_init(&setbar, 1);
    if constexpr (META) mbar_init(&kpbar, kW);
    fence_mbar_init();
    s_abort = 0;
    s_merge = 0;
    OC_SSTAMP(10, globaltimer_ns());
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&kmap)) : "memory");
    // The first slabs are requested before the previous kernel in the stream
    // has finished: a kernel only starts early behind one of this library's
    // scorer, compaction or attention kernels, and none of them writes keys.
    for (int k = 0; k < kStages && k < n_units; ++k) issue(k);
  }
  // Launched as a programmatic dependent: the kernel may start while the one
  // before it in the stream (one of this library's, which write no keys and
  // no queries) is still running.  Streaming and transforming the keys and
  // staging the queries only read inputs, so they start at once; the
  // epilogue warps wait for the previous kernel (pdl_wait) before the first
  // write of an output or of the workspace, the compute warps before the
  // attention phase.
  pdl_trigger();
  __syncthreads();  // barrier initialisation is visible; the only CTA-wide barrier
  if (tid == 0) OC_SSTAMP(1, globaltimer_ns());
  FusedSet fs = {};
#ifdef OC_TIMING
  unsigned long long t_wait = 0;
#endif

  // Warps kW .. kW+NE-1 run the tile epilogues (bound, zeta, keep) while the
  // 16 compute warps go on with the next tiles.  Epilogue warp e owns tile
  // buffer e and the tiles e, e + NE, ...; the buffer is handed over on
  // tfull[e] (16 arrivals) and handed back on tempty[e].
  if (warp >= kW) {
    const int e = warp - kW;
    const int qrows = q_cached ? (int)(q_elems / D) : 0;
    if (q_cached) {
      // Queries and their squared norms, staged once (only these warps read them).
      const uint4* src = reinterpret_cast<const uint4*>(a.q);
      uint4* dst = reinterpret_cast<uint4*>(s_q);
      for (size_t i = e * 32 + lane; i < q_elems / 8; i += NE * 32) dst[i] = src[i];
      asm volatile("bar.sync 1, %0;" ::"r"(NE * 32) : "memory");
      for (int r = e; r < qrows; r += NE) {
        float nrm = 0.f;
#pragma unroll
        for (int c = lane; c < D; c += 32) {
          const float qv = __bfloat162float(s_q[(size_t)r * D + c]);
          nrm = fmaf(qv, qv, nrm);
        }
        nrm = warp_sum(nrm);
        if (lane == 0) s_qn[r] = nrm;
      }
      asm volatile("bar.sync 1, %0;" ::"r"(NE * 32) : "memory");
    }
    // This warp's tiles are e, e + NE, ...; with META the decisions of the
    // first 32 (tiles < kMetaPre) are made by the compute warps before the
    // wait for the previous kernel (the metadata and the queries are
    // inputs), one warp per tile; lane i picks up tile e + i NE's.
    int meta_kp = 0;
    if constexpr (META) {
      const int n_mine_tiles = e < my_tiles ? (my_tiles - 1 - e) / NE + 1 : 0;
      if (!mbar_wait(&kpbar, 0)) {
        s_abort = 1;
        if (lane == 0) atomicExch(&g_score_status, 1);
      }
      if (lane < min(n_mine_tiles, 32)) meta_kp = s_kpre[e + lane * NE];
    }
    // Outputs and the workspace are written from here on.
    pdl_wait();
    if constexpr (FUSED) {
      if (e == 0 && lane == 0) {
        s_seq = __ldcg(f.epoch);
        s_set = s_seq & 1;
        OC_SSTAMP(8, globaltimer_ns());
      }
      asm volatile("bar.sync 1, %0;" ::"r"(NE * 32) : "memory");
      fs = fused_set(f, a.nb, s_set);
      if (blockIdx.x == 0) {
        // The other set was last used by the previous call, which has
        // completed: clear it for the next call.
        int* other = f.sets + (size_t)(s_set ^ 1) * f.set_ints;
        for (int i = e * 32 + lane; i < f.set_ints; i += NE * 32) other[i] = 0;
      }
      if (e == 0 && lane == 0) mbar_arrive(&setbar);  // the compute warps may read s_set
    }
    if constexpr (META) {
      // Decisions from write-time metadata, 32 tiles at a time: lane i
      // counts tile i's head in (the atomics of the 32 tiles in flight
      // together); the last head of a block publishes it as in the key path.
      const int n_mine_tiles = e < my_tiles ? (my_tiles - 1 - e) / NE + 1 : 0;
      for (int c0 = 0; c0 < n_mine_tiles; c0 += 32) {
        if (c0 > 0)
          for (int i = 0; i < min(n_mine_tiles - c0, 32); ++i) {
            const int kp = meta_keep<D>(a, e + (c0 + i) * NE, q_cached, s_q, s_qn, lane);
            if (lane == i) meta_kp = kp;
          }
        int row_done = 0, b = 0;
        if (c0 + lane < n_mine_tiles) {
          const int t = blockIdx.x + (e + (c0 + lane) * NE) * gridDim.x;
          const int h = t % a.H;
          const int j = (t / a.H) % a.nb;
          b = t / (a.H * a.nb);
          const int kp = meta_kp;
          if (a.keep) a.keep[((size_t)b * a.nb + j) * a.H + h] = (uint8_t)kp;
          const int bj = b * a.nb + j;
          const int old = atomicAdd(fs.blk_state + bj, 1 + (kp << 16));
          if ((old & 0xffff) == a.H - 1) {
            const bool kept = (old >> 16) + kp > 0;
            const int rw = atom_add_acq_rel(fs.row + b, kept ? 0x10001 : 1);
            if (kept) st_release(fs.queue + (size_t)b * a.nb + (rw >> 16), j + 1);
            row_done = (rw & 0xffff) == a.nb - 1;
          }
        }
        for (unsigned m = __ballot_sync(0xffffffffu, row_done); m; m &= m - 1) {
          const int bb = __shfl_sync(0xffffffffu, b, __ffs(m) - 1);
          fused_write_perm(fs.blk_state + (size_t)bb * a.nb, a.nb, f.perm + (size_t)bb * a.nb, f.count + bb, lane);
          __syncwarp();
          if (lane == 0) {
            __threadfence();
            if (atom_add_acq_rel(fs.decided_all, 1) == f.B - 1) atomicAdd(f.epoch, 1);
          }
        }
        __syncwarp();
      }
    } else
    for (int tile = e; tile < my_tiles; tile += NE) {
      const int tb = e;
      if (!__all_sync(0xffffffffu, mbar_wait(&tfull[tb], (tile / NE) & 1))) {
        s_abort = 1;
        if (lane == 0) atomicExch(&g_score_status, 1);
        if constexpr (FUSED) break;
        else return;
      }
      const int t = blockIdx.x + tile * gridDim.x;
      const int h = t % a.H;
      const int j = (t / a.H) % a.nb;
      const int b = t / (a.H * a.nb);
      // Group energies over the 16 warps (lanes 4q .. 4q+3 sum group q); group
      // 0 gets the exact between-half term: the sum over 64 offsets of
      // (y - mu)^2 = SS0 + SS1 + 16 (mu0 - mu1)^2.
      const int q8 = lane >> 2, wq = lane & 3;
      float gv = (s_grp[tb][wq][q8] + s_grp[tb][wq + 4][q8]) + (s_grp[tb][wq + 8][q8] + s_grp[tb][wq + 12][q8]);
      gv += __shfl_xor_sync(0xffffffffu, gv, 1);
      gv += __shfl_xor_sync(0xffffffffu, gv, 2);
      float between = 0.f, e_dc = 0.f;
#pragma unroll
      for (int c = lane; c < D; c += 32) {
        const float m0 = s_mu[tb][0][c], m1 = s_mu[tb][1][c];
        const float dm = m0 - m1;
        between = fmaf(16.0f * dm, dm, between);
        const float dcv = (32.0f * (m0 + m1)) / kNorm;  // WHT coefficient 0
        s_dcw[tb][c] = dcv;
        e_dc = fmaf(dcv, dcv, e_dc);
      }
      between = warp_sum(between);
      e_dc = warp_sum(e_dc);
      __syncwarp();
      float g[8];
#pragma unroll
      for (int q = 0; q < 8; ++q) g[q] = __shfl_sync(0xffffffffu, gv, 4 * q);
      g[0] += between;
#pragma unroll
      for (int q = 0; q < 8; ++q) g[q] *= 0.125f;  // (64 / 512) Parseval factor of the inner transform
      float e_ac = 0.f;
#pragma unroll
      for (int q = 0; q < 8; ++q) e_ac += g[q];
      const float e_lo = band_from_groups(a.bands.lo[0], a.bands.hi[0], g, e_dc);
      const float e_mi = band_from_groups(a.bands.lo[1], a.bands.hi[1], g, e_dc);
      const float e_hi = band_from_groups(a.bands.lo[2], a.bands.hi[2], g, e_dc);
      const size_t cell = ((size_t)b * a.nb + j) * a.H + h;
      const float* dcp = s_dcw[tb];
      if (a.dc)
        for (int c = lane; c < D; c += 32) a.dc[cell * D + c] = dcp[c];
      float bmax = -INFINITY;
      if (a.q) {
        // rows = Sq * G <= 8 on this path: all rows' dot products at once,
        // reduced so that lanes 4r .. 4r+3 hold row r.
        const int rows = a.Sq * a.G;
        const float sqrt_d = sqrtf((float)D);
        const float resid_scale = sqrtf(e_ac);
        const __nv_bfloat16* qb = q_cached ? s_q : reinterpret_cast<const __nv_bfloat16*>(a.q);
        float dv[8];
#pragma unroll
        for (int r = 0; r < 8; ++r) dv[r] = 0.f;
#pragma unroll
        for (int c = lane; c < D; c += 32) {
          const float mean = dcp[c] / kNorm;  // block mean = DC / sqrt(512)
#pragma unroll
          for (int r = 0; r < 8; ++r)
            if (r < rows) {
              const int s = r / a.G, gq = r - s * a.G;
              const size_t qrow = ((size_t)b * a.Sq + s) * a.Hq + (size_t)h * a.G + gq;
              dv[r] = fmaf(__bfloat162float(qb[qrow * D + c]), mean, dv[r]);
            }
        }
        const float dot = transpose_sum8(dv, lane);
        const int r = lane >> 2;
        float nrm = 0.f;
        size_t qrow = 0;
        if (r < rows) {
          const int s = r / a.G, gq = r - s * a.G;
          qrow = ((size_t)b * a.Sq + s) * a.Hq + (size_t)h * a.G + gq;
        }
        if (q_cached) {
          if (r < rows) nrm = s_qn[qrow];
        } else {
          for (int rr = 0; rr < rows; ++rr) {
            const int s = rr / a.G, gq = rr - s * a.G;
            const size_t qr = ((size_t)b * a.Sq + s) * a.Hq + (size_t)h * a.G + gq;
            float n2 = 0.f;
            for (int c = lane; c < D; c += 32) {
              const float qv = __bfloat162float(qb[qr * D + c]);
              n2 = fmaf(qv, qv, n2);
            }
            n2 = warp_sum(n2);
            if (rr == r) nrm = n2;
          }
        }
        float bound = -INFINITY;
        if (r < rows) {
          bound = dot / sqrt_d + (sqrtf(nrm) * resid_scale) / sqrt_d;
          if (a.bounds && (lane & 3) == 0) {
            const int s = r / a.G, gq = r - s * a.G;
            a.bounds[(((size_t)b * a.Sq + s) * a.nb + j) * a.Hq + (size_t)h * a.G + gq] = bound;
          }
        }
        bmax = warp_max(bound);
      }
      int row_done = 0;  // fused: this epilogue completed batch row b's decisions
      if (lane == 0) {
        const float z = e_hi / (e_lo + 1e-6f);
        if (a.e_low) a.e_low[cell] = e_lo;
        if (a.e_mid) a.e_mid[cell] = e_mi;
        if (a.e_high) a.e_high[cell] = e_hi;
        if (a.zeta) a.zeta[cell] = z;
        if (a.e_ac) a.e_ac[cell] = e_ac;
        if (a.q && a.bound_max) a.bound_max[cell] = bmax;
        const int kp = ((a.q ? bmax >= a.tau : true) && z <= a.zeta_max) ? 1 : 0;
        if (a.keep) a.keep[cell] = (uint8_t)kp;
        if constexpr (FUSED) {
          // Count this head in; the last head of the block decides it.
          const int bj = b * a.nb + j;
          const int old = atomicAdd(fs.blk_state + bj, 1 + (kp << 16));
          if ((old & 0xffff) == a.H - 1) {
            // One word per batch row counts decided and kept blocks; a kept
            // block's queue slot is the kept count before it.
            const bool kept = (old >> 16) + kp > 0;
            const int rw = atom_add_acq_rel(fs.row + b, kept ? 0x10001 : 1);
            if (kept) st_release(fs.queue + (size_t)b * a.nb + (rw >> 16), j + 1);
            row_done = (rw & 0xffff) == a.nb - 1;
          }
        }
      }
      if constexpr (FUSED) {
        // The last decision of batch row b: its permutation and count, and,
        // for the grid's last row, the epoch step that hands the next call
        // the other counter set (every CTA has read the epoch by now: each
        // one scored a tile before any row could be complete).
        if (__shfl_sync(0xffffffffu, row_done, 0)) {
          fused_write_perm(fs.blk_state + (size_t)b * a.nb, a.nb, f.perm + (size_t)b * a.nb, f.count + b, lane);
          __syncwarp();
          if (lane == 0) {
            __threadfence();
            if (atom_add_acq_rel(fs.decided_all, 1) == f.B - 1) atomicAdd(f.epoch, 1);
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[tb]);
    }
    if (lane == 0 && e == 0) OC_SSTAMP(4, globaltimer_ns());
    if constexpr (FUSED) {
      // The epilogue warp whose last tile comes earliest (tile my_tiles - NE)
      // becomes the producer of the attention units: lane 0 feeds the stage
      // ring once the scorer has released each stage for the last time.
      if (e == my_tiles % NE) {
        if (lane == 0) {
          const int grp = blockIdx.x % f.NG, b = grp / a.H, h = grp % a.H;
          const int* qb = fs.queue + (size_t)b * a.nb;
          // Per stage (bit s): used = a unit was put in the stage and its
          // release is still to be awaited; phase = parity of that release
          // on empty[s].
          uint32_t used = (1u << (n_units < kStages ? n_units : kStages)) - 1u, phase = 0;
          constexpr int CPB = kBlock / kFusedChunk;  // units per block
          // Units are claimed one ahead: the claim's round trip and the first
          // look at its queue slot overlap the wait for a free stage.  The
          // queue entry is all that is needed from its publisher (keys and
          // values are inputs), so relaxed loads poll it; the end-of-queue
          // test acquires the row word.
          // Units are claimed in pairs (one atomic and one queue look per two
          // 128-token chunks of the same block: kUnitClaim divides CPB).
          constexpr int kUnitClaim = 2;
          static_assert(CPB % kUnitClaim == 0, "a claim stays within one block");
          int w = atomicAdd(fs.grp_ctr + grp, kUnitClaim);
          int w_end = w + kUnitClaim;
          int vq = w / CPB < a.nb ? ld_relaxed(qb + w / CPB) : 0;
          OC_SSTAMP(9, 0);
          for (int k = n_units;; ++k) {
            const int s = k % kStages;
            if (used >> s & 1u) {
              if (!mbar_wait(&empty[s], phase >> s & 1u)) { s_abort = 1; atomicExch(&g_score_status, 1); }
              phase ^= 1u << s;
            }
            used |= 1u << s;
            int desc = -1;
            const uint64_t t0 = globaltimer_ns();
            if (!s_abort) {
              const int slot = w / CPB;
              int v = vq;
              for (int it = 0; slot < a.nb; ++it) {
                if (v > 0) { desc = (v - 1) * CPB + w % CPB; break; }
                if ((it & 3) == 3) {
                  const int rw = ld_acquire(fs.row + b);
                  if ((rw & 0xffff) == a.nb && slot >= (rw >> 16)) break;  // past the last kept block
                }
                if (globaltimer_ns() - t0 > g_wait_limit_ns) { s_abort = 1; atomicExch(&g_score_status, 1); break; }
                __nanosleep(32);
                v = ld_relaxed(qb + slot);
              }
            }
#ifdef OC_TIMING
            g_sstamp[blockIdx.x][9] += globaltimer_ns() - t0;
#endif
            s_desc[s] = desc;
            if (k == n_units) OC_SSTAMP(15, globaltimer_ns());
            if (desc < 0) {
              mbar_arrive(&full[s]);  // end of the run: the consumers stop at this unit
              break;
            }
            const int j = desc / CPB, cc = desc % CPB;
            uint8_t* dst = smem + (size_t)s * kSlabB;
            const int y = b * a.S + j * kBlock + cc * kFusedChunk;
            mbar_expect_tx(&full[s], kSlabB);
#pragma unroll
            for (int jb = 0; jb < D / 64; ++jb) {
              tma_load_2d(dst + jb * (kFusedChunk * 128), &amap_k, &full[s], h * D + jb * 64, y);
              tma_load_2d(dst + kSlabB / 2 + jb * (kFusedChunk * 128), &amap_v, &full[s], h * D + jb * 64, y);
            }
            if (++w == w_end) {
              w = atomicAdd(fs.grp_ctr + grp, kUnitClaim);
              w_end = w + kUnitClaim;
              vq = w / CPB < a.nb ? ld_relaxed(qb + w / CPB) : 0;
            } else {
              vq = desc / CPB + 1;  // the same block: its queue entry is known
            }
          }
        }
      }
    }
    return;
  }

  // Stage layout (4-D box: 64 channels x 8 i_hi x 32 i_lo, per half of the
  // inner offsets): row = (i_lo % 32) * 8 + i_hi, 128 bytes, 16-byte chunk ch
  // at chunk ch ^ i_hi (128-byte swizzle, row % 8 == i_hi).  The 8 rows of one
  // 8x8 matrix (i_hi = 0..7 at one i_lo) are consecutive rows in distinct
  // bank groups.  Lane (matrix lane / 8, row lane % 8) addresses:
  const uint32_t lane_off = (uint32_t)hb * (kSlabB / 2) + (uint32_t)((lane >> 3) * 8 + (lane & 7)) * 128 +
                            (uint32_t)((ch ^ (lane & 7)) << 4);
  if constexpr (META) {
    // Keep decisions of this CTA's tiles < kMetaPre, one warp per tile (the
    // compute warps are otherwise idle until the attention phase), handed to
    // the epilogue warps through s_kpre; the queries are read from global
    // memory (their shared-memory copy is being staged meanwhile).
    for (int t = warp; t < min(my_tiles, kMetaPre); t += kW) {
      const int kp = meta_keep<D>(a, t, false, nullptr, nullptr, lane);
      if (lane == 0) s_kpre[t] = kp;
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&kpbar);
  }
  for (int tile = 0; tile < (META ? 0 : my_tiles); ++tile) {
    const int tb = tile % NBUF;
    if (tile >= NBUF && !__all_sync(0xffffffffu, mbar_wait(&tempty[tb], (tile / NBUF - 1) & 1))) {
      s_abort = 1;
      if (lane == 0) atomicExch(&g_score_status, 1);
      if constexpr (FUSED) goto scored;
      else return;
    }
    float gacc = 0.f;  // this lane's share of the energy of coefficient group g
    for (int part = 0; part < PARTS; ++part) {
      const int k = tile * PARTS + part;
      const int stage = k % kStages;
      // A copy that never completes sets the abort flag: every warp stops
      // waiting and leaves (the fused kernel goes on to its end barriers).
      if (__any_sync(0xffffffffu, s_abort)) {
        if constexpr (FUSED) goto scored;
        else return;
      }
#ifdef OC_TIMING
      const unsigned long long tw0 = globaltimer_ns();
#endif
      if (!__all_sync(0xffffffffu, mbar_wait(&full[stage], (k / kStages) & 1))) {
        s_abort = 1;
        if (lane == 0) atomicExch(&g_score_status, 1);
        if constexpr (FUSED) goto scored;
        else return;
      }
#ifdef OC_TIMING
      const unsigned long long tw1 = globaltimer_ns();
      t_wait += tw1 - tw0;
      if (warp == 0 && lane == 0) { s_tarr[stage] = tw1; if (k == 0) OC_SSTAMP(2, tw1); }
#endif
      // 32 transposed 8x8 matrices: B operands (k = i_hi, n = channel) of
      // the inner offsets 32hb + 4s + m, m = 0..3.
      const uint32_t sbase = smem_u32(smem + (size_t)stage * kSlabB) + lane_off;
      uint32_t bm[8][4];
#pragma unroll
      for (int s = 0; s < 8; ++s) ldsm_x4_trans(bm[s], sbase + s * 4096);
      // This warp is done with the stage; the last of the 16 warps refills it.
      __threadfence_block();
      __syncwarp();
      if (lane == 0) {
        if (atomicAdd(&s_rel[stage], 1) == kW - 1) {
          s_rel[stage] = 0;
          if (k + kStages < n_units) {
            if (!s_abort) {
              fence_proxy_async();
              issue(k + kStages);
#ifdef OC_TIMING
              s_trel += globaltimer_ns() - s_tarr[stage];
#endif
            }
          } else if constexpr (FUSED) {
            // Last scoring use of this stage: hand it to the producer.
            fence_proxy_async();
            mbar_arrive(&empty[stage]);
          }
        }
      }
      // z = H8 x over i_hi for two inner offsets per MMA: rows 0-7 of D are
      // groups q = 0..7 at the first offset, rows 8-15 at the second.  Lane
      // (g, c4) receives group g at channels 2c4, 2c4 + 1 of its chunk.
      // Row g = 0 is y0, whose per-channel mean is needed: it is accumulated
      // relative to a pivot (its first value) as sum and sum of squares, so
      // the centred sum loses nothing to cancellation.
      float d[4];
      mma_h8(d, hA, bm[0][0], bm[0][1], 0.f, 0.f);
      const float p0 = g == 0 ? d[0] : 0.f, p1 = g == 0 ? d[1] : 0.f;
      const f32x2 piv = pack2(p0, p1);
      f32x2 s1 = sub2(pack2(d[2], d[3]), piv);
      f32x2 s2 = fma2(s1, s1, pack2(0.f, 0.f));
      {
        f32x2 da = sub2(pack2(d[0], d[1]), piv);  // zero on row 0; z on the others
        s2 = fma2(da, da, s2);
      }
#pragma unroll
      for (int s = 0; s < 8; ++s) {
#pragma unroll
        for (int m = 0; m < 2; ++m) {
          if (s == 0 && m == 0) continue;
          mma_h8(d, hA, bm[s][2 * m], bm[s][2 * m + 1], -p0, -p1);  // D = z - pivot
          const f32x2 da = pack2(d[0], d[1]), db = pack2(d[2], d[3]);
          s1 = add2(s1, add2(da, db));
          s2 = fma2(da, da, s2);
          s2 = fma2(db, db, s2);
        }
      }
      float s1a, s1b, s2a, s2b;
      unpack2(s1, s1a, s1b);
      unpack2(s2, s2a, s2b);
      if (g == 0) {
        // 32 offsets: mean = pivot + S1 / 32, centred squares = S2 - S1^2 / 32
        s_mu[tb][hb][part * kSlabC + ch * 8 + 2 * c4] = p0 + s1a * (1.0f / 32.0f);
        s_mu[tb][hb][part * kSlabC + ch * 8 + 2 * c4 + 1] = p1 + s1b * (1.0f / 32.0f);
        gacc += fmaf(-s1a * (1.0f / 32.0f), s1a, s2a) + fmaf(-s1b * (1.0f / 32.0f), s1b, s2b);
      } else {
        gacc += s2a + s2b;
      }
    }
    gacc += __shfl_xor_sync(0xffffffffu, gacc, 1);
    gacc += __shfl_xor_sync(0xffffffffu, gacc, 2);
    if (c4 == 0) s_grp[tb][warp][g] = gacc;
    // Publish this warp's share of the tile to the epilogue warp.
    __threadfence_block();
    __syncwarp();
    if (lane == 0) mbar_arrive(&tfull[tb]);
  }
#ifdef OC_TIMING
  if (warp == 0 && lane == 0) {
    OC_SSTAMP(3, globaltimer_ns());
    OC_SSTAMP(5, t_wait);
    OC_SSTAMP(6, s_trel);
    OC_SSTAMP(7, n_units);
  }
#endif
scored:
  if constexpr (FUSED) {
    static_assert(!FUSED || D == 128, "the fused decode layer is built for head_dim 128");
    // The attention phase writes partials into the workspace: after the
    // previous kernel, with this call's counter set.
    if (!__all_sync(0xffffffffu, mbar_wait(&setbar, 0))) {
      s_abort = 1;
      if (lane == 0) atomicExch(&g_score_status, 1);
    }
    pdl_wait();
    fs = fused_set(f, a.nb, s_set);
    // ---- attention over the retained blocks of group (bq, hq) ----
    const int grp = blockIdx.x % f.NG, bq = grp / a.H, hq = grp % a.H;
    const int tg = warp & 7;    // tokens 16 tg .. 16 tg + 15 of each unit
    const int chh = warp >> 3;  // value channels 64 chh .. 64 chh + 63
    // A fragments of Q: row g of the tile is query row g of KV head hq
    // (adaptive_attention.py:60-70 with GQA rows s * G + gq); rows 8..15 and
    // rows >= R are zero.
    uint32_t qa[D / 16][2];
    {
      const uint32_t* qrow = nullptr;
      if (g < f.R) {
        const int s = g / a.G, gq = g - s * a.G;
        qrow = reinterpret_cast<const uint32_t*>(reinterpret_cast<const __nv_bfloat16*>(a.q) +
                                                 (((size_t)bq * a.Sq + s) * a.Hq + (size_t)hq * a.G + gq) * D);
      }
#pragma unroll
      for (int ks = 0; ks < D / 16; ++ks) {
        qa[ks][0] = qrow ? qrow[8 * ks + c4] : 0u;      // channels 16 ks + 2 c4, +1
        qa[ks][1] = qrow ? qrow[8 * ks + 4 + c4] : 0u;  // channels 16 ks + 8 + 2 c4, +1
      }
    }
    // Online softmax (log2 units) of this warp's tokens, row g:
    // running max, this lane's share of the sum, output channels
    // 64 chh + 8 nt + 2 c4, +1.
    if (tid == 0) { OC_SSTAMP(11, globaltimer_ns()); OC_SSTAMP(18, 0); OC_SSTAMP(19, 0); }
    float m_run = -INFINITY, l_run = 0.f;
    float o[8][2];
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) o[nt][0] = o[nt][1] = 0.f;
    const int mm = lane >> 3, rr = lane & 7;
    for (int k = n_units;; ++k) {
      const int stage = k % kStages;
      if (__any_sync(0xffffffffu, s_abort)) break;
#ifdef OC_TIMING
      const unsigned long long tw0a = globaltimer_ns();
#endif
      if (!__all_sync(0xffffffffu, mbar_wait(&full[stage], (k / kStages) & 1))) {
        s_abort = 1;
        if (lane == 0) atomicExch(&g_score_status, 1);
        break;
      }
#ifdef OC_TIMING
      if (tid == 0) { g_sstamp[blockIdx.x][19] += globaltimer_ns() - tw0a; g_sstamp[blockIdx.x][18] += 1; }
#endif
      if (s_desc[stage] < 0) break;
      if (tid == 0 && k == n_units) OC_SSTAMP(12, globaltimer_ns());
      const uint32_t kbase = smem_u32(smem + (size_t)stage * kSlabB), vbase = kbase + kSlabB / 2;
      // S = Q K^T for tokens 16 tg + (0..7 | 8..15)
      float sa[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
      for (int ks = 0; ks < D / 16; ++ks) {
        uint32_t kb[4];
        ldsm_x4(kb, kbase + swz<kFusedChunk>(16 * tg + 8 * (mm >> 1) + rr, 2 * ks + (mm & 1)));
        const uint32_t af[4] = {qa[ks][0], 0u, qa[ks][1], 0u};
        mma_bf16_16816(sa[0], af, kb[0], kb[1]);
        mma_bf16_16816(sa[1], af, kb[2], kb[3]);
      }
      // V fragments of the warp's 16 tokens and 64 channels, then release.
      uint32_t vb[4][4];
#pragma unroll
      for (int np = 0; np < 4; ++np)
        ldsm_x4_t(vb[np], vbase + swz<kFusedChunk>(16 * tg + 8 * (mm & 1) + rr, 2 * (4 * chh + np) + (mm >> 1)));
      __threadfence_block();
      __syncwarp();
      if (lane == 0 && atomicAdd(&s_rel[stage], 1) == kW - 1) {
        s_rel[stage] = 0;
        fence_proxy_async();
        mbar_arrive(&empty[stage]);
      }
      const float x0 = sa[0][0] * f.scale_log2, x1 = sa[0][1] * f.scale_log2;
      const float x2 = sa[1][0] * f.scale_log2, x3 = sa[1][1] * f.scale_log2;
      float mx = fmaxf(fmaxf(x0, x1), fmaxf(x2, x3));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
      const float mn = fmaxf(m_run, mx);
      const float alpha = exp2f(m_run - mn);
      const float p0 = exp2f(x0 - mn), p1 = exp2f(x1 - mn), p2 = exp2f(x2 - mn), p3 = exp2f(x3 - mn);
      l_run = fmaf(l_run, alpha, (p0 + p1) + (p2 + p3));
      m_run = mn;
      const uint32_t pa[4] = {pack_bf16x2(p0, p1), 0u, pack_bf16x2(p2, p3), 0u};
#pragma unroll
      for (int np = 0; np < 4; ++np)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          float d[4] = {o[2 * np + e][0] * alpha, o[2 * np + e][1] * alpha, 0.f, 0.f};
          mma_bf16_16816(d, pa, vb[np][2 * e], vb[np][2 * e + 1]);
          o[2 * np + e][0] = d[0];
          o[2 * np + e][1] = d[1];
        }
    }
    if (tid == 0) OC_SSTAMP(13, globaltimer_ns());
    float l = l_run + __shfl_xor_sync(0xffffffffu, l_run, 1);
    l += __shfl_xor_sync(0xffffffffu, l, 2);
    // Combine the 16 warp states into the CTA's partial (the ring is idle:
    // every issued unit has been consumed and nothing more is issued).
    asm volatile("bar.sync 2, %0;" ::"r"(kScoreThreads) : "memory");
    float* cm = reinterpret_cast<float*>(smem);  // [kW][8] max
    float* cl = cm + kW * 8;                     // [kW][8] sum
    float* co = cl + kW * 8;                     // [kW][8][64] output
    if (c4 == 0) { cm[warp * 8 + g] = m_run; cl[warp * 8 + g] = l; }
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      co[(warp * 8 + g) * 64 + 8 * nt + 2 * c4] = o[nt][0];
      co[(warp * 8 + g) * 64 + 8 * nt + 2 * c4 + 1] = o[nt][1];
    }
    asm volatile("bar.sync 2, %0;" ::"r"(kScoreThreads) : "memory");
    const size_t pbase = (size_t)grp * f.cpg + blockIdx.x / f.NG;
    for (int x = tid; x < f.R * D; x += kScoreThreads) {
      const int r = x / D, d = x - r * D, hh = d >> 6, dl = d & 63;
      float M = -INFINITY;
#pragma unroll
      for (int t = 0; t < 8; ++t) M = fmaxf(M, cm[(hh * 8 + t) * 8 + r]);
      float L = 0.f, O = 0.f;
      if (M != -INFINITY)
#pragma unroll
        for (int t = 0; t < 8; ++t) {
          const int w = hh * 8 + t;
          const float wt = exp2f(cm[w * 8 + r] - M);
          L = fmaf(cl[w * 8 + r], wt, L);
          O = fmaf(co[(w * 8 + r) * 64 + dl], wt, O);
        }
      f.part_o[(pbase * kFusedMaxRows + r) * D + d] = O;
      if (d == 0) { f.part_m[pbase * kFusedMaxRows + r] = M; f.part_l[pbase * kFusedMaxRows + r] = L; }
    }
    asm volatile("bar.sync 2, %0;" ::"r"(kScoreThreads) : "memory");
    const int n_grp = ((int)gridDim.x - 1 - grp) / f.NG + 1;  // CTAs serving this group
    if (tid == 0) {
      // Release: the CTA's partial (ordered before by the barrier) is
      // visible to whichever CTA sees the last count.
      s_merge = atom_add_acq_rel(fs.grp_done + grp, 1) == n_grp - 1;
      OC_SSTAMP(16, s_merge);
      OC_SSTAMP(17, globaltimer_ns());
    }
    asm volatile("bar.sync 2, %0;" ::"r"(kScoreThreads) : "memory");
    if (s_merge) {
      // Last CTA of the group: log-sum-exp merge of its n_grp partials, o / l
      // (adaptive_attention.py:72-76; zeros when no block is retained,
      // indirect_attention.py:150-151).  kMergeRound partials per round,
      // their loads issued together.
      const size_t g0 = (size_t)grp * f.cpg;
      for (int x = tid; x < f.R * D; x += kScoreThreads) {
        const int r = x / D, d = x - r * D;
        float M = -INFINITY, L = 0.f, O = 0.f;
        for (int i0 = 0; i0 < n_grp; i0 += kMergeRound) {
          float mv[kMergeRound], lv[kMergeRound], ov[kMergeRound];
#pragma unroll
          for (int u = 0; u < kMergeRound; ++u) {
            const size_t pr = (g0 + i0 + u) * kFusedMaxRows + r;
            const bool in = i0 + u < n_grp;
            mv[u] = in ? __ldcg(f.part_m + pr) : -INFINITY;
            lv[u] = in ? __ldcg(f.part_l + pr) : 0.f;
            ov[u] = in ? __ldcg(f.part_o + pr * D + d) : 0.f;
          }
          float mc = M;
#pragma unroll
          for (int u = 0; u < kMergeRound; ++u) mc = fmaxf(mc, mv[u]);
          if (mc != -INFINITY) {
            const float sc = exp2f(M - mc);
            L *= sc;
            O *= sc;
#pragma unroll
            for (int u = 0; u < kMergeRound; ++u) {
              const float w = exp2f(mv[u] - mc);
              L = fmaf(lv[u], w, L);
              O = fmaf(ov[u], w, O);
            }
            M = mc;
          }
        }
        const int s = r / a.G, gq = r - s * a.G;
        const size_t orow = ((size_t)bq * a.Sq + s) * a.Hq + (size_t)hq * a.G + gq;
        if (f.px.P > 0) {
          // This shard's partial of group grp into slot [parity][rank][grp]
          // of every rank's exchange region (plain stores over NVLink).
          // Each word carries its float and the call number + 1, so no
          // fence or flag is needed: the reader waits for each word.
          const size_t slot = ((size_t)(s_seq & 1) * f.px.P + f.px.rank) * f.NG + grp;
          const uint64_t tag = (uint64_t)(uint32_t)(s_seq + 1) << 32;
          for (int p = 0; p < f.px.P; ++p) {
            uint64_t* blk = reinterpret_cast<uint64_t*>(f.px.bases[p]) + slot * kXchgBlock;
            xchg_put(blk + 16 + r * D + d, tag | __float_as_uint(O));
            if (d == 0) {
              xchg_put(blk + r, tag | __float_as_uint(M));
              xchg_put(blk + 8 + r, tag | __float_as_uint(L));
            }
          }
        } else if (f.pm) {
          // Unnormalised partial of this shard for a cross-shard merge.
          f.po[orow * D + d] = O;
          if (d == 0) { f.pm[orow] = M; f.pl[orow] = L; }
        } else {
          const float y = L > 0.f ? O / L : 0.f;
          if (f.out_bf16) reinterpret_cast<__nv_bfloat16*>(f.out)[orow * D + d] = __float2bfloat16_rn(y);
          else reinterpret_cast<float*>(f.out)[orow * D + d] = y;
        }
      }
    }
    if (f.px.P > 0 && s_merge) {
      PeerMergeArgs pa;
      pa.px = f.px;
      pa.NG = f.NG; pa.R = f.R; pa.G = a.G; pa.Sq = a.Sq; pa.Hq = a.Hq;
      pa.out = f.out; pa.out_bf16 = f.out_bf16;
      if (tid == 0) OC_SSTAMP(20, globaltimer_ns());
      fused_peer_merge(pa, grp, bq, hq, s_seq, tid, &s_abort);
      if (tid == 0) OC_SSTAMP(21, globaltimer_ns());
    }
    if (tid == 0) OC_SSTAMP(14, globaltimer_ns());
  }
}

// ---------------------------------------------------------------------------
// Full 9-stage butterfly on a shared-memory slab of 512 x 32 float32,
// stage order h = 1, 2, ..., 256 and "a + b" to the lower / "a - b" to the
// upper row exactly as fwht.py:25-58 (bit-identical float32 results).
// ---------------------------------------------------------------------------
constexpr int kSlab = 32;

__device__ __forceinline__ void slab_fwht(float (*s)[kSlab]) {
  const int c = threadIdx.x & 31;
  const int p0 = threadIdx.x >> 5;  // 8 pair rows per pass
#pragma unroll 1
  for (int hs = 1; hs < kBlock; hs <<= 1) {
    __syncthreads();
#pragma unroll 8
    for (int p = p0; p < kBlock / 2; p += kThreads / 32) {
      const int lo = (p / hs) * (2 * hs) + (p % hs);
      const int hi = lo + hs;
      const float x = s[lo][c], y = s[hi][c];
      s[lo][c] = x + y;
      s[hi][c] = x - y;
    }
  }
  __syncthreads();
}

template <typename T>
__device__ __forceinline__ void load_slab(float (*s)[kSlab], const T* src, size_t row_stride,
                                          int ncols_valid) {
  for (int i = threadIdx.x; i < kBlock * kSlab; i += kThreads) {
    const int r = i / kSlab, c = i % kSlab;
    s[r][c] = c < ncols_valid ? to_f32<T>(src[(size_t)r * row_stride + c]) : 0.f;
  }
}

template <typename T>
__global__ void __launch_bounds__(kThreads)
score_full_kernel(ScoreArgs a) {
  extern __shared__ float dyn[];
  float (*s)[kSlab] = reinterpret_cast<float (*)[kSlab]>(dyn);
  float* s_dc = dyn + kBlock * kSlab;           // [D]
  __shared__ float s_acc[kThreads / 32][4];
  __shared__ float s_band[4];
  __shared__ float s_red[kThreads / 32];

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int D = a.D;
  const int h = blockIdx.x % a.H;
  const int j = (blockIdx.x / a.H) % a.nb;
  const int b = blockIdx.x / (a.H * a.nb);
  const T* base = reinterpret_cast<const T*>(a.keys) +
                  (((size_t)b * a.S + (size_t)j * kBlock) * a.H + h) * D;
  const size_t tok_stride = (size_t)a.H * D;

  float acc[4] = {0.f, 0.f, 0.f, 0.f};  // low, mid, high, AC
  for (int c0 = 0; c0 < D; c0 += kSlab) {
    __syncthreads();
    load_slab<T>(s, base + c0, tok_stride, min(kSlab, D - c0));
    slab_fwht(s);
    for (int i = tid; i < kBlock * kSlab; i += kThreads) {
      const int k = i / kSlab, c = i % kSlab;
      if (c0 + c >= D) continue;
      const float coef = s[k][c] / kNorm;
      if (k == 0) { s_dc[c0 + c] = coef; }
      const float e = coef * coef;
      if (k >= 1) acc[3] += e;
#pragma unroll
      for (int bnd = 0; bnd < 3; ++bnd)
        if (k >= a.bands.lo[bnd] && k < a.bands.hi[bnd]) acc[bnd] += e;
    }
  }
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const float v = warp_sum(acc[q]);
    if (lane == 0) s_acc[warp][q] = v;
  }
  __syncthreads();
  if (tid < 4) {
    float v = 0.f;
    for (int w = 0; w < kThreads / 32; ++w) v += s_acc[w][tid];
    s_band[tid] = v;
  }
  __syncthreads();
  score_epilogue<T>(a, b, j, h, s_dc, s_band, s_red);
}

// Stand-alone fwht_512 over (512, N): one CTA per 32-column slab.
template <typename T>
__global__ void __launch_bounds__(kThreads)
fwht512_kernel(const T* x, float* y, int64_t n) {
  extern __shared__ float dyn[];
  float (*s)[kSlab] = reinterpret_cast<float (*)[kSlab]>(dyn);
  const int64_t c0 = (int64_t)blockIdx.x * kSlab;
  const int valid = (int)((n - c0) < kSlab ? (n - c0) : kSlab);
  load_slab<T>(s, x + c0, (size_t)n, valid);
  slab_fwht(s);
  for (int i = threadIdx.x; i < kBlock * kSlab; i += kThreads) {
    const int r = i / kSlab, c = i % kSlab;
    if (c < valid) y[(size_t)r * n + c0 + c] = s[r][c] / kNorm;
  }
}

constexpr size_t kSlabBytes = (size_t)kBlock * kSlab * sizeof(float);

bool bands_partial_ok(const Bands& bd) {
  for (int i = 0; i < 3; ++i) {
    const int e[2] = {bd.lo[i], bd.hi[i]};
    for (int q = 0; q < 2; ++q)
      if (!(e[q] == 0 || e[q] == 1 || e[q] % 64 == 0)) return false;
  }
  return true;
}

// Keys viewed as (channel, i_hi, i_lo, block) with token = 512 block +
// 64 i_hi + i_lo, so that a box lands in shared memory i_hi fastest.
int encode_score_map(CUtensorMap* map, const void* keys, int H, int D, int64_t blocks) {
  const uint64_t cols = (uint64_t)H * D, row_b = cols * 2;
  const uint64_t dims[4] = {cols, 8, 64, (uint64_t)blocks};
  const uint64_t strides[3] = {64 * row_b, row_b, (uint64_t)kBlock * row_b};
  const uint32_t box[4] = {(uint32_t)kSlabC, 8, 32, 1};
  return encode_map_4d(map, keys, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, dims, strides, box, true);
}

template <int D>
int launch_tma(const ScoreArgs& a, int ntiles, cudaStream_t st) {
  CUtensorMap map;
  const uint64_t key[4] = {1, (uint64_t)a.keys, (uint64_t)a.H | ((uint64_t)D << 32), (uint64_t)(ntiles / a.H) * kBlock};
  int rc = 0;
  if (!map_cache_get(key, &map) && !(rc = encode_score_map(&map, a.keys, a.H, D, ntiles / a.H)))
    map_cache_put(key, map);
  if (rc) return set_error(OC_ERR_CUDA, "oc_score_blocks: tensor map encode failed (%d)", rc);
  const int smem = kStages * kSlabB + kQCacheBytes + 1024;
  static std::atomic<uint64_t> s_setup{0};
  if (first_on_device(s_setup))
    cudaFuncSetAttribute(score_tma_kernel<D, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  const int grid = ntiles < device_sm_count() ? ntiles : device_sm_count();
  const FusedArgs none = {};
  const cudaError_t e = launch_pdl(score_tma_kernel<D, false>, dim3(grid), dim3(kScoreThreads + kEpiWarps * 32),
                                   smem, st, map, map, map, a, ntiles, none);
  if (e != cudaSuccess) return set_error(OC_ERR_CUDA, "score_tma_kernel: %s", cudaGetErrorString(e));
  return check_launch("score_tma_kernel");
}

// Workspace of the fused decode layer: the epoch and two counter sets
// (zero before the first call), then the per-CTA partials.
struct FusedLayout {
  size_t counters, bytes;
  int NG, cpg, set_ints;
};
FusedLayout fused_layout(int B, int nb, int Hkv) {
  FusedLayout L;
  L.NG = B * Hkv;
  L.cpg = (kFusedMaxGrid + L.NG - 1) / L.NG;
  L.set_ints = fused_set_ints(B, nb, L.NG);
  const size_t ints = 1 + 2 * (size_t)L.set_ints;
  L.counters = (ints * 4 + 255) / 256 * 256;
  const size_t parts = (size_t)L.NG * L.cpg * kFusedMaxRows;
  L.bytes = L.counters + ((parts * 2 + parts * 128) * 4 + 255) / 256 * 256;
  return L;
}

template <typename T>
int launch_score(const ScoreArgs& a, int mode, int ncta, cudaStream_t st) {
  if constexpr (Elem<T>::kCode == OC_BF16) {
    // The pipelined scorer evaluates the bound in one warp per tile; with
    // many query rows (chunked prefill) the 8-warp kernel below is used.
    if (mode == 1 && (!a.q || a.Sq * a.G <= 8)) {
      switch (a.D) {
        case 64: return launch_tma<64>(a, ncta, st);
        case 128: return launch_tma<128>(a, ncta, st);
        case 256: return launch_tma<256>(a, ncta, st);
      }
    }
  }
  if (mode == 1 || mode == 3) {
    switch (a.D) {
      case 64: score_partial_kernel<T, 64><<<ncta, kThreads, 0, st>>>(a); break;
      case 128: score_partial_kernel<T, 128><<<ncta, kThreads, 0, st>>>(a); break;
      case 256: score_partial_kernel<T, 256><<<ncta, kThreads, 0, st>>>(a); break;
      default: return set_error(OC_ERR_SHAPE, "head_dim %d not in {64,128,256}", a.D);
    }
    return check_launch("score_partial_kernel");
  }
  const size_t smem = kSlabBytes + (size_t)a.D * sizeof(float);
  // Per call: the attribute is per device, and one process may drive several.
  cudaFuncSetAttribute(score_full_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  score_full_kernel<T><<<ncta, kThreads, smem, st>>>(a);
  return check_launch("score_full_kernel");
}

// Host side of the fused decode layer, one instantiation per kernel form
// (the key-scoring one here, the metadata one in oc_score_meta.cu, so that
// neither form's code generation depends on the other's).
template <bool META>
int decode_fused_impl(const void* q, const void* k, const void* v, int batch, int q_len, int q_heads, int kv_heads,
                 int head_dim, int seq_len, float tau, float zeta_max, uint8_t* keep, int32_t* perm, int32_t* count,
                 void* out, int out_dtype, float* pm, float* pl, float* po, void* ws, size_t ws_bytes,
                 cudaStream_t st, const PeerXchg* px, const float* meta_dc, const float* meta_eac,
                 const float* meta_zeta) {
  if (head_dim != 128 || !q || q_len < 1 || kv_heads < 1 || q_heads % kv_heads) return OC_ERR_UNSUPPORTED;
  const int G = q_heads / kv_heads, R = q_len * G, nb = seq_len / kBlock;
  // Counts share an int32 with 16 bits each (blk_state, the row word): at
  // most 32767 blocks per row and 32767 KV heads keep them non-negative.
  if (R > kFusedMaxRows || nb < 1 || nb > 0x7fff || kv_heads > 0x7fff) return OC_ERR_UNSUPPORTED;
  if (out_dtype != OC_BF16 && out_dtype != OC_F32) return OC_ERR_UNSUPPORTED;
  const FusedLayout L = fused_layout(batch, nb, kv_heads);
  const int64_t ntiles = (int64_t)batch * nb * kv_heads;
  if (ntiles >= (1ll << 31)) return OC_ERR_UNSUPPORTED;
  int grid = device_sm_count();
  if (grid > kFusedMaxGrid) grid = kFusedMaxGrid;
  if (ntiles < grid) grid = (int)ntiles;
  if (L.NG > grid || !ws || ws_bytes < L.bytes) return OC_ERR_UNSUPPORTED;
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || (reinterpret_cast<uintptr_t>(ws) & 255))
    return OC_ERR_UNSUPPORTED;

  ScoreArgs a = {};
  a.keys = k; a.q = q; a.S = seq_len; a.H = kv_heads; a.D = head_dim; a.nb = nb;
  a.Sq = q_len; a.Hq = q_heads; a.G = G;
  a.bands = Bands{{1, 64, 256}, {64, 256, kBlock}};
  a.tau = tau; a.zeta_max = zeta_max; a.keep = keep;
  FusedArgs f = {};
  f.epoch = reinterpret_cast<int*>(ws);
  f.sets = f.epoch + 1;
  f.set_ints = L.set_ints;
  float* pf = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(ws) + L.counters);
  const size_t parts = (size_t)L.NG * L.cpg * kFusedMaxRows;
  f.part_m = pf; f.part_l = pf + parts; f.part_o = pf + 2 * parts;
  f.out = out; f.out_bf16 = out_dtype == OC_BF16;
  f.pm = pm; f.pl = pl; f.po = po;
  f.perm = perm; f.count = count;
  f.B = batch; f.NG = L.NG; f.cpg = L.cpg; f.R = R;
  f.scale_log2 = 1.4426950408889634f / sqrtf((float)head_dim);
  if (px) f.px = *px;
  // Decisions from write-time metadata: all three arrays.
  if (META && (!meta_dc || !meta_eac || !meta_zeta)) return OC_ERR_NULL;
  if (META) {
    a.dc = const_cast<float*>(meta_dc);
    a.e_ac = const_cast<float*>(meta_eac);
    a.zeta = const_cast<float*>(meta_zeta);
  }

  CUtensorMap km, ak, av;
  const uint64_t cols = (uint64_t)kv_heads * 128, rows = (uint64_t)batch * seq_len;
  int rc = 0;
  const uint64_t kk[4] = {1, (uint64_t)k, (uint64_t)kv_heads | (128ull << 32), rows};
  const uint64_t ka[4] = {2, (uint64_t)k, cols, rows};
  const uint64_t kv[4] = {2, (uint64_t)v, cols, rows};
  if (!map_cache_get(kk, &km) && !(rc = encode_score_map(&km, k, kv_heads, 128, (int64_t)batch * nb)))
    map_cache_put(kk, km);
  if (!rc && !map_cache_get(ka, &ak) &&
      !(rc = encode_map_2d(&ak, k, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, cols, rows, 64, kFusedChunk, true)))
    map_cache_put(ka, ak);
  if (!rc && !map_cache_get(kv, &av) &&
      !(rc = encode_map_2d(&av, v, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, cols, rows, 64, kFusedChunk, true)))
    map_cache_put(kv, av);
  if (rc) return set_error(OC_ERR_CUDA, "oc_decode_step: tensor map encode failed (%d)", rc);
  const int smem = kStages * kSlabB + kQCacheBytes + 1024;
  // Once per device: the shared-memory opt-in, and the check that a CTA of
  // this size fits on every SM (the persistent grid relies on all its CTAs
  // being resident at once; with less room the separate kernels run instead).
  auto kern = score_tma_kernel<128, true, META>;
  static std::atomic<uint64_t> s_setup{0}, s_fits{0};
  if (first_on_device(s_setup)) {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    int per_sm = 0;
    int dev = 0;
    cudaGetDevice(&dev);
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kFusedThreads, smem) == cudaSuccess &&
        per_sm >= 1 && dev < kMaxCachedDevices)
      s_fits.fetch_or(1ull << dev);
  }
  {
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= kMaxCachedDevices || !(s_fits.load() & (1ull << dev))) return OC_ERR_UNSUPPORTED;
  }
  const cudaError_t e = launch_pdl(kern, dim3(grid), dim3(kFusedThreads), smem, st, km, ak, av, a, (int)ntiles, f);
  if (e != cudaSuccess) return set_error(OC_ERR_CUDA, "score_tma_kernel (fused): %s", cudaGetErrorString(e));
  return check_launch("score_tma_kernel (fused)");
}

}  // namespace
}  // namespace oc

#ifndef OC_SCORE_META_TU
using namespace oc;

extern "C" int oc_fwht512(const void* x, int x_dtype, int64_t ncols, float* y, oc_stream_t stream) {
  OC_REQUIRE(x && y, OC_ERR_NULL, "oc_fwht512: null pointer");
  OC_REQUIRE(ncols >= 0, OC_ERR_SHAPE, "oc_fwht512: ncols < 0");
  if (ncols == 0) return OC_OK;
  const int64_t grid = (ncols + kSlab - 1) / kSlab;
  OC_REQUIRE(grid < (1ll << 31), OC_ERR_CAPACITY, "oc_fwht512: too many columns");
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  cudaFuncSetAttribute(fwht512_kernel<float>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSlabBytes);
  cudaFuncSetAttribute(fwht512_kernel<__nv_bfloat16>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSlabBytes);
  if (x_dtype == OC_F32)
    fwht512_kernel<float><<<(unsigned)grid, kThreads, kSlabBytes, st>>>((const float*)x, y, ncols);
  else if (x_dtype == OC_BF16)
    fwht512_kernel<__nv_bfloat16><<<(unsigned)grid, kThreads, kSlabBytes, st>>>(
        (const __nv_bfloat16*)x, y, ncols);
  else
    return set_error(OC_ERR_DTYPE, "oc_fwht512: dtype %d", x_dtype);
  return check_launch("fwht512_kernel");
}

namespace oc {
int score_blocks_impl(const void* keys, const void* q, int dtype, int batch, int seq_len, int kv_heads,
                      int head_dim, int q_len, int q_heads, int bl0, int bl1, int bm0, int bm1, int bh0, int bh1,
                      float tau, float zeta_max, float* dc, float* e_low, float* e_mid, float* e_high, float* zeta,
                      float* bound_max, float* bounds, uint8_t* keep, float* e_ac, int mode, oc_stream_t stream);
}  // namespace oc

extern "C" int oc_score_blocks(const void* keys, const void* q, int dtype,
                               int batch, int seq_len, int kv_heads, int head_dim,
                               int q_len, int q_heads,
                               int bl0, int bl1, int bm0, int bm1, int bh0, int bh1,
                               float tau, float zeta_max,
                               float* dc, float* e_low, float* e_mid, float* e_high,
                               float* zeta, float* bound_max, float* bounds, uint8_t* keep,
                               int mode, oc_stream_t stream) {
  return score_blocks_impl(keys, q, dtype, batch, seq_len, kv_heads, head_dim, q_len, q_heads, bl0, bl1, bm0, bm1,
                           bh0, bh1, tau, zeta_max, dc, e_low, e_mid, e_high, zeta, bound_max, bounds, keep,
                           nullptr, mode, stream);
}

extern "C" int oc_block_metadata(const void* keys, int dtype, int batch, int seq_len, int kv_heads, int head_dim,
                                 float* dc, float* e_ac, float* zeta, oc_stream_t stream) {
  OC_REQUIRE(dc || e_ac || zeta, OC_ERR_NULL, "oc_block_metadata: no output");
  return score_blocks_impl(keys, nullptr, dtype, batch, seq_len, kv_heads, head_dim, 0, 0, 1, 64, 64, 256, 256,
                           512, 0.f, 0.f, dc, nullptr, nullptr, nullptr, zeta, nullptr, nullptr, nullptr, e_ac, 0,
                           stream);
}

namespace oc {
int score_blocks_impl(const void* keys, const void* q, int dtype, int batch, int seq_len, int kv_heads,
                      int head_dim, int q_len, int q_heads, int bl0, int bl1, int bm0, int bm1, int bh0, int bh1,
                      float tau, float zeta_max, float* dc, float* e_low, float* e_mid, float* e_high, float* zeta,
                      float* bound_max, float* bounds, uint8_t* keep, float* e_ac, int mode, oc_stream_t stream) {
  OC_REQUIRE(keys, OC_ERR_NULL, "oc_score_blocks: keys is NULL");
  OC_REQUIRE(batch >= 1 && kv_heads >= 1, OC_ERR_SHAPE, "oc_score_blocks: batch/kv_heads < 1");
  OC_REQUIRE(seq_len >= 0 && seq_len % kBlock == 0, OC_ERR_SHAPE,
             "oc_score_blocks: seq_len %d is not a multiple of 512", seq_len);
  OC_REQUIRE(head_dim == 64 || head_dim == 128 || head_dim == 256, OC_ERR_SHAPE,
             "oc_score_blocks: head_dim %d not in {64,128,256}", head_dim);
  OC_REQUIRE(dtype == OC_F32 || dtype == OC_BF16, OC_ERR_DTYPE, "oc_score_blocks: dtype %d", dtype);
  OC_REQUIRE(aligned16(keys), OC_ERR_ALIGN, "oc_score_blocks: keys not 16-byte aligned");
  OC_REQUIRE(!q || aligned16(q), OC_ERR_ALIGN, "oc_score_blocks: q not 16-byte aligned");
  if (q) {
    OC_REQUIRE(q_len >= 1 && q_heads >= 1 && q_heads % kv_heads == 0, OC_ERR_SHAPE,
               "oc_score_blocks: q_heads %d must be a positive multiple of kv_heads %d (q_len %d)",
               q_heads, kv_heads, q_len);
  }
  Bands bd{{bl0, bm0, bh0}, {bl1, bm1, bh1}};
  for (int i = 0; i < 3; ++i)
    OC_REQUIRE(bd.lo[i] >= 0 && bd.hi[i] <= kBlock && bd.lo[i] <= bd.hi[i], OC_ERR_SHAPE,
               "oc_score_blocks: band %d = [%d, %d) outside [0, 512)", i, bd.lo[i], bd.hi[i]);
  if (mode == 0) mode = bands_partial_ok(bd) ? 1 : 2;
  OC_REQUIRE(mode >= 1 && mode <= 3, OC_ERR_SHAPE, "oc_score_blocks: mode %d", mode);
  OC_REQUIRE(mode == 2 || bands_partial_ok(bd), OC_ERR_SHAPE,
             "oc_score_blocks: modes 1 and 3 need band edges in {0, 1, 64k}");
  const int nb = seq_len / kBlock;
  const int64_t ncta = (int64_t)batch * nb * kv_heads;
  if (ncta == 0) return OC_OK;
  OC_REQUIRE(ncta < (1ll << 31), OC_ERR_CAPACITY, "oc_score_blocks: too many blocks");
  ScoreArgs a = {};
  a.keys = keys; a.q = q; a.S = seq_len; a.H = kv_heads; a.D = head_dim; a.nb = nb;
  a.Sq = q ? q_len : 0; a.Hq = q ? q_heads : 0; a.G = q ? q_heads / kv_heads : 1;
  a.bands = bd; a.tau = tau; a.zeta_max = zeta_max;
  a.dc = dc; a.e_low = e_low; a.e_mid = e_mid; a.e_high = e_high; a.zeta = zeta;
  a.bound_max = bound_max; a.bounds = q ? bounds : nullptr; a.keep = keep; a.e_ac = e_ac;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (dtype == OC_F32) return launch_score<float>(a, mode, (int)ncta, st);
  return launch_score<__nv_bfloat16>(a, mode, (int)ncta, st);
}
}  // namespace oc

// ---------------------------------------------------------------------------
// The two gates from write-time metadata (no key is read): one warp per
// (batch, block, kv head) cell computes the bound of every query row of the
// group from the cached DC coefficients and E_AC (spectral_energy.py:150-177),
// its max (:195), and the keep bit with the cached zeta (:196, :231-234).
// ---------------------------------------------------------------------------
namespace oc {
namespace {
// Where the metadata of logical cell (b, j, h) lives: the cell itself, or,
// for a paged cache, page table[b][j] of a pool of num_pages pages (-1: an
// invalid page, whose block is never kept).
struct MetaSrc {
  const int32_t* table;
  int table_stride, num_pages;
};
__device__ __forceinline__ int64_t meta_src(const MetaSrc& m, int b, int j, int h, int nb, int H) {
  if (!m.table) return ((int64_t)b * nb + j) * H + h;
  const int p = m.table[(size_t)b * m.table_stride + j];
  return (p >= 0 && p < m.num_pages) ? (int64_t)p * H + h : -1;
}

template <typename T>
__global__ void __launch_bounds__(256)
meta_gates_kernel(const float* __restrict__ dc, const float* __restrict__ e_ac, const float* __restrict__ zeta,
                  const T* __restrict__ q, int nb, int H, int D, int Sq, int Hq, int G, int64_t cells, float tau,
                  float zeta_max, float* bound_max, float* bounds, uint8_t* keep, MetaSrc ms) {
  const int lane = threadIdx.x & 31;
  const int64_t cell = (int64_t)blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
  if (cell >= cells) return;
  const int h = (int)(cell % H);
  const int j = (int)((cell / H) % nb);
  const int b = (int)(cell / ((int64_t)H * nb));
  const int64_t src = meta_src(ms, b, j, h, nb, H);
  if (src < 0) {
    if (lane == 0) {
      if (bound_max) bound_max[cell] = -INFINITY;
      if (keep) keep[cell] = 0;
    }
    return;
  }
  const float sqrt_d = sqrtf((float)D);
  const float resid_scale = sqrtf(e_ac[src]);
  const float* dcc = dc + src * D;
  float bmax = -INFINITY;
  const int rows = Sq * G;
  for (int r = 0; r < rows; ++r) {
    const int s = r / G, gq = r - s * G;
    const size_t qrow = ((size_t)b * Sq + s) * Hq + (size_t)h * G + gq;
    const T* qr = q + qrow * D;
    float dot = 0.f, nrm = 0.f;
    for (int c = lane; c < D; c += 32) {
      const float qv = to_f32<T>(qr[c]);
      dot = fmaf(qv, dcc[c] / kNorm, dot);  // block mean = DC / sqrt(512)
      nrm = fmaf(qv, qv, nrm);
    }
    dot = warp_sum(dot);
    nrm = warp_sum(nrm);
    const float bound = dot / sqrt_d + (sqrtf(nrm) * resid_scale) / sqrt_d;
    if (bounds && lane == 0) bounds[(((size_t)b * Sq + s) * nb + j) * Hq + (size_t)h * G + gq] = bound;
    bmax = fmaxf(bmax, bound);
  }
  if (lane == 0) {
    if (bound_max) bound_max[cell] = bmax;
    if (keep) keep[cell] = (bmax >= tau && zeta[src] <= zeta_max) ? 1 : 0;
  }
}
}  // namespace
}  // namespace oc

namespace oc {
namespace {
// ---------------------------------------------------------------------------
// The same gates for long query chunks (chunked prefill: thousands of query
// rows per KV head).  The bounds of all rows against all blocks are a small
// float32 GEMM (rows x D) . (D x blocks) per (batch, KV head), tiled so that
// every query row is read once per 64 blocks instead of once per block:
//   meta_bound_init_kernel  bound_max <- ordered key of -inf
//   meta_bound_gemm_kernel  CTA = 128 rows x 64 blocks of one (b, h); each
//                           thread 8 rows x 4 blocks; row norms on the way;
//                           bound per (row, block) (optionally stored), max
//                           over the CTA's rows, atomicMax of the ordered
//                           integer key into bound_max
//   meta_bound_gates_kernel key -> float, keep = bound >= tau && zeta <= zeta_max
// The per-term arithmetic is the warp kernel's: mean = DC / sqrt(512) in
// float32, dot in float32, bound = dot / sqrt(D) + sqrt(|q|^2) sqrt(E_AC) / sqrt(D).
// ---------------------------------------------------------------------------
// Monotone map of float32 onto int32 (for atomicMax over floats of any sign).
__device__ __forceinline__ int f2key(float f) {
  const int i = __float_as_int(f);
  return i >= 0 ? i : i ^ 0x7fffffff;
}
__device__ __forceinline__ float key2f(int k) { return __int_as_float(k >= 0 ? k : k ^ 0x7fffffff); }

__global__ void meta_bound_init_kernel(int* key, int64_t cells) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < cells) key[i] = f2key(-INFINITY);
}

constexpr int kMbRows = 128, kMbBlk = 64, kMbK = 32;
constexpr int kMetaGemmMinRows = 32;  // query rows per KV head above which the GEMM form is used

template <typename T>
__global__ void __launch_bounds__(256)
meta_bound_gemm_kernel(const float* __restrict__ dc, const float* __restrict__ e_ac, const T* __restrict__ q,
                       int nb, int H, int D, int Sq, int Hq, int G, int* key, float* bounds, MetaSrc ms) {
  __shared__ float qs[kMbK][kMbRows + 4];
  __shared__ float ds[kMbK][kMbBlk + 4];
  __shared__ float s_nrm[kMbRows];
  __shared__ float s_max[16][kMbBlk];
  const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
  const int bh = blockIdx.y, h = bh % H, b = bh / H;
  const int r0 = blockIdx.x * kMbRows, j0 = blockIdx.z * kMbBlk;
  const int rows = Sq * G;
  // loader roles: q row lr (two threads per row, 16 dims each), dc block ld
  const int lr = tid >> 1, lhalf = tid & 1;
  const int grow = r0 + lr;
  const T* qrow = nullptr;
  if (grow < rows) {
    const int s = grow / G, g = grow - s * G;
    qrow = q + (((size_t)b * Sq + s) * Hq + (size_t)h * G + g) * D;
  }
  const int lb = tid >> 2, lq = tid & 3;  // dc: block lb, 8 dims at lq*8
  const int64_t dsrc = (j0 + lb < nb) ? meta_src(ms, b, j0 + lb, h, nb, H) : -1;
  const float* dcrow = dsrc >= 0 ? dc + dsrc * D : nullptr;
  float acc[8][4];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int c = 0; c < 4; ++c) acc[i][c] = 0.f;
  float nrm = 0.f;
  for (int k0 = 0; k0 < D; k0 += kMbK) {
#pragma unroll
    for (int e = 0; e < 16; ++e) {
      const int k = lhalf * 16 + e;
      const float v = qrow ? to_f32<T>(qrow[k0 + k]) : 0.f;
      nrm = fmaf(v, v, nrm);
      qs[k][lr] = v;
    }
#pragma unroll
    for (int e = 0; e < 8; ++e) ds[lq * 8 + e][lb] = dcrow ? dcrow[k0 + lq * 8 + e] / kNorm : 0.f;
    __syncthreads();
#pragma unroll
    for (int k = 0; k < kMbK; ++k) {
      float a[8], bv[4];
#pragma unroll
      for (int i = 0; i < 8; ++i) a[i] = qs[k][ty * 8 + i];
#pragma unroll
      for (int c = 0; c < 4; ++c) bv[c] = ds[k][tx * 4 + c];
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int c = 0; c < 4; ++c) acc[i][c] = fmaf(a[i], bv[c], acc[i][c]);
    }
    __syncthreads();
  }
  nrm += __shfl_xor_sync(0xffffffffu, nrm, 1);
  if (lhalf == 0) s_nrm[lr] = nrm;
  __syncthreads();
  const float sqrt_d = sqrtf((float)D);
  float bm[4];
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    const int j = j0 + tx * 4 + c;
    const int64_t esrc = j < nb ? meta_src(ms, b, j, h, nb, H) : -1;
    const float rs = esrc >= 0 ? sqrtf(e_ac[esrc]) : 0.f;
    bm[c] = -INFINITY;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int r = r0 + ty * 8 + i;
      if (r < rows && esrc >= 0) {
        const float bound = acc[i][c] / sqrt_d + (sqrtf(s_nrm[ty * 8 + i]) * rs) / sqrt_d;
        if (bounds) {
          const int s = r / G, g = r - s * G;
          bounds[(((size_t)b * Sq + s) * nb + j) * Hq + (size_t)h * G + g] = bound;
        }
        bm[c] = fmaxf(bm[c], bound);
      }
    }
    s_max[ty][tx * 4 + c] = bm[c];
  }
  __syncthreads();
  if (tid < kMbBlk && j0 + tid < nb) {
    float m = s_max[0][tid];
#pragma unroll
    for (int y = 1; y < 16; ++y) m = fmaxf(m, s_max[y][tid]);
    atomicMax(&key[((size_t)b * nb + j0 + tid) * H + h], f2key(m));
  }
}

// The same bound GEMM on the tensor cores for bfloat16 queries:
// mma.sync m16n8k8 with tf32 operands and float32 accumulation.  A bfloat16
// query is exact in tf32 (8 of its 10 mantissa bits); each block mean is
// split into a tf32 part and the tf32 of its remainder (two MMAs), so the
// dot keeps about 21 bits of the mean, against 24 for the float32 FMA chain
// of meta_bound_gemm_kernel — both differ from the float64 sum of the oracle
// only by rounding.  CTA = 128 rows x 64 blocks of one (b, h), 8 warps of
// 32 rows x 32 blocks; the K dimension is staged 32 at a time.
constexpr int kMtLdq = kMbRows + 8, kMtLdb = kMbBlk + 8;  // row pitch = 8 mod 32 banks: conflict-free fragments

__device__ __forceinline__ uint32_t tf32_rna(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return r;
}

__device__ __forceinline__ void mma_tf32(float* c, const uint32_t* a, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__global__ void __launch_bounds__(256)
meta_bound_mma_kernel(const float* __restrict__ dc, const float* __restrict__ e_ac,
                      const __nv_bfloat16* __restrict__ q, int nb, int H, int D, int Sq, int Hq, int G, int* key,
                      float* bounds, MetaSrc ms) {
  __shared__ float qs[kMbK][kMtLdq];
  __shared__ uint32_t dh[kMbK][kMtLdb], dl[kMbK][kMtLdb];
  __shared__ float s_nrm[kMbRows];
  __shared__ float s_rs[kMbBlk];
  __shared__ float s_max[4][kMbBlk];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = lane >> 2, c4 = lane & 3;
  const int wr = (warp & 3) * 32, wc = (warp >> 2) * 32;  // warp tile origin: rows, blocks
  const int bh = blockIdx.y, h = bh % H, b = bh / H;
  const int r0 = blockIdx.x * kMbRows, j0 = blockIdx.z * kMbBlk;
  const int rows = Sq * G;
  // loaders: query row lr (two threads per row, 16 dims each as two 16-byte
  // vectors); block lb (four threads per block, 8 dims each as two float4)
  const int lr = tid >> 1, lhalf = tid & 1;
  const __nv_bfloat16* qrow = nullptr;
  if (r0 + lr < rows) {
    const int s = (r0 + lr) / G, gq = (r0 + lr) - s * G;
    qrow = q + (((size_t)b * Sq + s) * Hq + (size_t)h * G + gq) * D;
  }
  const int lb = tid >> 2, lq = tid & 3;
  const int64_t dsrc = (j0 + lb < nb) ? meta_src(ms, b, j0 + lb, h, nb, H) : -1;
  const float* dcrow = dsrc >= 0 ? dc + dsrc * D : nullptr;
  if (tid < kMbBlk) {
    const int64_t es = (j0 + tid < nb) ? meta_src(ms, b, j0 + tid, h, nb, H) : -1;
    s_rs[tid] = es >= 0 ? sqrtf(e_ac[es]) : -1.f;  // -1: no block
  }
  float acc[2][4][4];
#pragma unroll
  for (int m = 0; m < 2; ++m)
#pragma unroll
    for (int n = 0; n < 4; ++n)
#pragma unroll
      for (int c = 0; c < 4; ++c) acc[m][n][c] = 0.f;
  float nrm = 0.f;
  for (int k0 = 0; k0 < D; k0 += kMbK) {
    {
      uint4 v[2] = {make_uint4(0, 0, 0, 0), make_uint4(0, 0, 0, 0)};
      if (qrow) {
        const uint4* src = reinterpret_cast<const uint4*>(qrow + k0 + lhalf * 16);
        v[0] = src[0];
        v[1] = src[1];
      }
      const __nv_bfloat16* e16 = reinterpret_cast<const __nv_bfloat16*>(v);
#pragma unroll
      for (int e = 0; e < 16; ++e) {
        const float x = __bfloat162float(e16[e]);
        nrm = fmaf(x, x, nrm);
        qs[lhalf * 16 + e][lr] = x;
      }
    }
    {
      float4 v[2] = {make_float4(0.f, 0.f, 0.f, 0.f), make_float4(0.f, 0.f, 0.f, 0.f)};
      if (dcrow) {
        const float4* src = reinterpret_cast<const float4*>(dcrow + k0 + lq * 8);
        v[0] = src[0];
        v[1] = src[1];
      }
      const float* f = reinterpret_cast<const float*>(v);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const float mean = f[e] / kNorm;  // block mean = DC / sqrt(512), as in the FMA form
        const uint32_t hi = tf32_rna(mean);
        dh[lq * 8 + e][lb] = hi;
        dl[lq * 8 + e][lb] = tf32_rna(mean - __uint_as_float(hi));
      }
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < kMbK; kk += 8) {
      uint32_t a[2][4];
#pragma unroll
      for (int m = 0; m < 2; ++m) {
        const int rr = wr + m * 16 + g;
        a[m][0] = __float_as_uint(qs[kk + c4][rr]);
        a[m][1] = __float_as_uint(qs[kk + c4][rr + 8]);
        a[m][2] = __float_as_uint(qs[kk + c4 + 4][rr]);
        a[m][3] = __float_as_uint(qs[kk + c4 + 4][rr + 8]);
      }
#pragma unroll
      for (int n = 0; n < 4; ++n) {
        const int cc = wc + n * 8 + g;
        const uint32_t h0 = dh[kk + c4][cc], h1 = dh[kk + c4 + 4][cc];
        const uint32_t l0 = dl[kk + c4][cc], l1 = dl[kk + c4 + 4][cc];
#pragma unroll
        for (int m = 0; m < 2; ++m) {
          mma_tf32(acc[m][n], a[m], l0, l1);
          mma_tf32(acc[m][n], a[m], h0, h1);
        }
      }
    }
    __syncthreads();
  }
  nrm += __shfl_xor_sync(0xffffffffu, nrm, 1);
  if (lhalf == 0) s_nrm[lr] = nrm;
  __syncthreads();
  const float sqrt_d = sqrtf((float)D);
#pragma unroll
  for (int n = 0; n < 4; ++n) {
#pragma unroll
    for (int c = 0; c < 2; ++c) {
      const int jl = wc + n * 8 + 2 * c4 + c;  // block within the CTA tile
      const float rs = s_rs[jl];
      float bm = -INFINITY;
#pragma unroll
      for (int m = 0; m < 2; ++m)
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) {
          const int rl = wr + m * 16 + g + 8 * hf;
          const int r = r0 + rl;
          if (r < rows && rs >= 0.f) {
            const float bound = acc[m][n][2 * hf + c] / sqrt_d + (sqrtf(s_nrm[rl]) * rs) / sqrt_d;
            if (bounds) {
              const int s = r / G, gq = r - s * G;
              bounds[(((size_t)b * Sq + s) * nb + j0 + jl) * Hq + (size_t)h * G + gq] = bound;
            }
            bm = fmaxf(bm, bound);
          }
        }
      // max over the 8 row groups g (lanes of equal c4)
      bm = fmaxf(bm, __shfl_xor_sync(0xffffffffu, bm, 4));
      bm = fmaxf(bm, __shfl_xor_sync(0xffffffffu, bm, 8));
      bm = fmaxf(bm, __shfl_xor_sync(0xffffffffu, bm, 16));
      if (g == 0) s_max[warp & 3][jl] = bm;
    }
  }
  __syncthreads();
  if (tid < kMbBlk && j0 + tid < nb && s_rs[tid] >= 0.f) {
    const float m = fmaxf(fmaxf(s_max[0][tid], s_max[1][tid]), fmaxf(s_max[2][tid], s_max[3][tid]));
    atomicMax(&key[((size_t)b * nb + j0 + tid) * H + h], f2key(m));
  }
}

// The bound GEMM on the 5th-generation tensor cores (tcgen05, accumulators
// in tensor memory) for bfloat16 queries with head_dim 128.  A bfloat16
// query is exact as an MMA operand; each block mean (DC / sqrt(512) in
// float32, as in the FMA form) is split into three bfloat16 parts
// m = p1 + p2 + p3 (24 significant bits, the float32 mean up to its last
// bit), so one M128 N192 K16 kind::f16 MMA per 16 channels gives q . p1,
// q . p2 and q . p3 in three column ranges of float32 accumulators, summed
// in the epilogue (smallest first).  The bound is
// (q . m + |q| sqrt(E_AC)) * (1 / sqrt(D)): the FMA form's terms, one
// rounding apart.
// CTA = one (b, h), 64 blocks, tpc row tiles of 128 query rows (gq adjacent
// query heads x 128 / gq positions, so each position's rows are one
// contiguous run).  16 warps: thread 0 issues the TMA loads of the row tiles
// (a ring of three) and the MMAs, into two tensor-memory accumulators so that
// a tile's MMA overlaps the previous tile's epilogue; there warp w reads tensor-memory
// lanes 32 (w % 4) .. + 31 (rows) and block columns 16 (w / 4) .. + 15, and
// every thread keeps a running max per block over its rows; the CTA ends with
// one max per block (atomicMax of the ordered key, as in the FMA form).
constexpr int kBtRows = 128, kBtBlk = 64, kBtN = 3 * kBtBlk, kBtThreads = 512;
constexpr int kBtCols = kBtBlk / (kBtThreads / 128);  // block columns per thread: 16
constexpr int kBtATile = kBtRows * 128 * 2;  // bf16 row tile: two 128B-swizzled boxes of 64 channels
constexpr int kBtBBox = kBtN * 128;          // 192 rows x 64 channels of bf16
constexpr int kBtABufs = 3;  // query row-tile ring
struct BtSmem {
  unsigned char a[kBtABufs][kBtATile];
  unsigned char bm[2][kBtBBox];
  uint64_t a_full[kBtABufs], mma_done[2];
  uint32_t tmem;
  float s_rs[kBtBlk];
  float s_nrm[2][kBtThreads / 128][kBtRows];  // partial squared row norms by column group, per accumulator
  float s_max[4][kBtBlk];
};
constexpr size_t kBtSmemBytes = sizeof(BtSmem) + 1024;

// 16 consecutive fp32 columns of this thread's lane, loaded without waiting:
// the registers are valid only after tmem_ld_wait().
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
}

// Waits for this thread's outstanding tensor-memory loads, then passes each of
// the n loaded registers through an empty volatile statement after the wait,
// so that no use of them can be scheduled before it.
template <int n>
__device__ __forceinline__ void tmem_ld_wait(uint32_t* r) {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < n; ++i) asm volatile("" : "+r"(r[i]));
}

__global__ void __launch_bounds__(kBtThreads, 1)
meta_bound_tc_kernel(const __grid_constant__ CUtensorMap mq, const float* __restrict__ dc,
                     const float* __restrict__ e_ac, int nb, int H, int Sq, int Hq, int G, int gq, int ntiles, int tpc,
                     int* key, float* bounds, MetaSrc ms) {
  constexpr int D = 128;
  extern __shared__ unsigned char bt_raw[];
  BtSmem& sm = *reinterpret_cast<BtSmem*>((reinterpret_cast<uintptr_t>(bt_raw) + 1023) & ~uintptr_t(1023));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int quarter = warp & 3, cg = warp >> 2;  // tensor-memory lane quarter, column group
  const int row = quarter * 32 + lane;           // row of the tile (tensor-memory lane)
  const int bh = blockIdx.y, h = bh % H, b = bh / H;
  const int j0 = blockIdx.z * kBtBlk;
  const int t0 = blockIdx.x * tpc;
  const int nt = min(tpc, ntiles - t0);
  if (tid == 0) {
    for (int i = 0; i < kBtABufs; ++i) mbar_init(&sm.a_full[i], 1);
    mbar_init(&sm.mma_done[0], 1);
    mbar_init(&sm.mma_done[1], 1);
    fence_mbar_init();
  }
  if (warp == 0) {  // two accumulators of 192 columns, at columns 0 and 256
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&sm.tmem)),
                 "r"(512)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  if (tid < kBtBlk) {
    const int64_t es = (j0 + tid < nb) ? meta_src(ms, b, j0 + tid, h, nb, H) : -1;
    sm.s_rs[tid] = es >= 0 ? sqrtf(e_ac[es]) : -1.f;  // -1: no block
  }
  {
    // B operand: rows p * 64 + jj (part p of block jj's mean), K-major,
    // 128-byte swizzle (16-byte chunk c of row n at chunk c ^ (n % 8)).
    // Thread: block jj, channels 16 kq .. 16 kq + 15 (two 16-byte chunks).
    const int jj = tid >> 3, kq = tid & 7;
    const int kb = kq >> 2;  // box of 64 channels
    const int64_t src = (j0 + jj < nb) ? meta_src(ms, b, j0 + jj, h, nb, H) : -1;
    const float* rowp = src >= 0 ? dc + src * D + kq * 16 : nullptr;
#pragma unroll
    for (int cc = 0; cc < 2; ++cc) {
      const int c = (kq & 3) * 2 + cc;  // 16-byte chunk within the box's 128-byte row
      float v[8];
      if (rowp) {
        const float4 x = reinterpret_cast<const float4*>(rowp)[2 * cc];
        const float4 y = reinterpret_cast<const float4*>(rowp)[2 * cc + 1];
        v[0] = x.x; v[1] = x.y; v[2] = x.z; v[3] = x.w; v[4] = y.x; v[5] = y.y; v[6] = y.z; v[7] = y.w;
      } else {
#pragma unroll
        for (int e = 0; e < 8; ++e) v[e] = 0.f;
      }
      uint32_t pk[3][4];
#pragma unroll
      for (int e = 0; e < 8; e += 2) {
        float r0 = v[e] / kNorm, r1 = v[e + 1] / kNorm;
#pragma unroll
        for (int p = 0; p < 3; ++p) {
          const __nv_bfloat16 h0 = __float2bfloat16_rn(r0), h1 = __float2bfloat16_rn(r1);
          pk[p][e / 2] = (uint32_t)__bfloat16_as_ushort(h0) | ((uint32_t)__bfloat16_as_ushort(h1) << 16);
          r0 -= __bfloat162float(h0);
          r1 -= __bfloat162float(h1);
        }
      }
#pragma unroll
      for (int p = 0; p < 3; ++p) {
        const int n = p * kBtBlk + jj;
        *reinterpret_cast<uint4*>(sm.bm[kb] + n * 128 + ((c ^ (n & 7)) << 4)) =
            make_uint4(pk[p][0], pk[p][1], pk[p][2], pk[p][3]);
      }
    }
  }
  fence_proxy_async();  // the B operand written by threads is read by the tensor cores
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sm.tmem;
  // A row tile: gq query heads (of this KV head's G) x 128 / gq positions,
  // row r = position s0 + r / gq, head hq0 + r % gq
  const int ng = G / gq, ppt = kBtRows / gq;
  auto load_tile = [&](int t) {
    const int T = t0 + t, hq = h * G + (T % ng) * gq, s0 = (T / ng) * ppt;
    uint64_t* bar = &sm.a_full[t % kBtABufs];
    mbar_expect_tx(bar, kBtATile);
    tma_load_3d(sm.a[t % kBtABufs], &mq, bar, 0, hq, b * Sq + s0);
    tma_load_3d(sm.a[t % kBtABufs] + kBtATile / 2, &mq, bar, 64, hq, b * Sq + s0);
  };
  if (tid == 0)
    for (int t = 0; t < kBtABufs && t < nt; ++t) load_tile(t);
  float rmax[kBtCols], rs[kBtCols];
#pragma unroll
  for (int i = 0; i < kBtCols; ++i) {
    rmax[i] = -INFINITY;
    rs[i] = sm.s_rs[cg * kBtCols + i];
  }
  const float inv_sqrt_d = 1.f / sqrtf((float)D);
  constexpr uint32_t kId = tc_idesc_bf16(kBtRows, kBtN, 0);
  const uint32_t t_row = tmem + ((uint32_t)(quarter * 32) << 16) + cg * kBtCols;
  // Tile t: its MMA (accumulator t % 2) is issued in iteration t, its
  // epilogue runs in iteration t + 1, overlapping the MMA of tile t + 1.
  bool ok = true;
  for (int t = 0; t <= nt; ++t) {
    if (t < nt) {
      const int buf = t % kBtABufs;
      const bool got = mbar_wait(&sm.a_full[buf], (t / kBtABufs) & 1);
      if (__syncthreads_or(!got)) { ok = false; break; }
      {
        // partial squared norm of row `row` over this column group's 32 channels
        float nrm4[4] = {0.f, 0.f, 0.f, 0.f};  // four independent chains
#pragma unroll
        for (int c4 = 0; c4 < 4; ++c4) {
          const int c = cg * 4 + c4, kb = c >> 3, cl = c & 7;
          const uint4 w = *reinterpret_cast<const uint4*>(sm.a[buf] + kb * (kBtATile / 2) + row * 128 +
                                                          ((cl ^ (row & 7)) << 4));
          const uint32_t u[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float lo = __uint_as_float(u[e] << 16), hi = __uint_as_float(u[e] & 0xffff0000u);
            nrm4[e] = fmaf(lo, lo, nrm4[e]);
            nrm4[e] = fmaf(hi, hi, nrm4[e]);
          }
        }
        sm.s_nrm[t & 1][cg][row] = (nrm4[0] + nrm4[1]) + (nrm4[2] + nrm4[3]);
      }
      if (tid == 0) {
        tc_fence_after();
        const uint32_t ab = smem_u32(sm.a[buf]), bb = smem_u32(sm.bm[0]);
        const uint32_t acc = tmem + (uint32_t)(t & 1) * 256;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint64_t ad = sdesc(ab + (kk >> 2) * (kBtATile / 2) + (kk & 3) * 32, 16, 1024);
          const uint64_t bd = sdesc(bb + (kk >> 2) * kBtBBox + (kk & 3) * 32, 16, 1024);
          umma_bf16(acc, ad, bd, kId, kk > 0 ? 1 : 0);
        }
        umma_commit(&sm.mma_done[t & 1]);
      }
    }
    if (t == 0) continue;
    const int e = t - 1;  // the tile whose epilogue runs now
    const bool done = mbar_wait(&sm.mma_done[e & 1], (e >> 1) & 1);
    tc_fence_after();
    if (__syncthreads_or(!done)) { ok = false; break; }
    // tile e's MMA is complete and every thread read its buffer (before the
    // barrier of iteration e): the buffer takes tile e + 3
    if (tid == 0 && e + kBtABufs < nt) load_tile(e + kBtABufs);
    const int T = t0 + e, hq = h * G + (T % ng) * gq + row % gq, s = (T / ng) * ppt + row / gq;
    const bool valid = s < Sq;
    const float rn = sqrtf((sm.s_nrm[e & 1][0][row] + sm.s_nrm[e & 1][1][row]) +
                           (sm.s_nrm[e & 1][2][row] + sm.s_nrm[e & 1][3][row]));
    const uint32_t t_acc = t_row + (uint32_t)(e & 1) * 256;
    // the three partial-dot column ranges of this row: three loads in
    // flight, one wait
    uint32_t xr[3 * kBtCols];
    tmem_ld16(t_acc, xr);
    tmem_ld16(t_acc + kBtBlk, xr + kBtCols);
    tmem_ld16(t_acc + 2 * kBtBlk, xr + 2 * kBtCols);
    tmem_ld_wait<3 * kBtCols>(xr);
    // rmax keeps the unscaled maximum; the 1/sqrt(D) scale is applied once
    // per block at the end (rounding is monotonic, so the scaled maximum is
    // the same float).  Columns of absent blocks (rs < 0) are never read.
    if (valid) {
      if (bounds) {
#pragma unroll
        for (int i = 0; i < kBtCols; ++i) {
          if (rs[i] >= 0.f) {
            const float u = fmaf(rn, rs[i], __uint_as_float(xr[2 * kBtCols + i]) + __uint_as_float(xr[kBtCols + i]) +
                                                __uint_as_float(xr[i]));
            bounds[(((size_t)b * Sq + s) * nb + j0 + cg * kBtCols + i) * Hq + hq] = u * inv_sqrt_d;
            rmax[i] = fmaxf(rmax[i], u);
          }
        }
      } else {
#pragma unroll
        for (int i = 0; i < kBtCols; ++i)
          rmax[i] = fmaxf(rmax[i], fmaf(rn, rs[i], __uint_as_float(xr[2 * kBtCols + i]) +
                                                       __uint_as_float(xr[kBtCols + i]) + __uint_as_float(xr[i])));
      }
    }
    tc_fence_before();
    __syncthreads();  // accumulator e % 2 and norms e % 2 read: tile e + 2 may reuse them
  }
  if (!ok && tid == 0) atomicExch(&g_score_status, 1);
#pragma unroll
  for (int i = 0; i < kBtCols; ++i) {
    float m = rmax[i];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (lane == 0) sm.s_max[quarter][cg * kBtCols + i] = m;
  }
  tc_fence_before();
  __syncthreads();
  if (ok && tid < kBtBlk && j0 + tid < nb && sm.s_rs[tid] >= 0.f) {
    const float m = fmaxf(fmaxf(sm.s_max[0][tid], sm.s_max[1][tid]), fmaxf(sm.s_max[2][tid], sm.s_max[3][tid]));
    atomicMax(&key[((size_t)b * nb + j0 + tid) * H + h], f2key(m * inv_sqrt_d));
  }
  if (warp == 0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512) : "memory");
  }
}

__global__ void meta_bound_gates_kernel(float* bound_max, const float* __restrict__ zeta, int64_t cells, float tau,
                                        float zeta_max, uint8_t* keep, int nb, int H, MetaSrc ms) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= cells) return;
  const float bm = key2f(reinterpret_cast<int*>(bound_max)[i]);
  bound_max[i] = bm;
  const int h = (int)(i % H), j = (int)((i / H) % nb), b = (int)(i / ((int64_t)H * nb));
  const int64_t src = meta_src(ms, b, j, h, nb, H);
  if (keep) keep[i] = (src >= 0 && bm >= tau && zeta[src] <= zeta_max) ? 1 : 0;
}

template <typename T>
int launch_meta_bound_gemm(const float* dc, const float* e_ac, const float* zeta, const T* q, int B, int nb, int H,
                           int D, int Sq, int Hq, float tau, float zeta_max, float* bound_max, float* bounds,
                           uint8_t* keep, cudaStream_t st, MetaSrc ms) {
  const int64_t cells = (int64_t)B * nb * H;
  const int G = Hq / H;
  const int64_t rows = (int64_t)Sq * G;
  const int64_t gx = (rows + kMbRows - 1) / kMbRows;
  OC_REQUIRE(gx < (1ll << 31) && (int64_t)B * H < 65536 && (nb + kMbBlk - 1) / kMbBlk < 65536, OC_ERR_CAPACITY,
             "oc_score_from_metadata: grid too large");
  const unsigned g1 = (unsigned)((cells + 255) / 256);
  int* key = reinterpret_cast<int*>(bound_max);
  meta_bound_init_kernel<<<g1, 256, 0, st>>>(key, cells);
  dim3 grid((unsigned)gx, (unsigned)(B * H), (unsigned)((nb + kMbBlk - 1) / kMbBlk));
  if constexpr (std::is_same<T, __nv_bfloat16>::value) {
    if (D == 128 && aligned16(q) && aligned16(dc) && (int64_t)B * Sq < INT32_MAX) {
      // tcgen05 form: q as a (B*Sq, Hq, 128) tensor map, row tiles of 128
      // positions of one query head
      // a box of gq adjacent query heads x 128 / gq positions: 128 rows of
      // 128 bytes in runs of gq * 128 contiguous bytes
      const int gq = (G <= kBtRows && kBtRows % G == 0) ? G : 1;
      CUtensorMap mq;
      const uint64_t mkey[4] = {5, (uint64_t)q, (uint64_t)Hq | ((uint64_t)gq << 32), (uint64_t)B * Sq};
      if (!map_cache_get(mkey, &mq)) {
        const uint64_t dims[3] = {128, (uint64_t)Hq, (uint64_t)B * Sq};
        const uint64_t strides[2] = {256, (uint64_t)Hq * 256};
        const uint32_t box[3] = {64, (uint32_t)gq, (uint32_t)(kBtRows / gq)};
        const int r = encode_map_3d(&mq, q, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, dims, strides, box, true);
        if (r) return set_error(OC_ERR_CUDA, "oc_score_from_metadata: tensor map for q failed (CUresult %d)", r);
        map_cache_put(mkey, mq);
      }
      static std::atomic<uint64_t> s_setup{0};
      if (first_on_device(s_setup)) {
        cudaError_t e = cudaFuncSetAttribute(meta_bound_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)kBtSmemBytes);
        if (e != cudaSuccess) return set_error(OC_ERR_CUDA, "oc_score_from_metadata: %s", cudaGetErrorString(e));
      }
      // row tiles per CTA: one wave of at most one CTA per SM (one fits per SM)
      const int ntiles = (G / gq) * ((Sq + kBtRows / gq - 1) / (kBtRows / gq));
      const int64_t cols = (int64_t)B * H * ((nb + kBtBlk - 1) / kBtBlk);
      const int64_t per_col = std::max<int64_t>(1, device_sm_count() / cols);
      const int tpc = (int)((ntiles + per_col - 1) / per_col);
      dim3 tgrid((unsigned)((ntiles + tpc - 1) / tpc), (unsigned)(B * H), (unsigned)((nb + kBtBlk - 1) / kBtBlk));
      meta_bound_tc_kernel<<<tgrid, kBtThreads, kBtSmemBytes, st>>>(mq, dc, e_ac, nb, H, Sq, Hq, G, gq, ntiles, tpc, key,
                                                                    bounds, ms);
      meta_bound_gates_kernel<<<g1, 256, 0, st>>>(bound_max, zeta, cells, tau, zeta_max, keep, nb, H, ms);
      return check_launch("meta_bound_tc_kernel");
    }
    if (aligned16(q) && aligned16(dc)) {
      meta_bound_mma_kernel<<<grid, 256, 0, st>>>(dc, e_ac, q, nb, H, D, Sq, Hq, G, key, bounds, ms);
      meta_bound_gates_kernel<<<g1, 256, 0, st>>>(bound_max, zeta, cells, tau, zeta_max, keep, nb, H, ms);
      return check_launch("meta_bound_mma_kernel");
    }
  }
  meta_bound_gemm_kernel<T><<<grid, 256, 0, st>>>(dc, e_ac, q, nb, H, D, Sq, Hq, G, key, bounds, ms);
  meta_bound_gates_kernel<<<g1, 256, 0, st>>>(bound_max, zeta, cells, tau, zeta_max, keep, nb, H, ms);
  return check_launch("meta_bound_gemm_kernel");
}

}  // namespace
}  // namespace oc

namespace oc {
namespace {
int score_from_metadata_impl(const float* dc, const float* e_ac, const float* zeta, const void* q, int q_dtype,
                             int batch, int num_blocks, int kv_heads, int head_dim, int q_len, int q_heads, float tau,
                             float zeta_max, float* bound_max, float* bounds, uint8_t* keep, MetaSrc ms,
                             oc_stream_t stream) {
  OC_REQUIRE(dc && e_ac && zeta && q, OC_ERR_NULL, "oc_score_from_metadata: null input");
  OC_REQUIRE(bound_max || bounds || keep, OC_ERR_NULL, "oc_score_from_metadata: no output");
  OC_REQUIRE(batch >= 1 && num_blocks >= 0 && kv_heads >= 1 && head_dim >= 1 && q_len >= 1 &&
                 q_heads >= 1 && q_heads % kv_heads == 0,
             OC_ERR_SHAPE, "oc_score_from_metadata: bad shape");
  const int64_t cells = (int64_t)batch * num_blocks * kv_heads;
  if (cells == 0) return OC_OK;
  const int64_t grid = (cells + 7) / 8;
  OC_REQUIRE(grid < (1ll << 31), OC_ERR_CAPACITY, "oc_score_from_metadata: too many blocks");
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const int G = q_heads / kv_heads;
  // Long query chunks: the tiled bound GEMM (bound_max doubles as its
  // atomic-max scratch, so it must be given).
  if ((int64_t)q_len * G > kMetaGemmMinRows && bound_max && head_dim % kMbK == 0) {
    if (q_dtype == OC_F32)
      return launch_meta_bound_gemm<float>(dc, e_ac, zeta, (const float*)q, batch, num_blocks, kv_heads, head_dim,
                                           q_len, q_heads, tau, zeta_max, bound_max, bounds, keep, st, ms);
    if (q_dtype == OC_BF16)
      return launch_meta_bound_gemm<__nv_bfloat16>(dc, e_ac, zeta, (const __nv_bfloat16*)q, batch, num_blocks,
                                                   kv_heads, head_dim, q_len, q_heads, tau, zeta_max, bound_max,
                                                   bounds, keep, st, ms);
  }
  if (q_dtype == OC_F32)
    meta_gates_kernel<float><<<(unsigned)grid, 256, 0, st>>>(dc, e_ac, zeta, (const float*)q, num_blocks, kv_heads,
                                                             head_dim, q_len, q_heads, G, cells, tau, zeta_max,
                                                             bound_max, bounds, keep, ms);
  else if (q_dtype == OC_BF16)
    meta_gates_kernel<__nv_bfloat16><<<(unsigned)grid, 256, 0, st>>>(
        dc, e_ac, zeta, (const __nv_bfloat16*)q, num_blocks, kv_heads, head_dim, q_len, q_heads, G, cells, tau,
        zeta_max, bound_max, bounds, keep, ms);
  else
    return set_error(OC_ERR_DTYPE, "oc_score_from_metadata: q dtype %d", q_dtype);
  return check_launch("meta_gates_kernel");
}
}  // namespace
}  // namespace oc

extern "C" int oc_score_from_metadata(const float* dc, const float* e_ac, const float* zeta, const void* q,
                                      int q_dtype, int batch, int num_blocks, int kv_heads, int head_dim,
                                      int q_len, int q_heads, float tau, float zeta_max, float* bound_max,
                                      float* bounds, uint8_t* keep, oc_stream_t stream) {
  return oc::score_from_metadata_impl(dc, e_ac, zeta, q, q_dtype, batch, num_blocks, kv_heads, head_dim, q_len,
                                      q_heads, tau, zeta_max, bound_max, bounds, keep, oc::MetaSrc{nullptr, 0, 0},
                                      stream);
}

extern "C" int oc_score_from_metadata_paged(const float* dc_pool, const float* e_ac_pool, const float* zeta_pool,
                                            int num_pages, const int32_t* block_table, int table_stride,
                                            const void* q, int q_dtype, int batch, int num_blocks, int kv_heads,
                                            int head_dim, int q_len, int q_heads, float tau, float zeta_max,
                                            float* bound_max, float* bounds, uint8_t* keep, oc_stream_t stream) {
  OC_REQUIRE(block_table, OC_ERR_NULL, "oc_score_from_metadata_paged: block_table is NULL");
  OC_REQUIRE(num_pages >= 1 && table_stride >= num_blocks, OC_ERR_SHAPE,
             "oc_score_from_metadata_paged: num_pages %d, table_stride %d < num_blocks %d", num_pages, table_stride,
             num_blocks);
  return oc::score_from_metadata_impl(dc_pool, e_ac_pool, zeta_pool, q, q_dtype, batch, num_blocks, kv_heads,
                                      head_dim, q_len, q_heads, tau, zeta_max, bound_max, bounds, keep,
                                      oc::MetaSrc{block_table, table_stride, num_pages}, stream);
}

namespace oc {
int wait_limit_score(unsigned long long ns) {
  const int rc = set_wait_limit_here(ns);
  return rc ? rc : wait_limit_score_meta(ns);
}
int score_status(int* status, int reset) {
  // this unit's flag, or'ed with the metadata form's (oc_score_meta.cu)
  cudaError_t e = cudaMemcpyFromSymbol(status, g_score_status, sizeof(int));
  if (e != cudaSuccess) return set_error(OC_ERR_CUDA, "oc_device_status: %s", cudaGetErrorString(e));
  if (reset) {
    const int zero = 0;
    e = cudaMemcpyToSymbol(g_score_status, &zero, sizeof(int));
    if (e != cudaSuccess) return set_error(OC_ERR_CUDA, "oc_device_status: %s", cudaGetErrorString(e));
  }
  int meta = 0;
  const int rc = score_status_meta(&meta, reset);
  if (rc) return rc;
  *status |= meta;
  return OC_OK;
}
}  // namespace oc

#ifdef OC_TIMING
extern "C" int oc_probe_read_score_stamps(unsigned long long* host, int n) {
  return (int)cudaMemcpyFromSymbol(host, oc::g_sstamp, sizeof(unsigned long long) * 24 * n);
}
#endif

// ---------------------------------------------------------------------------
// Fused decode layer: host side.
// ---------------------------------------------------------------------------
namespace oc {

size_t xchg_region_bytes(int P, int NG) {
  return ((size_t)2 * P * NG * kXchgBlock * sizeof(uint64_t) + 255) / 256 * 256;
}

size_t decode_fused_bytes(int batch, int seq_len, int kv_heads) {
  return fused_layout(batch, seq_len / kBlock, kv_heads).bytes;
}

int decode_fused(const void* q, const void* k, const void* v, int batch, int q_len, int q_heads, int kv_heads,
                 int head_dim, int seq_len, float tau, float zeta_max, uint8_t* keep, int32_t* perm, int32_t* count,
                 void* out, int out_dtype, float* pm, float* pl, float* po, void* ws, size_t ws_bytes,
                 cudaStream_t st, const PeerXchg* px, const float* meta_dc, const float* meta_eac,
                 const float* meta_zeta) {
  if (meta_dc || meta_eac || meta_zeta)
    return decode_fused_meta(q, k, v, batch, q_len, q_heads, kv_heads, head_dim, seq_len, tau, zeta_max, keep, perm,
                             count, out, out_dtype, pm, pl, po, ws, ws_bytes, st, px, meta_dc, meta_eac, meta_zeta);
  return decode_fused_impl<false>(q, k, v, batch, q_len, q_heads, kv_heads, head_dim, seq_len, tau, zeta_max, keep,
                                  perm, count, out, out_dtype, pm, pl, po, ws, ws_bytes, st, px, nullptr, nullptr,
                                  nullptr);
}

}  // namespace oc
#else  // OC_SCORE_META_TU: the metadata form of the fused layer only

namespace oc {
int decode_fused_meta(const void* q, const void* k, const void* v, int batch, int q_len, int q_heads, int kv_heads,
                      int head_dim, int seq_len, float tau, float zeta_max, uint8_t* keep, int32_t* perm,
                      int32_t* count, void* out, int out_dtype, float* pm, float* pl, float* po, void* ws,
                      size_t ws_bytes, cudaStream_t st, const PeerXchg* px, const float* meta_dc,
                      const float* meta_eac, const float* meta_zeta) {
  return decode_fused_impl<true>(q, k, v, batch, q_len, q_heads, kv_heads, head_dim, seq_len, tau, zeta_max, keep,
                                 perm, count, out, out_dtype, pm, pl, po, ws, ws_bytes, st, px, meta_dc, meta_eac,
                                 meta_zeta);
}
int wait_limit_score_meta(unsigned long long ns) { return set_wait_limit_here(ns); }
int score_status_meta(int* status, int reset) {
  cudaError_t e = cudaMemcpyFromSymbol(status, g_score_status, sizeof(int));
  if (e != cudaSuccess) return set_error(OC_ERR_CUDA, "oc_device_status: %s", cudaGetErrorString(e));
  if (reset) {
    const int zero = 0;
    e = cudaMemcpyToSymbol(g_score_status, &zero, sizeof(int));
    if (e != cudaSuccess) return set_error(OC_ERR_CUDA, "oc_device_status: %s", cudaGetErrorString(e));
  }
  return OC_OK;
}
}  // namespace oc

#ifdef OC_TIMING
extern "C" int oc_probe_read_score_stamps_meta(unsigned long long* host, int n) {
  return (int)cudaMemcpyFromSymbol(host, oc::g_sstamp, sizeof(unsigned long long) * 24 * n);
}
#endif
#endif  // OC_SCORE_META_TU
