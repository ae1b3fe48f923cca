// Chunked-prefill indirect block attention on the 5th-generation tensor cores
// (tcgen05 + tensor memory), for query chunks long enough to make attention
// compute-bound: every query row of a chunk attends to the tokens of the
// retained blocks idx[0 .. count) of its batch row (and KV head, for per-head
// lists), with a streaming (online) softmax.
//
// Semantics: the per-block loop of indirect_attention / _multihead_loop
// (src/orthocache/indirect_attention.py:29-83, adaptive_attention.py:90-120)
// for any seq_len_q: logits = q.k / sqrt(D) in float32, softmax over all
// retained tokens, output o / l cast to the output dtype; count == 0 gives
// zeros (indirect_attention.py:150-151).  GQA: query head hq reads KV head
// hq / (Hq / Hkv).  No causal mask (the reference has none).
//
// Design (one persistent CTA per SM, 320 threads):
//   * a work unit is (batch row b, KV head h, two row tiles of 128 query rows
//     each); the two tiles share every K and V tile the unit streams, so the
//     tensor pipe alternates between them while the other tile's softmax runs;
//   * warp 8 is the TMA producer: the unit's two query tiles (32 KB each,
//     128B-swizzled boxes of 128 rows x 64 channels), then K_0, V_0, K_1,
//     V_1, ... (128 tokens x 128 channels, 32 KB each) into a 5-slot ring;
//   * warp 9 allocates 512 tensor-memory columns (per tile: S = 128 fp32
//     columns, O = 128 fp32 columns) and one of its threads issues every
//     tcgen05.mma: S_t = Q_t K_j^T (A and B K-major in shared memory) and
//     O_t += P_t V_j (P from tensor memory, V MN-major in shared memory),
//     8 instructions of M128 N128 K16 each, with tcgen05.commit to mbarriers;
//   * warps 0-3 / 4-7 are the softmax warpgroups of tile 0 / 1: each thread
//     owns one query row (tensor-memory lane), loads its 128 logits with
//     tcgen05.ld, keeps the running max and sum, writes P as bfloat16 pairs
//     over the logits in tensor memory (tcgen05.st), and rescales O in tensor
//     memory only when its row max grows by more than 2^8 (the stale max
//     stays exact: the final o / l uses the same max for both); one eighth
//     of the exponentials run as a polynomial on the FMA pipe, the scaling,
//     row sums and polynomial in paired (.f32x2) instructions;
//   * the issue order per KV tile j is PV_0(j-1), S_0(j), PV_1(j-1), S_1(j):
//     the commit that publishes S_t(j) also covers PV_t(j-1), so a softmax
//     warpgroup that sees S_t(j) may rescale O_t and overwrite P_t, and
//     tensor-core operations of one thread run in issue order, so S_t(j+1)
//     overwrites P_t(j) only after PV_t(j) has read it.
// Every mbarrier wait is bounded; a wait that gives up sets g_prefill_status
// and an abort flag so that all warps leave their loops and the CTA frees its
// tensor memory.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "oc_common.cuh"
#include "oc_mma.cuh"
#include "oc_tma.cuh"
#include "oc_tcgen05.cuh"

namespace oc {

__device__ int g_prefill_status = 0;

namespace {

constexpr int kPfRows = 128;        // query rows per tile (UMMA M)
constexpr int kPfTok = 128;         // tokens per K/V tile (UMMA N of QK^T, K of PV)
constexpr int kPfD = 128;           // head_dim
constexpr int kPfSlots = 5;         // K/V ring slots
constexpr int kPfTileBytes = kPfRows * kPfD * 2;  // 32 KB, every tile in the kernel
constexpr int kPfBoxBytes = kPfTileBytes / 2;     // one 128 x 64 box
constexpr int kPfThreads = 320;
constexpr int kPfProducerWarp = 8;
constexpr int kPfMmaWarp = 9;
constexpr int kPfTmemCols = 512;

struct PfSmem {
  // tiles first, each 1024-byte aligned (the 128B swizzle repeats every 1024 B)
  unsigned char q[2][kPfTileBytes];
  unsigned char kv[kPfSlots][kPfTileBytes];
  uint64_t kv_full[kPfSlots], kv_empty[kPfSlots];
  uint64_t q_full, q_empty;
  uint64_t s_full[2], p_full[2], o_free[2];
  uint64_t drain;
  uint32_t tmem_base;
  int abort;
};
constexpr size_t kPfSmemBytes = sizeof(PfSmem) + 1024;  // + alignment slack

struct PfArgs {
  const int32_t* idx;
  const int32_t* count;
  void* out;
  int out_dtype;
  int B, Sq, Hq, Hkv, S, bs, max_blocks;
  int kv_rows;  // token rows of K / V per batch row (S; 0 for a page pool shared by the batch)
  int idx_stride, idx_hstride, count_stride, count_hstride;
  int G, nqt, tiles_per_head, npairs, units;
  float scale_log2;  // log2(e) / sqrt(D)
};

// ---- tcgen05 helpers (inline PTX, sm_100a) --------------------------------

// Instruction descriptor of kind::f16 for this kernel's M = 128, N = 128
// tiles (A K-major; B K-major for b_mn = 0, MN-major for b_mn = 1).
__host__ __device__ constexpr uint32_t idesc_bf16(int b_mn) { return tc_idesc_bf16(kPfRows, kPfTok, b_mn); }

// Paired fp32 arithmetic (sm_100a .f32x2 forms): one instruction for two
// lanes of a float2, halving the issue slots of the softmax's FMA work.
__device__ __forceinline__ uint64_t f2_pack(float a, float b) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ void f2_unpack(uint64_t r, float& a, float& b) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(r));
}
__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}
__device__ __forceinline__ uint64_t f2_add(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}

// 2^x for a pair of values on the FMA pipe, for the share of the
// exponentials taken off the MUFU unit.  x = n + f with n = floor(x) found
// without a conversion instruction (those issue on the same narrow pipe as
// MUFU): adding 1.5 * 2^23 with rounding toward -inf leaves floor(x) in the
// low mantissa bits of t, and bits(t) << 23 is exactly n << 23 modulo 2^32.
// 2^f on [0, 1) is the cubic through the four Chebyshev nodes of the
// interval (relative error < 1e-4, below the bfloat16 rounding that P
// gets); 2^n is added to the exponent field.  x is clamped to >= -126 so that
// the exponent field never wraps (the result there is ~1e-38, i.e. zero).
__device__ __forceinline__ void poly_ex2x2(float x0, float x1, float& y0, float& y1) {
  const uint64_t kMagic = f2_pack(12582912.f, 12582912.f);
  const uint64_t x = f2_pack(fmaxf(x0, -126.f), fmaxf(x1, -126.f));
  uint64_t t, n, f;
  asm("add.rm.f32x2 %0, %1, %2;" : "=l"(t) : "l"(x), "l"(kMagic));
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(n) : "l"(t), "l"(kMagic));
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(f) : "l"(x), "l"(n));
  uint64_t p = f2_fma(f2_pack(0.0789672570f, 0.0789672570f), f, f2_pack(0.2246931558f, 0.2246931558f));
  p = f2_fma(p, f, f2_pack(0.6963247711f, 0.6963247711f));
  p = f2_fma(p, f, f2_pack(0.9999002882f, 0.9999002882f));
  float p0, p1, t0, t1;
  f2_unpack(p, p0, p1);
  f2_unpack(t, t0, t1);
  y0 = __uint_as_float(__float_as_uint(t0) * (1u << 23) + __float_as_uint(p0));
  y1 = __uint_as_float(__float_as_uint(t1) * (1u << 23) + __float_as_uint(p1));
}

// Chunks of 8 exponentials per 64 that run as poly_ex2x2: one in eight.
// (Measured on config 2: shares of 0 and 1/8 are equally fast, 1/4 is 2 %
// slower, 3/8 and 1/2 slower still, so MUFU is not what bounds the kernel.)
__host__ __device__ constexpr bool poly_chunk(int c) { return c == 7; }

// Three-input maximum (one instruction on sm_100a).
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

__device__ __forceinline__ float fast_ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}


// ---- work decomposition ---------------------------------------------------

struct PfUnit {
  int b, h, n;        // batch row, KV head, K/V tiles to stream (count * bs / 128)
  int ntile;          // row tiles in this unit (1 or 2)
  int hq[2], q0[2];   // query head and first query position of each tile
  const int32_t* idx;
};

__device__ __forceinline__ PfUnit pf_unit(const PfArgs& a, int u) {
  PfUnit w;
  const int pair = u % a.npairs;
  const int bh = u / a.npairs;
  w.h = bh % a.Hkv;
  w.b = bh / a.Hkv;
  const int r0 = 2 * pair;
  w.ntile = (r0 + 1 < a.tiles_per_head) ? 2 : 1;
#pragma unroll
  for (int t = 0; t < 2; ++t) {
    const int r = r0 + t;  // row tile r: query head g = r % G of the group, position tile r / G
    w.hq[t] = w.h * a.G + r % a.G;
    w.q0[t] = (r / a.G) * kPfRows;
  }
  int c = a.count[(size_t)w.b * a.count_stride + (size_t)w.h * a.count_hstride];
  c = c < 0 ? 0 : (c > a.max_blocks ? a.max_blocks : c);
  w.n = c * (a.bs / kPfTok);
  w.idx = a.idx + (size_t)w.b * a.idx_stride + (size_t)w.h * a.idx_hstride;
  return w;
}

// First token (row of the (B*S, Hkv, D) view) of K/V tile j of a unit.
__device__ __forceinline__ int pf_token(const PfArgs& a, const PfUnit& w, int j) {
  const int tpb = a.bs / kPfTok;
  const int blk = w.idx[j / tpb];
  return w.b * a.kv_rows + blk * a.bs + (j % tpb) * kPfTok;
}

__device__ __forceinline__ bool pf_wait(PfSmem& sm, uint64_t* bar, uint32_t parity) {
  if (mbar_wait(bar, parity)) return true;
  atomicExch(&g_prefill_status, 1);
  *(volatile int*)&sm.abort = 1;
  return false;
}
__device__ __forceinline__ bool pf_aborted(PfSmem& sm) { return *(volatile int*)&sm.abort != 0; }

// Store one finished output row (128 channels) of this thread.
template <typename TO>
__device__ __forceinline__ void pf_store_row(TO* dst, const float* v, float inv_l);
template <>
__device__ __forceinline__ void pf_store_row<__nv_bfloat16>(__nv_bfloat16* dst, const float* v, float inv_l) {
  uint4* d = reinterpret_cast<uint4*>(dst);
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    uint4 w;
    w.x = pack_bf16x2(v[8 * c + 0] * inv_l, v[8 * c + 1] * inv_l);
    w.y = pack_bf16x2(v[8 * c + 2] * inv_l, v[8 * c + 3] * inv_l);
    w.z = pack_bf16x2(v[8 * c + 4] * inv_l, v[8 * c + 5] * inv_l);
    w.w = pack_bf16x2(v[8 * c + 6] * inv_l, v[8 * c + 7] * inv_l);
    d[c] = w;
  }
}
template <>
__device__ __forceinline__ void pf_store_row<float>(float* dst, const float* v, float inv_l) {
  float4* d = reinterpret_cast<float4*>(dst);
#pragma unroll
  for (int c = 0; c < 8; ++c)
    d[c] = make_float4(v[4 * c] * inv_l, v[4 * c + 1] * inv_l, v[4 * c + 2] * inv_l, v[4 * c + 3] * inv_l);
}

template <typename TO>
__device__ void pf_softmax(PfSmem& sm, const PfArgs& a, int t, uint32_t tmem) {
  const int row = threadIdx.x & 127;           // query row of the tile == TMEM lane
  const int warp_lane0 = (threadIdx.x & 96);   // first TMEM lane of this warp
  const uint32_t t_s = tmem + ((uint32_t)warp_lane0 << 16) + t * 256;
  const uint32_t t_o = t_s + 128;
  uint32_t s_ph = 0;
  for (int u = blockIdx.x; u < a.units; u += gridDim.x) {
    const PfUnit w = pf_unit(a, u);
    if (t >= w.ntile) continue;
    const int qpos = (t ? w.q0[1] : w.q0[0]) + row;
    const int hq = t ? w.hq[1] : w.hq[0];
    TO* orow = reinterpret_cast<TO*>(a.out) + (((size_t)w.b * a.Sq + qpos) * a.Hq + hq) * kPfD;
    if (w.n == 0) {
      if (qpos < a.Sq) {
        float z[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) z[i] = 0.f;
#pragma unroll
        for (int c = 0; c < 4; ++c) pf_store_row<TO>(orow + 32 * c, z, 0.f);
      }
      continue;
    }
    float m_used = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < w.n; ++j) {
      if (pf_aborted(sm) || !pf_wait(sm, &sm.s_full[t], s_ph)) { ok = false; break; }
      s_ph ^= 1;
      tc_fence_after();
      // Row max over the 128 logits in two halves of 64 columns (the register
      // budget is that of 3 warps per SM sub-partition, 168 registers); the
      // first half (read second) stays in registers for its exponentials, the
      // other is read again.
      float s[64];
      tmem_ld64_wait(t_s + 64, s);
      // Eight independent running maxima (a single chain of 128 dependent
      // max operations would sit on the critical path of every K/V tile).
      float m8[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        m8[k] = fmax3(s[k], s[8 + k], s[16 + k]);
        m8[k] = fmax3(m8[k], s[24 + k], s[32 + k]);
        m8[k] = fmax3(m8[k], s[40 + k], s[48 + k]);
        m8[k] = fmaxf(m8[k], s[56 + k]);
      }
      tmem_ld64_wait(t_s, s);
#pragma unroll
      for (int i = 0; i < 64; i += 16)
#pragma unroll
        for (int k = 0; k < 8; ++k) m8[k] = fmax3(m8[k], s[i + k], s[i + 8 + k]);
      float mx = fmaxf(fmaxf(fmaxf(m8[0], m8[1]), fmaxf(m8[2], m8[3])), fmaxf(fmaxf(m8[4], m8[5]), fmaxf(m8[6], m8[7])));
      mx *= a.scale_log2;
      const bool need = mx > m_used + 8.f;
      if (__any_sync(0xffffffffu, need)) {
        const float m_new = need ? mx : m_used;
        const float alpha = fast_ex2(m_used - m_new);  // 0 on the first tile (m_used = -inf)
        if (j > 0) {
#pragma unroll 1
          for (int c = 0; c < 4; ++c) {
            float o[32];
            tmem_ld32_wait(t_o + 32 * c, o);
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] *= alpha;
            tmem_st32(t_o + 32 * c, o);
          }
        }
        l *= alpha;
        m_used = m_new;
      }
      // P = exp2(s * scale - m) as bfloat16 pairs written over S in tensor
      // memory (column c holds tokens 2c, 2c + 1), the A operand of P.V.
      // Tokens 0-63 go to columns 0-31, whose logits are already in
      // registers; tokens 64-127 to columns 32-63, after their logits (columns
      // 64-127, untouched so far) have been read.  One chunk of 8 in 8 takes
      // its exponentials on the FMA pipe.  Independent partial sums (as for
      // the max), four float2 pairs.
      uint64_t r2[4] = {0, 0, 0, 0};
      const uint64_t sc2 = f2_pack(a.scale_log2, a.scale_log2), nm2 = f2_pack(-m_used, -m_used);
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        if (half == 1) tmem_ld64_wait(t_s + 64, s);
        uint32_t pk[32];
#pragma unroll
        for (int c = 0; c < 8; ++c) {
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            float x0, x1, p0, p1;
            f2_unpack(f2_fma(f2_pack(s[8 * c + 2 * i], s[8 * c + 2 * i + 1]), sc2, nm2), x0, x1);
            if (poly_chunk(c)) {
              poly_ex2x2(x0, x1, p0, p1);
            } else {
              p0 = fast_ex2(x0);
              p1 = fast_ex2(x1);
            }
            r2[i] = f2_add(r2[i], f2_pack(p0, p1));
            pk[4 * c + i] = pack_bf16x2(p0, p1);
          }
        }
        tmem_st32u(t_s + 32 * half, pk);
      }
      tc_wait_st();  // P and any rescaled O are in tensor memory
      {
        float r[8];
#pragma unroll
        for (int i = 0; i < 4; ++i) f2_unpack(r2[i], r[2 * i], r[2 * i + 1]);
        l += ((r[0] + r[1]) + (r[2] + r[3])) + ((r[4] + r[5]) + (r[6] + r[7]));
      }
      tc_fence_before();
      mbar_arrive(&sm.p_full[t]);
    }
    if (!ok) break;
    // the last commit of the unit covers the final PV: O is complete
    if (pf_aborted(sm) || !pf_wait(sm, &sm.s_full[t], s_ph)) break;
    s_ph ^= 1;
    tc_fence_after();
    const float inv_l = 1.f / l;
#pragma unroll 1
    for (int c = 0; c < 4; ++c) {
      float o[32];
      tmem_ld32_wait(t_o + 32 * c, o);
      if (qpos < a.Sq) pf_store_row<TO>(orow + 32 * c, o, inv_l);
    }
    // O of this tile is read: the next unit's first S_t may be committed
    // (without this hand-over two phases of s_full[t] could complete between
    // two polls of this warpgroup).
    tc_fence_before();
    mbar_arrive(&sm.o_free[t]);
  }
}

__device__ void pf_producer(PfSmem& sm, const PfArgs& a, const CUtensorMap* mq, const CUtensorMap* mk,
                            const CUtensorMap* mv) {
  uint32_t q_ph = 0;
  uint32_t L = 0;  // running K/V load index: slot L % kPfSlots, use L / kPfSlots
  for (int u = blockIdx.x; u < a.units; u += gridDim.x) {
    const PfUnit w = pf_unit(a, u);
    if (w.n == 0) continue;
    if (pf_aborted(sm) || !pf_wait(sm, &sm.q_empty, q_ph ^ 1)) return;
    q_ph ^= 1;
    mbar_expect_tx(&sm.q_full, (uint32_t)(w.ntile * kPfTileBytes));
#pragma unroll
    for (int t = 0; t < 2; ++t) {
      if (t < w.ntile) {
        const int y = w.hq[t], z = w.b * a.Sq + w.q0[t];
        tma_load_3d(sm.q[t], mq, &sm.q_full, 0, y, z);
        tma_load_3d(sm.q[t] + kPfBoxBytes, mq, &sm.q_full, 64, y, z);
      }
    }
    for (int j = 0; j < w.n; ++j) {
      const int tok = pf_token(a, w, j);
#pragma unroll
      for (int kv = 0; kv < 2; ++kv, ++L) {
        const uint32_t slot = L % kPfSlots, use = L / kPfSlots;
        if (pf_aborted(sm) || !pf_wait(sm, &sm.kv_empty[slot], (use & 1) ^ 1)) return;
        mbar_expect_tx(&sm.kv_full[slot], kPfTileBytes);
        const CUtensorMap* m = kv ? mv : mk;
        tma_load_3d(sm.kv[slot], m, &sm.kv_full[slot], 0, w.h, tok);
        tma_load_3d(sm.kv[slot] + kPfBoxBytes, m, &sm.kv_full[slot], 64, w.h, tok);
      }
    }
  }
}

__device__ void pf_mma(PfSmem& sm, const PfArgs& a, uint32_t tmem) {
  constexpr uint32_t kIdQK = idesc_bf16(0), kIdPV = idesc_bf16(1);
  uint32_t q_ph = 0, p_ph = 0, o_ph = 0;  // bit t: phase of p_full[t] / o_free[t]
  uint32_t L = 0;
  for (int u = blockIdx.x; u < a.units; u += gridDim.x) {
    const PfUnit w = pf_unit(a, u);
    if (w.n == 0) continue;
    if (pf_aborted(sm) || !pf_wait(sm, &sm.q_full, q_ph)) return;
    q_ph ^= 1;
    tc_fence_after();
    uint32_t vslot_prev = 0;
    for (int j = 0; j <= w.n; ++j) {
      uint32_t kslot = 0;
      if (j < w.n) {
        kslot = L % kPfSlots;
        if (pf_aborted(sm) || !pf_wait(sm, &sm.kv_full[kslot], (L / kPfSlots) & 1)) return;
        tc_fence_after();
      }
      if (j > 0) {  // V_{j-1} is load L - 1
        if (pf_aborted(sm) || !pf_wait(sm, &sm.kv_full[vslot_prev], ((L - 1) / kPfSlots) & 1)) return;
        tc_fence_after();
      }
#pragma unroll
      for (int t = 0; t < 2; ++t) {
        if (t >= w.ntile) break;
        const uint32_t d_s = tmem + t * 256, d_o = d_s + 128;
        const uint32_t qa = smem_u32(sm.q[t]);
        if (j > 0) {
          if (pf_aborted(sm) || !pf_wait(sm, &sm.p_full[t], (p_ph >> t) & 1)) return;
          p_ph ^= 1u << t;
          tc_fence_after();
          const uint32_t vb = smem_u32(sm.kv[vslot_prev]);
#pragma unroll
          for (int kk = 0; kk < 8; ++kk) {
            const uint64_t bd = sdesc(vb + kk * 2048, kPfBoxBytes, 1024);
            umma_bf16_ts(d_o, d_s + kk * 8, bd, kIdPV, (j > 1 || kk > 0) ? 1 : 0);
          }
          if (t == w.ntile - 1) umma_commit(&sm.kv_empty[vslot_prev]);
        }
        if (j == 0) {  // the softmax warpgroup has read the previous unit's O_t
          if (pf_aborted(sm) || !pf_wait(sm, &sm.o_free[t], ((o_ph >> t) & 1) ^ 1)) return;
          o_ph ^= 1u << t;
          tc_fence_after();
        }
        if (j < w.n) {
          const uint32_t kb = smem_u32(sm.kv[kslot]);
#pragma unroll
          for (int kk = 0; kk < 8; ++kk) {
            const uint64_t ad = sdesc(qa + (kk >> 2) * kPfBoxBytes + (kk & 3) * 32, 16, 1024);
            const uint64_t bd = sdesc(kb + (kk >> 2) * kPfBoxBytes + (kk & 3) * 32, 16, 1024);
            umma_bf16(d_s, ad, bd, kIdQK, kk > 0 ? 1 : 0);
          }
        }
        umma_commit(&sm.s_full[t]);
        if (j < w.n && t == w.ntile - 1) {
          umma_commit(&sm.kv_empty[kslot]);
          if (j == w.n - 1) umma_commit(&sm.q_empty);
        }
      }
      if (j < w.n) {
        vslot_prev = (L + 1) % kPfSlots;
        L += 2;
      }
    }
  }
}

template <typename TO>
__global__ void __launch_bounds__(kPfThreads, 1)
    prefill_attn_kernel(const __grid_constant__ CUtensorMap mq, const __grid_constant__ CUtensorMap mk,
                        const __grid_constant__ CUtensorMap mv, const PfArgs a) {
  extern __shared__ unsigned char pf_raw[];
  PfSmem& sm = *reinterpret_cast<PfSmem*>((reinterpret_cast<uintptr_t>(pf_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5;
  if (threadIdx.x == 0) {
    for (int i = 0; i < kPfSlots; ++i) {
      mbar_init(&sm.kv_full[i], 1);
      mbar_init(&sm.kv_empty[i], 1);
    }
    mbar_init(&sm.q_full, 1);
    mbar_init(&sm.q_empty, 1);
    for (int t = 0; t < 2; ++t) {
      mbar_init(&sm.s_full[t], 1);
      mbar_init(&sm.p_full[t], 128);
      mbar_init(&sm.o_free[t], 128);
    }
    mbar_init(&sm.drain, 1);
    sm.abort = 0;
    fence_mbar_init();
  }
  if (warp == kPfMmaWarp) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&sm.tmem_base)),
                 "r"(kPfTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sm.tmem_base;

  if (warp < 8) {
    pf_softmax<TO>(sm, a, warp >> 2, tmem);
  } else if (warp == kPfProducerWarp) {
    if ((threadIdx.x & 31) == 0) pf_producer(sm, a, &mq, &mk, &mv);
  } else {
    if ((threadIdx.x & 31) == 0) {
      pf_mma(sm, a, tmem);
      // wait (bounded) for every MMA still in flight before the memory is freed
      umma_commit(&sm.drain);
      if (!mbar_wait(&sm.drain, 0)) atomicExch(&g_prefill_status, 1);
    }
    __syncwarp();
  }
  tc_fence_before();
  __syncthreads();
  if (warp == kPfMmaWarp) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kPfTmemCols) : "memory");
  }
}

int pf_map(CUtensorMap* m, const void* base, int inner_heads, int64_t rows, const char* what) {
  const uint64_t dims[3] = {(uint64_t)kPfD, (uint64_t)inner_heads, (uint64_t)rows};
  const uint64_t strides[2] = {(uint64_t)kPfD * 2, (uint64_t)inner_heads * kPfD * 2};
  const uint32_t box[3] = {64, 1, (uint32_t)kPfRows};
  const uint64_t key[4] = {3, (uint64_t)base, (uint64_t)inner_heads, (uint64_t)rows};
  if (map_cache_get(key, m)) return OC_OK;
  const int r = encode_map_3d(m, base, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, dims, strides, box, true);
  if (r) return set_error(OC_ERR_CUDA, "oc_prefill_attention: tensor map for %s failed (CUresult %d)", what, r);
  map_cache_put(key, *m);
  return OC_OK;
}

}  // namespace

int wait_limit_prefill(unsigned long long ns) { return set_wait_limit_here(ns); }
int prefill_status(int* status, int reset) {
  cudaError_t e = cudaMemcpyFromSymbol(status, g_prefill_status, sizeof(int));
  if (e != cudaSuccess) return set_error(OC_ERR_CUDA, "oc_device_status: %s", cudaGetErrorString(e));
  if (reset) {
    const int zero = 0;
    e = cudaMemcpyToSymbol(g_prefill_status, &zero, sizeof(int));
    if (e != cudaSuccess) return set_error(OC_ERR_CUDA, "oc_device_status: %s", cudaGetErrorString(e));
  }
  return OC_OK;
}

}  // namespace oc

using namespace oc;

namespace {
// pool_pages > 0: k / v are a pool of pool_pages blocks shared by the batch
// and idx holds pool pages; seq_len is then the logical capacity.
int prefill_impl(const void* q, const void* k, const void* v, int dtype, const int32_t* idx, int idx_stride,
                 int idx_head_stride, const int32_t* count, int count_stride, int count_head_stride, int batch,
                 int q_len, int q_heads, int kv_heads, int head_dim, int seq_len, int block_size, int max_blocks,
                 void* out, int out_dtype, oc_stream_t stream, int pool_pages) {
  OC_REQUIRE(q && k && v && idx && count && out, OC_ERR_NULL, "oc_prefill_attention: NULL pointer");
  OC_REQUIRE(dtype == OC_BF16, OC_ERR_DTYPE, "oc_prefill_attention: inputs must be bfloat16");
  OC_REQUIRE(out_dtype == OC_BF16 || out_dtype == OC_F32, OC_ERR_DTYPE, "oc_prefill_attention: bad out dtype");
  OC_REQUIRE(head_dim == kPfD, OC_ERR_SHAPE, "oc_prefill_attention: head_dim must be 128");
  OC_REQUIRE(batch >= 1 && q_len >= 1 && kv_heads >= 1 && q_heads >= kv_heads && q_heads % kv_heads == 0,
             OC_ERR_SHAPE, "oc_prefill_attention: bad batch / heads");
  OC_REQUIRE(block_size >= kPfTok && block_size % kPfTok == 0, OC_ERR_SHAPE,
             "oc_prefill_attention: block_size must be a multiple of 128");
  OC_REQUIRE(seq_len >= block_size && seq_len % block_size == 0, OC_ERR_SHAPE,
             "oc_prefill_attention: seq_len must be a multiple of block_size");
  OC_REQUIRE(max_blocks >= 0 && max_blocks <= seq_len / block_size, OC_ERR_SHAPE,
             "oc_prefill_attention: max_blocks out of range");
  OC_REQUIRE(idx_stride >= 0 && idx_head_stride >= 0 && count_stride >= 0 && count_head_stride >= 0, OC_ERR_SHAPE,
             "oc_prefill_attention: negative stride");
  OC_REQUIRE(aligned16(q) && aligned16(k) && aligned16(v) && aligned16(out), OC_ERR_ALIGN,
             "oc_prefill_attention: q/k/v/out must be 16-byte aligned");
  OC_REQUIRE((int64_t)batch * seq_len < INT32_MAX && (int64_t)batch * q_len < INT32_MAX, OC_ERR_SHAPE,
             "oc_prefill_attention: too many rows");

  PfArgs a;
  a.idx = idx;
  a.count = count;
  a.out = out;
  a.out_dtype = out_dtype;
  a.B = batch;
  a.Sq = q_len;
  a.Hq = q_heads;
  a.Hkv = kv_heads;
  a.S = seq_len;
  a.kv_rows = pool_pages > 0 ? 0 : seq_len;
  a.bs = block_size;
  a.max_blocks = max_blocks;
  a.idx_stride = idx_stride;
  a.idx_hstride = idx_head_stride;
  a.count_stride = count_stride;
  a.count_hstride = count_head_stride;
  a.G = q_heads / kv_heads;
  a.nqt = (q_len + kPfRows - 1) / kPfRows;
  a.tiles_per_head = a.G * a.nqt;
  a.npairs = (a.tiles_per_head + 1) / 2;
  const int64_t units = (int64_t)batch * kv_heads * a.npairs;
  OC_REQUIRE(units < INT32_MAX, OC_ERR_SHAPE, "oc_prefill_attention: too many work units");
  a.units = (int)units;
  a.scale_log2 = 1.4426950408889634f / sqrtf((float)head_dim);

  CUtensorMap mq, mk, mv;
  int rc = pf_map(&mq, q, q_heads, (int64_t)batch * q_len, "q");
  const int64_t kv_total = pool_pages > 0 ? (int64_t)pool_pages * block_size : (int64_t)batch * seq_len;
  if (!rc) rc = pf_map(&mk, k, kv_heads, kv_total, "k");
  if (!rc) rc = pf_map(&mv, v, kv_heads, kv_total, "v");
  if (rc) return rc;

  auto kern = out_dtype == OC_BF16 ? prefill_attn_kernel<__nv_bfloat16> : prefill_attn_kernel<float>;
  static std::atomic<uint64_t> s_setup[2] = {{0}, {0}};
  if (first_on_device(s_setup[out_dtype == OC_BF16])) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kPfSmemBytes);
    if (e != cudaSuccess) return set_error(OC_ERR_CUDA, "oc_prefill_attention: %s", cudaGetErrorString(e));
  }
  const int sms = device_sm_count();
  const int grid = (int)(units < sms ? units : sms);
  kern<<<grid, kPfThreads, kPfSmemBytes, reinterpret_cast<cudaStream_t>(stream)>>>(mq, mk, mv, a);
  return check_launch("prefill_attn_kernel");
}
}  // namespace

extern "C" int oc_prefill_attention(const void* q, const void* k, const void* v, int dtype,
                                    const int32_t* idx, int idx_stride, int idx_head_stride,
                                    const int32_t* count, int count_stride, int count_head_stride,
                                    int batch, int q_len, int q_heads, int kv_heads, int head_dim,
                                    int seq_len, int block_size, int max_blocks,
                                    void* out, int out_dtype, oc_stream_t stream) {
  return prefill_impl(q, k, v, dtype, idx, idx_stride, idx_head_stride, count, count_stride, count_head_stride, batch,
                      q_len, q_heads, kv_heads, head_dim, seq_len, block_size, max_blocks, out, out_dtype, stream, 0);
}

extern "C" size_t oc_prefill_attention_paged_workspace_bytes(int batch, int max_blocks) {
  if (batch < 1 || max_blocks < 0) return 0;
  return ((size_t)batch * max_blocks * sizeof(int32_t) + 255) / 256 * 256;
}

extern "C" int oc_prefill_attention_paged(const void* q, const void* k_pool, const void* v_pool, int dtype,
                                          const int32_t* block_table, int table_stride, const int32_t* idx,
                                          int idx_stride, const int32_t* count, int count_stride, int batch,
                                          int q_len, int q_heads, int kv_heads, int head_dim, int num_pages,
                                          int block_size, int max_blocks, void* out, int out_dtype, void* workspace,
                                          size_t workspace_bytes, oc_stream_t stream) {
  OC_REQUIRE(block_table && idx && count && workspace, OC_ERR_NULL, "oc_prefill_attention_paged: NULL pointer");
  OC_REQUIRE(num_pages >= 1 && table_stride >= 1 && max_blocks >= 0 && max_blocks <= table_stride && batch >= 1,
             OC_ERR_SHAPE, "oc_prefill_attention_paged: num_pages %d, table_stride %d, max_blocks %d", num_pages,
             table_stride, max_blocks);
  OC_REQUIRE((int64_t)num_pages * block_size < INT32_MAX, OC_ERR_SHAPE, "oc_prefill_attention_paged: pool too large");
  const size_t need = oc_prefill_attention_paged_workspace_bytes(batch, max_blocks);
  OC_REQUIRE(workspace_bytes >= need, OC_ERR_CAPACITY, "oc_prefill_attention_paged: workspace %zu < %zu bytes",
             workspace_bytes, need);
  int32_t* phys = static_cast<int32_t*>(workspace);
  int rc = compose_page_lists(block_table, table_stride, table_stride, idx, idx_stride, count, count_stride, batch,
                              max_blocks, num_pages, phys, reinterpret_cast<cudaStream_t>(stream));
  if (rc) return rc;
  return prefill_impl(q, k_pool, v_pool, dtype, phys, max_blocks, 0, count, count_stride, 0, batch, q_len, q_heads,
                      kv_heads, head_dim, table_stride * block_size, block_size, max_blocks, out, out_dtype, stream,
                      num_pages);
}

