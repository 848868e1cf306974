// Exact block-gated attention backward on the 5th-generation tensor cores.
//
// Two owner kernels, no floating atomics (deterministic):
//   dQ  kernel: CTA = 128 query rows; per key tile S = Q K^T and dP = dO V^T
//               (tcgen05, TMEM), the gate-aware dA per score, then
//               dQ += dA K with dA read straight from TMEM.
//   dKV kernel: CTA = 128 keys; per query tile the same S / dP / dA, with P
//               and dA written to shared memory (128-byte swizzle) so that
//               dV += P^T dO and dK += dA^T Q run as tcgen05 MMAs whose A
//               operand is MN-major.
// A prologue kernel computes delta = dO.O and rho = dO.RC - delta * PR per
// row and the per-128-row position bounds used to skip invisible tiles.
//
// Per score (base-2 logits a, block log-mass s_b, e = 2^(a - blockmax)):
//   p      = e * 2^(blockmax + s_b - zr - L)      (remote block)
//          = e * 2^(blockmax - L)                 (local key)
//   direct = p * (dP - delta)
//   dA     = direct + e * (2^(blockmax - s_b) * sum_block(direct)
//                          - 2^(blockmax - zr) * rho)   (remote only)
// scaled by the softmax scale. Blocks of up to 32 keys are finished inside a
// 32-column chunk in one pass (one exp2 per score); 64/128-key blocks use a
// three-pass scheme over TMEM (three exp2 per score).
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "../common/sm100.cuh"
#include "../common/tma.cuh"
#include "gated_common.cuh"
#include "gated_noalloc.h"

#include <cstdio>
#include <mutex>

namespace eb {
namespace {

using namespace sm100;

constexpr int kT = 128;            // rows (queries or keys) per CTA and per tile
constexpr int kTmemCols = 512;
constexpr float kLog2e = 1.4426950408889634f;

struct BwdParams {
  const int* pos;        // [B, Q]
  const float* lse;      // [B, Q, H] natural log
  const float* zr;       // [B, Q, H]
  const float* delta;    // [B, Q, H]
  const float* rho;      // [B, Q, H]
  const int* bounds;     // [B, q_tiles, 3]: max_pos, remote_end, local_start
  __nv_bfloat16* dq;
  __nv_bfloat16* dk;
  __nv_bfloat16* dv;
  ErrorSlot* err;
  int queries, keys, heads, q_tiles;
  float scale, scale_log2;
};

// ---------------------------------------------------------------------------
// prologue
// ---------------------------------------------------------------------------

__global__ void __launch_bounds__(256)
delta_rho_kernel(const __nv_bfloat16* __restrict__ dout, const __nv_bfloat16* __restrict__ out,
                 const float* __restrict__ rc, const float* __restrict__ pr, float* __restrict__ delta,
                 float* __restrict__ rho, int64_t rows, int dim) {
  const int64_t row = blockIdx.x * 8LL + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  float d = 0.f, r = 0.f;
  for (int i = lane; i < dim; i += 32) {
    const float g = __bfloat162float(dout[row * dim + i]);
    d += g * __bfloat162float(out[row * dim + i]);
    r += g * rc[row * dim + i];
  }
  d = warp_sum(d);
  r = warp_sum(r);
  if (lane == 0) {
    delta[row] = d;
    rho[row] = r - d * pr[row];
  }
}

template <int B>
__global__ void __launch_bounds__(kT)
tile_bounds_kernel(const int* __restrict__ pos, int* __restrict__ bounds, int queries, int q_tiles) {
  __shared__ int red[3][4];
  const int tile = blockIdx.x, batch = blockIdx.y;
  const int q = tile * kT + threadIdx.x;
  int p = q < queries ? pos[static_cast<int64_t>(batch) * queries + q] : -1;
  int mx = p, re = 0, ls = 1 << 30;
  if (p >= 0) {
    const int first_local = (p / B - 1) * B;
    re = max(0, first_local);
    ls = max(0, first_local);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    mx = max(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    re = max(re, __shfl_xor_sync(0xffffffffu, re, o));
    ls = min(ls, __shfl_xor_sync(0xffffffffu, ls, o));
  }
  if ((threadIdx.x & 31) == 0) {
    red[0][threadIdx.x >> 5] = mx;
    red[1][threadIdx.x >> 5] = re;
    red[2][threadIdx.x >> 5] = ls;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int* out = bounds + (static_cast<int64_t>(batch) * q_tiles + tile) * 3;
    out[0] = max(max(red[0][0], red[0][1]), max(red[0][2], red[0][3]));
    out[1] = max(max(red[1][0], red[1][1]), max(red[1][2], red[1][3]));
    out[2] = min(min(red[2][0], red[2][1]), min(red[2][2], red[2][3]));
  }
}

// ---------------------------------------------------------------------------
// per-row gradient engine (thread = query row, 128 keys of one tile)
// ---------------------------------------------------------------------------

struct RowStats {
  int pos, first_local, pb;
  float lse2, zr2, delta, rho;
};

EB_DEVICE void load_row32(uint32_t addr, float (&x)[32]) {
  uint32_t r[32];
  tmem_ld32(addr, r);
  tc_wait_ld();
#pragma unroll
  for (int i = 0; i < 32; ++i) x[i] = __uint_as_float(r[i]);
}

// Calls sink(c0, p[32], da[32]) for c0 = 0, 32, 64, 96. `fast`: every key of
// the tile is an in-range remote key for every live row of the CTA (no masks,
// finite scores), so the block log-masses come from raw scores with the scale
// folded into one FFMA per exponent and no local terms exist.
template <int B, typename Sink>
EB_DEVICE void grad_row(uint32_t s_addr, uint32_t dp_addr, int k0, int keys, const RowStats& st,
                        float scale_log2, float scale, bool fast, int c_begin, int c_end, Sink&& sink) {
  const bool live = st.pos >= 0;
  if constexpr (B <= 32) {
    constexpr int kSeg = 32 / B;
    if (fast) {
#pragma unroll 1
      for (int c0 = c_begin; c0 < c_end; c0 += 32) {
        float a[32], dp[32], p[32], da[32];
        load_row32(s_addr + c0, a);
        load_row32(dp_addr + c0, dp);
#pragma unroll
        for (int g = 0; g < kSeg; ++g) {
          float m = a[g * B];
#pragma unroll
          for (int i = 1; i < B; ++i) m = fmaxf(m, a[g * B + i]);
          const float ms = m * scale_log2;
          float sum = 0.f;
#pragma unroll
          for (int i = 0; i < B; ++i) {
            const float e = ex2(fmaf(a[g * B + i], scale_log2, -ms));
            a[g * B + i] = e;
            sum += e;
          }
          const float sb = ms + lg2(sum);
          const float f = live ? ex2(ms + sb - st.zr2 - st.lse2) : 0.f;
          float rb = 0.f;
#pragma unroll
          for (int i = 0; i < B; ++i) {
            const float pv = a[g * B + i] * f;
            const float direct = pv * (dp[g * B + i] - st.delta);
            p[g * B + i] = pv;
            da[g * B + i] = direct;
            rb += direct;
          }
          const float gate = live ? ex2(ms - sb) * rb - ex2(ms - st.zr2) * st.rho : 0.f;
#pragma unroll
          for (int i = 0; i < B; ++i) da[g * B + i] = (da[g * B + i] + a[g * B + i] * gate) * scale;
        }
        sink(c0, p, da);
      }
      return;
    }
#pragma unroll 1
    for (int c0 = c_begin; c0 < c_end; c0 += 32) {
      float a[32], dp[32], p[32], da[32];
      load_row32(s_addr + c0, a);
      load_row32(dp_addr + c0, dp);
#pragma unroll
      for (int i = 0; i < 32; ++i) a[i] = (k0 + c0 + i < keys) ? a[i] * scale_log2 : kNegInf;
#pragma unroll
      for (int g = 0; g < kSeg; ++g) {
        float m = kNegInf;
#pragma unroll
        for (int i = 0; i < B; ++i) m = fmaxf(m, a[g * B + i]);
        float sum = 0.f;
#pragma unroll
        for (int i = 0; i < B; ++i) {
          const float e = m == kNegInf ? 0.f : ex2(a[g * B + i] - m);
          p[g * B + i] = e;          // e for now
          sum += e;
        }
        const float sb = m == kNegInf ? kNegInf : m + lg2(sum);
        const int block = (k0 + c0) / B + g;
        const bool remote = live && block < st.pb - 1 && m != kNegInf;
        const float f = remote ? ex2(m + sb - st.zr2 - st.lse2) : (m == kNegInf ? 0.f : ex2(m - st.lse2));
        float rb = 0.f;
#pragma unroll
        for (int i = 0; i < B; ++i) {
          const int key = k0 + c0 + g * B + i;
          const bool local = live && key >= st.first_local && key <= st.pos && key < keys;
          const float e = p[g * B + i];
          const float pv = (remote || local) ? e * f : 0.f;
          const float direct = pv * (dp[g * B + i] - st.delta);
          p[g * B + i] = pv;
          da[g * B + i] = direct;
          rb += direct;
          dp[g * B + i] = e;         // keep e for the gate term
        }
        if (remote) {
          const float g1 = ex2(m - sb) * rb, g2 = ex2(m - st.zr2) * st.rho;
#pragma unroll
          for (int i = 0; i < B; ++i) da[g * B + i] += dp[g * B + i] * (g1 - g2);
        }
      }
#pragma unroll
      for (int i = 0; i < 32; ++i) da[i] *= scale;
      sink(c0, p, da);
    }
  } else {
    constexpr int kChunks = B / 32;             // chunks per block
    constexpr int kSeg = kT / B;                // blocks per tile
    float m[kSeg], sum[kSeg], sb[kSeg], rb[kSeg];
#pragma unroll
    for (int g = 0; g < kSeg; ++g) {
      m[g] = kNegInf;
      sum[g] = 0.f;
      rb[g] = 0.f;
    }
    // Pass A: online block max / mass.
#pragma unroll 1
    for (int c = c_begin / 32; c < c_end / 32; ++c) {
      float a[32];
      load_row32(s_addr + c * 32, a);
      const int g = c / kChunks;
      float cm = kNegInf;
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        a[i] = (k0 + c * 32 + i < keys) ? a[i] * scale_log2 : kNegInf;
        cm = fmaxf(cm, a[i]);
      }
      const float nm = fmaxf(m[g], cm);
      if (nm != kNegInf) {
        float s = m[g] == kNegInf ? 0.f : sum[g] * ex2(m[g] - nm);
#pragma unroll
        for (int i = 0; i < 32; ++i) s += ex2(a[i] - nm);
        sum[g] = s;
        m[g] = nm;
      }
    }
#pragma unroll
    for (int g = 0; g < kSeg; ++g) sb[g] = m[g] == kNegInf ? kNegInf : m[g] + lg2(sum[g]);
    auto probs = [&](int c, float (&a)[32], float (&dp)[32], float (&p)[32], float (&e)[32], bool& remote) {
      const int g = c / kChunks;
      const int block = (k0 + c * 32) / B;
      remote = live && block < st.pb - 1 && m[g] != kNegInf;
      const float f = remote ? ex2(m[g] + sb[g] - st.zr2 - st.lse2) : (m[g] == kNegInf ? 0.f : ex2(m[g] - st.lse2));
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const int key = k0 + c * 32 + i;
        const float x = key < keys ? a[i] * scale_log2 : kNegInf;
        const bool local = live && key >= st.first_local && key <= st.pos && key < keys;
        e[i] = m[g] == kNegInf ? 0.f : ex2(x - m[g]);
        p[i] = (remote || local) ? e[i] * f : 0.f;
      }
    };
    // Pass B: block sums of the direct term.
#pragma unroll 1
    for (int c = c_begin / 32; c < c_end / 32; ++c) {
      float a[32], dp[32], p[32], e[32];
      bool remote;
      load_row32(s_addr + c * 32, a);
      load_row32(dp_addr + c * 32, dp);
      probs(c, a, dp, p, e, remote);
      float s = 0.f;
#pragma unroll
      for (int i = 0; i < 32; ++i) s += p[i] * (dp[i] - st.delta);
      rb[c / kChunks] += s;
    }
    // Pass C: dA.
#pragma unroll 1
    for (int c = c_begin / 32; c < c_end / 32; ++c) {
      float a[32], dp[32], p[32], e[32], da[32];
      bool remote;
      load_row32(s_addr + c * 32, a);
      load_row32(dp_addr + c * 32, dp);
      probs(c, a, dp, p, e, remote);
      const int g = c / kChunks;
      const float g1 = remote ? ex2(m[g] - sb[g]) * rb[g] : 0.f;
      const float g2 = remote ? ex2(m[g] - st.zr2) * st.rho : 0.f;
#pragma unroll
      for (int i = 0; i < 32; ++i) da[i] = (p[i] * (dp[i] - st.delta) + e[i] * (g1 - g2)) * scale;
      sink(c * 32, p, da);
    }
  }
}

EB_DEVICE RowStats row_stats(const BwdParams& p, int batch, int head, int q) {
  RowStats st;
  if (q < p.queries) {
    const int64_t s = (static_cast<int64_t>(batch) * p.queries + q) * p.heads + head;
    st.pos = p.pos[static_cast<int64_t>(batch) * p.queries + q];
    const float l = p.lse[s], z = p.zr[s];
    st.lse2 = l == kNegInf ? 0.f : l * kLog2e;
    st.zr2 = z == kNegInf ? 0.f : z * kLog2e;
    st.delta = p.delta[s];
    st.rho = p.rho[s];
  } else {
    st.pos = -1;
    st.lse2 = st.zr2 = st.delta = st.rho = 0.f;
  }
  st.pb = st.pos >= 0 ? st.pos : 0;
  return st;
}

template <int B>
EB_DEVICE void finish_stats(RowStats& st) {
  st.pb = st.pos >= 0 ? st.pos / B : 0;
  st.first_local = (st.pb - 1) * B;
}

// ---------------------------------------------------------------------------
// dQ kernel
// ---------------------------------------------------------------------------

template <int D>
struct alignas(1024) DqSmem {
  // K/V ring depth: four stages at head dim 64 so that the loads of the next
  // tiles are in flight while a tile's MMAs and gradient arithmetic run; two
  // at head dim 128 (64 KB per stage).
  static constexpr int kStagesKV = D == 64 ? 4 : 2;
  __nv_bfloat16 q[kT * D];
  __nv_bfloat16 g[kT * D];
  __nv_bfloat16 k[kStagesKV][kT * D];
  __nv_bfloat16 v[kStagesKV][kT * D];
  uint64_t qg_full, kv_full[kStagesKV], kv_empty[kStagesKV], sdp_full, da_full, dq_done;
  uint32_t tmem_base;
  int abort;
};

// SPLIT = number of gradient warpgroups: with 2 (blocks of at most 64 keys)
// each warpgroup owns 64 of the 128 key columns of every tile, so a row's
// work is done by two threads at once; no value crosses the column halves.
constexpr int threads_for(int split) { return 128 + 128 * split; }

template <int D, int B, int SPLIT>
__global__ void __launch_bounds__(threads_for(SPLIT), 1)
gated_dq_tc_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tg,
                   const __grid_constant__ CUtensorMap tk, const __grid_constant__ CUtensorMap tv, BwdParams p) {
  extern __shared__ __align__(1024) uint8_t raw_smem[];
  DqSmem<D>& sm = *reinterpret_cast<DqSmem<D>*>(
      (reinterpret_cast<uintptr_t>(raw_smem) + 1023) & ~static_cast<uintptr_t>(1023));
  constexpr int kS = DqSmem<D>::kStagesKV;
  constexpr int kHalves = D / 64, kBox = 128 * 64;
  // dA (bf16) lives in its own TMEM columns when two warpgroups write it
  // concurrently (one warpgroup's dA may not overwrite the other's S).
  constexpr uint32_t kDaCol = SPLIT == 2 ? 384 : 0;
  const int q_tile = gridDim.x - 1 - blockIdx.x;
  const int head = blockIdx.y, batch = blockIdx.z;
  const int q0 = q_tile * kT;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  volatile int* abort = &sm.abort;
  if (threadIdx.x == 0) {
    mbar_init(&sm.qg_full, 1);
    for (int s = 0; s < kS; ++s) {
      mbar_init(&sm.kv_full[s], 1);
      mbar_init(&sm.kv_empty[s], 1);
    }
    mbar_init(&sm.sdp_full, 1);
    mbar_init(&sm.da_full, 128 * SPLIT);
    mbar_init(&sm.dq_done, 1);
    sm.abort = 0;
    fence_barrier_init();
  }
  if (warp == 2) tmem_alloc(&sm.tmem_base, kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sm.tmem_base;
  const int* bnd = p.bounds + (static_cast<int64_t>(batch) * p.q_tiles + q_tile) * 3;
  const int max_pos = bnd[0];
  const int limit = min(p.keys, max_pos + 1);
  const int tiles = limit > 0 ? (limit + kT - 1) / kT : 0;
  if (warp == 0) {
    if (lane == 0 && tiles > 0) {
      mbar_expect_tx(&sm.qg_full, 2 * kT * D * 2);
      for (int h = 0; h < kHalves; ++h) {
        tma_load_4d(sm.q + h * kBox, &tq, &sm.qg_full, h * 64, head, q0, batch);
        tma_load_4d(sm.g + h * kBox, &tg, &sm.qg_full, h * 64, head, q0, batch);
      }
      int issued = 0;
      for (int j = 0; j < tiles; ++j) {
        const int s = j % kS;
        if (j >= kS && !mbar_wait(&sm.kv_empty[s], ((j / kS) - 1) & 1, abort, p.err, kSiteKvEmpty)) break;
        mbar_expect_tx(&sm.kv_full[s], 2 * kT * D * 2);
        for (int h = 0; h < kHalves; ++h) {
          tma_load_4d(sm.k[s] + h * kBox, &tk, &sm.kv_full[s], h * 64, head, j * kT, batch);
          tma_load_4d(sm.v[s] + h * kBox, &tv, &sm.kv_full[s], h * 64, head, j * kT, batch);
        }
        ++issued;
      }
      if (*abort) {
        for (int j = max(0, issued - kS); j < issued; ++j)
          mbar_wait(&sm.kv_full[j % kS], (j / kS) & 1, abort, nullptr, kSiteDrain);
        mbar_wait(&sm.qg_full, 0, abort, nullptr, kSiteDrain);
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && tiles > 0) {
      const uint32_t id_s = idesc_bf16(kT, kT, false, false);
      const uint32_t id_dq = idesc_bf16(kT, D, false, true);
      const uint32_t q_addr = smem_u32(sm.q), g_addr = smem_u32(sm.g);
      bool ok = mbar_wait(&sm.qg_full, 0, abort, p.err, kSiteQFull);
      for (int j = 0; ok && j < tiles; ++j) {
        const int s = j % kS;
        if (!mbar_wait(&sm.kv_full[s], (j / kS) & 1, abort, p.err, kSiteKvFull)) break;
        tc_fence_after();
        const uint32_t k_addr = smem_u32(sm.k[s]), v_addr = smem_u32(sm.v[s]);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (kk / 4) * kBox * 2 + (kk % 4) * 32;
          mma_ss(tmem, smem_desc_sw128(q_addr + off, 16, 1024), smem_desc_sw128(k_addr + off, 16, 1024), id_s,
                 kk > 0);
          mma_ss(tmem + 128, smem_desc_sw128(g_addr + off, 16, 1024), smem_desc_sw128(v_addr + off, 16, 1024),
                 id_s, kk > 0);
        }
        tc_commit(&sm.sdp_full);
        if (!mbar_wait(&sm.da_full, j & 1, abort, p.err, kSitePFull)) break;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < kT / 16; ++kk)
          mma_ts(tmem + 256, tmem + kDaCol + kk * 8, smem_desc_sw128(k_addr + kk * 2048, kBox * 2, 1024), id_dq,
                 (j > 0 || kk > 0) ? 1u : 0u);
        tc_commit(&sm.kv_empty[s]);
        tc_commit(&sm.dq_done);
      }
    }
  } else if (warp >= 4) {
    const int wg = (warp - 4) >> 2;
    const int row = (threadIdx.x - 128) & (kT - 1);
    const uint32_t lane_addr = tmem + (static_cast<uint32_t>(((warp - 4) & 3) * 32) << 16);
    const int c_begin = SPLIT == 2 ? wg * 64 : 0, c_end = SPLIT == 2 ? c_begin + 64 : kT;
    RowStats st = row_stats(p, batch, head, q0 + row);
    finish_stats<B>(st);
    bool ok = true;
    for (int j = 0; j < tiles; ++j) {
      if (!__all_sync(0xffffffffu, mbar_wait(&sm.sdp_full, j & 1, abort, p.err, kSiteSFull))) {
        ok = false;
        break;
      }
      tc_fence_after();
      const bool fast = (j + 1) * kT <= bnd[2] && (j + 1) * kT <= p.keys;
      grad_row<B>(lane_addr, lane_addr + 128, j * kT, p.keys, st, p.scale_log2, p.scale, fast, c_begin, c_end,
                  [&](int c0, const float (&pv)[32], const float (&da)[32]) {
                    uint32_t packed[16];
#pragma unroll
                    for (int i = 0; i < 16; ++i) packed[i] = pack_bf16(da[2 * i], da[2 * i + 1]);
                    tmem_st16(lane_addr + kDaCol + c0 / 2, packed);
                  });
      tc_wait_st();
      tc_fence_before();
      mbar_arrive(&sm.da_full);
    }
    if (ok && tiles > 0) ok = mbar_wait(&sm.dq_done, (tiles - 1) & 1, abort, p.err, kSiteODone);
    // Warp-uniform from here on: tcgen05.ld is warp-collective.
    const bool have = __all_sync(0xffffffffu, ok) && tiles > 0;
    tc_fence_after();
    const int q = q0 + row;
    const bool write = q < p.queries;
    __nv_bfloat16* out = p.dq + ((static_cast<int64_t>(batch) * p.queries + (write ? q : 0)) * p.heads + head) * D;
    constexpr int kCols = SPLIT == 2 ? D / 2 : D;   // dQ columns stored by this warpgroup
#pragma unroll
    for (int cc = 0; cc < kCols; cc += 32) {
      const int c = (SPLIT == 2 ? wg * kCols : 0) + cc;
      float x[32];
      if (have) {
        load_row32(lane_addr + 256 + c, x);
      } else {
#pragma unroll
        for (int i = 0; i < 32; ++i) x[i] = 0.f;
      }
#pragma unroll
      for (int i = 0; i < 32; i += 8) {
        uint32_t packed[4];
#pragma unroll
        for (int t = 0; t < 4; ++t) packed[t] = pack_bf16(x[i + 2 * t], x[i + 2 * t + 1]);
        if (write) *reinterpret_cast<uint4*>(out + c + i) = make_uint4(packed[0], packed[1], packed[2], packed[3]);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// ---------------------------------------------------------------------------
// dK/dV kernel
// ---------------------------------------------------------------------------

// Query-side stages of the dK/dV kernel: Q, dO and the P / dA tiles written
// for the dV / dK MMAs are double-buffered when they fit (head dim 64: 224 KB
// of shared memory), so that the next query tile's loads and S / dP MMAs do
// not wait for the previous tile's dV / dK MMAs.
template <int D>
constexpr int dkv_stages() { return D <= 64 ? 2 : 1; }

template <int D>
struct alignas(1024) DkvSmem {
  static constexpr int kStagesQ = dkv_stages<D>();
  __nv_bfloat16 k[kT * D];
  __nv_bfloat16 v[kT * D];
  __nv_bfloat16 q[kStagesQ][kT * D];
  __nv_bfloat16 g[kStagesQ][kT * D];
  __nv_bfloat16 pt[kStagesQ][kT * kT];    // P as [query][key], two 64-key swizzled boxes
  __nv_bfloat16 dat[kStagesQ][kT * kT];   // dA, same layout
  uint64_t kv_full, qg_full[kStagesQ], qg_free[kStagesQ], sdp_full, pda_full, acc_done;
  uint32_t tmem_base;
  int abort;
};

// Byte offset of (row, 16-byte chunk) in a [128 rows x 64 bf16] 128B-swizzled box.
EB_DEVICE uint32_t sw128_offset(int row, int chunk) { return row * 128 + ((chunk ^ (row & 7)) << 4); }

template <int D, int B, int SPLIT>
__global__ void __launch_bounds__(threads_for(SPLIT), 1)
gated_dkv_tc_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tg,
                    const __grid_constant__ CUtensorMap tk, const __grid_constant__ CUtensorMap tv, BwdParams p) {
  extern __shared__ __align__(1024) uint8_t raw_smem[];
  DkvSmem<D>& sm = *reinterpret_cast<DkvSmem<D>*>(
      (reinterpret_cast<uintptr_t>(raw_smem) + 1023) & ~static_cast<uintptr_t>(1023));
  constexpr int kHalves = D / 64, kBox = 128 * 64;
  const int k_tile = blockIdx.x, head = blockIdx.y, batch = blockIdx.z;
  const int k0 = k_tile * kT;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  volatile int* abort = &sm.abort;
  constexpr int kQS = DkvSmem<D>::kStagesQ;
  if (threadIdx.x == 0) {
    mbar_init(&sm.kv_full, 1);
    for (int s = 0; s < kQS; ++s) {
      mbar_init(&sm.qg_full[s], 1);
      mbar_init(&sm.qg_free[s], 1);
    }
    mbar_init(&sm.sdp_full, 1);
    mbar_init(&sm.pda_full, 128 * SPLIT);
    mbar_init(&sm.acc_done, 1);
    sm.abort = 0;
    fence_barrier_init();
  }
  if (warp == 2) tmem_alloc(&sm.tmem_base, kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sm.tmem_base;
  // Query tiles that see at least one key of this tile.
  auto visible = [&](int i) { return p.bounds[(static_cast<int64_t>(batch) * p.q_tiles + i) * 3] >= k0; };
  int count = 0;
  for (int i = 0; i < p.q_tiles; ++i) count += visible(i) ? 1 : 0;
  if (warp == 0) {
    if (lane == 0 && count > 0) {
      mbar_expect_tx(&sm.kv_full, 2 * kT * D * 2);
      for (int h = 0; h < kHalves; ++h) {
        tma_load_4d(sm.k + h * kBox, &tk, &sm.kv_full, h * 64, head, k0, batch);
        tma_load_4d(sm.v + h * kBox, &tv, &sm.kv_full, h * 64, head, k0, batch);
      }
      int n = 0;
      for (int i = 0; i < p.q_tiles; ++i) {
        if (!visible(i)) continue;
        const int s = n % kQS, use = n / kQS;
        if (n >= kQS && !mbar_wait(&sm.qg_free[s], (use - 1) & 1, abort, p.err, kSiteKvEmpty)) break;
        mbar_expect_tx(&sm.qg_full[s], 2 * kT * D * 2);
        for (int h = 0; h < kHalves; ++h) {
          tma_load_4d(sm.q[s] + h * kBox, &tq, &sm.qg_full[s], h * 64, head, i * kT, batch);
          tma_load_4d(sm.g[s] + h * kBox, &tg, &sm.qg_full[s], h * 64, head, i * kT, batch);
        }
        ++n;
      }
      if (*abort) {   // let issued copies land before the CTA exits
        mbar_wait(&sm.kv_full, 0, abort, nullptr, kSiteDrain);
        for (int m = max(0, n - kQS); m < n; ++m)
          mbar_wait(&sm.qg_full[m % kQS], (m / kQS) & 1, abort, nullptr, kSiteDrain);
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && count > 0) {
      const uint32_t id_s = idesc_bf16(kT, kT, false, false);
      const uint32_t id_acc = idesc_bf16(kT, D, true, true);
      const uint32_t k_addr = smem_u32(sm.k), v_addr = smem_u32(sm.v);
      // S = Q K^T and dP = dO V^T of visible query tile n (stage n % kQS).
      auto issue_sdp = [&](int n) {
        const int s = n % kQS;
        const uint32_t q_addr = smem_u32(sm.q[s]), g_addr = smem_u32(sm.g[s]);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (kk / 4) * kBox * 2 + (kk % 4) * 32;
          mma_ss(tmem, smem_desc_sw128(q_addr + off, 16, 1024), smem_desc_sw128(k_addr + off, 16, 1024), id_s,
                 kk > 0);
          mma_ss(tmem + 128, smem_desc_sw128(g_addr + off, 16, 1024), smem_desc_sw128(v_addr + off, 16, 1024),
                 id_s, kk > 0);
        }
        tc_commit(&sm.sdp_full);
      };
      // dV += P^T dO and dK += dA^T Q of tile n; then its stage is free.
      auto issue_acc = [&](int n) {
        const int s = n % kQS;
        const uint32_t q_addr = smem_u32(sm.q[s]), g_addr = smem_u32(sm.g[s]);
        const uint32_t pt_addr = smem_u32(sm.pt[s]), da_addr = smem_u32(sm.dat[s]);
#pragma unroll
        for (int kk = 0; kk < kT / 16; ++kk) {
          // A = P^T / dA^T: M = keys (MN-major, two 64-key boxes), K = 16 queries.
          const uint64_t a_p = smem_desc_sw128(pt_addr + kk * 2048, kBox * 2, 1024);
          const uint64_t a_d = smem_desc_sw128(da_addr + kk * 2048, kBox * 2, 1024);
          const uint64_t b_g = smem_desc_sw128(g_addr + kk * 2048, kBox * 2, 1024);
          const uint64_t b_q = smem_desc_sw128(q_addr + kk * 2048, kBox * 2, 1024);
          const uint32_t acc = (n > 0 || kk > 0) ? 1u : 0u;
          mma_ss(tmem + 256 + D, a_p, b_g, id_acc, acc);   // dV += P^T dO
          mma_ss(tmem + 256, a_d, b_q, id_acc, acc);       // dK += dA^T Q
        }
        tc_commit(&sm.qg_free[s]);
      };
      bool ok = mbar_wait(&sm.kv_full, 0, abort, p.err, kSiteKvFull);
      int done = 0;   // tiles whose dV / dK MMAs are issued
      for (int n = 0; ok && n < count; ++n) {
        if (!mbar_wait(&sm.qg_full[n % kQS], (n / kQS) & 1, abort, p.err, kSiteQFull)) break;
        tc_fence_after();
        issue_sdp(n);
        // With two stages the previous tile's dV / dK run under this tile's
        // gradient math; with one they must finish before its stage reloads.
        if (kQS == 2 && n > 0) issue_acc(done++);
        if (!mbar_wait(&sm.pda_full, n & 1, abort, p.err, kSitePFull)) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (kQS == 1) issue_acc(done++);
      }
      if (ok && done < count) issue_acc(done++);
      if (ok) tc_commit(&sm.acc_done);
    }
  } else if (warp >= 4) {
    const int wg = (warp - 4) >> 2;
    const int row = (threadIdx.x - 128) & (kT - 1);
    const uint32_t lane_addr = tmem + (static_cast<uint32_t>(((warp - 4) & 3) * 32) << 16);
    const int c_begin = SPLIT == 2 ? wg * 64 : 0, c_end = SPLIT == 2 ? c_begin + 64 : kT;
    bool ok = true;
    int n = 0;
    for (int i = 0; i < p.q_tiles && ok; ++i) {
      if (!visible(i)) continue;
      const int s = n % kQS;
      uint8_t* pt = reinterpret_cast<uint8_t*>(sm.pt[s]);
      uint8_t* dat = reinterpret_cast<uint8_t*>(sm.dat[s]);
      RowStats st = row_stats(p, batch, head, i * kT + row);
      finish_stats<B>(st);
      // The stage's P / dA buffers are free once the dV / dK MMAs that read
      // them (tile n - kQS) have completed.
      const bool stage_free = n < kQS || mbar_wait(&sm.qg_free[s], ((n / kQS) - 1) & 1, abort, p.err, kSiteKvEmpty);
      if (!__all_sync(0xffffffffu, stage_free && mbar_wait(&sm.sdp_full, n & 1, abort, p.err, kSiteSFull))) {
        ok = false;
        break;
      }
      tc_fence_after();
      const int local_start_i = p.bounds[(static_cast<int64_t>(batch) * p.q_tiles + i) * 3 + 2];
      const bool fast = k0 + kT <= local_start_i && k0 + kT <= p.keys;
      grad_row<B>(lane_addr, lane_addr + 128, k0, p.keys, st, p.scale_log2, p.scale, fast, c_begin, c_end,
                  [&](int c0, const float (&pv)[32], const float (&da)[32]) {
                    const int box = c0 / 64, chunk0 = (c0 % 64) / 8;
#pragma unroll
                    for (int t = 0; t < 4; ++t) {
                      const uint32_t off = box * kBox * 2 + sw128_offset(row, chunk0 + t);
                      *reinterpret_cast<uint4*>(pt + off) =
                          make_uint4(pack_bf16(pv[8 * t], pv[8 * t + 1]), pack_bf16(pv[8 * t + 2], pv[8 * t + 3]),
                                     pack_bf16(pv[8 * t + 4], pv[8 * t + 5]), pack_bf16(pv[8 * t + 6], pv[8 * t + 7]));
                      *reinterpret_cast<uint4*>(dat + off) =
                          make_uint4(pack_bf16(da[8 * t], da[8 * t + 1]), pack_bf16(da[8 * t + 2], da[8 * t + 3]),
                                     pack_bf16(da[8 * t + 4], da[8 * t + 5]), pack_bf16(da[8 * t + 6], da[8 * t + 7]));
                    }
                  });
      // Make generic-proxy shared stores visible to the tensor cores.
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      tc_fence_before();
      mbar_arrive(&sm.pda_full);
      ++n;
    }
    if (ok && count > 0) ok = mbar_wait(&sm.acc_done, 0, abort, p.err, kSiteODone);   // committed once, after the last MMA
    const bool have = __all_sync(0xffffffffu, ok) && count > 0;
    tc_fence_after();
    // Epilogue: thread = key row of the dK/dV accumulators (warp-uniform TMEM loads).
    const int key = k0 + row;
    const bool write = key < p.keys;
    const int64_t base = ((static_cast<int64_t>(batch) * p.keys + (write ? key : 0)) * p.heads + head) * D;
#pragma unroll
    for (int which = 0; which < 2; ++which) {
      if (SPLIT == 2 && which != wg) continue;       // warpgroup 0 stores dK, warpgroup 1 dV
      __nv_bfloat16* out = (which == 0 ? p.dk : p.dv) + base;
#pragma unroll
      for (int c = 0; c < D; c += 32) {
        float x[32];
        if (have) {
          load_row32(lane_addr + 256 + which * D + c, x);
        } else {
#pragma unroll
          for (int t = 0; t < 32; ++t) x[t] = 0.f;
        }
#pragma unroll
        for (int t = 0; t < 32; t += 8) {
          uint32_t packed[4];
#pragma unroll
          for (int u = 0; u < 4; ++u) packed[u] = pack_bf16(x[t + 2 * u], x[t + 2 * u + 1]);
          if (write) *reinterpret_cast<uint4*>(out + c + t) = make_uint4(packed[0], packed[1], packed[2], packed[3]);
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

template <int D, int B>
void launch_bwd(const at::Tensor& grad, const at::Tensor& q, const at::Tensor& k, const at::Tensor& v,
                const BwdParams& params, cudaStream_t stream) {
  const int batch = q.size(0), queries = q.size(1), heads = q.size(2), keys = k.size(1);
  CUtensorMap tq = make_bhld_map(q.data_ptr(), batch, queries, heads, D, kT);
  CUtensorMap tg = make_bhld_map(grad.data_ptr(), batch, queries, heads, D, kT);
  CUtensorMap tk = make_bhld_map(k.data_ptr(), batch, keys, heads, D, kT);
  CUtensorMap tv = make_bhld_map(v.data_ptr(), batch, keys, heads, D, kT);
  // Two gradient warpgroups when a gate block fits in a column half.
  constexpr int kSplit = B <= 64 ? 2 : 1;
  {
    const size_t smem = sizeof(DqSmem<D>) + 1024;
    auto kernel = gated_dq_tc_kernel<D, B, kSplit>;
    EB_CUDA_CHECK(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    kernel<<<dim3((queries + kT - 1) / kT, heads, batch), threads_for(kSplit), smem, stream>>>(tq, tg, tk, tv,
                                                                                               params);
  }
  {
    const size_t smem = sizeof(DkvSmem<D>) + 1024;
    auto kernel = gated_dkv_tc_kernel<D, B, kSplit>;
    EB_CUDA_CHECK(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    kernel<<<dim3((keys + kT - 1) / kT, heads, batch), threads_for(kSplit), smem, stream>>>(tq, tg, tk, tv,
                                                                                            params);
  }
}

}  // namespace

void gated_bwd_tc_launch(const at::Tensor& grad, const at::Tensor& q, const at::Tensor& k, const at::Tensor& v,
                         const at::Tensor& pos, const at::Tensor& out, const at::Tensor& rc, const at::Tensor& pr,
                         const at::Tensor& zr, const at::Tensor& lse, int64_t block, at::Tensor& dq,
                         at::Tensor& dk, at::Tensor& dv) {
  const int batch = q.size(0), queries = q.size(1), heads = q.size(2), d = q.size(3);
  auto stream = at::cuda::getCurrentCUDAStream();
  auto delta = at::empty_like(pr);
  auto rho = at::empty_like(pr);
  const int64_t rows = static_cast<int64_t>(batch) * queries * heads;
  delta_rho_kernel<<<static_cast<unsigned>((rows + 7) / 8), 256, 0, stream>>>(
      reinterpret_cast<const __nv_bfloat16*>(grad.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(out.data_ptr()),
      rc.data_ptr<float>(), pr.data_ptr<float>(), delta.data_ptr<float>(), rho.data_ptr<float>(), rows, d);
  const int q_tiles = (queries + kT - 1) / kT;
  auto bounds = at::empty({batch, q_tiles, 3}, pos.options());
  switch (block) {
    case 16: tile_bounds_kernel<16><<<dim3(q_tiles, batch), kT, 0, stream>>>(pos.data_ptr<int>(), bounds.data_ptr<int>(), queries, q_tiles); break;
    case 32: tile_bounds_kernel<32><<<dim3(q_tiles, batch), kT, 0, stream>>>(pos.data_ptr<int>(), bounds.data_ptr<int>(), queries, q_tiles); break;
    case 64: tile_bounds_kernel<64><<<dim3(q_tiles, batch), kT, 0, stream>>>(pos.data_ptr<int>(), bounds.data_ptr<int>(), queries, q_tiles); break;
    default: tile_bounds_kernel<128><<<dim3(q_tiles, batch), kT, 0, stream>>>(pos.data_ptr<int>(), bounds.data_ptr<int>(), queries, q_tiles); break;
  }
  BwdParams params{pos.data_ptr<int>(),
                   lse.data_ptr<float>(),
                   zr.data_ptr<float>(),
                   delta.data_ptr<float>(),
                   rho.data_ptr<float>(),
                   bounds.data_ptr<int>(),
                   reinterpret_cast<__nv_bfloat16*>(dq.data_ptr()),
                   reinterpret_cast<__nv_bfloat16*>(dk.data_ptr()),
                   reinterpret_cast<__nv_bfloat16*>(dv.data_ptr()),
                   device_error_slot(q.device().index()),
                   queries,
                   static_cast<int>(k.size(1)),
                   heads,
                   q_tiles,
                   static_cast<float>(1.0 / std::sqrt(static_cast<double>(d))),
                   static_cast<float>(kLog2e / std::sqrt(static_cast<double>(d)))};
#define EB_BWD_CASE(DD, BB) \
  if (d == DD && block == BB) { launch_bwd<DD, BB>(grad, q, k, v, params, stream); C10_CUDA_KERNEL_LAUNCH_CHECK(); count_launch(4); return; }
  EB_BWD_CASE(64, 16) EB_BWD_CASE(64, 32) EB_BWD_CASE(64, 64) EB_BWD_CASE(64, 128)
  EB_BWD_CASE(128, 16) EB_BWD_CASE(128, 32) EB_BWD_CASE(128, 64) EB_BWD_CASE(128, 128)
#undef EB_BWD_CASE
  TORCH_CHECK(false, "no tcgen05 gated-attention backward for head_dim ", d, " block ", block);
}

}  // namespace eb

// ===========================================================================
// No-allocation entry point
// ===========================================================================
//
// Declared in gated_noalloc.h. This entry point has no counterpart in the
// reference framework; it exists for callers that must not allocate device
// memory: code running inside a custom allocator or memory pool callback,
// real-time or embedded hosts that pre-reserve all memory up front, and
// runtimes that forbid cudaMalloc after start-up (for example while other
// work is being recorded into a stream). Such callers cannot use
// gated_attention_bwd above, because that path allocates its per-row scratch
// (delta, rho) and per-tile position bounds with the PyTorch allocator.
//
// Here that scratch lives in one file-scope device array of fixed size.
// Limits: batch * queries * heads <= kNoAllocMaxRows and
// batch * ceil(queries / 128) <= kNoAllocMaxTiles; larger calls are rejected
// with an error message. Every GPU that loads this library keeps the array
// (about 4.2 MiB) resident until the process exits. All calls on a device
// share it and it keeps the previous call's contents, so calls whose GPU work
// may overlap (for example calls on two streams of one device) race on it;
// the caller must serialise them.
namespace eb {
namespace {

constexpr int64_t kNoAllocMaxRows = int64_t(1) << 19;    // delta + rho: 2 x 2 MiB
constexpr int64_t kNoAllocMaxTiles = int64_t(1) << 14;   // bounds: 192 KiB
constexpr size_t kNoAllocRowBytes = sizeof(float) * kNoAllocMaxRows;
constexpr size_t kNoAllocBoundBytes = sizeof(int) * 3 * kNoAllocMaxTiles;
constexpr size_t kNoAllocBytes = 2 * kNoAllocRowBytes + kNoAllocBoundBytes + 256;

// The scratch array. In host code this name is only a stand-in, never a
// device address: the host takes the address with cudaGetSymbolAddress.
static __device__ __align__(256) unsigned char noalloc_scratch[kNoAllocBytes];

std::mutex noalloc_lock;
unsigned char* noalloc_base[64] = {nullptr};

int noalloc_fail(char* msg, int cap, const char* text, int code) {
  if (msg != nullptr && cap > 0) {
    std::snprintf(msg, static_cast<size_t>(cap), "%s", text);
  }
  return code;
}

// Set-up, once per device, with that device current (the caller's current
// device): look up the device address of the scratch array.
int noalloc_scratch_address(int device, unsigned char** out, char* msg, int cap) {
  std::lock_guard<std::mutex> guard(noalloc_lock);
  if (noalloc_base[device] == nullptr) {
    void* ptr = nullptr;
    const cudaError_t rc = cudaGetSymbolAddress(&ptr, noalloc_scratch);
    if (rc != cudaSuccess || ptr == nullptr) {
      char text[256];
      std::snprintf(text, sizeof(text), "cudaGetSymbolAddress(noalloc_scratch) failed: %s",
                    cudaGetErrorString(rc));
      return noalloc_fail(msg, cap, text, 2);
    }
    noalloc_base[device] = static_cast<unsigned char*>(ptr);
  }
  *out = noalloc_base[device];
  return 0;
}

// The same kernels and warpgroup split as launch_bwd (two gradient warpgroups
// for gate blocks of at most 64 keys). Returns the first CUDA error of the
// attribute calls or the launches.
template <int D, int B>
cudaError_t noalloc_launch(const void* grad, const void* q, const void* k, const void* v, int batch, int queries,
                           int keys, int heads, const BwdParams& params, cudaStream_t stream) {
  constexpr int kSplit = B <= 64 ? 2 : 1;
  CUtensorMap tq = make_bhld_map(const_cast<void*>(q), batch, queries, heads, D, kT);
  CUtensorMap tg = make_bhld_map(const_cast<void*>(grad), batch, queries, heads, D, kT);
  CUtensorMap tk = make_bhld_map(const_cast<void*>(k), batch, keys, heads, D, kT);
  CUtensorMap tv = make_bhld_map(const_cast<void*>(v), batch, keys, heads, D, kT);
  const size_t smem_q = sizeof(DqSmem<D>) + 1024, smem_kv = sizeof(DkvSmem<D>) + 1024;
  cudaError_t rc = cudaFuncSetAttribute(gated_dq_tc_kernel<D, B, kSplit>,
                                        cudaFuncAttributeMaxDynamicSharedMemorySize, smem_q);
  if (rc != cudaSuccess) return rc;
  rc = cudaFuncSetAttribute(gated_dkv_tc_kernel<D, B, kSplit>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_kv);
  if (rc != cudaSuccess) return rc;
  gated_dq_tc_kernel<D, B, kSplit><<<dim3((queries + kT - 1) / kT, heads, batch), threads_for(kSplit), smem_q,
                                     stream>>>(tq, tg, tk, tv, params);
  rc = cudaGetLastError();
  if (rc != cudaSuccess) return rc;
  gated_dkv_tc_kernel<D, B, kSplit><<<dim3((keys + kT - 1) / kT, heads, batch), threads_for(kSplit), smem_kv,
                                      stream>>>(tq, tg, tk, tv, params);
  return cudaGetLastError();
}

sm100::ErrorSlot* noalloc_error_slot(unsigned char* base) {
  return reinterpret_cast<sm100::ErrorSlot*>(base + 2 * kNoAllocRowBytes + kNoAllocBoundBytes);
}

}  // namespace
}  // namespace eb

extern "C" int eb_gated_attention_bwd_noalloc(const void* grad, const void* q, const void* k, const void* v,
                                              const int* pos, const void* out, const float* rc, const float* pr,
                                              const float* zr, const float* lse, void* dq, void* dk, void* dv,
                                              int batch, int queries, int keys, int heads, int head_dim,
                                              int block, void* stream_handle, char* error_message,
                                              int error_capacity) {
  using namespace eb;
  char* msg = error_message;
  const int cap = error_capacity;
  if (batch < 1 || queries < 1 || keys < 1 || heads < 1)
    return noalloc_fail(msg, cap, "sizes must be positive", 1);
  if (!((head_dim == 64 || head_dim == 128) && (block == 16 || block == 32 || block == 64 || block == 128)))
    return noalloc_fail(msg, cap, "unsupported shape: head_dim must be 64 or 128 and block 16/32/64/128", 1);
  const int64_t rows = static_cast<int64_t>(batch) * queries * heads;
  const int q_tiles = (queries + kT - 1) / kT;
  if (rows > kNoAllocMaxRows) {
    char text[192];
    std::snprintf(text, sizeof(text), "batch*queries*heads = %lld exceeds the scratch limit %lld",
                  static_cast<long long>(rows), static_cast<long long>(kNoAllocMaxRows));
    return noalloc_fail(msg, cap, text, 1);
  }
  if (static_cast<int64_t>(batch) * q_tiles > kNoAllocMaxTiles)
    return noalloc_fail(msg, cap, "batch * ceil(queries/128) exceeds the scratch tile limit", 1);
  // An error left by earlier work of this thread is not this call's: report it
  // without launching, and leave it pending for its owner.
  const cudaError_t pending = cudaPeekAtLastError();
  if (pending != cudaSuccess) {
    char text[256];
    std::snprintf(text, sizeof(text), "a CUDA error is pending from earlier work: %s", cudaGetErrorString(pending));
    return noalloc_fail(msg, cap, text, 2);
  }
  int device = 0;
  if (cudaGetDevice(&device) != cudaSuccess || device < 0 || device >= 64)
    return noalloc_fail(msg, cap, "no current CUDA device", 2);
  unsigned char* base = nullptr;
  if (int rc_setup = noalloc_scratch_address(device, &base, msg, cap)) return rc_setup;
  auto* delta = reinterpret_cast<float*>(base);
  auto* rho = reinterpret_cast<float*>(base + kNoAllocRowBytes);
  auto* bounds = reinterpret_cast<int*>(base + 2 * kNoAllocRowBytes);
  sm100::ErrorSlot* err = noalloc_error_slot(base);
  cudaStream_t stream = static_cast<cudaStream_t>(stream_handle);
  // delta, rho and bounds are fully rewritten below; only the error slot must start at zero.
  if (cudaMemsetAsync(err, 0, sizeof(sm100::ErrorSlot), stream) != cudaSuccess)
    return noalloc_fail(msg, cap, "cudaMemsetAsync of the error slot failed", 2);
  delta_rho_kernel<<<static_cast<unsigned>((rows + 7) / 8), 256, 0, stream>>>(
      static_cast<const __nv_bfloat16*>(grad), static_cast<const __nv_bfloat16*>(out), rc, pr, delta, rho, rows,
      head_dim);
  switch (block) {
    case 16: tile_bounds_kernel<16><<<dim3(q_tiles, batch), kT, 0, stream>>>(pos, bounds, queries, q_tiles); break;
    case 32: tile_bounds_kernel<32><<<dim3(q_tiles, batch), kT, 0, stream>>>(pos, bounds, queries, q_tiles); break;
    case 64: tile_bounds_kernel<64><<<dim3(q_tiles, batch), kT, 0, stream>>>(pos, bounds, queries, q_tiles); break;
    default: tile_bounds_kernel<128><<<dim3(q_tiles, batch), kT, 0, stream>>>(pos, bounds, queries, q_tiles); break;
  }
  BwdParams params{pos, lse, zr, delta, rho, bounds,
                   static_cast<__nv_bfloat16*>(dq), static_cast<__nv_bfloat16*>(dk), static_cast<__nv_bfloat16*>(dv),
                   err, queries, keys, heads, q_tiles,
                   static_cast<float>(1.0 / std::sqrt(static_cast<double>(head_dim))),
                   static_cast<float>(kLog2e / std::sqrt(static_cast<double>(head_dim)))};
  cudaError_t launched = cudaSuccess;
  try {
#define EB_NOALLOC_CASE(DD, BB) \
    if (head_dim == DD && block == BB) \
      launched = noalloc_launch<DD, BB>(grad, q, k, v, batch, queries, keys, heads, params, stream);
    EB_NOALLOC_CASE(64, 16) EB_NOALLOC_CASE(64, 32) EB_NOALLOC_CASE(64, 64) EB_NOALLOC_CASE(64, 128)
    EB_NOALLOC_CASE(128, 16) EB_NOALLOC_CASE(128, 32) EB_NOALLOC_CASE(128, 64) EB_NOALLOC_CASE(128, 128)
#undef EB_NOALLOC_CASE
  } catch (const std::exception& exc) {   // tensor-map encoding rejected an operand
    return noalloc_fail(msg, cap, exc.what(), 3);
  }
  if (launched != cudaSuccess) return noalloc_fail(msg, cap, cudaGetErrorString(launched), 2);
  return 0;
}

// Reads the bounded-wait record of the allocation-free backward on `device`
// and clears it. The kernels of that entry point give up a wait after about a
// second (a peer or copy that never arrived); they then stop early, leave
// dQ/dK/dV incomplete, and record which wait gave up (*site, a WaitSite id,
// 0 when none did) and in which CTA (*cta). The entry point's return code
// cannot say so, because the kernels finish after it returns: synchronise the
// stream of the call, then call this. It copies 8 bytes with cudaMemcpy and
// clears them with cudaMemset (no allocation), and makes `device` current for
// the duration of the call. Returns 0, or a nonzero code with a message in
// error_message when the device is invalid or a copy failed.
extern "C" int eb_gated_attention_bwd_noalloc_status(int device, int* site, int* cta, char* error_message,
                                                     int error_capacity) {
  using namespace eb;
  if (site == nullptr || cta == nullptr) return noalloc_fail(error_message, error_capacity, "null output", 1);
  *site = 0;
  *cta = 0;
  int count = 0;
  if (cudaGetDeviceCount(&count) != cudaSuccess || device < 0 || device >= count || device >= 64)
    return noalloc_fail(error_message, error_capacity, "invalid device", 1);
  int previous = 0;
  if (cudaGetDevice(&previous) != cudaSuccess) return noalloc_fail(error_message, error_capacity, "no device", 2);
  if (cudaSetDevice(device) != cudaSuccess) return noalloc_fail(error_message, error_capacity, "cudaSetDevice failed", 2);
  int rc = 0;
  unsigned char* base = nullptr;
  rc = noalloc_scratch_address(device, &base, error_message, error_capacity);
  if (rc == 0) {
    sm100::ErrorSlot slot{0, 0};
    sm100::ErrorSlot* dev_slot = noalloc_error_slot(base);
    if (cudaMemcpy(&slot, dev_slot, sizeof(slot), cudaMemcpyDeviceToHost) != cudaSuccess ||
        cudaMemset(dev_slot, 0, sizeof(slot)) != cudaSuccess) {
      rc = noalloc_fail(error_message, error_capacity, "reading the error record failed", 2);
    } else {
      *site = slot.code;
      *cta = slot.block;
    }
  }
  cudaSetDevice(previous);
  return rc;
}
