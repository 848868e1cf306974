// Local halo window attention on the 5th-generation tensor cores: block 16,
// head dim 64, bf16 (the shape of every Stack preset), sm_100a.
//
// Same semantics as local_halo.cu: query row t of block g attends causally
// to keys of blocks g-1 and g (the previous block comes from `prev` at a
// chunk start, or is masked), keys limited to [valid_start, start + n), RoPE
// applied on load relative to the window (only query/key distances enter
// the scores, so the CTA origin is used: 16 rows before its first query).
//
// Forward, persistent: one CTA per SM walks the units (128 query rows of one
// (batch, head)) u = blockIdx.x, blockIdx.x + gridDim.x, ...; the CTA's
// iteration i uses shared-memory stage i % 3 and TMEM buffer i % 2:
//   warp 0      TMA: Q [128 x 64], K and V [144 x 64] (halo block + 128
//               rows; a chunk start reads the halo from `prev`, or zero
//               fill), up to three units ahead
//   warp 1      S = Q K^T for all 128 x 144 (query, key) pairs into TMEM
//               buffer i % 2 (the band is 32 keys wide; the extra columns
//               cost nothing that matters at this size)
//   warp 3      O = P V with P read from TMEM (A-from-TMEM MMA form); its
//               completion frees the unit's shared-memory stage
//   warps 4-7   compute warpgroup of the even iterations, warps 8-11 of the
//   / 8-11      odd ones: rotate Q and K in shared memory (128-byte swizzled
//               rows), then thread = query row: softmax over its 32-key
//               window, P (bf16, normalised, zeros outside the window)
//               written back to TMEM, then the epilogue stores O and the
//               row's log-sum-exp.
// The two warpgroups work on consecutive units at the same time and the
// loads run ahead of both, so the copy engine, the tensor core and the
// softmax arithmetic overlap across units instead of following each other
// inside one unit.
// TMEM per buffer: S / P columns [0, 144), O [160, 224); two buffers of 256
// columns. The backward kernels are described below.
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <cstdio>
#include <cstdlib>
#include <map>
#include <mutex>

#include "../common/sm100.cuh"
#include "../common/tma.cuh"

namespace eb {
namespace {

using namespace sm100;

constexpr int kB = 16;
constexpr int kD = 64;
constexpr int kM = 128;                 // query rows per CTA
constexpr int kKeys = kM + kB;          // 144 key rows per CTA
constexpr int kThreads = 256;
constexpr uint32_t kTmemCols = 256;
constexpr uint32_t kOCol = 160;
constexpr int kTable = kM + 2 * kB;     // rotation offsets 0 .. 159
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

struct LtArgs {
  int n, heads;
  int64_t start, valid_start;
  int has_prev;
  const float* cos;    // [kTable, 32]
  const float* sin;
  __nv_bfloat16* out;  // [B, n, H * 64]
  float* lse;          // [B, n, H]
  ErrorSlot* err;
};

constexpr int kFwdStages = 3;
constexpr int kFwdThreads = 384;
constexpr uint32_t kFwdBuf = 256;       // TMEM columns per buffer

struct alignas(1024) LtSmem {
  __nv_bfloat16 q[kFwdStages][kM * kD];
  __nv_bfloat16 k[kFwdStages][kKeys * kD];
  __nv_bfloat16 v[kFwdStages][kKeys * kD];
  uint64_t q_full[kFwdStages], k_full[kFwdStages], v_full[kFwdStages], stage_free[kFwdStages];
  uint64_t rot_done[2], s_full[2], p_full[2], o_full[2], tmem_free[2];
  uint32_t tmem_base;
  int abort;
};

// Unit u -> (first query row, head, batch); the query tile varies fastest,
// so CTAs that run at the same time read neighbouring rows (shared halos).
struct LtUnit {
  int t0, head, batch;
};

EB_DEVICE LtUnit unit_of(int u, int tiles, int heads) {
  LtUnit x;
  x.t0 = (u % tiles) * kM;
  const int bh = u / tiles;
  x.head = bh % heads;
  x.batch = bh / heads;
  return x;
}

EB_DEVICE bool key_ok(const LtArgs& a, int t) {
  if (t < 0 && !a.has_prev) return false;
  return t < a.n && a.start + t >= a.valid_start;
}

// Rotate rows [0, ROWS) of a 64-wide bf16 tile stored with the 128-byte
// swizzle (row r at r * 128 bytes, 16-byte chunk c at chunk c ^ (r & 7)) by
// the RoPE angle of offset (r + off0): dims d and d + 32 form a pair. 128
// threads; thread tid always owns chunk c = tid & 3 of rows r0 + 32 k
// (r0 = tid / 4), so it reads the table twice, for its first row and for the
// 32-row step, and advances by the angle-addition formulas
//   cos(a + b) = cos a cos b - sin a sin b,  sin(a + b) = sin a cos b + cos a sin b
// (at most four steps of fp32 rounding, far below the bf16 output).
template <int ROWS>
EB_DEVICE void rotate_tile(__nv_bfloat16* tile, int off0, const float* cos_t, const float* sin_t, int tid) {
  constexpr int kPer = (ROWS * 4 + 127) / 128;
  uint8_t* base = reinterpret_cast<uint8_t*>(tile);
  const int r0 = tid >> 2, c = tid & 3;
  // Table rows are 128 bytes and the 8 angles of chunk c start 32 bytes in.
  const float4* c0p = reinterpret_cast<const float4*>(cos_t + (r0 + off0) * 32 + 8 * c);
  const float4* s0p = reinterpret_cast<const float4*>(sin_t + (r0 + off0) * 32 + 8 * c);
  const float4* cdp = reinterpret_cast<const float4*>(cos_t + 32 * 32 + 8 * c);
  const float4* sdp = reinterpret_cast<const float4*>(sin_t + 32 * 32 + 8 * c);
  const float4 c0a = __ldg(c0p), c0b = __ldg(c0p + 1), s0a = __ldg(s0p), s0b = __ldg(s0p + 1);
  const float4 cda = __ldg(cdp), cdb = __ldg(cdp + 1), sda = __ldg(sdp), sdb = __ldg(sdp + 1);
  float cs[8] = {c0a.x, c0a.y, c0a.z, c0a.w, c0b.x, c0b.y, c0b.z, c0b.w};
  float sn[8] = {s0a.x, s0a.y, s0a.z, s0a.w, s0b.x, s0b.y, s0b.z, s0b.w};
  const float cd[8] = {cda.x, cda.y, cda.z, cda.w, cdb.x, cdb.y, cdb.z, cdb.w};
  const float sd[8] = {sda.x, sda.y, sda.z, sda.w, sdb.x, sdb.y, sdb.z, sdb.w};
#pragma unroll
  for (int k = 0; k < kPer; ++k) {
    const int r = r0 + 32 * k;
    if (r < ROWS) {
      uint4* lo = reinterpret_cast<uint4*>(base + r * 128 + ((c ^ (r & 7)) << 4));
      uint4* hi = reinterpret_cast<uint4*>(base + r * 128 + (((c + 4) ^ (r & 7)) << 4));
      uint4 xa = *lo, xb = *hi;
      __nv_bfloat162* pa = reinterpret_cast<__nv_bfloat162*>(&xa);
      __nv_bfloat162* pb = reinterpret_cast<__nv_bfloat162*>(&xb);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 x1 = __bfloat1622float2(pa[i]), x2 = __bfloat1622float2(pb[i]);
        const float ca = cs[2 * i], cb = cs[2 * i + 1], sa = sn[2 * i], sb = sn[2 * i + 1];
        pa[i] = __floats2bfloat162_rn(x1.x * ca - x2.x * sa, x1.y * cb - x2.y * sb);
        pb[i] = __floats2bfloat162_rn(x2.x * ca + x1.x * sa, x2.y * cb + x1.y * sb);
      }
      *lo = xa;
      *hi = xb;
    }
    if (k + 1 < kPer) {
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float cn = cs[j] * cd[j] - sn[j] * sd[j];
        sn[j] = sn[j] * cd[j] + cs[j] * sd[j];
        cs[j] = cn;
      }
    }
  }
}

__global__ void __launch_bounds__(kFwdThreads, 1)
local_tc_fwd_kernel(const __grid_constant__ CUtensorMap t_main, const __grid_constant__ CUtensorMap t_halo,
                    const __grid_constant__ CUtensorMap t_prev, LtArgs a, int units, int tiles) {
  extern __shared__ __align__(1024) uint8_t raw_smem[];
  LtSmem& sm = *reinterpret_cast<LtSmem*>((reinterpret_cast<uintptr_t>(raw_smem) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int first = blockIdx.x, step = gridDim.x;
  const int H = a.heads;
  volatile int* abort = &sm.abort;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kFwdStages; ++s) {
      mbar_init(&sm.q_full[s], 1);
      mbar_init(&sm.k_full[s], 1);
      mbar_init(&sm.v_full[s], 1);
      mbar_init(&sm.stage_free[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&sm.rot_done[b], 128);
      mbar_init(&sm.s_full[b], 1);
      mbar_init(&sm.p_full[b], 128);
      mbar_init(&sm.o_full[b], 1);
      mbar_init(&sm.tmem_free[b], 128);
    }
    sm.abort = 0;
    fence_barrier_init();
  }
  if (warp == 2) tmem_alloc(&sm.tmem_base, 2 * kFwdBuf);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sm.tmem_base;

  if (warp == 0) {
    if (lane == 0) {
      prefetch_tensormap(&t_main);
      prefetch_tensormap(&t_halo);
      if (a.has_prev) prefetch_tensormap(&t_prev);
      int issued = 0;
      for (int i = 0, u = first; u < units; u += step, ++i) {
        const int s = i % kFwdStages;
        if (i >= kFwdStages &&
            !mbar_wait(&sm.stage_free[s], ((i / kFwdStages) - 1) & 1, abort, a.err, kSiteKvEmpty))
          break;
        const LtUnit x = unit_of(u, tiles, H);
        const bool from_prev = x.t0 == 0 && a.has_prev;
        mbar_expect_tx(&sm.q_full[s], kM * kD * 2);
        tma_load_4d(sm.q[s], &t_main, &sm.q_full[s], 0, x.head, x.t0, x.batch);
        for (int part = 1; part <= 2; ++part) {
          uint64_t* bar = part == 1 ? &sm.k_full[s] : &sm.v_full[s];
          __nv_bfloat16* dst = part == 1 ? sm.k[s] : sm.v[s];
          mbar_expect_tx(bar, kKeys * kD * 2);
          if (from_prev) tma_load_4d(dst, &t_prev, bar, 0, part * H + x.head, 0, x.batch);
          else tma_load_4d(dst, &t_halo, bar, 0, part * H + x.head, x.t0 - kB, x.batch);   // zero fill before row 0
          tma_load_4d(dst + kB * kD, &t_main, bar, 0, part * H + x.head, x.t0, x.batch);
        }
        ++issued;
      }
      if (*abort) {   // let this CTA's copies in flight land before it exits
        for (int i = issued > kFwdStages ? issued - kFwdStages : 0; i < issued; ++i) {
          const int s = i % kFwdStages;
          const uint32_t ph = (i / kFwdStages) & 1;
          mbar_wait(&sm.q_full[s], ph, abort, nullptr, kSiteDrain);
          mbar_wait(&sm.k_full[s], ph, abort, nullptr, kSiteDrain);
          mbar_wait(&sm.v_full[s], ph, abort, nullptr, kSiteDrain);
        }
      }
    }
  } else if (warp == 1) {
    // S = Q K^T of every iteration, in order, into TMEM buffer i % 2 once the
    // unit is rotated and the buffer's previous O has been read out.
    if (lane == 0) {
      const uint32_t id_s = idesc_bf16(kM, kKeys, false, false);
      for (int i = 0, u = first; u < units; u += step, ++i) {
        const int s = i % kFwdStages, b = i & 1, j = i >> 1;
        if (!mbar_wait(&sm.rot_done[b], j & 1, abort, a.err, kSiteQFull)) break;
        if (i >= 2 && !mbar_wait(&sm.tmem_free[b], (j - 1) & 1, abort, a.err, kSiteODone)) break;
        tc_fence_after();
        const uint32_t q_addr = smem_u32(sm.q[s]), k_addr = smem_u32(sm.k[s]);
#pragma unroll
        for (int kk = 0; kk < kD / 16; ++kk)
          mma_ss(tmem + b * kFwdBuf, smem_desc_sw128(q_addr + kk * 32, 16, 1024),
                 smem_desc_sw128(k_addr + kk * 32, 16, 1024), id_s, kk > 0);
        tc_commit(&sm.s_full[b]);
      }
    }
  } else if (warp == 3) {
    // O = P V of every iteration, in order; its completion also frees the stage.
    if (lane == 0) {
      const uint32_t id_pv = idesc_bf16(kM, kD, false, true);
      for (int i = 0, u = first; u < units; u += step, ++i) {
        const int s = i % kFwdStages, b = i & 1, j = i >> 1;
        if (!mbar_wait(&sm.v_full[s], (i / kFwdStages) & 1, abort, a.err, kSiteKvFull)) break;
        if (!mbar_wait(&sm.p_full[b], j & 1, abort, a.err, kSitePFull)) break;
        tc_fence_after();
        const uint32_t v_addr = smem_u32(sm.v[s]);
        const uint32_t buf = tmem + b * kFwdBuf;
#pragma unroll
        for (int kk = 0; kk < kKeys / 16; ++kk)
          mma_ts(buf + kOCol, buf + kk * 8, smem_desc_sw128(v_addr + kk * 2048, kKeys * 128, 1024), id_pv, kk > 0);
        tc_commit(&sm.o_full[b]);
        tc_commit(&sm.stage_free[s]);
      }
    }
  } else if (warp >= 4) {
    const int grp = (warp - 4) >> 2;            // this warpgroup takes iterations i = grp, grp + 2, ...
    const int w = warp & 3;                     // TMEM lane quarter
    const int tid = threadIdx.x - 128 - grp * 128;
    const int r = tid;
    const int off = lane >= 16 ? kB : 0;        // window start relative to the warp's first column 32 w
    for (int i = grp, u = first + grp * step; u < units; u += 2 * step, i += 2) {
      const int s = i % kFwdStages, j = i >> 1;
      const uint32_t ph = (i / kFwdStages) & 1;
      const uint32_t lane_addr = tmem + grp * kFwdBuf + (static_cast<uint32_t>(w * 32) << 16);
      const LtUnit x = unit_of(u, tiles, H);
      const int t0 = x.t0, t = t0 + r;
      // 1. Rotate Q (offsets 16..143) as soon as it lands, then K (0..143), in place.
      bool ok = __all_sync(0xffffffffu, mbar_wait(&sm.q_full[s], ph, abort, a.err, kSiteQFull));
      if (ok) rotate_tile<kM>(sm.q[s], kB, a.cos, a.sin, tid);
      ok = ok && __all_sync(0xffffffffu, mbar_wait(&sm.k_full[s], ph, abort, a.err, kSiteKvFull));
      if (ok) rotate_tile<kKeys>(sm.k[s], 0, a.cos, a.sin, tid);
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      mbar_arrive(&sm.rot_done[grp]);
      // 2. Softmax of row r over its window: keys 16 * (r / 16) .. + 31 (unit key index).
      float lse_row = kNegInf;
      float p[48];
      ok = ok && __all_sync(0xffffffffu, mbar_wait(&sm.s_full[grp], j & 1, abort, a.err, kSiteSFull));
      if (ok) {
        tc_fence_after();
        uint32_t s0[32], s1[16];
        tmem_ld32(lane_addr + 32 * w, s0);
        tmem_ld16(lane_addr + 32 * w + 32, s1);
        tc_wait_ld();
        const float scale = 0.125f * kLog2e;
        float m = kNegInf;
#pragma unroll
        for (int jj = 0; jj < 48; ++jj) {
          const int kk = 32 * w + jj;                  // unit key index; token t0 - 16 + kk
          const bool in = jj >= off && jj < off + 2 * kB && kk <= r + kB && key_ok(a, t0 - kB + kk) && t < a.n;
          const float xs = __uint_as_float(jj < 32 ? s0[jj] : s1[jj - 32]) * scale;
          p[jj] = in ? xs : kNegInf;
          m = fmaxf(m, p[jj]);
        }
        float sum = 0.f;
#pragma unroll
        for (int jj = 0; jj < 48; ++jj) {
          p[jj] = m == kNegInf ? 0.f : ex2(p[jj] - m);
          sum += p[jj];
        }
        const float inv = sum > 0.f ? 1.f / sum : 0.f;
#pragma unroll
        for (int jj = 0; jj < 48; ++jj) p[jj] *= inv;
        lse_row = sum > 0.f ? (m + lg2(sum)) * kLn2 : kNegInf;
        // P as bf16 pairs over all 144 key columns (72 TMEM columns): the band
        // of this warp is pair columns [16 w, 16 w + 24), the rest is zero.
        uint32_t zero[8];
#pragma unroll
        for (int c = 0; c < 8; ++c) zero[c] = 0u;
#pragma unroll
        for (int chunk = 0; chunk < kKeys / 16; ++chunk)
          if (chunk < 2 * w || chunk > 2 * w + 2) tmem_st8(lane_addr + chunk * 8, zero);
#pragma unroll
        for (int rel = 0; rel < 3; ++rel) {          // band chunks 2w .. 2w+2 (16 keys each)
          uint32_t packed[8];
#pragma unroll
          for (int c = 0; c < 8; ++c) packed[c] = pack_bf16(p[rel * 16 + 2 * c], p[rel * 16 + 2 * c + 1]);
          tmem_st8(lane_addr + (2 * w + rel) * 8, packed);
        }
        tc_wait_st();
      }
      tc_fence_before();
      mbar_arrive(&sm.p_full[grp]);
      // 3. Epilogue: O rows (already normalised) and the row's log-sum-exp; the
      //    buffer is handed back as soon as O is in registers.
      ok = ok && __all_sync(0xffffffffu, mbar_wait(&sm.o_full[grp], j & 1, abort, a.err, kSiteODone));
      uint32_t o0[32], o1[32];
      if (ok) {
        tc_fence_after();
        tmem_ld32(lane_addr + kOCol, o0);
        tmem_ld32(lane_addr + kOCol + 32, o1);
        tc_wait_ld();
      }
      tc_fence_before();
      mbar_arrive(&sm.tmem_free[grp]);
      if (!ok) break;
      if (t < a.n) {
        uint4* dst = reinterpret_cast<uint4*>(a.out + ((static_cast<int64_t>(x.batch) * a.n + t) * H + x.head) * kD);
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          const uint32_t* src = c < 4 ? o0 + 8 * c : o1 + 8 * (c - 4);
          dst[c] = make_uint4(pack_bf16(__uint_as_float(src[0]), __uint_as_float(src[1])),
                              pack_bf16(__uint_as_float(src[2]), __uint_as_float(src[3])),
                              pack_bf16(__uint_as_float(src[4]), __uint_as_float(src[5])),
                              pack_bf16(__uint_as_float(src[6]), __uint_as_float(src[7])));
        }
        a.lse[(static_cast<int64_t>(x.batch) * a.n + t) * H + x.head] = lse_row;
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(tmem, 2 * kFwdBuf);
  }
}

// ---------------------------------------------------------------------------
// backward
//
// dQ kernel (query owner), one CTA = 128 query rows of one (batch, head):
//   S = Q K^T and dP = dO V^T (128 x 144 each, sequentially in the same TMEM
//   columns), P = exp(S - lse) from the forward's log-sum-exp, dS = P (dP -
//   delta) on the 32-key window (bf16 into TMEM), dQ = dS K (A-from-TMEM),
//   then RoPE is undone on dQ. delta = rowsum(dO o O) is formed here and
//   stored for the key kernel.
// dK/dV kernel (key owner), one CTA = 128 key rows [s0, s0+128); its
//   queries are [s0, s0+144) (the next block also sees the last key block):
//   S^T = K Q^T and dP^T = V dO^T (128 x 144), P^T and dS^T on the window,
//   dV = P^T dO and dK = dS^T Q (both A-from-TMEM), RoPE undone on dK. An
//   extra CTA owns the halo block (`prev`), whose gradient goes to dprev.
// Every element is written by exactly one CTA: no atomics, deterministic.
// ---------------------------------------------------------------------------

struct LtBwdArgs {
  int n, heads;
  int64_t start, valid_start;
  int has_prev;
  const float* cos;
  const float* sin;
  const __nv_bfloat16* out;     // [B, n, H * 64]
  const __nv_bfloat16* dout;
  const float* lse;             // [B, n, H]
  float* delta;                 // [B, n, H] (written by the dQ kernel)
  __nv_bfloat16* dqkv;          // [B, n, 3, H, 64]
  __nv_bfloat16* dprev;         // [B, 16, 3, H, 64] or nullptr
  ErrorSlot* err;
};

struct alignas(1024) LtDqSmem {
  __nv_bfloat16 q[kM * kD];
  __nv_bfloat16 g[kM * kD];     // dO
  __nv_bfloat16 k[kKeys * kD];
  __nv_bfloat16 v[kKeys * kD];
  uint64_t q_full, g_full, k_full, v_full, rot_done, s_full, s_read, dp_full, ds_full, dq_full;
  uint32_t tmem_base;
  int abort;
};

EB_DEVICE bool bwd_key_ok(const LtBwdArgs& a, int t) {
  if (t < 0 && !a.has_prev) return false;
  return t < a.n && a.start + t >= a.valid_start;
}

// RoPE backward on a 64-wide fp32 row held as 64 values: x = R(-theta) y.
EB_DEVICE void unrotate_row(float (&y)[64], int offset, const float* cos_t, const float* sin_t) {
  const float4* cs = reinterpret_cast<const float4*>(cos_t + offset * 32);    // 128-byte table rows
  const float4* sn = reinterpret_cast<const float4*>(sin_t + offset * 32);
#pragma unroll
  for (int i4 = 0; i4 < 8; ++i4) {
    const float4 c4 = __ldg(cs + i4), s4 = __ldg(sn + i4);
    const float cc[4] = {c4.x, c4.y, c4.z, c4.w}, ss[4] = {s4.x, s4.y, s4.z, s4.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int i = 4 * i4 + j;
      const float a = y[i], b = y[i + 32];
      y[i] = a * cc[j] + b * ss[j];
      y[i + 32] = b * cc[j] - a * ss[j];
    }
  }
}

EB_DEVICE void store_row64(__nv_bfloat16* dst, const float (&y)[64]) {
  uint4* d = reinterpret_cast<uint4*>(dst);
#pragma unroll
  for (int c = 0; c < 8; ++c)
    d[c] = make_uint4(pack_bf16(y[8 * c], y[8 * c + 1]), pack_bf16(y[8 * c + 2], y[8 * c + 3]),
                      pack_bf16(y[8 * c + 4], y[8 * c + 5]), pack_bf16(y[8 * c + 6], y[8 * c + 7]));
}

EB_DEVICE void load_tmem64(uint32_t addr, float (&y)[64]) {
  uint32_t r0[32], r1[32];
  tmem_ld32(addr, r0);
  tmem_ld32(addr + 32, r1);
  tc_wait_ld();
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    y[i] = __uint_as_float(r0[i]);
    y[i + 32] = __uint_as_float(r1[i]);
  }
}

// 48 fp32 TMEM columns starting at `addr` (the warp's band).
EB_DEVICE void load_band48(uint32_t addr, float (&x)[48]) {
  uint32_t r0[32], r1[16];
  tmem_ld32(addr, r0);
  tmem_ld16(addr + 32, r1);
  tc_wait_ld();
#pragma unroll
  for (int j = 0; j < 32; ++j) x[j] = __uint_as_float(r0[j]);
#pragma unroll
  for (int j = 0; j < 16; ++j) x[32 + j] = __uint_as_float(r1[j]);
}

// 48 band values as bf16 pairs into the 72 pair columns at `addr` (zeros
// outside this warp's band: pair columns [16 w, 16 w + 24)).
EB_DEVICE void store_band_bf16(uint32_t addr, int w, const float (&x)[48]) {
  uint32_t zero[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) zero[i] = 0u;
#pragma unroll
  for (int chunk = 0; chunk < kKeys / 16; ++chunk)
    if (chunk < 2 * w || chunk > 2 * w + 2) tmem_st8(addr + chunk * 8, zero);
#pragma unroll
  for (int rel = 0; rel < 3; ++rel) {
    uint32_t packed[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) packed[i] = pack_bf16(x[rel * 16 + 2 * i], x[rel * 16 + 2 * i + 1]);
    tmem_st8(addr + (2 * w + rel) * 8, packed);
  }
}

__global__ void __launch_bounds__(kThreads, 2)
local_tc_dq_kernel(const __grid_constant__ CUtensorMap t_main, const __grid_constant__ CUtensorMap t_halo,
                   const __grid_constant__ CUtensorMap t_prev, const __grid_constant__ CUtensorMap t_dout,
                   LtBwdArgs a) {
  extern __shared__ __align__(1024) uint8_t raw_smem[];
  LtDqSmem& sm = *reinterpret_cast<LtDqSmem*>((reinterpret_cast<uintptr_t>(raw_smem) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int head = blockIdx.y, batch = blockIdx.z;
  const int t0 = blockIdx.x * kM;
  const int H = a.heads;
  volatile int* abort = &sm.abort;
  if (threadIdx.x == 0) {
    mbar_init(&sm.q_full, 1);
    mbar_init(&sm.g_full, 1);
    mbar_init(&sm.k_full, 1);
    mbar_init(&sm.v_full, 1);
    mbar_init(&sm.rot_done, 128);
    mbar_init(&sm.s_full, 1);
    mbar_init(&sm.s_read, 128);
    mbar_init(&sm.dp_full, 1);
    mbar_init(&sm.ds_full, 128);
    mbar_init(&sm.dq_full, 1);
    sm.abort = 0;
    fence_barrier_init();
  }
  if (warp == 2) tmem_alloc(&sm.tmem_base, kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sm.tmem_base;

  if (warp == 0) {
    if (lane == 0) {
      prefetch_tensormap(&t_main);
      prefetch_tensormap(&t_halo);
      prefetch_tensormap(&t_dout);
      const bool from_prev = t0 == 0 && a.has_prev;
      mbar_expect_tx(&sm.q_full, kM * kD * 2);
      tma_load_4d(sm.q, &t_main, &sm.q_full, 0, head, t0, batch);
      mbar_expect_tx(&sm.g_full, kM * kD * 2);
      tma_load_4d(sm.g, &t_dout, &sm.g_full, 0, head, t0, batch);
      for (int part = 1; part <= 2; ++part) {
        uint64_t* bar = part == 1 ? &sm.k_full : &sm.v_full;
        __nv_bfloat16* dst = part == 1 ? sm.k : sm.v;
        mbar_expect_tx(bar, kKeys * kD * 2);
        if (from_prev) tma_load_4d(dst, &t_prev, bar, 0, part * H + head, 0, batch);
        else tma_load_4d(dst, &t_halo, bar, 0, part * H + head, t0 - kB, batch);
        tma_load_4d(dst + kB * kD, &t_main, bar, 0, part * H + head, t0, batch);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t id_s = idesc_bf16(kM, kKeys, false, false);
      const uint32_t id_dq = idesc_bf16(kM, kD, false, true);
      bool ok = mbar_wait(&sm.rot_done, 0, abort, a.err, kSiteQFull);
      if (ok) {
        tc_fence_after();
        const uint32_t q_addr = smem_u32(sm.q), k_addr = smem_u32(sm.k);
#pragma unroll
        for (int kk = 0; kk < kD / 16; ++kk)
          mma_ss(tmem, smem_desc_sw128(q_addr + kk * 32, 16, 1024), smem_desc_sw128(k_addr + kk * 32, 16, 1024), id_s,
                 kk > 0);
        tc_commit(&sm.s_full);
        ok = mbar_wait(&sm.g_full, 0, abort, a.err, kSiteKvFull) && mbar_wait(&sm.v_full, 0, abort, a.err, kSiteKvFull) &&
             mbar_wait(&sm.s_read, 0, abort, a.err, kSitePFull);
      }
      if (ok) {
        tc_fence_after();
        const uint32_t g_addr = smem_u32(sm.g), v_addr = smem_u32(sm.v);
#pragma unroll
        for (int kk = 0; kk < kD / 16; ++kk)
          mma_ss(tmem, smem_desc_sw128(g_addr + kk * 32, 16, 1024), smem_desc_sw128(v_addr + kk * 32, 16, 1024), id_s,
                 kk > 0);
        tc_commit(&sm.dp_full);
        ok = mbar_wait(&sm.ds_full, 0, abort, a.err, kSitePFull);
      }
      if (ok) {
        tc_fence_after();
        const uint32_t k_addr = smem_u32(sm.k);
#pragma unroll
        for (int kk = 0; kk < kKeys / 16; ++kk)
          mma_ts(tmem + kOCol, tmem + kk * 8, smem_desc_sw128(k_addr + kk * 2048, kKeys * 128, 1024), id_dq, kk > 0);
        tc_commit(&sm.dq_full);
      }
    }
  } else if (warp >= 4) {
    const int tid = threadIdx.x - 128;
    const int w = warp - 4;
    const uint32_t lane_addr = tmem + (static_cast<uint32_t>(w * 32) << 16);
    bool ok = __all_sync(0xffffffffu, mbar_wait(&sm.q_full, 0, abort, a.err, kSiteQFull));
    if (ok) rotate_tile<kM>(sm.q, kB, a.cos, a.sin, tid);
    ok = ok && __all_sync(0xffffffffu, mbar_wait(&sm.k_full, 0, abort, a.err, kSiteKvFull));
    if (ok) rotate_tile<kKeys>(sm.k, 0, a.cos, a.sin, tid);
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    mbar_arrive(&sm.rot_done);
    // Row statistics: lse (base 2) and delta = dO . O (stored for the key kernel).
    const int r = tid, t = t0 + r;
    const bool row_ok = t < a.n;
    float lse2 = 0.f, delta = 0.f;
    if (row_ok) {
      const int64_t s = (static_cast<int64_t>(batch) * a.n + t) * H + head;
      const float l = a.lse[s];
      lse2 = l == kNegInf ? 0.f : l * kLog2e;
      const uint4* go = reinterpret_cast<const uint4*>(a.dout + s * kD);
      const uint4* oo = reinterpret_cast<const uint4*>(a.out + s * kD);
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        const uint4 gu = go[c], ou = oo[c];
        const __nv_bfloat162* gp = reinterpret_cast<const __nv_bfloat162*>(&gu);
        const __nv_bfloat162* op = reinterpret_cast<const __nv_bfloat162*>(&ou);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float2 gf = __bfloat1622float2(gp[i]), of = __bfloat1622float2(op[i]);
          delta += gf.x * of.x + gf.y * of.y;
        }
      }
      a.delta[s] = delta;
    }
    const int off = lane >= 16 ? kB : 0;
    float p[48];
    ok = ok && __all_sync(0xffffffffu, mbar_wait(&sm.s_full, 0, abort, a.err, kSiteSFull));
    if (ok) {
      tc_fence_after();
      float x[48];
      load_band48(lane_addr + 32 * w, x);
      const float scale = 0.125f * kLog2e;
#pragma unroll
      for (int j = 0; j < 48; ++j) {
        const int kk = 32 * w + j;
        const bool in = row_ok && j >= off && j < off + 2 * kB && kk <= r + kB && bwd_key_ok(a, t0 - kB + kk);
        p[j] = in ? ex2(fmaf(x[j], scale, -lse2)) : 0.f;
      }
    }
    tc_fence_before();
    mbar_arrive(&sm.s_read);
    ok = ok && __all_sync(0xffffffffu, mbar_wait(&sm.dp_full, 0, abort, a.err, kSiteSFull));
    if (ok) {
      tc_fence_after();
      float dp[48];
      load_band48(lane_addr + 32 * w, dp);
#pragma unroll
      for (int j = 0; j < 48; ++j) dp[j] = p[j] * (dp[j] - delta);
      store_band_bf16(lane_addr, w, dp);
      tc_wait_st();
    }
    tc_fence_before();
    mbar_arrive(&sm.ds_full);
    ok = ok && __all_sync(0xffffffffu, mbar_wait(&sm.dq_full, 0, abort, a.err, kSiteODone));
    if (ok) {
      tc_fence_after();
      float y[64];
      load_tmem64(lane_addr + kOCol, y);
#pragma unroll
      for (int i = 0; i < 64; ++i) y[i] *= 0.125f;
      unrotate_row(y, r + kB, a.cos, a.sin);
      if (row_ok) store_row64(a.dqkv + ((static_cast<int64_t>(batch) * a.n + t) * 3 * H + head) * kD, y);
    }
  }
  if (warp == 0 && lane == 0 && *abort) {
    mbar_wait(&sm.q_full, 0, abort, nullptr, kSiteDrain);
    mbar_wait(&sm.g_full, 0, abort, nullptr, kSiteDrain);
    mbar_wait(&sm.k_full, 0, abort, nullptr, kSiteDrain);
    mbar_wait(&sm.v_full, 0, abort, nullptr, kSiteDrain);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

struct alignas(1024) LtDkvSmem {
  __nv_bfloat16 k[kM * kD];
  __nv_bfloat16 v[kM * kD];
  __nv_bfloat16 q[kKeys * kD];     // query rows s0 .. s0 + 143
  __nv_bfloat16 g[kKeys * kD];     // dO rows s0 .. s0 + 143
  float lse2[kKeys], delta[kKeys];
  uint64_t k_full, v_full, q_full, g_full, rot_done, s_full, dp_full, p_full, ds_full, dv_full, dk_full;
  uint32_t tmem_base;
  int abort;
};

constexpr uint32_t kDkvTmemCols = 512;
constexpr int kDkvThreads = 384;          // control warps 0-3 + two compute warpgroups
constexpr uint32_t kColDp = 160, kColDs = 160, kColDv = 320, kColDk = 384;

__global__ void __launch_bounds__(kDkvThreads, 1)
local_tc_dkv_kernel(const __grid_constant__ CUtensorMap t_main, const __grid_constant__ CUtensorMap t_halo,
                    const __grid_constant__ CUtensorMap t_prev, const __grid_constant__ CUtensorMap t_dout,
                    const __grid_constant__ CUtensorMap t_dout16, LtBwdArgs a, int owner_ctas) {
  extern __shared__ __align__(1024) uint8_t raw_smem[];
  LtDkvSmem& sm = *reinterpret_cast<LtDkvSmem*>((reinterpret_cast<uintptr_t>(raw_smem) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int head = blockIdx.y, batch = blockIdx.z;
  const bool halo_cta = static_cast<int>(blockIdx.x) >= owner_ctas;   // keys of `prev`: rows s0 + 112 .. s0 + 127
  const int s0 = halo_cta ? -kM : static_cast<int>(blockIdx.x) * kM;
  const int H = a.heads;
  volatile int* abort = &sm.abort;
  if (threadIdx.x == 0) {
    mbar_init(&sm.k_full, 1);
    mbar_init(&sm.v_full, 1);
    mbar_init(&sm.q_full, 1);
    mbar_init(&sm.g_full, 1);
    mbar_init(&sm.rot_done, 256);
    mbar_init(&sm.s_full, 1);
    mbar_init(&sm.dp_full, 1);
    mbar_init(&sm.p_full, 256);
    mbar_init(&sm.ds_full, 256);
    mbar_init(&sm.dv_full, 1);
    mbar_init(&sm.dk_full, 1);
    sm.abort = 0;
    fence_barrier_init();
  }
  if (warp == 2) tmem_alloc(&sm.tmem_base, kDkvTmemCols);
  // Per-query statistics of rows s0 .. s0 + 143 (base-2 lse, delta).
  for (int i = threadIdx.x; i < kKeys; i += kDkvThreads) {
    const int t = s0 + i;
    float l2 = 0.f, d = 0.f;
    if (t >= 0 && t < a.n) {
      const int64_t s = (static_cast<int64_t>(batch) * a.n + t) * H + head;
      const float l = a.lse[s];
      l2 = l == kNegInf ? 0.f : l * kLog2e;
      d = a.delta[s];
    }
    sm.lse2[i] = l2;
    sm.delta[i] = d;
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sm.tmem_base;

  if (warp == 0) {
    if (lane == 0) {
      prefetch_tensormap(&t_main);
      prefetch_tensormap(&t_halo);
      prefetch_tensormap(&t_dout);
      prefetch_tensormap(&t_dout16);
      for (int part = 1; part <= 2; ++part) {
        uint64_t* bar = part == 1 ? &sm.k_full : &sm.v_full;
        __nv_bfloat16* dst = part == 1 ? sm.k : sm.v;
        mbar_expect_tx(bar, kM * kD * 2);
        if (halo_cta) {
          // Rows -128 .. -17 do not exist (zero fill, one 16-row box each);
          // rows -16 .. -1 are the halo block `prev`.
          for (int j = 0; j < kM / kB - 1; ++j)
            tma_load_4d(dst + j * kB * kD, &t_halo, bar, 0, part * H + head, s0 + j * kB, batch);
          tma_load_4d(dst + (kM - kB) * kD, &t_prev, bar, 0, part * H + head, 0, batch);
        } else {
          tma_load_4d(dst, &t_main, bar, 0, part * H + head, s0, batch);
        }
      }
      mbar_expect_tx(&sm.q_full, kKeys * kD * 2);
      tma_load_4d(sm.q, &t_main, &sm.q_full, 0, head, s0, batch);
      tma_load_4d(sm.q + kM * kD, &t_halo, &sm.q_full, 0, head, s0 + kM, batch);
      mbar_expect_tx(&sm.g_full, kKeys * kD * 2);
      tma_load_4d(sm.g, &t_dout, &sm.g_full, 0, head, s0, batch);
      tma_load_4d(sm.g + kM * kD, &t_dout16, &sm.g_full, 0, head, s0 + kM, batch);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t id_s = idesc_bf16(kM, kKeys, false, false);
      const uint32_t id_acc = idesc_bf16(kM, kD, false, true);
      // dP^T = V dO^T needs no rotation: issue it first.
      bool ok = mbar_wait(&sm.v_full, 0, abort, a.err, kSiteKvFull) && mbar_wait(&sm.g_full, 0, abort, a.err, kSiteKvFull);
      if (ok) {
        tc_fence_after();
        const uint32_t v_addr = smem_u32(sm.v), g_addr = smem_u32(sm.g);
#pragma unroll
        for (int kk = 0; kk < kD / 16; ++kk)
          mma_ss(tmem + kColDp, smem_desc_sw128(v_addr + kk * 32, 16, 1024), smem_desc_sw128(g_addr + kk * 32, 16, 1024),
                 id_s, kk > 0);
        tc_commit(&sm.dp_full);
        ok = mbar_wait(&sm.rot_done, 0, abort, a.err, kSiteQFull);
      }
      if (ok) {
        tc_fence_after();
        const uint32_t k_addr = smem_u32(sm.k), q_addr = smem_u32(sm.q);
#pragma unroll
        for (int kk = 0; kk < kD / 16; ++kk)
          mma_ss(tmem, smem_desc_sw128(k_addr + kk * 32, 16, 1024), smem_desc_sw128(q_addr + kk * 32, 16, 1024), id_s,
                 kk > 0);
        tc_commit(&sm.s_full);
        ok = mbar_wait(&sm.p_full, 0, abort, a.err, kSitePFull);
      }
      if (ok) {
        tc_fence_after();
        const uint32_t g_addr = smem_u32(sm.g);
#pragma unroll
        for (int kk = 0; kk < kKeys / 16; ++kk)   // dV = P^T dO
          mma_ts(tmem + kColDv, tmem + kk * 8, smem_desc_sw128(g_addr + kk * 2048, kKeys * 128, 1024), id_acc, kk > 0);
        tc_commit(&sm.dv_full);
        ok = mbar_wait(&sm.ds_full, 0, abort, a.err, kSitePFull);
      }
      if (ok) {
        tc_fence_after();
        const uint32_t q_addr = smem_u32(sm.q);
#pragma unroll
        for (int kk = 0; kk < kKeys / 16; ++kk)   // dK = dS^T Q
          mma_ts(tmem + kColDk, tmem + kColDs + kk * 8, smem_desc_sw128(q_addr + kk * 2048, kKeys * 128, 1024), id_acc,
                 kk > 0);
        tc_commit(&sm.dk_full);
      }
    }
  } else if (warp >= 4) {
    // Two compute warpgroups share every key row (TMEM lane): group 0 (warps
    // 4-7) owns band columns j in [0, 32) and dV, group 1 (warps 8-11) owns
    // j in [32, 48), the zero columns outside the band and dK. P^T and dS^T
    // overwrite the fp32 columns they are computed from, so both groups load
    // their values before either stores (named barrier over the 256 threads).
    const int grp = (warp - 4) >> 2;
    const int w = warp & 3;                        // TMEM lane quarter: rows 32 w ..
    const int tid = threadIdx.x - 128 - grp * 128;
    const uint32_t lane_addr = tmem + (static_cast<uint32_t>(w * 32) << 16);
    // Origin 16 rows before s0: key row k at offset k + 16, query row i at i + 16.
    // Group 0 rotates K while group 1 rotates Q.
    bool ok;
    if (grp == 0) {
      ok = __all_sync(0xffffffffu, mbar_wait(&sm.k_full, 0, abort, a.err, kSiteKvFull));
      if (ok) rotate_tile<kM>(sm.k, kB, a.cos, a.sin, tid);
    } else {
      ok = __all_sync(0xffffffffu, mbar_wait(&sm.q_full, 0, abort, a.err, kSiteQFull));
      if (ok) rotate_tile<kKeys>(sm.q, kB, a.cos, a.sin, tid);
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    mbar_arrive(&sm.rot_done);
    const int kr = tid, tk = s0 + kr;              // key row and token
    const bool key_live = bwd_key_ok(a, tk) && (!halo_cta || kr >= kM - kB);
    const int off = lane >= 16 ? kB : 0;           // query window start relative to column 32 w
    const int j0 = grp == 0 ? 0 : 32, nj = grp == 0 ? 32 : 16;
    uint32_t zero[8];
#pragma unroll
    for (int c = 0; c < 8; ++c) zero[c] = 0u;
    // Stores this group's 16-column chunks of band values v (bf16 pairs) at `addr`.
    auto store_mine = [&](uint32_t addr, const float (&v)[32]) {
#pragma unroll
      for (int rel = 0; rel < 2; ++rel) {
        if (rel * 16 < nj) {
          uint32_t packed[8];
#pragma unroll
          for (int c = 0; c < 8; ++c) packed[c] = pack_bf16(v[rel * 16 + 2 * c], v[rel * 16 + 2 * c + 1]);
          tmem_st8(addr + (2 * w + j0 / 16 + rel) * 8, packed);
        }
      }
      if (grp == 1) {
#pragma unroll
        for (int chunk = 0; chunk < kKeys / 16; ++chunk)
          if (chunk < 2 * w || chunk > 2 * w + 2) tmem_st8(addr + chunk * 8, zero);
      }
    };
    auto load_mine = [&](uint32_t addr, float (&v)[32]) {
      uint32_t r[32];
      if (grp == 0) {
        tmem_ld32(addr + 32 * w, r);
      } else {
        uint32_t r16[16];
        tmem_ld16(addr + 32 * w + 32, r16);
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          r[i] = r16[i];
          r[i + 16] = 0u;
        }
      }
      tc_wait_ld();
#pragma unroll
      for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
    };
    float p[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) p[i] = 0.f;
    ok = ok && __all_sync(0xffffffffu, mbar_wait(&sm.s_full, 0, abort, a.err, kSiteSFull));
    if (ok) {
      tc_fence_after();
      float x[32];
      load_mine(0, x);
      const float scale = 0.125f * kLog2e;
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const int j = j0 + i;
        const int qi = 32 * w + j, tq = s0 + qi;   // query index in [0, 144) and token
        const bool in = i < nj && key_live && j >= off && j < off + 2 * kB && qi >= kr && tq >= 0 && tq < a.n;
        p[i] = in ? ex2(fmaf(x[i], scale, -sm.lse2[qi < kKeys ? qi : kKeys - 1])) : 0.f;
      }
    }
    asm volatile("bar.sync 1, 256;" ::: "memory");
    if (ok) {
      store_mine(lane_addr, p);                    // P^T over S^T's columns
      tc_wait_st();
    }
    tc_fence_before();
    mbar_arrive(&sm.p_full);
    ok = ok && __all_sync(0xffffffffu, mbar_wait(&sm.dp_full, 0, abort, a.err, kSiteSFull));
    float dp[32];
    if (ok) {
      tc_fence_after();
      load_mine(kColDp, dp);
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const int qi = 32 * w + j0 + i;
        dp[i] = i < nj ? p[i] * (dp[i] - sm.delta[qi < kKeys ? qi : kKeys - 1]) : 0.f;
      }
    }
    asm volatile("bar.sync 2, 256;" ::: "memory");
    if (ok) {
      store_mine(lane_addr + kColDs, dp);          // dS^T over dP^T's columns
      tc_wait_st();
    }
    tc_fence_before();
    mbar_arrive(&sm.ds_full);
    ok = ok && __all_sync(0xffffffffu, grp == 0 ? mbar_wait(&sm.dv_full, 0, abort, a.err, kSiteODone)
                                                : mbar_wait(&sm.dk_full, 0, abort, a.err, kSiteODone));
    if (ok) {
      tc_fence_after();
      float y[64];
      __nv_bfloat16* base = nullptr;
      if (halo_cta) {
        if (kr >= kM - kB) base = a.dprev + ((static_cast<int64_t>(batch) * kB + (kr - (kM - kB))) * 3 * H + head) * kD;
      } else if (tk < a.n) {
        base = a.dqkv + ((static_cast<int64_t>(batch) * a.n + tk) * 3 * H + head) * kD;
      }
      if (grp == 0) {
        load_tmem64(lane_addr + kColDv, y);
        if (base) store_row64(base + 2 * H * kD, y);
      } else {
        load_tmem64(lane_addr + kColDk, y);
#pragma unroll
        for (int i = 0; i < 64; ++i) y[i] *= 0.125f;
        unrotate_row(y, kr + kB, a.cos, a.sin);
        if (base) store_row64(base + H * kD, y);
      }
    }
  }
  if (warp == 0 && lane == 0 && *abort) {
    mbar_wait(&sm.k_full, 0, abort, nullptr, kSiteDrain);
    mbar_wait(&sm.v_full, 0, abort, nullptr, kSiteDrain);
    mbar_wait(&sm.q_full, 0, abort, nullptr, kSiteDrain);
    mbar_wait(&sm.g_full, 0, abort, nullptr, kSiteDrain);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(tmem, kDkvTmemCols);
  }
}

std::pair<at::Tensor, at::Tensor> tc_tables(const at::Device& device) {
  // Never destroyed: tensors must not be freed by static destructors after the
  // CUDA allocator has shut down at process exit.
  static std::mutex lock;
  static auto& cache = *new std::map<int, std::pair<at::Tensor, at::Tensor>>();
  const std::lock_guard<std::mutex> guard(lock);
  auto hit = cache.find(device.index());
  if (hit != cache.end()) return hit->second;
  auto offsets = at::arange(0, kTable, at::TensorOptions().dtype(at::kFloat));
  auto index = at::arange(0, kD, 2, at::TensorOptions().dtype(at::kFloat));
  auto inv = at::pow(10000.0, -index / static_cast<double>(kD));
  auto angles = offsets.unsqueeze(1) * inv.unsqueeze(0);
  auto value = std::make_pair(angles.cos().to(device).contiguous(), angles.sin().to(device).contiguous());
  cache.emplace(device.index(), value);
  return value;
}

// qkv [B, n, 3, H, 64] viewed as (64, 3H, n, B); boxes of 64 x 1 x rows x 1.
CUtensorMap qkv_map(const void* base, int batch, int n, int heads, int rows) {
  return make_bhld_map(const_cast<void*>(base), batch, n, 3 * heads, kD, rows);
}

}  // namespace

bool local_tc_supported(const at::Tensor& qkv, int64_t block) {
  return qkv.is_cuda() && qkv.scalar_type() == at::kBFloat16 && block == kB && qkv.size(-1) == kD &&
         qkv.is_contiguous();
}

std::vector<at::Tensor> local_tc_fwd(const at::Tensor& qkv, const c10::optional<at::Tensor>& prev, int64_t start,
                                     int64_t valid_start, int64_t n) {
  TORCH_CHECK(local_tc_supported(qkv, kB), "local_tc_fwd: contiguous bf16 [B, n, 3, H, 64] with block 16");
  const int batch = qkv.size(0), heads = qkv.size(3);
  TORCH_CHECK(qkv.size(1) == n && qkv.size(2) == 3, "local_tc_fwd: qkv must be [B, n, 3, H, 64]");
  const c10::cuda::CUDAGuard guard(qkv.device());
  auto out = at::empty({batch, n, heads * kD}, qkv.options());
  auto lse = at::empty({batch, n, heads}, qkv.options().dtype(at::kFloat));
  if (n == 0) return {out, lse};
  auto tables = tc_tables(qkv.device());
  const bool has_prev = prev.has_value() && prev->defined();
  at::Tensor prev_c;
  if (has_prev) {
    prev_c = prev->contiguous();
    TORCH_CHECK(prev_c.scalar_type() == at::kBFloat16 && prev_c.size(0) == batch && prev_c.size(1) == kB &&
                    prev_c.size(2) == 3 && prev_c.size(3) == heads && prev_c.size(4) == kD,
                "local_tc_fwd: prev must be [B, 16, 3, H, 64] bf16");
  }
  CUtensorMap t_main = qkv_map(qkv.data_ptr(), batch, n, heads, kM);
  CUtensorMap t_halo = qkv_map(qkv.data_ptr(), batch, n, heads, kB);
  CUtensorMap t_prev = has_prev ? qkv_map(prev_c.data_ptr(), batch, kB, heads, kB) : t_halo;
  LtArgs args{static_cast<int>(n), heads, start, valid_start, has_prev ? 1 : 0,
              tables.first.data_ptr<float>(), tables.second.data_ptr<float>(),
              reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), lse.data_ptr<float>(),
              device_error_slot(qkv.device().index())};
  // Persistent: one CTA per SM (all 512 TMEM columns, three shared-memory stages).
  const size_t smem = sizeof(LtSmem) + 1024;
  auto kernel = local_tc_fwd_kernel;
  EB_CUDA_CHECK(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
  const int tiles = (n + kM - 1) / kM;
  const int units = tiles * heads * batch;
  const int sms = at::cuda::getCurrentDeviceProperties()->multiProcessorCount;
  kernel<<<std::min(units, sms), kFwdThreads, smem, at::cuda::getCurrentCUDAStream()>>>(t_main, t_halo, t_prev,
                                                                                       args, units, tiles);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  count_launch(1);
  return {out, lse};
}


std::vector<at::Tensor> local_tc_bwd(const at::Tensor& dout, const at::Tensor& qkv, const c10::optional<at::Tensor>& prev,
                                     const at::Tensor& out, const at::Tensor& lse, int64_t start, int64_t valid_start,
                                     int64_t n) {
  TORCH_CHECK(local_tc_supported(qkv, kB), "local_tc_bwd: contiguous bf16 [B, n, 3, H, 64] with block 16");
  const int batch = qkv.size(0), heads = qkv.size(3);
  TORCH_CHECK(dout.is_contiguous() && dout.scalar_type() == at::kBFloat16 && dout.sizes() == out.sizes() &&
                  out.is_contiguous() && lse.is_contiguous(), "local_tc_bwd: dout/out [B, n, H*64] bf16");
  const c10::cuda::CUDAGuard guard(qkv.device());
  auto dqkv = at::empty_like(qkv);
  const bool has_prev = prev.has_value() && prev->defined();
  at::Tensor prev_c, dprev;
  if (has_prev) {
    prev_c = prev->contiguous();
    dprev = at::zeros_like(prev_c);
  }
  if (n == 0) return {dqkv, dprev};
  // The q part of dqkv is fully written by the dQ kernel and the k/v parts by
  // the key kernel; dprev's q part stays zero.
  auto delta = at::empty({batch, n, heads}, qkv.options().dtype(at::kFloat));
  auto tables = tc_tables(qkv.device());
  CUtensorMap t_main = qkv_map(qkv.data_ptr(), batch, n, heads, kM);
  CUtensorMap t_halo = qkv_map(qkv.data_ptr(), batch, n, heads, kB);
  CUtensorMap t_prev = has_prev ? qkv_map(prev_c.data_ptr(), batch, kB, heads, kB) : t_halo;
  CUtensorMap t_dout = make_bhld_map(dout.data_ptr(), batch, n, heads, kD, kM);
  CUtensorMap t_dout16 = make_bhld_map(dout.data_ptr(), batch, n, heads, kD, kB);
  LtBwdArgs args{static_cast<int>(n), heads, start, valid_start, has_prev ? 1 : 0,
                 tables.first.data_ptr<float>(), tables.second.data_ptr<float>(),
                 reinterpret_cast<const __nv_bfloat16*>(out.data_ptr()),
                 reinterpret_cast<const __nv_bfloat16*>(dout.data_ptr()), lse.data_ptr<float>(),
                 delta.data_ptr<float>(), reinterpret_cast<__nv_bfloat16*>(dqkv.data_ptr()),
                 has_prev ? reinterpret_cast<__nv_bfloat16*>(dprev.data_ptr()) : nullptr,
                 device_error_slot(qkv.device().index())};
  auto stream = at::cuda::getCurrentCUDAStream();
  const int ctas = (n + kM - 1) / kM;
  // EB200_DEBUG_LOCAL=1: synchronise and report after every step (diagnostics).
  static const bool debug = std::getenv("EB200_DEBUG_LOCAL") != nullptr;
  auto trace = [&](const char* what) {
    if (!debug) return;
    const cudaError_t e = cudaStreamSynchronize(stream);
    std::fprintf(stderr, "[local_tc_bwd] %s: %s (n=%lld B=%d H=%d qkv=%p dout=%p out=%p lse=%p dqkv=%p)\n", what,
                 cudaGetErrorString(e), static_cast<long long>(n), batch, heads, qkv.data_ptr(), dout.data_ptr(),
                 out.data_ptr(), lse.data_ptr(), dqkv.data_ptr());
    std::fflush(stderr);
  };
  trace("start");
  {
    const size_t smem = std::max<size_t>(sizeof(LtDqSmem) + 1024, 80 * 1024);
    auto kernel = local_tc_dq_kernel;
    EB_CUDA_CHECK(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    // Two CTAs per SM need the maximum shared-memory carveout.
    EB_CUDA_CHECK(cudaFuncSetAttribute(kernel, cudaFuncAttributePreferredSharedMemoryCarveout, 100));
    trace("dq attribute");
    kernel<<<dim3(ctas, heads, batch), kThreads, smem, stream>>>(t_main, t_halo, t_prev, t_dout, args);
    C10_CUDA_KERNEL_LAUNCH_CHECK();
    trace("dq kernel");
  }
  {
    // One CTA per SM: the kernel holds all 512 TMEM columns.
    const size_t smem = std::max<size_t>(sizeof(LtDkvSmem) + 1024, 120 * 1024);
    auto kernel = local_tc_dkv_kernel;
    EB_CUDA_CHECK(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    trace("dkv attribute");
    kernel<<<dim3(ctas + (has_prev ? 1 : 0), heads, batch), kDkvThreads, smem, stream>>>(t_main, t_halo, t_prev, t_dout,
                                                                                       t_dout16, args, ctas);
    C10_CUDA_KERNEL_LAUNCH_CHECK();
    trace("dkv kernel");
  }
  count_launch(2);
  return {dqkv, dprev};
}

}  // namespace eb
