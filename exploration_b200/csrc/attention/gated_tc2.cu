// Exact block-gated attention forward, two query tiles per CTA (head dim 64).
//
// Same mathematics and per-row state as gated_tc.cu (one exp2 per score
// serving the block log-mass and both probabilities, stale-max online
// softmax, pure-remote fast path). The difference is the schedule: the CTA
// owns two 128-row query tiles (A and B) of one (batch, head) and streams
// each K/V tile once for both, and two softmax warpgroups work on A and B
// in parallel while the single MMA thread alternates between them:
//
//   warp 0      TMA: Q_A, Q_B once, then K/V tiles (2-stage ring)
//   warp 1      MMA: S_A(0), S_B(0); then per key tile j:
//                 PV_A(j) -> S_A(j+1) once softmax A released P_A(j),
//                 PV_B(j) -> S_B(j+1) once softmax B released P_B(j)
//   warp 2      TMEM allocator (512 columns)
//   warps 4-7   softmax/gate of tile A (thread = query row)
//   warps 8-11  softmax/gate of tile B
//
// TMEM: tile A S/P [0,128), O_remote [128,192), O_local [192,256); tile B
// the same at +256. Each tile has its own bounds (a tile stops at its own
// last visible key tile).
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "../common/sm100.cuh"
#include "../common/tma.cuh"

namespace eb {
namespace {

using namespace sm100;

constexpr int kD = 64;
constexpr int kM = 128;
constexpr int kN = 128;
constexpr int kStages = 2;
constexpr int kThreads = 384;
constexpr uint32_t kTmemCols = 512;
constexpr float kRescaleThreshold = 8.f;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

struct alignas(1024) Tc2Smem {
  __nv_bfloat16 q[2][kM * kD];
  __nv_bfloat16 k[kStages][kN * kD];
  __nv_bfloat16 v[kStages][kN * kD];
  uint64_t q_full;
  uint64_t kv_full[kStages], kv_empty[kStages];
  uint64_t s_full[2], p_full[2], o_done[2];
  uint32_t tmem_base;
  int abort;
  int pos[2][kM];
};

struct Tc2Params {
  const int* pos;
  __nv_bfloat16* out;
  float* rc;
  float* pr;
  float* zr;
  float* lse;
  ErrorSlot* err;
  int queries, keys, heads;
  float scale_log2;
};

EB_DEVICE float log2_add2(float a, float b) {
  const float m = fmaxf(a, b);
  if (m == kNegInf) return kNegInf;
  return m + lg2(ex2(a - m) + ex2(b - m));
}

struct TileBounds {
  int max_pos, remote_end, local_start, min_first_local, tiles;
};

template <int B>
EB_DEVICE TileBounds tile_bounds(const int* pos, int keys) {
  TileBounds t{-1, 0, 1 << 30, 1 << 30, 0};
  for (int r = 0; r < kM; ++r) {
    const int p = pos[r];
    if (p < 0) continue;
    t.max_pos = max(t.max_pos, p);
    const int first_local = (p / B - 1) * B;
    t.remote_end = max(t.remote_end, first_local);
    t.local_start = min(t.local_start, max(first_local, 0));
    t.min_first_local = min(t.min_first_local, first_local);
  }
  const int limit = min(keys, t.max_pos + 1);
  t.tiles = limit > 0 ? (limit + kN - 1) / kN : 0;
  return t;
}

EB_DEVICE bool remote_used(const TileBounds& t, int j) { return j * kN < t.remote_end; }
EB_DEVICE bool local_used(const TileBounds& t, int j) {
  return t.max_pos >= 0 && j * kN + kN > t.local_start && j * kN <= t.max_pos;
}
EB_DEVICE bool pure_remote(const TileBounds& t, int j, int keys) {
  return (j + 1) * kN <= t.min_first_local && (j + 1) * kN <= keys;
}

struct RowState {
  float m_r, d_r, m_l, d_l, zr;
};

// One key tile of one query row (thread = row, warp-collective TMEM access).
// Returns false when a bounded wait gave up.
template <int B>
EB_DEVICE bool softmax_tile(RowState& st, uint32_t lane_addr, uint32_t s_col, uint32_t o_col, int j, int pos,
                            const TileBounds& tb, const Tc2Params& p, uint64_t* o_done, volatile int* abort) {
  constexpr int kSeg = kN / B;
  float e[kN];
#pragma unroll
  for (int c = 0; c < kN; c += 32) {
    uint32_t r[32];
    tmem_ld32(lane_addr + s_col + c, r);
#pragma unroll
    for (int i = 0; i < 32; ++i) e[c + i] = __uint_as_float(r[i]);
  }
  tc_wait_ld();
  const int k0 = j * kN;
  const int pb = pos >= 0 ? pos / B : 0;
  const int first_local = (pb - 1) * B;
  auto rescale_o = [&](float alpha_r, float alpha_l, int cols) -> bool {
    const bool waited = j == 0 || mbar_wait(o_done, (j - 1) & 1, abort, p.err, kSiteODone);
    if (!__all_sync(0xffffffffu, waited)) return false;
    tc_fence_after();
#pragma unroll
    for (int c = 0; c < 2 * kD; c += 32) {
      if (c >= cols) break;
      uint32_t r[32];
      tmem_ld32(lane_addr + o_col + c, r);
      tc_wait_ld();
      const float f = c < kD ? alpha_r : alpha_l;
#pragma unroll
      for (int i = 0; i < 32; ++i) r[i] = __float_as_uint(__uint_as_float(r[i]) * f);
      tmem_st32(lane_addr + o_col + c, r);
    }
    return true;
  };
  if (pure_remote(tb, j, p.keys)) {
    const bool row_ok = pos >= 0;
    float seg_max[kSeg], seg_lse[kSeg];
    float tz = kNegInf, remote_max = kNegInf;
#pragma unroll
    for (int g = 0; g < kSeg; ++g) {
      float m = e[g * B];
#pragma unroll
      for (int c = 1; c < B; ++c) m = fmaxf(m, e[g * B + c]);
      const float ms = m * p.scale_log2;
      float sum = 0.f;
#pragma unroll
      for (int c = 0; c < B; ++c) {
        const float x = ex2(fmaf(e[g * B + c], p.scale_log2, -ms));
        e[g * B + c] = x;
        sum += x;
      }
      seg_max[g] = ms;
      seg_lse[g] = ms + lg2(sum);
      tz = log2_add2(tz, seg_lse[g]);
      remote_max = fmaxf(remote_max, ms + seg_lse[g]);
    }
    if (!row_ok) {
      tz = kNegInf;
      remote_max = kNegInf;
    }
    st.zr = log2_add2(st.zr, tz);
    float alpha_r = 1.f;
    bool rescale = false;
    if (remote_max > st.m_r + kRescaleThreshold || (st.m_r == kNegInf && remote_max != kNegInf)) {
      alpha_r = (st.m_r == kNegInf) ? 0.f : ex2(st.m_r - remote_max);
      rescale = st.d_r > 0.f;
      st.m_r = remote_max;
    }
    if (__any_sync(0xffffffffu, rescale) && !rescale_o(alpha_r, 1.f, kD)) return false;
    st.d_r *= alpha_r;
    float fr[kSeg];
#pragma unroll
    for (int g = 0; g < kSeg; ++g) {
      fr[g] = row_ok ? ex2(seg_max[g] + seg_lse[g] - st.m_r) : 0.f;
      if (row_ok) st.d_r += ex2(2.f * seg_lse[g] - st.m_r);
    }
#pragma unroll
    for (int c0 = 0; c0 < kN; c0 += 32) {
      uint32_t packed_r[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const int c = c0 + 2 * i;
        packed_r[i] = pack_bf16(e[c] * fr[c / B], e[c + 1] * fr[(c + 1) / B]);
      }
      tmem_st16(lane_addr + s_col + c0 / 2, packed_r);
    }
    tc_wait_st();
    return true;
  }
  // Generic tile: masks, local window, partial blocks.
  float local_max = kNegInf;
#pragma unroll
  for (int c = 0; c < kN; ++c) {
    const int key = k0 + c;
    e[c] = key < p.keys ? e[c] * p.scale_log2 : kNegInf;
    const bool loc = pos >= 0 && key >= first_local && key <= pos;
    if (loc) local_max = fmaxf(local_max, e[c]);
  }
  float seg_max[kSeg], seg_lse[kSeg];
#pragma unroll
  for (int g = 0; g < kSeg; ++g) {
    float m = kNegInf;
#pragma unroll
    for (int c = 0; c < B; ++c) m = fmaxf(m, e[g * B + c]);
    float sum = 0.f;
#pragma unroll
    for (int c = 0; c < B; ++c) {
      const float x = (m == kNegInf) ? 0.f : ex2(e[g * B + c] - m);
      e[g * B + c] = x;
      sum += x;
    }
    seg_max[g] = m;
    seg_lse[g] = (m == kNegInf) ? kNegInf : m + lg2(sum);
  }
  float tz = kNegInf, remote_max = kNegInf;
#pragma unroll
  for (int g = 0; g < kSeg; ++g) {
    const bool rem = pos >= 0 && (k0 / B + g) < pb - 1;
    if (rem && seg_lse[g] != kNegInf) {
      tz = log2_add2(tz, seg_lse[g]);
      remote_max = fmaxf(remote_max, seg_max[g] + seg_lse[g]);
    }
  }
  st.zr = log2_add2(st.zr, tz);
  bool rescale = false;
  float alpha_r = 1.f, alpha_l = 1.f;
  if (remote_max > st.m_r + kRescaleThreshold || (st.m_r == kNegInf && remote_max != kNegInf)) {
    alpha_r = (st.m_r == kNegInf) ? 0.f : ex2(st.m_r - remote_max);
    rescale |= st.d_r > 0.f;
    st.m_r = remote_max;
  }
  if (local_max > st.m_l + kRescaleThreshold || (st.m_l == kNegInf && local_max != kNegInf)) {
    alpha_l = (st.m_l == kNegInf) ? 0.f : ex2(st.m_l - local_max);
    rescale |= st.d_l > 0.f;
    st.m_l = local_max;
  }
  if (__any_sync(0xffffffffu, rescale) && !rescale_o(alpha_r, alpha_l, 2 * kD)) return false;
  st.d_r *= alpha_r;
  st.d_l *= alpha_l;
  const bool use_r = remote_used(tb, j), use_l = local_used(tb, j);
  float fr[kSeg], fl[kSeg];
#pragma unroll
  for (int g = 0; g < kSeg; ++g) {
    const bool rem = pos >= 0 && (k0 / B + g) < pb - 1 && seg_lse[g] != kNegInf;
    fr[g] = rem ? ex2(seg_max[g] + seg_lse[g] - st.m_r) : 0.f;
    if (rem) st.d_r += ex2(2.f * seg_lse[g] - st.m_r);
    fl[g] = (st.m_l == kNegInf || seg_max[g] == kNegInf) ? 0.f : ex2(seg_max[g] - st.m_l);
  }
#pragma unroll
  for (int c0 = 0; c0 < kN; c0 += 32) {
    uint32_t packed_r[16], packed_l[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const int c = c0 + 2 * i;
      const float r0 = e[c] * fr[c / B], r1 = e[c + 1] * fr[(c + 1) / B];
      packed_r[i] = pack_bf16(r0, r1);
      const int key0 = k0 + c, key1 = key0 + 1;
      const bool l0 = pos >= 0 && key0 >= first_local && key0 <= pos && key0 < p.keys;
      const bool l1 = pos >= 0 && key1 >= first_local && key1 <= pos && key1 < p.keys;
      const float x0 = l0 ? e[c] * fl[c / B] : 0.f, x1 = l1 ? e[c + 1] * fl[(c + 1) / B] : 0.f;
      st.d_l += x0 + x1;
      packed_l[i] = pack_bf16(x0, x1);
    }
    if (use_r) tmem_st16(lane_addr + s_col + c0 / 2, packed_r);
    if (use_l) tmem_st16(lane_addr + s_col + 64 + c0 / 2, packed_l);
  }
  tc_wait_st();
  return true;
}

template <int B>
__global__ void __launch_bounds__(kThreads, 1)
gated_fwd_tc2_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                     const __grid_constant__ CUtensorMap tv, Tc2Params p) {
  extern __shared__ __align__(1024) uint8_t raw_smem[];
  Tc2Smem& sm = *reinterpret_cast<Tc2Smem*>((reinterpret_cast<uintptr_t>(raw_smem) + 1023) & ~uintptr_t(1023));
  const int pair = gridDim.x - 1 - blockIdx.x;   // heaviest (latest) pairs first
  const int head = blockIdx.y, batch = blockIdx.z;
  const int q0 = pair * 2 * kM;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  volatile int* abort = &sm.abort;
  if (threadIdx.x == 0) {
    mbar_init(&sm.q_full, 1);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&sm.kv_full[s], 1);
      mbar_init(&sm.kv_empty[s], 1);
    }
    for (int t = 0; t < 2; ++t) {
      mbar_init(&sm.s_full[t], 1);
      mbar_init(&sm.p_full[t], 128);
      mbar_init(&sm.o_done[t], 1);
    }
    sm.abort = 0;
    fence_barrier_init();
  }
  if (warp == 2) tmem_alloc(&sm.tmem_base, kTmemCols);
  for (int i = threadIdx.x; i < 2 * kM; i += kThreads) {
    const int q = q0 + i;
    sm.pos[i / kM][i % kM] = q < p.queries ? p.pos[static_cast<int64_t>(batch) * p.queries + q] : -1;
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sm.tmem_base;
  const TileBounds tb[2] = {tile_bounds<B>(sm.pos[0], p.keys), tile_bounds<B>(sm.pos[1], p.keys)};
  const int tiles = max(tb[0].tiles, tb[1].tiles);
  // Register split (launched with 168 per thread = 64512 per CTA): warpgroup 0
  // (TMA, MMA, TMEM owner, idle) gives back to 40, the two softmax
  // warpgroups take 232 each: 128 * 40 + 256 * 232 = 64512.

  if (warp < 4) {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 40;\n" ::: "memory");
  if (warp == 0) {
    if (lane == 0 && tiles > 0) {
      prefetch_tensormap(&tq);
      prefetch_tensormap(&tk);
      prefetch_tensormap(&tv);
      mbar_expect_tx(&sm.q_full, 2 * kM * kD * 2);
      tma_load_4d(sm.q[0], &tq, &sm.q_full, 0, head, q0, batch);
      tma_load_4d(sm.q[1], &tq, &sm.q_full, 0, head, q0 + kM, batch);
      int issued = 0;
      for (int j = 0; j < tiles; ++j) {
        const int s = j % kStages;
        if (j >= kStages && !mbar_wait(&sm.kv_empty[s], ((j / kStages) - 1) & 1, abort, p.err, kSiteKvEmpty)) break;
        mbar_expect_tx(&sm.kv_full[s], 2 * kN * kD * 2);
        tma_load_4d(sm.k[s], &tk, &sm.kv_full[s], 0, head, j * kN, batch);
        tma_load_4d(sm.v[s], &tv, &sm.kv_full[s], 0, head, j * kN, batch);
        ++issued;
      }
      if (*abort) {
        for (int j = max(0, issued - kStages); j < issued; ++j)
          mbar_wait(&sm.kv_full[j % kStages], (j / kStages) & 1, abort, nullptr, kSiteDrain);
        mbar_wait(&sm.q_full, 0, abort, nullptr, kSiteDrain);
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && tiles > 0) {
      const uint32_t id_s = idesc_bf16(kM, kN, false, false);
      const uint32_t id_pv = idesc_bf16(kM, kD, false, true);
      auto issue_s = [&](int t, int j) {
        const uint32_t q_addr = smem_u32(sm.q[t]), k_addr = smem_u32(sm.k[j % kStages]);
#pragma unroll
        for (int kk = 0; kk < kD / 16; ++kk)
          mma_ss(tmem + t * 256, smem_desc_sw128(q_addr + kk * 32, 16, 1024),
                 smem_desc_sw128(k_addr + kk * 32, 16, 1024), id_s, kk > 0);
        tc_commit(&sm.s_full[t]);
      };
      auto issue_pv = [&](int t, int j) {
        const uint32_t v_addr = smem_u32(sm.v[j % kStages]);
        const uint32_t base = tmem + t * 256;
        if (remote_used(tb[t], j)) {
#pragma unroll
          for (int kk = 0; kk < kN / 16; ++kk)
            mma_ts(base + 128, base + kk * 8, smem_desc_sw128(v_addr + kk * 2048, kN * 128, 1024), id_pv, 1);
        }
        if (local_used(tb[t], j)) {
#pragma unroll
          for (int kk = 0; kk < kN / 16; ++kk)
            mma_ts(base + 128 + kD, base + 64 + kk * 8, smem_desc_sw128(v_addr + kk * 2048, kN * 128, 1024), id_pv,
                   1);
        }
        tc_commit(&sm.o_done[t]);
      };
      bool ok = mbar_wait(&sm.q_full, 0, abort, p.err, kSiteQFull) &&
                mbar_wait(&sm.kv_full[0], 0, abort, p.err, kSiteKvFull);
      if (ok) {
        tc_fence_after();
        for (int t = 0; t < 2; ++t)
          if (tb[t].tiles > 0) issue_s(t, 0);
      }
      for (int j = 0; ok && j < tiles; ++j) {
        for (int t = 0; ok && t < 2; ++t) {
          if (j >= tb[t].tiles) continue;
          if (!mbar_wait(&sm.p_full[t], j & 1, abort, p.err, kSitePFull)) {
            ok = false;
            break;
          }
          tc_fence_after();
          issue_pv(t, j);
          if (j + 1 < tb[t].tiles) {
            if (!mbar_wait(&sm.kv_full[(j + 1) % kStages], ((j + 1) / kStages) & 1, abort, p.err, kSiteKvFull)) {
              ok = false;
              break;
            }
            tc_fence_after();
            issue_s(t, j + 1);
          }
        }
        if (ok) tc_commit(&sm.kv_empty[j % kStages]);
      }
    }
  }
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 232;\n" ::: "memory");
    const int t = (warp - 4) >> 2;                   // query tile of this warpgroup
    const int row = (threadIdx.x - 128) & (kM - 1);
    const uint32_t lane_addr = tmem + (static_cast<uint32_t>(((warp - 4) & 3) * 32) << 16);
    const uint32_t s_col = t * 256, o_col = t * 256 + 128;
    const int pos = sm.pos[t][row];
    const TileBounds& mine = tb[t];
    {
      uint32_t zero[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) zero[i] = 0u;
#pragma unroll
      for (int c = 0; c < 2 * kD; c += 32) tmem_st32(lane_addr + o_col + c, zero);
      tc_wait_st();
    }
    RowState st{kNegInf, 0.f, kNegInf, 0.f, kNegInf};
    bool ok = true;
    for (int j = 0; j < mine.tiles; ++j) {
      if (!__all_sync(0xffffffffu, mbar_wait(&sm.s_full[t], j & 1, abort, p.err, kSiteSFull))) {
        ok = false;
        break;
      }
      tc_fence_after();
      if (!softmax_tile<B>(st, lane_addr, s_col, o_col, j, pos, mine, p, &sm.o_done[t], abort)) {
        ok = false;
        break;
      }
      tc_fence_before();
      mbar_arrive(&sm.p_full[t]);
    }
    if (ok && mine.tiles > 0) ok = mbar_wait(&sm.o_done[t], (mine.tiles - 1) & 1, abort, p.err, kSiteODone);
    ok = __all_sync(0xffffffffu, ok);
    tc_fence_after();
    const int qrow = q0 + t * kM + row;
    const bool write = qrow < p.queries;
    const float lr = (st.d_r > 0.f) ? st.m_r + lg2(st.d_r) - (st.zr == kNegInf ? 0.f : st.zr) : kNegInf;
    const float ll = (st.d_l > 0.f) ? st.m_l + lg2(st.d_l) : kNegInf;
    const float total = log2_add2(lr, ll);
    const float ref = total == kNegInf ? 0.f : total;
    const float prob_r = lr == kNegInf ? 0.f : ex2(lr - ref);
    const float prob_l = ll == kNegInf ? 0.f : ex2(ll - ref);
    const float wr = (ok && st.d_r > 0.f) ? prob_r / st.d_r : 0.f;
    const float wl = (ok && st.d_l > 0.f) ? prob_l / st.d_l : 0.f;
    const int64_t sidx = (static_cast<int64_t>(batch) * p.queries + (write ? qrow : 0)) * p.heads + head;
    if (write) {
      p.pr[sidx] = prob_r;
      p.zr[sidx] = st.zr == kNegInf ? kNegInf : st.zr * kLn2;
      p.lse[sidx] = total == kNegInf ? kNegInf : total * kLn2;
    }
    __nv_bfloat16* orow = p.out + sidx * kD;
    float* rrow = p.rc + sidx * kD;
    {
#pragma unroll
      for (int c = 0; c < kD; c += 32) {
        uint32_t rr[32], ll_[32];
        tmem_ld32(lane_addr + o_col + c, rr);
        tmem_ld32(lane_addr + o_col + kD + c, ll_);
        tc_wait_ld();
#pragma unroll
        for (int i = 0; i < 32; i += 8) {
          float remote[8];
          uint32_t packed[4];
#pragma unroll
          for (int u = 0; u < 8; ++u) remote[u] = __uint_as_float(rr[i + u]) * wr;
#pragma unroll
          for (int u = 0; u < 4; ++u)
            packed[u] = pack_bf16(remote[2 * u] + __uint_as_float(ll_[i + 2 * u]) * wl,
                                  remote[2 * u + 1] + __uint_as_float(ll_[i + 2 * u + 1]) * wl);
          if (write) {
            *reinterpret_cast<uint4*>(orow + c + i) = make_uint4(packed[0], packed[1], packed[2], packed[3]);
            *reinterpret_cast<float4*>(rrow + c + i) = make_float4(remote[0], remote[1], remote[2], remote[3]);
            *reinterpret_cast<float4*>(rrow + c + i + 4) = make_float4(remote[4], remote[5], remote[6], remote[7]);
          }
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

template <int B>
void launch2(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, const Tc2Params& params,
             cudaStream_t stream) {
  const int batch = q.size(0), queries = q.size(1), heads = q.size(2), keys = k.size(1);
  CUtensorMap tq = make_bhld_map(q.data_ptr(), batch, queries, heads, kD, 128);
  CUtensorMap tk = make_bhld_map(k.data_ptr(), batch, keys, heads, kD, 128);
  CUtensorMap tv = make_bhld_map(v.data_ptr(), batch, keys, heads, kD, 128);
  const size_t smem = sizeof(Tc2Smem) + 1024;
  auto kernel = gated_fwd_tc2_kernel<B>;
  EB_CUDA_CHECK(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
  dim3 grid((queries + 2 * kM - 1) / (2 * kM), heads, batch);
  kernel<<<grid, kThreads, smem, stream>>>(tq, tk, tv, params);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  count_launch(1);
}

}  // namespace

bool gated_tc2_supported(const at::Tensor& q, int64_t block) {
  return q.scalar_type() == at::kBFloat16 && q.size(3) == kD && block >= 16 && block <= 128 &&
         (block & (block - 1)) == 0;
}

void gated_fwd_tc2_launch(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, const at::Tensor& pos,
                          int64_t block, at::Tensor& out, at::Tensor& rc, at::Tensor& pr, at::Tensor& zr,
                          at::Tensor& lse) {
  Tc2Params params{pos.data_ptr<int>(),
                   reinterpret_cast<__nv_bfloat16*>(out.data_ptr()),
                   rc.data_ptr<float>(),
                   pr.data_ptr<float>(),
                   zr.data_ptr<float>(),
                   lse.data_ptr<float>(),
                   device_error_slot(q.device().index()),
                   static_cast<int>(q.size(1)),
                   static_cast<int>(k.size(1)),
                   static_cast<int>(q.size(2)),
                   static_cast<float>(kLog2e / std::sqrt(static_cast<double>(q.size(3))))};
  auto stream = at::cuda::getCurrentCUDAStream();
  switch (block) {
    case 16: return launch2<16>(q, k, v, params, stream);
    case 32: return launch2<32>(q, k, v, params, stream);
    case 64: return launch2<64>(q, k, v, params, stream);
    default: return launch2<128>(q, k, v, params, stream);
  }
}

}  // namespace eb
