// Exact block-gated attention forward on the 5th-generation tensor cores.
//
// One CTA = 128 query rows of one (batch, head); key tiles of 128.
// Warp roles (352 threads for gate blocks of at most 64 keys, else 224):
//   warp 0      TMA producer: Q once, then K/V tiles into a 4-stage ring
//               (2 stages for head dim 128)
//   warp 1      MMA issuer (one thread): S = Q K^T into TMEM (double
//               buffered), then O_r += P_r V and O_l += P_l V with P read
//               straight from TMEM (tcgen05.mma A-from-TMEM form)
//   warp 2      TMEM allocator (512 columns)
//   warps 3-6   softmax/gate warpgroup(s): thread i owns query row i (TMEM
//   (and 7-10)  lane i); with two warpgroups each takes 64 of the tile's 128
//               score columns, so two warps per SM sub-partition work
//               through the per-score arithmetic (one warp per
//               sub-partition was latency-bound: the tile's chain of
//               dependent exp2 / max / sum steps left issue slots idle)
//
// Gate math per row in base-2 units: with a = q.k * scale * log2(e), a
// block's log-mass is s_j = log2 sum 2^a over its b keys. One exp2 per
// score (e = 2^(a - blockmax)) serves the block sum, the remote probability
// p_r = e * 2^(blockmax + s_j - m_r) and the local one p_l = e *
// 2^(blockmax - m_l); the remote denominator gains 2^(2 s_j - m_r) per block
// and log Z_R accumulates the blocks' s_j. Statistics that span the whole
// tile are combined across the two warpgroups once per tile. Both online-softmax states keep a
// stale maximum unless it grows by more than 2^8 (then O is rescaled in
// TMEM), so the MMA and softmax warps rarely wait on each other.
//
// TMEM columns: S/P buffer 0 [0,128), buffer 1 [128,256), O_remote
// [256,256+D), O_local [256+D,256+2D). P (bf16 pairs) overwrites its S
// buffer: remote in the first 64 columns, local in the next 64.
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cudaTypedefs.h>
#include <torch/extension.h>

#include "../common/sm100.cuh"
#include "../common/tma.cuh"
#include "gated_common.cuh"

namespace eb {
namespace {

using namespace sm100;

constexpr int kM = 128;          // query rows per CTA
constexpr int kN = 128;          // keys per tile
constexpr int kTmemCols = 512;
constexpr float kRescaleThreshold = 8.f;   // log2 units
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;
// log2 of the gate block size (the largest log2 of a block's sum of 2^(a - max)).
template <int B>
constexpr float kLog2B = B == 16 ? 4.f : B == 32 ? 5.f : B == 64 ? 6.f : B == 128 ? 7.f : B == 8 ? 3.f : 10.f;

template <int D>
struct alignas(1024) TcSmem {
  // K/V ring depth. A key tile is one MMA-and-softmax step of well under a
  // microsecond, while its TMA load (from L2 or HBM) takes longer; with two
  // stages the step waited for the load of the tile two ahead (head dim 64:
  // 2.4 us per tile step at the training shape). Head dim 128 keeps two
  // stages (64 KB each).
  static constexpr int kStages = D == 64 ? 4 : 2;
  __nv_bfloat16 q[kM * D];
  __nv_bfloat16 k[kStages][kN * D];
  __nv_bfloat16 v[kStages][kN * D];
  uint64_t q_full;
  uint64_t kv_full[kStages];
  uint64_t kv_empty[kStages];
  uint64_t s_full[2];
  uint64_t p_full[2];
  uint64_t o_done;
  uint64_t xch_bar[2];
  uint32_t tmem_base;
  int abort;
  int pos[kM];
  float xch[2][2][4][kM];   // [round parity][warpgroup][value][row]: row statistics swapped per tile
};

struct TcParams {
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

EB_DEVICE float log2_add(float a, float b) {
  const float m = fmaxf(a, b);
  if (m == kNegInf) return kNegInf;
  return m + lg2(ex2(a - m) + ex2(b - m));
}

// Softmax warpgroups per CTA: two share each row when a gate block fits in
// half a key tile, one otherwise.
template <int B>
constexpr int kSplitFor = B <= 64 ? 2 : 1;
// Warps 0-2 are the producer, the MMA issuer and the TMEM owner; softmax warp
// s is hardware warp 3 + s, so it reaches TMEM lanes 32 * ((3 + s) % 4) and
// each group of four covers all 128 rows. (No idle fourth control warp: with
// two softmax warpgroups that leaves each thread 184 registers instead of 168.)
template <int B>
constexpr int kThreadsFor = 96 + 128 * kSplitFor<B>;
constexpr int kFirstSoftmaxWarp = 3;

template <int D, int B>
__global__ void __launch_bounds__(kThreadsFor<B>, 1)
gated_fwd_tc_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                    const __grid_constant__ CUtensorMap tv, TcParams p) {
  extern __shared__ __align__(1024) uint8_t raw_smem[];
  TcSmem<D>& sm = *reinterpret_cast<TcSmem<D>*>(
      (reinterpret_cast<uintptr_t>(raw_smem) + 1023) & ~static_cast<uintptr_t>(1023));
  constexpr int kHalves = D / 64;
  constexpr int kBox = 128 * 64;                 // elements per TMA box
  constexpr int kStages = TcSmem<D>::kStages;
  constexpr int kSplit = kSplitFor<B>;
  constexpr int kCols = kN / kSplit;             // score columns per softmax warpgroup
  constexpr int kSegW = kCols / B;               // gate blocks per softmax warpgroup
  constexpr int kOCols = D / kSplit;             // accumulator columns each warpgroup rescales and stores
  const int q_tile = gridDim.x - 1 - blockIdx.x; // heaviest (latest) tiles first
  const int head = blockIdx.y, batch = blockIdx.z;
  const int q0 = q_tile * kM;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  volatile int* abort = &sm.abort;

  if (threadIdx.x == 0) {
    mbar_init(&sm.q_full, 1);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&sm.kv_full[s], 1);
      mbar_init(&sm.kv_empty[s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&sm.s_full[s], 1);
      mbar_init(&sm.p_full[s], 128 * kSplit);
      mbar_init(&sm.xch_bar[s], 128 * kSplit);
    }
    mbar_init(&sm.o_done, 1);
    sm.abort = 0;
    fence_barrier_init();
  }
  if (warp == 2) tmem_alloc(&sm.tmem_base, kTmemCols);
  if (threadIdx.x < kM) {
    const int row = threadIdx.x;
    sm.pos[row] = (q0 + row < p.queries) ? p.pos[static_cast<int64_t>(batch) * p.queries + q0 + row] : -1;
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sm.tmem_base;

  // Tile-level bounds shared by every role.
  int max_pos = -1, remote_end = 0, local_start = 1 << 30, min_first_local = 1 << 30;
  for (int r = 0; r < kM; ++r) {
    const int pr_ = sm.pos[r];
    if (pr_ < 0) continue;
    max_pos = max(max_pos, pr_);
    const int first_local = (pr_ / B - 1) * B;   // may be negative: no remote keys
    remote_end = max(remote_end, first_local);
    local_start = min(local_start, max(first_local, 0));
    min_first_local = min(min_first_local, first_local);
  }
  const int limit = min(p.keys, max_pos + 1);
  const int tiles = limit > 0 ? (limit + kN - 1) / kN : 0;
  auto remote_used = [&](int j) { return j * kN < remote_end; };
  auto local_used = [&](int j) { return max_pos >= 0 && j * kN + kN > local_start && j * kN <= max_pos; };
  // Every key of tile j is an in-range remote key for every valid row of the
  // CTA: no masks, no local state, finite scores.
  auto pure_remote = [&](int j) { return (j + 1) * kN <= min_first_local && (j + 1) * kN <= p.keys; };

  if (warp == 0) {
    if (lane == 0 && tiles > 0) {
      prefetch_tensormap(&tq);
      prefetch_tensormap(&tk);
      prefetch_tensormap(&tv);
      mbar_expect_tx(&sm.q_full, kM * D * 2);
      for (int h = 0; h < kHalves; ++h) tma_load_4d(sm.q + h * kBox, &tq, &sm.q_full, h * 64, head, q0, batch);
      int issued = 0;
      for (int j = 0; j < tiles; ++j) {
        const int s = j % kStages;
        if (j >= kStages && !mbar_wait(&sm.kv_empty[s], ((j / kStages) - 1) & 1, abort, p.err, kSiteKvEmpty)) break;
        mbar_expect_tx(&sm.kv_full[s], 2 * kN * D * 2);
        for (int h = 0; h < kHalves; ++h) {
          tma_load_4d(sm.k[s] + h * kBox, &tk, &sm.kv_full[s], h * 64, head, j * kN, batch);
          tma_load_4d(sm.v[s] + h * kBox, &tv, &sm.kv_full[s], h * 64, head, j * kN, batch);
        }
        ++issued;
      }
      if (*abort) {   // let issued copies land before the CTA exits
        for (int j = max(0, issued - kStages); j < issued; ++j)
          mbar_wait(&sm.kv_full[j % kStages], (j / kStages) & 1, abort, nullptr, kSiteDrain);
        mbar_wait(&sm.q_full, 0, abort, nullptr, kSiteDrain);
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && tiles > 0) {
      const uint32_t id_s = idesc_bf16(kM, kN, false, false);
      const uint32_t id_pv = idesc_bf16(kM, D, false, true);
      const uint32_t q_addr = smem_u32(sm.q);
      auto issue_s = [&](int j) {
        const int s = j % kStages, buf = j & 1;
        const uint32_t k_addr = smem_u32(sm.k[s]);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (kk / 4) * kBox * 2 + (kk % 4) * 32;
          mma_ss(tmem + buf * 128, smem_desc_sw128(q_addr + off, 16, 1024), smem_desc_sw128(k_addr + off, 16, 1024),
                 id_s, kk > 0);
        }
        tc_commit(&sm.s_full[buf]);
      };
      bool ok = mbar_wait(&sm.q_full, 0, abort, p.err, kSiteQFull) &&
                mbar_wait(&sm.kv_full[0], 0, abort, p.err, kSiteKvFull);
      if (ok) {
        tc_fence_after();
        issue_s(0);
      }
      for (int j = 0; ok && j < tiles; ++j) {
        if (j + 1 < tiles) {
          if (!mbar_wait(&sm.kv_full[(j + 1) % kStages], ((j + 1) / kStages) & 1, abort, p.err, kSiteKvFull)) break;
          tc_fence_after();
          issue_s(j + 1);
        }
        if (!mbar_wait(&sm.p_full[j & 1], (j >> 1) & 1, abort, p.err, kSitePFull)) break;
        tc_fence_after();
        const int s = j % kStages, buf = j & 1;
        const uint32_t v_addr = smem_u32(sm.v[s]);
        const uint32_t p_base = tmem + buf * 128;
        if (remote_used(j)) {
#pragma unroll
          for (int kk = 0; kk < kN / 16; ++kk)
            mma_ts(tmem + 256, p_base + kk * 8, smem_desc_sw128(v_addr + kk * 2048, kBox * 2, 1024), id_pv, 1);
        }
        if (local_used(j)) {
#pragma unroll
          for (int kk = 0; kk < kN / 16; ++kk)
            mma_ts(tmem + 256 + D, p_base + 64 + kk * 8, smem_desc_sw128(v_addr + kk * 2048, kBox * 2, 1024), id_pv,
                   1);
        }
        tc_commit(&sm.kv_empty[s]);
        tc_commit(&sm.o_done);
      }
    }
  } else if (warp >= kFirstSoftmaxWarp) {
    // Softmax/gate warpgroups. With kSplit = 2 (gate blocks of at most 64
    // keys) two warpgroups share every query row (TMEM lane): warpgroup grp
    // owns score columns [grp * 64, grp * 64 + 64) of each tile, half of the
    // accumulator columns for rescaling and the epilogue, and partial
    // denominators; once per tile they swap the row statistics that span the
    // whole tile (tile maximum and mass, remote and local maxima) through
    // shared memory, so both take identical rescaling decisions. Every P
    // write follows that swap, i.e. both halves of S are already in registers
    // when either warpgroup overwrites S with P.
    const int grp = (warp - kFirstSoftmaxWarp) >> 2;
    const int row = (warp & 3) * 32 + lane;       // TMEM lane of this thread
    const int col0 = grp * kCols;                 // first key column of the tile owned here
    const uint32_t lane_addr = tmem + (static_cast<uint32_t>((warp & 3) * 32) << 16);
    const int pos = sm.pos[row];
    const int pb = pos >= 0 ? pos / B : 0;
    const int first_local = (pb - 1) * B;
    int round = 0;
    // Sends this warpgroup's four row values and receives the other's (bounded wait).
    auto swap = [&](const float (&mine)[4], float (&other)[4]) -> bool {
      if constexpr (kSplit == 1) {
        return true;
      } else {
        const int slot = round & 1;
#pragma unroll
        for (int k = 0; k < 4; ++k) sm.xch[slot][grp][k][row] = mine[k];
        tc_fence_before();
        mbar_arrive(&sm.xch_bar[slot]);
        const bool done = __all_sync(0xffffffffu, mbar_wait(&sm.xch_bar[slot], (round >> 1) & 1, abort, p.err,
                                                            kSiteSFull));
        tc_fence_after();
#pragma unroll
        for (int k = 0; k < 4; ++k) other[k] = sm.xch[slot][grp ^ 1][k][row];
        ++round;
        return done;
      }
    };
    // Zero this warpgroup's share of both accumulators (the MMAs always accumulate).
    {
      uint32_t zero[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) zero[i] = 0u;
#pragma unroll
      for (int c = 0; c < kOCols; c += 32) {
        tmem_st32(lane_addr + 256 + grp * kOCols + c, zero);
        tmem_st32(lane_addr + 256 + D + grp * kOCols + c, zero);
      }
      tc_wait_st();
    }
    // Running row state; d_r and d_l are this warpgroup's partial denominators.
    float m_r = kNegInf, d_r = 0.f, m_l = kNegInf, d_l = 0.f, zr = kNegInf;
    bool ok = true;
    // Multiplies this warpgroup's share of O_remote by ar and of O_local by al.
    auto rescale_o = [&](float ar, float al) {
#pragma unroll
      for (int c = 0; c < kOCols; c += 32) {
#pragma unroll
        for (int part = 0; part < 2; ++part) {
          const float f = part == 0 ? ar : al;
          if (__all_sync(0xffffffffu, f == 1.f)) continue;   // tcgen05.ld/st are warp-collective
          uint32_t r[32];
          const uint32_t addr = lane_addr + 256 + part * D + grp * kOCols + c;
          tmem_ld32(addr, r);
          tc_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) r[i] = __float_as_uint(__uint_as_float(r[i]) * f);
          tmem_st32(addr, r);
        }
      }
    };
    for (int j = 0; j < tiles; ++j) {
      const int buf = j & 1;
      if (!__all_sync(0xffffffffu, mbar_wait(&sm.s_full[buf], (j >> 1) & 1, abort, p.err, kSiteSFull))) {
        ok = false;
        break;
      }
      tc_fence_after();
      float e[kCols];
#pragma unroll
      for (int c = 0; c < kCols; c += 32) {
        uint32_t r[32];
        tmem_ld32(lane_addr + buf * 128 + col0 + c, r);
#pragma unroll
        for (int i = 0; i < 32; ++i) e[c + i] = __uint_as_float(r[i]);
      }
      tc_wait_ld();
      const int k0 = j * kN + col0;               // key index of this warpgroup's first column
      if (pure_remote(j)) {
        // Fast path (most tiles of a long sequence). Per block g: ms = its
        // maximum (scaled), sum = sum of 2^(a - ms), so its log-mass is
        // s_g = ms + log2(sum). Everything below is expressed through ms and
        // sum (two exp2 per block, no per-block log2):
        //   remote weight factor 2^(ms + s_g - m_r) = sum * 2^(2 ms - m_r),
        //   denominator term     2^(2 s_g - m_r)    = factor * sum,
        //   log Z_R of the tile  = M + log2(sum_g sum * 2^(ms - M)), M = max ms,
        //   stabiliser           2 ms + log2(B) >= ms + s_g  (an upper bound
        //                        is enough: it only shifts the scale of P).
        const bool row_ok = pos >= 0;
        float seg_max[kSegW], seg_sum[kSegW];
        float tile_max = kNegInf, remote_max = kNegInf;
#pragma unroll
        for (int g = 0; g < kSegW; ++g) {
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
          seg_sum[g] = sum;
          tile_max = fmaxf(tile_max, ms);
          remote_max = fmaxf(remote_max, 2.f * ms + kLog2B<B>);
        }
        float mass = 0.f;
#pragma unroll
        for (int g = 0; g < kSegW; ++g) mass += seg_sum[g] * ex2(seg_max[g] - tile_max);
        if constexpr (kSplit == 2) {
          const float mine[4] = {tile_max, mass, remote_max, 0.f};
          float other[4];
          if (!swap(mine, other)) {
            ok = false;
            break;
          }
          const float both = fmaxf(tile_max, other[0]);
          mass = mass * ex2(tile_max - both) + other[1] * ex2(other[0] - both);
          tile_max = both;
          remote_max = fmaxf(remote_max, other[2]);
        }
        float tz = kNegInf;
        if (row_ok) tz = tile_max + lg2(mass);
        else remote_max = kNegInf;
        zr = log2_add(zr, tz);
        float alpha_r = 1.f;
        bool rescale = false;
        if (remote_max > m_r + kRescaleThreshold || (m_r == kNegInf && remote_max != kNegInf)) {
          alpha_r = (m_r == kNegInf) ? 0.f : ex2(m_r - remote_max);
          rescale = d_r > 0.f || m_r != kNegInf;
          m_r = remote_max;
        }
        if (__any_sync(0xffffffffu, rescale)) {
          const bool waited = j == 0 || mbar_wait(&sm.o_done, (j - 1) & 1, abort, p.err, kSiteODone);
          if (!__all_sync(0xffffffffu, waited)) {
            ok = false;
            break;
          }
          tc_fence_after();
          rescale_o(alpha_r, 1.f);
        }
        d_r *= alpha_r;
        float fr[kSegW];
#pragma unroll
        for (int g = 0; g < kSegW; ++g) {
          fr[g] = row_ok ? seg_sum[g] * ex2(2.f * seg_max[g] - m_r) : 0.f;
          d_r += fr[g] * seg_sum[g];
        }
#pragma unroll
        for (int c0 = 0; c0 < kCols; c0 += 32) {
          uint32_t packed_r[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const int c = c0 + 2 * i;
            packed_r[i] = pack_bf16(e[c] * fr[c / B], e[c + 1] * fr[(c + 1) / B]);
          }
          tmem_st16(lane_addr + buf * 128 + (col0 + c0) / 2, packed_r);
        }
        tc_wait_st();
        tc_fence_before();
        mbar_arrive(&sm.p_full[buf]);
        continue;
      }
      // Scaled base-2 logits; keys past N are -inf.
      float local_max = kNegInf;
#pragma unroll
      for (int c = 0; c < kCols; ++c) {
        const int key = k0 + c;
        e[c] = key < p.keys ? e[c] * p.scale_log2 : kNegInf;
        const bool loc = pos >= 0 && key >= first_local && key <= pos;
        if (loc) local_max = fmaxf(local_max, e[c]);
      }
      float seg_max[kSegW], seg_lse[kSegW];
#pragma unroll
      for (int g = 0; g < kSegW; ++g) {
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
      // Remote blocks: log Z_R and the remote maximum.
      float tz = kNegInf, remote_max = kNegInf;
#pragma unroll
      for (int g = 0; g < kSegW; ++g) {
        const bool rem = pos >= 0 && (k0 / B + g) < pb - 1;
        if (rem && seg_lse[g] != kNegInf) {
          tz = log2_add(tz, seg_lse[g]);
          remote_max = fmaxf(remote_max, seg_max[g] + seg_lse[g]);
        }
      }
      if constexpr (kSplit == 2) {
        const float mine[4] = {tz, remote_max, local_max, 0.f};
        float other[4];
        if (!swap(mine, other)) {
          ok = false;
          break;
        }
        tz = log2_add(tz, other[0]);
        remote_max = fmaxf(remote_max, other[1]);
        local_max = fmaxf(local_max, other[2]);
      }
      zr = log2_add(zr, tz);
      bool rescale = false;
      float alpha_r = 1.f, alpha_l = 1.f;
      if (remote_max > m_r + kRescaleThreshold || (m_r == kNegInf && remote_max != kNegInf)) {
        alpha_r = (m_r == kNegInf) ? 0.f : ex2(m_r - remote_max);
        rescale |= d_r > 0.f || m_r != kNegInf;
        m_r = remote_max;
      }
      if (local_max > m_l + kRescaleThreshold || (m_l == kNegInf && local_max != kNegInf)) {
        alpha_l = (m_l == kNegInf) ? 0.f : ex2(m_l - local_max);
        rescale |= d_l > 0.f || m_l != kNegInf;
        m_l = local_max;
      }
      // tcgen05.ld/st are warp-collective: the whole warp rescales when any lane must.
      if (__any_sync(0xffffffffu, rescale)) {
        // O must be stable: wait for the previous tile's PV.
        const bool waited = j == 0 || mbar_wait(&sm.o_done, (j - 1) & 1, abort, p.err, kSiteODone);
        if (!__all_sync(0xffffffffu, waited)) {
          ok = false;
          break;
        }
        tc_fence_after();
        rescale_o(alpha_r, alpha_l);
      }
      d_r *= alpha_r;
      d_l *= alpha_l;
      const bool use_r = remote_used(j), use_l = local_used(j);
      float fr[kSegW], fl[kSegW];
#pragma unroll
      for (int g = 0; g < kSegW; ++g) {
        const bool rem = pos >= 0 && (k0 / B + g) < pb - 1 && seg_lse[g] != kNegInf;
        fr[g] = rem ? ex2(seg_max[g] + seg_lse[g] - m_r) : 0.f;
        if (rem) d_r += ex2(2.f * seg_lse[g] - m_r);
        fl[g] = (m_l == kNegInf || seg_max[g] == kNegInf) ? 0.f : ex2(seg_max[g] - m_l);
      }
#pragma unroll
      for (int c0 = 0; c0 < kCols; c0 += 32) {
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
          d_l += x0 + x1;
          packed_l[i] = pack_bf16(x0, x1);
        }
        if (use_r) tmem_st16(lane_addr + buf * 128 + (col0 + c0) / 2, packed_r);
        if (use_l) tmem_st16(lane_addr + buf * 128 + 64 + (col0 + c0) / 2, packed_l);
      }
      tc_wait_st();
      tc_fence_before();
      mbar_arrive(&sm.p_full[buf]);
    }
    if (ok && tiles > 0) ok = mbar_wait(&sm.o_done, (tiles - 1) & 1, abort, p.err, kSiteODone);
    ok = __all_sync(0xffffffffu, ok);
    if constexpr (kSplit == 2) {
      // Whole-row denominators from the two partial sums.
      const float mine[4] = {d_r, d_l, 0.f, 0.f};
      float other[4] = {0.f, 0.f, 0.f, 0.f};
      ok = swap(mine, other) && ok;
      d_r += other[0];
      d_l += other[1];
    }
    tc_fence_after();
    const int qrow = q0 + row;
    const bool write = qrow < p.queries;
    {
      const float lr = (d_r > 0.f) ? m_r + lg2(d_r) - (zr == kNegInf ? 0.f : zr) : kNegInf;
      const float ll = (d_l > 0.f) ? m_l + lg2(d_l) : kNegInf;
      const float total = log2_add(lr, ll);
      const float ref = total == kNegInf ? 0.f : total;
      const float prob_r = lr == kNegInf ? 0.f : ex2(lr - ref);
      const float prob_l = ll == kNegInf ? 0.f : ex2(ll - ref);
      const float wr = (ok && d_r > 0.f) ? prob_r / d_r : 0.f;
      const float wl = (ok && d_l > 0.f) ? prob_l / d_l : 0.f;
      const int64_t s = (static_cast<int64_t>(batch) * p.queries + (write ? qrow : 0)) * p.heads + head;
      if (write && grp == 0) {
        p.pr[s] = prob_r;
        p.zr[s] = zr == kNegInf ? kNegInf : zr * kLn2;
        p.lse[s] = total == kNegInf ? kNegInf : total * kLn2;
      }
      __nv_bfloat16* orow = p.out + s * D;
      float* rrow = p.rc + s * D;
#pragma unroll
      for (int c = grp * kOCols; c < (grp + 1) * kOCols; c += 32) {
        uint32_t rr[32], ll_[32];
        tmem_ld32(lane_addr + 256 + c, rr);
        tmem_ld32(lane_addr + 256 + D + c, ll_);
        tc_wait_ld();
#pragma unroll
        for (int i = 0; i < 32; i += 8) {
          float remote[8];
          uint32_t packed[4];
#pragma unroll
          for (int t = 0; t < 8; ++t) remote[t] = __uint_as_float(rr[i + t]) * wr;
#pragma unroll
          for (int t = 0; t < 4; ++t)
            packed[t] = pack_bf16(remote[2 * t] + __uint_as_float(ll_[i + 2 * t]) * wl,
                                  remote[2 * t + 1] + __uint_as_float(ll_[i + 2 * t + 1]) * wl);
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

template <int D, int B>
void launch(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, const TcParams& params,
            cudaStream_t stream) {
  const int batch = q.size(0), queries = q.size(1), heads = q.size(2), keys = k.size(1);
  CUtensorMap tq = make_bhld_map(q.data_ptr(), batch, queries, heads, D, 128);
  CUtensorMap tk = make_bhld_map(k.data_ptr(), batch, keys, heads, D, 128);
  CUtensorMap tv = make_bhld_map(v.data_ptr(), batch, keys, heads, D, 128);
  const size_t smem = std::max<size_t>(sizeof(TcSmem<D>) + 1024, 120 * 1024);
  auto kernel = gated_fwd_tc_kernel<D, B>;
  EB_CUDA_CHECK(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
  dim3 grid((queries + kM - 1) / kM, heads, batch);
  kernel<<<grid, kThreadsFor<B>, smem, stream>>>(tq, tk, tv, params);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  count_launch(1);
}

}  // namespace

bool gated_tc_supported(const at::Tensor& q, int64_t block) {
  const int64_t d = q.size(3);
  return q.scalar_type() == at::kBFloat16 && (d == 64 || d == 128) && block >= 16 && block <= 128 &&
         (block & (block - 1)) == 0;
}

void gated_fwd_tc_launch(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, const at::Tensor& pos,
                         int64_t block, at::Tensor& out, at::Tensor& rc, at::Tensor& pr, at::Tensor& zr,
                         at::Tensor& lse) {
  TcParams params{pos.data_ptr<int>(),
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
  const int d = q.size(3);
#define EB_GATED_CASE(DD, BB) \
  if (d == DD && block == BB) return launch<DD, BB>(q, k, v, params, stream);
  EB_GATED_CASE(64, 16) EB_GATED_CASE(64, 32) EB_GATED_CASE(64, 64) EB_GATED_CASE(64, 128)
  EB_GATED_CASE(128, 16) EB_GATED_CASE(128, 32) EB_GATED_CASE(128, 64) EB_GATED_CASE(128, 128)
#undef EB_GATED_CASE
  TORCH_CHECK(false, "no tcgen05 gated-attention instance for head_dim ", d, " block ", block);
}

}  // namespace eb
