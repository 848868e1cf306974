// Exact block scores on the tensor cores and a fused per-row top-k (sm_100a).
//
// Scoring a query against every gate block of a long KV cache reads all of
// K once; it is bandwidth-bound (1M keys x 4 heads x 64 dims x 2 bytes =
// 512 MB). One CTA owns a contiguous range of 128-key tiles of one (batch,
// head) and all queries of the call (N = queries rounded up to 16, <= 256):
//   warp 0      TMA: Q once, K tiles through a 4-stage ring
//   warp 1      S^T = K Q^T  (M = 128 keys, N = queries, K = head dim) into
//               one of two TMEM buffers
//   warps 4-7   thread = key row: scale, block log-sum-exp over the b keys of
//               each gate block (b = 16 or 32: a shuffle reduction inside the
//               half/full warp), visibility (block entirely before the
//               query's local window and complete), one fp32 store per
//               (query, block). A running log-sum-exp per query gives this
//               CTA's part of log Z_R.
// The selection kernel then takes each (batch, query, head) row of block
// scores, forms log Z_R and the top-k by a 4-pass radix select on the
// order-preserving integer image of the floats, and sorts the k winners
// (descending score, then ascending block id) with a bitonic network.
//
// Reference: st/kernels/sparse.py:9-35 (scores) and st/ops/sparse.py:130-139
// (torch topk / logsumexp).
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "../common/sm100.cuh"
#include "../common/tma.cuh"

namespace eb {
namespace {

using namespace sm100;

constexpr int kTile = 128;
constexpr int kStages = 4;
constexpr int kThreads = 384;   // warps 0-3: TMA, MMA, TMEM owner, idle; 4-11: epilogue

struct ScoreArgs {
  const int* pos;        // [B, Q] (this call's query rows)
  float* scores;         // [B, Q, H, G]
  float* zr_part;        // [B, Q, H, ctas]
  int queries, heads, keys, block, groups, tiles, tiles_per_cta, ctas;
  int64_t first;         // absolute token of key 0
  float scale;           // 1 / sqrt(head dim)
  ErrorSlot* err;
};

template <int D, int N>
struct alignas(1024) ScoreSmem {
  __nv_bfloat16 k[kStages][kTile * D];
  __nv_bfloat16 q[N * D];
  uint64_t full[kStages], empty[kStages], q_full, acc_full[2], acc_empty[2];
  uint32_t tmem_base;
  int abort;
  int pos[N];
};

// Up to 16 queries the kernel fits 80 registers, so two CTAs share an SM (the
// host sizes the grid for two per SM).
template <int D, int N, int B>
__global__ void __launch_bounds__(kThreads, N <= 16 ? 2 : 1)
block_scores_tc_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk, ScoreArgs a) {
  extern __shared__ __align__(1024) uint8_t raw_smem[];
  using Smem = ScoreSmem<D, N>;
  Smem& sm = *reinterpret_cast<Smem*>((reinterpret_cast<uintptr_t>(raw_smem) + 1023) & ~uintptr_t(1023));
  constexpr int kHalves = D / 64;
  constexpr uint32_t kCols = 2 * N <= 32 ? 32 : (2 * N <= 64 ? 64 : (2 * N <= 128 ? 128 : (2 * N <= 256 ? 256 : 512)));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int bh = blockIdx.y, batch = bh / a.heads, head = bh % a.heads;
  const int tile0 = blockIdx.x * a.tiles_per_cta;
  const int tile1 = min(a.tiles, tile0 + a.tiles_per_cta);
  const int count = max(0, tile1 - tile0);
  volatile int* abort = &sm.abort;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&sm.full[s], 1);
      mbar_init(&sm.empty[s], 1);
    }
    mbar_init(&sm.q_full, 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&sm.acc_full[s], 1);
      mbar_init(&sm.acc_empty[s], 256);
    }
    sm.abort = 0;
    fence_barrier_init();
  }
  for (int i = threadIdx.x; i < N; i += kThreads)
    sm.pos[i] = i < a.queries ? a.pos[static_cast<int64_t>(batch) * a.queries + i] : -1;
  if (warp == 2) tmem_alloc(&sm.tmem_base, kCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sm.tmem_base;

  if (warp == 0) {
    if (lane == 0 && count > 0) {
      prefetch_tensormap(&tq);
      prefetch_tensormap(&tk);
      mbar_expect_tx(&sm.q_full, N * D * 2);
      for (int h = 0; h < kHalves; ++h) tma_load_4d(sm.q + h * N * 64, &tq, &sm.q_full, h * 64, head, 0, batch);
      int issued = 0;
      for (int i = 0; i < count; ++i) {
        const int s = i % kStages;
        if (i >= kStages && !mbar_wait(&sm.empty[s], ((i / kStages) - 1) & 1, abort, a.err, kSiteKvEmpty)) break;
        mbar_expect_tx(&sm.full[s], kTile * D * 2);
        for (int h = 0; h < kHalves; ++h)
          tma_load_4d(sm.k[s] + h * kTile * 64, &tk, &sm.full[s], h * 64, head, (tile0 + i) * kTile, batch);
        ++issued;
      }
      if (*abort) {
        for (int i = max(0, issued - kStages); i < issued; ++i)
          mbar_wait(&sm.full[i % kStages], (i / kStages) & 1, abort, nullptr, kSiteDrain);
        mbar_wait(&sm.q_full, 0, abort, nullptr, kSiteDrain);
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && count > 0) {
      const uint32_t idesc = idesc_bf16(kTile, N, false, false);
      bool ok = mbar_wait(&sm.q_full, 0, abort, a.err, kSiteQFull);
      const uint32_t q_addr = smem_u32(sm.q);
      for (int i = 0; ok && i < count; ++i) {
        const int s = i % kStages, buf = i & 1;
        if (i >= 2 && !mbar_wait(&sm.acc_empty[buf], ((i >> 1) - 1) & 1, abort, a.err, kSiteODone)) break;
        if (!mbar_wait(&sm.full[s], (i / kStages) & 1, abort, a.err, kSiteKvFull)) break;
        tc_fence_after();
        const uint32_t k_addr = smem_u32(sm.k[s]);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t ka = k_addr + (kk / 4) * kTile * 128 + (kk % 4) * 32;
          const uint32_t qa = q_addr + (kk / 4) * N * 128 + (kk % 4) * 32;
          mma_ss(tmem + buf * N, smem_desc_sw128(ka, 16, 1024), smem_desc_sw128(qa, 16, 1024), idesc, kk > 0);
        }
        tc_commit(&sm.empty[s]);
        tc_commit(&sm.acc_full[buf]);
      }
    }
  } else if (warp >= 4) {
    constexpr int kHalf = N / 2;                      // query columns per warpgroup
    const int ew = warp - 4, grp = ew >> 2, w = ew & 3;
    const uint32_t lane_addr = tmem + (static_cast<uint32_t>(w * 32) << 16);
    const float scale2 = a.scale * 1.4426950408889634f;
    // Running base-2 (max, sum) of this CTA's visible block scores per query.
    // After the reductions below, lane l of a block's lane group holds query
    // l % 8 of each group of eight query columns (lanes l and l + 8 hold the
    // same), so the first eight lanes of every block finish one query each.
    constexpr int kGroups = kHalf / 8;
    float zm[kGroups], zs[kGroups];
#pragma unroll
    for (int c = 0; c < kGroups; ++c) {
      zm[c] = kNegInf;
      zs[c] = 0.f;
    }
    const bool finisher = (lane % B) < 8;
    const int qsel = lane & 7;
    for (int i = 0; i < count; ++i) {
      const int buf = i & 1;
      if (!__all_sync(0xffffffffu, mbar_wait(&sm.acc_full[buf], (i >> 1) & 1, abort, a.err, kSiteSFull))) break;
      tc_fence_after();
      const int tile = tile0 + i;
      const int key = tile * kTile + w * 32 + lane;          // key index within this call
      const int g = key / B;                                 // gate block within this call
      const bool full = (g + 1) * B <= a.keys;
      const int64_t gid = (a.first + static_cast<int64_t>(g) * B) / B;
      uint32_t r[kHalf];
      if constexpr (kHalf == 8) {
        uint32_t (&r8)[8] = reinterpret_cast<uint32_t(&)[8]>(r);
        tmem_ld8(lane_addr + buf * N + grp * kHalf, r8);
      } else {
        uint32_t (&r16)[16] = reinterpret_cast<uint32_t(&)[16]>(r);
        tmem_ld16(lane_addr + buf * N + grp * kHalf, r16);
      }
      tc_wait_ld();
      tc_fence_before();
      mbar_arrive(&sm.acc_empty[buf]);                        // the values are in registers
#pragma unroll
      for (int j0 = 0; j0 < kHalf; j0 += 8) {
        float x[8], m[8], e[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          x[j] = key < a.keys ? __uint_as_float(r[j0 + j]) * scale2 : kNegInf;
          m[j] = x[j];
        }
        // Block maxima on every lane of the block (each step for all eight
        // columns before the next, so the shuffle latencies overlap).
#pragma unroll
        for (int o = 1; o < B; o <<= 1) {
#pragma unroll
          for (int j = 0; j < 8; ++j) m[j] = fmaxf(m[j], __shfl_xor_sync(0xffffffffu, m[j], o));
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) e[j] = m[j] == kNegInf ? 0.f : ex2(x[j] - m[j]);
        // Block sums: plain butterfly steps down to 8 lanes, then three
        // transposing steps, each keeping the half of the columns picked by
        // the lane bit (and the matching maxima, which need no exchange).
#pragma unroll
        for (int o = B / 2; o >= 8; o >>= 1) {
#pragma unroll
          for (int j = 0; j < 8; ++j) e[j] += __shfl_xor_sync(0xffffffffu, e[j], o);
        }
#pragma unroll
        for (int s2 = 4; s2 >= 1; s2 >>= 1) {
          const bool upper = (lane & s2) != 0;
#pragma unroll
          for (int t = 0; t < s2; ++t) {
            const float send = upper ? e[t] : e[t + s2];
            e[t] = (upper ? e[t + s2] : e[t]) + __shfl_xor_sync(0xffffffffu, send, s2);
            m[t] = upper ? m[t + s2] : m[t];
          }
        }
        const float sum = e[0], mq = m[0];                     // query j0 + qsel of this block
        const int c = grp * kHalf + j0 + qsel;
        const int p = sm.pos[c];
        const bool visible = full && p >= 0 && gid < p / B - 1 && c < a.queries && mq != kNegInf;
        if (finisher && c < a.queries && g < a.groups) {
          const float sb2 = visible ? mq + lg2(sum) : kNegInf;
          a.scores[((static_cast<int64_t>(batch) * a.queries + c) * a.heads + head) * a.groups + g] =
              visible ? sb2 * 0.6931471805599453f : kNegInf;
          if (visible) {
            const int gi = j0 / 8;
            if (sb2 > zm[gi]) {
              zs[gi] = zs[gi] * ex2(zm[gi] - sb2) + 1.f;
              zm[gi] = sb2;
            } else {
              zs[gi] += ex2(sb2 - zm[gi]);
            }
          }
        }
      }
    }
    // Combine owners and warps: per query, the (max, sum) pairs of up to
    // 4 warps x (32 / B) owners of this warpgroup.
    constexpr int kOwners = 32 / B;
    __shared__ float zpart[2][4 * kOwners][kHalf][2];
    if (finisher) {
#pragma unroll
      for (int gi = 0; gi < kGroups; ++gi) {
        zpart[grp][w * kOwners + lane / B][gi * 8 + qsel][0] = zm[gi];
        zpart[grp][w * kOwners + lane / B][gi * 8 + qsel][1] = zs[gi];
      }
    }
    asm volatile("bar.sync 1, 256;" ::: "memory");
    const int t = threadIdx.x - 128;
    if (t < N) {
      const int gg = t / kHalf, j = t % kHalf;
      float m = kNegInf;
      for (int o = 0; o < 4 * kOwners; ++o) m = fmaxf(m, zpart[gg][o][j][0]);
      float sum = 0.f;
      if (m != kNegInf)
        for (int o = 0; o < 4 * kOwners; ++o)
          if (zpart[gg][o][j][0] != kNegInf) sum += zpart[gg][o][j][1] * ex2(zpart[gg][o][j][0] - m);
      if (t < a.queries)
        a.zr_part[((static_cast<int64_t>(batch) * a.queries + t) * a.heads + head) * a.ctas + blockIdx.x] =
            m == kNegInf ? kNegInf : (m + lg2(sum)) * 0.6931471805599453f;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(tmem, kCols);
  }
}

// ---------------------------------------------------------------------------
// per-row top-k by radix select + bitonic sort; log Z_R from the CTA parts
// ---------------------------------------------------------------------------

constexpr int kSelThreads = 512;
constexpr int kMaxK = 1024;

EB_DEVICE uint32_t order_key(float f) {
  const uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

constexpr int kSelPerThread = 8;                       // segment values held in registers per thread
constexpr int kSelWarps = kSelThreads / 32;

// Exclusive prefix (and total) of one count per thread over the CTA, in
// thread order; `scratch` holds kSelWarps + 1 ints.
EB_DEVICE int block_exclusive_scan(int value, int* scratch, int& total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int incl = value;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += y;
  }
  if (lane == 31) scratch[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    int w = lane < kSelWarps ? scratch[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += y;
    }
    if (lane < kSelWarps) scratch[lane] = w;      // inclusive warp totals
    if (lane == kSelWarps - 1) scratch[kSelWarps] = w;
  }
  __syncthreads();
  const int before = (warp > 0 ? scratch[warp - 1] : 0) + incl - value;
  total = scratch[kSelWarps];
  __syncthreads();
  return before;
}

// Top-k of one segment of `len` values (row `blockIdx.y`, segment `blockIdx.x`
// of `seg_len`, at most kSelThreads * kSelPerThread values): the segment is
// read once into registers (value i of the segment is element i / kSelThreads
// of thread i % kSelThreads), a 4-pass radix select over the order-preserving
// integer image finds the k-th largest key (each pass: a shared histogram,
// then one warp scans the 256 digit counts), the winners are gathered by
// prefix counts in position order (ties at the threshold: lowest positions
// first) and sorted by (score desc, index asc) with a bitonic network.
// `idx_in` (nullable) maps positions to the indices used for ties and output.
__global__ void __launch_bounds__(kSelThreads)
topk_select_kernel(const float* __restrict__ values, const int* __restrict__ idx_in, int row_len, int seg_len, int k,
                   float* __restrict__ out_v, int* __restrict__ out_i, int64_t* __restrict__ out_ids, int64_t id_base) {
  __shared__ uint32_t hist[256];
  __shared__ uint32_t sel_prefix;
  __shared__ int sel_remaining;
  __shared__ int scan_scratch[kSelWarps + 1];
  __shared__ float cand_v[kMaxK];
  __shared__ int cand_i[kMaxK];
  const int64_t row = blockIdx.y;
  const int seg = blockIdx.x, segs = gridDim.x;
  const int lo = seg * seg_len;
  const int len = max(0, min(seg_len, row_len - lo));
  const float* x = values + row * row_len + lo;
  const int* ix = idx_in != nullptr ? idx_in + row * row_len + lo : nullptr;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int kk = min(k, len);
  uint32_t keys[kSelPerThread];
#pragma unroll
  for (int j = 0; j < kSelPerThread; ++j) {
    const int i = j * kSelThreads + tid;
    keys[j] = i < len ? order_key(x[i]) : 0u;     // 0 sorts below every real key
  }
  uint32_t prefix = 0, mask = 0;
  int remaining = kk;
  for (int shift = 24; shift >= 0 && kk > 0; shift -= 8) {
    for (int i = tid; i < 256; i += kSelThreads) hist[i] = 0;
    __syncthreads();
#pragma unroll
    for (int j = 0; j < kSelPerThread; ++j) {
      const int i = j * kSelThreads + tid;
      if (i < len && (keys[j] & mask) == prefix) atomicAdd(&hist[(keys[j] >> shift) & 255u], 1u);
    }
    __syncthreads();
    if (warp == 0) {
      // Counts from the top digit down: lane l holds digits 255 - 8l .. 248 - 8l.
      int c[8], sum = 0;
#pragma unroll
      for (int t = 0; t < 8; ++t) {
        c[t] = static_cast<int>(hist[255 - (8 * lane + t)]);
        sum += c[t];
      }
      int incl = sum;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += y;
      }
      const int excl = incl - sum;
      // The digit where the running count (from the top) first reaches `remaining`.
      const bool mine = excl < remaining && incl >= remaining;
      if (mine) {
        int acc = excl;
        int t = 0;
        for (; t < 7; ++t) {
          if (acc + c[t] >= remaining) break;
          acc += c[t];
        }
        sel_prefix = prefix | (static_cast<uint32_t>(255 - (8 * lane + t)) << shift);
        sel_remaining = remaining - acc;
      }
    }
    __syncthreads();
    prefix = sel_prefix;
    remaining = sel_remaining;
    mask |= 255u << shift;
    __syncthreads();
  }
  const int take_eq = remaining;
  const int gt_total = kk - take_eq;
  // Gather in position order: values above the threshold, then the first
  // `take_eq` equal to it.
  int base_gt = 0, base_eq = 0;
#pragma unroll
  for (int j = 0; j < kSelPerThread; ++j) {
    const int i = j * kSelThreads + tid;
    const bool valid = i < len && kk > 0;
    const bool gt = valid && keys[j] > prefix, eq = valid && keys[j] == prefix;
    int total_gt = 0, total_eq = 0;
    const int rank_gt = block_exclusive_scan(gt ? 1 : 0, scan_scratch, total_gt);
    const int rank_eq = block_exclusive_scan(eq ? 1 : 0, scan_scratch, total_eq);
    if (gt) {
      cand_v[base_gt + rank_gt] = x[i];
      cand_i[base_gt + rank_gt] = ix != nullptr ? ix[i] : lo + i;
    }
    if (eq && base_eq + rank_eq < take_eq) {
      cand_v[gt_total + base_eq + rank_eq] = x[i];
      cand_i[gt_total + base_eq + rank_eq] = ix != nullptr ? ix[i] : lo + i;
    }
    base_gt += total_gt;
    base_eq += total_eq;
  }
  __syncthreads();
  int n2 = 1;
  while (n2 < k) n2 <<= 1;
  for (int i = kk + tid; i < n2; i += kSelThreads) {
    cand_v[i] = kNegInf;
    cand_i[i] = 0x7fffffff;
  }
  __syncthreads();
  for (int size = 2; size <= n2; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int i = tid; i < n2; i += kSelThreads) {
        const int j = i ^ stride;
        if (j > i) {
          const bool desc = (i & size) == 0;
          const float vi = cand_v[i], vj = cand_v[j];
          const int ii = cand_i[i], ij = cand_i[j];
          const bool i_first = vi > vj || (vi == vj && ii < ij);
          if (desc != i_first) {
            cand_v[i] = vj;
            cand_v[j] = vi;
            cand_i[i] = ij;
            cand_i[j] = ii;
          }
        }
      }
      __syncthreads();
    }
  }
  const int64_t out_base = (row * segs + seg) * static_cast<int64_t>(k);
  for (int i = tid; i < k; i += kSelThreads) {
    if (out_v != nullptr) out_v[out_base + i] = cand_v[i];
    if (out_i != nullptr) out_i[out_base + i] = cand_i[i];
    if (out_ids != nullptr) out_ids[out_base + i] = id_base + cand_i[i];
  }
}

// log Z_R of each row from the scoring CTAs' parts (natural-log units).
__global__ void zr_combine_kernel(const float* __restrict__ zr_part, int ctas, int rows, float* __restrict__ zr) {
  const int row = blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  float m = kNegInf;
  for (int i = lane; i < ctas; i += 32) m = fmaxf(m, zr_part[static_cast<int64_t>(row) * ctas + i]);
  m = warp_max(m);
  float s = 0.f;
  for (int i = lane; i < ctas; i += 32) {
    const float v = zr_part[static_cast<int64_t>(row) * ctas + i];
    s += v == kNegInf ? 0.f : expf(v - m);
  }
  s = warp_sum(s);
  if (lane == 0) zr[row] = (m == kNegInf || s <= 0.f) ? kNegInf : m + logf(s);
}

template <int D, int N, int B>
void launch_scores(const at::Tensor& q, const at::Tensor& k, ScoreArgs& args, int batch, int heads,
                   cudaStream_t stream) {
  CUtensorMap tq = make_bhld_map(q.data_ptr(), batch, q.size(1), heads, D, N);
  CUtensorMap tk = make_bhld_map(k.data_ptr(), batch, k.size(1), heads, D, kTile);
  const size_t smem = sizeof(ScoreSmem<D, N>) + 1024;
  auto kernel = block_scores_tc_kernel<D, N, B>;
  EB_CUDA_CHECK(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
  kernel<<<dim3(args.ctas, batch * heads), kThreads, smem, stream>>>(tq, tk, args);
}

template <int D, int N>
void dispatch_block(const at::Tensor& q, const at::Tensor& k, ScoreArgs& args, int batch, int heads, int block,
                    cudaStream_t stream) {
  if (block == 16) launch_scores<D, N, 16>(q, k, args, batch, heads, stream);
  else launch_scores<D, N, 32>(q, k, args, batch, heads, stream);
}

template <int D>
void dispatch_n(const at::Tensor& q, const at::Tensor& k, ScoreArgs& args, int batch, int heads, int block,
                cudaStream_t stream) {
  const int n = q.size(1);
  if (n <= 16) dispatch_block<D, 16>(q, k, args, batch, heads, block, stream);
  else dispatch_block<D, 32>(q, k, args, batch, heads, block, stream);
}

}  // namespace

bool block_scores_tc_supported(const at::Tensor& q, const at::Tensor& k, int64_t block, int64_t topk) {
  const int64_t d = q.size(3);
  return q.is_cuda() && q.scalar_type() == at::kBFloat16 && k.scalar_type() == at::kBFloat16 && q.is_contiguous() &&
         k.is_contiguous() && (d == 64 || d == 128) && (block == 16 || block == 32) && q.size(1) <= 32 &&
         topk >= 1 && topk <= kMaxK;
}

// Exact block scores over k (tokens [first, first + keys)), log Z_R and the
// top-k per (batch, query, head): returns (scores [B,Q,H,k'], ids, log_zr)
// with k' = min(topk, blocks), like torch.topk + logsumexp over the scores.
std::vector<at::Tensor> block_scores_topk_tc(const at::Tensor& q, const at::Tensor& k, const at::Tensor& pos,
                                             int64_t block, int64_t first, int64_t topk) {
  TORCH_CHECK(block_scores_tc_supported(q, k, block, topk), "block_scores_topk_tc: unsupported shape");
  TORCH_CHECK(pos.scalar_type() == at::kInt && pos.is_contiguous(), "positions int32");
  TORCH_CHECK(first % block == 0, "first must be block aligned");
  const c10::cuda::CUDAGuard guard(q.device());
  const int batch = q.size(0), queries = q.size(1), heads = q.size(2), dim = q.size(3);
  const int keys = k.size(1);
  const int groups = (keys + block - 1) / block;
  const int tiles = (keys + kTile - 1) / kTile;
  int sms = 0;
  EB_CUDA_CHECK(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, q.device().index()));
  const int want = std::max(1, 2 * sms / std::max(1, batch * heads));
  const int per = std::max(4, (tiles + want - 1) / want);
  const int ctas = std::max(1, (tiles + per - 1) / per);
  auto fopt = q.options().dtype(at::kFloat);
  auto scores = at::empty({batch, queries, heads, groups}, fopt);
  auto zr_part = at::empty({batch, queries, heads, ctas}, fopt);
  ScoreArgs args{pos.data_ptr<int>(), scores.data_ptr<float>(), zr_part.data_ptr<float>(), queries, heads, keys,
                 static_cast<int>(block), groups, tiles, per, ctas, first, 1.f / std::sqrt(static_cast<float>(dim)),
                 device_error_slot(q.device().index())};
  auto stream = at::cuda::getCurrentCUDAStream();
  if (dim == 64) dispatch_n<64>(q, k, args, batch, heads, static_cast<int>(block), stream);
  else dispatch_n<128>(q, k, args, batch, heads, static_cast<int>(block), stream);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  const int64_t kk = std::min<int64_t>(topk, groups);
  auto top = at::empty({batch, queries, heads, kk}, fopt);
  auto ids = at::empty({batch, queries, heads, kk}, q.options().dtype(at::kLong));
  auto zr = at::empty({batch, queries, heads}, fopt);
  const int rows = batch * queries * heads;
  // Top-kk of every segment of kSegLen scores (a selection CTA holds at most
  // kSelThreads * kSelPerThread values), then of the segments' winners, level
  // by level until one segment remains.
  constexpr int kSegLen = kSelThreads * kSelPerThread;
  at::Tensor level_v = scores, level_i;
  int len = groups;
  int launches = 1;
  while (true) {
    const int segs = (len + kSegLen - 1) / kSegLen;
    const int* idx = level_i.defined() ? level_i.data_ptr<int>() : nullptr;
    if (segs == 1) {
      topk_select_kernel<<<dim3(1, rows), kSelThreads, 0, stream>>>(level_v.data_ptr<float>(), idx, len, len,
                                                                     static_cast<int>(kk), top.data_ptr<float>(),
                                                                     nullptr, ids.data_ptr<int64_t>(), first / block);
      ++launches;
      break;
    }
    auto next_v = at::empty({rows, segs, kk}, fopt);
    auto next_i = at::empty({rows, segs, kk}, q.options().dtype(at::kInt));
    topk_select_kernel<<<dim3(segs, rows), kSelThreads, 0, stream>>>(
        level_v.data_ptr<float>(), idx, len, kSegLen, static_cast<int>(kk), next_v.data_ptr<float>(),
        next_i.data_ptr<int>(), nullptr, 0);
    ++launches;
    level_v = next_v;
    level_i = next_i;
    len = static_cast<int>(segs * kk);
  }
  zr_combine_kernel<<<(rows + 7) / 8, 256, 0, stream>>>(zr_part.data_ptr<float>(), ctas, rows, zr.data_ptr<float>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  count_launch(launches + 1);
  return {top, ids, zr};
}

}  // namespace eb
