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
    // Running base-2 (max, sum) of this CTA's visible block scores per query;
    // only block-owner lanes (lane % B == 0) accumulate.
    float zm[kHalf], zs[kHalf];
#pragma unroll
    for (int c = 0; c < kHalf; ++c) {
      zm[c] = kNegInf;
      zs[c] = 0.f;
    }
    const bool owner = (lane % B) == 0;
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
      // Eight query columns at a time, each reduction step issued for all
      // eight before the next, so the shuffle latencies overlap.
#pragma unroll
      for (int j0 = 0; j0 < kHalf; j0 += 8) {
        float x[8], m[8], e[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          x[j] = key < a.keys ? __uint_as_float(r[j0 + j]) * scale2 : kNegInf;
          m[j] = x[j];
        }
#pragma unroll
        for (int o = 1; o < B; o <<= 1) {
#pragma unroll
          for (int j = 0; j < 8; ++j) m[j] = fmaxf(m[j], __shfl_xor_sync(0xffffffffu, m[j], o));
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) e[j] = m[j] == kNegInf ? 0.f : ex2(x[j] - m[j]);
#pragma unroll
        for (int o = 1; o < B; o <<= 1) {
#pragma unroll
          for (int j = 0; j < 8; ++j) e[j] += __shfl_xor_sync(0xffffffffu, e[j], o);
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const int jj = j0 + j;
          const int c = grp * kHalf + jj;
          const int p = sm.pos[c];
          const bool visible = full && p >= 0 && gid < p / B - 1 && c < a.queries && m[j] != kNegInf;
          if (owner && c < a.queries && g < a.groups) {
            const float sb2 = visible ? m[j] + lg2(e[j]) : kNegInf;
            a.scores[((static_cast<int64_t>(batch) * a.queries + c) * a.heads + head) * a.groups + g] =
                visible ? sb2 * 0.6931471805599453f : kNegInf;
            if (visible) {
              if (sb2 > zm[jj]) {
                zs[jj] = zs[jj] * ex2(zm[jj] - sb2) + 1.f;
                zm[jj] = sb2;
              } else {
                zs[jj] += ex2(sb2 - zm[jj]);
              }
            }
          }
        }
      }
    }
    // Combine owners and warps: per query, the (max, sum) pairs of up to
    // 4 warps x (32 / B) owners of this warpgroup.
    constexpr int kOwners = 32 / B;
    __shared__ float zpart[2][4 * kOwners][kHalf][2];
    if (owner) {
#pragma unroll
      for (int j = 0; j < kHalf; ++j) {
        zpart[grp][w * kOwners + lane / B][j][0] = zm[j];
        zpart[grp][w * kOwners + lane / B][j][1] = zs[j];
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

// Top-k of one segment of `len` values (row `blockIdx.y`, segment `blockIdx.x`
// of `seg_len`): radix select of the k-th largest order key, then the winners
// sorted by (score desc, index asc). `idx_in` (nullable) maps positions to
// the indices used for ties and output; candidates beyond `len` are padding.
__global__ void __launch_bounds__(kSelThreads)
topk_select_kernel(const float* __restrict__ values, const int* __restrict__ idx_in, int row_len, int seg_len, int k,
                   float* __restrict__ out_v, int* __restrict__ out_i, int64_t* __restrict__ out_ids, int64_t id_base) {
  __shared__ uint32_t hist[256];
  __shared__ uint32_t sel_prefix;
  __shared__ int sel_remaining, n_gt;
  __shared__ float cand_v[kMaxK];
  __shared__ int cand_i[kMaxK];
  const int64_t row = blockIdx.y;
  const int seg = blockIdx.x, segs = gridDim.x;
  const int lo = seg * seg_len;
  const int len = max(0, min(seg_len, row_len - lo));
  const float* x = values + row * row_len + lo;
  const int* ix = idx_in != nullptr ? idx_in + row * row_len + lo : nullptr;
  const int tid = threadIdx.x;
  const int kk = min(k, len);
  uint32_t prefix = 0, mask = 0;
  int remaining = kk;
  for (int shift = 24; shift >= 0 && kk > 0; shift -= 8) {
    for (int i = tid; i < 256; i += kSelThreads) hist[i] = 0;
    __syncthreads();
    for (int i = tid; i < len; i += kSelThreads) {
      const uint32_t key = order_key(x[i]);
      if ((key & mask) == prefix) atomicAdd(&hist[(key >> shift) & 255u], 1u);
    }
    __syncthreads();
    if (tid == 0) {
      int acc = 0, digit = 255;
      for (; digit > 0; --digit) {
        if (acc + static_cast<int>(hist[digit]) >= remaining) break;
        acc += hist[digit];
      }
      sel_prefix = prefix | (static_cast<uint32_t>(digit) << shift);
      sel_remaining = remaining - acc;
    }
    __syncthreads();
    prefix = sel_prefix;
    remaining = sel_remaining;
    mask |= 255u << shift;
    __syncthreads();
  }
  if (tid == 0) n_gt = 0;
  __syncthreads();
  const int take_eq = remaining;
  const int gt_total = kk - take_eq;
  for (int i = tid; i < len && kk > 0; i += kSelThreads) {
    const uint32_t key = order_key(x[i]);
    if (key > prefix) {
      const int slot = atomicAdd(&n_gt, 1);
      cand_v[slot] = x[i];
      cand_i[slot] = ix != nullptr ? ix[i] : lo + i;
    }
  }
  __syncthreads();
  if (tid < 32 && kk > 0) {   // ties at the threshold: lowest positions first
    int taken = 0;
    for (int base = 0; base < len && taken < take_eq; base += 32) {
      const int i = base + tid;
      const bool eq = i < len && order_key(x[i]) == prefix;
      const unsigned ballot = __ballot_sync(0xffffffffu, eq);
      const int before = __popc(ballot & ((1u << tid) - 1u));
      if (eq && taken + before < take_eq) {
        cand_v[gt_total + taken + before] = x[i];
        cand_i[gt_total + taken + before] = ix != nullptr ? ix[i] : lo + i;
      }
      taken += __popc(ballot);
    }
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
  // Stage 1: top-kk of each segment of kSegLen block scores; stage 2: of the candidates.
  constexpr int kSegLen = 4096;
  const int segs = (groups + kSegLen - 1) / kSegLen;
  if (segs == 1) {
    topk_select_kernel<<<dim3(1, rows), kSelThreads, 0, stream>>>(scores.data_ptr<float>(), nullptr, groups, groups,
                                                                   static_cast<int>(kk), top.data_ptr<float>(), nullptr,
                                                                   ids.data_ptr<int64_t>(), first / block);
  } else {
    auto cand_v = at::empty({rows, segs, kk}, fopt);
    auto cand_i = at::empty({rows, segs, kk}, q.options().dtype(at::kInt));
    topk_select_kernel<<<dim3(segs, rows), kSelThreads, 0, stream>>>(
        scores.data_ptr<float>(), nullptr, groups, kSegLen, static_cast<int>(kk), cand_v.data_ptr<float>(),
        cand_i.data_ptr<int>(), nullptr, 0);
    const int cand_len = static_cast<int>(segs * kk);
    topk_select_kernel<<<dim3(1, rows), kSelThreads, 0, stream>>>(
        cand_v.data_ptr<float>(), cand_i.data_ptr<int>(), cand_len, cand_len, static_cast<int>(kk),
        top.data_ptr<float>(), nullptr, ids.data_ptr<int64_t>(), first / block);
  }
  zr_combine_kernel<<<(rows + 7) / 8, 256, 0, stream>>>(zr_part.data_ptr<float>(), ctas, rows, zr.data_ptr<float>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  count_launch(segs == 1 ? 3 : 4);
  return {top, ids, zr};
}

}  // namespace eb
