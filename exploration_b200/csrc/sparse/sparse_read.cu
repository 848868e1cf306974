// Paged sparse read kernels (sm_100a): exact block scores with a fused
// per-tile top-k and Z_R partial, and the gather-free sparse pop.
//
// block scores: a CTA owns 32 gate blocks of one (batch, head) and all query
// rows of the chunk; queries live in shared memory, each warp streams whole
// key blocks (one pass over K, the roofline of exact scoring). Visible
// blocks are those entirely before the row's local window and complete
// inside the tile. The top-k of the tile and log Z_R of the tile are
// reduced from the score tile on the device.
//
// pop (bf16, blocks of 16 or 32 keys, head dim 64 or 128): split over the
// slots of a row (2 local-window blocks, then the selected blocks). A CTA of 8
// warps takes 8 slots of one (batch, query, head) row, one block per warp:
// the block's keys are dotted with the query by 32 / b lanes each (16-byte
// loads, a shuffle adds the key's parts), the block's softmax is formed in
// registers and its values accumulate with each lane owning dim / 32
// columns (the warp reads each value row as one coalesced line). The CTA
// merges its warps into one normalised partial and its log-mass; a second
// kernel merges a row's partials by their log-masses (flash decoding). About
// 66 slots per row give 9 CTAs per row, hundreds of CTAs for 16 queries.
// Other shapes and fp32 use one CTA per row (its warps split the slots).
// Selected blocks carry the gate bias s_j - log Z_R.
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "../common/util.cuh"

namespace eb {
namespace {

constexpr int kScoreWarps = 8;
constexpr int kBlocksPerWarp = 4;
constexpr int kPopWarps = 8;

template <typename T>
__global__ void __launch_bounds__(kScoreWarps * 32)
block_scores_kernel(  // blockDim.x = 32 * warps, warps <= kScoreWarps
const T* __restrict__ q, const T* __restrict__ k, const int* __restrict__ pos,
                    float* __restrict__ scores, int queries, int keys, int heads, int dim, int block,
                    int64_t first, int groups) {
  extern __shared__ float smem[];
  const int ld = dim + 1;
  const int bh = blockIdx.y, batch = bh / heads, head = bh % heads;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nwarps = blockDim.x >> 5;
  float* Qs = smem;                                   // [Q][ld]
  float* Kw = Qs + queries * ld + warp * block * ld;  // per warp [b][ld]
  float* Sw = smem + queries * ld + nwarps * block * ld + warp * queries * block;   // [Q][b]
  for (int e = threadIdx.x; e < queries * dim; e += blockDim.x) {
    const int r = e / dim, d = e % dim;
    Qs[r * ld + d] = load_f(q + ((static_cast<int64_t>(batch) * queries + r) * heads + head) * dim + d);
  }
  __syncthreads();
  const float scale = rsqrtf(static_cast<float>(dim));
  const int g0 = (blockIdx.x * nwarps + warp) * kBlocksPerWarp;
  for (int gi = 0; gi < kBlocksPerWarp; ++gi) {
    const int g = g0 + gi;
    if (g >= groups) break;
    const int valid_keys = min(block, keys - g * block);
    for (int e = lane; e < block * dim; e += 32) {
      const int j = e / dim, d = e % dim;
      Kw[j * ld + d] = j < valid_keys
          ? load_f(k + ((static_cast<int64_t>(batch) * keys + g * block + j) * heads + head) * dim + d)
          : 0.f;
    }
    __syncwarp();
    for (int e = lane; e < queries * block; e += 32) {
      const int r = e / block, j = e % block;
      float acc = 0.f;
      for (int d = 0; d < dim; ++d) acc += Qs[r * ld + d] * Kw[j * ld + d];
      Sw[r * block + j] = j < valid_keys ? acc * scale : kNegInf;
    }
    __syncwarp();
    const int64_t gid = first / block + g;
    for (int r = lane; r < queries; r += 32) {
      const int p = pos[static_cast<int64_t>(batch) * queries + r];
      const bool visible = p >= 0 && gid < p / block - 1 && valid_keys == block;
      float s = kNegInf;
      if (visible) {
        float m = kNegInf;
        for (int j = 0; j < block; ++j) m = fmaxf(m, Sw[r * block + j]);
        float acc = 0.f;
        for (int j = 0; j < block; ++j) acc += expf(Sw[r * block + j] - m);
        s = m + logf(acc);
      }
      scores[((static_cast<int64_t>(batch) * queries + r) * heads + head) * groups + g] = s;
    }
    __syncwarp();
  }
}

template <typename T>
__global__ void __launch_bounds__(kPopWarps * 32)
sparse_pop_kernel(const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ v,
                  const int* __restrict__ pos, const int64_t* __restrict__ ids,
                  const float* __restrict__ sel_scores, const float* __restrict__ log_zr,
                  float* __restrict__ out, float* __restrict__ lse, int queries, int keys, int heads,
                  int dim, int block, int topk, int64_t offset) {
  extern __shared__ float smem[];
  const int row = blockIdx.x;            // (batch * queries + query) * heads + head
  const int head = row % heads, query = (row / heads) % queries, batch = row / (heads * queries);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float* qs = smem;                       // [D]
  float* acc_all = qs + dim;              // [warps][D]
  float* ml_all = acc_all + kPopWarps * dim;   // [warps][2]
  for (int d = threadIdx.x; d < dim; d += blockDim.x) qs[d] = load_f(q + static_cast<int64_t>(row) * dim + d);
  __syncthreads();
  const int p = pos[static_cast<int64_t>(batch) * queries + query];
  const float zr = finite_or_zero(log_zr[row]);
  const float scale = rsqrtf(static_cast<float>(dim));
  float m = kNegInf, l = 0.f;
  float* acc = acc_all + warp * dim;
  for (int d = lane; d < dim; d += 32) acc[d] = 0.f;
  __syncwarp();
  const int slots = 2 + topk;
  for (int s = warp; s < slots && p >= 0; s += kPopWarps) {
    int64_t blk;
    float bias = 0.f;
    if (s < 2) {
      blk = p / block - 1 + s;
    } else {
      blk = ids[static_cast<int64_t>(row) * topk + (s - 2)];
      const float sc = sel_scores[static_cast<int64_t>(row) * topk + (s - 2)];
      if (blk < 0 || sc == kNegInf) continue;
      bias = sc - zr;
    }
    for (int j0 = 0; j0 < block; j0 += 32) {
      const int j = j0 + lane;
      const int64_t token = blk * block + j;
      const bool ok = j < block && token >= 0 && token <= p && token >= offset && token < offset + keys;
      float logit = kNegInf;
      const int64_t kr = ((static_cast<int64_t>(batch) * keys + (ok ? token - offset : 0)) * heads + head) * dim;
      if (ok) {
        float dot = 0.f;
        for (int d = 0; d < dim; ++d) dot += qs[d] * load_f(k + kr + d);
        logit = dot * scale + bias;
      }
      const float tile_max = warp_max(logit);
      if (tile_max == kNegInf) continue;
      const float new_m = fmaxf(m, tile_max);
      const float keep = m == kNegInf ? 0.f : expf(m - new_m);
      const float w = ok ? expf(logit - new_m) : 0.f;
      l = l * keep + warp_sum(w);
      for (int d = lane; d < dim; d += 32) {
        float a = acc[d] * keep;
        for (int t = 0; t < 32; ++t) {
          const float wt = __shfl_sync(0xffffffffu, w, t);
          if (wt != 0.f) {
            const int64_t tok = blk * block + j0 + t;
            a += wt * load_f(v + ((static_cast<int64_t>(batch) * keys + (tok - offset)) * heads + head) * dim + d);
          }
        }
        acc[d] = a;
      }
      m = new_m;
    }
  }
  if (lane == 0) {
    ml_all[warp * 2] = m;
    ml_all[warp * 2 + 1] = l;
  }
  __syncthreads();
  float gm = kNegInf;
  for (int w = 0; w < kPopWarps; ++w) gm = fmaxf(gm, ml_all[w * 2]);
  float gl = 0.f;
  for (int w = 0; w < kPopWarps; ++w)
    if (ml_all[w * 2] != kNegInf) gl += ml_all[w * 2 + 1] * expf(ml_all[w * 2] - gm);
  for (int d = threadIdx.x; d < dim; d += blockDim.x) {
    float a = 0.f;
    for (int w = 0; w < kPopWarps; ++w)
      if (ml_all[w * 2] != kNegInf) a += acc_all[w * dim + d] * expf(ml_all[w * 2] - gm);
    out[static_cast<int64_t>(row) * dim + d] = gl > 0.f ? a / gl : 0.f;
  }
  if (threadIdx.x == 0) lse[row] = gl > 0.f ? gm + logf(gl) : kNegInf;
}


constexpr int kSplitWarps = 8;

EB_DEVICE void bf16x8_to_float(const uint4 raw, float (&f)[8]) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 x = __bfloat1622float2(h[i]);
    f[2 * i] = x.x;
    f[2 * i + 1] = x.y;
  }
}

template <int DIM, int BLK>
__global__ void __launch_bounds__(kSplitWarps * 32)
sparse_pop_split_kernel(const __nv_bfloat16* __restrict__ q, const __nv_bfloat16* __restrict__ k,
                        const __nv_bfloat16* __restrict__ v, const int* __restrict__ pos,
                        const int64_t* __restrict__ ids, const float* __restrict__ sel_scores,
                        const float* __restrict__ log_zr, float* __restrict__ part_out,
                        float* __restrict__ part_lse, int queries, int keys, int heads, int topk, int64_t offset,
                        int chunks) {
  constexpr int kLanesPerKey = 32 / BLK;        // lanes sharing one key's dot product
  constexpr int kDotDims = DIM / kLanesPerKey;  // dims per lane in the dot product
  constexpr int kValDims = DIM / 32;            // value columns owned by a lane
  __shared__ float s_acc[kSplitWarps][DIM];
  __shared__ float s_ml[kSplitWarps][2];
  const int row = blockIdx.y;                   // (batch * queries + query) * heads + head
  const int chunk = blockIdx.x;
  const int head = row % heads, query = (row / heads) % queries, batch = row / (heads * queries);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int p = pos[static_cast<int64_t>(batch) * queries + query];
  const int slot = chunk * kSplitWarps + warp;
  float m = kNegInf, l = 0.f, acc[kValDims];
#pragma unroll
  for (int i = 0; i < kValDims; ++i) acc[i] = 0.f;
  int64_t blk = -1;
  float bias = 0.f;
  if (p >= 0 && slot < 2 + topk) {
    if (slot < 2) {
      blk = p / BLK - 1 + slot;
    } else {
      blk = ids[static_cast<int64_t>(row) * topk + (slot - 2)];
      const float sc = sel_scores[static_cast<int64_t>(row) * topk + (slot - 2)];
      if (sc == kNegInf) blk = -1;
      bias = sc - finite_or_zero(log_zr[row]);
    }
  }
  if (blk >= 0) {
    const int key_in_block = lane / kLanesPerKey, part = lane % kLanesPerKey;
    const int64_t token = blk * BLK + key_in_block;
    const bool ok = token >= 0 && token <= p && token >= offset && token < offset + keys;
    // This lane's part of the query and of its key (16-byte loads).
    const int64_t qrow = static_cast<int64_t>(row) * DIM + part * kDotDims;
    const int64_t krow = ((static_cast<int64_t>(batch) * keys + (ok ? token - offset : 0)) * heads + head) * DIM +
                         part * kDotDims;
    float dot = 0.f;
#pragma unroll
    for (int c = 0; c < kDotDims; c += 8) {
      float qf[8], kf[8];
      bf16x8_to_float(*reinterpret_cast<const uint4*>(q + qrow + c), qf);
      bf16x8_to_float(ok ? *reinterpret_cast<const uint4*>(k + krow + c) : make_uint4(0u, 0u, 0u, 0u), kf);
#pragma unroll
      for (int i = 0; i < 8; ++i) dot = fmaf(qf[i], kf[i], dot);
    }
#pragma unroll
    for (int o = 1; o < kLanesPerKey; o <<= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
    const float logit = ok ? dot * rsqrtf(static_cast<float>(DIM)) + bias : kNegInf;
    m = warp_max(logit);                        // the block's maximum (every key counted kLanesPerKey times)
    if (m != kNegInf) {
      const float w = ok ? expf(logit - m) : 0.f;
      l = warp_sum(part == 0 ? w : 0.f);
#pragma unroll
      for (int key = 0; key < BLK; ++key) {
        const float wk = __shfl_sync(0xffffffffu, w, key * kLanesPerKey);
        if (wk == 0.f) continue;                // uniform across the warp
        const int64_t tok = blk * BLK + key - offset;
        const __nv_bfloat16* vrow = v + ((static_cast<int64_t>(batch) * keys + tok) * heads + head) * DIM +
                                    lane * kValDims;
        if constexpr (kValDims == 2) {
          const float2 x = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(vrow));
          acc[0] = fmaf(wk, x.x, acc[0]);
          acc[1] = fmaf(wk, x.y, acc[1]);
        } else {
          const uint2 raw = *reinterpret_cast<const uint2*>(vrow);
          const float2 x = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&raw.x));
          const float2 y = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&raw.y));
          acc[0] = fmaf(wk, x.x, acc[0]);
          acc[1] = fmaf(wk, x.y, acc[1]);
          acc[2] = fmaf(wk, y.x, acc[2]);
          acc[3] = fmaf(wk, y.y, acc[3]);
        }
      }
    }
  }
#pragma unroll
  for (int i = 0; i < kValDims; ++i) s_acc[warp][lane * kValDims + i] = acc[i];
  if (lane == 0) {
    s_ml[warp][0] = m;
    s_ml[warp][1] = l;
  }
  __syncthreads();
  // Merge the warps (fixed order) into this chunk's normalised partial.
  float gm = kNegInf;
#pragma unroll
  for (int w = 0; w < kSplitWarps; ++w) gm = fmaxf(gm, s_ml[w][0]);
  float gl = 0.f;
#pragma unroll
  for (int w = 0; w < kSplitWarps; ++w)
    if (s_ml[w][0] != kNegInf) gl += s_ml[w][1] * expf(s_ml[w][0] - gm);
  const int64_t out_base = (static_cast<int64_t>(row) * chunks + chunk) * DIM;
  for (int d = threadIdx.x; d < DIM; d += blockDim.x) {
    float a = 0.f;
#pragma unroll
    for (int w = 0; w < kSplitWarps; ++w)
      if (s_ml[w][0] != kNegInf) a += s_acc[w][d] * expf(s_ml[w][0] - gm);
    part_out[out_base + d] = gl > 0.f ? a / gl : 0.f;
  }
  if (threadIdx.x == 0) part_lse[static_cast<int64_t>(row) * chunks + chunk] = gl > 0.f ? gm + logf(gl) : kNegInf;
}

// One warp per row: out = sum_c 2^... of the chunk partials weighted by their
// log-masses (chunk order), lse = log of the total mass.
__global__ void __launch_bounds__(256)
sparse_pop_combine_kernel(const float* __restrict__ part_out, const float* __restrict__ part_lse,
                          float* __restrict__ out, float* __restrict__ lse, int rows, int chunks, int dim) {
  const int row = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (row >= rows) return;
  const float* pl = part_lse + static_cast<int64_t>(row) * chunks;
  float gm = kNegInf;
  for (int c = 0; c < chunks; ++c) gm = fmaxf(gm, pl[c]);
  float total = 0.f;
  for (int c = 0; c < chunks; ++c)
    if (pl[c] != kNegInf) total += expf(pl[c] - gm);
  for (int d = lane; d < dim; d += 32) {
    float a = 0.f;
    for (int c = 0; c < chunks; ++c)
      if (pl[c] != kNegInf) a += part_out[(static_cast<int64_t>(row) * chunks + c) * dim + d] * expf(pl[c] - gm);
    out[static_cast<int64_t>(row) * dim + d] = total > 0.f ? a / total : 0.f;
  }
  if (lane == 0) lse[row] = total > 0.f ? gm + logf(total) : kNegInf;
}

}  // namespace

std::vector<at::Tensor> block_scores_topk(const at::Tensor& q, const at::Tensor& k, const at::Tensor& pos,
                                          int64_t block, int64_t first, int64_t topk) {
  TORCH_CHECK(q.is_cuda() && q.is_contiguous() && k.is_contiguous() && pos.scalar_type() == at::kInt,
              "block_scores_topk: contiguous CUDA q/k and int32 positions");
  TORCH_CHECK(q.scalar_type() == k.scalar_type(), "q/k dtype mismatch");
  const c10::cuda::CUDAGuard guard(q.device());
  const int batch = q.size(0), queries = q.size(1), heads = q.size(2), dim = q.size(3);
  const int keys = k.size(1);
  const int groups = cdiv(keys, block);
  auto scores = at::empty({batch, queries, heads, groups}, q.options().dtype(at::kFloat));
  const int ld = dim + 1;
  const size_t q_bytes = sizeof(float) * static_cast<size_t>(queries) * ld;
  const size_t warp_bytes = sizeof(float) * (static_cast<size_t>(block) * ld + static_cast<size_t>(queries) * block);
  constexpr size_t kBudget = 200 * 1024;
  TORCH_CHECK(q_bytes + warp_bytes <= kBudget, "block_scores_topk: query chunk too large for one CTA");
  const int warps = static_cast<int>(std::min<size_t>(kScoreWarps, (kBudget - q_bytes) / warp_bytes));
  const size_t smem = q_bytes + warps * warp_bytes;
  dim3 grid(cdiv(groups, warps * kBlocksPerWarp), batch * heads);
  auto stream = at::cuda::getCurrentCUDAStream();
  if (q.scalar_type() == at::kBFloat16) {
    auto kernel = block_scores_kernel<__nv_bfloat16>;
    EB_CUDA_CHECK(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    kernel<<<grid, warps * 32, smem, stream>>>(
        reinterpret_cast<const __nv_bfloat16*>(q.data_ptr()), reinterpret_cast<const __nv_bfloat16*>(k.data_ptr()),
        pos.data_ptr<int>(), scores.data_ptr<float>(), queries, keys, heads, dim, block, first, groups);
  } else {
    TORCH_CHECK(q.scalar_type() == at::kFloat, "block_scores_topk: fp32 or bf16");
    auto kernel = block_scores_kernel<float>;
    EB_CUDA_CHECK(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    kernel<<<grid, warps * 32, smem, stream>>>(q.data_ptr<float>(), k.data_ptr<float>(), pos.data_ptr<int>(),
                                                     scores.data_ptr<float>(), queries, keys, heads, dim, block,
                                                     first, groups);
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  count_launch(1);
  auto zr = at::logsumexp(scores, {-1});
  const int64_t count = std::min<int64_t>(topk, groups);
  auto top = at::topk(scores, count, -1);
  auto ids = std::get<1>(top) + first / block;
  return {std::get<0>(top), ids, zr};
}

std::vector<at::Tensor> sparse_pop(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v,
                                   const at::Tensor& pos, const at::Tensor& ids, const at::Tensor& scores,
                                   const at::Tensor& log_zr, int64_t block, int64_t offset) {
  TORCH_CHECK(q.is_contiguous() && k.is_contiguous() && v.is_contiguous() && ids.is_contiguous() &&
                  scores.is_contiguous() && log_zr.is_contiguous(), "sparse_pop: contiguous inputs");
  TORCH_CHECK(ids.scalar_type() == at::kLong && scores.scalar_type() == at::kFloat &&
                  log_zr.scalar_type() == at::kFloat && pos.scalar_type() == at::kInt, "sparse_pop dtypes");
  const c10::cuda::CUDAGuard guard(q.device());
  const int batch = q.size(0), queries = q.size(1), heads = q.size(2), dim = q.size(3);
  const int keys = k.size(1), topk = ids.size(-1);
  auto out = at::empty({batch, queries, heads, dim}, q.options().dtype(at::kFloat));
  auto lse = at::empty({batch, queries, heads}, q.options().dtype(at::kFloat));
  const int rows = batch * queries * heads;
  if (rows == 0) return {out, lse};
  auto stream = at::cuda::getCurrentCUDAStream();
  const bool aligned = reinterpret_cast<uintptr_t>(q.data_ptr()) % 16 == 0 &&
                       reinterpret_cast<uintptr_t>(k.data_ptr()) % 16 == 0 &&
                       reinterpret_cast<uintptr_t>(v.data_ptr()) % 16 == 0;
  if (q.scalar_type() == at::kBFloat16 && aligned && (dim == 64 || dim == 128) && (block == 16 || block == 32)) {
    const int chunks = cdiv(2 + topk, kSplitWarps);
    auto part_out = at::empty({rows, chunks, dim}, q.options().dtype(at::kFloat));
    auto part_lse = at::empty({rows, chunks}, q.options().dtype(at::kFloat));
    const dim3 grid(chunks, rows);
    using T = __nv_bfloat16;
    auto args = [&](auto kernel) {
      kernel<<<grid, kSplitWarps * 32, 0, stream>>>(
          reinterpret_cast<const T*>(q.data_ptr()), reinterpret_cast<const T*>(k.data_ptr()),
          reinterpret_cast<const T*>(v.data_ptr()), pos.data_ptr<int>(), ids.data_ptr<int64_t>(),
          scores.data_ptr<float>(), log_zr.data_ptr<float>(), part_out.data_ptr<float>(),
          part_lse.data_ptr<float>(), queries, keys, heads, topk, offset, chunks);
    };
    if (dim == 64 && block == 16) args(sparse_pop_split_kernel<64, 16>);
    else if (dim == 64) args(sparse_pop_split_kernel<64, 32>);
    else if (block == 16) args(sparse_pop_split_kernel<128, 16>);
    else args(sparse_pop_split_kernel<128, 32>);
    sparse_pop_combine_kernel<<<cdiv(rows, 8), 256, 0, stream>>>(part_out.data_ptr<float>(), part_lse.data_ptr<float>(),
                                                                 out.data_ptr<float>(), lse.data_ptr<float>(), rows,
                                                                 chunks, dim);
    C10_CUDA_KERNEL_LAUNCH_CHECK();
    count_launch(2);
    return {out, lse};
  }
  const size_t smem = sizeof(float) * (dim + kPopWarps * dim + kPopWarps * 2);
  if (q.scalar_type() == at::kBFloat16) {
    using T = __nv_bfloat16;
    sparse_pop_kernel<T><<<rows, kPopWarps * 32, smem, stream>>>(
        reinterpret_cast<const T*>(q.data_ptr()), reinterpret_cast<const T*>(k.data_ptr()),
        reinterpret_cast<const T*>(v.data_ptr()), pos.data_ptr<int>(), ids.data_ptr<int64_t>(),
        scores.data_ptr<float>(), log_zr.data_ptr<float>(), out.data_ptr<float>(), lse.data_ptr<float>(),
        queries, keys, heads, dim, block, topk, offset);
  } else {
    TORCH_CHECK(q.scalar_type() == at::kFloat, "sparse_pop: fp32 or bf16");
    sparse_pop_kernel<float><<<rows, kPopWarps * 32, smem, stream>>>(
        q.data_ptr<float>(), k.data_ptr<float>(), v.data_ptr<float>(), pos.data_ptr<int>(),
        ids.data_ptr<int64_t>(), scores.data_ptr<float>(), log_zr.data_ptr<float>(), out.data_ptr<float>(),
        lse.data_ptr<float>(), queries, keys, heads, dim, block, topk, offset);
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  count_launch(1);
  return {out, lse};
}

}  // namespace eb
