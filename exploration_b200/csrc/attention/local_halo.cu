// Local halo window attention with fused rotary embedding (sm_100a).
//
// Query row r of block g attends to the 2b keys of blocks g-1 and g (window
// column c in [0, 2b)), causally (c <= b + r), restricted to absolute key
// positions in [valid_start, start + n). Block -1 is the halo block passed
// in `prev` (or masked). RoPE is relative to the query block origin: queries
// rotate by r and window keys by c - b, so the kernel reads the raw qkv
// projection and rotates on load (no rotated copy of q/k ever hits HBM).
//
// One CTA owns one (block, head, batch). Forward writes the context and the
// per-row log-sum-exp. Backward is owner-computes and atomic-free: the CTA of
// block g writes dq of query block g and dk/dv of key block g, which collect
// contributions from query blocks g (key at window column b + j) and g + 1
// (key at column j). Rotations compose, so queries of block g + 1 are
// rotated by r + b and every key of block g keeps rotation j.
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <map>
#include <mutex>
#include <tuple>

#include "../common/util.cuh"

namespace eb {
namespace {

constexpr int kLocalThreads = 128;
constexpr int kLocalWarps = kLocalThreads / 32;

struct LocalArgs {
  const void* qkv;     // [B, n, 3, H, D]
  const void* prev;    // [B, b, 3, H, D] or nullptr
  const float* cos;    // [3b, D/2] rotation offsets -b .. 2b-1
  const float* sin;
  int n, heads, dim, block;
  int64_t start, valid_start;
};

template <typename T>
EB_DEVICE const T* qkv_row(const LocalArgs& a, int batch, int token, int part, int head) {
  // token in [-b, n): negative rows come from the halo block.
  const int64_t stride_tok = 3LL * a.heads * a.dim;
  if (token < 0) {
    const T* p = static_cast<const T*>(a.prev);
    return p + (static_cast<int64_t>(batch) * a.block + (token + a.block)) * stride_tok +
           (static_cast<int64_t>(part) * a.heads + head) * a.dim;
  }
  const T* q = static_cast<const T*>(a.qkv);
  return q + (static_cast<int64_t>(batch) * a.n + token) * stride_tok +
         (static_cast<int64_t>(part) * a.heads + head) * a.dim;
}

EB_DEVICE bool key_valid(const LocalArgs& a, int token) {
  const int64_t kp = a.start + token;
  if (token < 0 && a.prev == nullptr) return false;
  return kp >= a.valid_start && kp < a.start + a.n && token < a.n;
}

// Load one D-vector rotated by `offset` (fp32) into smem row `dst`.
template <typename T>
EB_DEVICE void load_rotated(float* dst, const T* src, const LocalArgs& a, int offset, bool valid,
                            int lane_begin, int lane_step) {
  const int half = a.dim / 2;
  const float* cs = a.cos + static_cast<int64_t>(offset + a.block) * half;
  const float* sn = a.sin + static_cast<int64_t>(offset + a.block) * half;
  for (int i = lane_begin; i < half; i += lane_step) {
    float x1 = valid ? load_f(src + i) : 0.f;
    float x2 = valid ? load_f(src + i + half) : 0.f;
    dst[i] = x1 * cs[i] - x2 * sn[i];
    dst[i + half] = x2 * cs[i] + x1 * sn[i];
  }
}

template <typename T>
EB_DEVICE void load_plain(float* dst, const T* src, int dim, bool valid, int lane_begin, int lane_step) {
  for (int i = lane_begin; i < dim; i += lane_step) dst[i] = valid ? load_f(src + i) : 0.f;
}

template <typename T>
__global__ void __launch_bounds__(kLocalThreads)
local_fwd_kernel(LocalArgs a, T* __restrict__ out, float* __restrict__ lse) {
  extern __shared__ float smem[];
  const int g = blockIdx.x, head = blockIdx.y, batch = blockIdx.z;
  const int b = a.block, D = a.dim, ld = D + 1, W = 2 * b;
  float* K = smem;                       // [2b][D+1] rotated keys
  float* V = K + W * ld;                 // [2b][D+1]
  float* Qw = V + W * ld;                // [warps][D]
  float* Pw = Qw + kLocalWarps * D;      // [warps][2b]
  bool* valid = reinterpret_cast<bool*>(Pw + kLocalWarps * W);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // Stage the window: one warp per key row.
  for (int c = warp; c < W; c += kLocalWarps) {
    const int token = (g - 1) * b + c;
    const bool ok = key_valid(a, token);
    if (lane == 0) valid[c] = ok;
    load_rotated(K + c * ld, qkv_row<T>(a, batch, ok ? token : 0, 1, head), a, c - b, ok, lane, 32);
    load_plain(V + c * ld, qkv_row<T>(a, batch, ok ? token : 0, 2, head), D, ok, lane, 32);
  }
  __syncthreads();
  const float scale = rsqrtf(static_cast<float>(D));
  for (int r = warp; r < b; r += kLocalWarps) {
    const int token = g * b + r;
    if (token >= a.n) break;
    float* q = Qw + warp * D;
    load_rotated(q, qkv_row<T>(a, batch, token, 0, head), a, r, true, lane, 32);
    __syncwarp();
    float* p = Pw + warp * W;
    float mx = kNegInf;
    for (int c = lane; c < W; c += 32) {
      float s = kNegInf;
      if (c <= b + r && valid[c]) {
        const float* kr = K + c * ld;
        float acc = 0.f;
        for (int d = 0; d < D; ++d) acc += q[d] * kr[d];
        s = acc * scale;
      }
      p[c] = s;
      mx = fmaxf(mx, s);
    }
    mx = warp_max(mx);
    float sum = 0.f;
    for (int c = lane; c < W; c += 32) {
      float e = p[c] == kNegInf ? 0.f : expf(p[c] - mx);
      p[c] = e;
      sum += e;
    }
    sum = warp_sum(sum);
    __syncwarp();
    const float inv = 1.f / sum;
    T* orow = out + (static_cast<int64_t>(batch) * a.n + token) * a.heads * D + static_cast<int64_t>(head) * D;
    for (int d = lane; d < D; d += 32) {
      float acc = 0.f;
      for (int c = 0; c < W; ++c) acc += p[c] * V[c * ld + d];
      orow[d] = cast_f<T>(acc * inv);
    }
    if (lane == 0) lse[(static_cast<int64_t>(batch) * a.n + token) * a.heads + head] = mx + logf(sum);
    __syncwarp();
  }
}

template <typename T>
__global__ void __launch_bounds__(kLocalThreads)
local_bwd_kernel(LocalArgs a, const T* __restrict__ dout, const T* __restrict__ out,
                 const float* __restrict__ lse, T* __restrict__ dqkv, T* __restrict__ dprev) {
  extern __shared__ float smem[];
  const int g = blockIdx.x, head = blockIdx.y, batch = blockIdx.z;
  const int b = a.block, D = a.dim, ld = D + 1, W = 2 * b;
  const int groups = cdiv(a.n, b);
  const bool has_next = g + 1 < groups;
  float* K = smem;              // [2b][ld] window keys of block g (rotated c - b)
  float* V = K + W * ld;        // [2b][ld]
  float* Q0 = V + W * ld;       // [b][ld] queries of block g (rotated r)
  float* Q1 = Q0 + b * ld;      // [b][ld] queries of block g+1 (rotated r + b)
  float* G0 = Q1 + b * ld;      // [b][ld] dout of block g
  float* G1 = G0 + b * ld;      // [b][ld] dout of block g+1
  float* P0 = G1 + b * ld;      // [b][2b] probabilities, block g
  float* S0 = P0 + b * W;       // [b][2b] dS, block g
  float* P1 = S0 + b * W;       // [b][b] probabilities of block g+1 on keys of block g
  float* S1 = P1 + b * b;       // [b][b]
  bool* valid = reinterpret_cast<bool*>(S1 + b * b);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t row_stride = static_cast<int64_t>(a.heads) * D;
  for (int c = warp; c < W; c += kLocalWarps) {
    const int token = (g - 1) * b + c;
    const bool ok = key_valid(a, token);
    if (lane == 0) valid[c] = ok;
    load_rotated(K + c * ld, qkv_row<T>(a, batch, ok ? token : 0, 1, head), a, c - b, ok, lane, 32);
    load_plain(V + c * ld, qkv_row<T>(a, batch, ok ? token : 0, 2, head), D, ok, lane, 32);
  }
  for (int r = warp; r < b; r += kLocalWarps) {
    const int t0 = g * b + r, t1 = (g + 1) * b + r;
    const bool ok0 = t0 < a.n, ok1 = has_next && t1 < a.n;
    load_rotated(Q0 + r * ld, qkv_row<T>(a, batch, ok0 ? t0 : 0, 0, head), a, r, ok0, lane, 32);
    load_rotated(Q1 + r * ld, qkv_row<T>(a, batch, ok1 ? t1 : 0, 0, head), a, r + b, ok1, lane, 32);
    const T* d0 = dout + (static_cast<int64_t>(batch) * a.n + (ok0 ? t0 : 0)) * row_stride + head * D;
    const T* d1 = dout + (static_cast<int64_t>(batch) * a.n + (ok1 ? t1 : 0)) * row_stride + head * D;
    load_plain(G0 + r * ld, d0, D, ok0, lane, 32);
    load_plain(G1 + r * ld, d1, D, ok1, lane, 32);
  }
  __syncthreads();
  const float scale = rsqrtf(static_cast<float>(D));
  // Probabilities and dS of query block g over its whole window.
  for (int r = warp; r < b; r += kLocalWarps) {
    const int t0 = g * b + r;
    const bool ok0 = t0 < a.n;
    float delta = 0.f, l = 0.f;
    if (ok0) {
      const T* o = out + (static_cast<int64_t>(batch) * a.n + t0) * row_stride + head * D;
      for (int d = lane; d < D; d += 32) delta += G0[r * ld + d] * load_f(o + d);
      delta = warp_sum(delta);
      l = lse[(static_cast<int64_t>(batch) * a.n + t0) * a.heads + head];
    }
    for (int c = lane; c < W; c += 32) {
      float p = 0.f, ds = 0.f;
      if (ok0 && c <= b + r && valid[c]) {
        float s = 0.f, dp = 0.f;
        for (int d = 0; d < D; ++d) {
          s += Q0[r * ld + d] * K[c * ld + d];
          dp += G0[r * ld + d] * V[c * ld + d];
        }
        p = expf(s * scale - l);
        ds = p * (dp - delta);
      }
      P0[r * W + c] = p;
      S0[r * W + c] = ds;
    }
    // Query block g + 1 against the keys of block g (its previous block).
    const int t1 = (g + 1) * b + r;
    const bool ok1 = has_next && t1 < a.n;
    float delta1 = 0.f, l1 = 0.f;
    if (ok1) {
      const T* o = out + (static_cast<int64_t>(batch) * a.n + t1) * row_stride + head * D;
      for (int d = lane; d < D; d += 32) delta1 += G1[r * ld + d] * load_f(o + d);
      delta1 = warp_sum(delta1);
      l1 = lse[(static_cast<int64_t>(batch) * a.n + t1) * a.heads + head];
    }
    for (int j = lane; j < b; j += 32) {
      float p = 0.f, ds = 0.f;
      if (ok1 && valid[b + j]) {
        float s = 0.f, dp = 0.f;
        for (int d = 0; d < D; ++d) {
          s += Q1[r * ld + d] * K[(b + j) * ld + d];
          dp += G1[r * ld + d] * V[(b + j) * ld + d];
        }
        p = expf(s * scale - l1);
        ds = p * (dp - delta1);
      }
      P1[r * b + j] = p;
      S1[r * b + j] = ds;
    }
  }
  __syncthreads();
  const int half = D / 2;
  // dq of block g: un-rotate sum_c dS[r][c] K[c] by offset r.
  for (int r = warp; r < b; r += kLocalWarps) {
    const int t0 = g * b + r;
    if (t0 >= a.n) continue;
    T* dq = dqkv + (static_cast<int64_t>(batch) * a.n + t0) * 3 * row_stride + head * D;
    const float* cs = a.cos + static_cast<int64_t>(r + b) * half;
    const float* sn = a.sin + static_cast<int64_t>(r + b) * half;
    for (int i = lane; i < half; i += 32) {
      float g1 = 0.f, g2 = 0.f;
      for (int c = 0; c < W; ++c) {
        const float w = S0[r * W + c];
        g1 += w * K[c * ld + i];
        g2 += w * K[c * ld + i + half];
      }
      dq[i] = cast_f<T>((g1 * cs[i] + g2 * sn[i]) * scale);
      dq[i + half] = cast_f<T>((g2 * cs[i] - g1 * sn[i]) * scale);
    }
  }
  // dk/dv of block g (offset j) from query blocks g and g + 1.
  for (int j = warp; j < b; j += kLocalWarps) {
    const int tk = g * b + j;
    if (tk >= a.n) continue;
    T* dk = dqkv + (static_cast<int64_t>(batch) * a.n + tk) * 3 * row_stride + row_stride + head * D;
    T* dv = dk + row_stride;
    const float* cs = a.cos + static_cast<int64_t>(j + b) * half;
    const float* sn = a.sin + static_cast<int64_t>(j + b) * half;
    for (int i = lane; i < half; i += 32) {
      float k1 = 0.f, k2 = 0.f, v1 = 0.f, v2 = 0.f;
      for (int r = 0; r < b; ++r) {
        const float w0 = S0[r * W + b + j], w1 = S1[r * b + j];
        k1 += w0 * Q0[r * ld + i] + w1 * Q1[r * ld + i];
        k2 += w0 * Q0[r * ld + i + half] + w1 * Q1[r * ld + i + half];
        const float p0 = P0[r * W + b + j], p1 = P1[r * b + j];
        v1 += p0 * G0[r * ld + i] + p1 * G1[r * ld + i];
        v2 += p0 * G0[r * ld + i + half] + p1 * G1[r * ld + i + half];
      }
      dk[i] = cast_f<T>((k1 * cs[i] + k2 * sn[i]) * scale);
      dk[i + half] = cast_f<T>((k2 * cs[i] - k1 * sn[i]) * scale);
      dv[i] = cast_f<T>(v1);
      dv[i + half] = cast_f<T>(v2);
    }
  }
  // Halo block (keys of block -1) receive gradient from query block 0 only.
  if (g == 0 && dprev != nullptr) {
    for (int j = warp; j < b; j += kLocalWarps) {
      T* dk = dprev + (static_cast<int64_t>(batch) * b + j) * 3 * row_stride + row_stride + head * D;
      T* dv = dk + row_stride;
      const float* cs = a.cos + static_cast<int64_t>(j) * half;   // offset j - b
      const float* sn = a.sin + static_cast<int64_t>(j) * half;
      for (int i = lane; i < half; i += 32) {
        float k1 = 0.f, k2 = 0.f, v1 = 0.f, v2 = 0.f;
        for (int r = 0; r < b; ++r) {
          const float w0 = S0[r * W + j], p0 = P0[r * W + j];
          k1 += w0 * Q0[r * ld + i];
          k2 += w0 * Q0[r * ld + i + half];
          v1 += p0 * G0[r * ld + i];
          v2 += p0 * G0[r * ld + i + half];
        }
        dk[i] = cast_f<T>((k1 * cs[i] + k2 * sn[i]) * scale);
        dk[i + half] = cast_f<T>((k2 * cs[i] - k1 * sn[i]) * scale);
        dv[i] = cast_f<T>(v1);
        dv[i + half] = cast_f<T>(v2);
      }
    }
  }
}

size_t fwd_smem(int b, int D) {
  const int ld = D + 1, W = 2 * b;
  return sizeof(float) * (2 * W * ld + kLocalWarps * D + kLocalWarps * W) + W;
}

size_t bwd_smem(int b, int D) {
  const int ld = D + 1, W = 2 * b;
  return sizeof(float) * (2 * W * ld + 4 * b * ld + 2 * b * W + 2 * b * b) + W;
}

std::pair<at::Tensor, at::Tensor> rope_tables(int block, int dim, const at::Device& device) {
  // Offsets -b .. 2b-1; float32 angles as in the torch reference. Built once
  // per (device, block, dim) and kept, so no host->device copy happens inside
  // a captured CUDA graph.
  static std::mutex lock;
  static auto& cache = *new std::map<std::tuple<int, int, int>, std::pair<at::Tensor, at::Tensor>>();
  const std::lock_guard<std::mutex> guard(lock);
  const auto key = std::make_tuple(static_cast<int>(device.index()), block, dim);
  auto hit = cache.find(key);
  if (hit != cache.end()) return hit->second;
  auto offsets = at::arange(-block, 2 * block, at::TensorOptions().dtype(at::kFloat));
  auto index = at::arange(0, dim, 2, at::TensorOptions().dtype(at::kFloat));
  auto inv = at::pow(10000.0, -index / static_cast<double>(dim));
  auto angles = offsets.unsqueeze(1) * inv.unsqueeze(0);
  auto value = std::make_pair(angles.cos().to(device).contiguous(), angles.sin().to(device).contiguous());
  cache.emplace(key, value);
  return value;
}

}  // namespace

bool local16_supported(int block, int dim);
std::vector<at::Tensor> local16_fwd_launch(const at::Tensor& qkv, const c10::optional<at::Tensor>& prev,
                                           int64_t start, int64_t valid_start, int64_t n);
std::vector<at::Tensor> local16_bwd_launch(const at::Tensor& dout, const at::Tensor& qkv,
                                           const c10::optional<at::Tensor>& prev, const at::Tensor& out,
                                           const at::Tensor& lse, int64_t start, int64_t valid_start, int64_t n);

bool local_attention_supported(int block, int dim) {
  return block >= 1 && block <= 128 && dim % 2 == 0 && dim <= 256 && bwd_smem(block, dim) <= 200 * 1024;
}

std::vector<at::Tensor> local_attention_fwd(const at::Tensor& qkv, const c10::optional<at::Tensor>& prev,
                                            int64_t start, int64_t valid_start, int64_t n, int64_t block) {
  TORCH_CHECK(qkv.is_cuda() && qkv.dim() == 5 && qkv.size(2) == 3 && qkv.is_contiguous(), "qkv [B,n,3,H,D]");
  TORCH_CHECK(qkv.size(1) == n, "qkv rows must equal n");
  const int batch = qkv.size(0), heads = qkv.size(3), dim = qkv.size(4);
  TORCH_CHECK(local_attention_supported(block, dim), "unsupported local attention shape");
  const c10::cuda::CUDAGuard guard(qkv.device());
  if (local16_supported(block, dim) && n > 0) return local16_fwd_launch(qkv, prev, start, valid_start, n);
  auto tables = rope_tables(block, dim, qkv.device());
  LocalArgs a{qkv.data_ptr(), prev.has_value() ? prev->data_ptr() : nullptr, tables.first.data_ptr<float>(),
              tables.second.data_ptr<float>(), static_cast<int>(n), heads, dim, static_cast<int>(block),
              start, valid_start};
  auto out = at::empty({batch, n, heads * dim}, qkv.options());
  auto lse = at::empty({batch, n, heads}, qkv.options().dtype(at::kFloat));
  if (n == 0) return {out, lse};
  dim3 grid(cdiv(n, block), heads, batch);
  const size_t smem = fwd_smem(block, dim);
  auto stream = at::cuda::getCurrentCUDAStream();
  if (qkv.scalar_type() == at::kBFloat16) {
    auto kernel = local_fwd_kernel<__nv_bfloat16>;
    EB_CUDA_CHECK(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    kernel<<<grid, kLocalThreads, smem, stream>>>(a, reinterpret_cast<__nv_bfloat16*>(out.data_ptr()),
                                                  lse.data_ptr<float>());
  } else {
    TORCH_CHECK(qkv.scalar_type() == at::kFloat, "qkv must be fp32 or bf16");
    auto kernel = local_fwd_kernel<float>;
    EB_CUDA_CHECK(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    kernel<<<grid, kLocalThreads, smem, stream>>>(a, out.data_ptr<float>(), lse.data_ptr<float>());
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  count_launch(1);
  return {out, lse};
}

std::vector<at::Tensor> local_attention_bwd(const at::Tensor& dout, const at::Tensor& qkv,
                                            const c10::optional<at::Tensor>& prev, const at::Tensor& out,
                                            const at::Tensor& lse, int64_t start, int64_t valid_start,
                                            int64_t n, int64_t block) {
  TORCH_CHECK(dout.is_contiguous() && dout.sizes() == out.sizes(), "dout must match out");
  const int batch = qkv.size(0), heads = qkv.size(3), dim = qkv.size(4);
  const c10::cuda::CUDAGuard guard(qkv.device());
  if (local16_supported(block, dim) && n > 0)
    return local16_bwd_launch(dout, qkv, prev, out, lse, start, valid_start, n);
  auto tables = rope_tables(block, dim, qkv.device());
  LocalArgs a{qkv.data_ptr(), prev.has_value() ? prev->data_ptr() : nullptr, tables.first.data_ptr<float>(),
              tables.second.data_ptr<float>(), static_cast<int>(n), heads, dim, static_cast<int>(block),
              start, valid_start};
  auto dqkv = at::empty_like(qkv);
  at::Tensor dprev;
  if (prev.has_value()) dprev = at::zeros_like(*prev);
  if (n == 0) return {dqkv, dprev};
  dim3 grid(cdiv(n, block), heads, batch);
  const size_t smem = bwd_smem(block, dim);
  auto stream = at::cuda::getCurrentCUDAStream();
  if (qkv.scalar_type() == at::kBFloat16) {
    using T = __nv_bfloat16;
    auto kernel = local_bwd_kernel<T>;
    EB_CUDA_CHECK(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    kernel<<<grid, kLocalThreads, smem, stream>>>(
        a, reinterpret_cast<const T*>(dout.data_ptr()), reinterpret_cast<const T*>(out.data_ptr()),
        lse.data_ptr<float>(), reinterpret_cast<T*>(dqkv.data_ptr()),
        prev.has_value() ? reinterpret_cast<T*>(dprev.data_ptr()) : nullptr);
  } else {
    auto kernel = local_bwd_kernel<float>;
    EB_CUDA_CHECK(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    kernel<<<grid, kLocalThreads, smem, stream>>>(a, dout.data_ptr<float>(), out.data_ptr<float>(),
                                                  lse.data_ptr<float>(), dqkv.data_ptr<float>(),
                                                  prev.has_value() ? dprev.data_ptr<float>() : nullptr);
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  count_launch(1);
  return {dqkv, dprev};
}

}  // namespace eb
