// Data-parallel gradient reduction over NVLink peer memory (sm_100a).
//
// Every rank keeps its flat fp32 gradient buffer and the bf16 shadow of its
// parameters in a symmetric heap: one region per rank, mapped by every peer,
// identical offsets everywhere. The reduction then needs no collective
// library and no staging copies:
//
// * grad_reduce_bucket (one launch per gradient bucket, on a side stream,
//   as soon as backward has produced the bucket). A bucket [lo, hi) is cut
//   into `world` slices of q elements; rank r owns slice r. The kernel first
//   announces "my bucket is final" to every peer (system-scope release store
//   into the peer's arrival word) and waits, bounded, until every peer has
//   announced the same. Each thread then loads one 16-byte vector of the
//   owned slice from all ranks at once (world loads in flight), adds them in
//   rank order (the same order on every launch, so results are
//   deterministic), applies the bucket scale and stores the sum either
//   locally (reduce-scatter: the ZeRO-1 owner is the only rank that needs
//   it) or into every rank's buffer (all-reduce: parameters that every rank
//   updates). The sum of squares of the reduced values, the gradient-norm
//   contribution of the slice, comes out of the same pass as one partial per
//   CTA, so clipping needs no second read of the gradient.
// * grad_norm_exchange (once per step, after the last bucket): adds the
//   partials in a fixed order, stores the rank's total into every peer's
//   norm word, waits for all ranks (bounded) and writes the global squared
//   norm, summed in rank order, to `hyper[3]` on every rank. It doubles as
//   the end-of-reduction barrier: no rank passes it before every rank's
//   bucket kernels (and their peer stores) are complete, and it advances the
//   device-side epoch, so a captured CUDA graph replays correctly.
// * flat_adamw_peer: AdamW over an owned slice that also writes the updated
//   bf16 shadow into every rank's shadow buffer (the ZeRO-1 parameter
//   all-gather as peer stores fused into the update; 16-byte stores).
//
// Ownership makes the kernels race-free without locks: slice r of a bucket
// is read and written only by rank r, and all-reduce stores of one element
// follow that thread's loads of it. Waits are bounded by wall time
// (globaltimer); on expiry the kernel records kSitePeer in the device error
// slot and returns, so the host raises instead of hanging. No multicast
// object and no `multimem` access is used: plain peer loads and stores.
//
// The reference reduces gradients with DDP (NCCL all-reduce buckets,
// st/runtime/engine.py:85-87), shards AdamW with ZeroRedundancyOptimizer
// (engine.py:105-112) and clips with clip_grad_norm_ (engine.py:179).
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <vector>

#include "../common/peer.cuh"
#include "../common/sm100.cuh"
#include "../common/tma.cuh"

namespace eb {
namespace {

using namespace sm100;

constexpr int kMaxRanks = 8;
constexpr int kMaxBuckets = 256;
constexpr int kReduceThreads = 256;
constexpr int kLoads = 16;       // 16-byte loads in flight per thread in grad_reduce_kernel
// Flag-slot layout (32-bit words, identical on every rank):
//   [b * 8 + s]            rank s arrived at bucket b (epoch)
//   [kFin + s]             rank s finished the step's reduction (epoch)
//   [kNorm + s]            rank s's squared-norm contribution (float bits)
//   [kEpoch]               this rank's last completed epoch (local only)
constexpr int kFin = kMaxBuckets * 8;
constexpr int kNorm = kFin + 8;
constexpr int kEpoch = kNorm + 8;
constexpr int kFlagWords = kEpoch + 8;

struct PeerF32 {
  float4* p[kMaxRanks];
};
struct PeerFlags {
  unsigned int* p[kMaxRanks];
};
struct PeerBf16 {
  uint4* p[kMaxRanks];
};

// Bounded wait until every rank's word [base + s] reached `epoch`.
// Thread s < world polls word s; returns false on timeout (reported).
EB_DEVICE bool wait_all(const unsigned int* words, int world, unsigned int epoch, uint64_t timeout_ns,
                        ErrorSlot* err) {
  __shared__ int failed;
  if (threadIdx.x == 0) failed = 0;
  __syncthreads();
  if (threadIdx.x < world) {
    const uint64_t start = global_ns();
    while (static_cast<int>(load_acquire_sys(words + threadIdx.x) - epoch) < 0) {
      if (global_ns() - start > timeout_ns) {
        report(err, kSitePeer);
        failed = 1;
        break;
      }
    }
  }
  __syncthreads();
  return failed == 0;
}

EB_DEVICE float block_sum(float v, float* scratch) {
  v = warp_sum(v);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) scratch[warp] = v;
  __syncthreads();
  float total = 0.f;
  if (warp == 0) {
    total = lane < static_cast<int>(blockDim.x >> 5) ? scratch[lane] : 0.f;
    total = warp_sum(total);
  }
  return total;    // valid in thread 0
}

template <int W>
__global__ void __launch_bounds__(kReduceThreads)
grad_reduce_kernel(PeerF32 grads, PeerFlags flags, int rank, int64_t s0, int64_t s1, int bucket, int all_reduce,
                   float scale, float* __restrict__ partial, uint64_t timeout_ns, ErrorSlot* err) {
  __shared__ float scratch[kReduceThreads / 32];
  const unsigned int epoch = *reinterpret_cast<volatile unsigned int*>(flags.p[rank] + kEpoch) + 1u;
  if (blockIdx.x == 0 && threadIdx.x < W) {
    __threadfence_system();
    store_release_sys(flags.p[threadIdx.x] + bucket * 8 + rank, epoch);
  }
  if (!wait_all(flags.p[rank] + bucket * 8, W, epoch, timeout_ns, err)) return;
  // Every thread keeps kLoads 16-byte loads in flight (U vectors from each of
  // the W ranks) before it adds anything: a peer load takes microseconds over
  // NVLink, so the bandwidth follows the bytes in flight. One vector per rank
  // and thread (32 CTAs of 512 threads) reached about 110 GB/s at W = 2,
  // eight about 290 GB/s. The ranks are still added in rank order.
  constexpr int U = kLoads / W > 0 ? kLoads / W : 1;
  float acc = 0.f;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * kReduceThreads;
  const int64_t end = s1 / 4;
  for (int64_t i0 = s0 / 4 + blockIdx.x * static_cast<int64_t>(kReduceThreads) + threadIdx.x; i0 < end;
       i0 += stride * U) {
    float4 v[U][W];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t i = i0 + u * stride;
      if (i < end) {
#pragma unroll
        for (int r = 0; r < W; ++r) v[u][r] = __ldcg(grads.p[r] + i);
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t i = i0 + u * stride;
      if (i >= end) break;
      float4 s = v[u][0];
#pragma unroll
      for (int r = 1; r < W; ++r) {
        s.x += v[u][r].x;
        s.y += v[u][r].y;
        s.z += v[u][r].z;
        s.w += v[u][r].w;
      }
      s.x *= scale;
      s.y *= scale;
      s.z *= scale;
      s.w *= scale;
      acc += s.x * s.x + s.y * s.y + s.z * s.z + s.w * s.w;
      if (all_reduce) {
#pragma unroll
        for (int r = 0; r < W; ++r) grads.p[r][i] = s;
      } else {
        grads.p[rank][i] = s;
      }
    }
  }
  if (all_reduce) __threadfence_system();
  const float total = block_sum(acc, scratch);
  if (threadIdx.x == 0) partial[blockIdx.x] = total;
}

__global__ void __launch_bounds__(1024)
grad_norm_exchange_kernel(const float* __restrict__ partial, int count, PeerFlags flags, int rank, int world,
                          float* __restrict__ hyper, uint64_t timeout_ns, ErrorSlot* err) {
  __shared__ float scratch[32];
  float acc = 0.f;
  for (int i = threadIdx.x; i < count; i += blockDim.x) acc += partial[i];
  const float mine = block_sum(acc, scratch);
  unsigned int* own = flags.p[rank];
  const unsigned int epoch = *reinterpret_cast<volatile unsigned int*>(own + kEpoch) + 1u;
  __shared__ float shared_mine;
  if (threadIdx.x == 0) shared_mine = mine;
  __syncthreads();
  if (threadIdx.x < world) {
    __threadfence_system();
    store_relaxed_sys(flags.p[threadIdx.x] + kNorm + rank, __float_as_uint(shared_mine));
    store_release_sys(flags.p[threadIdx.x] + kFin + rank, epoch);
  }
  const bool ok = wait_all(own + kFin, world, epoch, timeout_ns, err);
  if (threadIdx.x == 0) {
    float total = 0.f;
    for (int s = 0; s < world; ++s) total += __uint_as_float(load_acquire_sys(own + kNorm + s));
    hyper[3] = ok ? total : __int_as_float(0x7fc00000);      // NaN: the optimizer skips the step
    *reinterpret_cast<volatile unsigned int*>(own + kEpoch) = epoch;
  }
}

EB_DEVICE uint32_t pack2_bf16(float a, float b) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

EB_DEVICE void adamw4(float4& p, const float4 g, float4& m, float4& v, float scale, float beta1, float beta2,
                      float eps, float step_size, float inv_sqrt_bc2, float keep) {
  float* pp = &p.x;
  const float* gg = &g.x;
  float* mm = &m.x;
  float* vv = &v.x;
#pragma unroll
  for (int t = 0; t < 4; ++t) {
    const float gt = gg[t] * scale;
    mm[t] = beta1 * mm[t] + (1.f - beta1) * gt;
    vv[t] = beta2 * vv[t] + (1.f - beta2) * gt * gt;
    pp[t] = pp[t] * keep - step_size * mm[t] / (sqrtf(vv[t]) * inv_sqrt_bc2 + eps);
  }
}

// Same arithmetic as flat_adamw (fused/flat_optim.cu); 8 elements per step so
// the shadow leaves as one 16-byte store per rank.
__global__ void __launch_bounds__(256)
flat_adamw_peer_kernel(float4* __restrict__ p, const float4* __restrict__ g, float4* __restrict__ m,
                       float4* __restrict__ v, PeerBf16 shadows, int rank, int world, int64_t n8,
                       const float* __restrict__ hyper, const float* __restrict__ loss_check, float beta1,
                       float beta2, float eps, float decay) {
  const float lr = hyper[0], step = hyper[1], max_norm = hyper[2], sq = hyper[3];
  const float lc = loss_check != nullptr ? *loss_check : 0.f;
  if (!isfinite(sq) || !isfinite(lc)) return;
  float scale = 1.f;
  if (max_norm > 0.f) scale = fminf(max_norm / (sqrtf(sq) + 1e-6f), 1.f);
  const float bc1 = 1.f - powf(beta1, step);
  const float bc2 = 1.f - powf(beta2, step);
  const float step_size = lr / bc1;
  const float inv_sqrt_bc2 = 1.f / sqrtf(bc2);
  const float keep = 1.f - lr * decay;
  for (int64_t i = blockIdx.x * 256ll + threadIdx.x; i < n8; i += static_cast<int64_t>(gridDim.x) * 256) {
    float4 p0 = p[2 * i], p1 = p[2 * i + 1], m0 = m[2 * i], m1 = m[2 * i + 1], v0 = v[2 * i], v1 = v[2 * i + 1];
    const float4 g0 = g[2 * i], g1 = g[2 * i + 1];
    adamw4(p0, g0, m0, v0, scale, beta1, beta2, eps, step_size, inv_sqrt_bc2, keep);
    adamw4(p1, g1, m1, v1, scale, beta1, beta2, eps, step_size, inv_sqrt_bc2, keep);
    p[2 * i] = p0;
    p[2 * i + 1] = p1;
    m[2 * i] = m0;
    m[2 * i + 1] = m1;
    v[2 * i] = v0;
    v[2 * i + 1] = v1;
    const uint4 packed = make_uint4(pack2_bf16(p0.x, p0.y), pack2_bf16(p0.z, p0.w), pack2_bf16(p1.x, p1.y),
                                    pack2_bf16(p1.z, p1.w));
    for (int r = 0; r < world; ++r) shadows.p[(rank + r) % world][i] = packed;
  }
  __threadfence_system();
}

uint64_t timeout_ns_of(double seconds) { return static_cast<uint64_t>(seconds * 1e9); }

void check_ranks(size_t world, int64_t rank) {
  TORCH_CHECK(world >= 1 && world <= kMaxRanks && rank >= 0 && rank < static_cast<int64_t>(world),
              "grad_reduce: bad world/rank");
}

}  // namespace

int64_t grad_flag_bytes() { return static_cast<int64_t>(kFlagWords) * 4; }

int64_t grad_reduce_max_buckets() { return kMaxBuckets; }

// Reduce slice `rank` of bucket [lo, hi) (slice length q) across all ranks.
// grads[r] / flags[r]: device addresses of rank r's flat gradient and flag slot.
void grad_reduce_bucket(const std::vector<int64_t>& grads, const std::vector<int64_t>& flags, int64_t rank,
                        int64_t bucket, int64_t lo, int64_t hi, int64_t q, bool all_reduce, double scale,
                        at::Tensor& partial, double timeout_s) {
  const size_t world = grads.size();
  check_ranks(world, rank);
  TORCH_CHECK(flags.size() == world, "grad_reduce: one flag slot per rank");
  TORCH_CHECK(bucket >= 0 && bucket < kMaxBuckets, "grad_reduce: at most ", kMaxBuckets, " buckets");
  TORCH_CHECK(lo % 4 == 0 && hi % 4 == 0 && q % 4 == 0 && lo <= hi, "grad_reduce: bounds must be multiples of 4");
  TORCH_CHECK(partial.is_cuda() && partial.scalar_type() == at::kFloat && partial.is_contiguous(),
              "grad_reduce: partial must be a contiguous fp32 CUDA tensor");
  PeerF32 g{};
  PeerFlags f{};
  for (size_t r = 0; r < world; ++r) {
    TORCH_CHECK(grads[r] % 16 == 0 && flags[r] % 16 == 0, "grad_reduce: 16-byte aligned buffers");
    g.p[r] = reinterpret_cast<float4*>(grads[r]);
    f.p[r] = reinterpret_cast<unsigned int*>(flags[r]);
  }
  const int64_t s0 = std::min(hi, lo + rank * q), s1 = std::min(hi, s0 + q);
  const int64_t n4 = (s1 - s0) / 4;
  const int blocks = static_cast<int>(partial.numel());
  TORCH_CHECK(blocks >= 1, "grad_reduce: partial needs one slot per CTA");
  (void)n4;
  const c10::cuda::CUDAGuard guard(partial.device());
  auto stream = at::cuda::getCurrentCUDAStream();
  ErrorSlot* err = device_error_slot(partial.get_device());
  const uint64_t t = timeout_ns_of(timeout_s);
  const float sc = static_cast<float>(scale);
  float* part = partial.data_ptr<float>();
  const int b = static_cast<int>(bucket), ar = all_reduce ? 1 : 0, rk = static_cast<int>(rank);
  switch (world) {
#define EB_REDUCE_CASE(W)                                                                                      \
  case W:                                                                                                      \
    grad_reduce_kernel<W><<<blocks, kReduceThreads, 0, stream>>>(g, f, rk, s0, s1, b, ar, sc, part, t, err); \
    break;
    EB_REDUCE_CASE(1)
    EB_REDUCE_CASE(2)
    EB_REDUCE_CASE(3)
    EB_REDUCE_CASE(4)
    EB_REDUCE_CASE(5)
    EB_REDUCE_CASE(6)
    EB_REDUCE_CASE(7)
    EB_REDUCE_CASE(8)
#undef EB_REDUCE_CASE
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  count_launch(1);
}

// hyper[3] = global squared gradient norm; end-of-reduction barrier.
void grad_norm_exchange(const at::Tensor& partial, const std::vector<int64_t>& flags, int64_t rank, at::Tensor& hyper,
                        double timeout_s) {
  const size_t world = flags.size();
  check_ranks(world, rank);
  TORCH_CHECK(partial.is_cuda() && partial.scalar_type() == at::kFloat && partial.is_contiguous(),
              "grad_norm_exchange: partial fp32");
  TORCH_CHECK(hyper.is_cuda() && hyper.scalar_type() == at::kFloat && hyper.numel() >= 4, "hyper [4] fp32");
  PeerFlags f{};
  for (size_t r = 0; r < world; ++r) f.p[r] = reinterpret_cast<unsigned int*>(flags[r]);
  const c10::cuda::CUDAGuard guard(partial.device());
  grad_norm_exchange_kernel<<<1, 1024, 0, at::cuda::getCurrentCUDAStream()>>>(
      partial.data_ptr<float>(), static_cast<int>(partial.numel()), f, static_cast<int>(rank),
      static_cast<int>(world), hyper.data_ptr<float>(), timeout_ns_of(timeout_s),
      device_error_slot(partial.get_device()));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  count_launch(1);
}

// AdamW over an owned slice; the bf16 shadow goes to shadows[r] (same offset on every rank).
void flat_adamw_peer(at::Tensor& param, const at::Tensor& grad, at::Tensor& exp_avg, at::Tensor& exp_avg_sq,
                     const std::vector<int64_t>& shadows, int64_t rank, const at::Tensor& hyper,
                     const c10::optional<at::Tensor>& loss_check, double beta1, double beta2, double eps,
                     double decay) {
  const size_t world = shadows.size();
  check_ranks(world, rank);
  const int64_t n = param.numel();
  const at::Tensor* tensors[] = {&param, &grad, &exp_avg, &exp_avg_sq};
  for (const at::Tensor* t : tensors) {
    TORCH_CHECK(t->is_cuda() && t->scalar_type() == at::kFloat && t->is_contiguous() && t->numel() == n &&
                    reinterpret_cast<uintptr_t>(t->data_ptr()) % 16 == 0,
                "flat_adamw_peer: contiguous 16-byte aligned fp32 tensors of one size");
  }
  TORCH_CHECK(n % 8 == 0, "flat_adamw_peer: a multiple of 8 elements");
  TORCH_CHECK(hyper.is_cuda() && hyper.scalar_type() == at::kFloat && hyper.numel() >= 4, "hyper [4] fp32");
  PeerBf16 sh{};
  for (size_t r = 0; r < world; ++r) {
    TORCH_CHECK(shadows[r] % 16 == 0, "flat_adamw_peer: 16-byte aligned shadows");
    sh.p[r] = reinterpret_cast<uint4*>(shadows[r]);
  }
  const float* lc = nullptr;
  if (loss_check.has_value() && loss_check->defined()) {
    TORCH_CHECK(loss_check->is_cuda() && loss_check->scalar_type() == at::kFloat, "loss_check fp32");
    lc = loss_check->data_ptr<float>();
  }
  if (n == 0) return;
  const c10::cuda::CUDAGuard guard(param.device());
  const int64_t n8 = n / 8;
  const int blocks = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>((n8 + 255) / 256, 148 * 4)));
  flat_adamw_peer_kernel<<<blocks, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<float4*>(param.data_ptr()), reinterpret_cast<const float4*>(grad.data_ptr()),
      reinterpret_cast<float4*>(exp_avg.data_ptr()), reinterpret_cast<float4*>(exp_avg_sq.data_ptr()), sh,
      static_cast<int>(rank), static_cast<int>(world), n8, hyper.data_ptr<float>(), lc, static_cast<float>(beta1),
      static_cast<float>(beta2), static_cast<float>(eps), static_cast<float>(decay));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  count_launch(1);
}

}  // namespace eb
