// Persistent tcgen05 GEMM with fused epilogues (sm_100a).
//
//   C[M, N] = alpha * sum_k A[m, k] * B[n, k]        (bf16 in, fp32 accumulate)
//
// A and B are each either K-major (k contiguous: x and W of y = x W^T) or
// MN-major (m / n contiguous: the transposed operands of the backward
// GEMMs), so all three GEMMs of a linear layer (y = x W^T, dx = dy W,
// dW = dy^T x) run without a transpose copy.
//
// CTA = one SM, persistent over 128 x BN output tiles (grouped order for
// L2 reuse). Warp 0 streams A/B k-slices (64 deep, 128-byte swizzle) through
// a 4-stage TMA ring; warp 1 issues tcgen05.mma (M=128, N=BN, K=16) into one
// of two TMEM accumulators; warps 4-7 drain the other accumulator (thread =
// output row) through the fused epilogue while the next tile accumulates.
//
// Epilogues: bf16 store | fp32 store | fp32 accumulate-into (weight grads) |
// bias + exact GELU -> bf16 (pre-activation kept for backward) |
// bias + fp32 residual -> fp32 (residual stream) |
// GELU backward (acc * gelu'(pre)) -> bf16 with per-tile column sums for the
// bias gradient.
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "../common/sm100.cuh"
#include "../common/tma.cuh"

namespace eb {
namespace {

using namespace sm100;

constexpr int kBM = 128;
constexpr int kBK = 64;
constexpr int kStages = 4;
constexpr int kThreads = 256;
constexpr int kGroupM = 8;

enum Epilogue : int {
  kStoreBf16 = 0,
  kStoreF32 = 1,
  kAccumF32 = 2,
  kBiasGeluBf16 = 3,
  kBiasResidualF32 = 4,
  kGeluBackBf16 = 5,
};

struct GemmArgs {
  int M, N, K;
  void* out;
  int64_t ldo;
  const float* bias;       // [N]
  const float* residual;   // fp32 [M, ldr]
  int64_t ldr;
  __nv_bfloat16* aux;      // pre-activation (written by kBiasGeluBf16, read by kGeluBackBf16)
  int64_t ld_aux;
  float* col_partial;      // [tiles_m, N] fp32 partial column sums (kGeluBackBf16)
  float alpha;
  ErrorSlot* err;
};

template <int BN>
struct alignas(1024) GemmSmem {
  __nv_bfloat16 a[kStages][kBM * kBK];
  __nv_bfloat16 b[kStages][BN * kBK];
  uint64_t full[kStages], empty[kStages], acc_full[2], acc_empty[2];
  uint32_t tmem_base;
  int abort;
  float colsum[4][BN];     // per-warp column partials of the GELU-backward epilogue
};

EB_DEVICE float gelu_f(float v) { return 0.5f * v * (1.f + erff(v * 0.70710678118654752f)); }
EB_DEVICE float gelu_grad_f(float v) {
  return 0.5f * (1.f + erff(v * 0.70710678118654752f)) + v * expf(-0.5f * v * v) * 0.39894228040143268f;
}

EB_DEVICE void tile_coords(int tile, int tiles_m, int tiles_n, int& tm, int& tn) {
  const int per_group = kGroupM * tiles_n;
  const int group = tile / per_group;
  const int first_m = group * kGroupM;
  const int rows = min(tiles_m - first_m, kGroupM);
  const int in_group = tile % per_group;
  tm = first_m + in_group % rows;
  tn = in_group / rows;
}

template <int BN, bool A_MN, bool B_MN, int EPI>
__global__ void __launch_bounds__(kThreads, 1)
gemm_tc_kernel(const __grid_constant__ CUtensorMap ta, const __grid_constant__ CUtensorMap tb, GemmArgs g) {
  extern __shared__ __align__(1024) uint8_t raw_smem[];
  GemmSmem<BN>& sm = *reinterpret_cast<GemmSmem<BN>*>(
      (reinterpret_cast<uintptr_t>(raw_smem) + 1023) & ~static_cast<uintptr_t>(1023));
  constexpr uint32_t kTmemCols = 2 * BN <= 32 ? 32 : (2 * BN <= 64 ? 64 : (2 * BN <= 128 ? 128 : (2 * BN <= 256 ? 256 : 512)));
  constexpr uint32_t kStageBytes = (kBM + BN) * kBK * 2;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tiles_m = (g.M + kBM - 1) / kBM, tiles_n = (g.N + BN - 1) / BN;
  const int tiles = tiles_m * tiles_n;
  const int k_blocks = (g.K + kBK - 1) / kBK;
  volatile int* abort = &sm.abort;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&sm.full[s], 1);
      mbar_init(&sm.empty[s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&sm.acc_full[s], 1);
      mbar_init(&sm.acc_empty[s], 128);
    }
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
      prefetch_tensormap(&ta);
      prefetch_tensormap(&tb);
      int it = 0;   // global k-slice counter across tiles
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < tiles; tile += gridDim.x) {
        int tm, tn;
        tile_coords(tile, tiles_m, tiles_n, tm, tn);
        for (int kb = 0; kb < k_blocks; ++kb, ++it) {
          const int s = it % kStages;
          if (it >= kStages && !mbar_wait(&sm.empty[s], ((it / kStages) - 1) & 1, abort, g.err, kSiteGemm)) {
            ok = false;
            break;
          }
          mbar_expect_tx(&sm.full[s], kStageBytes);
          const int k0 = kb * kBK;
          if constexpr (A_MN) {   // A stored [K, M]: boxes of 64 m x 64 k
            tma_load_2d(sm.a[s], &ta, &sm.full[s], tm * kBM, k0);
            tma_load_2d(sm.a[s] + 64 * kBK, &ta, &sm.full[s], tm * kBM + 64, k0);
          } else {                // A stored [M, K]: one box of 64 k x 128 m
            tma_load_2d(sm.a[s], &ta, &sm.full[s], k0, tm * kBM);
          }
          if constexpr (B_MN) {   // B stored [K, N]: BN/64 boxes of 64 n x 64 k
#pragma unroll
            for (int j = 0; j < BN / 64; ++j)
              tma_load_2d(sm.b[s] + j * 64 * kBK, &tb, &sm.full[s], tn * BN + 64 * j, k0);
          } else {                // B stored [N, K]: one box of 64 k x BN n
            tma_load_2d(sm.b[s], &tb, &sm.full[s], k0, tn * BN);
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = idesc_bf16(kBM, BN, A_MN, B_MN);
      int it = 0, local = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < tiles; tile += gridDim.x, ++local) {
        const int acc = local & 1;
        if (local >= 2 && !mbar_wait(&sm.acc_empty[acc], ((local >> 1) - 1) & 1, abort, g.err, kSiteGemm)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem + acc * BN;
        for (int kb = 0; kb < k_blocks; ++kb, ++it) {
          const int s = it % kStages;
          if (!mbar_wait(&sm.full[s], (it / kStages) & 1, abort, g.err, kSiteGemm)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(sm.a[s]), b_addr = smem_u32(sm.b[s]);
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk) {
            const uint64_t da = A_MN ? smem_desc_sw128(a_addr + kk * 2048, 64 * kBK * 2, 1024)
                                     : smem_desc_sw128(a_addr + kk * 32, 16, 1024);
            const uint64_t db = B_MN ? smem_desc_sw128(b_addr + kk * 2048, 64 * kBK * 2, 1024)
                                     : smem_desc_sw128(b_addr + kk * 32, 16, 1024);
            mma_ss(d_tmem, da, db, idesc, (kb > 0 || kk > 0) ? 1u : 0u);
          }
          tc_commit(&sm.empty[s]);
        }
        if (ok) tc_commit(&sm.acc_full[acc]);
      }
    }
  } else if (warp >= 4) {
    const int ew = warp - 4;
    const int row = threadIdx.x - 128;
    const uint32_t lane_addr = tmem + (static_cast<uint32_t>(ew * 32) << 16);
    int local = 0;
    for (int tile = blockIdx.x; tile < tiles; tile += gridDim.x, ++local) {
      int tm, tn;
      tile_coords(tile, tiles_m, tiles_n, tm, tn);
      const int acc = local & 1;
      const bool ready = mbar_wait(&sm.acc_full[acc], (local >> 1) & 1, abort, g.err, kSiteGemm);
      if (!__all_sync(0xffffffffu, ready)) break;
      tc_fence_after();
      const int m = tm * kBM + row;
      const bool row_ok = m < g.M;
      if constexpr (EPI == kGeluBackBf16) {
        for (int c = lane; c < BN; c += 32) sm.colsum[ew][c] = 0.f;
        __syncwarp();
      }
#pragma unroll 1
      for (int c0 = 0; c0 < BN; c0 += 32) {
        uint32_t r[32];
        tmem_ld32(lane_addr + acc * BN + c0, r);
        tc_wait_ld();
        const int n0 = tn * BN + c0;
        float v[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]) * g.alpha;
        const bool full_chunk = n0 + 32 <= g.N;
        if constexpr (EPI == kStoreBf16 || EPI == kBiasGeluBf16) {
          __nv_bfloat16* orow = static_cast<__nv_bfloat16*>(g.out) + static_cast<int64_t>(m) * g.ldo + n0;
          __nv_bfloat16* arow = EPI == kBiasGeluBf16 ? g.aux + static_cast<int64_t>(m) * g.ld_aux + n0 : nullptr;
#pragma unroll
          for (int i = 0; i < 32; i += 8) {
            float pre[8], post[8];
#pragma unroll
            for (int t = 0; t < 8; ++t) {
              pre[t] = v[i + t];
              if constexpr (EPI == kBiasGeluBf16) {
                const int n = n0 + i + t;
                pre[t] += n < g.N ? g.bias[n] : 0.f;
                post[t] = gelu_f(pre[t]);
              } else {
                post[t] = pre[t];
              }
            }
            if (row_ok && full_chunk) {
              *reinterpret_cast<uint4*>(orow + i) = make_uint4(pack_bf16(post[0], post[1]), pack_bf16(post[2], post[3]),
                                                               pack_bf16(post[4], post[5]), pack_bf16(post[6], post[7]));
              if constexpr (EPI == kBiasGeluBf16)
                *reinterpret_cast<uint4*>(arow + i) = make_uint4(pack_bf16(pre[0], pre[1]), pack_bf16(pre[2], pre[3]),
                                                                 pack_bf16(pre[4], pre[5]), pack_bf16(pre[6], pre[7]));
            } else if (row_ok) {
#pragma unroll
              for (int t = 0; t < 8; ++t) {
                if (n0 + i + t < g.N) {
                  orow[i + t] = __float2bfloat16(post[t]);
                  if constexpr (EPI == kBiasGeluBf16) arow[i + t] = __float2bfloat16(pre[t]);
                }
              }
            }
          }
        } else if constexpr (EPI == kStoreF32 || EPI == kAccumF32 || EPI == kBiasResidualF32) {
          float* orow = static_cast<float*>(g.out) + static_cast<int64_t>(m) * g.ldo + n0;
          const float* rrow = EPI == kBiasResidualF32 ? g.residual + static_cast<int64_t>(m) * g.ldr + n0 : nullptr;
#pragma unroll
          for (int i = 0; i < 32; i += 4) {
            float o[4];
#pragma unroll
            for (int t = 0; t < 4; ++t) o[t] = v[i + t];
            if (row_ok && full_chunk) {
              if constexpr (EPI == kAccumF32) {
                const float4 prev = *reinterpret_cast<const float4*>(orow + i);
                o[0] += prev.x; o[1] += prev.y; o[2] += prev.z; o[3] += prev.w;
              } else if constexpr (EPI == kBiasResidualF32) {
                const float4 res = *reinterpret_cast<const float4*>(rrow + i);
                o[0] += res.x + (g.bias ? g.bias[n0 + i] : 0.f);
                o[1] += res.y + (g.bias ? g.bias[n0 + i + 1] : 0.f);
                o[2] += res.z + (g.bias ? g.bias[n0 + i + 2] : 0.f);
                o[3] += res.w + (g.bias ? g.bias[n0 + i + 3] : 0.f);
              }
              *reinterpret_cast<float4*>(orow + i) = make_float4(o[0], o[1], o[2], o[3]);
            } else if (row_ok) {
#pragma unroll
              for (int t = 0; t < 4; ++t) {
                const int n = n0 + i + t;
                if (n < g.N) {
                  float val = o[t];
                  if constexpr (EPI == kAccumF32) val += orow[i + t];
                  if constexpr (EPI == kBiasResidualF32) val += rrow[i + t] + (g.bias ? g.bias[n] : 0.f);
                  orow[i + t] = val;
                }
              }
            }
          }
        } else if constexpr (EPI == kGeluBackBf16) {
          __nv_bfloat16* orow = static_cast<__nv_bfloat16*>(g.out) + static_cast<int64_t>(m) * g.ldo + n0;
          const __nv_bfloat16* arow = g.aux + static_cast<int64_t>(m) * g.ld_aux + n0;
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const int n = n0 + i;
            float d = 0.f;
            if (row_ok && n < g.N) {
              d = v[i] * gelu_grad_f(__bfloat162float(arow[i]));
              orow[i] = __float2bfloat16(d);
            }
            // Column partial sums over this warp's 32 rows (deterministic tree).
            float s = d;
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
            if (lane == 0) sm.colsum[ew][c0 + i] = s;
          }
        }
      }
      if constexpr (EPI == kGeluBackBf16) {
        // Combine the four warps' partials of this tile; one row per tile of output.
        asm volatile("bar.sync 1, 128;" ::: "memory");
        for (int c = row; c < BN; c += 128) {
          const int n = tn * BN + c;
          if (n < g.N)
            g.col_partial[static_cast<int64_t>(tm) * g.N + n] =
                sm.colsum[0][c] + sm.colsum[1][c] + sm.colsum[2][c] + sm.colsum[3][c];
        }
        asm volatile("bar.sync 1, 128;" ::: "memory");
      }
      tc_fence_before();
      mbar_arrive(&sm.acc_empty[acc]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// Operand descriptor: row-major storage [rows, cols] with a leading dimension.
struct Operand {
  const at::Tensor* t;
  bool mn_major;   // true: stored [K, M or N]; false: stored [M or N, K]
};

template <int BN, bool A_MN, bool B_MN, int EPI>
void run_gemm(const at::Tensor& a, const at::Tensor& b, int M, int N, int K, GemmArgs& args, cudaStream_t stream) {
  // TMA maps: inner (contiguous) dimension first.
  CUtensorMap ta = A_MN ? make_matrix_map(a.data_ptr(), K, M, a.stride(0), kBK)     // [K, M], box 64m x 64k
                        : make_matrix_map(a.data_ptr(), M, K, a.stride(0), kBM);    // [M, K], box 64k x 128m
  CUtensorMap tb = B_MN ? make_matrix_map(b.data_ptr(), K, N, b.stride(0), kBK)
                        : make_matrix_map(b.data_ptr(), N, K, b.stride(0), BN);
  const int tiles = ((M + kBM - 1) / kBM) * ((N + BN - 1) / BN);
  int sms = 0;
  EB_CUDA_CHECK(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, a.device().index()));
  const int grid = std::min(tiles, sms);
  const size_t smem = sizeof(GemmSmem<BN>) + 1024;
  auto kernel = gemm_tc_kernel<BN, A_MN, B_MN, EPI>;
  EB_CUDA_CHECK(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
  kernel<<<grid, kThreads, smem, stream>>>(ta, tb, args);
}

template <bool A_MN, bool B_MN, int EPI>
void dispatch_bn(const at::Tensor& a, const at::Tensor& b, int M, int N, int K, GemmArgs& args,
                 cudaStream_t stream) {
  // Wide tiles when there is enough work to fill the GPU; narrow ones otherwise.
  const int sms = 148;
  const long tiles256 = ((M + kBM - 1) / kBM) * static_cast<long>((N + 255) / 256);
  if (N >= 256 && tiles256 >= sms) run_gemm<256, A_MN, B_MN, EPI>(a, b, M, N, K, args, stream);
  else run_gemm<128, A_MN, B_MN, EPI>(a, b, M, N, K, args, stream);
}

template <int EPI>
void dispatch_layout(const at::Tensor& a, bool a_mn, const at::Tensor& b, bool b_mn, int M, int N, int K,
                     GemmArgs& args, cudaStream_t stream) {
  if (!a_mn && !b_mn) dispatch_bn<false, false, EPI>(a, b, M, N, K, args, stream);
  else if (!a_mn && b_mn) dispatch_bn<false, true, EPI>(a, b, M, N, K, args, stream);
  else if (a_mn && !b_mn) dispatch_bn<true, false, EPI>(a, b, M, N, K, args, stream);
  else dispatch_bn<true, true, EPI>(a, b, M, N, K, args, stream);
}

bool aligned16(const at::Tensor& t) {
  return reinterpret_cast<uintptr_t>(t.data_ptr()) % 16 == 0 && (t.stride(0) * 2) % 16 == 0 && t.stride(1) == 1;
}

}  // namespace

bool gemm_supported(const at::Tensor& a, bool a_mn, const at::Tensor& b, bool b_mn) {
  return a.is_cuda() && b.is_cuda() && a.scalar_type() == at::kBFloat16 && b.scalar_type() == at::kBFloat16 &&
         a.dim() == 2 && b.dim() == 2 && aligned16(a) && aligned16(b);
}

// out = epilogue(alpha * op(A) op(B)^T) where op(A) is [M, K] and op(B) is [N, K].
// a_mn: A is stored [K, M]; b_mn: B is stored [K, N]. Optional tensors may be undefined.
void gemm(const at::Tensor& a, bool a_mn, const at::Tensor& b, bool b_mn, at::Tensor& out, int64_t epilogue,
          double alpha, const c10::optional<at::Tensor>& bias, const c10::optional<at::Tensor>& residual,
          const c10::optional<at::Tensor>& aux, const c10::optional<at::Tensor>& col_partial) {
  TORCH_CHECK(gemm_supported(a, a_mn, b, b_mn), "gemm: bf16 2-D operands with 16-byte aligned rows required");
  const int M = a_mn ? a.size(1) : a.size(0);
  const int K = a_mn ? a.size(0) : a.size(1);
  const int N = b_mn ? b.size(1) : b.size(0);
  TORCH_CHECK((b_mn ? b.size(0) : b.size(1)) == K, "gemm: inner dimensions differ");
  TORCH_CHECK(out.dim() == 2 && out.size(0) == M && out.size(1) == N && out.stride(1) == 1, "gemm: bad output");
  const c10::cuda::CUDAGuard guard(a.device());
  GemmArgs args{};
  args.M = M;
  args.N = N;
  args.K = K;
  args.out = out.data_ptr();
  args.ldo = out.stride(0);
  args.alpha = static_cast<float>(alpha);
  args.bias = bias.has_value() && bias->defined() ? bias->data_ptr<float>() : nullptr;
  if (residual.has_value() && residual->defined()) {
    args.residual = residual->data_ptr<float>();
    args.ldr = residual->stride(0);
  }
  if (aux.has_value() && aux->defined()) {
    args.aux = reinterpret_cast<__nv_bfloat16*>(aux->data_ptr());
    args.ld_aux = aux->stride(0);
  }
  if (col_partial.has_value() && col_partial->defined()) args.col_partial = col_partial->data_ptr<float>();
  args.err = device_error_slot(a.device().index());
  auto stream = at::cuda::getCurrentCUDAStream();
  switch (epilogue) {
    case kStoreBf16:
      TORCH_CHECK(out.scalar_type() == at::kBFloat16, "bf16 output");
      dispatch_layout<kStoreBf16>(a, a_mn, b, b_mn, M, N, K, args, stream); break;
    case kStoreF32:
      TORCH_CHECK(out.scalar_type() == at::kFloat, "fp32 output");
      dispatch_layout<kStoreF32>(a, a_mn, b, b_mn, M, N, K, args, stream); break;
    case kAccumF32:
      TORCH_CHECK(out.scalar_type() == at::kFloat, "fp32 output");
      dispatch_layout<kAccumF32>(a, a_mn, b, b_mn, M, N, K, args, stream); break;
    case kBiasGeluBf16:
      TORCH_CHECK(out.scalar_type() == at::kBFloat16 && args.aux && args.bias, "bias/aux needed");
      dispatch_layout<kBiasGeluBf16>(a, a_mn, b, b_mn, M, N, K, args, stream); break;
    case kBiasResidualF32:
      TORCH_CHECK(out.scalar_type() == at::kFloat && args.residual, "fp32 residual needed");
      dispatch_layout<kBiasResidualF32>(a, a_mn, b, b_mn, M, N, K, args, stream); break;
    case kGeluBackBf16:
      TORCH_CHECK(out.scalar_type() == at::kBFloat16 && args.aux && args.col_partial, "aux/partials needed");
      dispatch_layout<kGeluBackBf16>(a, a_mn, b, b_mn, M, N, K, args, stream); break;
    default:
      TORCH_CHECK(false, "unknown epilogue ", epilogue);
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  count_launch(1);
}

int64_t gemm_tile_m() { return kBM; }

}  // namespace eb
