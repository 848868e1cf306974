// Persistent tcgen05 GEMM with fused epilogues (sm_100a).
//
//   C[M, N] = alpha * sum_k A[m, k] * B[n, k]        (bf16 in, fp32 accumulate)
//
// A and B are each either K-major (k contiguous: x and W of y = x W^T) or
// MN-major (m / n contiguous: the transposed operands of the backward
// GEMMs), so all three GEMMs of a linear layer (y = x W^T, dx = dy W,
// dW = dy^T x) run without a transpose copy.
//
// Persistent over (128 * CTAS) x BN output tiles (grouped order for L2
// reuse). With CTAS = 1 a CTA owns an SM and a 128 x BN tile. With CTAS = 2 a
// 2-CTA cluster runs one cta_group::2 MMA of 256 x BN: each CTA stages its 128
// rows of A and BN/2 columns of B, so an SM holds half the B tile (half the
// shared-memory traffic per FLOP of the single-CTA form) and keeps 6 stages in
// flight; the even CTA issues the MMAs and both CTAs drain their 128
// accumulator rows. Warp 0 streams A/B k-slices (64 deep, 128-byte swizzle)
// through the TMA ring; warp 1 issues tcgen05.mma (K=16) into one of two TMEM
// accumulators; warps 4-11 drain the other accumulator (thread = output row)
// through the fused epilogue while the next tile accumulates.
//
// Epilogues: bf16 store | fp32 store | fp32 accumulate-into (weight grads) |
// bias + exact GELU -> bf16 (gelu'(pre-activation) kept for backward) |
// bias + fp32 residual -> fp32 (residual stream) |
// GELU backward (acc * the kept gelu') -> bf16 with per-tile column sums for
// the bias gradient | peer scatter (Ulysses to-heads).
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <cstdlib>
#include <string>

#include "../common/sm100.cuh"
#include "../common/tma.cuh"

namespace eb {
namespace {

using namespace sm100;

constexpr int kBM = 128;
constexpr int kBK = 64;
constexpr int kStages = 4;
constexpr int kThreads = 384;   // warps 0-3: TMA, MMA, TMEM owner, idle; 4-11: epilogue
constexpr int kGroupM = 8;

enum Epilogue : int {
  kStoreBf16 = 0,
  kStoreF32 = 1,
  kAccumF32 = 2,
  kBiasGeluBf16 = 3,
  kBiasResidualF32 = 4,
  kGeluBackBf16 = 5,
  kScatterBf16 = 6,        // bf16 tile stored straight into the owning rank's buffer (Ulysses to-heads)
};

constexpr int kMaxPeers = 8;

// Ulysses layout shared by the peer-scatter epilogue and the peer-gather A
// operand. Every rank holds a buffer [parts, batch, n_total, C] for its C =
// heads_per_rank * head_dim columns of each part (q; or k and v) over the
// whole sequence; rank r's sequence shard is rows [r * n_local, (r+1) * n_local).
// In the sequence layout a row has parts * dim columns, dim = world * C.
struct PeerLayout {
  int world, rank, parts, batch, n_local, n_total, C, dim;
  int tma_store;                   // scatter through TMA stores of 32 x 32 blocks (PeerMaps hold the targets)
  __nv_bfloat16* dst[kMaxPeers];   // scatter targets (possibly peer memory)
};

struct PeerMaps {
  CUtensorMap map[kMaxPeers];      // gather sources or scatter targets, one 3-D map per rank
};

// Targets of the TMA epilogue: the output [planes, M, N] (planes = K splits)
// and, for bias+GELU, the kept derivative [M, N]; 32 x 32 boxes (make_epilogue_map).
struct OutMaps {
  CUtensorMap out, aux;
};

struct GemmArgs {
  int M, N, K;
  void* out;
  int64_t ldo;
  const float* bias;       // [N]
  const float* residual;   // fp32 [M, ldr]
  int64_t ldr;
  __nv_bfloat16* aux;      // gelu'(pre-activation) (written by kBiasGeluBf16, read by kGeluBackBf16)
  int64_t ld_aux;
  float* col_partial;      // [tiles_m, N] fp32 partial column sums (kGeluBackBf16)
  float alpha;
  int splits;              // K split into this many ranges; split s writes out + s * split_stride (fp32 partials)
  int64_t split_stride;
  int vec;                 // 1: every row start and leading dimension allows 8/16-byte vector access
  int tma_out;             // 1: the epilogue writes through shared memory with TMA (OutMaps hold the targets)
  ErrorSlot* err;
  PeerLayout peer;
};

template <int BN, int CTAS>
struct GemmShape {
  static constexpr int kTileM = kBM * CTAS;                   // rows of one output tile
  static constexpr int kBNc = BN / CTAS;                      // B rows (n) staged by each CTA
  static constexpr int kStagesN = CTAS == 2 ? 6 : kStages;
  static constexpr uint32_t kStageBytes = (kBM + kBNc) * kBK * 2;   // per CTA
};

template <int BN, int CTAS>
struct alignas(1024) GemmSmem {
  using Shape = GemmShape<BN, CTAS>;
  __nv_bfloat16 a[Shape::kStagesN][kBM * kBK];
  __nv_bfloat16 b[Shape::kStagesN][Shape::kBNc * kBK];
  uint64_t full[Shape::kStagesN], empty[Shape::kStagesN], acc_full[2], acc_empty[2];
  uint32_t tmem_base;
  int abort;
  // Per epilogue warp, 4 KB: a 32-row output box for the TMA epilogue (32 fp32
  // or, in the first 2 KB, 32 bf16 columns; bias+GELU's derivative box in the
  // second 2 KB); the GELU-backward column partials at byte 2048. The
  // register-path epilogue stages 32 rows x 16 fp32 columns in the first 2 KB,
  // the peer scatter a 32 x 32 bf16 block.
  alignas(1024) uint8_t stage[8][4096];
};

EB_DEVICE float rcp_approx(float x) {
  float y;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Exact GELU and its derivative: gelu(v) = v * Phi(v), gelu'(v) = Phi(v) +
// v * phi(v) (Phi/phi: standard normal cdf/pdf). erf comes from Abramowitz &
// Stegun, Handbook of Mathematical Functions, formula 7.1.26 (absolute error
// <= 1.5e-7, far below the bf16 rounding of both outputs):
//   erf(x) = 1 - t (a1 + t (a2 + t (a3 + t (a4 + t a5)))) exp(-x^2),
//   t = 1 / (1 + p x), x >= 0.
// With x = |v| / sqrt(2), exp(-x^2) = exp(-v^2 / 2) is also the exponential
// of phi(v), so both outputs cost one exp2 and one reciprocal.
EB_DEVICE void gelu_and_grad(float v, float& y, float& dy) {
  const float x = fabsf(v) * 0.70710678118654752f;
  const float t = rcp_approx(fmaf(0.3275911f, x, 1.f));
  const float poly =
      t * fmaf(t, fmaf(t, fmaf(t, fmaf(t, 1.061405429f, -1.453152027f), 1.421413741f), -0.284496736f), 0.254829592f);
  const float e = ex2(v * v * -0.72134752044448170f);          // exp(-v^2 / 2) = 2^(-v^2 log2(e) / 2)
  const float cdf = 0.5f + copysignf(0.5f - 0.5f * poly * e, v);
  y = v * cdf;
  dy = fmaf(v * e, 0.39894228040143268f, cdf);
}

EB_DEVICE float4 load_bias4(const float* bias, int n, int N) {
  if (n + 4 <= N && (reinterpret_cast<uintptr_t>(bias + n) & 15) == 0) return *reinterpret_cast<const float4*>(bias + n);
  float b[4];
#pragma unroll
  for (int t = 0; t < 4; ++t) b[t] = n + t < N ? bias[n + t] : 0.f;
  return make_float4(b[0], b[1], b[2], b[3]);
}

// Four consecutive outputs (m, n..n+3) of one row. Vector accesses need the
// row start aligned (checked on the host: GemmArgs::vec) and n + 4 <= N.
template <int EPI>
EB_DEVICE void epilogue4(const GemmArgs& g, int64_t ooff, int m, int n, float4 v4, float4 b4, float (&cs)[4],
                         uint2 aux_raw) {
  float v[4] = {v4.x, v4.y, v4.z, v4.w};
  const float bb[4] = {b4.x, b4.y, b4.z, b4.w};
  const bool vec = g.vec && n + 4 <= g.N;
  const int cnt = min(4, g.N - n);
  if constexpr (EPI == kStoreBf16 || EPI == kBiasGeluBf16) {
    __nv_bfloat16* o = static_cast<__nv_bfloat16*>(g.out) + static_cast<int64_t>(m) * g.ldo + n;
    float pre[4];   // kBiasGeluBf16: gelu'(pre-activation), the backward's multiplier
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      if constexpr (EPI == kBiasGeluBf16) {
        gelu_and_grad(v[t] + bb[t], v[t], pre[t]);
      } else {
        pre[t] = v[t];
      }
    }
    if (vec) {
      *reinterpret_cast<uint2*>(o) = make_uint2(pack_bf16(v[0], v[1]), pack_bf16(v[2], v[3]));
      if constexpr (EPI == kBiasGeluBf16)
        *reinterpret_cast<uint2*>(g.aux + static_cast<int64_t>(m) * g.ld_aux + n) =
            make_uint2(pack_bf16(pre[0], pre[1]), pack_bf16(pre[2], pre[3]));
    } else {
      for (int t = 0; t < cnt; ++t) {
        o[t] = __float2bfloat16(v[t]);
        if constexpr (EPI == kBiasGeluBf16) g.aux[static_cast<int64_t>(m) * g.ld_aux + n + t] = __float2bfloat16(pre[t]);
      }
    }
  } else if constexpr (EPI == kStoreF32 || EPI == kAccumF32 || EPI == kBiasResidualF32) {
    float* o = static_cast<float*>(g.out) + ooff + static_cast<int64_t>(m) * g.ldo + n;
    const float* res = EPI == kBiasResidualF32 ? g.residual + static_cast<int64_t>(m) * g.ldr + n : nullptr;
    if (vec) {
      if constexpr (EPI == kAccumF32) {
        const float4 p = *reinterpret_cast<const float4*>(o);
        v[0] += p.x; v[1] += p.y; v[2] += p.z; v[3] += p.w;
      } else if constexpr (EPI == kBiasResidualF32) {
        const float4 p = *reinterpret_cast<const float4*>(res);
        v[0] += p.x + bb[0]; v[1] += p.y + bb[1]; v[2] += p.z + bb[2]; v[3] += p.w + bb[3];
      }
      *reinterpret_cast<float4*>(o) = make_float4(v[0], v[1], v[2], v[3]);
    } else {
      for (int t = 0; t < cnt; ++t) {
        float val = v[t];
        if constexpr (EPI == kAccumF32) val += o[t];
        if constexpr (EPI == kBiasResidualF32) val += res[t] + bb[t];
        o[t] = val;
      }
    }
  } else if constexpr (EPI == kScatterBf16) {
    // Sequence-layout element (m, n) -> owner's head-layout buffer.
    const PeerLayout& L = g.peer;
    const int b = m / L.n_local, t = m - b * L.n_local;
    const int part = n / L.dim, within = n - part * L.dim;
    const int owner = within / L.C, c = within - owner * L.C;
    __nv_bfloat16* o = L.dst[owner] +
                       (static_cast<int64_t>(part * L.batch + b) * L.n_total + L.rank * L.n_local + t) * L.C + c;
    if (vec && c + 4 <= L.C) {
      *reinterpret_cast<uint2*>(o) = make_uint2(pack_bf16(v[0], v[1]), pack_bf16(v[2], v[3]));
    } else {
      for (int q = 0; q < cnt; ++q) {
        const int nn = n + q, pp = nn / L.dim, ww = nn - pp * L.dim, ow = ww / L.C, cc = ww - ow * L.C;
        L.dst[ow][(static_cast<int64_t>(pp * L.batch + b) * L.n_total + L.rank * L.n_local + t) * L.C + cc] =
            __float2bfloat16(v[q]);
      }
    }
  } else if constexpr (EPI == kGeluBackBf16) {
    __nv_bfloat16* o = static_cast<__nv_bfloat16*>(g.out) + static_cast<int64_t>(m) * g.ldo + n;
    const __nv_bfloat16* a = g.aux + static_cast<int64_t>(m) * g.ld_aux + n;
    float pre[4] = {0.f, 0.f, 0.f, 0.f};
    if (vec) {
      const uint2 raw = aux_raw;               // loaded by the caller ahead of the TMEM wait
      const __nv_bfloat162 p0 = *reinterpret_cast<const __nv_bfloat162*>(&raw.x);
      const __nv_bfloat162 p1 = *reinterpret_cast<const __nv_bfloat162*>(&raw.y);
      pre[0] = __low2float(p0); pre[1] = __high2float(p0); pre[2] = __low2float(p1); pre[3] = __high2float(p1);
    } else {
      for (int t = 0; t < cnt; ++t) pre[t] = __bfloat162float(a[t]);
    }
    float d[4];
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      d[t] = t < cnt ? v[t] * pre[t] : 0.f;
      cs[t] += d[t];
    }
    if (vec) {
      *reinterpret_cast<uint2*>(o) = make_uint2(pack_bf16(d[0], d[1]), pack_bf16(d[2], d[3]));
    } else {
      for (int t = 0; t < cnt; ++t) o[t] = __float2bfloat16(d[t]);
    }
  }
}

// Sum over the warp's 32 lanes of each of 32 per-lane values: afterwards lane
// j holds the sum of everyone's v[j]. Five exchange rounds (16, 8, 4, 2, 1
// values); in each, a lane keeps the half of its columns selected by its lane
// bit and adds its partner's copy of that half.
EB_DEVICE float lane_transpose_sum(float (&v)[32], int lane) {
#pragma unroll
  for (int s = 16; s >= 1; s >>= 1) {
    const bool upper = (lane & s) != 0;
#pragma unroll
    for (int k = 0; k < s; ++k) {
      const float send = upper ? v[k] : v[k + s];
      const float keep = upper ? v[k + s] : v[k];
      v[k] = keep + __shfl_xor_sync(0xffffffffu, send, s);
    }
  }
  return v[0];
}

// Byte offset of the 16-byte unit `unit` of row `row` in a swizzled box whose
// rows are 64 bytes (64-byte swizzle) or 128 bytes (128-byte swizzle) wide;
// the box starts on a 1024-byte boundary. Eight consecutive rows writing the
// same unit hit eight different bank groups.
template <int kRowBytes>
EB_DEVICE uint32_t swizzled(int row, int unit) {
  if constexpr (kRowBytes == 64) return row * 64 + ((unit ^ ((row >> 1) & 3)) << 4);
  else return row * 128 + ((unit ^ (row & 7)) << 4);
}

// The TMA epilogue of one accumulator tile for one epilogue warp: its 32 rows
// (lane = row, from TMEM lanes) by its column half, 32 columns per chunk.
// The chunk's values are finished in registers (bias, GELU, residual, kept
// derivative), written to the warp's swizzled 32-row box in shared memory and
// stored (fp32 accumulation: reduced with an element-wise add) by one TMA
// instruction; the TMA engine clips rows and columns outside the matrix. The
// box is reused once the previous store has read it. GELU backward also
// leaves the warp's column sums at byte 2048 of its staging area.
template <int BN, int EPI>
EB_DEVICE void tma_epilogue(const GemmArgs& g, const OutMaps& om, uint8_t* stage, uint32_t taddr, int row0,
                            int col_base, int grp, int lane, int plane) {
  constexpr bool kF32 = EPI == kStoreF32 || EPI == kAccumF32 || EPI == kBiasResidualF32;
  const int m = row0 + lane;
  const bool row_ok = m < g.M;
  float* colsum = reinterpret_cast<float*>(stage + 2048);
#pragma unroll 1
  for (int c0 = grp * (BN / 2); c0 < (grp + 1) * (BN / 2); c0 += 32) {
    const int n0 = col_base + c0;
    if (n0 >= g.N) break;                           // uniform across the warp
    const bool full = n0 + 32 <= g.N;
    // Per-row operands of the chunk, issued before the TMEM load is awaited.
    uint4 aux_raw[4];
    float4 res[8];
    if constexpr (EPI == kGeluBackBf16) {
      const __nv_bfloat16* a = g.aux + static_cast<int64_t>(m) * g.ld_aux + n0;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        aux_raw[q] = make_uint4(0u, 0u, 0u, 0u);
        if (row_ok && full) aux_raw[q] = *reinterpret_cast<const uint4*>(a + 8 * q);
      }
      if (row_ok && !full) {
        __nv_bfloat16* e = reinterpret_cast<__nv_bfloat16*>(aux_raw);
        for (int j = 0; j < 32 && n0 + j < g.N; ++j) e[j] = a[j];
      }
    }
    if constexpr (EPI == kBiasResidualF32) {
      const float* rrow = g.residual + static_cast<int64_t>(m) * g.ldr + n0;
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        res[q] = make_float4(0.f, 0.f, 0.f, 0.f);
        if (row_ok && full) res[q] = *reinterpret_cast<const float4*>(rrow + 4 * q);
      }
      if (row_ok && !full) {
        float* e = reinterpret_cast<float*>(res);
        for (int j = 0; j < 32 && n0 + j < g.N; ++j) e[j] = rrow[j];
      }
    }
    uint32_t r[32];
    tmem_ld32(taddr + c0, r);
    tc_wait_ld();
    float v[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]) * g.alpha;
    float kept[32];                                  // bias+GELU: gelu'(pre-activation)
    if constexpr (EPI == kBiasGeluBf16 || EPI == kBiasResidualF32) {
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const float4 b4 = g.bias ? load_bias4(g.bias, n0 + 4 * q, g.N) : make_float4(0.f, 0.f, 0.f, 0.f);
        const float bb[4] = {b4.x, b4.y, b4.z, b4.w};
#pragma unroll
        for (int t = 0; t < 4; ++t) {
          float& x = v[4 * q + t];
          if constexpr (EPI == kBiasGeluBf16) {
            gelu_and_grad(x + bb[t], x, kept[4 * q + t]);
          } else {
            const float rr[4] = {res[q].x, res[q].y, res[q].z, res[q].w};
            x += bb[t] + rr[t];
          }
        }
      }
    }
    if constexpr (EPI == kGeluBackBf16) {
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const uint32_t w[4] = {aux_raw[q].x, aux_raw[q].y, aux_raw[q].z, aux_raw[q].w};
#pragma unroll
        for (int t = 0; t < 4; ++t) {
          const __nv_bfloat162 p2 = *reinterpret_cast<const __nv_bfloat162*>(&w[t]);
          v[8 * q + 2 * t] *= __low2float(p2);
          v[8 * q + 2 * t + 1] *= __high2float(p2);
        }
      }
    }
    if (lane == 0) bulk_wait_read_all();             // the previous chunk's stores have read the box
    __syncwarp();
    if constexpr (kF32) {
#pragma unroll
      for (int u = 0; u < 8; ++u)
        *reinterpret_cast<float4*>(stage + swizzled<128>(lane, u)) =
            make_float4(v[4 * u], v[4 * u + 1], v[4 * u + 2], v[4 * u + 3]);
    } else {
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const float* x = v + 8 * u;
        *reinterpret_cast<uint4*>(stage + swizzled<64>(lane, u)) =
            make_uint4(pack_bf16(x[0], x[1]), pack_bf16(x[2], x[3]), pack_bf16(x[4], x[5]), pack_bf16(x[6], x[7]));
      }
      if constexpr (EPI == kBiasGeluBf16) {
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const float* x = kept + 8 * u;
          *reinterpret_cast<uint4*>(stage + 2048 + swizzled<64>(lane, u)) =
              make_uint4(pack_bf16(x[0], x[1]), pack_bf16(x[2], x[3]), pack_bf16(x[4], x[5]), pack_bf16(x[6], x[7]));
        }
      }
    }
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0 && row0 < g.M) {
      if constexpr (EPI == kAccumF32) tma_reduce_add_3d(&om.out, stage, n0, row0, plane);
      else tma_store_3d(&om.out, stage, n0, row0, plane);
      if constexpr (EPI == kBiasGeluBf16) tma_store_3d(&om.aux, stage + 2048, n0, row0, 0);
      bulk_commit();
    }
    if constexpr (EPI == kGeluBackBf16) {
      // Column sums of this chunk over the warp's rows (rows past M hold zeros).
      const float sum = lane_transpose_sum(v, lane);
      colsum[c0 - grp * (BN / 2) + lane] = sum;
    }
  }
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

template <int BN, bool A_MN, bool B_MN, int EPI, bool GATHER_A, int CTAS>
__global__ void __launch_bounds__(kThreads, 1)
gemm_tc_kernel(const __grid_constant__ CUtensorMap ta, const __grid_constant__ CUtensorMap tb, GemmArgs g,
               const __grid_constant__ PeerMaps pm, const __grid_constant__ OutMaps om) {
  static_assert(CTAS == 1 || (CTAS == 2 && !GATHER_A && EPI != kScatterBf16), "peer paths run on single CTAs");
  using Shape = GemmShape<BN, CTAS>;
  constexpr int kS = Shape::kStagesN;
  constexpr int kTileM = Shape::kTileM;
  constexpr int kBNc = Shape::kBNc;
  extern __shared__ __align__(1024) uint8_t raw_smem[];
  GemmSmem<BN, CTAS>& sm = *reinterpret_cast<GemmSmem<BN, CTAS>*>(
      (reinterpret_cast<uintptr_t>(raw_smem) + 1023) & ~static_cast<uintptr_t>(1023));
  constexpr uint32_t kTmemCols = 2 * BN <= 32 ? 32 : (2 * BN <= 64 ? 64 : (2 * BN <= 128 ? 128 : (2 * BN <= 256 ? 256 : 512)));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = CTAS == 2 ? cluster_ctarank() : 0;    // position in the CTA pair
  const int group = blockIdx.x / CTAS, groups = gridDim.x / CTAS;
  const int tiles_m = (g.M + kTileM - 1) / kTileM, tiles_n = (g.N + BN - 1) / BN;
  const int tiles = tiles_m * tiles_n;
  const int units = tiles * g.splits;     // (split, tile) pairs; consecutive units share a K range
  const int k_blocks = (g.K + kBK - 1) / kBK;
  volatile int* abort = &sm.abort;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kS; ++s) {
      mbar_init(&sm.full[s], 1);
      mbar_init(&sm.empty[s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&sm.acc_full[s], 1);
      mbar_init(&sm.acc_empty[s], 8 * CTAS);   // one arrival per epilogue warp of every CTA of the group
    }
    sm.abort = 0;
    fence_barrier_init();
  }
  if (warp == 2) {
    if constexpr (CTAS == 2) tmem_alloc_pair(&sm.tmem_base, kTmemCols);
    else tmem_alloc(&sm.tmem_base, kTmemCols);
  }
  tc_fence_before();
  if constexpr (CTAS == 2) cluster_sync();    // the peer's barriers are initialised before anyone signals them
  else __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sm.tmem_base;

  if (warp == 0) {
    if (lane == 0) {
      if constexpr (GATHER_A) {
        for (int r = 0; r < g.peer.world; ++r) prefetch_tensormap(&pm.map[r]);
      } else {
        prefetch_tensormap(&ta);
      }
      prefetch_tensormap(&tb);
      int it = 0;   // global k-slice counter across tiles
      bool ok = true;
      for (int unit = group; ok && unit < units; unit += groups) {
        const int split = unit / tiles, tile = unit - split * tiles;
        int tm, tn;
        tile_coords(tile, tiles_m, tiles_n, tm, tn);
        const int kb0 = split * k_blocks / g.splits, kb1 = (split + 1) * k_blocks / g.splits;
        const int m0 = tm * kTileM + static_cast<int>(rank) * kBM;     // this CTA's A rows
        const int n0 = tn * BN + static_cast<int>(rank) * kBNc;        // this CTA's B rows (output columns)
        for (int kb = kb0; kb < kb1; ++kb, ++it) {
          const int s = it % kS;
          if (it >= kS && !mbar_wait(&sm.empty[s], ((it / kS) - 1) & 1, abort, g.err, kSiteGemm)) {
            ok = false;
            break;
          }
          const int k0 = kb * kBK;
          if constexpr (CTAS == 2) {
            // Both CTAs' bytes complete on the leader's barrier; the leader
            // arms it for the pair (its arrival is the barrier's only one).
            const uint32_t bar = cluster_addr(&sm.full[s], 0);
            if (rank == 0) mbar_expect_tx(&sm.full[s], CTAS * Shape::kStageBytes);
            if constexpr (A_MN) {
              tma_load_2d_pair(sm.a[s], &ta, bar, m0, k0);
              tma_load_2d_pair(sm.a[s] + 64 * kBK, &ta, bar, m0 + 64, k0);
            } else {
              tma_load_2d_pair(sm.a[s], &ta, bar, k0, m0);
            }
            if constexpr (B_MN) {
#pragma unroll
              for (int j = 0; j < kBNc / 64; ++j) tma_load_2d_pair(sm.b[s] + j * 64 * kBK, &tb, bar, n0 + 64 * j, k0);
            } else {
              tma_load_2d_pair(sm.b[s], &tb, bar, k0, n0);
            }
            continue;
          }
          mbar_expect_tx(&sm.full[s], Shape::kStageBytes);
          if constexpr (GATHER_A) {
            // A = the sequence layout of rank-sharded head buffers: the 64-wide
            // k-slice lives on one owner; rows are this rank's shard.
            const PeerLayout& L = g.peer;
            const int b = m0 / L.n_local, t0 = m0 - b * L.n_local;
            const int part = k0 / L.dim, within = k0 - part * L.dim;
            const int owner = within / L.C, col = within - owner * L.C;
            tma_load_3d(sm.a[s], &pm.map[owner], &sm.full[s], col, L.rank * L.n_local + t0, part * L.batch + b);
          } else if constexpr (A_MN) {   // A stored [K, M]: boxes of 64 m x 64 k
            tma_load_2d(sm.a[s], &ta, &sm.full[s], m0, k0);
            tma_load_2d(sm.a[s] + 64 * kBK, &ta, &sm.full[s], m0 + 64, k0);
          } else {                // A stored [M, K]: one box of 64 k x 128 m
            tma_load_2d(sm.a[s], &ta, &sm.full[s], k0, m0);
          }
          if constexpr (B_MN) {   // B stored [K, N]: BN/64 boxes of 64 n x 64 k
#pragma unroll
            for (int j = 0; j < BN / 64; ++j)
              tma_load_2d(sm.b[s] + j * 64 * kBK, &tb, &sm.full[s], n0 + 64 * j, k0);
          } else {                // B stored [N, K]: one box of 64 k x BN n
            tma_load_2d(sm.b[s], &tb, &sm.full[s], k0, n0);
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && rank == 0) {
      const uint32_t idesc = idesc_bf16(kTileM, BN, A_MN, B_MN);
      int it = 0, local = 0;
      bool ok = true;
      for (int unit = group; ok && unit < units; unit += groups, ++local) {
        const int split = unit / tiles;
        const int kb0 = split * k_blocks / g.splits, kb1 = (split + 1) * k_blocks / g.splits;
        const int acc = local & 1;
        if (local >= 2 && !mbar_wait(&sm.acc_empty[acc], ((local >> 1) - 1) & 1, abort, g.err, kSiteGemm)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem + acc * BN;
        for (int kb = kb0; kb < kb1; ++kb, ++it) {
          const int s = it % kS;
          if (!mbar_wait(&sm.full[s], (it / kS) & 1, abort, g.err, kSiteGemm)) {
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
            if constexpr (CTAS == 2) mma_ss_pair(d_tmem, da, db, idesc, (kb > kb0 || kk > 0) ? 1u : 0u);
            else mma_ss(d_tmem, da, db, idesc, (kb > kb0 || kk > 0) ? 1u : 0u);
          }
          if constexpr (CTAS == 2) {          // the stage is free in both CTAs
            tc_commit_pair(cluster_addr(&sm.empty[s], 0));
            tc_commit_pair(cluster_addr(&sm.empty[s], 1));
          } else {
            tc_commit(&sm.empty[s]);
          }
        }
        if (ok) {
          if constexpr (CTAS == 2) {
            tc_commit_pair(cluster_addr(&sm.acc_full[acc], 0));
            tc_commit_pair(cluster_addr(&sm.acc_full[acc], 1));
          } else {
            tc_commit(&sm.acc_full[acc]);
          }
        }
      }
    }
  } else if (warp >= 4) {
    // Two epilogue warpgroups split the tile's columns. Each warp owns 32
    // accumulator lanes (rows); a row's values go through a small swizzled
    // shared-memory stage so that global loads/stores are coalesced (four
    // lanes cover 16 consecutive columns of one row).
    const int ew = warp - 4;                  // 0..7
    const int grp = ew >> 2;                  // column half of the tile
    const int wr = ew & 3;                    // TMEM lane quarter (rows 32*wr..)
    const uint32_t lane_addr = tmem + (static_cast<uint32_t>(wr * 32) << 16);
    float4* stage = reinterpret_cast<float4*>(sm.stage[ew]);
    float* colsum = reinterpret_cast<float*>(sm.stage[ew] + 2048);   // this warp's column partials
    const int rq = lane >> 2, u = lane & 3;
    int local = 0;
    for (int unit = group; unit < units; unit += groups, ++local) {
      const int split = unit / tiles, tile = unit - split * tiles;
      const int64_t ooff = static_cast<int64_t>(split) * g.split_stride;
      int tm, tn;
      tile_coords(tile, tiles_m, tiles_n, tm, tn);
      const int row0 = tm * kTileM + static_cast<int>(rank) * kBM;   // this CTA's accumulator rows
      const int acc = local & 1;
      const bool ready = mbar_wait(&sm.acc_full[acc], (local >> 1) & 1, abort, g.err, kSiteGemm);
      if (!__all_sync(0xffffffffu, ready)) break;
      tc_fence_after();
      bool tma_done = false;
      if constexpr (EPI != kScatterBf16) {
        if (g.tma_out) {
          tma_epilogue<BN, EPI>(g, om, sm.stage[ew], lane_addr + acc * BN, row0 + wr * 32, tn * BN, grp, lane,
                                g.splits > 1 ? split : 0);
          tma_done = true;
        }
      }
#pragma unroll 1
      for (int c0 = grp * (BN / 2); !tma_done && c0 < (grp + 1) * (BN / 2); c0 += 32) {
        uint32_t r[32];
        tmem_ld32(lane_addr + acc * BN + c0, r);
        if constexpr (EPI == kScatterBf16) {
          if (g.peer.tma_store) {
            // The warp's 32 rows x these 32 columns go to one owner as one TMA
            // store: each lane packs its row (64 bytes) into the staging block.
            tc_wait_ld();
            const int n = tn * BN + c0;
            if (n >= g.N) continue;
            __nv_bfloat16* block = reinterpret_cast<__nv_bfloat16*>(stage);
            if (lane == 0) bulk_wait_read_all();             // the previous store has read the block
            __syncwarp();
            uint4* row = reinterpret_cast<uint4*>(block + lane * 32);
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              const uint32_t* v = r + 8 * q;
              row[q] = make_uint4(pack_bf16(__uint_as_float(v[0]) * g.alpha, __uint_as_float(v[1]) * g.alpha),
                                  pack_bf16(__uint_as_float(v[2]) * g.alpha, __uint_as_float(v[3]) * g.alpha),
                                  pack_bf16(__uint_as_float(v[4]) * g.alpha, __uint_as_float(v[5]) * g.alpha),
                                  pack_bf16(__uint_as_float(v[6]) * g.alpha, __uint_as_float(v[7]) * g.alpha));
            }
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
              const PeerLayout& L = g.peer;
              const int m0 = row0 + wr * 32;
              const int b = m0 / L.n_local, t0 = m0 - b * L.n_local;
              const int part = n / L.dim, within = n - part * L.dim;
              const int owner = within / L.C, c = within - owner * L.C;
              tma_store_3d(&pm.map[owner], block, c, L.rank * L.n_local + t0, part * L.batch + b);
              bulk_commit();
            }
            continue;
          }
        }
        // GELU backward: the kept gelu' of this chunk's 8 (row, 4-column) groups is
        // loaded while the TMEM load is in flight.
        uint2 aux_raw[2][4];
#pragma unroll
        for (int half = 0; half < 2; ++half) {
#pragma unroll
          for (int it = 0; it < 4; ++it) {
            aux_raw[half][it] = make_uint2(0u, 0u);
            if constexpr (EPI == kGeluBackBf16) {
              const int m = row0 + wr * 32 + it * 8 + rq;
              const int n = tn * BN + c0 + half * 16 + 4 * u;
              if (g.vec && m < g.M && n + 4 <= g.N)
                aux_raw[half][it] = *reinterpret_cast<const uint2*>(g.aux + static_cast<int64_t>(m) * g.ld_aux + n);
            }
          }
        }
        tc_wait_ld();
#pragma unroll
        for (int half = 0; half < 2; ++half) {
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const int j = half * 16 + 4 * q;
            stage[lane * 4 + (q ^ ((lane >> 1) & 3))] =
                make_float4(__uint_as_float(r[j]) * g.alpha, __uint_as_float(r[j + 1]) * g.alpha,
                            __uint_as_float(r[j + 2]) * g.alpha, __uint_as_float(r[j + 3]) * g.alpha);
          }
          __syncwarp();
          const int n = tn * BN + c0 + half * 16 + 4 * u;
          float4 bias4 = make_float4(0.f, 0.f, 0.f, 0.f);
          if constexpr (EPI == kBiasGeluBf16 || EPI == kBiasResidualF32) {
            if (g.bias) bias4 = load_bias4(g.bias, n, g.N);
          }
          float cs[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
          for (int it = 0; it < 4; ++it) {
            const int rr = it * 8 + rq;
            const float4 v = stage[rr * 4 + (u ^ ((rr >> 1) & 3))];
            const int m = row0 + wr * 32 + rr;
            if (m < g.M && n < g.N) epilogue4<EPI>(g, ooff, m, n, v, bias4, cs, aux_raw[half][it]);
          }
          __syncwarp();
          if constexpr (EPI == kGeluBackBf16) {
#pragma unroll
            for (int t = 0; t < 4; ++t) {
#pragma unroll
              for (int o = 4; o < 32; o <<= 1) cs[t] += __shfl_xor_sync(0xffffffffu, cs[t], o);
            }
            if (lane < 4) {
              float* dst = &colsum[c0 - grp * (BN / 2) + half * 16 + 4 * u];
              dst[0] = cs[0]; dst[1] = cs[1]; dst[2] = cs[2]; dst[3] = cs[3];
            }
          }
        }
      }
      if constexpr (EPI == kGeluBackBf16) {
        // Combine the group's four row-quarters; one partial row per output tile.
        const int gt = threadIdx.x - 128 - grp * 128;
        auto part = [&](int w) { return reinterpret_cast<const float*>(sm.stage[w] + 2048); };
        asm volatile("bar.sync %0, 128;" ::"r"(1 + grp) : "memory");
        for (int c = gt; c < BN / 2; c += 128) {
          const int n = tn * BN + grp * (BN / 2) + c;
          if (n < g.N)
            g.col_partial[static_cast<int64_t>(row0 / kBM) * g.N + n] =
                part(grp * 4)[c] + part(grp * 4 + 1)[c] + part(grp * 4 + 2)[c] + part(grp * 4 + 3)[c];
        }
        asm volatile("bar.sync %0, 128;" ::"r"(1 + grp) : "memory");
      }
      // The warp's TMEM reads are complete (tcgen05.wait::ld above); one
      // arrival per warp frees the accumulator (the leader's barrier).
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if constexpr (CTAS == 2) mbar_arrive_cluster(cluster_addr(&sm.acc_empty[acc], 0));
        else mbar_arrive(&sm.acc_empty[acc]);
      }
    }
    if constexpr (EPI != kScatterBf16) {
      if (g.tma_out && lane == 0) bulk_wait_all();   // the epilogue's stores are complete
    }
    // Peer stores complete at system scope before the kernel ends, so a
    // barrier issued after it publishes them.
    if constexpr (EPI == kScatterBf16) {
      if (g.peer.tma_store && lane == 0) bulk_wait_all();   // this warp's stores are complete
      __threadfence_system();
    }
  }
  tc_fence_before();
  if constexpr (CTAS == 2) cluster_sync();     // neither CTA leaves while the pair's MMAs may read its memory
  else __syncthreads();
  if (warp == 2) {
    tc_fence_after();
    if constexpr (CTAS == 2) tmem_dealloc_pair(tmem, kTmemCols);
    else tmem_dealloc(tmem, kTmemCols);
  }
}

int sm_count(int device) {
  static int cached[64] = {0};
  if (device < 0 || device >= 64) device = 0;
  if (cached[device] == 0) {
    int sms = 0;
    EB_CUDA_CHECK(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device));
    cached[device] = sms;
  }
  return cached[device];
}

template <int BN, bool A_MN, bool B_MN, int EPI, bool GATHER_A, int CTAS = 1>
void launch_gemm(const CUtensorMap& ta, const PeerMaps& pm, const at::Tensor& b, int M, int N, int K,
                 GemmArgs& args, cudaStream_t stream, const OutMaps& om = OutMaps{}) {
  using Shape = GemmShape<BN, CTAS>;
  CUtensorMap tb = B_MN ? make_matrix_map(b.data_ptr(), K, N, b.stride(0), kBK)              // [K, N], box 64n x 64k
                        : make_matrix_map(b.data_ptr(), N, K, b.stride(0), Shape::kBNc);     // [N, K], box 64k x n
  const int units = ((M + Shape::kTileM - 1) / Shape::kTileM) * ((N + BN - 1) / BN) * std::max(1, args.splits);
  const size_t smem = sizeof(GemmSmem<BN, CTAS>) + 1024;
  auto kernel = gemm_tc_kernel<BN, A_MN, B_MN, EPI, GATHER_A, CTAS>;
  EB_CUDA_CHECK(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
  const int device = b.device().index();
  if constexpr (CTAS == 1) {
    const int grid = std::min(units, sm_count(device));
    kernel<<<grid, kThreads, smem, stream>>>(ta, tb, args, pm, om);
  } else {
    // One CTA pair per pair of SMs that can hold one: as many clusters as fit at once.
    static int resident[64] = {0};
    cudaLaunchAttribute attr{};
    attr.id = cudaLaunchAttributeClusterDimension;
    attr.val.clusterDim.x = CTAS;
    attr.val.clusterDim.y = 1;
    attr.val.clusterDim.z = 1;
    cudaLaunchConfig_t cfg{};
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    const int slot = device >= 0 && device < 64 ? device : 0;
    if (resident[slot] == 0) {
      cfg.gridDim = dim3(sm_count(device));
      int clusters = 0;
      EB_CUDA_CHECK(cudaOccupancyMaxActiveClusters(&clusters, kernel, &cfg));
      resident[slot] = std::max(1, clusters);
    }
    cfg.gridDim = dim3(CTAS * std::min(units, resident[slot]));
    EB_CUDA_CHECK(cudaLaunchKernelEx(&cfg, kernel, ta, tb, args, pm, om));
  }
}

// Output tile shapes: 128 x 128 and 128 x 256 on one CTA, 256 x 256 on a CTA pair.
enum TileShape : int { kShapeAuto = 0, kShapeNarrow = 1, kShapeWide = 2, kShapePair = 3 };

template <int BN, bool A_MN, bool B_MN, int EPI, int CTAS = 1>
void run_gemm(const at::Tensor& a, const at::Tensor& b, int M, int N, int K, GemmArgs& args, cudaStream_t stream,
              const PeerMaps* pm = nullptr) {
  // TMA maps: inner (contiguous) dimension first. Each CTA stages 128 rows of A.
  CUtensorMap ta = A_MN ? make_matrix_map(a.data_ptr(), K, M, a.stride(0), kBK)     // [K, M], box 64m x 64k
                        : make_matrix_map(a.data_ptr(), M, K, a.stride(0), kBM);    // [M, K], box 64k x 128m
  PeerMaps none{};
  OutMaps om{};
  if constexpr (EPI != kScatterBf16) {
    if (args.tma_out) {
      constexpr bool kF32 = EPI == kStoreF32 || EPI == kAccumF32 || EPI == kBiasResidualF32;
      const int planes = std::max(1, args.splits);
      const int64_t plane = planes > 1 ? args.split_stride : static_cast<int64_t>(M) * args.ldo;
      om.out = make_epilogue_map(args.out, planes, M, N, args.ldo, plane, kF32);
      if constexpr (EPI == kBiasGeluBf16)
        om.aux = make_epilogue_map(args.aux, 1, M, N, args.ld_aux, static_cast<int64_t>(M) * args.ld_aux, false);
    }
  }
  launch_gemm<BN, A_MN, B_MN, EPI, false, CTAS>(ta, pm ? *pm : none, b, M, N, K, args, stream, om);
}

// The TMA epilogue needs 16-byte aligned rows in the output and in the
// row-wise operands it reads (residual, kept derivative); EB200_GEMM_TMA_EPILOGUE=0
// selects the register-path epilogue everywhere.
bool tma_epilogue_ok(const GemmArgs& args, int out_elem) {
  static const bool off = std::getenv("EB200_GEMM_TMA_EPILOGUE") != nullptr &&
                          std::string(std::getenv("EB200_GEMM_TMA_EPILOGUE")) == "0";
  auto ok = [](const void* p, int64_t ld, int elem) {
    return p == nullptr || ((reinterpret_cast<uintptr_t>(p) % 16) == 0 && (ld * elem) % 16 == 0);
  };
  return !off && args.out != nullptr && ok(args.out, args.ldo, out_elem) && ok(args.residual, args.ldr, 4) &&
         ok(args.aux, args.ld_aux, 2);
}

bool wide_tiles(int M, int N) {
  // Wide tiles when there is enough work to fill the GPU; narrow ones otherwise.
  const long tiles256 = ((M + kBM - 1) / kBM) * static_cast<long>((N + 255) / 256);
  return N >= 256 && tiles256 >= 148;
}

struct GemmPlan {
  int shape;
  int splits;
};

// Tile shape and K split from a small cost model in units of one 128 x 128 x 64
// MMA step of one SM: waves x (k-blocks per unit x tile width x relative cost
// per FLOP + the tile's epilogue), plus, when K is split, the partials' round
// trip through L2 (written once, read once, and the output). Per FLOP a
// 128-wide tile moves twice the B bytes of a 256-wide one (about 15% slower);
// a CTA pair stages half of B per SM (about 15% faster than a single CTA).
// Weight gradients (M, N <= a few thousand, K = tokens) are the shapes that
// split; token-major GEMMs have enough tiles without it.
GemmPlan plan_gemm(int M, int N, int K, int sms, bool can_split) {
  const int k_blocks = (K + kBK - 1) / kBK;
  constexpr double kStepSeconds = 256.0 / 1.9e9;   // one 128x128x64 step at ~8K FLOP/clock
  constexpr double kPartialBandwidth = 8e12;        // partials stay in L2 between the two kernels
  GemmPlan best{N >= 256 ? kShapeWide : kShapeNarrow, 1};
  double best_t = 1e300;
  for (int shape : {kShapePair, kShapeWide, kShapeNarrow}) {
    const int tile_m = shape == kShapePair ? 2 * kBM : kBM;
    const int bn = shape == kShapeNarrow ? 128 : 256;
    if (bn == 256 && N < 256) continue;
    if (shape == kShapePair && M < tile_m) continue;
    const int slots = shape == kShapePair ? sms / 2 : sms;
    const double cost = shape == kShapeNarrow ? 1.15 : (shape == kShapePair ? 0.85 : 1.0);
    const long tiles = static_cast<long>((M + tile_m - 1) / tile_m) * ((N + bn - 1) / bn);
    const int max_split = can_split ? std::max(1, std::min(16, k_blocks / 4)) : 1;
    for (int sp = 1; sp <= max_split; ++sp) {
      const long units = tiles * sp;
      const long waves = (units + slots - 1) / slots;
      const double kb = static_cast<double>((k_blocks + sp - 1) / sp);
      const double unit_t = kb * (bn / 128.0) * cost + 2.0 * bn / 128.0;
      double t = static_cast<double>(waves) * unit_t;
      if (sp > 1) t += (sp + 2.0) * M * static_cast<double>(N) * 4.0 / kPartialBandwidth / kStepSeconds;
      if (t < best_t * 0.97) {
        best_t = t;
        best = GemmPlan{shape, sp};
      }
    }
  }
  return best;
}

// shape: a TileShape (kShapeAuto = the cost model's choice without a split).
template <bool A_MN, bool B_MN, int EPI>
void dispatch_bn(const at::Tensor& a, const at::Tensor& b, int M, int N, int K, GemmArgs& args,
                 cudaStream_t stream, int shape) {
  if (shape == kShapeAuto) shape = plan_gemm(M, N, K, sm_count(a.device().index()), false).shape;
  // A pair tile needs rows for both CTAs; a 256-wide tile needs 256 columns.
  if (shape == kShapePair && M < 2 * kBM) shape = kShapeWide;
  if (shape != kShapeNarrow && N < 256) shape = kShapeNarrow;
  if (shape == kShapePair) run_gemm<256, A_MN, B_MN, EPI, 2>(a, b, M, N, K, args, stream);
  else if (shape == kShapeWide) run_gemm<256, A_MN, B_MN, EPI>(a, b, M, N, K, args, stream);
  else run_gemm<128, A_MN, B_MN, EPI>(a, b, M, N, K, args, stream);
}

template <int EPI>
void dispatch_layout(const at::Tensor& a, bool a_mn, const at::Tensor& b, bool b_mn, int M, int N, int K,
                     GemmArgs& args, cudaStream_t stream, int shape = kShapeAuto) {
  if (!a_mn && !b_mn) dispatch_bn<false, false, EPI>(a, b, M, N, K, args, stream, shape);
  else if (!a_mn && b_mn) dispatch_bn<false, true, EPI>(a, b, M, N, K, args, stream, shape);
  else if (a_mn && !b_mn) dispatch_bn<true, false, EPI>(a, b, M, N, K, args, stream, shape);
  else dispatch_bn<true, true, EPI>(a, b, M, N, K, args, stream, shape);
}

// Sums the split partials ws[0..splits) in split order (so the result does
// not depend on which CTA finished first) and stores (or adds) them into the
// contiguous output. Four consecutive elements per thread.
template <bool kBf16Out>
__global__ void __launch_bounds__(256) splitk_reduce_kernel(const float4* __restrict__ ws, int splits, int64_t n4,
                                                            int64_t stride4, void* __restrict__ out, int accumulate) {
  const int64_t step = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n4; i += step) {
    float4 acc = ws[i];
    for (int s = 1; s < splits; ++s) {
      const float4 p = ws[s * stride4 + i];
      acc.x += p.x; acc.y += p.y; acc.z += p.z; acc.w += p.w;
    }
    if constexpr (kBf16Out) {
      static_cast<uint2*>(out)[i] = make_uint2(pack_bf16(acc.x, acc.y), pack_bf16(acc.z, acc.w));
    } else {
      float4* o = static_cast<float4*>(out) + i;
      if (accumulate) {
        const float4 old = *o;
        acc.x = old.x + acc.x; acc.y = old.y + acc.y; acc.z = old.z + acc.z; acc.w = old.w + acc.w;
      }
      *o = acc;
    }
  }
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
// shape: a TileShape to force (tests), 0 = chosen from the problem size.
void gemm(const at::Tensor& a, bool a_mn, const at::Tensor& b, bool b_mn, at::Tensor& out, int64_t epilogue,
          double alpha, const c10::optional<at::Tensor>& bias, const c10::optional<at::Tensor>& residual,
          const c10::optional<at::Tensor>& aux, const c10::optional<at::Tensor>& col_partial, int64_t shape) {
  TORCH_CHECK(shape >= kShapeAuto && shape <= kShapePair, "gemm: tile shape 0..3");
  TORCH_CHECK(gemm_supported(a, a_mn, b, b_mn), "gemm: bf16 2-D operands with 16-byte aligned rows required");
  const int M = a_mn ? a.size(1) : a.size(0);
  const int K = a_mn ? a.size(0) : a.size(1);
  const int N = b_mn ? b.size(1) : b.size(0);
  TORCH_CHECK((b_mn ? b.size(0) : b.size(1)) == K, "gemm: inner dimensions differ");
  TORCH_CHECK(out.dim() == 2 && out.size(0) == M && out.size(1) == N && out.stride(1) == 1, "gemm: bad output");
  const c10::cuda::CUDAGuard guard(a.device());
  GemmArgs args{};
  args.splits = 1;
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
  {
    // Vector epilogue accesses: 4 elements per access at column multiples of 4.
    auto ok = [](const void* p, int64_t ld, int elem) {
      return p == nullptr || ((reinterpret_cast<uintptr_t>(p) % 16) == 0 && (ld * elem) % 16 == 0);
    };
    args.vec = ok(args.out, args.ldo, out.element_size()) && ok(args.residual, args.ldr, 4) &&
               ok(args.aux, args.ld_aux, 2);
  }
  args.tma_out = tma_epilogue_ok(args, out.element_size()) ? 1 : 0;
  auto stream = at::cuda::getCurrentCUDAStream();
  switch (epilogue) {
    case kStoreBf16:
      TORCH_CHECK(out.scalar_type() == at::kBFloat16, "bf16 output");
      dispatch_layout<kStoreBf16>(a, a_mn, b, b_mn, M, N, K, args, stream, static_cast<int>(shape)); break;
    case kStoreF32:
      TORCH_CHECK(out.scalar_type() == at::kFloat, "fp32 output");
      dispatch_layout<kStoreF32>(a, a_mn, b, b_mn, M, N, K, args, stream, static_cast<int>(shape)); break;
    case kAccumF32:
      TORCH_CHECK(out.scalar_type() == at::kFloat, "fp32 output");
      dispatch_layout<kAccumF32>(a, a_mn, b, b_mn, M, N, K, args, stream, static_cast<int>(shape)); break;
    case kBiasGeluBf16:
      TORCH_CHECK(out.scalar_type() == at::kBFloat16 && args.aux && args.bias, "bias/aux needed");
      dispatch_layout<kBiasGeluBf16>(a, a_mn, b, b_mn, M, N, K, args, stream, static_cast<int>(shape)); break;
    case kBiasResidualF32:
      TORCH_CHECK(out.scalar_type() == at::kFloat && args.residual, "fp32 residual needed");
      dispatch_layout<kBiasResidualF32>(a, a_mn, b, b_mn, M, N, K, args, stream, static_cast<int>(shape)); break;
    case kGeluBackBf16:
      TORCH_CHECK(out.scalar_type() == at::kBFloat16 && args.aux && args.col_partial, "aux/partials needed");
      dispatch_layout<kGeluBackBf16>(a, a_mn, b, b_mn, M, N, K, args, stream, static_cast<int>(shape)); break;
    default:
      TORCH_CHECK(false, "unknown epilogue ", epilogue);
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  count_launch(1);
}

namespace {

PeerLayout make_layout(int64_t world, int64_t rank, int64_t parts, int64_t batch, int64_t n_local, int64_t C) {
  TORCH_CHECK(world >= 1 && world <= kMaxPeers && rank >= 0 && rank < world, "ulysses gemm: bad world/rank");
  TORCH_CHECK(parts >= 1 && batch >= 1 && n_local >= 1 && C >= 1, "ulysses gemm: bad layout");
  PeerLayout L{};
  L.world = static_cast<int>(world);
  L.rank = static_cast<int>(rank);
  L.parts = static_cast<int>(parts);
  L.batch = static_cast<int>(batch);
  L.n_local = static_cast<int>(n_local);
  L.n_total = static_cast<int>(n_local * world);
  L.C = static_cast<int>(C);
  L.dim = static_cast<int>(world * C);
  return L;
}

GemmArgs base_args(int M, int N, int K, const at::Tensor& ref) {
  GemmArgs args{};
  args.splits = 1;
  args.M = M;
  args.N = N;
  args.K = K;
  args.alpha = 1.f;
  args.err = device_error_slot(ref.device().index());
  return args;
}

}  // namespace

// Ulysses to-heads fused with its projection: Y = A op(B)^T in the sequence
// layout [batch * n_local, parts * world * C] is never materialised; each
// 4-column group goes to `dst[owner]`, the owner's [parts, batch, n_total, C]
// buffer (peer memory). Caller synchronises ranks afterwards.
void gemm_scatter(const at::Tensor& a, const at::Tensor& b, bool b_mn, const std::vector<int64_t>& dst,
                  int64_t rank, int64_t parts, int64_t batch, int64_t n_local, int64_t C) {
  TORCH_CHECK(gemm_supported(a, false, b, b_mn), "gemm_scatter: bf16 2-D operands with 16-byte aligned rows");
  const int64_t world = static_cast<int64_t>(dst.size());
  PeerLayout L = make_layout(world, rank, parts, batch, n_local, C);
  const int M = a.size(0), K = a.size(1);
  const int N = b_mn ? b.size(1) : b.size(0);
  TORCH_CHECK(M == batch * n_local && N == parts * world * C, "gemm_scatter: shapes do not match the layout");
  TORCH_CHECK((b_mn ? b.size(0) : b.size(1)) == K, "gemm_scatter: inner dimensions differ");
  for (int r = 0; r < world; ++r) {
    TORCH_CHECK(dst[r] % 16 == 0, "gemm_scatter: destination must be 16-byte aligned");
    L.dst[r] = reinterpret_cast<__nv_bfloat16*>(dst[r]);
  }
  const c10::cuda::CUDAGuard guard(a.device());
  GemmArgs args = base_args(M, N, K, a);
  args.vec = (C % 4) == 0;
  // 32 x 32 blocks stay inside one owner's columns and one batch's rows.
  static const bool tma_off = std::getenv("EB200_SCATTER_TMA") != nullptr &&
                              std::string(std::getenv("EB200_SCATTER_TMA")) == "0";
  L.tma_store = !tma_off && C % 32 == 0 && n_local % 32 == 0 ? 1 : 0;
  args.peer = L;
  PeerMaps pm{};
  if (L.tma_store)
    for (int r = 0; r < world; ++r)
      pm.map[r] = make_store_plane_map(reinterpret_cast<const void*>(dst[r]), parts * batch, L.n_total, C, 32, 32);
  auto stream = at::cuda::getCurrentCUDAStream();
  if (b_mn) {
    if (wide_tiles(M, N)) run_gemm<256, false, true, kScatterBf16>(a, b, M, N, K, args, stream, &pm);
    else run_gemm<128, false, true, kScatterBf16>(a, b, M, N, K, args, stream, &pm);
  } else {
    if (wide_tiles(M, N)) run_gemm<256, false, false, kScatterBf16>(a, b, M, N, K, args, stream, &pm);
    else run_gemm<128, false, false, kScatterBf16>(a, b, M, N, K, args, stream, &pm);
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  count_launch(1);
}

namespace {
template <int EPI>
void gather_dispatch(const PeerMaps& pm, const at::Tensor& b, bool b_mn, int M, int N, int K, GemmArgs& args,
                     cudaStream_t stream) {
  CUtensorMap none{};
  const bool wide = wide_tiles(M, N);
  if (b_mn) {
    if (wide) launch_gemm<256, false, true, EPI, true>(none, pm, b, M, N, K, args, stream);
    else launch_gemm<128, false, true, EPI, true>(none, pm, b, M, N, K, args, stream);
  } else {
    if (wide) launch_gemm<256, false, false, EPI, true>(none, pm, b, M, N, K, args, stream);
    else launch_gemm<128, false, false, EPI, true>(none, pm, b, M, N, K, args, stream);
  }
}
}  // namespace

// Ulysses to-sequence fused with the next projection: A[m, k] is read tile
// by tile with TMA straight from the owners' [parts, batch, n_total, C]
// buffers (`src[r]`, peer memory; plain tiled loads), out = epilogue(A op(B)^T).
void gemm_gather(const std::vector<int64_t>& src, int64_t rank, int64_t parts, int64_t batch, int64_t n_local,
                 int64_t C, const at::Tensor& b, bool b_mn, at::Tensor& out, int64_t epilogue,
                 const c10::optional<at::Tensor>& bias, const c10::optional<at::Tensor>& residual) {
  const int64_t world = static_cast<int64_t>(src.size());
  PeerLayout L = make_layout(world, rank, parts, batch, n_local, C);
  TORCH_CHECK(C % 64 == 0, "gemm_gather: heads_per_rank * head_dim must be a multiple of 64");
  TORCH_CHECK(n_local % kBM == 0, "gemm_gather: the local shard must be a multiple of 128 rows");
  TORCH_CHECK(b.is_cuda() && b.scalar_type() == at::kBFloat16 && b.dim() == 2 && aligned16(b), "gemm_gather: B");
  const int M = batch * n_local, K = parts * world * C;
  const int N = b_mn ? b.size(1) : b.size(0);
  TORCH_CHECK((b_mn ? b.size(0) : b.size(1)) == K, "gemm_gather: inner dimensions differ");
  TORCH_CHECK(out.dim() == 2 && out.size(0) == M && out.size(1) == N && out.stride(1) == 1, "gemm_gather: bad output");
  const c10::cuda::CUDAGuard guard(b.device());
  PeerMaps pm{};
  for (int r = 0; r < world; ++r)
    pm.map[r] = make_plane_map(reinterpret_cast<const void*>(src[r]), parts * batch, L.n_total, C, kBM);
  GemmArgs args = base_args(M, N, K, b);
  args.peer = L;
  args.out = out.data_ptr();
  args.ldo = out.stride(0);
  args.bias = bias.has_value() && bias->defined() ? bias->data_ptr<float>() : nullptr;
  if (residual.has_value() && residual->defined()) {
    TORCH_CHECK(residual->scalar_type() == at::kFloat && residual->stride(1) == 1, "gemm_gather: fp32 residual");
    args.residual = residual->data_ptr<float>();
    args.ldr = residual->stride(0);
  }
  auto ok = [](const void* p, int64_t ld, int elem) {
    return p == nullptr || ((reinterpret_cast<uintptr_t>(p) % 16) == 0 && (ld * elem) % 16 == 0);
  };
  args.vec = ok(args.out, args.ldo, out.element_size()) && ok(args.residual, args.ldr, 4);
  auto stream = at::cuda::getCurrentCUDAStream();
  switch (epilogue) {
    case kStoreBf16:
      TORCH_CHECK(out.scalar_type() == at::kBFloat16, "bf16 output");
      gather_dispatch<kStoreBf16>(pm, b, b_mn, M, N, K, args, stream); break;
    case kBiasResidualF32:
      TORCH_CHECK(out.scalar_type() == at::kFloat && args.residual, "fp32 residual needed");
      gather_dispatch<kBiasResidualF32>(pm, b, b_mn, M, N, K, args, stream); break;
    default:
      TORCH_CHECK(false, "gemm_gather: epilogue ", epilogue, " is not instantiated");
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  count_launch(1);
}

// out = op(A) op(B)^T (store) or out += op(A) op(B)^T (accumulate, fp32 out)
// with no fused epilogue: the linear layers' plain forwards (bf16 or fp32
// logits), their input gradients (dx = dy W, B MN-major) and their weight
// gradients (dW = dy^T x, both operands MN-major, accumulated into the fp32
// gradient). Few-tile shapes split K: fp32 partials of each split go to a
// workspace and one reduce kernel sums them in a fixed order (deterministic,
// no atomics) into the output. `splits`: 0 = chosen by the cost model.
// Returns the split count used.
int64_t gemm_plain(const at::Tensor& a, bool a_mn, const at::Tensor& b, bool b_mn, at::Tensor& out, bool accumulate,
                   int64_t splits, int64_t shape) {
  TORCH_CHECK(shape >= kShapeAuto && shape <= kShapePair, "gemm_plain: tile shape 0..3");
  TORCH_CHECK(gemm_supported(a, a_mn, b, b_mn), "gemm_plain: bf16 2-D operands with 16-byte aligned rows required");
  const int M = a_mn ? a.size(1) : a.size(0);
  const int K = a_mn ? a.size(0) : a.size(1);
  const int N = b_mn ? b.size(1) : b.size(0);
  TORCH_CHECK((b_mn ? b.size(0) : b.size(1)) == K, "gemm_plain: inner dimensions differ");
  TORCH_CHECK(out.dim() == 2 && out.size(0) == M && out.size(1) == N && out.stride(1) == 1, "gemm_plain: bad output");
  const bool bf16_out = out.scalar_type() == at::kBFloat16;
  TORCH_CHECK(bf16_out || out.scalar_type() == at::kFloat, "gemm_plain: bf16 or fp32 output");
  TORCH_CHECK(!(accumulate && bf16_out), "gemm_plain: accumulation needs an fp32 output");
  const c10::cuda::CUDAGuard guard(a.device());
  const int sms = sm_count(a.device().index());
  const int k_blocks = (K + kBK - 1) / kBK;
  // The reduce kernel reads and writes four contiguous elements at a time.
  const bool can_split = out.is_contiguous() && N % 4 == 0 &&
                         reinterpret_cast<uintptr_t>(out.data_ptr()) % 16 == 0 && k_blocks >= 2;
  GemmPlan plan = plan_gemm(M, N, K, sms, can_split);
  if (splits > 0) plan.splits = can_split ? static_cast<int>(std::min<int64_t>(splits, k_blocks)) : 1;
  if (shape != kShapeAuto) plan.shape = static_cast<int>(shape);
  auto stream = at::cuda::getCurrentCUDAStream();
  GemmArgs args = base_args(M, N, K, a);
  args.ldo = out.stride(0);
  if (plan.splits == 1) {
    args.out = out.data_ptr();
    args.vec = (reinterpret_cast<uintptr_t>(out.data_ptr()) % 16) == 0 && (args.ldo * out.element_size()) % 16 == 0;
    args.tma_out = tma_epilogue_ok(args, out.element_size()) ? 1 : 0;
    if (bf16_out) dispatch_layout<kStoreBf16>(a, a_mn, b, b_mn, M, N, K, args, stream, plan.shape);
    else if (accumulate) dispatch_layout<kAccumF32>(a, a_mn, b, b_mn, M, N, K, args, stream, plan.shape);
    else dispatch_layout<kStoreF32>(a, a_mn, b, b_mn, M, N, K, args, stream, plan.shape);
    C10_CUDA_KERNEL_LAUNCH_CHECK();
    count_launch(1);
    return 1;
  }
  auto ws = at::empty({plan.splits, static_cast<int64_t>(M), static_cast<int64_t>(N)}, out.options().dtype(at::kFloat));
  args.out = ws.data_ptr();
  args.ldo = N;
  args.splits = plan.splits;
  args.split_stride = static_cast<int64_t>(M) * N;
  args.vec = 1;
  args.tma_out = tma_epilogue_ok(args, 4) ? 1 : 0;
  dispatch_layout<kStoreF32>(a, a_mn, b, b_mn, M, N, K, args, stream, plan.shape);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  const int64_t n4 = static_cast<int64_t>(M) * N / 4;
  const int grid = static_cast<int>(std::min<int64_t>((n4 + 255) / 256, static_cast<int64_t>(sms) * 8));
  if (bf16_out)
    splitk_reduce_kernel<true><<<grid, 256, 0, stream>>>(reinterpret_cast<const float4*>(ws.data_ptr()),
                                                         plan.splits, n4, n4, out.data_ptr(), 0);
  else
    splitk_reduce_kernel<false><<<grid, 256, 0, stream>>>(reinterpret_cast<const float4*>(ws.data_ptr()),
                                                          plan.splits, n4, n4, out.data_ptr(), accumulate ? 1 : 0);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  count_launch(2);
  return plan.splits;
}

// The plan gemm_plain would use: (tile shape: 1 = 128 x 128, 2 = 128 x 256,
// 3 = 256 x 256 on a CTA pair; splits), for tests and tools.
std::vector<int64_t> gemm_plain_plan(int64_t M, int64_t N, int64_t K, int64_t sms) {
  const GemmPlan plan = plan_gemm(static_cast<int>(M), static_cast<int>(N), static_cast<int>(K),
                                  static_cast<int>(sms), N % 4 == 0 && (K + kBK - 1) / kBK >= 2);
  return {plan.shape, plan.splits};
}

int64_t gemm_tile_m() { return kBM; }

}  // namespace eb
