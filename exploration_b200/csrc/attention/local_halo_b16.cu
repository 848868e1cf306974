// Local halo window attention, specialised for block 16 and head_dim 64 (the
// shape of every Stack preset), sm_100a.
//
// Same semantics as local_halo.cu (window of the previous and the current
// 16-token block, causal, keys limited to [valid_start, start + n), RoPE
// relative to the query), but a CTA covers 128 query rows (8 blocks) of one
// head, so each key row is staged once instead of twice, and every thread
// computes 4 x 4 (scores) or 4 x 8 (context, gradients) register
// micro-tiles, reading shared memory once per 4-8 FMAs.
//
// Rotations are taken relative to the CTA origin (16 rows before its first
// query). RoPE only depends on the query/key distance, so this equals the
// block-relative convention of the reference up to fp32 rounding of the
// angle tables.
//
// Backward (owner computes, no atomics): the CTA of key rows [s, s + 128)
// recomputes P and dS for its own 8 query blocks and for the first block of
// the next CTA (whose window starts in this CTA's last block), then writes
// dQ of its query rows and dK/dV of its key rows.
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "../common/util.cuh"

namespace eb {
namespace {

constexpr int kB = 16;        // gate block
constexpr int kD = 64;        // head dim
constexpr int kRowsCta = 128; // query rows per CTA
constexpr int kThreads = 256; // 8 warps: warp w owns query block w
constexpr int kLdS = 65;      // padded fp32 row for scalar access
constexpr int kLdV = 68;      // 16-byte aligned fp32 row for float4 access
constexpr int kLdP = 33;

struct Args {
  const void* qkv;     // [B, n, 3, H, 64]
  const void* prev;    // [B, 16, 3, H, 64] or nullptr
  const float* cos;    // [kTable, 32] for offsets 0 .. kTable-1
  const float* sin;
  int n, heads;
  int64_t start, valid_start;
};
constexpr int kTable = kRowsCta + 2 * kB;   // offsets used by the backward: up to 160

template <typename T>
EB_DEVICE const T* row_ptr(const Args& a, int batch, int t, int part, int head) {
  const int64_t stride = 3LL * a.heads * kD;
  if (t < 0)
    return static_cast<const T*>(a.prev) + (static_cast<int64_t>(batch) * kB + t + kB) * stride +
           (static_cast<int64_t>(part) * a.heads + head) * kD;
  return static_cast<const T*>(a.qkv) + (static_cast<int64_t>(batch) * a.n + t) * stride +
         (static_cast<int64_t>(part) * a.heads + head) * kD;
}

EB_DEVICE bool key_ok(const Args& a, int t) {
  if (t < 0 && a.prev == nullptr) return false;
  return t < a.n && a.start + t >= a.valid_start;
}

template <typename T>
EB_DEVICE void load8(const T* src, float (&x)[8]);
template <>
EB_DEVICE void load8<__nv_bfloat16>(const __nv_bfloat16* src, float (&x)[8]) {
  const uint4 u = *reinterpret_cast<const uint4*>(src);
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __bfloat1622float2(h[i]);
    x[2 * i] = f.x;
    x[2 * i + 1] = f.y;
  }
}
template <>
EB_DEVICE void load8<float>(const float* src, float (&x)[8]) {
  const float4 a = *reinterpret_cast<const float4*>(src);
  const float4 b = *reinterpret_cast<const float4*>(src + 4);
  x[0] = a.x; x[1] = a.y; x[2] = a.z; x[3] = a.w; x[4] = b.x; x[5] = b.y; x[6] = b.z; x[7] = b.w;
}

template <typename T>
EB_DEVICE void store8(T* dst, const float (&x)[8]);
template <>
EB_DEVICE void store8<__nv_bfloat16>(__nv_bfloat16* dst, const float (&x)[8]) {
  uint4 u;
  __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(x[2 * i], x[2 * i + 1]);
  *reinterpret_cast<uint4*>(dst) = u;
}
template <>
EB_DEVICE void store8<float>(float* dst, const float (&x)[8]) {
  *reinterpret_cast<float4*>(dst) = make_float4(x[0], x[1], x[2], x[3]);
  *reinterpret_cast<float4*>(dst + 4) = make_float4(x[4], x[5], x[6], x[7]);
}

// Stage `rows` rows of part `part` starting at token t0, rotated by offset
// (row index + off0) when `rotate`; invalid rows are zero.
template <typename T>
EB_DEVICE void stage_rows(float* dst, int ld, const Args& a, int batch, int head, int part, int t0, int rows,
                          bool rotate, int off0, bool keys) {
  if (rotate) {
    for (int item = threadIdx.x; item < rows * 4; item += kThreads) {
      const int r = item >> 2, c = item & 3;
      const int t = t0 + r;
      const bool ok = keys ? key_ok(a, t) : (t >= 0 && t < a.n);
      float x1[8], x2[8];
      if (ok) {
        const T* src = row_ptr<T>(a, batch, t, part, head);
        load8<T>(src + 8 * c, x1);
        load8<T>(src + 8 * c + 32, x2);
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) x1[i] = x2[i] = 0.f;
      }
      const float* cs = a.cos + (r + off0) * 32 + 8 * c;
      const float* sn = a.sin + (r + off0) * 32 + 8 * c;
      float* d = dst + r * ld + 8 * c;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        d[i] = x1[i] * cs[i] - x2[i] * sn[i];
        d[i + 32] = x2[i] * cs[i] + x1[i] * sn[i];
      }
    }
  } else {
    for (int item = threadIdx.x; item < rows * 8; item += kThreads) {
      const int r = item >> 3, c = item & 7;
      const int t = t0 + r;
      const bool ok = keys ? key_ok(a, t) : (t >= 0 && t < a.n);
      float x[8];
      if (ok) {
        load8<T>(row_ptr<T>(a, batch, t, part, head) + 8 * c, x);
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) x[i] = 0.f;
      }
      float* d = dst + r * ld + 8 * c;
#pragma unroll
      for (int i = 0; i < 8; ++i) d[i] = x[i];
    }
  }
}

template <typename T>
__global__ void __launch_bounds__(kThreads)
local16_fwd(Args a, T* __restrict__ out, float* __restrict__ lse) {
  extern __shared__ float smem[];
  float* Ks = smem;                          // [144][65] keys t0-16 .. t0+127 (rotated)
  float* Vs = Ks + (kRowsCta + kB) * kLdS;   // [144][68]
  float* Qs = Vs + (kRowsCta + kB) * kLdV;   // [128][65] (rotated)
  float* Ps = Qs + kRowsCta * kLdS;          // [8][16][33]
  bool* valid = reinterpret_cast<bool*>(Ps + 8 * kB * kLdP);   // [144]
  const int head = blockIdx.y, batch = blockIdx.z;
  const int t0 = blockIdx.x * kRowsCta;      // first query row of the CTA
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  stage_rows<T>(Ks, kLdS, a, batch, head, 1, t0 - kB, kRowsCta + kB, true, 0, true);
  stage_rows<T>(Vs, kLdV, a, batch, head, 2, t0 - kB, kRowsCta + kB, false, 0, true);
  stage_rows<T>(Qs, kLdS, a, batch, head, 0, t0, kRowsCta, true, kB, false);
  for (int r = threadIdx.x; r < kRowsCta + kB; r += kThreads) valid[r] = key_ok(a, t0 - kB + r);
  __syncthreads();
  const int w = warp;                        // query block within the CTA
  const int rg = lane >> 3, kg = lane & 7;   // 4 rows x 4 keys per lane
  const float scale = 0.125f;                // 1 / sqrt(64)
  float acc[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;
  const float* qb = Qs + (w * kB + 4 * rg) * kLdS;
  const float* kb = Ks + (w * kB + 4 * kg) * kLdS;
#pragma unroll 8
  for (int d = 0; d < kD; ++d) {
    float q[4], k[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) q[i] = qb[i * kLdS + d];
#pragma unroll
    for (int j = 0; j < 4; ++j) k[j] = kb[j * kLdS + d];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) acc[i][j] += q[i] * k[j];
  }
  float* pw = Ps + w * kB * kLdP;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int r = 4 * rg + i;
    float s[4], m = kNegInf;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int c = 4 * kg + j;
      const bool ok = c <= kB + r && valid[w * kB + c];
      s[j] = ok ? acc[i][j] * scale : kNegInf;
      m = fmaxf(m, s[j]);
    }
#pragma unroll
    for (int o = 1; o < 8; o <<= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    float sum = 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      s[j] = (s[j] == kNegInf) ? 0.f : expf(s[j] - m);
      sum += s[j];
    }
#pragma unroll
    for (int o = 1; o < 8; o <<= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    const float inv = sum > 0.f ? 1.f / sum : 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j) pw[r * kLdP + 4 * kg + j] = s[j] * inv;
    const int t = t0 + w * kB + r;
    if (kg == 0 && t < a.n) lse[(static_cast<int64_t>(batch) * a.n + t) * a.heads + head] = m + logf(sum);
  }
  __syncwarp();
  // Context: lane -> 4 rows x 8 dims.
  const int dg = lane & 7;
  float o[4][8];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) o[i][j] = 0.f;
  const float* vb = Vs + (w * kB) * kLdV + 8 * dg;
#pragma unroll 4
  for (int c = 0; c < 2 * kB; ++c) {
    const float4 v0 = *reinterpret_cast<const float4*>(vb + c * kLdV);
    const float4 v1 = *reinterpret_cast<const float4*>(vb + c * kLdV + 4);
    const float vv[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float p = pw[(4 * rg + i) * kLdP + c];
#pragma unroll
      for (int j = 0; j < 8; ++j) o[i][j] += p * vv[j];
    }
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int t = t0 + w * kB + 4 * rg + i;
    if (t < a.n) store8<T>(out + (static_cast<int64_t>(batch) * a.n + t) * a.heads * kD + head * kD + 8 * dg, o[i]);
  }
}

template <typename T>
__global__ void __launch_bounds__(kThreads)
local16_bwd(Args a, const T* __restrict__ dout, const T* __restrict__ out, const float* __restrict__ lse,
            T* __restrict__ dqkv, T* __restrict__ dprev) {
  extern __shared__ float smem[];
  constexpr int kQRows = kRowsCta + kB;      // 9 query blocks
  float* Qs = smem;                          // [144][65]: query rows s .. s+143 (rotated, offset +16)
  float* Gs = Qs + kQRows * kLdS;            // [144][68]: dO rows s .. s+143
  float* Ks = Gs + kQRows * kLdV;            // [144][65]: key rows s-16 .. s+127 (rotated)
  float* Vs = Ks + kQRows * kLdS;            // [144][68]
  float* Pb = Vs + kQRows * kLdV;            // [9][16][33]
  float* Sb = Pb + 9 * kB * kLdP;            // [9][16][33] dS
  float* rowf = Sb + 9 * kB * kLdP;          // [144][2]: lse, delta
  bool* valid = reinterpret_cast<bool*>(rowf + 2 * kQRows);
  const int head = blockIdx.y, batch = blockIdx.z;
  const int s0 = blockIdx.x * kRowsCta;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  stage_rows<T>(Ks, kLdS, a, batch, head, 1, s0 - kB, kQRows, true, 0, true);
  stage_rows<T>(Vs, kLdV, a, batch, head, 2, s0 - kB, kQRows, false, 0, true);
  stage_rows<T>(Qs, kLdS, a, batch, head, 0, s0, kQRows, true, kB, false);
  // dO rows (plain copy) and per-row lse / delta.
  const int64_t row_stride = static_cast<int64_t>(a.heads) * kD;
  for (int item = threadIdx.x; item < kQRows * 8; item += kThreads) {
    const int r = item >> 3, c = item & 7;
    const int t = s0 + r;
    float x[8];
    if (t < a.n) {
      load8<T>(dout + (static_cast<int64_t>(batch) * a.n + t) * row_stride + head * kD + 8 * c, x);
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) x[i] = 0.f;
    }
    float* d = Gs + r * kLdV + 8 * c;
#pragma unroll
    for (int i = 0; i < 8; ++i) d[i] = x[i];
  }
  for (int r = warp; r < kQRows; r += 8) {
    const int t = s0 + r;
    float delta = 0.f, l = 0.f;
    if (t < a.n) {
      const int64_t base = (static_cast<int64_t>(batch) * a.n + t) * row_stride + head * kD;
      for (int d = lane; d < kD; d += 32) delta += load_f(dout + base + d) * load_f(out + base + d);
      l = lse[(static_cast<int64_t>(batch) * a.n + t) * a.heads + head];
    }
    delta = warp_sum(delta);
    if (lane == 0) {
      rowf[2 * r] = l;
      rowf[2 * r + 1] = delta;
    }
  }
  for (int r = threadIdx.x; r < kQRows; r += kThreads) valid[r] = key_ok(a, s0 - kB + r);
  __syncthreads();
  const float scale = 0.125f;
  const int rg = lane >> 3, kg = lane & 7;
  // P and dS for query blocks 0..7 (warp w) and block 8 (warp 0, keys of block 7 only).
  for (int blk = warp; blk < 9; blk += 8) {
    const int ncols = blk < 8 ? 2 * kB : kB;
    float sacc[4][4], pacc[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) sacc[i][j] = pacc[i][j] = 0.f;
    if (4 * kg < ncols) {
      const float* qb = Qs + (blk * kB + 4 * rg) * kLdS;
      const float* gb = Gs + (blk * kB + 4 * rg) * kLdV;
      const float* kb = Ks + (blk * kB + 4 * kg) * kLdS;
      const float* vb = Vs + (blk * kB + 4 * kg) * kLdV;
#pragma unroll 4
      for (int d = 0; d < kD; ++d) {
        float q[4], g[4], k[4], v[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          q[i] = qb[i * kLdS + d];
          g[i] = gb[i * kLdV + d];
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          k[j] = kb[j * kLdS + d];
          v[j] = vb[j * kLdV + d];
        }
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            sacc[i][j] += q[i] * k[j];
            pacc[i][j] += g[i] * v[j];
          }
      }
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int r = 4 * rg + i;
      const int qr = blk * kB + r;
      const bool row_ok = s0 + qr < a.n;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int c = 4 * kg + j;
        float p = 0.f, ds = 0.f;
        if (row_ok && c < ncols && c <= kB + r && valid[blk * kB + c]) {
          p = expf(sacc[i][j] * scale - rowf[2 * qr]);
          ds = p * (pacc[i][j] - rowf[2 * qr + 1]);
        }
        if (c < 2 * kB) {
          Pb[(blk * kB + r) * kLdP + c] = p;
          Sb[(blk * kB + r) * kLdP + c] = ds;
        }
      }
    }
  }
  __syncthreads();
  const int dg = lane & 7;
  // dQ of query block w: sum_c dS[r][c] K[c], un-rotated by the query offset.
  {
    const int w = warp;
    float acc[4][8];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[i][j] = 0.f;
    for (int c = 0; c < 2 * kB; ++c) {
      float k1[4], k2[4];   // dims [4dg, 4dg+4) and +32: paired halves for the inverse rotation
      const float* kr = Ks + (w * kB + c) * kLdS;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        k1[j] = kr[4 * dg + j];
        k2[j] = kr[4 * dg + j + 32];
      }
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float ds = Sb[(w * kB + 4 * rg + i) * kLdP + c];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          acc[i][j] += ds * k1[j];
          acc[i][j + 4] += ds * k2[j];
        }
      }
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int r = w * kB + 4 * rg + i;
      const int t = s0 + r;
      if (t >= a.n) continue;
      const float* cs = a.cos + (r + kB) * 32 + 4 * dg;
      const float* sn = a.sin + (r + kB) * 32 + 4 * dg;
      T* dq = dqkv + (static_cast<int64_t>(batch) * a.n + t) * 3 * row_stride + head * kD;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float g1 = acc[i][j], g2 = acc[i][j + 4];
        dq[4 * dg + j] = cast_f<T>((g1 * cs[j] + g2 * sn[j]) * scale);
        dq[4 * dg + j + 32] = cast_f<T>((g2 * cs[j] - g1 * sn[j]) * scale);
      }
    }
  }
  // dK / dV of key block w (key rows s0 + 16w + j): from query blocks w (column 16 + j) and w + 1 (column j).
  {
    const int w = warp;
    const int jg = rg;     // 4 keys per lane group
    float ak[4][8], av[4][8];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 8; ++j) ak[i][j] = av[i][j] = 0.f;
#pragma unroll 1
    for (int part = 0; part < 2; ++part) {
      const int blk = w + part;        // query block
      const int col0 = part == 0 ? kB : 0;
      for (int r = 0; r < kB; ++r) {
        const int qr = blk * kB + r;
        float q1[4], q2[4];
        const float* qrow = Qs + qr * kLdS;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          q1[j] = qrow[4 * dg + j];
          q2[j] = qrow[4 * dg + j + 32];
        }
        const float4 g0 = *reinterpret_cast<const float4*>(Gs + qr * kLdV + 4 * dg);
        const float4 g1 = *reinterpret_cast<const float4*>(Gs + qr * kLdV + 4 * dg + 32);
        const float gg[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int c = col0 + 4 * jg + i;
          const float ds = Sb[qr * kLdP + c], p = Pb[qr * kLdP + c];
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            ak[i][j] += ds * q1[j];
            ak[i][j + 4] += ds * q2[j];
          }
#pragma unroll
          for (int j = 0; j < 8; ++j) av[i][j] += p * gg[j];
        }
      }
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int kr = w * kB + 4 * jg + i;     // key row within the CTA (0..127)
      const int t = s0 + kr;
      if (t >= a.n) continue;
      const float* cs = a.cos + (kr + kB) * 32 + 4 * dg;
      const float* sn = a.sin + (kr + kB) * 32 + 4 * dg;
      T* dk = dqkv + (static_cast<int64_t>(batch) * a.n + t) * 3 * row_stride + row_stride + head * kD;
      T* dv = dk + row_stride;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float g1 = ak[i][j], g2 = ak[i][j + 4];
        dk[4 * dg + j] = cast_f<T>((g1 * cs[j] + g2 * sn[j]) * scale);
        dk[4 * dg + j + 32] = cast_f<T>((g2 * cs[j] - g1 * sn[j]) * scale);
        dv[4 * dg + j] = cast_f<T>(av[i][j]);
        dv[4 * dg + j + 32] = cast_f<T>(av[i][j + 4]);
      }
    }
  }
  // Halo block: keys -16 .. -1 receive gradient from query block 0 (columns 0..15).
  if (blockIdx.x == 0 && dprev != nullptr && warp == 0) {
    const int jg = rg;
    float ak[4][8], av[4][8];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 8; ++j) ak[i][j] = av[i][j] = 0.f;
    for (int r = 0; r < kB; ++r) {
      float q1[4], q2[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        q1[j] = Qs[r * kLdS + 4 * dg + j];
        q2[j] = Qs[r * kLdS + 4 * dg + j + 32];
      }
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int c = 4 * jg + i;
        const float ds = Sb[r * kLdP + c], p = Pb[r * kLdP + c];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          ak[i][j] += ds * q1[j];
          ak[i][j + 4] += ds * q2[j];
          av[i][j] += p * Gs[r * kLdV + 4 * dg + j];
          av[i][j + 4] += p * Gs[r * kLdV + 4 * dg + j + 32];
        }
      }
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int j_key = 4 * jg + i;          // halo row, key offset j_key relative to the CTA origin
      const float* cs = a.cos + j_key * 32 + 4 * dg;
      const float* sn = a.sin + j_key * 32 + 4 * dg;
      T* dk = dprev + (static_cast<int64_t>(batch) * kB + j_key) * 3 * row_stride + row_stride + head * kD;
      T* dv = dk + row_stride;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float g1 = ak[i][j], g2 = ak[i][j + 4];
        dk[4 * dg + j] = cast_f<T>((g1 * cs[j] + g2 * sn[j]) * scale);
        dk[4 * dg + j + 32] = cast_f<T>((g2 * cs[j] - g1 * sn[j]) * scale);
        dv[4 * dg + j] = cast_f<T>(av[i][j]);
        dv[4 * dg + j + 32] = cast_f<T>(av[i][j + 4]);
      }
    }
  }
}

constexpr size_t kFwdSmem = sizeof(float) * ((kRowsCta + kB) * (kLdS + kLdV) + kRowsCta * kLdS + 8 * kB * kLdP) +
                            (kRowsCta + kB);
constexpr size_t kBwdSmem = sizeof(float) * ((kRowsCta + kB) * (2 * kLdS + 2 * kLdV) + 2 * 9 * kB * kLdP +
                                             2 * (kRowsCta + kB)) + (kRowsCta + kB);

std::pair<at::Tensor, at::Tensor> tables(const at::Device& device) {
  // Never destroyed (see the note on static tensors in local_tc.cu's tables).
  static at::Tensor* cos_t = new at::Tensor[16];
  static at::Tensor* sin_t = new at::Tensor[16];
  const int idx = device.index();
  if (!cos_t[idx].defined()) {
    auto offsets = at::arange(0, kTable, at::TensorOptions().dtype(at::kFloat));
    auto index = at::arange(0, kD, 2, at::TensorOptions().dtype(at::kFloat));
    auto inv = at::pow(10000.0, -index / static_cast<double>(kD));
    auto angles = offsets.unsqueeze(1) * inv.unsqueeze(0);
    cos_t[idx] = angles.cos().to(device).contiguous();
    sin_t[idx] = angles.sin().to(device).contiguous();
  }
  return {cos_t[idx], sin_t[idx]};
}

}  // namespace

bool local16_supported(int block, int dim) { return block == kB && dim == kD; }

std::vector<at::Tensor> local16_fwd_launch(const at::Tensor& qkv, const c10::optional<at::Tensor>& prev,
                                           int64_t start, int64_t valid_start, int64_t n) {
  const int batch = qkv.size(0), heads = qkv.size(3);
  auto t = tables(qkv.device());
  Args a{qkv.data_ptr(), prev.has_value() ? prev->data_ptr() : nullptr, t.first.data_ptr<float>(),
         t.second.data_ptr<float>(), static_cast<int>(n), heads, start, valid_start};
  auto out = at::empty({batch, n, heads * kD}, qkv.options());
  auto lse = at::empty({batch, n, heads}, qkv.options().dtype(at::kFloat));
  dim3 grid((n + kRowsCta - 1) / kRowsCta, heads, batch);
  auto stream = at::cuda::getCurrentCUDAStream();
  if (qkv.scalar_type() == at::kBFloat16) {
    EB_CUDA_CHECK(cudaFuncSetAttribute(local16_fwd<__nv_bfloat16>, cudaFuncAttributeMaxDynamicSharedMemorySize, kFwdSmem));
    local16_fwd<__nv_bfloat16><<<grid, kThreads, kFwdSmem, stream>>>(
        a, reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), lse.data_ptr<float>());
  } else {
    EB_CUDA_CHECK(cudaFuncSetAttribute(local16_fwd<float>, cudaFuncAttributeMaxDynamicSharedMemorySize, kFwdSmem));
    local16_fwd<float><<<grid, kThreads, kFwdSmem, stream>>>(a, out.data_ptr<float>(), lse.data_ptr<float>());
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  count_launch(1);
  return {out, lse};
}

std::vector<at::Tensor> local16_bwd_launch(const at::Tensor& dout, const at::Tensor& qkv,
                                           const c10::optional<at::Tensor>& prev, const at::Tensor& out,
                                           const at::Tensor& lse, int64_t start, int64_t valid_start, int64_t n) {
  const int batch = qkv.size(0), heads = qkv.size(3);
  auto t = tables(qkv.device());
  Args a{qkv.data_ptr(), prev.has_value() ? prev->data_ptr() : nullptr, t.first.data_ptr<float>(),
         t.second.data_ptr<float>(), static_cast<int>(n), heads, start, valid_start};
  auto dqkv = at::empty_like(qkv);
  at::Tensor dprev;
  if (prev.has_value()) dprev = at::zeros_like(*prev);
  dim3 grid((n + kRowsCta - 1) / kRowsCta, heads, batch);
  auto stream = at::cuda::getCurrentCUDAStream();
  if (qkv.scalar_type() == at::kBFloat16) {
    using T = __nv_bfloat16;
    EB_CUDA_CHECK(cudaFuncSetAttribute(local16_bwd<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, kBwdSmem));
    local16_bwd<T><<<grid, kThreads, kBwdSmem, stream>>>(
        a, reinterpret_cast<const T*>(dout.data_ptr()), reinterpret_cast<const T*>(out.data_ptr()),
        lse.data_ptr<float>(), reinterpret_cast<T*>(dqkv.data_ptr()),
        prev.has_value() ? reinterpret_cast<T*>(dprev.data_ptr()) : nullptr);
  } else {
    EB_CUDA_CHECK(cudaFuncSetAttribute(local16_bwd<float>, cudaFuncAttributeMaxDynamicSharedMemorySize, kBwdSmem));
    local16_bwd<float><<<grid, kThreads, kBwdSmem, stream>>>(a, dout.data_ptr<float>(), out.data_ptr<float>(),
                                                              lse.data_ptr<float>(), dqkv.data_ptr<float>(),
                                                              prev.has_value() ? dprev.data_ptr<float>() : nullptr);
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  count_launch(1);
  return {dqkv, dprev};
}

}  // namespace eb
