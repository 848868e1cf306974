// Exact block-gated dense attention, fp32-accumulating CUDA-core kernels.
//
// These kernels serve fp32 inputs (IEEE fp32 products, no TF32, matching
// the reference's fp32 tolerance) and the head dims / block sizes the
// tcgen05 kernel does not specialise. Layout: q [B,Q,H,D], k/v [B,N,H,D],
// pos [B,Q] int32 (-1 = padding row).
//
// Tiling: a CTA owns 16 query rows of one (batch, head) and streams key
// tiles of T = max(b, 32) keys (a whole number of gate blocks, so each
// block's log-mass is computed inside one tile). Shared memory holds one
// K-or-V tile at a time (fp32, padded rows), so D = 256 with b = 128 fits.
//
// Backward ownership (no atomics, deterministic): the dQ kernel owns query
// rows, the dK/dV kernel owns key tiles and, for wide D, a slice of the
// head dimension (the probabilities are recomputed per slice).
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "../common/util.cuh"
#include "gated_common.cuh"

namespace eb {
namespace {

constexpr int kRows = 16;
constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kMaxAcc = 16;   // per-thread accumulators (16 rows x D<=256 over 256 threads)

template <typename T>
EB_DEVICE void load_tile(float* dst, int ld, const T* src, int64_t row0, int rows_valid, int rows,
                         int heads, int head, int dim) {
  // src row r at ((row0 + r) * heads + head) * dim; rows >= rows_valid are zero.
  for (int e = threadIdx.x; e < rows * dim; e += kThreads) {
    const int r = e / dim, d = e % dim;
    dst[r * ld + d] = r < rows_valid ? load_f(src + ((row0 + r) * heads + head) * dim + d) : 0.f;
  }
}

// S[r][c] = q_r . k_c over D for 16 rows x T keys (unscaled).
EB_DEVICE void tile_dots(float* S, const float* Qs, const float* Ks, int ld, int TK, int dim) {
  for (int e = threadIdx.x; e < kRows * TK; e += kThreads) {
    const int r = e / TK, c = e % TK;
    const float* q = Qs + r * ld;
    const float* k = Ks + c * ld;
    float acc = 0.f;
    for (int d = 0; d < dim; ++d) acc += q[d] * k[d];
    S[r * TK + c] = acc;
  }
}

// Per-row logits a (scaled, -inf past N) and per-key block log-mass sb of one tile.
// One warp per row; T <= 128 so a lane holds at most 4 columns.
EB_DEVICE void row_block_scores(const float* S, int TK, int row, int k0, int nk, int b, float scale,
                                float a[4], float sb[4]) {
  const int lane = threadIdx.x & 31;
  const int per = TK / 32 > 0 ? TK / 32 : 1;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    a[i] = kNegInf;
    sb[i] = kNegInf;
  }
  for (int i = 0; i < per; ++i) {
    const int c = lane + 32 * i;
    if (c < TK && k0 + c < nk) a[i] = S[row * TK + c] * scale;
  }
  if (b <= 32) {
    for (int i = 0; i < per; ++i) {
      float m = a[i];
      for (int o = b >> 1; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
      float e = (m == kNegInf) ? 0.f : expf(a[i] - m);
      for (int o = b >> 1; o > 0; o >>= 1) e += __shfl_xor_sync(0xffffffffu, e, o);
      sb[i] = (m == kNegInf) ? kNegInf : m + logf(e);
    }
  } else {   // T == b: the tile is one gate block
    float m = kNegInf;
    for (int i = 0; i < per; ++i) m = fmaxf(m, a[i]);
    m = warp_max(m);
    float e = 0.f;
    for (int i = 0; i < per; ++i) e += (a[i] == kNegInf) ? 0.f : expf(a[i] - m);
    e = warp_sum(e);
    const float s = (m == kNegInf) ? kNegInf : m + logf(e);
    for (int i = 0; i < per; ++i) sb[i] = s;
  }
}

// Segmented (per gate block) sum of x over the tile, same lane mapping.
EB_DEVICE void block_sums(int TK, int b, float x[4], float out[4]) {
  const int per = TK / 32 > 0 ? TK / 32 : 1;
  if (b <= 32) {
    for (int i = 0; i < per; ++i) {
      float v = x[i];
      for (int o = b >> 1; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
      out[i] = v;
    }
  } else {
    float v = 0.f;
    for (int i = 0; i < per; ++i) v += x[i];
    v = warp_sum(v);
    for (int i = 0; i < per; ++i) out[i] = v;
  }
}

struct GatedParams {
  const void* q;
  const void* k;
  const void* v;
  const int* pos;
  int batch, queries, keys, heads, dim, block;
  float scale;
};

template <typename T>
__global__ void __launch_bounds__(kThreads)
gated_fwd_simt(GatedParams p, T* __restrict__ out, float* __restrict__ rc, float* __restrict__ pr,
               float* __restrict__ zr_out, float* __restrict__ lse_out) {
  extern __shared__ float smem[];
  const int D = p.dim, ld = D + 1, b = p.block;
  const int TK = tile_keys(b);
  const int q0 = blockIdx.x * kRows;
  const int bh = blockIdx.y, batch = bh / p.heads, head = bh % p.heads;
  float* Qs = smem;                     // [16][ld]
  float* KV = Qs + kRows * ld;          // [T][ld]
  float* S = KV + TK * ld;               // [16][T]
  float* PR = S + kRows * TK;            // [16][T] remote probabilities
  float* PL = PR + kRows * TK;           // [16][T] local probabilities
  float* AR = PL + kRows * TK;           // [16] remote rescale
  float* AL = AR + kRows;               // [16] local rescale
  float* FR = AL + kRows;               // [16] final remote factor
  float* FL = FR + kRows;               // [16] final local factor
  int* P = reinterpret_cast<int*>(FL + kRows);   // [16] positions
  const int rows_valid = min(kRows, p.queries - q0);
  const T* qb = static_cast<const T*>(p.q) + static_cast<int64_t>(batch) * p.queries * p.heads * D;
  const T* kb = static_cast<const T*>(p.k) + static_cast<int64_t>(batch) * p.keys * p.heads * D;
  const T* vb = static_cast<const T*>(p.v) + static_cast<int64_t>(batch) * p.keys * p.heads * D;
  load_tile(Qs, ld, qb, q0, rows_valid, kRows, p.heads, head, D);
  if (threadIdx.x < kRows)
    P[threadIdx.x] = threadIdx.x < rows_valid ? p.pos[static_cast<int64_t>(batch) * p.queries + q0 + threadIdx.x] : -1;
  __syncthreads();
  int max_pos = -1;
  for (int r = 0; r < kRows; ++r) max_pos = max(max_pos, P[r]);
  const int limit = min(p.keys, max_pos + 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // Row state (two rows per warp), replicated across the warp's lanes.
  float mr[2] = {kNegInf, kNegInf}, dr[2] = {0.f, 0.f}, ml[2] = {kNegInf, kNegInf}, dl[2] = {0.f, 0.f};
  float zr[2] = {kNegInf, kNegInf};
  // Accumulators: thread owns row t/16 and columns (t%16) + 16*i.
  const int my_row = threadIdx.x / 16, my_col = threadIdx.x % 16;
  float nr[kMaxAcc], nl[kMaxAcc];
#pragma unroll
  for (int i = 0; i < kMaxAcc; ++i) nr[i] = nl[i] = 0.f;
  for (int k0 = 0; k0 < limit; k0 += TK) {
    load_tile(KV, ld, kb, k0, min(TK, p.keys - k0), TK, p.heads, head, D);
    __syncthreads();
    tile_dots(S, Qs, KV, ld, TK, D);
    __syncthreads();
    for (int w = 0; w < 2; ++w) {
      const int row = warp * 2 + w;
      const int pos = P[row];
      float a[4], sb[4];
      row_block_scores(S, TK, row, k0, p.keys, b, p.scale, a, sb);
      const int per = TK / 32 > 0 ? TK / 32 : 1;
      bool rem[4], loc[4];
      float tz_max = kNegInf, lrmax = kNegInf, llmax = kNegInf;
      for (int i = 0; i < per; ++i) {
        const int key = k0 + lane + 32 * i;
        const int kbk = key / b, pb = pos >= 0 ? pos / b : 0;
        rem[i] = pos >= 0 && key < p.keys && kbk < pb - 1;
        loc[i] = pos >= 0 && key < p.keys && kbk >= pb - 1 && key <= pos;
        if (rem[i] && (key % b) == 0) tz_max = fmaxf(tz_max, sb[i]);
        if (rem[i]) lrmax = fmaxf(lrmax, a[i] + sb[i]);
        if (loc[i]) llmax = fmaxf(llmax, a[i]);
      }
      tz_max = warp_max(tz_max);
      lrmax = warp_max(lrmax);
      llmax = warp_max(llmax);
      float tz = 0.f;
      for (int i = 0; i < per; ++i) {
        const int key = k0 + lane + 32 * i;
        if (rem[i] && (key % b) == 0) tz += expf(sb[i] - tz_max);
      }
      tz = warp_sum(tz);
      if (tz_max != kNegInf) zr[w] = log_add(zr[w], tz_max + logf(tz));
      const float mr_new = fmaxf(mr[w], lrmax), ml_new = fmaxf(ml[w], llmax);
      const float mr_ref = finite_or_zero(mr_new), ml_ref = finite_or_zero(ml_new);
      float sum_r = 0.f, sum_l = 0.f;
      for (int i = 0; i < per; ++i) {
        const int c = lane + 32 * i;
        const float er = rem[i] ? expf(a[i] + sb[i] - mr_ref) : 0.f;
        const float el = loc[i] ? expf(a[i] - ml_ref) : 0.f;
        if (c < TK) {
          PR[row * TK + c] = er;
          PL[row * TK + c] = el;
        }
        sum_r += er;
        sum_l += el;
      }
      sum_r = warp_sum(sum_r);
      sum_l = warp_sum(sum_l);
      const float alpha_r = mr[w] == kNegInf ? 0.f : expf(mr[w] - mr_ref);
      const float alpha_l = ml[w] == kNegInf ? 0.f : expf(ml[w] - ml_ref);
      dr[w] = dr[w] * alpha_r + sum_r;
      dl[w] = dl[w] * alpha_l + sum_l;
      mr[w] = mr_new;
      ml[w] = ml_new;
      if (lane == 0) {
        AR[row] = alpha_r;
        AL[row] = alpha_l;
      }
    }
    __syncthreads();
    load_tile(KV, ld, vb, k0, min(TK, p.keys - k0), TK, p.heads, head, D);
    __syncthreads();
    {
      const float ar = AR[my_row], al = AL[my_row];
      const float* prow = PR + my_row * TK;
      const float* lrow = PL + my_row * TK;
#pragma unroll
      for (int i = 0; i < kMaxAcc; ++i) {
        const int d = i * 16 + my_col;
        if (d < D) {
          float accr = nr[i] * ar, accl = nl[i] * al;
          for (int c = 0; c < TK; ++c) {
            const float vv = KV[c * ld + d];
            accr += prow[c] * vv;
            accl += lrow[c] * vv;
          }
          nr[i] = accr;
          nl[i] = accl;
        }
      }
    }
    __syncthreads();
  }
  for (int w = 0; w < 2; ++w) {
    const int row = warp * 2 + w;
    const float lr = (dr[w] > 0.f) ? mr[w] + logf(dr[w]) - finite_or_zero(zr[w]) : kNegInf;
    const float ll = (dl[w] > 0.f) ? ml[w] + logf(dl[w]) : kNegInf;
    const float total = log_add(lr, ll);
    const float ref = finite_or_zero(total);
    const float prob_r = lr == kNegInf ? 0.f : expf(lr - ref);
    const float prob_l = ll == kNegInf ? 0.f : expf(ll - ref);
    if (lane == 0) {
      FR[row] = dr[w] > 0.f ? prob_r / dr[w] : 0.f;
      FL[row] = dl[w] > 0.f ? prob_l / dl[w] : 0.f;
      if (row < rows_valid) {
        const int64_t s = (static_cast<int64_t>(batch) * p.queries + q0 + row) * p.heads + head;
        pr[s] = prob_r;
        zr_out[s] = zr[w];
        lse_out[s] = total;
      }
    }
  }
  __syncthreads();
  if (my_row < rows_valid) {
    const float fr = FR[my_row], fl = FL[my_row];
    const int64_t base = ((static_cast<int64_t>(batch) * p.queries + q0 + my_row) * p.heads + head) * D;
#pragma unroll
    for (int i = 0; i < kMaxAcc; ++i) {
      const int d = i * 16 + my_col;
      if (d < D) {
        const float remote = nr[i] * fr;
        rc[base + d] = remote;
        out[base + d] = cast_f<T>(remote + nl[i] * fl);
      }
    }
  }
}

// Shared per-tile backward math for one warp-row: recompute probabilities and
// the gate-aware logit gradient da (already multiplied by the softmax scale).
EB_DEVICE void tile_grad_row(const float* S, const float* DP, int TK, int row, int k0, int nk, int b,
                             float scale, int pos, float zr, float lse, float delta, float rho,
                             float* prob_out, float* da_out) {
  const int lane = threadIdx.x & 31;
  const int per = TK / 32 > 0 ? TK / 32 : 1;
  float a[4], sb[4], direct[4], rb[4], prob[4];
  bool rem[4];
  row_block_scores(S, TK, row, k0, nk, b, scale, a, sb);
  for (int i = 0; i < per; ++i) {
    const int c = lane + 32 * i;
    const int key = k0 + c;
    const int pb = pos >= 0 ? pos / b : 0;
    rem[i] = pos >= 0 && key < nk && key / b < pb - 1;
    const bool loc = pos >= 0 && key < nk && key / b >= pb - 1 && key <= pos;
    prob[i] = rem[i] ? expf(a[i] + sb[i] - zr - lse) : (loc ? expf(a[i] - lse) : 0.f);
    direct[i] = prob[i] * ((c < TK ? DP[row * TK + c] : 0.f) - delta);
  }
  block_sums(TK, b, direct, rb);
  for (int i = 0; i < per; ++i) {
    const int c = lane + 32 * i;
    float g = 0.f;
    if (rem[i]) g = expf(a[i] - sb[i]) * rb[i] - expf(a[i] - zr) * rho;
    if (c < TK) {
      prob_out[row * TK + c] = prob[i];
      da_out[row * TK + c] = (direct[i] + g) * scale;
    }
  }
}

// delta = dO . O and rho = dO . RC - delta * PR for one row (warp-cooperative).
template <typename T>
EB_DEVICE void row_delta_rho(const T* go, const T* o, const float* rcp, float prob_remote, int dim,
                             float& delta, float& rho) {
  const int lane = threadIdx.x & 31;
  float dd = 0.f, rr = 0.f;
  for (int d = lane; d < dim; d += 32) {
    const float g = load_f(go + d);
    dd += g * load_f(o + d);
    rr += g * rcp[d];
  }
  delta = warp_sum(dd);
  rho = warp_sum(rr) - delta * prob_remote;
}

struct GatedBwdParams {
  GatedParams f;
  const void* dout;
  const void* out;
  const float* rc;
  const float* pr;
  const float* zr;
  const float* lse;
};

template <typename T>
__global__ void __launch_bounds__(kThreads)
gated_dq_simt(GatedBwdParams bp, T* __restrict__ dq) {
  extern __shared__ float smem[];
  const GatedParams& p = bp.f;
  const int D = p.dim, ld = D + 1, b = p.block;
  const int TK = tile_keys(b);
  const int q0 = blockIdx.x * kRows;
  const int bh = blockIdx.y, batch = bh / p.heads, head = bh % p.heads;
  float* Qs = smem;
  float* Gs = Qs + kRows * ld;
  float* KV = Gs + kRows * ld;
  float* S = KV + TK * ld;
  float* DP = S + kRows * TK;
  float* PB = DP + kRows * TK;
  float* DA = PB + kRows * TK;
  float* RowF = DA + kRows * TK;            // [16][4]: zr, lse, delta, rho
  int* P = reinterpret_cast<int*>(RowF + kRows * 4);
  const int rows_valid = min(kRows, p.queries - q0);
  const int64_t qoff = static_cast<int64_t>(batch) * p.queries * p.heads * D;
  const int64_t koff = static_cast<int64_t>(batch) * p.keys * p.heads * D;
  load_tile(Qs, ld, static_cast<const T*>(p.q) + qoff, q0, rows_valid, kRows, p.heads, head, D);
  load_tile(Gs, ld, static_cast<const T*>(bp.dout) + qoff, q0, rows_valid, kRows, p.heads, head, D);
  if (threadIdx.x < kRows)
    P[threadIdx.x] = threadIdx.x < rows_valid ? p.pos[static_cast<int64_t>(batch) * p.queries + q0 + threadIdx.x] : -1;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int w = 0; w < 2; ++w) {
    const int row = warp * 2 + w;
    float delta = 0.f, rho = 0.f, z = 0.f, l = 0.f;
    if (row < rows_valid) {
      const int64_t s = (static_cast<int64_t>(batch) * p.queries + q0 + row) * p.heads + head;
      const int64_t e = s * D;
      row_delta_rho(static_cast<const T*>(bp.dout) + e, static_cast<const T*>(bp.out) + e, bp.rc + e,
                    bp.pr[s], D, delta, rho);
      z = finite_or_zero(bp.zr[s]);
      l = finite_or_zero(bp.lse[s]);
    }
    if (lane == 0) {
      RowF[row * 4 + 0] = z;
      RowF[row * 4 + 1] = l;
      RowF[row * 4 + 2] = delta;
      RowF[row * 4 + 3] = rho;
    }
  }
  __syncthreads();
  int max_pos = -1;
  for (int r = 0; r < kRows; ++r) max_pos = max(max_pos, P[r]);
  const int limit = min(p.keys, max_pos + 1);
  const int my_row = threadIdx.x / 16, my_col = threadIdx.x % 16;
  float acc[kMaxAcc];
#pragma unroll
  for (int i = 0; i < kMaxAcc; ++i) acc[i] = 0.f;
  const T* kb = static_cast<const T*>(p.k) + koff;
  const T* vb = static_cast<const T*>(p.v) + koff;
  for (int k0 = 0; k0 < limit; k0 += TK) {
    const int kv = min(TK, p.keys - k0);
    load_tile(KV, ld, kb, k0, kv, TK, p.heads, head, D);
    __syncthreads();
    tile_dots(S, Qs, KV, ld, TK, D);
    __syncthreads();
    load_tile(KV, ld, vb, k0, kv, TK, p.heads, head, D);
    __syncthreads();
    tile_dots(DP, Gs, KV, ld, TK, D);
    __syncthreads();
    for (int w = 0; w < 2; ++w) {
      const int row = warp * 2 + w;
      tile_grad_row(S, DP, TK, row, k0, p.keys, b, p.scale, P[row], RowF[row * 4], RowF[row * 4 + 1],
                    RowF[row * 4 + 2], RowF[row * 4 + 3], PB, DA);
    }
    load_tile(KV, ld, kb, k0, kv, TK, p.heads, head, D);
    __syncthreads();
    const float* darow = DA + my_row * TK;
#pragma unroll
    for (int i = 0; i < kMaxAcc; ++i) {
      const int d = i * 16 + my_col;
      if (d < D) {
        float a = acc[i];
        for (int c = 0; c < TK; ++c) a += darow[c] * KV[c * ld + d];
        acc[i] = a;
      }
    }
    __syncthreads();
  }
  if (my_row < rows_valid) {
    const int64_t base = ((static_cast<int64_t>(batch) * p.queries + q0 + my_row) * p.heads + head) * D;
#pragma unroll
    for (int i = 0; i < kMaxAcc; ++i)
      if (i * 16 + my_col < D) dq[base + i * 16 + my_col] = cast_f<T>(acc[i]);
  }
}

template <typename T>
__global__ void __launch_bounds__(kThreads)
gated_dkv_simt(GatedBwdParams bp, T* __restrict__ dk, T* __restrict__ dv, int dslice) {
  extern __shared__ float smem[];
  const GatedParams& p = bp.f;
  const int D = p.dim, ld = D + 1, b = p.block;
  const int TK = tile_keys(b);
  const int k0 = blockIdx.x * TK;
  const int bh = blockIdx.y, batch = bh / p.heads, head = bh % p.heads;
  const int d0 = blockIdx.z * dslice, dn = min(dslice, D - d0);
  float* Qs = smem;
  float* Gs = Qs + kRows * ld;
  float* KV = Gs + kRows * ld;
  float* S = KV + TK * ld;
  float* DP = S + kRows * TK;
  float* PB = DP + kRows * TK;
  float* DA = PB + kRows * TK;
  float* RowF = DA + kRows * TK;
  int* P = reinterpret_cast<int*>(RowF + kRows * 4);
  const int kv = min(TK, p.keys - k0);
  const int64_t qoff = static_cast<int64_t>(batch) * p.queries * p.heads * D;
  const int64_t koff = static_cast<int64_t>(batch) * p.keys * p.heads * D;
  const T* kb = static_cast<const T*>(p.k) + koff;
  const T* vb = static_cast<const T*>(p.v) + koff;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // Thread owns outputs e = threadIdx.x + kThreads * i of the [T][dn] slice.
  float ak[kMaxAcc * 2], av[kMaxAcc * 2];
#pragma unroll
  for (int i = 0; i < kMaxAcc * 2; ++i) ak[i] = av[i] = 0.f;
  const int outputs = TK * dn;
  for (int q0 = 0; q0 < p.queries; q0 += kRows) {
    const int rows_valid = min(kRows, p.queries - q0);
    if (threadIdx.x < kRows)
      P[threadIdx.x] = threadIdx.x < rows_valid ? p.pos[static_cast<int64_t>(batch) * p.queries + q0 + threadIdx.x] : -1;
    __syncthreads();
    int max_pos = -1;
    for (int r = 0; r < kRows; ++r) max_pos = max(max_pos, P[r]);
    if (max_pos < k0) {       // no row of this tile sees these keys
      __syncthreads();
      continue;
    }
    load_tile(Qs, ld, static_cast<const T*>(p.q) + qoff, q0, rows_valid, kRows, p.heads, head, D);
    load_tile(Gs, ld, static_cast<const T*>(bp.dout) + qoff, q0, rows_valid, kRows, p.heads, head, D);
    for (int w = 0; w < 2; ++w) {
      const int row = warp * 2 + w;
      float delta = 0.f, rho = 0.f, z = 0.f, l = 0.f;
      if (row < rows_valid) {
        const int64_t s = (static_cast<int64_t>(batch) * p.queries + q0 + row) * p.heads + head;
        const int64_t e = s * D;
        row_delta_rho(static_cast<const T*>(bp.dout) + e, static_cast<const T*>(bp.out) + e, bp.rc + e,
                      bp.pr[s], D, delta, rho);
        z = finite_or_zero(bp.zr[s]);
        l = finite_or_zero(bp.lse[s]);
      }
      if (lane == 0) {
        RowF[row * 4 + 0] = z;
        RowF[row * 4 + 1] = l;
        RowF[row * 4 + 2] = delta;
        RowF[row * 4 + 3] = rho;
      }
    }
    load_tile(KV, ld, kb, k0, kv, TK, p.heads, head, D);
    __syncthreads();
    tile_dots(S, Qs, KV, ld, TK, D);
    __syncthreads();
    load_tile(KV, ld, vb, k0, kv, TK, p.heads, head, D);
    __syncthreads();
    tile_dots(DP, Gs, KV, ld, TK, D);
    __syncthreads();
    for (int w = 0; w < 2; ++w) {
      const int row = warp * 2 + w;
      tile_grad_row(S, DP, TK, row, k0, p.keys, b, p.scale, P[row], RowF[row * 4], RowF[row * 4 + 1],
                    RowF[row * 4 + 2], RowF[row * 4 + 3], PB, DA);
    }
    __syncthreads();
#pragma unroll
    for (int i = 0; i < 2 * kMaxAcc; ++i) {
      const int e = i * kThreads + threadIdx.x;
      if (e < outputs) {
        const int c = e / dn, d = d0 + e % dn;
        float gk = ak[i], gv = av[i];
        for (int r = 0; r < kRows; ++r) {
          gk += DA[r * TK + c] * Qs[r * ld + d];
          gv += PB[r * TK + c] * Gs[r * ld + d];
        }
        ak[i] = gk;
        av[i] = gv;
      }
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 2 * kMaxAcc; ++i) {
    const int e = i * kThreads + threadIdx.x;
    const int c = e / dn, d = d0 + e % dn;
    if (e < outputs && c < kv) {
      const int64_t o = ((static_cast<int64_t>(batch) * p.keys + k0 + c) * p.heads + head) * D + d;
      dk[o] = cast_f<T>(ak[i]);
      dv[o] = cast_f<T>(av[i]);
    }
  }
}

size_t smem_fwd(int D, int TK) {
  const int ld = D + 1;
  return sizeof(float) * (kRows * ld + TK * ld + 3 * kRows * TK + 4 * kRows) + sizeof(int) * kRows;
}

size_t smem_bwd(int D, int TK) {
  const int ld = D + 1;
  return sizeof(float) * (2 * kRows * ld + TK * ld + 4 * kRows * TK + 4 * kRows) + sizeof(int) * kRows;
}

int dkv_slice(int D, int TK) {
  // Accumulators: T * slice / kThreads <= 2 * kMaxAcc per thread.
  int slice = D;
  while (TK * slice > kThreads * kMaxAcc * 2) slice = (slice + 1) / 2;
  return slice;
}

template <typename T>
void launch_simt(const GatedParams& p, at::Tensor& out, at::Tensor& rc, at::Tensor& pr, at::Tensor& zr,
                 at::Tensor& lse, cudaStream_t stream) {
  const int tk = tile_keys(p.block);
  const size_t smem = smem_fwd(p.dim, tk);
  auto kernel = gated_fwd_simt<T>;
  EB_CUDA_CHECK(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
  dim3 grid(cdiv(p.queries, kRows), p.batch * p.heads);
  kernel<<<grid, kThreads, smem, stream>>>(p, reinterpret_cast<T*>(out.data_ptr()), rc.data_ptr<float>(),
                                           pr.data_ptr<float>(), zr.data_ptr<float>(), lse.data_ptr<float>());
}

template <typename T>
void launch_simt_bwd(const GatedBwdParams& bp, at::Tensor& dq, at::Tensor& dk, at::Tensor& dv,
                     cudaStream_t stream) {
  const GatedParams& p = bp.f;
  const int tk = tile_keys(p.block);
  const size_t smem = smem_bwd(p.dim, tk);
  auto kq = gated_dq_simt<T>;
  EB_CUDA_CHECK(cudaFuncSetAttribute(kq, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
  kq<<<dim3(cdiv(p.queries, kRows), p.batch * p.heads), kThreads, smem, stream>>>(
      bp, reinterpret_cast<T*>(dq.data_ptr()));
  const int slice = dkv_slice(p.dim, tk);
  auto kkv = gated_dkv_simt<T>;
  EB_CUDA_CHECK(cudaFuncSetAttribute(kkv, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
  kkv<<<dim3(cdiv(p.keys, tk), p.batch * p.heads, cdiv(p.dim, slice)), kThreads, smem, stream>>>(
      bp, reinterpret_cast<T*>(dk.data_ptr()), reinterpret_cast<T*>(dv.data_ptr()), slice);
}

}  // namespace

void gated_fwd_simt_launch(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, const at::Tensor& pos,
                           int64_t block, at::Tensor& out, at::Tensor& rc, at::Tensor& pr, at::Tensor& zr,
                           at::Tensor& lse) {
  GatedParams p{q.data_ptr(), k.data_ptr(), v.data_ptr(), pos.data_ptr<int>(), static_cast<int>(q.size(0)),
                static_cast<int>(q.size(1)), static_cast<int>(k.size(1)), static_cast<int>(q.size(2)),
                static_cast<int>(q.size(3)), static_cast<int>(block), 1.f / std::sqrt(static_cast<float>(q.size(3)))};
  auto stream = at::cuda::getCurrentCUDAStream();
  if (q.scalar_type() == at::kFloat) launch_simt<float>(p, out, rc, pr, zr, lse, stream);
  else launch_simt<__nv_bfloat16>(p, out, rc, pr, zr, lse, stream);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  count_launch(1);
}

void gated_bwd_simt_launch(const at::Tensor& grad, const at::Tensor& q, const at::Tensor& k, const at::Tensor& v,
                           const at::Tensor& pos, const at::Tensor& out, const at::Tensor& rc,
                           const at::Tensor& pr, const at::Tensor& zr, const at::Tensor& lse, int64_t block,
                           at::Tensor& dq, at::Tensor& dk, at::Tensor& dv) {
  GatedParams p{q.data_ptr(), k.data_ptr(), v.data_ptr(), pos.data_ptr<int>(), static_cast<int>(q.size(0)),
                static_cast<int>(q.size(1)), static_cast<int>(k.size(1)), static_cast<int>(q.size(2)),
                static_cast<int>(q.size(3)), static_cast<int>(block), 1.f / std::sqrt(static_cast<float>(q.size(3)))};
  GatedBwdParams bp{p, grad.data_ptr(), out.data_ptr(), rc.data_ptr<float>(), pr.data_ptr<float>(),
                    zr.data_ptr<float>(), lse.data_ptr<float>()};
  auto stream = at::cuda::getCurrentCUDAStream();
  if (q.scalar_type() == at::kFloat) launch_simt_bwd<float>(bp, dq, dk, dv, stream);
  else launch_simt_bwd<__nv_bfloat16>(bp, dq, dk, dv, stream);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  count_launch(2);
}

}  // namespace eb
