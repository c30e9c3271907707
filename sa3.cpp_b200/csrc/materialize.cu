// materialize.cu -- linears whose adapter is applied through a materialized effective weight:
// the families the trainer cannot apply functionally (dora-cols, bora, and the -xs forms of every
// family, src/train_dit.h:90-164), and lora / dora-rows too when asked.
//
// Forward (src/train_lora.h:275-329), per call:
//   V     = W + s * (B A)             or, for -xs, W + s * (U M) V^T      f32 [out][in]
//   rows  rs[o] = m_r[o] / sqrt(sum_i V^2 + in * 1e-12)    (dora-rows: m, bora: m_r; else 1)
//   cols  cs[i] = m_c[i] / sqrt(sum_o (rs V)^2 + out * 1e-12)  (dora-cols: m, bora: m_c; else 1)
//   W_eff = rs[o] * V * cs[i], kept as the f16 operand of the GEMMs
//   y     = x W_eff^T + bias                                 (tcgen05 GEMM)
// Backward:
//   dx    = dy W_eff                                         (tcgen05 GEMM, W_eff read MN-major)
//   G     = dy^T x                                           (tcgen05 GEMM, K = tokens)
//   then through the column and row normalisations (the derivative of v / n(v) along a row or
//   column is (g - v <g, v> / n^2) / n), dD = s dV, and the low-rank factors:
//   dB = dD A^T, dA = B^T dD, or dM = U^T dD V for -xs (U, V frozen), dm / dm_r / dm_c.
// The W-sized passes are HBM-bound f32 streams (V and G are each written once and read at most
// twice); the three GEMMs carry the FLOPs.
#include "../../include/sa3k.h"
#include "linear.h"
#include "materialize.h"
#include "lora_kernels.h"
#include "sa3k_common.cuh"
#include "sa3k_internal.h"
#include "weight_value.cuh"

#include <cstring>
#include <string>

namespace sa3k {
namespace {

constexpr float kMatEps = 1e-12f;
constexpr int kMatMaxRank = 16;
constexpr int kSlotMat = 57;

__device__ __forceinline__ double warp_sum(double v) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
  return v;
}
__device__ __forceinline__ float warp_sumf(float v) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
  return v;
}

// -xs: P = U M [out][r] (the row factor of the update) and Q = V^T [r][in].
__global__ void mat_xs_prep_kernel(const float* __restrict__ U, const float* __restrict__ M,
                                   const float* __restrict__ Vb, int64_t out, int64_t in, int r,
                                   float* __restrict__ P, float* __restrict__ Q) {
  const int64_t n1 = out * r, n = n1 + (int64_t)r * in;
  for (int64_t k = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; k < n; k += (int64_t)gridDim.x * blockDim.x) {
    if (k < n1) {
      const int64_t o = k / r;
      const int b = (int)(k % r);
      float acc = 0.f;
      for (int a = 0; a < r; ++a) acc = fmaf(U[o * r + a], M[a * r + b], acc);
      P[k] = acc;
    } else {
      const int64_t q = k - n1;
      Q[q] = Vb[(q % in) * r + q / in];
    }
  }
}

// V = W + s P Q; rn2[o] = sum_i V^2 + in eps (f64 sum) and rs[o] = mr[o] / sqrt(rn2[o]) (1
// without a row magnitude).  A block of 128 threads takes two rows, its threads spread over the
// columns; each Q chunk read serves both rows, and the row sums are reduced in shared memory.
constexpr int kBdThreads = 128, kBdRows = 2, kBdWarps = kBdThreads / 32;
__global__ void __launch_bounds__(kBdThreads) mat_build_kernel(const Weight w, const float* __restrict__ P,
                                                               const float* __restrict__ Q, int r, float s,
                                                               const float* __restrict__ mr, float* __restrict__ V,
                                                               double* __restrict__ rn2, float* __restrict__ rs) {
  __shared__ float ps[kBdRows][kMatMaxRank];
  __shared__ double red[kBdWarps][kBdRows];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t o0 = (int64_t)blockIdx.x * kBdRows, in = w.in;
  const int nr = (int)min((int64_t)kBdRows, w.out - o0);
  if (tid < kBdRows * kMatMaxRank) {
    const int u = tid / kMatMaxRank, j = tid % kMatMaxRank;
    ps[u][j] = (u < nr && j < r) ? s * P[(o0 + u) * r + j] : 0.f;
  }
  __syncthreads();
  double acc[kBdRows] = {0.0, 0.0};
  for (int64_t i = 4 * tid; i < in; i += 4 * kBdThreads) {
    float v[kBdRows][4];
#pragma unroll
    for (int u = 0; u < kBdRows; ++u) {
      if (u < nr) wval4(w, o0 + u, i, v[u]);
      else v[u][0] = v[u][1] = v[u][2] = v[u][3] = 0.f;
    }
    for (int j = 0; j < r; ++j) {
      const float4 q = __ldg(reinterpret_cast<const float4*>(Q + (int64_t)j * in + i));
#pragma unroll
      for (int u = 0; u < kBdRows; ++u) {
        const float pj = ps[u][j];
        v[u][0] = fmaf(pj, q.x, v[u][0]);
        v[u][1] = fmaf(pj, q.y, v[u][1]);
        v[u][2] = fmaf(pj, q.z, v[u][2]);
        v[u][3] = fmaf(pj, q.w, v[u][3]);
      }
    }
#pragma unroll
    for (int u = 0; u < kBdRows; ++u) {
      if (u >= nr) break;
      *reinterpret_cast<float4*>(V + (o0 + u) * in + i) = make_float4(v[u][0], v[u][1], v[u][2], v[u][3]);
#pragma unroll
      for (int c = 0; c < 4; ++c) acc[u] += (double)v[u][c] * (double)v[u][c];
    }
  }
#pragma unroll
  for (int u = 0; u < kBdRows; ++u) {
    const double t = warp_sum(acc[u]);
    if (lane == 0) red[warp][u] = t;
  }
  __syncthreads();
  if (tid < nr) {
    double n2 = (double)in * (double)kMatEps;
#pragma unroll
    for (int k = 0; k < kBdWarps; ++k) n2 += red[k][tid];
    rn2[o0 + tid] = n2;
    rs[o0 + tid] = mr ? mr[o0 + tid] / (float)sqrt(n2) : 1.0f;
  }
}

// Column sums over a slice of rows, added into acc[i] (f64 atomics), four columns per thread and
// four rows of loads in flight:
//   G null: sum_o (rs V)^2          (the column norms of the row-scaled V)
//   else:   sum_o G (rs V)          (<g, r> along a column in the backward)
constexpr int kColThreads = 128;
__global__ void __launch_bounds__(kColThreads) mat_colsum_kernel(const float* __restrict__ V, const float* __restrict__ G,
                                                                 const float* __restrict__ rs, int64_t out, int64_t in,
                                                                 int64_t rows_per, double* __restrict__ acc) {
  const int64_t i = 4 * ((int64_t)blockIdx.x * blockDim.x + threadIdx.x);
  if (i >= in) return;
  const int64_t o0 = (int64_t)blockIdx.y * rows_per, o1 = min(out, o0 + rows_per);
  double a[4] = {0.0, 0.0, 0.0, 0.0};
  auto add = [&](const float4& v, const float4& g, float r) {
    const float rv[4] = {r * v.x, r * v.y, r * v.z, r * v.w};
    const float gv[4] = {g.x, g.y, g.z, g.w};
#pragma unroll
    for (int c = 0; c < 4; ++c) a[c] += G ? (double)gv[c] * (double)rv[c] : (double)rv[c] * (double)rv[c];
  };
  const float4 zero = make_float4(0.f, 0.f, 0.f, 0.f);
  int64_t o = o0;
  for (; o + 4 <= o1; o += 4) {
    float4 v[4], g[4];
    float r[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      v[u] = *reinterpret_cast<const float4*>(V + (o + u) * in + i);
      g[u] = G ? *reinterpret_cast<const float4*>(G + (o + u) * in + i) : zero;
      r[u] = rs[o + u];
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) add(v[u], g[u], r[u]);
  }
  for (; o < o1; ++o)
    add(*reinterpret_cast<const float4*>(V + o * in + i), G ? *reinterpret_cast<const float4*>(G + o * in + i) : zero,
        rs[o]);
  if (o1 > o0) {
#pragma unroll
    for (int c = 0; c < 4; ++c) atomicAdd(acc + i + c, a[c]);
  }
}

// Column factors: cs[i] = mc[i] / cn[i] (1 without a column magnitude), cn^2 = csq + out eps.
// With tc (the backward): cfac = cs, tcn[i] = tc / cn^2 and dmc[i] = tc / cn.
__global__ void mat_colfac_kernel(const double* __restrict__ csq, const double* __restrict__ tc,
                                  const float* __restrict__ mc, int64_t out, int64_t in, float* __restrict__ cs,
                                  float* __restrict__ tcn, float* __restrict__ dmc, int acc) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= in) return;
  if (!mc) {
    cs[i] = 1.0f;
    return;
  }
  const double n2 = csq[i] + (double)out * (double)kMatEps, n = sqrt(n2);
  cs[i] = (float)((double)mc[i] / n);
  if (tc) {
    tcn[i] = (float)(tc[i] / n2);
    if (dmc) dmc[i] = (float)(tc[i] / n) + (acc ? dmc[i] : 0.f);
  }
}

// W_eff = rs[o] V cs[i] as f16 (the GEMM operand) and, when asked, f32.
__global__ void mat_weff_kernel(const float* __restrict__ V, const float* __restrict__ rs,
                                const float* __restrict__ cs, int64_t out, int64_t in,
                                __half* __restrict__ wb, float* __restrict__ wf) {
  const int64_t n4 = out * in / 4;
  for (int64_t k = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; k < n4; k += (int64_t)gridDim.x * blockDim.x) {
    const int64_t e = 4 * k, o = e / in, i = e % in;
    const float4 v = reinterpret_cast<const float4*>(V)[k];
    const float4 c = *reinterpret_cast<const float4*>(cs + i);
    const float r = rs[o];
    const float4 y = make_float4(r * v.x * c.x, r * v.y * c.y, r * v.z * c.z, r * v.w * c.w);
    if (wf) reinterpret_cast<float4*>(wf)[k] = y;
    uint2 p;
    p.x = pack_f16x2(y.x, y.y);
    p.y = pack_f16x2(y.z, y.w);
    reinterpret_cast<uint2*>(wb)[k] = p;
  }
}

// The row pass of the backward: dD = s dV as f16 (the operand of the dB / dA GEMMs):
//   dR = cols ? cs[i] (G - rs V tcn[i]) : G
//   rows: t = sum_i dR V, dmr[o] += t / rn, dV = rs (dR - V t / rn^2), else dV = dR
// A block of 128 threads takes two rows, its threads spread over the columns (many warps per SM
// even for 1536-row weights), and the row sums are reduced through shared memory.
constexpr int kRbThreads = 128, kRbRows = 2, kRbWarps = kRbThreads / 32;
__global__ void __launch_bounds__(kRbThreads) mat_rowbwd_kernel(const float* __restrict__ G,
                                                                const float* __restrict__ V,
                                                                const float* __restrict__ rs,
                                                                const double* __restrict__ rn2,
                                                                const float* __restrict__ cs,
                                                                const float* __restrict__ tcn, int64_t out,
                                                                int64_t in, float s, int rows, int cols,
                                                                float* __restrict__ dmr,
                                                                __half* __restrict__ dDb) {
  __shared__ double red_t[kRbWarps][kRbRows];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t o0 = (int64_t)blockIdx.x * kRbRows;
  const int nr = (int)min((int64_t)kRbRows, out - o0);
  float ro[kRbRows], t_over[kRbRows];
#pragma unroll
  for (int u = 0; u < kRbRows; ++u) {
    ro[u] = u < nr ? rs[o0 + u] : 0.f;
    t_over[u] = 0.f;
  }
  // dR of 4 columns of row u (cf / tc: the column factors of those columns)
  auto dr4 = [&](const float4& gv, const float4& vv, const float4& cf, const float4& tc, float r0, float (&d)[4]) {
    if (cols) {
      d[0] = cf.x * (gv.x - r0 * vv.x * tc.x);
      d[1] = cf.y * (gv.y - r0 * vv.y * tc.y);
      d[2] = cf.z * (gv.z - r0 * vv.z * tc.z);
      d[3] = cf.w * (gv.w - r0 * vv.w * tc.w);
    } else {
      d[0] = gv.x; d[1] = gv.y; d[2] = gv.z; d[3] = gv.w;
    }
  };
  const float4 one4 = make_float4(1.f, 1.f, 1.f, 1.f);
  if (rows) {
    double t[kRbRows] = {0.0, 0.0};
    for (int64_t i = 4 * tid; i < in; i += 4 * kRbThreads) {
      const float4 cf = cols ? *reinterpret_cast<const float4*>(cs + i) : one4;
      const float4 tc = cols ? *reinterpret_cast<const float4*>(tcn + i) : one4;
#pragma unroll
      for (int u = 0; u < kRbRows; ++u) {
        if (u >= nr) break;
        const float4 gv = *reinterpret_cast<const float4*>(G + (o0 + u) * in + i);
        const float4 vv = *reinterpret_cast<const float4*>(V + (o0 + u) * in + i);
        float d[4];
        dr4(gv, vv, cf, tc, ro[u], d);
        t[u] += (double)d[0] * vv.x + (double)d[1] * vv.y + (double)d[2] * vv.z + (double)d[3] * vv.w;
      }
    }
#pragma unroll
    for (int u = 0; u < kRbRows; ++u) {
      const double w = warp_sum(t[u]);
      if (lane == 0) red_t[warp][u] = w;
    }
    __syncthreads();
#pragma unroll
    for (int u = 0; u < kRbRows; ++u) {
      if (u >= nr) break;
      double tt = 0.0;
#pragma unroll
      for (int k = 0; k < kRbWarps; ++k) tt += red_t[k][u];
      t_over[u] = (float)(tt / rn2[o0 + u]);
      if (tid == 0) dmr[o0 + u] += (float)(tt / sqrt(rn2[o0 + u]));
    }
  }
  for (int64_t i = 4 * tid; i < in; i += 4 * kRbThreads) {
    const float4 cf = cols ? *reinterpret_cast<const float4*>(cs + i) : one4;
    const float4 tc = cols ? *reinterpret_cast<const float4*>(tcn + i) : one4;
#pragma unroll
    for (int u = 0; u < kRbRows; ++u) {
      if (u >= nr) break;
      const float4 gv = *reinterpret_cast<const float4*>(G + (o0 + u) * in + i);
      const float4 vv = *reinterpret_cast<const float4*>(V + (o0 + u) * in + i);
      float d[4];
      dr4(gv, vv, cf, tc, ro[u], d);
      const float vx[4] = {vv.x, vv.y, vv.z, vv.w};
#pragma unroll
      for (int c = 0; c < 4; ++c) d[c] = s * (rows ? ro[u] * (d[c] - vx[c] * t_over[u]) : d[c]);
      uint2 pk;
      pk.x = pack_f16x2(d[0], d[1]);
      pk.y = pack_f16x2(d[2], d[3]);
      *reinterpret_cast<uint2*>(dDb + (o0 + u) * in + i) = pk;
    }
  }
}

// dM[a][b] = sum_o U[o][a] PG[o][b] (PG = dD V), one block per (a, b).
__global__ void mat_dm_xs_kernel(const float* __restrict__ U, const float* __restrict__ PG, int64_t out, int r,
                                 float* __restrict__ dM, int acc_out) {
  const int a = blockIdx.x / r, b = blockIdx.x % r;
  float acc = 0.f;
  for (int64_t o = threadIdx.x; o < out; o += blockDim.x) acc = fmaf(U[o * r + a], PG[o * r + b], acc);
  __shared__ float red[32];
  acc = warp_sumf(acc);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
    v = warp_sumf(v);
    if (threadIdx.x == 0) dM[blockIdx.x] = v + (acc_out ? dM[blockIdx.x] : 0.f);
  }
}

// dst[o][s] = src[s][o] for f16 src [S][out] -> dst [out][ld] (ld even), 64 x 64 tiles: every
// thread moves f16 pairs, so a warp reads and writes 128 contiguous bytes (even widths).
__global__ void transpose_f16_kernel(const __half* __restrict__ src, int64_t S, int64_t out,
                                           __half* __restrict__ dst, int64_t ld) {
  __shared__ __half t[64][66];   // [s][o], padded
  const int64_t s0 = (int64_t)blockIdx.x * 64, o0 = (int64_t)blockIdx.y * 64;
  const int tx = threadIdx.x;
  const __half zero = __float2half_rn(0.f);
  for (int k = threadIdx.y; k < 64; k += blockDim.y) {
    const int64_t s = s0 + k, o = o0 + 2 * tx;
    __half2 v;
    v.x = zero;
    v.y = zero;
    if (s < S && o < out) {
      if ((out & 1) == 0) {
        v = *reinterpret_cast<const __half2*>(src + s * out + o);
      } else {   // odd widths: rows are not 4-byte aligned
        v.x = src[s * out + o];
        if (o + 1 < out) v.y = src[s * out + o + 1];
      }
    }
    t[k][2 * tx] = v.x;
    t[k][2 * tx + 1] = v.y;
  }
  __syncthreads();
  for (int k = threadIdx.y; k < 64; k += blockDim.y) {
    const int64_t o = o0 + k, s = s0 + 2 * tx;
    if (o >= out || s >= S) continue;
    if (s + 1 < S) {
      __half2 v;
      v.x = t[2 * tx][k];
      v.y = t[2 * tx + 1][k];
      *reinterpret_cast<__half2*>(dst + o * ld + s) = v;   // ld and s even
    } else {
      dst[o * ld + s] = t[2 * tx][k];
    }
  }
}

// nrm[i] = sqrt(sum_o W[o][i]^2), one thread per column, f64 sums.
__global__ void mat_col_norms_kernel(const Weight w, float* __restrict__ nrm) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= w.in) return;
  double a = 0.0;
  for (int64_t o = 0; o < w.out; ++o) {
    const double v = (double)wval(w, o, i);
    a += v * v;
  }
  nrm[i] = (float)sqrt(a);
}

// Per-step f16 operands of the weight-gradient GEMMs: Qb [r][in] = Q (A, or V^T for -xs) and,
// for the standard families, Btb [r][out] = B^T.
__global__ void mat_pack_kernel(const float* __restrict__ Q, const float* __restrict__ B, int64_t out, int64_t in,
                                int r, __half* __restrict__ Qb, __half* __restrict__ Btb) {
  const int64_t n1 = (int64_t)r * in, n = n1 + (B ? (int64_t)r * out : 0);
  for (int64_t k = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; k < n; k += (int64_t)gridDim.x * blockDim.x) {
    if (k < n1) {
      Qb[k] = __float2half_rn(Q[k]);
    } else {
      const int64_t q = k - n1, j = q / out, o = q % out;
      Btb[q] = __float2half_rn(B[o * r + j]);
    }
  }
}

struct MatPlan {
  bool xs = false, rows = false, cols = false;
  const float* mr = nullptr;   // row magnitude (dora-rows m, bora m_r)
  const float* mc = nullptr;   // column magnitude (dora-cols m, bora m_c)
};

bool parse_type(const sa3k_mat_adapter* ad, MatPlan& p, std::string& err) {
  if (!ad->adapter_type) {
    err = "adapter_type is NULL";
    return false;
  }
  std::string t = ad->adapter_type;
  p.xs = t.size() >= 3 && t.compare(t.size() - 3, 3, "-xs") == 0;
  if (p.xs) t = t.substr(0, t.size() - 3);
  if (t == "lora") {
  } else if (t == "dora-rows") {
    p.rows = true;
    p.mr = ad->m;
  } else if (t == "dora-cols") {
    p.cols = true;
    p.mc = ad->m;
  } else if (t == "bora") {
    p.rows = p.cols = true;
    p.mr = ad->m_r;
    p.mc = ad->m_c;
  } else {
    err = "unknown adapter_type " + std::string(ad->adapter_type);
    return false;
  }
  if ((p.rows && !p.mr) || (p.cols && !p.mc)) {
    err = "adapter magnitude missing for " + std::string(ad->adapter_type);
    return false;
  }
  if (ad->rank < 1 || ad->rank > kMatMaxRank) {
    err = "materialized adapters take rank 1..16";
    return false;
  }
  if (p.xs ? (!ad->U || !ad->V || !ad->M) : (!ad->A || !ad->B)) {
    err = p.xs ? "-xs adapters need U, V and M" : "adapters need A and B";
    return false;
  }
  if (!p.xs && (reinterpret_cast<uintptr_t>(ad->A) & 15)) {
    err = "A must be 16-byte aligned";
    return false;
  }
  return true;
}

// Slices of rows for the column kernels (blocks of `cols` columns): about four blocks per SM,
// at least 16 rows a slice.
int64_t col_rows_per(Ctx* c, int64_t out, int64_t in, int64_t cols) {
  const int64_t cb = (in + cols - 1) / cols;
  int64_t splits = (int64_t)(4 * c->sm_count) / cb;
  splits = splits < 1 ? 1 : splits;
  const int64_t rp = (out + splits - 1) / splits;
  return rp < 16 ? 16 : rp;
}
constexpr int64_t kColBlockCols = 4 * kColThreads;

int mat_check(const sa3k_weight* w, const sa3k_mat_adapter* ad, int64_t S, MatPlan& p, std::string& err) {
  if (!parse_type(ad, p, err)) return 1;
  if (w->w.in % 64 != 0) {
    err = "in must be a multiple of 64";
    return 1;
  }
  if (S <= 0) {
    err = "S must be positive";
    return 1;
  }
  return 0;
}

// The target form of one call's adapter, its buffers and the call's scratch (x, dy as f16, G,
// the transposed dy, dD) carved from one context scratch slot.
struct MatCall {
  MatTarget t;
  __half *xb = nullptr, *dyb = nullptr, *dyt = nullptr, *dDb = nullptr;
  float* G = nullptr;
  int64_t ldt = 0;
};

bool mat_prepare(Ctx* c, const Weight* w, const sa3k_mat_adapter* ad, const MatPlan& p, const sa3k_mat_grads* g,
                 int64_t S, bool bwd, MatCall& mc, std::string& err) {
  MatTarget& t = mc.t;
  t.xs = p.xs; t.rows = p.rows; t.cols = p.cols;
  t.rank = ad->rank; t.s = ad->scale; t.w = w; t.in = w->in; t.out = w->out;
  t.A = ad->A; t.B = ad->B; t.U = ad->U; t.Vb = ad->V; t.M = ad->M; t.mr = p.mr; t.mc = p.mc;
  if (g) {
    t.dA = g->dA; t.dB = g->dB; t.dM = g->dM;
    t.dmr = p.rows ? (p.cols ? g->dm_r : g->dm) : nullptr;
    t.dmc = p.cols ? (p.rows ? g->dm_c : g->dm) : nullptr;
  }
  const int64_t in = w->in, out = w->out, wn = in * out;
  mc.ldt = (S + 7) / 8 * 8;
  auto al = [](size_t b) { return (b + 255) / 256 * 256; };
  const size_t tb = al(mat_target_bytes(in, out, ad->rank)), xb = al(2 * (size_t)(S * in));
  const size_t extra = bwd ? al(2 * (size_t)(S * out)) + al(2 * (size_t)(out * mc.ldt)) + al(2 * (size_t)wn) +
                                 al(4 * (size_t)wn)
                           : 0;
  uint8_t* base = static_cast<uint8_t*>(scratch_get(c, kSlotMat, tb + xb + extra, err));
  if (!base) return false;
  mat_target_bind(t, base);
  mc.xb = reinterpret_cast<__half*>(base + tb);
  if (bwd) {
    uint8_t* q = base + tb + xb;
    mc.dyb = reinterpret_cast<__half*>(q); q += al(2 * (size_t)(S * out));
    mc.dyt = reinterpret_cast<__half*>(q); q += al(2 * (size_t)(out * mc.ldt));
    mc.dDb = reinterpret_cast<__half*>(q); q += al(2 * (size_t)wn);
    mc.G = reinterpret_cast<float*>(q);
  }
  return true;
}

int mat_run(Ctx* c, const Weight* w, const sa3k_mat_adapter* ad, const MatPlan& p, const float* bias, const float* x,
            const float* dy, int64_t S, float* y, float* dx, const sa3k_mat_grads* g, std::string& err) {
  const int64_t in = w->in, out = w->out;
  const int r = ad->rank;
  const cudaStream_t st = c->stream;
  const bool bwd = dy != nullptr;
  MatCall mc;
  if (!mat_prepare(c, w, ad, p, g, S, bwd, mc, err)) return 1;
  MatTarget& t = mc.t;
  if (mat_target_build(c, t, nullptr, err)) return 1;
  if (k_cvt_f16(c, x, S * in, mc.xb, err)) return 1;
  if (y) {
    GemmDesc d;   // y = x W_eff^T + bias
    d.M = (int)S; d.N = (int)out; d.K = (int)in;
    d.a = mc.xb; d.lda = in;
    d.bsrc = kB_F16_KMAJOR; d.b = t.wb; d.ldb = in;
    d.col_bias = bias;
    d.out = y; d.ldo = out;
    d.name = "mat.fwd";
    if (gemm(c, d, err)) return 1;
  }
  if (!bwd) return 0;
  // the gradients are written: clear them, then the target pass adds into them
  auto zero = [&](float* q, int64_t n) {
    return !q || cudaMemsetAsync(q, 0, sizeof(float) * (size_t)n, st) == cudaSuccess;
  };
  if (!zero(t.dA, (int64_t)r * in) || !zero(t.dB, out * r) || !zero(t.dM, (int64_t)r * r) || !zero(t.dmr, out) ||
      !zero(t.dmc, in))
    return check_launch("memset", err);
  if (k_cvt_f16(c, dy, S * out, mc.dyb, err)) return 1;
  if (dx) {
    GemmDesc d;   // dx = dy W_eff
    d.M = (int)S; d.N = (int)in; d.K = (int)out;
    d.a = mc.dyb; d.lda = out;
    d.bsrc = kB_F16_MNMAJOR; d.b = t.wb; d.ldb = in;
    d.out = dx; d.ldo = in;
    d.name = "mat.dx";
    if (gemm(c, d, err)) return 1;
  }
  return mat_target_backward(c, t, mc.dyb, S, mc.xb, mc.G, mc.dyt, mc.ldt, mc.dDb, err);
}

int mfail(char* err, int len, const std::string& msg) {
  if (err && len > 0) {
    std::strncpy(err, msg.c_str(), (size_t)len - 1);
    err[len - 1] = 0;
  }
  return 1;
}

}  // namespace

size_t mat_target_bytes(int64_t in, int64_t out, int rank) {
  auto al = [](size_t b) { return (b + 255) / 256 * 256; };
  const size_t wn = (size_t)(in * out);
  return al(4 * wn) + al(2 * wn) + 2 * al(4 * (size_t)out * rank) + al(4 * (size_t)rank * in) + al(4 * out) +
         2 * al(4 * in) + al(8 * out) + 2 * al(8 * in) + al(2 * (size_t)rank * in) + al(2 * (size_t)rank * out);
}

void mat_target_bind(MatTarget& t, void* mem) {
  auto al = [](size_t b) { return (b + 255) / 256 * 256; };
  uint8_t* p = static_cast<uint8_t*>(mem);
  auto take = [&](size_t bytes) { uint8_t* q = p; p += al(bytes); return q; };
  const size_t wn = (size_t)(t.in * t.out);
  t.V = reinterpret_cast<float*>(take(4 * wn));
  t.wb = reinterpret_cast<__half*>(take(2 * wn));
  t.P = reinterpret_cast<float*>(take(4 * (size_t)t.out * t.rank));
  t.PG = reinterpret_cast<float*>(take(4 * (size_t)t.out * t.rank));
  t.Q = reinterpret_cast<float*>(take(4 * (size_t)t.rank * t.in));
  t.rs = reinterpret_cast<float*>(take(4 * t.out));
  t.cs = reinterpret_cast<float*>(take(4 * t.in));
  t.tcn = reinterpret_cast<float*>(take(4 * t.in));
  t.rn2 = reinterpret_cast<double*>(take(8 * t.out));
  t.csq = reinterpret_cast<double*>(take(8 * t.in));
  t.tc = reinterpret_cast<double*>(take(8 * t.in));
  t.Qb = reinterpret_cast<__half*>(take(2 * (size_t)t.rank * t.in));
  t.Btb = reinterpret_cast<__half*>(take(2 * (size_t)t.rank * t.out));
}

int mat_target_build(Ctx* c, MatTarget& t, float* weff_f32, std::string& err) {
  const int64_t in = t.in, out = t.out;
  const int r = t.rank;
  const cudaStream_t st = c->stream;
  const float* P = t.B;
  const float* Q = t.A;
  if (t.xs) {
    if (!t.U || !t.Vb) {
      err = "the -xs adapter has no U / V bases";
      return 1;
    }
    ProfScope prof_(c, "mat.xs_prep");
    mat_xs_prep_kernel<<<(unsigned)(2 * c->sm_count), 256, 0, st>>>(t.U, t.M, t.Vb, out, in, r, t.P, t.Q);
    if (check_launch("mat xs prep", err)) return 1;
    P = t.P;
    Q = t.Q;
  }
  {
    ProfScope prof_(c, "mat.build");
    mat_build_kernel<<<(unsigned)((out + kBdRows - 1) / kBdRows), kBdThreads, 0, st>>>(*t.w, P, Q, r, t.s,
                                                                                      t.rows ? t.mr : nullptr, t.V,
                                                                                      t.rn2, t.rs);
    if (check_launch("mat build", err)) return 1;
  }
  if (t.cols) {
    ProfScope prof_(c, "mat.cols");
    if (cudaMemsetAsync(t.csq, 0, sizeof(double) * in, st) != cudaSuccess) return check_launch("memset", err);
    const int64_t rp = col_rows_per(c, out, in, kColBlockCols);
    mat_colsum_kernel<<<dim3((unsigned)((in + kColBlockCols - 1) / kColBlockCols), (unsigned)((out + rp - 1) / rp)),
                        kColThreads, 0, st>>>(t.V, nullptr, t.rs, out, in, rp, t.csq);
    if (check_launch("mat colsum", err)) return 1;
  }
  ProfScope prof_(c, "mat.weff");
  mat_colfac_kernel<<<(unsigned)((in + 255) / 256), 256, 0, st>>>(t.csq, nullptr, t.cols ? t.mc : nullptr, out, in,
                                                                 t.cs, nullptr, nullptr, 0);
  if (check_launch("mat colfac", err)) return 1;
  mat_weff_kernel<<<(unsigned)(4 * c->sm_count), 256, 0, st>>>(t.V, t.rs, t.cs, out, in, t.wb, weff_f32);
  if (check_launch("mat weff", err)) return 1;
  mat_pack_kernel<<<(unsigned)(c->sm_count), 256, 0, st>>>(Q, t.xs ? nullptr : t.B, out, in, r, t.Qb, t.Btb);
  return check_launch("mat pack", err);
}

int mat_target_backward(Ctx* c, MatTarget& t, const __half* dz, int64_t M, const __half* x,
                        float* G, __half* dzt, int64_t ldt, __half* dDb, std::string& err) {
  const int64_t in = t.in, out = t.out;
  const int r = t.rank;
  const cudaStream_t st = c->stream;
  if (ldt < M || ldt % 8) {
    err = "mat backward: transposed gradient pitch";
    return 1;
  }
  {
    ProfScope prof_(c, "mat.transpose");
    transpose_f16_kernel<<<dim3((unsigned)((M + 63) / 64), (unsigned)((out + 63) / 64)), dim3(32, 8), 0, st>>>(
        dz, M, out, dzt, ldt);
    if (check_launch("mat transpose", err)) return 1;
  }
  {
    GemmDesc d;   // G = dz^T x  [out][in], K = token rows
    d.M = (int)out; d.N = (int)in; d.K = (int)M;
    d.a = dzt; d.lda = ldt;
    d.bsrc = kB_F16_MNMAJOR; d.b = x; d.ldb = in;
    d.out = G; d.ldo = in;
    d.name = "mat.dW";
    if (gemm(c, d, err)) return 1;
  }
  if (t.cols) {
    ProfScope prof_(c, "mat.cols_bwd");
    if (cudaMemsetAsync(t.tc, 0, sizeof(double) * in, st) != cudaSuccess) return check_launch("memset", err);
    const int64_t rp = col_rows_per(c, out, in, kColBlockCols);
    mat_colsum_kernel<<<dim3((unsigned)((in + kColBlockCols - 1) / kColBlockCols), (unsigned)((out + rp - 1) / rp)),
                        kColThreads, 0, st>>>(t.V, G, t.rs, out, in, rp, t.tc);
    if (check_launch("mat colsum bwd", err)) return 1;
    mat_colfac_kernel<<<(unsigned)((in + 255) / 256), 256, 0, st>>>(t.csq, t.tc, t.mc, out, in, t.cs, t.tcn, t.dmc, 1);
    if (check_launch("mat colfac bwd", err)) return 1;
  }
  {
    ProfScope prof_(c, "mat.rows_bwd");
    mat_rowbwd_kernel<<<(unsigned)((out + kRbRows - 1) / kRbRows), kRbThreads, 0, st>>>(
        G, t.V, t.rs, t.rn2, t.cs, t.tcn, out, in, t.s, t.rows ? 1 : 0, t.cols ? 1 : 0, t.rows ? t.dmr : nullptr, dDb);
    if (check_launch("mat rows bwd", err)) return 1;
  }
  if (t.xs && cudaMemsetAsync(t.PG, 0, sizeof(float) * (size_t)out * r, st) != cudaSuccess)
    return check_launch("memset", err);
  {
    GemmDesc d;   // dB += dD A^T, or PG = dD V (-xs)  [out][r], K = in
    d.M = (int)out; d.N = r; d.K = (int)in;
    d.a = dDb; d.lda = in;
    d.bsrc = kB_F16_KMAJOR; d.b = t.Qb; d.ldb = in;
    d.out = t.xs ? t.PG : t.dB; d.ldo = r; d.accumulate = 1; d.bn = 16;
    d.atomic_split = 1;
    d.name = "mat.dB";
    if (gemm(c, d, err)) return 1;
  }
  if (t.xs) {
    ProfScope prof_(c, "mat.dM");
    mat_dm_xs_kernel<<<(unsigned)(r * r), 256, 0, st>>>(t.U, t.PG, out, r, t.dM, 1);
    return check_launch("mat dM", err);
  }
  GemmDesc d;   // dA^T += dD^T B  [in][r] (dD read MN-major), stored transposed as dA [r][in]
  d.M = (int)in; d.N = r; d.K = (int)out;
  d.a = dDb; d.lda = in; d.a_mn = 1;
  d.bsrc = kB_F16_KMAJOR; d.b = t.Btb; d.ldb = out;
  d.out = t.dA; d.ldo = in; d.out_trans = 1; d.accumulate = 1; d.bn = 16;
  d.atomic_split = 1;
  d.name = "mat.dA";
  return gemm(c, d, err);
}

int mat_col_norms(Ctx* c, const Weight* w, float* nrm, std::string& err) {
  ProfScope prof_(c, "col norms");
  mat_col_norms_kernel<<<(unsigned)((w->in + 255) / 256), 256, 0, c->stream>>>(*w, nrm);
  return check_launch("col norms", err);
}

}  // namespace sa3k

using namespace sa3k;

extern "C" {

int sa3k_mat_effective_weight(sa3k_ctx* ctx, const sa3k_weight* w, const sa3k_mat_adapter* ad, float* weff,
                              char* err, int err_len) {
  if (!ctx || !w || !ad || !weff) return mfail(err, err_len, "NULL argument");
  MatPlan p;
  std::string e;
  if (mat_check(w, ad, 1, p, e)) return mfail(err, err_len, e);
  Ctx* c = &ctx->c;
  cudaSetDevice(c->device);
  MatCall mc;
  if (!mat_prepare(c, &w->w, ad, p, nullptr, 1, false, mc, e) || mat_target_build(c, mc.t, weff, e))
    return mfail(err, err_len, e);
  return 0;
}

int sa3k_linear_mat_fwd(sa3k_ctx* ctx, const sa3k_weight* w, const sa3k_mat_adapter* ad, const float* bias,
                        const float* x, int64_t S, float* y, char* err, int err_len) {
  if (!ctx || !w || !ad || !x || !y) return mfail(err, err_len, "NULL argument");
  if (S <= 0) return mfail(err, err_len, "S must be positive");
  MatPlan p;
  std::string e;
  if (mat_check(w, ad, S, p, e)) return mfail(err, err_len, e);
  cudaSetDevice(ctx->c.device);
  if (mat_run(&ctx->c, &w->w, ad, p, bias, x, nullptr, S, y, nullptr, nullptr, e)) return mfail(err, err_len, e);
  return 0;
}

int sa3k_linear_mat_fwd_bwd(sa3k_ctx* ctx, const sa3k_weight* w, const sa3k_mat_adapter* ad, const float* bias,
                            const float* x, const float* dy, int64_t S, float* y, float* dx, const sa3k_mat_grads* g,
                            char* err, int err_len) {
  if (!ctx || !w || !ad || !x || !dy || !g) return mfail(err, err_len, "NULL argument");
  if (S <= 0) return mfail(err, err_len, "S must be positive");
  MatPlan p;
  std::string e;
  if (mat_check(w, ad, S, p, e)) return mfail(err, err_len, e);
  if (p.xs ? !g->dM : (!g->dA || !g->dB)) return mfail(err, err_len, p.xs ? "-xs adapters need dM" : "need dA and dB");
  if (p.rows && p.cols ? (!g->dm_r || !g->dm_c) : ((p.rows || p.cols) && !g->dm))
    return mfail(err, err_len, "magnitude gradients missing");
  cudaSetDevice(ctx->c.device);
  if (mat_run(&ctx->c, &w->w, ad, p, bias, x, dy, S, y, dx, g, e)) return mfail(err, err_len, e);
  return 0;
}

}  // extern "C"
