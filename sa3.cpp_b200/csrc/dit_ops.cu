// dit_ops.cu -- the memory-bound pieces of one DiT block, forward and backward.
//
// Each kernel restates a group of ggml ops of dit_block (src/dit.h:164-266) in the autodiff-safe
// form the training graph uses, plus the derivative ggml_build_backward_expand produces for it:
//   rms_norm + adaLN modulate   src/nn.h:40-42, src/dit.h:177-185    (RMS_NORM(_BACK), MUL, ADD)
//   qk rms_norm + partial RoPE  src/dit.h:195, src/nn.h:53-59       (ROPE NEOX and its backward)
//   gate + residual             src/dit.h:186-193, 223, 265          (h / (exp(g - 1) + 1))
//   SwiGLU                      src/dit.h:259-264                    (SILU(_BACK), MUL)
//   adaLN vectors               src/dit.h:174-176                    (ssg + gcond)
//   MSE loss                    src/train_ckpt.h:226-228
// All are vectorized row kernels (one warp per row or 128-bit grid-stride loops).
#include "attention.h"
#include "sa3k_common.cuh"

namespace sa3k {
namespace {

// RoPE angle of pair i (< rot/2) at position pos: pos * base^(-2i/rot); its (cos, sin) come from
// a table built once per (positions, rot, base) rather than from sincos in every warp.
// (cos, sin) of NeoX RoPE, twice: position-major tab[pos * half + i] (the head-preparation
// kernels, 8 lanes per row) and frequency-major tab[n + i * tps + pos] (the GEMM epilogue, one
// row per lane: consecutive lanes read consecutive positions)
__global__ void rope_table_kernel(int tps, int rot, float log2_base, float2* __restrict__ tab) {
  const int half = rot / 2, n = tps * half;
  const int e = blockIdx.x * blockDim.x + threadIdx.x;
  if (e >= n) return;
  const int pos = e / half, i = e % half;
  const float freq = exp2f(-2.0f * (float)i / (float)rot * log2_base);
  float sn, cs;
  sincosf((float)pos * freq, &sn, &cs);
  tab[e] = make_float2(cs, sn);
  tab[n + (long)i * tps + pos] = make_float2(cs, sn);
}

// Head preparation kernels: 8 lanes per head row.  Lane l of a warp: row group q = l >> 3 (four
// token rows at a time), element chunk j = l & 7 (head elements 8j .. 8j + 7, two 16-byte loads).
// Per-row sums take three shuffles inside the 8-lane group.  NeoX RoPE pairs (i, i + rot/2),
// i < rot/2: rot 32 pairs chunks j and j ^ 2 (j < 4), rot 64 pairs chunks j and j ^ 4.  A block
// is 8 warps on 8 consecutive heads of one slice (512 contiguous columns) and kHpRows token rows.
struct HeadSlices {
  HeadSlice s[5];
  int n;
  // the slices repeated `reps` times, repetition r shifted by r col_step columns, r gamma_step
  // gamma values and r rstd_step rstd entries (the context K / V of every block in one launch)
  int reps = 1, col_step = 0, gamma_step = 0;
  long rstd_step = 0;
};
constexpr int kHpRows = 16;
constexpr int kQkvRows = 32;   // qkv_bwd_dz: more rows per block, fewer dg atomics
constexpr int kQkvSets = 4;    // qkv_bwd_dz: row sets whose loads are in flight together

__device__ __forceinline__ float sum8(float v) {
  v += __shfl_xor_sync(0xffffffffu, v, 1);
  v += __shfl_xor_sync(0xffffffffu, v, 2);
  v += __shfl_xor_sync(0xffffffffu, v, 4);
  return v;
}

__device__ __forceinline__ void ld8(const float* p, float (&v)[8]) {
  const float4 a = reinterpret_cast<const float4*>(p)[0], b = reinterpret_cast<const float4*>(p)[1];
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}

__device__ __forceinline__ void ld8(const __half* p, float (&v)[8]) {
  const uint4 w = *reinterpret_cast<const uint4*>(p);
  const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&ww[k]));
    v[2 * k] = f.x;
    v[2 * k + 1] = f.y;
  }
}

__device__ __forceinline__ void st8(float* p, const float (&v)[8]) {
  reinterpret_cast<float4*>(p)[0] = make_float4(v[0], v[1], v[2], v[3]);
  reinterpret_cast<float4*>(p)[1] = make_float4(v[4], v[5], v[6], v[7]);
}

__device__ __forceinline__ void st8_f16(__half* p, const float (&v)[8]) {
  uint4 o;
  o.x = pack_f16x2(v[0], v[1]);
  o.y = pack_f16x2(v[2], v[3]);
  o.z = pack_f16x2(v[4], v[5]);
  o.w = pack_f16x2(v[6], v[7]);
  *reinterpret_cast<uint4*>(p) = o;
}

// Sum over the block (blockDim.x a multiple of 32, at most 1024); every thread gets the total.
// `red` holds 32 floats of shared memory, used once per kernel.
__device__ __forceinline__ float block_sum(float v, float* red) {
  v = warp_sum(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31, nw = blockDim.x >> 5;
  if (l == 0) red[w] = v;
  __syncthreads();
  return warp_sum(l < nw ? red[l] : 0.f);
}

// rms_norm + adaLN modulate of one row per block, one thread per 8 columns: every load of the row
// (x, gamma, the sample's scale / shift) is issued before the row reduction, so the whole row is
// in flight at once.  h = f16(x rstd gamma (1 + sc) + sh), rstd = 1 / sqrt(mean(x^2) + eps).
__global__ void __launch_bounds__(1024) rmsnorm_mod_fwd_kernel(const float* __restrict__ x, int T, int D,
                                                               const float* __restrict__ gamma,
                                                               const float* __restrict__ sc,
                                                               const float* __restrict__ sh, long mod_stride, int tps,
                                                               float eps, __half* __restrict__ h,
                                                               float* __restrict__ rstd) {
  pdl_prologue();
  __shared__ float red[32];
  const int row = blockIdx.x, c = 8 * threadIdx.x;
  const bool act = c < D;
  const long s = row / tps;
  float v[8], gm[8], a[8], b[8];
  if (act) {
    ld8(x + (long)row * D + c, v);
    ld8(gamma + c, gm);
    if (sc) {
      ld8(sc + s * mod_stride + c, a);
      ld8(sh + s * mod_stride + c, b);
    }
  } else {
#pragma unroll
    for (int k = 0; k < 8; ++k) v[k] = 0.f;
  }
  float ss = 0.f;
#pragma unroll
  for (int k = 0; k < 8; ++k) ss = fmaf(v[k], v[k], ss);
  const float r = rsqrtf(block_sum(ss, red) / (float)D + eps);
  if (threadIdx.x == 0 && rstd) rstd[row] = r;
  if (!act) return;
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    v[k] *= r * gm[k];
    if (sc) v[k] = fmaf(v[k], 1.f + a[k], b[k]);
  }
  st8_f16(h + (long)row * D + c, v);
}

// The residual step of a block half fused with the norm that follows it, one row per block, one
// thread per 8 columns: x_out = x_in + y (gate null: the cross-attention residual) or
// x_in + y s (s = the sample's gate vector, sigmoid(1 - g) as the modulation kernel leaves it),
// then h = f16(rms_norm(x_out) gamma (1 + sc) + sh) and its rstd, as rmsnorm_mod_fwd.
__global__ void __launch_bounds__(1024) residual_norm_kernel(const float* __restrict__ x_in,
                                                             const float* __restrict__ y,
                                                             const float* __restrict__ gate, long gstride, int T,
                                                             int D, int tps, float* __restrict__ x_out,
                                                             const float* __restrict__ gamma,
                                                             const float* __restrict__ sc,
                                                             const float* __restrict__ sh, long mod_stride, float eps,
                                                             __half* __restrict__ h, float* __restrict__ rstd) {
  pdl_prologue();
  __shared__ float red[32];
  const int row = blockIdx.x, c = 8 * threadIdx.x;
  const bool act = c < D;
  const long s = row / tps;
  const long e = (long)row * D + c;
  float v[8], w[8], gv[8], gm[8], a[8], b[8];
  if (act) {
    ld8(x_in + e, v);
    ld8(y + e, w);
    if (gate) ld8(gate + s * gstride + c, gv);
#pragma unroll
    for (int k = 0; k < 8; ++k) v[k] = gate ? fmaf(w[k], gv[k], v[k]) : v[k] + w[k];
    st8(x_out + e, v);
  } else {
#pragma unroll
    for (int k = 0; k < 8; ++k) v[k] = 0.f;
  }
  float ss = 0.f;
#pragma unroll
  for (int k = 0; k < 8; ++k) ss = fmaf(v[k], v[k], ss);
  const float r = rsqrtf(block_sum(ss, red) / (float)D + eps);
  if (threadIdx.x == 0 && rstd) rstd[row] = r;
  if (!act) return;
  // the row-invariant vectors (gamma, the sample's scale / shift: cache-resident) only now, so
  // they hold no registers while the row's own loads are in flight
  ld8(gamma + c, gm);
  if (sc) {
    ld8(sc + s * mod_stride + c, a);
    ld8(sh + s * mod_stride + c, b);
  }
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    v[k] *= r * gm[k];
    if (sc) v[k] = fmaf(v[k], 1.f + a[k], b[k]);
  }
  st8_f16(h + e, v);
}

// Backward of rmsnorm_mod_fwd, one row per block (as the forward): with dn = dh gamma (1 + sc),
// gx += rstd (dn - x rstd^2 mean(dn x)); gx_h (nullable) receives f16(gx) as well.
__global__ void __launch_bounds__(1024) rmsnorm_mod_bwd_kernel(const float* __restrict__ dh,
                                                               const float* __restrict__ x,
                                                               const float* __restrict__ rstd, int T, int D,
                                                               const float* __restrict__ gamma,
                                                               const float* __restrict__ sc, long mod_stride, int tps,
                                                               float* __restrict__ gx,
                                                               __half* __restrict__ gx_h) {
  pdl_prologue();
  __shared__ float red[32];
  const int row = blockIdx.x, c = 8 * threadIdx.x;
  const bool act = c < D;
  const long s = row / tps;
  const long e = (long)row * D + c;
  float v[8], d[8], gm[8], a[8], g[8];
  const float r = rstd[row];
  if (act) {
    ld8(x + e, v);
    ld8(dh + e, d);
    ld8(gamma + c, gm);
    ld8(gx + e, g);
    if (sc) ld8(sc + s * mod_stride + c, a);
  } else {
#pragma unroll
    for (int k = 0; k < 8; ++k) v[k] = d[k] = 0.f;
  }
  float dot = 0.f;
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    if (act) d[k] *= gm[k] * (sc ? 1.f + a[k] : 1.f);   // dn
    dot = fmaf(d[k], v[k], dot);
  }
  dot = block_sum(dot, red) * r / (float)D;   // rstd mean(dn x)
  if (!act) return;
#pragma unroll
  for (int k = 0; k < 8; ++k) g[k] += r * (d[k] - v[k] * r * dot);
  st8(gx + e, g);
  if (gx_h) st8_f16(gx_h + e, g);
}

// RoPE of this lane's chunk j at position pos (inverse rotation when inv): first element of a pair
// x cos -/+ partner sin, second partner sin +/- ... ; all lanes take part in the shuffles.
__device__ __forceinline__ void rope8(float (&v)[8], int j, int pos, int rot, const float2* __restrict__ tab, bool inv) {
  const int half = rot / 2, px = rot == 32 ? 2 : 4;
  float pv[8];
#pragma unroll
  for (int k = 0; k < 8; ++k) pv[k] = __shfl_xor_sync(0xffffffffu, v[k], px);
  if (rot == 64 || j < 4) {
    const bool first = (j & px) == 0;
    const float4* cs = reinterpret_cast<const float4*>(tab + pos * half + ((8 * j) & (half - 1)));
#pragma unroll
    for (int k2 = 0; k2 < 4; ++k2) {
      const float4 c = cs[k2];   // (cos, sin) of elements 2 k2 and 2 k2 + 1 of the chunk
      const float c0 = c.x, s0 = inv ? -c.y : c.y, c1 = c.z, s1 = inv ? -c.w : c.w;
      if (first) {
        v[2 * k2] = v[2 * k2] * c0 - pv[2 * k2] * s0;
        v[2 * k2 + 1] = v[2 * k2 + 1] * c1 - pv[2 * k2 + 1] * s1;
      } else {
        v[2 * k2] = pv[2 * k2] * s0 + v[2 * k2] * c0;
        v[2 * k2 + 1] = pv[2 * k2 + 1] * s1 + v[2 * k2 + 1] * c1;
      }
    }
  }
}

// Grid (ceil(H * nslices / 8), ceil(T / kHpRows)).
template <typename Y>
__global__ void __launch_bounds__(256) head_prep_fwd_kernel(const Y* __restrict__ y, int T, int ncols, int H,
                                                            const HeadSlices slices, int tps, float eps, int rot,
                                                            const float2* __restrict__ tab,
                                                            __half* __restrict__ out) {
  pdl_prologue();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, j = lane & 7, q = lane >> 3;
  const int pair = blockIdx.x * 8 + warp;
  if (pair >= H * slices.n * slices.reps) return;
  const int rp = pair / (H * slices.n), pr = pair - rp * H * slices.n;
  const int si = pr / H, h = pr % H;
  HeadSlice sl = slices.s[si];
  sl.col += rp * slices.col_step;
  if (sl.gamma) sl.gamma += rp * slices.gamma_step;
  if (sl.rstd) sl.rstd += rp * slices.rstd_step;
  const int col = sl.col + h * 64 + 8 * j;
  float gm[8];
  if (sl.gamma) ld8(sl.gamma + 8 * j, gm);
  else {
#pragma unroll
    for (int k = 0; k < 8; ++k) gm[k] = 1.f;
  }
  const int tb0 = blockIdx.y * kHpRows;
  int pos = (tb0 + q) % tps;
  // every row's load first (the rstd stores below may alias y for the compiler)
  float vr[kHpRows / 4][8];
#pragma unroll
  for (int it = 0; it < kHpRows / 4; ++it) {
    const int t = tb0 + 4 * it + q;
    if (t < T) {
      ld8(y + (long)t * ncols + col, vr[it]);
    } else {
#pragma unroll
      for (int k = 0; k < 8; ++k) vr[it][k] = 0.f;
    }
  }
#pragma unroll
  for (int it = 0; it < kHpRows / 4; ++it) {
    const int t = tb0 + 4 * it + q;
    const bool valid = t < T;
    float (&v)[8] = vr[it];
    if (sl.gamma) {
      float ss = 0.f;
#pragma unroll
      for (int k = 0; k < 8; ++k) ss = fmaf(v[k], v[k], ss);
      const float r = rsqrtf(sum8(ss) / 64.f + eps);
      if (valid && j == 0 && sl.rstd) sl.rstd[(long)t * H + h] = r;
#pragma unroll
      for (int k = 0; k < 8; ++k) v[k] *= r * gm[k];
    }
    if (sl.rope && (rot == 32 || rot == 64)) rope8(v, j, pos, rot, tab, false);
    if (valid) st8_f16(out + (long)t * ncols + col, v);
    pos += 4;
    while (pos >= tps) pos -= tps;
  }
}

// Backward of one slice.  Grid (ceil(H / 8), ceil(T / kHpRows)).
__global__ void __launch_bounds__(256) head_prep_bwd_kernel(const float* g, long g_ld, const float* __restrict__ y,
                                                            int T, int ncols, int H, HeadSlice sl, int tps, int rot,
                                                            const float2* __restrict__ tab, float gscale,
                                                            const float* g2, long g2_ld, float* dy,
                                                            __half* dy_h) {
  pdl_prologue();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, j = lane & 7, q = lane >> 3;
  const int h = blockIdx.x * 8 + warp;
  if (h >= H) return;
  float gm[8];
  if (sl.gamma) ld8(sl.gamma + 8 * j, gm);
  const int tb0 = blockIdx.y * kHpRows;
  int pos = (tb0 + q) % tps;
  // every row set's loads first (gradient, the second stream's, the projection output, rstd),
  // then the arithmetic and stores row set by row set
  constexpr int NS = kHpRows / 4;
  float ga[NS][8], ya[NS][8], ra[NS];
#pragma unroll
  for (int it = 0; it < NS; ++it) {
    const int t = tb0 + 4 * it + q;
    ra[it] = 0.f;
    if (t < T) {
      ld8(g + (long)t * g_ld + h * 64 + 8 * j, ga[it]);
      if (sl.gamma) {
        ld8(y + (long)t * ncols + sl.col + h * 64 + 8 * j, ya[it]);
        ra[it] = sl.rstd[(long)t * H + h];
      }
    } else {
#pragma unroll
      for (int k = 0; k < 8; ++k) ga[it][k] = ya[it][k] = 0.f;
    }
  }
#pragma unroll
  for (int it = 0; it < NS; ++it) {
    const int t = tb0 + 4 * it + q;
    const bool valid = t < T;
    float(&gv)[8] = ga[it];
    float(&yv)[8] = ya[it];
    const float r = ra[it];
    if (valid && g2) {
      float w[8];
      ld8(g2 + (long)t * g2_ld + h * 64 + 8 * j, w);
#pragma unroll
      for (int k = 0; k < 8; ++k) gv[k] -= w[k];
    }
#pragma unroll
    for (int k = 0; k < 8; ++k) gv[k] *= gscale;
    if (sl.rope && (rot == 32 || rot == 64)) rope8(gv, j, pos, rot, tab, true);
    if (sl.gamma) {
      float dot = 0.f;
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        yv[k] *= r;            // normalized input
        gv[k] *= gm[k];        // gradient w.r.t. the normalized input
        dot = fmaf(gv[k], yv[k], dot);
      }
      const float mean = sum8(dot) / 64.f;
#pragma unroll
      for (int k = 0; k < 8; ++k) gv[k] = r * (gv[k] - yv[k] * mean);
    }
    if (valid) {
      if (dy_h) st8_f16(dy_h + (long)t * ncols + sl.col + h * 64 + 8 * j, gv);
      else st8(dy + (long)t * ncols + sl.col + h * 64 + 8 * j, gv);
    }
    pos += 4;
    while (pos >= tps) pos -= tps;
  }
}

// The self-attention head preparation's backward (q and k: inverse RoPE, then the per-head
// rms-norm backward; v: identity) fused with the qkv projection's backward prologue: writes
// dz = f16(g * dy) and adds colsum(dy * y / g) into dg (DoRA; g null: dz = f16(dy)), with
// y = the projection output qkv (no bias).  Block = 8 warps on 8 consecutive head slices of
// [q heads | k heads | v heads (| qd heads | kd heads)] and kHpRows token rows; each lane adds
// its 8 columns' dg sums (summed over the warp's four row groups first) once.
// Differential attention (nsl = 5): the qd / kd gradients in dq3 come from the second softmax
// stream run on +dO, so they enter negated, and the v gradient is dq3's minus dv2 (that
// stream's dV).  Grid (ceil(nsl H / 8), ceil(T / kHpRows)).
__global__ void __launch_bounds__(256, 2) qkv_bwd_dz_kernel(const float* __restrict__ dq3,
                                                            const __half* __restrict__ qkv, int T, int D, int H,
                                                            int nsl, const float* __restrict__ rq,
                                                            const float* __restrict__ rk, const float* __restrict__ rq2,
                                                            const float* __restrict__ rk2, const float* __restrict__ dv2,
                                                            const float* __restrict__ gq, const float* __restrict__ gk,
                                                            int tps, int rot, const float2* __restrict__ tab,
                                                            const float* __restrict__ g, __half* __restrict__ dz,
                                                            float* __restrict__ dg) {
  pdl_prologue();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, j = lane & 7, q = lane >> 3;
  const int hs = blockIdx.x * 8 + warp;
  if (hs >= nsl * H) return;
  const int slice = hs / H, h = hs % H;
  const int ncols = nsl * D, col = slice * D + h * 64 + 8 * j;
  const bool norm = slice != 2;
  const bool qside = slice == 0 || slice == 3;
  const float* rs = slice == 0 ? rq : slice == 1 ? rk : slice == 3 ? rq2 : rk2;
  const float sgn = slice >= 3 ? -1.f : 1.f;
  const bool sub_dv2 = slice == 2 && dv2 != nullptr;
  float gm[8], gd[8], acc[8];
  if (norm) ld8((qside ? gq : gk) + 8 * j, gm);
  if (g) ld8(g + col, gd);
#pragma unroll
  for (int k = 0; k < 8; ++k) acc[k] = 0.f;
  const int tb0 = blockIdx.y * kQkvRows;
  float igd[8];
#pragma unroll
  for (int k = 0; k < 8; ++k) igd[k] = g ? 1.f / gd[k] : 1.f;
  // kQkvSets row sets in flight per thread: their raw loads (f32 gradient as two float4, f16 qkv
  // as one uint4) are all issued before any of them is processed (the dz stores in between may
  // alias the inputs for the compiler)
  for (int it0 = 0; it0 < kQkvRows / 4 && tb0 + 4 * it0 < T; it0 += kQkvSets) {
    float4 ga[kQkvSets][2];
    uint4 ya[kQkvSets];
    float ra[kQkvSets];
#pragma unroll
    for (int u = 0; u < kQkvSets; ++u) {
      const int t = tb0 + 4 * (it0 + u) + q;
      ra[u] = 0.f;
      if (it0 + u < kQkvRows / 4 && t < T) {
        const float4* gp = reinterpret_cast<const float4*>(dq3 + (long)t * ncols + col);
        ga[u][0] = gp[0];
        ga[u][1] = gp[1];
        ya[u] = (norm || g) ? *reinterpret_cast<const uint4*>(qkv + (long)t * ncols + col) : make_uint4(0u, 0u, 0u, 0u);
        if (norm) ra[u] = rs[(long)t * H + h];
      } else {
        ga[u][0] = ga[u][1] = make_float4(0.f, 0.f, 0.f, 0.f);
        ya[u] = make_uint4(0u, 0u, 0u, 0u);
      }
    }
#pragma unroll
    for (int u = 0; u < kQkvSets; ++u) {
      const int t = tb0 + 4 * (it0 + u) + q;
      const bool valid = it0 + u < kQkvRows / 4 && t < T;
      float gv[8] = {ga[u][0].x, ga[u][0].y, ga[u][0].z, ga[u][0].w, ga[u][1].x, ga[u][1].y, ga[u][1].z, ga[u][1].w};
      float yv[8];
      {
        const uint32_t yw[4] = {ya[u].x, ya[u].y, ya[u].z, ya[u].w};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&yw[k]));
          yv[2 * k] = f.x;
          yv[2 * k + 1] = f.y;
        }
      }
      const float r = ra[u];
      if (valid && sub_dv2) {
        float w[8];
        ld8(dv2 + (long)t * D + h * 64 + 8 * j, w);
#pragma unroll
        for (int k = 0; k < 8; ++k) gv[k] -= w[k];
      }
      if (sgn < 0.f) {
#pragma unroll
        for (int k = 0; k < 8; ++k) gv[k] = -gv[k];
      }
      if (norm) {
        if (rot == 32 || rot == 64) rope8(gv, j, (valid ? t : 0) % tps, rot, tab, true);
        float dot = 0.f;
#pragma unroll
        for (int k = 0; k < 8; ++k) dot = fmaf(gv[k] * gm[k], yv[k] * r, dot);
        const float mean = sum8(dot) / 64.f;
#pragma unroll
        for (int k = 0; k < 8; ++k) gv[k] = r * (gv[k] * gm[k] - yv[k] * r * mean);
      }
      if (g) {
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          acc[k] = fmaf(gv[k], yv[k] * igd[k], acc[k]);
          gv[k] *= gd[k];
        }
      }
      if (valid) st8_f16(dz + (long)t * ncols + col, gv);
    }
  }
  if (g) {
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      acc[k] += __shfl_xor_sync(0xffffffffu, acc[k], 8);
      acc[k] += __shfl_xor_sync(0xffffffffu, acc[k], 16);
      if (q == 0) atomicAdd(dg + col + k, acc[k]);
    }
  }
}

// Grid (ceil(D / 4 / 256), rows): thread = 4 consecutive columns of one row.
__global__ void gate_residual_kernel(const float* __restrict__ x_in, const float* __restrict__ y,
                                     const float* __restrict__ gate, long gstride, int T, int D, int tps,
                                     float* __restrict__ x_out) {
  pdl_prologue();
  const int cidx = 4 * (blockIdx.x * blockDim.x + threadIdx.x);
  if (cidx >= D) return;
  for (int t = blockIdx.y; t < T; t += gridDim.y) {
    const long e = (long)t * D + cidx;
    const float4 gv = *reinterpret_cast<const float4*>(gate + (long)(t / tps) * gstride + cidx);
    const float4 a = *reinterpret_cast<const float4*>(x_in + e);
    const float4 b = *reinterpret_cast<const float4*>(y + e);
    *reinterpret_cast<float4*>(x_out + e) =
        make_float4(a.x + b.x * gv.x, a.y + b.y * gv.y, a.z + b.z * gv.z, a.w + b.w * gv.w);
  }
}

__global__ void gate_bwd_kernel(const float* __restrict__ gx, const float* __restrict__ gate, long gstride, int T,
                                int D, int tps, float* __restrict__ dy) {
  pdl_prologue();
  const int cidx = 4 * (blockIdx.x * blockDim.x + threadIdx.x);
  if (cidx >= D) return;
  for (int t = blockIdx.y; t < T; t += gridDim.y) {
    const long e = (long)t * D + cidx;
    const float4 gv = *reinterpret_cast<const float4*>(gate + (long)(t / tps) * gstride + cidx);
    const float4 a = *reinterpret_cast<const float4*>(gx + e);
    *reinterpret_cast<float4*>(dy + e) = make_float4(a.x * gv.x, a.y * gv.y, a.z * gv.z, a.w * gv.w);
  }
}

__global__ void add_kernel(const float* __restrict__ x, const float* __restrict__ y, long n, float* __restrict__ out) {
  pdl_prologue();
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x) out[i] = x[i] + y[i];
}

__device__ __forceinline__ float sigm(float x) { return 1.f / (1.f + __expf(-x)); }

// out = x - y for f16 vectors, 8 values per thread (difference taken in f32)
__global__ void sub_f16_kernel(const __half* __restrict__ x, const __half* __restrict__ y, long n8,
                                __half* __restrict__ out) {
  pdl_prologue();
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < n8; i += (long)gridDim.x * blockDim.x) {
    const uint4 a = reinterpret_cast<const uint4*>(x)[i], b = reinterpret_cast<const uint4*>(y)[i];
    const uint32_t aw[4] = {a.x, a.y, a.z, a.w}, bw[4] = {b.x, b.y, b.z, b.w};
    uint32_t o[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float2 fa = __half22float2(*reinterpret_cast<const __half2*>(&aw[k]));
      const float2 fb = __half22float2(*reinterpret_cast<const __half2*>(&bw[k]));
      o[k] = pack_f16x2(fa.x - fb.x, fa.y - fb.y);
    }
    reinterpret_cast<uint4*>(out)[i] = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

// SwiGLU over rows: f[t] = [val (I) | gate (I)], a[t] = val * silu(gate).  Grid (I / 4 / 256
// column blocks, T rows): each thread owns 4 consecutive columns of one row (128-bit accesses).
// act = f16(val * silu(gate)) of the ff.proj output f = [val | gate] (f16 rows of 2I), eight
// columns per thread (16-byte loads and stores)
__global__ void swiglu_fwd_kernel(const __half* __restrict__ f, int T, int I, __half* __restrict__ a) {
  pdl_prologue();
  const int j = 8 * (blockIdx.x * blockDim.x + threadIdx.x);
  if (j >= I) return;
  for (int t = blockIdx.y; t < T; t += gridDim.y) {
    const __half* fr = f + (long)t * 2 * I;
    const uint4 v4 = *reinterpret_cast<const uint4*>(fr + j);
    const uint4 g4 = *reinterpret_cast<const uint4*>(fr + I + j);
    const uint32_t vw[4] = {v4.x, v4.y, v4.z, v4.w}, gw[4] = {g4.x, g4.y, g4.z, g4.w};
    uint32_t o[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float2 v = __half22float2(*reinterpret_cast<const __half2*>(&vw[k]));
      const float2 g = __half22float2(*reinterpret_cast<const __half2*>(&gw[k]));
      o[k] = pack_f16x2(v.x * g.x * sigm(g.x), v.y * g.y * sigm(g.y));
    }
    *reinterpret_cast<uint4*>(a + (long)t * I + j) = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

__global__ void silu_f16_kernel(const float* __restrict__ x, long n, __half* __restrict__ out) {
  pdl_prologue();
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x) {
    const float v = x[i];
    out[i] = __float2half_rn(v * sigm(v));
  }
}

// out = dy * silu'(h), silu'(h) = sigmoid(h) (1 + h (1 - sigmoid(h)))   (out may alias dy)
__global__ void silu_bwd_kernel(const float* dy, const float* __restrict__ h, long n, float* out) {
  pdl_prologue();
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x) {
    const float v = h[i], sg = sigm(v);
    out[i] = dy[i] * sg * (1.f + v * (1.f - sg));
  }
}

// Per-sample column sums for the adaLN modulation gradient (the vectors of a block are per
// sample: rows t of sample b = t / tps).  One thread per column, blockIdx.y = sample, blockIdx.z
// = a slice of the sample's rows; the partial sums are added into the [B][row stride] outputs.
//   norm (x non-null): h = n (1 + sc) + sh with n = x rstd gamma:
//       dsc[b][c] += gamma[c] sum_t dh x rstd,   dsh[b][c] += sum_t dh
//   gate (x null): out = res + y s, s = sigmoid(1 - g) (the modulation vectors hold s itself):
//       dg[b][c] += -s (1 - s) sum_t dh y  (here dh = the gradient of the block half's output,
//       y = the gated branch)
constexpr int kColRows = 128;
__global__ void __launch_bounds__(128) mod_colsum_kernel(const float* __restrict__ dh, const float* __restrict__ x,
                                                         const float* __restrict__ rstd,
                                                         const float* __restrict__ gamma,
                                                         const float* __restrict__ y, const float* __restrict__ gate,
                                                         long gate_stride, int T, int D, int tps, long out_stride,
                                                         float* __restrict__ o1, float* __restrict__ o2) {
  pdl_prologue();
  const int c = blockIdx.x * 128 + threadIdx.x, b = blockIdx.y;
  if (c >= D) return;
  const int t0 = b * tps + blockIdx.z * kColRows;
  const int t1 = min(b * tps + tps, min(t0 + kColRows, T));
  float a1 = 0.f, a2 = 0.f;
  for (int t = t0; t < t1; ++t) {
    const float g = dh[(long)t * D + c];
    if (x) {
      a1 = fmaf(g, x[(long)t * D + c] * rstd[t], a1);
      a2 += g;
    } else {
      a1 = fmaf(g, y[(long)t * D + c], a1);
    }
  }
  if (t1 <= t0) return;
  if (x) {
    atomicAdd(o1 + (long)b * out_stride + c, gamma[c] * a1);
    atomicAdd(o2 + (long)b * out_stride + c, a2);
  } else {
    const float s = gate[(long)b * gate_stride + c];
    atomicAdd(o1 + (long)b * out_stride + c, -s * (1.f - s) * a1);
  }
}

// mod[l][b][j] = ssg[l][j] + gcond[b][j] for L blocks (ssg, mod with block strides 6D, B 6D);
// slots 2 and 5 (the gates) leave as sigmoid(1 - v)
__global__ void modulation_kernel(const float* __restrict__ ssg, const float* __restrict__ gcond, int L, int B, int D,
                                  float* __restrict__ mod) {
  pdl_prologue();
  const long per = 6L * D, n = (long)L * B * per;
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x) {
    const long l = i / ((long)B * per), bi = i - l * B * per, j = bi % per;
    float v = ssg[l * per + j] + gcond[bi];
    const int slot = (int)(j / D);
    if (slot == 2 || slot == 5) v = 1.f / (__expf(v - 1.f) + 1.f);   // h * sigmoid(1 - g)
    mod[i] = v;
  }
}

__global__ void mse_kernel(const float* __restrict__ vel, const float* __restrict__ tgt, const float* __restrict__ wt,
                           long per, float inv, float gscale, float* __restrict__ loss, float* __restrict__ dvel) {
  pdl_prologue();
  const int b = blockIdx.y;
  float acc = 0.f;
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < per; i += (long)gridDim.x * blockDim.x) {
    const long e = (long)b * per + i;
    const float d = vel[e] - tgt[e];
    if (wt) {   // inpaint: sum of w (v - t)^2, the weights carry the normalisation
      acc += wt[e] * d * d;
      if (dvel) dvel[e] = 2.f * wt[e] * d * gscale;
    } else {
      acc += d * d;
      if (dvel) dvel[e] = 2.f * d * inv * gscale;
    }
  }
  acc = warp_sum(acc);
  __shared__ float part[32];
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < (blockDim.x >> 5) ? part[threadIdx.x] : 0.f;
    v = warp_sum(v);
    if (threadIdx.x == 0) atomicAdd(loss + b, wt ? v : v * inv);
  }
}

// dst[r][c] = c < w ? f16(src[r][c]) : 0 for c < ld (a row-padded f16 copy)
__global__ void pad_f16_kernel(const float* __restrict__ src, long rows, int w, __half* __restrict__ dst, long ld) {
  pdl_prologue();
  const long n = rows * ld;
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x) {
    const long r = i / ld;
    const int cc = (int)(i - r * ld);
    dst[i] = __float2half_rn(cc < w ? src[r * w + cc] : 0.f);
  }
}

// dst[b S + t][:] = y[b S + t][:] + (t >= mem ? le[b (S - mem) + t - mem][:] : 0); dst may be y
__global__ void add_local_kernel(const float* y, const float* __restrict__ le, long rows, int S, int mem, int D,
                                 float* dst) {
  pdl_prologue();
  const long n = rows * D;
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x) {
    const long r = i / D;
    const int col = (int)(i - r * D);
    const long b = r / S;
    const int t = (int)(r - b * S);
    float v = y[i];
    if (t >= mem) v += le[(b * (S - mem) + (t - mem)) * D + col];
    dst[i] = v;
  }
}

__global__ void scale_kernel(float4* __restrict__ x, long n4, float s) {
  pdl_prologue();
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += (long)gridDim.x * blockDim.x) {
    float4 v = x[i];
    v.x *= s; v.y *= s; v.z *= s; v.w *= s;
    x[i] = v;
  }
}

__global__ void scale_tail_kernel(float* __restrict__ x, long from, long n, float s) {
  pdl_prologue();
  for (long i = from + threadIdx.x; i < n; i += blockDim.x) x[i] *= s;
}

__global__ void copy_rows_kernel(const float* __restrict__ src, int src_rows_per, int src_off, float* __restrict__ dst,
                                 __half* __restrict__ dst_h, int dst_rows_per, int dst_off, int B, int rows,
                                 int D) {
  pdl_prologue();
  const long n = (long)B * rows * D;
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x) {
    const long d = i % D, r = (i / D) % rows, b = i / ((long)D * rows);
    const float v = src[((long)b * src_rows_per + src_off + r) * D + d];
    const long o = ((long)b * dst_rows_per + dst_off + r) * D + d;
    if (dst) dst[o] = v;
    if (dst_h) dst_h[o] = __float2half_rn(v);
  }
}

// The same copy with 16-byte rows (D % 4 == 0, 16-byte aligned pointers): one block row per
// copied row (grid-stride over rows), thread = 4 columns, no index division per element.
__global__ void copy_rows4_kernel(const float* __restrict__ src, int src_rows_per, int src_off, float* __restrict__ dst,
                                  __half* __restrict__ dst_h, int dst_rows_per, int dst_off, int B, int rows, int D) {
  pdl_prologue();
  const int c = 4 * (blockIdx.x * blockDim.x + threadIdx.x);
  if (c >= D) return;
  for (int rr = blockIdx.y; rr < B * rows; rr += gridDim.y) {
    const int b = rr / rows, r = rr - b * rows;
    const float4 v = *reinterpret_cast<const float4*>(src + ((long)b * src_rows_per + src_off + r) * D + c);
    const long o = ((long)b * dst_rows_per + dst_off + r) * D + c;
    if (dst) *reinterpret_cast<float4*>(dst + o) = v;
    if (dst_h) *reinterpret_cast<uint2*>(dst_h + o) = make_uint2(pack_f16x2(v.x, v.y), pack_f16x2(v.z, v.w));
  }
}

unsigned gs(long n, int threads = 256) {
  long b = (n + threads - 1) / threads;
  if (b > 148 * 16) b = 148 * 16;
  return (unsigned)(b < 1 ? 1 : b);
}

}  // namespace

// one block per row, one thread per 8 columns, in whole warps
static int row_block(int D, std::string& err) {
  if (D % 8 || D > 8192) { err = "rms_norm: D must be a multiple of 8 and at most 8192"; return 0; }
  return (D / 8 + 31) / 32 * 32;
}

int k_rmsnorm_mod_fwd(Ctx* c, const float* x, int T, int D, const float* gamma, const float* sc, const float* sh,
                      long mod_stride, int tps, float eps, __half* h, float* rstd, std::string& err) {
  const int nt = row_block(D, err);
  if (!nt) return 1;
  ProfScope prof_(c, "rmsnorm_mod_fwd");
  launch_pdl(c, rmsnorm_mod_fwd_kernel, (unsigned)T, nt, 0, x, T, D, gamma, sc, sh, mod_stride, tps, eps, h, rstd);
  return check_launch("rmsnorm_mod_fwd", err);
}

int k_residual_norm(Ctx* c, const float* x_in, const float* y, const float* gate, long gstride, int T, int D, int tps,
                    float* x_out, const float* gamma, const float* sc, const float* sh, long mod_stride, float eps,
                    __half* h, float* rstd, std::string& err) {
  const int nt = row_block(D, err);
  if (!nt) return 1;
  ProfScope prof_(c, "residual_norm");
  launch_pdl(c, residual_norm_kernel, (unsigned)T, nt, 0, x_in, y, gate, gstride, T, D, tps, x_out, gamma, sc, sh,
             mod_stride, eps, h, rstd);
  return check_launch("residual_norm", err);
}

int k_rmsnorm_mod_bwd(Ctx* c, const float* dh, const float* x, const float* rstd, int T, int D, const float* gamma,
                      const float* sc, long mod_stride, int tps, float* gx, __half* gx_h, std::string& err) {
  const int nt = row_block(D, err);
  if (!nt) return 1;
  ProfScope prof_(c, "rmsnorm_mod_bwd");
  launch_pdl(c, rmsnorm_mod_bwd_kernel, (unsigned)T, nt, 0, dh, x, rstd, T, D, gamma, sc, mod_stride, tps, gx, gx_h);
  return check_launch("rmsnorm_mod_bwd", err);
}

// (cos, sin) table of the context for (tps, rot, base); rebuilt only when one of them changes
const float2* k_rope_table(Ctx* c, int tps, int rot, float rope_base, std::string& err) {
  if (rot == 0) return nullptr;
  const size_t bytes = 2 * sizeof(float2) * (size_t)tps * (rot / 2);
  void* tab = scratch_get(c, kSlotRope, bytes, err);
  if (!tab) return nullptr;
  if (tab != c->rope_tab || c->rope_tps != tps || c->rope_rot != rot || c->rope_base != rope_base) {
    ++c->gen;   // recorded graphs may rely on the table's previous contents
    const int n = tps * (rot / 2);
    rope_table_kernel<<<(unsigned)((n + 255) / 256), 256, 0, c->stream>>>(tps, rot, log2f(rope_base),
                                                                            static_cast<float2*>(tab));
    if (check_launch("rope table", err)) return nullptr;
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    cudaStreamIsCapturing(c->stream, &cs);
    if (cs == cudaStreamCaptureStatusNone) {   // a captured build only exists once the graph runs
      c->rope_tab = tab;
      c->rope_tps = tps;
      c->rope_rot = rot;
      c->rope_base = rope_base;
    }
  }
  return static_cast<const float2*>(tab);
}

template <typename Y>
static int head_prep_fwd_t(Ctx* c, const Y* y, int T, int ncols, int H, const HeadSlice* slices, int nslices, int tps,
                           float eps, int rot, float rope_base, __half* out, std::string& err, int reps = 1,
                           int col_step = 0, int gamma_step = 0, long rstd_step = 0) {
  if (rot != 0 && rot != 32 && rot != 64) { err = "rope: rot must be 32 or 64"; return 1; }
  if (nslices < 1 || nslices > 5) { err = "head_prep: 1..5 slices"; return 1; }
  if (reps < 1) { err = "head_prep: reps must be positive"; return 1; }
  HeadSlices hs{};
  hs.reps = reps; hs.col_step = col_step; hs.gamma_step = gamma_step; hs.rstd_step = rstd_step;
  bool any_rope = false;
  for (int i = 0; i < nslices; ++i) {
    hs.s[i] = slices[i];
    any_rope = any_rope || slices[i].rope;
  }
  hs.n = nslices;
  const float2* tab = nullptr;
  if (any_rope && rot && !(tab = k_rope_table(c, tps, rot, rope_base, err))) return 1;
  ProfScope prof_(c, "head_prep_fwd");
  if ((T + kHpRows - 1) / kHpRows > 65535) { err = "head prep: too many rows"; return 1; }
  const dim3 grid((unsigned)((H * nslices * reps + 7) / 8), (unsigned)((T + kHpRows - 1) / kHpRows));
  launch_pdl(c, head_prep_fwd_kernel<Y>, grid, 256, 0, y, T, ncols, H, hs, tps, eps, rot, tab, out);
  return check_launch("head_prep_fwd", err);
}

int k_head_prep_fwd(Ctx* c, const float* y, int T, int ncols, int H, const HeadSlice* slices, int nslices, int tps,
                    float eps, int rot, float rope_base, __half* out, std::string& err) {
  return head_prep_fwd_t(c, y, T, ncols, H, slices, nslices, tps, eps, rot, rope_base, out, err);
}

int k_head_prep_fwd_reps(Ctx* c, const float* y, int T, int ncols, int H, const HeadSlice* slices, int nslices,
                         int tps, float eps, int rot, float rope_base, __half* out, int reps, int col_step,
                         int gamma_step, long rstd_step, std::string& err) {
  return head_prep_fwd_t(c, y, T, ncols, H, slices, nslices, tps, eps, rot, rope_base, out, err, reps, col_step,
                         gamma_step, rstd_step);
}

int k_head_prep_fwd(Ctx* c, const __half* y, int T, int ncols, int H, const HeadSlice* slices, int nslices,
                    int tps, float eps, int rot, float rope_base, __half* out, std::string& err) {
  return head_prep_fwd_t(c, y, T, ncols, H, slices, nslices, tps, eps, rot, rope_base, out, err);
}

int k_qkv_bwd_dz(Ctx* c, const float* dq3, const __half* qkv, int T, int D, int H, int nsl, const float* rq,
                 const float* rk, const float* rq2, const float* rk2, const float* dv2, const float* gq, const float* gk,
                 int tps, int rot, float rope_base, const float* g, __half* dz, float* dg, std::string& err) {
  if (nsl != 3 && nsl != 5) { err = "qkv backward: 3 or 5 slices"; return 1; }
  const float2* tab = nullptr;
  if (rot && !(tab = k_rope_table(c, tps, rot, rope_base, err))) return 1;
  if ((T + kQkvRows - 1) / kQkvRows > 65535) { err = "qkv backward: too many rows"; return 1; }
  if (g && cudaMemsetAsync(dg, 0, sizeof(float) * nsl * D, c->stream) != cudaSuccess) return check_launch("memset", err);
  ProfScope prof_(c, "qkv_bwd_dz");
  launch_pdl(c, qkv_bwd_dz_kernel, dim3((unsigned)((nsl * H + 7) / 8), (unsigned)((T + kQkvRows - 1) / kQkvRows)), 256,
             0, dq3, qkv, T, D, H, nsl, rq, rk, rq2, rk2, dv2, gq, gk, tps, rot, tab, g, dz, dg);
  return check_launch("qkv_bwd_dz", err);
}

int k_head_prep_bwd(Ctx* c, const float* g, long g_ld, const float* y, int T, int ncols, int H, const HeadSlice& sl,
                    int tps, int rot, float rope_base, float* dy, __half* dy_h, std::string& err,
                    float gscale, const float* g2, long g2_ld) {
  const float2* tab = nullptr;
  if (sl.rope && rot && !(tab = k_rope_table(c, tps, rot, rope_base, err))) return 1;
  ProfScope prof_(c, "head_prep_bwd");
  if ((T + kHpRows - 1) / kHpRows > 65535) { err = "head prep: too many rows"; return 1; }
  const dim3 grid((unsigned)((H + 7) / 8), (unsigned)((T + kHpRows - 1) / kHpRows));
  launch_pdl(c, head_prep_bwd_kernel, grid, 256, 0, g, g_ld, y, T, ncols, H, sl, tps, rot, tab, gscale, g2, g2_ld, dy,
             dy_h);
  return check_launch("head_prep_bwd", err);
}

int k_gate_residual(Ctx* c, const float* x_in, const float* y, const float* gate, long gstride, int T, int D, int tps,
                    float* x_out, std::string& err) {
  ProfScope prof_(c, "gate_residual");
  if (D % 4) { err = "gate: the width must be a multiple of 4"; return 1; }
  launch_pdl(c, gate_residual_kernel, dim3((unsigned)((D / 4 + 255) / 256), (unsigned)(T < 65535 ? T : 65535)), 256, 0, x_in, y, gate, gstride, T, D, tps, x_out);
  return check_launch("gate_residual", err);
}

int k_gate_bwd(Ctx* c, const float* gx, const float* gate, long gstride, int T, int D, int tps, float* dy,
               std::string& err) {
  ProfScope prof_(c, "gate_bwd");
  if (D % 4) { err = "gate: the width must be a multiple of 4"; return 1; }
  launch_pdl(c, gate_bwd_kernel, dim3((unsigned)((D / 4 + 255) / 256), (unsigned)(T < 65535 ? T : 65535)), 256, 0, gx, gate, gstride, T, D, tps, dy);
  return check_launch("gate_bwd", err);
}

int k_sub_f16(Ctx* c, const __half* x, const __half* y, long n, __half* out, std::string& err) {
  if (n % 8) { err = "sub: n must be a multiple of 8"; return 1; }
  ProfScope prof_(c, "sub_f16");
  launch_pdl(c, sub_f16_kernel, gs(n / 8), 256, 0, x, y, n / 8, out);
  return check_launch("sub_f16", err);
}

int k_add(Ctx* c, const float* x, const float* y, long n, float* out, std::string& err) {
  ProfScope prof_(c, "add");
  launch_pdl(c, add_kernel, gs(n), 256, 0, x, y, n, out);
  return check_launch("add", err);
}

int k_swiglu_fwd(Ctx* c, const __half* f, int T, int I, __half* a, std::string& err) {
  ProfScope prof_(c, "swiglu_fwd");
  if (I % 8) { err = "swiglu: the hidden width must be a multiple of 8"; return 1; }
  launch_pdl(c, swiglu_fwd_kernel, dim3((unsigned)((I / 8 + 255) / 256), (unsigned)(T < 65535 ? T : 65535)), 256, 0,
             f, T, I, a);
  return check_launch("swiglu_fwd", err);
}

int k_silu_f16(Ctx* c, const float* x, long n, __half* out, std::string& err) {
  ProfScope prof_(c, "silu");
  launch_pdl(c, silu_f16_kernel, gs(n), 256, 0, x, n, out);
  return check_launch("silu", err);
}

int k_silu_bwd(Ctx* c, const float* dy, const float* h, long n, float* out, std::string& err) {
  ProfScope prof_(c, "silu_bwd");
  launch_pdl(c, silu_bwd_kernel, gs(n), 256, 0, dy, h, n, out);
  return check_launch("silu_bwd", err);
}

static int mod_colsum(Ctx* c, const float* dh, const float* x, const float* rstd, const float* gamma, const float* y,
                      const float* gate, long gate_stride, int T, int D, int tps, long out_stride, float* o1, float* o2,
                      std::string& err) {
  if (T % tps) { err = "modulation gradient: rows must be whole samples"; return 1; }
  const dim3 grid((unsigned)((D + 127) / 128), (unsigned)(T / tps), (unsigned)((tps + kColRows - 1) / kColRows));
  ProfScope prof_(c, "mod_grad");
  launch_pdl(c, mod_colsum_kernel, grid, 128, 0, dh, x, rstd, gamma, y, gate, gate_stride, T, D, tps, out_stride, o1,
             o2);
  return check_launch("mod_grad", err);
}

int k_mod_grad_norm(Ctx* c, const float* dh, const float* x, const float* rstd, const float* gamma, int T, int D,
                    int tps, long out_stride, float* dsc, float* dsh, std::string& err) {
  return mod_colsum(c, dh, x, rstd, gamma, nullptr, nullptr, 0, T, D, tps, out_stride, dsc, dsh, err);
}

int k_mod_grad_gate(Ctx* c, const float* gy, const float* y, const float* gate, long gate_stride, int T, int D, int tps,
                    long out_stride, float* dgate, std::string& err) {
  return mod_colsum(c, gy, nullptr, nullptr, nullptr, y, gate, gate_stride, T, D, tps, out_stride, dgate, nullptr, err);
}

int k_modulation(Ctx* c, const float* ssg, const float* gcond, int B, int D, float* mod, std::string& err, int L) {
  ProfScope prof_(c, "modulation");
  launch_pdl(c, modulation_kernel, gs((long)L * B * 6 * D), 256, 0, ssg, gcond, L, B, D, mod);
  return check_launch("modulation", err);
}

int k_mse(Ctx* c, const float* vel, const float* target, int B, long per, float* loss, float* dvel, float grad_scale,
          const float* weight, std::string& err) {
  ProfScope prof_(c, "mse");
  if (cudaMemsetAsync(loss, 0, sizeof(float) * B, c->stream) != cudaSuccess) return check_launch("mse memset", err);
  dim3 grid(16, (unsigned)B);
  launch_pdl(c, mse_kernel, grid, 256, 0, vel, target, weight, per, 1.0f / (float)per, grad_scale, loss, dvel);
  return check_launch("mse", err);
}

int k_pad_f16(Ctx* c, const float* src, long rows, int w, __half* dst, long ld, std::string& err) {
  ProfScope prof_(c, "pad_f16");
  launch_pdl(c, pad_f16_kernel, gs(rows * ld), 256, 0, src, rows, w, dst, ld);
  return check_launch("pad_f16", err);
}

int k_add_local(Ctx* c, const float* y, const float* le, int B, int S, int mem, int D, float* dst, std::string& err) {
  ProfScope prof_(c, "add_local");
  launch_pdl(c, add_local_kernel, gs((long)B * S * D), 256, 0, y, le, (long)B * S, S, mem, D, dst);
  return check_launch("add_local", err);
}

int k_scale(Ctx* c, float* x, long n, float s, std::string& err) {
  ProfScope prof_(c, "scale");
  if (n <= 0) return 0;
  const long n4 = (reinterpret_cast<uintptr_t>(x) & 15) == 0 ? n / 4 : 0;
  if (n4 > 0) {
    const long blocks = std::min<long>((n4 + 255) / 256, (long)c->sm_count * 8);
    launch_pdl(c, scale_kernel, (unsigned)blocks, 256, 0, reinterpret_cast<float4*>(x), n4, s);
  }
  if (4 * n4 < n) launch_pdl(c, scale_tail_kernel, 1, 256, 0, x, 4 * n4, n, s);
  return check_launch("scale", err);
}

int k_copy_rows(Ctx* c, const float* src, int src_rows_per, int src_off, float* dst, __half* dst_h,
                int dst_rows_per, int dst_off, int B, int rows, int D, std::string& err) {
  ProfScope prof_(c, "copy_rows");
  const auto al16 = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15) == 0; };
  if (D % 4 == 0 && al16(src) && (!dst || al16(dst)) && (!dst_h || (reinterpret_cast<uintptr_t>(dst_h) & 7) == 0) &&
      B > 0 && rows > 0) {
    const long nrows = (long)B * rows;
    const dim3 grid((unsigned)((D / 4 + 255) / 256), (unsigned)(nrows < 65535 ? nrows : 65535));
    launch_pdl(c, copy_rows4_kernel, grid, 256, 0, src, src_rows_per, src_off, dst, dst_h, dst_rows_per, dst_off, B,
               rows, D);
    return check_launch("copy_rows", err);
  }
  launch_pdl(c, copy_rows_kernel, gs((long)B * rows * D), 256, 0, src, src_rows_per, src_off, dst, dst_h, dst_rows_per,
                                                                  dst_off, B, rows, D);
  return check_launch("copy_rows", err);
}

}  // namespace sa3k
