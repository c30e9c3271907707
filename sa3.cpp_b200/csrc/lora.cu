// lora.cu -- the small, memory-bound kernels around the adapter GEMMs of dit_lin.
//
// dit_lin (src/dit.h:92-149) with a functional LoRA / DoRA-rows adapter computes
//   z = x W^T + s (x A^T) B^T,   y = g * z + bias,   g = m / sqrt(nsq),
//   nsq = bns + 2 s t2 + s^2 t3,  t2 = rowsum((W A^T) * B),  t3 = rowsum((B A A^T) * B)
// and ggml differentiates it (src/train_ckpt.h:400).  The contractions run on the tcgen05 GEMM
// engine; these kernels do the rank-16 bookkeeping in between: operand packing to f16, A A^T,
// the DoRA norm, the backward prologue dz = g * dy with dg = colsum(dy * z), and the DoRA
// backward terms for dA, dB and dm.  Ranks up to 16 are padded to 16 (zero rows / columns).
#include "sa3k_common.cuh"
#include "sa3k_internal.h"
#include "lora_kernels.h"

#include <algorithm>

namespace sa3k {

constexpr int R = 16;   // padded rank

__global__ void cvt_f16_kernel(const float* __restrict__ src, int64_t n, __half* __restrict__ dst) {
  pdl_prologue();
  const int64_t n4 = n / 4;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += stride) {
    const float4 v = reinterpret_cast<const float4*>(src)[i];
    uint2 o;
    o.x = pack_f16x2(v.x, v.y);
    o.y = pack_f16x2(v.z, v.w);
    reinterpret_cast<uint2*>(dst)[i] = o;
  }
  for (int64_t i = n4 * 4 + (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride)
    dst[i] = __float2half_rn(src[i]);
}

// Adapter operand forms.  A f32 [rank][in], B f32 [out][rank].
//   a_h  f16 [16][in]    (rows >= rank zero)      B operand of u = x A^T, A operand of W A^T
//   at_x  f16 [in][64]    A^T in columns 0..15     K-extension B operand of dx
//   b_x   f16 [out][64]   s B in columns 0..15     K-extension B operand of y
//   bt_h f16 [16][out]   B^T                      B operand of du = dz B
__global__ void prep_adapter_kernel(const float* __restrict__ A, const float* __restrict__ B, int rank, float s,
                                    int64_t in, int64_t out, __half* __restrict__ a_h,
                                    __half* __restrict__ at_x, __half* __restrict__ b_x,
                                    __half* __restrict__ bt_h) {
  pdl_prologue();
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  const int64_t t0 = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  for (int64_t k = t0; k < in * 64; k += stride) {
    const int64_t i = k / 64;
    const int c = (int)(k % 64);
    const float a = (c < rank) ? A[(int64_t)c * in + i] : 0.f;
    at_x[k] = __float2half_rn(a);
    if (c < R) a_h[(int64_t)c * in + i] = __float2half_rn(a);
  }
  for (int64_t k = t0; k < out * 64; k += stride) {
    const int64_t o = k / 64;
    const int c = (int)(k % 64);
    const float b = (c < rank) ? B[o * rank + c] : 0.f;
    b_x[k] = __float2half_rn(s * b);
    if (c < R) bt_h[(int64_t)c * out + o] = __float2half_rn(b);
  }
}

// AAt[r1][r2] = sum_i A[r1][i] A[r2][i] (f32 accumulate).  Block r1 of 16; each of its 256
// threads sums a strided slice of `in` for all 16 r2, then the block reduces.
__global__ void aat_kernel(const float* __restrict__ A, int rank, int64_t in, float* __restrict__ aat) {
  pdl_prologue();
  const int r1 = blockIdx.x;
  float acc[R];
#pragma unroll
  for (int r = 0; r < R; ++r) acc[r] = 0.f;
  if (r1 < rank) {
    for (int64_t i = threadIdx.x; i < in; i += blockDim.x) {
      const float a1 = A[(int64_t)r1 * in + i];
#pragma unroll
      for (int r = 0; r < R; ++r) acc[r] = r < rank ? fmaf(a1, A[(int64_t)r * in + i], acc[r]) : 0.f;
    }
  }
  __shared__ float part[8][R];
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const float v = warp_sum(acc[r]);
    if (lane == 0) part[wid][r] = v;
  }
  __syncthreads();
  if (threadIdx.x < R) {
    float v = 0.f;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) v += part[w][threadIdx.x];
    aat[r1 * R + threadIdx.x] = v;
  }
}

// DoRA-rows norm per output row o (src/dit.h:126-144):
//   t2 = sum_r P[o][r] B[o][r]   (P = W A^T, given transposed as pt[16][out])
//   t3 = sum_r (B AAt)[o][r] B[o][r]
//   nsq = bns + 2 s t2 + s^2 t3 ;  g = m / sqrt(nsq)
__global__ void dora_norm_kernel(const float* __restrict__ pt, const float* __restrict__ B, int rank,
                                 int64_t out, const float* __restrict__ aat, const float* __restrict__ bns,
                                 const float* __restrict__ m, float s, float* __restrict__ nsq,
                                 float* __restrict__ g) {
  pdl_prologue();
  __shared__ float saat[R * R];
  saat[threadIdx.x % (R * R)] = aat[threadIdx.x % (R * R)];
  __syncthreads();
  const int64_t o = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (o >= out) return;
  float b[R];
#pragma unroll
  for (int r = 0; r < R; ++r) b[r] = r < rank ? B[o * rank + r] : 0.f;
  float t2 = 0.f, t3 = 0.f;
#pragma unroll
  for (int r = 0; r < R; ++r) {
    t2 = fmaf(pt[(int64_t)r * out + o], b[r], t2);
    float bar = 0.f;
#pragma unroll
    for (int k = 0; k < R; ++k) bar = fmaf(b[k], saat[k * R + r], bar);
    t3 = fmaf(bar, b[r], t3);
  }
  const float n2 = bns[o] + 2.f * s * t2 + s * s * t3;
  nsq[o] = n2;
  g[o] = m[o] / sqrtf(n2);
}

// ---------------------------------------------------------------- producers fused with the prologue
// The upstream gradient dy of an adapted linear is produced here and never stored in f32: the
// kernels write dz = f16(g * dy) (f16(dy) without DoRA) and add colsum(dy * z) into dg, with
// z = (y - bias) / g the pre-scale output of the forward.  Thread = 4 columns, block = kFuseTok
// rows (one f32 atomic per column and block).
constexpr int kFuseTok = 32;
constexpr int kGateRows = 16;

__device__ __forceinline__ void dz_store4(__half* dz, const float (&dy)[4], const float (&gv)[4], bool dora) {
  uint2 pk;
  pk.x = pack_f16x2(dora ? dy[0] * gv[0] : dy[0], dora ? dy[1] * gv[1] : dy[1]);
  pk.y = pack_f16x2(dora ? dy[2] * gv[2] : dy[2], dora ? dy[3] * gv[3] : dy[3]);
  *reinterpret_cast<uint2*>(dz) = pk;
}

// dy = gx * gate[sample] (the gate backward of src/dit.h:186-193).  Block (128, 4): thread x owns
// 4 columns, thread y four consecutive rows of each kGateRows-row chunk the block visits (loads
// first); dg is summed over y in shared memory before one atomic per column.
__global__ void __launch_bounds__(512) gate_bwd_dz_kernel(const float* __restrict__ gx, const float* __restrict__ gate,
                                                          long gstride, int T, int D, int tps,
                                                          const float* __restrict__ y, const float* __restrict__ bias,
                                                          const float* __restrict__ g, __half* __restrict__ dz,
                                                          float* __restrict__ dg) {
  pdl_prologue();
  __shared__ float4 red[4][128];
  const int c0 = 4 * (blockIdx.x * blockDim.x + threadIdx.x);
  const bool col_ok = c0 < D;
  const bool dora = g != nullptr;
  float gv[4] = {1.f, 1.f, 1.f, 1.f}, inv[4] = {1.f, 1.f, 1.f, 1.f}, bv[4] = {0.f, 0.f, 0.f, 0.f};
  if (dora && col_ok) {
    const float4 g4 = *reinterpret_cast<const float4*>(g + c0);
    gv[0] = g4.x; gv[1] = g4.y; gv[2] = g4.z; gv[3] = g4.w;
#pragma unroll
    for (int e = 0; e < 4; ++e) inv[e] = 1.f / gv[e];
    if (bias) {
      const float4 b4 = *reinterpret_cast<const float4*>(bias + c0);
      bv[0] = b4.x; bv[1] = b4.y; bv[2] = b4.z; bv[3] = b4.w;
    }
  }
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  // grid-stride over chunks of kGateRows rows (thread y: four consecutive rows of a chunk), so a
  // grid of about two blocks per SM covers any T with one dg atomic per column and block
  const int nchunk = (T + kGateRows - 1) / kGateRows;
  for (int ch = blockIdx.y; ch < nchunk && col_ok; ch += gridDim.y) {
    const int tb = ch * kGateRows + 4 * threadIdx.y, t1 = min(T, tb + 4);
    if (tb >= t1) continue;
    float4 gt[4], av[4], yv[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int t = min(tb + u, t1 - 1);          // rows past the end repeat the last (not stored)
      const long e = (long)t * D + c0;
      gt[u] = *reinterpret_cast<const float4*>(gate + (long)(t / tps) * gstride + c0);
      av[u] = *reinterpret_cast<const float4*>(gx + e);
      if (dora) yv[u] = *reinterpret_cast<const float4*>(y + e);
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      if (tb + u >= t1) break;
      const long e = (long)(tb + u) * D + c0;
      const float dy[4] = {av[u].x * gt[u].x, av[u].y * gt[u].y, av[u].z * gt[u].z, av[u].w * gt[u].w};
      dz_store4(dz + e, dy, gv, dora);
      if (dora) {
        acc[0] = fmaf(dy[0], (yv[u].x - bv[0]) * inv[0], acc[0]);
        acc[1] = fmaf(dy[1], (yv[u].y - bv[1]) * inv[1], acc[1]);
        acc[2] = fmaf(dy[2], (yv[u].z - bv[2]) * inv[2], acc[2]);
        acc[3] = fmaf(dy[3], (yv[u].w - bv[3]) * inv[3], acc[3]);
      }
    }
  }
  if (dora) {
    red[threadIdx.y][threadIdx.x] = make_float4(acc[0], acc[1], acc[2], acc[3]);
    __syncthreads();
    if (threadIdx.y == 0 && col_ok) {
      float4 sum = red[0][threadIdx.x];
#pragma unroll
      for (int q = 1; q < 4; ++q) {
        const float4 v = red[q][threadIdx.x];
        sum.x += v.x; sum.y += v.y; sum.z += v.z; sum.w += v.w;
      }
      atomicAdd(dg + c0, sum.x);
      atomicAdd(dg + c0 + 1, sum.y);
      atomicAdd(dg + c0 + 2, sum.z);
      atomicAdd(dg + c0 + 3, sum.w);
    }
  }
}

// SwiGLU backward (src/dit.h:259-264): f[t] = [val | gate] is the ff.proj output (f16), da (f16)
// the gradient of val * silu(gate); dy = [d val | d gate] is the ff.proj output gradient (2I
// columns).  Thread = 8 columns of val and the matching 8 of gate (16-byte loads and stores);
// the blocks walk chunks of kSwiRows rows grid-stride (every row's loads of a chunk issued
// first), with a grid of kSwiBlocks blocks per SM, so no partial last wave is left; dz = f16(g dy)
// and, for DoRA, dg += colsum(dy (y - bias) / g) with the reciprocals of g taken once per thread.
constexpr int kSwiRows = 4;
constexpr int kSwiBlocks = 3;

__device__ __forceinline__ void f16x8(const uint4 w, float (&v)[8]) {
  const uint32_t u[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&u[k]));
    v[2 * k] = a.x;
    v[2 * k + 1] = a.y;
  }
}

__device__ __forceinline__ void f32x8(const float* p, float (&v)[8]) {
  const float4 a = reinterpret_cast<const float4*>(p)[0], b = reinterpret_cast<const float4*>(p)[1];
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}

__device__ __forceinline__ uint4 f16x8_pack(const float (&v)[8]) {
  return make_uint4(pack_f16x2(v[0], v[1]), pack_f16x2(v[2], v[3]), pack_f16x2(v[4], v[5]), pack_f16x2(v[6], v[7]));
}

__global__ void __launch_bounds__(128, kSwiBlocks)
    swiglu_bwd_dz_kernel(const __half* __restrict__ da, const __half* __restrict__ f, int T, int I,
                         const float* __restrict__ bias, const float* __restrict__ g, __half* __restrict__ dz,
                         float* __restrict__ dg) {
  pdl_prologue();
  const int j = 8 * (blockIdx.x * blockDim.x + threadIdx.x);
  if (j >= I) return;
  const bool dora = g != nullptr;
  float gv[8], gg[8], igv[8], igg[8], bv[8], bg[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) gv[e] = gg[e] = igv[e] = igg[e] = 1.f, bv[e] = bg[e] = 0.f;
  if (dora) {
    f32x8(g + j, gv);
    f32x8(g + I + j, gg);
#pragma unroll
    for (int e = 0; e < 8; ++e) igv[e] = 1.f / gv[e], igg[e] = 1.f / gg[e];
    if (bias) {
      f32x8(bias + j, bv);
      f32x8(bias + I + j, bg);
    }
  }
  float accv[8], accg[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) accv[e] = accg[e] = 0.f;
  for (int tb = blockIdx.y * kSwiRows; tb < T; tb += gridDim.y * kSwiRows) {
    const int t1 = min(T, tb + kSwiRows);
    uint4 v4[kSwiRows], g4[kSwiRows], d4[kSwiRows];
#pragma unroll
    for (int u = 0; u < kSwiRows; ++u) {             // every row's loads first
      const int t = min(tb + u, t1 - 1);
      const __half* fr = f + (long)t * 2 * I;
      v4[u] = *reinterpret_cast<const uint4*>(fr + j);
      g4[u] = *reinterpret_cast<const uint4*>(fr + I + j);
      d4[u] = *reinterpret_cast<const uint4*>(da + (long)t * I + j);
    }
#pragma unroll
    for (int u = 0; u < kSwiRows; ++u) {
      const int t = tb + u;
      if (t >= t1) break;
      float vv[8], ga[8], dd[8], dv[8], dgl[8];
      f16x8(v4[u], vv);
      f16x8(g4[u], ga);
      f16x8(d4[u], dd);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const float sg = __fdividef(1.f, 1.f + __expf(-ga[e]));
        dv[e] = dd[e] * ga[e] * sg;
        dgl[e] = dd[e] * vv[e] * sg * (1.f + ga[e] * (1.f - sg));
        if (dora) {
          accv[e] = fmaf(dv[e], (vv[e] - bv[e]) * igv[e], accv[e]);
          accg[e] = fmaf(dgl[e], (ga[e] - bg[e]) * igg[e], accg[e]);
          dv[e] *= gv[e];
          dgl[e] *= gg[e];
        }
      }
      __half* zr = dz + (long)t * 2 * I;
      *reinterpret_cast<uint4*>(zr + j) = f16x8_pack(dv);
      *reinterpret_cast<uint4*>(zr + I + j) = f16x8_pack(dgl);
    }
  }
  if (dora) {
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      atomicAdd(dg + j + e, accv[e]);
      atomicAdd(dg + I + j + e, accg[e]);
    }
  }
}

// ---------------------------------------------------------------- grouped adapter preparation
// The same three preparations for every adapter of a model in one launch each (grid.y = adapter),
// driven by a device array of PrepDesc built once when the adapters are bound.
__global__ void prep_all_kernel(const PrepDesc* __restrict__ descs) {
  pdl_prologue();
  const PrepDesc d = descs[blockIdx.y];
  const int stride = gridDim.x * blockDim.x;
  const int t0 = blockIdx.x * blockDim.x + threadIdx.x;
  const int nin = (int)d.in * 64, nout = (int)d.out * 64;
  // each output walked in its own row-major order, so every store is coalesced: at_x [in][64] and
  // b_x [out][64] along the padded rank (the A reads of at_x stride through A, which stays in
  // cache), a_h [16][in] and bt_h [16][out] along in / out
  for (int k = t0; k < nin; k += stride) {
    const int i = k >> 6, c = k & 63;
    d.at_x[k] = __float2half_rn((c < d.rank) ? d.A[(int64_t)c * d.in + i] : 0.f);
  }
  for (int k = t0; k < R * (int)d.in; k += stride) {
    const int c = k / (int)d.in;
    d.a_h[k] = __float2half_rn((c < d.rank) ? d.A[k] : 0.f);
  }
  for (int k = t0; k < nout; k += stride) {
    const int o = k >> 6, c = k & 63;
    d.b_x[k] = __float2half_rn((c < d.rank) ? d.s * d.B[(int64_t)o * d.rank + c] : 0.f);
  }
  for (int k = t0; k < R * (int)d.out; k += stride) {
    const int c = k / (int)d.out, o = k - c * (int)d.out;
    d.bt_h[k] = __float2half_rn((c < d.rank) ? d.B[(int64_t)o * d.rank + c] : 0.f);
  }
}

__global__ void aat_all_kernel(const PrepDesc* __restrict__ descs) {
  pdl_prologue();
  const PrepDesc d = descs[blockIdx.y];
  if (!d.dora) return;
  const int r1 = blockIdx.x;
  float acc[R];
#pragma unroll
  for (int r = 0; r < R; ++r) acc[r] = 0.f;
  if (r1 < d.rank) {
    for (int64_t i = threadIdx.x; i < d.in; i += blockDim.x) {
      const float a1 = d.A[(int64_t)r1 * d.in + i];
#pragma unroll
      for (int r = 0; r < R; ++r) acc[r] = r < d.rank ? fmaf(a1, d.A[(int64_t)r * d.in + i], acc[r]) : 0.f;
    }
  }
  __shared__ float part[8][R];
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const float v = warp_sum(acc[r]);
    if (lane == 0) part[wid][r] = v;
  }
  __syncthreads();
  if (threadIdx.x < R) {
    float v = 0.f;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) v += part[w][threadIdx.x];
    d.aat[r1 * R + threadIdx.x] = v;
  }
}

__global__ void dora_norm_all_kernel(const PrepDesc* __restrict__ descs) {
  pdl_prologue();
  const PrepDesc d = descs[blockIdx.y];
  if (!d.dora) return;
  __shared__ float saat[R * R];
  saat[threadIdx.x % (R * R)] = d.aat[threadIdx.x % (R * R)];
  __syncthreads();
  const int64_t o = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (o >= d.out) return;
  float b[R];
#pragma unroll
  for (int r = 0; r < R; ++r) b[r] = r < d.rank ? d.B[o * d.rank + r] : 0.f;
  float t2 = 0.f, t3 = 0.f;
#pragma unroll
  for (int r = 0; r < R; ++r) {
    t2 = fmaf(d.pt[(int64_t)r * d.out + o], b[r], t2);
    float bar = 0.f;
#pragma unroll
    for (int k = 0; k < R; ++k) bar = fmaf(b[k], saat[k * R + r], bar);
    t3 = fmaf(bar, b[r], t3);
  }
  const float n2 = d.bns[o] + 2.f * d.s * t2 + d.s * d.s * t3;
  d.nsq[o] = n2;
  d.g[o] = d.m[o] / sqrtf(n2);
}

// Backward prologue over dy[S][out] (one thread per column, TOK rows per block):
//   dz = f16(g * dy) ;  dg[o] += sum_t dy[t][o] * (y[t][o] - bias[o]) / g[o]   (dora only)
// With g == null this is the plain f32 -> f16 conversion of dy.
constexpr int kProTok = 32;
__global__ void bwd_prologue_kernel(const float* __restrict__ dy, const float* __restrict__ y,
                                    const float* __restrict__ bias, const float* __restrict__ g,
                                    int64_t S, int64_t out, __half* __restrict__ dz,
                                    float* __restrict__ dg) {
  pdl_prologue();
  const int64_t o = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (o >= out) return;
  const int64_t t0 = (int64_t)blockIdx.y * kProTok;
  const int64_t t1 = t0 + kProTok < S ? t0 + kProTok : S;
  if (!g) {
    for (int64_t t = t0; t < t1; ++t) dz[t * out + o] = __float2half_rn(dy[t * out + o]);
    return;
  }
  const float go = g[o], bo = bias ? bias[o] : 0.f, inv = 1.f / go;
  float acc = 0.f;
  for (int64_t t = t0; t < t1; ++t) {
    const float d = dy[t * out + o];
    dz[t * out + o] = __float2half_rn(d * go);
    acc = fmaf(d, (y[t * out + o] - bo) * inv, acc);
  }
  atomicAdd(dg + o, acc);
}

// DoRA backward per output row o (the derivative of the norm expression above):
//   dm  = dg / sqrt(nsq)                      dnsq = -0.5 dg g / nsq
//   dt2 = 2 s dnsq, dt3 = s^2 dnsq
//   dB[o][r] += dt2 P[o][r] + 2 dt3 (B AAt)[o][r]
//   cb[r][o] = f16(dt2 B[o][r])   (A operand of dA += cb W, a rank-16 quant GEMM)
//   c3[r][k] += dt3 B[o][r] B[o][k]           (dA += 2 c3 A afterwards)
// 128 rows per block.  Phase 1: one thread per row (dm, dB, cb; the row's dt3 B[o][:] and B[o][:]
// go to shared memory).  Phase 2: thread (r, k), r <= k < R, sums dt3 B[o][r] B[o][k] over the
// block's rows and adds it to c3 (one atomic per entry and block).
constexpr int kDoraRows = 128;
__device__ __forceinline__ void dora_bwd_rows(int blk, const float* __restrict__ pt, const float* __restrict__ B,
                                              int rank, int64_t out, const float* __restrict__ aat,
                                              const float* __restrict__ nsq, const float* __restrict__ g,
                                              const float* __restrict__ dg, float s, float* __restrict__ dm,
                                              int dm_accumulate, float* __restrict__ dB,
                                              __half* __restrict__ cb, float* __restrict__ c3) {
  __shared__ float saat[R * R];
  __shared__ float sb[kDoraRows][R + 1];    // B[o][:]          (+1: no bank conflicts on columns)
  __shared__ float sbt[kDoraRows][R + 1];   // dt3[o] B[o][:]
  for (int e = threadIdx.x; e < R * R; e += blockDim.x) saat[e] = aat[e];
  __syncthreads();
  const int row = threadIdx.x;
  const int64_t o = (int64_t)blk * kDoraRows + row;
  float b[R];
  float dt3 = 0.f;
#pragma unroll
  for (int r = 0; r < R; ++r) b[r] = 0.f;
  if (o < out) {
#pragma unroll
    for (int r = 0; r < R; ++r) b[r] = r < rank ? B[o * rank + r] : 0.f;
    const float n2 = nsq[o], d = dg[o];
    const float dmo = d / sqrtf(n2);
    if (dm) dm[o] = dm_accumulate ? dm[o] + dmo : dmo;
    const float dn = -0.5f * d * g[o] / n2;
    const float dt2 = 2.f * s * dn;
    dt3 = s * s * dn;
#pragma unroll
    for (int r = 0; r < R; ++r) {
      float bar = 0.f;
#pragma unroll
      for (int k = 0; k < R; ++k) bar = fmaf(b[k], saat[k * R + r], bar);
      if (r < rank) dB[o * rank + r] += dt2 * pt[(int64_t)r * out + o] + 2.f * dt3 * bar;
      cb[(int64_t)r * out + o] = __float2half_rn(dt2 * b[r]);
    }
  }
#pragma unroll
  for (int r = 0; r < R; ++r) {
    sb[row][r] = b[r];
    sbt[row][r] = dt3 * b[r];
  }
  __syncthreads();
  // 136 (r <= k) entries of the symmetric R x R block sum
  const int nrows = (int)min((int64_t)kDoraRows, out - (int64_t)blk * kDoraRows);
  for (int e = threadIdx.x; e < R * (R + 1) / 2; e += blockDim.x) {
    int r = 0, rem = e;
    while (rem >= R - r) { rem -= R - r; ++r; }
    const int k = r + rem;
    if (r >= rank || k >= rank) continue;
    float acc = 0.f;
    for (int q = 0; q < nrows; ++q) acc = fmaf(sbt[q][r], sb[q][k], acc);
    atomicAdd(c3 + r * R + k, acc);
    if (k != r) atomicAdd(c3 + k * R + r, acc);
  }
}

__global__ void __launch_bounds__(kDoraRows) dora_bwd_kernel(
    const float* __restrict__ pt, const float* __restrict__ B, int rank, int64_t out, const float* __restrict__ aat,
    const float* __restrict__ nsq, const float* __restrict__ g, const float* __restrict__ dg, float s,
    float* __restrict__ dm, int dm_accumulate, float* __restrict__ dB, __half* __restrict__ cb,
    float* __restrict__ c3) {
  pdl_prologue();
  dora_bwd_rows(blockIdx.x, pt, B, rank, out, aat, nsq, g, dg, s, dm, dm_accumulate, dB, cb, c3);
}

// All DoRA adapters of a group at once: blockIdx.y = adapter, blockIdx.x = 128-row block of its
// output rows (blocks past an adapter's rows return at once).  dm, dB accumulate.
__global__ void __launch_bounds__(kDoraRows) dora_bwd_all_kernel(const PrepDesc* __restrict__ descs) {
  pdl_prologue();
  const PrepDesc& d = descs[blockIdx.y];
  if (!d.dora || (int64_t)blockIdx.x * kDoraRows >= d.out) return;
  dora_bwd_rows(blockIdx.x, d.pt, d.B, d.rank, d.out, d.aat, d.nsq, d.g, d.dg, d.s, d.dm, 1, d.dB, d.cb, d.c3);
}

// dA[r][i] += 2 sum_q c3[r][q] A[q][i] for all DoRA adapters: blockIdx.y = adapter, 256 (r, i)
// entries per block.
__global__ void dora_da_c3_all_kernel(const PrepDesc* __restrict__ descs) {
  pdl_prologue();
  const PrepDesc& d = descs[blockIdx.y];
  if (!d.dora) return;
  __shared__ float s3[R * R];
  if (threadIdx.x < R * R) s3[threadIdx.x] = d.c3[threadIdx.x];
  __syncthreads();
  const int64_t n = (int64_t)d.rank * d.in;
  for (int64_t k = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; k < n; k += (int64_t)gridDim.x * blockDim.x) {
    const int r = (int)(k / d.in);
    const int64_t i = k % d.in;
    float acc = 0.f;
    for (int q = 0; q < d.rank; ++q) acc = fmaf(s3[r * R + q], d.A[(int64_t)q * d.in + i], acc);
    d.dA[k] += 2.f * acc;
  }
}

// dA[r][i] += 2 sum_k c3[r][k] A[k][i]
__global__ void dora_da_c3_kernel(const float* __restrict__ c3, const float* __restrict__ A, int rank,
                                  int64_t in, float* __restrict__ dA) {
  pdl_prologue();
  __shared__ float s3[R * R];
  if (threadIdx.x < R * R) s3[threadIdx.x] = c3[threadIdx.x];
  __syncthreads();
  const int64_t k = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (k >= (int64_t)rank * in) return;
  const int r = (int)(k / in);
  const int64_t i = k % in;
  float acc = 0.f;
  for (int q = 0; q < rank; ++q) acc = fmaf(s3[r * R + q], A[(int64_t)q * in + i], acc);
  dA[k] += 2.f * acc;
}

// ----------------------------------------------------------------------------- launchers
static unsigned grid1d(int64_t n, int threads, int cap = 148 * 16) {
  int64_t b = (n + threads - 1) / threads;
  if (b > cap) b = cap;
  return (unsigned)(b < 1 ? 1 : b);
}

int k_cvt_f16(Ctx* c, const float* src, int64_t n, __half* dst, std::string& err) {
  ProfScope prof_(c, "cvt_f16");
  launch_pdl(c, cvt_f16_kernel, grid1d(n / 4 + 1, 256), 256, 0, src, n, dst);
  return check_launch("cvt_f16", err);
}

int k_prep_adapter(Ctx* c, const float* A, const float* B, int rank, float s, int64_t in, int64_t out,
                   __half* a_h, __half* at_x, __half* b_x, __half* bt_h,
                   std::string& err) {
  ProfScope prof_(c, "prep_adapter");
  launch_pdl(c, prep_adapter_kernel, grid1d((in + out) * 64, 256), 256, 0, A, B, rank, s, in, out, a_h, at_x, b_x,
                                                                             bt_h);
  return check_launch("prep_adapter", err);
}

int k_aat(Ctx* c, const float* A, int rank, int64_t in, float* aat, std::string& err) {
  ProfScope prof_(c, "aat");
  launch_pdl(c, aat_kernel, R, 256, 0, A, rank, in, aat);
  return check_launch("aat", err);
}

int k_dora_norm(Ctx* c, const float* pt, const float* B, int rank, int64_t out, const float* aat,
                const float* bns, const float* m, float s, float* nsq, float* g, std::string& err) {
  ProfScope prof_(c, "dora_norm");
  launch_pdl(c, dora_norm_kernel, (unsigned)((out + 255) / 256), 256, 0, pt, B, rank, out, aat, bns, m, s, nsq, g);
  return check_launch("dora_norm", err);
}

int k_bwd_prologue(Ctx* c, const float* dy, const float* y, const float* bias, const float* g, int64_t S,
                   int64_t out, __half* dz, float* dg, std::string& err) {
  ProfScope prof_(c, "bwd_prologue");
  dim3 grid((unsigned)((out + 255) / 256), (unsigned)((S + kProTok - 1) / kProTok));
  launch_pdl(c, bwd_prologue_kernel, grid, 256, 0, dy, y, bias, g, S, out, dz, dg);
  return check_launch("bwd_prologue", err);
}

int k_dora_bwd(Ctx* c, const float* pt, const float* B, int rank, int64_t out, const float* aat,
               const float* nsq, const float* g, const float* dg, float s, float* dm, int dm_acc,
               float* dB, __half* cb, float* c3, std::string& err) {
  ProfScope prof_(c, "dora_bwd");
  launch_pdl(c, dora_bwd_kernel, (unsigned)((out + kDoraRows - 1) / kDoraRows), kDoraRows, 0, 
      pt, B, rank, out, aat, nsq, g, dg, s, dm, dm_acc, dB, cb, c3);
  return check_launch("dora_bwd", err);
}

int k_gate_bwd_dz(Ctx* c, const float* gx, const float* gate, long gstride, int T, int D, int tps, const float* y,
                  const float* bias, const float* g, __half* dz, float* dg, std::string& err) {
  if (D % 4) { err = "gate: the width must be a multiple of 4"; return 1; }
  const unsigned gx_blocks = (unsigned)((D / 4 + 127) / 128), nchunk = (unsigned)((T + kGateRows - 1) / kGateRows);
  const unsigned gy = std::max(1u, std::min(nchunk, (unsigned)(2 * c->sm_count) / gx_blocks));
  if (g && cudaMemsetAsync(dg, 0, sizeof(float) * D, c->stream) != cudaSuccess) return check_launch("memset", err);
  ProfScope prof_(c, "gate_bwd_dz");
  launch_pdl(c, gate_bwd_dz_kernel, dim3(gx_blocks, gy), dim3(128, 4), 0, gx, gate, gstride, T, D, tps, y, bias, g, dz,
             dg);
  return check_launch("gate_bwd_dz", err);
}

int k_swiglu_bwd_dz(Ctx* c, const __half* da, const __half* f, int T, int I, const float* bias,
                    const float* g,
                    __half* dz, float* dg, std::string& err) {
  if (I % 8) { err = "swiglu: the hidden width must be a multiple of 8"; return 1; }
  if (g && cudaMemsetAsync(dg, 0, sizeof(float) * 2 * I, c->stream) != cudaSuccess) return check_launch("memset", err);
  ProfScope prof_(c, "swiglu_bwd_dz");
  const unsigned gx = (unsigned)((I / 8 + 127) / 128), nchunk = (unsigned)((T + kSwiRows - 1) / kSwiRows);
  const unsigned gy = std::max(1u, std::min(nchunk, (unsigned)(kSwiBlocks * c->sm_count) / gx));
  launch_pdl(c, swiglu_bwd_dz_kernel, dim3(gx, gy), 128, 0, da, f, T, I, bias, g, dz, dg);
  return check_launch("swiglu_bwd_dz", err);
}

int k_prep_all(Ctx* c, const PrepDesc* descs, int n, std::string& err) {
  ProfScope prof_(c, "prep_adapter");
  launch_pdl(c, prep_all_kernel, dim3(48, (unsigned)n), 256, 0, descs);
  return check_launch("prep_all", err);
}

int k_aat_all(Ctx* c, const PrepDesc* descs, int n, std::string& err) {
  ProfScope prof_(c, "aat");
  launch_pdl(c, aat_all_kernel, dim3(R, (unsigned)n), 256, 0, descs);
  return check_launch("aat_all", err);
}

int k_dora_norm_all(Ctx* c, const PrepDesc* descs, int n, int64_t max_out, std::string& err) {
  ProfScope prof_(c, "dora_norm");
  launch_pdl(c, dora_norm_all_kernel, dim3((unsigned)((max_out + 255) / 256), (unsigned)n), 256, 0, descs);
  return check_launch("dora_norm_all", err);
}

int k_dora_bwd_all(Ctx* c, const PrepDesc* descs, int n, int64_t max_out, std::string& err) {
  ProfScope prof_(c, "dora_bwd");
  launch_pdl(c, dora_bwd_all_kernel, dim3((unsigned)((max_out + kDoraRows - 1) / kDoraRows), (unsigned)n), kDoraRows, 0, descs);
  return check_launch("dora_bwd_all", err);
}

int k_dora_da_c3_all(Ctx* c, const PrepDesc* descs, int n, std::string& err) {
  ProfScope prof_(c, "dora_da_c3");
  launch_pdl(c, dora_da_c3_all_kernel, dim3(64, (unsigned)n), 256, 0, descs);
  return check_launch("dora_da_c3_all", err);
}

int k_dora_da_c3(Ctx* c, const float* c3, const float* A, int rank, int64_t in, float* dA, std::string& err) {
  ProfScope prof_(c, "dora_da_c3");
  launch_pdl(c, dora_da_c3_kernel, (unsigned)(((int64_t)rank * in + 255) / 256), 256, 0, c3, A, rank, in, dA);
  return check_launch("dora_da_c3", err);
}


// ---------------------------------------------------------------- rank-16 projections
// u^T = f16(alpha (X Bm^T))^T for an adapter of rank <= 16: X [M][K] f16 (row stride ldx), Bm
// [16][K] f16 (rows past the rank are zero), out [16][ldu] f16.  The forward's u = x A^T and the
// backward's du = s dz B have this shape.  16 outputs per row make it a pure stream of X (2 bytes
// per element against 32 FLOPs): the kernel is shaped for HBM, not for the tensor pipe (a
// 128-row tcgen05 tile gives a 4352-row X only 34 CTAs, which cannot pull HBM's rate).
// Block = 8 warps on 16 rows; each warp streams a contiguous eighth of the 32-wide k chunks,
// keeping the X loads of the next 4 chunks in flight while it multiplies the current 4, with
// warp-level m16n8k16 MMAs (two n-halves of the 16 outputs); the eight partial tiles are summed
// in shared memory.  Within a chunk the k order is permuted so that a lane reads its X row slice
// and its Bm slice as one 16-byte load each: lane (g, c) holds k 8c .. 8c + 7 of the chunk; the
// first MMA takes k 8c .. 8c + 3 as its fragment pairs (2c, 2c + 8), the second k 8c + 4 .. 8c + 7.
// X and Bm share the permutation, so the sum is unchanged.  Needs K % 32 == 0.
constexpr int kR16Warps = 8, kR16Unroll = 4;

__device__ __forceinline__ void mma_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                          uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__global__ void __launch_bounds__(32 * kR16Warps) r16_proj_kernel(const __half* __restrict__ x, long ldx, int M,
                                                                   int K, const __half* __restrict__ bm, float alpha,
                                                                   __half* __restrict__ ut, long ldu) {
  pdl_prologue();
  __shared__ float red[kR16Warps][16][17];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, c = lane & 3;
  const int m0 = blockIdx.x * 16;
  const long ra = min(m0 + g, M - 1), rb = min(m0 + g + 8, M - 1);   // clamped: stores are guarded
  const __half* xa = x + ra * ldx + 8 * c;
  const __half* xb = x + rb * ldx + 8 * c;
  const __half* ba = bm + (long)g * K + 8 * c;
  const __half* bb = bm + (long)(g + 8) * K + 8 * c;
  float d0[4] = {0.f, 0.f, 0.f, 0.f}, d1[4] = {0.f, 0.f, 0.f, 0.f};
  // warp w streams the contiguous chunk range [c_lo, c_hi): at any moment the warps of a block
  // read 8 different 512-byte row segments rather than one narrow column band of every row
  const int nch = K / 32, per = (nch + kR16Warps - 1) / kR16Warps;
  const int c_lo = warp * per, c_hi = min(nch, c_lo + per);
  // two register groups of kR16Unroll chunks: the next group's loads are in flight while the
  // current one is multiplied
  uint4 a0[kR16Unroll], b0[kR16Unroll], a1[kR16Unroll], b1[kR16Unroll];
  auto load = [&](uint4 (&va)[kR16Unroll], uint4 (&vb)[kR16Unroll], int ch0) {
#pragma unroll
    for (int u = 0; u < kR16Unroll; ++u) {
      const int ch = min(ch0 + u, c_hi - 1);
      va[u] = __ldcs(reinterpret_cast<const uint4*>(xa + 32 * ch));
      vb[u] = __ldcs(reinterpret_cast<const uint4*>(xb + 32 * ch));
    }
  };
  auto mul = [&](const uint4 (&va)[kR16Unroll], const uint4 (&vb)[kR16Unroll], int ch0) {
#pragma unroll
    for (int u = 0; u < kR16Unroll; ++u) {
      const int ch = ch0 + u;
      if (ch >= c_hi) break;
      const uint4 wa = __ldg(reinterpret_cast<const uint4*>(ba + 32 * ch));   // Bm: L1 / L2 resident
      const uint4 wb = __ldg(reinterpret_cast<const uint4*>(bb + 32 * ch));
      mma_16816(d0, va[u].x, vb[u].x, va[u].y, vb[u].y, wa.x, wa.y);
      mma_16816(d1, va[u].x, vb[u].x, va[u].y, vb[u].y, wb.x, wb.y);
      mma_16816(d0, va[u].z, vb[u].z, va[u].w, vb[u].w, wa.z, wa.w);
      mma_16816(d1, va[u].z, vb[u].z, va[u].w, vb[u].w, wb.z, wb.w);
    }
  };
  if (c_lo < c_hi) load(a0, b0, c_lo);
  for (int ch0 = c_lo; ch0 < c_hi; ch0 += 2 * kR16Unroll) {
    if (ch0 + kR16Unroll < c_hi) load(a1, b1, ch0 + kR16Unroll);
    mul(a0, b0, ch0);
    if (ch0 + kR16Unroll >= c_hi) break;
    if (ch0 + 2 * kR16Unroll < c_hi) load(a0, b0, ch0 + 2 * kR16Unroll);
    mul(a1, b1, ch0 + kR16Unroll);
  }
  // accumulator fragment: rows g, g + 8; outputs 2c, 2c + 1 (d0) and 8 + 2c, 8 + 2c + 1 (d1)
  red[warp][g][2 * c] = d0[0];
  red[warp][g][2 * c + 1] = d0[1];
  red[warp][g + 8][2 * c] = d0[2];
  red[warp][g + 8][2 * c + 1] = d0[3];
  red[warp][g][8 + 2 * c] = d1[0];
  red[warp][g][8 + 2 * c + 1] = d1[1];
  red[warp][g + 8][8 + 2 * c] = d1[2];
  red[warp][g + 8][8 + 2 * c + 1] = d1[3];
  __syncthreads();
#pragma unroll
  for (int i = threadIdx.x; i < 256; i += 32 * kR16Warps) {
    const int r = i >> 4, row = i & 15;
    float v = 0.f;
#pragma unroll
    for (int w = 0; w < kR16Warps; ++w) v += red[w][row][r];
    if (m0 + row < M) ut[(long)r * ldu + m0 + row] = __float2half_rn(alpha * v);
  }
}

int k_r16_proj(Ctx* c, const __half* x, long ldx, int64_t M, int64_t K, const __half* bm, float alpha, __half* ut,
               long ldu, const char* name, std::string& err) {
  if (M <= 0 || K <= 0 || K % 32 || ldx % 8 || (reinterpret_cast<uintptr_t>(x) & 15) ||
      (reinterpret_cast<uintptr_t>(bm) & 15)) {
    err = "rank-16 projection: K must be a positive multiple of 32 and the operands 16-byte aligned";
    return 1;
  }
  if ((M + 15) / 16 > 0x7fffffffL) { err = "rank-16 projection: too many rows"; return 1; }
  ProfScope prof_(c, name);
  launch_pdl(c, r16_proj_kernel, dim3((unsigned)((M + 15) / 16)), 32 * kR16Warps, 0, x, ldx, (int)M, (int)K, bm, alpha,
             ut, ldu);
  return check_launch("r16_proj", err);
}

}  // namespace sa3k
