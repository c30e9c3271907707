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

__global__ void rmsnorm_mod_fwd_kernel(const float* __restrict__ x, int T, int D, const float* __restrict__ gamma,
                                       const float* __restrict__ sc, const float* __restrict__ sh, long mod_stride,
                                       int tps, float eps, __nv_bfloat16* __restrict__ h, float* __restrict__ rstd) {
  pdl_prologue();
  const int row = blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
  if (row >= T) return;
  const int lane = threadIdx.x & 31;
  const float4* xr = reinterpret_cast<const float4*>(x + (long)row * D);
  float ss = 0.f;
  for (int i = lane; i < D / 4; i += 32) {
    const float4 v = xr[i];
    ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
  }
  ss = warp_sum(ss);
  const float r = rsqrtf(ss / (float)D + eps);
  if (lane == 0 && rstd) rstd[row] = r;
  const int s = row / tps;
  const float* scs = sc ? sc + (long)s * mod_stride : nullptr;
  const float* shs = sh ? sh + (long)s * mod_stride : nullptr;
  uint2* hr = reinterpret_cast<uint2*>(h + (long)row * D);
  for (int i = lane; i < D / 4; i += 32) {
    const float4 v = xr[i];
    const float4 gm = reinterpret_cast<const float4*>(gamma)[i];
    float o[4] = {v.x * r * gm.x, v.y * r * gm.y, v.z * r * gm.z, v.w * r * gm.w};
    if (scs) {
      const float4 a = reinterpret_cast<const float4*>(scs)[i];
      const float4 b = reinterpret_cast<const float4*>(shs)[i];
      o[0] = o[0] * (1.f + a.x) + b.x;
      o[1] = o[1] * (1.f + a.y) + b.y;
      o[2] = o[2] * (1.f + a.z) + b.z;
      o[3] = o[3] * (1.f + a.w) + b.w;
    }
    uint2 pk;
    pk.x = pack_bf16x2(o[0], o[1]);
    pk.y = pack_bf16x2(o[2], o[3]);
    hr[i] = pk;
  }
}

__global__ void rmsnorm_mod_bwd_kernel(const float* __restrict__ dh, const float* __restrict__ x,
                                       const float* __restrict__ rstd, int T, int D, const float* __restrict__ gamma,
                                       const float* __restrict__ sc, long mod_stride, int tps, float* __restrict__ gx) {
  pdl_prologue();
  const int row = blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
  if (row >= T) return;
  const int lane = threadIdx.x & 31;
  const float r = rstd[row];
  const int s = row / tps;
  const float* scs = sc ? sc + (long)s * mod_stride : nullptr;
  const float4* xr = reinterpret_cast<const float4*>(x + (long)row * D);
  const float4* dr = reinterpret_cast<const float4*>(dh + (long)row * D);
  float dot = 0.f;
  for (int i = lane; i < D / 4; i += 32) {
    const float4 v = xr[i], d = dr[i], gm = reinterpret_cast<const float4*>(gamma)[i];
    float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
    if (scs) a = reinterpret_cast<const float4*>(scs)[i];
    dot += d.x * gm.x * (1.f + a.x) * v.x + d.y * gm.y * (1.f + a.y) * v.y + d.z * gm.z * (1.f + a.z) * v.z +
           d.w * gm.w * (1.f + a.w) * v.w;
  }
  dot = warp_sum(dot) * r / (float)D;   // mean(dn * n)
  float4* gr = reinterpret_cast<float4*>(gx + (long)row * D);
  for (int i = lane; i < D / 4; i += 32) {
    const float4 v = xr[i], d = dr[i], gm = reinterpret_cast<const float4*>(gamma)[i];
    float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
    if (scs) a = reinterpret_cast<const float4*>(scs)[i];
    float4 gv = gr[i];
    gv.x += r * (d.x * gm.x * (1.f + a.x) - v.x * r * dot);
    gv.y += r * (d.y * gm.y * (1.f + a.y) - v.y * r * dot);
    gv.z += r * (d.z * gm.z * (1.f + a.z) - v.z * r * dot);
    gv.w += r * (d.w * gm.w * (1.f + a.w) - v.w * r * dot);
    gr[i] = gv;
  }
}

// RoPE angle of pair i (< rot/2) at position pos: pos * base^(-2i/rot); its (cos, sin) come from
// a table built once per (positions, rot, base) rather than from sincos in every warp.
__global__ void rope_table_kernel(int tps, int rot, float log2_base, float2* __restrict__ tab) {
  const int half = rot / 2;
  const int e = blockIdx.x * blockDim.x + threadIdx.x;
  if (e >= tps * half) return;
  const int pos = e / half, i = e % half;
  const float freq = exp2f(-2.0f * (float)i / (float)rot * log2_base);
  float sn, cs;
  sincosf((float)pos * freq, &sn, &cs);
  tab[e] = make_float2(cs, sn);
}

// One warp per (slice, head) and kHeadRows consecutive token rows; lane l holds head elements
// 2l and 2l + 1 (one 8-byte load and one 4-byte bf16x2 store per row).  All rows' loads are
// issued before any row is processed.  RoPE partners: rot 32 pairs (i, i + 16), i < 16, live in
// lanes l and l ^ 8 (lanes 0..15); rot 64 pairs (i, i + 32) in lanes l and l ^ 16.
struct HeadSlices {
  HeadSlice s[5];
  int n;
};
constexpr int kHeadRows = 8;

// cos / sin of the two NeoX pairs (e & (rot/2 - 1)) of head elements e = 2l, 2l + 1
__device__ __forceinline__ float4 rope_cs2(const float2* __restrict__ tab, int pos, int lane, int rot) {
  const int half = rot / 2;
  return *reinterpret_cast<const float4*>(tab + pos * half + ((2 * lane) & (half - 1)));
}

// Grid (ceil(H * nslices / 8), ceil(T / kHeadRows)); warp w of block x = (slice, head) pair 8 x + w.
__global__ void head_prep_fwd_kernel(const float* __restrict__ y, int T, int ncols, int H, const HeadSlices slices,
                                     int tps, float eps, int rot, const float2* __restrict__ tab,
                                     __nv_bfloat16* __restrict__ out) {
  pdl_prologue();
  const int nslices = slices.n;
  const int pair = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (pair >= H * nslices) return;
  const int lane = threadIdx.x & 31;
  const int si = pair % nslices, h = pair / nslices;
  const HeadSlice sl = slices.s[si];
  const int t0 = blockIdx.y * kHeadRows;
  const float2 gm = sl.gamma ? reinterpret_cast<const float2*>(sl.gamma)[lane] : make_float2(1.f, 1.f);
  float2 v[kHeadRows];
#pragma unroll
  for (int r = 0; r < kHeadRows; ++r)
    v[r] = t0 + r < T ? reinterpret_cast<const float2*>(y + (long)(t0 + r) * ncols + sl.col + h * 64)[lane]
                      : make_float2(0.f, 0.f);
#pragma unroll
  for (int r = 0; r < kHeadRows; ++r) {
    const int t = t0 + r;
    if (t >= T) break;
    float a = v[r].x, b = v[r].y;
    if (sl.gamma) {
      const float rr = rsqrtf(warp_sum(a * a + b * b) / 64.f + eps);
      if (lane == 0 && sl.rstd) sl.rstd[(long)t * H + h] = rr;
      a *= rr * gm.x;
      b *= rr * gm.y;
    }
    if (sl.rope && (rot == 32 || rot == 64)) {
      const int px = rot == 32 ? 8 : 16;
      const float pa = __shfl_xor_sync(0xffffffffu, a, px), pb = __shfl_xor_sync(0xffffffffu, b, px);
      if (rot == 64 || lane < 16) {
        const float4 cs = rope_cs2(tab, t % tps, lane, rot);
        if ((lane & px) == 0) {   // first element of the pair: x cos - partner sin
          a = a * cs.x - pa * cs.y;
          b = b * cs.z - pb * cs.w;
        } else {                  // second: partner sin + x cos
          a = pa * cs.y + a * cs.x;
          b = pb * cs.w + b * cs.z;
        }
      }
    }
    reinterpret_cast<__nv_bfloat162*>(out + (long)t * ncols + sl.col + h * 64)[lane] = __floats2bfloat162_rn(a, b);
  }
}

__global__ void head_prep_bwd_kernel(const float* g, long g_ld, const float* __restrict__ y, int T, int ncols, int H,
                                     HeadSlice sl, int tps, int rot, const float2* __restrict__ tab, float* dy) {
  pdl_prologue();
  const int h = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (h >= H) return;
  const int lane = threadIdx.x & 31;
  const int t0 = blockIdx.y * kHeadRows;
  const float2 gm = sl.gamma ? reinterpret_cast<const float2*>(sl.gamma)[lane] : make_float2(1.f, 1.f);
  float2 gv[kHeadRows], yv[kHeadRows];
  float rs[kHeadRows];
#pragma unroll
  for (int r = 0; r < kHeadRows; ++r) {
    const int t = t0 + r;
    const bool in = t < T;
    gv[r] = in ? reinterpret_cast<const float2*>(g + (long)t * g_ld + h * 64)[lane] : make_float2(0.f, 0.f);
    yv[r] = in && sl.gamma ? reinterpret_cast<const float2*>(y + (long)t * ncols + sl.col + h * 64)[lane]
                           : make_float2(0.f, 0.f);
    rs[r] = in && sl.gamma ? sl.rstd[(long)t * H + h] : 0.f;
  }
#pragma unroll
  for (int r = 0; r < kHeadRows; ++r) {
    const int t = t0 + r;
    if (t >= T) break;
    float ga = gv[r].x, gb = gv[r].y;
    if (sl.rope && (rot == 32 || rot == 64)) {   // inverse rotation of the gradient
      const int px = rot == 32 ? 8 : 16;
      const float pa = __shfl_xor_sync(0xffffffffu, ga, px), pb = __shfl_xor_sync(0xffffffffu, gb, px);
      if (rot == 64 || lane < 16) {
        const float4 cs = rope_cs2(tab, t % tps, lane, rot);
        if ((lane & px) == 0) {
          ga = ga * cs.x + pa * cs.y;
          gb = gb * cs.z + pb * cs.w;
        } else {
          ga = -pa * cs.y + ga * cs.x;
          gb = -pb * cs.w + gb * cs.z;
        }
      }
    }
    if (sl.gamma) {
      const float rr = rs[r];
      const float na = yv[r].x * rr, nb = yv[r].y * rr;
      const float da = ga * gm.x, db = gb * gm.y;
      const float mean = warp_sum(da * na + db * nb) / 64.f;
      ga = rr * (da - na * mean);
      gb = rr * (db - nb * mean);
    }
    reinterpret_cast<float2*>(dy + (long)t * ncols + sl.col + h * 64)[lane] = make_float2(ga, gb);
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

// SwiGLU over rows: f[t] = [val (I) | gate (I)], a[t] = val * silu(gate).  Grid (I / 4 / 256
// column blocks, T rows): each thread owns 4 consecutive columns of one row (128-bit accesses).
__global__ void swiglu_fwd_kernel(const float* __restrict__ f, int T, int I, __nv_bfloat16* __restrict__ a) {
  pdl_prologue();
  const int j = 4 * (blockIdx.x * blockDim.x + threadIdx.x);
  if (j >= I) return;
  for (int t = blockIdx.y; t < T; t += gridDim.y) {
  const float* fr = f + (long)t * 2 * I;
  const float4 v = *reinterpret_cast<const float4*>(fr + j);
  const float4 gl = *reinterpret_cast<const float4*>(fr + I + j);
  uint2 pk;
  pk.x = pack_bf16x2(v.x * gl.x * sigm(gl.x), v.y * gl.y * sigm(gl.y));
  pk.y = pack_bf16x2(v.z * gl.z * sigm(gl.z), v.w * gl.w * sigm(gl.w));
  *reinterpret_cast<uint2*>(a + (long)t * I + j) = pk;
  }
}

__global__ void swiglu_bwd_kernel(const float* __restrict__ da, const float* __restrict__ f, int T, int I,
                                  float* __restrict__ df) {
  pdl_prologue();
  const int j = 4 * (blockIdx.x * blockDim.x + threadIdx.x);
  if (j >= I) return;
  for (int t = blockIdx.y; t < T; t += gridDim.y) {
  const float* fr = f + (long)t * 2 * I;
  const float4 v = *reinterpret_cast<const float4*>(fr + j);
  const float4 gl = *reinterpret_cast<const float4*>(fr + I + j);
  const float4 d = *reinterpret_cast<const float4*>(da + (long)t * I + j);
  const float vv[4] = {v.x, v.y, v.z, v.w}, gg[4] = {gl.x, gl.y, gl.z, gl.w}, dd[4] = {d.x, d.y, d.z, d.w};
  float dv[4], dgl[4];
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const float sg = sigm(gg[e]);
    dv[e] = dd[e] * gg[e] * sg;
    dgl[e] = dd[e] * vv[e] * sg * (1.f + gg[e] * (1.f - sg));
  }
  float* dr = df + (long)t * 2 * I;
  *reinterpret_cast<float4*>(dr + j) = make_float4(dv[0], dv[1], dv[2], dv[3]);
  *reinterpret_cast<float4*>(dr + I + j) = make_float4(dgl[0], dgl[1], dgl[2], dgl[3]);
  }
}

__global__ void silu_bf16_kernel(const float* __restrict__ x, long n, __nv_bfloat16* __restrict__ out) {
  pdl_prologue();
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x) {
    const float v = x[i];
    out[i] = __float2bfloat16_rn(v * sigm(v));
  }
}

__global__ void modulation_kernel(const float* __restrict__ ssg, const float* __restrict__ gcond, int B, int D,
                                  float* __restrict__ mod) {
  pdl_prologue();
  const long n = (long)B * 6 * D;
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x) {
    const long j = i % (6L * D);
    float v = ssg[j] + gcond[i];
    const int slot = (int)(j / D);
    if (slot == 2 || slot == 5) v = 1.f / (__expf(v - 1.f) + 1.f);   // h * sigmoid(1 - g)
    mod[i] = v;
  }
}

__global__ void mse_kernel(const float* __restrict__ vel, const float* __restrict__ tgt, long per, float inv,
                           float* __restrict__ loss, float* __restrict__ dvel) {
  pdl_prologue();
  const int b = blockIdx.y;
  float acc = 0.f;
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < per; i += (long)gridDim.x * blockDim.x) {
    const long e = (long)b * per + i;
    const float d = vel[e] - tgt[e];
    acc += d * d;
    if (dvel) dvel[e] = 2.f * d * inv;
  }
  acc = warp_sum(acc);
  __shared__ float part[32];
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < (blockDim.x >> 5) ? part[threadIdx.x] : 0.f;
    v = warp_sum(v);
    if (threadIdx.x == 0) atomicAdd(loss + b, v * inv);
  }
}

__global__ void copy_rows_kernel(const float* __restrict__ src, int src_rows_per, int src_off, float* __restrict__ dst,
                                 __nv_bfloat16* __restrict__ dst_bf, int dst_rows_per, int dst_off, int B, int rows,
                                 int D) {
  pdl_prologue();
  const long n = (long)B * rows * D;
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x) {
    const long d = i % D, r = (i / D) % rows, b = i / ((long)D * rows);
    const float v = src[((long)b * src_rows_per + src_off + r) * D + d];
    const long o = ((long)b * dst_rows_per + dst_off + r) * D + d;
    if (dst) dst[o] = v;
    if (dst_bf) dst_bf[o] = __float2bfloat16_rn(v);
  }
}

unsigned gs(long n, int threads = 256) {
  long b = (n + threads - 1) / threads;
  if (b > 148 * 16) b = 148 * 16;
  return (unsigned)(b < 1 ? 1 : b);
}

}  // namespace

int k_rmsnorm_mod_fwd(Ctx* c, const float* x, int T, int D, const float* gamma, const float* sc, const float* sh,
                      long mod_stride, int tps, float eps, __nv_bfloat16* h, float* rstd, std::string& err) {
  if (D % 4) { err = "rms_norm: D % 4"; return 1; }
  ProfScope prof_(c, "rmsnorm_mod_fwd");
  launch_pdl(c, rmsnorm_mod_fwd_kernel, (unsigned)((T + 7) / 8), 256, 0, x, T, D, gamma, sc, sh, mod_stride, tps, eps, h, rstd);
  return check_launch("rmsnorm_mod_fwd", err);
}

int k_rmsnorm_mod_bwd(Ctx* c, const float* dh, const float* x, const float* rstd, int T, int D, const float* gamma,
                      const float* sc, long mod_stride, int tps, float* gx, std::string& err) {
  ProfScope prof_(c, "rmsnorm_mod_bwd");
  launch_pdl(c, rmsnorm_mod_bwd_kernel, (unsigned)((T + 7) / 8), 256, 0, dh, x, rstd, T, D, gamma, sc, mod_stride, tps, gx);
  return check_launch("rmsnorm_mod_bwd", err);
}

// (cos, sin) table of the context for (tps, rot, base); rebuilt only when one of them changes
static const float2* rope_table(Ctx* c, int tps, int rot, float rope_base, std::string& err) {
  if (rot == 0) return nullptr;
  const size_t bytes = sizeof(float2) * (size_t)tps * (rot / 2);
  void* tab = scratch_get(c, kSlotRope, bytes, err);
  if (!tab) return nullptr;
  if (tab != c->rope_tab || c->rope_tps != tps || c->rope_rot != rot || c->rope_base != rope_base) {
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

int k_head_prep_fwd(Ctx* c, const float* y, int T, int ncols, int H, const HeadSlice* slices, int nslices, int tps,
                    float eps, int rot, float rope_base, __nv_bfloat16* out, std::string& err) {
  if (rot != 0 && rot != 32 && rot != 64) { err = "rope: rot must be 32 or 64"; return 1; }
  if (nslices < 1 || nslices > 5) { err = "head_prep: 1..5 slices"; return 1; }
  HeadSlices hs{};
  bool any_rope = false;
  for (int i = 0; i < nslices; ++i) {
    hs.s[i] = slices[i];
    any_rope = any_rope || slices[i].rope;
  }
  hs.n = nslices;
  const float2* tab = nullptr;
  if (any_rope && rot && !(tab = rope_table(c, tps, rot, rope_base, err))) return 1;
  ProfScope prof_(c, "head_prep_fwd");
  if ((T + kHeadRows - 1) / kHeadRows > 65535) { err = "head prep: too many rows"; return 1; }
  const dim3 grid((unsigned)((H * nslices + 7) / 8), (unsigned)((T + kHeadRows - 1) / kHeadRows));
  launch_pdl(c, head_prep_fwd_kernel, grid, 256, 0, y, T, ncols, H, hs, tps, eps, rot, tab, out);
  return check_launch("head_prep_fwd", err);
}

int k_head_prep_bwd(Ctx* c, const float* g, long g_ld, const float* y, int T, int ncols, int H, const HeadSlice& sl,
                    int tps, int rot, float rope_base, float* dy, std::string& err) {
  const float2* tab = nullptr;
  if (sl.rope && rot && !(tab = rope_table(c, tps, rot, rope_base, err))) return 1;
  ProfScope prof_(c, "head_prep_bwd");
  if ((T + kHeadRows - 1) / kHeadRows > 65535) { err = "head prep: too many rows"; return 1; }
  const dim3 grid((unsigned)((H + 7) / 8), (unsigned)((T + kHeadRows - 1) / kHeadRows));
  launch_pdl(c, head_prep_bwd_kernel, grid, 256, 0, g, g_ld, y, T, ncols, H, sl, tps, rot, tab, dy);
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

int k_add(Ctx* c, const float* x, const float* y, long n, float* out, std::string& err) {
  ProfScope prof_(c, "add");
  launch_pdl(c, add_kernel, gs(n), 256, 0, x, y, n, out);
  return check_launch("add", err);
}

int k_swiglu_fwd(Ctx* c, const float* f, int T, int I, __nv_bfloat16* a, std::string& err) {
  ProfScope prof_(c, "swiglu_fwd");
  if (I % 4) { err = "swiglu: the hidden width must be a multiple of 4"; return 1; }
  launch_pdl(c, swiglu_fwd_kernel, dim3((unsigned)((I / 4 + 255) / 256), (unsigned)(T < 65535 ? T : 65535)), 256, 0, f, T, I, a);
  return check_launch("swiglu_fwd", err);
}

int k_swiglu_bwd(Ctx* c, const float* da, const float* f, int T, int I, float* df, std::string& err) {
  ProfScope prof_(c, "swiglu_bwd");
  if (I % 4) { err = "swiglu: the hidden width must be a multiple of 4"; return 1; }
  launch_pdl(c, swiglu_bwd_kernel, dim3((unsigned)((I / 4 + 255) / 256), (unsigned)(T < 65535 ? T : 65535)), 256, 0, da, f, T, I, df);
  return check_launch("swiglu_bwd", err);
}

int k_silu_bf16(Ctx* c, const float* x, long n, __nv_bfloat16* out, std::string& err) {
  ProfScope prof_(c, "silu");
  launch_pdl(c, silu_bf16_kernel, gs(n), 256, 0, x, n, out);
  return check_launch("silu", err);
}

int k_modulation(Ctx* c, const float* ssg, const float* gcond, int B, int D, float* mod, std::string& err) {
  ProfScope prof_(c, "modulation");
  launch_pdl(c, modulation_kernel, gs((long)B * 6 * D), 256, 0, ssg, gcond, B, D, mod);
  return check_launch("modulation", err);
}

int k_mse(Ctx* c, const float* vel, const float* target, int B, long per, float* loss, float* dvel, std::string& err) {
  ProfScope prof_(c, "mse");
  if (cudaMemsetAsync(loss, 0, sizeof(float) * B, c->stream) != cudaSuccess) return check_launch("mse memset", err);
  dim3 grid(16, (unsigned)B);
  launch_pdl(c, mse_kernel, grid, 256, 0, vel, target, per, 1.0f / (float)per, loss, dvel);
  return check_launch("mse", err);
}

int k_copy_rows(Ctx* c, const float* src, int src_rows_per, int src_off, float* dst, __nv_bfloat16* dst_bf,
                int dst_rows_per, int dst_off, int B, int rows, int D, std::string& err) {
  ProfScope prof_(c, "copy_rows");
  launch_pdl(c, copy_rows_kernel, gs((long)B * rows * D), 256, 0, src, src_rows_per, src_off, dst, dst_bf, dst_rows_per,
                                                                  dst_off, B, rows, D);
  return check_launch("copy_rows", err);
}

}  // namespace sa3k
