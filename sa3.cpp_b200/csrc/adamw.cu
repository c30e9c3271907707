// adamw.cu -- gradient average, global-norm clip and AdamW over the flat adapter buffers.
//
// Replaces the host loops of src/train_loop.h:147-211 (train_average_and_clip +
// train_apply_accumulated_adamw) and src/train_optimizer.h:42-65 (adamw_update_vector).
// Every adapter tensor of a training state lives in one flat f32 buffer (parameters, gradients,
// first and second moments), so the whole update is one HBM-bound elementwise pass.
//
// The arithmetic is written with explicit round-to-nearest intrinsics so nvcc cannot contract
// it into FMAs: each element goes through exactly the f32 operations of the reference, in its
// order, and the result is bit-identical to the reference's CPU code for the same inputs and the
// same bias corrections (computed on the host with the reference's std::pow(float, float)).
// Only the f64 sum of squares for the clip norm differs in summation order.
#include "sa3k_common.cuh"
#include "lora_kernels.h"

namespace sa3k {

// acc += sum_i (g_i * inv)^2 in f64, where g_i * inv is rounded to f32 first as the
// reference averages in place before it accumulates (src/train_loop.h:150-160).
__global__ void sumsq_kernel(const float* __restrict__ g, int64_t n, float inv, double* __restrict__ acc) {
  pdl_prologue();
  double s = 0.0;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  const int64_t t0 = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  int64_t head = 0;
  if ((reinterpret_cast<uintptr_t>(g) & 15) == 0) {   // 128-bit loads over the aligned groups of four
    const float4* g4 = reinterpret_cast<const float4*>(g);
    for (int64_t i = t0; i < n / 4; i += stride) {
      const float4 q = g4[i];
      const float a = __fmul_rn(q.x, inv), b = __fmul_rn(q.y, inv), c = __fmul_rn(q.z, inv), d = __fmul_rn(q.w, inv);
      s += (double)a * (double)a + (double)b * (double)b + (double)c * (double)c + (double)d * (double)d;
    }
    head = 4 * (n / 4);
  }
  for (int64_t i = head + t0; i < n; i += stride) {
    const float v = __fmul_rn(g[i], inv);
    s += (double)v * (double)v;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  __shared__ double ws[32];
  if ((threadIdx.x & 31) == 0) ws[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x < 32) {
    double t = threadIdx.x < (blockDim.x >> 5) ? ws[threadIdx.x] : 0.0;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
    if (threadIdx.x == 0) atomicAdd(acc, t);
  }
}

// scales[0] = 1/count, scales[1] = clip factor (1 when no clipping applies), norm_out = norm.
__global__ void clip_scale_kernel(const double* __restrict__ sumsq, float grad_clip, float inv_count,
                                  float* __restrict__ scales, double* __restrict__ norm_out) {
  pdl_prologue();
  const double norm = sqrt(*sumsq);
  if (norm_out) *norm_out = norm;
  scales[0] = inv_count;
  scales[1] = (grad_clip > 0.0f && norm > (double)grad_clip) ? (float)((double)grad_clip / (norm + 1e-6)) : 1.0f;
}

// One element of the reference's update (src/train_optimizer.h:42-65), operation for operation.
struct AdamWStep {
  float lr, b1, b2, eps, wd, b1c, b2c, inv, clip, omb1, omb2;
  __device__ __forceinline__ void operator()(float& p, float g, float& m, float& v) const {
    if (inv != 1.0f) g = __fmul_rn(g, inv);
    if (clip != 1.0f) g = __fmul_rn(g, clip);
    const float mi = __fadd_rn(__fmul_rn(b1, m), __fmul_rn(omb1, g));
    const float vi = __fadd_rn(__fmul_rn(b2, v), __fmul_rn(__fmul_rn(omb2, g), g));
    m = mi;
    v = vi;
    const float mh = __fdiv_rn(mi, b1c);
    const float vh = __fdiv_rn(vi, b2c);
    const float upd = __fadd_rn(__fdiv_rn(mh, __fadd_rn(__fsqrt_rn(vh), eps)), __fmul_rn(wd, p));
    p = __fsub_rn(p, __fmul_rn(lr, upd));
  }
};

__device__ __forceinline__ AdamWStep adamw_step(float lr, float b1, float b2, float eps, float wd, float b1c,
                                                float b2c, const float* scales) {
  return AdamWStep{lr, b1, b2, eps, wd, b1c, b2c, scales ? scales[0] : 1.0f, scales ? scales[1] : 1.0f, 1.0f - b1,
                   1.0f - b2};
}

__global__ void adamw_kernel(float* __restrict__ p, const float* __restrict__ g, float* __restrict__ m,
                             float* __restrict__ v, int64_t n, float lr, float b1, float b2, float eps,
                             float wd, float b1c, float b2c, const float* __restrict__ scales) {
  pdl_prologue();
  const AdamWStep st = adamw_step(lr, b1, b2, eps, wd, b1c, b2c, scales);
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
    float pi = p[i], mi = m[i], vi = v[i];
    st(pi, g[i], mi, vi);
    p[i] = pi;
    m[i] = mi;
    v[i] = vi;
  }
}

// The same over 16-byte aligned buffers: four elements per thread and iteration as one 128-bit
// load / store of each of p, g, m and v (n4 = n / 4 groups; the host runs the last n % 4
// elements through the scalar kernel).
__global__ void adamw4_kernel(float4* __restrict__ p, const float4* __restrict__ g, float4* __restrict__ m,
                              float4* __restrict__ v, int64_t n4, float lr, float b1, float b2, float eps, float wd,
                              float b1c, float b2c, const float* __restrict__ scales) {
  pdl_prologue();
  const AdamWStep st = adamw_step(lr, b1, b2, eps, wd, b1c, b2c, scales);
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += stride) {
    float4 pi = p[i], mi = m[i], vi = v[i];
    const float4 gi = g[i];
    st(pi.x, gi.x, mi.x, vi.x);
    st(pi.y, gi.y, mi.y, vi.y);
    st(pi.z, gi.z, mi.z, vi.z);
    st(pi.w, gi.w, mi.w, vi.w);
    p[i] = pi;
    m[i] = mi;
    v[i] = vi;
  }
}

static unsigned blocks_for(int64_t n) {
  int64_t b = (n + 255) / 256;
  if (b > 148 * 8) b = 148 * 8;
  return (unsigned)(b < 1 ? 1 : b);
}

int k_sumsq(Ctx* c, const float* g, int64_t n, float inv, double* acc, std::string& err) {
  ProfScope prof_(c, "sumsq");
  launch_pdl(c, sumsq_kernel, blocks_for(n), 256, 0, g, n, inv, acc);
  return check_launch("sumsq", err);
}

int k_clip_scale(Ctx* c, const double* sumsq, float grad_clip, float inv_count, float* scales,
                 double* norm_out, std::string& err) {
  ProfScope prof_(c, "clip_scale");
  launch_pdl(c, clip_scale_kernel, 1, 1, 0, sumsq, grad_clip, inv_count, scales, norm_out);
  return check_launch("clip_scale", err);
}

int k_adamw(Ctx* c, float* p, const float* g, float* m, float* v, int64_t n, float lr, float b1, float b2,
            float eps, float wd, float b1c, float b2c, const float* scales, std::string& err) {
  ProfScope prof_(c, "adamw");
  auto al16 = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15) == 0; };
  int64_t done = 0;
  if (al16(p) && al16(g) && al16(m) && al16(v) && n >= 4) {
    const int64_t n4 = n / 4;
    launch_pdl(c, adamw4_kernel, blocks_for(n4), 256, 0, reinterpret_cast<float4*>(p),
               reinterpret_cast<const float4*>(g), reinterpret_cast<float4*>(m), reinterpret_cast<float4*>(v), n4, lr,
               b1, b2, eps, wd, b1c, b2c, scales);
    if (check_launch("adamw", err)) return 1;
    done = 4 * n4;
  }
  if (done == n) return 0;
  launch_pdl(c, adamw_kernel, blocks_for(n - done), 256, 0, p + done, g + done, m + done, v + done, n - done, lr, b1,
             b2, eps, wd, b1c, b2c, scales);
  return check_launch("adamw", err);
}

}  // namespace sa3k
