// quant.cu -- frozen base weights: GGUF block bytes -> the device layout the GEMM engine reads.
//
// The reference hands ggml the raw GGUF rows (src/gguf_model.h:318-329 uploads them as-is) and
// ggml's type traits dequantize per row (src/lora.h:52-74, to_float).  Here the bytes are
// uploaded once and repacked on the device into separate code and scale planes, which TMA can
// tile (a 34-byte Q8_0 block is not 16-byte aligned):
//   Q8_0: codes int8 [out][in];         scales f32   [in/32][out] = d
//   Q4_K: codes u8   [out][in/2] (element 2j in the low nibble of byte j, 2j+1 in the high);
//         scales float2 [in/32][out] = (d*sc, dmin*m) for each 32-element sub-block.
//   F16 / F32: f16 [out][in].
// value(o, i) = code * d (Q8_0) or (d*sc) * code - dmin*m (Q4_K) in f32 is exactly what
// ggml-quants.c computes; dequant_kernel below is the bit-exactness probe for that claim.
#include "sa3k_internal.h"
#include "weight_value.cuh"

namespace sa3k {

// ---- Q8_0: 34-byte blocks {f16 d, int8 q[32]} along `in` ----
__global__ void repack_q8_0_kernel(const uint8_t* __restrict__ raw, int64_t in, int64_t out,
                                   int8_t* __restrict__ codes, float* __restrict__ scales) {
  const int64_t nb = in / 32;
  const int64_t blk = (int64_t)blockIdx.x * blockDim.y + threadIdx.y;   // one warp per block
  if (blk >= nb * out) return;
  const int64_t o = blk / nb, b = blk % nb;
  const uint8_t* p = raw + (o * nb + b) * 34;
  const int l = threadIdx.x;
  codes[o * in + b * 32 + l] = (int8_t)p[2 + l];
  if (l == 0) {
    const uint16_t dh = (uint16_t)p[0] | ((uint16_t)p[1] << 8);
    scales[b * out + o] = __half2float(__ushort_as_half(dh));
  }
}

// ---- Q4_K: 144-byte super-blocks {f16 d, f16 dmin, 12 B scales, 128 B nibbles} along `in` ----
__device__ __forceinline__ void q4k_scale_min(const uint8_t* s, int j, int& sc, int& mn) {
  if (j < 4) {
    sc = s[j] & 63;
    mn = s[j + 4] & 63;
  } else {
    sc = (s[j + 4] & 0x0f) | ((s[j - 4] >> 6) << 4);
    mn = (s[j + 4] >> 4) | ((s[j] >> 6) << 4);
  }
}

__global__ void repack_q4_k_kernel(const uint8_t* __restrict__ raw, int64_t in, int64_t out,
                                   uint8_t* __restrict__ codes, float2* __restrict__ scales) {
  const int64_t nsb = in / 256;
  const int64_t sblk = (int64_t)blockIdx.x * blockDim.y + threadIdx.y;   // one warp per super-block
  if (sblk >= nsb * out) return;
  const int64_t o = sblk / nsb, b = sblk % nsb;
  const uint8_t* p = raw + (o * nsb + b) * 144;
  const float d = __half2float(__ushort_as_half((uint16_t)(p[0] | (p[1] << 8))));
  const float dmin = __half2float(__ushort_as_half((uint16_t)(p[2] | (p[3] << 8))));
  const uint8_t* qs = p + 16;
  const int l = threadIdx.x;   // 0..31
  // element e of sub-block sb: byte qs[(sb/2)*32 + e], nibble (sb & 1)
  // output byte j (0..127) of this super-block holds elements 2j, 2j+1
#pragma unroll
  for (int t = 0; t < 4; ++t) {
    const int j = l + 32 * t;                 // output byte
    const int e0 = 2 * j, e1 = 2 * j + 1;     // elements in 0..255
    const int sb0 = e0 >> 5, sb1 = e1 >> 5;   // same sub-block (e0 even)
    const uint8_t b0 = qs[(sb0 >> 1) * 32 + (e0 & 31)];
    const uint8_t b1 = qs[(sb1 >> 1) * 32 + (e1 & 31)];
    const int q0 = (sb0 & 1) ? (b0 >> 4) : (b0 & 15);
    const int q1 = (sb1 & 1) ? (b1 >> 4) : (b1 & 15);
    codes[o * (in / 2) + b * 128 + j] = (uint8_t)(q0 | (q1 << 4));
  }
  if (l < 8) {
    int sc, mn;
    q4k_scale_min(p + 4, l, sc, mn);
    scales[(b * 8 + l) * out + o] = make_float2(d * (float)sc, dmin * (float)mn);
  }
}

__global__ void repack_f16_kernel(const __half* __restrict__ src, int64_t n, __half* __restrict__ dst) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    dst[i] = __float2half_rn(__half2float(src[i]));
}

__global__ void repack_f32_kernel(const float* __restrict__ src, int64_t n, __half* __restrict__ dst) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    dst[i] = __float2half_rn(src[i]);
}

__global__ void dequant_kernel(const Weight w, float* __restrict__ dst) {
  const int64_t n = w.in * w.out;
  for (int64_t k = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; k < n; k += (int64_t)gridDim.x * blockDim.x)
    dst[k] = wval(w, k / w.in, k % w.in);
}

// bns[o] = sum_i W[o,i]^2 + in*eps and norm[o] = sqrt(sum_i W[o,i]^2), f64 accumulation
// (src/train_lora.h:141-174).  One warp per output row.
__global__ void row_norms_kernel(const Weight w, float eps, float* __restrict__ nsq, float* __restrict__ nrm) {
  const int64_t o = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  if (o >= w.out) return;
  const int lane = threadIdx.x & 31;
  double s = 0.0;
  for (int64_t i = lane; i < w.in; i += 32) {
    const double v = (double)wval(w, o, i);
    s += v * v;
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
  if (lane == 0) {
    if (nsq) nsq[o] = (float)(s + (double)w.in * (double)eps);
    if (nrm) nrm[o] = (float)sqrt(s);
  }
}

// f16 operand copy of a quantized weight: the exact f32 dequantized value, rounded once.
__global__ void dequant_f16_kernel(const Weight w, __half* __restrict__ dst) {
  const int64_t n = w.in * w.out;
  for (int64_t k = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; k < n; k += (int64_t)gridDim.x * blockDim.x)
    dst[k] = __float2half_rn(wval(w, k / w.in, k % w.in));
}

int weight_cache_f16(Ctx* c, Weight* w, std::string& err) {
  ProfScope prof_(c, "weight cache");
  dequant_f16_kernel<<<1184, 256, 0, c->stream>>>(*w, w->f16);
  return check_launch("weight cache", err);
}

int weight_repack(Ctx* c, Weight* w, std::string& err) {
  ProfScope prof_(c, "weight repack");
  const cudaStream_t st = c->stream;
  if (w->type == kTypeQ8_0) {
    const int64_t nblk = w->in / 32 * w->out;
    dim3 blk(32, 8);
    repack_q8_0_kernel<<<(unsigned)((nblk + 7) / 8), blk, 0, st>>>(
        reinterpret_cast<const uint8_t*>(w->raw), w->in, w->out, w->codes, w->scales);
  } else if (w->type == kTypeQ4_K) {
    const int64_t nblk = w->in / 256 * w->out;
    dim3 blk(32, 8);
    repack_q4_k_kernel<<<(unsigned)((nblk + 7) / 8), blk, 0, st>>>(
        reinterpret_cast<const uint8_t*>(w->raw), w->in, w->out,
        reinterpret_cast<uint8_t*>(w->codes), reinterpret_cast<float2*>(w->scales));
  } else if (w->type == kTypeF16) {
    repack_f16_kernel<<<1184, 256, 0, st>>>(reinterpret_cast<const __half*>(w->raw), w->in * w->out, w->f16);
  } else {
    repack_f32_kernel<<<1184, 256, 0, st>>>(reinterpret_cast<const float*>(w->raw), w->in * w->out, w->f16);
  }
  return check_launch("weight repack", err);
}

// codes_t[i][o] = codes[o][i] (Q8_0 bytes, or Q4_K nibbles: codes_t byte i*(out/2) + o/2 holds o
// even in the low nibble), one 64 x 64 tile of elements per block through shared memory.
__global__ void transpose_codes_kernel(const uint8_t* __restrict__ codes, int64_t in, int64_t out, int q4,
                                       uint8_t* __restrict__ codes_t) {
  __shared__ uint8_t tile[64][65];
  const int64_t o0 = (int64_t)blockIdx.y * 64, i0 = (int64_t)blockIdx.x * 64;
  for (int e = threadIdx.x; e < 64 * 64; e += blockDim.x) {
    const int r = e / 64, cl = e % 64;   // element (o0 + r, i0 + cl)
    const int64_t o = o0 + r, i = i0 + cl;
    uint8_t v = 0;
    if (o < out && i < in) {
      if (q4) {
        const uint8_t b = codes[o * (in / 2) + i / 2];
        v = (i & 1) ? (uint8_t)(b >> 4) : (uint8_t)(b & 0x0F);
      } else {
        v = codes[o * in + i];
      }
    }
    tile[r][cl] = v;
  }
  __syncthreads();
  if (q4) {
    for (int e = threadIdx.x; e < 64 * 32; e += blockDim.x) {
      const int cl = e / 32, rp = e % 32;   // output row i0 + cl, byte (o0 + 2 rp) / 2
      const int64_t i = i0 + cl, o = o0 + 2 * rp;
      if (i < in && o < out) codes_t[i * (out / 2) + o / 2] = (uint8_t)(tile[2 * rp][cl] | (tile[2 * rp + 1][cl] << 4));
    }
  } else {
    for (int e = threadIdx.x; e < 64 * 64; e += blockDim.x) {
      const int cl = e / 64, r = e % 64;
      const int64_t i = i0 + cl, o = o0 + r;
      if (i < in && o < out) codes_t[i * out + o] = tile[r][cl];
    }
  }
}

int weight_transpose_codes(Ctx* c, Weight* w, std::string& err) {
  if (w->codes_t) return 0;
  if (w->type != kTypeQ8_0 && w->type != kTypeQ4_K) {
    err = "transposed codes exist only for Q8_0 / Q4_K weights";
    return 1;
  }
  const bool q4 = w->type == kTypeQ4_K;
  if (q4 && (w->out & 1)) {
    err = "Q4_K transposed codes need an even out";
    return 1;
  }
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(c->stream, &cs) != cudaSuccess || cs != cudaStreamCaptureStatusNone) {
    cudaGetLastError();
    err = "transposed weight codes are made on the first eager call, not inside a stream capture";
    return 1;
  }
  const size_t bytes = q4 ? (size_t)(w->in * (w->out / 2)) : (size_t)(w->in * w->out);
  if (cudaMalloc(&w->codes_t, bytes) != cudaSuccess) {
    w->codes_t = nullptr;
    cudaGetLastError();
    err = "out of device memory (transposed weight codes)";
    return 1;
  }
  ProfScope prof_(c, "weight transpose");
  dim3 grid((unsigned)((w->in + 63) / 64), (unsigned)((w->out + 63) / 64));
  transpose_codes_kernel<<<grid, 256, 0, c->stream>>>(reinterpret_cast<const uint8_t*>(w->codes), w->in, w->out,
                                                       q4 ? 1 : 0, reinterpret_cast<uint8_t*>(w->codes_t));
  return check_launch("weight transpose", err);
}

int weight_dequant(Ctx* c, const Weight* w, float* dst, std::string& err) {
  ProfScope prof_(c, "dequant");
  dequant_kernel<<<1184, 256, 0, c->stream>>>(*w, dst);
  return check_launch("dequant", err);
}

int weight_row_norms(Ctx* c, const Weight* w, float eps, float* nsq, float* nrm, std::string& err) {
  ProfScope prof_(c, "row norms");
  row_norms_kernel<<<(unsigned)((w->out + 7) / 8), 256, 0, c->stream>>>(*w, eps, nsq, nrm);
  return check_launch("row norms", err);
}

}  // namespace sa3k
