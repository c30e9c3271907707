// gemm_wq.cuh -- quantized-weight GEMM with the dequantized weight as the tensor-memory operand.
//
// The frozen base of a linear (Q8_0 / Q4_K codes + block scales, quant.cu's layouts) times an
// f16 activation, computed transposed so that the weight is the MMA's A operand:
//
//   D[f][t] = sum_k Wop[f][k] * X[t][k]        f = 128 output features per tile (TMEM lanes)
//                                               t = 128 tokens per tile (the MMA's N)
//   NT (forward, y = x W^T):    Wop[f][k] = W[f][k]   (f = out, k = in)
//   TN (input grad, dx = dy W): Wop[f][k] = W[k][f]   (f = in,  k = out), read from the
//                                                      transposed codes (codes_t, [in][out])
//
// Why this form: a tcgen05 MMA reads its B operand from shared memory but may take A from tensor
// memory.  Dequantizing the weight straight into tensor memory (registers -> tcgen05.st) keeps the
// f16 weight tile out of shared memory: per 128-k stage the shared-memory traffic is the
// activation tile (32 KB, written by TMA, read by the MMA) plus the 1-byte codes and the scales
// (18 KB, written by TMA, read once by the dequant warps), where dequantizing into a shared-memory
// f16 operand tile would add 64 KB of f16 writes and reads for the same MMA work.
//
// Warp roles (736 threads) and their three rings:
//   warp 0        activation producer (X ring, kWqXStages): the tile [128 t][128 k] f16 as two
//                 128B-swizzled 64-k halves; for the K = 16 extension the u^T tile [16][128 t].
//                 A slot is freed by the MMA that read it.
//   warp 1        TMEM owner and MMA issue (A from TMEM, B from shared memory), 8 MMAs a stage
//   warps 2-5     epilogue: one warp per TMEM lane quarter, all 128 token columns
//   warps 6-21    dequant: four warps per lane quarter, 32 of the 128 k of a stage each, from
//                 the codes ring into the A ring (kWqAStages, tensor memory; freed by the MMA)
//   warp 22       codes producer (C ring, kWqCStages): codes [128 f][128 k] (128B swizzle; Q4_K
//                 64 bytes a row, 64B swizzle) and the stage's block scales.  A slot is freed by
//                 the dequant warps once they hold its values, so the codes run ahead of the MMA.
//
// Tensor memory (512 columns): two 128-column accumulators and kWqAStages A stages of 64 columns
// (128 f16 per lane).  The dequantized value is the exact f32 product of the reference's
// dequantization rounded once to f16 -- the same value the f16 operand cache holds.
#pragma once

#include "gemm_tc.cuh"

namespace sa3k {

struct WqArgs {
  int M, N, K;               // tokens, features, contraction
  int nt;                    // 1: forward (W[f][k]), 0: transposed (W[k][f] from codes_t)
  int has_ext;               // one K = 16 extension MMA: A = ext_b [N][64] f16 (cols 0..15), B = u^T
  const __half* ext_b;
  const float* col_scale;    // per feature (nullable)
  const float* col_bias;     // per feature (nullable)
  float alpha;
  float* out;                // f32 out[t * ldo + f] (out_trans: out[f * ldo + t]); nullable
  long ldo;
  int out_trans;
  int accumulate;
  __half* out_h;             // f16 h_scale * value, [t][ldo_h] (out_h_trans: [f][ldo_h]); nullable
  long ldo_h;
  int out_h_trans;
  float h_scale;
  __half* out_h_t;           // second f16 output, transposed [f][ldo_h_t] (nullable)
  long ldo_h_t;
  int* err;
};

constexpr int kWqF = 128, kWqT = 128, kWqK = 128, kWqXStages = 4, kWqAStages = 4, kWqCStages = 5;

template <int QT>
struct WqSmem {
  static constexpr int X_BYTES = kWqT * kWqK * 2;                  // 32 KB: two 64-k halves (128B swizzle)
  static constexpr int C_BYTES = kWqF * kWqK / (QT == 0 ? 1 : 2);  // codes of 128 features x 128 k
  static constexpr int SC_BYTES = (QT == 0 ? 4 : 8) * 512;         // 4 x 128 scales (f32 or float2)
  static constexpr int OFF_X = 0;
  static constexpr int OFF_C = OFF_X + kWqXStages * X_BYTES;
  static constexpr int OFF_SC = OFF_C + kWqCStages * C_BYTES;
  static constexpr int OFF_BAR = OFF_SC + kWqCStages * SC_BYTES;
  static constexpr int BAR_BYTES = (2 * kWqXStages + 2 * kWqAStages + 2 * kWqCStages + 4) * 8 + 16;
  static constexpr int DYN = OFF_BAR + BAR_BYTES + 1024;
  static_assert(DYN <= 232448, "shared memory budget (227 KB)");
};

constexpr int kWqEpiWarps = 4, kWqDqWarps = 16;
constexpr int kWqCodeWarp = 2 + kWqEpiWarps + kWqDqWarps;   // the codes / scales producer
constexpr int kWqThreads = 32 * (kWqCodeWarp + 1);

__device__ __forceinline__ void tmem_st8(uint32_t taddr, const uint32_t (&r)[8]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"r"(taddr), "r"(r[0]),
      "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7])
      : "memory");
}

__device__ __forceinline__ void tmem_st16_w(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}

__device__ __forceinline__ void tmem_st32_w(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, "
      "%17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]),
      "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]),
      "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}

__device__ __forceinline__ void tmem_st_wait_w() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// 8 int8 codes (two words) times per-pair scales s01, s23, s45, s67 (TN: the scale changes with k)
__device__ __forceinline__ uint4 q8_chunk4(uint2 q, uint64_t s01, uint64_t s23, uint64_t s45, uint64_t s67) {
  const uint32_t w[2] = {q.x ^ 0x80808080u, q.y ^ 0x80808080u};
  const uint64_t bias = f2(-8388736.0f, -8388736.0f);
  const uint64_t sc[4] = {s01, s23, s45, s67};
  uint32_t o[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const uint32_t ww = w[k >> 1];
    const int b = 2 * (k & 1);
    float lo, hi;
    f2split(fmul2(fadd2(f2(magic_code(ww, b), magic_code(ww, b + 1)), bias), sc[k]), lo, hi);
    o[k] = pack_f16x2(lo, hi);
  }
  return make_uint4(o[0], o[1], o[2], o[3]);
}

// 8 Q4_K codes (one word of nibbles, element 2b low nibble of byte b) with per-pair (d, m)
__device__ __forceinline__ uint4 q4_chunk4(uint32_t nib, const uint64_t (&dd)[4], const uint64_t (&mm)[4]) {
  const uint32_t lo4 = nib & 0x0F0F0F0Fu, hi4 = (nib >> 4) & 0x0F0F0F0Fu;
  const uint64_t bias = f2(-8388608.0f, -8388608.0f);
  uint32_t o[4];
#pragma unroll
  for (int b = 0; b < 4; ++b) {
    float v0, v1;
    f2split(ffma2(dd[b], fadd2(f2(magic_code(lo4, b), magic_code(hi4, b)), bias), mm[b]), v0, v1);
    o[b] = pack_f16x2(v0, v1);
  }
  return make_uint4(o[0], o[1], o[2], o[3]);
}

// 8 int8 codes (two words) times f16 scales in packed f16 arithmetic.  A Q8_0 block scale is an
// f16 value and a code an integer of at most 7 bits, so their product is exact in f32 and the f32
// path's one rounding to f16 equals the one rounding of an f16 multiply: bit-identical values.
// A biased byte b = code + 128 placed under the f16 exponent of 1024 (0x64bb) is 1024 + b
// exactly; subtracting 1152 leaves the code.  dd01 .. dd67: the scale of each element pair.
__device__ __forceinline__ uint4 q8_chunk_h(uint2 q, uint32_t dd01, uint32_t dd23, uint32_t dd45, uint32_t dd67) {
  const uint32_t w0 = q.x ^ 0x80808080u, w1 = q.y ^ 0x80808080u;
  const __half2 bias = __halves2half2(__ushort_as_half((unsigned short)0x6480u),
                                      __ushort_as_half((unsigned short)0x6480u));
  const uint32_t p[4] = {__byte_perm(w0, 0x64646464u, 0x5140u), __byte_perm(w0, 0x64646464u, 0x5342u),
                         __byte_perm(w1, 0x64646464u, 0x5140u), __byte_perm(w1, 0x64646464u, 0x5342u)};
  const uint32_t dd[4] = {dd01, dd23, dd45, dd67};
  uint32_t o[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const __half2 v = __hmul2(__hsub2(*reinterpret_cast<const __half2*>(&p[k]), bias),
                              *reinterpret_cast<const __half2*>(&dd[k]));
    o[k] = *reinterpret_cast<const uint32_t*>(&v);
  }
  return make_uint4(o[0], o[1], o[2], o[3]);
}

__device__ __forceinline__ uint32_t h2bits(float a, float b) {
  const __half2 v = __floats2half2_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&v);
}

// Dequantize this thread's part of a stage into 16 packed f16 pairs: row r of the 128-feature
// tile (quarter q = r / 32) and k 32h .. 32h + 31 of the stage, from the stage's codes cst and
// block scales sc in shared memory (TMA layouts: codes 128B-swizzled rows, Q4_K 64B-swizzled).
template <int QT>
__device__ __forceinline__ void wq_dequant(const uint8_t* cst, const uint8_t* sc, bool nt, int r, int q, int h,
                                           uint32_t (&rg)[16]) {
  // codes of row r, k 32h .. 32h + 31 (rows beyond N and k beyond K read TMA's zero fill)
  uint4 ca, cb = make_uint4(0, 0, 0, 0);
  if (QT == 0) {   // 128-byte rows, 128B swizzle: 16-byte chunk c at c ^ (r & 7)
    ca = *reinterpret_cast<const uint4*>(cst + r * 128 + 16 * ((2 * h) ^ (r & 7)));
    cb = *reinterpret_cast<const uint4*>(cst + r * 128 + 16 * ((2 * h + 1) ^ (r & 7)));
  } else {         // 64-byte rows, 64B swizzle: chunk c at c ^ ((r >> 1) & 3)
    ca = *reinterpret_cast<const uint4*>(cst + r * 64 + 16 * (h ^ ((r >> 1) & 3)));
  }
  if (nt) {
    // one block scale for the 32 k: scales [4 k-blocks][128 f], block h
    if (QT == 0) {
      const float d = reinterpret_cast<const float*>(sc)[h * 128 + r];
      const uint32_t dd = h2bits(d, d);   // exact: d is an f16 value
      const uint4 c0 = q8_chunk_h(make_uint2(ca.x, ca.y), dd, dd, dd, dd);
      const uint4 c1 = q8_chunk_h(make_uint2(ca.z, ca.w), dd, dd, dd, dd);
      const uint4 c2 = q8_chunk_h(make_uint2(cb.x, cb.y), dd, dd, dd, dd);
      const uint4 c3 = q8_chunk_h(make_uint2(cb.z, cb.w), dd, dd, dd, dd);
      const uint32_t t16[16] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w,
                                c2.x, c2.y, c2.z, c2.w, c3.x, c3.y, c3.z, c3.w};
#pragma unroll
      for (int j2 = 0; j2 < 16; ++j2) rg[j2] = t16[j2];
    } else {
      const float2 dm = reinterpret_cast<const float2*>(sc)[h * 128 + r];
      const uint64_t d4[4] = {f2(dm.x, dm.x), f2(dm.x, dm.x), f2(dm.x, dm.x), f2(dm.x, dm.x)};
      const uint64_t m4[4] = {f2(-dm.y, -dm.y), f2(-dm.y, -dm.y), f2(-dm.y, -dm.y), f2(-dm.y, -dm.y)};
      const uint32_t words[4] = {ca.x, ca.y, ca.z, ca.w};
#pragma unroll
      for (int w4 = 0; w4 < 4; ++w4) {
        const uint4 o = q4_chunk4(words[w4], d4, m4);
        rg[4 * w4] = o.x; rg[4 * w4 + 1] = o.y; rg[4 * w4 + 2] = o.z; rg[4 * w4 + 3] = o.w;
      }
    }
  } else {
    // the scale changes with k (k = the weight's output row): scales [4 f-blocks][128 k]
    if (QT == 0) {
      const float4* sq = reinterpret_cast<const float4*>(sc) + q * 32 + h * 8;   // 32 floats
      const uint32_t wv[8] = {ca.x, ca.y, ca.z, ca.w, cb.x, cb.y, cb.z, cb.w};
#pragma unroll
      for (int g = 0; g < 4; ++g) {   // 8 k per group: two float4 of scales
        const float4 s0 = sq[2 * g], s1 = sq[2 * g + 1];
        const uint4 o = q8_chunk_h(make_uint2(wv[2 * g], wv[2 * g + 1]), h2bits(s0.x, s0.y),
                                   h2bits(s0.z, s0.w), h2bits(s1.x, s1.y), h2bits(s1.z, s1.w));
        rg[4 * g] = o.x; rg[4 * g + 1] = o.y; rg[4 * g + 2] = o.z; rg[4 * g + 3] = o.w;
      }
    } else {
      const float4* sq = reinterpret_cast<const float4*>(sc) + q * 64 + h * 16;   // 32 float2
      const uint32_t words[4] = {ca.x, ca.y, ca.z, ca.w};
#pragma unroll
      for (int g = 0; g < 4; ++g) {   // 8 k: four float4 = (d0, m0, d1, m1) pairs
        uint64_t d4[4], m4[4];
#pragma unroll
        for (int p = 0; p < 4; ++p) {
          const float4 dm = sq[4 * g + p];
          d4[p] = f2(dm.x, dm.z);
          m4[p] = f2(-dm.y, -dm.w);
        }
        const uint4 o = q4_chunk4(words[g], d4, m4);
        rg[4 * g] = o.x; rg[4 * g + 1] = o.y; rg[4 * g + 2] = o.z; rg[4 * g + 3] = o.w;
      }
    }
  }
}

// Epilogue of one accumulator: lane = feature f (TMEM lane), the tile's kWqT token columns from
// tacc; out = alpha * col_scale[f] * acc + col_bias[f] into the outputs args names.  `have` false
// (an aborted tile): the TMEM reads still run (warp-aligned), nothing is stored.
__device__ __forceinline__ void wq_drain(const WqArgs& args, uint32_t tacc, int f, int t0, bool have) {
  const bool fin = f < args.N;
  float cs = args.alpha, cb = 0.f;
  if (fin && args.col_scale) cs *= args.col_scale[f];
  if (fin && args.col_bias) cb = args.col_bias[f];
#pragma unroll 1
  for (int c0 = 0; c0 < kWqT; c0 += 32) {
    uint32_t v[32];
    tmem_ld32(tacc + (uint32_t)c0, v);
    tmem_ld_wait();
    if (!have || !fin) continue;
    const int tb = t0 + c0;
    float x[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) x[j] = __uint_as_float(v[j]) * cs + cb;
    if (args.out && !args.out_trans) {
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        if (tb + j >= args.M) break;
        float* dst = args.out + (long)(tb + j) * args.ldo + f;
        *dst = args.accumulate ? *dst + x[j] : x[j];
      }
    }
    if (args.out && args.out_trans) {
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        if (tb + j >= args.M) break;
        float* dst = args.out + (long)f * args.ldo + tb + j;
        *dst = args.accumulate ? *dst + x[j] : x[j];
      }
    }
    if (args.out_h) {
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        if (tb + j >= args.M) break;
        const __half hv = __float2half_rn(x[j] * args.h_scale);
        if (args.out_h_trans) args.out_h[(long)f * args.ldo_h + tb + j] = hv;
        else args.out_h[(long)(tb + j) * args.ldo_h + f] = hv;
      }
    }
    if (args.out_h_t) {
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        if (tb + j >= args.M) break;
        args.out_h_t[(long)f * args.ldo_h_t + tb + j] = __float2half_rn(x[j]);
      }
    }
  }
}

template <int QT>
__global__ void __launch_bounds__(kWqThreads, 1)
    gemm_wq_kernel(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_c,
                   const __grid_constant__ CUtensorMap tm_sc, const __grid_constant__ CUtensorMap tm_u,
                   const __grid_constant__ WqArgs args) {
  using L = WqSmem<QT>;
  extern __shared__ uint8_t smem_raw[];
  pdl_trigger();
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t* xfull = reinterpret_cast<uint64_t*>(smem + L::OFF_BAR);
  uint64_t* xempty = xfull + kWqXStages;
  uint64_t* afull = xempty + kWqXStages;
  uint64_t* aempty = afull + kWqAStages;
  uint64_t* cfull = aempty + kWqAStages;
  uint64_t* cempty = cfull + kWqCStages;
  uint64_t* tfull = cempty + kWqCStages;   // [2]
  uint64_t* tempty = tfull + 2;            // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tiles_f = (args.N + kWqF - 1) / kWqF;
  const int tiles_t = (args.M + kWqT - 1) / kWqT;
  const int ntiles = tiles_f * tiles_t;
  const int nkb = (args.K + kWqK - 1) / kWqK;
  const int total = nkb + (args.has_ext ? 1 : 0);   // k-steps per tile

  if (warp == 0 && lane == 0) {
    for (int s = 0; s < kWqXStages; ++s) {
      mbar_init(&xfull[s], 1);
      mbar_init(&xempty[s], 1);
    }
    for (int s = 0; s < kWqAStages; ++s) {
      mbar_init(&afull[s], 32 * kWqDqWarps);
      mbar_init(&aempty[s], 1);
    }
    for (int s = 0; s < kWqCStages; ++s) {
      mbar_init(&cfull[s], 1);
      mbar_init(&cempty[s], 32 * kWqDqWarps);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 32 * kWqEpiWarps);
    }
    *abort_flag = 0;
    fence_barrier_init();
    tma_prefetch_desc(&tm_x);
    tma_prefetch_desc(&tm_c);
    tma_prefetch_desc(&tm_sc);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
    tc_fence_before();
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tmem_slot;
  const uint32_t tA = tbase + 2 * kWqT;   // A stages (kWqK / 2 columns each) after the two accumulators
  pdl_wait();

  // (waiting threads sleep between polls: the dequant warps share the SM's issue slots with
  // the polls of the others)
  auto wait = [&](uint64_t* bar, uint32_t parity, int code) -> bool {
    if (*abort_flag) return false;
    const uint32_t a = smem_u32(bar);
    if (mbar_try_wait(a, parity)) return true;
    const unsigned long long t0 = globaltimer();
    for (uint32_t i = 1;; ++i) {
      if (mbar_try_wait_sleep(a, parity, 200)) return true;
      if ((i & 63u) == 0) {
        if (*abort_flag) return false;
        if (globaltimer() - t0 > kWaitLimitNs) {
          record_error(args.err, code);
          *abort_flag = 1;
          return false;
        }
      }
    }
  };

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      int it = 0;
      bool ok = true;
      for (int item = blockIdx.x; item < ntiles && ok; item += gridDim.x) {
        const int t0 = (item / tiles_f) * kWqT;
        for (int kb = 0; kb < total; ++kb, ++it) {
          const int s = it % kWqXStages;
          const uint32_t use = (uint32_t)(it / kWqXStages);
          if (it >= kWqXStages && !wait(&xempty[s], (use & 1u) ^ 1u, kErrTimeoutEmpty)) { ok = false; break; }
          uint8_t* xs = smem + L::OFF_X + s * L::X_BYTES;
          if (kb < nkb) {
            mbar_arrive_expect_tx(&xfull[s], (uint32_t)L::X_BYTES);
            tma_load_2d(xs, &tm_x, &xfull[s], kb * kWqK, t0);
            tma_load_2d(xs + L::X_BYTES / 2, &tm_x, &xfull[s], kb * kWqK + 64, t0);
          } else {
            // extension: u^T rows t0 .. t0 + 127 as two MN-major 64 (t) x 16 (k) boxes
            mbar_arrive_expect_tx(&xfull[s], (uint32_t)(2 * 64 * 16 * 2));
            tma_load_2d(xs, &tm_u, &xfull[s], t0, 0);
            tma_load_2d(xs + 2048, &tm_u, &xfull[s], t0 + 64, 0);
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issue
    const WaiterW<> wt{abort_flag, args.err};
    const uint32_t idesc = make_idesc_f16(kWqF, kWqT, 0, 0);       // B = activation tile, K-major
    const uint32_t idesc_ext = make_idesc_f16(kWqF, kWqT, 0, 1);   // B = u^T, MN-major
    const uint64_t xdesc0 = make_sdesc(smem_u32(smem + L::OFF_X), 16, 1024);
    const uint64_t udesc0 = make_sdesc(smem_u32(smem + L::OFF_X), 2048, 1024);
    int it = 0, ti = 0;
    bool ok = true;
    for (int item = blockIdx.x; item < ntiles && ok; item += gridDim.x, ++ti) {
      const int a = ti & 1;
      const uint32_t ause = (uint32_t)(ti >> 1);
      if (ti >= 2 && !wt(&tempty[a], (ause & 1u) ^ 1u, kErrTimeoutOther)) { ok = false; break; }
      tc_fence_after();
      const uint32_t d_tmem = tbase + (uint32_t)(a * kWqT);
      for (int kb = 0; kb < total; ++kb, ++it) {
        const int s = it % kWqXStages, as = it % kWqAStages;
        if (!wt(&xfull[s], (uint32_t)(it / kWqXStages) & 1u, kErrTimeoutFull)) { ok = false; break; }
        if (!wt(&afull[as], (uint32_t)(it / kWqAStages) & 1u, kErrTimeoutReady)) { ok = false; break; }
        tc_fence_after();
        const uint32_t xoff = (uint32_t)(s * L::X_BYTES) >> 4;
        const uint32_t a_tm = tA + (uint32_t)(as * (kWqK / 2));
        if (kb < nkb) {
#pragma unroll
          for (int kk = 0; kk < kWqK / 16; ++kk)   // 64-k halves of the stage at +0 and +16 KB
            umma_ts_w(d_tmem, a_tm + (uint32_t)(kk * 8),
                      xdesc0 + xoff + (uint32_t)((kk >> 2) * (L::X_BYTES / 2 >> 4)) + (uint32_t)((kk & 3) * 2), idesc,
                      (kb > 0 || kk > 0) ? 1u : 0u);
        } else {
          umma_ts_w(d_tmem, a_tm, udesc0 + xoff, idesc_ext, total > 1 ? 1u : 0u);
        }
        umma_commit_w(&xempty[s]);
        umma_commit_w(&aempty[as]);
      }
      if (ok) umma_commit_w(&tfull[a]);
    }
  } else if (warp < 2 + kWqEpiWarps) {
    // ------------------------------------------------------------ epilogue
    // Lane = feature f, TMEM column = token: a warp store of one token row covers 32 consecutive
    // features (128 contiguous bytes of f32 output).
    const int q = warp & 3;
    int ti = 0;
    for (int item = blockIdx.x; item < ntiles; item += gridDim.x, ++ti) {
      const int f0 = (item % tiles_f) * kWqF, t0 = (item / tiles_f) * kWqT;
      const int a = ti & 1;
      const bool have = wait(&tfull[a], (uint32_t)(ti >> 1) & 1u, kErrTimeoutAccum);
      tc_fence_after();
      wq_drain(args, tbase + (uint32_t)(a * kWqT) + ((uint32_t)(32 * q) << 16), f0 + 32 * q + lane, t0, have);
      tc_fence_before();
      mbar_arrive(&tempty[a]);
    }
  } else if (warp == kWqCodeWarp) {
    // ------------------------------------------------------------ codes / scales producer
    // Its ring is released by the dequant warps as soon as they hold a stage's values, not by
    // the MMA: the codes run ahead of the activations by up to kWqCStages.
    if (lane == 0) {
      int ic = 0;
      bool ok = true;
      for (int item = blockIdx.x; item < ntiles && ok; item += gridDim.x) {
        const int f0 = (item % tiles_f) * kWqF;
        for (int kb = 0; kb < nkb; ++kb, ++ic) {
          const int s = ic % kWqCStages;
          if (ic >= kWqCStages && !wait(&cempty[s], ((uint32_t)(ic / kWqCStages) & 1u) ^ 1u, kErrTimeoutEmpty)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&cfull[s], (uint32_t)(L::C_BYTES + L::SC_BYTES));
          tma_load_2d(smem + L::OFF_C + s * L::C_BYTES, &tm_c, &cfull[s], kb * kWqK / (QT == 0 ? 1 : 2), f0);
          uint8_t* sc = smem + L::OFF_SC + s * L::SC_BYTES;
          if (args.nt) tma_load_2d(sc, &tm_sc, &cfull[s], f0, kb * 4);        // [4 k-blocks][128 f]
          else tma_load_2d(sc, &tm_sc, &cfull[s], kb * kWqK, f0 / 32);         // [4 f-blocks][128 k]
        }
      }
    }
  } else {
    // ------------------------------------------------------------ dequant into tensor memory
    // Thread = one feature row r of the A tile (lane of quarter q) and one half (32 k) of a stage.
    const int q = warp & 3, h = (warp - 2 - kWqEpiWarps) / 4;
    const int r = 32 * q + lane;
    const uint32_t lane_off = (uint32_t)(32 * q) << 16;
    int it = 0, ic = 0;
    bool ok = true;
    for (int item = blockIdx.x; item < ntiles && ok; item += gridDim.x) {
      const int f = (item % tiles_f) * kWqF + r;
      for (int kb = 0; kb < total; ++kb, ++it) {
        const int as = it % kWqAStages;
        uint32_t rg[16];
        if (kb >= nkb) {
          // extension: the 16 f16 of ext_b row f
          uint4 ca = make_uint4(0, 0, 0, 0), cb = ca;
          if (h == 0 && f < args.N) {
            const uint4* p = reinterpret_cast<const uint4*>(args.ext_b + (long)f * 64);
            ca = __ldg(p);
            cb = __ldg(p + 1);
          }
          rg[0] = ca.x; rg[1] = ca.y; rg[2] = ca.z; rg[3] = ca.w;
          rg[4] = cb.x; rg[5] = cb.y; rg[6] = cb.z; rg[7] = cb.w;
        } else {
          // the stage's codes and scales (TMA), dequantized into registers; each thread hands
          // the slot back to the codes producer before it waits for a free A stage
          const int cs = ic % kWqCStages;
          if (!wait(&cfull[cs], (uint32_t)(ic / kWqCStages) & 1u, kErrTimeoutFull)) { ok = false; break; }
          ++ic;
          wq_dequant<QT>(smem + L::OFF_C + cs * L::C_BYTES, smem + L::OFF_SC + cs * L::SC_BYTES, args.nt != 0, r, q, h,
                         rg);
          mbar_arrive(&cempty[cs]);
        }
        // a free A stage (the MMA that read it is done)
        if (it >= kWqAStages && !wait(&aempty[as], ((uint32_t)(it / kWqAStages) & 1u) ^ 1u, kErrTimeoutEmpty)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t dst = tA + (uint32_t)(as * (kWqK / 2)) + lane_off;
        if (kb >= nkb) {
          if (h == 0) {
            const uint32_t rr[8] = {rg[0], rg[1], rg[2], rg[3], rg[4], rg[5], rg[6], rg[7]};
            tmem_st8(dst, rr);
          }
        } else {
          tmem_st16_w(dst + (uint32_t)(16 * h), rg);
        }
        tmem_st_wait_w();
        tc_fence_before();
        mbar_arrive(&afull[as]);
      }
    }
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tbase, 512);
  }
}

}  // namespace sa3k
