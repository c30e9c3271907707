// gemm_tc.cuh -- the tcgen05 GEMM engine behind every contraction of the adapter-training path.
//
//   D[M x N] (f32, in TMEM) = sum_k Aop[m, k] * Bop[n, k]   (+ one optional K = 16 "extension")
//
// It replaces ggml's MUL_MAT / OUT_PROD for the calls of src/dit.h:107,120-121,132,136-137 and
// their backward (ggml_build_backward_expand at src/train_ckpt.h:400).  One CTA computes one
// 128 x BN output tile with a warp-specialized pipeline:
//
//   warp 0      TMA producer: A tile (bf16) + B tile (bf16) or the raw quantized B bytes + scales
//   warp 1      TMEM allocator and the single MMA-issuing thread (tcgen05.mma kind::f16)
//   warps 2-5   dequant stage (quantized B only): raw bytes -> bf16 in the 128B-swizzled UMMA
//               layout, then the epilogue: tcgen05.ld of the accumulator -> scale/bias -> global
//
// Operand layouts in shared memory (bf16, 128-byte swizzle, BK = 64 = one swizzle row):
//   K-major:  [rows][64] -- row r at r*128 B, 8-row groups of 1024 B (SBO = 1024);
//             advancing K by 16 moves the start address by 32 B.
//   MN-major: [64 k-rows][64 mn] atoms of 8 KB, atom j (mn 64j..) at j*8192 (LBO = 8192),
//             8-k-row groups at 1024 B (SBO = 1024); advancing K by 16 moves by 2048 B.
//
// B operand modes (BMODE):
//   0  bf16 K-major via TMA  ([N][K] row-major in HBM)
//   1  bf16 MN-major via TMA ([K][N] row-major in HBM)
//   2  Q8_0 "NT": W[out = N][in = K] quantized along K, dequantized K-major      (forward)
//   3  Q8_0 "TN": W[out = K][in = N] quantized along N, dequantized MN-major     (dX = W^T dy)
//   4  Q4_K "NT", 5  Q4_K "TN": as 2 / 3 with 4-bit codes.
// Quantized weights live in HBM repacked by quant.cu: int8 codes (Q8_0) or natural-order nibble
// pairs (Q4_K) as [out][in], and per-32-element scales as [in/32][out] f32 (Q8_0: d) or
// float2 (Q4_K: d*sc, dmin*m) -- the same numbers the GGUF blocks encode, so the dequantized
// values are bit-identical to ggml's to_float (then rounded once to bf16 for the tensor core).
#pragma once

#include "sa3k_common.cuh"

namespace sa3k {

struct GemmArgs {
  int M, N, K;              // K: main reduction length (the last 64-block may be ragged)
  int has_ext;              // add one K = 16 MMA from the extension operands
  const float* col_scale;   // per-column multiplier (nullable)
  const float* col_bias;    // per-column bias, added after scaling (nullable)
  float alpha;              // global multiplier
  float* out;               // f32 output (nullable)
  long ldo;                 // its leading dimension (elements)
  int out_trans;            // 0: out[m*ldo + n]; 1: out[n*ldo + m]
  int accumulate;           // add into out instead of overwriting
  __nv_bfloat16* out_bf;    // bf16 output (nullable), same scale/bias as out
  long ldo_bf;
  int out_bf_trans;
  int splits;               // split-K: work item = (tile, split); 1 = no split
  int kb_per_split;         // 64-wide k-blocks per split
  float* partial;           // split-K: raw f32 partial sums [splits][M][N] (epilogue deferred)
  int tma_out;              // 1: f32 `out` via TMA store / reduce-add; 2: bf16 `out_bf` via TMA
                            //    store; 0: direct stores (split-K partials, transposed or dual outputs)
  int atomic;               // split-K: every split adds its (scaled) part into `out` with atomics
  int* err;                 // device error word
};

constexpr int kBM = 128, kBK = 64;

template <int BMODE>
struct BModeTraits {
  static constexpr bool quant = BMODE >= 2;
  static constexpr bool mn = (BMODE == 1 || BMODE == 3 || BMODE == 5);
  static constexpr bool q8 = (BMODE == 2 || BMODE == 3);
  static constexpr bool q4 = (BMODE == 4 || BMODE == 5);
};

__host__ __device__ constexpr int align_up(int x, int a) { return (x + a - 1) / a * a; }

// Warp roles: 0 TMA producer, 1 TMEM owner + MMA issuer, 2..5 epilogue, 6.. dequant (quant only).
template <int BMODE>
struct GemmRoles {
  static constexpr int EPI_WARPS = 4;
  static constexpr int DQ_WARPS = BModeTraits<BMODE>::quant ? 8 : 0;
  static constexpr int THREADS = 32 * (2 + EPI_WARPS + DQ_WARPS);
  static constexpr int DQ_THREADS = 32 * DQ_WARPS;
};

template <int BN, int STAGES, int BMODE>
struct GemmSmem {
  static constexpr int A_BYTES = kBM * kBK * 2;
  static constexpr int B_BYTES = BN * kBK * 2;
  static constexpr int RAW_BYTES =
      BModeTraits<BMODE>::q8 ? BN * kBK : BModeTraits<BMODE>::q4 ? BN * kBK / 2 : 0;
  static constexpr int SC_BYTES =
      BModeTraits<BMODE>::q8 ? BN * 2 * 4 : BModeTraits<BMODE>::q4 ? BN * 2 * 8 : 0;
  static constexpr int RAW_STRIDE = align_up(RAW_BYTES, 128);
  static constexpr int SC_STRIDE = align_up(SC_BYTES, 128);
  static constexpr int OFF_A = 0;
  static constexpr int OFF_B = OFF_A + STAGES * A_BYTES;
  static constexpr int OFF_RAW = OFF_B + STAGES * B_BYTES;
  static constexpr int OFF_SC = OFF_RAW + STAGES * RAW_STRIDE;
  // epilogue: two 4 KB staging buffers per epilogue warp (32 rows x 128 B, 128B-swizzled), the
  // source of the TMA stores (or of the coalescing transpose on the direct path)
  static constexpr int OFF_STAGE = align_up(OFF_SC + STAGES * SC_STRIDE, 1024);
  static constexpr int STAGE_BYTES = 4096;
  // two staging buffers per warp when they fit next to the pipeline stages, else one
  static constexpr int STAGE_BUFS = (OFF_STAGE + 4 * 2 * STAGE_BYTES + 1024 + 256 <= 232448) ? 2 : 1;
  static constexpr int OFF_BAR = OFF_STAGE + 4 * STAGE_BUFS * STAGE_BYTES;
  static constexpr int BAR_BYTES = (3 * STAGES + 4) * 8 + 16;
  static constexpr int TOTAL = OFF_BAR + BAR_BYTES;
  static constexpr int DYN = TOTAL + 1024;   // slack for 1024-byte alignment of the base
  static constexpr int ACC_COLS = BN < 32 ? 32 : BN;           // one accumulator buffer
  // double-buffered; the allocation is a power of two >= 32 columns
  static constexpr int TMEM_COLS = 2 * ACC_COLS <= 64 ? 64 : 2 * ACC_COLS <= 128 ? 128
                                 : 2 * ACC_COLS <= 256 ? 256 : 512;
  static_assert(2 * ACC_COLS <= 512, "two accumulators must fit the 512 TMEM columns");
  static_assert(DYN <= 232448, "shared memory budget (227 KB)");
};

// ------------------------------------------------------------------ dequantization stages
// NT threads of the dequant warps each write BN*8/NT 16-byte chunks (8 bf16) of the B stage.

__device__ __forceinline__ uint4 q8_chunk(uint2 q, float s) {
  uint4 o;
  const int8_t* qb = reinterpret_cast<const int8_t*>(&q);
  o.x = pack_bf16x2((float)qb[0] * s, (float)qb[1] * s);
  o.y = pack_bf16x2((float)qb[2] * s, (float)qb[3] * s);
  o.z = pack_bf16x2((float)qb[4] * s, (float)qb[5] * s);
  o.w = pack_bf16x2((float)qb[6] * s, (float)qb[7] * s);
  return o;
}

__device__ __forceinline__ uint4 q4_chunk(uint32_t nib, float d, float m) {
  // nib holds 8 codes, element 2b in the low nibble of byte b, 2b+1 in the high nibble;
  // d*q is exact in f32 (<= 21 significant bits), so the FMA below rounds exactly like ggml's
  // separate multiply and subtract.
  uint4 o;
  float v[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) v[e] = d * (float)((nib >> (4 * e)) & 0xFu) - m;
  o.x = pack_bf16x2(v[0], v[1]);
  o.y = pack_bf16x2(v[2], v[3]);
  o.z = pack_bf16x2(v[4], v[5]);
  o.w = pack_bf16x2(v[6], v[7]);
  return o;
}

// K-major destination chunk (row r, 16-byte column chunk c) of a [rows][64] 128B-swizzled tile.
__device__ __forceinline__ uint4* kmajor_chunk(uint8_t* bst, int r, int c) {
  return reinterpret_cast<uint4*>(bst + r * 128 + ((c ^ (r & 7)) << 4));
}

// MN-major destination chunk (k-row k, 8-element mn chunk cn) of [64 k][BN mn] atoms.
__device__ __forceinline__ uint4* mnmajor_chunk(uint8_t* bst, int k, int cn) {
  const int atom = cn >> 3, ch = cn & 7;
  return reinterpret_cast<uint4*>(bst + atom * 8192 + (k >> 3) * 1024 + (k & 7) * 128 + ((ch ^ (k & 7)) << 4));
}

template <int BN, int BMODE, int NT>
__device__ __forceinline__ void dequant_stage(const uint8_t* raw, const uint8_t* sc, uint8_t* bst, int tid) {
  constexpr int PER = BN * 8 / NT;
  static_assert(BN * 8 % NT == 0, "dequant split");
#pragma unroll
  for (int j = 0; j < PER; ++j) {
    const int idx = tid + NT * j;
    if (BMODE == 2) {          // Q8_0 NT: raw [BN][64] int8, sc [2][BN] f32
      const int r = idx >> 3, c = idx & 7;
      const uint2 q = *reinterpret_cast<const uint2*>(raw + r * 64 + c * 8);
      *kmajor_chunk(bst, r, c) = q8_chunk(q, reinterpret_cast<const float*>(sc)[(c >> 2) * BN + r]);
    } else if (BMODE == 3) {   // Q8_0 TN: raw [64][BN] int8, sc [BN/32][64] f32
      const int k = idx / (BN / 8), cn = idx % (BN / 8);
      const uint2 q = *reinterpret_cast<const uint2*>(raw + k * BN + cn * 8);
      *mnmajor_chunk(bst, k, cn) = q8_chunk(q, reinterpret_cast<const float*>(sc)[(cn >> 2) * 64 + k]);
    } else if (BMODE == 4) {   // Q4_K NT: raw [BN][32] bytes, sc [2][BN] float2
      const int r = idx >> 3, c = idx & 7;
      const uint32_t nib = *reinterpret_cast<const uint32_t*>(raw + r * 32 + c * 4);
      const float2 s = reinterpret_cast<const float2*>(sc)[(c >> 2) * BN + r];
      *kmajor_chunk(bst, r, c) = q4_chunk(nib, s.x, s.y);
    } else if (BMODE == 5) {   // Q4_K TN: raw [64][BN/2] bytes, sc [BN/32][64] float2
      const int k = idx / (BN / 8), cn = idx % (BN / 8);
      const uint32_t nib = *reinterpret_cast<const uint32_t*>(raw + k * (BN / 2) + cn * 4);
      const float2 s = reinterpret_cast<const float2*>(sc)[(cn >> 2) * 64 + k];
      *mnmajor_chunk(bst, k, cn) = q4_chunk(nib, s.x, s.y);
    }
  }
}

// ------------------------------------------------------------------ split-K reduction
// out = epilogue(alpha * sum_s partial[s]) with the same column scale / bias / accumulate /
// transpose / bf16 options as the GEMM epilogue.  Deterministic (fixed summation order).
__global__ void splitk_reduce_kernel(const GemmArgs args) {
  const long mn = (long)args.M * args.N;
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < mn; i += (long)gridDim.x * blockDim.x) {
    const int m = (int)(i / args.N), n = (int)(i % args.N);
    float x = 0.f;
    for (int sp = 0; sp < args.splits; ++sp) x += args.partial[(long)sp * mn + i];
    x *= args.alpha;
    if (args.col_scale) x *= args.col_scale[n];
    if (args.col_bias) x += args.col_bias[n];
    if (args.out) {
      float* dst = args.out_trans ? args.out + (long)n * args.ldo + m : args.out + (long)m * args.ldo + n;
      *dst = args.accumulate ? *dst + x : x;
    }
    if (args.out_bf) {
      __nv_bfloat16* dst = args.out_bf_trans ? args.out_bf + (long)n * args.ldo_bf + m : args.out_bf + (long)m * args.ldo_bf + n;
      *dst = __float2bfloat16_rn(x);
    }
  }
}

// ------------------------------------------------------------------ epilogue arithmetic
// f[j] = acc[j] * (alpha * col_scale[n0 + j]) + col_bias[n0 + j] for 32 accumulator columns
// (raw sums for split-K partials).  Column vectors are read 4 at a time (the same addresses for
// every lane of the warp: broadcast loads).
__device__ __forceinline__ void epi_columns(const uint32_t (&v)[32], float* f, int n0, const GemmArgs& args,
                                            bool raw, const float* col_bias) {
  if (raw || !(args.col_scale || col_bias)) {
    const float al = raw ? 1.f : args.alpha;
#pragma unroll
    for (int j = 0; j < 32; ++j) f[j] = __uint_as_float(v[j]) * al + 0.f;
  } else if (n0 + 32 <= args.N) {
#pragma unroll
    for (int j = 0; j < 32; j += 4) {
      float4 s4 = make_float4(1.f, 1.f, 1.f, 1.f), b4 = make_float4(0.f, 0.f, 0.f, 0.f);
      if (args.col_scale) s4 = __ldg(reinterpret_cast<const float4*>(args.col_scale + n0 + j));
      if (col_bias) b4 = __ldg(reinterpret_cast<const float4*>(col_bias + n0 + j));
      f[j] = __uint_as_float(v[j]) * (args.alpha * s4.x) + b4.x;
      f[j + 1] = __uint_as_float(v[j + 1]) * (args.alpha * s4.y) + b4.y;
      f[j + 2] = __uint_as_float(v[j + 2]) * (args.alpha * s4.z) + b4.z;
      f[j + 3] = __uint_as_float(v[j + 3]) * (args.alpha * s4.w) + b4.w;
    }
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      const int n = n0 + j;
      float cs = args.alpha, cb = 0.f;
      if (n < args.N) {
        if (args.col_scale) cs *= args.col_scale[n];
        if (col_bias) cb = col_bias[n];
      }
      f[j] = __uint_as_float(v[j]) * cs + cb;
    }
  }
}

// ------------------------------------------------------------------ the kernel
// Persistent: gridDim.x CTAs walk the work items blockIdx.x, blockIdx.x + gridDim.x, ...; an item
// is an output tile t (m-tile t % tiles_m, n-tile t / tiles_m, so co-resident CTAs share B
// columns) and, with split-K, one K-range of it.
// The accumulator is double-buffered in TMEM: the epilogue drains tile i while the MMA warp
// accumulates tile i + 1.
template <int BN, int STAGES, int BMODE, bool A_MN>
__global__ void __launch_bounds__(GemmRoles<BMODE>::THREADS, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b,
                   const __grid_constant__ CUtensorMap tm_bs, const __grid_constant__ CUtensorMap tm_ea,
                   const __grid_constant__ CUtensorMap tm_eb, const __grid_constant__ CUtensorMap tm_out,
                   const GemmArgs args) {
  using T = BModeTraits<BMODE>;
  using L = GemmSmem<BN, STAGES, BMODE>;
  using R = GemmRoles<BMODE>;
  static_assert(BN % 16 == 0 && BN >= 16 && BN <= 256, "UMMA M=128 needs N % 16 == 0, 16..256");
  static_assert(!T::mn || BN % 64 == 0, "MN-major B tiles are built from 64-wide atoms");

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::OFF_BAR);
  uint64_t* empty = full + STAGES;
  uint64_t* bready = empty + STAGES;
  uint64_t* tfull = bready + STAGES;     // [2] accumulator ready for the epilogue
  uint64_t* tempty = tfull + 2;          // [2] accumulator drained by the epilogue
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tiles_m = (args.M + kBM - 1) / kBM;
  const int tiles_n = (args.N + BN - 1) / BN;
  const int ntiles = tiles_m * tiles_n;
  const int nitems = ntiles * args.splits;
  const int nkb_all = (args.K + kBK - 1) / kBK;   // a ragged last block reads TMA zero fill
  // item -> (tile, split); split s covers k-blocks [s*kps, min(nkb_all, (s+1)*kps)) and the last
  // split also runs the K = 16 extension
  auto item_kb = [&](int item, int& kb0, int& nkb, int& total) {
    const int split = item / ntiles;
    kb0 = split * args.kb_per_split;
    nkb = min(nkb_all - kb0, args.kb_per_split);
    total = nkb + ((args.has_ext && split == args.splits - 1) ? 1 : 0);
  };

  if (warp == 0 && lane == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
      mbar_init(&bready[s], R::DQ_THREADS > 0 ? R::DQ_THREADS : 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 32 * R::EPI_WARPS);
    }
    *abort_flag = 0;
    fence_barrier_init();
    fence_proxy_async_smem();
    tma_prefetch_desc(&tm_a);
    tma_prefetch_desc(&tm_b);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, L::TMEM_COLS);
    tmem_relinquish();
    tc_fence_before();
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tmem_slot;

  auto wait = [&](uint64_t* bar, uint32_t parity, int code) -> bool {
    if (*abort_flag) return false;
    const uint32_t a = smem_u32(bar);
    if (mbar_try_wait(a, parity)) return true;
    const unsigned long long t0 = globaltimer();
    for (uint32_t i = 1;; ++i) {
      if (mbar_try_wait(a, parity)) return true;
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
      for (int item = blockIdx.x; item < nitems && ok; item += gridDim.x) {
        const int t = item % ntiles;
        const int m0 = (t % tiles_m) * kBM, n0 = (t / tiles_m) * BN;
        int kb0, nkb, total;
        item_kb(item, kb0, nkb, total);
        for (int kb = 0; kb < total; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t use = (uint32_t)(it / STAGES);
          if (it >= STAGES && !wait(&empty[s], (use & 1u) ^ 1u, kErrTimeoutEmpty)) { ok = false; break; }
          uint8_t* a_st = smem + L::OFF_A + s * L::A_BYTES;
          uint8_t* b_st = smem + L::OFF_B + s * L::B_BYTES;
          if (kb < nkb) {
            const int k0 = (kb0 + kb) * kBK;
            const uint32_t bbytes = T::quant ? (uint32_t)(L::RAW_BYTES + L::SC_BYTES) : (uint32_t)L::B_BYTES;
            mbar_arrive_expect_tx(&full[s], (uint32_t)L::A_BYTES + bbytes);
            if (A_MN) {
              tma_load_2d(a_st, &tm_a, &full[s], m0, k0);
              tma_load_2d(a_st + 8192, &tm_a, &full[s], m0 + 64, k0);
            } else {
              tma_load_2d(a_st, &tm_a, &full[s], k0, m0);
            }
            uint8_t* raw = smem + L::OFF_RAW + s * L::RAW_STRIDE;
            uint8_t* sc = smem + L::OFF_SC + s * L::SC_STRIDE;
            if (BMODE == 0) {
              tma_load_2d(b_st, &tm_b, &full[s], k0, n0);
            } else if (BMODE == 1) {
#pragma unroll
              for (int j = 0; j < BN / 64; ++j) tma_load_2d(b_st + j * 8192, &tm_b, &full[s], n0 + 64 * j, k0);
            } else if (BMODE == 2) {
              tma_load_2d(raw, &tm_b, &full[s], k0, n0);
              tma_load_2d(sc, &tm_bs, &full[s], n0, k0 / 32);
            } else if (BMODE == 3) {
              tma_load_2d(raw, &tm_b, &full[s], n0, k0);
              tma_load_2d(sc, &tm_bs, &full[s], k0, n0 / 32);
            } else if (BMODE == 4) {
              tma_load_2d(raw, &tm_b, &full[s], k0 / 2, n0);
              tma_load_2d(sc, &tm_bs, &full[s], n0, k0 / 32);
            } else {
              tma_load_2d(raw, &tm_b, &full[s], n0 / 2, k0);
              tma_load_2d(sc, &tm_bs, &full[s], k0, n0 / 32);
            }
          } else {
            mbar_arrive_expect_tx(&full[s], (uint32_t)(L::A_BYTES + L::B_BYTES));
            tma_load_2d(a_st, &tm_ea, &full[s], 0, m0);
            tma_load_2d(b_st, &tm_eb, &full[s], 0, n0);
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t idesc = make_idesc_bf16(kBM, BN, A_MN ? 1 : 0, T::mn ? 1 : 0);
      const uint32_t idesc_ext = make_idesc_bf16(kBM, BN, 0, 0);
      int it = 0, ti = 0;
      bool ok = true;
      for (int item = blockIdx.x; item < nitems && ok; item += gridDim.x, ++ti) {
        int kb0, nkb, total;
        item_kb(item, kb0, nkb, total);
        const int a = ti & 1;
        const uint32_t ause = (uint32_t)(ti >> 1);
        if (ti >= 2 && !wait(&tempty[a], (ause & 1u) ^ 1u, kErrTimeoutOther)) { ok = false; break; }
        tc_fence_after();
        const uint32_t d_tmem = tbase + (uint32_t)(a * L::ACC_COLS);
        for (int kb = 0; kb < total; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t use = (uint32_t)(it / STAGES);
          if (!wait(&full[s], use & 1u, kErrTimeoutFull)) { ok = false; break; }
          if (T::quant && !wait(&bready[s], use & 1u, kErrTimeoutReady)) { ok = false; break; }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(smem + L::OFF_A + s * L::A_BYTES);
          const uint32_t b_addr = smem_u32(smem + L::OFF_B + s * L::B_BYTES);
          if (kb < nkb) {
#pragma unroll
            for (int kk = 0; kk < kBK / 16; ++kk) {
              const uint64_t ad = A_MN ? make_sdesc(a_addr + kk * 2048, 8192, 1024)
                                       : make_sdesc(a_addr + kk * 32, 16, 1024);
              const uint64_t bd = T::mn ? make_sdesc(b_addr + kk * 2048, 8192, 1024)
                                        : make_sdesc(b_addr + kk * 32, 16, 1024);
              umma_bf16(d_tmem, ad, bd, idesc, (kb > 0 || kk > 0) ? 1u : 0u);
            }
          } else {
            umma_bf16(d_tmem, make_sdesc(a_addr, 16, 1024), make_sdesc(b_addr, 16, 1024), idesc_ext,
                      total > 1 ? 1u : 0u);
          }
          umma_commit(&empty[s]);
        }
        if (ok) umma_commit(&tfull[a]);
      }
    }
  } else if (warp < 2 + R::EPI_WARPS) {
    // ------------------------------------------------------------ epilogue
    // Each warp drains its 32 TMEM lanes (32 output rows).  TMA path (args.tma_out): 32 f32 (or
    // 64 bf16) columns per step are written into a 128B-swizzled 32-row staging buffer and sent
    // with one asynchronous TMA store (reduce-add when accumulating); two buffers alternate.
    // Direct path: the same staging buffer transposes each 32 x 32 block so every global store
    // is one coalesced row segment; transposed outputs are already coalesced across lanes.
    const int q = warp & 3;   // TMEM lane quarter this warp may access
    uint8_t* stg = smem + L::OFF_STAGE + (warp - 2) * L::STAGE_BUFS * L::STAGE_BYTES;
    const bool split_out = args.partial != nullptr;   // raw partial sums (reduced by a second pass)
    const int cstep = args.tma_out == 2 ? 64 : 32;
    int nstore = 0;
    int ti = 0;
    for (int item = blockIdx.x; item < nitems; item += gridDim.x, ++ti) {
      const int t = item % ntiles;
      const int a = ti & 1;
      const uint32_t ause = (uint32_t)(ti >> 1);
      const int m0 = (t % tiles_m) * kBM, n0 = (t / tiles_m) * BN;
      const bool have = wait(&tfull[a], ause & 1u, kErrTimeoutAccum);
      tc_fence_after();
      const int rbase = m0 + 32 * q;               // first row of this warp
      const uint32_t tacc = tbase + (uint32_t)(a * L::ACC_COLS) + ((uint32_t)(32 * q) << 16);
#pragma unroll 1
      for (int c0 = 0; c0 < BN; c0 += cstep) {
        float f[64];
        const int nb = n0 + c0;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          if (h == 1 && cstep == 32) break;
          const int cc = c0 + 32 * h;
          uint32_t v[32];
          if (BN - cc >= 32) {
            tmem_ld32(tacc + (uint32_t)cc, v);
          } else {
            tmem_ld16(tacc + (uint32_t)cc, *reinterpret_cast<uint32_t(*)[16]>(&v[0]));
          }
          tmem_ld_wait();
          // with atomic split-K every split adds its scaled part; only split 0 adds the bias
          epi_columns(v, f + 32 * h, nb + 32 * h, args, split_out,
                      (args.atomic && item >= ntiles) ? nullptr : args.col_bias);
        }
        if (!have || nb >= args.N) continue;
        if (args.tma_out) {
          // ---- TMA store path: swizzled staging (16-byte chunk c of row r at c ^ (r & 7))
          uint8_t* buf = stg + (L::STAGE_BUFS == 2 ? (nstore & 1) : 0) * L::STAGE_BYTES;
          if (nstore >= L::STAGE_BUFS) {
            // the store that last used this buffer must have read it
            if (lane == 0) {
              if (L::STAGE_BUFS == 2) bulk_wait_read<1>();
              else bulk_wait_read<0>();
            }
            __syncwarp();
          }
          if (args.tma_out == 1) {
#pragma unroll
            for (int c = 0; c < 8; ++c)
              *reinterpret_cast<float4*>(buf + lane * 128 + ((c ^ (lane & 7)) << 4)) =
                  make_float4(f[4 * c], f[4 * c + 1], f[4 * c + 2], f[4 * c + 3]);
          } else {
#pragma unroll
            for (int c = 0; c < 8; ++c) {
              uint4 o;
              o.x = pack_bf16x2(f[8 * c], f[8 * c + 1]);
              o.y = pack_bf16x2(f[8 * c + 2], f[8 * c + 3]);
              o.z = pack_bf16x2(f[8 * c + 4], f[8 * c + 5]);
              o.w = pack_bf16x2(f[8 * c + 6], f[8 * c + 7]);
              *reinterpret_cast<uint4*>(buf + lane * 128 + ((c ^ (lane & 7)) << 4)) = o;
            }
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            if (args.accumulate) tma_reduce_add_2d(&tm_out, buf, nb, rbase);
            else tma_store_2d(&tm_out, buf, nb, rbase);
            bulk_commit();
          }
          ++nstore;
          continue;
        }
        // ---- direct path
        const int ncols = min(min(32, BN - c0), args.N - nb);
        const int myrow = rbase + lane;
        if (args.out && args.out_trans) {          // lanes are consecutive rows: coalesced
          if (myrow < args.M) {
#pragma unroll
            for (int j = 0; j < 32; ++j) {   // static indices keep f[] in registers
              if (j >= ncols) break;
              float* dst = args.out + (long)(nb + j) * args.ldo + myrow;
              if (args.atomic) atomicAdd(dst, f[j]);
              else *dst = args.accumulate ? *dst + f[j] : f[j];
            }
          }
        }
        if (args.out_bf && args.out_bf_trans) {
          if (myrow < args.M) {
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              if (j >= ncols) break;
              args.out_bf[(long)(nb + j) * args.ldo_bf + myrow] = __float2bfloat16_rn(f[j]);
            }
          }
        }
        if (split_out || (args.out && !args.out_trans) || (args.out_bf && !args.out_bf_trans)) {
          float* st32 = reinterpret_cast<float*>(stg);     // 32 x 32 f32, XOR-swizzled columns
#pragma unroll
          for (int j = 0; j < 32; ++j) st32[lane * 32 + (j ^ lane)] = f[j];
          __syncwarp();
          float* pbase = split_out ? args.partial + (long)(item / ntiles) * args.M * args.N : nullptr;
          for (int r = 0; r < 32; ++r) {
            const int row = rbase + r;
            if (row >= args.M || lane >= ncols) continue;
            const float x = st32[r * 32 + (lane ^ r)];
            if (split_out) {
              pbase[(long)row * args.N + nb + lane] = x;
              continue;
            }
            if (args.out && !args.out_trans) {
              float* dst = args.out + (long)row * args.ldo + nb + lane;
              if (args.atomic) atomicAdd(dst, x);
              else *dst = args.accumulate ? *dst + x : x;
            }
            if (args.out_bf && !args.out_bf_trans) args.out_bf[(long)row * args.ldo_bf + nb + lane] = __float2bfloat16_rn(x);
          }
          __syncwarp();
        }
      }
      tc_fence_before();
      mbar_arrive(&tempty[a]);
    }
    if (lane == 0) bulk_wait_all();       // staging buffers must outlive the in-flight stores
    __syncwarp();
  } else {
    // ------------------------------------------------------------ dequant warps (quant modes)
    if constexpr (T::quant) {
      const int tid = threadIdx.x - 32 * (2 + R::EPI_WARPS);
      int it = 0;
      bool ok = true;
      for (int item = blockIdx.x; item < nitems && ok; item += gridDim.x) {
        int kb0, nkb, total;
        item_kb(item, kb0, nkb, total);
        for (int kb = 0; kb < total; ++kb, ++it) {
          // Every stage use is observed (and acknowledged on bready), the extension stage too
          // (it is loaded as bf16 by TMA and needs no work): skipping a phase would make the
          // next parity wait on this barrier alias with an older phase.
          const int s = it % STAGES;
          const uint32_t use = (uint32_t)(it / STAGES);
          if (!wait(&full[s], use & 1u, kErrTimeoutFull)) { ok = false; break; }
          if (kb < nkb) {
            const uint8_t* raw = smem + L::OFF_RAW + s * L::RAW_STRIDE;
            const uint8_t* sc = smem + L::OFF_SC + s * L::SC_STRIDE;
            uint8_t* b_st = smem + L::OFF_B + s * L::B_BYTES;
            dequant_stage<BN, BMODE, R::DQ_THREADS>(raw, sc, b_st, tid);
            fence_proxy_async_smem();
          }
          mbar_arrive(&bready[s]);
        }
      }
    }
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tbase, L::TMEM_COLS);
  }
}

}  // namespace sa3k
