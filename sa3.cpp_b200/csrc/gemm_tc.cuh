// gemm_tc.cuh -- the tcgen05 GEMM engine behind every contraction of the adapter-training path.
//
//   D[M x N] (f32, in TMEM) = sum_k Aop[m, k] * Bop[n, k]   (+ one optional K = 16 "extension")
//
// It replaces ggml's MUL_MAT / OUT_PROD for the calls of src/dit.h:107,120-121,132,136-137 and
// their backward (ggml_build_backward_expand at src/train_ckpt.h:400).  One CTA computes one
// 128 x BN output tile with a warp-specialized pipeline:
//
//   warp 0      TMA producer: A tile (f16) + B tile (f16) or the raw quantized B bytes + scales
//   warp 1      TMEM allocator and MMA issue (tcgen05.mma kind::f16, one elected lane)
//   warps 2-5   dequant stage (quantized B only): raw bytes -> f16 in the 128B-swizzled UMMA
//               layout, then the epilogue: tcgen05.ld of the accumulator -> scale/bias -> global
//
// Operand layouts in shared memory (f16, 128-byte swizzle, BK = 64 = one swizzle row):
//   K-major:  [rows][64] -- row r at r*128 B, 8-row groups of 1024 B (SBO = 1024);
//             advancing K by 16 moves the start address by 32 B.
//   MN-major: [64 k-rows][64 mn] atoms of 8 KB, atom j (mn 64j..) at j*8192 (LBO = 8192),
//             8-k-row groups at 1024 B (SBO = 1024); advancing K by 16 moves by 2048 B.
//
// B operand modes (BMODE):
//   0  f16 K-major via TMA  ([N][K] row-major in HBM)
//   1  f16 MN-major via TMA ([K][N] row-major in HBM)
//   2  Q8_0 "NT": W[out = N][in = K] quantized along K, dequantized K-major      (forward)
//   3  Q8_0 "TN": W[out = K][in = N] quantized along N, dequantized MN-major     (dX = W^T dy)
//   4  Q4_K "NT", 5  Q4_K "TN": as 2 / 3 with 4-bit codes.
// Quantized weights live in HBM repacked by quant.cu: int8 codes (Q8_0) or natural-order nibble
// pairs (Q4_K) as [out][in], and per-32-element scales as [in/32][out] f32 (Q8_0: d) or
// float2 (Q4_K: d*sc, dmin*m) -- the same numbers the GGUF blocks encode, so the dequantized
// values are bit-identical to ggml's to_float (then rounded once to f16 for the tensor core).
#pragma once

#include "sa3k_common.cuh"
#include "sa3k_internal.h"

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
  __half* out_h;    // f16 output (nullable): h_scale * the value written to out
  long ldo_h;
  int out_h_trans;
  float h_scale;
  __half* out_h_t;  // second f16 output, transposed: out_h_t[n * ldo_h_t + m] (nullable)
  long ldo_h_t;
  int splits;               // split-K: work item = (tile, split); 1 = no split
  int kb_per_split;         // 64-wide k-blocks per split
  float* partial;           // split-K: raw f32 partial sums [splits][M][N]; the CTA that finishes a
                            //   tile's last split sums them in split order and runs the epilogue
  int* tile_cnt;            // split-K: per-tile count of finished splits (zero between launches)
  int tail_t0;              // tail split: tiles [tail_t0, ntiles) (the last, partial round) run as
  int tail_parts;           //   tail_parts K ranges of tail_kbps k-blocks each, added into the
  int tail_kbps;            //   output (pre-zeroed unless accumulating); tail_parts <= 1: off
  int tma_out;              // 1: f32 `out` via TMA store / reduce-add; 2: f16 `out_h` via TMA
                            //    store; 0: direct stores (split-K partials, transposed or dual outputs)
  int atomic;               // split-K: every split adds its (scaled) part into `out` with atomics
  int has_hp;               // the fused head preparation below applies (CTA-pair kernel)
  HeadPrepEpi hp;
  int* err;                 // device error word
};

constexpr int kBM = 128, kBK = 64;

// A work item of the persistent GEMM kernels: tile t and its K range [kb0, kb0 + nkb) of 64-wide
// k-blocks; total adds the K = 16 extension stage to the last range.  Items [0, tail_t0) are
// whole tiles; with a tail split the remaining tiles are each split into tail_parts ranges
// (every CTA then gets about the same work); with split-K item = split * ntiles + tile.
struct WorkItem {
  int t, kb0, nkb, total;
  bool first;   // the range that adds the bias
  bool add;     // tail part: add into the output
};

template <typename Args>
__device__ __forceinline__ WorkItem decode_item(const Args& a, int item, int ntiles, int nkb_all) {
  WorkItem w;
  bool last;
  if (a.tail_parts > 1 && item >= a.tail_t0) {
    const int j = item - a.tail_t0, part = j % a.tail_parts;
    w.t = a.tail_t0 + j / a.tail_parts;
    w.kb0 = part * a.tail_kbps;
    w.nkb = min(nkb_all - w.kb0, a.tail_kbps);
    w.first = part == 0;
    last = part == a.tail_parts - 1;
    w.add = true;
  } else {
    const int split = item / ntiles;
    w.t = item % ntiles;
    w.kb0 = split * a.kb_per_split;
    w.nkb = min(nkb_all - w.kb0, a.kb_per_split);
    w.first = split == 0;
    last = split == a.splits - 1;
    w.add = false;
  }
  w.total = w.nkb + ((a.has_ext && last) ? 1 : 0);
  return w;
}

template <typename Args>
__device__ __forceinline__ int num_items(const Args& a, int ntiles) {
  return a.tail_parts > 1 ? a.tail_t0 + (ntiles - a.tail_t0) * a.tail_parts : ntiles * a.splits;
}
// the K = 16 extension's A tile: 128 rows of u^T as two 64 (M) x 16 (K) MN-major boxes
constexpr int kExtABytes = 128 * 16 * 2;

template <int BMODE>
struct BModeTraits {
  static constexpr bool quant = BMODE >= 2;
  static constexpr bool mn = (BMODE == 1 || BMODE == 3 || BMODE == 5);
  static constexpr bool q8 = (BMODE == 2 || BMODE == 3);
  static constexpr bool q4 = (BMODE == 4 || BMODE == 5);
};

__host__ __device__ constexpr int align_up(int x, int a) { return (x + a - 1) / a * a; }

// Warp roles: 0 TMA producer, 1 TMEM owner + MMA issuer, then the epilogue warps (8 for f16
// operands: two per TMEM lane quarter, splitting the accumulator columns; 4 with the dequant
// stage), then the dequant warps (quantized B only).
template <int BMODE>
struct GemmRoles {
  static constexpr int EPI_WARPS = BModeTraits<BMODE>::quant ? 4 : 8;
  static constexpr int DQ_WARPS = BModeTraits<BMODE>::quant ? 8 : 0;
  static constexpr int THREADS = 32 * (2 + EPI_WARPS + DQ_WARPS);
  static constexpr int DQ_THREADS = 32 * DQ_WARPS;
};

template <int BN, int STAGES, int BMODE>
struct GemmSmem {
  static constexpr int EPI_WARPS = GemmRoles<BMODE>::EPI_WARPS;
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
  // epilogue: 4 KB staging buffers per epilogue warp (32 rows x 128 B, 128B-swizzled), the
  // source of the TMA stores (or of the coalescing transpose on the direct path)
  static constexpr int OFF_STAGE = align_up(OFF_SC + STAGES * SC_STRIDE, 1024);
  static constexpr int STAGE_BYTES = 4096;
  // two staging buffers per warp when they fit next to the pipeline stages, else one
  static constexpr int STAGE_BUFS =
      (OFF_STAGE + EPI_WARPS * 2 * STAGE_BYTES + (3 * STAGES + 4) * 8 + 16 + 1024 <= 232448) ? 2 : 1;
  static constexpr int OFF_BAR = OFF_STAGE + EPI_WARPS * STAGE_BUFS * STAGE_BYTES;
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
// NT threads of the dequant warps each write BN*8/NT 16-byte chunks (8 f16) of the B stage.

// Codes to f32 without the int-to-float conversion unit (a quarter-rate pipe): a byte c placed in
// the low mantissa byte of 2^23 (bits 0x4B0000cc, one byte permute) is the float 2^23 + c
// exactly, and subtracting the bias recovers the code exactly, so the products below round once,
// like the f32 multiply of the reference dequantization.
__device__ __forceinline__ float magic_code(uint32_t w, int b) {
  return __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7540u + (uint32_t)b));
}

// 8 int8 codes (two words) times the block scale s: the signed codes are biased by 128 (an xor of
// the sign bits) so that each byte is 0 .. 255, then 2^23 + 128 is subtracted.
__device__ __forceinline__ uint4 q8_chunk(uint2 q, float s) {
  const uint32_t w[2] = {q.x ^ 0x80808080u, q.y ^ 0x80808080u};
  const uint64_t bias = f2(-8388736.0f, -8388736.0f), sc = f2(s, s);
  uint32_t o[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const uint32_t ww = w[k >> 1];
    const int b = 2 * (k & 1);
    float lo, hi;
    f2split(fmul2(fadd2(f2(magic_code(ww, b), magic_code(ww, b + 1)), bias), sc), lo, hi);
    o[k] = pack_f16x2(lo, hi);
  }
  return make_uint4(o[0], o[1], o[2], o[3]);
}

__device__ __forceinline__ uint4 q4_chunk(uint32_t nib, float d, float m) {
  // nib holds 8 codes, element 2b in the low nibble of byte b, 2b+1 in the high nibble;
  // d*q is exact in f32 (<= 21 significant bits), so the FMA below rounds exactly like ggml's
  // separate multiply and subtract.
  const uint32_t lo4 = nib & 0x0F0F0F0Fu, hi4 = (nib >> 4) & 0x0F0F0F0Fu;
  const uint64_t bias = f2(-8388608.0f, -8388608.0f), dd = f2(d, d), mm = f2(-m, -m);
  uint32_t o[4];
#pragma unroll
  for (int b = 0; b < 4; ++b) {   // elements 2b (low nibble) and 2b + 1 (high nibble)
    float v0, v1;
    f2split(ffma2(dd, fadd2(f2(magic_code(lo4, b), magic_code(hi4, b)), bias), mm), v0, v1);
    o[b] = pack_f16x2(v0, v1);
  }
  return make_uint4(o[0], o[1], o[2], o[3]);
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

// ------------------------------------------------------------------ split-K completion
// The tile [m0, m0 + rows) x [n0, n0 + cols) of out = epilogue(alpha * sum_s partial[s]), summed in
// split order (deterministic) by the nt threads tid = 0 .. nt-1.  Partials are read from L2
// (__ldcg: other CTAs wrote them).  Four columns per thread when N % 4 == 0 (n0 is a multiple of
// the N tile); the mapping is column-fastest for row-major outputs (coalesced partial reads and
// output writes) and row-fastest when an output is transposed.
__device__ __forceinline__ void splitk_finish(const GemmArgs& args, int m0, int n0, int rows, int cols, int tid,
                                              int nt) {
  const long mn = (long)args.M * args.N;
  const bool trans = args.out_trans || args.out_h_trans || args.out_h_t;
  const int vw = (args.N % 4 == 0) ? 4 : 1;
  const int cg = (cols + vw - 1) / vw;
  for (int e = tid; e < rows * cg; e += nt) {
    const int r = trans ? e % rows : e / cg, cq = trans ? e / rows : e % cg;
    const int row = m0 + r, col0 = n0 + vw * cq;
    const float* src = args.partial + (long)row * args.N + col0;
    float x[4] = {0.f, 0.f, 0.f, 0.f};
    if (vw == 4) {
#pragma unroll 4
      for (int sp = 0; sp < args.splits; ++sp) {
        const float4 p = __ldcg(reinterpret_cast<const float4*>(src + sp * mn));
        x[0] += p.x; x[1] += p.y; x[2] += p.z; x[3] += p.w;
      }
    } else {
#pragma unroll 4
      for (int sp = 0; sp < args.splits; ++sp) x[0] += __ldcg(src + sp * mn);
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int col = col0 + u;
      if (u >= vw || col >= n0 + cols) break;
      float v = x[u] * args.alpha;
      if (args.col_scale) v *= args.col_scale[col];
      if (args.col_bias) v += args.col_bias[col];
      if (args.out) {
        float* dst = args.out_trans ? args.out + (long)col * args.ldo + row : args.out + (long)row * args.ldo + col;
        *dst = args.accumulate ? *dst + v : v;
      }
      if (args.out_h) {
        __half* dst = args.out_h_trans ? args.out_h + (long)col * args.ldo_h + row
                                               : args.out_h + (long)row * args.ldo_h + col;
        *dst = __float2half_rn(v * args.h_scale);
      }
      if (args.out_h_t) args.out_h_t[(long)col * args.ldo_h_t + row] = __float2half_rn(v);
    }
  }
}

// The same for a 16-wide output (N = 16): thread `tid` < rows owns one row and loads every
// split's 16 partial sums (64 contiguous bytes each).  This path runs once per tile, so its code
// is kept small (cold instruction fetches dominate otherwise): the finished row goes through the
// thread's shared-memory slot `stage` (16 floats) and is written by one short loop.
__device__ __forceinline__ void splitk_finish_rows16(const GemmArgs& args, int m0, int rows, int tid, float* stage) {
  if (tid >= rows) return;
  const long mn4 = (long)args.M * args.N / 4;
  const int row = m0 + tid;
  const float4* src = reinterpret_cast<const float4*>(args.partial + (long)row * args.N);
  float4 x0 = make_float4(0.f, 0.f, 0.f, 0.f), x1 = x0, x2 = x0, x3 = x0;
#pragma unroll 1
  for (int sp = 0; sp < args.splits; ++sp) {
    const float4* s = src + sp * mn4;
    const float4 p0 = __ldcg(s), p1 = __ldcg(s + 1), p2 = __ldcg(s + 2), p3 = __ldcg(s + 3);
    x0.x += p0.x; x0.y += p0.y; x0.z += p0.z; x0.w += p0.w;
    x1.x += p1.x; x1.y += p1.y; x1.z += p1.z; x1.w += p1.w;
    x2.x += p2.x; x2.y += p2.y; x2.z += p2.z; x2.w += p2.w;
    x3.x += p3.x; x3.y += p3.y; x3.z += p3.z; x3.w += p3.w;
  }
  float4* st = reinterpret_cast<float4*>(stage);
  st[0] = x0; st[1] = x1; st[2] = x2; st[3] = x3;
#pragma unroll 1
  for (int col = 0; col < 16; ++col) {
    float v = stage[col] * args.alpha;
    if (args.col_scale) v *= args.col_scale[col];
    if (args.col_bias) v += args.col_bias[col];
    if (args.out) {
      float* dst = args.out_trans ? args.out + (long)col * args.ldo + row : args.out + (long)row * args.ldo + col;
      *dst = args.accumulate ? *dst + v : v;
    }
    if (args.out_h) {
      __half* dst = args.out_h_trans ? args.out_h + (long)col * args.ldo_h + row
                                             : args.out_h + (long)row * args.ldo_h + col;
      *dst = __float2half_rn(v * args.h_scale);
    }
    if (args.out_h_t) args.out_h_t[(long)col * args.ldo_h_t + row] = __float2half_rn(v);
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
                   const __grid_constant__ GemmArgs args) {
  using T = BModeTraits<BMODE>;
  using L = GemmSmem<BN, STAGES, BMODE>;
  using R = GemmRoles<BMODE>;
  static_assert(BN % 16 == 0 && BN >= 16 && BN <= 256, "UMMA M=128 needs N % 16 == 0, 16..256");
  static_assert(!T::mn || BN % 64 == 0, "MN-major B tiles are built from 64-wide atoms");

  extern __shared__ uint8_t smem_raw[];
  pdl_trigger();   // the next kernel may be scheduled once every CTA of this grid runs
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
  const int nitems = num_items(args, ntiles);
  const int nkb_all = (args.K + kBK - 1) / kBK;   // a ragged last block reads TMA zero fill

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
  pdl_wait();      // outputs of earlier kernels are read only from here on

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
        const WorkItem w = decode_item(args, item, ntiles, nkb_all);
        const int m0 = (w.t % tiles_m) * kBM, n0 = (w.t / tiles_m) * BN;
        const int kb0 = w.kb0, nkb = w.nkb, total = w.total;
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
            // K = 16 extension: u^T rows m0 .. m0 + 127 as two MN-major 64 x 16 boxes, B ext tile
            mbar_arrive_expect_tx(&full[s], (uint32_t)(kExtABytes + L::B_BYTES));
            tma_load_2d(a_st, &tm_ea, &full[s], m0, 0);
            tma_load_2d(a_st + kExtABytes / 2, &tm_ea, &full[s], m0 + 64, 0);
            tma_load_2d(b_st, &tm_eb, &full[s], 0, n0);
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    // The whole warp runs the loop with warp-uniform values and one elected lane issues each
    // tcgen05 instruction.  Descriptors are built once; the start-address field (bits 0-13,
    // address >> 4) is advanced by adding the byte offset >> 4 (shared addresses stay below
    // 2^18, so the field never carries into the next one).
    const WaiterW<> wt{abort_flag, args.err};
    const uint32_t idesc = make_idesc_f16(kBM, BN, A_MN ? 1 : 0, T::mn ? 1 : 0);
    const uint32_t idesc_ext = make_idesc_f16(kBM, BN, 1, 0);   // A = u^T read MN-major
    const uint64_t adesc0 = A_MN ? make_sdesc(smem_u32(smem + L::OFF_A), 8192, 1024)
                                 : make_sdesc(smem_u32(smem + L::OFF_A), 16, 1024);
    const uint64_t bdesc0 = T::mn ? make_sdesc(smem_u32(smem + L::OFF_B), 8192, 1024)
                                  : make_sdesc(smem_u32(smem + L::OFF_B), 16, 1024);
    const uint64_t bdesc0_k = make_sdesc(smem_u32(smem + L::OFF_B), 16, 1024);
    const uint64_t adesc0_ext = make_sdesc(smem_u32(smem + L::OFF_A), kExtABytes / 2, 1024);
    constexpr uint32_t A_KSTEP = A_MN ? 2048 >> 4 : 32 >> 4;
    constexpr uint32_t B_KSTEP = T::mn ? 2048 >> 4 : 32 >> 4;
    int it = 0, ti = 0;
    bool ok = true;
    for (int item = blockIdx.x; item < nitems && ok; item += gridDim.x, ++ti) {
      const WorkItem w = decode_item(args, item, ntiles, nkb_all);
      const int nkb = w.nkb, total = w.total;
      const int a = ti & 1;
      const uint32_t ause = (uint32_t)(ti >> 1);
      if (ti >= 2 && !wt(&tempty[a], (ause & 1u) ^ 1u, kErrTimeoutOther)) { ok = false; break; }
      tc_fence_after();
      const uint32_t d_tmem = tbase + (uint32_t)(a * L::ACC_COLS);
      for (int kb = 0; kb < total; ++kb, ++it) {
        const int s = it % STAGES;
        const uint32_t use = (uint32_t)(it / STAGES);
        if (!wt(&full[s], use & 1u, kErrTimeoutFull)) { ok = false; break; }
        if (T::quant && !wt(&bready[s], use & 1u, kErrTimeoutReady)) { ok = false; break; }
        tc_fence_after();
        const uint32_t aoff = (uint32_t)(s * L::A_BYTES) >> 4, boff = (uint32_t)(s * L::B_BYTES) >> 4;
        if (kb < nkb) {
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk)
            umma_f16_w(d_tmem, adesc0 + aoff + kk * A_KSTEP, bdesc0 + boff + kk * B_KSTEP, idesc,
                        (kb > 0 || kk > 0) ? 1u : 0u);
        } else {
          umma_f16_w(d_tmem, adesc0_ext + aoff, bdesc0_k + boff, idesc_ext, total > 1 ? 1u : 0u);
        }
        umma_commit_w(&empty[s]);
      }
      if (ok) umma_commit_w(&tfull[a]);
    }
  } else if (warp < 2 + R::EPI_WARPS) {
    // ------------------------------------------------------------ epilogue
    // Each warp drains 32 TMEM lanes (32 output rows); with 8 epilogue warps the two warps of a
    // lane quarter take alternate column chunks.  TMA path (args.tma_out): 32 f32 (or 64 f16)
    // columns per step are written into a 128B-swizzled 32-row staging buffer and sent with one
    // asynchronous TMA store (reduce-add when accumulating); two buffers alternate when they fit.
    // Direct path: the same staging buffer transposes each 32 x 32 block so every global store
    // is one coalesced row segment; transposed outputs are already coalesced across lanes.
    const int q = warp & 3;   // TMEM lane quarter this warp may access
    constexpr int NH = R::EPI_WARPS / 4;   // warps per lane quarter
    const int half = (warp - 2) / 4;       // this warp's chunks: chunk % NH == half
    uint8_t* stg = smem + L::OFF_STAGE + (warp - 2) * L::STAGE_BUFS * L::STAGE_BYTES;
    const bool split_out = args.partial != nullptr;   // raw partial sums, reduced by the last split
    const int cstep = args.tma_out == 2 ? 64 : 32;
    volatile int* last_split = reinterpret_cast<volatile int*>(tmem_slot + 2);
    int nstore = 0;
    int ti = 0;
    for (int item = blockIdx.x; item < nitems; item += gridDim.x, ++ti) {
      const WorkItem w = decode_item(args, item, ntiles, nkb_all);
      const int t = w.t;
      // parts of a split tile add into the output; only the first part adds the bias
      const bool add = w.add || args.atomic;
      const float* bias = (w.first || !add) ? args.col_bias : nullptr;
      const int a = ti & 1;
      const uint32_t ause = (uint32_t)(ti >> 1);
      const int m0 = (t % tiles_m) * kBM, n0 = (t / tiles_m) * BN;
      const bool have = wait(&tfull[a], ause & 1u, kErrTimeoutAccum);
      tc_fence_after();
      const int rbase = m0 + 32 * q;               // first row of this warp
      const uint32_t tacc = tbase + (uint32_t)(a * L::ACC_COLS) + ((uint32_t)(32 * q) << 16);
#pragma unroll 1
      for (int c0 = half * cstep; c0 < BN; c0 += NH * cstep) {
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
          epi_columns(v, f + 32 * h, nb + 32 * h, args, split_out, bias);
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
              o.x = pack_f16x2(f[8 * c], f[8 * c + 1]);
              o.y = pack_f16x2(f[8 * c + 2], f[8 * c + 3]);
              o.z = pack_f16x2(f[8 * c + 4], f[8 * c + 5]);
              o.w = pack_f16x2(f[8 * c + 6], f[8 * c + 7]);
              *reinterpret_cast<uint4*>(buf + lane * 128 + ((c ^ (lane & 7)) << 4)) = o;
            }
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            if (args.accumulate || w.add) tma_reduce_add_2d(&tm_out, buf, nb, rbase);
            else tma_store_2d(&tm_out, buf, nb, rbase);
            bulk_commit();
          }
          ++nstore;
          continue;
        }
        // ---- direct path
        const int ncols = min(min(32, BN - c0), args.N - nb);
        const int myrow = rbase + lane;
        if (!split_out && myrow < args.M) {        // transposed outputs: lanes are consecutive rows
#pragma unroll
          for (int j = 0; j < 32; ++j) {           // static indices keep f[] in registers
            if (j >= ncols) break;
            if (args.out && args.out_trans) {
              float* dst = args.out + (long)(nb + j) * args.ldo + myrow;
              if (add) atomicAdd(dst, f[j]);
              else *dst = args.accumulate ? *dst + f[j] : f[j];
            }
            if (args.out_h && args.out_h_trans)
              args.out_h[(long)(nb + j) * args.ldo_h + myrow] = __float2half_rn(f[j] * args.h_scale);
            if (args.out_h_t) args.out_h_t[(long)(nb + j) * args.ldo_h_t + myrow] = __float2half_rn(f[j]);
          }
        }
        if (BN == 16 && split_out && args.N == 16) {
          // narrow tile: each lane stores its row's 16 partial sums as four 16-byte pieces
          if (myrow < args.M) {
            float4* dst = reinterpret_cast<float4*>(args.partial + (long)(item / ntiles) * args.M * args.N +
                                                    (long)myrow * args.N + nb);
#pragma unroll
            for (int c = 0; c < 4; ++c) dst[c] = make_float4(f[4 * c], f[4 * c + 1], f[4 * c + 2], f[4 * c + 3]);
          }
          continue;
        }
        if (split_out || (args.out && !args.out_trans) || (args.out_h && !args.out_h_trans)) {
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
              if (add) atomicAdd(dst, x);
              else *dst = args.accumulate ? *dst + x : x;
            }
            if (args.out_h && !args.out_h_trans)
              args.out_h[(long)row * args.ldo_h + nb + lane] = __float2half_rn(x * args.h_scale);
          }
          __syncwarp();
        }
      }
      if (split_out) {
        // ---- split-K: the CTA that completes the tile's last split reduces it.  Every thread
        // makes its partial stores visible, one thread counts the split in, and the last one
        // sums the splits in order 0, 1, ... (deterministic) from L2 and runs the epilogue.
        __threadfence();
        named_bar(1, 32 * R::EPI_WARPS);
        if (warp == 2 && lane == 0) {
          const int prev = atomicAdd(args.tile_cnt + t, 1);
          const int last = prev == args.splits - 1;
          if (last) args.tile_cnt[t] = 0;        // ready for the next launch
          *last_split = last;
        }
        named_bar(1, 32 * R::EPI_WARPS);
        if (*last_split) {
          __threadfence();
          if (BN == 16 && args.N == 16)
            splitk_finish_rows16(args, m0, min(kBM, args.M - m0), threadIdx.x - 64,
                                 reinterpret_cast<float*>(stg) + 16 * lane);
          else splitk_finish(args, m0, n0, min(kBM, args.M - m0), min(BN, args.N - n0), threadIdx.x - 64,
                             32 * R::EPI_WARPS);
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
        const WorkItem w = decode_item(args, item, ntiles, nkb_all);
        const int nkb = w.nkb, total = w.total;
        for (int kb = 0; kb < total; ++kb, ++it) {
          // Every stage use is observed (and acknowledged on bready), the extension stage too
          // (it is loaded as f16 by TMA and needs no work): skipping a phase would make the
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
