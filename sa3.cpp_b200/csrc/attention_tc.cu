// attention_tc.cu -- scaled-dot-product attention on the tcgen05 tensor cores, head_dim 64.
//
// Same contract as attention.cu (nn::sdpa, src/nn.h:135-144, with the band mask of
// src/same_ae.h:96-106): O = softmax(scale q k^T) v per (batch, head), the row log-sum-exp kept
// in log2 units, and the backward in two deterministic passes (no atomics):
//   dq pass   (CTA per 128 queries, loop over 64-key tiles):    dQ = scale dS K
//   dkdv pass (CTA per 128 keys, loop over 64-query tiles):     dV = P^T dO, dK = scale dS^T Q
// with P = exp2(s * scale * log2 e - lse), dP = dO V^T, dS = P o (dP - D), D = rowsum(dO o O).
//
// One CTA = 6 warps, two CTAs per SM (each holds 256 TMEM columns), so one CTA's softmax work
// overlaps the other's tensor-core work:
//   warp 0     TMA producer: the CTA's fixed tile once, then a ring of streamed tiles
//   warp 1     TMEM owner and the single thread issuing tcgen05.mma
//   warps 2-5  one thread per TMEM lane (= tile row): softmax / dS arithmetic on the f32
//              accumulators read with tcgen05.ld; P and dS go back into TMEM as packed bf16 and
//              feed the next MMA directly as its A operand (A from tensor memory)
// Tiles come in by TMA from the strided (batch, head, row) layout through 4-D tensor maps whose
// per-batch row extent zero-fills rows past the sequence; keys past Sk and outside the band are
// masked in the softmax.  Every wait is bounded (2 s), like the GEMM engine's.
#include "attention.h"
#include "sa3k_common.cuh"
#include "sa3k_internal.h"

#include <cmath>

namespace sa3k {
namespace {

constexpr float kLog2e = 1.4426950408889634f;

struct TcArgs {
  int B, H, Sq, Sk, window;
  float sl2;                 // scale * log2(e)
  float scale;
  int q_tm, k_tm, v_tm, o_tm, do_tm;   // tensor-map coordinate order: 1 = (d, h, s, b), 0 = (d, s, h, b)
  __nv_bfloat16* o; long o_sb, o_sh, o_ld;
  float* lse;                // forward output [B*H][Sq]
  const float* lse_in;       // backward input
  float* Dsum;               // [B*H][Sq]: written by the dq pass, read by the dk / dv pass
  float* dq; long dq_sb, dq_sh, dq_ld;
  float* dk; long dk_sb, dk_sh, dk_ld;
  float* dv; long dv_sb, dv_sh, dv_ld;
  int* err;
};

// ------------------------------------------------------------------------------ primitives
__device__ __forceinline__ void tma_load_4d(void* dst, const CUtensorMap* m, uint64_t* bar, int c0, int c1, int c2,
                                            int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
      : "memory");
}

// rows [row0, row0 + n) of head h of batch b (map coordinate order per `tm`)
__device__ __forceinline__ void load_rows(void* dst, const CUtensorMap* m, uint64_t* bar, int tm, int b, int h,
                                          int row0) {
  if (tm) tma_load_4d(dst, m, bar, 0, h, row0, b);
  else tma_load_4d(dst, m, bar, 0, row0, h, b);
}

// D (tmem) (+)= A (tmem, bf16 packed two per column) * B (smem descriptor)
__device__ __forceinline__ void umma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc,
                                        uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}

__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Packed pairs of f32 (sm_100 f32x2 arithmetic: two lanes of work per instruction).
__device__ __forceinline__ uint64_t f2(float a, float b) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ void f2split(uint64_t r, float& a, float& b) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(r));
}
__device__ __forceinline__ uint64_t ffma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t fadd2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t fmul2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}

// every (row, key) of a rows x keys tile is inside [0, Sk) and the band
__device__ __forceinline__ bool tile_visible(int r0, int nr, int k0, int nk, int Sk, int window) {
  if (k0 + nk > Sk) return false;
  if (window < 0) return true;
  return max(r0 + nr - 1 - k0, k0 + nk - 1 - r0) <= window;
}

// K-major [rows][64] bf16 tile (128-byte rows, 128B swizzle): descriptor at k-step kk (16 wide)
__device__ __forceinline__ uint64_t kdesc(uint32_t base, int kk) { return make_sdesc(base + kk * 32, 16, 1024); }
// the same tile read MN-major (its rows are the reduction index): 16 rows per k-step
__device__ __forceinline__ uint64_t mndesc(uint32_t base, int kk) { return make_sdesc(base + kk * 2048, 8192, 1024); }

struct Waiter {
  volatile int* abort_flag;
  int* err;
  __device__ __forceinline__ bool operator()(uint64_t* bar, uint32_t parity, int code) const {
    if (*abort_flag) return false;
    const uint32_t a = smem_u32(bar);
    if (mbar_try_wait(a, parity)) return true;
    const unsigned long long t0 = globaltimer();
    for (uint32_t i = 1;; ++i) {
      if (mbar_try_wait(a, parity)) return true;
      if ((i & 63u) == 0) {
        if (*abort_flag) return false;
        if (globaltimer() - t0 > kWaitLimitNs) {
          record_error(err, code);
          *abort_flag = 1;
          return false;
        }
      }
    }
  }
};

__device__ __forceinline__ bool visible(int qi, int kj, int Sk, int window) {
  return kj < Sk && (window < 0 || abs(qi - kj) <= window);
}

// [lo, hi) range of `tile`-sized tiles of the other side that rows [r0, r0 + n) can see
__device__ __forceinline__ void tile_range(int r0, int n, int other, int window, int tile, int& t0, int& t1) {
  t0 = 0;
  t1 = (other + tile - 1) / tile;
  if (window >= 0) {
    const int lo = r0 - window, hi = r0 + n - 1 + window;
    t0 = max(0, lo) / tile;
    t1 = min(t1, max(0, hi) / tile + 1);
    if (t1 < t0) t1 = t0;
  }
}

// Warp roles of all three kernels (10 warps): warp 0 TMA producer, warp 1 TMEM owner + MMA
// issuer, warps 2-5 = warpgroup 0 and warps 6-9 = warpgroup 1 of softmax threads (thread <->
// TMEM lane <-> tile row; warp w reaches lanes 32 (w % 4) .. +32).  Streamed tiles are 64 rows
// and sit in a 4-deep ring.  The two warpgroups keep the tensor core busy while they work: in
// the forward each owns its own 128-query tile; in the backward passes they take alternate
// streamed tiles and the MMA thread folds their results into one accumulator in tile order.
constexpr int kWarpsTC = 10;
// Each CTA holds all 512 TMEM columns; a shared-memory request above half the SM keeps a second
// CTA from being placed beside it (it would only wait in tcgen05.alloc).
constexpr int kSmemFloor = 120 * 1024;
constexpr int smem_req(int bytes) { return bytes + 1024 > kSmemFloor ? bytes + 1024 : kSmemFloor; }
constexpr int kThreadsTC = 32 * kWarpsTC;
constexpr int NSTAGE = 4;

// ============================================================================== forward
// CTA: two 128-query tiles of one (b, h) (warpgroup g: rows qbase + 128 g ..), key tiles of 64.
// TMEM, per warpgroup at 192 g: S0 [0, 64), S1 [64, 128) (double-buffered scores; P overwrites
// the first 32 columns as packed bf16), O [128, 192).
// smem: Q0 16 KB | Q1 16 KB | 4 x (K 8 KB, V 8 KB) | barriers
constexpr int F_SMEM = 32768 + NSTAGE * 16384 + 512;

__global__ void __launch_bounds__(kThreadsTC, 1)
    attn_tc_fwd_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                       const __grid_constant__ CUtensorMap tm_v, const TcArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;
  uint8_t* sKV = smem + 32768;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + 32768 + NSTAGE * 16384);
  uint64_t* q_full = bars;
  uint64_t* kv_full = bars + 1;
  uint64_t* kv_empty = kv_full + NSTAGE;
  uint64_t* s_full = kv_empty + NSTAGE;   // [2 groups][2 buffers]
  uint64_t* p_full = s_full + 4;          // [2]
  uint64_t* o_done = p_full + 2;          // [2]
  uint64_t* o_full = o_done + 2;          // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(o_full + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int bh = blockIdx.y, b = bh / a.H, h = bh % a.H;
  const int qbase = blockIdx.x * 256;
  const int ngrp = qbase + 128 < a.Sq ? 2 : 1;
  int kt0, kt1;
  tile_range(qbase, 128 * ngrp, a.Sk, a.window, 64, kt0, kt1);
  const int nkt = kt1 - kt0;

  if (warp == 0 && lane == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < NSTAGE; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    for (int i = 0; i < 4; ++i) mbar_init(&s_full[i], 1);
    for (int g = 0; g < 2; ++g) {
      mbar_init(&p_full[g], 4);
      mbar_init(&o_done[g], 1);
      mbar_init(&o_full[g], 1);
    }
    *abort_flag = 0;
    fence_barrier_init();
    tma_prefetch_desc(&tm_q);
    tma_prefetch_desc(&tm_k);
    tma_prefetch_desc(&tm_v);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
    tc_fence_before();
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tmem_slot;
  const Waiter wait{abort_flag, a.err};

  if (warp == 0) {
    if (lane == 0) {
      mbar_arrive_expect_tx(q_full, 16384u * (uint32_t)ngrp);
      for (int g = 0; g < ngrp; ++g) load_rows(sQ + 16384 * g, &tm_q, q_full, a.q_tm, b, h, qbase + 128 * g);
      for (int j = 0; j < nkt; ++j) {
        const int s = j % NSTAGE;
        const uint32_t use = (uint32_t)(j / NSTAGE);
        if (j >= NSTAGE && !wait(&kv_empty[s], (use & 1u) ^ 1u, kErrTimeoutEmpty)) break;
        uint8_t* st = sKV + s * 16384;
        mbar_arrive_expect_tx(&kv_full[s], 16384);
        load_rows(st, &tm_k, &kv_full[s], a.k_tm, b, h, (kt0 + j) * 64);
        load_rows(st + 8192, &tm_v, &kv_full[s], a.v_tm, b, h, (kt0 + j) * 64);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t id_qk = make_idesc_bf16(128, 64, 0, 0);   // S[128 q][64 k] = Q K^T
      const uint32_t id_pv = make_idesc_bf16(128, 64, 0, 1);   // O[128 q][64 d] += P V (V MN-major)
      bool ok = wait(q_full, 0, kErrTimeoutFull);
      auto qk = [&](int j) -> bool {
        const int s = j % NSTAGE;
        if (!wait(&kv_full[s], (uint32_t)(j / NSTAGE) & 1u, kErrTimeoutFull)) return false;
        tc_fence_after();
        const uint32_t ka = smem_u32(sKV + s * 16384);
        for (int g = 0; g < ngrp; ++g) {
          const uint32_t qa = smem_u32(sQ + 16384 * g), tS = tbase + 192 * g + 64 * (j & 1);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) umma_bf16(tS, kdesc(qa, kk), kdesc(ka, kk), id_qk, kk > 0 ? 1u : 0u);
          umma_commit(&s_full[2 * g + (j & 1)]);
        }
        return true;
      };
      if (ok && nkt > 0) ok = qk(0);
      if (ok && nkt > 1) ok = qk(1);
      for (int j = 0; j < nkt && ok; ++j) {
        const int s = j % NSTAGE;
        const uint32_t va = smem_u32(sKV + s * 16384) + 8192;
        for (int g = 0; g < ngrp && ok; ++g) {
          if (!wait(&p_full[g], (uint32_t)(j & 1), kErrTimeoutReady)) { ok = false; break; }
          tc_fence_after();
          const uint32_t tS = tbase + 192 * g + 64 * (j & 1), tO = tbase + 192 * g + 128;
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)   // 64 keys = 4 k-steps; P at S columns [0, 32)
            umma_ts(tO, tS + kk * 8, mndesc(va, kk), id_pv, (j > 0 || kk > 0) ? 1u : 0u);
          umma_commit(&o_done[g]);
        }
        if (!ok) break;
        umma_commit(&kv_empty[s]);
        if (j + 2 < nkt) ok = qk(j + 2);
      }
      for (int g = 0; g < ngrp; ++g) umma_commit(&o_full[g]);
    }
  } else {
    // ------------------------------------------------------------ softmax + epilogue
    const int g = (warp - 2) >> 2;
    const int quarter = warp & 3;
    const int row = 32 * quarter + lane;
    const int r0 = qbase + 128 * g, qi = r0 + row;
    const uint32_t lane_off = (uint32_t)(32 * quarter) << 16;
    const uint32_t tO = tbase + 192 * g + 128;
    if (g < ngrp) {
      float m_used = -INFINITY, l = 0.f;
      bool ok = true;
      for (int j = 0; j < nkt; ++j) {
        if (!wait(&s_full[2 * g + (j & 1)], (uint32_t)((j >> 1) & 1), kErrTimeoutAccum)) { ok = false; break; }
        tc_fence_after();
        const uint32_t tS = tbase + 192 * g + 64 * (j & 1);
        uint32_t v[64];
        tmem_ld32(tS + lane_off, *reinterpret_cast<uint32_t(*)[32]>(&v[0]));
        tmem_ld32(tS + lane_off + 32, *reinterpret_cast<uint32_t(*)[32]>(&v[32]));
        tmem_ld_wait();
        const int k0 = (kt0 + j) * 64;
        if (!tile_visible(r0, 128, k0, 64, a.Sk, a.window)) {
#pragma unroll
          for (int c = 0; c < 64; ++c)
            if (!visible(qi, k0 + c, a.Sk, a.window)) v[c] = __float_as_uint(-INFINITY);
        }
        float mraw = -INFINITY;   // row max of the raw scores (scale > 0 keeps the order)
#pragma unroll
        for (int c = 0; c < 64; c += 2) mraw = fmaxf(mraw, fmaxf(__uint_as_float(v[c]), __uint_as_float(v[c + 1])));
        const float mx = mraw * a.sl2;
        // lazy rescaling: keep the exponent base unless the row max grew by more than 2^8
        const bool grow = mx > m_used + 8.f;
        float alpha = 1.f;
        if (grow) {
          alpha = m_used == -INFINITY ? 0.f : ex2(m_used - mx);
          m_used = mx;
        }
        // O is stable once the previous tile's P V has completed
        if (j > 0 && !wait(&o_done[g], (uint32_t)((j - 1) & 1), kErrTimeoutAccum)) { ok = false; break; }
        if (__any_sync(0xffffffffu, grow && j > 0)) {
#pragma unroll 1
          for (int c = 0; c < 4; ++c) {
            uint32_t o[16];
            tmem_ld16(tO + lane_off + 16 * c, o);
            tmem_ld_wait();
#pragma unroll
            for (int e = 0; e < 16; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * alpha);
            tmem_st16(tO + lane_off + 16 * c, o);
          }
        }
        l *= alpha;
        const float mb = m_used == -INFINITY ? 0.f : m_used;
        const uint64_t sc2 = f2(a.sl2, a.sl2), nb2 = f2(-mb, -mb);
        uint64_t lsum = f2(0.f, 0.f);
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          uint32_t pk[16];
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            float x0, x1;
            f2split(ffma2(f2(__uint_as_float(v[32 * c + 2 * e]), __uint_as_float(v[32 * c + 2 * e + 1])), sc2, nb2),
                    x0, x1);
            const float p0 = ex2(x0), p1 = ex2(x1);
            lsum = fadd2(lsum, f2(p0, p1));
            pk[e] = pack_bf16x2(p0, p1);
          }
          tmem_st16(tS + lane_off + 16 * c, pk);
        }
        {
          float l0, l1;
          f2split(lsum, l0, l1);
          l += l0 + l1;
        }
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&p_full[g]);
      }
      const bool have = ok && wait(&o_full[g], 0, kErrTimeoutAccum) && nkt > 0;
      tc_fence_after();
      if (ok && nkt == 0 && qi < a.Sq) {     // no visible key: O = 0 (an empty softmax row)
        uint4* dst = reinterpret_cast<uint4*>(a.o + b * a.o_sb + h * a.o_sh + (long)qi * a.o_ld);
#pragma unroll
        for (int c = 0; c < 8; ++c) dst[c] = make_uint4(0u, 0u, 0u, 0u);
        if (a.lse) a.lse[(long)bh * a.Sq + qi] = log2f(1e-30f);
      }
      if (have) {
        uint32_t o[64];
        tmem_ld32(tO + lane_off, *reinterpret_cast<uint32_t(*)[32]>(&o[0]));
        tmem_ld32(tO + lane_off + 32, *reinterpret_cast<uint32_t(*)[32]>(&o[32]));
        tmem_ld_wait();
        if (qi < a.Sq) {
          const float inv = l > 0.f ? 1.f / l : 0.f;
          uint4* dst = reinterpret_cast<uint4*>(a.o + b * a.o_sb + h * a.o_sh + (long)qi * a.o_ld);
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            uint4 w4;
            w4.x = pack_bf16x2(__uint_as_float(o[8 * c]) * inv, __uint_as_float(o[8 * c + 1]) * inv);
            w4.y = pack_bf16x2(__uint_as_float(o[8 * c + 2]) * inv, __uint_as_float(o[8 * c + 3]) * inv);
            w4.z = pack_bf16x2(__uint_as_float(o[8 * c + 4]) * inv, __uint_as_float(o[8 * c + 5]) * inv);
            w4.w = pack_bf16x2(__uint_as_float(o[8 * c + 6]) * inv, __uint_as_float(o[8 * c + 7]) * inv);
            dst[c] = w4;
          }
          if (a.lse) a.lse[(long)bh * a.Sq + qi] = (m_used == -INFINITY ? 0.f : m_used) + log2f(fmaxf(l, 1e-30f));
        }
      }
    }
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tbase, 512);
  }
}

// ============================================================================== dq pass
// CTA: 128 queries of one (b, h); key tiles of 64, warpgroup g takes tiles j = g, g + 2, ...
// TMEM: buffer g at 128 g: S [0, 64) (dS overwrites [0, 32) as packed bf16), dP [64, 128);
// dQ at 256 (64 columns).  The softmax threads also form D = rowsum(dO o O) for their row
// (written to Dsum for the dk / dv pass).
// smem: Q 16 KB | dO 16 KB | 4 x (K 8 KB, V 8 KB) | barriers
constexpr int Q_SMEM = 32768 + NSTAGE * 16384 + 512;

__global__ void __launch_bounds__(kThreadsTC, 1)
    attn_tc_dq_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_do,
                      const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_v,
                      const TcArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;
  uint8_t* sdO = smem + 16384;
  uint8_t* sKV = smem + 32768;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + 32768 + NSTAGE * 16384);
  uint64_t* q_full = bars;
  uint64_t* kv_full = bars + 1;
  uint64_t* kv_empty = kv_full + NSTAGE;
  uint64_t* s_full = kv_empty + NSTAGE;   // [2]
  uint64_t* ds_full = s_full + 2;         // [2]
  uint64_t* acc_full = ds_full + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_full + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int bh = blockIdx.y, b = bh / a.H, h = bh % a.H;
  const int q0 = blockIdx.x * 128;
  int kt0, kt1;
  tile_range(q0, 128, a.Sk, a.window, 64, kt0, kt1);
  const int nkt = kt1 - kt0;

  if (warp == 0 && lane == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < NSTAGE; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    for (int g = 0; g < 2; ++g) {
      mbar_init(&s_full[g], 1);
      mbar_init(&ds_full[g], 4);
    }
    mbar_init(acc_full, 1);
    *abort_flag = 0;
    fence_barrier_init();
    tma_prefetch_desc(&tm_k);
    tma_prefetch_desc(&tm_v);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
    tc_fence_before();
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tmem_slot;
  const uint32_t tQ = tbase + 256;
  const Waiter wait{abort_flag, a.err};

  if (warp == 0) {
    if (lane == 0) {
      mbar_arrive_expect_tx(q_full, 32768);
      load_rows(sQ, &tm_q, q_full, a.q_tm, b, h, q0);
      load_rows(sdO, &tm_do, q_full, a.do_tm, b, h, q0);
      for (int j = 0; j < nkt; ++j) {
        const int s = j % NSTAGE;
        const uint32_t use = (uint32_t)(j / NSTAGE);
        if (j >= NSTAGE && !wait(&kv_empty[s], (use & 1u) ^ 1u, kErrTimeoutEmpty)) break;
        uint8_t* st = sKV + s * 16384;
        mbar_arrive_expect_tx(&kv_full[s], 16384);
        load_rows(st, &tm_k, &kv_full[s], a.k_tm, b, h, (kt0 + j) * 64);
        load_rows(st + 8192, &tm_v, &kv_full[s], a.v_tm, b, h, (kt0 + j) * 64);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t id_s = make_idesc_bf16(128, 64, 0, 0);    // S = Q K^T, dP = dO V^T  [128 q][64 k]
      const uint32_t id_dq = make_idesc_bf16(128, 64, 0, 1);   // dQ[128 q][64 d] += dS K (K MN-major)
      bool ok = wait(q_full, 0, kErrTimeoutFull);
      const uint32_t qa = smem_u32(sQ), da = smem_u32(sdO);
      auto sd = [&](int j) -> bool {
        const int s = j % NSTAGE;
        if (!wait(&kv_full[s], (uint32_t)(j / NSTAGE) & 1u, kErrTimeoutFull)) return false;
        tc_fence_after();
        const uint32_t ka = smem_u32(sKV + s * 16384), va = ka + 8192, tS = tbase + 128 * (j & 1);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) umma_bf16(tS, kdesc(qa, kk), kdesc(ka, kk), id_s, kk > 0 ? 1u : 0u);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) umma_bf16(tS + 64, kdesc(da, kk), kdesc(va, kk), id_s, kk > 0 ? 1u : 0u);
        umma_commit(&s_full[j & 1]);
        return true;
      };
      if (ok && nkt > 0) ok = sd(0);
      if (ok && nkt > 1) ok = sd(1);
      for (int j = 0; j < nkt && ok; ++j) {
        const int s = j % NSTAGE;
        if (!wait(&ds_full[j & 1], (uint32_t)((j >> 1) & 1), kErrTimeoutReady)) { ok = false; break; }
        tc_fence_after();
        const uint32_t ka = smem_u32(sKV + s * 16384), tS = tbase + 128 * (j & 1);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)   // 64 keys = 4 k-steps; dS at S columns [0, 32)
          umma_ts(tQ, tS + kk * 8, mndesc(ka, kk), id_dq, (j > 0 || kk > 0) ? 1u : 0u);
        umma_commit(&kv_empty[s]);
        if (j + 2 < nkt) ok = sd(j + 2);
      }
      umma_commit(acc_full);
    }
  } else {
    const int g = (warp - 2) >> 2;
    const int quarter = warp & 3;
    const int row = 32 * quarter + lane;
    const int qi = q0 + row;
    const uint32_t lane_off = (uint32_t)(32 * quarter) << 16;
    const bool qok = qi < a.Sq;
    const float lse = qok ? a.lse_in[(long)bh * a.Sq + qi] : INFINITY;
    bool ok = wait(q_full, 0, kErrTimeoutFull);
    // D = rowsum(dO o O): dO from the swizzled smem tile, O from global
    float Dq = 0.f;
    if (ok && qok) {
      const uint4* orow = reinterpret_cast<const uint4*>(a.o + b * a.o_sb + h * a.o_sh + (long)qi * a.o_ld);
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        const uint4 ov = orow[c];
        const uint4 dv = *reinterpret_cast<const uint4*>(sdO + row * 128 + ((c ^ (row & 7)) << 4));
        const __nv_bfloat162* o2 = reinterpret_cast<const __nv_bfloat162*>(&ov);
        const __nv_bfloat162* d2 = reinterpret_cast<const __nv_bfloat162*>(&dv);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 of = __bfloat1622float2(o2[e]), df = __bfloat1622float2(d2[e]);
          Dq = fmaf(of.x, df.x, Dq);
          Dq = fmaf(of.y, df.y, Dq);
        }
      }
      if (g == 0) a.Dsum[(long)bh * a.Sq + qi] = Dq;
    }
    for (int j = g; j < nkt && ok; j += 2) {
      if (!wait(&s_full[g], (uint32_t)((j >> 1) & 1), kErrTimeoutAccum)) { ok = false; break; }
      tc_fence_after();
      const uint32_t tS = tbase + 128 * g;
      uint32_t sv[64], pv[64];
      tmem_ld32(tS + lane_off, *reinterpret_cast<uint32_t(*)[32]>(&sv[0]));
      tmem_ld32(tS + lane_off + 32, *reinterpret_cast<uint32_t(*)[32]>(&sv[32]));
      tmem_ld32(tS + 64 + lane_off, *reinterpret_cast<uint32_t(*)[32]>(&pv[0]));
      tmem_ld32(tS + 64 + lane_off + 32, *reinterpret_cast<uint32_t(*)[32]>(&pv[32]));
      tmem_ld_wait();
      const int k0 = (kt0 + j) * 64;
      if (!tile_visible(q0, 128, k0, 64, a.Sk, a.window)) {
#pragma unroll
        for (int c = 0; c < 64; ++c)
          if (!visible(qi, k0 + c, a.Sk, a.window)) sv[c] = __float_as_uint(-INFINITY);
      }
      const uint64_t sc2 = f2(a.sl2, a.sl2), nl2 = f2(-lse, -lse), nd2 = f2(-Dq, -Dq);
      uint32_t pk[32];   // dS row as packed bf16 pairs: column e holds keys 2e, 2e + 1
#pragma unroll
      for (int e = 0; e < 32; ++e) {
        float x0, x1, d0, d1;
        f2split(ffma2(f2(__uint_as_float(sv[2 * e]), __uint_as_float(sv[2 * e + 1])), sc2, nl2), x0, x1);
        const uint64_t pp = f2(ex2(x0), ex2(x1));
        f2split(fmul2(pp, fadd2(f2(__uint_as_float(pv[2 * e]), __uint_as_float(pv[2 * e + 1])), nd2)), d0, d1);
        pk[e] = pack_bf16x2(d0, d1);
      }
      tmem_st16(tS + lane_off, *reinterpret_cast<uint32_t(*)[16]>(&pk[0]));
      tmem_st16(tS + lane_off + 16, *reinterpret_cast<uint32_t(*)[16]>(&pk[16]));
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&ds_full[g]);
    }
    const bool have = ok && wait(acc_full, 0, kErrTimeoutAccum) && nkt > 0;
    tc_fence_after();
    // warpgroup g writes dQ columns [32 g, 32 g + 32)
    float4* dst = reinterpret_cast<float4*>(a.dq + b * a.dq_sb + h * a.dq_sh + (long)qi * a.dq_ld + 32 * g);
    if (ok && nkt == 0 && qok) {
#pragma unroll
      for (int c = 0; c < 8; ++c) dst[c] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    if (have) {
      uint32_t o[32];
      tmem_ld32(tQ + lane_off + 32 * g, o);
      tmem_ld_wait();
      if (qok) {
#pragma unroll
        for (int c = 0; c < 8; ++c)
          dst[c] = make_float4(__uint_as_float(o[4 * c]) * a.scale, __uint_as_float(o[4 * c + 1]) * a.scale,
                               __uint_as_float(o[4 * c + 2]) * a.scale, __uint_as_float(o[4 * c + 3]) * a.scale);
      }
    }
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tbase, 512);
  }
}

// ============================================================================== dkdv pass
// CTA: 128 keys of one (b, h); query tiles of 64, warpgroup g takes tiles i = g, g + 2, ...
// TMEM: buffer g at 128 g: S^T [0, 64) (P^T overwrites [0, 32)), dP^T [64, 128) (dS^T overwrites
// [64, 96)); dV at 256, dK at 320.
// smem: K 16 KB | V 16 KB | 4 x (Q 8 KB, dO 8 KB) | lse / D per warpgroup (x2) | barriers
constexpr int KV_SMEM = 32768 + NSTAGE * 16384 + 2048 + 512;

__global__ void __launch_bounds__(kThreadsTC, 1)
    attn_tc_dkdv_kernel(const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_v,
                        const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_do,
                        const TcArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sK = smem;
  uint8_t* sV = smem + 16384;
  uint8_t* sQd = smem + 32768;
  float* s_ld = reinterpret_cast<float*>(smem + 32768 + NSTAGE * 16384);   // [2 groups][2 bufs][lse 64 | D 64]
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + 32768 + NSTAGE * 16384 + 2048);
  uint64_t* kv_full = bars;
  uint64_t* q_full = bars + 1;
  uint64_t* q_empty = q_full + NSTAGE;
  uint64_t* s_full = q_empty + NSTAGE;    // [2]
  uint64_t* ds_full = s_full + 2;         // [2]
  uint64_t* acc_full = ds_full + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_full + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int bh = blockIdx.y, b = bh / a.H, h = bh % a.H;
  const int k0 = blockIdx.x * 128;
  int qt0, qt1;
  tile_range(k0, 128, a.Sq, a.window, 64, qt0, qt1);
  const int nqt = qt1 - qt0;

  if (warp == 0 && lane == 0) {
    mbar_init(kv_full, 1);
    for (int s = 0; s < NSTAGE; ++s) {
      mbar_init(&q_full[s], 1);
      mbar_init(&q_empty[s], 1);
    }
    for (int g = 0; g < 2; ++g) {
      mbar_init(&s_full[g], 1);
      mbar_init(&ds_full[g], 4);
    }
    mbar_init(acc_full, 1);
    *abort_flag = 0;
    fence_barrier_init();
    tma_prefetch_desc(&tm_q);
    tma_prefetch_desc(&tm_do);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
    tc_fence_before();
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tmem_slot;
  const uint32_t tV = tbase + 256, tK = tbase + 320;
  const Waiter wait{abort_flag, a.err};

  if (warp == 0) {
    if (lane == 0) {
      mbar_arrive_expect_tx(kv_full, 32768);
      load_rows(sK, &tm_k, kv_full, a.k_tm, b, h, k0);
      load_rows(sV, &tm_v, kv_full, a.v_tm, b, h, k0);
      for (int i = 0; i < nqt; ++i) {
        const int s = i % NSTAGE;
        const uint32_t use = (uint32_t)(i / NSTAGE);
        if (i >= NSTAGE && !wait(&q_empty[s], (use & 1u) ^ 1u, kErrTimeoutEmpty)) break;
        uint8_t* st = sQd + s * 16384;
        mbar_arrive_expect_tx(&q_full[s], 16384);
        load_rows(st, &tm_q, &q_full[s], a.q_tm, b, h, (qt0 + i) * 64);
        load_rows(st + 8192, &tm_do, &q_full[s], a.do_tm, b, h, (qt0 + i) * 64);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t id_s = make_idesc_bf16(128, 64, 0, 0);    // S^T = K Q^T, dP^T = V dO^T  [128 k][64 q]
      const uint32_t id_g = make_idesc_bf16(128, 64, 0, 1);    // dV / dK [128 k][64 d] (dO / Q MN-major)
      bool ok = wait(kv_full, 0, kErrTimeoutFull);
      const uint32_t ka = smem_u32(sK), va = smem_u32(sV);
      auto sd = [&](int i) -> bool {
        const int s = i % NSTAGE;
        if (!wait(&q_full[s], (uint32_t)(i / NSTAGE) & 1u, kErrTimeoutFull)) return false;
        tc_fence_after();
        const uint32_t qa = smem_u32(sQd + s * 16384), da = qa + 8192, tS = tbase + 128 * (i & 1);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) umma_bf16(tS, kdesc(ka, kk), kdesc(qa, kk), id_s, kk > 0 ? 1u : 0u);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) umma_bf16(tS + 64, kdesc(va, kk), kdesc(da, kk), id_s, kk > 0 ? 1u : 0u);
        umma_commit(&s_full[i & 1]);
        return true;
      };
      if (ok && nqt > 0) ok = sd(0);
      if (ok && nqt > 1) ok = sd(1);
      for (int i = 0; i < nqt && ok; ++i) {
        const int s = i % NSTAGE;
        if (!wait(&ds_full[i & 1], (uint32_t)((i >> 1) & 1), kErrTimeoutReady)) { ok = false; break; }
        tc_fence_after();
        const uint32_t qa = smem_u32(sQd + s * 16384), da = qa + 8192, tS = tbase + 128 * (i & 1);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)   // 64 queries = 4 k-steps; P^T at S^T columns [0, 32)
          umma_ts(tV, tS + kk * 8, mndesc(da, kk), id_g, (i > 0 || kk > 0) ? 1u : 0u);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)   // dS^T at dP^T columns [0, 32)
          umma_ts(tK, tS + 64 + kk * 8, mndesc(qa, kk), id_g, (i > 0 || kk > 0) ? 1u : 0u);
        umma_commit(&q_empty[s]);
        if (i + 2 < nqt) ok = sd(i + 2);
      }
      umma_commit(acc_full);
    }
  } else {
    const int g = (warp - 2) >> 2;
    const int quarter = warp & 3;
    const int row = 32 * quarter + lane;
    const int kj = k0 + row;
    const int t = threadIdx.x - 64 - 128 * g;   // 0..127 within the warpgroup
    const uint32_t lane_off = (uint32_t)(32 * quarter) << 16;
    bool ok = true;
    int it = 0;
    for (int i = g; i < nqt; i += 2, ++it) {
      const int q0 = (qt0 + i) * 64;
      float* lse_b = s_ld + 256 * g + 128 * (it & 1);
      float* D_b = lse_b + 64;
      {
        const int c = t & 63, qi = q0 + c;
        const bool qok = qi < a.Sq;
        if (t < 64) lse_b[c] = qok ? a.lse_in[(long)bh * a.Sq + qi] : INFINITY;
        else D_b[c] = qok ? a.Dsum[(long)bh * a.Sq + qi] : 0.f;
      }
      if (g == 0) named_bar(1, 128);   // every warp of the group passes it once per tile, also after an abort
      else named_bar(2, 128);
      if (ok) ok = wait(&s_full[g], (uint32_t)(it & 1), kErrTimeoutAccum);
      if (!ok) continue;
      tc_fence_after();
      const uint32_t tS = tbase + 128 * g;
      uint32_t sv[64], pv[64];
      tmem_ld32(tS + lane_off, *reinterpret_cast<uint32_t(*)[32]>(&sv[0]));
      tmem_ld32(tS + lane_off + 32, *reinterpret_cast<uint32_t(*)[32]>(&sv[32]));
      tmem_ld32(tS + 64 + lane_off, *reinterpret_cast<uint32_t(*)[32]>(&pv[0]));
      tmem_ld32(tS + 64 + lane_off + 32, *reinterpret_cast<uint32_t(*)[32]>(&pv[32]));
      tmem_ld_wait();
      if (!tile_visible(k0, 128, q0, 64, a.Sq, a.window) || kj >= a.Sk) {
        // (queries past Sq already carry lse = +inf, so P = 0 there)
#pragma unroll
        for (int c = 0; c < 64; ++c)
          if (!visible(q0 + c, kj, a.Sk, a.window)) sv[c] = __float_as_uint(-INFINITY);
      }
      const uint64_t sc2 = f2(a.sl2, a.sl2);
      const float2* lse2 = reinterpret_cast<const float2*>(lse_b);
      const float2* D2 = reinterpret_cast<const float2*>(D_b);
      uint32_t pk[32], dk[32];
#pragma unroll
      for (int e = 0; e < 32; ++e) {
        const float2 lz = lse2[e], dz = D2[e];      // smem broadcast reads
        float x0, x1, d0, d1;
        f2split(ffma2(f2(__uint_as_float(sv[2 * e]), __uint_as_float(sv[2 * e + 1])), sc2, f2(-lz.x, -lz.y)), x0, x1);
        const float p0 = ex2(x0), p1 = ex2(x1);
        f2split(fmul2(f2(p0, p1), fadd2(f2(__uint_as_float(pv[2 * e]), __uint_as_float(pv[2 * e + 1])),
                                        f2(-dz.x, -dz.y))), d0, d1);
        pk[e] = pack_bf16x2(p0, p1);
        dk[e] = pack_bf16x2(d0, d1);
      }
      tmem_st16(tS + lane_off, *reinterpret_cast<uint32_t(*)[16]>(&pk[0]));
      tmem_st16(tS + lane_off + 16, *reinterpret_cast<uint32_t(*)[16]>(&pk[16]));
      tmem_st16(tS + 64 + lane_off, *reinterpret_cast<uint32_t(*)[16]>(&dk[0]));
      tmem_st16(tS + 64 + lane_off + 16, *reinterpret_cast<uint32_t(*)[16]>(&dk[16]));
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&ds_full[g]);
    }
    const bool have = ok && wait(acc_full, 0, kErrTimeoutAccum) && nqt > 0;
    tc_fence_after();
    const bool kok = kj < a.Sk;
    // warpgroup 0 writes dV, warpgroup 1 writes dK
    float4* dst = g == 0 ? reinterpret_cast<float4*>(a.dv + b * a.dv_sb + h * a.dv_sh + (long)kj * a.dv_ld)
                         : reinterpret_cast<float4*>(a.dk + b * a.dk_sb + h * a.dk_sh + (long)kj * a.dk_ld);
    const float mul = g == 0 ? 1.f : a.scale;
    if (ok && nqt == 0 && kok) {
#pragma unroll
      for (int c = 0; c < 16; ++c) dst[c] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    if (have) {
      uint32_t o[64];
      const uint32_t tacc = g == 0 ? tV : tK;
      tmem_ld32(tacc + lane_off, *reinterpret_cast<uint32_t(*)[32]>(&o[0]));
      tmem_ld32(tacc + lane_off + 32, *reinterpret_cast<uint32_t(*)[32]>(&o[32]));
      tmem_ld_wait();
      if (kok) {
#pragma unroll
        for (int c = 0; c < 16; ++c)
          dst[c] = make_float4(__uint_as_float(o[4 * c]) * mul, __uint_as_float(o[4 * c + 1]) * mul,
                               __uint_as_float(o[4 * c + 2]) * mul, __uint_as_float(o[4 * c + 3]) * mul);
      }
    }
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tbase, 512);
  }
}

// ------------------------------------------------------------------------------ host side
// 4-D tensor map over a strided (b, h, s, d) bf16 tensor: the smaller of the head / row strides
// goes second so the strides grow; the box is `rows` rows x 64 d of one (b, h).
int make_map4(CUtensorMap* m, const __nv_bfloat16* base, long sb, long sh, long ld, int B, int H, int S, int rows,
              int& tm, std::string& err) {
  PFN_encodeTiled enc = encode_tiled_fn(err);
  if (!enc) return 1;
  if ((reinterpret_cast<uintptr_t>(base) & 15) || (sh % 8) || (ld % 8) || (sb % 8)) {
    err = "attention: tensor strides must be multiples of 8 elements";
    return 1;
  }
  tm = sh <= ld ? 1 : 0;
  const long s1 = tm ? sh : ld, s2 = tm ? ld : sh;
  const long n1 = tm ? H : S, n2 = tm ? S : H;
  long s3 = sb;
  if (B == 1) {
    s3 = s2 * n2;                         // unused extent-1 dimension: any valid stride
  } else if (s3 < s2 * n2) {
    err = "attention: batch stride overlaps the heads / rows of a batch";
    return 1;
  }
  cuuint64_t dims[4] = {64, (cuuint64_t)n1, (cuuint64_t)n2, (cuuint64_t)B};
  cuuint64_t strides[3] = {(cuuint64_t)s1 * 2, (cuuint64_t)s2 * 2, (cuuint64_t)s3 * 2};
  cuuint32_t box[4] = {64, tm ? 1u : (cuuint32_t)rows, tm ? (cuuint32_t)rows : 1u, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  const CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<__nv_bfloat16*>(base), dims, strides, box,
                         estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    err = "attention: cuTensorMapEncodeTiled failed (" + std::to_string((int)r) + ")";
    return 1;
  }
  return 0;
}

TcArgs tc_args(const AttnArgs& p) {
  TcArgs a{};
  a.B = p.B; a.H = p.H; a.Sq = p.Sq; a.Sk = p.Sk; a.window = p.window;
  a.scale = p.scale;
  a.sl2 = p.scale * kLog2e;
  a.o = p.o; a.o_sb = p.o_sb; a.o_sh = p.o_sh; a.o_ld = p.o_ld;
  a.lse = p.lse;
  a.lse_in = p.lse;
  a.Dsum = p.Dsum;
  a.dq = p.dq; a.dq_sb = p.dq_sb; a.dq_sh = p.dq_sh; a.dq_ld = p.dq_ld;
  a.dk = p.dk; a.dk_sb = p.dk_sb; a.dk_sh = p.dk_sh; a.dk_ld = p.dk_ld;
  a.dv = p.dv; a.dv_sb = p.dv_sb; a.dv_sh = p.dv_sh; a.dv_ld = p.dv_ld;
  return a;
}

int set_tc_attrs(std::string& err) {
  static bool done = false;
  if (done) return 0;
  if (cudaFuncSetAttribute(attn_tc_fwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_req(F_SMEM)) != cudaSuccess ||
      cudaFuncSetAttribute(attn_tc_dq_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_req(Q_SMEM)) != cudaSuccess ||
      cudaFuncSetAttribute(attn_tc_dkdv_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_req(KV_SMEM)) != cudaSuccess)
    return check_launch("attention tc smem attributes", err);
  done = true;
  return 0;
}

}  // namespace

bool attn_tc_supported(const AttnArgs& p) {
  auto al = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15) == 0; };
  auto st = [](long a, long b, long c) { return a % 8 == 0 && b % 8 == 0 && c % 8 == 0; };
  return p.head_dim == 64 && al(p.q) && al(p.k) && al(p.v) && al(p.o) && st(p.q_sb, p.q_sh, p.q_ld) &&
         st(p.k_sb, p.k_sh, p.k_ld) && st(p.v_sb, p.v_sh, p.v_ld) && st(p.o_sb, p.o_sh, p.o_ld) &&
         (!p.dO || (al(p.dO) && st(p.dO_sb, p.dO_sh, p.dO_ld))) &&
         (!p.dq || (al(p.dq) && p.dq_ld % 4 == 0 && p.dq_sb % 4 == 0 && p.dq_sh % 4 == 0)) &&
         (!p.dk || (al(p.dk) && p.dk_ld % 4 == 0 && p.dk_sb % 4 == 0 && p.dk_sh % 4 == 0)) &&
         (!p.dv || (al(p.dv) && p.dv_ld % 4 == 0 && p.dv_sb % 4 == 0 && p.dv_sh % 4 == 0)) &&
         (!p.o || (p.o_ld % 8 == 0));
}

int attn_tc_forward(Ctx* c, const AttnArgs& p, std::string& err) {
  if (set_tc_attrs(err)) return 1;
  TcArgs a = tc_args(p);
  a.err = c->d_err;
  CUtensorMap mq, mk, mv;
  if (make_map4(&mq, p.q, p.q_sb, p.q_sh, p.q_ld, p.B, p.H, p.Sq, 128, a.q_tm, err) ||
      make_map4(&mk, p.k, p.k_sb, p.k_sh, p.k_ld, p.B, p.H, p.Sk, 64, a.k_tm, err) ||
      make_map4(&mv, p.v, p.v_sb, p.v_sh, p.v_ld, p.B, p.H, p.Sk, 64, a.v_tm, err))
    return 1;
  ProfScope prof_(c, "attn.fwd");
  dim3 grid((unsigned)((p.Sq + 255) / 256), (unsigned)(p.B * p.H));
  attn_tc_fwd_kernel<<<grid, kThreadsTC, smem_req(F_SMEM), c->stream>>>(mq, mk, mv, a);
  return check_launch("attn tc fwd", err);
}

int attn_tc_grads(Ctx* c, const AttnArgs& p, bool want_dkdv, std::string& err) {
  if (set_tc_attrs(err)) return 1;
  TcArgs a = tc_args(p);
  a.err = c->d_err;
  {
    CUtensorMap mq, mdo, mk, mv;
    if (make_map4(&mq, p.q, p.q_sb, p.q_sh, p.q_ld, p.B, p.H, p.Sq, 128, a.q_tm, err) ||
        make_map4(&mdo, p.dO, p.dO_sb, p.dO_sh, p.dO_ld, p.B, p.H, p.Sq, 128, a.do_tm, err) ||
        make_map4(&mk, p.k, p.k_sb, p.k_sh, p.k_ld, p.B, p.H, p.Sk, 64, a.k_tm, err) ||
        make_map4(&mv, p.v, p.v_sb, p.v_sh, p.v_ld, p.B, p.H, p.Sk, 64, a.v_tm, err))
      return 1;
    ProfScope prof_(c, "attn.bwd_dq");
    dim3 grid((unsigned)((p.Sq + 127) / 128), (unsigned)(p.B * p.H));
    attn_tc_dq_kernel<<<grid, kThreadsTC, smem_req(Q_SMEM), c->stream>>>(mq, mdo, mk, mv, a);
    if (check_launch("attn tc dq", err)) return 1;
  }
  if (want_dkdv) {
    CUtensorMap mk, mv, mq, mdo;
    if (make_map4(&mk, p.k, p.k_sb, p.k_sh, p.k_ld, p.B, p.H, p.Sk, 128, a.k_tm, err) ||
        make_map4(&mv, p.v, p.v_sb, p.v_sh, p.v_ld, p.B, p.H, p.Sk, 128, a.v_tm, err) ||
        make_map4(&mq, p.q, p.q_sb, p.q_sh, p.q_ld, p.B, p.H, p.Sq, 64, a.q_tm, err) ||
        make_map4(&mdo, p.dO, p.dO_sb, p.dO_sh, p.dO_ld, p.B, p.H, p.Sq, 64, a.do_tm, err))
      return 1;
    ProfScope prof_(c, "attn.bwd_dkdv");
    dim3 grid((unsigned)((p.Sk + 127) / 128), (unsigned)(p.B * p.H));
    attn_tc_dkdv_kernel<<<grid, kThreadsTC, smem_req(KV_SMEM), c->stream>>>(mk, mv, mq, mdo, a);
    if (check_launch("attn tc dkdv", err)) return 1;
  }
  return 0;
}

}  // namespace sa3k
