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
//              accumulators read with tcgen05.ld; P and dS go back into TMEM as packed f16 and
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
  int q_tm, k_tm, v_tm, o_tm, do_tm, dq_tm;   // tensor-map coordinate order: 1 = (d, h, s, b), 0 = (d, s, h, b)
  __half* o; long o_sb, o_sh, o_ld;
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

__device__ __forceinline__ void tma_store_4d(const CUtensorMap* m, const void* src, int c0, int c1, int c2, int c3) {
  asm volatile("cp.async.bulk.tensor.4d.global.shared::cta.bulk_group [%0, {%2, %3, %4, %5}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(m)),
               "r"(smem_u32(src)), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
               : "memory");
}

// rows [row0, row0 + n) of head h of batch b (map coordinate order per `tm`)
__device__ __forceinline__ void load_rows(void* dst, const CUtensorMap* m, uint64_t* bar, int tm, int b, int h,
                                          int row0) {
  if (tm) tma_load_4d(dst, m, bar, 0, h, row0, b);
  else tma_load_4d(dst, m, bar, 0, row0, h, b);
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

__device__ __forceinline__ uint64_t fadd2_rm(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rm.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}

// 2^x for two values on the FMA / integer pipes instead of the MUFU unit (part of the softmax
// exponentials run here so that both kinds of pipe share the work).  Method: Cody-Waite range
// reduction x = n + f with n = floor(x) (x + 1.5 * 2^23 rounded toward -inf leaves n in the low
// mantissa bits) and f in [0, 1), a degree-3 polynomial for 2^f fitted here by iteratively
// reweighted least squares for minimax relative error (< 8e-5 on [0, 1)), and n added into the
// exponent field.  x is clamped to >= -125, so arguments below give ~2^-125 instead of 0 (far
// below what the f16 P or the f32 row sum register).
// which pairs of every 8 take ex2_poly2 (3 of 8: the MUFU and FMA pipes then finish together)
__device__ constexpr bool kPolyPair[8] = {true, false, false, true, false, true, false, false};

__device__ __forceinline__ void ex2_poly2(float x0, float x1, float& y0, float& y1) {
  constexpr float kMagic = 12582912.0f;   // 1.5 * 2^23
  const uint64_t x = f2(fmaxf(x0, -125.f), fmaxf(x1, -125.f));
  const uint64_t t = fadd2_rm(x, f2(kMagic, kMagic));           // kMagic + floor(x), exact
  const uint64_t n = fadd2(t, f2(-kMagic, -kMagic));             // floor(x)
  const uint64_t fr = ffma2(n, f2(-1.f, -1.f), x);               // x - floor(x), in [0, 1)
  uint64_t p = ffma2(f2(0.07802403f, 0.07802403f), fr, f2(0.22606707f, 0.22606707f));
  p = ffma2(p, fr, f2(0.69583398f, 0.69583398f));
  p = ffma2(p, fr, f2(0.99992514f, 0.99992514f));
  float p0, p1, t0, t1;
  f2split(p, p0, p1);
  f2split(t, t0, t1);
  const int mb = __float_as_int(kMagic);
  y0 = __int_as_float(__float_as_int(p0) + ((__float_as_int(t0) - mb) << 23));
  y1 = __int_as_float(__float_as_int(p1) + ((__float_as_int(t1) - mb) << 23));
}

__device__ __forceinline__ float max3(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

// max of 64 values held as raw f32 bits (four independent chains of three-input max)
__device__ __forceinline__ float rowmax64(const uint32_t (&v)[64]) {
  float m[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
  for (int c = 0; c < 64; c += 8)
#pragma unroll
    for (int u = 0; u < 4; ++u) m[u] = max3(m[u], __uint_as_float(v[c + 2 * u]), __uint_as_float(v[c + 2 * u + 1]));
  return fmaxf(fmaxf(m[0], m[1]), fmaxf(m[2], m[3]));
}

// every (row, key) of a rows x keys tile is inside [0, Sk) and the band
__device__ __forceinline__ bool tile_visible(int r0, int nr, int k0, int nk, int Sk, int window) {
  if (k0 + nk > Sk) return false;
  if (window < 0) return true;
  return max(r0 + nr - 1 - k0, k0 + nk - 1 - r0) <= window;
}

// K-major [rows][64] f16 tile (128-byte rows, 128B swizzle): descriptor of the tile, and the
// descriptor at k-step kk (16 wide = 32 bytes further: +2 in the start-address field)
__device__ __forceinline__ uint64_t kdesc0(uint32_t base) { return make_sdesc(base, 16, 1024); }
__device__ __forceinline__ uint64_t kstep(uint64_t d0, int kk) { return d0 + (uint64_t)(2 * kk); }
// the same tile read MN-major (its rows are the reduction index): 16 rows = 2048 bytes per k-step
__device__ __forceinline__ uint64_t mndesc0(uint32_t base) { return make_sdesc(base, 8192, 1024); }
__device__ __forceinline__ uint64_t mnstep(uint64_t d0, int kk) { return d0 + (uint64_t)(128 * kk); }

struct Waiter {
  volatile int* abort_flag;
  int* err;
  __device__ __forceinline__ bool operator()(uint64_t* bar, uint32_t parity, int code) const {
    const uint32_t a = smem_u32(bar);
    if (mbar_try_wait(a, parity)) return true;     // fast path: already complete
    if (*abort_flag) return false;
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

// Warp roles of all three kernels (11 warps): warp 0 TMA producer, warp 1 TMEM owner and issuer
// of the score MMAs, warp 10 issuer of the gradient / output MMAs (two issue streams, synchronised
// through barriers, so neither waits on the other's instruction issue), warps 2-5 = warpgroup 0
// and warps 6-9 = warpgroup 1 of softmax threads (thread <-> TMEM lane <-> tile row; warp w
// reaches lanes 32 (w % 4) .. +32).  Streamed tiles are 64 rows
// and sit in a 4-deep ring.  The two warpgroups keep the tensor core busy while they work: in
// the forward each owns its own 128-query tile; in the backward passes they take alternate
// streamed tiles and the MMA thread folds their results into one accumulator in tile order.
constexpr int kWarpsTC = 11;
// Each CTA holds all 512 TMEM columns; a shared-memory request above half the SM keeps a second
// CTA from being placed beside it (it would only wait in tcgen05.alloc).
constexpr int kSmemFloor = 120 * 1024;
constexpr int smem_req(int bytes) { return bytes + 1024 > kSmemFloor ? bytes + 1024 : kSmemFloor; }
constexpr int kThreadsTC = 32 * kWarpsTC;
constexpr int NSTAGE = 4;

// Work order of the grid-per-tile kernels and of the dq pass's items: every full tile of every
// (b, h) first (the tiles of one (b, h) adjacent), then the (b, h)s' partial last tiles, so that
// the short tiles fill the last round of SMs instead of being spread through it.  Linear index
// L of nbh (b, h)s with `full` full tiles each (+ one partial when `part`) -> (bh, tile).
__device__ __forceinline__ void heavy_first(int L, int nbh, int full, int& bh, int& tile) {
  if (L < nbh * full) {
    bh = L / full;
    tile = L % full;
  } else {
    bh = L - nbh * full;
    tile = full;
  }
}

// ============================================================================== forward
// CTA: two 128-query tiles of one (b, h) (warpgroup g: rows qbase + 128 g ..), key tiles of 64.
// TMEM, per warpgroup at 256 g: S0, S1, S2 at [0, 64), [64, 128), [128, 192) (scores of three
// key tiles in flight; P overwrites the first 32 columns of its buffer as packed f16), O at
// [192, 256).
// smem: Q0 16 KB | Q1 16 KB | 4 x (K 8 KB, V 8 KB) | barriers
constexpr int F_SMEM = 32768 + NSTAGE * 16384 + 512;

__global__ void __launch_bounds__(kThreadsTC, 1)
    attn_tc_fwd_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                       const __grid_constant__ CUtensorMap tm_v, const TcArgs a) {
  extern __shared__ uint8_t smem_raw[];
  pdl_trigger();   // the next kernel may be scheduled once every CTA of this grid runs
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;
  uint8_t* sKV = smem + 32768;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + 32768 + NSTAGE * 16384);
  uint64_t* q_full = bars;
  uint64_t* kv_full = bars + 1;
  uint64_t* kv_empty = kv_full + NSTAGE;
  uint64_t* s_full = kv_empty + NSTAGE;   // [2 groups][3 buffers]
  uint64_t* p_full = s_full + 6;          // [2]
  uint64_t* o_done = p_full + 2;          // [2]
  uint64_t* o_full = o_done + 2;          // [2]
  uint64_t* pv_done = o_full + 2;         // [2 groups][3 buffers]: P V has read the buffer's P
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(pv_done + 6);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int bh, qt;
  heavy_first((int)(blockIdx.y * gridDim.x + blockIdx.x), (int)gridDim.y, a.Sq / 256, bh, qt);
  const int b = bh / a.H, h = bh % a.H;
  const int qbase = qt * 256;
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
    for (int i = 0; i < 6; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&pv_done[i], 1);
    }
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
  pdl_wait();      // outputs of earlier kernels are read only from here on
  const Waiter wait{abort_flag, a.err};     // single-thread roles (the TMA producer)
  const WaiterW<> waitw{abort_flag, a.err};   // whole-warp roles (MMA issue, softmax)

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
    {   // scores S = Q K^T of tile j for both groups into buffer j % 3, once P V (j - 3) read it
      const uint32_t id_qk = make_idesc_f16(128, 64, 0, 0);   // S[128 q][64 k] = Q K^T
      bool ok = waitw(q_full, 0, kErrTimeoutFull);
      for (int j = 0; j < nkt && ok; ++j) {
        const int s = j % NSTAGE;
        if (!waitw(&kv_full[s], (uint32_t)(j / NSTAGE) & 1u, kErrTimeoutFull)) { ok = false; break; }
        const uint64_t kd = kdesc0(smem_u32(sKV + s * 16384));
        for (int g = 0; g < ngrp && ok; ++g) {
          if (j >= 3 && !waitw(&pv_done[3 * g + j % 3], (uint32_t)(((j / 3) - 1) & 1), kErrTimeoutOther)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t qd = kdesc0(smem_u32(sQ + 16384 * g));
          const uint32_t tS = tbase + 256 * g + 64 * (j % 3);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) umma_f16_w(tS, kstep(qd, kk), kstep(kd, kk), id_qk, kk > 0 ? 1u : 0u);
          umma_commit_w(&s_full[3 * g + (j % 3)]);
        }
      }
    }
  } else if (warp == 10) {
    {   // O += P V of tile j for each group once its P is in TMEM
      const uint32_t id_pv = make_idesc_f16(128, 64, 0, 1);   // O[128 q][64 d] += P V (V MN-major)
      bool ok = true;
      for (int j = 0; j < nkt && ok; ++j) {
        const int s = j % NSTAGE;
        const uint64_t vd = mndesc0(smem_u32(sKV + s * 16384) + 8192);
        for (int g = 0; g < ngrp && ok; ++g) {
          if (!waitw(&p_full[g], (uint32_t)(j & 1), kErrTimeoutReady)) { ok = false; break; }
          tc_fence_after();
          const uint32_t tS = tbase + 256 * g + 64 * (j % 3), tO = tbase + 256 * g + 192;
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)   // 64 keys = 4 k-steps; P at S columns [0, 32)
            umma_ts_w(tO, tS + kk * 8, mnstep(vd, kk), id_pv, (j > 0 || kk > 0) ? 1u : 0u);
          umma_commit_w(&o_done[g]);
          umma_commit_w(&pv_done[3 * g + j % 3]);
        }
        // (the score MMAs of tile j completed before any P of it existed: K is free as well)
        if (ok) umma_commit_w(&kv_empty[s]);
      }
      for (int g = 0; g < ngrp; ++g) umma_commit_w(&o_full[g]);
    }
  } else {   // warps 2 .. 9
    // ------------------------------------------------------------ softmax + epilogue
    const int g = (warp - 2) >> 2;
    const int quarter = warp & 3;
    const int row = 32 * quarter + lane;
    const int r0 = qbase + 128 * g, qi = r0 + row;
    const uint32_t lane_off = (uint32_t)(32 * quarter) << 16;
    const uint32_t tO = tbase + 256 * g + 192;
    if (g < ngrp) {
      float m_used = -INFINITY, l = 0.f;
      bool ok = true;
      for (int j = 0; j < nkt; ++j) {
        if (!waitw(&s_full[3 * g + (j % 3)], (uint32_t)((j / 3) & 1), kErrTimeoutAccum)) { ok = false; break; }
        tc_fence_after();
        const uint32_t tS = tbase + 256 * g + 64 * (j % 3);
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
        const float mx = rowmax64(v) * a.sl2;   // (scale > 0 keeps the order of the raw scores)
        // lazy rescaling: keep the exponent base unless the row max grew by more than 2^8
        const bool grow = mx > m_used + 8.f;
        float alpha = 1.f;
        if (grow) {
          alpha = m_used == -INFINITY ? 0.f : ex2(m_used - mx);
          m_used = mx;
        }
        // O is stable once the previous tile's P V has completed (o_done phase j - 1).  That phase
        // is consumed exactly once per tile: here when O must be rescaled, else just before P_j is
        // handed to the MMA (it has normally completed long before).
        bool waited = false;
        if (__any_sync(0xffffffffu, grow && j > 0)) {
          if (!waitw(&o_done[g], (uint32_t)((j - 1) & 1), kErrTimeoutAccum)) { ok = false; break; }
          waited = true;
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
        uint64_t lsum[2] = {f2(0.f, 0.f), f2(0.f, 0.f)};
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          uint32_t pk[16];
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            float x0, x1;
            f2split(ffma2(f2(__uint_as_float(v[32 * c + 2 * e]), __uint_as_float(v[32 * c + 2 * e + 1])), sc2, nb2),
                    x0, x1);
            float p0, p1;
            if (kPolyPair[e & 7]) {      // a share of the exponentials on the FMA pipes
              ex2_poly2(x0, x1, p0, p1);
            } else {
              p0 = ex2(x0);
              p1 = ex2(x1);
            }
            lsum[e & 1] = fadd2(lsum[e & 1], f2(p0, p1));
            pk[e] = pack_f16x2(p0, p1);
          }
          tmem_st16(tS + lane_off + 16 * c, pk);
        }
        {
          float l0, l1, l2, l3;
          f2split(lsum[0], l0, l1);
          f2split(lsum[1], l2, l3);
          l += (l0 + l1) + (l2 + l3);
        }
        tmem_st_wait();
        tc_fence_before();
        if (j > 0 && !waited && !waitw(&o_done[g], (uint32_t)((j - 1) & 1), kErrTimeoutAccum)) { ok = false; break; }
        __syncwarp();
        if (lane == 0) mbar_arrive(&p_full[g]);
      }
      const bool have = ok && waitw(&o_full[g], 0, kErrTimeoutAccum) && nkt > 0;
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
            w4.x = pack_f16x2(__uint_as_float(o[8 * c]) * inv, __uint_as_float(o[8 * c + 1]) * inv);
            w4.y = pack_f16x2(__uint_as_float(o[8 * c + 2]) * inv, __uint_as_float(o[8 * c + 3]) * inv);
            w4.z = pack_f16x2(__uint_as_float(o[8 * c + 4]) * inv, __uint_as_float(o[8 * c + 5]) * inv);
            w4.w = pack_f16x2(__uint_as_float(o[8 * c + 6]) * inv, __uint_as_float(o[8 * c + 7]) * inv);
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
// Persistent: CTA c walks the work items c, c + gridDim.x, ...; an item is 128 queries of one
// (b, h) (items of one (b, h) are adjacent, so co-running CTAs share its K / V in L2).  The key
// tiles (64) of consecutive items form one stream: the TMA ring, the three score buffers and the
// warpgroup that handles a tile (the stream index's parity) all run on across items, and the
// next item's Q / dO load while the current item finishes.
// TMEM: score buffers at 128 b (b < 3): S [0, 64) (dS overwrites [0, 32) as packed f16),
// dP [64, 128); two dQ accumulators at 384 and 448 (alternate items).  The softmax threads also
// form D = rowsum(dO o O) of their row (stored to Dsum for the dk / dv pass).
// The row's O comes in with Q and dO (TMA, an item ahead), so D needs no global load at the
// item boundary; dQ leaves through swizzled shared-memory staging and TMA stores.
// smem: 2 x (Q 16 KB, dO 16 KB, O 16 KB) | 5 x (K 8 KB, V 8 KB) | 8 x 4 KB dQ staging | barriers
constexpr int Q_STAGES = 5;
constexpr int Q_SMEM = 98304 + Q_STAGES * 16384 + 32768 + 512;

struct ItemCursor {   // walks this CTA's items and their key tiles
  int item, nitems, step, qtiles, Sq, Sk, window, tile;
  int bh, r0, t0, t1;       // current item: (b, h), first row, visible other-side tile range
  __device__ __forceinline__ void load() {
    int qt;
    heavy_first(item, nitems / qtiles, Sq / 128, bh, qt);
    r0 = qt * 128;
    tile_range(r0, 128, Sk, window, tile, t0, t1);
  }
  __device__ __forceinline__ bool valid() const { return item < nitems; }
  __device__ __forceinline__ void next() {
    item += step;
    if (item < nitems) load();
  }
};

__global__ void __launch_bounds__(kThreadsTC, 1)
    attn_tc_dq_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_do,
                      const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_v,
                      const __grid_constant__ CUtensorMap tm_o, const __grid_constant__ CUtensorMap tm_dq,
                      const TcArgs a) {
  extern __shared__ uint8_t smem_raw[];
  pdl_trigger();   // the next kernel may be scheduled once every CTA of this grid runs
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQd = smem;                  // [2 items][Q 16 KB | dO 16 KB | O 16 KB]
  uint8_t* sKV = smem + 98304;
  uint8_t* sStage = sKV + Q_STAGES * 16384;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sStage + 32768);
  uint64_t* q_full = bars;              // [2]
  uint64_t* q_empty = q_full + 2;       // [2]
  uint64_t* kv_full = q_empty + 2;      // [Q_STAGES]
  uint64_t* kv_empty = kv_full + Q_STAGES;
  uint64_t* s_full = kv_empty + Q_STAGES;   // [3 buffers]
  uint64_t* ds_full = s_full + 3;         // [3 buffers]
  uint64_t* acc_full = ds_full + 3;       // [2]
  uint64_t* acc_empty = acc_full + 2;     // [2]
  uint64_t* dq_done = acc_empty + 2;      // [3 buffers]: the dQ MMA has read the buffer's dS
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(dq_done + 3);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int qtiles = (a.Sq + 127) / 128;
  const int nitems = a.B * a.H * qtiles;
  auto cursor = [&]() {
    ItemCursor c{(int)blockIdx.x, nitems, (int)gridDim.x, qtiles, a.Sq, a.Sk, a.window, 64, 0, 0, 0, 0};
    if (c.valid()) c.load();
    return c;
  };

  if (warp == 0 && lane == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&q_full[i], 1);
      mbar_init(&q_empty[i], 1);
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], 8);
    }
    for (int s = 0; s < Q_STAGES; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    for (int i = 0; i < 3; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&ds_full[i], 4);
      mbar_init(&dq_done[i], 1);
    }
    *abort_flag = 0;
    fence_barrier_init();
    tma_prefetch_desc(&tm_q);
    tma_prefetch_desc(&tm_do);
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
  pdl_wait();      // outputs of earlier kernels are read only from here on
  const Waiter wait{abort_flag, a.err};     // single-thread roles (the TMA producer)
  const WaiterW<> waitw{abort_flag, a.err};   // whole-warp roles (MMA issue, softmax)

  if (warp == 0) {
    if (lane == 0) {
      ItemCursor c = cursor();
      int t = 0, ii = 0;     // ii counts the items that have key tiles (empty ones touch no barrier)
      bool ok = true;
      for (; c.valid() && ok; c.next()) {
        if (c.t0 == c.t1) continue;
        const int ib = ii & 1;
        const int b = c.bh / a.H, h = c.bh % a.H;
        if (ii >= 2 && !wait(&q_empty[ib], (uint32_t)(((ii >> 1) - 1) & 1), kErrTimeoutEmpty)) break;
        mbar_arrive_expect_tx(&q_full[ib], 49152);
        load_rows(sQd + 49152 * ib, &tm_q, &q_full[ib], a.q_tm, b, h, c.r0);
        load_rows(sQd + 49152 * ib + 16384, &tm_do, &q_full[ib], a.do_tm, b, h, c.r0);
        load_rows(sQd + 49152 * ib + 32768, &tm_o, &q_full[ib], a.o_tm, b, h, c.r0);
        for (int kt = c.t0; kt < c.t1; ++kt, ++t) {
          const int s = t % Q_STAGES;
          const uint32_t use = (uint32_t)(t / Q_STAGES);
          if (t >= Q_STAGES && !wait(&kv_empty[s], (use & 1u) ^ 1u, kErrTimeoutEmpty)) { ok = false; break; }
          uint8_t* st = sKV + s * 16384;
          mbar_arrive_expect_tx(&kv_full[s], 16384);
          load_rows(st, &tm_k, &kv_full[s], a.k_tm, b, h, kt * 64);
          load_rows(st + 8192, &tm_v, &kv_full[s], a.v_tm, b, h, kt * 64);
        }
        ++ii;
      }
    }
  } else if (warp == 1 || warp == 10) {
    {   // the whole warp walks the schedule (uniform operands); one elected lane issues
      const uint32_t id_s = make_idesc_f16(128, 64, 0, 0);    // S = Q K^T, dP = dO V^T  [128 q][64 k]
      const uint32_t id_dq = make_idesc_f16(128, 64, 0, 1);   // dQ[128 q][64 d] += dS K (K MN-major)
      bool ok = true;
      // a cursor over the key-tile stream, resting on a tile of an item that has some (the item
      // counter ii, which picks the Q / dO / O buffer and the accumulator, counts only those)
      auto normalize = [&](ItemCursor& c, int& kt) {
        while (c.valid() && c.t0 == c.t1) { c.next(); if (c.valid()) kt = c.t0; }
      };
      auto advance = [&](ItemCursor& c, int& ii, int& kt) {
        if (++kt < c.t1) return;
        c.next();
        ++ii;
        if (c.valid()) kt = c.t0;
        normalize(c, kt);
      };
      ItemCursor c = cursor();
      int ii = 0, kt = c.valid() ? c.t0 : 0, t = 0;
      normalize(c, kt);
      if (warp == 1) {
        // scores: S = Q K^T and dP = dO V^T of tile t into buffer t % 3, once dQ(t - 3) has read it
        while (ok && c.valid()) {
          const int ib = ii & 1;
          if (t >= 3 && !waitw(&dq_done[t % 3], (uint32_t)(((t / 3) - 1) & 1), kErrTimeoutOther)) { ok = false; break; }
          if (kt == c.t0 && !waitw(&q_full[ib], (uint32_t)((ii >> 1) & 1), kErrTimeoutFull)) { ok = false; break; }
          const int s = t % Q_STAGES;
          if (!waitw(&kv_full[s], (uint32_t)(t / Q_STAGES) & 1u, kErrTimeoutFull)) { ok = false; break; }
          tc_fence_after();
          const uint32_t qa = smem_u32(sQd + 49152 * ib);
          const uint64_t qd = kdesc0(qa), dd = kdesc0(qa + 16384);
          const uint32_t ka = smem_u32(sKV + s * 16384), tS = tbase + 128 * (t % 3);
          const uint64_t kd = kdesc0(ka), vd = kdesc0(ka + 8192);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) umma_f16_w(tS, kstep(qd, kk), kstep(kd, kk), id_s, kk > 0 ? 1u : 0u);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) umma_f16_w(tS + 64, kstep(dd, kk), kstep(vd, kk), id_s, kk > 0 ? 1u : 0u);
          umma_commit_w(&s_full[t % 3]);
          ++t;
          advance(c, ii, kt);
        }
      } else {
        // gradient: dQ += dS K of tile t once its dS is in TMEM
        while (ok && c.valid()) {
          const int ia = ii & 1;
          const bool first = kt == c.t0, last = kt + 1 == c.t1;
          if (!waitw(&ds_full[t % 3], (uint32_t)((t / 3) & 1), kErrTimeoutReady)) { ok = false; break; }
          if (first && ii >= 2 && !waitw(&acc_empty[ia], (uint32_t)(((ii >> 1) - 1) & 1), kErrTimeoutOther)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const int s = t % Q_STAGES;
          const uint64_t kmn = mndesc0(smem_u32(sKV + s * 16384));
          const uint32_t tS = tbase + 128 * (t % 3), tQ = tbase + 384 + 64 * ia;
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)   // 64 keys = 4 k-steps; dS at S columns [0, 32)
            umma_ts_w(tQ, tS + kk * 8, mnstep(kmn, kk), id_dq, (!first || kk > 0) ? 1u : 0u);
          // (the score MMAs of tile t completed before its dS existed, so these commits also
          // cover their reads of K / V and of the item's Q / dO)
          umma_commit_w(&dq_done[t % 3]);
          umma_commit_w(&kv_empty[s]);
          if (last) {
            umma_commit_w(&acc_full[ia]);
            umma_commit_w(&q_empty[ia]);
          }
          ++t;
          advance(c, ii, kt);
        }
      }
    }
  } else {   // warps 2 .. 9
    const int g = (warp - 2) >> 2;
    const int quarter = warp & 3;
    const int row = 32 * quarter + lane;
    const uint32_t lane_off = (uint32_t)(32 * quarter) << 16;
    ItemCursor c = cursor();
    bool ok = true;
    int t = 0, ii = 0;
    uint8_t* stg = sStage + (warp - 2) * 4096;   // this warp's 32 rows x 32 f32 of dQ
    // lse of the row in the next item that has key tiles, fetched one item ahead
    auto next_item = [&](ItemCursor cn) {
      cn.next();
      while (cn.valid() && cn.t0 == cn.t1) cn.next();
      return cn;
    };
    auto fetch_lse = [&](const ItemCursor& cn) -> float {
      if (!cn.valid()) return INFINITY;
      const int qi = cn.r0 + row;
      return qi < a.Sq ? a.lse_in[(long)cn.bh * a.Sq + qi] : INFINITY;
    };
    ItemCursor cf = c;
    while (cf.valid() && cf.t0 == cf.t1) cf.next();
    float lse_next = fetch_lse(cf);
    for (; c.valid(); c.next()) {
      const int ib = ii & 1, ia = ii & 1;
      const int b = c.bh / a.H, h = c.bh % a.H;
      const int q0 = c.r0, qi = q0 + row;
      const bool qok = qi < a.Sq;
      const int nkt = c.t1 - c.t0;
      if (nkt == 0) {     // no visible key: dQ = 0; the item touches no barrier or buffer
        if (qok) {
          float4* dz = reinterpret_cast<float4*>(a.dq + b * a.dq_sb + h * a.dq_sh + (long)qi * a.dq_ld + 32 * g);
#pragma unroll
          for (int cc = 0; cc < 8; ++cc) dz[cc] = make_float4(0.f, 0.f, 0.f, 0.f);
          if (g == 0) a.Dsum[(long)c.bh * a.Sq + qi] = 0.f;
        }
        continue;
      }
      ++ii;
      const float lse = lse_next;
      lse_next = fetch_lse(next_item(c));
      if (ok) ok = waitw(&q_full[ib], (uint32_t)(((ii - 1) >> 1) & 1), kErrTimeoutFull);
      // D = rowsum(dO o O) from the swizzled dO and O tiles in shared memory
      float Dq = 0.f;
      if (ok) {
        const uint8_t* sdO = sQd + 49152 * ib + 16384;
        const uint8_t* sO = sdO + 16384;
#pragma unroll
        for (int cc = 0; cc < 8; ++cc) {
          const int off = row * 128 + ((cc ^ (row & 7)) << 4);
          const uint4 ov = *reinterpret_cast<const uint4*>(sO + off);
          const uint4 dv = *reinterpret_cast<const uint4*>(sdO + off);
          const __half2* o2 = reinterpret_cast<const __half2*>(&ov);
          const __half2* d2 = reinterpret_cast<const __half2*>(&dv);
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float2 of = __half22float2(o2[e]), df = __half22float2(d2[e]);
            Dq = fmaf(of.x, df.x, Dq);
            Dq = fmaf(of.y, df.y, Dq);
          }
        }
        if (!qok) Dq = 0.f;
        if (g == 0 && qok) a.Dsum[(long)c.bh * a.Sq + qi] = Dq;
      }
      for (int j = 0; j < nkt; ++j, ++t) {
        if ((t & 1) != g || !ok) continue;
        if (!waitw(&s_full[t % 3], (uint32_t)((t / 3) & 1), kErrTimeoutAccum)) { ok = false; continue; }
        tc_fence_after();
        const uint32_t tS = tbase + 128 * (t % 3);
        const int k0 = (c.t0 + j) * 64;
        const bool edge = !tile_visible(q0, 128, k0, 64, a.Sk, a.window);
        const uint64_t sc2 = f2(a.sl2, a.sl2), nl2 = f2(-lse, -lse), nd2 = f2(-Dq, -Dq);
        // two halves of 32 keys: S / dP of a half in, its dS row (packed f16 pairs, column e of
        // the slot holds keys 2e, 2e + 1) out to the half's 16 columns, which the other half no
        // longer reads
#pragma unroll 1
        for (int hf = 0; hf < 2; ++hf) {
          uint32_t sv[32], pv[32];
          tmem_ld32(tS + lane_off + 32 * hf, sv);
          tmem_ld32(tS + 64 + lane_off + 32 * hf, pv);
          tmem_ld_wait();
          if (edge) {
#pragma unroll
            for (int cc = 0; cc < 32; ++cc)
              if (!visible(qi, k0 + 32 * hf + cc, a.Sk, a.window)) sv[cc] = __float_as_uint(-INFINITY);
          }
          uint32_t pk[16];
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            float x0, x1, d0, d1;
            f2split(ffma2(f2(__uint_as_float(sv[2 * e]), __uint_as_float(sv[2 * e + 1])), sc2, nl2), x0, x1);
            float p0, p1;
            if (kPolyPair[e & 7]) {      // a share of the exponentials on the FMA pipes
              ex2_poly2(x0, x1, p0, p1);
            } else {
              p0 = ex2(x0);
              p1 = ex2(x1);
            }
            const uint64_t pp = f2(p0, p1);
            f2split(fmul2(pp, fadd2(f2(__uint_as_float(pv[2 * e]), __uint_as_float(pv[2 * e + 1])), nd2)), d0, d1);
            pk[e] = pack_f16x2(d0, d1);
          }
          tmem_st16(tS + lane_off + 16 * hf, pk);
        }
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&ds_full[t % 3]);
      }
      // epilogue of the item: warpgroup g stores dQ columns [32 g, 32 g + 32) of its 32 rows
      const bool have = ok && waitw(&acc_full[ia], (uint32_t)(((ii - 1) >> 1) & 1), kErrTimeoutAccum);
      ok = have;
      tc_fence_after();
      if (have) {
        uint32_t o[32];
        tmem_ld32(tbase + 384 + 64 * ia + 32 * g + lane_off, o);
        tmem_ld_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&acc_empty[ia]);   // the accumulator is free again
        if (lane == 0) bulk_wait_read<0>();             // the previous item's store has read stg
        __syncwarp();
#pragma unroll
        for (int cc = 0; cc < 8; ++cc)
          *reinterpret_cast<float4*>(stg + lane * 128 + ((cc ^ (lane & 7)) << 4)) =
              make_float4(__uint_as_float(o[4 * cc]) * a.scale, __uint_as_float(o[4 * cc + 1]) * a.scale,
                          __uint_as_float(o[4 * cc + 2]) * a.scale, __uint_as_float(o[4 * cc + 3]) * a.scale);
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          const int r0 = q0 + 32 * quarter;
          if (a.dq_tm) tma_store_4d(&tm_dq, stg, 32 * g, h, r0, b);
          else tma_store_4d(&tm_dq, stg, 32 * g, r0, h, b);
          bulk_commit();
        }
      }
    }
    if (lane == 0) bulk_wait_all();
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tbase, 512);
  }
}

// ============================================================================== dkdv pass
// CTA: 128 keys of one (b, h); query tiles of 64, warpgroup g takes tiles i = g, g + 2, ...
// TMEM: three buffers (query tiles in flight) at 128 b: S^T [0, 64) (P^T overwrites [0, 32)),
// dP^T [64, 128) (dS^T overwrites [64, 96)); dV at 384, dK at 448.
// smem: K 16 KB | V 16 KB | 4 x (Q 8 KB, dO 8 KB) | lse / D per warpgroup (x2) | barriers
constexpr int KV_SMEM = 32768 + NSTAGE * 16384 + 2048 + 512;

__global__ void __launch_bounds__(kThreadsTC, 1)
    attn_tc_dkdv_kernel(const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_v,
                        const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_do,
                        const TcArgs a) {
  extern __shared__ uint8_t smem_raw[];
  pdl_trigger();   // the next kernel may be scheduled once every CTA of this grid runs
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sK = smem;
  uint8_t* sV = smem + 16384;
  uint8_t* sQd = smem + 32768;
  // [2 groups][2 bufs][32 query pairs][lse 2 | D 2]: one 16-byte broadcast read per pair
  float* s_ld = reinterpret_cast<float*>(smem + 32768 + NSTAGE * 16384);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + 32768 + NSTAGE * 16384 + 2048);
  uint64_t* kv_full = bars;
  uint64_t* q_full = bars + 1;
  uint64_t* q_empty = q_full + NSTAGE;
  uint64_t* s_full = q_empty + NSTAGE;    // [3 buffers]
  uint64_t* ds_full = s_full + 3;         // [3 buffers]
  uint64_t* acc_full = ds_full + 3;
  uint64_t* gd_done = acc_full + 1;       // [3 buffers]: dV / dK MMAs have read the buffer
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(gd_done + 3);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int bh, kt;
  heavy_first((int)(blockIdx.y * gridDim.x + blockIdx.x), (int)gridDim.y, a.Sk / 128, bh, kt);
  const int b = bh / a.H, h = bh % a.H;
  const int k0 = kt * 128;
  int qt0, qt1;
  tile_range(k0, 128, a.Sq, a.window, 64, qt0, qt1);
  const int nqt = qt1 - qt0;

  if (warp == 0 && lane == 0) {
    mbar_init(kv_full, 1);
    for (int s = 0; s < NSTAGE; ++s) {
      mbar_init(&q_full[s], 1);
      mbar_init(&q_empty[s], 1);
    }
    for (int i = 0; i < 3; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&ds_full[i], 4);
      mbar_init(&gd_done[i], 1);
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
  pdl_wait();      // outputs of earlier kernels are read only from here on
  const uint32_t tV = tbase + 384, tK = tbase + 448;
  const Waiter wait{abort_flag, a.err};     // single-thread roles (the TMA producer)
  const WaiterW<> waitw{abort_flag, a.err};   // whole-warp roles (MMA issue, softmax)

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
    {   // S^T = K Q^T and dP^T = V dO^T of query tile i into buffer i % 3, once dV / dK (i - 3) read it
      const uint32_t id_s = make_idesc_f16(128, 64, 0, 0);    // S^T, dP^T [128 k][64 q]
      bool ok = waitw(kv_full, 0, kErrTimeoutFull);
      const uint64_t kd = kdesc0(smem_u32(sK)), vd = kdesc0(smem_u32(sV));
      for (int i = 0; i < nqt && ok; ++i) {
        const int s = i % NSTAGE;
        if (i >= 3 && !waitw(&gd_done[i % 3], (uint32_t)(((i / 3) - 1) & 1), kErrTimeoutOther)) { ok = false; break; }
        if (!waitw(&q_full[s], (uint32_t)(i / NSTAGE) & 1u, kErrTimeoutFull)) { ok = false; break; }
        tc_fence_after();
        const uint32_t qa = smem_u32(sQd + s * 16384), tS = tbase + 128 * (i % 3);
        const uint64_t qd = kdesc0(qa), dd = kdesc0(qa + 8192);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) umma_f16_w(tS, kstep(kd, kk), kstep(qd, kk), id_s, kk > 0 ? 1u : 0u);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) umma_f16_w(tS + 64, kstep(vd, kk), kstep(dd, kk), id_s, kk > 0 ? 1u : 0u);
        umma_commit_w(&s_full[i % 3]);
      }
    }
  } else if (warp == 10) {
    {   // dV += P^T dO and dK += dS^T Q of query tile i once P^T / dS^T are in TMEM
      const uint32_t id_g = make_idesc_f16(128, 64, 0, 1);    // dV / dK [128 k][64 d] (dO / Q MN-major)
      bool ok = true;
      for (int i = 0; i < nqt && ok; ++i) {
        const int s = i % NSTAGE;
        if (!waitw(&ds_full[i % 3], (uint32_t)((i / 3) & 1), kErrTimeoutReady)) { ok = false; break; }
        tc_fence_after();
        const uint32_t qa = smem_u32(sQd + s * 16384), tS = tbase + 128 * (i % 3);
        const uint64_t qmn = mndesc0(qa), dmn = mndesc0(qa + 8192);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)   // 64 queries = 4 k-steps; P^T at S^T columns [0, 32)
          umma_ts_w(tV, tS + kk * 8, mnstep(dmn, kk), id_g, (i > 0 || kk > 0) ? 1u : 0u);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)   // dS^T at dP^T columns [0, 32)
          umma_ts_w(tK, tS + 64 + kk * 8, mnstep(qmn, kk), id_g, (i > 0 || kk > 0) ? 1u : 0u);
        // (the score MMAs of tile i completed before its P^T existed: Q / dO are free as well)
        umma_commit_w(&gd_done[i % 3]);
        umma_commit_w(&q_empty[s]);
      }
      umma_commit_w(acc_full);
    }
  } else {   // warps 2 .. 9
    const int g = (warp - 2) >> 2;
    const int quarter = warp & 3;
    const int row = 32 * quarter + lane;
    const int kj = k0 + row;
    const int t = threadIdx.x - 64 - 128 * g;   // 0..127 within the warpgroup
    const uint32_t lane_off = (uint32_t)(32 * quarter) << 16;
    bool ok = true;
    int it = 0;
    // thread t holds lse (t < 64) or D (t >= 64) of query t % 64 of a tile; the value for the
    // group's next tile is fetched one tile ahead so its latency hides behind the current one
    auto fetch = [&](int i) -> float {
      const int qi = (qt0 + i) * 64 + (t & 63);
      if (qi >= a.Sq) return t < 64 ? INFINITY : 0.f;
      return t < 64 ? a.lse_in[(long)bh * a.Sq + qi] : a.Dsum[(long)bh * a.Sq + qi];
    };
    float next = g < nqt ? fetch(g) : 0.f;
    for (int i = g; i < nqt; i += 2, ++it) {
      const int q0 = (qt0 + i) * 64;
      float* lse_b = s_ld + 256 * g + 128 * (it & 1);
      lse_b[4 * ((t & 63) >> 1) + (t >= 64 ? 2 : 0) + (t & 1)] = next;
      if (i + 2 < nqt) next = fetch(i + 2);
      if (g == 0) named_bar(1, 128);   // every warp of the group passes it once per tile, also after an abort
      else named_bar(2, 128);
      if (ok) ok = waitw(&s_full[i % 3], (uint32_t)((i / 3) & 1), kErrTimeoutAccum);
      if (!ok) continue;
      tc_fence_after();
      const uint32_t tS = tbase + 128 * (i % 3);
      const bool edge = !tile_visible(k0, 128, q0, 64, a.Sq, a.window) || kj >= a.Sk;
      const uint64_t sc2 = f2(a.sl2, a.sl2);
      const float4* ld4 = reinterpret_cast<const float4*>(lse_b);
      // two halves of 32 queries: S^T / dP^T of a half in, its P^T / dS^T (packed f16) out to the
      // first 16 columns of the half's slot (the packed halves never overlap columns still to read),
      // so about 100 values per thread are live instead of 192
#pragma unroll 1
      for (int hf = 0; hf < 2; ++hf) {
        uint32_t sv[32], pv[32];
        tmem_ld32(tS + lane_off + 32 * hf, sv);
        tmem_ld32(tS + 64 + lane_off + 32 * hf, pv);
        tmem_ld_wait();
        if (edge) {
          // (queries past Sq already carry lse = +inf, so P = 0 there)
#pragma unroll
          for (int c = 0; c < 32; ++c)
            if (!visible(q0 + 32 * hf + c, kj, a.Sk, a.window)) sv[c] = __float_as_uint(-INFINITY);
        }
        uint32_t pk[16], dk[16];
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          const float4 w4 = ld4[16 * hf + e];      // smem broadcast read: lse and D of queries 2e, 2e + 1
          const float2 lz = make_float2(w4.x, w4.y), dz = make_float2(w4.z, w4.w);
          float x0, x1, d0, d1;
          f2split(ffma2(f2(__uint_as_float(sv[2 * e]), __uint_as_float(sv[2 * e + 1])), sc2, f2(-lz.x, -lz.y)), x0,
                  x1);
          float p0, p1;
          if (kPolyPair[e & 7]) {      // a share of the exponentials on the FMA pipes
            ex2_poly2(x0, x1, p0, p1);
          } else {
            p0 = ex2(x0);
            p1 = ex2(x1);
          }
          f2split(fmul2(f2(p0, p1), fadd2(f2(__uint_as_float(pv[2 * e]), __uint_as_float(pv[2 * e + 1])),
                                          f2(-dz.x, -dz.y))), d0, d1);
          pk[e] = pack_f16x2(p0, p1);
          dk[e] = pack_f16x2(d0, d1);
        }
        tmem_st16(tS + lane_off + 16 * hf, pk);
        tmem_st16(tS + 64 + lane_off + 16 * hf, dk);
      }
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&ds_full[i % 3]);
    }
    const bool have = ok && waitw(acc_full, 0, kErrTimeoutAccum) && nqt > 0;
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

// ============================================================================== short key range
// Attention whose keys fit one 128-wide tile (1 <= Sk <= 128, no band): the cross-attention to the
// 128 conditioning tokens.  With one or two 64-key tiles per 128 queries, the general kernels spend
// each CTA on load / MMA / softmax / epilogue latencies in series.  These kernels are persistent
// over 128-query items (CTA c takes a contiguous range of them), load an item's Q (dO, O) and the
// head's whole K / V in one TMA transaction into one of two buffers (K / V only when the buffer's
// previous item had another head), and keep two items in flight:
// softmax warpgroup g takes the CTA's items i with i % 2 == g, on its own TMEM buffer, while the
// MMA warp already issues the next item's score MMAs.  Keys at or past Sk (TMA zero fill) are
// masked to -inf.
constexpr int SF_BUF = 3 * 16384;                 // forward: Q | K | V of one item
constexpr int SF_STG = 8 * 4096;                  // forward: 32 rows x 128 B of O per softmax warp
constexpr int SF_SMEM = 2 * SF_BUF + SF_STG + 256;
constexpr int SQ_BUF = 5 * 16384;                 // dq pass: Q | dO | O | K | V of one item
constexpr int SQ_STG = 8 * 8192;                  // dq pass: 32 rows x 256 B of dQ per softmax warp
constexpr int SQ_SMEM = 2 * SQ_BUF + SQ_STG + 256;

// CTA c's items: a contiguous range of the (b, h, 128-query tile) order, so that consecutive items
// of a CTA mostly share their head and a buffer's K / V can stay in place
__device__ __forceinline__ void short_range(int nitems, int& first, int& n) {
  const int G = (int)gridDim.x, c = (int)blockIdx.x, per = nitems / G, rem = nitems % G;
  first = c * per + min(c, rem);
  n = per + (c < rem ? 1 : 0);
}

// Forward.  TMEM buffer g at 192 g: S [0, 128) (P overwrites [0, 64) as packed f16), O [128, 192).
__global__ void __launch_bounds__(kThreadsTC, 1)
    attn_short_fwd_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                          const __grid_constant__ CUtensorMap tm_v, const TcArgs a) {
  extern __shared__ uint8_t smem_raw[];
  pdl_trigger();
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sstg = smem + 2 * SF_BUF;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sstg + SF_STG);
  uint64_t* in_full = bars;            // [2] TMA -> MMA
  uint64_t* in_empty = in_full + 2;    // [2] P V done -> TMA
  uint64_t* s_full = in_empty + 2;     // [2] S MMAs done -> softmax
  uint64_t* p_full = s_full + 2;       // [2] P in TMEM -> MMA (one arrival per softmax warp)
  uint64_t* o_full = p_full + 2;       // [2] P V done -> epilogue
  uint64_t* o_empty = o_full + 2;      // [2] epilogue read O -> the buffer's next S MMAs
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(o_empty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int qtiles = (a.Sq + 127) / 128, nitems = a.B * a.H * qtiles;
  int first, n;
  short_range(nitems, first, n);
  auto item_of = [&](int i, int& b, int& h, int& bh, int& q0) {
    const int item = first + i;
    bh = item / qtiles;
    q0 = (item % qtiles) * 128;
    b = bh / a.H;
    h = bh % a.H;
  };

  if (warp == 0 && lane == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&in_full[i], 1);
      mbar_init(&in_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 4);
      mbar_init(&o_full[i], 1);
      mbar_init(&o_empty[i], 4);
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
  pdl_wait();
  const Waiter wait{abort_flag, a.err};
  const WaiterW<> waitw{abort_flag, a.err};

  if (warp == 0) {
    if (lane == 0) {
      for (int i = 0; i < n; ++i) {
        int b, h, bh, q0;
        item_of(i, b, h, bh, q0);
        const int bf = i & 1;
        if (i >= 2 && !wait(&in_empty[bf], (uint32_t)(((i >> 1) - 1) & 1), kErrTimeoutEmpty)) break;
        uint8_t* buf = smem + bf * SF_BUF;
        int pb, ph_, pbh = -1, pq;
        if (i >= 2) item_of(i - 2, pb, ph_, pbh, pq);
        const bool kv = pbh != bh;     // the buffer holds another head's K / V
        mbar_arrive_expect_tx(&in_full[bf], (uint32_t)(kv ? SF_BUF : 16384));
        load_rows(buf, &tm_q, &in_full[bf], a.q_tm, b, h, q0);
        if (kv) {
          load_rows(buf + 16384, &tm_k, &in_full[bf], a.k_tm, b, h, 0);
          load_rows(buf + 32768, &tm_v, &in_full[bf], a.v_tm, b, h, 0);
        }
      }
    }
  } else if (warp == 1) {
    const uint32_t id_s = make_idesc_f16(128, 128, 0, 0);   // S[128 q][128 k] = Q K^T
    const uint32_t id_o = make_idesc_f16(128, 64, 0, 1);    // O[128 q][64 d] = P V (V MN-major)
    auto issue_s = [&](int i) -> bool {
      const int bf = i & 1;
      if (!waitw(&in_full[bf], (uint32_t)((i >> 1) & 1), kErrTimeoutFull)) return false;
      if (i >= 2 && !waitw(&o_empty[bf], (uint32_t)(((i >> 1) - 1) & 1), kErrTimeoutOther)) return false;
      tc_fence_after();
      const uint32_t ba = smem_u32(smem + bf * SF_BUF);
      const uint64_t qd = kdesc0(ba), kd = kdesc0(ba + 16384);
      const uint32_t tS = tbase + 192 * bf;
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) umma_f16_w(tS, kstep(qd, kk), kstep(kd, kk), id_s, kk > 0 ? 1u : 0u);
      umma_commit_w(&s_full[bf]);
      return true;
    };
    bool ok = n == 0 || issue_s(0);
    for (int i = 0; i < n && ok; ++i) {
      const int bf = i & 1;
      if (i + 1 < n && !issue_s(i + 1)) { ok = false; break; }
      if (!waitw(&p_full[bf], (uint32_t)((i >> 1) & 1), kErrTimeoutReady)) { ok = false; break; }
      tc_fence_after();
      const uint64_t vd = mndesc0(smem_u32(smem + bf * SF_BUF + 32768));
      const uint32_t tS = tbase + 192 * bf, tO = tS + 128;
#pragma unroll
      for (int kk = 0; kk < 8; ++kk)   // 128 keys = 8 k-steps; P at S columns [0, 64)
        umma_ts_w(tO, tS + kk * 8, mnstep(vd, kk), id_o, kk > 0 ? 1u : 0u);
      umma_commit_w(&o_full[bf]);
      umma_commit_w(&in_empty[bf]);
    }
  } else if (warp < 10) {
    const int g = (warp - 2) >> 2;
    const int quarter = warp & 3;
    const int row = 32 * quarter + lane;
    const uint32_t lane_off = (uint32_t)(32 * quarter) << 16;
    const uint32_t tS = tbase + 192 * g, tO = tS + 128;
    bool ok = true;
    for (int i = g; i < n && ok; i += 2) {
      int b, h, bh, q0;
      item_of(i, b, h, bh, q0);
      const int qi = q0 + row;
      const uint32_t ph = (uint32_t)((i >> 1) & 1);
      if (!waitw(&s_full[g], ph, kErrTimeoutAccum)) { ok = false; break; }
      tc_fence_after();
      // pass 1: the row max over the visible keys
      float mx = -INFINITY;
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        uint32_t v[32];
        tmem_ld32(tS + lane_off + 32 * c, v);
        tmem_ld_wait();
#pragma unroll
        for (int e = 0; e < 32; ++e)
          if (32 * c + e < a.Sk) mx = fmaxf(mx, __uint_as_float(v[e]));
      }
      const float mb = mx == -INFINITY ? 0.f : mx * a.sl2;   // (scale > 0 keeps the order)
      // pass 2: P = 2^(s scale log2 e - m) as packed f16; chunk c's 32 keys go to columns
      // [16 c, 16 c + 16), which the later chunks no longer read
      const uint64_t sc2 = f2(a.sl2, a.sl2), nb2 = f2(-mb, -mb);
      uint64_t lsum[2] = {f2(0.f, 0.f), f2(0.f, 0.f)};
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        uint32_t v[32];
        tmem_ld32(tS + lane_off + 32 * c, v);
        tmem_ld_wait();
        if (32 * c + 32 > a.Sk) {
#pragma unroll
          for (int e = 0; e < 32; ++e)
            if (32 * c + e >= a.Sk) v[e] = __float_as_uint(-INFINITY);
        }
        uint32_t pk[16];
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          float x0, x1, p0, p1;
          f2split(ffma2(f2(__uint_as_float(v[2 * e]), __uint_as_float(v[2 * e + 1])), sc2, nb2), x0, x1);
          if (kPolyPair[e & 7]) {
            ex2_poly2(x0, x1, p0, p1);
            if (32 * c + 2 * e >= a.Sk) p0 = 0.f;       // (the polynomial clamps -inf to 2^-125)
            if (32 * c + 2 * e + 1 >= a.Sk) p1 = 0.f;
          } else {
            p0 = ex2(x0);
            p1 = ex2(x1);
          }
          lsum[e & 1] = fadd2(lsum[e & 1], f2(p0, p1));
          pk[e] = pack_f16x2(p0, p1);
        }
        tmem_st16(tS + lane_off + 16 * c, pk);
      }
      float l;
      {
        float l0, l1, l2, l3;
        f2split(lsum[0], l0, l1);
        f2split(lsum[1], l2, l3);
        l = (l0 + l1) + (l2 + l3);
      }
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[g]);
      // epilogue: O / l to the f16 output, the row's log2-sum-exp
      if (!waitw(&o_full[g], ph, kErrTimeoutAccum)) { ok = false; break; }
      tc_fence_after();
      uint32_t o[64];
      tmem_ld32(tO + lane_off, *reinterpret_cast<uint32_t(*)[32]>(&o[0]));
      tmem_ld32(tO + lane_off + 32, *reinterpret_cast<uint32_t(*)[32]>(&o[32]));
      tmem_ld_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&o_empty[g]);
      // O / l through this warp's staging rows (16-byte chunk c of row r at c ^ (r & 7)), then
      // stored four rows (4 x 128 contiguous bytes) per warp instruction
      {
        const float inv = l > 0.f ? 1.f / l : 0.f;
        uint8_t* stg = sstg + (warp - 2) * 4096;
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          uint4 w4;
          w4.x = pack_f16x2(__uint_as_float(o[8 * c]) * inv, __uint_as_float(o[8 * c + 1]) * inv);
          w4.y = pack_f16x2(__uint_as_float(o[8 * c + 2]) * inv, __uint_as_float(o[8 * c + 3]) * inv);
          w4.z = pack_f16x2(__uint_as_float(o[8 * c + 4]) * inv, __uint_as_float(o[8 * c + 5]) * inv);
          w4.w = pack_f16x2(__uint_as_float(o[8 * c + 6]) * inv, __uint_as_float(o[8 * c + 7]) * inv);
          *reinterpret_cast<uint4*>(stg + lane * 128 + ((c ^ (lane & 7)) << 4)) = w4;
        }
        __syncwarp();
#pragma unroll
        for (int it = 0; it < 8; ++it) {
          const int r = 4 * it + (lane >> 3), c = lane & 7, qr = q0 + 32 * quarter + r;
          const uint4 w4 = *reinterpret_cast<const uint4*>(stg + r * 128 + ((c ^ (r & 7)) << 4));
          if (qr < a.Sq) reinterpret_cast<uint4*>(a.o + b * a.o_sb + h * a.o_sh + (long)qr * a.o_ld)[c] = w4;
        }
        __syncwarp();
        if (qi < a.Sq && a.lse) a.lse[(long)bh * a.Sq + qi] = mb + log2f(fmaxf(l, 1e-30f));
      }
    }
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tbase, 512);
  }
}

// dQ pass (and D = rowsum(dO o O) for the dk / dv pass).  TMEM buffer g at 256 g: S [0, 128) (dS
// overwrites [0, 64) as packed f16), dP [128, 256) (dQ accumulates into [128, 192) once every dP
// value has been read).
__global__ void __launch_bounds__(kThreadsTC, 1)
    attn_short_dq_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_do,
                         const __grid_constant__ CUtensorMap tm_o, const __grid_constant__ CUtensorMap tm_k,
                         const __grid_constant__ CUtensorMap tm_v, const TcArgs a) {
  extern __shared__ uint8_t smem_raw[];
  pdl_trigger();
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sstg = smem + 2 * SQ_BUF;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sstg + SQ_STG);
  uint64_t* in_full = bars;            // [2] TMA -> MMA and softmax (D)
  uint64_t* in_empty = in_full + 2;    // [2] dQ MMAs done -> TMA
  uint64_t* sp_full = in_empty + 2;    // [2] S and dP MMAs done -> softmax
  uint64_t* ds_full = sp_full + 2;     // [2] dS in TMEM -> MMA (one arrival per softmax warp)
  uint64_t* dq_full = ds_full + 2;     // [2] dQ MMAs done -> epilogue
  uint64_t* dq_empty = dq_full + 2;    // [2] epilogue read dQ -> the buffer's next MMAs
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(dq_empty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int qtiles = (a.Sq + 127) / 128, nitems = a.B * a.H * qtiles;
  int first, n;
  short_range(nitems, first, n);
  auto item_of = [&](int i, int& b, int& h, int& bh, int& q0) {
    const int item = first + i;
    bh = item / qtiles;
    q0 = (item % qtiles) * 128;
    b = bh / a.H;
    h = bh % a.H;
  };

  if (warp == 0 && lane == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&in_full[i], 1);
      mbar_init(&in_empty[i], 1);
      mbar_init(&sp_full[i], 1);
      mbar_init(&ds_full[i], 4);
      mbar_init(&dq_full[i], 1);
      mbar_init(&dq_empty[i], 4);
    }
    *abort_flag = 0;
    fence_barrier_init();
    tma_prefetch_desc(&tm_q);
    tma_prefetch_desc(&tm_do);
    tma_prefetch_desc(&tm_o);
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
  pdl_wait();
  const Waiter wait{abort_flag, a.err};
  const WaiterW<> waitw{abort_flag, a.err};

  if (warp == 0) {
    if (lane == 0) {
      for (int i = 0; i < n; ++i) {
        int b, h, bh, q0;
        item_of(i, b, h, bh, q0);
        const int bf = i & 1;
        if (i >= 2 && !wait(&in_empty[bf], (uint32_t)(((i >> 1) - 1) & 1), kErrTimeoutEmpty)) break;
        uint8_t* buf = smem + bf * SQ_BUF;
        int pb, ph_, pbh = -1, pq;
        if (i >= 2) item_of(i - 2, pb, ph_, pbh, pq);
        const bool kv = pbh != bh;     // the buffer holds another head's K / V
        mbar_arrive_expect_tx(&in_full[bf], (uint32_t)(kv ? SQ_BUF : 49152));
        load_rows(buf, &tm_q, &in_full[bf], a.q_tm, b, h, q0);
        load_rows(buf + 16384, &tm_do, &in_full[bf], a.do_tm, b, h, q0);
        load_rows(buf + 32768, &tm_o, &in_full[bf], a.o_tm, b, h, q0);
        if (kv) {
          load_rows(buf + 49152, &tm_k, &in_full[bf], a.k_tm, b, h, 0);
          load_rows(buf + 65536, &tm_v, &in_full[bf], a.v_tm, b, h, 0);
        }
      }
    }
  } else if (warp == 1) {
    const uint32_t id_s = make_idesc_f16(128, 128, 0, 0);    // S = Q K^T, dP = dO V^T  [128 q][128 k]
    const uint32_t id_dq = make_idesc_f16(128, 64, 0, 1);    // dQ[128 q][64 d] = dS K (K MN-major)
    auto issue_sp = [&](int i) -> bool {
      const int bf = i & 1;
      if (!waitw(&in_full[bf], (uint32_t)((i >> 1) & 1), kErrTimeoutFull)) return false;
      if (i >= 2 && !waitw(&dq_empty[bf], (uint32_t)(((i >> 1) - 1) & 1), kErrTimeoutOther)) return false;
      tc_fence_after();
      const uint32_t ba = smem_u32(smem + bf * SQ_BUF);
      const uint64_t qd = kdesc0(ba), dd = kdesc0(ba + 16384), kd = kdesc0(ba + 49152), vd = kdesc0(ba + 65536);
      const uint32_t tS = tbase + 256 * bf;
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) umma_f16_w(tS, kstep(qd, kk), kstep(kd, kk), id_s, kk > 0 ? 1u : 0u);
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) umma_f16_w(tS + 128, kstep(dd, kk), kstep(vd, kk), id_s, kk > 0 ? 1u : 0u);
      umma_commit_w(&sp_full[bf]);
      return true;
    };
    bool ok = n == 0 || issue_sp(0);
    for (int i = 0; i < n && ok; ++i) {
      const int bf = i & 1;
      if (i + 1 < n && !issue_sp(i + 1)) { ok = false; break; }
      if (!waitw(&ds_full[bf], (uint32_t)((i >> 1) & 1), kErrTimeoutReady)) { ok = false; break; }
      tc_fence_after();
      const uint64_t kmn = mndesc0(smem_u32(smem + bf * SQ_BUF + 49152));
      const uint32_t tS = tbase + 256 * bf, tQ = tS + 128;
#pragma unroll
      for (int kk = 0; kk < 8; ++kk)   // 128 keys = 8 k-steps; dS at S columns [0, 64)
        umma_ts_w(tQ, tS + kk * 8, mnstep(kmn, kk), id_dq, kk > 0 ? 1u : 0u);
      umma_commit_w(&dq_full[bf]);
      umma_commit_w(&in_empty[bf]);
    }
  } else if (warp < 10) {
    const int g = (warp - 2) >> 2;
    const int quarter = warp & 3;
    const int row = 32 * quarter + lane;
    const uint32_t lane_off = (uint32_t)(32 * quarter) << 16;
    const uint32_t tS = tbase + 256 * g, tP = tS + 128;
    bool ok = true;
    for (int i = g; i < n && ok; i += 2) {
      int b, h, bh, q0;
      item_of(i, b, h, bh, q0);
      const int qi = q0 + row;
      const bool qok = qi < a.Sq;
      const uint32_t ph = (uint32_t)((i >> 1) & 1);
      const float lse = qok ? a.lse_in[(long)bh * a.Sq + qi] : INFINITY;
      if (!waitw(&in_full[g], ph, kErrTimeoutFull)) { ok = false; break; }
      // D = rowsum(dO o O) from the swizzled dO and O tiles in shared memory
      float Dq = 0.f;
      {
        const uint8_t* sdO = smem + g * SQ_BUF + 16384;
        const uint8_t* sO = sdO + 16384;
#pragma unroll
        for (int cc = 0; cc < 8; ++cc) {
          const int off = row * 128 + ((cc ^ (row & 7)) << 4);
          const uint4 ov = *reinterpret_cast<const uint4*>(sO + off);
          const uint4 dv = *reinterpret_cast<const uint4*>(sdO + off);
          const __half2* o2 = reinterpret_cast<const __half2*>(&ov);
          const __half2* d2 = reinterpret_cast<const __half2*>(&dv);
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float2 of = __half22float2(o2[e]), df = __half22float2(d2[e]);
            Dq = fmaf(of.x, df.x, Dq);
            Dq = fmaf(of.y, df.y, Dq);
          }
        }
      }
      if (!qok) Dq = 0.f;
      if (qok) a.Dsum[(long)bh * a.Sq + qi] = Dq;
      if (!waitw(&sp_full[g], ph, kErrTimeoutAccum)) { ok = false; break; }
      tc_fence_after();
      const uint64_t sc2 = f2(a.sl2, a.sl2), nl2 = f2(-lse, -lse), nd2 = f2(-Dq, -Dq);
      // chunk c's 32 keys: S / dP in, dS (packed f16) out to columns [16 c, 16 c + 16)
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        uint32_t sv[32], pv[32];
        tmem_ld32(tS + lane_off + 32 * c, sv);
        tmem_ld32(tP + lane_off + 32 * c, pv);
        tmem_ld_wait();
        uint32_t pk[16];
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          float x0, x1, p0, p1, d0, d1;
          f2split(ffma2(f2(__uint_as_float(sv[2 * e]), __uint_as_float(sv[2 * e + 1])), sc2, nl2), x0, x1);
          if (kPolyPair[e & 7]) {
            ex2_poly2(x0, x1, p0, p1);
          } else {
            p0 = ex2(x0);
            p1 = ex2(x1);
          }
          if (32 * c + 2 * e >= a.Sk) p0 = 0.f;        // keys past Sk (zero-filled rows)
          if (32 * c + 2 * e + 1 >= a.Sk) p1 = 0.f;
          f2split(fmul2(f2(p0, p1), fadd2(f2(__uint_as_float(pv[2 * e]), __uint_as_float(pv[2 * e + 1])), nd2)), d0,
                  d1);
          pk[e] = pack_f16x2(d0, d1);
        }
        tmem_st16(tS + lane_off + 16 * c, pk);
      }
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&ds_full[g]);
      // epilogue: scale dQ to the f32 output
      if (!waitw(&dq_full[g], ph, kErrTimeoutAccum)) { ok = false; break; }
      tc_fence_after();
      uint32_t o[64];
      tmem_ld32(tP + lane_off, *reinterpret_cast<uint32_t(*)[32]>(&o[0]));
      tmem_ld32(tP + lane_off + 32, *reinterpret_cast<uint32_t(*)[32]>(&o[32]));
      tmem_ld_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&dq_empty[g]);
      // dQ through this warp's staging rows (16-byte chunk c of row r at c ^ (r & 15)), then
      // stored two rows (2 x 256 contiguous bytes) per warp instruction
      {
        uint8_t* stg = sstg + (warp - 2) * 8192;
#pragma unroll
        for (int c = 0; c < 16; ++c)
          *reinterpret_cast<float4*>(stg + lane * 256 + ((c ^ (lane & 15)) << 4)) =
              make_float4(__uint_as_float(o[4 * c]) * a.scale, __uint_as_float(o[4 * c + 1]) * a.scale,
                          __uint_as_float(o[4 * c + 2]) * a.scale, __uint_as_float(o[4 * c + 3]) * a.scale);
        __syncwarp();
#pragma unroll
        for (int it = 0; it < 16; ++it) {
          const int r = 2 * it + (lane >> 4), c = lane & 15, qr = q0 + 32 * quarter + r;
          const float4 v4 = *reinterpret_cast<const float4*>(stg + r * 256 + ((c ^ (r & 15)) << 4));
          if (qr < a.Sq) reinterpret_cast<float4*>(a.dq + b * a.dq_sb + h * a.dq_sh + (long)qr * a.dq_ld)[c] = v4;
        }
        __syncwarp();
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
// 4-D tensor map over a strided (b, h, s, d) tensor with 64 values per row (d): the smaller of
// the head / row strides goes second so the strides grow; the box is `rows` rows x `box_d`
// values of one (b, h) (box_d x element size = 128 bytes, the swizzle span).
int make_map4t(CUtensorMap* m, CUtensorMapDataType dt, int esize, const void* base, long sb, long sh, long ld,
               int B, int H, int S, int box_d, int rows, int& tm, std::string& err) {
  PFN_encodeTiled enc = encode_tiled_fn(err);
  if (!enc) return 1;
  if ((reinterpret_cast<uintptr_t>(base) & 15) || (sh * esize) % 16 || (ld * esize) % 16 || (sb * esize) % 16) {
    err = "attention: tensor rows and strides must be 16-byte aligned";
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
  cuuint64_t strides[3] = {(cuuint64_t)(s1 * esize), (cuuint64_t)(s2 * esize), (cuuint64_t)(s3 * esize)};
  cuuint32_t box[4] = {(cuuint32_t)box_d, tm ? 1u : (cuuint32_t)rows, tm ? (cuuint32_t)rows : 1u, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  const CUresult r = enc(m, dt, 4, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                         CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    err = "attention: cuTensorMapEncodeTiled failed (" + std::to_string((int)r) + ")";
    return 1;
  }
  return 0;
}

int make_map4(CUtensorMap* m, const __half* base, long sb, long sh, long ld, int B, int H, int S, int rows,
              int& tm, std::string& err) {
  return make_map4t(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, base, sb, sh, ld, B, H, S, 64, rows, tm, err);
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

int set_tc_attrs(int device, std::string& err) {
  const char* what = "attention tc smem attributes";
  return smem_attr(reinterpret_cast<const void*>(attn_tc_fwd_kernel), smem_req(F_SMEM), device, what, err) ||
         smem_attr(reinterpret_cast<const void*>(attn_tc_dq_kernel), smem_req(Q_SMEM), device, what, err) ||
         smem_attr(reinterpret_cast<const void*>(attn_tc_dkdv_kernel), smem_req(KV_SMEM), device, what, err) ||
         smem_attr(reinterpret_cast<const void*>(attn_short_fwd_kernel), smem_req(SF_SMEM), device, what, err) ||
         smem_attr(reinterpret_cast<const void*>(attn_short_dq_kernel), smem_req(SQ_SMEM), device, what, err);
}

// the keys fit one 128-wide tile and there is no band: the short-range kernels
bool short_keys(const AttnArgs& p) { return p.Sk >= 1 && p.Sk <= 128 && p.window < 0; }

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
  if (set_tc_attrs(c->device, err)) return 1;
  TcArgs a = tc_args(p);
  a.err = c->d_err;
  CUtensorMap mq, mk, mv;
  const int kv_rows = short_keys(p) ? 128 : 64;
  if (make_map4(&mq, p.q, p.q_sb, p.q_sh, p.q_ld, p.B, p.H, p.Sq, 128, a.q_tm, err) ||
      make_map4(&mk, p.k, p.k_sb, p.k_sh, p.k_ld, p.B, p.H, p.Sk, kv_rows, a.k_tm, err) ||
      make_map4(&mv, p.v, p.v_sb, p.v_sh, p.v_ld, p.B, p.H, p.Sk, kv_rows, a.v_tm, err))
    return 1;
  ProfScope prof_(c, "attn.fwd");
  if (short_keys(p)) {   // persistent over 128-query items
    const long items = (long)p.B * p.H * ((p.Sq + 127) / 128);
    const unsigned grid = (unsigned)(items < (long)c->sm_count ? items : (long)c->sm_count);
    launch_pdl(c, attn_short_fwd_kernel, grid, kThreadsTC, smem_req(SF_SMEM), mq, mk, mv, a);
    return check_launch("attn short fwd", err);
  }
  dim3 grid((unsigned)((p.Sq + 255) / 256), (unsigned)(p.B * p.H));
  launch_pdl(c, attn_tc_fwd_kernel, grid, kThreadsTC, smem_req(F_SMEM), mq, mk, mv, a);
  return check_launch("attn tc fwd", err);
}

int attn_tc_grads(Ctx* c, const AttnArgs& p, bool want_dkdv, std::string& err) {
  if (set_tc_attrs(c->device, err)) return 1;
  TcArgs a = tc_args(p);
  a.err = c->d_err;
  {
    CUtensorMap mq, mdo, mk, mv, mo, mdq;
    if (short_keys(p)) {
      if (make_map4(&mq, p.q, p.q_sb, p.q_sh, p.q_ld, p.B, p.H, p.Sq, 128, a.q_tm, err) ||
          make_map4(&mdo, p.dO, p.dO_sb, p.dO_sh, p.dO_ld, p.B, p.H, p.Sq, 128, a.do_tm, err) ||
          make_map4(&mo, p.o, p.o_sb, p.o_sh, p.o_ld, p.B, p.H, p.Sq, 128, a.o_tm, err) ||
          make_map4(&mk, p.k, p.k_sb, p.k_sh, p.k_ld, p.B, p.H, p.Sk, 128, a.k_tm, err) ||
          make_map4(&mv, p.v, p.v_sb, p.v_sh, p.v_ld, p.B, p.H, p.Sk, 128, a.v_tm, err))
        return 1;
      ProfScope prof_(c, "attn.bwd_dq");
      const long items = (long)p.B * p.H * ((p.Sq + 127) / 128);
      const unsigned grid = (unsigned)(items < (long)c->sm_count ? items : (long)c->sm_count);
      launch_pdl(c, attn_short_dq_kernel, grid, kThreadsTC, smem_req(SQ_SMEM), mq, mdo, mo, mk, mv, a);
      if (check_launch("attn short dq", err)) return 1;
    } else {
      if (make_map4(&mq, p.q, p.q_sb, p.q_sh, p.q_ld, p.B, p.H, p.Sq, 128, a.q_tm, err) ||
          make_map4(&mdo, p.dO, p.dO_sb, p.dO_sh, p.dO_ld, p.B, p.H, p.Sq, 128, a.do_tm, err) ||
          make_map4(&mk, p.k, p.k_sb, p.k_sh, p.k_ld, p.B, p.H, p.Sk, 64, a.k_tm, err) ||
          make_map4(&mv, p.v, p.v_sb, p.v_sh, p.v_ld, p.B, p.H, p.Sk, 64, a.v_tm, err) ||
          make_map4(&mo, p.o, p.o_sb, p.o_sh, p.o_ld, p.B, p.H, p.Sq, 128, a.o_tm, err) ||
          make_map4t(&mdq, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, p.dq, p.dq_sb, p.dq_sh, p.dq_ld, p.B, p.H, p.Sq, 32, 32,
                     a.dq_tm, err))
        return 1;
      ProfScope prof_(c, "attn.bwd_dq");
      const long items = (long)p.B * p.H * ((p.Sq + 127) / 128);   // persistent: one CTA per SM at most
      const unsigned grid = (unsigned)(items < (long)c->sm_count ? items : (long)c->sm_count);
      launch_pdl(c, attn_tc_dq_kernel, grid, kThreadsTC, smem_req(Q_SMEM), mq, mdo, mk, mv, mo, mdq, a);
      if (check_launch("attn tc dq", err)) return 1;
    }
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
    launch_pdl(c, attn_tc_dkdv_kernel, grid, kThreadsTC, smem_req(KV_SMEM), mk, mv, mq, mdo, a);
    if (check_launch("attn tc dkdv", err)) return 1;
  }
  return 0;
}

}  // namespace sa3k
