// attention.cu -- scaled-dot-product attention forward and backward, head_dim 64.
//
// Replaces nn::sdpa (src/nn.h:135-144: mul_mat(k, q) -> soft_max_ext(scale) -> mul_mat(v^T, kq))
// and its autodiff backward (SOFT_MAX_BACK + OUT_PROD), for the DiT's dense self-attention
// (src/dit.h:199-221), its cross-attention to the conditioning (src/dit.h:225-240) and the
// banded variant |q - k| <= window (the mask of src/same_ae.h:96-106).
//
// Flash-style tiling: nothing of size S x S touches HBM.  Forward keeps a running row max / sum
// and writes O and the row log-sum-exp; the backward recomputes P from that LSE.  The backward
// is split into two deterministic passes without atomics:
//   dq pass   (one CTA per 64 queries, loop over keys):  dQ = scale * dS K
//   dkdv pass (one CTA per 64 keys, loop over queries):  dV = P^T dO,  dK = scale * dS^T Q
// with dS = P o (dP - D), dP = dO V^T, D = rowsum(dO o O).
// Tiles are f16 in 128-byte rows with the 16-byte chunks XOR-swizzled by (row & 7); the
// products run on mma.sync m16n8k16 (f16 in, f32 accumulate).
//
// Tensor addressing: element (b, h, s, d) of q is at q + b*sb + h*sh + s*ld + d, so q / k / v
// can be read straight out of the token-major qkv buffer [B][S][3*dim] and O / dO live in the
// token-major [B][S][dim] layout the out-projection reads.
#include "sa3k_common.cuh"
#include "sa3k_internal.h"
#include "attention.h"

namespace sa3k {
namespace {

constexpr int HD = 64;      // head dim
constexpr int TQ = 64;      // queries per CTA / tile
constexpr int TK = 64;      // keys per tile
constexpr int NT = 128;     // threads per CTA (4 warps x 16 rows)
constexpr float kLog2e = 1.4426950408889634f;

__device__ __forceinline__ uint32_t toff(int r, int c) { return (uint32_t)((r * 8 + (c ^ (r & 7))) * 16); }

__device__ __forceinline__ void cp_async16(uint32_t saddr, const void* g, bool pred) {
  const int sz = pred ? 16 : 0;   // src-size 0 zero-fills the 16 bytes
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(saddr), "l"(g), "r"(sz) : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(addr));
}
__device__ __forceinline__ void mma16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// [64 rows][64 f16] tile from rows row0.. of a strided tensor (rows >= nrows read as zero).
__device__ __forceinline__ void load_tile(uint32_t sbase, const __half* g, long ld, int row0, int nrows,
                                          int tid) {
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int idx = tid + NT * i;
    const int r = idx >> 3, c = idx & 7;
    const bool ok = row0 + r < nrows;
    cp_async16(sbase + toff(r, c), ok ? (const void*)(g + (long)(row0 + r) * ld + c * 8) : (const void*)g, ok);
  }
}

// A fragments (16 rows x 64 cols, row-major in the tile) for 4 k-steps of 16.
__device__ __forceinline__ void load_a_frags(uint32_t (&a)[4][4], uint32_t sbase, int r0, int lane) {
#pragma unroll
  for (int ks = 0; ks < 4; ++ks) ldsm_x4(a[ks], sbase + toff(r0 + (lane & 15), ks * 2 + (lane >> 4)));
}

// acc[16 x 64] += A[16 x 64] * T^T where T is a [64 n][64 k] tile (k contiguous): B = T^T.
__device__ __forceinline__ void mma_abt(float (&acc)[8][4], const uint32_t (&a)[4][4], uint32_t tbase, int lane) {
#pragma unroll
  for (int np = 0; np < 4; ++np) {
#pragma unroll
    for (int ks = 0; ks < 4; ++ks) {
      uint32_t b[4];
      ldsm_x4(b, tbase + toff(16 * np + (lane & 7) + ((lane >> 4) << 3), ks * 2 + ((lane >> 3) & 1)));
      mma16816(acc[2 * np], a[ks], b[0], b[1]);
      mma16816(acc[2 * np + 1], a[ks], b[2], b[3]);
    }
  }
}

// acc[16 x 64] += A[16 x 64 k] * T where T is a [64 k][64 n] tile (n contiguous).
__device__ __forceinline__ void mma_ab(float (&acc)[8][4], const uint32_t (&a)[4][4], uint32_t tbase, int lane) {
#pragma unroll
  for (int np = 0; np < 4; ++np) {
#pragma unroll
    for (int ks = 0; ks < 4; ++ks) {
      uint32_t b[4];
      ldsm_x4_t(b, tbase + toff(16 * ks + (lane & 7) + (((lane >> 3) & 1) << 3), np * 2 + (lane >> 4)));
      mma16816(acc[2 * np], a[ks], b[0], b[1]);
      mma16816(acc[2 * np + 1], a[ks], b[2], b[3]);
    }
  }
}

// f32 accumulator fragments [16 x 64] -> f16 A fragments (the FA2 register reuse).
__device__ __forceinline__ void acc_to_a(uint32_t (&a)[4][4], const float (&c)[8][4]) {
#pragma unroll
  for (int ks = 0; ks < 4; ++ks) {
    a[ks][0] = pack_f16x2(c[2 * ks][0], c[2 * ks][1]);
    a[ks][1] = pack_f16x2(c[2 * ks][2], c[2 * ks][3]);
    a[ks][2] = pack_f16x2(c[2 * ks + 1][0], c[2 * ks + 1][1]);
    a[ks][3] = pack_f16x2(c[2 * ks + 1][2], c[2 * ks + 1][3]);
  }
}

__device__ __forceinline__ void zero(float (&c)[8][4]) {
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) c[i][j] = 0.f;
}

__device__ __forceinline__ bool visible(int qi, int kj, int Sk, int window) {
  return kj < Sk && (window < 0 || abs(qi - kj) <= window);
}

// key-tile range a query tile [q0, q0 + 64) can see
__device__ __forceinline__ void key_range(int q0, int Sk, int window, int& kt0, int& kt1) {
  kt0 = 0;
  kt1 = (Sk + TK - 1) / TK;
  if (window >= 0) {
    const int lo = q0 - window, hi = q0 + TQ - 1 + window;
    kt0 = max(0, lo) / TK;
    kt1 = min(kt1, hi / TK + 1);
  }
}

// ---------------------------------------------------------------------------------- forward
__global__ void __launch_bounds__(NT) attn_fwd_kernel(const AttnArgs p) {
  pdl_prologue();
  extern __shared__ __align__(1024) uint8_t sm[];    // Q, K[2], V[2]
  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
  const int g = lane >> 2, t4 = lane & 3;
  const int bh = blockIdx.y, b = bh / p.H, h = bh % p.H;
  const int q0 = blockIdx.x * TQ;
  const __half* qg = p.q + b * p.q_sb + h * p.q_sh;
  const __half* kg = p.k + b * p.k_sb + h * p.k_sh;
  const __half* vg = p.v + b * p.v_sb + h * p.v_sh;
  const uint32_t sQ = smem_u32(sm), sK = sQ + 8192, sV = sQ + 3 * 8192;
  int kt0, kt1;
  key_range(q0, p.Sk, p.window, kt0, kt1);

  load_tile(sQ, qg, p.q_ld, q0, p.Sq, tid);
  cp_commit();
  if (kt0 < kt1) {
    load_tile(sK, kg, p.k_ld, kt0 * TK, p.Sk, tid);
    load_tile(sV, vg, p.v_ld, kt0 * TK, p.Sk, tid);
  }
  cp_commit();
  cp_wait<1>();
  __syncthreads();
  uint32_t qa[4][4];
  load_a_frags(qa, sQ, 16 * w, lane);

  const float sl2 = p.scale * kLog2e;
  float m[2] = {-INFINITY, -INFINITY}, l[2] = {0.f, 0.f};
  float o[8][4];
  zero(o);
  const int qr[2] = {q0 + 16 * w + g, q0 + 16 * w + g + 8};
  for (int kt = kt0; kt < kt1; ++kt) {
    const int buf = (kt - kt0) & 1;
    if (kt + 1 < kt1) {
      load_tile(sK + (buf ^ 1) * 8192, kg, p.k_ld, (kt + 1) * TK, p.Sk, tid);
      load_tile(sV + (buf ^ 1) * 8192, vg, p.v_ld, (kt + 1) * TK, p.Sk, tid);
    }
    cp_commit();
    cp_wait<1>();
    __syncthreads();
    float s[8][4];
    zero(s);
    mma_abt(s, qa, sK + buf * 8192, lane);
    float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int nt = 0; nt < 8; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int kj = kt * TK + nt * 8 + 2 * t4 + (e & 1);
        const float x = visible(qr[e >> 1], kj, p.Sk, p.window) ? s[nt][e] * sl2 : -INFINITY;
        s[nt][e] = x;
        mx[e >> 1] = fmaxf(mx[e >> 1], x);
      }
    float alpha[2], mu[2];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 1));
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 2));
      const float mn = fmaxf(m[r], mx[r]);
      mu[r] = mn == -INFINITY ? 0.f : mn;
      alpha[r] = exp2f(m[r] - mu[r]);
      m[r] = mn;
      l[r] *= alpha[r];
    }
#pragma unroll
    for (int nt = 0; nt < 8; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float pe = exp2f(s[nt][e] - mu[e >> 1]);
        s[nt][e] = pe;
        l[e >> 1] += pe;
        o[nt][e] *= alpha[e >> 1];
      }
    uint32_t pa[4][4];
    acc_to_a(pa, s);
    mma_ab(o, pa, sV + buf * 8192, lane);
    __syncthreads();
  }
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    l[r] += __shfl_xor_sync(0xffffffffu, l[r], 1);
    l[r] += __shfl_xor_sync(0xffffffffu, l[r], 2);
  }
  __half* og = p.o + b * p.o_sb + h * p.o_sh;
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int qi = qr[r];
    if (qi >= p.Sq) continue;
    const float inv = l[r] > 0.f ? 1.f / l[r] : 0.f;
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      const uint32_t v2 = pack_f16x2(o[nt][2 * r] * inv, o[nt][2 * r + 1] * inv);
      *reinterpret_cast<uint32_t*>(og + (long)qi * p.o_ld + nt * 8 + 2 * t4) = v2;
    }
    if (t4 == 0 && p.lse) p.lse[(long)bh * p.Sq + qi] = (m[r] == -INFINITY ? 0.f : m[r]) + log2f(fmaxf(l[r], 1e-30f));
  }
}

// D[bh][q] = sum_d dO[b,h,q,d] * O[b,h,q,d]  (one warp per (bh, q) row)
__global__ void attn_bwd_pre_kernel(const AttnArgs p) {
  pdl_prologue();
  const long row = (long)blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
  const long nrows = (long)p.B * p.H * p.Sq;
  if (row >= nrows) return;
  const int lane = threadIdx.x & 31;
  const int bh = (int)(row / p.Sq), qi = (int)(row % p.Sq);
  const int b = bh / p.H, h = bh % p.H;
  const __half2 d2 = reinterpret_cast<const __half2*>(p.dO + b * p.dO_sb + h * p.dO_sh + (long)qi * p.dO_ld)[lane];
  const __half2 o2 = reinterpret_cast<const __half2*>(p.o + b * p.o_sb + h * p.o_sh + (long)qi * p.o_ld)[lane];
  float acc = __half2float(d2.x) * __half2float(o2.x) + __half2float(d2.y) * __half2float(o2.y);
  acc = warp_sum(acc);
  if (lane == 0) p.Dsum[row] = acc;
}

// ---------------------------------------------------------------------------------- dq pass
__global__ void __launch_bounds__(NT) attn_bwd_dq_kernel(const AttnArgs p) {
  pdl_prologue();
  extern __shared__ __align__(1024) uint8_t sm[];    // Q, dO, K[2], V[2]
  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
  const int g = lane >> 2, t4 = lane & 3;
  const int bh = blockIdx.y, b = bh / p.H, h = bh % p.H;
  const int q0 = blockIdx.x * TQ;
  const __half* qg = p.q + b * p.q_sb + h * p.q_sh;
  const __half* kg = p.k + b * p.k_sb + h * p.k_sh;
  const __half* vg = p.v + b * p.v_sb + h * p.v_sh;
  const __half* dog = p.dO + b * p.dO_sb + h * p.dO_sh;
  const uint32_t sQ = smem_u32(sm), sD = sQ + 8192, sK = sQ + 2 * 8192, sV = sQ + 4 * 8192;
  int kt0, kt1;
  key_range(q0, p.Sk, p.window, kt0, kt1);
  load_tile(sQ, qg, p.q_ld, q0, p.Sq, tid);
  load_tile(sD, dog, p.dO_ld, q0, p.Sq, tid);
  cp_commit();
  if (kt0 < kt1) {
    load_tile(sK, kg, p.k_ld, kt0 * TK, p.Sk, tid);
    load_tile(sV, vg, p.v_ld, kt0 * TK, p.Sk, tid);
  }
  cp_commit();
  cp_wait<1>();
  __syncthreads();
  uint32_t qa[4][4], da[4][4];
  load_a_frags(qa, sQ, 16 * w, lane);
  load_a_frags(da, sD, 16 * w, lane);
  const int qr[2] = {q0 + 16 * w + g, q0 + 16 * w + g + 8};
  float lse[2], Dr[2];
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const bool ok = qr[r] < p.Sq;
    lse[r] = ok ? p.lse[(long)bh * p.Sq + qr[r]] : 0.f;
    Dr[r] = ok ? p.Dsum[(long)bh * p.Sq + qr[r]] : 0.f;
  }
  const float sl2 = p.scale * kLog2e;
  float dq[8][4];
  zero(dq);
  for (int kt = kt0; kt < kt1; ++kt) {
    const int buf = (kt - kt0) & 1;
    if (kt + 1 < kt1) {
      load_tile(sK + (buf ^ 1) * 8192, kg, p.k_ld, (kt + 1) * TK, p.Sk, tid);
      load_tile(sV + (buf ^ 1) * 8192, vg, p.v_ld, (kt + 1) * TK, p.Sk, tid);
    }
    cp_commit();
    cp_wait<1>();
    __syncthreads();
    float s[8][4], dp[8][4];
    zero(s);
    zero(dp);
    mma_abt(s, qa, sK + buf * 8192, lane);
    mma_abt(dp, da, sV + buf * 8192, lane);
#pragma unroll
    for (int nt = 0; nt < 8; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int r = e >> 1;
        const int kj = kt * TK + nt * 8 + 2 * t4 + (e & 1);
        const float pe = visible(qr[r], kj, p.Sk, p.window) ? exp2f(s[nt][e] * sl2 - lse[r]) : 0.f;
        s[nt][e] = pe * (dp[nt][e] - Dr[r]) * p.scale;   // dS (scaled)
      }
    uint32_t sa[4][4];
    acc_to_a(sa, s);
    mma_ab(dq, sa, sK + buf * 8192, lane);
    __syncthreads();
  }
  float* dqg = p.dq + b * p.dq_sb + h * p.dq_sh;
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    if (qr[r] >= p.Sq) continue;
#pragma unroll
    for (int nt = 0; nt < 8; ++nt)
      *reinterpret_cast<float2*>(dqg + (long)qr[r] * p.dq_ld + nt * 8 + 2 * t4) = make_float2(dq[nt][2 * r], dq[nt][2 * r + 1]);
  }
}

// ---------------------------------------------------------------------------------- dkdv pass
__global__ void __launch_bounds__(NT) attn_bwd_dkdv_kernel(const AttnArgs p) {
  pdl_prologue();
  extern __shared__ __align__(1024) uint8_t sm[];    // K, V, Q[2], dO[2], then lse / D [2][64]
  float (*s_lse)[TQ] = reinterpret_cast<float (*)[TQ]>(sm + 8192 * 6);
  float (*s_D)[TQ] = reinterpret_cast<float (*)[TQ]>(sm + 8192 * 6 + 2 * TQ * 4);
  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
  const int g = lane >> 2, t4 = lane & 3;
  const int bh = blockIdx.y, b = bh / p.H, h = bh % p.H;
  const int k0 = blockIdx.x * TK;
  const __half* qg = p.q + b * p.q_sb + h * p.q_sh;
  const __half* kg = p.k + b * p.k_sb + h * p.k_sh;
  const __half* vg = p.v + b * p.v_sb + h * p.v_sh;
  const __half* dog = p.dO + b * p.dO_sb + h * p.dO_sh;
  const uint32_t sK = smem_u32(sm), sV = sK + 8192, sQ = sK + 2 * 8192, sD = sK + 4 * 8192;
  // query tiles that can see this key tile
  int qt0 = 0, qt1 = (p.Sq + TQ - 1) / TQ;
  if (p.window >= 0) {
    qt0 = max(0, k0 - p.window) / TQ;
    qt1 = min(qt1, (k0 + TK - 1 + p.window) / TQ + 1);
  }
  auto load_q = [&](int qt, int buf) {
    load_tile(sQ + buf * 8192, qg, p.q_ld, qt * TQ, p.Sq, tid);
    load_tile(sD + buf * 8192, dog, p.dO_ld, qt * TQ, p.Sq, tid);
    if (tid < TQ) {
      const int qi = qt * TQ + tid;
      s_lse[buf][tid] = qi < p.Sq ? p.lse[(long)bh * p.Sq + qi] : 0.f;
      s_D[buf][tid] = qi < p.Sq ? p.Dsum[(long)bh * p.Sq + qi] : 0.f;
    }
  };
  load_tile(sK, kg, p.k_ld, k0, p.Sk, tid);
  load_tile(sV, vg, p.v_ld, k0, p.Sk, tid);
  cp_commit();
  if (qt0 < qt1) load_q(qt0, 0);
  cp_commit();
  cp_wait<1>();
  __syncthreads();
  uint32_t ka[4][4], va[4][4];
  load_a_frags(ka, sK, 16 * w, lane);
  load_a_frags(va, sV, 16 * w, lane);
  const int kr[2] = {k0 + 16 * w + g, k0 + 16 * w + g + 8};
  const float sl2 = p.scale * kLog2e;
  float dk[8][4], dv[8][4];
  zero(dk);
  zero(dv);
  for (int qt = qt0; qt < qt1; ++qt) {
    const int buf = (qt - qt0) & 1;
    if (qt + 1 < qt1) load_q(qt + 1, buf ^ 1);
    cp_commit();
    cp_wait<1>();
    __syncthreads();
    float st[8][4], dpt[8][4];
    zero(st);
    zero(dpt);
    mma_abt(st, ka, sQ + buf * 8192, lane);    // S^T = K Q^T   [16 keys x 64 queries]
    mma_abt(dpt, va, sD + buf * 8192, lane);   // dP^T = V dO^T
#pragma unroll
    for (int nt = 0; nt < 8; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int ql = nt * 8 + 2 * t4 + (e & 1);
        const int qi = qt * TQ + ql;
        const bool ok = qi < p.Sq && visible(qi, kr[e >> 1], p.Sk, p.window);
        const float pe = ok ? exp2f(st[nt][e] * sl2 - s_lse[buf][ql]) : 0.f;
        st[nt][e] = pe;                                               // P^T
        dpt[nt][e] = pe * (dpt[nt][e] - s_D[buf][ql]) * p.scale;      // dS^T (scaled)
      }
    uint32_t pa[4][4], sa[4][4];
    acc_to_a(pa, st);
    acc_to_a(sa, dpt);
    mma_ab(dv, pa, sD + buf * 8192, lane);     // dV += P^T dO
    mma_ab(dk, sa, sQ + buf * 8192, lane);     // dK += dS^T Q
    __syncthreads();
  }
  float* dkg = p.dk + b * p.dk_sb + h * p.dk_sh;
  float* dvg = p.dv + b * p.dv_sb + h * p.dv_sh;
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    if (kr[r] >= p.Sk) continue;
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      *reinterpret_cast<float2*>(dkg + (long)kr[r] * p.dk_ld + nt * 8 + 2 * t4) = make_float2(dk[nt][2 * r], dk[nt][2 * r + 1]);
      *reinterpret_cast<float2*>(dvg + (long)kr[r] * p.dv_ld + nt * 8 + 2 * t4) = make_float2(dv[nt][2 * r], dv[nt][2 * r + 1]);
    }
  }
}

}  // namespace

constexpr int kSmemFwd = 8192 * 5, kSmemDq = 8192 * 6, kSmemDkdv = 8192 * 6 + 4 * TQ * 4;

static int set_attrs(int device, std::string& err) {
  const char* what = "attention smem attributes";
  return smem_attr(reinterpret_cast<const void*>(attn_fwd_kernel), kSmemFwd, device, what, err) ||
         smem_attr(reinterpret_cast<const void*>(attn_bwd_dq_kernel), kSmemDq, device, what, err) ||
         smem_attr(reinterpret_cast<const void*>(attn_bwd_dkdv_kernel), kSmemDkdv, device, what, err);
}

int attn_forward(Ctx* c, const AttnArgs& a, std::string& err) {
  if (a.head_dim != HD) { err = "attention: head_dim must be 64"; return 1; }
  if (c->attn_tc && attn_tc_supported(a)) return attn_tc_forward(c, a, err);
  if (set_attrs(c->device, err)) return 1;
  ProfScope prof_(c, "attn.fwd");
  dim3 grid((unsigned)((a.Sq + TQ - 1) / TQ), (unsigned)(a.B * a.H));
  launch_pdl(c, attn_fwd_kernel, grid, NT, kSmemFwd, a);
  return check_launch("attn fwd", err);
}

int attn_backward(Ctx* c, const AttnArgs& a, bool want_dkdv, std::string& err) {
  if (a.head_dim != HD) { err = "attention: head_dim must be 64"; return 1; }
  // the tcgen05 dq pass forms D = rowsum(dO o O) itself
  if (c->attn_tc && attn_tc_supported(a)) return attn_tc_grads(c, a, want_dkdv, err);
  if (set_attrs(c->device, err)) return 1;
  {
    ProfScope prof_(c, "attn.bwd_pre");
    const long rows = (long)a.B * a.H * a.Sq;
    launch_pdl(c, attn_bwd_pre_kernel, (unsigned)((rows + 7) / 8), 256, 0, a);
    if (check_launch("attn bwd pre", err)) return 1;
  }
  {
    ProfScope prof_(c, "attn.bwd_dq");
    dim3 grid((unsigned)((a.Sq + TQ - 1) / TQ), (unsigned)(a.B * a.H));
    launch_pdl(c, attn_bwd_dq_kernel, grid, NT, kSmemDq, a);
    if (check_launch("attn bwd dq", err)) return 1;
  }
  if (want_dkdv) {
    ProfScope prof_(c, "attn.bwd_dkdv");
    dim3 grid((unsigned)((a.Sk + TK - 1) / TK), (unsigned)(a.B * a.H));
    launch_pdl(c, attn_bwd_dkdv_kernel, grid, NT, kSmemDkdv, a);
    if (check_launch("attn bwd dkdv", err)) return 1;
  }
  return 0;
}

}  // namespace sa3k
