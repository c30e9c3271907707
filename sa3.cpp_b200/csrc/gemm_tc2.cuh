// gemm_tc2.cuh -- the CTA-pair (tcgen05 cta_group::2) form of the GEMM engine, for f16 operands.
//
// A cluster of two CTAs on two SMs computes one 256 x BN output tile with M = 256 UMMAs:
//   CTA r (r = %cluster_ctarank) loads rows [128 r, 128 r + 128) of the A tile and columns
//   [r BN/2, (r+1) BN/2) of the B tile into its own shared memory (plain TMA loads: each CTA
//   fetches only its own half, nothing is multicast), and holds rows 128 r .. of the f32
//   accumulator in its own TMEM.  The even CTA's MMA warp (one elected lane) issues every
//   tcgen05.mma.cta_group::2, which reads both CTAs' operand halves.
// Each SM therefore streams 128 x 64 of A and BN/2 x 64 of B per k-block instead of 128 x 64 and
// BN x 64: the shared-memory traffic per tensor-core cycle falls by a quarter at BN = 256, which
// is what lets the tensor pipe run close to its peak.
//
// Barriers (per CTA, same offsets in both):
//   full[s]    even CTA only: armed with the bytes of both halves; both CTAs' TMA loads complete
//              on it (cta_group::2 loads may signal the peer's barrier)
//   empty[s]   both CTAs: the MMA commit arrives on both (tcgen05.commit ... multicast::cluster)
//   tfull[a]   both CTAs: accumulator a complete (multicast commit)
//   tempty[a]  even CTA only: one arrival per epilogue warp of both CTAs (remote arrives)
// Every wait is bounded like the one-CTA kernel's; both CTAs always reach the final cluster
// barrier, so neither leaves while the peer may still read its shared memory.
#pragma once

#include "gemm_tc.cuh"

namespace sa3k {

__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// Address of the same shared-memory location in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t addr, uint32_t rank) {
  uint32_t d;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(d) : "r"(addr), "r"(rank));
  return d;
}

__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_remote(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}

// TMA tile load into this CTA's shared memory whose completion is signalled on an mbarrier that
// may live in the peer CTA of the pair (cluster address).  Not a multicast load.
__device__ __forceinline__ void tma_load_2d_pair(void* smem_dst, const CUtensorMap* m, uint32_t bar_cluster,
                                                 int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(bar_cluster), "r"(x), "r"(y)
      : "memory");
}

__device__ __forceinline__ void tmem_alloc_pair(uint32_t* slot, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot)),
               "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// tcgen05.mma.cta_group::2, issued warp-wide: warp-uniform operands, one elected lane issues.
__device__ __forceinline__ void umma_f16_pair_w(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                                 uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p, e;\n\t"
      "elect.sync _|e, 0xffffffff;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "@e tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive once on the mbarrier at this offset in both CTAs of the pair when every MMA issued so
// far has completed (warp-wide, one elected lane).
__device__ __forceinline__ void umma_commit_pair_w(uint64_t* bar) {
  asm volatile(
      "{\n\t.reg .pred e;\n\t"
      "elect.sync _|e, 0xffffffff;\n\t"
      "@e tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;\n\t}" ::"r"(
          smem_u32(bar)),
      "h"((uint16_t)0x3)
      : "memory");
}

// NeoX rotation of the first 2 HALF dims of a head: dims i and i + HALF rotate together by the
// (cos, sin) pair cs[i * tps] of the row's position (frequency-major table, so the lanes of a warp,
// on consecutive rows, read consecutive pairs)
template <int HALF>
__device__ __forceinline__ void head_rope(float (&v)[64], const float2* cs, int tps) {
#pragma unroll
  for (int i = 0; i < HALF; ++i) {
    const float2 t = __ldg(cs + (long)i * tps);
    const float a = v[i], b = v[i + HALF];
    v[i] = a * t.x - b * t.y;
    v[i + HALF] = b * t.x + a * t.y;
  }
}

// The fused head preparation of one 64-column head of `row` (HeadPrepEpi): f holds the GEMM's
// f32 values of columns nb .. nb + 63.  q and k heads only: v is read from the GEMM's own output.
__device__ __forceinline__ void head_prep_epi(const HeadPrepEpi& p, const float* f, int nb, int row) {
  const int slice = nb / p.D, h = (nb - slice * p.D) >> 6;
  if (slice >= 2) return;
  float v[64];
#pragma unroll
  for (int k = 0; k < 64; ++k) v[k] = f[k];
  {
    const float* gm = slice == 0 ? p.gq : p.gk;
    float ss = 0.f;
#pragma unroll
    for (int k = 0; k < 64; ++k) ss = fmaf(v[k], v[k], ss);
    const float r = rsqrtf(ss / 64.f + p.eps);
    (slice == 0 ? p.rq : p.rk)[(long)row * p.H + h] = r;
#pragma unroll
    for (int k = 0; k < 64; k += 4) {
      const float4 g4 = __ldg(reinterpret_cast<const float4*>(gm + k));
      v[k] *= r * g4.x; v[k + 1] *= r * g4.y; v[k + 2] *= r * g4.z; v[k + 3] *= r * g4.w;
    }
    if (p.tab && p.rot == 32) head_rope<16>(v, p.tab + row % p.tps, p.tps);
    else if (p.tab && p.rot == 64) head_rope<32>(v, p.tab + row % p.tps, p.tps);
  }
  uint4* dst = reinterpret_cast<uint4*>(p.out + (long)row * p.ld + nb);
#pragma unroll
  for (int c = 0; c < 8; ++c)
    dst[c] = make_uint4(pack_f16x2(v[8 * c], v[8 * c + 1]), pack_f16x2(v[8 * c + 2], v[8 * c + 3]),
                        pack_f16x2(v[8 * c + 4], v[8 * c + 5]), pack_f16x2(v[8 * c + 6], v[8 * c + 7]));
}

constexpr int kPairEpiWarps = 8;        // two per TMEM lane quarter, alternate column chunks
constexpr int kPairThreads = 32 * (2 + kPairEpiWarps);

template <int BN, int STAGES>
struct Gemm2Smem {
  static constexpr int BH = BN / 2;                  // B rows (N) held by each CTA
  static constexpr int A_BYTES = kBM * kBK * 2;      // 16 KB
  static constexpr int B_BYTES = BH * kBK * 2;
  static constexpr int OFF_A = 0;
  static constexpr int OFF_B = OFF_A + STAGES * A_BYTES;
  static constexpr int OFF_STAGE = align_up(OFF_B + STAGES * B_BYTES, 1024);
  static constexpr int STAGE_BYTES = 4096;
  static constexpr int STAGE_BUFS =
      (OFF_STAGE + kPairEpiWarps * 2 * STAGE_BYTES + (2 * STAGES + 4) * 8 + 16 + 1024 <= 232448) ? 2 : 1;
  static constexpr int OFF_BAR = OFF_STAGE + kPairEpiWarps * STAGE_BUFS * STAGE_BYTES;
  static constexpr int BAR_BYTES = (2 * STAGES + 4) * 8 + 16;
  static constexpr int TOTAL = OFF_BAR + BAR_BYTES;
  static constexpr int DYN = TOTAL + 1024;
  static constexpr int ACC_COLS = BN;
  static constexpr int TMEM_COLS = 2 * BN <= 256 ? 256 : 512;   // a power of two
  static_assert(BN == 128 || BN == 192 || BN == 256, "pair tiles are 256 x 128, 192 or 256");
  static_assert(DYN <= 232448, "shared memory budget (227 KB)");
};

// BMODE 0: B is [N][K] row-major (K-major); 1: B is [K][N] row-major (MN-major).  A is [M][K].
template <int BN, int STAGES, int BMODE>
__global__ void __launch_bounds__(kPairThreads, 1)
    gemm_tc2_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b,
                    const __grid_constant__ CUtensorMap tm_ea, const __grid_constant__ CUtensorMap tm_eb,
                    const __grid_constant__ CUtensorMap tm_out, const __grid_constant__ GemmArgs args) {
  using L = Gemm2Smem<BN, STAGES>;
  constexpr bool BMN = BMODE == 1;
  constexpr int EPI_WARPS = kPairEpiWarps;
  constexpr int PM = 2 * kBM;                        // rows of a pair tile
  static_assert(!BMN || L::BH % 64 == 0, "MN-major B halves are built from 64-wide atoms");

  extern __shared__ uint8_t smem_raw[];
  pdl_trigger();   // the next kernel may be scheduled once every CTA of this grid runs
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::OFF_BAR);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;      // [2]
  uint64_t* tempty = tfull + 2;          // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int cluster = blockIdx.x >> 1, nclusters = gridDim.x >> 1;
  const int tiles_m = (args.M + PM - 1) / PM;
  const int tiles_n = (args.N + BN - 1) / BN;
  const int ntiles = tiles_m * tiles_n;
  const int nkb_all = (args.K + kBK - 1) / kBK;
  const int nitems = num_items(args, ntiles);   // work items over pair tiles (gemm_tc.cuh)

  if (warp == 0 && lane == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 2 * EPI_WARPS);
    }
    *abort_flag = 0;
    fence_barrier_init();
    fence_proxy_async_smem();
    tma_prefetch_desc(&tm_a);
    tma_prefetch_desc(&tm_b);
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, L::TMEM_COLS);
    tmem_relinquish_pair();
    tc_fence_before();
  }
  cluster_sync_all();      // barriers of both CTAs initialised, TMEM allocated in both
  tc_fence_after();
  const uint32_t tbase = *tmem_slot;
  pdl_wait();      // outputs of earlier kernels are read only from here on

  auto wait = [&](uint64_t* bar, uint32_t parity, int code, bool cluster_scope) -> bool {
    if (*abort_flag) return false;
    const uint32_t a = smem_u32(bar);
    auto probe = [&]() { return cluster_scope ? mbar_try_wait_cluster(a, parity) : mbar_try_wait(a, parity); };
    if (probe()) return true;
    const unsigned long long t0 = globaltimer();
    for (uint32_t i = 1;; ++i) {
      if (probe()) return true;
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
    // ------------------------------------------------------------ TMA producer (both CTAs)
    if (lane == 0) {
      const uint32_t full0 = mapa_shared(smem_u32(full), 0);   // the even CTA's full[0]
      int it = 0;
      bool ok = true;
      for (int item = cluster; item < nitems && ok; item += nclusters) {
        const WorkItem w = decode_item(args, item, ntiles, nkb_all);
        const int m0 = (w.t % tiles_m) * PM + (int)rank * kBM;
        const int n0 = (w.t / tiles_m) * BN + (int)rank * L::BH;
        const int nkb = w.nkb, total = w.total;
        for (int kb = 0; kb < total; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t use = (uint32_t)(it / STAGES);
          if (it >= STAGES && !wait(&empty[s], (use & 1u) ^ 1u, kErrTimeoutEmpty, true)) { ok = false; break; }
          uint8_t* a_st = smem + L::OFF_A + s * L::A_BYTES;
          uint8_t* b_st = smem + L::OFF_B + s * L::B_BYTES;
          const uint32_t fb = full0 + (uint32_t)(s * 8);
          if (leader)
            mbar_arrive_expect_tx(&full[s], 2u * (uint32_t)((kb < nkb ? L::A_BYTES : kExtABytes) + L::B_BYTES));
          if (kb < nkb) {
            const int k0 = (w.kb0 + kb) * kBK;
            tma_load_2d_pair(a_st, &tm_a, fb, k0, m0);
            if (!BMN) {
              tma_load_2d_pair(b_st, &tm_b, fb, k0, n0);
            } else {
#pragma unroll
              for (int j = 0; j < L::BH / 64; ++j) tma_load_2d_pair(b_st + j * 8192, &tm_b, fb, n0 + 64 * j, k0);
            }
          } else {
            tma_load_2d_pair(a_st, &tm_ea, fb, m0, 0);               // u^T, MN-major
            tma_load_2d_pair(a_st + kExtABytes / 2, &tm_ea, fb, m0 + 64, 0);
            tma_load_2d_pair(b_st, &tm_eb, fb, 0, n0);
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (even CTA)
    // Warp-wide with one elected issuing lane and descriptors built once (see gemm_tc.cuh).
    if (leader) {
      const WaiterW<true> wt{abort_flag, args.err};
      const uint32_t idesc = make_idesc_f16(PM, BN, 0, BMN ? 1 : 0);
      const uint32_t idesc_ext = make_idesc_f16(PM, BN, 1, 0);   // A = u^T read MN-major
      const uint64_t adesc0 = make_sdesc(smem_u32(smem + L::OFF_A), 16, 1024);
      const uint64_t bdesc0 = BMN ? make_sdesc(smem_u32(smem + L::OFF_B), 8192, 1024)
                                  : make_sdesc(smem_u32(smem + L::OFF_B), 16, 1024);
      const uint64_t bdesc0_k = make_sdesc(smem_u32(smem + L::OFF_B), 16, 1024);
      const uint64_t adesc0_ext = make_sdesc(smem_u32(smem + L::OFF_A), kExtABytes / 2, 1024);
      constexpr uint32_t B_KSTEP = BMN ? 2048 >> 4 : 32 >> 4;
      int it = 0, ti = 0;
      bool ok = true;
      for (int item = cluster; item < nitems && ok; item += nclusters, ++ti) {
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
          tc_fence_after();
          const uint32_t aoff = (uint32_t)(s * L::A_BYTES) >> 4, boff = (uint32_t)(s * L::B_BYTES) >> 4;
          if (kb < nkb) {
#pragma unroll
            for (int kk = 0; kk < kBK / 16; ++kk)
              umma_f16_pair_w(d_tmem, adesc0 + aoff + kk * 2u, bdesc0 + boff + kk * B_KSTEP, idesc,
                               (kb > 0 || kk > 0) ? 1u : 0u);
          } else {
            umma_f16_pair_w(d_tmem, adesc0_ext + aoff, bdesc0_k + boff, idesc_ext, total > 1 ? 1u : 0u);
          }
          umma_commit_pair_w(&empty[s]);
        }
        if (ok) umma_commit_pair_w(&tfull[a]);
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue (both CTAs)
    const int q = warp & 3;
    constexpr int NH = EPI_WARPS / 4;      // warps per TMEM lane quarter
    const int half = (warp - 2) / 4;       // this warp's chunks: chunk % NH == half
    uint8_t* stg = smem + L::OFF_STAGE + (warp - 2) * L::STAGE_BUFS * L::STAGE_BYTES;
    const int cstep = args.tma_out == 2 ? 64 : 32;
    const uint32_t tempty0 = mapa_shared(smem_u32(tempty), 0);
    int nstore = 0, ti = 0;
    for (int item = cluster; item < nitems; item += nclusters, ++ti) {
      const WorkItem w = decode_item(args, item, ntiles, nkb_all);
      const int t = w.t;
      const float* bias = w.first ? args.col_bias : nullptr;   // tail parts: the first adds the bias
      const int a = ti & 1;
      const uint32_t ause = (uint32_t)(ti >> 1);
      const int m0 = (t % tiles_m) * PM + (int)rank * kBM, n0 = (t / tiles_m) * BN;
      const bool have = wait(&tfull[a], ause & 1u, kErrTimeoutAccum, true);
      tc_fence_after();
      const int rbase = m0 + 32 * q;
      const uint32_t tacc = tbase + (uint32_t)(a * L::ACC_COLS) + ((uint32_t)(32 * q) << 16);
#pragma unroll 1
      for (int c0 = half * cstep; c0 < BN; c0 += NH * cstep) {
        float f[64];
        const int nb = n0 + c0;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          if (h == 1 && cstep == 32) break;
          uint32_t v[32];
          tmem_ld32(tacc + (uint32_t)(c0 + 32 * h), v);
          tmem_ld_wait();
          epi_columns(v, f + 32 * h, nb + 32 * h, args, false, bias);
        }
        if (!have || nb >= args.N) continue;
        if (args.has_hp && rbase + lane < args.M) head_prep_epi(args.hp, f, nb, rbase + lane);   // (cstep is 64)
        if (args.tma_out) {
          uint8_t* buf = stg + (L::STAGE_BUFS == 2 ? (nstore & 1) : 0) * L::STAGE_BYTES;
          if (nstore >= L::STAGE_BUFS) {
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
        // direct path (row-major f32 and / or f16, or transposed outputs)
        const int ncols = min(32, args.N - nb);
        const int myrow = rbase + lane;
        if (args.out && args.out_trans) {
          if (myrow < args.M) {
#pragma unroll
            for (int j = 0; j < 32; ++j) {   // static indices keep f[] in registers
              if (j >= ncols) break;
              float* dst = args.out + (long)(nb + j) * args.ldo + myrow;
              if (w.add) atomicAdd(dst, f[j]);
              else *dst = args.accumulate ? *dst + f[j] : f[j];
            }
          }
        }
        if (args.out_h && args.out_h_trans) {
          if (myrow < args.M) {
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              if (j >= ncols) break;
              args.out_h[(long)(nb + j) * args.ldo_h + myrow] = __float2half_rn(f[j]);
            }
          }
        }
        if ((args.out && !args.out_trans) || (args.out_h && !args.out_h_trans)) {
          float* st32 = reinterpret_cast<float*>(stg);
#pragma unroll
          for (int j = 0; j < 32; ++j) st32[lane * 32 + (j ^ lane)] = f[j];
          __syncwarp();
          for (int r = 0; r < 32; ++r) {
            const int row = rbase + r;
            if (row >= args.M || lane >= ncols) continue;
            const float x = st32[r * 32 + (lane ^ r)];
            if (args.out && !args.out_trans) {
              float* dst = args.out + (long)row * args.ldo + nb + lane;
              if (w.add) atomicAdd(dst, x);
              else *dst = args.accumulate ? *dst + x : x;
            }
            if (args.out_h && !args.out_h_trans) args.out_h[(long)row * args.ldo_h + nb + lane] = __float2half_rn(x);
          }
          __syncwarp();
        }
      }
      // this warp's TMEM reads of accumulator a are complete: tell the MMA thread (even CTA)
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_remote(tempty0 + (uint32_t)(a * 8));
    }
    if (lane == 0) bulk_wait_all();
    __syncwarp();
  }
  tc_fence_before();
  cluster_sync_all();      // no CTA leaves while its peer may still use its shared memory
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tbase, L::TMEM_COLS);
  }
}

}  // namespace sa3k
