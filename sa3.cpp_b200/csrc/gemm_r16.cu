// gemm_r16.cu -- grouped rank-16 GEMMs on the tcgen05 tensor cores: many independent problems
//
//   out (+)= alpha * Aop[M x K] * Bop[K x N],  N <= 16,  one launch for the whole group
//
// The adapter gradients of the backward pass (dB = s dz^T u, dA = du^T x, the DoRA term
// dA += (dt2 B)^T W, src/train_lora.h's functional LoRA / DoRA backward as derived by
// ggml_build_backward_expand, src/train_ckpt.h:400) and the DoRA P = W A^T of the forward are all
// such "skinny" contractions over a long K: they only stream their A operand (an activation,
// an output gradient or the f16 base copy) once.  Run one at a time they are latency-bound
// launches of a few dozen CTAs; grouped, every SM streams A tiles at HBM speed.
//
// Work items are (problem, 128-row M tile, K range); persistent CTAs walk the global item list.
// Each CTA: warp 0 TMA producer (A tile 128 x 64 f16, K-major or MN-major, and the 16 x 64 B
// tile), warp 1 TMEM owner + MMA issue (tcgen05.mma kind::f16, M = 128, N = 16, one elected
// lane), warps 2-5 epilogue (tcgen05.ld of the 128 x 16 f32 accumulator, alpha, f32 atomic add
// or plain store).  The accumulator is double-buffered in TMEM (2 x 16 columns).
// Problem descriptors (with their TMA tensor maps) live in device memory; the per-problem item
// offsets are staged in shared memory for the item -> problem search.
#include "gemm_r16.h"
#include "sa3k_common.cuh"

#include <algorithm>
#include <cstring>

namespace sa3k {

struct alignas(128) R16Problem {
  CUtensorMap ta;          // A: K-major dims {K, M} box {64, 128}; MN-major dims {M, K} box {64, 64}
  CUtensorMap tb;          // B: K-major [N][ldb] dims {K, 16} box {64, 16}
  int M, N, K, a_mn;
  int tiles_m, kbps, nkb, item0;
  int out_trans, atomic;
  long ldo;
  float alpha;
  float* out;
};

namespace {

constexpr int kStages = 11;
constexpr int kA = 128 * 64 * 2;     // A stage bytes
constexpr int kB = 16 * 64 * 2;      // B stage bytes
constexpr int kMaxProblems = 1024;
constexpr int kOffA = 0;
constexpr int kOffB = kOffA + kStages * kA;
constexpr int kOffItem0 = kOffB + kStages * kB;
constexpr int kOffBar = kOffItem0 + kMaxProblems * 4;
constexpr int kBarBytes = (2 * kStages + 4) * 8 + 16;
constexpr int kDyn = kOffBar + kBarBytes + 1024;
static_assert(kDyn <= 232448, "shared memory budget");
constexpr int kThreads = 192;

__device__ __forceinline__ int find_problem(const int* item0, int nprob, int item) {
  int lo = 0, hi = nprob - 1;
  while (lo < hi) {            // last p with item0[p] <= item
    const int mid = (lo + hi + 1) >> 1;
    if (item0[mid] <= item) lo = mid;
    else hi = mid - 1;
  }
  return lo;
}

struct ItemPos {
  int p, m0, kb0, nkb;
};

__device__ __forceinline__ ItemPos locate(const R16Problem* probs, const int* item0, int nprob, int item) {
  ItemPos r;
  r.p = find_problem(item0, nprob, item);
  const R16Problem& P = probs[r.p];
  const int local = item - item0[r.p];
  const int tm = P.tiles_m;
  r.m0 = (local % tm) * 128;
  r.kb0 = (local / tm) * P.kbps;
  r.nkb = min(P.nkb - r.kb0, P.kbps);
  return r;
}

__global__ void __launch_bounds__(kThreads, 1)
    r16_group_kernel(const R16Problem* __restrict__ probs, int nprob, int nitems, int* err) {
  extern __shared__ uint8_t smem_raw[];
  pdl_trigger();   // the next kernel may be scheduled once every CTA of this grid runs
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  int* item0 = reinterpret_cast<int*>(smem + kOffItem0);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kOffBar);
  uint64_t* empty = full + kStages;
  uint64_t* tfull = empty + kStages;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  for (int p = threadIdx.x; p < nprob; p += blockDim.x) item0[p] = probs[p].item0;
  if (warp == 0 && lane == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 128);
    }
    *abort_flag = 0;
    fence_barrier_init();
    fence_proxy_async_smem();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 32);
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
          record_error(err, code);
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
        const ItemPos ip = locate(probs, item0, nprob, item);
        const R16Problem* P = probs + ip.p;
        const int a_mn = P->a_mn;
        for (int kb = 0; kb < ip.nkb; ++kb, ++it) {
          const int s = it % kStages;
          const uint32_t use = (uint32_t)(it / kStages);
          if (it >= kStages && !wait(&empty[s], (use & 1u) ^ 1u, kErrTimeoutEmpty)) { ok = false; break; }
          uint8_t* a_st = smem + kOffA + s * kA;
          uint8_t* b_st = smem + kOffB + s * kB;
          const int k0 = (ip.kb0 + kb) * 64;
          mbar_arrive_expect_tx(&full[s], (uint32_t)(kA + kB));
          if (a_mn) {
            tma_load_2d(a_st, &P->ta, &full[s], ip.m0, k0);
            tma_load_2d(a_st + 8192, &P->ta, &full[s], ip.m0 + 64, k0);
          } else {
            tma_load_2d(a_st, &P->ta, &full[s], k0, ip.m0);
          }
          tma_load_2d(b_st, &P->tb, &full[s], k0, 0);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issue (warp-wide)
    const WaiterW<> wt{abort_flag, err};
    const uint32_t aoff0 = smem_u32(smem + kOffA), boff0 = smem_u32(smem + kOffB);
    const uint64_t bdesc0 = make_sdesc(boff0, 16, 1024);
    const uint64_t adesc_k = make_sdesc(aoff0, 16, 1024), adesc_mn = make_sdesc(aoff0, 8192, 1024);
    const uint32_t idesc_k = make_idesc_f16(128, 16, 0, 0), idesc_mn = make_idesc_f16(128, 16, 1, 0);
    int it = 0, ti = 0;
    bool ok = true;
    for (int item = blockIdx.x; item < nitems && ok; item += gridDim.x, ++ti) {
      const ItemPos ip = locate(probs, item0, nprob, item);
      const int a_mn = probs[ip.p].a_mn;
      const uint64_t adesc0 = a_mn ? adesc_mn : adesc_k;
      const uint32_t idesc = a_mn ? idesc_mn : idesc_k;
      const uint32_t akstep = a_mn ? (2048u >> 4) : (32u >> 4);
      const int a = ti & 1;
      const uint32_t ause = (uint32_t)(ti >> 1);
      if (ti >= 2 && !wt(&tempty[a], (ause & 1u) ^ 1u, kErrTimeoutOther)) { ok = false; break; }
      tc_fence_after();
      const uint32_t d_tmem = tbase + (uint32_t)(a * 16);
      for (int kb = 0; kb < ip.nkb; ++kb, ++it) {
        const int s = it % kStages;
        const uint32_t use = (uint32_t)(it / kStages);
        if (!wt(&full[s], use & 1u, kErrTimeoutFull)) { ok = false; break; }
        tc_fence_after();
        const uint32_t aoff = (uint32_t)(s * kA) >> 4, boff = (uint32_t)(s * kB) >> 4;
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          umma_f16_w(d_tmem, adesc0 + aoff + kk * akstep, bdesc0 + boff + kk * 2u, idesc,
                      (kb > 0 || kk > 0) ? 1u : 0u);
        umma_commit_w(&empty[s]);
      }
      if (ok) umma_commit_w(&tfull[a]);
    }
  } else {
    // ------------------------------------------------------------ epilogue (warps 2-5)
    const int q = warp & 3;
    int ti = 0;
    for (int item = blockIdx.x; item < nitems; item += gridDim.x, ++ti) {
      const ItemPos ip = locate(probs, item0, nprob, item);
      const R16Problem* P = probs + ip.p;
      const int a = ti & 1;
      const uint32_t ause = (uint32_t)(ti >> 1);
      const bool have = wait(&tfull[a], ause & 1u, kErrTimeoutAccum);
      tc_fence_after();
      uint32_t v[16];
      tmem_ld16(tbase + (uint32_t)(a * 16) + ((uint32_t)(32 * q) << 16), v);
      tmem_ld_wait();
      const int row = ip.m0 + 32 * q + lane;
      if (have && ip.nkb > 0 && row < P->M) {
        const float alpha = P->alpha;
        float* out = P->out;
        const long ldo = P->ldo;
        const int n = P->N, tr = P->out_trans, at = P->atomic;
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          if (j >= n) break;
          const float x = __uint_as_float(v[j]) * alpha;
          float* dst = tr ? out + (long)j * ldo + row : out + (long)row * ldo + j;
          if (at) atomicAdd(dst, x);
          else *dst = x;
        }
      }
      tc_fence_before();
      mbar_arrive(&tempty[a]);
    }
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tbase, 32);
  }
}

}  // namespace

static int map2d(CUtensorMap* m, const void* base, uint64_t inner, uint64_t outer, uint64_t row_bytes,
                 uint32_t box_inner, uint32_t box_outer, const char* what, std::string& err) {
  PFN_encodeTiled enc = encode_tiled_fn(err);
  if (!enc) return 1;
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0 || (row_bytes & 15) != 0) {
    err = std::string(what) + ": TMA needs 16-byte aligned base and row pitch";
    return 1;
  }
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  if (enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS) {
    err = std::string(what) + ": cuTensorMapEncodeTiled failed";
    return 1;
  }
  return 0;
}

int r16_group_build(Ctx* c, const std::vector<R16Job>& jobs, int kb_target, R16Group& g, std::string& err) {
  r16_group_free(g);
  if (jobs.empty()) return 0;
  if ((int)jobs.size() > kMaxProblems) {
    err = "r16 group: too many problems";
    return 1;
  }
  std::vector<R16Problem> probs(jobs.size());
  long items = 0;
  for (size_t i = 0; i < jobs.size(); ++i) {
    const R16Job& j = jobs[i];
    R16Problem& P = probs[i];
    std::memset(&P, 0, sizeof P);
    if (j.M <= 0 || j.K <= 0 || j.N <= 0 || j.N > 16 || !j.a || !j.b || !j.out) {
      err = "r16 group: bad problem";
      return 1;
    }
    if (j.a_mn) {
      if (map2d(&P.ta, j.a, (uint64_t)j.M, (uint64_t)j.K, (uint64_t)j.lda * 2, 64, 64, "r16 A (MN-major)", err)) return 1;
    } else {
      if (map2d(&P.ta, j.a, (uint64_t)j.K, (uint64_t)j.M, (uint64_t)j.lda * 2, 64, 128, "r16 A", err)) return 1;
    }
    if (map2d(&P.tb, j.b, (uint64_t)j.K, 16, (uint64_t)j.ldb * 2, 64, 16, "r16 B", err)) return 1;
    P.M = j.M; P.N = j.N; P.K = j.K; P.a_mn = j.a_mn;
    P.tiles_m = (j.M + 127) / 128;
    P.nkb = (j.K + 63) / 64;
    int splits = j.atomic ? (P.nkb + kb_target - 1) / kb_target : 1;
    if (splits < 1) splits = 1;
    P.kbps = (P.nkb + splits - 1) / splits;
    splits = (P.nkb + P.kbps - 1) / P.kbps;
    P.item0 = (int)items;
    items += (long)P.tiles_m * splits;
    P.out_trans = j.out_trans; P.atomic = j.atomic; P.ldo = j.ldo; P.alpha = j.alpha; P.out = j.out;
  }
  if (items > (1L << 30)) {
    err = "r16 group: too many work items";
    return 1;
  }
  if (cudaMalloc(&g.table, sizeof(R16Problem) * probs.size()) != cudaSuccess) {
    cudaGetLastError();
    err = "r16 group: out of device memory";
    g.table = nullptr;
    return 1;
  }
  if (cudaMemcpy(g.table, probs.data(), sizeof(R16Problem) * probs.size(), cudaMemcpyHostToDevice) != cudaSuccess) {
    err = "r16 group: table upload failed";
    r16_group_free(g);
    return 1;
  }
  g.nprob = (int)probs.size();
  g.nitems = (int)items;
  return 0;
}

void r16_group_free(R16Group& g) {
  if (g.table) cudaFree(g.table);
  g.table = nullptr;
  g.nprob = g.nitems = 0;
}

int r16_group_run(Ctx* c, const R16Group& g, const char* name, std::string& err) {
  if (!g.table || g.nitems == 0) return 0;
  if (smem_attr(reinterpret_cast<const void*>(r16_group_kernel), kDyn, c->device, "r16 smem attribute", err)) return 1;
  const int grid = std::min<long>(g.nitems, (long)c->sm_count);
  ProfScope prof_(c, name);
  launch_pdl(c, r16_group_kernel, grid, kThreads, kDyn, static_cast<const R16Problem*>(g.table), g.nprob, g.nitems,
                                                        c->d_err);
  return check_launch("r16_group", err);
}

}  // namespace sa3k
