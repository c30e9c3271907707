// gemm_tc.cu -- host side of the tcgen05 GEMM engine: tensor maps, tile choice, launch.
#include "gemm_tc.cuh"
#include "gemm_tc2.cuh"
#include "gemm_wq.cuh"
#include "sa3k_internal.h"

#include <algorithm>
#include <atomic>
#include <cstdio>
#include <mutex>
#include <set>

namespace sa3k {

PFN_encodeTiled encode_tiled_fn(std::string& err) {
  static PFN_encodeTiled fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_encodeTiled>(p);
  });
  if (!fn) err = "cuTensorMapEncodeTiled is unavailable (no CUDA driver)";
  return fn;
}

int smem_attr(const void* kern, int bytes, int device, const char* what, std::string& err) {
  static std::mutex mu;
  static std::set<std::pair<const void*, int>> done;
  std::lock_guard<std::mutex> lock(mu);
  if (done.count({kern, device})) return 0;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) != cudaSuccess)
    return check_launch(what, err);
  done.insert({kern, device});
  return 0;
}

// 2-D tensor map over a row-major [outer][inner] array with `row_bytes` between rows.
static int make_map(CUtensorMap* m, CUtensorMapDataType dt, const void* base, uint64_t inner,
                    uint64_t outer, uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer,
                    CUtensorMapSwizzle sw, const char* what, std::string& err) {
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
  const CUresult r = enc(m, dt, 2, const_cast<void*>(base), dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    char buf[256];
    snprintf(buf, sizeof buf, "%s: cuTensorMapEncodeTiled failed (%d) dims=%llu x %llu box=%u x %u",
             what, (int)r, (unsigned long long)inner, (unsigned long long)outer, box_inner, box_outer);
    err = buf;
    return 1;
  }
  return 0;
}

// Per-tile split counters of the split-K GEMMs (split-K runs only with at most sm_count / 2
// output tiles).  Zeroed once when allocated; the kernel resets each counter it completes.
static int* split_counters(Ctx* c, std::string& err) {
  constexpr size_t kCounters = 1024;
  const bool fresh = (int)c->scratch.size() <= kSlotSplitCnt || !c->scratch[(size_t)kSlotSplitCnt].ptr;
  int* p = static_cast<int*>(scratch_get(c, kSlotSplitCnt, kCounters * sizeof(int), err));
  if (!p) return nullptr;
  if (fresh && cudaMemsetAsync(p, 0, kCounters * sizeof(int), c->stream) != cudaSuccess) {
    check_launch("split counters", err);
    return nullptr;
  }
  if ((size_t)c->sm_count / 2 > kCounters) {
    err = "gemm: too many SMs for the split-K counters";
    return nullptr;
  }
  return p;
}

// Tail split: when the tiles leave a last, partial round on `slots` CTAs (or CTA pairs), split
// each of those tiles' K range into parts spread over every slot; the parts add into the output,
// which is zeroed first over the column band of the tail tiles unless the GEMM accumulates.
// f32 output only (f16 partial sums cannot be added), no split-K.
static int plan_tail(Ctx* c, const GemmDesc& d, GemmArgs& a, long tiles, long slots, int tiles_m, int bn,
                     std::string& err) {
  const int nkb = (d.K + kBK - 1) / kBK;
  a.tail_t0 = (int)tiles;
  a.tail_parts = 1;
  a.tail_kbps = nkb;
  if (a.splits != 1 || !d.out || d.out_h || d.out_h_t || tiles <= slots) return 0;
  const long rem = tiles % slots;
  if (rem == 0) return 0;
  int parts = (int)(slots / rem);
  if (parts > nkb / 4) parts = nkb / 4;           // keep >= 4 k-blocks per part
  if (parts < 2) return 0;
  const int kbps = (nkb + parts - 1) / parts;
  parts = (nkb + kbps - 1) / kbps;
  if (parts < 2) return 0;
  a.tail_t0 = (int)(tiles - rem);
  a.tail_parts = parts;
  a.tail_kbps = kbps;
  if (!d.accumulate) {
    const long col0 = (long)(a.tail_t0 / tiles_m) * bn;
    const cudaError_t e =
        d.out_trans ? cudaMemset2DAsync(d.out + col0 * d.ldo, (size_t)d.ldo * 4, 0, (size_t)d.M * 4, (size_t)(d.N - col0),
                                        c->stream)
                    : cudaMemset2DAsync(d.out + col0, (size_t)d.ldo * 4, 0, (size_t)(d.N - col0) * 4, (size_t)d.M,
                                        c->stream);
    if (e != cudaSuccess) return check_launch("gemm tail memset", err);
  }
  return 0;
}

template <int BN, int STAGES, int BMODE, bool A_MN>
static int launch(Ctx* c, const GemmDesc& d, const CUtensorMap& ta, const CUtensorMap& tb,
                  const CUtensorMap& tbs, const CUtensorMap& tea, const CUtensorMap& teb,
                  const GemmArgs& args, std::string& err) {
  using L = GemmSmem<BN, STAGES, BMODE>;
  const auto SW = CU_TENSOR_MAP_SWIZZLE_128B;
  using R = GemmRoles<BMODE>;
  auto kern = gemm_tc_kernel<BN, STAGES, BMODE, A_MN>;
  if (smem_attr(reinterpret_cast<const void*>(kern), L::DYN, c->device, "gemm smem attribute", err)) return 1;
  const long tiles = (long)((d.M + kBM - 1) / kBM) * ((d.N + BN - 1) / BN);
  GemmArgs a = args;
  // split-K when the output has too few tiles to fill the GPU and K is long
  const int nkb = (d.K + kBK - 1) / kBK;
  a.splits = 1;
  a.kb_per_split = nkb > 0 ? nkb : 1;
  a.partial = nullptr;
  // (splits that end in the in-kernel reduction keep >= 16 k-blocks each: below that the
  // reduction by the last CTA of a tile costs more than the shorter K loop saves; a 16-wide
  // tile's reduction reads only 8 KB a split, so the rank-16 GEMMs split down to 4 k-blocks)
  const int min_kb = ((d.atomic_split && d.out && !d.out_h) || BN == 16) ? 4 : 16;
  if (tiles * 2 <= (long)c->sm_count && nkb >= 2 * min_kb) {
    int splits = (int)((long)c->sm_count / tiles);
    if (splits > nkb / min_kb) splits = nkb / min_kb;
    if (splits > 1) {
      const int kps = (nkb + splits - 1) / splits;
      splits = (nkb + kps - 1) / kps;
      a.splits = splits;
      a.kb_per_split = kps;
      if (d.atomic_split && d.out && !d.out_h) {
        // the splits add into `out` directly; without accumulation it starts from zero
        a.atomic = 1;
        if (!d.accumulate) {
          const size_t rows = d.out_trans ? (size_t)d.N : (size_t)d.M, cols = d.out_trans ? (size_t)d.M : (size_t)d.N;
          if (cudaMemset2DAsync(d.out, (size_t)d.ldo * sizeof(float), 0, cols * sizeof(float), rows, c->stream) !=
              cudaSuccess)
            return check_launch("gemm atomic split-K memset", err);
        }
      } else {
        float* part = static_cast<float*>(scratch_get(c, kSlotSplitK, (size_t)splits * d.M * d.N * sizeof(float), err));
        if (!part) return 1;
        a.partial = part;
        a.tile_cnt = split_counters(c, err);
        if (!a.tile_cnt) return 1;
      }
    }
  }
  if (plan_tail(c, d, a, tiles, (long)c->sm_count, (d.M + kBM - 1) / kBM, BN, err)) return 1;
  // epilogue through TMA stores when the output is a single row-major tensor
  CUtensorMap tout = ta;
  a.tma_out = 0;
  if (a.splits == 1) {
    std::string e2;
    if (d.out && !d.out_h && !d.out_h_t && !d.out_trans && (d.ldo % 4) == 0 &&
        (reinterpret_cast<uintptr_t>(d.out) & 15) == 0 &&
        !make_map(&tout, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, d.out, d.N, d.M, d.ldo * 4, 32, 32, SW, "out", e2))
      a.tma_out = 1;
    else if (d.out_h && !d.out && !d.out_h_trans && !d.out_h_t && d.h_scale == 1.0f && BN >= 64 && (d.ldo_h % 8) == 0 &&
             (reinterpret_cast<uintptr_t>(d.out_h) & 15) == 0 &&
             !make_map(&tout, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, d.out_h, d.N, d.M, d.ldo_h * 2, 64, 32, SW, "out_h", e2))
      a.tma_out = 2;
  }
  const long items = a.tail_parts > 1 ? a.tail_t0 + (tiles - a.tail_t0) * a.tail_parts : tiles * a.splits;
  const unsigned grid = (unsigned)(items < (long)c->sm_count ? items : (long)c->sm_count);
  {
    ProfScope prof_(c, d.name);
    launch_pdl(c, kern, grid, R::THREADS, L::DYN, ta, tb, tbs, tea, teb, tout, a);
    if (check_launch("gemm_tc", err)) return 1;
  }
  return 0;
}

// CTA-pair launch (cta_group::2, clusters of 2): f16 operands, no split-K.
template <int BN, int STAGES, int BMODE>
static int launch_pair(Ctx* c, const GemmDesc& d, const CUtensorMap& ta, const CUtensorMap& tb,
                       const CUtensorMap& tea, const CUtensorMap& teb, const GemmArgs& args, std::string& err) {
  using L = Gemm2Smem<BN, STAGES>;
  const auto SW = CU_TENSOR_MAP_SWIZZLE_128B;
  auto kern = gemm_tc2_kernel<BN, STAGES, BMODE>;
  if (smem_attr(reinterpret_cast<const void*>(kern), L::DYN, c->device, "gemm pair smem attribute", err)) return 1;
  // (the cluster occupancy is a property of the kernel and the sm_100 part, the same on every device)
  static std::atomic<int> max_clusters{0};
  if (!max_clusters.load()) {
    cudaLaunchConfig_t q = {};
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = 2; at[0].val.clusterDim.y = 1; at[0].val.clusterDim.z = 1;
    q.gridDim = dim3(2 * (unsigned)(c->sm_count / 2));
    q.blockDim = dim3(kPairThreads);
    q.dynamicSmemBytes = L::DYN;
    q.attrs = at;
    q.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, kern, &q) != cudaSuccess || n <= 0) {
      cudaGetLastError();
      n = c->sm_count / 2;
    }
    max_clusters.store(n);
  }
  GemmArgs a = args;
  a.splits = 1;
  a.kb_per_split = (d.K + kBK - 1) / kBK;
  a.partial = nullptr;
  CUtensorMap tout = ta;
  a.tma_out = 0;
  {
    std::string e2;
    if (d.out && !d.out_h && !d.out_trans && (d.ldo % 4) == 0 && (reinterpret_cast<uintptr_t>(d.out) & 15) == 0 &&
        !make_map(&tout, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, d.out, d.N, d.M, d.ldo * 4, 32, 32, SW, "out", e2))
      a.tma_out = 1;
    else if (d.out_h && !d.out && !d.out_h_trans && (d.ldo_h % 8) == 0 &&
             (reinterpret_cast<uintptr_t>(d.out_h) & 15) == 0 &&
             !make_map(&tout, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, d.out_h, d.N, d.M, d.ldo_h * 2, 64, 32, SW, "out_h", e2))
      a.tma_out = 2;
  }
  if (d.hp && (a.tma_out != 2 || d.N != 3 * d.hp->D || d.hp->D % 64)) {
    err = "gemm: the fused head preparation needs an aligned row-major f16 output of [q | k | v]";
    return 1;
  }
  const long tiles = (long)((d.M + 2 * kBM - 1) / (2 * kBM)) * ((d.N + BN - 1) / BN);
  if (plan_tail(c, d, a, tiles, (long)max_clusters, (d.M + 2 * kBM - 1) / (2 * kBM), BN, err)) return 1;
  const long items = a.tail_parts > 1 ? a.tail_t0 + (tiles - a.tail_t0) * a.tail_parts : tiles;
  const long clusters = items < (long)max_clusters ? items : (long)max_clusters;
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute at[2];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = 2; at[0].val.clusterDim.y = 1; at[0].val.clusterDim.z = 1;
  at[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[1].val.programmaticStreamSerializationAllowed = use_pdl(c) ? 1 : 0;
  cfg.gridDim = dim3((unsigned)(2 * clusters));
  cfg.blockDim = dim3(kPairThreads);
  cfg.dynamicSmemBytes = L::DYN;
  cfg.stream = c->stream;
  cfg.attrs = at;
  cfg.numAttrs = 2;
  ProfScope prof_(c, d.name);
  if (cudaLaunchKernelEx(&cfg, kern, ta, tb, tea, teb, tout, a) != cudaSuccess) return check_launch("gemm_tc2", err);
  return check_launch("gemm_tc2", err);
}

// N tile for the main GEMMs from a wave-quantized cost model: waves x per-tile time, the time of
// a 128 x bn tile taken as bn / eff(bn) + a fixed prologue / epilogue share.  eff() is the
// measured per-tile tensor efficiency of the one-CTA kernel (narrow tiles stream more operand
// bytes per MMA cycle); quantized B operands have only the 128 / 256 instantiations.
static int pick_bn(const Ctx* c, int M, int N, bool quant) {
  if (N <= 128) return 128;
  const long tm = (M + kBM - 1) / kBM;
  auto cost = [&](int bn, double eff) {
    const long tiles = tm * ((N + bn - 1) / bn);
    const long waves = (tiles + (long)c->sm_count - 1) / (long)c->sm_count;
    return (double)waves * (bn / eff + 16.0);
  };
  int best = 256;
  double bc = cost(256, 1.0);
  if (!quant && cost(192, 0.90) < bc) { best = 192; bc = cost(192, 0.90); }
  if (cost(128, 0.72) < bc) best = 128;
  return best;
}

// A GEMM over a quantized base with the weight dequantized into tensor memory (gemm_wq.cuh): the
// forward y = x W^T (NT) or the input gradient dx = dy W (TN, from the transposed codes).
static int gemm_wq(Ctx* c, const GemmDesc& d, std::string& err) {
  Weight* w = const_cast<Weight*>(d.w);   // the transposed codes are a lazily made cache
  const bool nt = d.bsrc == kB_WEIGHT_NT;
  const bool q4 = w->type == kTypeQ4_K;
  if (d.a_mn) { err = "gemm: MN-major A is not supported with an in-kernel dequantized base"; return 1; }
  if (!nt && weight_transpose_codes(c, w, err)) return 1;
  const auto F16 = CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  const auto U8 = CU_TENSOR_MAP_DATA_TYPE_UINT8;
  const auto SW = CU_TENSOR_MAP_SWIZZLE_128B;
  const auto NOSW = CU_TENSOR_MAP_SWIZZLE_NONE;
  const auto SCT = q4 ? CU_TENSOR_MAP_DATA_TYPE_UINT64 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
  const long sc_elem = q4 ? 8 : 4;
  // codes as [N features][code_ld bytes]: 64 (Q8_0) or 32 (Q4_K) bytes of k per feature per stage
  const void* codes = nt ? (const void*)w->codes : (const void*)w->codes_t;
  const long code_ld = nt ? (q4 ? w->in / 2 : w->in) : (q4 ? w->out / 2 : w->out);
  CUtensorMap tx, tc, tsc, tu;
  if (make_map(&tx, F16, d.a, d.K, d.M, d.lda * 2, 64, kWqT, SW, "activation", err)) return 1;
  if (make_map(&tc, U8, codes, code_ld, d.N, code_ld, q4 ? kWqK / 2 : kWqK, kWqF,
               q4 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_128B, "codes", err))
    return 1;
  // scales [in/32][out]: NT boxes of 4 k-blocks x 128 features, TN of 4 feature blocks x 128 k
  if (nt) {
    if (make_map(&tsc, SCT, w->scales, w->out, w->in / 32, w->out * sc_elem, kWqF, 4, NOSW, "scales", err)) return 1;
  } else {
    if (make_map(&tsc, SCT, w->scales, w->out, w->in / 32, w->out * sc_elem, kWqK, 4, NOSW, "scales", err)) return 1;
  }
  if (d.ext_at) {
    if (make_map(&tu, F16, d.ext_at, d.M, 16, d.ld_ext * 2, 64, 16, SW, "ext u^T", err)) return 1;
  } else {
    tu = tx;
  }
  WqArgs a;
  a.M = d.M; a.N = d.N; a.K = d.K;
  a.nt = nt ? 1 : 0;
  a.has_ext = d.ext_at ? 1 : 0;
  a.ext_b = d.ext_b;
  a.col_scale = d.col_scale; a.col_bias = d.col_bias; a.alpha = d.alpha;
  a.out = d.out; a.ldo = d.ldo; a.out_trans = d.out_trans; a.accumulate = d.accumulate;
  a.out_h = d.out_h; a.ldo_h = d.ldo_h; a.out_h_trans = d.out_h_trans; a.h_scale = d.h_scale;
  a.out_h_t = d.out_h_t; a.ldo_h_t = d.ldo_h_t;
  a.err = c->d_err;
  const long tiles = (long)((d.N + kWqF - 1) / kWqF) * ((d.M + kWqT - 1) / kWqT);
  const unsigned grid = (unsigned)std::min<long>(tiles, (long)c->sm_count);
  auto launch_q = [&](auto kern, int dyn) -> int {
    if (smem_attr(reinterpret_cast<const void*>(kern), dyn, c->device, "gemm_wq smem attribute", err)) return 1;
    ProfScope prof_(c, d.name);
    launch_pdl(c, kern, dim3(grid), dim3(kWqThreads), (size_t)dyn, tx, tc, tsc, tu, a);
    return check_launch("gemm_wq", err);
  };
  return q4 ? launch_q(gemm_wq_kernel<1>, WqSmem<1>::DYN) : launch_q(gemm_wq_kernel<0>, WqSmem<0>::DYN);
}

// The tensor-memory dequant kernel reads the codes by TMA: their rows must be 16-byte multiples.
static bool wq_fits(const GemmDesc& d) {
  const Weight* w = d.w;
  const bool q4 = w->type == kTypeQ4_K;
  const long code_ld = d.bsrc == kB_WEIGHT_NT ? (q4 ? w->in / 2 : w->in) : (q4 ? w->out / 2 : w->out);
  return !d.a_mn && code_ld % 16 == 0 && (!q4 || d.bsrc == kB_WEIGHT_NT || w->out % 2 == 0);
}

bool gemm_pair_applies(const Ctx* c, int M, int N, bool f16_b) {
  if (!c->gemm_pair || !f16_b || M < 2 * kBM || N < 256) return false;
  if (c->gemm_pair == 2) return true;
  if (c->tile_n != 0) return false;
  const long clusters = (long)(c->sm_count / 2);
  const long tm2 = (M + 2 * kBM - 1) / (2 * kBM);
  return tm2 * ((N + 255) / 256) >= clusters;
}

int gemm(Ctx* c, const GemmDesc& d, std::string& err) {
  if (d.M <= 0 || d.N <= 0 || d.K < 0 || (d.K == 0 && !d.ext_at)) {
    err = "gemm: need M, N > 0 and K > 0";
    return 1;
  }
  const bool weight_b = d.bsrc == kB_WEIGHT_NT || d.bsrc == kB_WEIGHT_TN;
  // quantized weights run through the in-smem dequant path unless a f16 operand copy exists
  // and the context has not asked for the in-smem path explicitly
  const bool quant = weight_b && d.w && (d.w->type == kTypeQ8_0 || d.w->type == kTypeQ4_K) &&
                     !(d.w->f16 && !c->smem_dequant);
  if (d.hp && quant) { err = "gemm: the fused head preparation needs an f16 weight operand"; return 1; }
  if (quant && c->dequant_tmem && wq_fits(d)) {
    // (inside a stream capture the transposed codes of an input-gradient GEMM cannot be made: such
    // a GEMM keeps to the shared-memory dequant path until an eager call has made them)
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    const bool capturing = cudaStreamIsCapturing(c->stream, &cs) == cudaSuccess && cs != cudaStreamCaptureStatusNone;
    if (d.bsrc == kB_WEIGHT_NT || d.w->codes_t || !capturing) return gemm_wq(c, d, err);
  }
  int bn = d.bn;
  if (bn == 128) bn = c->tile_n ? c->tile_n : pick_bn(c, d.M, d.N, quant);
  if (quant && bn == 192) bn = 256;
  if (!(bn == 16 || bn == 128 || bn == 192 || bn == 256)) {
    err = "gemm: unsupported N tile";
    return 1;
  }
  CUtensorMap ta, tb, tbs, tea, teb;
  memset(&tbs, 0, sizeof tbs);
  memset(&tea, 0, sizeof tea);
  memset(&teb, 0, sizeof teb);
  const auto BF = CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  const auto SW = CU_TENSOR_MAP_SWIZZLE_128B;
  const auto NOSW = CU_TENSOR_MAP_SWIZZLE_NONE;

  if (d.a_mn) {
    if (make_map(&ta, BF, d.a, d.M, d.K, d.lda * 2, 64, 64, SW, "A (MN-major)", err)) return 1;
  } else {
    if (make_map(&ta, BF, d.a, d.K, d.M, d.lda * 2, 64, kBM, SW, "A", err)) return 1;
  }
  int bmode = 0;
  if (d.bsrc == kB_F16_KMAJOR) {
    bmode = 0;
    if (make_map(&tb, BF, d.b, d.K, d.N, d.ldb * 2, 64, bn, SW, "B", err)) return 1;
  } else if (d.bsrc == kB_F16_MNMAJOR) {
    bmode = 1;
    if (make_map(&tb, BF, d.b, d.N, d.K, d.ldb * 2, 64, 64, SW, "B (MN-major)", err)) return 1;
  } else {
    const Weight* w = d.w;
    const bool nt = d.bsrc == kB_WEIGHT_NT;
    if (nt ? (w->out != d.N || w->in != d.K) : (w->out != d.K || w->in != d.N)) {
      err = "gemm: weight shape does not match the GEMM";
      return 1;
    }
    if (quant && w->type == kTypeQ8_0) {
      bmode = nt ? 2 : 3;
      const auto U8 = CU_TENSOR_MAP_DATA_TYPE_UINT8;
      const auto F32 = CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
      if (nt) {
        if (make_map(&tb, U8, w->codes, w->in, w->out, w->in, 64, bn, NOSW, "Q8_0 codes", err)) return 1;
        if (make_map(&tbs, F32, w->scales, w->out, w->in / 32, w->out * 4, bn, 2, NOSW, "Q8_0 scales", err)) return 1;
      } else {
        if (make_map(&tb, U8, w->codes, w->in, w->out, w->in, bn, 64, NOSW, "Q8_0 codes", err)) return 1;
        if (make_map(&tbs, F32, w->scales, w->out, w->in / 32, w->out * 4, 64, bn / 32, NOSW, "Q8_0 scales", err)) return 1;
      }
    } else if (quant && w->type == kTypeQ4_K) {
      bmode = nt ? 4 : 5;
      const auto U8 = CU_TENSOR_MAP_DATA_TYPE_UINT8;
      const auto U64 = CU_TENSOR_MAP_DATA_TYPE_UINT64;
      if (nt) {
        if (make_map(&tb, U8, w->codes, w->in / 2, w->out, w->in / 2, 32, bn, NOSW, "Q4_K codes", err)) return 1;
        if (make_map(&tbs, U64, w->scales, w->out, w->in / 32, w->out * 8, bn, 2, NOSW, "Q4_K scales", err)) return 1;
      } else {
        if (make_map(&tb, U8, w->codes, w->in / 2, w->out, w->in / 2, bn / 2, 64, NOSW, "Q4_K codes", err)) return 1;
        if (make_map(&tbs, U64, w->scales, w->out, w->in / 32, w->out * 8, 64, bn / 32, NOSW, "Q4_K scales", err)) return 1;
      }
    } else {
      // F16 / F32 bases, and quantized bases with a dequantized cache, run on the f16 copy
      if (nt) {
        bmode = 0;
        if (make_map(&tb, BF, w->f16, w->in, w->out, w->in * 2, 64, bn, SW, "W f16", err)) return 1;
      } else {
        bmode = 1;
        if (make_map(&tb, BF, w->f16, w->in, w->out, w->in * 2, 64, 64, SW, "W^T f16", err)) return 1;
      }
    }
  }
  if (d.ext_at) {
    // u^T [16][ld_ext] read MN-major: boxes of 64 rows (M) x 16 (K)
    if (make_map(&tea, BF, d.ext_at, d.M, 16, d.ld_ext * 2, 64, 16, SW, "ext A", err)) return 1;
    if (make_map(&teb, BF, d.ext_b, 64, d.N, 128, 64, bn, SW, "ext B", err)) return 1;
  } else {
    tea = ta;
    teb = tb;
  }
  if (bmode < 2) tbs = tb;   // unused by the kernel; keep it a valid map

  GemmArgs a;
  a.M = d.M; a.N = d.N; a.K = d.K;
  a.has_ext = d.ext_at ? 1 : 0;
  a.col_scale = d.col_scale; a.col_bias = d.col_bias; a.alpha = d.alpha;
  a.out = d.out; a.ldo = d.ldo; a.out_trans = d.out_trans; a.accumulate = d.accumulate;
  a.out_h = d.out_h; a.ldo_h = d.ldo_h; a.out_h_trans = d.out_h_trans; a.h_scale = d.h_scale;
  a.out_h_t = d.out_h_t; a.ldo_h_t = d.ldo_h_t;
  a.tile_cnt = nullptr;
  a.tail_t0 = 0;
  a.tail_parts = 1;
  a.tail_kbps = 0;
  a.err = c->d_err;
  a.splits = 1;
  a.kb_per_split = 1;
  a.partial = nullptr;
  a.tma_out = 0;
  a.atomic = 0;
  a.has_hp = d.hp ? 1 : 0;
  if (d.hp) a.hp = *d.hp;

  if (bn == 16) {
    if (bmode != 0) { err = "gemm: N tile 16 supports f16 K-major B only"; return 1; }
    return d.a_mn ? launch<16, 8, 0, true>(c, d, ta, tb, tbs, tea, teb, a, err)
                  : launch<16, 8, 0, false>(c, d, ta, tb, tbs, tea, teb, a, err);
  }
  if (d.a_mn) { err = "gemm: MN-major A is only instantiated with the 16-wide N tile"; return 1; }
  // CTA pairs for the f16-operand GEMMs with at least one full round of pair tiles (measured on
  // the DiT shapes: pairs match or beat the one-CTA kernel from there on; half the B bytes per
  // SM per MMA cycle).  The pair N tile (256, or 192 for K-major B) minimises rounds x tile
  // width / efficiency, 256 x 192 pair tiles running at about 0.85 of 256 x 256 per column.
  // gemm_pair 2 forces pairs wherever they apply (tile_n 192 picks 256 x 192 pair tiles).
  if (c->gemm_pair && bmode < 2 && d.M >= 2 * kBM && d.N >= 256 && !d.out_h_t && d.h_scale == 1.0f) {
    int bp = 0;
    if (c->gemm_pair == 2) {
      bp = (c->tile_n == 192 && bmode == 0) ? 192 : 256;
    } else if (c->tile_n == 0) {
      const long clusters = (long)(c->sm_count / 2);
      const long tm2 = (d.M + 2 * kBM - 1) / (2 * kBM);
      const long t256 = tm2 * ((d.N + 255) / 256), t192 = tm2 * ((d.N + 191) / 192);
      if (t256 >= clusters) {
        const double c256 = (double)((t256 + clusters - 1) / clusters) * 256.0;
        const double c192 = (double)((t192 + clusters - 1) / clusters) * 192.0 / 0.85;
        bp = (bmode == 0 && c192 < c256) ? 192 : 256;
      }
    }
    if (bp) {
      CUtensorMap tb2 = tb, tea2 = tea, teb2 = teb;
      // B halves: BN/2 rows (K-major) per CTA; MN-major B keeps its 64-wide atoms
      if (bmode == 0) {
        const void* bptr = d.bsrc == kB_F16_KMAJOR ? d.b : d.w->f16;
        const long bk = d.bsrc == kB_F16_KMAJOR ? d.K : d.w->in;
        const long bld = d.bsrc == kB_F16_KMAJOR ? d.ldb * 2 : d.w->in * 2;
        if (make_map(&tb2, BF, bptr, bk, d.N, bld, 64, bp / 2, SW, "B half", err)) return 1;
      }
      if (d.ext_at) {
        if (make_map(&teb2, BF, d.ext_b, 64, d.N, 128, 64, bp / 2, SW, "ext B half", err)) return 1;
      }
      if (d.hp && bmode != 0) { err = "gemm: the fused head preparation needs a K-major B operand"; return 1; }
      if (bp == 192) return launch_pair<192, 6, 0>(c, d, ta, tb2, tea2, teb2, a, err);
      return bmode == 0 ? launch_pair<256, 6, 0>(c, d, ta, tb2, tea2, teb2, a, err)
                        : launch_pair<256, 6, 1>(c, d, ta, tb2, tea2, teb2, a, err);
    }
  }
  if (d.hp) { err = "gemm: the fused head preparation runs on the CTA-pair kernel only"; return 1; }
  if (bn == 256) {
    switch (bmode) {
      case 0: return launch<256, 4, 0, false>(c, d, ta, tb, tbs, tea, teb, a, err);
      case 1: return launch<256, 4, 1, false>(c, d, ta, tb, tbs, tea, teb, a, err);
      case 2: return launch<256, 3, 2, false>(c, d, ta, tb, tbs, tea, teb, a, err);
      case 3: return launch<256, 3, 3, false>(c, d, ta, tb, tbs, tea, teb, a, err);
      case 4: return launch<256, 3, 4, false>(c, d, ta, tb, tbs, tea, teb, a, err);
      default: return launch<256, 3, 5, false>(c, d, ta, tb, tbs, tea, teb, a, err);
    }
  }
  if (bn == 192) {
    if (bmode == 0) return launch<192, 4, 0, false>(c, d, ta, tb, tbs, tea, teb, a, err);
    return launch<192, 4, 1, false>(c, d, ta, tb, tbs, tea, teb, a, err);
  }
  switch (bmode) {
    case 0: return launch<128, 6, 0, false>(c, d, ta, tb, tbs, tea, teb, a, err);
    case 1: return launch<128, 6, 1, false>(c, d, ta, tb, tbs, tea, teb, a, err);
    case 2: return launch<128, 4, 2, false>(c, d, ta, tb, tbs, tea, teb, a, err);
    case 3: return launch<128, 4, 3, false>(c, d, ta, tb, tbs, tea, teb, a, err);
    case 4: return launch<128, 4, 4, false>(c, d, ta, tb, tbs, tea, teb, a, err);
    default: return launch<128, 4, 5, false>(c, d, ta, tb, tbs, tea, teb, a, err);
  }
}

}  // namespace sa3k
