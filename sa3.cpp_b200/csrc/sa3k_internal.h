// sa3k_internal.h -- types shared by the sa3k translation units (not part of the C ABI).
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>
#include <utility>
#include <vector>

namespace sa3k {

// ggml type ids (ggml.h enum ggml_type) for the formats the path accepts.
enum : int { kTypeF32 = 0, kTypeF16 = 1, kTypeQ8_0 = 8, kTypeQ4_K = 12 };

struct Ctx;

// A frozen base weight W[out][in] in device memory (see quant.cu for the layouts).
struct Weight {
  int type = kTypeF32;
  int64_t in = 0, out = 0;
  void* raw = nullptr;               // F16/F32: the original values (dequant probe, row norms)
  int8_t* codes = nullptr;           // Q8_0 int8 [out][in] | Q4_K nibble pairs [out][in/2]
  float* scales = nullptr;           // Q8_0 f32 [in/32][out] | Q4_K float2 [in/32][out]
  __half* f16 = nullptr;     // f16 [out][in] operand copy (F16/F32 always; Q8_0/Q4_K
                                     // when the context keeps a dequantized cache)
  int8_t* codes_t = nullptr;         // Q8_0 int8 [in][out] | Q4_K nibble pairs [in][out/2]: the codes
                                     // transposed, made on the first input-gradient GEMM that
                                     // dequantizes in the kernel (gemm_wq)
  int device = 0;
};

// Growable device scratch owned by a context.
struct Scratch {
  void* ptr = nullptr;
  size_t bytes = 0;
};

// Per launch-class counters (the counterpart of the reference's SA3_TRAIN_PROFILE timers,
// src/train_loop.h:314-437): launches are always counted; with timing on, every launch is
// bracketed by CUDA events on the context's stream.
struct ProfEntry {
  std::string name;
  long long launches = 0;
  double ms = 0.0;
  std::vector<std::pair<cudaEvent_t, cudaEvent_t>> pending;
};

struct Ctx {
  int device = 0;
  cudaStream_t stream = nullptr;
  bool own_stream = false;
  int* d_err = nullptr;              // device error word written by bounded waits
  std::vector<Scratch> scratch;      // indexed by the slot enums of the callers
  size_t sm_count = 148;
  bool timing = false;
  bool timing_graph = false;         // timing events live in a captured CUDA graph
  bool weight_cache = true;          // quantized weights keep a dequantized f16 operand copy
  bool smem_dequant = false;         // force the in-smem dequant GEMM path for quantized weights
  int tile_n = 0;                    // main-GEMM N tile: 0 = cost model, 128 or 256 = fixed
  int gemm_pair = 1;                 // CTA-pair (cta_group::2) GEMMs: 0 never, 1 where they pay, 2 always
  bool attn_tc = true;               // tcgen05 attention kernels (else the mma.sync ones)
  bool pdl = true;                   // programmatic dependent launch between consecutive kernels
  bool step_graph = true;            // the DiT step records and replays a CUDA graph
  bool dequant_tmem = true;          // in-kernel dequantization into tensor memory (gemm_wq)
  bool fuse_head_prep = true;        // DiT: q / k head preparation in the qkv GEMM's epilogue
  // bumped whenever something a recorded graph may depend on changes: an option, a scratch
  // buffer reallocated, the RoPE table rebuilt
  uint64_t gen = 0;
  // NeoX RoPE (cos, sin) table for (positions, rot, base), kept in scratch slot kSlotRope
  const void* rope_tab = nullptr;
  int rope_tps = 0, rope_rot = 0;
  float rope_base = 0.f;
  std::vector<ProfEntry> prof;
  std::vector<cudaEvent_t> ev_pool;
};

// RAII bracket around one kernel launch of class `name`.
struct ProfScope {
  Ctx* c;
  int idx = -1;
  cudaEvent_t e0 = nullptr;
  ProfScope(Ctx* ctx, const char* name);
  ~ProfScope();
};

// Run-time lookup of the driver entry point (the library does not link libcuda, so it loads on
// machines without a GPU driver; every call then fails with a clear error instead).
typedef CUresult (*PFN_encodeTiled)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                    const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                    const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                    CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
PFN_encodeTiled encode_tiled_fn(std::string& err);

// Programmatic dependent launch for eager launches (measured on the DiT step: it hides part of
// each launch's latency when kernels are launched one by one, while a captured CUDA graph replays
// faster without the programmatic edges).
inline bool use_pdl(Ctx* c) {
  if (!c->pdl) return false;
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  return cudaStreamIsCapturing(c->stream, &cs) == cudaSuccess && cs == cudaStreamCaptureStatusNone;
}

// Launch `kern` on the context's stream with programmatic stream serialization (the kernel
// starts with pdl_prologue or waits with pdl_wait before reading its predecessors' outputs).
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(Ctx* c, void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = c->stream;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = use_pdl(c) ? 1 : 0;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

// cudaFuncAttributeMaxDynamicSharedMemorySize of `kern` on `device` (the current device), set once
// per (kernel, device): the attribute is per device, and contexts may live on several devices of
// one process and be driven from several threads.
int smem_attr(const void* kern, int bytes, int device, const char* what, std::string& err);

inline int check_launch(const char* what, std::string& err) {
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    err = std::string(what) + ": " + cudaGetErrorString(e);
    return 1;
  }
  return 0;
}

// Scratch slots owned by a context (see api.cu for the linear path's slots).
enum : int { kSlotSplitK = 63, kSlotHeadSlices = 62, kSlotRope = 61, kSlotSplitCnt = 60, kSlotChainX = 59,
             kSlotChainU = 58 };

// Scratch slot `slot` of at least `bytes` (grows; contents are not preserved on growth).
void* scratch_get(Ctx* c, int slot, size_t bytes, std::string& err);

int weight_repack(Ctx* c, Weight* w, std::string& err);
// codes_t of a Q8_0 / Q4_K weight (allocated and filled once; a no-op when present)
int weight_transpose_codes(Ctx* c, Weight* w, std::string& err);
int weight_cache_f16(Ctx* c, Weight* w, std::string& err);
int weight_dequant(Ctx* c, const Weight* w, float* dst, std::string& err);
int weight_row_norms(Ctx* c, const Weight* w, float eps, float* nsq, float* nrm, std::string& err);

// ----------------------------------------------------------------------------- GEMM engine
// B operand sources.
enum BSource : int {
  kB_F16_KMAJOR = 0,   // f16 [N][K]
  kB_F16_MNMAJOR = 1,  // f16 [K][N]
  kB_WEIGHT_NT = 2,     // weight W[out = N][in = K]           (y = x W^T)
  kB_WEIGHT_TN = 3,     // weight W[out = K][in = N], used as W^T (dx = dy W)
};

// Head preparation fused into the epilogue of a self-attention qkv projection (the CTA-pair GEMM
// with an f16 output): for output columns [0, 2 D) (q and k) each 64-column head gets its RMS
// norm (gq / gk, rstd stored to rq / rk [M][H]) and then the NeoX rotation of its first rot dims
// at the row's position (row % tps); columns [2 D, 3 D) (v) are copied.  The prepared heads go to
// `out` [M][ld] f16; the GEMM's own f16 output keeps the values before preparation.
struct HeadPrepEpi {
  __half* out = nullptr;
  long ld = 0;
  const float* gq = nullptr;
  const float* gk = nullptr;
  float* rq = nullptr;
  float* rk = nullptr;
  const float2* tab = nullptr;   // [rot / 2][tps] (cos, sin), frequency-major; null: no rotation
  int tps = 0, rot = 0, D = 0, H = 0;
  float eps = 0.f;
};

struct GemmDesc {
  int M = 0, N = 0, K = 0;
  // A: f16, K-major [M][lda] or (a_mn) MN-major [K][lda]
  const __half* a = nullptr;
  long lda = 0;
  int a_mn = 0;
  // B
  int bsrc = kB_F16_KMAJOR;
  const __half* b = nullptr;
  long ldb = 0;
  const Weight* w = nullptr;
  // K = 16 extension: ext_at f16 [16][ld_ext] (the rank-16 left factor transposed, read
  // MN-major), ext_b f16 [N][64] (columns 16..63 are not read)
  const __half* ext_at = nullptr;
  long ld_ext = 0;
  const __half* ext_b = nullptr;
  // epilogue
  const float* col_scale = nullptr;
  const float* col_bias = nullptr;
  float alpha = 1.0f;
  float* out = nullptr;
  long ldo = 0;
  int out_trans = 0;
  int accumulate = 0;
  __half* out_h = nullptr;    // h_scale * the f32 value, row-major or (out_h_trans) transposed
  long ldo_h = 0;
  int out_h_trans = 0;
  float h_scale = 1.0f;
  __half* out_h_t = nullptr;  // the unscaled value again as f16, transposed [N][ldo_h_t]
  long ldo_h_t = 0;
  int bn = 128;         // N tile (16, 128)
  // split-K partial sums may be added into `out` with f32 atomics (no reduction pass; the
  // summation order, and so the last bits, vary from run to run).  f32 `out` only.
  int atomic_split = 0;
  const HeadPrepEpi* hp = nullptr;   // fused head preparation (CTA-pair path, f16 output only)
  const char* name = "gemm";   // launch class for the profiler
};

int gemm(Ctx* c, const GemmDesc& d, std::string& err);
// true when gemm() runs an M x N GEMM with an f16 B operand (f16_b) on the CTA-pair kernel
bool gemm_pair_applies(const Ctx* c, int M, int N, bool f16_b);

}  // namespace sa3k

// The opaque handles of the C ABI (include/sa3k.h) wrap the internal objects.
struct sa3k_ctx {
  sa3k::Ctx c;
};
struct sa3k_weight {
  sa3k::Weight w;
};
