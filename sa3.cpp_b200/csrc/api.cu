// api.cu -- the sa3k C ABI (include/sa3k.h): contexts, weights, dit_lin forward / backward and
// the optimizer, orchestrated over the tcgen05 GEMM engine and the small kernels.
#include "../../include/sa3k.h"
#include "attention.h"
#include "linear.h"
#include "lora_kernels.h"
#include "sa3k_internal.h"
#include "materialize.h"
#include "sa3k_common.cuh"

#include <cmath>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <new>

namespace sa3k {

static int fill_err(char* err, int len, const std::string& msg) {
  if (err && len > 0) {
    std::strncpy(err, msg.c_str(), (size_t)len - 1);
    err[len - 1] = 0;
  }
  return 1;
}

void* scratch_get(Ctx* c, int slot, size_t bytes, std::string& err) {
  if ((int)c->scratch.size() <= slot) c->scratch.resize((size_t)slot + 1);
  Scratch& s = c->scratch[(size_t)slot];
  if (s.bytes < bytes) {
    ++c->gen;   // recorded graphs may hold the old buffer
    if (s.ptr) {
      cudaStreamSynchronize(c->stream);
      cudaFree(s.ptr);
      s.ptr = nullptr;
      s.bytes = 0;
    }
    const size_t want = (bytes + 255) & ~(size_t)255;
    if (cudaMalloc(&s.ptr, want) != cudaSuccess) {
      cudaGetLastError();
      err = "out of device memory for scratch";
      return nullptr;
    }
    s.bytes = want;
  }
  return s.ptr;
}

// Scratch slots of the C-ABI linear entry points.
enum Slot : int {
  kS_XBF = 0, kS_PREP, kS_UT, kS_DZ, kS_DG, kS_DUT, kS_CB, kS_C3, kS_HOST_IO, kS_OPT,
  kS_COUNT
};

static int64_t pad64(int64_t v) { return (v + 63) / 64 * 64; }

template <class T>
static bool get(Ctx* c, int slot, int64_t count, T*& p, std::string& err) {
  p = static_cast<T*>(scratch_get(c, slot, (size_t)count * sizeof(T), err));
  return p != nullptr;
}

// The C-ABI linear: f32 activations in, the adapter prepared per call.  y_out: forward output
// (null = no forward); y_in: the forward output the DoRA backward needs when no forward runs.
static int linear_run(Ctx* c, const Weight* w, const sa3k_adapter* ad, const float* bias, const float* x,
                      const float* dy, int64_t S, float* y_out, const float* y_in, float* dx, float* dA,
                      float* dB, float* dm, int accumulate, std::string& err) {
  const int64_t in = w->in, out = w->out;
  const bool adapter = ad != nullptr;
  const bool dora = adapter && ad->magnitude != nullptr;
  const bool fwd = y_out != nullptr;
  const bool bwd = dy != nullptr;
  if (S <= 0) { err = "S must be positive"; return 1; }
  if (in % 64 != 0) { err = "in must be a multiple of 64"; return 1; }
  if (adapter && (ad->rank < 1 || ad->rank > 16 || !ad->A || !ad->B)) { err = "adapter rank must be 1..16 with A and B"; return 1; }
  if (dora && !ad->base_norm_sq) { err = "dora adapter needs base_norm_sq"; return 1; }
  if (bwd && !fwd && dora && !y_in) { err = "dora backward needs the forward output y"; return 1; }
  const int64_t s_pad = pad64(S);
  __half* x_h;
  if (!get(c, kS_XBF, S * in, x_h, err)) return 1;
  if (k_cvt_f16(c, x, S * in, x_h, err)) return 1;

  AdapterPrep prep;
  __half* ut = nullptr;
  if (adapter) {
    prep.rank = ad->rank; prep.in = in; prep.out = out; prep.s = ad->scale;
    prep.A = ad->A; prep.B = ad->B; prep.m = dora ? ad->magnitude : nullptr; prep.bns = ad->base_norm_sq;
    void* mem = scratch_get(c, kS_PREP, adapter_prep_bytes(in, out, dora), err);
    if (!mem) return 1;
    adapter_bind(prep, mem);
    if (adapter_prepare(c, w, prep, err)) return 1;
    if (!get(c, kS_UT, 16 * s_pad, ut, err))
      return 1;
  }
  if (fwd || (bwd && adapter)) {
    // the backward needs u^T, which the forward produces; a backward-only call recomputes it
    LinearFwd f;
    f.w = w; f.ad = adapter ? &prep : nullptr; f.bias = bias; f.x_h = x_h; f.M = S;
    f.y = y_out; f.ut = ut; f.ut_ld = s_pad;
    if (!fwd) {
      // u only (the main GEMM is skipped without an output)
      if (lora_u(c, x_h, S, in, prep, ut, s_pad, err)) return 1;
    } else if (linear_forward(c, f, err)) {
      return 1;
    }
  }
  if (!bwd) return 0;
  LinearBwd b;
  b.w = w; b.ad = adapter ? &prep : nullptr; b.bias = bias; b.x_h = x_h; b.y = fwd ? y_out : y_in; b.dy = dy;
  b.M = S; b.ut = ut; b.ut_ld = s_pad;
  b.dx = dx; b.dx_accumulate = accumulate;
  b.dA = dA; b.dB = dB; b.dm = dm; b.grad_accumulate = accumulate;
  if (!get(c, kS_DZ, S * out, b.dz, err)) return 1;
  if (dora && (!get(c, kS_DG, out, b.dg, err) || !get(c, kS_CB, 16 * out, b.cb, err) || !get(c, kS_C3, 256, b.c3, err)))
    return 1;
  if (adapter && !get(c, kS_DUT, 16 * s_pad, b.dut, err)) return 1;
  return linear_backward(c, b, err);
}

// Record a timing event; inside a stream capture it must become an event-record node of the
// graph (cudaEventRecordExternal), otherwise it would only be a capture dependency.
static void record_event(cudaEvent_t e, cudaStream_t st) {
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  cudaStreamIsCapturing(st, &cs);
  if (cs == cudaStreamCaptureStatusActive) cudaEventRecordWithFlags(e, st, cudaEventRecordExternal);
  else cudaEventRecord(e, st);
}

ProfScope::ProfScope(Ctx* ctx, const char* name) : c(ctx) {
  for (size_t i = 0; i < c->prof.size(); ++i)
    if (c->prof[i].name == name) { idx = (int)i; break; }
  if (idx < 0) {
    c->prof.push_back(ProfEntry{});
    c->prof.back().name = name;
    idx = (int)c->prof.size() - 1;
  }
  c->prof[(size_t)idx].launches += 1;
  if (c->timing) {
    if (c->ev_pool.empty()) {
      cudaEvent_t e;
      cudaEventCreate(&e);
      c->ev_pool.push_back(e);
    }
    e0 = c->ev_pool.back();
    c->ev_pool.pop_back();
    record_event(e0, c->stream);
  }
}

ProfScope::~ProfScope() {
  if (!e0) return;
  cudaEvent_t e1;
  if (c->ev_pool.empty()) cudaEventCreate(&e1);
  else { e1 = c->ev_pool.back(); c->ev_pool.pop_back(); }
  record_event(e1, c->stream);
  c->prof[(size_t)idx].pending.emplace_back(e0, e1);
}

// Eager mode (timing 1): add the elapsed times of the recorded pairs and recycle the events.
// Graph mode (timing 2): the pairs were captured into a graph and are re-recorded by each
// replay; report the most recent replay's times and keep the pairs.
static void prof_collect(Ctx* c) {
  cudaStreamSynchronize(c->stream);
  for (ProfEntry& p : c->prof) {
    if (c->timing_graph) p.ms = 0.0;
    for (auto& ev : p.pending) {
      float ms = 0.f;
      if (cudaEventElapsedTime(&ms, ev.first, ev.second) == cudaSuccess) p.ms += ms;
      if (!c->timing_graph) {
        c->ev_pool.push_back(ev.first);
        c->ev_pool.push_back(ev.second);
      }
    }
    if (!c->timing_graph) p.pending.clear();
  }
  cudaGetLastError();
}

static int adamw_bias_corrections(const sa3k_adamw_params* hp, int step, float& b1c, float& b2c) {
  // exactly the reference's float expressions (src/train_optimizer.h:55-56)
  b1c = 1.0f - std::pow(hp->beta1, (float)step);
  b2c = 1.0f - std::pow(hp->beta2, (float)step);
  return 0;
}

}  // namespace sa3k

using namespace sa3k;

extern "C" {

const char* sa3k_version(void) { return "sa3k 0.1.0 (sm_100a)"; }

int sa3k_ctx_create(int device, sa3k_ctx** out, char* err, int err_len) {
  if (!out) return fill_err(err, err_len, "out is NULL");
  *out = nullptr;
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0) {
    cudaGetLastError();
    return fill_err(err, err_len, "no CUDA device available (sa3k has no CPU fallback)");
  }
  if (device < 0 || device >= n) return fill_err(err, err_len, "device ordinal out of range");
  cudaDeviceProp prop;
  if (cudaGetDeviceProperties(&prop, device) != cudaSuccess) return fill_err(err, err_len, "cudaGetDeviceProperties failed");
  if (prop.major != 10) return fill_err(err, err_len, "sa3k kernels are built for sm_100a (B200); device is sm_" +
                                                          std::to_string(prop.major) + std::to_string(prop.minor));
  if (cudaSetDevice(device) != cudaSuccess) return fill_err(err, err_len, "cudaSetDevice failed");
  sa3k_ctx* c = new (std::nothrow) sa3k_ctx();
  if (!c) return fill_err(err, err_len, "out of host memory");
  c->c.device = device;
  c->c.sm_count = (size_t)prop.multiProcessorCount;
  if (cudaStreamCreateWithFlags(&c->c.stream, cudaStreamNonBlocking) != cudaSuccess ||
      cudaMalloc(&c->c.d_err, sizeof(int)) != cudaSuccess || cudaMemset(c->c.d_err, 0, sizeof(int)) != cudaSuccess) {
    delete c;
    return fill_err(err, err_len, "failed to create the context stream / error word");
  }
  c->c.own_stream = true;
  *out = c;
  return 0;
}

void sa3k_ctx_destroy(sa3k_ctx* ctx) {
  if (!ctx) return;
  cudaSetDevice(ctx->c.device);
  prof_collect(&ctx->c);
  for (cudaEvent_t e : ctx->c.ev_pool) cudaEventDestroy(e);
  for (auto& s : ctx->c.scratch)
    if (s.ptr) cudaFree(s.ptr);
  if (ctx->c.d_err) cudaFree(ctx->c.d_err);
  if (ctx->c.own_stream) cudaStreamDestroy(ctx->c.stream);
  delete ctx;
}

int sa3k_ctx_set_stream(sa3k_ctx* ctx, void* stream, char* err, int err_len) {
  if (!ctx) return fill_err(err, err_len, "ctx is NULL");
  cudaSetDevice(ctx->c.device);
  if (ctx->c.own_stream) {
    cudaStreamSynchronize(ctx->c.stream);
    cudaStreamDestroy(ctx->c.stream);
    ctx->c.own_stream = false;
  }
  ctx->c.stream = static_cast<cudaStream_t>(stream);   // NULL is CUDA's legacy default stream
  return 0;
}

int sa3k_ctx_set_option(sa3k_ctx* ctx, int option, int64_t value, char* err, int err_len) {
  if (!ctx) return fill_err(err, err_len, "ctx is NULL");
  ++ctx->c.gen;
  switch (option) {
    case SA3K_OPT_WEIGHT_F16_CACHE: ctx->c.weight_cache = value != 0; return 0;
    case SA3K_OPT_SMEM_DEQUANT: ctx->c.smem_dequant = value != 0; return 0;
    case SA3K_OPT_GEMM_TILE_N:
      if (value != 0 && value != 128 && value != 192 && value != 256)
        return fill_err(err, err_len, "tile N must be 0, 128, 192 or 256");
      ctx->c.tile_n = (int)value;
      return 0;
    case SA3K_OPT_GEMM_PAIR:
      if (value < 0 || value > 2) return fill_err(err, err_len, "GEMM pair option must be 0, 1 or 2");
      ctx->c.gemm_pair = (int)value;
      return 0;
    case SA3K_OPT_ATTN_TC: ctx->c.attn_tc = value != 0; return 0;
    case SA3K_OPT_PDL: ctx->c.pdl = value != 0; return 0;
    case SA3K_OPT_STEP_GRAPH: ctx->c.step_graph = value != 0; return 0;
    case SA3K_OPT_DEQUANT_TMEM: ctx->c.dequant_tmem = value != 0; return 0;
    case SA3K_OPT_FUSE_HEAD_PREP: ctx->c.fuse_head_prep = value != 0; return 0;
    default: return fill_err(err, err_len, "unknown option");
  }
}

int sa3k_sync(sa3k_ctx* ctx, char* err, int err_len) {
  if (!ctx) return fill_err(err, err_len, "ctx is NULL");
  cudaSetDevice(ctx->c.device);
  cudaError_t e = cudaStreamSynchronize(ctx->c.stream);
  if (e != cudaSuccess) return fill_err(err, err_len, std::string("CUDA error: ") + cudaGetErrorString(e));
  int code = 0;
  if (cudaMemcpy(&code, ctx->c.d_err, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess)
    return fill_err(err, err_len, "failed to read the device error word");
  if (code != 0) {
    cudaMemset(ctx->c.d_err, 0, sizeof(int));
    return fill_err(err, err_len, "device wait timed out inside a kernel (code " + std::to_string(code) + ")");
  }
  return 0;
}

// One thread waits on a shared-memory mbarrier that nothing arrives at, through the same bounded
// wait as every pipeline of the library: the wait runs out, records kErrTimeoutOther in the
// context's error word and the kernel returns.
__global__ void wait_probe_kernel(int* err, unsigned long long limit_ns) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x != 0) return;
  sa3k::mbar_init(&bar, 1);
  sa3k::fence_barrier_init();
  sa3k::mbar_wait(&bar, 0u, err, sa3k::kErrTimeoutOther, limit_ns);
}

int sa3k_check_bounded_wait(sa3k_ctx* ctx, int limit_us, char* err, int err_len) {
  if (!ctx) return fill_err(err, err_len, "ctx is NULL");
  if (limit_us < 1 || limit_us > 2000000) return fill_err(err, err_len, "limit_us must be in 1 .. 2000000");
  cudaSetDevice(ctx->c.device);
  wait_probe_kernel<<<1, 32, 0, ctx->c.stream>>>(ctx->c.d_err, 1000ull * (unsigned long long)limit_us);
  std::string e;
  if (check_launch("wait probe", e)) return fill_err(err, err_len, e);
  return 0;
}

int sa3k_profile_enable(sa3k_ctx* ctx, int timing, char* err, int err_len) {
  if (!ctx) return fill_err(err, err_len, "ctx is NULL");
  if (timing < 0 || timing > 2) return fill_err(err, err_len, "timing must be 0, 1 or 2");
  cudaSetDevice(ctx->c.device);
  if (ctx->c.timing_graph) {   // release the graph-owned event pairs
    for (ProfEntry& p : ctx->c.prof)
      for (auto& ev : p.pending) { ctx->c.ev_pool.push_back(ev.first); ctx->c.ev_pool.push_back(ev.second); }
    for (ProfEntry& p : ctx->c.prof) p.pending.clear();
    ctx->c.timing_graph = false;
  }
  prof_collect(&ctx->c);
  ctx->c.prof.clear();
  ctx->c.timing = timing != 0;
  ctx->c.timing_graph = timing == 2;
  return 0;
}

int sa3k_profile_read(sa3k_ctx* ctx, sa3k_profile_entry* out, int max, int* n_out, char* err, int err_len) {
  if (!ctx || !n_out) return fill_err(err, err_len, "NULL argument");
  cudaSetDevice(ctx->c.device);
  prof_collect(&ctx->c);
  int n = 0;
  for (const ProfEntry& p : ctx->c.prof) {
    if (out && n < max) {
      std::memset(out[n].name, 0, sizeof out[n].name);
      std::strncpy(out[n].name, p.name.c_str(), sizeof out[n].name - 1);
      out[n].launches = p.launches;
      out[n].total_ms = p.ms;
    }
    ++n;
  }
  *n_out = n;
  return 0;
}

int sa3k_weight_upload(sa3k_ctx* ctx, int type, const void* blocks, int64_t in, int64_t out, sa3k_weight** wout,
                       char* err, int err_len) {
  if (!ctx || !blocks || !wout) return fill_err(err, err_len, "NULL argument");
  *wout = nullptr;
  if (in <= 0 || out <= 0) return fill_err(err, err_len, "weight dims must be positive");
  if (in % 64 != 0) return fill_err(err, err_len, "weight `in` must be a multiple of 64");
  size_t raw_bytes = 0;
  switch (type) {
    case kTypeF32: raw_bytes = (size_t)(in * out * 4); break;
    case kTypeF16: raw_bytes = (size_t)(in * out * 2); break;
    case kTypeQ8_0: raw_bytes = (size_t)(in / 32 * 34 * out); break;
    case kTypeQ4_K:
      if (in % 256 != 0) return fill_err(err, err_len, "Q4_K needs `in` to be a multiple of 256");
      raw_bytes = (size_t)(in / 256 * 144 * out);
      break;
    default: return fill_err(err, err_len, "unsupported ggml type (F32, F16, Q8_0, Q4_K)");
  }
  cudaSetDevice(ctx->c.device);
  sa3k_weight* h = new (std::nothrow) sa3k_weight();
  if (!h) return fill_err(err, err_len, "out of host memory");
  Weight& w = h->w;
  w.type = type; w.in = in; w.out = out; w.device = ctx->c.device;
  std::string e;
  auto fail = [&](const std::string& msg) {
    if (w.raw) cudaFree(w.raw);
    if (w.codes) cudaFree(w.codes);
    if (w.scales) cudaFree(w.scales);
    if (w.f16) cudaFree(w.f16);
    if (w.codes_t) cudaFree(w.codes_t);
    delete h;
    cudaGetLastError();
    return fill_err(err, err_len, msg);
  };
  if (cudaMalloc(&w.raw, raw_bytes) != cudaSuccess) return fail("out of device memory (weight)");
  if (cudaMemcpyAsync(w.raw, blocks, raw_bytes, cudaMemcpyHostToDevice, ctx->c.stream) != cudaSuccess)
    return fail("weight upload copy failed");
  if (type == kTypeQ8_0) {
    if (cudaMalloc(&w.codes, (size_t)(in * out)) != cudaSuccess ||
        cudaMalloc(&w.scales, (size_t)(in / 32 * out * 4)) != cudaSuccess)
      return fail("out of device memory (weight)");
  } else if (type == kTypeQ4_K) {
    if (cudaMalloc(&w.codes, (size_t)(in / 2 * out)) != cudaSuccess ||
        cudaMalloc(&w.scales, (size_t)(in / 32 * out * 8)) != cudaSuccess)
      return fail("out of device memory (weight)");
  } else {
    if (cudaMalloc(&w.f16, (size_t)(in * out * 2)) != cudaSuccess) return fail("out of device memory (weight)");
  }
  if (weight_repack(&ctx->c, &w, e)) return fail(e);
  if ((type == kTypeQ8_0 || type == kTypeQ4_K) && ctx->c.weight_cache) {
    if (cudaMalloc(&w.f16, (size_t)(in * out * 2)) != cudaSuccess) return fail("out of device memory (weight cache)");
    if (weight_cache_f16(&ctx->c, &w, e)) return fail(e);
  }
  if (cudaStreamSynchronize(ctx->c.stream) != cudaSuccess) return fail("weight repack failed");
  if (type == kTypeQ8_0 || type == kTypeQ4_K) {   // codes + scales carry every bit of the blocks
    cudaFree(w.raw);
    w.raw = nullptr;
  }
  *wout = h;
  return 0;
}

void sa3k_weight_free(sa3k_weight* h) {
  if (!h) return;
  Weight& w = h->w;
  cudaSetDevice(w.device);   // cudaFree waits for the device's outstanding work
  if (w.raw) cudaFree(w.raw);
  if (w.codes) cudaFree(w.codes);
  if (w.scales) cudaFree(w.scales);
  if (w.f16) cudaFree(w.f16);
  if (w.codes_t) cudaFree(w.codes_t);
  delete h;
}

int sa3k_dequant(sa3k_ctx* ctx, const sa3k_weight* w, float* dst, char* err, int err_len) {
  if (!ctx || !w || !dst) return fill_err(err, err_len, "NULL argument");
  cudaSetDevice(ctx->c.device);
  std::string e;
  if (weight_dequant(&ctx->c, &w->w, dst, e)) return fill_err(err, err_len, e);
  return 0;
}

int sa3k_row_norms(sa3k_ctx* ctx, const sa3k_weight* w, float eps, float* nsq, float* nrm, char* err, int err_len) {
  if (!ctx || !w) return fill_err(err, err_len, "NULL argument");
  cudaSetDevice(ctx->c.device);
  std::string e;
  if (weight_row_norms(&ctx->c, &w->w, eps, nsq, nrm, e)) return fill_err(err, err_len, e);
  return 0;
}

int sa3k_col_norms(sa3k_ctx* ctx, const sa3k_weight* w, float* nrm, char* err, int err_len) {
  if (!ctx || !w || !nrm) return fill_err(err, err_len, "NULL argument");
  cudaSetDevice(ctx->c.device);
  std::string e;
  if (mat_col_norms(&ctx->c, &w->w, nrm, e)) return fill_err(err, err_len, e);
  return 0;
}

int sa3k_linear_fwd(sa3k_ctx* ctx, const sa3k_weight* w, const sa3k_adapter* ad, const float* bias,
                    const float* x, int64_t S, float* y, char* err, int err_len) {
  if (!ctx || !w || !x || !y) return fill_err(err, err_len, "NULL argument");
  cudaSetDevice(ctx->c.device);
  std::string e;
  if (linear_run(&ctx->c, &w->w, ad, bias, x, nullptr, S, y, nullptr, nullptr, nullptr, nullptr, nullptr, 0, e))
    return fill_err(err, err_len, e);
  return 0;
}

int sa3k_linear_bwd(sa3k_ctx* ctx, const sa3k_weight* w, const sa3k_adapter* ad, const float* bias,
                    const float* x, const float* y, const float* dy, int64_t S, float* dx, float* dA, float* dB,
                    float* dm, int accumulate, char* err, int err_len) {
  if (!ctx || !w || !x || !dy) return fill_err(err, err_len, "NULL argument");
  if (ad && (!dA || !dB || (ad->magnitude && !dm))) return fill_err(err, err_len, "adapter gradients need dA, dB (and dm)");
  cudaSetDevice(ctx->c.device);
  std::string e;
  if (linear_run(&ctx->c, &w->w, ad, bias, x, dy, S, nullptr, y, dx, dA, dB, dm, accumulate, e))
    return fill_err(err, err_len, e);
  return 0;
}

int sa3k_linear_fwd_bwd(sa3k_ctx* ctx, const sa3k_weight* w, const sa3k_adapter* ad, const float* bias,
                        const float* x, const float* dy, int64_t S, float* y, float* dx, float* dA, float* dB,
                        float* dm, char* err, int err_len) {
  if (!ctx || !w || !x || !dy || !y) return fill_err(err, err_len, "NULL argument");
  if (ad && (!dA || !dB || (ad->magnitude && !dm))) return fill_err(err, err_len, "adapter gradients need dA, dB (and dm)");
  cudaSetDevice(ctx->c.device);
  std::string e;
  if (linear_run(&ctx->c, &w->w, ad, bias, x, dy, S, y, nullptr, dx, dA, dB, dm, 0, e)) return fill_err(err, err_len, e);
  return 0;
}

int sa3k_linear_fwd_bwd_host(sa3k_ctx* ctx, const sa3k_weight* w, const sa3k_adapter* adh, const float* bias_h,
                             const float* x_h, const float* dy_h, int64_t S, float* y_h, float* dx_h, float* dA_h,
                             float* dB_h, float* dm_h, char* err, int err_len) {
  if (!ctx || !w || !x_h || !dy_h || !y_h) return fill_err(err, err_len, "NULL argument");
  // the adapter is validated before its host arrays are read (their sizes follow from the rank)
  if (adh && (adh->rank < 1 || adh->rank > 16 || !adh->A || !adh->B))
    return fill_err(err, err_len, "adapter rank must be 1..16 with A and B");
  if (S <= 0) return fill_err(err, err_len, "S must be positive");
  Ctx* c = &ctx->c;
  cudaSetDevice(c->device);
  const int64_t in = w->w.in, out = w->w.out;
  const int rank = adh ? adh->rank : 0;
  const bool dora = adh && adh->magnitude;
  // one device block: x, dy, y, dx, A, B, m, bns, bias, dA, dB, dm
  const int64_t n_x = S * in, n_dy = S * out;
  const int64_t n_a = (int64_t)rank * in, n_b = out * rank;
  const int64_t total = 2 * n_x + 2 * n_dy + 2 * n_a + 2 * n_b + 4 * out + 64;
  std::string e;
  float* base = static_cast<float*>(scratch_get(c, kS_HOST_IO, (size_t)total * sizeof(float), e));
  if (!base) return fill_err(err, err_len, e);
  auto take = [&](int64_t n) { float* p = base; base += (n + 15) / 16 * 16; return p; };
  float *x = take(n_x), *dy = take(n_dy), *y = take(n_dy), *dx = take(n_x);
  float *A = take(n_a), *B = take(n_b), *m = take(out), *bns = take(out), *bias = take(out);
  float *dA = take(n_a), *dB = take(n_b), *dm = take(out);
  const cudaStream_t st = c->stream;
  auto h2d = [&](float* d, const float* h, int64_t n) {
    return cudaMemcpyAsync(d, h, (size_t)n * sizeof(float), cudaMemcpyHostToDevice, st) == cudaSuccess;
  };
  auto d2h = [&](float* h, const float* d, int64_t n) {
    return cudaMemcpyAsync(h, d, (size_t)n * sizeof(float), cudaMemcpyDeviceToHost, st) == cudaSuccess;
  };
  bool ok = h2d(x, x_h, n_x) && h2d(dy, dy_h, n_dy);
  if (bias_h) ok = ok && h2d(bias, bias_h, out);
  sa3k_adapter ad{};
  if (adh) {
    ok = ok && h2d(A, adh->A, n_a) && h2d(B, adh->B, n_b);
    if (dora) ok = ok && h2d(m, adh->magnitude, out) && h2d(bns, adh->base_norm_sq, out);
    ad.A = A; ad.B = B; ad.magnitude = dora ? m : nullptr; ad.base_norm_sq = dora ? bns : nullptr;
    ad.scale = adh->scale; ad.rank = rank;
  }
  if (!ok) return fill_err(err, err_len, "host->device copy failed");
  if (linear_run(c, &w->w, adh ? &ad : nullptr, bias_h ? bias : nullptr, x, dy, S, y, nullptr, dx_h ? dx : nullptr,
                 adh ? dA : nullptr, adh ? dB : nullptr, dora ? dm : nullptr, 0, e))
    return fill_err(err, err_len, e);
  ok = d2h(y_h, y, n_dy);
  if (dx_h) ok = ok && d2h(dx_h, dx, n_x);
  if (adh) {
    if (dA_h) ok = ok && d2h(dA_h, dA, n_a);
    if (dB_h) ok = ok && d2h(dB_h, dB, n_b);
    if (dora && dm_h) ok = ok && d2h(dm_h, dm, out);
  }
  if (!ok) return fill_err(err, err_len, "device->host copy failed");
  if (cudaStreamSynchronize(st) != cudaSuccess) return fill_err(err, err_len, "linear step failed");
  return 0;
}

static void set4(const sa3k_tensor4* t, const __half*& p, long& sb, long& sh, long& ld) {
  p = static_cast<const __half*>(t->data);
  sb = (long)t->batch_stride;
  sh = (long)t->head_stride;
  ld = (long)t->row_stride;
}

static int attn_args(int B, int H, int Sq, int Sk, int head_dim, float scale, int window, const sa3k_tensor4* q,
                     const sa3k_tensor4* k, const sa3k_tensor4* v, const sa3k_tensor4* o, AttnArgs& a,
                     std::string& err) {
  if (!q || !k || !v || !o || !q->data || !k->data || !v->data || !o->data) { err = "NULL tensor"; return 1; }
  if (B <= 0 || H <= 0 || Sq <= 0 || Sk <= 0) { err = "attention dims must be positive"; return 1; }
  a.B = B; a.H = H; a.Sq = Sq; a.Sk = Sk; a.head_dim = head_dim; a.scale = scale; a.window = window;
  set4(q, a.q, a.q_sb, a.q_sh, a.q_ld);
  set4(k, a.k, a.k_sb, a.k_sh, a.k_ld);
  set4(v, a.v, a.v_sb, a.v_sh, a.v_ld);
  a.o = static_cast<__half*>(o->data);
  a.o_sb = (long)o->batch_stride; a.o_sh = (long)o->head_stride; a.o_ld = (long)o->row_stride;
  for (long st : {a.q_ld, a.k_ld, a.v_ld, a.o_ld})
    if (st % 8) { err = "attention rows must be 16-byte aligned (row_stride % 8 == 0)"; return 1; }
  return 0;
}

int sa3k_attention_fwd(sa3k_ctx* ctx, int B, int H, int Sq, int Sk, int head_dim, float scale, int window,
                       const sa3k_tensor4* q, const sa3k_tensor4* k, const sa3k_tensor4* v, const sa3k_tensor4* o,
                       float* lse, char* err, int err_len) {
  if (!ctx) return fill_err(err, err_len, "ctx is NULL");
  cudaSetDevice(ctx->c.device);
  std::string e;
  AttnArgs a;
  if (attn_args(B, H, Sq, Sk, head_dim, scale, window, q, k, v, o, a, e)) return fill_err(err, err_len, e);
  a.lse = lse;
  if (attn_forward(&ctx->c, a, e)) return fill_err(err, err_len, e);
  return 0;
}

int sa3k_attention_bwd(sa3k_ctx* ctx, int B, int H, int Sq, int Sk, int head_dim, float scale, int window,
                       const sa3k_tensor4* q, const sa3k_tensor4* k, const sa3k_tensor4* v, const sa3k_tensor4* o,
                       const sa3k_tensor4* dO, const float* lse, const sa3k_tensor4* dq, const sa3k_tensor4* dk,
                       const sa3k_tensor4* dv, char* err, int err_len) {
  if (!ctx || !dO || !dq || !lse) return fill_err(err, err_len, "NULL argument");
  cudaSetDevice(ctx->c.device);
  std::string e;
  AttnArgs a;
  if (attn_args(B, H, Sq, Sk, head_dim, scale, window, q, k, v, o, a, e)) return fill_err(err, err_len, e);
  a.lse = const_cast<float*>(lse);
  set4(dO, a.dO, a.dO_sb, a.dO_sh, a.dO_ld);
  a.dq = static_cast<float*>(dq->data); a.dq_sb = (long)dq->batch_stride; a.dq_sh = (long)dq->head_stride;
  a.dq_ld = (long)dq->row_stride;
  const bool kv = dk && dv && dk->data && dv->data;
  if (kv) {
    a.dk = static_cast<float*>(dk->data); a.dk_sb = (long)dk->batch_stride; a.dk_sh = (long)dk->head_stride;
    a.dk_ld = (long)dk->row_stride;
    a.dv = static_cast<float*>(dv->data); a.dv_sb = (long)dv->batch_stride; a.dv_sh = (long)dv->head_stride;
    a.dv_ld = (long)dv->row_stride;
  }
  float* dsum = static_cast<float*>(scratch_get(&ctx->c, kS_OPT + 1, sizeof(float) * (size_t)B * H * Sq, e));
  if (!dsum) return fill_err(err, err_len, e);
  a.Dsum = dsum;
  if (attn_backward(&ctx->c, a, kv, e)) return fill_err(err, err_len, e);
  return 0;
}

// ------------------------------------------------------------------ attention backward, fixed scratch
// The one scratch buffer of the attention backward (D = rowsum(dO o O), one float per (b, h, query
// row)) lives in this file-scope device array instead of context scratch, so the entry point
// below never allocates device memory.  Its device address is looked up once per device.
constexpr int64_t kNoAllocDsumRows = int64_t(1) << 20;           // 4 MiB of f32
static __device__ __align__(256) float g_noalloc_dsum[kNoAllocDsumRows];
constexpr int kNoAllocMaxDevices = 64;
static float* g_noalloc_dsum_addr[kNoAllocMaxDevices] = {};
static std::mutex g_noalloc_mu;

int sa3k_attention_bwd_noalloc(sa3k_ctx* ctx, int B, int H, int Sq, int Sk, int head_dim, float scale,
                               int window, const sa3k_tensor4* q, const sa3k_tensor4* k,
                               const sa3k_tensor4* v, const sa3k_tensor4* o, const sa3k_tensor4* dO,
                               const float* lse, const sa3k_tensor4* dq, const sa3k_tensor4* dk,
                               const sa3k_tensor4* dv, char* err, int err_len) {
  if (!ctx || !dO || !dq || !lse) return fill_err(err, err_len, "NULL argument");
  const int dev = ctx->c.device;
  if (dev < 0 || dev >= kNoAllocMaxDevices) return fill_err(err, err_len, "device index out of range");
  if (B <= 0 || H <= 0 || Sq <= 0) return fill_err(err, err_len, "B, H and Sq must be positive");
  const int64_t rows = (int64_t)B * H * Sq;
  if (rows > kNoAllocDsumRows) {
    char msg[160];
    std::snprintf(msg, sizeof msg,
                  "sa3k_attention_bwd_noalloc: B*H*Sq = %lld exceeds its fixed scratch of %lld rows",
                  (long long)rows, (long long)kNoAllocDsumRows);
    return fill_err(err, err_len, msg);
  }
  if (cudaSetDevice(dev) != cudaSuccess) return fill_err(err, err_len, "cudaSetDevice failed");
  float* dsum = nullptr;
  {
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    if (!g_noalloc_dsum_addr[dev]) {
      void* p = nullptr;
      const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_dsum);
      if (e != cudaSuccess) {
        cudaGetLastError();
        return fill_err(err, err_len, std::string("cudaGetSymbolAddress of the fixed scratch failed: ") +
                                          cudaGetErrorString(e));
      }
      g_noalloc_dsum_addr[dev] = static_cast<float*>(p);
    }
    dsum = g_noalloc_dsum_addr[dev];
  }
  std::string e;
  AttnArgs a;
  if (attn_args(B, H, Sq, Sk, head_dim, scale, window, q, k, v, o, a, e)) return fill_err(err, err_len, e);
  a.lse = const_cast<float*>(lse);
  set4(dO, a.dO, a.dO_sb, a.dO_sh, a.dO_ld);
  a.dq = static_cast<float*>(dq->data); a.dq_sb = (long)dq->batch_stride; a.dq_sh = (long)dq->head_stride;
  a.dq_ld = (long)dq->row_stride;
  const bool kv = dk && dv && dk->data && dv->data;
  if (kv) {
    a.dk = static_cast<float*>(dk->data); a.dk_sb = (long)dk->batch_stride; a.dk_sh = (long)dk->head_stride;
    a.dk_ld = (long)dk->row_stride;
    a.dv = static_cast<float*>(dv->data); a.dv_sb = (long)dv->batch_stride; a.dv_sh = (long)dv->head_stride;
    a.dv_ld = (long)dv->row_stride;
  }
  // every D entry is written by the pre-pass before the dq / dk-dv passes read it: no clearing
  a.Dsum = dsum;
  if (attn_backward(&ctx->c, a, kv, e)) return fill_err(err, err_len, e);
  return 0;
}

int sa3k_head_prep_fwd(sa3k_ctx* ctx, const float* y, int T, int ncols, int H, const sa3k_head_slice* slices,
                       int nslices, int tps, float eps, int rot, float rope_base, void* out, char* err, int err_len) {
  if (!ctx || !y || !slices || !out) return fill_err(err, err_len, "NULL argument");
  if (nslices < 1 || nslices > 5) return fill_err(err, err_len, "1..5 slices");
  cudaSetDevice(ctx->c.device);
  HeadSlice hs[5];
  for (int i = 0; i < nslices; ++i) {
    hs[i].col = slices[i].col; hs[i].gamma = slices[i].gamma; hs[i].rope = slices[i].rope; hs[i].rstd = slices[i].rstd;
    if (hs[i].col % 64 || hs[i].col + H * 64 > ncols) return fill_err(err, err_len, "slice outside y");
  }
  std::string e;
  if (k_head_prep_fwd(&ctx->c, y, T, ncols, H, hs, nslices, tps, eps, rot, rope_base,
                      static_cast<__half*>(out), e))
    return fill_err(err, err_len, e);
  return 0;
}

int sa3k_head_prep_bwd(sa3k_ctx* ctx, const float* g, int64_t g_ld, const float* y, int T, int ncols, int H,
                       const sa3k_head_slice* slice, int tps, int rot, float rope_base, float* dy, char* err,
                       int err_len) {
  if (!ctx || !g || !y || !slice || !dy) return fill_err(err, err_len, "NULL argument");
  cudaSetDevice(ctx->c.device);
  HeadSlice hs;
  hs.col = slice->col; hs.gamma = slice->gamma; hs.rope = slice->rope; hs.rstd = slice->rstd;
  std::string e;
  if (k_head_prep_bwd(&ctx->c, g, (long)g_ld, y, T, ncols, H, hs, tps, rot, rope_base, dy, nullptr, e))
    return fill_err(err, err_len, e);
  return 0;
}

int sa3k_adamw(sa3k_ctx* ctx, float* p, const float* g, float* m, float* v, int64_t n, const sa3k_adamw_params* hp,
               int step, char* err, int err_len) {
  if (!ctx || !p || !g || !m || !v || !hp) return fill_err(err, err_len, "NULL argument");
  if (step <= 0) return fill_err(err, err_len, "AdamW step must be positive");
  cudaSetDevice(ctx->c.device);
  float b1c, b2c;
  adamw_bias_corrections(hp, step, b1c, b2c);
  std::string e;
  if (k_adamw(&ctx->c, p, g, m, v, n, hp->learning_rate, hp->beta1, hp->beta2, hp->eps, hp->weight_decay, b1c, b2c,
              nullptr, e))
    return fill_err(err, err_len, e);
  return 0;
}

int sa3k_average_clip_adamw(sa3k_ctx* ctx, float* p, const float* g, float* m, float* v, int64_t n, int count,
                            const sa3k_adamw_params* hp, int step, double* grad_norm_out, char* err, int err_len) {
  if (!ctx || !p || !g || !m || !v || !hp) return fill_err(err, err_len, "NULL argument");
  if (count <= 0) return fill_err(err, err_len, "cannot apply empty gradient batch");
  if (step <= 0) return fill_err(err, err_len, "AdamW step must be positive");
  Ctx* c = &ctx->c;
  cudaSetDevice(c->device);
  std::string e;
  // [0]: f64 sum of squares, [1]: f64 norm, then 2 floats of scales
  double* acc = static_cast<double*>(scratch_get(c, kS_OPT, 64, e));
  if (!acc) return fill_err(err, err_len, e);
  float* scales = reinterpret_cast<float*>(acc + 2);
  const float inv = count > 1 ? 1.0f / (float)count : 1.0f;
  if (cudaMemsetAsync(acc, 0, sizeof(double), c->stream) != cudaSuccess) return fill_err(err, err_len, "memset failed");
  if (k_sumsq(c, g, n, inv, acc, e) || k_clip_scale(c, acc, hp->grad_clip, inv, scales, acc + 1, e))
    return fill_err(err, err_len, e);
  float b1c, b2c;
  adamw_bias_corrections(hp, step, b1c, b2c);
  if (k_adamw(c, p, g, m, v, n, hp->learning_rate, hp->beta1, hp->beta2, hp->eps, hp->weight_decay, b1c, b2c, scales, e))
    return fill_err(err, err_len, e);
  if (grad_norm_out) {
    if (cudaMemcpyAsync(grad_norm_out, acc + 1, sizeof(double), cudaMemcpyDeviceToHost, c->stream) != cudaSuccess ||
        cudaStreamSynchronize(c->stream) != cudaSuccess)
      return fill_err(err, err_len, "failed to read the gradient norm");
  }
  return 0;
}

}  // extern "C"
