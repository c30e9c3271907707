// lora_chain.cu -- inference with a chain of functional adapters over a frozen (quantized) base:
// build_functional_lora (src/lora.h:372-622) folded on the device, and the dit_lin term path it
// feeds (src/dit.h:108-117):
//
//   y = b * (x W^T) + sum_k s_k (x A_k^T) B'_k^T + bias,   B'_k = B_k * g_k (row scale)
//
// For a chain of adapters k = 0..n-1 (lora or dora-rows, s_k = alpha_k / rank_k * strength_k),
// every dora-rows adapter j rescales the rows of the weight accumulated so far,
// V_j = b W + sum_{k<=j} s_k g_k B_k A_k, by d_j = m_j / |V_j|_row, folded into the base
// coefficient b and the residual coefficients g_k (k <= j).  The row norms need only low-rank
// quantities: nsq0 = |W|_row^2 + in eps (the base row norms), T2_k = rowdot(W A_k^T, B_k) and the
// Gram terms G_kl = rowdot(B_k (A_k A_l^T), B_l).
//
// On the device: one P = W A^T GEMM per 16 ranks of the chain, one A A^T kernel, one fold kernel
// (one thread per output row walks the chain) that writes b and the extension operand
// B'' = s_k g_k B_k / b in f16.  The forward is then the fused LoRA GEMM of the training path:
// u = x A_cat^T (rank <= 16 in all), y = b * (x W^T + u B''^T) + bias in one GEMM.  A chain of more
// than 16 ranks, or with a row where b = 0, runs the base GEMM with column scale b and adds each
// 16-rank group u_g (s g B)_g^T with one more accumulating K = 16 GEMM.
#include "../../include/sa3k.h"
#include "linear.h"
#include "lora_kernels.h"
#include "sa3k_common.cuh"

#include <algorithm>
#include <cstring>
#include <vector>

namespace sa3k {
namespace {

constexpr int kMaxTerms = 16;
constexpr int kMaxRank = 64;   // all terms of a chain together

struct ChainTermDev {
  const float* B;       // [out][rank]
  const float* m;       // [out] (dora) or null
  int col, rank;        // first column of the term in the concatenated rank space
  float s;
};

struct ChainArgs {
  ChainTermDev t[kMaxTerms];
  int n, R, groups;
  int any_dora;
  int fused;            // B'' is divided by b (extension inside the base GEMM)
};

// A_cat A_cat^T [R][R] in f32 (one block per entry, a block-wide dot over `in`)
__global__ void aat_cat_kernel(const float* __restrict__ A, int R, int64_t in, float* __restrict__ aat) {
  const int r = blockIdx.x / R, c = blockIdx.x % R;
  float acc = 0.f;
  for (int64_t i = threadIdx.x; i < in; i += blockDim.x) acc = fmaf(A[(int64_t)r * in + i], A[(int64_t)c * in + i], acc);
  __shared__ float red[8];
  acc = warp_sum(acc);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x == 0) {
    float s = 0.f;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) s += red[w];
    aat[r * R + c] = s;
  }
}

// One thread per output row o: the chain walk of build_functional_lora (src/lora.h:531-554), then
// b[o] and B''[group][o][64] (columns of the group's 16 ranks; the rest zero).
__global__ void chain_fold_kernel(const __grid_constant__ ChainArgs a, const float* __restrict__ pt,
                                  const float* __restrict__ aat, const float* __restrict__ nsq0, int64_t out,
                                  float* __restrict__ bsc, __half* __restrict__ bx, int* __restrict__ zero_rows) {
  const int64_t o = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (o >= out) return;
  const int n = a.n, R = a.R;
  float bv[kMaxRank];
  for (int k = 0; k < n; ++k)
    for (int r = 0; r < a.t[k].rank; ++r) bv[a.t[k].col + r] = a.t[k].B[o * a.t[k].rank + r];
  float t2[kMaxTerms], g[kMaxTerms];
  if (a.any_dora) {
    for (int k = 0; k < n; ++k) {
      float s = 0.f;
      for (int r = 0; r < a.t[k].rank; ++r) s = fmaf(pt[(int64_t)(a.t[k].col + r) * out + o], bv[a.t[k].col + r], s);
      t2[k] = s;
    }
  }
  // G_kl = sum_{r in k, c in l} B_k[o][r] (A A^T)[r][c] B_l[o][c]
  auto gram = [&](int k, int l) {
    float s = 0.f;
    for (int r = 0; r < a.t[k].rank; ++r) {
      float q = 0.f;
      for (int c = 0; c < a.t[l].rank; ++c) q = fmaf(aat[(a.t[k].col + r) * R + a.t[l].col + c], bv[a.t[l].col + c], q);
      s = fmaf(bv[a.t[k].col + r], q, s);
    }
    return s;
  };
  float b = 1.f;
  bool has_b = false;
  for (int k = 0; k < n; ++k) g[k] = 1.f;
  for (int j = 0; j < n; ++j) {
    if (!a.t[j].m) continue;
    float nsq = has_b ? nsq0[o] * b * b : nsq0[o];
    for (int k = 0; k <= j; ++k) nsq += t2[k] * g[k] * 2.f * a.t[k].s * (has_b ? b : 1.f);
    for (int k = 0; k <= j; ++k)
      for (int l = k; l <= j; ++l) nsq += gram(k, l) * g[k] * g[l] * a.t[k].s * a.t[l].s * (k == l ? 1.f : 2.f);
    const float d = a.t[j].m[o] / sqrtf(nsq);
    b = has_b ? b * d : d;
    has_b = true;
    for (int k = 0; k <= j; ++k) g[k] *= d;
  }
  if (a.any_dora) {
    bsc[o] = b;
    if (b == 0.f) atomicAdd(zero_rows, 1);
  }
  const float inv = a.fused && has_b && b != 0.f ? 1.f / b : 1.f;
  for (int gi = 0; gi < a.groups; ++gi)
    for (int c = 0; c < 64; ++c) {
      const int idx = gi * 16 + c;
      float v = 0.f;
      if (c < 16 && idx < R)
        for (int k = 0; k < n; ++k)
          if (idx >= a.t[k].col && idx < a.t[k].col + a.t[k].rank) v = a.t[k].s * g[k] * bv[idx] * inv;
      bx[((int64_t)gi * out + o) * 64 + c] = __float2half_rn(v);
    }
}

}  // namespace

struct LoraChain {
  int R = 0, groups = 0, n = 0;
  bool any_dora = false, fused = false;
  int64_t in = 0, out = 0;
  __half* a_h = nullptr;   // [16 groups][in] f16 (A_cat, zero rows past R)
  __half* bx = nullptr;     // [groups][out][64] f16 (s g B, / b when fused)
  float* bsc = nullptr;            // [out] base scale b (any dora)
  void* mem = nullptr;
  ~LoraChain() {
    if (mem) cudaFree(mem);
  }
};

static int chain_build(Ctx* c, const Weight* w, const sa3k_chain_term* terms, int n, LoraChain& ch, std::string& err) {
  if (n < 1 || n > kMaxTerms) { err = "a chain holds 1 to 16 adapters"; return 1; }
  const int64_t in = w->in, out = w->out;
  ChainArgs a{};
  int R = 0;
  bool any_dora = false;
  for (int k = 0; k < n; ++k) {
    const sa3k_chain_term& t = terms[k];
    if (!t.A || !t.B || t.rank < 1) { err = "chain term needs A, B and rank >= 1"; return 1; }
    a.t[k] = ChainTermDev{t.B, t.magnitude, R, t.rank, t.scale};
    R += t.rank;
    any_dora = any_dora || t.magnitude;
  }
  if (R > kMaxRank) { err = "a chain holds at most 64 ranks in all"; return 1; }
  if (in % 64) { err = "in must be a multiple of 64"; return 1; }
  const int groups = (R + 15) / 16;
  a.n = n; a.R = R; a.groups = groups; a.any_dora = any_dora ? 1 : 0;
  ch.R = R; ch.groups = groups; ch.n = n; ch.any_dora = any_dora; ch.in = in; ch.out = out;
  // device memory: a_h, bx, bsc, A_cat f32, P^T f32, A A^T, nsq0, the zero-row counter
  auto al = [](size_t b) { return (b + 255) & ~(size_t)255; };
  const size_t b_abf = al((size_t)16 * groups * in * 2), b_bx = al((size_t)groups * out * 64 * 2), b_bsc = al(out * 4);
  const size_t b_acat = al((size_t)R * in * 4), b_pt = al((size_t)16 * groups * out * 4), b_aat = al((size_t)R * R * 4);
  const size_t b_nsq = al(out * 4), b_cnt = 256;
  if (cudaMalloc(&ch.mem, b_abf + b_bx + b_bsc + b_acat + b_pt + b_aat + b_nsq + b_cnt) != cudaSuccess) {
    cudaGetLastError();
    err = "out of device memory for the adapter chain";
    return 1;
  }
  char* q = static_cast<char*>(ch.mem);
  ch.a_h = reinterpret_cast<__half*>(q); q += b_abf;
  ch.bx = reinterpret_cast<__half*>(q); q += b_bx;
  ch.bsc = reinterpret_cast<float*>(q); q += b_bsc;
  float* acat = reinterpret_cast<float*>(q); q += b_acat;
  float* pt = reinterpret_cast<float*>(q); q += b_pt;
  float* aat = reinterpret_cast<float*>(q); q += b_aat;
  float* nsq0 = reinterpret_cast<float*>(q); q += b_nsq;
  int* zero_rows = reinterpret_cast<int*>(q);
  cudaStream_t st = c->stream;
  if (cudaMemsetAsync(ch.a_h, 0, b_abf, st) != cudaSuccess || cudaMemsetAsync(zero_rows, 0, sizeof(int), st) != cudaSuccess)
    return check_launch("memset", err);
  for (int k = 0; k < n; ++k)
    if (cudaMemcpyAsync(acat + (int64_t)a.t[k].col * in, terms[k].A, sizeof(float) * terms[k].rank * in,
                        cudaMemcpyDeviceToDevice, st) != cudaSuccess)
      return check_launch("copy", err);
  if (k_cvt_f16(c, acat, (int64_t)R * in, ch.a_h, err)) return 1;
  if (any_dora) {
    if (weight_row_norms(c, w, 1e-12f, nsq0, nullptr, err)) return 1;   // |W|_row^2 + in eps
    for (int gi = 0; gi < groups; ++gi) {   // P^T rows of group gi = (W A_g^T)^T
      AdapterPrep p;
      p.in = in; p.out = out; p.rank = 16;
      p.a_h = ch.a_h + (int64_t)gi * 16 * in;
      p.pt = pt + (int64_t)gi * 16 * out;
      if (adapter_dora_p(c, w, p, err)) return 1;
    }
    aat_cat_kernel<<<(unsigned)(R * R), 256, 0, st>>>(acat, R, in, aat);
    if (check_launch("chain A A^T", err)) return 1;
  }
  // fused unless the chain is wider than one extension or some base scale is 0 (known after the
  // fold: fold once for the group path first, check, fold again divided by b)
  a.fused = 0;
  chain_fold_kernel<<<(unsigned)((out + 127) / 128), 128, 0, st>>>(a, pt, aat, nsq0, out, ch.bsc, ch.bx, zero_rows);
  if (check_launch("chain fold", err)) return 1;
  int zr = 0;
  if (cudaMemcpyAsync(&zr, zero_rows, sizeof(int), cudaMemcpyDeviceToHost, st) != cudaSuccess ||
      cudaStreamSynchronize(st) != cudaSuccess)
    return check_launch("chain fold", err);
  ch.fused = groups == 1 && zr == 0;
  if (ch.fused && any_dora) {
    a.fused = 1;
    chain_fold_kernel<<<(unsigned)((out + 127) / 128), 128, 0, st>>>(a, pt, aat, nsq0, out, ch.bsc, ch.bx, zero_rows);
    if (check_launch("chain fold", err)) return 1;
  }
  return 0;
}

static int chain_forward(Ctx* c, const Weight* w, const LoraChain& ch, const float* bias, const __half* x_h,
                         int64_t M, float* y, __half* u_buf, int64_t u_ld, std::string& err) {
  if (ch.fused) {
    AdapterPrep p;   // the training path's fused forward with the chain's operands
    p.in = ch.in; p.out = ch.out; p.rank = 16; p.s = 1.f;
    p.a_h = ch.a_h;
    p.b_x = ch.bx;
    if (lora_u(c, x_h, M, ch.in, p, u_buf, u_ld, err)) return 1;
    GemmDesc g;
    g.M = (int)M; g.N = (int)ch.out; g.K = (int)ch.in;
    g.a = x_h; g.lda = ch.in;
    g.bsrc = kB_WEIGHT_NT; g.w = w;
    g.ext_at = u_buf; g.ld_ext = u_ld; g.ext_b = ch.bx;
    g.col_scale = ch.any_dora ? ch.bsc : nullptr;
    g.col_bias = bias;
    g.out = y; g.ldo = ch.out;
    g.name = "linear.fwd";
    return gemm(c, g, err);
  }
  // u_all = x A_cat^T [M][16 groups] (row-major), base GEMM, one K = 16 GEMM per group
  const int RP = 16 * ch.groups;
  {
    GemmDesc g;
    g.M = (int)M; g.N = RP; g.K = (int)ch.in;
    g.a = x_h; g.lda = ch.in;
    g.bsrc = kB_F16_KMAJOR; g.b = ch.a_h; g.ldb = ch.in;
    g.out_h = u_buf; g.ldo_h = RP;
    g.bn = 16;
    g.name = "lora.u";
    if (gemm(c, g, err)) return 1;
  }
  {
    GemmDesc g;
    g.M = (int)M; g.N = (int)ch.out; g.K = (int)ch.in;
    g.a = x_h; g.lda = ch.in;
    g.bsrc = kB_WEIGHT_NT; g.w = w;
    g.col_scale = ch.any_dora ? ch.bsc : nullptr;
    g.col_bias = bias;
    g.out = y; g.ldo = ch.out;
    g.name = "linear.fwd";
    if (gemm(c, g, err)) return 1;
  }
  for (int gi = 0; gi < ch.groups; ++gi) {
    GemmDesc g;
    g.M = (int)M; g.N = (int)ch.out; g.K = 16;
    g.a = u_buf + 16 * gi; g.lda = RP;
    g.bsrc = kB_F16_KMAJOR; g.b = ch.bx + (int64_t)gi * ch.out * 64; g.ldb = 64;
    g.out = y; g.ldo = ch.out; g.accumulate = 1;
    g.name = "lora.chain";
    if (gemm(c, g, err)) return 1;
  }
  return 0;
}

}  // namespace sa3k

using namespace sa3k;

struct sa3k_lora_chain {
  LoraChain ch;
  const sa3k_weight* w = nullptr;
};

static int lfail(char* err, int len, const std::string& msg) {
  if (err && len > 0) {
    std::strncpy(err, msg.c_str(), (size_t)len - 1);
    err[len - 1] = 0;
  }
  return 1;
}

extern "C" {

int sa3k_lora_chain_build(sa3k_ctx* ctx, const sa3k_weight* w, const sa3k_chain_term* terms, int n,
                          sa3k_lora_chain** out, char* err, int err_len) {
  if (!ctx || !w || !terms || !out) return lfail(err, err_len, "NULL argument");
  cudaSetDevice(ctx->c.device);
  sa3k_lora_chain* h = new (std::nothrow) sa3k_lora_chain();
  if (!h) return lfail(err, err_len, "out of host memory");
  h->w = w;
  std::string e;
  if (chain_build(&ctx->c, &w->w, terms, n, h->ch, e)) {
    delete h;
    return lfail(err, err_len, e);
  }
  *out = h;
  return 0;
}

void sa3k_lora_chain_free(sa3k_lora_chain* chain) { delete chain; }

int sa3k_lora_chain_info(const sa3k_lora_chain* chain, int* total_rank, int* fused) {
  if (!chain) return 1;
  if (total_rank) *total_rank = chain->ch.R;
  if (fused) *fused = chain->ch.fused ? 1 : 0;
  return 0;
}

int sa3k_linear_fwd_chain(sa3k_ctx* ctx, const sa3k_weight* w, const sa3k_lora_chain* chain, const float* bias,
                          const float* x, int64_t S, float* y, char* err, int err_len) {
  if (!ctx || !w || !chain || !x || !y) return lfail(err, err_len, "NULL argument");
  if (chain->w != w) return lfail(err, err_len, "the chain was built for another weight");
  if (S <= 0) return lfail(err, err_len, "S must be positive");
  Ctx* c = &ctx->c;
  cudaSetDevice(c->device);
  std::string e;
  const int64_t in = w->w.in, s_pad = (S + 63) / 64 * 64;
  __half* x_h = static_cast<__half*>(scratch_get(c, kSlotChainX, sizeof(__half) * S * in, e));
  __half* u = x_h ? static_cast<__half*>(scratch_get(c, kSlotChainU, sizeof(__half) * 64 * s_pad, e))
                          : nullptr;
  if (!x_h || !u) return lfail(err, err_len, e);
  if (k_cvt_f16(c, x, S * in, x_h, e)) return lfail(err, err_len, e);
  if (chain_forward(c, &w->w, chain->ch, bias, x_h, S, y, u, chain->ch.fused ? s_pad : 16 * chain->ch.groups, e))
    return lfail(err, err_len, e);
  return 0;
}

}  // extern "C"
