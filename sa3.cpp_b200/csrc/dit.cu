// dit.cu -- the DiT adapter-training step on one GPU: forward through the frozen (quantized)
// DiT with functional LoRA / DoRA-rows adapters, MSE v-objective loss, full backward to the
// adapter gradients, and the averaged + clipped AdamW update.
//
// Reference: dit_head / dit_block / dit_tail (src/dit.h:164-323) built into training graphs by
// build_train_dit_ckpt (src/train_ckpt.h:143-474) and run per sample by
// run_train_dit_accumulate_ckpt (src/train_loop.h:309-441); the update is
// train_apply_accumulated_adamw (src/train_loop.h:173-211).
//
// Differences of execution (not of math):
//  * a batch of B samples runs as one pass: every linear sees M = B * (mem + T) token rows, the
//    per-sample pieces (adaLN vectors, attention, positions, loss) are indexed by sample; the
//    adapter gradients are the sum over samples, as the reference's host accumulation.
//  * all activations stay resident in HBM (about 0.6 GB per block at batch 4, medium width), so
//    the backward does not recompute the forward; the reference's checkpointed VJP
//    (src/train_ckpt.h:12-18) is the same gradient.
//  * adapters live in one flat f32 buffer [A | B | m] per target, gradients and moments alike;
//    the A/B operand packing and the DoRA norms are prepared once per step.
//  * any 2-D DiT weight can carry an adapter (the reference's `full` and `core` scopes,
//    src/train_lora.h:54-95): the per-block projections, and the head / tail linears; the
//    gradient reaches the head through x0, the context and gcond as in the reference's head VJP
//    (src/train_ckpt.h:440-470), and those backward pieces run only when a target needs them.
#include "../../include/sa3k.h"
#include "attention.h"
#include "gemm_r16.h"
#include "gguf_io.h"
#include "linear.h"
#include "lora_kernels.h"
#include "materialize.h"

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <sys/stat.h>
#include <string>
#include <vector>

namespace sa3k {

struct DitTarget {
  std::string name;
  const Weight* w = nullptr;
  int64_t in = 0, out = 0;
  int64_t offA = 0, offB = 0, offM = -1;   // into the flat adapter state
  float* bns = nullptr;                    // [out]
  AdapterPrep prep;
  // rows: the token rows this linear sees in a step (B (mem + T), B ctx, B T or B); ut_ld their
  // pitch rounded up to 64.  The forward keeps u^T [16][ut_ld] f16 in ut; the step's inputs of
  // the grouped adapter-gradient pass (activation arena): dz [rows][out] f16, dg [out], du^T
  // [16][ut_ld] f16, cb [16][out] f16 (dora), c3 [16][16]; and the forward's input rows x_h
  int64_t rows = 0, ut_ld = 0;
  // inert: an adapter on a weight the step never computes with (the inpaint local.* projections
  // without a local-conditioning input): carried with zero gradients, left out of every
  // per-step adapter kernel; act = the index among the other (active) targets
  bool inert = false;
  int act = -1;
  __half *ut = nullptr, *dz = nullptr, *dut = nullptr, *cb = nullptr;
  float *dg = nullptr, *c3 = nullptr;
  const __half* x_h = nullptr;
  // materialized families (dora-cols, bora, every -xs form): W_eff built once per step, the
  // forward and dX GEMMs on it, the weight gradient per backward (outside the functional
  // adapters' grouped preparation and gradient passes).  offMc: the bora column magnitude;
  // offX: M_xs; U [out][rank] / Vb [in][rank]: the frozen -xs bases (device)
  bool mat = false;
  MatTarget mt;
  int64_t offMc = -1, offX = -1;
  float *U = nullptr, *Vb = nullptr;
};

struct DitBlockAct {
  float *x = nullptr, *rstd_a = nullptr, *rq = nullptr, *rk = nullptr, *lse_a = nullptr;
  __half* qkv = nullptr;   // qkv projection output, f16 (read by the head preparation and its backward)
  float *yo = nullptr, *x1 = nullptr, *rstd_c = nullptr, *qf = nullptr, *rcq = nullptr, *kvf = nullptr;
  float *rck = nullptr, *lse_c = nullptr, *x2 = nullptr, *rstd_f = nullptr, *yf = nullptr;
  __half* ff = nullptr;   // ff.proj output [val | gate], f16 (read by the SwiGLU forward and backward)
  float* mod = nullptr;
  __half *h_a = nullptr, *qkvb = nullptr, *oa = nullptr, *hc = nullptr, *cq = nullptr, *kvb = nullptr;
  __half *oc = nullptr, *hf = nullptr, *act = nullptr;
  // differential attention: both softmax streams' outputs (oa = o1 - o2, oc = oc1 - oc2), the
  // second stream's log-sum-exp and the rstd of its q / k heads (null otherwise)
  __half *o1 = nullptr, *o2 = nullptr, *oc1 = nullptr, *oc2 = nullptr;
  float *lse_a2 = nullptr, *lse_c2 = nullptr, *rq2 = nullptr, *rk2 = nullptr, *rcq2 = nullptr, *rck2 = nullptr;
  float* yc = nullptr;   // cross.out output, kept when that linear has an adapter
  int64_t kv_ld = 0;     // row stride of kvf / kvb (depth x their width when the blocks share them)
};

struct DitModel {
  Ctx* c = nullptr;
  sa3k_ctx* handle = nullptr;
  int device = 0;
  sa3k_dit_config cfg{};
  std::map<std::string, Weight*> W;
  std::vector<sa3k_weight*> weights;   // owned weight handles (W points into them)
  std::map<std::string, float*> V;
  // weights kept on the host only: inpaint local.* projections whose `in` the GEMM engine does
  // not tile (dit.local_dim = 257); [out][in] f32 with their (in, out)
  std::map<std::string, std::vector<float>> host_w;
  std::map<std::string, std::pair<int64_t, int64_t>> host_shape;
  // the same weights zero-padded to a multiple of 64 in `in` on the device: the inpaint local.0
  // projection of the local-conditioning input, run by the GEMM engine (name -> padded weight)
  std::map<std::string, Weight*> Wpad;
  // inpaint: the current call carries a local-conditioning input and loss weights
  // (sa3k_dit_forward_backward_inpaint); local_ld = dit.local_dim rounded up to 64
  bool inpaint = false;
  int64_t local_ld = 0;
  float *in_local = nullptr, *in_lw = nullptr, *lmid = nullptr;
  __half *local_h = nullptr, *lmid_h = nullptr;
  std::vector<void*> owned;            // device allocations of this model
  // adapters
  bool dora = false;
  bool mat = false;                    // a materialized family (every target is a DitTarget::mat)
  std::string adapter_type = "lora";
  float* mat_G = nullptr;              // [max out*in] f32 weight-gradient scratch (materialized)
  __half* mat_dzt = nullptr;    // [max out][mat_ldt] f16 transposed output gradient
  __half* mat_dD = nullptr;     // [max out*in] f16 dD of the normalisation backward
  int64_t mat_ldt = 0;
  int rank = 0;
  float alpha = 1.f, s = 1.f;
  std::vector<DitTarget> tg;
  std::map<std::string, int> tix;
  float *p = nullptr, *g = nullptr, *am = nullptr, *av = nullptr;
  int64_t np = 0;
  void* prep_mem = nullptr;
  PrepDesc* prep_desc = nullptr;       // device descriptors of the active adapters (grouped preparation)
  int n_active = 0;
  int64_t max_out = 0;
  // grouped rank-16 GEMMs: DoRA P = W A^T of every adapter (forward preparation) and every
  // adapter's dB / dA contractions (end of the backward); bound to the activation arena
  R16Group r16_prep, r16_grads;
  float* c3_all = nullptr;
  // activations for shape (B, T, C)
  int B = 0, T = 0, C = 0;
  void* arena = nullptr;
  size_t arena_bytes = 0;
  std::vector<DitBlockAct> blk;
  float* x_final = nullptr;
  // inputs
  float *in_x = nullptr, *in_target = nullptr, *in_tfeat = nullptr, *in_cross = nullptr, *in_glob = nullptr;
  // head
  float *te_h = nullptr, *te = nullptr, *g_h = nullptr, *gsum = nullptr, *gce_h = nullptr, *gcond = nullptr;
  float *ctx_h = nullptr, *pre = nullptr, *xin0 = nullptr;
  __half *tfeat_b = nullptr, *te_hb = nullptr, *glob_b = nullptr, *g_hb = nullptr, *gsum_b = nullptr;
  __half *gce_hb = nullptr, *cross_b = nullptr, *ctx_hb = nullptr, *context_b = nullptr, *xt_b = nullptr;
  __half* xp_b = nullptr;
  // tail
  __half *xT_b = nullptr, *pout_b = nullptr;
  float *pout = nullptr, *vel = nullptr, *dvel = nullptr, *loss = nullptr, *dp = nullptr, *dxT = nullptr;
  // backward temporaries
  float *gx = nullptr, *dtmp = nullptr, *dh = nullptr, *dq3 = nullptr, *Dsum = nullptr;
  float* dv2 = nullptr;   // differential: dV of the second softmax stream (run on +dO)
  // forward outputs kept for the backward of head / tail adapters (linear output without the
  // residual it is added to)
  float *pre_lin = nullptr, *vel_lin = nullptr, *g_y = nullptr, *ctx_y = nullptr;
  // backward buffers of the optional pieces: cross q gradient (adapted cross.q), cross k / v
  // gradients and the context gradient (adapted cross.kv or cond_embed), gcond and gsum
  // gradients (adapted gce / time_embed / global_embed), x0 rows (adapted proj_in / pre_conv)
  float *dqf = nullptr, *dkv = nullptr, *dkvf = nullptr, *dvc2 = nullptr, *dctx = nullptr, *dmlp = nullptr;
  float *dgcond = nullptr, *dgsum = nullptr, *dxin0 = nullptr, *dxp = nullptr;
  bool need_ctx = false, need_mod = false, need_x0 = false;
  __half *dO_b = nullptr, *dact_b = nullptr;   // dact_b: the SwiGLU output gradient, f16
  // the context K / V projections of every block as one GEMM (no adapter on any cross.kv, nothing
  // differentiated through them): the blocks' f16 weights stacked [depth x Dk][dim], refilled when
  // the model generation changes; the outputs kvf_all (f32) / kvb_all (prepared, f16) are
  // [MC][depth x Dk], block l at column l Dk
  bool kv_batched = false;
  __half* kv_w_all = nullptr;
  // every block's ssg vector stacked [depth][6 dim] (refilled with the stacked K / V weights), so
  // one launch forms all blocks' adaLN vectors into mod_all [depth][B][6 dim]
  float* ssg_all = nullptr;
  uint64_t ssg_mgen = ~0ull;
  float* mod_all = nullptr;
  // with the batched context K / V and no differential streams, their head preparation is one
  // launch too: the blocks' cross.k_norm gammas stacked [depth][64] (refilled with ssg_all), the
  // blocks' rstd of the context keys contiguous in rck_all [depth][MC][H]
  bool kvp_batched = false;
  float* gck_all = nullptr;
  float* rck_all = nullptr;
  uint64_t kvw_mgen = ~0ull;
  float* kvf_all = nullptr;
  __half* kvb_all = nullptr;
  // linear scratch
  float *dg = nullptr, *c3 = nullptr;
  __half *dut = nullptr, *dz = nullptr, *cb = nullptr;
  int64_t ut_ld = 0;

  // the step recorded as a CUDA graph (SA3K_OPT_STEP_GRAPH): valid for shape (gB, gT, gC) while
  // the context generation is g_cgen and the model generation g_mgen; launch counts per profile
  // class of one replay (so the context's launch counters stay true)
  uint64_t gen = 0;                                 // bumped by set_tensor / init_adapters
  cudaGraphExec_t step_exec = nullptr;
  int gB = 0, gT = 0, gC = 0;
  uint64_t g_cgen = 0, g_mgen = 0;
  std::vector<std::pair<std::string, long long>> g_launches;
  cudaStream_t cap_stream = nullptr;                // private stream the graph is recorded on
  bool warm = false;                                // one eager call at the current key done
  int wB = 0, wT = 0, wC = 0;
  uint64_t w_cgen = 0, w_mgen = 0;

  ~DitModel() {
    if (step_exec) cudaGraphExecDestroy(step_exec);
    if (cap_stream) cudaStreamDestroy(cap_stream);
    r16_group_free(r16_prep);
    r16_group_free(r16_grads);
    for (void* q : owned) cudaFree(q);
    if (arena) cudaFree(arena);
    for (sa3k_weight* h : weights) sa3k_weight_free(h);
  }

  int Sfull() const { return cfg.mem_tokens + T; }
  int qkv_cols() const { return (cfg.differential ? 5 : 3) * cfg.dim; }
  int cq_cols() const { return (cfg.differential ? 2 : 1) * cfg.dim; }    // cross.q output
  int ckv_cols() const { return (cfg.differential ? 3 : 2) * cfg.dim; }   // cross.kv output
  std::string bname(int l, const char* suffix) const { return "dit." + std::to_string(l) + "." + suffix; }
  const Weight* weight(const std::string& n, std::string& err) const {
    auto it = W.find(n);
    if (it == W.end()) { err = "missing weight " + n; return nullptr; }
    return it->second;
  }
  const float* vec(const std::string& n, std::string& err) const {
    auto it = V.find(n);
    if (it == V.end()) { err = "missing tensor " + n; return nullptr; }
    return it->second;
  }
};

static void* dmalloc(DitModel& m, size_t bytes, std::string& err) {
  void* q = nullptr;
  if (cudaMalloc(&q, bytes) != cudaSuccess) {
    cudaGetLastError();
    err = "out of device memory";
    return nullptr;
  }
  m.owned.push_back(q);
  return q;
}

// ------------------------------------------------------------------ grouped adapter passes
// After the activation arena moved: bind every adapter to its block's input rows and u^T, refresh
// the device descriptors (now with the gradient pointers), and build the grouped rank-16 GEMMs
// of the DoRA preparation and of the adapter gradients.
// The linear a weight name belongs to: its f16 input rows in the activation arena (null for a
// name that is not a linear of the DiT) and how many rows it sees per step.
static int64_t target_rows(const DitModel& m, const std::string& n) {
  const int64_t B = m.B;
  if (n.compare(0, 4, "dit.") == 0 && n.size() > 4 && n[4] >= '0' && n[4] <= '9')
    return n.find(".cross.kv.") != std::string::npos ? B * m.C : B * m.Sfull();
  if (n.find("time_embed.") != std::string::npos || n.find("global_embed.") != std::string::npos ||
      n.find(".gce.") != std::string::npos)
    return B;
  if (n.find("cond_embed.") != std::string::npos) return B * m.C;
  return B * m.T;   // pre_conv, proj_in, proj_out, post_conv
}

static const __half* target_input(const DitModel& m, const std::string& n) {
  if (n.compare(0, 4, "dit.") != 0) return nullptr;
  const std::string r = n.substr(4);
  if (!r.empty() && r[0] >= '0' && r[0] <= '9') {
    const size_t dot = r.find('.');
    const long l = std::strtol(r.substr(0, dot).c_str(), nullptr, 10);
    if (dot == std::string::npos || l < 0 || l >= m.cfg.depth) return nullptr;
    const DitBlockAct& a = m.blk[(size_t)l];
    const std::string k = r.substr(dot + 1);
    if (k == "self.qkv.weight") return a.h_a;
    if (k == "self.out.weight") return a.oa;
    if (k == "cross.q.weight") return a.hc;
    if (k == "cross.kv.weight") return m.context_b;
    if (k == "cross.out.weight") return a.oc;
    if (k == "ff.proj.weight") return a.hf;
    if (k == "ff.out.weight") return a.act;
    return nullptr;
  }
  static const struct { const char* name; __half* DitModel::*x; } kHead[] = {
      {"time_embed.0.weight", &DitModel::tfeat_b}, {"time_embed.2.weight", &DitModel::te_hb},
      {"global_embed.0.weight", &DitModel::glob_b}, {"global_embed.2.weight", &DitModel::g_hb},
      {"gce.0.weight", &DitModel::gsum_b},          {"gce.2.weight", &DitModel::gce_hb},
      {"cond_embed.0.weight", &DitModel::cross_b},  {"cond_embed.2.weight", &DitModel::ctx_hb},
      {"pre_conv.weight", &DitModel::xt_b},         {"proj_in.weight", &DitModel::xp_b},
      {"proj_out.weight", &DitModel::xT_b},         {"post_conv.weight", &DitModel::pout_b}};
  for (const auto& h : kHead)
    if (r == h.name) return m.*(h.x);
  return nullptr;
}

static bool has_target(const DitModel& m, const char* fragment) {
  for (const DitTarget& t : m.tg)
    if (t.name.find(fragment) != std::string::npos) return true;
  return false;
}

static int bind_adapter_grads(DitModel& m, std::string& err) {
  for (DitTarget& t : m.tg) {
    if (t.inert) continue;
    t.x_h = target_input(m, t.name);
    if (!t.x_h) {
      err = "adapter target " + t.name + " is not a linear of the DiT";
      return 1;
    }
  }
  std::vector<PrepDesc> descs;
  std::vector<R16Job> prep, grads;
  for (DitTarget& t : m.tg) {
    if (t.inert || t.mat) continue;
    const AdapterPrep& p = t.prep;
    PrepDesc pd{};
    pd.A = p.A; pd.B = p.B; pd.m = p.m; pd.bns = p.bns;
    pd.rank = p.rank; pd.dora = p.dora() ? 1 : 0; pd.s = p.s; pd.in = p.in; pd.out = p.out;
    pd.a_h = p.a_h; pd.at_x = p.at_x; pd.b_x = p.b_x; pd.bt_h = p.bt_h;
    pd.pt = p.pt; pd.aat = p.aat; pd.nsq = p.nsq; pd.g = p.g;
    pd.dg = t.dg; pd.dB = m.g + t.offB; pd.dA = m.g + t.offA; pd.dm = t.offM >= 0 ? m.g + t.offM : nullptr;
    pd.cb = t.cb; pd.c3 = t.c3;
    descs.push_back(pd);
    const int64_t M = t.rows;
    R16Job j;
    // dB [out][rank] += s dz^T u     (A = dz read MN-major, K = the M token rows)
    j = R16Job();
    j.a = t.dz; j.lda = t.out; j.a_mn = 1; j.M = (int)t.out; j.N = p.rank; j.K = (int)M;
    j.b = t.ut; j.ldb = t.ut_ld; j.alpha = p.s;
    j.out = m.g + t.offB; j.ldo = p.rank; j.atomic = 1;
    grads.push_back(j);
    // dA [rank][in] += du^T x        (A = x read MN-major, stored transposed)
    j = R16Job();
    j.a = t.x_h; j.lda = t.in; j.a_mn = 1; j.M = (int)t.in; j.N = p.rank; j.K = (int)M;
    j.b = t.dut; j.ldb = t.ut_ld;
    j.out = m.g + t.offA; j.ldo = t.in; j.out_trans = 1; j.atomic = 1;
    grads.push_back(j);
    if (p.dora() && t.w->f16) {
      // dA += (dt2 B)^T W             (A = the f16 base copy read MN-major, K = out)
      j = R16Job();
      j.a = t.w->f16; j.lda = t.in; j.a_mn = 1; j.M = (int)t.in; j.N = p.rank; j.K = (int)t.out;
      j.b = t.cb; j.ldb = t.out;
      j.out = m.g + t.offA; j.ldo = t.in; j.out_trans = 1; j.atomic = 1;
      grads.push_back(j);
      // P^T [16][out] = (W A^T)^T
      j = R16Job();
      j.a = t.w->f16; j.lda = t.in; j.a_mn = 0; j.M = (int)t.out; j.N = 16; j.K = (int)t.in;
      j.b = p.a_h; j.ldb = t.in;
      j.out = p.pt; j.ldo = t.out; j.out_trans = 1; j.atomic = 0;
      prep.push_back(j);
    }
  }
  if (!descs.empty() &&
      cudaMemcpy(m.prep_desc, descs.data(), sizeof(PrepDesc) * descs.size(), cudaMemcpyHostToDevice) != cudaSuccess) {
    err = "adapter descriptor upload failed";
    return 1;
  }
  // every DoRA base needs its f16 copy for the grouped P and dA terms (else the per-adapter
  // GEMMs over the quantized codes run instead)
  bool all_f16 = true;
  for (DitTarget& t : m.tg) all_f16 = all_f16 && (t.inert || t.mat || !t.prep.dora() || t.w->f16);
  r16_group_free(m.r16_prep);
  r16_group_free(m.r16_grads);
  if (!all_f16 || grads.empty()) return 0;
  if (!prep.empty() && r16_group_build(m.c, prep, 24, m.r16_prep, err)) return 1;
  return r16_group_build(m.c, grads, 24, m.r16_grads, err);
}

// ------------------------------------------------------------------ activation arena
static int alloc_acts(DitModel& m, int B, int T, int C, std::string& err) {
  if (m.arena && m.B == B && m.T == T && m.C == C) return 0;
  if (m.arena) { cudaStreamSynchronize(m.c->stream); cudaFree(m.arena); m.arena = nullptr; }
  const sa3k_dit_config& k = m.cfg;
  m.B = B; m.T = T; m.C = C;
  const int64_t S = m.Sfull(), M = (int64_t)B * S, D = k.dim, Hh = k.heads, I = k.ff_inner;
  const int64_t Q = m.qkv_cols(), MC = (int64_t)B * C, MT = (int64_t)B * T;
  const int64_t Dq = m.cq_cols(), Dk = m.ckv_cols();
  const bool diff = k.differential != 0;
  const int64_t Mx = std::max(M, MC);
  m.ut_ld = (Mx + 63) / 64 * 64;
  m.need_ctx = has_target(m, "cond_embed.");
  m.need_mod = has_target(m, "time_embed.") || has_target(m, "global_embed.") || has_target(m, ".gce.");
  m.need_x0 = has_target(m, "pre_conv.") || has_target(m, "proj_in.");
  const bool any_cq = has_target(m, ".cross.q."), need_kv = m.need_ctx || has_target(m, ".cross.kv.");
  m.kv_batched = !need_kv && k.depth > 1;
  const int64_t kv_ld = m.kv_batched ? (int64_t)k.depth * Dk : Dk;
  // two passes: measure, then carve
  for (int pass = 0; pass < 2; ++pass) {
    char* base = static_cast<char*>(m.arena);
    size_t off = 0;
    auto take = [&](size_t bytes) -> void* {
      void* r = pass ? base + off : nullptr;
      off += (bytes + 255) & ~(size_t)255;
      return r;
    };
    auto f = [&](int64_t n) { return static_cast<float*>(take(n * 4)); };
    auto h = [&](int64_t n) { return static_cast<__half*>(take(n * 2)); };
    m.kvf_all = m.kv_batched ? f(MC * kv_ld) : nullptr;
    m.mod_all = f((int64_t)k.depth * B * 6 * D);
    m.kvp_batched = m.kv_batched && !diff;
    m.rck_all = m.kvp_batched ? f((int64_t)k.depth * MC * Hh) : nullptr;
    m.kvb_all = m.kv_batched ? h(MC * kv_ld) : nullptr;
    m.blk.assign(k.depth, DitBlockAct{});
    for (int l = 0; l < k.depth; ++l) {
      DitBlockAct& a = m.blk[l];
      a.x = f(M * D); a.rstd_a = f(M); a.h_a = h(M * D); a.qkv = h(M * Q); a.qkvb = h(M * Q);
      a.rq = f(M * Hh); a.rk = f(M * Hh); a.oa = h(M * D); a.lse_a = f(B * Hh * S); a.yo = f(M * D);
      a.x1 = f(M * D); a.rstd_c = f(M); a.hc = h(M * D); a.qf = f(M * Dq); a.cq = h(M * Dq); a.rcq = f(M * Hh);
      if (m.kv_batched) {
        a.kvf = m.kvf_all ? m.kvf_all + l * Dk : nullptr;
        a.kvb = m.kvb_all ? m.kvb_all + l * Dk : nullptr;
      } else {
        a.kvf = f(MC * Dk); a.kvb = h(MC * Dk);
      }
      a.kv_ld = kv_ld;
      if (m.kvp_batched) a.rck = m.rck_all ? m.rck_all + (int64_t)l * MC * Hh : nullptr;
      else a.rck = f(MC * Hh);
      a.oc = h(M * D); a.lse_c = f(B * Hh * S);
      if (diff) {
        a.o1 = h(M * D); a.o2 = h(M * D); a.oc1 = h(M * D); a.oc2 = h(M * D);
        a.lse_a2 = f(B * Hh * S); a.lse_c2 = f(B * Hh * S); a.rq2 = f(M * Hh); a.rk2 = f(M * Hh); a.rcq2 = f(M * Hh);
        a.rck2 = f(MC * Hh);
      }
      a.x2 = f(M * D); a.rstd_f = f(M); a.hf = h(M * D); a.ff = h(M * 2 * I); a.act = h(M * I); a.yf = f(M * D);
      a.mod = m.mod_all ? m.mod_all + (int64_t)l * B * 6 * D : nullptr;
      a.yc = m.tix.count(m.bname(l, "cross.out.weight")) ? f(M * D) : nullptr;
    }
    m.x_final = f(M * D);
    m.in_x = f(MT * k.io); m.in_target = f(MT * k.io); m.in_tfeat = f(B * k.time_dim);
    m.in_cross = f(MC * k.cond_dim); m.in_glob = f(B * k.cond_dim);
    m.te_h = f(B * D); m.te = f(B * D); m.g_h = f(B * D); m.gsum = f(B * D); m.gce_h = f(B * D); m.gcond = f(B * 6 * D);
    m.ctx_h = f(MC * D); m.pre = f(MT * k.io); m.xin0 = f(MT * D);
    m.tfeat_b = h(B * k.time_dim); m.te_hb = h(B * D); m.glob_b = h(B * k.cond_dim); m.g_hb = h(B * D);
    m.gsum_b = h(B * D); m.gce_hb = h(B * D); m.cross_b = h(MC * k.cond_dim); m.ctx_hb = h(MC * D);
    m.context_b = h(MC * D); m.xt_b = h(MT * k.io); m.xp_b = h(MT * k.io);
    m.xT_b = h(MT * D); m.pout_b = h(MT * k.io); m.pout = f(MT * k.io); m.vel = f(MT * k.io); m.dvel = f(MT * k.io);
    m.loss = f(64); m.dp = f(MT * k.io); m.dxT = f(MT * D);
    const int64_t wide = std::max<int64_t>(std::max<int64_t>(Q, 2 * I), D);
    m.gx = f(M * D); m.dtmp = f(M * wide); m.dh = f(M * D); m.dact_b = h(M * I); m.dq3 = f(M * Q);
    if (k.local_dim > 0) {   // inpaint local conditioning (used only by the calls that carry it)
      m.local_ld = ((int64_t)k.local_dim + 63) / 64 * 64;
      m.in_local = f(MT * k.local_dim); m.in_lw = f(MT * k.io); m.lmid = f(MT * D);
      m.local_h = h(MT * m.local_ld); m.lmid_h = h(MT * D);
    }
    m.Dsum = f(B * Hh * S); m.dO_b = h(M * D);
    m.dv2 = diff ? f(M * D) : nullptr;
    m.pre_lin = f(MT * k.io); m.vel_lin = f(MT * k.io); m.g_y = f(B * D); m.ctx_y = f(MC * D);
    m.dqf = any_cq ? f(M * Dq) : nullptr;
    m.dkv = need_kv ? f(MC * Dk) : nullptr;
    m.dkvf = need_kv ? f(MC * Dk) : nullptr;
    m.dvc2 = need_kv && diff ? f(MC * D) : nullptr;
    m.dctx = m.need_ctx ? f(MC * D) : nullptr;
    m.dmlp = m.need_ctx || m.need_mod ? f(std::max<int64_t>(MC, B) * D) : nullptr;
    m.dgcond = m.need_mod ? f(B * 6 * D) : nullptr;
    m.dgsum = m.need_mod ? f(B * D) : nullptr;
    m.dxin0 = m.need_x0 ? f(MT * D) : nullptr;
    m.dxp = m.need_x0 ? f(MT * k.io) : nullptr;
    const int64_t maxout = std::max<int64_t>(wide, 6 * D);
    m.dg = f(maxout); m.c3 = f(256);
    m.dut = h(16 * m.ut_ld); m.dz = h(Mx * maxout); m.cb = h(16 * maxout);
    m.c3_all = f(256 * (int64_t)std::max(m.n_active, 1));
    for (size_t i = 0; i < m.tg.size(); ++i) {
      DitTarget& t = m.tg[i];
      if (t.inert) continue;
      t.rows = target_rows(m, t.name);
      t.ut_ld = (t.rows + 63) / 64 * 64;
      t.ut = h(16 * t.ut_ld);
      t.dz = h(t.rows * t.out); t.dg = f(t.out); t.dut = h(16 * t.ut_ld);
      t.cb = m.dora ? h(16 * t.out) : nullptr;
      t.c3 = m.c3_all && t.act >= 0 ? m.c3_all + 256 * (int64_t)t.act : nullptr;
    }
    if (m.mat) {   // weight-gradient scratch of the materialized targets, reused target by target
      int64_t wn = 0, mo = 0, mr = 0;
      for (const DitTarget& t : m.tg) {
        if (t.inert) continue;
        wn = std::max<int64_t>(wn, t.in * t.out);
        mo = std::max<int64_t>(mo, t.out);
        mr = std::max<int64_t>(mr, t.rows);
      }
      m.mat_ldt = (mr + 7) / 8 * 8;
      m.mat_G = f(wn);
      m.mat_dD = h(wn);
      m.mat_dzt = h(mo * m.mat_ldt);
    }
    if (pass == 0) {
      m.arena_bytes = off;
      if (cudaMalloc(&m.arena, off) != cudaSuccess) {
        cudaGetLastError();
        err = "out of device memory for DiT activations (" + std::to_string(off >> 20) + " MiB)";
        m.arena = nullptr;
        return 1;
      }
    }
  }
  return bind_adapter_grads(m, err);
}

// ------------------------------------------------------------------ linear helpers
static int lin_fwd(DitModel& m, const Weight* w, const DitTarget* t, const float* bias, const __half* x,
                   int64_t M, float* y, __half* y_h, std::string& err, const HeadPrepEpi* hp = nullptr) {
  if (t && t->mat) {
    if (t->rows != M || t->x_h != x) { err = "adapter " + t->name + " bound to other input rows"; return 1; }
    GemmDesc g;   // y = x W_eff^T + bias
    g.M = (int)M; g.N = (int)t->out; g.K = (int)t->in;
    g.a = x; g.lda = t->in;
    g.bsrc = kB_F16_KMAJOR; g.b = t->mt.wb; g.ldb = t->in;
    g.col_bias = bias;
    g.out = y; g.ldo = t->out;
    g.out_h = y_h; g.ldo_h = t->out;
    g.name = "linear.fwd";
    return gemm(m.c, g, err);
  }
  LinearFwd f;
  f.w = w; f.ad = t ? &t->prep : nullptr; f.bias = bias; f.x_h = x; f.M = M; f.y = y; f.y_h = y_h;
  f.hp = hp;
  if (t) {
    if (t->rows != M || t->x_h != x) { err = "adapter " + t->name + " bound to other input rows"; return 1; }
    f.ut = t->ut; f.ut_ld = t->ut_ld;
  }
  return linear_forward(m.c, f, err);
}

// dy == nullptr: dz_of(t) (and dg_of(t) for dora) were written by a fused producer of the gradient
static int lin_bwd(DitModel& m, const Weight* w, DitTarget* t, const float* bias, const __half* x,
                   const float* y, const float* dy, int64_t M, float* dx, int dx_acc, __half* dx_h,
                   std::string& err) {
  if (t && t->mat) {
    if (t->rows != M || t->x_h != x) { err = "adapter " + t->name + " bound to other input rows"; return 1; }
    // dz = f16(dy), or already written to m.dz by the fused producer of dy
    if (dy && k_cvt_f16(m.c, dy, M * t->out, m.dz, err)) return 1;
    if (dx || dx_h) {
      GemmDesc g;   // dx = dz W_eff
      g.M = (int)M; g.N = (int)t->in; g.K = (int)t->out;
      g.a = m.dz; g.lda = t->out;
      g.bsrc = kB_F16_MNMAJOR; g.b = t->mt.wb; g.ldb = t->in;
      g.out = dx; g.ldo = t->in; g.accumulate = dx_acc;
      g.out_h = dx_h; g.ldo_h = t->in;
      g.name = "linear.dx";
      if (gemm(m.c, g, err)) return 1;
    }
    return mat_target_backward(m.c, t->mt, m.dz, M, x, m.mat_G, m.mat_dzt, m.mat_ldt, m.mat_dD, err);
  }
  LinearBwd b;
  b.w = w; b.ad = t ? &t->prep : nullptr; b.bias = bias; b.x_h = x; b.y = y; b.dy = dy; b.M = M;
  b.dz_ready = dy == nullptr;
  b.dx = dx; b.dx_accumulate = dx_acc; b.dx_h = dx_h;
  b.ut_ld = m.ut_ld;
  if (t) {
    if (t->rows != M || t->x_h != x) { err = "adapter " + t->name + " bound to other input rows"; return 1; }
    b.ut = t->ut; b.ut_ld = t->ut_ld;
    b.dA = m.g + t->offA; b.dB = m.g + t->offB; b.dm = t->offM >= 0 ? m.g + t->offM : nullptr;
    b.grad_accumulate = 1;
  }
  b.dz = m.dz; b.dg = m.dg; b.dut = m.dut; b.cb = m.cb; b.c3 = m.c3;
  if (t && m.r16_grads.table) {
    // keep this adapter's dz / dg / du^T for the grouped gradient pass at the end of the backward
    b.dz = t->dz; b.dg = t->dg; b.dut = t->dut;
    b.defer_grads = true;
  }
  return linear_backward(m.c, b, err);
}

static DitTarget* target(DitModel& m, const std::string& name) {
  auto it = m.tix.find(name);
  return it == m.tix.end() ? nullptr : &m.tg[(size_t)it->second];
}

// MLP of dit_head: y = W2 silu(W1 x + b1) + b2 (src/dit.h:269-274), either linear adapted
static int mlp_silu(DitModel& m, const std::string& pfx, bool bias, const __half* x, int64_t M, float* h,
                    __half* hb, float* y, __half* y_h, std::string& err) {
  const Weight* w0 = m.weight(pfx + "0.weight", err);
  const Weight* w2 = m.weight(pfx + "2.weight", err);
  if (!w0 || !w2) return 1;
  const float* b0 = bias ? m.vec(pfx + "0.bias", err) : nullptr;
  const float* b2 = bias ? m.vec(pfx + "2.bias", err) : nullptr;
  if (bias && (!b0 || !b2)) return 1;
  if (lin_fwd(m, w0, target(m, pfx + "0.weight"), b0, x, M, h, nullptr, err)) return 1;
  if (k_silu_f16(m.c, h, M * w0->out, hb, err)) return 1;
  return lin_fwd(m, w2, target(m, pfx + "2.weight"), b2, hb, M, y, y_h, err);
}

// Backward of mlp_silu from dy = dL/dy [M][out]: the adapters' gradients and, with dx, dL/dx
// (overwritten).  h = W1 x + b1 and y are the forward's; nothing runs for a frozen MLP whose
// input gradient is not wanted.
static int mlp_silu_bwd(DitModel& m, const std::string& pfx, bool bias, const __half* x, int64_t M,
                        const float* h, const __half* hb, const float* y, const float* dy, float* dx,
                        std::string& err) {
  DitTarget *t0 = target(m, pfx + "0.weight"), *t2 = target(m, pfx + "2.weight");
  const bool inner = t0 || dx;
  if (!t2 && !inner) return 0;
  const Weight* w0 = m.weight(pfx + "0.weight", err);
  const Weight* w2 = m.weight(pfx + "2.weight", err);
  if (!w0 || !w2) return 1;
  const float* b0 = bias ? m.vec(pfx + "0.bias", err) : nullptr;
  const float* b2 = bias ? m.vec(pfx + "2.bias", err) : nullptr;
  if (bias && (!b0 || !b2)) return 1;
  if (lin_bwd(m, w2, t2, b2, hb, y, dy, M, inner ? m.dmlp : nullptr, 0, nullptr, err)) return 1;
  if (!inner) return 0;
  if (k_silu_bwd(m.c, m.dmlp, h, M * w0->out, m.dmlp, err)) return 1;
  return lin_bwd(m, w0, t0, b0, x, h, m.dmlp, M, dx, 0, nullptr, err);
}

// where the backward of linear `t` (null: a linear without adapter) expects its dz / dg
static __half* dz_of(DitModel& m, const DitTarget* t) {
  return t && !t->mat && m.r16_grads.table ? t->dz : m.dz;
}
static float* dg_of(DitModel& m, const DitTarget* t) { return t && !t->mat && m.r16_grads.table ? t->dg : m.dg; }

// self-attention of block `a` over the prepared [q | k | . (| qd | kd)] rows: softmax stream 0
// (q, k) or the differential stream 1 (qd, kd), both on v, output o [M][D] f16.  v takes no
// preparation and is read from the projection output itself.
static AttnArgs self_attn(const DitBlockAct& a, int B, int H, int S, int D, int Q, float scale, int st,
                          __half* o) {
  AttnArgs r;
  r.B = B; r.H = H; r.Sq = S; r.Sk = S; r.scale = scale; r.window = -1;
  r.q = a.qkvb + (st ? 3 * D : 0); r.q_sb = (long)S * Q; r.q_sh = 64; r.q_ld = Q;
  r.k = a.qkvb + (st ? 4 * D : D); r.k_sb = r.q_sb; r.k_sh = 64; r.k_ld = Q;
  r.v = a.qkv + 2 * D; r.v_sb = r.q_sb; r.v_sh = 64; r.v_ld = Q;
  r.o = o; r.o_sb = (long)S * D; r.o_sh = 64; r.o_ld = D;
  r.lse = st ? a.lse_a2 : a.lse_a;
  return r;
}

// cross-attention of block `a`: queries [cq (| cqd)] [M][Dq], context rows [ck (| ckd) | cv]
// [B C][Dk]; stream st as for self_attn
static AttnArgs cross_attn(const DitBlockAct& a, int B, int H, int S, int C, int D, int Dq, int Dk, float scale,
                           int st, __half* o) {
  AttnArgs r;
  r.B = B; r.H = H; r.Sq = S; r.Sk = C; r.scale = scale; r.window = -1;
  r.q = a.cq + st * D; r.q_sb = (long)S * Dq; r.q_sh = 64; r.q_ld = Dq;
  r.k = a.kvb + st * D; r.k_sb = (long)C * a.kv_ld; r.k_sh = 64; r.k_ld = a.kv_ld;
  r.v = a.kvb + (Dk - D); r.v_sb = r.k_sb; r.v_sh = 64; r.v_ld = a.kv_ld;
  r.o = o; r.o_sb = (long)S * D; r.o_sh = 64; r.o_ld = D;
  r.lse = st ? a.lse_c2 : a.lse_c;
  return r;
}

// The context K / V projections of all blocks (m.kv_batched): one GEMM over the stacked f16
// weights when every block's cross.kv has its f16 operand copy in use, else one GEMM per block;
// either way into kvf_all, block l at column l Dk.  The stacked copy is refilled when the model
// generation changed (set_tensor); a refill recorded into a caller's graph repeats on every
// replay, so it is only marked current when made outside a capture.
static int context_kv_all(DitModel& m, int64_t MC, int64_t Dk, std::string& err) {
  Ctx* c = m.c;
  const int L = m.cfg.depth;
  const int64_t ld = (int64_t)L * Dk;
  std::vector<const Weight*> w(L);
  bool stacked = true;
  for (int l = 0; l < L; ++l) {
    if (!(w[l] = m.weight(m.bname(l, "cross.kv.weight"), err))) return 1;
    if (w[l]->out != Dk || w[l]->in != w[0]->in) { err = "cross.kv weights of different shapes"; return 1; }
    stacked = stacked && w[l]->f16 &&
              (w[l]->type == kTypeF16 || w[l]->type == kTypeF32 || !c->smem_dequant);
  }
  const int64_t K = w[0]->in;
  if (!stacked) {
    for (int l = 0; l < L; ++l) {
      GemmDesc g;
      g.M = (int)MC; g.N = (int)Dk; g.K = (int)K;
      g.a = m.context_b; g.lda = K;
      g.bsrc = kB_WEIGHT_NT; g.w = w[l];
      g.out = m.kvf_all + l * Dk; g.ldo = ld;
      g.name = "linear.fwd";
      if (gemm(c, g, err)) return 1;
    }
    return 0;
  }
  if (!m.kv_w_all && !(m.kv_w_all = static_cast<__half*>(dmalloc(m, sizeof(__half) * (size_t)(ld * K), err))))
    return 1;
  if (m.kvw_mgen != m.gen) {
    for (int l = 0; l < L; ++l)
      if (cudaMemcpyAsync(m.kv_w_all + l * Dk * K, w[l]->f16, sizeof(__half) * (size_t)(Dk * K),
                          cudaMemcpyDeviceToDevice, c->stream) != cudaSuccess)
        return check_launch("stacked cross.kv weights", err);
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(c->stream, &cs) != cudaSuccess) cudaGetLastError();
    if (cs == cudaStreamCaptureStatusNone) m.kvw_mgen = m.gen;
  }
  GemmDesc g;   // kvf_all = context W_all^T
  g.M = (int)MC; g.N = (int)ld; g.K = (int)K;
  g.a = m.context_b; g.lda = K;
  g.bsrc = kB_F16_KMAJOR; g.b = m.kv_w_all; g.ldb = K;
  g.out = m.kvf_all; g.ldo = ld;
  g.name = "linear.fwd";
  return gemm(c, g, err);
}

// ------------------------------------------------------------------ forward + backward
static int dit_step(DitModel& m, std::string& err) {
  Ctx* c = m.c;
  const sa3k_dit_config& k = m.cfg;
  const int B = m.B, T = m.T, C = m.C, S = m.Sfull(), D = k.dim, H = k.heads, I = k.ff_inner;
  const int64_t M = (int64_t)B * S, MT = (int64_t)B * T, MC = (int64_t)B * C;
  const int Q = m.qkv_cols();
  const float scale = 1.0f / std::sqrt((float)k.head_dim);
  const bool diff = k.differential != 0;
  const int Dq = m.cq_cols(), Dk = m.ckv_cols();

  // Gradient scale: the loss gradient leaves the MSE kernel multiplied by gscale, a power of two
  // near io*T / 2, so the output gradient is (vel - target) in size and every gradient the backward
  // stores as an f16 operand (dz, du^T, dO, the SwiGLU output gradient) sits well inside the f16
  // normal range.  Every adapter-gradient contribution of the step is linear in the loss gradient
  // and adds into the flat buffer, so the buffer is multiplied by gscale before the step and by
  // 1 / gscale after it: both exact in f32, the accumulated gradients come out unscaled.
  const float gscale = std::exp2(std::floor(std::log2(0.5f * (float)T * (float)k.io)));
  if (m.np > 0 && k_scale(c, m.g, m.np, gscale, err)) return 1;
  if (m.inpaint && k_pad_f16(c, m.in_local, MT, k.local_dim, m.local_h, m.local_ld, err)) return 1;

  // adapters: operand forms + DoRA norms, once per step (grouped launches over all adapters; the
  // DoRA P = W A^T GEMMs run per adapter between them)
  const int nt = m.n_active;
  if (nt > 0 && k_prep_all(c, m.prep_desc, nt, err)) return 1;
  if (m.dora && nt > 0) {
    if (k_aat_all(c, m.prep_desc, nt, err)) return 1;
    if (m.r16_prep.table) {
      if (r16_group_run(c, m.r16_prep, "dora.P", err)) return 1;
    } else {
      for (DitTarget& t : m.tg)
        if (!t.inert && adapter_dora_p(c, t.w, t.prep, err)) return 1;
    }
    if (k_dora_norm_all(c, m.prep_desc, nt, m.max_out, err)) return 1;
  }
  // materialized families: W_eff of every target from this step's parameters
  for (DitTarget& t : m.tg)
    if (t.mat && !t.inert && mat_target_build(c, t.mt, nullptr, err)) return 1;

  // ---------------- head (src/dit.h:286-310)
  if (k_cvt_f16(c, m.in_tfeat, (int64_t)B * k.time_dim, m.tfeat_b, err)) return 1;
  if (mlp_silu(m, "dit.time_embed.", true, m.tfeat_b, B, m.te_h, m.te_hb, m.te, nullptr, err)) return 1;
  if (k_cvt_f16(c, m.in_glob, (int64_t)B * k.cond_dim, m.glob_b, err)) return 1;
  if (mlp_silu(m, "dit.global_embed.", false, m.glob_b, B, m.g_h, m.g_hb, m.g_y, nullptr, err)) return 1;
  if (k_add(c, m.g_y, m.te, (long)B * D, m.gsum, err)) return 1;
  if (k_cvt_f16(c, m.gsum, (int64_t)B * D, m.gsum_b, err)) return 1;
  if (mlp_silu(m, "dit.gce.", true, m.gsum_b, B, m.gce_h, m.gce_hb, m.gcond, nullptr, err)) return 1;
  if (k_cvt_f16(c, m.in_cross, MC * k.cond_dim, m.cross_b, err)) return 1;
  if (mlp_silu(m, "dit.cond_embed.", false, m.cross_b, MC, m.ctx_h, m.ctx_hb, m.ctx_y, m.context_b, err)) return 1;
  {
    const Weight* wpre = m.weight("dit.pre_conv.weight", err);
    const Weight* win = m.weight("dit.proj_in.weight", err);
    const float* mem = m.vec("dit.memory_tokens", err);
    if (!wpre || !win || !mem) return 1;
    if (k_cvt_f16(c, m.in_x, MT * k.io, m.xt_b, err)) return 1;
    if (lin_fwd(m, wpre, target(m, "dit.pre_conv.weight"), nullptr, m.xt_b, MT, m.pre_lin, nullptr, err)) return 1;
    if (k_add(c, m.pre_lin, m.in_x, (long)MT * k.io, m.pre, err)) return 1;
    if (k_cvt_f16(c, m.pre, MT * k.io, m.xp_b, err)) return 1;
    if (lin_fwd(m, win, target(m, "dit.proj_in.weight"), nullptr, m.xp_b, MT, m.xin0, nullptr, err)) return 1;
    float* x0 = m.blk[0].x;
    if (k_copy_rows(c, mem, 0, 0, x0, nullptr, S, 0, B, k.mem_tokens, D, err)) return 1;
    if (k_copy_rows(c, m.xin0, T, 0, x0, nullptr, S, k.mem_tokens, B, T, D, err)) return 1;
  }

  // ---------------- blocks (src/dit.h:164-266)
  // every block's adaLN vectors first: the residual kernel ending block l also forms the
  // modulated pre-norm input of block l + 1
  {
    const size_t per = sizeof(float) * 6 * (size_t)D;
    if (!m.ssg_all && !(m.ssg_all = static_cast<float*>(dmalloc(m, per * k.depth, err)))) return 1;
    if (m.kvp_batched && !m.gck_all && !(m.gck_all = static_cast<float*>(dmalloc(m, sizeof(float) * 64 * k.depth, err))))
      return 1;
    if (m.ssg_mgen != m.gen) {
      for (int l = 0; l < k.depth; ++l) {
        const float* ssg = m.vec(m.bname(l, "ssg"), err);
        if (!ssg) return 1;
        if (cudaMemcpyAsync(m.ssg_all + (size_t)l * 6 * D, ssg, per, cudaMemcpyDeviceToDevice, c->stream) != cudaSuccess)
          return check_launch("stacked ssg", err);
        if (m.kvp_batched) {
          const float* gck = m.vec(m.bname(l, "cross.k_norm.gamma"), err);
          if (!gck) return 1;
          if (cudaMemcpyAsync(m.gck_all + (size_t)l * 64, gck, sizeof(float) * 64, cudaMemcpyDeviceToDevice,
                              c->stream) != cudaSuccess)
            return check_launch("stacked k_norm gammas", err);
        }
      }
      cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
      if (cudaStreamIsCapturing(c->stream, &cs) != cudaSuccess) cudaGetLastError();
      if (cs == cudaStreamCaptureStatusNone) m.ssg_mgen = m.gen;   // (a captured refill repeats per replay)
    }
    if (k_modulation(c, m.ssg_all, m.gcond, B, D, m.mod_all, err, k.depth)) return 1;
  }
  if (m.kv_batched && context_kv_all(m, MC, Dk, err)) return 1;
  if (m.kvp_batched) {
    // [ck | cv] of every block: ck with its block's cross.k_norm, cv copied
    HeadSlice hs[2];
    hs[0].col = 0; hs[0].gamma = m.gck_all; hs[0].rstd = m.rck_all;
    hs[1].col = Dk - D;
    if (k_head_prep_fwd_reps(c, m.kvf_all, (int)MC, (int)((int64_t)k.depth * Dk), H, hs, 2, C, k.qk_eps, k.rot,
                             k.rope_base, m.kvb_all, k.depth, (int)Dk, 64, (long)MC * H, err))
      return 1;
  }
  for (int l = 0; l < k.depth; ++l) {
    DitBlockAct& a = m.blk[l];
    float* x_next = l + 1 < k.depth ? m.blk[l + 1].x : m.x_final;
    const Weight *wqkv = m.weight(m.bname(l, "self.qkv.weight"), err), *wout = m.weight(m.bname(l, "self.out.weight"), err);
    const Weight *wcq = m.weight(m.bname(l, "cross.q.weight"), err), *wckv = m.weight(m.bname(l, "cross.kv.weight"), err);
    const Weight *wco = m.weight(m.bname(l, "cross.out.weight"), err), *wfp = m.weight(m.bname(l, "ff.proj.weight"), err);
    const Weight* wfo = m.weight(m.bname(l, "ff.out.weight"), err);
    const float *ssg = m.vec(m.bname(l, "ssg"), err), *g_pre = m.vec(m.bname(l, "pre_norm.gamma"), err);
    const float *g_q = m.vec(m.bname(l, "self.q_norm.gamma"), err), *g_k = m.vec(m.bname(l, "self.k_norm.gamma"), err);
    const float *g_cn = m.vec(m.bname(l, "cross_norm.gamma"), err), *g_cq = m.vec(m.bname(l, "cross.q_norm.gamma"), err);
    const float *g_ck = m.vec(m.bname(l, "cross.k_norm.gamma"), err), *g_ff = m.vec(m.bname(l, "ff_norm.gamma"), err);
    const float *b_fp = m.vec(m.bname(l, "ff.proj.bias"), err), *b_fo = m.vec(m.bname(l, "ff.out.bias"), err);
    if (!wqkv || !wout || !wcq || !wckv || !wco || !wfp || !wfo || !ssg || !g_pre || !g_q || !g_k || !g_cn || !g_cq ||
        !g_ck || !g_ff || !b_fp || !b_fo)
      return 1;
    DitTarget *tq = target(m, m.bname(l, "self.qkv.weight")), *to = target(m, m.bname(l, "self.out.weight"));
    DitTarget *tp = target(m, m.bname(l, "ff.proj.weight")), *tf = target(m, m.bname(l, "ff.out.weight"));
    DitTarget *tcq = target(m, m.bname(l, "cross.q.weight")), *tkv = target(m, m.bname(l, "cross.kv.weight"));
    DitTarget* tco = target(m, m.bname(l, "cross.out.weight"));
    const long ms = 6L * D;
    // self-attention branch (block 0's pre-norm here; every later one ran fused with the residual
    // step that ended the previous block)
    if (l == 0 &&
        k_rmsnorm_mod_fwd(c, a.x, (int)M, D, g_pre, a.mod, a.mod + D, ms, S, k.norm_eps, a.h_a, a.rstd_a, err))
      return 1;
    // the q / k head preparation (RMS norm, RoPE) runs in the epilogue of the qkv GEMM when that
    // GEMM takes the CTA-pair kernel with the f16 weight operand (no differential slices, no
    // materialized qkv target); otherwise as its own pass over the projection output
    const bool f16_w = wqkv->type == kTypeF16 || wqkv->type == kTypeF32 || (wqkv->f16 && !c->smem_dequant);
    const bool fuse_hp = !diff && (k.rot == 0 || k.rot == 32 || k.rot == 64) && !(tq && tq->mat) && f16_w &&
                         c->fuse_head_prep && gemm_pair_applies(c, (int)M, Q, true);
    if (fuse_hp) {
      HeadPrepEpi hp;
      hp.out = a.qkvb; hp.ld = Q;
      hp.gq = g_q; hp.gk = g_k; hp.rq = a.rq; hp.rk = a.rk;
      hp.tab = k.rot ? k_rope_table(c, S, k.rot, k.rope_base, err) : nullptr;
      if (k.rot && !hp.tab) return 1;
      if (hp.tab) hp.tab += (long)S * (k.rot / 2);   // the frequency-major copy
      hp.tps = S; hp.rot = k.rot; hp.D = D; hp.H = H; hp.eps = k.qk_eps;
      if (lin_fwd(m, wqkv, tq, nullptr, a.h_a, M, nullptr, a.qkv, err, &hp)) return 1;
    } else {
    if (lin_fwd(m, wqkv, tq, nullptr, a.h_a, M, nullptr, a.qkv, err)) return 1;
    {
      // [q | k | v (| qd | kd)]: q / qd share q_norm, k / kd share k_norm, all four take RoPE;
      // v is left where the projection wrote it
      HeadSlice hs[4];
      hs[0].col = 0; hs[0].gamma = g_q; hs[0].rope = 1; hs[0].rstd = a.rq;
      hs[1].col = D; hs[1].gamma = g_k; hs[1].rope = 1; hs[1].rstd = a.rk;
      hs[2].col = 3 * D; hs[2].gamma = g_q; hs[2].rope = 1; hs[2].rstd = a.rq2;
      hs[3].col = 4 * D; hs[3].gamma = g_k; hs[3].rope = 1; hs[3].rstd = a.rk2;
      if (k_head_prep_fwd(c, a.qkv, (int)M, Q, H, hs, diff ? 4 : 2, S, k.qk_eps, k.rot, k.rope_base, a.qkvb, err))
        return 1;
    }
    }
    AttnArgs sa = self_attn(a, B, H, S, D, Q, scale, 0, diff ? a.o1 : a.oa);
    if (attn_forward(c, sa, err)) return 1;
    if (diff) {
      // differential attention (src/dit.h:152-158): o = sdpa(q, k, v) - sdpa(qd, kd, v)
      AttnArgs sd = self_attn(a, B, H, S, D, Q, scale, 1, a.o2);
      if (attn_forward(c, sd, err)) return 1;
      if (k_sub_f16(c, a.o1, a.o2, M * D, a.oa, err)) return 1;
    }
    if (lin_fwd(m, wout, to, nullptr, a.oa, M, a.yo, nullptr, err)) return 1;
    // x1 = x + gate(yo), then the cross-attention branch's norm of x1
    if (k_residual_norm(c, a.x, a.yo, a.mod + 2 * D, ms, (int)M, D, S, a.x1, g_cn, nullptr, nullptr, 0, k.norm_eps,
                        a.hc, a.rstd_c, err))
      return 1;
    if (lin_fwd(m, wcq, tcq, nullptr, a.hc, M, a.qf, nullptr, err)) return 1;
    {
      // [cq (| cqd)], both with cross.q_norm, no RoPE
      HeadSlice hs[2];
      hs[0].col = 0; hs[0].gamma = g_cq; hs[0].rstd = a.rcq;
      hs[1].col = D; hs[1].gamma = g_cq; hs[1].rstd = a.rcq2;
      if (k_head_prep_fwd(c, a.qf, (int)M, Dq, H, hs, diff ? 2 : 1, S, k.qk_eps, k.rot, k.rope_base, a.cq, err))
        return 1;
    }
    if (!m.kv_batched && lin_fwd(m, wckv, tkv, nullptr, m.context_b, MC, a.kvf, nullptr, err)) return 1;
    if (!m.kvp_batched) {
      // [ck (| ckd) | cv], ck / ckd with cross.k_norm
      HeadSlice hs[3];
      hs[0].col = 0; hs[0].gamma = g_ck; hs[0].rstd = a.rck;
      if (diff) { hs[1].col = D; hs[1].gamma = g_ck; hs[1].rstd = a.rck2; }
      hs[diff ? 2 : 1].col = Dk - D;
      if (k_head_prep_fwd(c, a.kvf, (int)MC, (int)a.kv_ld, H, hs, diff ? 3 : 2, C, k.qk_eps, k.rot, k.rope_base,
                          a.kvb, err))
        return 1;
    }
    AttnArgs ca = cross_attn(a, B, H, S, C, D, Dq, Dk, scale, 0, diff ? a.oc1 : a.oc);
    if (attn_forward(c, ca, err)) return 1;
    if (diff) {
      AttnArgs cd = cross_attn(a, B, H, S, C, D, Dq, Dk, scale, 1, a.oc2);
      if (attn_forward(c, cd, err)) return 1;
      if (k_sub_f16(c, a.oc1, a.oc2, M * D, a.oc, err)) return 1;
    }
    if (lin_fwd(m, wco, tco, nullptr, a.oc, M, tco ? a.yc : m.dtmp, nullptr, err)) return 1;
    if (m.inpaint) {
      // inpaint local conditioning (src/dit.h:244-254): local.2(silu(local.0(local))) added to
      // the T real tokens of every sample, the memory tokens + 0; the local.* projections are
      // frozen and the input is data, so nothing of this branch is differentiated
      const Weight* wl0 = m.Wpad.count(m.bname(l, "local.0.weight")) ? m.Wpad[m.bname(l, "local.0.weight")]
                                                                      : m.weight(m.bname(l, "local.0.weight"), err);
      const Weight* wl2 = m.weight(m.bname(l, "local.2.weight"), err);
      const float* bl0 = m.vec(m.bname(l, "local.0.bias"), err);
      const float* bl2 = m.vec(m.bname(l, "local.2.bias"), err);
      if (!wl0 || !wl2 || !bl0 || !bl2) return 1;
      if (lin_fwd(m, wl0, nullptr, bl0, m.local_h, MT, m.lmid, nullptr, err)) return 1;
      if (k_silu_f16(c, m.lmid, (long)MT * D, m.lmid_h, err)) return 1;
      if (lin_fwd(m, wl2, nullptr, bl2, m.lmid_h, MT, m.lmid, nullptr, err)) return 1;
      if (k_add_local(c, tco ? a.yc : m.dtmp, m.lmid, B, S, k.mem_tokens, D, m.dtmp, err)) return 1;
    }
    // x2 = x1 + cross-attention output, then the feed-forward branch's modulated norm of x2
    if (k_residual_norm(c, a.x1, (tco && !m.inpaint) ? a.yc : m.dtmp, nullptr, 0, (int)M, D, S, a.x2, g_ff, a.mod + 3 * D,
                        a.mod + 4 * D, ms, k.norm_eps, a.hf, a.rstd_f, err))
      return 1;
    if (lin_fwd(m, wfp, tp, b_fp, a.hf, M, nullptr, a.ff, err)) return 1;
    if (k_swiglu_fwd(c, a.ff, (int)M, I, a.act, err)) return 1;
    if (lin_fwd(m, wfo, tf, b_fo, a.act, M, a.yf, nullptr, err)) return 1;
    if (l + 1 < k.depth) {
      // x_next = x2 + gate(yf), then block l + 1's modulated pre-norm of it
      DitBlockAct& an = m.blk[l + 1];
      const float* g_pre_n = m.vec(m.bname(l + 1, "pre_norm.gamma"), err);
      if (!g_pre_n) return 1;
      if (k_residual_norm(c, a.x2, a.yf, a.mod + 5 * D, ms, (int)M, D, S, x_next, g_pre_n, an.mod, an.mod + D, ms,
                          k.norm_eps, an.h_a, an.rstd_a, err))
        return 1;
    } else if (k_gate_residual(c, a.x2, a.yf, a.mod + 5 * D, ms, (int)M, D, S, x_next, err)) {
      return 1;
    }
  }

  // ---------------- tail + loss (src/dit.h:314-323, src/train_ckpt.h:223-228)
  const Weight* wpo = m.weight("dit.proj_out.weight", err);
  const Weight* wpc = m.weight("dit.post_conv.weight", err);
  if (!wpo || !wpc) return 1;
  if (k_copy_rows(c, m.x_final, S, k.mem_tokens, nullptr, m.xT_b, T, 0, B, T, D, err)) return 1;
  DitTarget *tpo = target(m, "dit.proj_out.weight"), *tpc = target(m, "dit.post_conv.weight");
  if (lin_fwd(m, wpo, tpo, nullptr, m.xT_b, MT, m.pout, m.pout_b, err)) return 1;
  if (lin_fwd(m, wpc, tpc, nullptr, m.pout_b, MT, m.vel_lin, nullptr, err)) return 1;
  if (k_add(c, m.vel_lin, m.pout, (long)MT * k.io, m.vel, err)) return 1;
  if (k_mse(c, m.vel, m.in_target, B, (long)T * k.io, m.loss, m.dvel, gscale, m.inpaint ? m.in_lw : nullptr, err))
    return 1;

  // ---------------- backward
  if (cudaMemcpyAsync(m.dp, m.dvel, sizeof(float) * MT * k.io, cudaMemcpyDeviceToDevice, c->stream) != cudaSuccess)
    return check_launch("copy", err);
  if (lin_bwd(m, wpc, tpc, nullptr, m.pout_b, m.vel_lin, m.dvel, MT, m.dp, 1, nullptr, err)) return 1;
  if (lin_bwd(m, wpo, tpo, nullptr, m.xT_b, m.pout, m.dp, MT, m.dxT, 0, nullptr, err)) return 1;
  if (cudaMemsetAsync(m.gx, 0, sizeof(float) * M * D, c->stream) != cudaSuccess) return check_launch("memset", err);
  if (m.need_ctx && cudaMemsetAsync(m.dctx, 0, sizeof(float) * MC * D, c->stream) != cudaSuccess)
    return check_launch("memset", err);
  if (m.need_mod && cudaMemsetAsync(m.dgcond, 0, sizeof(float) * B * 6 * D, c->stream) != cudaSuccess)
    return check_launch("memset", err);
  if (k_copy_rows(c, m.dxT, T, 0, m.gx, nullptr, S, k.mem_tokens, B, T, D, err)) return 1;

  for (int l = k.depth - 1; l >= 0; --l) {
    DitBlockAct& a = m.blk[l];
    const Weight *wqkv = m.weight(m.bname(l, "self.qkv.weight"), err), *wout = m.weight(m.bname(l, "self.out.weight"), err);
    const Weight *wcq = m.weight(m.bname(l, "cross.q.weight"), err), *wco = m.weight(m.bname(l, "cross.out.weight"), err);
    const Weight *wfp = m.weight(m.bname(l, "ff.proj.weight"), err), *wfo = m.weight(m.bname(l, "ff.out.weight"), err);
    const float *g_pre = m.vec(m.bname(l, "pre_norm.gamma"), err), *g_q = m.vec(m.bname(l, "self.q_norm.gamma"), err);
    const float *g_k = m.vec(m.bname(l, "self.k_norm.gamma"), err), *g_cn = m.vec(m.bname(l, "cross_norm.gamma"), err);
    const float *g_cq = m.vec(m.bname(l, "cross.q_norm.gamma"), err), *g_ff = m.vec(m.bname(l, "ff_norm.gamma"), err);
    const float *b_fp = m.vec(m.bname(l, "ff.proj.bias"), err), *b_fo = m.vec(m.bname(l, "ff.out.bias"), err);
    const Weight* wckv = m.weight(m.bname(l, "cross.kv.weight"), err);
    const float* g_ck = m.vec(m.bname(l, "cross.k_norm.gamma"), err);
    DitTarget *tq = target(m, m.bname(l, "self.qkv.weight")), *to = target(m, m.bname(l, "self.out.weight"));
    DitTarget *tp = target(m, m.bname(l, "ff.proj.weight")), *tf = target(m, m.bname(l, "ff.out.weight"));
    DitTarget *tcq = target(m, m.bname(l, "cross.q.weight")), *tkv = target(m, m.bname(l, "cross.kv.weight"));
    DitTarget* tco = target(m, m.bname(l, "cross.out.weight"));
    const bool kv_grad = tkv || m.need_ctx;
    const long ms = 6L * D;
    // feed-forward branch
    // (the gate and SwiGLU backward write the adapted linears' dz / dg directly)
    if (m.need_mod && k_mod_grad_gate(c, m.gx, a.yf, a.mod + 5 * D, ms, (int)M, D, S, ms, m.dgcond + 5 * D, err))
      return 1;
    if (k_gate_bwd_dz(c, m.gx, a.mod + 5 * D, ms, (int)M, D, S, a.yf, b_fo, tf && tf->prep.dora() ? tf->prep.g : nullptr,
                      dz_of(m, tf), dg_of(m, tf), err))
      return 1;
    if (lin_bwd(m, wfo, tf, b_fo, a.act, a.yf, nullptr, M, nullptr, 0, m.dact_b, err)) return 1;
    if (k_swiglu_bwd_dz(c, m.dact_b, a.ff, (int)M, I, b_fp, tp && tp->prep.dora() ? tp->prep.g : nullptr, dz_of(m, tp),
                        dg_of(m, tp), err))
      return 1;
    // (dz / dg come from the SwiGLU backward, so the f32 output y is not needed here)
    if (lin_bwd(m, wfp, tp, b_fp, a.hf, nullptr, nullptr, M, m.dh, 0, nullptr, err)) return 1;
    if (m.need_mod && k_mod_grad_norm(c, m.dh, a.x2, a.rstd_f, g_ff, (int)M, D, S, ms, m.dgcond + 3 * D,
                                      m.dgcond + 4 * D, err))
      return 1;
    // (without a cross.out adapter the norm backward also leaves gx as f16 in m.dz: the input of
    // the cross.out backward; an adapted cross.out takes the f32 gradient)
    if (k_rmsnorm_mod_bwd(c, m.dh, a.x2, a.rstd_f, (int)M, D, g_ff, a.mod + 3 * D, ms, S, m.gx, tco ? nullptr : m.dz,
                          err))
      return 1;
    // cross-attention branch: dq always; dk / dv when cross.kv is adapted or the context's own
    // MLP is (the context gradient sums the blocks' cross.kv input gradients)
    if (tco) {
      if (lin_bwd(m, wco, tco, nullptr, a.oc, a.yc, m.gx, M, nullptr, 0, m.dO_b, err)) return 1;
    } else if (lin_bwd(m, wco, nullptr, nullptr, a.oc, nullptr, nullptr, M, nullptr, 0, m.dO_b, err)) {
      return 1;
    }
    for (int st = 0; st < (diff ? 2 : 1); ++st) {
      // stream st's dq into m.dtmp [M][Dq] columns st D.. (the second differential stream runs on
      // +dO, so its gradients enter the head backward negated); dk into m.dkv [MC][Dk] columns
      // st D.., dv of stream 0 into m.dkvf's v columns, of stream 1 into m.dvc2
      AttnArgs ca = cross_attn(a, B, H, S, C, D, Dq, Dk, scale, st, st ? a.oc2 : diff ? a.oc1 : a.oc);
      ca.dO = m.dO_b; ca.dO_sb = (long)S * D; ca.dO_sh = 64; ca.dO_ld = D;
      ca.Dsum = m.Dsum;
      ca.dq = m.dtmp + st * D; ca.dq_sb = (long)S * Dq; ca.dq_sh = 64; ca.dq_ld = Dq;
      if (kv_grad) {
        ca.dk = m.dkv + st * D; ca.dk_sb = (long)C * Dk; ca.dk_sh = 64; ca.dk_ld = Dk;
        if (st) {
          ca.dv = m.dvc2; ca.dv_sb = (long)C * D; ca.dv_sh = 64; ca.dv_ld = D;
        } else {
          ca.dv = m.dkvf + (Dk - D); ca.dv_sb = (long)C * Dk; ca.dv_sh = 64; ca.dv_ld = Dk;
        }
      }
      if (attn_backward(c, ca, kv_grad, err)) return 1;
      HeadSlice hs;
      hs.col = st * D; hs.gamma = g_cq; hs.rstd = st ? a.rcq2 : a.rcq;
      // f16 gradient straight into m.dz (the input of the cross.q backward), or f32 for an
      // adapted cross.q
      if (k_head_prep_bwd(c, m.dtmp + st * D, Dq, a.qf, (int)M, Dq, H, hs, S, k.rot, k.rope_base, tcq ? m.dqf : nullptr,
                          tcq ? nullptr : m.dz, err, st ? -1.0f : 1.0f))
        return 1;
    }
    if (lin_bwd(m, wcq, tcq, nullptr, a.hc, tcq ? a.qf : nullptr, tcq ? m.dqf : nullptr, M, m.dtmp, 0, nullptr, err))
      return 1;
    if (k_rmsnorm_mod_bwd(c, m.dtmp, a.x1, a.rstd_c, (int)M, D, g_cn, nullptr, 0, S, m.gx, nullptr, err)) return 1;
    if (kv_grad) {
      // [ck (| ckd) | cv] of the context rows: k-norm backward of each k slice, v = dv (- dv2)
      for (int st = 0; st < (diff ? 2 : 1); ++st) {
        HeadSlice hs;
        hs.col = st * D; hs.gamma = g_ck; hs.rstd = st ? a.rck2 : a.rck;
        if (k_head_prep_bwd(c, m.dkv + st * D, Dk, a.kvf, (int)MC, Dk, H, hs, C, k.rot, k.rope_base, m.dkvf, nullptr,
                            err, st ? -1.0f : 1.0f))
          return 1;
      }
      if (diff) {
        HeadSlice hv;
        hv.col = Dk - D;
        if (k_head_prep_bwd(c, m.dkvf + (Dk - D), Dk, a.kvf, (int)MC, Dk, H, hv, C, k.rot, k.rope_base, m.dkvf, nullptr,
                            err, 1.0f, m.dvc2, D))
          return 1;
      }
      if (lin_bwd(m, wckv, tkv, nullptr, m.context_b, a.kvf, m.dkvf, MC, m.need_ctx ? m.dctx : nullptr, 1, nullptr,
                  err))
        return 1;
    }
    // self-attention branch
    if (m.need_mod && k_mod_grad_gate(c, m.gx, a.yo, a.mod + 2 * D, ms, (int)M, D, S, ms, m.dgcond + 2 * D, err))
      return 1;
    if (k_gate_bwd_dz(c, m.gx, a.mod + 2 * D, ms, (int)M, D, S, a.yo, nullptr,
                      to && to->prep.dora() ? to->prep.g : nullptr, dz_of(m, to), dg_of(m, to), err))
      return 1;
    if (lin_bwd(m, wout, to, nullptr, a.oa, a.yo, nullptr, M, nullptr, 0, m.dO_b, err)) return 1;
    for (int st = 0; st < (diff ? 2 : 1); ++st) {
      // m.dq3 [M][Q] = [dq | dk | dv (| dqd' | dkd')]: the second differential stream runs on +dO
      // and leaves its (negated) q / k gradients in the last two slices and its dV in m.dv2
      AttnArgs sa = self_attn(a, B, H, S, D, Q, scale, st, st ? a.o2 : diff ? a.o1 : a.oa);
      sa.dO = m.dO_b; sa.dO_sb = (long)S * D; sa.dO_sh = 64; sa.dO_ld = D;
      sa.Dsum = m.Dsum;
      sa.dq = m.dq3 + (st ? 3 * D : 0); sa.dq_sb = (long)S * Q; sa.dq_sh = 64; sa.dq_ld = Q;
      sa.dk = m.dq3 + (st ? 4 * D : D); sa.dk_sb = sa.dq_sb; sa.dk_sh = 64; sa.dk_ld = Q;
      if (st) {
        sa.dv = m.dv2; sa.dv_sb = (long)S * D; sa.dv_sh = 64; sa.dv_ld = D;
      } else {
        sa.dv = m.dq3 + 2 * D; sa.dv_sb = sa.dq_sb; sa.dv_sh = 64; sa.dv_ld = Q;
      }
      if (attn_backward(c, sa, true, err)) return 1;
    }
    // q / k head preparation backward fused with the qkv projection's prologue
    if (k_qkv_bwd_dz(c, m.dq3, a.qkv, (int)M, D, H, diff ? 5 : 3, a.rq, a.rk, a.rq2, a.rk2, m.dv2, g_q, g_k, S,
                     k.rot, k.rope_base, tq && tq->prep.dora() ? tq->prep.g : nullptr, dz_of(m, tq), dg_of(m, tq),
                     err))
      return 1;
    // (dz / dg come from the fused head backward, so the f32 output y is not needed here)
    if (lin_bwd(m, wqkv, tq, nullptr, a.h_a, nullptr, nullptr, M, m.dh, 0, nullptr, err)) return 1;
    if (m.need_mod && k_mod_grad_norm(c, m.dh, a.x, a.rstd_a, g_pre, (int)M, D, S, ms, m.dgcond, m.dgcond + D, err))
      return 1;
    if (k_rmsnorm_mod_bwd(c, m.dh, a.x, a.rstd_a, (int)M, D, g_pre, a.mod, ms, S, m.gx, nullptr, err)) return 1;
  }
  // ---------------- head adapters (src/train_ckpt.h:440-470: the head's VJP against dL/dx0,
  // dL/dcontext and dL/dgcond)
  if (m.need_x0) {
    // x0 = [memory tokens | proj_in(x_in + pre_conv(x_in))]: the T rows of dL/dx0 per sample
    const Weight* wpre = m.weight("dit.pre_conv.weight", err);
    const Weight* win = m.weight("dit.proj_in.weight", err);
    if (!wpre || !win) return 1;
    DitTarget* tpre = target(m, "dit.pre_conv.weight");
    if (k_copy_rows(c, m.gx, S, k.mem_tokens, m.dxin0, nullptr, T, 0, B, T, D, err)) return 1;
    if (lin_bwd(m, win, target(m, "dit.proj_in.weight"), nullptr, m.xp_b, m.xin0, m.dxin0, MT, tpre ? m.dxp : nullptr,
                0, nullptr, err))
      return 1;
    if (tpre && lin_bwd(m, wpre, tpre, nullptr, m.xt_b, m.pre_lin, m.dxp, MT, nullptr, 0, nullptr, err)) return 1;
  }
  if (m.need_ctx && mlp_silu_bwd(m, "dit.cond_embed.", false, m.cross_b, MC, m.ctx_h, m.ctx_hb, m.ctx_y, m.dctx,
                                 nullptr, err))
    return 1;
  if (m.need_mod) {
    // gcond = gce(gsum), gsum = global_embed(glob) + time_embed(t): dL/dgsum feeds both
    const bool below = has_target(m, "time_embed.") || has_target(m, "global_embed.");
    if (mlp_silu_bwd(m, "dit.gce.", true, m.gsum_b, B, m.gce_h, m.gce_hb, m.gcond, m.dgcond, below ? m.dgsum : nullptr,
                     err))
      return 1;
    if (below) {
      if (mlp_silu_bwd(m, "dit.global_embed.", false, m.glob_b, B, m.g_h, m.g_hb, m.g_y, m.dgsum, nullptr, err)) return 1;
      if (mlp_silu_bwd(m, "dit.time_embed.", true, m.tfeat_b, B, m.te_h, m.te_hb, m.te, m.dgsum, nullptr, err)) return 1;
    }
  }
  // ---------------- adapter gradients, grouped over every adapter of the step: the DoRA row terms
  // (dm, dB, and the cb / c3 factors of dA), then one launch for all dB += s dz^T u,
  // dA += du^T x and dA += cb W contractions, then dA += 2 c3 A
  if (m.r16_grads.table) {
    if (m.dora) {
      if (cudaMemsetAsync(m.c3_all, 0, sizeof(float) * 256 * std::max(m.n_active, 1), c->stream) != cudaSuccess)
        return check_launch("memset", err);
      if (k_dora_bwd_all(c, m.prep_desc, nt, m.max_out, err)) return 1;
    }
    if (r16_group_run(c, m.r16_grads, "lora.grads", err)) return 1;
    if (m.dora && k_dora_da_c3_all(c, m.prep_desc, nt, err)) return 1;
  }
  if (m.np > 0 && k_scale(c, m.g, m.np, 1.0f / gscale, err)) return 1;
  return 0;
}

// The step through its recorded CUDA graph where that is possible: the first call at a shape (and
// context / model generation) runs eagerly and allocates everything, the second records the
// graph and replays it, later ones only replay.  A stream that is being captured (the caller
// records its own graph), profiling timing, or a failed recording runs the step eagerly.
static int run_step(DitModel& m, std::string& err) {
  Ctx* c = m.c;
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(c->stream, &cs) != cudaSuccess) cudaGetLastError();
  if (!c->step_graph || c->timing || cs != cudaStreamCaptureStatusNone) return dit_step(m, err);
  if (m.step_exec && m.gB == m.B && m.gT == m.T && m.gC == m.C && m.g_cgen == c->gen && m.g_mgen == m.gen) {
    if (cudaGraphLaunch(m.step_exec, c->stream) != cudaSuccess) return check_launch("step graph", err);
    for (const auto& pl : m.g_launches) {
      auto it = std::find_if(c->prof.begin(), c->prof.end(), [&](const ProfEntry& e) { return e.name == pl.first; });
      if (it == c->prof.end()) {
        c->prof.emplace_back();
        c->prof.back().name = pl.first;
        it = c->prof.end() - 1;
      }
      it->launches += pl.second;
    }
    return 0;
  }
  if (m.step_exec) {
    cudaGraphExecDestroy(m.step_exec);
    m.step_exec = nullptr;
  }
  const bool same = m.warm && m.wB == m.B && m.wT == m.T && m.wC == m.C && m.w_cgen == c->gen && m.w_mgen == m.gen;
  if (!same) {   // first call at this key: eager (allocations, caches)
    const int rc = dit_step(m, err);
    m.warm = rc == 0;
    m.wB = m.B; m.wT = m.T; m.wC = m.C; m.w_cgen = c->gen; m.w_mgen = m.gen;
    return rc;
  }
  // recorded on a private stream (the caller's may be the legacy default stream, which cannot
  // be captured); the graph is then launched on the caller's stream
  if (!m.cap_stream && cudaStreamCreateWithFlags(&m.cap_stream, cudaStreamNonBlocking) != cudaSuccess) {
    cudaGetLastError();
    m.cap_stream = nullptr;
    return dit_step(m, err);
  }
  std::vector<long long> before(c->prof.size());
  for (size_t i = 0; i < c->prof.size(); ++i) before[i] = c->prof[i].launches;
  const cudaStream_t user = c->stream;
  if (cudaStreamBeginCapture(m.cap_stream, cudaStreamCaptureModeThreadLocal) != cudaSuccess) {
    cudaGetLastError();
    return dit_step(m, err);
  }
  c->stream = m.cap_stream;
  std::string e2;
  const int rc = dit_step(m, e2);
  c->stream = user;
  cudaGraph_t g = nullptr;
  const cudaError_t ce = cudaStreamEndCapture(m.cap_stream, &g);
  cudaGraphExec_t exec = nullptr;
  const bool ok = rc == 0 && ce == cudaSuccess && g && cudaGraphInstantiate(&exec, g, 0) == cudaSuccess;
  if (g) cudaGraphDestroy(g);
  if (!ok) {   // nothing recorded ran: run the step eagerly and stay eager at this key
    cudaGetLastError();
    if (exec) cudaGraphExecDestroy(exec);
    m.warm = false;
    for (size_t i = 0; i < c->prof.size() && i < before.size(); ++i) c->prof[i].launches = before[i];
    return dit_step(m, err);
  }
  m.g_launches.clear();
  for (size_t i = 0; i < c->prof.size(); ++i) {
    const long long d = c->prof[i].launches - (i < before.size() ? before[i] : 0);
    if (d) m.g_launches.emplace_back(c->prof[i].name, d);
  }
  m.step_exec = exec;
  m.gB = m.B; m.gT = m.T; m.gC = m.C; m.g_cgen = c->gen; m.g_mgen = m.gen;
  if (cudaGraphLaunch(exec, c->stream) != cudaSuccess) return check_launch("step graph", err);
  return 0;
}

}  // namespace sa3k

using namespace sa3k;

struct sa3k_dit {
  DitModel m;
};

// ggml extents (ne0 = the contiguous dimension, ne1 = rows; 1 for vectors) of every tensor the
// step reads, from the config (the shapes dit_block / dit_head / dit_tail use, src/dit.h:106-147);
// false for a name the DiT does not have
static bool dit_tensor_shape(const sa3k_dit_config& k, const std::string& n, int64_t& ne0, int64_t& ne1) {
  const int64_t D = k.dim, io = k.io, cd = k.cond_dim, td = k.time_dim, I = k.ff_inner;
  const int64_t dq = k.differential ? 2 : 1;
  auto set = [&](int64_t a, int64_t b) { ne0 = a; ne1 = b; return true; };
  static const char* const kPrefix = "dit.";
  if (n.compare(0, 4, kPrefix) != 0) return false;
  const std::string r = n.substr(4);
  if (!r.empty() && r[0] >= '0' && r[0] <= '9') {
    const size_t dot = r.find('.');
    if (dot == std::string::npos) return false;
    const long l = std::strtol(r.substr(0, dot).c_str(), nullptr, 10);
    if (l < 0 || l >= k.depth) return false;
    const std::string b = r.substr(dot + 1);
    if (b == "ssg") return set(6 * D, 1);
    if (b == "pre_norm.gamma" || b == "cross_norm.gamma" || b == "ff_norm.gamma" || b == "ff.out.bias") return set(D, 1);
    if (b == "self.q_norm.gamma" || b == "self.k_norm.gamma" || b == "cross.q_norm.gamma" || b == "cross.k_norm.gamma")
      return set(k.head_dim, 1);
    if (b == "self.qkv.weight") return set(D, (dq + 1 + dq) * D);
    if (b == "self.out.weight" || b == "cross.out.weight") return set(D, D);
    if (b == "cross.q.weight") return set(D, dq * D);
    if (b == "cross.kv.weight") return set(D, (dq + 1) * D);
    if (b == "ff.proj.weight") return set(D, 2 * I);
    if (b == "ff.proj.bias") return set(2 * I, 1);
    if (b == "ff.out.weight") return set(I, D);
    if (k.local_dim > 0) {
      if (b == "local.0.weight") return set(k.local_dim, D);
      if (b == "local.2.weight") return set(D, D);
      if (b == "local.0.bias" || b == "local.2.bias") return set(D, 1);
    }
    return false;
  }
  if (r == "time_embed.0.weight") return set(td, D);
  if (r == "time_embed.0.bias" || r == "time_embed.2.bias" || r == "gce.0.bias") return set(D, 1);
  if (r == "time_embed.2.weight" || r == "global_embed.2.weight" || r == "gce.0.weight" ||
      r == "cond_embed.2.weight")
    return set(D, D);
  if (r == "global_embed.0.weight" || r == "cond_embed.0.weight") return set(cd, D);
  if (r == "gce.2.weight") return set(D, 6 * D);
  if (r == "gce.2.bias") return set(6 * D, 1);
  if (r == "pre_conv.weight" || r == "post_conv.weight") return set(io, io);
  if (r == "proj_in.weight") return set(io, D);
  if (r == "proj_out.weight") return set(D, io);
  if (r == "memory_tokens") return set(D, k.mem_tokens);
  return false;
}

static int dfail(char* err, int len, const std::string& msg) {
  if (err && len > 0) {
    std::strncpy(err, msg.c_str(), (size_t)len - 1);
    err[len - 1] = 0;
  }
  return 1;
}

extern "C" {

int sa3k_dit_create(sa3k_ctx* ctx, const sa3k_dit_config* cfg, sa3k_dit** out, char* err, int err_len) {
  if (!ctx || !cfg || !out) return dfail(err, err_len, "NULL argument");
  if (cfg->head_dim != 64) return dfail(err, err_len, "head_dim must be 64");
  if (cfg->dim != cfg->heads * cfg->head_dim) return dfail(err, err_len, "dim must equal heads * head_dim");
  if (cfg->dim % 64 || cfg->ff_inner % 64 || cfg->io % 64 || cfg->cond_dim % 64 || cfg->time_dim % 64)
    return dfail(err, err_len, "dim, ff_inner, io, cond_dim and time_dim must be multiples of 64");
  if (cfg->rot != 32 && cfg->rot != 64) return dfail(err, err_len, "rot must be 32 or 64");
  sa3k_dit* d = new (std::nothrow) sa3k_dit();
  if (!d) return dfail(err, err_len, "out of host memory");
  d->m.c = &ctx->c;
  d->m.handle = ctx;
  d->m.device = ctx->c.device;
  d->m.cfg = *cfg;
  *out = d;
  return 0;
}

void sa3k_dit_free(sa3k_dit* d) {
  if (!d) return;
  // the model's context may already be gone: use the device recorded at creation only
  // (cudaFree waits for the device's outstanding work)
  cudaSetDevice(d->m.device);
  delete d;
}

int sa3k_dit_set_tensor(sa3k_dit* d, const char* name, int type, const void* host, int64_t ne0, int64_t ne1,
                        char* err, int err_len) {
  if (!d || !name || !host) return dfail(err, err_len, "NULL argument");
  DitModel& m = d->m;
  cudaSetDevice(m.c->device);
  const std::string n(name);
  ++m.gen;
  int64_t x0 = 0, x1 = 0;
  if (!dit_tensor_shape(m.cfg, n, x0, x1)) return dfail(err, err_len, "not a tensor of this DiT: " + n);
  if (ne0 != x0 || (ne1 > 0 ? ne1 : 1) != x1)
    return dfail(err, err_len, n + ": shape [" + std::to_string(ne1) + "][" + std::to_string(ne0) + "], expected [" +
                                   std::to_string(x1) + "][" + std::to_string(x0) + "]");
  const bool is_weight = n.size() > 7 && n.compare(n.size() - 7, 7, ".weight") == 0;
  std::string e;
  if (is_weight && ne0 % 64 != 0) {
    // kept on the host (only the inpaint local.0 projection has such a width here)
    if (m.host_w.count(n)) return dfail(err, err_len, "tensor set twice: " + n);
    if (type != SA3K_TYPE_F32 && type != SA3K_TYPE_F16)
      return dfail(err, err_len, n + ": a weight whose width is not a multiple of 64 must be F32 or F16");
    std::vector<float> v((size_t)(ne0 * ne1));
    if (type == SA3K_TYPE_F32) {
      std::memcpy(v.data(), host, v.size() * 4);
    } else {
      const __half* hh = static_cast<const __half*>(host);
      for (size_t i = 0; i < v.size(); ++i) v[i] = __half2float(hh[i]);
    }
    // a device copy zero-padded to a multiple of 64 in `in` for the GEMM engine (the padding
    // meets zero columns of the padded input: the products are those of the logical weight)
    const int64_t ld = (ne0 + 63) / 64 * 64;
    std::vector<float> pad((size_t)(ld * ne1), 0.0f);
    for (int64_t o = 0; o < ne1; ++o) std::memcpy(&pad[(size_t)(o * ld)], &v[(size_t)(o * ne0)], 4 * (size_t)ne0);
    sa3k_weight* hp = nullptr;
    if (sa3k_weight_upload(m.handle, SA3K_TYPE_F32, pad.data(), ld, ne1, &hp, err, err_len)) return 1;
    m.weights.push_back(hp);
    m.Wpad[n] = &hp->w;
    m.host_w[n] = std::move(v);
    m.host_shape[n] = {ne0, ne1};
    return 0;
  }
  if (is_weight) {
    if (m.W.count(n)) return dfail(err, err_len, "tensor set twice: " + n);
    // the public upload path repacks the GGUF blocks; the model owns the handle afterwards
    sa3k_weight* h = nullptr;
    if (sa3k_weight_upload(m.handle, type, host, ne0, ne1, &h, err, err_len)) return 1;
    m.weights.push_back(h);
    m.W[n] = &h->w;
    return 0;
  }
  if (type != SA3K_TYPE_F32) return dfail(err, err_len, "1-D / non-weight tensors must be F32: " + n);
  const size_t bytes = (size_t)ne0 * (size_t)(ne1 > 0 ? ne1 : 1) * 4;
  float* dv = static_cast<float*>(dmalloc(m, bytes, e));
  if (!dv) return dfail(err, err_len, e);
  if (cudaMemcpy(dv, host, bytes, cudaMemcpyHostToDevice) != cudaSuccess) return dfail(err, err_len, "copy failed");
  m.V[n] = dv;
  return 0;
}

int sa3k_dit_init_adapters(sa3k_dit* d, const char* adapter_type, int rank, float alpha, const char* const* names,
                           int n, char* err, int err_len) {
  if (!d || !adapter_type || !names || n <= 0) return dfail(err, err_len, "NULL argument");
  DitModel& m = d->m;
  cudaSetDevice(m.c->device);
  const std::string at(adapter_type);
  // lora / dora-rows run functionally; the other families through a materialized W_eff
  // (src/train_dit.h:90-164)
  const bool xs = at.size() > 3 && at.compare(at.size() - 3, 3, "-xs") == 0;
  const std::string fam = xs ? at.substr(0, at.size() - 3) : at;
  if (fam != "lora" && fam != "dora-rows" && fam != "dora-cols" && fam != "bora")
    return dfail(err, err_len, "unknown adapter type " + at);
  if (rank < 1 || rank > 16) return dfail(err, err_len, "rank must be 1..16");
  if (!m.tg.empty()) return dfail(err, err_len, "adapters already initialised");
  ++m.gen;
  m.adapter_type = at;
  m.mat = xs || fam == "dora-cols" || fam == "bora";
  const bool mrows = fam == "dora-rows" || fam == "bora", mcols = fam == "dora-cols" || fam == "bora";
  m.dora = !m.mat && at == "dora-rows";
  m.rank = rank;
  m.alpha = alpha;
  m.s = alpha / (float)rank;
  int64_t off = 0;
  std::string e;
  for (int i = 0; i < n; ++i) {
    DitTarget t;
    t.name = names[i];
    auto it = m.W.find(t.name);
    auto ht = m.host_shape.find(t.name);
    if (it == m.W.end() && ht == m.host_shape.end())
      return dfail(err, err_len, "adapter target has no weight: " + t.name);
    t.inert = t.name.find(".local.") != std::string::npos;
    if (it != m.W.end()) {
      t.w = it->second;
      t.in = t.w->in;
      t.out = t.w->out;
    } else {
      t.in = ht->second.first;
      t.out = ht->second.second;
    }
    if (!t.inert && !t.w) return dfail(err, err_len, "adapter target has no device weight: " + t.name);
    t.mat = m.mat;
    if (!t.inert && !t.mat) t.act = m.n_active++;
    if (m.mat && xs) {   // trainable M_xs only; A / B absent (offA = offB = -1)
      t.offA = t.offB = -1;
      t.offX = off; off += (int64_t)rank * rank;
    } else {
      t.offA = off; off += (int64_t)rank * t.in;
      t.offB = off; off += t.out * rank;
    }
    if (m.dora || (m.mat && mrows)) { t.offM = off; off += t.out; }
    if (m.mat && mcols) {
      if (mrows) { t.offMc = off; off += t.in; }    // bora: m_r [out] at offM, m_c [in] at offMc
      else { t.offM = off; off += t.in; }          // dora-cols: m [in] at offM
    }
    m.tix[t.name] = (int)m.tg.size();
    m.tg.push_back(t);
  }
  m.np = off;
  for (float** b : {&m.p, &m.g, &m.am, &m.av}) {
    *b = static_cast<float*>(dmalloc(m, (size_t)off * 4, e));
    if (!*b) return dfail(err, err_len, e);
    cudaMemsetAsync(*b, 0, (size_t)off * 4, m.c->stream);
  }
  if (m.mat) {
    for (DitTarget& t : m.tg) {
      // magnitudes start at the base's row / column norms (train_row_norms / train_col_norms,
      // src/train_lora.h:141-190, 262-269)
      const int64_t om = t.offM, oc = mcols ? (mrows ? t.offMc : t.offM) : -1;
      if (t.w) {
        if (mrows && weight_row_norms(m.c, t.w, 1e-12f, nullptr, m.p + om, e)) return dfail(err, err_len, e);
        if (mcols && mat_col_norms(m.c, t.w, m.p + oc, e)) return dfail(err, err_len, e);
      } else if (mrows || mcols) {   // a host-only weight: the same f64 sums on the host
        const std::vector<float>& hw = m.host_w[t.name];
        std::vector<float> rn((size_t)t.out), cn((size_t)t.in);
        std::vector<double> ca((size_t)t.in, 0.0);
        for (int64_t o = 0; o < t.out; ++o) {
          double acc = 0.0;
          for (int64_t i = 0; i < t.in; ++i) {
            const double v = hw[(size_t)(o * t.in + i)];
            acc += v * v;
            ca[(size_t)i] += v * v;
          }
          rn[(size_t)o] = (float)std::sqrt(acc);
        }
        for (int64_t i = 0; i < t.in; ++i) cn[(size_t)i] = (float)std::sqrt(ca[(size_t)i]);
        if ((mrows && cudaMemcpy(m.p + om, rn.data(), 4 * rn.size(), cudaMemcpyHostToDevice) != cudaSuccess) ||
            (mcols && cudaMemcpy(m.p + oc, cn.data(), 4 * cn.size(), cudaMemcpyHostToDevice) != cudaSuccess))
          return dfail(err, err_len, "magnitude init copy failed");
      }
      if (t.inert) continue;
      MatTarget& mt = t.mt;
      mt.xs = xs; mt.rows = mrows; mt.cols = mcols;
      mt.rank = rank; mt.s = m.s; mt.w = t.w; mt.in = t.in; mt.out = t.out;
      if (xs) {
        t.U = static_cast<float*>(dmalloc(m, 4 * (size_t)t.out * rank, e));
        t.Vb = static_cast<float*>(dmalloc(m, 4 * (size_t)t.in * rank, e));
        if (!t.U || !t.Vb) return dfail(err, err_len, e);
        cudaMemsetAsync(t.U, 0, 4 * (size_t)t.out * rank, m.c->stream);
        cudaMemsetAsync(t.Vb, 0, 4 * (size_t)t.in * rank, m.c->stream);
        mt.U = t.U; mt.Vb = t.Vb; mt.M = m.p + t.offX; mt.dM = m.g + t.offX;
      } else {
        mt.A = m.p + t.offA; mt.B = m.p + t.offB; mt.dA = m.g + t.offA; mt.dB = m.g + t.offB;
      }
      if (mrows) { mt.mr = m.p + t.offM; mt.dmr = m.g + t.offM; }
      if (mcols) { mt.mc = m.p + oc; mt.dmc = m.g + oc; }
      void* mem = dmalloc(m, mat_target_bytes(t.in, t.out, rank), e);
      if (!mem) return dfail(err, err_len, e);
      mat_target_bind(mt, mem);
    }
    if (cudaStreamSynchronize(m.c->stream) != cudaSuccess) return dfail(err, err_len, "adapter init failed");
    return 0;
  }
  size_t prep_bytes = 256;
  for (DitTarget& t : m.tg)
    if (!t.inert) prep_bytes += adapter_prep_bytes(t.in, t.out, m.dora) + 256;
  char* pm = static_cast<char*>(dmalloc(m, prep_bytes, e));
  if (!pm) return dfail(err, err_len, e);
  for (DitTarget& t : m.tg) {
    AdapterPrep& p = t.prep;
    p.rank = rank; p.in = t.in; p.out = t.out; p.s = m.s;
    p.A = m.p + t.offA; p.B = m.p + t.offB;
    if (m.dora) {
      t.bns = static_cast<float*>(dmalloc(m, (size_t)t.out * 4, e));
      if (!t.bns) return dfail(err, err_len, e);
      p.m = m.p + t.offM;
      p.bns = t.bns;
      // base_norm_sq and the magnitude init = row norms of the dequantized base
      // (train_row_norm_sq / train_row_norms, src/train_lora.h:141-174,262-263)
      if (t.w) {
        if (weight_row_norms(m.c, t.w, 1e-12f, t.bns, m.p + t.offM, e)) return dfail(err, err_len, e);
      } else {   // a host-only weight: the same f64 sums on the host
        const std::vector<float>& hw = m.host_w[t.name];
        std::vector<float> nsq((size_t)t.out), nrm((size_t)t.out);
        for (int64_t o = 0; o < t.out; ++o) {
          double acc = 0.0;
          for (int64_t i = 0; i < t.in; ++i) acc += (double)hw[(size_t)(o * t.in + i)] * hw[(size_t)(o * t.in + i)];
          nsq[(size_t)o] = (float)(acc + (double)t.in * 1e-12);
          nrm[(size_t)o] = (float)std::sqrt(acc);
        }
        if (cudaMemcpy(t.bns, nsq.data(), 4 * nsq.size(), cudaMemcpyHostToDevice) != cudaSuccess ||
            cudaMemcpy(m.p + t.offM, nrm.data(), 4 * nrm.size(), cudaMemcpyHostToDevice) != cudaSuccess)
          return dfail(err, err_len, "magnitude init copy failed");
      }
    }
    if (t.inert) continue;
    adapter_bind(p, pm);
    pm += adapter_prep_bytes(t.in, t.out, m.dora) + 256;
  }
  // device descriptors of the active adapters for the grouped preparation kernels of every step
  std::vector<PrepDesc> descs;
  for (DitTarget& t : m.tg) {
    if (t.inert) continue;
    const AdapterPrep& p = t.prep;
    PrepDesc pd{};
    pd.A = p.A; pd.B = p.B; pd.m = p.m; pd.bns = p.bns;
    pd.rank = p.rank; pd.dora = p.dora() ? 1 : 0; pd.s = p.s; pd.in = p.in; pd.out = p.out;
    pd.a_h = p.a_h; pd.at_x = p.at_x; pd.b_x = p.b_x; pd.bt_h = p.bt_h;
    pd.pt = p.pt; pd.aat = p.aat; pd.nsq = p.nsq; pd.g = p.g;
    descs.push_back(pd);
    m.max_out = std::max(m.max_out, p.out);
  }
  m.prep_desc = static_cast<PrepDesc*>(dmalloc(m, sizeof(PrepDesc) * std::max<size_t>(descs.size(), 1), e));
  if (!m.prep_desc) return dfail(err, err_len, e);
  if (!descs.empty() &&
      cudaMemcpy(m.prep_desc, descs.data(), sizeof(PrepDesc) * descs.size(), cudaMemcpyHostToDevice) != cudaSuccess)
    return dfail(err, err_len, "adapter descriptor upload failed");
  if (cudaStreamSynchronize(m.c->stream) != cudaSuccess) return dfail(err, err_len, "adapter init failed");
  return 0;
}

int64_t sa3k_dit_adapter_size(const sa3k_dit* d) { return d ? d->m.np : 0; }

int sa3k_dit_adapter_offsets(const sa3k_dit* d, int idx, int64_t* offA, int64_t* offB, int64_t* offM) {
  if (!d || idx < 0 || idx >= (int)d->m.tg.size()) return 1;
  const DitTarget& t = d->m.tg[(size_t)idx];
  if (offA) *offA = t.offA;
  if (offB) *offB = t.offB;
  if (offM) *offM = t.offM;
  return 0;
}

int sa3k_dit_adapter_layout(const sa3k_dit* d, int idx, int64_t* offs) {
  if (!d || !offs || idx < 0 || idx >= (int)d->m.tg.size()) return 1;
  const DitTarget& t = d->m.tg[(size_t)idx];
  const bool bora = t.offMc >= 0;
  const bool cols = d->m.mat && (bora || d->m.adapter_type.rfind("dora-cols", 0) == 0);
  offs[0] = t.offA;
  offs[1] = t.offB;
  offs[2] = cols && !bora ? -1 : t.offM;   // row magnitude [out]
  offs[3] = bora ? t.offMc : (cols ? t.offM : -1);   // column magnitude [in]
  offs[4] = t.offX;
  return 0;
}

int sa3k_dit_set_xs_bases(sa3k_dit* d, const char* name, const float* U, const float* V, char* err, int err_len) {
  if (!d || !name || !U || !V) return dfail(err, err_len, "NULL argument");
  DitModel& m = d->m;
  auto it = m.tix.find(name);
  if (it == m.tix.end()) return dfail(err, err_len, std::string("no adapter target ") + name);
  DitTarget& t = m.tg[(size_t)it->second];
  if (!t.U) return dfail(err, err_len, "the adapters are not of an -xs family (or the target is inert)");
  cudaSetDevice(m.c->device);
  if (cudaMemcpy(t.U, U, 4 * (size_t)t.out * m.rank, cudaMemcpyHostToDevice) != cudaSuccess ||
      cudaMemcpy(t.Vb, V, 4 * (size_t)t.in * m.rank, cudaMemcpyHostToDevice) != cudaSuccess)
    return dfail(err, err_len, "basis copy failed");
  return 0;
}

int sa3k_dit_adapter_buffer(sa3k_dit* d, int which, float** dev_ptr, char* err, int err_len) {
  if (!d || !dev_ptr) return dfail(err, err_len, "NULL argument");
  float* b[4] = {d->m.p, d->m.g, d->m.am, d->m.av};
  if (which < 0 || which > 3) return dfail(err, err_len, "which must be 0 (params), 1 (grads), 2 (m), 3 (v)");
  *dev_ptr = b[which];
  return 0;
}

int sa3k_dit_adapter_copy(sa3k_dit* d, int which, float* buf, int64_t offset, int64_t count, int to_model,
                          char* err, int err_len) {
  if (!d || !buf) return dfail(err, err_len, "NULL argument");
  float* b[4] = {d->m.p, d->m.g, d->m.am, d->m.av};
  if (which < 0 || which > 3) return dfail(err, err_len, "which must be 0..3");
  if (offset < 0 || count < 0 || offset + count > d->m.np) return dfail(err, err_len, "range outside the state");
  cudaSetDevice(d->m.c->device);
  float* dev = b[which] + offset;
  const cudaError_t e = to_model ? cudaMemcpyAsync(dev, buf, (size_t)count * 4, cudaMemcpyDefault, d->m.c->stream)
                                 : cudaMemcpyAsync(buf, dev, (size_t)count * 4, cudaMemcpyDefault, d->m.c->stream);
  if (e != cudaSuccess || cudaStreamSynchronize(d->m.c->stream) != cudaSuccess) return dfail(err, err_len, "copy failed");
  return 0;
}

int sa3k_dit_zero_grads(sa3k_dit* d, char* err, int err_len) {
  if (!d) return dfail(err, err_len, "NULL argument");
  cudaSetDevice(d->m.c->device);
  if (cudaMemsetAsync(d->m.g, 0, (size_t)d->m.np * 4, d->m.c->stream) != cudaSuccess)
    return dfail(err, err_len, "memset failed");
  return 0;
}

int sa3k_dit_forward_backward(sa3k_dit* d, int B, int T, int ctx_len, const float* x_t, const float* target,
                              const float* t_feat, const float* cross, const float* global, float* loss,
                              char* err, int err_len) {
  if (!d || !x_t || !target || !t_feat || !cross || !global) return dfail(err, err_len, "NULL argument");
  DitModel& m = d->m;
  if (m.tg.empty()) return dfail(err, err_len, "no adapters: call sa3k_dit_init_adapters first");
  if (B <= 0 || B > 64 || T <= 0 || ctx_len <= 0) return dfail(err, err_len, "bad batch shape");
  cudaSetDevice(m.c->device);
  std::string e;
  if (alloc_acts(m, B, T, ctx_len, e)) return dfail(err, err_len, e);
  const sa3k_dit_config& k = m.cfg;
  const cudaStream_t st = m.c->stream;
  const int64_t MT = (int64_t)B * T;
  bool ok = cudaMemcpyAsync(m.in_x, x_t, sizeof(float) * MT * k.io, cudaMemcpyDefault, st) == cudaSuccess &&
            cudaMemcpyAsync(m.in_target, target, sizeof(float) * MT * k.io, cudaMemcpyDefault, st) == cudaSuccess &&
            cudaMemcpyAsync(m.in_tfeat, t_feat, sizeof(float) * B * k.time_dim, cudaMemcpyDefault, st) == cudaSuccess &&
            cudaMemcpyAsync(m.in_cross, cross, sizeof(float) * (size_t)B * ctx_len * k.cond_dim, cudaMemcpyDefault,
                            st) == cudaSuccess &&
            cudaMemcpyAsync(m.in_glob, global, sizeof(float) * B * k.cond_dim, cudaMemcpyDefault, st) == cudaSuccess;
  if (!ok) return dfail(err, err_len, "input copy failed");
  if (run_step(m, e)) return dfail(err, err_len, e);
  if (loss && cudaMemcpyAsync(loss, m.loss, sizeof(float) * B, cudaMemcpyDefault, st) != cudaSuccess)
    return dfail(err, err_len, "loss copy failed");
  return 0;
}

int sa3k_dit_forward_backward_inpaint(sa3k_dit* d, int B, int T, int ctx_len, const float* x_t, const float* target,
                                      const float* t_feat, const float* cross, const float* global,
                                      const float* local, const float* loss_weight, float* loss, char* err,
                                      int err_len) {
  if (!d || !local || !loss_weight) return dfail(err, err_len, "NULL argument");
  DitModel& m = d->m;
  const sa3k_dit_config& k = m.cfg;
  if (k.local_dim <= 0)
    return dfail(err, err_len, "inpainting requested but the DiT has no local-cond weights (dit.local_dim <= 0)");
  for (const DitTarget& t : m.tg)
    if (t.name.find(".local.") != std::string::npos)
      return dfail(err, err_len, "adapters on the local.* projections are not trained with an inpaint input here "
                                 "(the core scope leaves them out): " + t.name);
  if (m.tg.empty()) return dfail(err, err_len, "no adapters: call sa3k_dit_init_adapters first");
  if (B <= 0 || B > 64 || T <= 0 || ctx_len <= 0) return dfail(err, err_len, "bad batch shape");
  cudaSetDevice(m.c->device);
  std::string e;
  if (alloc_acts(m, B, T, ctx_len, e)) return dfail(err, err_len, e);
  const int64_t MT = (int64_t)B * T;
  const cudaStream_t st = m.c->stream;
  if (cudaMemcpyAsync(m.in_local, local, sizeof(float) * MT * k.local_dim, cudaMemcpyDefault, st) != cudaSuccess ||
      cudaMemcpyAsync(m.in_lw, loss_weight, sizeof(float) * MT * k.io, cudaMemcpyDefault, st) != cudaSuccess)
    return dfail(err, err_len, "input copy failed");
  // the inpaint step runs eagerly (the recorded step graph is the plain one)
  const bool graph = m.c->step_graph;
  m.c->step_graph = false;
  m.inpaint = true;
  const int rc = sa3k_dit_forward_backward(d, B, T, ctx_len, x_t, target, t_feat, cross, global, loss, err, err_len);
  m.inpaint = false;
  m.c->step_graph = graph;
  return rc;
}

int sa3k_dit_apply_adamw(sa3k_dit* d, int count, const sa3k_adamw_params* hp, int step, double* grad_norm_out,
                         char* err, int err_len) {
  if (!d) return dfail(err, err_len, "NULL argument");
  DitModel& m = d->m;
  return sa3k_average_clip_adamw(m.handle, m.p, m.g, m.am, m.av, m.np, count, hp, step, grad_norm_out, err, err_len);
}

int sa3k_dit_dp_apply_adamw(sa3k_dit* d, sa3k_dp_comm* comm, int samples_per_rank, const sa3k_adamw_params* hp,
                            int step, double* grad_norm_out, char* err, int err_len) {
  if (!d || !comm) return dfail(err, err_len, "NULL argument");
  DitModel& m = d->m;
  return sa3k_dp_allreduce_adamw(m.handle, comm, m.p, m.g, m.am, m.av, m.np, samples_per_rank, hp, step,
                                 grad_norm_out, err, err_len);
}


// ------------------------------------------------------------------ adapter / trainer-state files
// Targets in the reference's order (enumerate_train_lora_targets sorts them by weight name,
// src/train_lora.h:97-117), with their file stems (the weight name without ".weight").
static std::vector<size_t> file_order(const DitModel& m) {
  std::vector<size_t> o(m.tg.size());
  for (size_t i = 0; i < o.size(); ++i) o[i] = i;
  std::sort(o.begin(), o.end(), [&](size_t a, size_t b) { return m.tg[a].name < m.tg[b].name; });
  return o;
}

static std::string stem_of(const std::string& n) {
  return n.size() > 7 && n.compare(n.size() - 7, 7, ".weight") == 0 ? n.substr(0, n.size() - 7) : n;
}

static int fetch_flat(DitModel& m, const float* dev, std::vector<float>& host, std::string& err) {
  host.assign((size_t)m.np, 0.f);
  if (cudaStreamSynchronize(m.c->stream) != cudaSuccess ||
      cudaMemcpy(host.data(), dev, sizeof(float) * (size_t)m.np, cudaMemcpyDeviceToHost) != cudaSuccess) {
    cudaGetLastError();
    err = "adapter state copy to the host failed";
    return 1;
  }
  return 0;
}

static int store_flat(DitModel& m, float* dev, const std::vector<float>& host, std::string& err) {
  if (cudaStreamSynchronize(m.c->stream) != cudaSuccess ||
      cudaMemcpy(dev, host.data(), sizeof(float) * (size_t)m.np, cudaMemcpyHostToDevice) != cudaSuccess) {
    cudaGetLastError();
    err = "adapter state copy to the device failed";
    return 1;
  }
  return 0;
}

static std::string adapter_type_of(const DitModel& m) { return m.adapter_type; }

// The trainable tensors of one target in the flat state, named and ordered as the reference's
// adapter and trainer-state files hold them (src/train_checkpoint.h:68-99, src/train_resume.h:
// 319-331): lora_A, lora_B, M_xs, magnitude (dora-rows [out] / dora-cols [in]), magnitude_r,
// magnitude_c.
struct Part {
  const char* kind;
  int64_t off, count;
};
static std::vector<Part> target_parts(const DitModel& m, const DitTarget& t) {
  std::vector<Part> v;
  if (t.offA >= 0) v.push_back({"lora_A", t.offA, (int64_t)m.rank * t.in});
  if (t.offB >= 0) v.push_back({"lora_B", t.offB, t.out * m.rank});
  if (t.offX >= 0) v.push_back({"M_xs", t.offX, (int64_t)m.rank * m.rank});
  const bool cols = m.adapter_type.rfind("dora-cols", 0) == 0;
  if (t.offMc >= 0) {
    v.push_back({"magnitude_r", t.offM, t.out});
    v.push_back({"magnitude_c", t.offMc, t.in});
  } else if (t.offM >= 0) {
    v.push_back({"magnitude", t.offM, cols ? t.in : t.out});
  }
  return v;
}

static int write_adapter_file(DitModel& m, const std::string& path, std::string& err) {
  std::vector<float> p;
  if (fetch_flat(m, m.p, p, err)) return 1;
  std::vector<AdapterTargetView> v;
  std::vector<std::vector<float>> bases;   // the -xs U / V of each target, read back
  bases.reserve(2 * m.tg.size());
  for (size_t i : file_order(m)) {
    const DitTarget& t = m.tg[i];
    AdapterTargetView a;
    a.stem = stem_of(t.name);
    a.in = t.in;
    a.out = t.out;
    for (const Part& q : target_parts(m, t)) {
      const float* d = p.data() + q.off;
      const std::string k = q.kind;
      if (k == "lora_A") a.A = d;
      else if (k == "lora_B") a.B = d;
      else if (k == "M_xs") a.M = d;
      else if (k == "magnitude") { a.m = d; a.m_len = q.count; }
      else if (k == "magnitude_r") a.m_r = d;
      else a.m_c = d;
    }
    if (t.offX >= 0) {
      if (!t.U) {
        err = "the -xs target " + t.name + " has no device bases to write";
        return 1;
      }
      bases.emplace_back((size_t)(t.out * m.rank));
      bases.emplace_back((size_t)(t.in * m.rank));
      if (cudaMemcpy(bases[bases.size() - 2].data(), t.U, 4 * (size_t)t.out * m.rank, cudaMemcpyDeviceToHost) !=
              cudaSuccess ||
          cudaMemcpy(bases.back().data(), t.Vb, 4 * (size_t)t.in * m.rank, cudaMemcpyDeviceToHost) != cudaSuccess) {
        err = "basis read-back failed";
        return 1;
      }
      a.U = bases[bases.size() - 2].data();
      a.V = bases.back().data();
    }
    v.push_back(a);
  }
  return write_adapter_gguf(path, adapter_type_of(m), m.rank, m.alpha, v, err) ? 0 : 1;
}

// The adapter values of `path` into the host copy `p` of the flat parameters, with the checks of
// train_restore_adapter_values (src/train_resume.h:104-148): same type, rank and alpha, the same
// set of targets, every tensor of the expected size.
// bases: for -xs adapters, U and V of each target (index into m.tg), uploaded by the caller once
// the whole file has been checked.
struct XsBases {
  size_t target;
  std::vector<float> U, V;
};
static int read_adapter_file(const DitModel& m, const std::string& path, std::vector<float>& p,
                             std::vector<XsBases>& bases, std::string& err) {
  GgufFile f;
  if (!f.open(path, err)) return 1;
  const GgufValue* ty = f.find("lora.adapter_type");
  const GgufValue* rk = f.find("lora.rank");
  const GgufValue* al = f.find("lora.alpha");
  const std::string type = ty && ty->type == kGgufString ? ty->s : "lora";
  if (!rk || rk->type != kGgufU32 || !al || al->type != kGgufF32) {
    err = "adapter file has no lora.rank / lora.alpha: " + path;
    return 1;
  }
  if (type != adapter_type_of(m) || (int)rk->u != m.rank || (float)al->f != m.alpha) {
    err = "adapter type/rank/alpha of " + path + " does not match the model's adapters";
    return 1;
  }
  const GgufValue* nt = f.find("lora.n_targets");
  size_t stems = 0;
  if (nt && nt->type == kGgufU32) {
    stems = (size_t)nt->u;
  } else {
    for (const std::string& n : f.tensor_order)
      if (n.size() > 7 && n.compare(n.size() - 7, 7, ".lora_A") == 0) ++stems;
  }
  if (stems != m.tg.size()) {
    err = "adapter file target count does not match the model's adapters";
    return 1;
  }
  for (const DitTarget& t : m.tg) {
    const std::string st = stem_of(t.name);
    const std::vector<Part> parts = target_parts(m, t);
    for (const Part& q : parts) {
      std::vector<float> v;
      const std::string name = st + "." + q.kind;
      if (!f.tensors.count(name)) {
        err = "adapter file is missing " + name;
        return 1;
      }
      if (!f.read_f32(name, v, err)) return 1;
      if ((int64_t)v.size() != q.count) {
        err = "adapter tensor shape mismatch: " + name;
        return 1;
      }
      std::copy(v.begin(), v.end(), p.begin() + q.off);
    }
    if (t.offX >= 0) {
      XsBases b;
      b.target = (size_t)(&t - m.tg.data());
      if (!f.tensors.count(st + ".U") || !f.tensors.count(st + ".V")) {
        err = "adapter file is missing the -xs bases of " + st;
        return 1;
      }
      if (!f.read_f32(st + ".U", b.U, err) || !f.read_f32(st + ".V", b.V, err)) return 1;
      if ((int64_t)b.U.size() != t.out * m.rank || (int64_t)b.V.size() != t.in * m.rank) {
        err = "adapter basis shape mismatch: " + st;
        return 1;
      }
      bases.push_back(std::move(b));
    }
  }
  return 0;
}

static int upload_bases(DitModel& m, const std::vector<XsBases>& bases, std::string& err) {
  for (const XsBases& b : bases) {
    const DitTarget& t = m.tg[b.target];
    if (!t.U) continue;   // an inert target keeps no device bases
    if (cudaMemcpy(t.U, b.U.data(), 4 * b.U.size(), cudaMemcpyHostToDevice) != cudaSuccess ||
        cudaMemcpy(t.Vb, b.V.data(), 4 * b.V.size(), cudaMemcpyHostToDevice) != cudaSuccess) {
      err = "basis upload failed";
      return 1;
    }
  }
  return 0;
}

static bool file_exists(const std::string& p) {
  struct stat st;
  return stat(p.c_str(), &st) == 0;
}

static std::string base_name(const std::string& p) {
  const size_t k = p.find_last_of('/');
  return k == std::string::npos ? p : p.substr(k + 1);
}

int sa3k_dit_save_adapter(sa3k_dit* d, const char* path, char* err, int err_len) {
  if (!d || !path) return dfail(err, err_len, "NULL argument");
  DitModel& m = d->m;
  if (m.tg.empty()) return dfail(err, err_len, "no adapters");
  cudaSetDevice(m.c->device);
  std::string e;
  if (write_adapter_file(m, path, e)) return dfail(err, err_len, e);
  return 0;
}

int sa3k_dit_load_adapter(sa3k_dit* d, const char* path, char* err, int err_len) {
  if (!d || !path) return dfail(err, err_len, "NULL argument");
  DitModel& m = d->m;
  if (m.tg.empty()) return dfail(err, err_len, "no adapters: call sa3k_dit_init_adapters first");
  cudaSetDevice(m.c->device);
  std::string e;
  std::vector<float> p((size_t)m.np, 0.f);
  std::vector<XsBases> bases;
  if (read_adapter_file(m, path, p, bases, e) || store_flat(m, m.p, p, e) || upload_bases(m, bases, e))
    return dfail(err, err_len, e);
  return 0;
}

int sa3k_dit_save_checkpoint(sa3k_dit* d, const char* adapter_path, const char* state_path, int64_t step,
                             const sa3k_train_progress* pr, char* err, int err_len) {
  if (!d || !adapter_path || !state_path || !pr) return dfail(err, err_len, "NULL argument");
  DitModel& m = d->m;
  if (m.tg.empty()) return dfail(err, err_len, "no adapters");
  if (step <= 0 || !pr->order || pr->n_order <= 0 || pr->next_sample > (uint64_t)pr->n_order)
    return dfail(err, err_len, "cannot write invalid trainer continuation state");
  const std::string ap(adapter_path), sp(state_path);
  if (file_exists(ap) || file_exists(sp))
    return dfail(err, err_len, "refusing to overwrite an existing immutable training checkpoint at step " +
                                   std::to_string(step));
  cudaSetDevice(m.c->device);
  std::string e;
  std::vector<float> mom, vel;
  if (fetch_flat(m, m.am, mom, e) || fetch_flat(m, m.av, vel, e)) return dfail(err, err_len, e);
  const std::string atmp = ap + ".tmp", stmp = sp + ".tmp";
  std::remove(atmp.c_str());
  std::remove(stmp.c_str());
  auto cleanup = [&]() {
    std::remove(atmp.c_str());
    std::remove(stmp.c_str());
  };
  if (write_adapter_file(m, atmp, e)) {
    cleanup();
    return dfail(err, err_len, e);
  }
  const std::string fp = gguf_file_fingerprint(atmp, e);
  if (fp.empty()) {
    cleanup();
    return dfail(err, err_len, e);
  }
  // trainer state (write_train_state_gguf, src/train_resume.h:336-381)
  GgufWriter w;
  auto s = [](const char* x) { return std::string(x ? x : ""); };
  w.set_str("general.architecture", "sa3-trainer-state");
  w.set_str("general.name", "sa3 native trainer continuation state");
  w.set_u32("trainer.state_version", 1);
  w.set_u64("trainer.step", (uint64_t)step);
  w.set_u64("trainer.epoch", pr->epoch);
  w.set_u64("trainer.next_sample", pr->next_sample);
  w.set_u32("trainer.n_targets", (uint32_t)m.tg.size());
  w.set_str("trainer.adapter_file", base_name(ap));
  w.set_str("trainer.adapter_fingerprint", fp);
  w.set_str("trainer.compatibility", s(pr->compatibility));
  w.set_str("trainer.rng.shuffle", s(pr->rng_shuffle));
  w.set_str("trainer.rng.crop", s(pr->rng_crop));
  w.set_str("trainer.rng.cfg", s(pr->rng_cfg));
  w.set_str("trainer.rng.prompt", s(pr->rng_prompt));
  w.set_str("trainer.rng.inpaint", s(pr->rng_inpaint));
  w.set_str("trainer.rng.diffusion", s(pr->rng_diffusion));
  w.set_arr_u64("trainer.order", std::vector<uint64_t>(pr->order, pr->order + pr->n_order));
  std::vector<std::string> stems;
  for (size_t i : file_order(m)) stems.push_back(stem_of(m.tg[i].name));
  w.set_arr_str("trainer.targets", stems);
  for (size_t i : file_order(m)) {
    const DitTarget& t = m.tg[i];
    const std::string base = "optimizer." + stem_of(t.name) + ".";
    const std::vector<Part> parts = target_parts(m, t);
    for (const Part& q : parts) {
      w.add_f32(base + q.kind + ".m", {q.count}, mom.data() + q.off);
      w.add_f32(base + q.kind + ".v", {q.count}, vel.data() + q.off);
    }
  }
  if (!w.write(stmp, e)) {
    cleanup();
    return dfail(err, err_len, e);
  }
  // publish: the adapter first, the state last (its presence marks a complete pair)
  if (std::rename(atmp.c_str(), ap.c_str()) != 0) {
    cleanup();
    return dfail(err, err_len, "failed to publish adapter checkpoint " + ap);
  }
  if (std::rename(stmp.c_str(), sp.c_str()) != 0) {
    std::remove(stmp.c_str());
    return dfail(err, err_len, "adapter was written, but trainer state could not be published: " + sp);
  }
  return 0;
}

int sa3k_dit_load_checkpoint(sa3k_dit* d, const char* adapter_path, const char* state_path, int64_t* step,
                             char* err, int err_len) {
  if (!d || !adapter_path || !state_path || !step) return dfail(err, err_len, "NULL argument");
  DitModel& m = d->m;
  if (m.tg.empty()) return dfail(err, err_len, "no adapters: call sa3k_dit_init_adapters first");
  cudaSetDevice(m.c->device);
  std::string e;
  GgufFile f;
  if (!f.open(state_path, e)) return dfail(err, err_len, e);
  const GgufValue* arch = f.find("general.architecture");
  if (!arch || arch->type != kGgufString || arch->s != "sa3-trainer-state")
    return dfail(err, err_len, std::string("not an sa3 trainer-state GGUF: ") + state_path);
  const GgufValue* ver = f.find("trainer.state_version");
  if (!ver || ver->type != kGgufU32 || ver->u != 1) return dfail(err, err_len, "unsupported trainer-state version");
  const GgufValue* st = f.find("trainer.step");
  const GgufValue* fp = f.find("trainer.adapter_fingerprint");
  if (!st || st->type != kGgufU64 || !fp || fp->type != kGgufString)
    return dfail(err, err_len, "trainer state is missing its step or adapter fingerprint");
  const std::string actual = gguf_file_fingerprint(adapter_path, e);
  if (actual.empty()) return dfail(err, err_len, e);
  if (actual != fp->s) return dfail(err, err_len, "resume adapter does not match its trainer-state sidecar");
  const GgufValue* tg = f.find("trainer.targets");
  std::vector<std::string> stems;
  for (size_t i : file_order(m)) stems.push_back(stem_of(m.tg[i].name));
  if (!tg || tg->type != kGgufArray || tg->arr_type != kGgufString || tg->arr_s != stems)
    return dfail(err, err_len, "trainer state target inventory does not match the model's adapters");
  std::vector<float> p((size_t)m.np, 0.f), mom((size_t)m.np, 0.f), vel((size_t)m.np, 0.f);
  std::vector<XsBases> bases;
  if (read_adapter_file(m, adapter_path, p, bases, e)) return dfail(err, err_len, e);
  for (const DitTarget& t : m.tg) {
    const std::string base = "optimizer." + stem_of(t.name) + ".";
    const std::vector<Part> parts = target_parts(m, t);
    for (const Part& q : parts) {
      for (int k = 0; k < 2; ++k) {
        const std::string name = base + q.kind + (k ? ".v" : ".m");
        std::vector<float> v;
        if (!f.tensors.count(name)) return dfail(err, err_len, "trainer state is missing optimizer tensor " + name);
        if (!f.read_f32(name, v, e)) return dfail(err, err_len, e);
        if ((int64_t)v.size() != q.count) return dfail(err, err_len, "trainer optimizer tensor shape mismatch: " + name);
        std::copy(v.begin(), v.end(), (k ? vel : mom).begin() + q.off);
      }
    }
  }
  if (store_flat(m, m.p, p, e) || store_flat(m, m.am, mom, e) || store_flat(m, m.av, vel, e) ||
      upload_bases(m, bases, e))
    return dfail(err, err_len, e);
  *step = (int64_t)st->u;
  return 0;
}

}  // extern "C"
