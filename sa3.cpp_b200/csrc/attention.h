// attention.h -- attention and DiT elementwise kernels shared by the C ABI and the DiT step.
#pragma once

#include "sa3k_internal.h"

namespace sa3k {

// Strided f16 / f32 tensors: element (b, h, s, d) at ptr + b*sb + h*sh + s*ld + d.
struct AttnArgs {
  int B = 0, H = 0, Sq = 0, Sk = 0, head_dim = 64;
  float scale = 0.125f;
  int window = -1;                       // -1 dense, else keep |q - k| <= window
  const __half* q = nullptr; long q_sb = 0, q_sh = 0, q_ld = 0;
  const __half* k = nullptr; long k_sb = 0, k_sh = 0, k_ld = 0;
  const __half* v = nullptr; long v_sb = 0, v_sh = 0, v_ld = 0;
  __half* o = nullptr; long o_sb = 0, o_sh = 0, o_ld = 0;           // written by forward
  float* lse = nullptr;                  // [B*H][Sq], log2 units (row max + log2 of row sum)
  // backward
  const __half* dO = nullptr; long dO_sb = 0, dO_sh = 0, dO_ld = 0;
  float* Dsum = nullptr;                 // [B*H][Sq] scratch: rowsum(dO o O)
  float* dq = nullptr; long dq_sb = 0, dq_sh = 0, dq_ld = 0;
  float* dk = nullptr; long dk_sb = 0, dk_sh = 0, dk_ld = 0;
  float* dv = nullptr; long dv_sb = 0, dv_sh = 0, dv_ld = 0;
};

int attn_forward(Ctx* c, const AttnArgs& a, std::string& err);
// tcgen05 kernels (attention_tc.cu): used by attn_forward / attn_backward when the context allows
// them and the layout qualifies (16-byte aligned rows and strides)
bool attn_tc_supported(const AttnArgs& a);
int attn_tc_forward(Ctx* c, const AttnArgs& a, std::string& err);
int attn_tc_grads(Ctx* c, const AttnArgs& a, bool want_dkdv, std::string& err);
// dq always; dk / dv when want_dkdv (cross-attention to a frozen context needs only dq)
int attn_backward(Ctx* c, const AttnArgs& a, bool want_dkdv, std::string& err);

// ------------------------------------------------------------------ DiT elementwise (dit_ops.cu)
// h = rms_norm(x) * gamma * (1 + sc[sample]) + sh[sample]  -> f16, saves rstd per row
int k_rmsnorm_mod_fwd(Ctx* c, const float* x, int T, int D, const float* gamma, const float* sc, const float* sh,
                      long mod_stride, int tokens_per_sample, float eps, __half* h, float* rstd,
                      std::string& err);
// gx += d/dx of the above for upstream dh (gamma, sc, sh are frozen); gx_h (nullable) also
// receives the updated gx as f16
// x_out = x_in + y * gate[sample] (gate null: x_in + y), then the rmsnorm_mod_fwd of x_out
int k_residual_norm(Ctx* c, const float* x_in, const float* y, const float* gate, long gstride, int T, int D, int tps,
                    float* x_out, const float* gamma, const float* sc, const float* sh, long mod_stride, float eps,
                    __half* h, float* rstd, std::string& err);
int k_rmsnorm_mod_bwd(Ctx* c, const float* dh, const float* x, const float* rstd, int T, int D, const float* gamma,
                      const float* sc, long mod_stride, int tokens_per_sample, float* gx, __half* gx_h,
                      std::string& err);

// Per-head q/k preparation of a fused projection output y[T][ncols] (f32): for each slice (a
// column offset that is a multiple of the head width 64): rms-norm with gamma (if gamma), then
// partial NeoX RoPE of the first `rot` dims (if rope); written as f16 into out[T][ncols].
struct HeadSlice {
  int col = 0;            // first column of the slice
  const float* gamma = nullptr;   // null: copy only
  int rope = 0;           // apply RoPE after the norm
  float* rstd = nullptr;  // [T][H] saved for the backward (norm slices)
};
// NeoX RoPE (cos, sin) table [tps][rot / 2] of the context (null when rot == 0), followed by the
// same values frequency-major, [rot / 2][tps]
const float2* k_rope_table(Ctx* c, int tps, int rot, float rope_base, std::string& err);
int k_head_prep_fwd(Ctx* c, const float* y, int T, int ncols, int H, const HeadSlice* slices, int nslices,
                    int tokens_per_sample, float eps, int rot, float rope_base, __half* out, std::string& err);
// the same slices `reps` times, repetition r at r col_step columns, its gamma r gamma_step values
// on and its rstd r rstd_step entries on (one launch for every block's context K / V)
int k_head_prep_fwd_reps(Ctx* c, const float* y, int T, int ncols, int H, const HeadSlice* slices, int nslices,
                         int tokens_per_sample, float eps, int rot, float rope_base, __half* out, int reps,
                         int col_step, int gamma_step, long rstd_step, std::string& err);
// the same with f16 projection rows
int k_head_prep_fwd(Ctx* c, const __half* y, int T, int ncols, int H, const HeadSlice* slices, int nslices,
                    int tokens_per_sample, float eps, int rot, float rope_base, __half* out, std::string& err);
// Backward of one slice: g[T][H*64] (f32, gradient w.r.t. the prepared slice) -> dy slice of
// dy[T][ncols] (f32, overwritten; or, with dy_h, written as f16 there instead), using the
// forward input y and the saved rstd.
int k_head_prep_bwd(Ctx* c, const float* g, long g_ld, const float* y, int T, int ncols, int H, const HeadSlice& s,
                    int tokens_per_sample, int rot, float rope_base, float* dy, __half* dy_h,
                    std::string& err, float gscale = 1.0f,     // g enters as gscale (g - g2)
                    const float* g2 = nullptr, long g2_ld = 0);
// Self-attention q/k/v head preparation backward (dq3 = [dq | dk | dv] f32, or with nsl = 5 the
// differential layout [dq | dk | dv | dqd | dkd] whose second stream ran on +dO, dv2 its dV, and
// rq2 / rk2 its rstd; qkv = the projection output, f16) fused with the qkv projection's backward
// prologue: dz = f16(g * dy) [T][nsl D] and dg = colsum(dy * qkv / g) (DoRA g; null: plain f16
// conversion, dg untouched).
int k_qkv_bwd_dz(Ctx* c, const float* dq3, const __half* qkv, int T, int D, int H, int nsl, const float* rq,
                 const float* rk, const float* rq2, const float* rk2, const float* dv2, const float* gq,
                 const float* gk, int tokens_per_sample, int rot, float rope_base, const float* g,
                 __half* dz, float* dg, std::string& err);
// out = x - y (f16, n a multiple of 8)
int k_sub_f16(Ctx* c, const __half* x, const __half* y, long n, __half* out, std::string& err);

// x_out = x_in + y * gate[sample]  (gate already sigmoid(1 - g)); x_out may alias x_in
int k_gate_residual(Ctx* c, const float* x_in, const float* y, const float* gate, long gate_stride, int T, int D,
                    int tokens_per_sample, float* x_out, std::string& err);
// dy = gx * gate[sample]
int k_gate_bwd(Ctx* c, const float* gx, const float* gate, long gate_stride, int T, int D, int tokens_per_sample,
               float* dy, std::string& err);
// out = x + y (elementwise, n values); out may alias either input
int k_add(Ctx* c, const float* x, const float* y, long n, float* out, std::string& err);

// SwiGLU: f[T][2I] -> a[T][I] = f[:, :I] * silu(f[:, I:]) (f16); backward da -> df (f32)
// act = f16(val * silu(gate)) of f = [val | gate] (f16, rows of 2I)
int k_swiglu_fwd(Ctx* c, const __half* f, int T, int I, __half* a, std::string& err);

// silu in place (f32) and its f32 -> f16 copy for a following GEMM
int k_silu_f16(Ctx* c, const float* x, long n, __half* out, std::string& err);

// mod[b][i] = ssg[i] + gcond[b][i] for i < 6*D, and the two gates sigmoid(1 - g) in place of
// slots 2 and 5 (the adaLN-zero vectors of src/dit.h:174-193)
// out = dy * silu'(h) (elementwise; out may alias dy)
int k_silu_bwd(Ctx* c, const float* dy, const float* h, long n, float* out, std::string& err);
// adaLN modulation gradient, added per sample into [B][out_stride] rows (rows t of sample t / tps):
// of h = rms_norm(x) (1 + sc) + sh:  dsc += gamma * colsum(dh * x * rstd), dsh += colsum(dh);
// of out = res + y * s, s = sigmoid(1 - g) (gate holds s, as the modulation kernel leaves it):
// dg += -s (1 - s) colsum(gy * y)
int k_mod_grad_norm(Ctx* c, const float* dh, const float* x, const float* rstd, const float* gamma, int T, int D,
                    int tps, long out_stride, float* dsc, float* dsh, std::string& err);
int k_mod_grad_gate(Ctx* c, const float* gy, const float* y, const float* gate, long gate_stride, int T, int D, int tps,
                    long out_stride, float* dgate, std::string& err);
// L blocks at once: ssg [L][6D], mod [L][B][6D]
int k_modulation(Ctx* c, const float* ssg, const float* gcond, int B, int D, float* mod, std::string& err, int L = 1);

// loss[b] = sum((vel - target)^2) / (io*T) per sample; dvel = grad_scale * 2 (vel - target) / (io*T);
// with weight (nullable, [B][io*T]): loss[b] = sum(w (vel - target)^2), dvel = grad_scale * 2 w (vel - target)
int k_mse(Ctx* c, const float* vel, const float* target, int B, long per_sample, float* loss, float* dvel,
          float grad_scale, const float* weight, std::string& err);
// dst[r][c] = c < w ? f16(src[r][c]) : 0, rows of ld (>= w) f16
int k_pad_f16(Ctx* c, const float* src, long rows, int w, __half* dst, long ld, std::string& err);
// rows t >= mem of each sample (S rows) get le's row of that real token added: dst = y + le (dst may be y)
int k_add_local(Ctx* c, const float* y, const float* le, int B, int S, int mem, int D, float* dst, std::string& err);
// x *= s over n floats (in place)
int k_scale(Ctx* c, float* x, long n, float s, std::string& err);

// copy rows: dst[b*dst_rows_per + dst_off + r][:] = src[b*src_rows_per + src_off + r][:] for r < rows
// (f32 or f16 destination), used for the memory-token concat / drop of dit_head / dit_tail
int k_copy_rows(Ctx* c, const float* src, int src_rows_per, int src_off, float* dst, __half* dst_h,
                int dst_rows_per, int dst_off, int B, int rows, int D, std::string& err);

}  // namespace sa3k
