// linear.cu -- forward and backward of the adapted frozen-base linear over the tcgen05 engine.
//
// Forward (src/dit.h:106-147):
//   u = x A^T                               rank-16 GEMM, written as f16 u^T [16][M]
//   y = g * (x W^T  (+)  (s u) B^T) + bias  one GEMM: the LoRA term is a K = 16 extension of the
//                                           base MMA chain; g (DoRA) and bias in the epilogue
// Backward (what ggml_build_backward_expand derives for those ops, src/train_ckpt.h:400):
//   dz = g * dy,  dg = colsum(dy * (y - bias) / g)                  (prologue, dora)
//   du = s dz B                                                     rank-16 GEMM
//   dx = dz W  (+)  du A                                            one GEMM, K = 16 extension
//   dB = s dz^T u,  dA = du^T x                                     skinny GEMMs (split-K)
//   dora:  dm = dg / |.|,  dB += dt2 P + 2 dt3 (B A A^T),
//          dA += (dt2 B)^T W + 2 (B^T diag(dt3) B) A                rank-16 quant GEMM + 16x16
#include "linear.h"
#include "lora_kernels.h"

namespace sa3k {

static size_t al(size_t b) { return (b + 255) & ~(size_t)255; }

size_t adapter_prep_bytes(int64_t in, int64_t out, bool dora) {
  size_t b = al(16 * in * 2) + al(in * 64 * 2) + al(out * 64 * 2) + al(16 * out * 2);
  if (dora) b += al(16 * out * 4) + al(256 * 4) + al(out * 4) + al(out * 4);
  return b;
}

void adapter_bind(AdapterPrep& p, void* mem) {
  char* q = static_cast<char*>(mem);
  auto take = [&](size_t bytes) { void* r = q; q += al(bytes); return r; };
  p.a_h = static_cast<__half*>(take(16 * p.in * 2));
  p.at_x = static_cast<__half*>(take(p.in * 64 * 2));
  p.b_x = static_cast<__half*>(take(p.out * 64 * 2));
  p.bt_h = static_cast<__half*>(take(16 * p.out * 2));
  if (p.dora()) {
    p.pt = static_cast<float*>(take(16 * p.out * 4));
    p.aat = static_cast<float*>(take(256 * 4));
    p.nsq = static_cast<float*>(take(p.out * 4));
    p.g = static_cast<float*>(take(p.out * 4));
  }
}

int adapter_dora_p(Ctx* c, const Weight* w, AdapterPrep& p, std::string& err) {
  GemmDesc g;
  if (w->f16) {   // P = W A^T [out][16] with out as M, stored transposed as P^T [16][out]
    g.M = (int)p.out; g.N = 16; g.K = (int)p.in;
    g.a = w->f16; g.lda = p.in;
    g.bsrc = kB_F16_KMAJOR; g.b = p.a_h; g.ldb = p.in;
    g.out = p.pt; g.ldo = p.out; g.out_trans = 1; g.bn = 16;
  } else {         // quantized base without an operand copy: P^T = A W^T [16][out]
    g.M = 16; g.N = (int)p.out; g.K = (int)p.in;
    g.a = p.a_h; g.lda = p.in;
    g.bsrc = kB_WEIGHT_NT; g.w = w;
    g.out = p.pt; g.ldo = p.out;
  }
  g.name = "dora.P";
  return gemm(c, g, err);
}

int adapter_prepare(Ctx* c, const Weight* w, AdapterPrep& p, std::string& err) {
  if (k_prep_adapter(c, p.A, p.B, p.rank, p.s, p.in, p.out, p.a_h, p.at_x, p.b_x, p.bt_h, err)) return 1;
  if (!p.dora()) return 0;
  if (adapter_dora_p(c, w, p, err)) return 1;
  if (k_aat(c, p.A, p.rank, p.in, p.aat, err)) return 1;
  return k_dora_norm(c, p.pt, p.B, p.rank, p.out, p.aat, p.bns, p.m, p.s, p.nsq, p.g, err);
}

int lora_u(Ctx* c, const __half* x_h, int64_t M, int64_t in, const AdapterPrep& ad, __half* ut,
           int64_t ut_ld, std::string& err) {
  // u = x A^T  [M][16], written as ut = f16(u)^T [16][ut_ld]: the HBM-shaped rank-16 kernel, or
  // the GEMM engine for widths it does not take
  if (in % 32 == 0) return k_r16_proj(c, x_h, (long)in, M, in, ad.a_h, 1.0f, ut, (long)ut_ld, "lora.u", err);
  GemmDesc g;
  g.M = (int)M; g.N = 16; g.K = (int)in;
  g.a = x_h; g.lda = in;
  g.bsrc = kB_F16_KMAJOR; g.b = ad.a_h; g.ldb = in;
  g.out_h_t = ut; g.ldo_h_t = ut_ld;
  g.bn = 16;
  g.name = "lora.u";
  return gemm(c, g, err);
}

int linear_forward(Ctx* c, const LinearFwd& f, std::string& err) {
  const Weight* w = f.w;
  const AdapterPrep* ad = f.ad;
  if (ad && lora_u(c, f.x_h, f.M, w->in, *ad, f.ut, f.ut_ld, err)) return 1;
  GemmDesc g;   // y = g * (x W^T + s u B^T) + bias
  g.M = (int)f.M; g.N = (int)w->out; g.K = (int)w->in;
  g.a = f.x_h; g.lda = w->in;
  g.bsrc = kB_WEIGHT_NT; g.w = w;
  if (ad) { g.ext_at = f.ut; g.ld_ext = f.ut_ld; g.ext_b = ad->b_x; }
  g.col_scale = (ad && ad->dora()) ? ad->g : nullptr;
  g.col_bias = f.bias;
  g.out = f.y; g.ldo = w->out;
  g.out_h = f.y_h; g.ldo_h = w->out;
  g.hp = f.hp;
  g.name = "linear.fwd";
  return gemm(c, g, err);
}

int linear_backward(Ctx* c, const LinearBwd& b, std::string& err) {
  const Weight* w = b.w;
  const AdapterPrep* ad = b.ad;
  const bool dora = ad && ad->dora();
  const int64_t in = w->in, out = w->out;
  const int rank = ad ? ad->rank : 0;
  if (!b.dz_ready) {
    if (dora && cudaMemsetAsync(b.dg, 0, sizeof(float) * out, c->stream) != cudaSuccess)
      return check_launch("memset", err);
    if (k_bwd_prologue(c, b.dy, dora ? b.y : nullptr, b.bias, dora ? ad->g : nullptr, b.M, out, b.dz,
                       dora ? b.dg : nullptr, err))
      return 1;
  }
  if (ad && out % 32 == 0) {   // du = s dz B  [M][16], written as dut = f16(du)^T [16][ut_ld]
    if (k_r16_proj(c, b.dz, (long)out, b.M, out, ad->bt_h, ad->s, b.dut, (long)b.ut_ld, "lora.du", err)) return 1;
  } else if (ad) {
    GemmDesc g;   // (the GEMM engine for widths the rank-16 kernel does not take)
    g.M = (int)b.M; g.N = 16; g.K = (int)out;
    g.a = b.dz; g.lda = out;
    g.bsrc = kB_F16_KMAJOR; g.b = ad->bt_h; g.ldb = out;
    g.alpha = ad->s;
    g.out_h_t = b.dut; g.ldo_h_t = b.ut_ld;
    g.bn = 16;
    g.name = "lora.du";
    if (gemm(c, g, err)) return 1;
  }
  if (b.dx || b.dx_h) {
    GemmDesc g;   // dx = dz W + du A
    g.M = (int)b.M; g.N = (int)in; g.K = (int)out;
    g.a = b.dz; g.lda = out;
    g.bsrc = kB_WEIGHT_TN; g.w = w;
    if (ad) { g.ext_at = b.dut; g.ld_ext = b.ut_ld; g.ext_b = ad->at_x; }
    g.out = b.dx; g.ldo = in; g.accumulate = b.dx_accumulate;
    g.out_h = b.dx_h; g.ldo_h = in;
    g.name = "linear.dx";
    if (gemm(c, g, err)) return 1;
  }
  if (!ad || b.defer_grads) return 0;
  // The rank-16 gradient GEMMs run with the long dimension as M (full 128-row MMA tiles) and
  // add their split-K parts into the gradient with atomics.
  {
    GemmDesc g;   // dB = s dz^T u  [out][rank]
    g.M = (int)out; g.N = rank; g.K = (int)b.M;
    g.a = b.dz; g.lda = out; g.a_mn = 1;
    g.bsrc = kB_F16_KMAJOR; g.b = b.ut; g.ldb = b.ut_ld;
    g.alpha = ad->s;
    g.out = b.dB; g.ldo = rank; g.accumulate = b.grad_accumulate; g.bn = 16;
    g.atomic_split = 1;
    g.name = "lora.dB";
    if (gemm(c, g, err)) return 1;
  }
  {
    GemmDesc g;   // dA^T = x^T du  [in][rank], stored transposed as dA [rank][in]
    g.M = (int)in; g.N = rank; g.K = (int)b.M;
    g.a = b.x_h; g.lda = in; g.a_mn = 1;
    g.bsrc = kB_F16_KMAJOR; g.b = b.dut; g.ldb = b.ut_ld;
    g.out = b.dA; g.ldo = in; g.out_trans = 1; g.accumulate = b.grad_accumulate; g.bn = 16;
    g.atomic_split = 1;
    g.name = "lora.dA";
    if (gemm(c, g, err)) return 1;
  }
  if (!dora) return 0;
  if (cudaMemsetAsync(b.c3, 0, sizeof(float) * 256, c->stream) != cudaSuccess) return check_launch("memset", err);
  if (k_dora_bwd(c, ad->pt, ad->B, rank, out, ad->aat, ad->nsq, ad->g, b.dg, ad->s, b.dm, b.grad_accumulate, b.dB,
                 b.cb, b.c3, err))
    return 1;
  GemmDesc g;   // dA += (dt2 B)^T W
  if (w->f16) {   // as dA^T += W^T (dt2 B): the f16 operand copy read MN-major
    g.M = (int)in; g.N = rank; g.K = (int)out;
    g.a = w->f16; g.lda = in; g.a_mn = 1;
    g.bsrc = kB_F16_KMAJOR; g.b = b.cb; g.ldb = out;
    g.out = b.dA; g.ldo = in; g.out_trans = 1; g.accumulate = 1; g.bn = 16;
    g.atomic_split = 1;
  } else {         // quantized base without an operand copy: W^T dequantized in the GEMM
    g.M = rank; g.N = (int)in; g.K = (int)out;
    g.a = b.cb; g.lda = out;
    g.bsrc = kB_WEIGHT_TN; g.w = w;
    g.out = b.dA; g.ldo = in; g.accumulate = 1;
  }
  g.name = "dora.dA";
  if (gemm(c, g, err)) return 1;
  return k_dora_da_c3(c, b.c3, ad->A, rank, in, b.dA, err);
}

}  // namespace sa3k
