// lora_kernels.h -- launchers of the small kernels in lora.cu and adamw.cu.
#pragma once

#include "sa3k_internal.h"

namespace sa3k {

// One adapter's preparation inputs and outputs (device pointers), for the grouped kernels.
struct PrepDesc {
  const float* A;      // [rank][in]
  const float* B;      // [out][rank]
  const float* m;      // [out] (dora)
  const float* bns;    // [out] (dora)
  int rank, dora;
  float s;
  int64_t in, out;
  __half *a_h, *at_x, *b_x, *bt_h;
  float *pt, *aat, *nsq, *g;
  // gradients (grouped DoRA backward): dg [out] in, dm [out] / dB [out][rank] / dA [rank][in]
  // accumulated, cb [16][out] f16 and c3 [16][16] (zeroed before) out
  const float* dg;
  float *dm, *dB, *dA;
  __half* cb;
  float* c3;
};

int k_cvt_f16(Ctx* c, const float* src, int64_t n, __half* dst, std::string& err);
// grouped over n adapters (descs in device memory): operand packing, A A^T, DoRA norm
int k_prep_all(Ctx* c, const PrepDesc* descs, int n, std::string& err);
int k_aat_all(Ctx* c, const PrepDesc* descs, int n, std::string& err);
int k_dora_norm_all(Ctx* c, const PrepDesc* descs, int n, int64_t max_out, std::string& err);
// grouped DoRA backward (dm, dB, cb, c3 from dg) and the dA += 2 c3 A term, over n adapters
int k_dora_bwd_all(Ctx* c, const PrepDesc* descs, int n, int64_t max_out, std::string& err);
int k_dora_da_c3_all(Ctx* c, const PrepDesc* descs, int n, std::string& err);
int k_prep_adapter(Ctx* c, const float* A, const float* B, int rank, float s, int64_t in, int64_t out,
                   __half* a_h, __half* at_x, __half* b_x, __half* bt_h,
                   std::string& err);
int k_aat(Ctx* c, const float* A, int rank, int64_t in, float* aat, std::string& err);
int k_dora_norm(Ctx* c, const float* pt, const float* B, int rank, int64_t out, const float* aat,
                const float* bns, const float* m, float s, float* nsq, float* g, std::string& err);
// Producers of an adapted linear's output gradient fused with its backward prologue: write
// dz = f16(g * dy) and dg = colsum(dy * (y - bias) / g) (dg zeroed first; g null: dz = f16(dy)).
int k_gate_bwd_dz(Ctx* c, const float* gx, const float* gate, long gstride, int T, int D, int tps, const float* y,
                  const float* bias, const float* g, __half* dz, float* dg, std::string& err);
int k_swiglu_bwd_dz(Ctx* c, const __half* da, const __half* f, int T, int I, const float* bias,
                    const float* g, __half* dz, float* dg, std::string& err);
int k_bwd_prologue(Ctx* c, const float* dy, const float* y, const float* bias, const float* g, int64_t S,
                   int64_t out, __half* dz, float* dg, std::string& err);
int k_dora_bwd(Ctx* c, const float* pt, const float* B, int rank, int64_t out, const float* aat,
               const float* nsq, const float* g, const float* dg, float s, float* dm, int dm_acc,
               float* dB, __half* cb, float* c3, std::string& err);
int k_dora_da_c3(Ctx* c, const float* c3, const float* A, int rank, int64_t in, float* dA, std::string& err);
// ut = f16(alpha X Bm^T)^T for a rank <= 16 adapter: X [M][K] f16 (row stride ldx), Bm [16][K] f16,
// ut [16][ldu]; K % 32 == 0, 16-byte aligned operands (the forward's u = x A^T, the backward's du).
int k_r16_proj(Ctx* c, const __half* x, long ldx, int64_t M, int64_t K, const __half* bm, float alpha, __half* ut,
               long ldu, const char* name, std::string& err);

// adamw.cu
int k_sumsq(Ctx* c, const float* g, int64_t n, float inv, double* acc, std::string& err);
int k_clip_scale(Ctx* c, const double* sumsq, float grad_clip, float inv_count, float* scales,
                 double* norm_out, std::string& err);
int k_adamw(Ctx* c, float* p, const float* g, float* m, float* v, int64_t n, float lr, float b1, float b2,
            float eps, float wd, float b1c, float b2c, const float* scales, std::string& err);

}  // namespace sa3k
