// linear.h -- the adapted frozen-base linear (dit_lin, src/dit.h:92-149) as a reusable engine.
#pragma once

#include "sa3k_internal.h"

namespace sa3k {

// Per-step derived forms of one LoRA / DoRA-rows adapter.  The buffers are owned by the caller;
// adapter_prepare() fills them from A, B (and for DoRA m, base_norm_sq) once per optimizer step,
// and every forward / backward of that step reuses them.
struct AdapterPrep {
  int rank = 0;
  int64_t in = 0, out = 0;
  float s = 1.0f;                      // alpha / rank
  const float* A = nullptr;            // [rank][in]
  const float* B = nullptr;            // [out][rank]
  const float* m = nullptr;            // [out] dora-rows magnitude (null: plain LoRA)
  const float* bns = nullptr;          // [out] base row norm^2 + in*eps
  __half* a_h = nullptr;       // [16][in]
  __half* at_x = nullptr;       // [in][64]  A^T, extension operand of dx
  __half* b_x = nullptr;        // [out][64] B, extension operand of y
  __half* bt_h = nullptr;      // [16][out] B^T
  float* pt = nullptr;                 // [16][out] (W A^T)^T          (dora)
  float* aat = nullptr;                // [16][16]                      (dora)
  float* nsq = nullptr;                // [out] |W + s B A|_row^2       (dora)
  float* g = nullptr;                  // [out] m / sqrt(nsq)           (dora)
  bool dora() const { return m != nullptr; }
};

// bytes of device scratch one AdapterPrep needs (dora or not), laid out by adapter_bind()
size_t adapter_prep_bytes(int64_t in, int64_t out, bool dora);
void adapter_bind(AdapterPrep& p, void* mem);
int adapter_prepare(Ctx* c, const Weight* w, AdapterPrep& p, std::string& err);
// The DoRA P = W A^T GEMM of one adapter (its part of adapter_prepare between the grouped
// packing and the grouped norm).
int adapter_dora_p(Ctx* c, const Weight* w, AdapterPrep& p, std::string& err);

struct LinearFwd {
  const Weight* w = nullptr;
  const AdapterPrep* ad = nullptr;     // null: plain mul_mat
  const float* bias = nullptr;
  const __half* x_h = nullptr; // [M][in] f16 input
  int64_t M = 0;
  float* y = nullptr;                  // [M][out] f32 output (nullable)
  __half* y_h = nullptr;       // [M][out] f16 output (nullable)
  // adapter scratch: ut [16][ut_ld] f16 (u^T: the K = 16 extension operand, kept for backward)
  __half* ut = nullptr;
  int64_t ut_ld = 0;
  const HeadPrepEpi* hp = nullptr;     // fused head preparation of a qkv projection (see gemm())
};
int linear_forward(Ctx* c, const LinearFwd& f, std::string& err);
// u = x A^T of an adapter, written as ut = f16(u)^T [16][ut_ld]
int lora_u(Ctx* c, const __half* x_h, int64_t M, int64_t in, const AdapterPrep& ad, __half* ut,
           int64_t ut_ld, std::string& err);

struct LinearBwd {
  const Weight* w = nullptr;
  const AdapterPrep* ad = nullptr;
  const float* bias = nullptr;
  const __half* x_h = nullptr; // forward input [M][in]
  const float* y = nullptr;            // forward output [M][out] (needed by dora-rows)
  const float* dy = nullptr;           // upstream gradient [M][out] f32
  bool dz_ready = false;               // dz (and dg for dora) already written by a fused producer
  bool defer_grads = false;            // stop after dx: the caller computes dA / dB / dm later
                                       // (grouped over many adapters) from dz, dg, dut and u^T
  int64_t M = 0;
  const __half* ut = nullptr;   // u^T from the forward [16][ut_ld] (adapter)
  int64_t ut_ld = 0;
  float* dx = nullptr;                 // [M][in] f32 (nullable)
  int dx_accumulate = 0;
  __half* dx_h = nullptr;      // [M][in] f16 (nullable; not with dx_accumulate)
  float* dA = nullptr;                 // [rank][in]
  float* dB = nullptr;                 // [out][rank]
  float* dm = nullptr;                 // [out] (dora)
  int grad_accumulate = 0;
  // scratch: dz [M][out] f16, dg [out], dut [16][ut_ld] f16,
  // cb [16][out] f16, c3 [256]
  __half* dz = nullptr;
  float* dg = nullptr;
  __half* dut = nullptr;
  __half* cb = nullptr;
  float* c3 = nullptr;
};
int linear_backward(Ctx* c, const LinearBwd& b, std::string& err);

}  // namespace sa3k
