// materialize.h -- one materialized adapter (src/train_lora.h:275-329) as a part of a larger step:
// the effective weight built once per optimizer step, then any number of forward GEMMs on it,
// and a weight-gradient pass per backward that adds into the adapter's gradient buffers.
#pragma once

#include "sa3k_internal.h"

#include <string>

namespace sa3k {

struct MatTarget {
  // family: rows (dora-rows / bora row magnitude), cols (dora-cols / bora column magnitude),
  // xs (delta = U M V^T with U, V frozen)
  bool xs = false, rows = false, cols = false;
  int rank = 0;
  float s = 1.0f;
  const Weight* w = nullptr;
  int64_t in = 0, out = 0;
  // parameters (device): A [rank][in], B [out][rank]; or U [out][rank], V [in][rank], M [rank][rank]
  const float *A = nullptr, *B = nullptr, *U = nullptr, *Vb = nullptr, *M = nullptr;
  const float *mr = nullptr, *mc = nullptr;     // row magnitude [out], column magnitude [in]
  // gradients (device), added into
  float *dA = nullptr, *dB = nullptr, *dM = nullptr, *dmr = nullptr, *dmc = nullptr;
  // owned buffers (mat_target_bind): V f32 [out][in] and W_eff f16 [out][in] of this step, the
  // row / column factors and the low-rank scratch
  float *V = nullptr, *rs = nullptr, *cs = nullptr, *tcn = nullptr, *P = nullptr, *Q = nullptr, *PG = nullptr;
  double *rn2 = nullptr, *csq = nullptr, *tc = nullptr;
  __half* wb = nullptr;
  __half *Qb = nullptr, *Btb = nullptr;   // f16 A (or V^T) [rank][in] and B^T [rank][out]
};

size_t mat_target_bytes(int64_t in, int64_t out, int rank);
void mat_target_bind(MatTarget& t, void* mem);
// V, the row / column factors and W_eff (t.wb; also f32 into weff_f32 when not null) from the
// current parameters.
int mat_target_build(Ctx* c, MatTarget& t, float* weff_f32, std::string& err);
// The weight gradient of one backward: G = dz^T x (dz [M][out] f16, x [M][in] f16, K = M) into
// G [out][in] f32 scratch (dzt: [out][ldt] f16 scratch, ldt >= M, a multiple of 8), then the
// normalisation backward into dD = s dV (dDb: [out][in] f16 scratch) and the rank-r GEMMs on dD;
// the adapter gradients are added into t.dA / dB / dM / dmr / dmc.
int mat_target_backward(Ctx* c, MatTarget& t, const __half* dz, int64_t M, const __half* x,
                        float* G, __half* dzt, int64_t ldt, __half* dDb, std::string& err);
// nrm[i] = sqrt(sum_o W[o][i]^2) (f64 sums), the column-magnitude init (train_col_norms,
// src/train_lora.h:176-190).
int mat_col_norms(Ctx* c, const Weight* w, float* nrm, std::string& err);

}  // namespace sa3k
