// gemm_r16.h -- grouped rank-16 GEMMs (gemm_r16.cu): one launch for many skinny contractions.
#pragma once

#include <vector>

#include "sa3k_internal.h"

namespace sa3k {

// out (+)= alpha * Aop * Bop for one problem of a group:
//   Aop [M x K] f16: K-major A[m * lda + k] (a_mn 0) or MN-major A[k * lda + m] (a_mn 1)
//   Bop [K x N] f16, N <= 16, stored K-major as B[n * ldb + k] (rows n >= N are never used
//       in the output, but the 16 x 64 tile is loaded: ldb rows 0..15 must be readable)
//   out f32: out[m * ldo + n] or (out_trans) out[n * ldo + m]; atomic: added with f32 atomics
//       (K may then be split across CTAs), else stored once (no split).
struct R16Job {
  const __half* a = nullptr;
  long lda = 0;
  int a_mn = 0;
  int M = 0, N = 16, K = 0;
  const __half* b = nullptr;
  long ldb = 0;
  float alpha = 1.0f;
  float* out = nullptr;
  long ldo = 0;
  int out_trans = 0;
  int atomic = 0;
};

// A built group: the problem table (with TMA tensor maps, so the operand addresses are fixed)
// in device memory.
struct R16Group {
  void* table = nullptr;
  int nprob = 0, nitems = 0;
};

// Builds (synchronously uploads) the table; kb_target = 64-wide k-blocks per work item for the
// atomic problems.
int r16_group_build(Ctx* c, const std::vector<R16Job>& jobs, int kb_target, R16Group& g, std::string& err);
void r16_group_free(R16Group& g);
int r16_group_run(Ctx* c, const R16Group& g, const char* name, std::string& err);

}  // namespace sa3k
