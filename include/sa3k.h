/*
 * sa3k.h -- C ABI of the B200 (sm_100a) adapter-training hot path of sa3.cpp.
 *
 * Conventions follow the reference's libsa3 C ABI (src/libsa3.h:4-9): every call returns an int
 * status (0 = OK), failures fill `err` (a caller buffer of `err_len` bytes), no C++ exception
 * crosses the boundary, objects the library allocates are released by the library, and a
 * context is bound to one device and one CUDA stream and is not reentrant.
 *
 * Tensors are passed as plain pointers with the ggml layout of the reference, i.e. ggml
 * [ne0, ne1] = row-major [ne1][ne0]:
 *   W [in, out]  -> W[out][in], quantized blocks along `in`      (frozen base weight)
 *   x [in, S]    -> x[S][in]                                     (activations, f32)
 *   A [in, r]    -> A[r][in]          B [r, out] -> B[out][r]    (TrainLoraParam layout,
 *                                                                 src/train_lora.h:26-27)
 * Unless a name ends in _host, pointers are DEVICE pointers on the context's device.
 *
 * There is no CPU fallback: without an sm_100 device every call fails with an error.
 */
#ifndef SA3K_H
#define SA3K_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define SA3K_TYPE_F32 0
#define SA3K_TYPE_F16 1
#define SA3K_TYPE_Q8_0 8
#define SA3K_TYPE_Q4_K 12

typedef struct sa3k_ctx sa3k_ctx;
typedef struct sa3k_weight sa3k_weight;

/* Library version string.  Counterpart of sa3_version (src/libsa3.h:188). */
const char* sa3k_version(void);

/* Bind a context to CUDA device `device` (must be sm_100) with a private stream.
 * Replaces backend selection, make_backend (src/gguf_model.h:120-198). */
int sa3k_ctx_create(int device, sa3k_ctx** out, char* err, int err_len);
void sa3k_ctx_destroy(sa3k_ctx* ctx);

/* Run subsequent work on `cuda_stream`, a cudaStream_t of the context's device (NULL is CUDA's
 * legacy default stream).  The context's private stream is released on the first call.
 * No counterpart in the reference (ggml owns its streams). */
int sa3k_ctx_set_stream(sa3k_ctx* ctx, void* cuda_stream, char* err, int err_len);

/* Context options (sa3k_ctx_set_option).  No counterpart in the reference.
 *   SA3K_OPT_WEIGHT_F16_CACHE  1 (default): a Q8_0 / Q4_K weight uploaded afterwards also keeps
 *       an IEEE half (f16) operand copy, made once by the bit-exact dequantizer (the frozen base
 *       never changes, so the tensor cores then read f16 tiles directly).  0: codes + scales only.
 *   SA3K_OPT_SMEM_DEQUANT  1: GEMMs over quantized weights dequantize each TMA-loaded tile in
 *       shared memory even when an f16 copy exists.  0 (default): use the copy when present.
 * Both paths round the same f32 dequantized value once to f16, so results are identical.
 *
 * Operand type.  Every tensor-core contraction of the library (the GEMM engine, the rank-16
 * GEMMs, attention) reads IEEE half operands (11-bit significand) with f32 accumulation.  Against
 * bf16 (8-bit significand) at the same tensor-core rate this is 8x less rounding of the frozen
 * base weights, whose rounding error is the same for every token and so does not average out of
 * the adapter gradients.  The f16 range (largest 65504, normal down to 6.1e-5) suits normalized
 * activations; gradients are carried scaled: the DiT step multiplies its loss gradient by a
 * power of two and divides the adapter gradients by it again (exact), and the component
 * backward calls take the upstream gradient as given (callers with very small gradients scale
 * them the same way). */
#define SA3K_OPT_WEIGHT_F16_CACHE 1
#define SA3K_OPT_SMEM_DEQUANT 2
/* SA3K_OPT_GEMM_TILE_N  0 (default): the N tile of the large GEMMs comes from a wave-count cost
 *       model; 128, 192 or 256 fixes it (a tuning knob; results do not depend on it). */
#define SA3K_OPT_GEMM_TILE_N 3
/* SA3K_OPT_GEMM_PAIR  1 (default): f16-operand GEMMs with at least 256 rows and enough output
 *       tiles run on CTA pairs (tcgen05 cta_group::2, 256-row tiles); 0: one CTA per tile always;
 *       2: CTA pairs wherever they apply (a tuning knob; with SA3K_OPT_GEMM_TILE_N 192 the pair
 *       tiles are 256 x 192).  Results are identical either way (same per-element summation order). */
#define SA3K_OPT_GEMM_PAIR 4
/* SA3K_OPT_ATTN_TC  1 (default): attention on the tcgen05 tensor cores (TMEM accumulators, P and
 *       dS fed back from TMEM); 0: the mma.sync kernels.  Both compute in f16 with f32
 *       accumulation; results agree to rounding. */
#define SA3K_OPT_ATTN_TC 5
/* SA3K_OPT_PDL  1 (default): kernels launched outside a stream capture use programmatic
 *       dependent launch, so the next kernel of the stream is scheduled while the previous one
 *       drains (each kernel waits for its predecessor's results before reading them; captured
 *       graphs keep plain edges, which replay faster); 0: plain stream order always. */
#define SA3K_OPT_PDL 6
/* SA3K_OPT_STEP_GRAPH  1 (default): sa3k_dit_forward_backward records the step as a CUDA graph on
 *       its second call at a given (B, T, ctx_len) and replays it from then on (one launch per
 *       call instead of ~1000).  The graph is dropped and re-recorded after anything it depends on
 *       changes: tensors, adapters, context options or the context's scratch buffers.  Calls made
 *       while the stream is being captured, or with profiling timing on, run eagerly.
 *       0: every call launches its kernels one by one. */
#define SA3K_OPT_STEP_GRAPH 7
/* SA3K_OPT_DEQUANT_TMEM  1 (default): GEMMs that dequantize a Q8_0 / Q4_K base in the kernel (see
 *       SA3K_OPT_SMEM_DEQUANT; also every GEMM over a quantized base uploaded without the f16
 *       cache) compute the transposed product with the weight as the tensor-memory operand: the
 *       codes are read from global memory, dequantized in registers and written to tensor memory,
 *       so only the activation tile passes through shared memory.  The input-gradient GEMM reads a
 *       transposed copy of the codes, made once on its first eager call (1 byte per weight for
 *       Q8_0, half for Q4_K).  0: dequantize into a shared-memory B tile instead.  Results are
 *       identical up to the order of the f32 accumulation. */
#define SA3K_OPT_DEQUANT_TMEM 8
/* SA3K_OPT_FUSE_HEAD_PREP  1 (default): in the DiT step, the self-attention q / k head preparation
 *       (per-head RMS norm, NeoX RoPE) runs in the epilogue of the qkv projection GEMM whenever that
 *       GEMM takes the CTA-pair kernel with an f16 weight operand (no differential slices).  0: a
 *       separate pass over the projection output.  The two differ only in the rounding of the
 *       projection output before the norm (f32 in the epilogue, f16 in the separate pass). */
#define SA3K_OPT_FUSE_HEAD_PREP 9
int sa3k_ctx_set_option(sa3k_ctx* ctx, int option, int64_t value, char* err, int err_len);

/* Wait for the context's stream and report any asynchronous or device-side error (a bounded
 * wait that timed out inside a kernel is reported here and cleared).
 * Counterpart of the implicit sync in ggml_backend_tensor_get (src/train_loop.h:371). */
int sa3k_sync(sa3k_ctx* ctx, char* err, int err_len);

/* Failure-path check of the bounded device waits (no counterpart in the reference).  Launches,
 * on the context's stream, one kernel whose only wait is on a shared-memory barrier that nothing
 * completes, bounded by limit_us microseconds (1 .. 2,000,000) through the same wait routine as
 * every pipeline of this library.  The wait runs out, the kernel records the timeout in the
 * context's device error word and returns: the next sa3k_sync reports "device wait timed out"
 * and clears it, and the context stays usable.  Returns 0 when the kernel was launched. */
int sa3k_check_bounded_wait(sa3k_ctx* ctx, int limit_us, char* err, int err_len);

/* Per launch-class counters of this context: every kernel launch is counted by class
 * ("linear.fwd", "linear.dx", "lora.dA", "adamw", ...).  timing 1: each launch is also
 * bracketed by CUDA events on the context's stream and read sums the elapsed times.
 * timing 2 (graph): the events are recorded as event nodes of a CUDA graph being captured on
 * the context's stream; after each replay, read reports that replay's per-class times.
 * Enabling resets the counters.  Counterpart of the SA3_TRAIN_PROFILE phase timers
 * (src/train_loop.h:314-437). */
typedef struct sa3k_profile_entry {
  char name[48];
  int64_t launches;
  double total_ms;   /* summed event time of those launches (0 unless timing was on) */
} sa3k_profile_entry;

int sa3k_profile_enable(sa3k_ctx* ctx, int timing, char* err, int err_len);

/* Copy up to `max` entries into `out` (may be NULL to count) and the number of classes into
 * *n_out.  Synchronizes the context's stream. */
int sa3k_profile_read(sa3k_ctx* ctx, sa3k_profile_entry* out, int max, int* n_out, char* err,
                      int err_len);

/* Upload one frozen base weight from raw GGUF row bytes (host memory), ggml type
 * F32 / F16 / Q8_0 / Q4_K, and repack it for the tensor-core engine.  `in` must be a multiple of
 * 64 (Q8_0) or 256 (Q4_K).  Replaces the weight upload of load_gguf (src/gguf_model.h:318-329). */
int sa3k_weight_upload(sa3k_ctx* ctx, int ggml_type, const void* blocks_host, int64_t in,
                       int64_t out, sa3k_weight** w, char* err, int err_len);
void sa3k_weight_free(sa3k_weight* w);

/* dst[out][in] (f32) = the dequantized weight, bit-identical to ggml's to_float.
 * Counterpart of read_to_f32 (src/lora.h:52-74). */
int sa3k_dequant(sa3k_ctx* ctx, const sa3k_weight* w, float* dst, char* err, int err_len);

/* Per output row: base_norm_sq[o] = sum_i W[o][i]^2 + in*eps and norm[o] = sqrt(sum_i W^2),
 * f64 accumulation (either output may be NULL).  Replaces train_row_norm_sq and
 * train_row_norms (src/train_lora.h:141-174) for the DoRA constants and magnitude init. */
int sa3k_row_norms(sa3k_ctx* ctx, const sa3k_weight* w, float eps, float* base_norm_sq,
                   float* norm, char* err, int err_len);

/* Per input column: norm[i] = sqrt(sum_o W[o][i]^2), f64 accumulation.  Replaces train_col_norms
 * (src/train_lora.h:176-190), the magnitude init of dora-cols and bora's column magnitude. */
int sa3k_col_norms(sa3k_ctx* ctx, const sa3k_weight* w, float* norm, char* err, int err_len);

/* One functional adapter on a linear, as DitLoraParam (src/dit.h:65-88). rank <= 16. */
typedef struct sa3k_adapter {
  const float* A;             /* [rank][in]                                   */
  const float* B;             /* [out][rank]                                  */
  const float* magnitude;     /* [out] for dora-rows, else NULL                */
  const float* base_norm_sq;  /* [out] for dora-rows (sa3k_row_norms), else NULL */
  float scale;                /* alpha / rank                                 */
  int rank;
} sa3k_adapter;

/* y[S][out] = dit_lin(W, x) with the adapter (NULL: plain mul_mat) and optional bias[out]:
 *   y = g * (x W^T + s (x A^T) B^T) + bias,  g = m / |W + s B A|_row (dora-rows) or 1.
 * Replaces dit_lin (src/dit.h:92-149). */
int sa3k_linear_fwd(sa3k_ctx* ctx, const sa3k_weight* w, const sa3k_adapter* ad,
                    const float* bias, const float* x, int64_t S, float* y, char* err, int err_len);

/* ---- inference with a chain of functional adapters (build_functional_lora, src/lora.h:372-622,
 * and the DitLoraParam::terms path of dit_lin, src/dit.h:108-117) ----
 * One adapter of a chain, in chain order: A [rank][in], B [out][rank], magnitude [out] for
 * dora-rows (NULL for lora), scale = alpha / rank * strength.  Device pointers, read at build. */
typedef struct sa3k_chain_term {
  const float* A;
  const float* B;
  const float* magnitude;
  int rank;
  float scale;
} sa3k_chain_term;
typedef struct sa3k_lora_chain sa3k_lora_chain;
/* Folds the chain for weight w on the device: every dora-rows adapter rescales the rows of the
 * weight accumulated before it (base row norms, W A^T and A A^T terms; no materialized weight).
 * 1..16 adapters, at most 64 ranks in all.  The chain keeps its own device memory. */
int sa3k_lora_chain_build(sa3k_ctx* ctx, const sa3k_weight* w, const sa3k_chain_term* terms, int n,
                          sa3k_lora_chain** out, char* err, int err_len);
void sa3k_lora_chain_free(sa3k_lora_chain* chain);
/* total rank of the chain and whether its forward is one fused GEMM (rank <= 16 and no output row
 * whose base scale is 0); returns 0 */
int sa3k_lora_chain_info(const sa3k_lora_chain* chain, int* total_rank, int* fused);
/* y[S][out] = b * (x W^T) + sum_k scale_k (x A_k^T) B'_k^T + bias for the chain's weight (x, y,
 * bias f32 device). */
int sa3k_linear_fwd_chain(sa3k_ctx* ctx, const sa3k_weight* w, const sa3k_lora_chain* chain,
                          const float* bias, const float* x, int64_t S, float* y, char* err, int err_len);

/* A materialized adapter (src/train_lora.h:24-41, 275-329): the trainer's path for dora-cols,
 * bora and every "-xs" family (src/train_dit.h:90-164), available for lora / dora-rows too.
 *   V = W + scale * B A            (standard families; A [rank][in], B [out][rank])
 *   V = W + scale * U M V_xs^T     (-xs; U [out][rank], V_xs [in][rank] frozen, M [rank][rank])
 *   lora: W_eff = V;  dora-rows: m[out] * V / |V|_row;  dora-cols: m[in] * V / |V|_col;
 *   bora: m_c[in] * R / |R|_col with R = m_r[out] * V / |V|_row
 * (|v| = sqrt(sum v^2 + n * 1e-12) over the n values of a row or column).  rank 1..16; every
 * array f32 device memory, A 16-byte aligned. */
typedef struct sa3k_mat_adapter {
  const char* adapter_type;   /* "lora", "dora-rows", "dora-cols", "bora", each optionally "-xs" */
  int rank;
  float scale;                /* alpha / rank */
  const float* A;             /* [rank][in]   (standard) */
  const float* B;             /* [out][rank]  (standard) */
  const float* U;             /* [out][rank]  (-xs) */
  const float* V;             /* [in][rank]   (-xs) */
  const float* M;             /* [rank][rank] (-xs, trainable) */
  const float* m;             /* dora-rows [out] / dora-cols [in] */
  const float* m_r;           /* bora [out] */
  const float* m_c;           /* bora [in] */
} sa3k_mat_adapter;

/* Gradients written (not accumulated) by sa3k_linear_mat_fwd_bwd: dA, dB (standard) or dM
 * (-xs), dm (dora-rows, dora-cols) or dm_r, dm_c (bora); the others may be NULL. */
typedef struct sa3k_mat_grads {
  float* dA;
  float* dB;
  float* dM;
  float* dm;
  float* dm_r;
  float* dm_c;
} sa3k_mat_grads;

/* W_eff [out][in] f32 (train_lora_effective_weight, src/train_lora.h:299-329). */
int sa3k_mat_effective_weight(sa3k_ctx* ctx, const sa3k_weight* w, const sa3k_mat_adapter* ad, float* weff,
                              char* err, int err_len);
/* y[S][out] = x W_eff^T + bias (bias may be NULL): the dit_lin of an overridden weight. */
int sa3k_linear_mat_fwd(sa3k_ctx* ctx, const sa3k_weight* w, const sa3k_mat_adapter* ad, const float* bias,
                        const float* x, int64_t S, float* y, char* err, int err_len);
/* The forward (y may be NULL) and the backward for upstream dy[S][out]: dx[S][in] (may be NULL)
 * and the adapter gradients (what ggml_build_backward_expand derives for the override graph). */
int sa3k_linear_mat_fwd_bwd(sa3k_ctx* ctx, const sa3k_weight* w, const sa3k_mat_adapter* ad, const float* bias,
                            const float* x, const float* dy, int64_t S, float* y, float* dx,
                            const sa3k_mat_grads* g, char* err, int err_len);

/* Backward of sa3k_linear_fwd for upstream dy[S][out], given its inputs x and its output y.
 * Writes dx[S][in] (if non-NULL) and the adapter gradients dA[rank][in], dB[out][rank],
 * dm[out] (dora; each may be NULL when ad is NULL).  accumulate != 0 adds into dx/dA/dB/dm
 * instead of overwriting (gradient accumulation across samples / residual branches).
 * Replaces the OUT_PROD / MUL_MAT backward that ggml_build_backward_expand derives for dit_lin
 * (src/train_ckpt.h:400). */
int sa3k_linear_bwd(sa3k_ctx* ctx, const sa3k_weight* w, const sa3k_adapter* ad,
                    const float* bias, const float* x, const float* y, const float* dy, int64_t S,
                    float* dx, float* dA, float* dB, float* dm, int accumulate, char* err,
                    int err_len);

/* Forward + backward of one adapted linear in one call (shares u = x A^T and the DoRA norm
 * between the two passes).  Outputs y, dx, dA, dB, dm as above. */
int sa3k_linear_fwd_bwd(sa3k_ctx* ctx, const sa3k_weight* w, const sa3k_adapter* ad,
                        const float* bias, const float* x, const float* dy, int64_t S, float* y,
                        float* dx, float* dA, float* dB, float* dm, char* err, int err_len);

/* The same step with HOST buffers: copies x, dy and the adapter in, runs forward + backward and
 * copies y, dx, dA, dB, dm out (all host pointers; A/B/magnitude/base_norm_sq in `ad` are host
 * pointers too).  Mirrors what the reference does per step around ggml (tensor_set / graph
 * compute / tensor_get, src/train_loop.h:331-371). */
int sa3k_linear_fwd_bwd_host(sa3k_ctx* ctx, const sa3k_weight* w, const sa3k_adapter* ad_host,
                             const float* bias_host, const float* x_host, const float* dy_host,
                             int64_t S, float* y_host, float* dx_host, float* dA_host,
                             float* dB_host, float* dm_host, char* err, int err_len);

/* A strided 4-D tensor [B][H][S][head_dim]: element (b, h, s, d) is at
 * data + b*batch_stride + h*head_stride + s*row_stride + d (strides in elements).  This covers
 * head-major buffers and the token-major [B][S][H*head_dim] projection outputs alike. */
typedef struct sa3k_tensor4 {
  void* data;
  int64_t batch_stride, head_stride, row_stride;
} sa3k_tensor4;

/* o = softmax(scale * q k^T [+ band mask]) v per (batch, head), head_dim 64; q, k, v, o f16 (IEEE half).
 * window < 0: dense (the DiT's sdpa); window >= 0: keys with |i - j| <= window only (the banded
 * attention of BASELINE config 3).  lse [B*H][Sq] (f32, log2 units) is kept for the backward.
 * Replaces nn::sdpa (src/nn.h:135-144) and the band of attn_sliding (src/nn.h:79-100). */
int sa3k_attention_fwd(sa3k_ctx* ctx, int B, int H, int Sq, int Sk, int head_dim, float scale,
                       int window, const sa3k_tensor4* q, const sa3k_tensor4* k,
                       const sa3k_tensor4* v, const sa3k_tensor4* o, float* lse, char* err,
                       int err_len);

/* Backward of sa3k_attention_fwd for upstream dO (f16): dq, dk, dv (f32; dk and dv may be NULL
 * for a frozen key/value source such as the cross-attention context).  Replaces the
 * SOFT_MAX_BACK / OUT_PROD chain ggml derives for nn::sdpa. */
int sa3k_attention_bwd(sa3k_ctx* ctx, int B, int H, int Sq, int Sk, int head_dim, float scale,
                       int window, const sa3k_tensor4* q, const sa3k_tensor4* k,
                       const sa3k_tensor4* v, const sa3k_tensor4* o, const sa3k_tensor4* dO,
                       const float* lse, const sa3k_tensor4* dq, const sa3k_tensor4* dk,
                       const sa3k_tensor4* dv, char* err, int err_len);

/* sa3k_attention_bwd that never allocates device memory.  No counterpart in the reference: it is
 * for callers that must not allocate during a step -- a process whose device memory is all
 * pre-reserved by its own pool (a cudaMalloc would fail or fragment it), or a latency-sensitive
 * caller that cannot afford the device-wide synchronisation cudaMalloc / cudaFree may imply.
 * Its only scratch (one float per (batch, head, query row)) is a fixed device array inside the
 * library: B*H*Sq must be <= 1,048,576 (4 MiB), larger sizes are rejected with an error.  The
 * first call on each device looks up that array's address (cudaGetSymbolAddress, which may load
 * the library's device code); make that first call before capturing a stream.  All calls on one
 * device share the array, so two calls in flight at the same time (other streams, other
 * contexts, other threads) race: serialise them.  The looked-up address is kept for the life of
 * the process, so resetting a device (cudaDeviceReset, or another library resetting the primary
 * context) while this library is loaded is not supported.  Same arguments and results as
 * sa3k_attention_bwd. */
int sa3k_attention_bwd_noalloc(sa3k_ctx* ctx, int B, int H, int Sq, int Sk, int head_dim,
                               float scale, int window, const sa3k_tensor4* q,
                               const sa3k_tensor4* k, const sa3k_tensor4* v,
                               const sa3k_tensor4* o, const sa3k_tensor4* dO, const float* lse,
                               const sa3k_tensor4* dq, const sa3k_tensor4* dk,
                               const sa3k_tensor4* dv, char* err, int err_len);

/* One head slice of a fused projection output, for sa3k_head_prep_{fwd,bwd}. */
typedef struct sa3k_head_slice {
  int col;              /* first column of the slice in y (a multiple of 64)               */
  const float* gamma;   /* [64] qk RMSNorm weight, or NULL (no norm)                        */
  int rope;             /* apply partial NeoX RoPE after the norm                           */
  float* rstd;          /* [T][H] saved 1/rms per (token, head) when gamma != NULL          */
} sa3k_head_slice;

/* out[T][ncols] (f16) = per-head prepared slices of y[T][ncols] (f32): RMSNorm over each head's
 * 64 values with gamma (eps), then NeoX RoPE of the first `rot` (32 or 64) dims at position
 * (token index mod tokens_per_sample), base `rope_base`.  Replaces the qknorm + rope_neox of
 * dit_block (src/dit.h:195, 209-217; src/nn.h:53-59). */
int sa3k_head_prep_fwd(sa3k_ctx* ctx, const float* y, int T, int ncols, int H,
                       const sa3k_head_slice* slices, int nslices, int tokens_per_sample, float eps,
                       int rot, float rope_base, void* out_f16, char* err, int err_len);

/* Backward of one slice: g[T][H*64] (f32, row stride g_ld) is the gradient w.r.t. the prepared
 * slice; writes the gradient w.r.t. y into that slice of dy[T][ncols] (f32). */
int sa3k_head_prep_bwd(sa3k_ctx* ctx, const float* g, int64_t g_ld, const float* y, int T, int ncols,
                       int H, const sa3k_head_slice* slice, int tokens_per_sample, int rot,
                       float rope_base, float* dy, char* err, int err_len);

/* AdamW hyper-parameters, as TrainAdamWParams (src/train_optimizer.h:28-35). */
typedef struct sa3k_adamw_params {
  float learning_rate, beta1, beta2, eps, weight_decay, grad_clip;
} sa3k_adamw_params;

/* One AdamW update of n parameters with gradient g and moments m, v (updated in place), at
 * optimizer step `step` (>= 1).  Bit-identical to adamw_update_vector
 * (src/train_optimizer.h:42-65) for the same inputs. */
int sa3k_adamw(sa3k_ctx* ctx, float* p, const float* g, float* m, float* v, int64_t n,
               const sa3k_adamw_params* hp, int step, char* err, int err_len);

/* train_apply_accumulated_adamw over flat buffers (src/train_loop.h:147-211): average the
 * accumulated gradient g (n values, `count` samples), clip it to global L2 norm hp->grad_clip
 * (f64 norm; 0 disables), then AdamW.  g is left unmodified.  grad_norm_out (host, nullable)
 * receives the pre-clip norm; it forces a stream sync when requested. */
int sa3k_average_clip_adamw(sa3k_ctx* ctx, float* p, const float* g, float* m, float* v,
                            int64_t n, int count, const sa3k_adamw_params* hp, int step,
                            double* grad_norm_out, char* err, int err_len);

/* ------------------------------------------------------------------ the DiT training step */

/* DiT hyper-parameters, as DitConfig (src/dit.h:20-47) plus the SwiGLU inner width. */
typedef struct sa3k_dit_config {
  int io, dim, depth, heads, head_dim, cond_dim, mem_tokens, rot, time_dim, ff_inner, differential;
  float rope_base, norm_eps, qk_eps, time_min_freq, time_max_freq;
  /* inpaint local-conditioning width (dit.local_dim, src/dit.h:29-30; 0: none).  The per-block
   * dit.N.local.{0,2} tensors then load, and adapters on them are carried (saved, updated by
   * AdamW) with zero gradients: the training step takes no local-conditioning input, as the
   * reference's step without an inpaint input (src/dit.h:246). */
  int local_dim;
} sa3k_dit_config;

typedef struct sa3k_dit sa3k_dit;

/* A DiT bound to a context.  Replaces building the training graphs, build_train_dit_ckpt
 * (src/train_ckpt.h:143-474); the model keeps its activations resident, so no recompute. */
int sa3k_dit_create(sa3k_ctx* ctx, const sa3k_dit_config* cfg, sa3k_dit** out, char* err,
                    int err_len);
void sa3k_dit_free(sa3k_dit* dit);

/* Set one GGUF tensor by its name (the names dit.h reads, e.g. "dit.3.self.qkv.weight",
 * "dit.3.pre_norm.gamma", "dit.memory_tokens").  *.weight tensors may be F32 / F16 / Q8_0 / Q4_K
 * row bytes [ne1 = out][ne0 = in]; every other tensor is F32.  Replaces GgufModel loading
 * (src/gguf_model.h:280-331). */
int sa3k_dit_set_tensor(sa3k_dit* dit, const char* name, int ggml_type, const void* host,
                        int64_t ne0, int64_t ne1, char* err, int err_len);

/* Adapters of any family of the reference on the named weights (rank <= 16): "lora" and
 * "dora-rows" run functionally; "dora-cols", "bora" and every "-xs" form ("lora-xs",
 * "dora-rows-xs", "dora-cols-xs", "bora-xs") through a materialized W_eff rebuilt every step
 * (src/train_dit.h:90-164), the trainable tensors of each target laid out as
 * sa3k_dit_adapter_layout reports; an -xs target needs its frozen bases from
 * sa3k_dit_set_xs_bases before the first step.  Named weights: any 2-D
 * "*.weight" of the DiT, so the reference's `full` and `core` target scopes
 * (enumerate_train_lora_targets, src/train_lora.h:54-117) both fit; head adapters get their
 * gradient through x0, the context and gcond.  Allocates the flat adapter state [A | B | m] per target (order of `names`), zero; for
 * dora-rows computes base_norm_sq and initialises m to the base row norms (src/train_lora.h:
 * 141-174, 262-263).  A and B are then written by the caller through sa3k_dit_adapter_buffer.
 * Counterpart of init_train_lora_state (src/train_lora.h:205-273) for the device state. */
int sa3k_dit_init_adapters(sa3k_dit* dit, const char* adapter_type, int rank, float alpha,
                           const char* const* names, int n, char* err, int err_len);

/* Total floats of the flat adapter state and the offsets of target idx in it (offM = -1 for
 * plain LoRA). */
int64_t sa3k_dit_adapter_size(const sa3k_dit* dit);
int sa3k_dit_adapter_offsets(const sa3k_dit* dit, int idx, int64_t* offA, int64_t* offB,
                             int64_t* offM);
/* Offsets of target idx's tensors in the flat state, -1 where the family has none: offs[0] A
 * [rank][in], offs[1] B [out][rank], offs[2] the row magnitude [out] (dora-rows m, bora m_r),
 * offs[3] the column magnitude [in] (dora-cols m, bora m_c), offs[4] M_xs [rank][rank]
 * (TrainLoraParam, src/train_lora.h:24-33).  Magnitudes start at the base's row / column norms. */
int sa3k_dit_adapter_layout(const sa3k_dit* dit, int idx, int64_t* offs);
/* The frozen bases of an -xs target (host f32): U [out][rank], V [in][rank], the top-rank
 * singular vectors of the base the reference computes or loads at init (init_train_lora_state,
 * src/train_lora.h:223-251); the library takes them from the caller. */
int sa3k_dit_set_xs_bases(sa3k_dit* dit, const char* name, const float* U, const float* V, char* err,
                          int err_len);

/* Device pointer of a flat buffer: 0 parameters, 1 accumulated gradients, 2 AdamW m, 3 AdamW v
 * (TrainLoraState / TrainLoraGradAccum / TrainLoopState of src/train_loop.h:21-39). */
int sa3k_dit_adapter_buffer(sa3k_dit* dit, int which, float** dev_ptr, char* err, int err_len);

/* Copy `count` floats at `offset` of flat buffer `which` (as above) from buf into the model
 * (to_model != 0) or out of it into buf; buf may be host or device memory.  Synchronous.
 * Counterpart of upload_train_lora_state / train_read_grad (src/train_loop.h:41-73). */
int sa3k_dit_adapter_copy(sa3k_dit* dit, int which, float* buf, int64_t offset, int64_t count,
                          int to_model, char* err, int err_len);

/* Zero the accumulated gradients (train_clear_accum, src/train_loop.h:80-82). */
int sa3k_dit_zero_grads(sa3k_dit* dit, char* err, int err_len);

/* Forward + backward of B samples of T frames (replayed from a recorded CUDA graph, see
 * SA3K_OPT_STEP_GRAPH): x_t, target [B][T][io]; t_feat [B][time_dim]
 * (expo_features, src/sa3_pipeline.h:57-67); cross [B][ctx_len][cond_dim]; global [B][cond_dim]
 * (host or device pointers).  Adds the adapter gradients of the summed per-sample losses to the
 * accumulated gradients and writes the B per-sample losses (mean squared error over io*T) to
 * `loss` (host or device, nullable).  Replaces run_train_dit_accumulate_ckpt
 * (src/train_loop.h:309-441) called once per sample. */
int sa3k_dit_forward_backward(sa3k_dit* dit, int B, int T, int ctx_len, const float* x_t,
                              const float* target, const float* t_feat, const float* cross,
                              const float* global, float* loss, char* err, int err_len);

/* The same step with the inpaint objective (run_train_dit_accumulate_ckpt with a TrainInpaint,
 * src/train_loop.h:309-313, src/train_inpaint.h:145-201): local [B][T][local_dim] is the
 * local-add conditioning (build_train_inpaint: the frame mask, then the masked latent), added in
 * every block after the cross-attention as local.2(silu(local.0(local))) to the T real tokens
 * (src/dit.h:244-254); loss_weight [B][T][io] weights the squared error, loss[b] =
 * sum(w (v - target)^2) (src/train_ckpt.h:369).  The model needs dit.local_dim > 0; adapters on the
 * local.* projections themselves are refused (train the core scope).  Runs eagerly. */
int sa3k_dit_forward_backward_inpaint(sa3k_dit* dit, int B, int T, int ctx_len, const float* x_t,
                                      const float* target, const float* t_feat, const float* cross,
                                      const float* global, const float* local, const float* loss_weight,
                                      float* loss, char* err, int err_len);

/* ---- adapter and trainer-state files (the reference's GGUF formats) ----
 * Adapter file (write_train_lora_gguf / load_train_lora_gguf, src/train_checkpoint.h:42-173):
 * metadata general.architecture "sa3-lora", lora.adapter_type, lora.rank, lora.alpha,
 * lora.n_targets; per target <stem>.lora_A f32 ne {in, rank}, <stem>.lora_B ne {rank, out},
 * <stem>.magnitude ne {out} (dora-rows), stem = the weight name without ".weight", targets in
 * name order.  Such a file loads as an adapter in the reference's generator. */
int sa3k_dit_save_adapter(sa3k_dit* dit, const char* path, char* err, int err_len);
/* Adapter values from a file into the model's parameters (train_restore_adapter_values,
 * src/train_resume.h:104-148): type, rank and alpha must equal the model's adapters, the file
 * must hold exactly the model's targets with their shapes. */
int sa3k_dit_load_adapter(sa3k_dit* dit, const char* path, char* err, int err_len);

/* Dataset-side progress stored in the trainer-state file (TrainResumeProgress,
 * src/train_resume.h:23-37): the trainer's epoch, cursor and sample order, its compatibility
 * string and the serialized random-engine states of its samplers. */
typedef struct sa3k_train_progress {
  uint64_t epoch;
  uint64_t next_sample;
  const uint64_t* order;
  int64_t n_order;
  const char* compatibility;
  const char* rng_shuffle;
  const char* rng_crop;
  const char* rng_cfg;
  const char* rng_prompt;
  const char* rng_inpaint;
  const char* rng_diffusion;
} sa3k_train_progress;

/* Immutable checkpoint pair (write_train_checkpoint_pair, src/train_resume.h:502-538): the adapter
 * file and a trainer-state file (general.architecture "sa3-trainer-state", trainer.* metadata,
 * optimizer.<stem>.<lora_A|lora_B|magnitude>.<m|v> f32 AdamW moments) bound to the adapter by its
 * FNV-1a fingerprint.  Refuses to overwrite either file; both are written to ".tmp" names and
 * renamed, the state last.  `step` = the number of AdamW updates applied so far. */
int sa3k_dit_save_checkpoint(sa3k_dit* dit, const char* adapter_path, const char* state_path, int64_t step,
                             const sa3k_train_progress* progress, char* err, int err_len);
/* Restores parameters and AdamW moments from a pair (load_train_state_gguf,
 * src/train_resume.h:394-500): the adapter must match the state's fingerprint and the state's
 * target inventory the model's; returns the step.  The dataset-side progress is read back with
 * the sa3k_gguf_get_* calls below. */
int sa3k_dit_load_checkpoint(sa3k_dit* dit, const char* adapter_path, const char* state_path, int64_t* step,
                             char* err, int err_len);

/* Host-only file helpers (no device needed). */
/* An adapter file from host arrays (the same format as sa3k_dit_save_adapter); m may be NULL
 * (plain LoRA) or hold NULL entries. */
int sa3k_adapter_gguf_write(const char* path, const char* adapter_type, int rank, float alpha, int n,
                            const char* const* stems, const int64_t* in, const int64_t* out, const float* const* A,
                            const float* const* B, const float* const* m, char* err, int err_len);
/* Metadata of a GGUF file: a string (copied NUL-terminated into buf, its length to len_out), an
 * unsigned integer, an unsigned integer array (up to max elements, the count to n_out). */
int sa3k_gguf_get_string(const char* path, const char* key, char* buf, int64_t buf_len, int64_t* len_out,
                         char* err, int err_len);
int sa3k_gguf_get_u64(const char* path, const char* key, uint64_t* value, char* err, int err_len);
int sa3k_gguf_get_u64_array(const char* path, const char* key, uint64_t* out, int64_t max, int64_t* n_out,
                            char* err, int err_len);
/* An f32 tensor of a GGUF file (up to max values; the element count to n_out, dims to ne[4] and
 * n_dims). */
int sa3k_gguf_get_f32(const char* path, const char* name, float* out, int64_t max, int64_t* n_out, int64_t* ne,
                      int* n_dims, char* err, int err_len);

/* Average over `count` samples, clip, AdamW (train_apply_accumulated_adamw,
 * src/train_loop.h:173-211) on the flat state. */
int sa3k_dit_apply_adamw(sa3k_dit* dit, int count, const sa3k_adamw_params* hp, int step,
                         double* grad_norm_out, char* err, int err_len);

/* ---------------------------------------------------------------- data parallel (NCCL)
 * One process per GPU.  The reference trains on one device and sums per-sample gradients on the
 * host (src/train_loop.h:84-134) before train_average_and_clip (src/train_loop.h:147-171); over
 * ranks that sum becomes an all-reduce and the average divides by samples-per-rank x ranks, so
 * every rank applies the identical AdamW update.  NCCL is loaded at run time (libnccl.so.2, or
 * the path in SA3K_NCCL_LIBRARY); without it these calls return an error. */
typedef struct sa3k_dp_comm sa3k_dp_comm;

/* 128 opaque bytes made on one rank and handed to every rank (by the caller's own means). */
int sa3k_dp_unique_id(void* out, int out_len, char* err, int err_len);
/* Collective over all nranks processes (each with its own context / device).  The rendezvous is
 * bounded: a communicator whose ranks have not all joined within 300 s is aborted and the call
 * returns an error (sa3k_dp_comm_create_timeout sets the bound). */
int sa3k_dp_comm_create(sa3k_ctx* ctx, int nranks, int rank, const void* unique_id,
                        sa3k_dp_comm** out, char* err, int err_len);
int sa3k_dp_comm_create_timeout(sa3k_ctx* ctx, int nranks, int rank, const void* unique_id,
                                double timeout_s, sa3k_dp_comm** out, char* err, int err_len);
void sa3k_dp_comm_destroy(sa3k_dp_comm* comm);
int sa3k_dp_comm_info(const sa3k_dp_comm* comm, int* nranks, int* rank);
/* In-place sum of buf[n] (f32, device) over all ranks, on the context's stream. */
int sa3k_dp_allreduce_sum(sa3k_ctx* ctx, sa3k_dp_comm* comm, float* buf, int64_t n, char* err,
                          int err_len);
/* All-reduce g, then sa3k_average_clip_adamw with count = samples_per_rank x nranks: the
 * data-parallel form of train_apply_accumulated_adamw (src/train_loop.h:173-211). */
int sa3k_dp_allreduce_adamw(sa3k_ctx* ctx, sa3k_dp_comm* comm, float* p, float* g, float* m,
                            float* v, int64_t n, int samples_per_rank,
                            const sa3k_adamw_params* hp, int step, double* grad_norm_out,
                            char* err, int err_len);
/* sa3k_dp_allreduce_adamw on a DiT's flat adapter state. */
int sa3k_dit_dp_apply_adamw(sa3k_dit* dit, sa3k_dp_comm* comm, int samples_per_rank,
                            const sa3k_adamw_params* hp, int step, double* grad_norm_out,
                            char* err, int err_len);

#ifdef __cplusplus
}
#endif

#endif /* SA3K_H */
