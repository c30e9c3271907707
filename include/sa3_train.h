/*
 * sa3_train.h -- the reference's C++ training API (namespace sa3) over the B200 library.
 *
 * sa3.cpp's trainer (tools/sa3-train.cpp) drives one adapter-training step through header-only
 * functions of src/train_loop.h, src/train_ckpt.h, src/train_lora.h, src/train_optimizer.h and
 * src/train_diffusion.h on a ggml backend.  This header declares the same functions with the
 * same names, argument lists, types and error convention (bool return + std::string& err; the
 * model loader throws gguf_error as src/gguf_model.h does), with ggml_backend_t replaced by a
 * device context (sa3::Backend = sa3k_ctx*).  The trainer's step code compiles against it
 * unchanged apart from the backend argument; the implementation (sa3.cpp_b200/csrc/
 * sa3_train.cpp, linked into libsa3k.so) runs the step through the sa3k C ABI: the DiT forward
 * and backward, the gradient accumulation and the averaged, clipped AdamW all run on the GPU.
 *
 * Ownership follows the reference: the host owns the adapter state (TrainLoraState), the
 * optimizer moments (TrainLoopState) and the accumulated gradients (TrainLoraGradAccum) as
 * std::vector<float>; every step call uploads the adapters and downloads that sample's
 * gradients into the accumulator, and train_apply_accumulated_adamw runs the update on the device
 * the accumulator was filled on and writes parameters and moments back.  TrainDitCkpt owns the
 * device model (weights uploaded once per GgufModel and reused across rebuilds).
 */
#pragma once

#include "sa3k.h"

#include <cstdint>
#include <map>
#include <memory>
#include <random>
#include <stdexcept>
#include <string>
#include <vector>

namespace sa3 {

// ------------------------------------------------------------------ backend and model files
// Replaces ggml_backend_t / make_backend(cpu_threads) (src/gguf_model.h:120-198): a context on
// one CUDA device (sm_100).  make_backend throws gguf_error when no such device is usable.
using Backend = sa3k_ctx*;
Backend make_backend(int device = 0);
void free_backend(Backend backend);

struct gguf_error : std::runtime_error {
    using std::runtime_error::runtime_error;
};

// One tensor of a GGUF file: ggml type id, dims (ne[0] innermost) and its raw row bytes.
struct GgufTensor {
    int type = 0;
    int n_dims = 0;
    int64_t ne[4] = {1, 1, 1, 1};
    std::vector<uint8_t> data;
};

struct DitDevice;   // the uploaded device model of a GgufModel (internal)

// Replaces GgufModel (src/gguf_model.h:200-278): the tensors and metadata of a model file, held
// in host memory until a training graph uploads them.
struct GgufModel {
    Backend backend = nullptr;
    std::map<std::string, GgufTensor> tensors;
    std::map<std::string, uint64_t> u64_kv;      // unsigned / signed / bool metadata
    std::map<std::string, double> f64_kv;        // float metadata
    std::map<std::string, std::string> str_kv;   // string metadata
    std::shared_ptr<DitDevice> device;           // set by build_train_dit_ckpt, reused afterwards

    bool has(const std::string& name) const { return tensors.count(name) != 0; }
    const GgufTensor* get(const std::string& name) const;   // throws gguf_error when absent
    uint32_t u32(const std::string& key) const;             // throws gguf_error when absent
    float f32(const std::string& key) const;                // throws gguf_error when absent
};

// Replaces load_gguf (src/gguf_model.h:280-331): parses a GGUF v3 file; throws gguf_error.
GgufModel load_gguf(const char* path, Backend backend = nullptr);

// src/dit.h:20-47.  ff_inner (not a field of the reference) is read from dit.0.ff.proj.weight.
struct DitConfig {
    int io = 0, dim = 0, depth = 0, heads = 0, head_dim = 0, cond_dim = 0, mem_tokens = 0, rot = 0, time_dim = 0,
        local_dim = 0;
    float rope_base = 0, norm_eps = 0, qk_eps = 0, time_min_freq = 0, time_max_freq = 0;
    bool differential = true;
    int ff_inner = 0;
    static DitConfig from(const GgufModel& m);
};

// ------------------------------------------------------------------ adapter state (train_lora.h)
struct TrainLoraTarget {
    std::string weight_name;
    std::string stem;
    int64_t in = 0;
    int64_t out = 0;
};

struct TrainLoraParam {
    TrainLoraTarget target;
    std::vector<float> lora_A;       // [rank, in]
    std::vector<float> lora_B;       // [out, rank]
    std::vector<float> U;            // [out, rank] for -xs
    std::vector<float> V;            // [in, rank] for -xs
    std::vector<float> M_xs;         // [rank, rank] for -xs
    std::vector<float> magnitude;    // dora-rows [out] or dora-cols [in]
    std::vector<float> magnitude_r;  // bora [out]
    std::vector<float> magnitude_c;  // bora [in]
};

struct TrainLoraState {
    std::string adapter_type = "lora";
    int rank = 0;
    float alpha = 1.0f;
    std::vector<TrainLoraParam> params;
};

// src/train_lora.h:54-117: "full" (every 2-D dit.*.weight) or "core" (the per-block
// projections without local.*), then include / exclude substring filters.
struct TrainLoraScope {
    std::string name = "full";
    std::vector<std::string> include;
    std::vector<std::string> exclude;
};
bool train_lora_scope_known(const std::string& s);
std::vector<TrainLoraTarget> enumerate_train_lora_targets(const GgufModel& dit, const TrainLoraScope& scope = {});

// src/train_lora.h:205-273: A ~ kaiming-uniform U(-1/sqrt(in), 1/sqrt(in)) drawn from
// std::mt19937_64(seed) target after target, B = 0; magnitudes = the dequantized base's row
// (dora-rows, bora m_r) or column (dora-cols, bora m_c) norms, computed on the backend's device;
// -xs families take U / V from svd_bases (the randomized SVD of the reference is not built:
// without bases an -xs type is refused) and start M_xs at 0.  rank <= 16.
bool init_train_lora_state(const GgufModel& dit, const std::vector<TrainLoraTarget>& targets,
                           const std::string& adapter_type, int rank, float alpha, unsigned long long seed,
                           TrainLoraState& out, std::string& err, const GgufModel* svd_bases = nullptr);

// ------------------------------------------------------------------ optimizer (train_optimizer.h)
float inverse_lr(float base_lr, int step0, float inv_gamma, float power, float warmup, float final_lr);

struct TrainAdamWParams {
    float learning_rate = 1.0e-4f;
    float beta1 = 0.9f;
    float beta2 = 0.999f;
    float eps = 1.0e-8f;
    float weight_decay = 0.0f;
    float grad_clip = 0.0f;
};

struct TrainAdamWTensorState {
    std::vector<float> m;
    std::vector<float> v;
};

// ------------------------------------------------------------------ loop state (train_loop.h)
struct TrainLoopState {
    int step = 0;
    std::vector<TrainAdamWTensorState> A_state;
    std::vector<TrainAdamWTensorState> B_state;
    std::vector<TrainAdamWTensorState> mxs_state;
    std::vector<TrainAdamWTensorState> mag_state;
    std::vector<TrainAdamWTensorState> mag_r_state;
    std::vector<TrainAdamWTensorState> mag_c_state;
};

struct TrainLoraGradAccum {
    int count = 0;
    std::vector<std::vector<float>> A;
    std::vector<std::vector<float>> B;
    std::vector<std::vector<float>> mxs;
    std::vector<std::vector<float>> mag;
    std::vector<std::vector<float>> mag_r;
    std::vector<std::vector<float>> mag_c;
    std::shared_ptr<DitDevice> device;   // the device model the gradients were computed on
};

void train_clear_accum(TrainLoraGradAccum& accum);

// src/train_loop.h:173-211: step += 1; average over accum.count, global-norm clip, AdamW on
// every trainable vector; clears the accumulator.  Runs on the device the accumulator was filled
// on (the flat-buffer kernels of sa3k_average_clip_adamw, bit-exact with the reference's host
// loop), then writes the parameters and moments back into state and loop.
bool train_apply_accumulated_adamw(TrainLoraState& state, TrainLoraGradAccum& accum, TrainLoopState& loop,
                                   const TrainAdamWParams& hp, std::string& err, double* grad_norm_out = nullptr);

// ------------------------------------------------------------------ diffusion (train_diffusion.h)
struct TrainDiffusionSample {
    float t = 0.0f;
    std::vector<float> noise;
    std::vector<float> x_t;
    std::vector<float> velocity_target;
};

// src/train_diffusion.h:50-125: t ~ U(0, 1) or the truncated logit-normal draw, noise ~ N(0, 1)
// from one std::mt19937_64 stream; x_t = (1 - t) z + t n, v = n - z.  Same engine, same
// standard-library distributions and draw order, so a seed gives the reference's stream.
class TrainDiffusionSampler {
public:
    explicit TrainDiffusionSampler(unsigned long long seed, const std::string& mode = "uniform");
    bool sample(const std::vector<float>& z, TrainDiffusionSample& out, std::string& err);
    bool sample_at(const std::vector<float>& z, float t, TrainDiffusionSample& out, std::string& err);
    float draw_t();
    std::string serialize_state() const;
    bool restore_state(const std::string& state, std::string& err);

private:
    std::mt19937_64 rng_;
    std::string mode_;
    std::uniform_real_distribution<float> uniform_{0.0f, 1.0f};
    std::normal_distribution<float> normal_{0.0f, 1.0f};
};

// ------------------------------------------------------------------ conditioning and inpainting
// src/train_conditioning.h:16-22: cross [ctx rows][cond_dim] (the first ctx_len rows are read),
// global [cond_dim].
struct TrainConditioning {
    std::vector<float> cross;
    std::vector<float> global;
    int cond_dim = 0;
    int ctx_len = 0;
    int token_count = 0;
};

// src/train_inpaint.h:145-150: local [frames][local_dim] (the frame mask, then the masked latent)
// and loss_weight [frames][io] (build_train_inpaint).  A graph built with inpaint = true takes them
// every step: the local-add conditioning runs in every block on the device and the loss is the
// weighted sum.  Adapters on the local.* projections themselves are refused (the core scope).
enum class InpaintMaskType { Segments, FullMask, Causal, Spans };
struct TrainInpaint {
    std::vector<float> local;
    std::vector<float> loss_weight;
    InpaintMaskType type = InpaintMaskType::FullMask;
    int n_gen = 0, n_ctx = 0;
};

// ------------------------------------------------------------------ the checkpointed step (train_ckpt.h)
// Replaces TrainDitCkpt (src/train_ckpt.h:73-127).  pctx is non-null once built (the trainer
// tests it to decide whether to build).
struct TrainDitCkpt {
    void* pctx = nullptr;
    std::shared_ptr<DitDevice> device;
    bool inpaint = false;
    int frames = 0, cond_dim = 0, ctx_len = 0;
};

// src/train_ckpt.h:143-145: uploads the model's dit.* tensors (once per GgufModel; rebuilding
// for another shape reuses them) and the adapter layout of `lora`.
bool build_train_dit_ckpt(GgufModel& dit, const DitConfig& dc, const TrainLoraState& lora, int frames, int cond_dim,
                          int ctx_len, TrainDitCkpt& out, std::string& err, bool inpaint = false);
void free_train_dit_ckpt(TrainDitCkpt& ck);

// src/train_loop.h:309-313: one sample's forward + backward; adds its adapter gradients to accum
// (count += 1) and writes its loss.
bool run_train_dit_accumulate_ckpt(Backend backend, TrainDitCkpt& ck, const TrainLoraState& lora,
                                   TrainLoraGradAccum& accum, const TrainDiffusionSample& sample,
                                   const TrainConditioning& cond, const DitConfig& dc, float& loss_out,
                                   std::string& err, const TrainInpaint* inpaint = nullptr);

}  // namespace sa3
