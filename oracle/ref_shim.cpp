// oracle/ref_shim.cpp -- C entry points over the reference's own std-only headers.
//
// TEST INFRASTRUCTURE ONLY.  Compiled by oracle/Makefile against the reference tree's headers
// where they lie (-I <reference>/src); the headers are not copied.  The result,
// oracle/_ref/libsa3ref.so, is the reference's own CPU code for:
//   - AdamW:        src/train_optimizer.h:42-65   (sa3::adamw_update_vector)
//   - LR schedule:  src/train_optimizer.h:20-26   (sa3::inverse_lr)
//   - diffusion:    src/train_diffusion.h:50-125  (sa3::TrainDiffusionSampler: sample_at, draw_t)
// The average / global-norm clip of src/train_loop.h:147-171 sits in a header that pulls in
// ggml, so it cannot be compiled here; tests pin it through the oracle restatement instead.
#include "train_diffusion.h"
#include "train_optimizer.h"

#include <cstring>
#include <string>
#include <vector>

extern "C" {

// One AdamW update of n parameters; m, v are the moments (updated in place).
// Returns 0 on success, 1 with the reference's error text copied into err otherwise.
int sa3ref_adamw_update(float* param, const float* grad, float* m, float* v, long n, float lr,
                        float beta1, float beta2, float eps, float weight_decay, int step,
                        char* err, int err_len) {
    std::vector<float> p(param, param + n), g(grad, grad + n);
    sa3::TrainAdamWTensorState st;
    st.m.assign(m, m + n);
    st.v.assign(v, v + n);
    sa3::TrainAdamWParams hp;
    hp.learning_rate = lr;
    hp.beta1 = beta1;
    hp.beta2 = beta2;
    hp.eps = eps;
    hp.weight_decay = weight_decay;
    std::string e;
    if (!sa3::adamw_update_vector(p, g, st, hp, step, e)) {
        if (err && err_len > 0) {
            std::strncpy(err, e.c_str(), (size_t)err_len - 1);
            err[err_len - 1] = 0;
        }
        return 1;
    }
    std::memcpy(param, p.data(), sizeof(float) * (size_t)n);
    std::memcpy(m, st.m.data(), sizeof(float) * (size_t)n);
    std::memcpy(v, st.v.data(), sizeof(float) * (size_t)n);
    return 0;
}

float sa3ref_inverse_lr(float base_lr, int step0, float inv_gamma, float power, float warmup,
                        float final_lr) {
    return sa3::inverse_lr(base_lr, step0, inv_gamma, power, warmup, final_lr);
}

// x_t = (1-t) z + t n, v = n - z with the reference's seeded normal stream.
int sa3ref_diffusion_sample_at(unsigned long long seed, const float* z, long n, float t,
                               float* noise, float* x_t, float* v_target) {
    sa3::TrainDiffusionSampler s(seed);
    std::vector<float> zz(z, z + n);
    sa3::TrainDiffusionSample out;
    std::string e;
    if (!s.sample_at(zz, t, out, e)) return 1;
    std::memcpy(noise, out.noise.data(), sizeof(float) * (size_t)n);
    std::memcpy(x_t, out.x_t.data(), sizeof(float) * (size_t)n);
    std::memcpy(v_target, out.velocity_target.data(), sizeof(float) * (size_t)n);
    return 0;
}

// n_steps draws of one sampler stream: t_out[i] = draw_t(), then sample_at(z, t) fills
// noise[i*n ...]: the interleaving of the trainer's loop (draw_t, then the noise of that sample).
int sa3ref_diffusion_stream(unsigned long long seed, const char* mode, const float* z, long n, int n_steps,
                            float* t_out, float* noise) {
    sa3::TrainDiffusionSampler s(seed, mode);
    std::vector<float> zz(z, z + n);
    sa3::TrainDiffusionSample out;
    std::string e;
    for (int i = 0; i < n_steps; ++i) {
        t_out[i] = s.draw_t();
        if (!s.sample_at(zz, t_out[i], out, e)) return 1;
        std::memcpy(noise + (size_t)i * n, out.noise.data(), sizeof(float) * (size_t)n);
    }
    return 0;
}

}  // extern "C"
