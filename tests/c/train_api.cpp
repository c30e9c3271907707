// train_api.cpp -- drives the reference's training API (include/sa3_train.h, namespace sa3) the way
// tools/sa3-train.cpp does: load the DiT GGUF, enumerate targets, seeded init_train_lora_state,
// the diffusion sampler, build_train_dit_ckpt, run_train_dit_accumulate_ckpt per sample and
// train_apply_accumulated_adamw once per batch.  Every value the checks need is written to
// <out_dir> as raw float32 / float64 files; tests/test_gpu_host_api.py compares them with the
// float64 oracle and the reference's compiled sampler.
//
//   train_api cpu <out_dir>                         sampler streams + a "lora" init (no GPU)
//   train_api gpu <model.gguf> <inputs.bin> <out_dir>   two optimizer steps of two samples each
#include "sa3_train.h"

#include <cstdio>
#include <cstdlib>
#include <fstream>
#include <string>
#include <vector>

namespace {

void put(const std::string& path, const void* p, size_t bytes) {
    std::ofstream f(path, std::ios::binary);
    f.write(static_cast<const char*>(p), (std::streamsize)bytes);
    if (!f) {
        std::fprintf(stderr, "cannot write %s\n", path.c_str());
        std::exit(2);
    }
}
void putf(const std::string& path, const std::vector<float>& v) { put(path, v.data(), v.size() * sizeof(float)); }

// all trainable vectors of the state, target after target: lora_A, lora_B, magnitude
std::vector<float> flat_state(const sa3::TrainLoraState& st) {
    std::vector<float> out;
    for (const auto& p : st.params)
        for (const auto* v : {&p.lora_A, &p.lora_B, &p.magnitude}) out.insert(out.end(), v->begin(), v->end());
    return out;
}

int cpu_mode(const std::string& dir) {
    // sampler streams: per mode, 5 draws of t, each followed by the noise of a 7-value latent
    const std::vector<float> z = {0.5f, -1.f, 2.f, 0.25f, -0.75f, 1.5f, 0.f};
    for (const char* mode : {"uniform", "trunc_logit_normal"}) {
        sa3::TrainDiffusionSampler s(20240611ull, mode);
        std::vector<float> t, noise, xt, vt;
        std::string err;
        for (int i = 0; i < 5; ++i) {
            sa3::TrainDiffusionSample out;
            if (!s.sample(z, out, err)) {
                std::fprintf(stderr, "sample: %s\n", err.c_str());
                return 1;
            }
            t.push_back(out.t);
            noise.insert(noise.end(), out.noise.begin(), out.noise.end());
            xt.insert(xt.end(), out.x_t.begin(), out.x_t.end());
            vt.insert(vt.end(), out.velocity_target.begin(), out.velocity_target.end());
        }
        // a serialized state restores the stream exactly (the trainer's resume contract)
        const std::string state = s.serialize_state();
        sa3::TrainDiffusionSampler r(1ull, mode);
        if (!r.restore_state(state, err) || s.draw_t() != r.draw_t()) {
            std::fprintf(stderr, "sampler state did not round-trip\n");
            return 1;
        }
        const std::string m(mode);
        putf(dir + "/sampler_" + m + "_t.f32", t);
        putf(dir + "/sampler_" + m + "_noise.f32", noise);
        putf(dir + "/sampler_" + m + "_xt.f32", xt);
        putf(dir + "/sampler_" + m + "_v.f32", vt);
    }
    // "lora" init needs no device: A ~ kaiming-uniform from mt19937_64(seed), B = 0
    sa3::GgufModel model;
    const int64_t shapes[4][2] = {{96, 64}, {64, 160}, {128, 64}, {64, 64}};   // (in, out)
    const char* names[4] = {"dit.0.self.qkv.weight", "dit.0.ff.proj.weight", "dit.1.self.out.weight",
                            "dit.proj_in.weight"};
    for (int i = 0; i < 4; ++i) {
        sa3::GgufTensor t;
        t.type = 0;
        t.n_dims = 2;
        t.ne[0] = shapes[i][0];
        t.ne[1] = shapes[i][1];
        t.data.assign((size_t)(shapes[i][0] * shapes[i][1] * 4), 0);
        model.tensors[names[i]] = t;
    }
    sa3::GgufTensor vec;
    vec.type = 0;
    vec.n_dims = 1;
    vec.ne[0] = 64;
    vec.data.assign(256, 0);
    model.tensors["dit.0.pre_norm.gamma"] = vec;   // 1-D: never a target
    sa3::TrainLoraScope core;
    core.name = "core";
    auto targets = sa3::enumerate_train_lora_targets(model, core);
    auto all = sa3::enumerate_train_lora_targets(model);
    std::string err;
    sa3::TrainLoraState st;
    if (targets.size() != 3 || all.size() != 4 ||
        !sa3::init_train_lora_state(model, all, "lora", 4, 8.0f, 987654321ull, st, err)) {
        std::fprintf(stderr, "init: %zu %zu %s\n", targets.size(), all.size(), err.c_str());
        return 1;
    }
    std::vector<float> A, B;
    std::string order;
    for (const auto& p : st.params) {
        A.insert(A.end(), p.lora_A.begin(), p.lora_A.end());
        B.insert(B.end(), p.lora_B.begin(), p.lora_B.end());
        order += p.target.weight_name + "\n";
    }
    putf(dir + "/init_lora_A.f32", A);
    putf(dir + "/init_lora_B.f32", B);
    put(dir + "/init_order.txt", order.data(), order.size());
    // refused: rank above a target's width, unknown type, -xs without bases
    if (sa3::init_train_lora_state(model, all, "lora", 100, 1.f, 1ull, st, err) ||
        sa3::init_train_lora_state(model, all, "vera", 4, 1.f, 1ull, st, err) ||
        sa3::init_train_lora_state(model, all, "lora-xs", 4, 1.f, 1ull, st, err)) {
        std::fprintf(stderr, "an invalid init was accepted\n");
        return 1;
    }
    std::printf("OK\n");
    return 0;
}

int gpu_mode(const std::string& model_path, const std::string& inputs_path, const std::string& dir) {
    sa3::Backend be = sa3::make_backend(0);
    sa3::GgufModel model = sa3::load_gguf(model_path.c_str(), be);
    const sa3::DitConfig dc = sa3::DitConfig::from(model);
    // inputs: int32 header (n_samples, T, C), then z [n][T][io], cross [n][C][cond_dim], global [n][cond_dim]
    std::ifstream in(inputs_path, std::ios::binary);
    int32_t hdr[3];
    in.read(reinterpret_cast<char*>(hdr), sizeof hdr);
    const int n = hdr[0], T = hdr[1], C = hdr[2];
    std::vector<float> z((size_t)n * T * dc.io), cross((size_t)n * C * dc.cond_dim), glob((size_t)n * dc.cond_dim);
    in.read(reinterpret_cast<char*>(z.data()), (std::streamsize)(z.size() * 4));
    in.read(reinterpret_cast<char*>(cross.data()), (std::streamsize)(cross.size() * 4));
    in.read(reinterpret_cast<char*>(glob.data()), (std::streamsize)(glob.size() * 4));
    if (!in || n != 4) {
        std::fprintf(stderr, "bad inputs file\n");
        return 1;
    }
    sa3::TrainLoraScope scope;
    scope.include = {".self.qkv.", ".self.out.", ".ff.proj.", ".ff.out."};
    const auto targets = sa3::enumerate_train_lora_targets(model, scope);
    sa3::TrainLoraState lora;
    std::string err;
    if (!sa3::init_train_lora_state(model, targets, "dora-rows", 4, 8.0f, 1234ull, lora, err)) {
        std::fprintf(stderr, "init: %s\n", err.c_str());
        return 1;
    }
    putf(dir + "/state0.f32", flat_state(lora));
    std::string order;
    for (const auto& p : lora.params) order += p.target.weight_name + "\n";
    put(dir + "/order.txt", order.data(), order.size());

    sa3::TrainDiffusionSampler sampler(77ull, "uniform");
    sa3::TrainLoopState loop;
    sa3::TrainLoraGradAccum accum;
    sa3::TrainDitCkpt ck;
    sa3::TrainAdamWParams hp;
    hp.learning_rate = 1e-3f;
    hp.weight_decay = 0.01f;
    hp.grad_clip = 1.0f;
    const int batch = 2;
    for (int i = 0; i < n; ++i) {
        sa3::TrainConditioning cond;
        cond.cond_dim = dc.cond_dim;
        cond.ctx_len = C;
        cond.cross.assign(cross.begin() + (long)i * C * dc.cond_dim, cross.begin() + (long)(i + 1) * C * dc.cond_dim);
        cond.global.assign(glob.begin() + (long)i * dc.cond_dim, glob.begin() + (long)(i + 1) * dc.cond_dim);
        if (!ck.pctx && !sa3::build_train_dit_ckpt(model, dc, lora, T, cond.cond_dim, cond.ctx_len, ck, err)) {
            std::fprintf(stderr, "build: %s\n", err.c_str());
            return 1;
        }
        const std::vector<float> zi(z.begin() + (long)i * T * dc.io, z.begin() + (long)(i + 1) * T * dc.io);
        sa3::TrainDiffusionSample sample;
        if (!sampler.sample(zi, sample, err)) return 1;
        float loss = 0.f;
        if (!sa3::run_train_dit_accumulate_ckpt(be, ck, lora, accum, sample, cond, dc, loss, err)) {
            std::fprintf(stderr, "step: %s\n", err.c_str());
            return 1;
        }
        const std::string tag = dir + "/s" + std::to_string(i);
        putf(tag + "_xt.f32", sample.x_t);
        putf(tag + "_v.f32", sample.velocity_target);
        putf(tag + "_t.f32", {sample.t, loss});
        if (accum.count >= batch) {
            std::vector<float> g;
            for (size_t k = 0; k < lora.params.size(); ++k)
                for (const auto* v : {&accum.A[k], &accum.B[k], &accum.mag[k]}) g.insert(g.end(), v->begin(), v->end());
            const int step = loop.step + 1;
            putf(dir + "/grad" + std::to_string(step) + ".f32", g);
            double norm = 0.0;
            if (!sa3::train_apply_accumulated_adamw(lora, accum, loop, hp, err, &norm)) {
                std::fprintf(stderr, "adamw: %s\n", err.c_str());
                return 1;
            }
            if (accum.count != 0 || loop.step != step) return 1;
            put(dir + "/norm" + std::to_string(step) + ".f64", &norm, sizeof norm);
            putf(dir + "/state" + std::to_string(step) + ".f32", flat_state(lora));
            std::vector<float> mv;
            for (size_t k = 0; k < lora.params.size(); ++k)
                for (const auto* s : {&loop.A_state[k], &loop.B_state[k], &loop.mag_state[k]}) {
                    mv.insert(mv.end(), s->m.begin(), s->m.end());
                    mv.insert(mv.end(), s->v.begin(), s->v.end());
                }
            putf(dir + "/moments" + std::to_string(step) + ".f32", mv);
        }
    }
    // an empty batch and an inpaint input are refused
    sa3::TrainInpaint ip;
    float loss = 0.f;
    sa3::TrainDiffusionSample sample;
    std::vector<float> z0(z.begin(), z.begin() + (long)T * dc.io);
    sampler.sample(z0, sample, err);
    sa3::TrainConditioning cond;
    cond.cond_dim = dc.cond_dim;
    cond.ctx_len = C;
    cond.cross.assign(cross.begin(), cross.begin() + (long)C * dc.cond_dim);
    cond.global.assign(glob.begin(), glob.begin() + dc.cond_dim);
    if (sa3::train_apply_accumulated_adamw(lora, accum, loop, hp, err) ||
        sa3::run_train_dit_accumulate_ckpt(be, ck, lora, accum, sample, cond, dc, loss, err, &ip)) {
        std::fprintf(stderr, "an invalid call was accepted\n");
        return 1;
    }
    // the device model is released with its last owner, before the backend
    sa3::free_train_dit_ckpt(ck);
    accum.device.reset();
    model.device.reset();
    sa3::free_backend(be);
    std::printf("OK\n");
    return 0;
}

}  // namespace

int main(int argc, char** argv) {
    try {
        if (argc == 3 && std::string(argv[1]) == "cpu") return cpu_mode(argv[2]);
        if (argc == 5 && std::string(argv[1]) == "gpu") return gpu_mode(argv[2], argv[3], argv[4]);
    } catch (const sa3::gguf_error& e) {
        std::fprintf(stderr, "gguf_error: %s\n", e.what());
        return 1;
    }
    std::fprintf(stderr, "usage: train_api cpu <out_dir> | gpu <model.gguf> <inputs.bin> <out_dir>\n");
    return 2;
}
