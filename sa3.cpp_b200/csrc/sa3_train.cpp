// sa3_train.cpp -- the reference's namespace-sa3 training API (include/sa3_train.h) over the sa3k
// C ABI.  Host code: model files, adapter-state bookkeeping, the seeded initialisation and the
// diffusion sampler; every tensor computation of the step (DiT forward / backward, magnitude
// norms, average + clip + AdamW) runs on the device through sa3k_*.
#include "../../include/sa3_train.h"

#include "gguf_io.h"

#include <cuda_runtime.h>

#include <algorithm>
#include <array>
#include <cctype>
#include <cmath>
#include <cstring>
#include <sstream>

namespace sa3 {

// ------------------------------------------------------------------ the device model
struct DitDevice {
    sa3k_ctx* ctx = nullptr;
    sa3k_dit* dit = nullptr;
    DitConfig dc;
    std::string adapter_type;
    int rank = 0;
    float alpha = 0.f;
    std::vector<std::string> targets;
    std::vector<std::array<int64_t, 5>> layout;   // A, B, row magnitude, column magnitude, M_xs
    std::vector<int64_t> in, out;
    int64_t np = 0;
    std::vector<float> stage;                     // host image of one flat buffer
    ~DitDevice() {
        if (dit) sa3k_dit_free(dit);
    }
};

namespace {

constexpr int kErrLen = 1024;

bool fail(std::string& err, const std::string& msg) {
    err = msg;
    return false;
}

bool ok_or(int rc, const char* buf, std::string& err) {
    if (rc == 0) return true;
    err = buf;
    return false;
}

bool is_xs(const std::string& t) { return t.size() >= 3 && t.compare(t.size() - 3, 3, "-xs") == 0; }
std::string family(const std::string& t) { return is_xs(t) ? t.substr(0, t.size() - 3) : t; }

// Bytes of a ggml tensor of n elements (the block sizes of the GGUF formats).
bool type_bytes(int type, uint64_t n, uint64_t& bytes) {
    struct B { int id; uint64_t block, size; };
    static const B table[] = {{0, 1, 4},     {1, 1, 2},     {2, 32, 18},   {3, 32, 20},   {6, 32, 22},
                              {7, 32, 24},   {8, 32, 34},   {9, 32, 36},   {10, 256, 84}, {11, 256, 110},
                              {12, 256, 144}, {13, 256, 176}, {14, 256, 210}, {15, 256, 292}, {30, 1, 2}};
    for (const B& b : table)
        if (b.id == type) {
            if (n % b.block) return false;
            bytes = n / b.block * b.size;
            return true;
        }
    return false;
}

// src/sa3_pipeline.h:57-67: [cos, sin](t f 2 pi), f log-spaced in [min_f, max_f], f32 arithmetic.
void expo_features(float t, std::vector<float>& out, int dim, float min_f, float max_f) {
    const int half = dim / 2;
    const float lmin = std::log(min_f), lmax = std::log(max_f), two_pi = 6.28318530717958648f;
    out.assign((size_t)dim, 0.f);
    for (int i = 0; i < half; ++i) {
        const float ramp = half > 1 ? (float)i / (float)(half - 1) : 0.f;
        const float freq = std::exp(ramp * (lmax - lmin) + lmin);
        const float arg = t * freq * two_pi;
        out[(size_t)i] = std::cos(arg);
        out[(size_t)(half + i)] = std::sin(arg);
    }
}

// Which TrainLoraParam vector sits in which slot of the flat layout, by family.
struct Slots {
    std::vector<float>* v[5];
};
Slots slots_of(TrainLoraParam& p, const std::string& type) {
    const std::string f = family(type);
    Slots s{};
    s.v[0] = &p.lora_A;
    s.v[1] = &p.lora_B;
    s.v[2] = f == "dora-rows" ? &p.magnitude : f == "bora" ? &p.magnitude_r : nullptr;
    s.v[3] = f == "dora-cols" ? &p.magnitude : f == "bora" ? &p.magnitude_c : nullptr;
    s.v[4] = &p.M_xs;
    return s;
}
// the same slots of an accumulator / loop-state entry
template <typename V>
std::array<V*, 5> acc_slots(std::vector<V>& A, std::vector<V>& Bv, std::vector<V>& mag, std::vector<V>& mag_r,
                            std::vector<V>& mag_c, std::vector<V>& mxs, size_t i, const std::string& type) {
    const std::string f = family(type);
    return {&A[i], &Bv[i], f == "dora-rows" ? &mag[i] : f == "bora" ? &mag_r[i] : nullptr,
            f == "dora-cols" ? &mag[i] : f == "bora" ? &mag_c[i] : nullptr, &mxs[i]};
}

bool device_alive(const std::shared_ptr<DitDevice>& d, std::string& err) {
    if (!d || !d->dit) return fail(err, "training graph not built (build_train_dit_ckpt)");
    return true;
}

// Host vectors of state into the flat image (size checked against the layout).
bool pack_params(DitDevice& d, TrainLoraState& st, std::string& err) {
    if (st.params.size() != d.targets.size()) return fail(err, "adapter state does not match the training graph");
    d.stage.assign((size_t)d.np, 0.f);
    for (size_t i = 0; i < d.targets.size(); ++i) {
        Slots s = slots_of(st.params[i], d.adapter_type);
        for (int k = 0; k < 5; ++k) {
            const int64_t off = d.layout[i][(size_t)k];
            if (off < 0) continue;
            const int64_t n = k == 0 ? d.rank * d.in[i] : k == 1 ? d.out[i] * d.rank : k == 2 ? d.out[i]
                              : k == 3 ? d.in[i] : (int64_t)d.rank * d.rank;
            if (!s.v[k] || (int64_t)s.v[k]->size() != n)
                return fail(err, "adapter tensor of " + st.params[i].target.stem + " has the wrong size");
            std::memcpy(d.stage.data() + off, s.v[k]->data(), sizeof(float) * (size_t)n);
        }
    }
    return true;
}

int64_t slot_len(const DitDevice& d, size_t i, int k) {
    return k == 0 ? d.rank * d.in[i] : k == 1 ? d.out[i] * d.rank : k == 2 ? d.out[i] : k == 3 ? d.in[i]
                                                                                       : (int64_t)d.rank * d.rank;
}

}  // namespace

// ------------------------------------------------------------------ backend, model files
Backend make_backend(int device) {
    sa3k_ctx* c = nullptr;
    char e[kErrLen] = {0};
    if (sa3k_ctx_create(device, &c, e, kErrLen)) throw gguf_error(std::string("make_backend: ") + e);
    return c;
}

void free_backend(Backend backend) {
    if (backend) sa3k_ctx_destroy(backend);
}

const GgufTensor* GgufModel::get(const std::string& name) const {
    auto it = tensors.find(name);
    if (it == tensors.end()) throw gguf_error("missing tensor: " + name);
    return &it->second;
}

uint32_t GgufModel::u32(const std::string& key) const {
    auto it = u64_kv.find(key);
    if (it == u64_kv.end()) throw gguf_error("missing key: " + key);
    return (uint32_t)it->second;
}

float GgufModel::f32(const std::string& key) const {
    auto it = f64_kv.find(key);
    if (it == f64_kv.end()) throw gguf_error("missing key: " + key);
    return (float)it->second;
}

GgufModel load_gguf(const char* path, Backend backend) {
    sa3k::GgufFile f;
    std::string err;
    if (!path || !f.open(path, err)) throw gguf_error("failed to open " + std::string(path ? path : "(null)") + ": " + err);
    GgufModel m;
    m.backend = backend;
    for (const auto& kv : f.kv) {
        const sa3k::GgufValue& v = kv.second;
        if (v.type == sa3k::kGgufString) m.str_kv[kv.first] = v.s;
        else if (v.type == sa3k::kGgufF32 || v.type == sa3k::kGgufF64) m.f64_kv[kv.first] = v.f;
        else if (v.type != sa3k::kGgufArray) m.u64_kv[kv.first] = v.u;
    }
    for (const std::string& name : f.tensor_order) {
        const auto& t = f.tensors.at(name);
        GgufTensor g;
        g.type = (int)t.type;
        g.n_dims = (int)t.ne.size();
        uint64_t n = 1;
        for (size_t d = 0; d < t.ne.size(); ++d) {
            if (t.ne[d] <= 0) throw gguf_error("bad shape of tensor " + name);
            g.ne[d] = t.ne[d];
            n *= (uint64_t)t.ne[d];
        }
        uint64_t nb = 0;
        if (!type_bytes(g.type, n, nb)) throw gguf_error("unsupported ggml type " + std::to_string(g.type) + " of " + name);
        if (f.data_start + t.offset + nb > f.bytes.size()) throw gguf_error("truncated tensor data of " + name);
        const uint8_t* src = f.bytes.data() + f.data_start + t.offset;
        g.data.assign(src, src + nb);
        m.tensors.emplace(name, std::move(g));
    }
    return m;
}

DitConfig DitConfig::from(const GgufModel& m) {
    DitConfig c;
    auto dk = m.u64_kv.find("dit.differential");
    c.differential = dk == m.u64_kv.end() ? true : dk->second != 0;
    auto lk = m.u64_kv.find("dit.local_dim");
    c.local_dim = lk == m.u64_kv.end() ? 0 : (int)lk->second;
    c.io = (int)m.u32("dit.io");
    c.dim = (int)m.u32("dit.dim");
    c.depth = (int)m.u32("dit.depth");
    c.heads = (int)m.u32("dit.heads");
    c.head_dim = (int)m.u32("dit.head_dim");
    c.cond_dim = (int)m.u32("dit.cond_dim");
    c.mem_tokens = (int)m.u32("dit.mem_tokens");
    c.rot = (int)m.u32("dit.rot");
    c.time_dim = (int)m.u32("dit.time_dim");
    c.rope_base = m.f32("dit.rope_base");
    c.norm_eps = m.f32("dit.norm_eps");
    c.qk_eps = m.f32("dit.qk_eps");
    c.time_min_freq = m.f32("dit.time_min_freq");
    c.time_max_freq = m.f32("dit.time_max_freq");
    if (m.has("dit.0.ff.proj.weight")) c.ff_inner = (int)(m.get("dit.0.ff.proj.weight")->ne[1] / 2);
    return c;
}

// ------------------------------------------------------------------ targets and initialisation
bool train_lora_scope_known(const std::string& s) { return s == "full" || s == "core"; }

static bool is_block_weight(const std::string& name) {
    size_t i = 4;
    if (name.size() <= i || !std::isdigit((unsigned char)name[i])) return false;
    while (i < name.size() && std::isdigit((unsigned char)name[i])) i++;
    return i < name.size() && name[i] == '.';
}

static bool target_selected(const std::string& name, const TrainLoraScope& scope) {
    if (scope.name == "core") {
        if (!is_block_weight(name)) return false;
        if (name.find(".local.") != std::string::npos) return false;
    }
    if (!scope.include.empty() &&
        std::none_of(scope.include.begin(), scope.include.end(),
                     [&](const std::string& p) { return name.find(p) != std::string::npos; }))
        return false;
    return std::none_of(scope.exclude.begin(), scope.exclude.end(),
                        [&](const std::string& p) { return name.find(p) != std::string::npos; });
}

std::vector<TrainLoraTarget> enumerate_train_lora_targets(const GgufModel& dit, const TrainLoraScope& scope) {
    std::vector<TrainLoraTarget> out;
    for (const auto& kv : dit.tensors) {
        const std::string& name = kv.first;
        if (name.rfind("dit.", 0) != 0) continue;
        if (name.size() < 7 || name.compare(name.size() - 7, 7, ".weight") != 0) continue;
        int nd = kv.second.n_dims;
        while (nd > 1 && kv.second.ne[nd - 1] == 1) --nd;   // ggml_n_dims ignores trailing 1s
        if (nd != 2) continue;
        if (!target_selected(name, scope)) continue;
        TrainLoraTarget t;
        t.weight_name = name;
        t.stem = name.substr(0, name.size() - 7);
        t.in = kv.second.ne[0];
        t.out = kv.second.ne[1];
        if (t.in > 0 && t.out > 0) out.push_back(std::move(t));
    }
    std::sort(out.begin(), out.end(),
              [](const TrainLoraTarget& a, const TrainLoraTarget& b) { return a.weight_name < b.weight_name; });
    return out;
}

// first `rank` columns of a stored [rows][stored_rank] f32 basis (src/train_lora.h:192-203)
static bool copy_basis(const GgufTensor* t, int64_t rows, int rank, std::vector<float>& dst) {
    if (!t || t->type != 0 || t->ne[1] != rows || t->ne[0] < rank) return false;
    const int64_t sr = t->ne[0];
    const float* raw = reinterpret_cast<const float*>(t->data.data());
    dst.resize((size_t)(rows * rank));
    for (int64_t r = 0; r < rows; ++r)
        for (int a = 0; a < rank; ++a) dst[(size_t)(r * rank + a)] = raw[r * sr + a];
    return true;
}

// Row or column norms of one base weight on the backend's device (f64 accumulation there).
static bool device_norms(Backend be, const GgufTensor& w, bool rows, std::vector<float>& out, std::string& err) {
    char e[kErrLen] = {0};
    sa3k_weight* dw = nullptr;
    if (sa3k_weight_upload(be, w.type, w.data.data(), w.ne[0], w.ne[1], &dw, e, kErrLen)) return fail(err, e);
    const int64_t n = rows ? w.ne[1] : w.ne[0];
    float* d = nullptr;
    bool ok = cudaMalloc(&d, sizeof(float) * (size_t)n) == cudaSuccess;
    if (!ok) err = "device allocation failed";
    if (ok) ok = ok_or(rows ? sa3k_row_norms(be, dw, 0.f, nullptr, d, e, kErrLen) : sa3k_col_norms(be, dw, d, e, kErrLen),
                       e, err);
    if (ok) ok = ok_or(sa3k_sync(be, e, kErrLen), e, err);
    out.assign((size_t)n, 0.f);
    if (ok && cudaMemcpy(out.data(), d, sizeof(float) * (size_t)n, cudaMemcpyDeviceToHost) != cudaSuccess)
        ok = fail(err, "device copy failed");
    if (d) cudaFree(d);
    sa3k_weight_free(dw);
    return ok;
}

bool init_train_lora_state(const GgufModel& dit, const std::vector<TrainLoraTarget>& targets,
                           const std::string& adapter_type, int rank, float alpha, unsigned long long seed,
                           TrainLoraState& out, std::string& err, const GgufModel* svd_bases) {
    if (rank <= 0) return fail(err, "rank must be positive");
    const std::string f = family(adapter_type);
    if (f != "lora" && f != "dora-rows" && f != "dora-cols" && f != "bora")
        return fail(err, "unknown adapter type " + adapter_type);
    if (rank > 16) return fail(err, "rank must be <= 16 on this device path");
    const bool xs = is_xs(adapter_type);
    const bool need_norms = f != "lora";
    if (need_norms && !dit.backend) return fail(err, "the model has no backend for the magnitude initialisation");
    out = TrainLoraState{};
    out.adapter_type = adapter_type;
    out.rank = rank;
    out.alpha = alpha;
    std::mt19937_64 rng(seed);
    for (const TrainLoraTarget& t : targets) {
        if (rank > t.in || rank > t.out) return fail(err, "rank is infeasible for target " + t.stem);
        if (!dit.has(t.weight_name)) return fail(err, "missing tensor: " + t.weight_name);
        TrainLoraParam p;
        p.target = t;
        const GgufTensor& w = *dit.get(t.weight_name);
        if (xs) {
            const GgufTensor* Ut = svd_bases && svd_bases->has(t.stem + ".U") ? svd_bases->get(t.stem + ".U") : nullptr;
            const GgufTensor* Vt = svd_bases && svd_bases->has(t.stem + ".V") ? svd_bases->get(t.stem + ".V") : nullptr;
            if (!Ut && !Vt)
                return fail(err, "-xs adapters take their frozen bases from svd_bases (" + t.stem +
                                     ".U / .V); the randomized SVD initialisation is not built");
            if (!copy_basis(Ut, t.out, rank, p.U) || !copy_basis(Vt, t.in, rank, p.V))
                return fail(err, "svd bases shape mismatch for target " + t.stem);
            p.M_xs.assign((size_t)rank * rank, 0.0f);
        } else {
            p.lora_A.resize((size_t)(rank * t.in));
            p.lora_B.assign((size_t)(t.out * rank), 0.0f);
            const float bound = 1.0f / std::sqrt((float)t.in);
            std::uniform_real_distribution<float> kaiming(-bound, bound);
            for (float& v : p.lora_A) v = kaiming(rng);
        }
        if (f == "dora-rows") {
            if (!device_norms(dit.backend, w, true, p.magnitude, err)) return false;
        } else if (f == "dora-cols") {
            if (!device_norms(dit.backend, w, false, p.magnitude, err)) return false;
        } else if (f == "bora") {
            if (!device_norms(dit.backend, w, true, p.magnitude_r, err)) return false;
            if (!device_norms(dit.backend, w, false, p.magnitude_c, err)) return false;
        }
        out.params.push_back(std::move(p));
    }
    return true;
}

// ------------------------------------------------------------------ optimizer
float inverse_lr(float base_lr, int step0, float inv_gamma, float power, float warmup, float final_lr) {
    const double n = (double)step0;
    const double wf = warmup > 0.0f ? 1.0 - std::pow((double)warmup, n + 1.0) : 1.0;
    const double mult = std::pow(1.0 + n / (double)inv_gamma, -(double)power);
    return (float)(wf * std::max((double)final_lr, (double)base_lr * mult));
}

void train_clear_accum(TrainLoraGradAccum& accum) {
    accum.count = 0;
    for (auto* v : {&accum.A, &accum.B, &accum.mxs, &accum.mag, &accum.mag_r, &accum.mag_c})
        for (auto& g : *v) std::fill(g.begin(), g.end(), 0.0f);
}

bool train_apply_accumulated_adamw(TrainLoraState& state, TrainLoraGradAccum& accum, TrainLoopState& loop,
                                   const TrainAdamWParams& hp, std::string& err, double* grad_norm_out) {
    if (accum.count <= 0) return fail(err, "cannot apply empty gradient batch");
    if (!device_alive(accum.device, err)) return false;
    DitDevice& d = *accum.device;
    const size_t n = state.params.size();
    if (n != d.targets.size()) return fail(err, "adapter state does not match the training graph");
    loop.step += 1;
    for (auto* v : {&loop.A_state, &loop.B_state, &loop.mxs_state, &loop.mag_state, &loop.mag_r_state,
                    &loop.mag_c_state})
        v->resize(n);
    for (auto* v : {&accum.A, &accum.B, &accum.mxs, &accum.mag, &accum.mag_r, &accum.mag_c}) v->resize(n);
    char e[kErrLen] = {0};
    // parameters, then gradients, then the two moments, each through the flat host image
    if (!pack_params(d, state, err)) return false;
    if (!ok_or(sa3k_dit_adapter_copy(d.dit, 0, d.stage.data(), 0, d.np, 1, e, kErrLen), e, err)) return false;
    for (int which = 1; which <= 3; ++which) {
        d.stage.assign((size_t)d.np, 0.f);
        for (size_t i = 0; i < n; ++i) {
            std::array<std::vector<float>*, 5> sl{};
            if (which == 1) {
                sl = acc_slots(accum.A, accum.B, accum.mag, accum.mag_r, accum.mag_c, accum.mxs, i, d.adapter_type);
            } else {
                auto st = acc_slots(loop.A_state, loop.B_state, loop.mag_state, loop.mag_r_state, loop.mag_c_state,
                                    loop.mxs_state, i, d.adapter_type);
                for (int k = 0; k < 5; ++k) sl[(size_t)k] = st[(size_t)k] ? (which == 2 ? &st[(size_t)k]->m : &st[(size_t)k]->v) : nullptr;
            }
            for (int k = 0; k < 5; ++k) {
                const int64_t off = d.layout[i][(size_t)k];
                if (off < 0 || !sl[(size_t)k]) continue;
                const int64_t len = slot_len(d, i, k);
                std::vector<float>& v = *sl[(size_t)k];
                if ((int64_t)v.size() != len) {
                    if (which == 1 && !v.empty()) return fail(err, "accumulated gradient has the wrong size");
                    v.assign((size_t)len, 0.f);   // fresh moments (adamw_update_vector's first step)
                }
                std::memcpy(d.stage.data() + off, v.data(), sizeof(float) * (size_t)len);
            }
        }
        if (!ok_or(sa3k_dit_adapter_copy(d.dit, which, d.stage.data(), 0, d.np, 1, e, kErrLen), e, err)) return false;
    }
    sa3k_adamw_params p = {hp.learning_rate, hp.beta1, hp.beta2, hp.eps, hp.weight_decay, hp.grad_clip};
    double norm = 0.0;
    if (!ok_or(sa3k_dit_apply_adamw(d.dit, accum.count, &p, loop.step, &norm, e, kErrLen), e, err)) return false;
    if (grad_norm_out) *grad_norm_out = norm;
    // parameters and moments back into the host state
    for (int which : {0, 2, 3}) {
        d.stage.assign((size_t)d.np, 0.f);
        if (!ok_or(sa3k_dit_adapter_copy(d.dit, which, d.stage.data(), 0, d.np, 0, e, kErrLen), e, err)) return false;
        for (size_t i = 0; i < n; ++i) {
            std::array<std::vector<float>*, 5> sl{};
            if (which == 0) {
                Slots s = slots_of(state.params[i], d.adapter_type);
                for (int k = 0; k < 5; ++k) sl[(size_t)k] = s.v[k];
            } else {
                auto st = acc_slots(loop.A_state, loop.B_state, loop.mag_state, loop.mag_r_state, loop.mag_c_state,
                                    loop.mxs_state, i, d.adapter_type);
                for (int k = 0; k < 5; ++k) sl[(size_t)k] = st[(size_t)k] ? (which == 2 ? &st[(size_t)k]->m : &st[(size_t)k]->v) : nullptr;
            }
            for (int k = 0; k < 5; ++k) {
                const int64_t off = d.layout[i][(size_t)k];
                if (off < 0 || !sl[(size_t)k]) continue;
                const int64_t len = slot_len(d, i, k);
                sl[(size_t)k]->assign(d.stage.data() + off, d.stage.data() + off + len);
            }
        }
    }
    train_clear_accum(accum);
    return true;
}

// ------------------------------------------------------------------ diffusion sampler
// Acklam's rational approximation of the inverse normal CDF (published coefficients, about 1e-9
// relative accuracy), the same function the reference's truncated logit-normal draw uses.
static double norm_icdf(double p) {
    if (p <= 0.0) return -1e9;
    if (p >= 1.0) return 1e9;
    static const double a[6] = {-3.969683028665376e+01, 2.209460984245205e+02, -2.759285104469687e+02,
                                1.383577518672690e+02,  -3.066479806614716e+01, 2.506628277459239e+00};
    static const double b[5] = {-5.447609879822406e+01, 1.615858368580409e+02, -1.556989798598866e+02,
                                6.680131188771972e+01,  -1.328068155288572e+01};
    static const double c[6] = {-7.784894002430293e-03, -3.223964580411365e-01, -2.400758277161838e+00,
                                -2.549732539343734e+00, 4.374664141464968e+00,  2.938163982698783e+00};
    static const double d[4] = {7.784695709041462e-03, 3.224671290700398e-01, 2.445134137142996e+00,
                                3.754408661907416e+00};
    const double plow = 0.02425;
    auto tail = [&](double q) {
        return (((((c[0] * q + c[1]) * q + c[2]) * q + c[3]) * q + c[4]) * q + c[5]) /
               ((((d[0] * q + d[1]) * q + d[2]) * q + d[3]) * q + 1.0);
    };
    if (p < plow) return tail(std::sqrt(-2.0 * std::log(p)));
    if (p > 1.0 - plow) return -tail(std::sqrt(-2.0 * std::log(1.0 - p)));
    const double q = p - 0.5, r = q * q;
    return (((((a[0] * r + a[1]) * r + a[2]) * r + a[3]) * r + a[4]) * r + a[5]) * q /
           (((((b[0] * r + b[1]) * r + b[2]) * r + b[3]) * r + b[4]) * r + 1.0);
}

static double norm_cdf(double x) { return 0.5 * std::erfc(-x * 0.7071067811865476); }

TrainDiffusionSampler::TrainDiffusionSampler(unsigned long long seed, const std::string& mode) : rng_(seed), mode_(mode) {}

bool TrainDiffusionSampler::sample(const std::vector<float>& z, TrainDiffusionSample& out, std::string& err) {
    return sample_at(z, draw_t(), out, err);
}

bool TrainDiffusionSampler::sample_at(const std::vector<float>& z, float t, TrainDiffusionSample& out,
                                      std::string& err) {
    if (z.empty()) return fail(err, "latent vector is empty");
    out.t = t;
    out.noise.resize(z.size());
    out.x_t.resize(z.size());
    out.velocity_target.resize(z.size());
    for (size_t i = 0; i < z.size(); ++i) {
        const float n = normal_(rng_);
        out.noise[i] = n;
        out.x_t[i] = (1.0f - t) * z[i] + t * n;
        out.velocity_target[i] = n - z[i];
    }
    return true;
}

float TrainDiffusionSampler::draw_t() {
    if (mode_ == "trunc_logit_normal") {
        // the logistic-normal truncated at left = 0.075, rescaled to [0, 1] and flipped
        const double left = 0.075;
        const double lb = norm_cdf(std::log(left / (1.0 - left)));
        const double u = norm_cdf((double)normal_(rng_));
        double tc = lb + (1.0 - lb) * u;
        tc = std::min(std::max(tc, 1e-7), 1.0 - 1e-7);
        const double ts = 1.0 / (1.0 + std::exp(-norm_icdf(tc)));
        return (float)(1.0 - (ts - left) / (1.0 - left));
    }
    return uniform_(rng_);
}

std::string TrainDiffusionSampler::serialize_state() const {
    std::ostringstream s;
    s << rng_ << '\n' << uniform_ << '\n' << normal_;
    return s.str();
}

bool TrainDiffusionSampler::restore_state(const std::string& state, std::string& err) {
    std::istringstream s(state);
    std::mt19937_64 rng;
    std::uniform_real_distribution<float> uniform;
    std::normal_distribution<float> normal;
    if (!(s >> rng >> uniform >> normal)) return fail(err, "invalid diffusion sampler state");
    rng_ = rng;
    uniform_ = uniform;
    normal_ = normal;
    return true;
}

// ------------------------------------------------------------------ the step
bool build_train_dit_ckpt(GgufModel& dit, const DitConfig& dc, const TrainLoraState& lora, int frames, int cond_dim,
                          int ctx_len, TrainDitCkpt& out, std::string& err, bool inpaint) {
    if (frames <= 0 || cond_dim <= 0 || ctx_len <= 0) return fail(err, "invalid DiT training graph dimensions");
    if (inpaint && dc.local_dim <= 0)
        return fail(err, "inpainting requested but DiT has no local-cond weights (dit.local_dim <= 0)");
    if (!dit.backend) return fail(err, "the model has no backend (load_gguf(path, backend))");
    if (cond_dim != dc.cond_dim) return fail(err, "cond_dim does not match the model");
    std::vector<std::string> names;
    for (const TrainLoraParam& p : lora.params) names.push_back(p.target.weight_name);
    std::shared_ptr<DitDevice> dev = dit.device;
    const bool same = dev && dev->ctx == dit.backend && dev->adapter_type == lora.adapter_type && dev->rank == lora.rank &&
                      dev->alpha == lora.alpha && dev->targets == names;
    char e[kErrLen] = {0};
    if (!same) {
        dev = std::make_shared<DitDevice>();
        dev->ctx = dit.backend;
        dev->dc = dc;
        sa3k_dit_config k = {};
        k.io = dc.io; k.dim = dc.dim; k.depth = dc.depth; k.heads = dc.heads; k.head_dim = dc.head_dim;
        k.cond_dim = dc.cond_dim; k.mem_tokens = dc.mem_tokens; k.rot = dc.rot; k.time_dim = dc.time_dim;
        k.ff_inner = dc.ff_inner; k.differential = dc.differential ? 1 : 0; k.rope_base = dc.rope_base;
        k.norm_eps = dc.norm_eps; k.qk_eps = dc.qk_eps; k.time_min_freq = dc.time_min_freq;
        k.time_max_freq = dc.time_max_freq; k.local_dim = dc.local_dim;
        if (k.ff_inner <= 0) return fail(err, "DitConfig.ff_inner is unset (DitConfig::from reads it)");
        if (sa3k_dit_create(dit.backend, &k, &dev->dit, e, kErrLen)) return fail(err, e);
        for (const auto& kv : dit.tensors) {
            if (kv.first.rfind("dit.", 0) != 0) continue;
            const GgufTensor& t = kv.second;
            if (sa3k_dit_set_tensor(dev->dit, kv.first.c_str(), t.type, t.data.data(), t.ne[0], t.ne[1], e, kErrLen)) {
                if (std::strstr(e, "not a tensor")) continue;   // a dit.* tensor the training step does not read
                return fail(err, e);
            }
        }
        std::vector<const char*> cn;
        for (const std::string& s : names) cn.push_back(s.c_str());
        if (!cn.empty() && sa3k_dit_init_adapters(dev->dit, lora.adapter_type.c_str(), lora.rank, lora.alpha, cn.data(),
                                                  (int)cn.size(), e, kErrLen))
            return fail(err, e);
        dev->adapter_type = lora.adapter_type;
        dev->rank = lora.rank;
        dev->alpha = lora.alpha;
        dev->targets = names;
        dev->np = sa3k_dit_adapter_size(dev->dit);
        for (size_t i = 0; i < names.size(); ++i) {
            std::array<int64_t, 5> offs{};
            sa3k_dit_adapter_layout(dev->dit, (int)i, offs.data());
            dev->layout.push_back(offs);
            dev->in.push_back(lora.params[i].target.in);
            dev->out.push_back(lora.params[i].target.out);
            if (is_xs(lora.adapter_type) &&
                sa3k_dit_set_xs_bases(dev->dit, names[i].c_str(), lora.params[i].U.data(), lora.params[i].V.data(), e,
                                      kErrLen))
                return fail(err, e);
        }
        dit.device = dev;
    }
    out.device = dev;
    out.pctx = dev.get();
    out.inpaint = inpaint;
    out.frames = frames;
    out.cond_dim = cond_dim;
    out.ctx_len = ctx_len;
    return true;
}

void free_train_dit_ckpt(TrainDitCkpt& ck) {
    ck.device.reset();
    ck.pctx = nullptr;
    ck.frames = ck.cond_dim = ck.ctx_len = 0;
}

bool run_train_dit_accumulate_ckpt(Backend backend, TrainDitCkpt& ck, const TrainLoraState& lora,
                                   TrainLoraGradAccum& accum, const TrainDiffusionSample& sample,
                                   const TrainConditioning& cond, const DitConfig& dc, float& loss_out,
                                   std::string& err, const TrainInpaint* inpaint) {
    if (sample.x_t.empty() || sample.velocity_target.empty() || cond.cross.empty() || cond.global.empty())
        return fail(err, "training step inputs are empty");
    if (!device_alive(ck.device, err)) return false;
    if (ck.inpaint != (inpaint != nullptr))
        return fail(err, "inpaint graph/sample mismatch (local-cond present in one but not the other)");
    DitDevice& d = *ck.device;
    if (backend && backend != d.ctx) return fail(err, "backend differs from the one the graph was built on");
    const int64_t T = (int64_t)sample.x_t.size() / dc.io;
    if (T * dc.io != (int64_t)sample.x_t.size() || sample.velocity_target.size() != sample.x_t.size() || T != ck.frames)
        return fail(err, "latent size does not match the training graph");
    if ((int64_t)cond.cross.size() < (int64_t)ck.ctx_len * ck.cond_dim || (int)cond.global.size() != ck.cond_dim)
        return fail(err, "conditioning size does not match the training graph");
    char e[kErrLen] = {0};
    // adapters (one upload per call, as the reference's persistent tensors)
    TrainLoraState& st = const_cast<TrainLoraState&>(lora);   // read only: pack_params copies out
    if (!pack_params(d, st, err)) return false;
    if (!ok_or(sa3k_dit_adapter_copy(d.dit, 0, d.stage.data(), 0, d.np, 1, e, kErrLen), e, err)) return false;
    if (!ok_or(sa3k_dit_zero_grads(d.dit, e, kErrLen), e, err)) return false;
    std::vector<float> tf;
    expo_features(sample.t, tf, dc.time_dim, dc.time_min_freq, dc.time_max_freq);
    float loss = 0.f;
    if (inpaint) {
        if ((int64_t)inpaint->local.size() != T * dc.local_dim || (int64_t)inpaint->loss_weight.size() != T * dc.io)
            return fail(err, "inpaint input size does not match the training graph");
        if (!ok_or(sa3k_dit_forward_backward_inpaint(d.dit, 1, (int)T, ck.ctx_len, sample.x_t.data(),
                                                     sample.velocity_target.data(), tf.data(), cond.cross.data(),
                                                     cond.global.data(), inpaint->local.data(),
                                                     inpaint->loss_weight.data(), &loss, e, kErrLen),
                   e, err))
            return false;
    } else if (!ok_or(sa3k_dit_forward_backward(d.dit, 1, (int)T, ck.ctx_len, sample.x_t.data(),
                                                sample.velocity_target.data(), tf.data(), cond.cross.data(),
                                                cond.global.data(), &loss, e, kErrLen),
                      e, err)) {
        return false;
    }
    if (!ok_or(sa3k_sync(d.ctx, e, kErrLen), e, err)) return false;
    // this sample's gradients into the host accumulator
    d.stage.assign((size_t)d.np, 0.f);
    if (!ok_or(sa3k_dit_adapter_copy(d.dit, 1, d.stage.data(), 0, d.np, 0, e, kErrLen), e, err)) return false;
    const size_t n = d.targets.size();
    for (auto* v : {&accum.A, &accum.B, &accum.mxs, &accum.mag, &accum.mag_r, &accum.mag_c}) v->resize(n);
    for (size_t i = 0; i < n; ++i) {
        auto sl = acc_slots(accum.A, accum.B, accum.mag, accum.mag_r, accum.mag_c, accum.mxs, i, d.adapter_type);
        for (int k = 0; k < 5; ++k) {
            const int64_t off = d.layout[i][(size_t)k];
            if (off < 0 || !sl[(size_t)k]) continue;
            const int64_t len = slot_len(d, i, k);
            std::vector<float>& g = *sl[(size_t)k];
            if (g.empty()) g.assign((size_t)len, 0.f);
            if ((int64_t)g.size() != len) return fail(err, "gradient accumulator has the wrong size");
            for (int64_t j = 0; j < len; ++j) g[(size_t)j] += d.stage[(size_t)(off + j)];
        }
    }
    accum.count += 1;
    accum.device = ck.device;
    loss_out = loss;
    return true;
}

}  // namespace sa3
