// checkpoint.cu -- C-ABI entry points for the adapter and trainer-state files that need no
// device: writing an adapter file from host arrays and reading GGUF metadata / f32 tensors (the
// dataset loop of a trainer restores its cursor and random states from these).  Host code only.
#include "../../include/sa3k.h"
#include "gguf_io.h"

#include <algorithm>
#include <cstring>
#include <string>
#include <vector>

using namespace sa3k;

static int cfail(char* err, int len, const std::string& msg) {
  if (err && len > 0) {
    std::strncpy(err, msg.c_str(), (size_t)len - 1);
    err[len - 1] = 0;
  }
  return 1;
}

extern "C" {

int sa3k_adapter_gguf_write(const char* path, const char* adapter_type, int rank, float alpha, int n,
                            const char* const* stems, const int64_t* in, const int64_t* out, const float* const* A,
                            const float* const* B, const float* const* m, char* err, int err_len) {
  if (!path || !adapter_type || !stems || !in || !out || !A || !B || n <= 0 || rank <= 0)
    return cfail(err, err_len, "NULL argument or empty adapter");
  std::vector<AdapterTargetView> t((size_t)n);
  for (int i = 0; i < n; ++i) {
    if (!stems[i] || !A[i] || !B[i] || in[i] <= 0 || out[i] <= 0) return cfail(err, err_len, "bad adapter target");
    t[(size_t)i].stem = stems[i];
    t[(size_t)i].in = in[i];
    t[(size_t)i].out = out[i];
    t[(size_t)i].A = A[i];
    t[(size_t)i].B = B[i];
    t[(size_t)i].m = m ? m[i] : nullptr;
  }
  std::string e;
  if (!write_adapter_gguf(path, adapter_type, rank, alpha, t, e)) return cfail(err, err_len, e);
  return 0;
}

int sa3k_gguf_get_string(const char* path, const char* key, char* buf, int64_t buf_len, int64_t* len_out, char* err,
                         int err_len) {
  if (!path || !key) return cfail(err, err_len, "NULL argument");
  GgufFile f;
  std::string e;
  if (!f.open(path, e)) return cfail(err, err_len, e);
  const GgufValue* v = f.find(key);
  if (!v || v->type != kGgufString) return cfail(err, err_len, std::string("no string metadata ") + key);
  if (len_out) *len_out = (int64_t)v->s.size();
  if (buf && buf_len > 0) {
    const size_t n = std::min<size_t>((size_t)(buf_len - 1), v->s.size());
    std::memcpy(buf, v->s.data(), n);
    buf[n] = 0;
  }
  return 0;
}

int sa3k_gguf_get_u64(const char* path, const char* key, uint64_t* value, char* err, int err_len) {
  if (!path || !key || !value) return cfail(err, err_len, "NULL argument");
  GgufFile f;
  std::string e;
  if (!f.open(path, e)) return cfail(err, err_len, e);
  const GgufValue* v = f.find(key);
  if (!v || (v->type != kGgufU64 && v->type != kGgufU32 && v->type != kGgufU16 && v->type != kGgufU8))
    return cfail(err, err_len, std::string("no unsigned integer metadata ") + key);
  *value = v->u;
  return 0;
}

int sa3k_gguf_get_u64_array(const char* path, const char* key, uint64_t* out, int64_t max, int64_t* n_out, char* err,
                            int err_len) {
  if (!path || !key || !n_out) return cfail(err, err_len, "NULL argument");
  GgufFile f;
  std::string e;
  if (!f.open(path, e)) return cfail(err, err_len, e);
  const GgufValue* v = f.find(key);
  if (!v || v->type != kGgufArray || (v->arr_type != kGgufU64 && v->arr_type != kGgufU32))
    return cfail(err, err_len, std::string("no unsigned integer array metadata ") + key);
  *n_out = (int64_t)v->arr_u.size();
  for (int64_t i = 0; out && i < max && i < *n_out; ++i) out[i] = v->arr_u[(size_t)i];
  return 0;
}

int sa3k_gguf_get_f32(const char* path, const char* name, float* out, int64_t max, int64_t* n_out, int64_t* ne,
                      int* n_dims, char* err, int err_len) {
  if (!path || !name || !n_out) return cfail(err, err_len, "NULL argument");
  GgufFile f;
  std::string e;
  if (!f.open(path, e)) return cfail(err, err_len, e);
  std::vector<float> v;
  if (!f.read_f32(name, v, e)) return cfail(err, err_len, e);
  const GgufFile::Tensor& t = f.tensors.at(name);
  if (n_dims) *n_dims = (int)t.ne.size();
  for (size_t d = 0; ne && d < 4; ++d) ne[d] = d < t.ne.size() ? t.ne[d] : 1;
  *n_out = (int64_t)v.size();
  if (out) std::memcpy(out, v.data(), sizeof(float) * (size_t)std::min<int64_t>(max, *n_out));
  return 0;
}

}  // extern "C"
