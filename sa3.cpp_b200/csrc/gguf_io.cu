// gguf_io.cu -- GGUF version 3 reading and writing (host code only).
#include "gguf_io.h"

#include <cstdio>
#include <cstring>
#include <fstream>

namespace sa3k {

namespace {

constexpr uint32_t kMagic = 0x46554747u;   // "GGUF" read as a little-endian u32
constexpr uint32_t kVersion = 3;
constexpr uint32_t kTypeF32 = 0;           // ggml type id of f32 tensors

struct Out {
  std::vector<uint8_t> b;
  template <typename T>
  void put(T v) {
    const size_t n = b.size();
    b.resize(n + sizeof(T));
    std::memcpy(b.data() + n, &v, sizeof(T));
  }
  void str(const std::string& s) {
    put<uint64_t>(s.size());
    b.insert(b.end(), s.begin(), s.end());
  }
  void pad(size_t align) {
    while (b.size() % align) b.push_back(0);
  }
};

struct In {
  const std::vector<uint8_t>& b;
  size_t p = 0;
  bool ok = true;
  template <typename T>
  T get() {
    T v{};
    if (!ok || p + sizeof(T) > b.size()) {
      ok = false;
      return v;
    }
    std::memcpy(&v, b.data() + p, sizeof(T));
    p += sizeof(T);
    return v;
  }
  std::string str() {
    const uint64_t n = get<uint64_t>();
    if (!ok || n > b.size() - p) {
      ok = false;
      return {};
    }
    std::string s(reinterpret_cast<const char*>(b.data() + p), (size_t)n);
    p += (size_t)n;
    return s;
  }
};

size_t scalar_size(uint32_t t) {
  switch (t) {
    case kGgufU8: case kGgufI8: case kGgufBool: return 1;
    case kGgufU16: case kGgufI16: return 2;
    case kGgufU32: case kGgufI32: case kGgufF32: return 4;
    case kGgufU64: case kGgufI64: case kGgufF64: return 8;
    default: return 0;
  }
}

// one scalar of type t, integers widened into u (sign-extended), floats into f
bool read_scalar(In& in, uint32_t t, uint64_t& u, double& f) {
  switch (t) {
    case kGgufU8: u = in.get<uint8_t>(); break;
    case kGgufI8: u = (uint64_t)(int64_t)in.get<int8_t>(); break;
    case kGgufBool: u = in.get<uint8_t>() != 0; break;
    case kGgufU16: u = in.get<uint16_t>(); break;
    case kGgufI16: u = (uint64_t)(int64_t)in.get<int16_t>(); break;
    case kGgufU32: u = in.get<uint32_t>(); break;
    case kGgufI32: u = (uint64_t)(int64_t)in.get<int32_t>(); break;
    case kGgufU64: u = in.get<uint64_t>(); break;
    case kGgufI64: u = (uint64_t)in.get<int64_t>(); break;
    case kGgufF32: f = in.get<float>(); break;
    case kGgufF64: f = in.get<double>(); break;
    default: return false;
  }
  return in.ok;
}

void write_value(Out& o, const GgufValue& v) {
  o.put<uint32_t>(v.type);
  switch (v.type) {
    case kGgufString: o.str(v.s); break;
    case kGgufU32: o.put<uint32_t>((uint32_t)v.u); break;
    case kGgufU64: o.put<uint64_t>(v.u); break;
    case kGgufF32: o.put<float>((float)v.f); break;
    case kGgufArray:
      o.put<uint32_t>(v.arr_type);
      if (v.arr_type == kGgufString) {
        o.put<uint64_t>(v.arr_s.size());
        for (const std::string& s : v.arr_s) o.str(s);
      } else {   // u64 arrays are the only other kind written here
        o.put<uint64_t>(v.arr_u.size());
        for (uint64_t x : v.arr_u) o.put<uint64_t>(x);
      }
      break;
    default: break;
  }
}

}  // namespace

void GgufWriter::set_str(const std::string& k, const std::string& v) {
  GgufValue x;
  x.type = kGgufString;
  x.s = v;
  kv.emplace_back(k, x);
}
void GgufWriter::set_u32(const std::string& k, uint32_t v) {
  GgufValue x;
  x.type = kGgufU32;
  x.u = v;
  kv.emplace_back(k, x);
}
void GgufWriter::set_u64(const std::string& k, uint64_t v) {
  GgufValue x;
  x.type = kGgufU64;
  x.u = v;
  kv.emplace_back(k, x);
}
void GgufWriter::set_f32(const std::string& k, float v) {
  GgufValue x;
  x.type = kGgufF32;
  x.f = v;
  kv.emplace_back(k, x);
}
void GgufWriter::set_arr_u64(const std::string& k, const std::vector<uint64_t>& v) {
  GgufValue x;
  x.type = kGgufArray;
  x.arr_type = kGgufU64;
  x.arr_u = v;
  kv.emplace_back(k, x);
}
void GgufWriter::set_arr_str(const std::string& k, const std::vector<std::string>& v) {
  GgufValue x;
  x.type = kGgufArray;
  x.arr_type = kGgufString;
  x.arr_s = v;
  kv.emplace_back(k, x);
}
void GgufWriter::add_f32(const std::string& name, std::vector<int64_t> ne, const float* data) {
  tensors.push_back(Tensor{name, std::move(ne), data});
}

bool GgufWriter::write(const std::string& path, std::string& err) const {
  constexpr size_t kAlign = 32;
  Out o;
  o.put<uint32_t>(kMagic);
  o.put<uint32_t>(kVersion);
  o.put<uint64_t>(tensors.size());
  o.put<uint64_t>(kv.size());
  for (const auto& e : kv) {
    o.str(e.first);
    write_value(o, e.second);
  }
  uint64_t off = 0;
  std::vector<uint64_t> bytes(tensors.size());
  for (size_t i = 0; i < tensors.size(); ++i) {
    const Tensor& t = tensors[i];
    if (t.ne.empty() || t.ne.size() > 4) {
      err = "gguf: tensor " + t.name + " needs 1 to 4 dims";
      return false;
    }
    uint64_t n = 1;
    for (int64_t d : t.ne) {
      if (d <= 0) {
        err = "gguf: tensor " + t.name + " has an empty dim";
        return false;
      }
      n *= (uint64_t)d;
    }
    bytes[i] = n * sizeof(float);
    o.str(t.name);
    o.put<uint32_t>((uint32_t)t.ne.size());
    for (int64_t d : t.ne) o.put<uint64_t>((uint64_t)d);
    o.put<uint32_t>(kTypeF32);
    o.put<uint64_t>(off);
    off += (bytes[i] + kAlign - 1) / kAlign * kAlign;
  }
  o.pad(kAlign);
  for (size_t i = 0; i < tensors.size(); ++i) {
    const uint8_t* p = reinterpret_cast<const uint8_t*>(tensors[i].data);
    o.b.insert(o.b.end(), p, p + bytes[i]);
    o.pad(kAlign);
  }
  std::FILE* f = std::fopen(path.c_str(), "wb");
  if (!f) {
    err = "gguf: cannot open " + path + " for writing";
    return false;
  }
  const bool ok = std::fwrite(o.b.data(), 1, o.b.size(), f) == o.b.size();
  const bool closed = std::fclose(f) == 0;
  if (!ok || !closed) {
    err = "gguf: failed to write " + path;
    return false;
  }
  return true;
}

bool GgufFile::open(const std::string& path, std::string& err) {
  std::ifstream f(path, std::ios::binary);
  if (!f) {
    err = "gguf: cannot open " + path;
    return false;
  }
  bytes.assign(std::istreambuf_iterator<char>(f), std::istreambuf_iterator<char>());
  In in{bytes};
  if (in.get<uint32_t>() != kMagic || !in.ok) {
    err = "gguf: " + path + " is not a GGUF file";
    return false;
  }
  const uint32_t version = in.get<uint32_t>();
  if (version != 2 && version != 3) {
    err = "gguf: unsupported version " + std::to_string(version);
    return false;
  }
  const uint64_t nt = in.get<uint64_t>(), nkv = in.get<uint64_t>();
  if (!in.ok || nt > bytes.size() || nkv > bytes.size()) {
    err = "gguf: corrupt header";
    return false;
  }
  kv.clear();
  tensors.clear();
  tensor_order.clear();
  for (uint64_t i = 0; i < nkv && in.ok; ++i) {
    const std::string key = in.str();
    GgufValue v;
    v.type = in.get<uint32_t>();
    if (v.type == kGgufString) {
      v.s = in.str();
    } else if (v.type == kGgufArray) {
      v.arr_type = in.get<uint32_t>();
      const uint64_t n = in.get<uint64_t>();
      if (!in.ok || n > bytes.size()) {
        err = "gguf: corrupt array " + key;
        return false;
      }
      for (uint64_t k = 0; k < n && in.ok; ++k) {
        if (v.arr_type == kGgufString) {
          v.arr_s.push_back(in.str());
        } else {
          uint64_t u = 0;
          double fl = 0.0;
          if (scalar_size(v.arr_type) == 0 || !read_scalar(in, v.arr_type, u, fl)) {
            err = "gguf: unsupported array element type in " + key;
            return false;
          }
          v.arr_u.push_back(u);
          v.arr_f.push_back(fl);
        }
      }
    } else if (!read_scalar(in, v.type, v.u, v.f)) {
      err = "gguf: unsupported value type in " + key;
      return false;
    }
    kv[key] = v;
  }
  size_t align = 32;
  if (const GgufValue* a = find("general.alignment")) {
    if (a->u == 0 || (a->u & (a->u - 1)) || a->u > 4096) {
      err = "gguf: bad general.alignment";
      return false;
    }
    align = (size_t)a->u;
  }
  for (uint64_t i = 0; i < nt && in.ok; ++i) {
    const std::string name = in.str();
    Tensor t;
    const uint32_t nd = in.get<uint32_t>();
    if (!in.ok || nd == 0 || nd > 4) {
      err = "gguf: bad dims for tensor " + name;
      return false;
    }
    for (uint32_t d = 0; d < nd; ++d) t.ne.push_back((int64_t)in.get<uint64_t>());
    t.type = in.get<uint32_t>();
    t.offset = in.get<uint64_t>();
    if (tensors.count(name)) {
      err = "gguf: duplicate tensor " + name;
      return false;
    }
    tensors[name] = t;
    tensor_order.push_back(name);
  }
  if (!in.ok) {
    err = "gguf: truncated metadata in " + path;
    return false;
  }
  data_start = (in.p + align - 1) / align * align;
  if (data_start > bytes.size()) {
    err = "gguf: truncated file " + path;
    return false;
  }
  return true;
}

const GgufValue* GgufFile::find(const std::string& k) const {
  auto it = kv.find(k);
  return it == kv.end() ? nullptr : &it->second;
}

bool GgufFile::read_f32(const std::string& name, std::vector<float>& out, std::string& err) const {
  auto it = tensors.find(name);
  if (it == tensors.end()) {
    err = "gguf: no tensor " + name;
    return false;
  }
  const Tensor& t = it->second;
  if (t.type != kTypeF32) {
    err = "gguf: tensor " + name + " is not f32";
    return false;
  }
  uint64_t n = 1;
  for (int64_t d : t.ne) {
    if (d <= 0 || (uint64_t)d > bytes.size()) {
      err = "gguf: bad shape of " + name;
      return false;
    }
    n *= (uint64_t)d;
  }
  const uint64_t nb = n * sizeof(float);
  if (n > bytes.size() || t.offset > bytes.size() || data_start + t.offset + nb > bytes.size()) {
    err = "gguf: tensor " + name + " runs past the end of the file";
    return false;
  }
  out.resize((size_t)n);
  std::memcpy(out.data(), bytes.data() + data_start + t.offset, (size_t)nb);
  return true;
}

bool write_adapter_gguf(const std::string& path, const std::string& adapter_type, int rank, float alpha,
                        const std::vector<AdapterTargetView>& targets, std::string& err) {
  if (rank <= 0 || targets.empty()) {
    err = "cannot write an empty adapter file";
    return false;
  }
  GgufWriter w;
  w.set_str("general.architecture", "sa3-lora");
  w.set_str("general.name", "sa3 native trained adapter");
  w.set_str("lora.adapter_type", adapter_type);
  w.set_u32("lora.rank", (uint32_t)rank);
  w.set_f32("lora.alpha", alpha);
  w.set_u32("lora.n_targets", (uint32_t)targets.size());
  for (const AdapterTargetView& t : targets) {
    if (t.A) w.add_f32(t.stem + ".lora_A", {t.in, rank}, t.A);
    if (t.B) w.add_f32(t.stem + ".lora_B", {rank, t.out}, t.B);
    if (t.U) w.add_f32(t.stem + ".U", {rank, t.out}, t.U);
    if (t.V) w.add_f32(t.stem + ".V", {rank, t.in}, t.V);
    if (t.M) w.add_f32(t.stem + ".M_xs", {rank, rank}, t.M);
    if (t.m) w.add_f32(t.stem + ".magnitude", {t.m_len > 0 ? t.m_len : t.out}, t.m);
    if (t.m_r) w.add_f32(t.stem + ".magnitude_r", {t.out}, t.m_r);
    if (t.m_c) w.add_f32(t.stem + ".magnitude_c", {t.in}, t.m_c);
  }
  const std::string tmp = path + ".tmp";
  std::remove(tmp.c_str());
  if (!w.write(tmp, err)) return false;
  if (std::rename(tmp.c_str(), path.c_str()) != 0) {
    std::remove(tmp.c_str());
    err = "failed to publish adapter file " + path;
    return false;
  }
  return true;
}

std::string gguf_file_fingerprint(const std::string& path, std::string& err) {
  std::ifstream f(path, std::ios::binary);
  if (!f) {
    err = "cannot fingerprint checkpoint file: " + path;
    return {};
  }
  uint64_t h = 14695981039346656037ull;   // FNV-1a 64-bit offset basis and prime
  std::vector<char> buf(1u << 20);
  while (f) {
    f.read(buf.data(), (std::streamsize)buf.size());
    const std::streamsize got = f.gcount();
    for (std::streamsize i = 0; i < got; ++i) {
      h ^= (unsigned char)buf[(size_t)i];
      h *= 1099511628211ull;
    }
  }
  char s[40];
  std::snprintf(s, sizeof s, "fnv1a64:%016llx", (unsigned long long)h);
  return s;
}

}  // namespace sa3k
