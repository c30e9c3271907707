// gguf_io.h -- a small GGUF (version 3) reader and writer for the adapter and trainer-state files
// of the training path (host code).  The layout follows the published GGUF format: a header
// (magic "GGUF", version, tensor count, metadata count), typed key / value metadata, tensor
// infos (name, dims with ne[0] innermost, ggml type, data offset), then the tensor data, every
// tensor aligned to `general.alignment` (32 when absent).  Only F32 tensors are written or read:
// that is all adapter and optimizer tensors are (src/train_checkpoint.h:31-40).
#pragma once

#include <cstdint>
#include <map>
#include <string>
#include <vector>

namespace sa3k {

enum GgufValueType : uint32_t {
  kGgufU8 = 0, kGgufI8 = 1, kGgufU16 = 2, kGgufI16 = 3, kGgufU32 = 4, kGgufI32 = 5, kGgufF32 = 6,
  kGgufBool = 7, kGgufString = 8, kGgufArray = 9, kGgufU64 = 10, kGgufI64 = 11, kGgufF64 = 12
};

// One metadata value.  Scalars keep their bits in u (integers, bool) or f (floats); arrays keep
// their element type in arr_type and their elements in arr_u (integer types widened), arr_f or
// arr_s.
struct GgufValue {
  uint32_t type = kGgufU32;
  uint32_t arr_type = 0;
  uint64_t u = 0;
  double f = 0.0;
  std::string s;
  std::vector<uint64_t> arr_u;
  std::vector<double> arr_f;
  std::vector<std::string> arr_s;
};

struct GgufWriter {
  std::vector<std::pair<std::string, GgufValue>> kv;   // written in insertion order
  struct Tensor {
    std::string name;
    std::vector<int64_t> ne;    // ne[0] innermost
    const float* data = nullptr;
  };
  std::vector<Tensor> tensors;  // written in insertion order

  void set_str(const std::string& k, const std::string& v);
  void set_u32(const std::string& k, uint32_t v);
  void set_u64(const std::string& k, uint64_t v);
  void set_f32(const std::string& k, float v);
  void set_arr_u64(const std::string& k, const std::vector<uint64_t>& v);
  void set_arr_str(const std::string& k, const std::vector<std::string>& v);
  void add_f32(const std::string& name, std::vector<int64_t> ne, const float* data);
  bool write(const std::string& path, std::string& err) const;
};

struct GgufFile {
  struct Tensor {
    std::vector<int64_t> ne;
    uint32_t type = 0;
    uint64_t offset = 0;        // from the start of the data section
  };
  std::map<std::string, GgufValue> kv;
  std::map<std::string, Tensor> tensors;
  std::vector<std::string> tensor_order;
  std::vector<uint8_t> bytes;
  size_t data_start = 0;

  // Parses the whole file; every length and offset is checked against the file size.
  bool open(const std::string& path, std::string& err);
  const GgufValue* find(const std::string& k) const;
  // F32 tensor `name` into out (elements = product of ne)
  bool read_f32(const std::string& name, std::vector<float>& out, std::string& err) const;
};

// One adapter target as the adapter file stores it (write_train_lora_gguf,
// src/train_checkpoint.h:42-113), tensors in this order where present: <stem>.lora_A F32 ne
// {in, rank} (= A [rank][in]), .lora_B ne {rank, out} (= B [out][rank]), .U ne {rank, out},
// .V ne {rank, in}, .M_xs ne {rank, rank}, .magnitude, .magnitude_r ne {out}, .magnitude_c
// ne {in}.
struct AdapterTargetView {
  std::string stem;
  int64_t in = 0, out = 0;
  const float* A = nullptr;     // standard families
  const float* B = nullptr;
  const float* U = nullptr;     // -xs: U [out][rank], V [in][rank] (frozen), M_xs [rank][rank]
  const float* V = nullptr;
  const float* M = nullptr;
  const float* m = nullptr;     // magnitude (dora-rows [out], dora-cols [in]); null: none
  int64_t m_len = 0;            // its length (0: out)
  const float* m_r = nullptr;   // bora [out]
  const float* m_c = nullptr;   // bora [in]
};
// Writes the adapter file (metadata general.architecture "sa3-lora", general.name, lora.adapter_type,
// lora.rank, lora.alpha, lora.n_targets; tensors in target order) through path + ".tmp" and a rename.
bool write_adapter_gguf(const std::string& path, const std::string& adapter_type, int rank, float alpha,
                        const std::vector<AdapterTargetView>& targets, std::string& err);

// "fnv1a64:%016x" of a file's bytes: the binding between a trainer-state file and the adapter file
// written with it (train_resume_file_fingerprint, src/train_resume.h:165-179)
std::string gguf_file_fingerprint(const std::string& path, std::string& err);

}  // namespace sa3k
