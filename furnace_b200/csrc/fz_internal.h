// Internal declarations shared by the host runtime and the kernels.
#pragma once

#include <cstdint>
#include <cstring>
#include <map>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

#include "../../include/furnace.h"

namespace fz {

// Status-carrying exception used inside the library; the C ABI converts it
// into a return code plus fz_last_error().
struct Error : std::runtime_error {
  int code;
  Error(int c, const std::string& m) : std::runtime_error(m), code(c) {}
};

[[noreturn]] void fail(int code, const char* fmt, ...);
void set_last_error(const std::string& m);
// FZ_EINVAL with the formatted message unless cond holds (argument checks).
void need(bool cond, const char* fmt, ...);

// Runs f and converts what it throws into the C ABI's status code, the
// message going to fz_last_error().
template <class F>
int guard(F&& f) {
  try {
    f();
    return FZ_OK;
  } catch (const Error& e) {
    set_last_error(e.what());
    return e.code;
  } catch (const std::bad_alloc&) {
    set_last_error("host allocation failed");
    return FZ_ENOMEM;
  } catch (const std::exception& e) {
    set_last_error(e.what());
    return FZ_EINVAL;
  }
}

// Block geometry of the ggml types on the path (src/gguf.rs:206-216).
inline bool block_geom(uint32_t t, uint32_t* elems, uint32_t* bytes) {
  switch (t) {
    case FZ_F32: *elems = 1; *bytes = 4; return true;
    case FZ_F16: *elems = 1; *bytes = 2; return true;
    case FZ_Q8_0: *elems = 32; *bytes = 34; return true;
    case FZ_Q5_0: *elems = 32; *bytes = 22; return true;
    case FZ_Q4_K: *elems = 256; *bytes = 144; return true;
    case FZ_Q6_K: *elems = 256; *bytes = 210; return true;
    default: return false;
  }
}
inline bool is_quant(uint32_t t) { return t == FZ_Q8_0 || t == FZ_Q5_0 || t == FZ_Q4_K || t == FZ_Q6_K; }

// ---------------------------------------------------------------------------
// GGUF
// ---------------------------------------------------------------------------
struct MetaValue {
  uint32_t tag = 0;
  uint64_t u = 0;
  int64_t i = 0;
  double f = 0;
  std::string s;
  size_t array_len = 0;
  uint32_t array_tag = 0;
  size_t array_pos = 0;  // file offset of the first element
};

struct TensorEntry {
  std::string name;
  std::vector<uint64_t> dims;
  uint32_t dtype = 0;
  uint64_t offset = 0;
  uint64_t n_elements() const {
    uint64_t n = 1;
    for (auto d : dims) n *= d;
    return n;
  }
};

struct GgufFile {
  const uint8_t* base = nullptr;
  size_t size = 0;
  bool mapped = false;
  std::vector<uint8_t> owned;  // fz_open_bytes copy
  uint32_t version = 0;
  std::map<std::string, MetaValue> meta;
  std::vector<TensorEntry> tensors;
  std::map<std::string, size_t> index;
  size_t data_start = 0;

  ~GgufFile();
  void parse();
  const TensorEntry* find(const std::string& n) const {
    auto it = index.find(n);
    return it == index.end() ? nullptr : &tensors[it->second];
  }
  // GgufFile::tensor (src/gguf.rs:412-434)
  const uint8_t* tensor_data(const TensorEntry& t, uint64_t* nbytes) const;
  uint32_t meta_u32(const std::string& k) const;
  float meta_f32(const std::string& k) const;
  const std::string& meta_str(const std::string& k) const;
  size_t meta_array_len(const std::string& k) const;
  // GgufFile::meta_array elements as strings / integers (GgufValue::as_str,
  // as_i64, src/gguf.rs:136-163); fails on an element of another type
  std::vector<std::string> meta_str_array(const std::string& k) const;
  std::vector<int64_t> meta_int_array(const std::string& k) const;
};

// Whether [p, p + n) is well-formed UTF-8 (what Rust's String::from_utf8 accepts).
bool utf8_valid(const uint8_t* p, size_t n);

std::unique_ptr<GgufFile> open_gguf(const char* path);
std::unique_ptr<GgufFile> open_gguf_bytes(const void* data, size_t n);
fz_config config_from_gguf(const GgufFile& f);

}  // namespace fz

struct fz_file {
  std::unique_ptr<fz::GgufFile> g;
};
