// GGUF reader for the device loader.  Same acceptance rules as the reference
// parser (src/gguf.rs:315-363): magic "GGUF", version 2 or 3, every read
// bounds-checked, tensor dims <= 4, known ggml type ids, alignment from
// general.alignment (default 32, power of two), data start rounded up to it,
// and tensor data bounds checked at lookup (src/gguf.rs:412-434), strings
// well-formed UTF-8 (src/gguf.rs:71-75).  Metadata arrays are validated and
// skipped at parse time; their length and the offset of their first element
// are kept, and the tokenizer reads its tables from there.

#include <cstdarg>
#include <cstdio>
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include "fz_internal.h"

namespace fz {

static thread_local std::string g_last_error;

void set_last_error(const std::string& m) { g_last_error = m; }
const std::string& last_error() { return g_last_error; }

void fail(int code, const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  throw Error(code, buf);
}

void need(bool cond, const char* fmt, ...) {
  if (cond) return;
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  throw Error(FZ_EINVAL, buf);
}

namespace {

struct Reader {
  const uint8_t* p;
  size_t n, pos = 0;
  const uint8_t* take(size_t k) {
    if (k > n - pos) fail(FZ_EFORMAT, "unexpected EOF: need %zu bytes at offset %zu", k, pos);
    const uint8_t* r = p + pos;
    pos += k;
    return r;
  }
  template <class T>
  T get() {
    T v;
    memcpy(&v, take(sizeof(T)), sizeof(T));  // little-endian host (x86-64)
    return v;
  }
  std::string str() {
    uint64_t len = get<uint64_t>();
    if (len > n - pos) fail(FZ_EFORMAT, "unexpected EOF: need %llu bytes at offset %zu", (unsigned long long)len, pos);
    const uint8_t* s = take((size_t)len);
    if (!utf8_valid(s, (size_t)len)) fail(FZ_EFORMAT, "string is not valid UTF-8");
    return std::string((const char*)s, (size_t)len);
  }
};

// Byte size of one scalar metadata value, 0 for strings/arrays.
size_t scalar_size(uint32_t tag) {
  static const size_t sz[] = {1, 1, 2, 2, 4, 4, 4, 1, 0, 0, 8, 8, 8};
  return tag <= 12 ? sz[tag] : 0;
}

void read_value(Reader& r, uint32_t tag, MetaValue* v, int depth) {
  v->tag = tag;
  switch (tag) {
    case 0: v->u = r.get<uint8_t>(); v->i = (int64_t)v->u; break;
    case 1: v->i = r.get<int8_t>(); break;
    case 2: v->u = r.get<uint16_t>(); v->i = (int64_t)v->u; break;
    case 3: v->i = r.get<int16_t>(); break;
    case 4: v->u = r.get<uint32_t>(); v->i = (int64_t)v->u; break;
    case 5: v->i = r.get<int32_t>(); break;
    case 6: v->f = r.get<float>(); break;
    case 7: v->u = r.get<uint8_t>() != 0; break;
    case 8: v->s = r.str(); break;
    case 9: {
      uint32_t et = r.get<uint32_t>();
      uint64_t cnt = r.get<uint64_t>();
      v->array_tag = et;
      v->array_len = (size_t)cnt;
      v->array_pos = r.pos;
      if (depth > 8) fail(FZ_EFORMAT, "metadata arrays nested too deeply");
      size_t ss = scalar_size(et);
      if (ss) {
        if (cnt > (r.n - r.pos) / ss) fail(FZ_EFORMAT, "unexpected EOF: array of %llu items", (unsigned long long)cnt);
        r.take((size_t)cnt * ss);
      } else {
        MetaValue tmp;
        for (uint64_t k = 0; k < cnt; k++) read_value(r, et, &tmp, depth + 1);
      }
      break;
    }
    case 10: v->u = r.get<uint64_t>(); v->i = (int64_t)v->u; break;
    case 11: v->i = r.get<int64_t>(); break;
    case 12: v->f = r.get<double>(); break;
    default: fail(FZ_EFORMAT, "unknown metadata value type tag %u", tag);
  }
}

bool known_ggml_type(uint32_t v) {
  // the discriminants the reference accepts (src/gguf.rs:218-242)
  return v <= 3 || (v >= 6 && v <= 15) || (v >= 24 && v <= 28) || v == 30;
}

}  // namespace

GgufFile::~GgufFile() {
  if (mapped && base) munmap((void*)base, size);
}

void GgufFile::parse() {
  Reader r{base, size};
  const uint8_t* magic = r.take(4);
  if (memcmp(magic, "GGUF", 4) != 0)
    fail(FZ_EFORMAT, "not a GGUF file (bad magic %02x %02x %02x %02x)", magic[0], magic[1], magic[2], magic[3]);
  version = r.get<uint32_t>();
  if (version != 2 && version != 3) fail(FZ_EFORMAT, "unsupported GGUF version %u (only 2 and 3)", version);
  uint64_t n_tensors = r.get<uint64_t>();
  uint64_t n_kv = r.get<uint64_t>();
  for (uint64_t k = 0; k < n_kv; k++) {
    std::string key = r.str();
    uint32_t tag = r.get<uint32_t>();
    MetaValue v;
    try {
      read_value(r, tag, &v, 0);
    } catch (const Error& e) {
      fail(e.code, "metadata key '%s': %s", key.c_str(), e.what());
    }
    meta[key] = std::move(v);
  }
  for (uint64_t k = 0; k < n_tensors; k++) {
    TensorEntry t;
    t.name = r.str();
    uint32_t nd = r.get<uint32_t>();
    if (nd > 4) fail(FZ_EFORMAT, "tensor '%s' has %u dims, max is 4", t.name.c_str(), nd);
    for (uint32_t d = 0; d < nd; d++) t.dims.push_back(r.get<uint64_t>());
    t.dtype = r.get<uint32_t>();
    if (!known_ggml_type(t.dtype)) fail(FZ_EFORMAT, "tensor '%s': unsupported ggml tensor type %u", t.name.c_str(), t.dtype);
    t.offset = r.get<uint64_t>();
    index[t.name] = tensors.size();
    tensors.push_back(std::move(t));
  }
  uint64_t align = 32;
  auto it = meta.find("general.alignment");
  if (it != meta.end() && (it->second.tag == 4 || (it->second.tag == 10 && it->second.u <= 0xffffffffull)))
    align = it->second.u;
  if (align == 0 || (align & (align - 1))) fail(FZ_EFORMAT, "general.alignment %llu is not a power of two", (unsigned long long)align);
  size_t ds = (size_t)((r.pos + align - 1) / align * align);
  if (ds > size) fail(FZ_EFORMAT, "file truncated: tensor data would start at %zu but file is %zu bytes", ds, size);
  data_start = ds;
}

const uint8_t* GgufFile::tensor_data(const TensorEntry& t, uint64_t* nbytes) const {
  uint32_t be, bb;
  if (!block_geom(t.dtype, &be, &bb)) fail(FZ_EFORMAT, "tensor '%s': dtype %u not supported yet", t.name.c_str(), t.dtype);
  uint64_t n = t.n_elements();
  if (n % be) fail(FZ_EFORMAT, "tensor '%s' has %llu elements, not a multiple of block size %u", t.name.c_str(), (unsigned long long)n, be);
  uint64_t sz = n / be * bb;
  uint64_t start = data_start + t.offset;
  if (start < data_start || start > size || sz > size - start)
    fail(FZ_EFORMAT, "tensor '%s' data [%llu, %llu+%llu) runs past end of file (%zu bytes)", t.name.c_str(),
         (unsigned long long)start, (unsigned long long)start, (unsigned long long)sz, size);
  *nbytes = sz;
  return base + start;
}

uint32_t GgufFile::meta_u32(const std::string& k) const {
  auto it = meta.find(k);
  if (it != meta.end()) {
    if (it->second.tag == 4) return (uint32_t)it->second.u;
    if (it->second.tag == 10 && it->second.u <= 0xffffffffull) return (uint32_t)it->second.u;
  }
  fail(FZ_EFORMAT, "metadata key '%s' missing or not a u32", k.c_str());
}

float GgufFile::meta_f32(const std::string& k) const {
  auto it = meta.find(k);
  if (it != meta.end() && (it->second.tag == 6 || it->second.tag == 12)) return (float)it->second.f;
  fail(FZ_EFORMAT, "metadata key '%s' missing or not a float", k.c_str());
}

const std::string& GgufFile::meta_str(const std::string& k) const {
  auto it = meta.find(k);
  if (it != meta.end() && it->second.tag == 8) return it->second.s;
  fail(FZ_EFORMAT, "metadata key '%s' missing or not a string", k.c_str());
}

size_t GgufFile::meta_array_len(const std::string& k) const {
  auto it = meta.find(k);
  if (it != meta.end() && it->second.tag == 9) return it->second.array_len;
  fail(FZ_EFORMAT, "metadata key '%s' missing or not an array", k.c_str());
}

std::vector<std::string> GgufFile::meta_str_array(const std::string& k) const {
  auto it = meta.find(k);
  if (it == meta.end() || it->second.tag != 9) fail(FZ_EFORMAT, "metadata key '%s' missing or not an array", k.c_str());
  const MetaValue& v = it->second;
  std::vector<std::string> out;
  if (v.array_len == 0) return out;
  if (v.array_tag != 8) fail(FZ_EFORMAT, "metadata key '%s': element is not a string", k.c_str());
  Reader r{base, size, v.array_pos};
  out.reserve(v.array_len);
  for (size_t i = 0; i < v.array_len; i++) out.push_back(r.str());
  return out;
}

std::vector<int64_t> GgufFile::meta_int_array(const std::string& k) const {
  auto it = meta.find(k);
  if (it == meta.end() || it->second.tag != 9) fail(FZ_EFORMAT, "metadata key '%s' missing or not an array", k.c_str());
  const MetaValue& v = it->second;
  std::vector<int64_t> out;
  if (v.array_len == 0) return out;
  const uint32_t t = v.array_tag;
  if (!(t <= 5 || t == 10 || t == 11)) fail(FZ_EFORMAT, "metadata key '%s': element is not an integer", k.c_str());
  Reader r{base, size, v.array_pos};
  out.reserve(v.array_len);
  for (size_t i = 0; i < v.array_len; i++) {
    MetaValue e;
    read_value(r, t, &e, 1);
    if (t == 10 && e.u > (uint64_t)INT64_MAX) fail(FZ_EFORMAT, "metadata key '%s': element is not an i64", k.c_str());
    out.push_back(e.i);
  }
  return out;
}

// Well-formed UTF-8 per Unicode table 3-7 (no overlongs, surrogates or code
// points above U+10FFFF).
bool utf8_valid(const uint8_t* p, size_t n) {
  size_t i = 0;
  while (i < n) {
    const uint8_t b = p[i];
    if (b < 0x80) {
      i++;
      continue;
    }
    size_t len;
    uint8_t lo = 0x80, hi = 0xBF;
    if (b >= 0xC2 && b <= 0xDF) {
      len = 2;
    } else if (b >= 0xE0 && b <= 0xEF) {
      len = 3;
      if (b == 0xE0) lo = 0xA0;
      if (b == 0xED) hi = 0x9F;
    } else if (b >= 0xF0 && b <= 0xF4) {
      len = 4;
      if (b == 0xF0) lo = 0x90;
      if (b == 0xF4) hi = 0x8F;
    } else {
      return false;
    }
    if (n - i < len || p[i + 1] < lo || p[i + 1] > hi) return false;
    for (size_t k = 2; k < len; k++)
      if (p[i + k] < 0x80 || p[i + k] > 0xBF) return false;
    i += len;
  }
  return true;
}

std::unique_ptr<GgufFile> open_gguf(const char* path) {
  int fd = ::open(path, O_RDONLY);
  if (fd < 0) fail(FZ_EIO, "cannot open %s", path);
  struct stat st;
  if (fstat(fd, &st) != 0) {
    ::close(fd);
    fail(FZ_EIO, "cannot stat %s", path);
  }
  auto g = std::make_unique<GgufFile>();
  g->size = (size_t)st.st_size;
  if (g->size) {
    void* p = mmap(nullptr, g->size, PROT_READ, MAP_SHARED, fd, 0);
    if (p == MAP_FAILED) {
      ::close(fd);
      fail(FZ_EIO, "cannot mmap %s", path);
    }
    g->base = (const uint8_t*)p;
    g->mapped = true;
  }
  ::close(fd);
  g->parse();
  return g;
}

std::unique_ptr<GgufFile> open_gguf_bytes(const void* data, size_t n) {
  auto g = std::make_unique<GgufFile>();
  g->owned.assign((const uint8_t*)data, (const uint8_t*)data + n);
  g->base = g->owned.data();
  g->size = n;
  g->parse();
  return g;
}

// Config::from_gguf (src/model.rs:41-60)
fz_config config_from_gguf(const GgufFile& f) {
  const std::string& arch = f.meta_str("general.architecture");
  if (arch != "qwen2") fail(FZ_EFORMAT, "architecture '%s' not supported", arch.c_str());
  fz_config c;
  c.n_heads = f.meta_u32("qwen2.attention.head_count");
  c.hidden = f.meta_u32("qwen2.embedding_length");
  if (c.n_heads == 0 || c.hidden % c.n_heads) fail(FZ_EFORMAT, "hidden %u not divisible by %u heads", c.hidden, c.n_heads);
  c.n_layers = f.meta_u32("qwen2.block_count");
  c.n_kv_heads = f.meta_u32("qwen2.attention.head_count_kv");
  c.ffn = f.meta_u32("qwen2.feed_forward_length");
  c.head_dim = c.hidden / c.n_heads;
  c.rope_theta = f.meta_f32("qwen2.rope.freq_base");
  c.rms_eps = f.meta_f32("qwen2.attention.layer_norm_rms_epsilon");
  c.vocab = (uint32_t)f.meta_array_len("tokenizer.ggml.tokens");
  c.context_length = f.meta_u32("qwen2.context_length");
  return c;
}

}  // namespace fz
