// furnace_oracle.cpp -- TEST INFRASTRUCTURE ONLY.
//
// A CPU restatement of the furnace reference's decode path, used as the parity
// checker for the CUDA implementation and as the timed CPU baseline.  Only the
// test suite, __graft_entry__.smoke() and bench.py's CPU-baseline leg load this
// library; the product (libfurnace_cuda.so) never links or calls it.
//
// Every function names the reference file:line it restates (paths inside the
// furnace project).  Floating-point evaluation order follows the reference
// exactly: the build uses -O2 -ffp-contract=off (Rust never contracts a*b+c
// into an FMA), left-to-right sums where Rust folds an iterator, the 8-lane
// dot of src/tensor.rs:146-160, and glibc powf/sinf/cosf/expf/sqrtf, which is
// what Rust's f32 methods call on Linux.
//
// Parallelism stands in for rayon: matmul output rows are split into chunks
// of 64 (src/tensor.rs:102-113, :114-135) over a persistent thread pool.
// Each output element is computed by exactly one thread with the same
// arithmetic, so results do not depend on the thread count.

#include <atomic>
#include <cmath>
#include <condition_variable>
#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <fcntl.h>
#include <functional>
#include <map>
#include <mutex>
#include <string>
#include <sys/mman.h>
#include <sys/stat.h>
#include <thread>
#include <unistd.h>
#include <vector>

namespace {

thread_local std::string g_err;

void set_err(const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  g_err = buf;
}

// ---------------------------------------------------------------------------
// f16 -> f32, exact (the `half` crate's to_f32 used at src/quant.rs:36,54,94).
// ---------------------------------------------------------------------------
float f16_to_f32(uint16_t h) {
  uint32_t sign = (uint32_t)(h >> 15) << 31;
  uint32_t exp = (h >> 10) & 0x1f;
  uint32_t man = h & 0x3ff;
  uint32_t bits;
  if (exp == 0) {
    if (man == 0) {
      bits = sign;
    } else {
      // subnormal: normalise
      int e = -1;
      do {
        man <<= 1;
        e++;
      } while (!(man & 0x400));
      man &= 0x3ff;
      bits = sign | ((uint32_t)(127 - 15 - e) << 23) | (man << 13);
    }
  } else if (exp == 31) {
    bits = sign | 0x7f800000u | (man << 13);
  } else {
    bits = sign | ((exp + 127 - 15) << 23) | (man << 13);
  }
  float f;
  memcpy(&f, &bits, 4);
  return f;
}

uint16_t rd16(const uint8_t* p) { return (uint16_t)(p[0] | (p[1] << 8)); }
uint32_t rd32(const uint8_t* p) {
  return (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) | ((uint32_t)p[3] << 24);
}

// ---------------------------------------------------------------------------
// Thread pool standing in for rayon's global pool (src/main.rs:167-176).
// ---------------------------------------------------------------------------
class Pool {
 public:
  explicit Pool(int n) { resize(n); }
  ~Pool() { stop_all(); }

  void resize(int n) {
    stop_all();
    if (n < 1) n = 1;
    nthreads_ = n;
    stop_ = false;
    for (int i = 1; i < n; i++) workers_.emplace_back([this] { loop(); });
  }
  int size() const { return nthreads_; }

  // Run fn(i) for i in [0, n) across the pool; returns when all are done.
  void parallel_for(size_t n, const std::function<void(size_t)>& fn) {
    if (n == 0) return;
    if (nthreads_ == 1 || n == 1) {
      for (size_t i = 0; i < n; i++) fn(i);
      return;
    }
    std::unique_lock<std::mutex> lk(m_);
    job_ = &fn;
    job_n_ = n;
    next_.store(0);
    active_ = (int)workers_.size();
    gen_++;
    lk.unlock();
    cv_.notify_all();
    drain();
    lk.lock();
    done_cv_.wait(lk, [this] { return active_ == 0; });
    job_ = nullptr;
  }

 private:
  void drain() {
    for (;;) {
      size_t i = next_.fetch_add(1);
      if (i >= job_n_) break;
      (*job_)(i);
    }
  }
  void loop() {
    uint64_t seen = 0;
    for (;;) {
      std::unique_lock<std::mutex> lk(m_);
      cv_.wait(lk, [&] { return stop_ || gen_ != seen; });
      if (stop_) return;
      seen = gen_;
      lk.unlock();
      drain();
      lk.lock();
      if (--active_ == 0) done_cv_.notify_all();
    }
  }
  void stop_all() {
    {
      std::lock_guard<std::mutex> lk(m_);
      stop_ = true;
    }
    cv_.notify_all();
    for (auto& t : workers_) t.join();
    workers_.clear();
  }

  int nthreads_ = 1;
  std::vector<std::thread> workers_;
  std::mutex m_;
  std::condition_variable cv_, done_cv_;
  bool stop_ = false;
  uint64_t gen_ = 0;
  int active_ = 0;
  const std::function<void(size_t)>* job_ = nullptr;
  size_t job_n_ = 0;
  std::atomic<size_t> next_{0};
};

Pool& pool() {
  static Pool p((int)std::max(1u, std::thread::hardware_concurrency()));
  return p;
}

// ---------------------------------------------------------------------------
// ggml types (src/gguf.rs:180-243) and block layouts (src/gguf.rs:206-216).
// ---------------------------------------------------------------------------
enum : uint32_t { T_F32 = 0, T_F16 = 1, T_Q5_0 = 6, T_Q8_0 = 8, T_Q4_K = 12, T_Q6_K = 14 };

bool block_layout(uint32_t t, size_t* elems, size_t* bytes) {
  switch (t) {
    case T_F32: *elems = 1; *bytes = 4; return true;
    case T_F16: *elems = 1; *bytes = 2; return true;
    case T_Q8_0: *elems = 32; *bytes = 34; return true;
    case T_Q5_0: *elems = 32; *bytes = 22; return true;
    case T_Q4_K: *elems = 256; *bytes = 144; return true;
    case T_Q6_K: *elems = 256; *bytes = 210; return true;
    default: return false;
  }
}

bool known_type(uint32_t v) {
  // src/gguf.rs:218-242: the discriminants the parser accepts
  switch (v) {
    case 0: case 1: case 2: case 3: case 6: case 7: case 8: case 9: case 10:
    case 11: case 12: case 13: case 14: case 15: case 24: case 25: case 26:
    case 27: case 28: case 30:
      return true;
    default:
      return false;
  }
}

// ---------------------------------------------------------------------------
// GGUF parsing (src/gguf.rs:23-76 Cursor, :83-171 values, :246-291 tensor
// info, :315-363 parse, :366-434 open/tensor).
// ---------------------------------------------------------------------------
struct Value {
  uint32_t tag = 0;
  uint64_t u = 0;   // unsigned / bool payload
  int64_t i = 0;    // signed payload
  double f = 0;     // float payload
  std::string s;
  std::vector<Value> arr;
  bool as_u32(uint32_t* out) const {  // src/gguf.rs:128-134
    if (tag == 4) { *out = (uint32_t)u; return true; }
    if (tag == 10) { if (u > 0xffffffffull) return false; *out = (uint32_t)u; return true; }
    return false;
  }
  bool as_f32(float* out) const {  // src/gguf.rs:150-156
    if (tag == 6) { *out = (float)f; return true; }
    if (tag == 12) { *out = (float)f; return true; }
    return false;
  }
};

struct Cursor {
  const uint8_t* d;
  size_t n, pos = 0;
  bool take(size_t k, const uint8_t** out) {
    if (pos + k < pos || pos + k > n) {
      set_err("unexpected EOF: need %zu bytes at offset %zu", k, pos);
      return false;
    }
    *out = d + pos;
    pos += k;
    return true;
  }
  bool u8(uint8_t* v) { const uint8_t* p; if (!take(1, &p)) return false; *v = p[0]; return true; }
  bool u16(uint16_t* v) { const uint8_t* p; if (!take(2, &p)) return false; *v = rd16(p); return true; }
  bool u32(uint32_t* v) { const uint8_t* p; if (!take(4, &p)) return false; *v = rd32(p); return true; }
  bool u64(uint64_t* v) {
    const uint8_t* p;
    if (!take(8, &p)) return false;
    *v = (uint64_t)rd32(p) | ((uint64_t)rd32(p + 4) << 32);
    return true;
  }
  bool str(std::string* s) {
    uint64_t len;
    if (!u64(&len)) return false;
    const uint8_t* p;
    if (!take((size_t)len, &p)) return false;
    s->assign((const char*)p, (size_t)len);
    return true;
  }
};

bool read_value(Cursor& c, uint32_t tag, Value* v) {
  v->tag = tag;
  switch (tag) {
    case 0: { uint8_t x; if (!c.u8(&x)) return false; v->u = x; v->i = x; return true; }
    case 1: { uint8_t x; if (!c.u8(&x)) return false; v->i = (int8_t)x; return true; }
    case 2: { uint16_t x; if (!c.u16(&x)) return false; v->u = x; v->i = x; return true; }
    case 3: { uint16_t x; if (!c.u16(&x)) return false; v->i = (int16_t)x; return true; }
    case 4: { uint32_t x; if (!c.u32(&x)) return false; v->u = x; v->i = x; return true; }
    case 5: { uint32_t x; if (!c.u32(&x)) return false; v->i = (int32_t)x; return true; }
    case 6: { uint32_t x; if (!c.u32(&x)) return false; float f; memcpy(&f, &x, 4); v->f = f; return true; }
    case 7: { uint8_t x; if (!c.u8(&x)) return false; v->u = x != 0; return true; }
    case 8: return c.str(&v->s);
    case 9: {
      uint32_t et;
      uint64_t cnt;
      if (!c.u32(&et) || !c.u64(&cnt)) return false;
      v->arr.reserve((size_t)std::min<uint64_t>(cnt, 1u << 20));
      for (uint64_t k = 0; k < cnt; k++) {
        Value e;
        if (!read_value(c, et, &e)) return false;
        v->arr.push_back(std::move(e));
      }
      return true;
    }
    case 10: return c.u64(&v->u);
    case 11: { uint64_t x; if (!c.u64(&x)) return false; v->i = (int64_t)x; return true; }
    case 12: { uint64_t x; if (!c.u64(&x)) return false; double f; memcpy(&f, &x, 8); v->f = f; return true; }
    default: set_err("unknown metadata value type tag %u", tag); return false;
  }
}

struct TensorInfo {
  std::string name;
  std::vector<uint64_t> dims;
  uint32_t dtype;
  uint64_t offset;
  size_t n_elements() const {
    size_t n = 1;
    for (auto d : dims) n *= (size_t)d;
    return n;
  }
};

struct File {
  uint8_t* map = nullptr;
  size_t size = 0;
  uint32_t version = 0;
  std::map<std::string, Value> meta;
  std::vector<TensorInfo> tensors;
  size_t data_start = 0;
  ~File() {
    if (map) munmap(map, size);
  }
  const TensorInfo* find(const std::string& n) const {
    for (auto& t : tensors)
      if (t.name == n) return &t;
    return nullptr;
  }
  // src/gguf.rs:412-434
  bool tensor(const std::string& n, const TensorInfo** info, const uint8_t** raw, size_t* nbytes) const {
    const TensorInfo* t = find(n);
    if (!t) { set_err("no tensor named '%s'", n.c_str()); return false; }
    size_t be, bb;
    if (!block_layout(t->dtype, &be, &bb)) { set_err("dtype %u not supported yet", t->dtype); return false; }
    size_t ne = t->n_elements();
    if (ne % be) { set_err("tensor '%s' has %zu elements, not a multiple of block size %zu", n.c_str(), ne, be); return false; }
    size_t sz = ne / be * bb;
    size_t start = data_start + (size_t)t->offset;
    if (start + sz < start || start + sz > size) {
      set_err("tensor '%s' data [%zu, %zu+%zu) runs past end of file (%zu bytes)", n.c_str(), start, start, sz, size);
      return false;
    }
    *info = t;
    *raw = map + start;
    *nbytes = sz;
    return true;
  }
};

// src/gguf.rs:315-363
bool parse(const uint8_t* data, size_t n, File* f) {
  Cursor c{data, n};
  const uint8_t* magic;
  if (!c.take(4, &magic)) return false;
  if (memcmp(magic, "GGUF", 4) != 0) {
    set_err("not a GGUF file (bad magic %02x %02x %02x %02x)", magic[0], magic[1], magic[2], magic[3]);
    return false;
  }
  if (!c.u32(&f->version)) return false;
  if (f->version != 2 && f->version != 3) {
    set_err("unsupported GGUF version %u (only 2 and 3)", f->version);
    return false;
  }
  uint64_t tcount, kvcount;
  if (!c.u64(&tcount) || !c.u64(&kvcount)) return false;
  for (uint64_t k = 0; k < kvcount; k++) {
    std::string key;
    uint32_t tag;
    if (!c.str(&key) || !c.u32(&tag)) return false;
    Value v;
    if (!read_value(c, tag, &v)) {
      g_err = "metadata key '" + key + "': " + g_err;
      return false;
    }
    f->meta[key] = std::move(v);
  }
  for (uint64_t k = 0; k < tcount; k++) {
    TensorInfo t;
    uint32_t nd;
    if (!c.str(&t.name) || !c.u32(&nd)) return false;
    if (nd > 4) { set_err("tensor '%s' has %u dims, max is 4", t.name.c_str(), nd); return false; }
    for (uint32_t d = 0; d < nd; d++) {
      uint64_t x;
      if (!c.u64(&x)) return false;
      t.dims.push_back(x);
    }
    uint32_t dt;
    if (!c.u32(&dt)) return false;
    if (!known_type(dt)) { set_err("tensor '%s': unsupported ggml tensor type %u", t.name.c_str(), dt); return false; }
    t.dtype = dt;
    if (!c.u64(&t.offset)) return false;
    f->tensors.push_back(std::move(t));
  }
  size_t align = 32;
  auto it = f->meta.find("general.alignment");
  if (it != f->meta.end()) {
    uint32_t a;
    if (it->second.as_u32(&a)) align = a;
  }
  if (align == 0 || (align & (align - 1))) {
    set_err("general.alignment %zu is not a power of two", align);
    return false;
  }
  size_t ds = (c.pos + align - 1) / align * align;
  if (ds > n) {
    set_err("file truncated: tensor data would start at %zu but file is %zu bytes", ds, n);
    return false;
  }
  f->data_start = ds;
  return true;
}

// ---------------------------------------------------------------------------
// Dequantization (src/quant.rs:17-168, :261-281).
// ---------------------------------------------------------------------------
void dequant_block_q8_0(const uint8_t* b, float* out) {  // src/quant.rs:35-39
  float d = f16_to_f32(rd16(b));
  for (int i = 0; i < 32; i++) out[i] = d * (float)(int8_t)b[2 + i];
}

void dequant_block_q5_0(const uint8_t* b, float* out) {  // src/quant.rs:53-63
  float d = f16_to_f32(rd16(b));
  uint32_t qh = rd32(b + 2);
  const uint8_t* qs = b + 6;
  for (int j = 0; j < 16; j++) {
    uint32_t hi0 = ((qh >> j) & 1) << 4;
    uint32_t hi1 = ((qh >> (j + 16)) & 1) << 4;
    out[j] = d * (float)((int32_t)((qs[j] & 0x0F) | hi0) - 16);
    out[j + 16] = d * (float)((int32_t)((qs[j] >> 4) | hi1) - 16);
  }
}

void q4k_scale_min(int j, const uint8_t* s, float* sc, float* m) {  // src/quant.rs:78-88
  uint8_t a, b;
  if (j < 4) {
    a = s[j] & 63;
    b = s[j + 4] & 63;
  } else {
    a = (uint8_t)((s[j + 4] & 0x0F) | ((s[j - 4] >> 6) << 4));
    b = (uint8_t)((s[j + 4] >> 4) | ((s[j] >> 6) << 4));
  }
  *sc = (float)a;
  *m = (float)b;
}

void dequant_block_q4_k(const uint8_t* b, float* out) {  // src/quant.rs:93-109
  float d = f16_to_f32(rd16(b));
  float dmin = f16_to_f32(rd16(b + 2));
  const uint8_t* scales = b + 4;
  const uint8_t* qs = b + 16;
  for (int j64 = 0; j64 < 4; j64++) {
    const uint8_t* q = qs + 32 * j64;
    float sc1, m1, sc2, m2;
    q4k_scale_min(2 * j64, scales, &sc1, &m1);
    q4k_scale_min(2 * j64 + 1, scales, &sc2, &m2);
    float d1 = d * sc1, min1 = dmin * m1;
    float d2 = d * sc2, min2 = dmin * m2;
    for (int l = 0; l < 32; l++) {
      out[64 * j64 + l] = d1 * (float)(q[l] & 0x0F) - min1;
      out[64 * j64 + 32 + l] = d2 * (float)(q[l] >> 4) - min2;
    }
  }
}

void dequant_block_q6_k(const uint8_t* b, float* out) {  // src/quant.rs:114-133
  float d = f16_to_f32(rd16(b + 208));
  for (int half = 0; half < 2; half++) {
    const uint8_t* ql = b + 64 * half;
    const uint8_t* qh = b + 128 + 32 * half;
    const uint8_t* sc = b + 192 + 8 * half;
    float* y = out + 128 * half;
    for (int l = 0; l < 32; l++) {
      int is = l / 16;
      int q1 = ((ql[l] & 0x0F) | (((int)qh[l] & 3) << 4)) - 32;
      int q2 = ((ql[l + 32] & 0x0F) | ((((int)qh[l] >> 2) & 3) << 4)) - 32;
      int q3 = ((ql[l] >> 4) | ((((int)qh[l] >> 4) & 3) << 4)) - 32;
      int q4 = ((ql[l + 32] >> 4) | ((((int)qh[l] >> 6) & 3) << 4)) - 32;
      y[l] = d * (float)(int8_t)sc[is] * (float)q1;
      y[l + 32] = d * (float)(int8_t)sc[is + 2] * (float)q2;
      y[l + 64] = d * (float)(int8_t)sc[is + 4] * (float)q3;
      y[l + 96] = d * (float)(int8_t)sc[is + 6] * (float)q4;
    }
  }
}

typedef void (*BlockFn)(const uint8_t*, float*);

bool block_fn(uint32_t t, BlockFn* fn, size_t* be, size_t* bb) {  // src/quant.rs:137-144
  switch (t) {
    case T_Q8_0: *fn = dequant_block_q8_0; *be = 32; *bb = 34; return true;
    case T_Q5_0: *fn = dequant_block_q5_0; *be = 32; *bb = 22; return true;
    case T_Q4_K: *fn = dequant_block_q4_k; *be = 256; *bb = 144; return true;
    case T_Q6_K: *fn = dequant_block_q6_k; *be = 256; *bb = 210; return true;
    default: return false;
  }
}

// src/quant.rs:261-281 (dequantize), :17-42 (Q8_0 checks), :147-167 (blocks)
bool dequantize(uint32_t t, const uint8_t* raw, size_t nbytes, size_t n, float* out) {
  if (t == T_F32) {
    if (nbytes != n * 4) { set_err("F32 data is %zu bytes, expected %zu", nbytes, n * 4); return false; }
    memcpy(out, raw, n * 4);
    return true;
  }
  BlockFn fn;
  size_t be, bb;
  if (!block_fn(t, &fn, &be, &bb)) { set_err("dequantization for type %u is not implemented", t); return false; }
  if (n % be) { set_err("element count %zu is not a multiple of %zu", n, be); return false; }
  size_t nb = n / be;
  if (nbytes != nb * bb) { set_err("data is %zu bytes, expected %zu (%zu blocks of %zu)", nbytes, nb * bb, nb, bb); return false; }
  for (size_t k = 0; k < nb; k++) fn(raw + k * bb, out + k * be);
  return true;
}

// ---------------------------------------------------------------------------
// Tensor ops (src/tensor.rs).
// ---------------------------------------------------------------------------
// 8-lane dot (src/tensor.rs:146-160)
float dot8(const float* a, const float* b, size_t n) {
  float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  size_t full = n / 8 * 8;
  for (size_t i = 0; i < full; i += 8)
    for (int j = 0; j < 8; j++) acc[j] += a[i + j] * b[i + j];
  float sum = 0.0f;
  for (int j = 0; j < 8; j++) sum += acc[j];
  for (size_t i = full; i < n; i++) sum += a[i] * b[i];
  return sum;
}

// matmul_with (src/tensor.rs:86-136): out[s][o] = row_dot(o, a[s]).
// Decode (seq == 1) splits outputs into chunks of 64; prefill streams each
// weight row once for every activation row.  Both compute each element with
// the same row_dot, so the split is a scheduling choice only.
void matmul_with(const float* a, size_t seq, size_t d_out, size_t d_in, float* out,
                 const std::function<float(size_t, const float*)>& row_dot) {
  size_t chunks = (d_out + 63) / 64;
  pool().parallel_for(chunks, [&](size_t c) {
    size_t o0 = c * 64, o1 = std::min(d_out, o0 + 64);
    for (size_t o = o0; o < o1; o++)
      for (size_t s = 0; s < seq; s++) out[s * d_out + o] = row_dot(o, a + s * d_in);
  });
}

// matmul_q8_0 (src/quant.rs:234-258)
void matmul_q8_0(const float* a, size_t seq, const uint8_t* raw, size_t d_out, size_t d_in, float* out) {
  size_t row_bytes = d_in / 32 * 34;
  matmul_with(a, seq, d_out, d_in, out, [&](size_t o, const float* arow) {
    const uint8_t* row = raw + o * row_bytes;
    float acc = 0.0f;
    for (size_t b = 0; b < d_in / 32; b++) {
      const uint8_t* blk = row + b * 34;
      float scale = f16_to_f32(rd16(blk));
      const float* ab = arow + b * 32;
      float lanes[8] = {0, 0, 0, 0, 0, 0, 0, 0};
      for (int j = 0; j < 4; j++)
        for (int l = 0; l < 8; l++) lanes[l] += ab[j * 8 + l] * (float)(int8_t)blk[2 + j * 8 + l];
      float s = 0.0f;
      for (int l = 0; l < 8; l++) s += lanes[l];
      acc += scale * s;
    }
    return acc;
  });
}

// matmul_blocks (src/quant.rs:198-227)
void matmul_blocks(const float* a, size_t seq, const uint8_t* raw, size_t d_out, size_t d_in,
                   size_t be, size_t bb, BlockFn fn, float* out) {
  size_t row_bytes = d_in / be * bb;
  if (seq > 1) {
    // Prefill: the reference re-dequantizes each block for every activation
    // row (src/tensor.rs:114-135 calling src/quant.rs:214-226).  The
    // dequantized values do not depend on the row, so each weight row is
    // decoded once here and every activation row runs the same per-block
    // `acc += dot(...)` sequence over it: identical results, less work.
    size_t chunks = (d_out + 63) / 64;
    pool().parallel_for(chunks, [&](size_t c) {
      std::vector<float> wrow(d_in);
      size_t o0 = c * 64, o1 = std::min(d_out, o0 + 64);
      for (size_t o = o0; o < o1; o++) {
        const uint8_t* row = raw + o * row_bytes;
        for (size_t b = 0; b < d_in / be; b++) fn(row + b * bb, wrow.data() + b * be);
        for (size_t s = 0; s < seq; s++) {
          const float* arow = a + s * d_in;
          float acc = 0.0f;
          for (size_t b = 0; b < d_in / be; b++) acc += dot8(arow + b * be, wrow.data() + b * be, be);
          out[s * d_out + o] = acc;
        }
      }
    });
    return;
  }
  matmul_with(a, seq, d_out, d_in, out, [&](size_t o, const float* arow) {
    const uint8_t* row = raw + o * row_bytes;
    float buf[256];
    float acc = 0.0f;
    for (size_t b = 0; b < d_in / be; b++) {
      fn(row + b * bb, buf);
      acc += dot8(arow + b * be, buf, be);
    }
    return acc;
  });
}

// matmul (src/tensor.rs:74-80): dense f32 weights
void matmul_f32(const float* a, size_t seq, const float* w, size_t d_out, size_t d_in, float* out) {
  matmul_with(a, seq, d_out, d_in, out, [&](size_t o, const float* arow) { return dot8(arow, w + o * d_in, d_in); });
}

// matmul_quant (src/quant.rs:170-193)
bool matmul_quant(const float* a, size_t seq, const uint8_t* raw, size_t nbytes, size_t d_out, size_t d_in,
                  uint32_t t, float* out) {
  BlockFn fn;
  size_t be, bb;
  if (!block_fn(t, &fn, &be, &bb)) { set_err("no fused matmul kernel for type %u", t); return false; }
  if (d_in % be) { set_err("matmul: in dim %zu not a multiple of %zu", d_in, be); return false; }
  if (nbytes != d_out * (d_in / be * bb)) { set_err("matmul: bad weight byte count"); return false; }
  if (t == T_Q8_0)
    matmul_q8_0(a, seq, raw, d_out, d_in, out);
  else
    matmul_blocks(a, seq, raw, d_out, d_in, be, bb, fn, out);
  return true;
}

// rmsnorm (src/tensor.rs:164-186)
void rmsnorm(const float* x, size_t rows, size_t cols, const float* w, float eps, float* out) {
  for (size_t r = 0; r < rows; r++) {
    const float* row = x + r * cols;
    float ss = 0.0f;
    for (size_t i = 0; i < cols; i++) ss += row[i] * row[i];
    float mean_sq = ss / (float)cols;
    float inv_rms = 1.0f / sqrtf(mean_sq + eps);
    for (size_t i = 0; i < cols; i++) out[r * cols + i] = row[i] * inv_rms * w[i];
  }
}

// softmax (src/tensor.rs:188-205)
void softmax(float* x, size_t rows, size_t cols) {
  for (size_t r = 0; r < rows; r++) {
    float* row = x + r * cols;
    float mx = -INFINITY;
    for (size_t i = 0; i < cols; i++) mx = fmaxf(mx, row[i]);
    float sum = 0.0f;
    for (size_t i = 0; i < cols; i++) {
      row[i] = expf(row[i] - mx);
      sum += row[i];
    }
    for (size_t i = 0; i < cols; i++) row[i] /= sum;
  }
}

// silu (src/tensor.rs:207-210) and swiglu (src/tensor.rs:213-227)
float silu1(float v) { return v / (1.0f + expf(-v)); }
float swiglu1(float g, float u) { return g / (1.0f + expf(-g)) * u; }

// rope (src/model.rs:193-217)
void rope(float* x, size_t seq, size_t n_heads, size_t hd, float theta, size_t start_pos) {
  size_t half = hd / 2;
  for (size_t s = 0; s < seq; s++) {
    float* row = x + s * n_heads * hd;
    for (size_t h = 0; h < n_heads; h++) {
      float* head = row + h * hd;
      for (size_t i = 0; i < half; i++) {
        float freq = powf(theta, -2.0f * (float)i / (float)hd);
        float angle = (float)(start_pos + s) * freq;
        float sn = sinf(angle), cs = cosf(angle);
        float a = head[i], b = head[i + half];
        head[i] = a * cs - b * sn;
        head[i + half] = a * sn + b * cs;
      }
    }
  }
}

// argmax, first max wins ties (src/generate.rs:69-77)
uint32_t argmax(const float* d, size_t n) {
  size_t best = 0;
  for (size_t i = 1; i < n; i++)
    if (d[i] > d[best]) best = i;
  return (uint32_t)best;
}

// ---------------------------------------------------------------------------
// Model (src/model.rs).
// ---------------------------------------------------------------------------
struct Config {  // src/model.rs:27-38
  uint32_t n_layers, n_heads, n_kv_heads, hidden, ffn, head_dim;
  float rope_theta, rms_eps;
  uint32_t vocab, context_length;
};

struct Weight {  // src/model.rs:66-74
  bool is_f32 = false;
  std::vector<float> f;  // [out, in] when is_f32
  const uint8_t* raw = nullptr;
  size_t nbytes = 0;
  uint32_t dtype = 0;
  size_t out = 0, in = 0;
  // Weight::matmul (src/model.rs:99-106)
  void matmul(const float* x, size_t seq, float* y) const {
    if (is_f32)
      matmul_f32(x, seq, f.data(), out, in, y);
    else
      matmul_quant(x, seq, raw, nbytes, out, in, dtype, y);
  }
};

struct Layer {  // src/model.rs:130-143
  std::vector<float> attn_norm, bq, bk, bv, ffn_norm;
  Weight wq, wk, wv, wo, w_gate, w_up, w_down;
};

struct Model {
  File file;
  Config cfg;
  Weight embedding, lm_head;
  std::vector<Layer> layers;
  std::vector<float> output_norm;
};

bool meta_u32(const File& f, const char* k, uint32_t* v) {
  auto it = f.meta.find(k);
  if (it == f.meta.end() || !it->second.as_u32(v)) { set_err("metadata key '%s' missing or not a u32", k); return false; }
  return true;
}
bool meta_f32(const File& f, const char* k, float* v) {
  auto it = f.meta.find(k);
  if (it == f.meta.end() || !it->second.as_f32(v)) { set_err("metadata key '%s' missing or not a float", k); return false; }
  return true;
}

// Config::from_gguf (src/model.rs:41-60)
bool config_from(const File& f, Config* c) {
  auto it = f.meta.find("general.architecture");
  if (it == f.meta.end() || it->second.tag != 8) { set_err("metadata key 'general.architecture' missing or not a string"); return false; }
  if (it->second.s != "qwen2") { set_err("architecture '%s' not supported", it->second.s.c_str()); return false; }
  uint32_t nh, hid;
  if (!meta_u32(f, "qwen2.attention.head_count", &nh) || !meta_u32(f, "qwen2.embedding_length", &hid)) return false;
  if (nh == 0 || hid % nh) { set_err("hidden %u not divisible by %u heads", hid, nh); return false; }
  c->n_heads = nh;
  c->hidden = hid;
  c->head_dim = hid / nh;
  if (!meta_u32(f, "qwen2.block_count", &c->n_layers) || !meta_u32(f, "qwen2.attention.head_count_kv", &c->n_kv_heads) ||
      !meta_u32(f, "qwen2.feed_forward_length", &c->ffn) || !meta_f32(f, "qwen2.rope.freq_base", &c->rope_theta) ||
      !meta_f32(f, "qwen2.attention.layer_norm_rms_epsilon", &c->rms_eps))
    return false;
  auto tk = f.meta.find("tokenizer.ggml.tokens");
  if (tk == f.meta.end() || tk->second.tag != 9) { set_err("metadata key 'tokenizer.ggml.tokens' missing or not an array"); return false; }
  c->vocab = (uint32_t)tk->second.arr.size();
  return meta_u32(f, "qwen2.context_length", &c->context_length);
}

// Tensor::from_gguf (src/tensor.rs:55-60): dequantize to f32
bool tensor_f32(const File& f, const std::string& name, std::vector<float>* out, size_t expect = 0) {
  const TensorInfo* info;
  const uint8_t* raw;
  size_t nb;
  if (!f.tensor(name, &info, &raw, &nb)) return false;
  size_t n = info->n_elements();
  if (expect && n != expect) { set_err("tensor '%s' has %zu elements, expected %zu", name.c_str(), n, expect); return false; }
  out->resize(n);
  return dequantize(info->dtype, raw, nb, n, out->data());
}

// load_weight (src/model.rs:112-126)
bool load_weight(const File& f, const std::string& name, bool use_f32, Weight* w) {
  const TensorInfo* info;
  const uint8_t* raw;
  size_t nb;
  if (!f.tensor(name, &info, &raw, &nb)) return false;
  BlockFn fn;
  size_t be, bb;
  bool fused = block_fn(info->dtype, &fn, &be, &bb);
  if (info->dims.size() != 2) { set_err("weight '%s' is not 2-D", name.c_str()); return false; }
  w->out = (size_t)info->dims[1];
  w->in = (size_t)info->dims[0];
  if (use_f32 || !fused) {
    w->is_f32 = true;
    return tensor_f32(f, name, &w->f);
  }
  w->raw = raw;
  w->nbytes = nb;
  w->dtype = info->dtype;
  return true;
}

// Model::load (src/model.rs:520-552)
bool model_load(Model* m, bool use_f32) {
  const File& f = m->file;
  if (!config_from(f, &m->cfg)) return false;
  const Config& c = m->cfg;
  if (!load_weight(f, "token_embd.weight", use_f32, &m->embedding)) return false;
  if (m->embedding.out != c.vocab || m->embedding.in != c.hidden) {
    set_err("token_embd is [%zu, %zu], config says [%u, %u]", m->embedding.out, m->embedding.in, c.vocab, c.hidden);
    return false;
  }
  m->layers.resize(c.n_layers);
  for (uint32_t i = 0; i < c.n_layers; i++) {
    Layer& L = m->layers[i];
    std::string p = "blk." + std::to_string(i) + ".";
    if (!tensor_f32(f, p + "attn_norm.weight", &L.attn_norm) || !load_weight(f, p + "attn_q.weight", use_f32, &L.wq) ||
        !tensor_f32(f, p + "attn_q.bias", &L.bq) || !load_weight(f, p + "attn_k.weight", use_f32, &L.wk) ||
        !tensor_f32(f, p + "attn_k.bias", &L.bk) || !load_weight(f, p + "attn_v.weight", use_f32, &L.wv) ||
        !tensor_f32(f, p + "attn_v.bias", &L.bv) || !load_weight(f, p + "attn_output.weight", use_f32, &L.wo) ||
        !tensor_f32(f, p + "ffn_norm.weight", &L.ffn_norm) || !load_weight(f, p + "ffn_gate.weight", use_f32, &L.w_gate) ||
        !load_weight(f, p + "ffn_up.weight", use_f32, &L.w_up) || !load_weight(f, p + "ffn_down.weight", use_f32, &L.w_down))
      return false;
    if (L.w_gate.out != c.ffn || L.w_gate.in != c.hidden) {
      set_err("blk.%u ffn_gate is [%zu, %zu], expected [%u, %u]", i, L.w_gate.out, L.w_gate.in, c.ffn, c.hidden);
      return false;
    }
  }
  if (!tensor_f32(f, "output_norm.weight", &m->output_norm)) return false;
  const char* head = f.find("output.weight") ? "output.weight" : "token_embd.weight";
  if (!load_weight(f, head, use_f32, &m->lm_head)) return false;
  if (m->lm_head.out != c.vocab || m->lm_head.in != c.hidden) {
    set_err("lm_head is [%zu, %zu], config says [%u, %u]", m->lm_head.out, m->lm_head.in, c.vocab, c.hidden);
    return false;
  }
  return true;
}

// linear (src/model.rs:169-186)
void linear(const float* x, size_t seq, const Weight& w, const std::vector<float>* bias, float* y) {
  w.matmul(x, seq, y);
  if (bias)
    for (size_t s = 0; s < seq; s++)
      for (size_t o = 0; o < w.out; o++) y[s * w.out + o] += (*bias)[o];
}

// KvCache (src/model.rs:321-363)
struct KvCache {
  std::vector<std::vector<float>> k, v;
  size_t len = 0, max_ctx = 0, kv_dim = 0;
  bool f16 = false;  // elements kept as IEEE binary16 (rounded to nearest even when appended)
};

// binary32 -> binary16, round to nearest even (overflow to infinity,
// gradual underflow); the device's __float2half_rn rounding.
uint16_t float_to_half_rne(float f) {
  uint32_t x;
  memcpy(&x, &f, 4);
  const uint32_t sign = (x >> 16) & 0x8000u, ex = (x >> 23) & 0xFFu;
  uint32_t man = x & 0x7FFFFFu;
  if (ex == 0xFF) return (uint16_t)(sign | 0x7C00u | (man ? 0x200u : 0u));
  const int e = (int)ex - 127 + 15;
  if (e >= 31) return (uint16_t)(sign | 0x7C00u);
  if (e <= 0) {
    if (e < -10) return (uint16_t)sign;
    man |= 0x800000u;
    const uint32_t shift = (uint32_t)(14 - e), rem = man & ((1u << shift) - 1), halfway = 1u << (shift - 1);
    uint32_t h = man >> shift;
    if (rem > halfway || (rem == halfway && (h & 1u))) h++;
    return (uint16_t)(sign | h);
  }
  uint32_t h = ((uint32_t)e << 10) | (man >> 13);
  const uint32_t rem = man & 0x1FFFu;
  if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h++;  // a carry moves to the next binade / infinity
  return (uint16_t)(sign | h);
}

float round_to_half(float f) { return f16_to_f32(float_to_half_rne(f)); }

// attention_scores_cached + softmax + attention_apply_cached
// (src/model.rs:371-438); the uncached variants (:224-290) are the same
// arithmetic with k/v taken from the current rows.
void attention(const float* q, size_t n_new, const float* kc, const float* vc, size_t total, size_t start_pos,
               size_t nh, size_t nkv, size_t hd, float* out) {
  size_t kv_dim = nkv * hd, group = nh / nkv;
  float scale = 1.0f / sqrtf((float)hd);
  std::vector<float> probs(nh * n_new * total);
  memset(out, 0, sizeof(float) * n_new * nh * hd);
  // Heads are independent: one task per head, each running the reference's
  // per-head loops unchanged (scores, softmax row by row, then p * v).  A
  // masked entry's probability is exactly 0 (exp(-inf)); its p * v term
  // (+0 or -0 for finite v) leaves the sum unchanged, so it is skipped.
  pool().parallel_for(nh, [&](size_t h) {
    size_t kv = h / group;
    for (size_t s = 0; s < n_new; s++) {
      const float* qh = q + s * nh * hd + h * hd;
      float* row = probs.data() + (h * n_new + s) * total;
      for (size_t t = 0; t < total; t++) {
        if (t <= start_pos + s) {
          const float* kh = kc + t * kv_dim + kv * hd;
          float d = 0.0f;
          for (size_t i = 0; i < hd; i++) d += qh[i] * kh[i];
          row[t] = d * scale;
        } else {
          row[t] = -INFINITY;
        }
      }
    }
    softmax(probs.data() + h * n_new * total, n_new, total);
    for (size_t s = 0; s < n_new; s++) {
      const float* row = probs.data() + (h * n_new + s) * total;
      float* oh = out + s * nh * hd + h * hd;
      const size_t lim = std::min(total, start_pos + s + 1);
      for (size_t t = 0; t < lim; t++) {
        float p = row[t];
        const float* vh = vc + t * kv_dim + kv * hd;
        for (size_t d = 0; d < hd; d++) oh[d] += p * vh[d];
      }
    }
  });
}

// layer_forward_cached (src/model.rs:444-478).  With cache == nullptr this is
// layer_forward (src/model.rs:294-315): K/V come from the current rows only.
void layer_forward(const float* x, size_t n_new, const Layer& L, const Config& c, KvCache* cache, size_t li,
                   size_t start_pos, float* out) {
  size_t nh = c.n_heads, nkv = c.n_kv_heads, hd = c.head_dim, H = c.hidden, F = c.ffn;
  size_t qd = nh * hd, kd = nkv * hd;
  std::vector<float> xn(n_new * H), q(n_new * qd), k(n_new * kd), v(n_new * kd), ctx(n_new * qd), attn(n_new * H);
  rmsnorm(x, n_new, H, L.attn_norm.data(), c.rms_eps, xn.data());
  linear(xn.data(), n_new, L.wq, &L.bq, q.data());
  linear(xn.data(), n_new, L.wk, &L.bk, k.data());
  linear(xn.data(), n_new, L.wv, &L.bv, v.data());
  rope(q.data(), n_new, nh, hd, c.rope_theta, start_pos);
  rope(k.data(), n_new, nkv, hd, c.rope_theta, start_pos);
  if (cache) {
    if (cache->f16)
      for (size_t i = 0; i < n_new * kd; i++) {
        k[i] = round_to_half(k[i]);
        v[i] = round_to_half(v[i]);
      }
    memcpy(cache->k[li].data() + start_pos * kd, k.data(), sizeof(float) * n_new * kd);
    memcpy(cache->v[li].data() + start_pos * kd, v.data(), sizeof(float) * n_new * kd);
    size_t total = start_pos + n_new;
    attention(q.data(), n_new, cache->k[li].data(), cache->v[li].data(), total, start_pos, nh, nkv, hd, ctx.data());
  } else {
    attention(q.data(), n_new, k.data(), v.data(), n_new, 0, nh, nkv, hd, ctx.data());
  }
  linear(ctx.data(), n_new, L.wo, nullptr, attn.data());
  std::vector<float> h1(n_new * H);
  for (size_t i = 0; i < n_new * H; i++) h1[i] = x[i] + attn[i];
  std::vector<float> hn(n_new * H), gate(n_new * F), up(n_new * F), ffn(n_new * H);
  rmsnorm(h1.data(), n_new, H, L.ffn_norm.data(), c.rms_eps, hn.data());
  linear(hn.data(), n_new, L.w_gate, nullptr, gate.data());
  linear(hn.data(), n_new, L.w_up, nullptr, up.data());
  for (size_t i = 0; i < n_new * F; i++) gate[i] = swiglu1(gate[i], up[i]);
  linear(gate.data(), n_new, L.w_down, nullptr, ffn.data());
  for (size_t i = 0; i < n_new * H; i++) out[i] = h1[i] + ffn[i];
}

// embed (src/model.rs:482-506)
bool embed(const Weight& e, const uint32_t* toks, size_t n, float* out) {
  size_t H = e.in;
  for (size_t s = 0; s < n; s++) {
    size_t t = toks[s];
    if (t >= e.out) { set_err("token id %zu out of range (vocab %zu)", t, e.out); return false; }
    if (e.is_f32) {
      memcpy(out + s * H, e.f.data() + t * H, H * 4);
    } else {
      size_t be, bb;
      block_layout(e.dtype, &be, &bb);
      size_t rb = H / be * bb;
      if (!dequantize(e.dtype, e.raw + t * rb, rb, H, out + s * H)) return false;
    }
  }
  return true;
}

// last_row_logits (src/model.rs:594-600)
void last_row_logits(const Model& m, const float* x, size_t n, float* logits) {
  size_t H = m.cfg.hidden;
  std::vector<float> xn(n * H);
  rmsnorm(x, n, H, m.output_norm.data(), m.cfg.rms_eps, xn.data());
  linear(xn.data() + (n - 1) * H, 1, m.lm_head, nullptr, logits);
}

// Model::forward_cached (src/model.rs:579-592)
bool forward_cached(const Model& m, const uint32_t* toks, size_t n, KvCache* cache, float* logits) {
  size_t start = cache->len;
  if (start + n > cache->max_ctx) { set_err("context overflow: %zu + %zu > max_ctx %zu", start, n, cache->max_ctx); return false; }
  size_t H = m.cfg.hidden;
  std::vector<float> x(n * H), y(n * H);
  if (!embed(m.embedding, toks, n, x.data())) return false;
  for (size_t i = 0; i < m.layers.size(); i++) {
    layer_forward(x.data(), n, m.layers[i], m.cfg, cache, i, start, y.data());
    x.swap(y);
  }
  cache->len += n;
  last_row_logits(m, x.data(), n, logits);
  return true;
}

// Model::forward_last (src/model.rs:569-575), uncached full recompute
bool forward_last(const Model& m, const uint32_t* toks, size_t n, float* logits) {
  size_t H = m.cfg.hidden;
  std::vector<float> x(n * H), y(n * H);
  if (!embed(m.embedding, toks, n, x.data())) return false;
  for (size_t i = 0; i < m.layers.size(); i++) {
    layer_forward(x.data(), n, m.layers[i], m.cfg, nullptr, i, 0, y.data());
    x.swap(y);
  }
  last_row_logits(m, x.data(), n, logits);
  return true;
}

// ---------------------------------------------------------------------------
// Sampler (src/sampler.rs).
// ---------------------------------------------------------------------------
struct Pcg32 {  // src/sampler.rs:6-34
  uint64_t state = 0, inc = (0xda3e39cb94b95bdbull << 1) | 1;
  explicit Pcg32(uint64_t seed) {
    next_u32();
    state += seed;
    next_u32();
  }
  uint32_t next_u32() {
    uint64_t old = state;
    state = old * 6364136223846793005ull + inc;
    uint32_t xs = (uint32_t)(((old >> 18) ^ old) >> 27);
    uint32_t rot = (uint32_t)(old >> 59);
    return (xs >> rot) | (xs << ((32 - rot) & 31));
  }
  float next_f32() { return (float)(next_u32() >> 8) / (float)(1u << 24); }
};

// apply_repeat_penalty (src/sampler.rs:39-55)
void apply_repeat_penalty(float* lg, const uint32_t* recent, size_t nr, float pen) {
  if (pen == 1.0f) return;
  std::vector<uint32_t> seen;
  for (size_t i = 0; i < nr; i++) {
    uint32_t t = recent[i];
    bool dup = false;
    for (auto s : seen) dup |= s == t;
    if (dup) continue;
    seen.push_back(t);
    float& l = lg[t];
    if (l > 0.0f) l /= pen;
    else l *= pen;
  }
}

struct Sampler {  // src/sampler.rs:57-155
  float temperature, top_p, repeat_penalty;
  size_t top_k, repeat_window = 64;
  Pcg32 rng;
  uint64_t draws = 0;
  Sampler(float t, size_t k, float p, float r, uint64_t seed) : temperature(t), top_p(p), repeat_penalty(r), top_k(k), rng(seed) {}

  // Sampler::filtered (src/sampler.rs:113-154)
  std::vector<std::pair<uint32_t, float>> filtered(const float* lg, size_t n) const {
    std::vector<std::pair<uint32_t, float>> c(n);
    for (size_t i = 0; i < n; i++) c[i] = {(uint32_t)i, lg[i] / temperature};
    // The reference partitions with select_nth_unstable then sorts with an
    // unstable sort; ties between equal logits can land in either order.
    // A stable descending sort is one of the orders it may produce, which is
    // what the known-answer tests pin.
    std::stable_sort(c.begin(), c.end(), [](const auto& a, const auto& b) { return a.second > b.second; });
    if (top_k > 0 && top_k < c.size()) c.resize(top_k);
    float mx = c[0].second, sum = 0.0f;
    for (auto& e : c) {
      e.second = expf(e.second - mx);
      sum += e.second;
    }
    for (auto& e : c) e.second /= sum;
    if (top_p < 1.0f) {
      float cum = 0.0f;
      size_t keep = c.size();
      for (size_t i = 0; i < c.size(); i++) {
        cum += c[i].second;
        if (cum >= top_p) {
          keep = i + 1;
          break;
        }
      }
      c.resize(keep);
      float s = 0.0f;
      for (auto& e : c) s += e.second;
      for (auto& e : c) e.second /= s;
    }
    return c;
  }

  // Sampler::sample (src/sampler.rs:86-108)
  uint32_t sample(const float* logits, size_t n, const uint32_t* recent, size_t nr) {
    std::vector<float> lg(logits, logits + n);
    apply_repeat_penalty(lg.data(), recent, nr, this->repeat_penalty);
    if (temperature == 0.0f || top_k == 1) return argmax(lg.data(), n);
    auto cand = filtered(lg.data(), n);
    float u = rng.next_f32();
    draws++;
    float cum = 0.0f;
    for (auto& e : cand) {
      cum += e.second;
      if (u < cum) return e.first;
    }
    return cand.back().first;
  }
};

}  // namespace

// ===========================================================================
// C API used by the tests (ctypes) and bench.py's CPU-baseline leg.
// ===========================================================================
extern "C" {

const char* orc_last_error() { return g_err.c_str(); }

void orc_set_threads(int n) { pool().resize(n); }
int orc_threads() { return pool().size(); }

float orc_f16_to_f32(uint16_t h) { return f16_to_f32(h); }

int orc_dequantize(uint32_t dtype, const uint8_t* raw, size_t nbytes, size_t n, float* out) {
  return dequantize(dtype, raw, nbytes, n, out) ? 0 : 1;
}

int orc_matmul_quant(const float* a, size_t seq, const uint8_t* raw, size_t nbytes, size_t d_out, size_t d_in,
                     uint32_t dtype, float* out) {
  return matmul_quant(a, seq, raw, nbytes, d_out, d_in, dtype, out) ? 0 : 1;
}

void orc_matmul_f32(const float* a, size_t seq, const float* w, size_t d_out, size_t d_in, float* out) {
  matmul_f32(a, seq, w, d_out, d_in, out);
}

float orc_dot(const float* a, const float* b, size_t n) { return dot8(a, b, n); }

void orc_rmsnorm(const float* x, size_t rows, size_t cols, const float* w, float eps, float* out) {
  rmsnorm(x, rows, cols, w, eps, out);
}

void orc_softmax(float* x, size_t rows, size_t cols) { softmax(x, rows, cols); }

void orc_silu(const float* x, size_t n, float* out) {
  for (size_t i = 0; i < n; i++) out[i] = silu1(x[i]);
}

void orc_swiglu(const float* g, const float* u, size_t n, float* out) {
  for (size_t i = 0; i < n; i++) out[i] = swiglu1(g[i], u[i]);
}

void orc_rope(float* x, size_t seq, size_t n_heads, size_t hd, float theta, size_t start_pos) {
  rope(x, seq, n_heads, hd, theta, start_pos);
}

// Uncached attention over `seq` rows (src/model.rs:224-290).
void orc_attention(const float* q, const float* k, const float* v, size_t seq, size_t nh, size_t nkv, size_t hd,
                   float* out) {
  attention(q, seq, k, v, seq, 0, nh, nkv, hd, out);
}

uint32_t orc_argmax(const float* d, size_t n) { return argmax(d, n); }

// --- GGUF file -------------------------------------------------------------
void* orc_gguf_open(const char* path) {
  int fd = open(path, O_RDONLY);
  if (fd < 0) { set_err("cannot open %s", path); return nullptr; }
  struct stat st;
  fstat(fd, &st);
  File* f = new File();
  f->size = (size_t)st.st_size;
  if (f->size) {
    void* p = mmap(nullptr, f->size, PROT_READ, MAP_PRIVATE, fd, 0);
    if (p == MAP_FAILED) { close(fd); delete f; set_err("mmap failed for %s", path); return nullptr; }
    f->map = (uint8_t*)p;
  }
  close(fd);
  if (!parse(f->map, f->size, f)) { delete f; return nullptr; }
  return f;
}

int orc_gguf_parse_bytes(const uint8_t* data, size_t n, uint32_t* version, size_t* n_tensors, size_t* n_meta,
                         size_t* data_start) {
  File f;
  if (!parse(data, n, &f)) return 1;
  *version = f.version;
  *n_tensors = f.tensors.size();
  *n_meta = f.meta.size();
  *data_start = f.data_start;
  return 0;
}

void orc_gguf_close(void* f) { delete (File*)f; }

// --- Model -----------------------------------------------------------------
void* orc_model_open(const char* path, int use_f32) {
  Model* m = new Model();
  int fd = open(path, O_RDONLY);
  if (fd < 0) { set_err("cannot open %s", path); delete m; return nullptr; }
  struct stat st;
  fstat(fd, &st);
  m->file.size = (size_t)st.st_size;
  void* p = mmap(nullptr, m->file.size, PROT_READ, MAP_PRIVATE, fd, 0);
  close(fd);
  if (p == MAP_FAILED) { set_err("mmap failed"); delete m; return nullptr; }
  m->file.map = (uint8_t*)p;
  if (!parse(m->file.map, m->file.size, &m->file) || !model_load(m, use_f32 != 0)) {
    delete m;
    return nullptr;
  }
  return m;
}

void orc_model_close(void* m) { delete (Model*)m; }

// n_layers, n_heads, n_kv_heads, hidden, ffn, head_dim, vocab, context_length
void orc_model_config(void* mp, uint32_t* u, float* f) {
  Model* m = (Model*)mp;
  const Config& c = m->cfg;
  u[0] = c.n_layers; u[1] = c.n_heads; u[2] = c.n_kv_heads; u[3] = c.hidden;
  u[4] = c.ffn; u[5] = c.head_dim; u[6] = c.vocab; u[7] = c.context_length;
  f[0] = c.rope_theta;
  f[1] = c.rms_eps;
}

// Restrict the model to its first n layers (layer-truncated parity variants).
void orc_model_truncate(void* mp, uint32_t n) {
  Model* m = (Model*)mp;
  if (n < m->layers.size()) {
    m->layers.resize(n);
    m->cfg.n_layers = n;
  }
}

void* orc_kv_new(void* mp, size_t max_ctx) {
  Model* m = (Model*)mp;
  KvCache* kv = new KvCache();
  kv->kv_dim = (size_t)m->cfg.n_kv_heads * m->cfg.head_dim;
  kv->max_ctx = max_ctx;
  kv->k.assign(m->cfg.n_layers, std::vector<float>(max_ctx * kv->kv_dim, 0.0f));
  kv->v.assign(m->cfg.n_layers, std::vector<float>(max_ctx * kv->kv_dim, 0.0f));
  return kv;
}
void orc_kv_free(void* kv) { delete (KvCache*)kv; }
void orc_kv_set_f16(void* kv, int on) { ((KvCache*)kv)->f16 = on != 0; }
uint16_t orc_float_to_half(float f) { return float_to_half_rne(f); }
size_t orc_kv_len(void* kv) { return ((KvCache*)kv)->len; }
void orc_kv_set_len(void* kv, size_t n) { ((KvCache*)kv)->len = n; }

// Read back layer `li`'s cached K (or V) rows [0, n) as [n, kv_dim].
int orc_kv_read(void* kvp, size_t li, int which_v, size_t n, float* out) {
  KvCache* kv = (KvCache*)kvp;
  if (li >= kv->k.size() || n > kv->max_ctx) { set_err("kv read out of range"); return 1; }
  const auto& src = which_v ? kv->v[li] : kv->k[li];
  memcpy(out, src.data(), sizeof(float) * n * kv->kv_dim);
  return 0;
}

// Overwrite layer `li`'s cached K (or V) rows [0, n) from [n, kv_dim] (the
// timed CPU baseline fills a long context with synthetic rows: the cost of
// a decode step does not depend on the cached values).
int orc_kv_write(void* kvp, size_t li, int which_v, size_t n, const float* in) {
  KvCache* kv = (KvCache*)kvp;
  if (li >= kv->k.size() || n > kv->max_ctx) { set_err("kv write out of range"); return 1; }
  auto& dst = which_v ? kv->v[li] : kv->k[li];
  memcpy(dst.data(), in, sizeof(float) * n * kv->kv_dim);
  return 0;
}

int orc_forward_cached(void* mp, void* kv, const uint32_t* toks, size_t n, float* logits) {
  if (n == 0) { set_err("forward with no tokens"); return 1; }
  return forward_cached(*(Model*)mp, toks, n, (KvCache*)kv, logits) ? 0 : 1;
}

int orc_forward_last(void* mp, const uint32_t* toks, size_t n, float* logits) {
  if (n == 0) { set_err("forward with no tokens"); return 1; }
  return forward_last(*(Model*)mp, toks, n, logits) ? 0 : 1;
}

// Embedding row dequantized exactly as embed() does.
int orc_embed(void* mp, const uint32_t* toks, size_t n, float* out) {
  return embed(((Model*)mp)->embedding, toks, n, out) ? 0 : 1;
}

// One layer_forward_cached call against layer li (staged parity checks).
int orc_layer_forward(void* mp, void* kvp, size_t li, const float* x, size_t n, size_t start_pos, float* out) {
  Model* m = (Model*)mp;
  if (li >= m->layers.size()) { set_err("layer %zu out of range", li); return 1; }
  layer_forward(x, n, m->layers[li], m->cfg, (KvCache*)kvp, li, start_pos, out);
  return 0;
}

// Tensor lookup: dtype, dims (ggml order), raw pointer into the map.
int orc_tensor(void* mp, const char* name, uint32_t* dtype, uint64_t* dims, uint32_t* n_dims, const uint8_t** raw,
               size_t* nbytes) {
  Model* m = (Model*)mp;
  const TensorInfo* info;
  if (!m->file.tensor(name, &info, raw, nbytes)) return 1;
  *dtype = info->dtype;
  *n_dims = (uint32_t)info->dims.size();
  for (size_t i = 0; i < info->dims.size(); i++) dims[i] = info->dims[i];
  return 0;
}

// --- Sampler ---------------------------------------------------------------
void* orc_sampler_new(float temp, size_t top_k, float top_p, float rep, uint64_t seed) {
  return new Sampler(temp, top_k, top_p, rep, seed);
}
void orc_sampler_free(void* s) { delete (Sampler*)s; }
uint32_t orc_sampler_sample(void* s, const float* logits, size_t n, const uint32_t* recent, size_t nr) {
  return ((Sampler*)s)->sample(logits, n, recent, nr);
}
uint64_t orc_sampler_draws(void* s) { return ((Sampler*)s)->draws; }
size_t orc_sampler_filtered(void* s, const float* logits, size_t n, uint32_t* ids, float* probs) {
  auto c = ((Sampler*)s)->filtered(logits, n);
  for (size_t i = 0; i < c.size(); i++) {
    ids[i] = c[i].first;
    probs[i] = c[i].second;
  }
  return c.size();
}
void orc_repeat_penalty(float* lg, const uint32_t* recent, size_t nr, float pen) { apply_repeat_penalty(lg, recent, nr, pen); }

// generate (src/generate.rs:83-157) without text streaming: prefill once,
// then sample/decode.  Returns the number of generated ids.  When
// step_logits is non-null, the logits each sample was drawn from are stored
// row by row (row 0 = prefill logits).  prefill_s / decode_s receive the
// wall-clock seconds of the prefill and of all decode forwards.
int orc_generate(void* mp, const uint32_t* prompt, size_t n_prompt, size_t max_new, const uint32_t* stop_ids,
                 size_t n_stop, void* sp, size_t max_ctx, uint32_t* out_ids, size_t* n_out, float* step_logits,
                 double* prefill_s, double* decode_s) {
  Model* m = (Model*)mp;
  Sampler* s = (Sampler*)sp;
  if (n_prompt + max_new > max_ctx) {
    set_err("prompt (%zu) + max tokens (%zu) exceeds context cap %zu", n_prompt, max_new, max_ctx);
    return 1;
  }
  void* kv = orc_kv_new(mp, max_ctx);
  size_t V = m->cfg.vocab;
  std::vector<float> logits(V);
  std::vector<uint32_t> context(prompt, prompt + n_prompt);
  auto now = [] {
    struct timespec ts;
    clock_gettime(CLOCK_MONOTONIC, &ts);
    return ts.tv_sec + ts.tv_nsec * 1e-9;
  };
  double t0 = now();
  if (!forward_cached(*m, prompt, n_prompt, (KvCache*)kv, logits.data())) { orc_kv_free(kv); return 1; }
  if (prefill_s) *prefill_s = now() - t0;
  double dsec = 0;
  size_t ng = 0;
  for (size_t step = 0; step < max_new; step++) {
    if (step_logits) memcpy(step_logits + step * V, logits.data(), V * 4);
    size_t window = context.size() > s->repeat_window ? context.size() - s->repeat_window : 0;
    uint32_t next = s->sample(logits.data(), V, context.data() + window, context.size() - window);
    bool stop = false;
    for (size_t i = 0; i < n_stop; i++) stop |= stop_ids[i] == next;
    if (stop) break;
    out_ids[ng++] = next;
    context.push_back(next);
    if (step + 1 == max_new) break;
    double t1 = now();
    if (!forward_cached(*m, &next, 1, (KvCache*)kv, logits.data())) { orc_kv_free(kv); return 1; }
    dsec += now() - t1;
  }
  if (decode_s) *decode_s = dsec;
  *n_out = ng;
  orc_kv_free(kv);
  return 0;
}

}  // extern "C"
