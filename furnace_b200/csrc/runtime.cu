// Host runtime: model upload (Model::load, src/model.rs:520-552), device KV
// cache (src/model.rs:321-363), the decode step as one captured CUDA graph,
// and the C ABI declared in include/furnace.h.

#include <cuda_runtime.h>

#include <chrono>
#include <thread>

#include <algorithm>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <memory>
#include <string>
#include <vector>

#include "fz_internal.h"
#include "kernels.h"
#include "nccl_dyn.h"

namespace fz {
const std::string& last_error();
}

using namespace fz;

#define CK(x)                                                                               \
  do {                                                                                      \
    cudaError_t e_ = (x);                                                                   \
    if (e_ != cudaSuccess) fail(FZ_ECUDA, "%s failed: %s", #x, cudaGetErrorString(e_));     \
  } while (0)

namespace {

// Device allocation that frees itself.
struct DevBuf {
  void* p = nullptr;
  size_t n = 0;
  DevBuf() = default;
  explicit DevBuf(size_t bytes) { alloc(bytes); }
  void alloc(size_t bytes) {
    release();
    if (bytes == 0) bytes = 16;
    cudaError_t e = cudaMalloc(&p, bytes);
    if (e != cudaSuccess) {
      p = nullptr;
      cudaGetLastError();
      fail(FZ_ENOMEM, "cudaMalloc(%zu) failed: %s", bytes, cudaGetErrorString(e));
    }
    n = bytes;
  }
  void release() {
    if (p) cudaFree(p);
    p = nullptr;
    n = 0;
  }
  ~DevBuf() { release(); }
  DevBuf(const DevBuf&) = delete;
  DevBuf& operator=(const DevBuf&) = delete;
  template <class T>
  T* as() const {
    return reinterpret_cast<T*>(p);
  }
};

struct Layer {
  float *attn_norm, *ffn_norm, *bqkv;  // bqkv = [bq | bk | bv]
  DevMat wq, wk, wv, wo, wgu, wd;      // wgu: gate/up rows interleaved
};

}  // namespace

struct fz_model {
  fz_config cfg{};
  int device = 0;
  cudaStream_t stream = nullptr;
  DevBuf weights;         // every quantized matrix
  DevBuf smalls;          // norms and biases (f32)
  DevMat embd, lm_head;
  float* out_norm = nullptr;
  std::vector<Layer> layers;
  uint64_t resident = 0, streamed = 0;
  // activations (f32) and the run records GEMVs read (see kernels.cu)
  DevBuf x, qkv, ctx, h, logits;
  DevBuf runs_h;  // ffn hidden as run records
  // attention output as run records, one buffer per distinct o_off value:
  // the layers sharing a buffer write the same records, so the records of
  // o_proj's padding columns are never written and stay zero
  std::vector<std::unique_ptr<DevBuf>> runs_ctx;
  std::vector<uint32_t> ctx_buf;  // per layer: index into runs_ctx
  DevBuf trace;             // decode-step timeline (FURNACE_B200_TRACE=<file>)
  std::string trace_path;
  // tensor parallelism: this rank's share (world == 1: everything)
  int rank = 0, world = 1;
  ncclComm_t comm = nullptr;
  // residual exchange through peer memory: this rank's receive buffer
  // (exported by CUDA IPC), the peers' buffers as mapped here, the epoch base
  DevBuf ar_buf, ar_base;
  ArPeers ar_peers{};
  bool ar_p2p = false;
  fz_tp_slice sl{};
  uint32_t nh_l = 0, nkv_l = 0, qd_l = 0, kd_l = 0;
  std::vector<uint32_t> o_off;  // per layer: ctx[0]'s column within o_proj's block-aligned input
  uint32_t o_w = 0;             // widest o_proj input (run records of ctx cover it)
  // batched prefill (tensor cores): activations of up to pf_cap tokens, the
  // fp16 hi/lo panels of one weight and of one activation matrix
  uint32_t pf_cap = 0;
  DevBuf pf_x, pf_qkv, pf_ctx, pf_h, pf_tok, pf_err, pf_wh, pf_wl, pf_xh, pf_xl;
  DevBuf pf_rexp, pf_texp;  // power-of-two exponents of the panel rows / token rows
  DevBuf smp_scratch, smp_out;  // device top-k of the sampler
  // the caches made for this model: fz_model_free releases their device
  // memory and detaches them, so they may be freed before or after it
  std::vector<fz_kv*> caches;
};

struct fz_kv {
  fz_model* m = nullptr;
  uint32_t max_ctx = 0, len = 0, splits = 0;
  uint32_t eb = 4;  // bytes per cached element: 4 (f32) or 2 (f16)
  // layer li's K (or V) block [nkv_l][max_ctx][hd] of this rank
  void* layer_k(uint32_t li, uint32_t nkv, uint32_t hd) const {
    return k.as<uint8_t>() + (uint64_t)li * nkv * max_ctx * hd * eb;
  }
  void* layer_v(uint32_t li, uint32_t nkv, uint32_t hd) const {
    return v.as<uint8_t>() + (uint64_t)li * nkv * max_ctx * hd * eb;
  }
  DevBuf k, v, rope_cs, partials, state, forced, ids;
  cudaGraphExec_t g_full = nullptr, g_layers = nullptr;
  // device memory and graphs back; the handle stays valid for fz_kv_free
  void release() {
    if (g_full) cudaGraphExecDestroy(g_full);
    if (g_layers) cudaGraphExecDestroy(g_layers);
    g_full = g_layers = nullptr;
    for (DevBuf* b : {&k, &v, &rope_cs, &partials, &state, &forced, &ids}) b->release();
  }
  ~fz_kv() { release(); }
};

struct fz_weight {
  DevBuf buf, runs;
  DevMat m;
};

// Sampler (src/sampler.rs:57-155) with its PCG32 stream (src/sampler.rs:6-34).
struct fz_sampler {
  float temperature = 0.f, top_p = 1.f, repeat_penalty = 1.f;
  uint32_t top_k = 0;
  uint64_t state = 0, inc = (0xda3e39cb94b95bdbull << 1) | 1;
  uint64_t draws = 0;
  uint32_t next_u32() {
    const uint64_t old = state;
    state = old * 6364136223846793005ull + inc;
    const uint32_t xs = (uint32_t)(((old >> 18) ^ old) >> 27), rot = (uint32_t)(old >> 59);
    return (xs >> rot) | (xs << ((32 - rot) & 31));
  }
  float next_f32() { return (float)(next_u32() >> 8) / (float)(1u << 24); }
  bool greedy() const { return temperature == 0.0f || top_k == 1; }
};

namespace {

uint64_t gguf_bytes(uint32_t dtype, uint64_t rows, uint32_t cols) {
  uint32_t be, bb;
  block_geom(dtype, &be, &bb);
  return rows * (cols / be) * bb;
}

// Host-to-device weight upload through two pinned host buffers and two device
// staging buffers: while the GPU copies one chunk and repacks it into the
// device layout, host threads gather the next chunk from the (memory-mapped)
// GGUF bytes into the other pinned buffer.
struct Uploader {
  cudaStream_t s;
  size_t cap;
  uint8_t* host[2] = {nullptr, nullptr};
  DevBuf dev[2];
  cudaEvent_t ev[2] = {nullptr, nullptr};
  bool busy[2] = {false, false};
  int cur = 0;
  unsigned nthreads;

  Uploader(cudaStream_t st, size_t c) : s(st), cap(c) {
    nthreads = std::max(1u, std::min(16u, std::thread::hardware_concurrency()));
    for (int i = 0; i < 2; i++) {
      CK(cudaMallocHost(&host[i], cap));
      dev[i].alloc(cap);
      CK(cudaEventCreateWithFlags(&ev[i], cudaEventDisableTiming));
    }
  }
  ~Uploader() {
    cudaStreamSynchronize(s);
    for (int i = 0; i < 2; i++) {
      if (host[i]) cudaFreeHost(host[i]);
      if (ev[i]) cudaEventDestroy(ev[i]);
    }
  }
  Uploader(const Uploader&) = delete;
  Uploader& operator=(const Uploader&) = delete;

  // Pack `segs` (host source, bytes) back to back into the free pinned
  // buffer, copy it to the device and run post(device pointer) on the
  // stream.  The segments' bytes must total at most cap.
  template <class Post>
  void push(const std::vector<std::pair<const uint8_t*, size_t>>& segs, Post post) {
    if (busy[cur]) CK(cudaEventSynchronize(ev[cur]));
    size_t total = 0;
    for (auto& g : segs) total += g.second;
    need(total <= cap, "upload chunk of %zu bytes exceeds the staging buffer", total);
    // split the bytes evenly over the threads, each copying its byte range
    // across segment boundaries
    uint8_t* dst = host[cur];
    auto work = [&](size_t b0, size_t b1) {
      size_t off = 0;
      for (auto& g : segs) {
        const size_t a = std::max(b0, off), e = std::min(b1, off + g.second);
        if (a < e) memcpy(dst + a, g.first + (a - off), e - a);
        off += g.second;
        if (off >= b1) break;
      }
    };
    const unsigned T = total >= (4u << 20) ? nthreads : 1u;
    std::vector<std::thread> th;
    for (unsigned t = 1; t < T; t++) th.emplace_back(work, total * t / T, total * (t + 1) / T);
    work(0, total / T);
    for (auto& x : th) x.join();
    CK(cudaMemcpyAsync(dev[cur].p, host[cur], total, cudaMemcpyHostToDevice, s));
    post(dev[cur].as<uint8_t>());
    CK(cudaEventRecord(ev[cur], s));
    busy[cur] = true;
    cur ^= 1;
  }
  void finish() { CK(cudaStreamSynchronize(s)); }
};

// Upload `rows` GGUF rows of a [rows, cols] weight (raw host bytes) into the
// device layout at dst.
void upload_rows(uint32_t dtype, const uint8_t* raw, uint64_t rows, uint32_t cols, uint8_t* dst, Uploader& up) {
  const uint64_t row_raw = gguf_bytes(dtype, 1, cols);
  const uint64_t chunk_rows = up.cap / row_raw;
  need(chunk_rows > 0, "staging buffer too small");
  for (uint64_t r0 = 0; r0 < rows; r0 += chunk_rows) {
    const uint64_t nr = std::min(chunk_rows, rows - r0);
    up.push({{raw + r0 * row_raw, nr * row_raw}}, [&](const uint8_t* d) {
      launch_repack(dtype, d, dst, (uint32_t)r0, (uint32_t)nr, (uint32_t)rows, cols, up.s);
    });
  }
}

// This rank's share of the model (see fz_tp_slice in include/furnace.h).
fz_tp_slice tp_slice(const fz_config& c, int r, int T) {
  need(T >= 1 && r >= 0 && r < T, "rank %d of %d", r, T);
  need(c.n_heads % T == 0 && c.n_kv_heads % T == 0, "%u heads / %u KV heads do not split over %d ranks", c.n_heads,
       c.n_kv_heads, T);
  fz_tp_slice s{};
  s.q_heads = c.n_heads / T;
  s.q_head0 = r * s.q_heads;
  s.kv_heads = c.n_kv_heads / T;
  s.kv_head0 = r * s.kv_heads;
  s.o_col0 = s.q_head0 * c.head_dim;
  s.o_cols = s.q_heads * c.head_dim;
  const uint32_t U = (c.ffn + 255) / 256;  // FFN slices on 256-element boundaries
  s.ffn0 = std::min(c.ffn, (uint32_t)((uint64_t)r * U / T) * 256);
  const uint32_t f1 = r + 1 == T ? c.ffn : std::min(c.ffn, (uint32_t)((uint64_t)(r + 1) * U / T) * 256);
  need(f1 > s.ffn0, "FFN %u too small for %d ranks", c.ffn, T);
  s.ffn_n = f1 - s.ffn0;
  const uint32_t vs = (c.vocab + T - 1) / T;
  s.vocab_pad = vs * T;
  s.vocab0 = r * vs;
  s.vocab_n = std::min(vs, c.vocab - std::min(c.vocab, s.vocab0));
  return s;
}

void nccl_check(ncclResult_t r, const char* what) {
  if (r != ncclSuccess) fail(FZ_ECUDA, "%s failed: %s", what, nccl().GetErrorString(r));
}

// Seconds a communicator call may make no progress (a peer that never joins,
// or stops taking part) before the communicator is aborted and the call
// fails with FZ_ETIMEOUT: FURNACE_B200_NCCL_TIMEOUT_S, default 300.
double nccl_timeout_s() {
  const char* e = getenv("FURNACE_B200_NCCL_TIMEOUT_S");
  const double v = e ? atof(e) : 0.0;
  return v > 0 ? v : 300.0;
}

// The result of a call on a (possibly non-blocking) communicator: while it
// reports ncclInProgress, poll ncclCommGetAsyncError; past the time limit,
// ncclCommAbort it (*comm becomes null) and fail with FZ_ETIMEOUT.
void nccl_comm_check(ncclComm_t* comm, ncclResult_t r, const char* what) {
  if (r == ncclInProgress && nccl().CommGetAsyncError) {
    const auto t0 = std::chrono::steady_clock::now();
    const double lim = nccl_timeout_s();
    for (;;) {
      ncclResult_t st = ncclSuccess;
      const ncclResult_t q = nccl().CommGetAsyncError(*comm, &st);
      if (q != ncclSuccess) {
        r = q;
        break;
      }
      if (st != ncclInProgress) {
        r = st;
        break;
      }
      if (std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count() > lim) {
        nccl().CommAbort(*comm);
        *comm = nullptr;
        fail(FZ_ETIMEOUT, "%s: no progress within %.0f s (a peer did not take part); communicator aborted", what,
             lim);
      }
      std::this_thread::sleep_for(std::chrono::microseconds(200));
    }
  }
  if (r != ncclSuccess) fail(FZ_ECUDA, "%s failed: %s", what, nccl().GetErrorString(r));
}

// Upload rows [0, rows) restricted to input columns [col0, col0 + ncols)
// (block-aligned) of a [rows, cols] GGUF weight: rows are gathered on the host.
void upload_cols(uint32_t dtype, const uint8_t* raw, uint64_t rows, uint32_t cols, uint32_t col0, uint32_t ncols,
                 uint8_t* dst, Uploader& up) {
  uint32_t be, bb;
  block_geom(dtype, &be, &bb);
  need(col0 % be == 0 && ncols % be == 0 && col0 + ncols <= cols, "column slice not block-aligned");
  const uint64_t row_raw = gguf_bytes(dtype, 1, cols), sl_raw = gguf_bytes(dtype, 1, ncols);
  const uint64_t off = (uint64_t)(col0 / be) * bb;
  const uint64_t chunk_rows = std::max<uint64_t>(1, up.cap / sl_raw);
  for (uint64_t r0 = 0; r0 < rows; r0 += chunk_rows) {
    const uint64_t nr = std::min(chunk_rows, rows - r0);
    std::vector<std::pair<const uint8_t*, size_t>> segs(nr);
    for (uint64_t r = 0; r < nr; r++) segs[r] = {raw + (r0 + r) * row_raw + off, sl_raw};
    up.push(segs, [&](const uint8_t* d) {
      launch_repack(dtype, d, dst, (uint32_t)r0, (uint32_t)nr, (uint32_t)rows, ncols, up.s);
    });
  }
}

const TensorEntry& tensor2d(const GgufFile& f, const std::string& name, uint64_t out, uint64_t in) {
  const TensorEntry* t = f.find(name);
  if (!t) fail(FZ_EFORMAT, "no tensor named '%s'", name.c_str());
  if (t->dims.size() != 2) fail(FZ_EFORMAT, "weight '%s' is not 2-D", name.c_str());
  if (t->dims[1] != out || t->dims[0] != in)
    fail(FZ_EFORMAT, "weight '%s' is [%llu, %llu], expected [%llu, %llu]", name.c_str(), (unsigned long long)t->dims[1],
         (unsigned long long)t->dims[0], (unsigned long long)out, (unsigned long long)in);
  if (!is_quant(t->dtype))
    fail(FZ_EFORMAT, "weight '%s' has dtype %u; the device path needs Q8_0, Q5_0, Q4_K or Q6_K", name.c_str(), t->dtype);
  return *t;
}

// f32 vector (norm or bias) of n elements, dequantized on the host if needed.
std::vector<float> vec_f32(const GgufFile& f, const std::string& name, uint64_t n) {
  const TensorEntry* t = f.find(name);
  if (!t) fail(FZ_EFORMAT, "no tensor named '%s'", name.c_str());
  if (t->n_elements() != n) fail(FZ_EFORMAT, "tensor '%s' has %llu elements, expected %llu", name.c_str(),
                                 (unsigned long long)t->n_elements(), (unsigned long long)n);
  uint64_t nb;
  const uint8_t* d = f.tensor_data(*t, &nb);
  if (t->dtype != FZ_F32) fail(FZ_EFORMAT, "tensor '%s' must be F32 (got dtype %u)", name.c_str(), t->dtype);
  std::vector<float> v(n);
  memcpy(v.data(), d, n * 4);
  return v;
}

void build_graphs(fz_kv* kv);

// Optional per-launch instrumentation (fz_step_profile): called with the op
// kind before (begin = true) and after each launch.
struct OpHook {
  virtual void at(int op, bool begin) = 0;
  virtual ~OpHook() = default;
};

// One decode step: embed -> layers -> [norm + lm_head + argmax] -> finalize.
// Every GEMV reads run records written by its predecessor's epilogue; RMSNorm
// inputs are x (.) w with 1/rms from the predecessor's sum-of-squares partials.
// The GEMV launches of one step in execution order: qkv, o_proj, gate_up,
// down per layer (src/model.rs:444-478), then lm_head (src/model.rs:594-600).
std::vector<GemvLaunch> step_gemvs(fz_kv* kv) {
  fz_model* m = kv->m;
  const fz_config& c = m->cfg;
  StepState* st = kv->state.as<StepState>();
  const uint32_t qd = m->qd_l, kd = m->kd_l;  // this rank's q / k widths
  // tensor parallelism: o_proj and down partial sums of ranks > 0 overwrite
  // x, rank 0 adds its partial to x, and the all-reduce that follows sums them
  const bool xch = m->world > 1 && m->ar_p2p;  // exchange through peer memory
  const int resid = m->rank == 0 || xch ? EPI_RESID : EPI_STORE;
  float* x = m->x.as<float>();
  float* qkv = m->qkv.as<float>();
  std::vector<GemvLaunch> gl(4 * c.n_layers + 1);
  // exchange k of the step: pushed by o_proj (2 li) and down (2 li + 1),
  // pulled by the next RMS-normalised GEMV
  auto ar = [&](GemvLaunch& g, uint32_t k, bool push) {
    if (!xch) return;
    g.ar_peers = m->ar_peers;
    g.ar_w = m->world;
    g.ar_rank = m->rank;
    g.ar_k = k;
    g.ar_h = c.hidden;
    g.ar_base = m->ar_base.as<uint32_t>();
    (push ? g.ar_push : g.ar_pull) = 1;
  };
  for (uint32_t li = 0; li < c.n_layers; li++) {
    Layer& L = m->layers[li];
    GemvLaunch& g = gl[4 * li];
    g.nseg = 3;
    g.seg[0] = GemvSeg{L.wq, L.bqkv, qkv};
    g.seg[1] = GemvSeg{L.wk, L.bqkv + qd, qkv + qd};
    g.seg[2] = GemvSeg{L.wv, L.bqkv + qd + kd, qkv + qd + kd};
    g.x = x;
    g.norm_w = L.attn_norm;
    g.eps = c.rms_eps;
    g.epilogue = EPI_STORE;
    GemvLaunch& go = gl[4 * li + 1];
    go.seg[0] = GemvSeg{L.wo, nullptr, x};
    go.in_runs = m->runs_ctx[m->ctx_buf[li]]->p;
    go.epilogue = resid;
    GemvLaunch& gu = gl[4 * li + 2];
    gu.seg[0] = GemvSeg{L.wgu, nullptr, nullptr};
    gu.x = x;
    gu.norm_w = L.ffn_norm;
    gu.eps = c.rms_eps;
    gu.epilogue = EPI_SWIGLU;
    gu.out_runs = m->runs_h.p;
    GemvLaunch& gd = gl[4 * li + 3];
    gd.seg[0] = GemvSeg{L.wd, nullptr, x};
    gd.in_runs = m->runs_h.p;
    gd.epilogue = resid;
    if (li > 0) ar(g, 2 * li - 1, false);
    ar(go, 2 * li, true);
    ar(gu, 2 * li, false);
    ar(gd, 2 * li + 1, true);
    for (GemvLaunch* p : {&g, &go, &gu, &gd}) p->state = st;
  }
  GemvLaunch& lm = gl[4 * c.n_layers];
  lm.seg[0] = GemvSeg{m->lm_head, nullptr, m->logits.as<float>() + m->sl.vocab0};
  lm.idx_base = m->sl.vocab0;
  lm.x = x;
  lm.norm_w = m->out_norm;
  lm.eps = c.rms_eps;
  lm.epilogue = EPI_LOGITS;
  lm.state = st;
  ar(lm, 2 * c.n_layers - 1, false);
  return gl;
}

AttnLaunch layer_attention(fz_kv* kv, uint32_t li, uint32_t splits) {
  fz_model* m = kv->m;
  const fz_config& c = m->cfg;
  const uint32_t hd = c.head_dim;
  AttnLaunch a{m->qkv.as<float>(), kv->rope_cs.as<float>(), kv->layer_k(li, m->nkv_l, hd),
               kv->layer_v(li, m->nkv_l, hd), m->ctx.as<float>(), m->runs_ctx[m->ctx_buf[li]]->p, kv->partials.as<float>(), m->nh_l,
               m->nkv_l, hd, kv->max_ctx, splits, kv->state.as<StepState>()};
  a.ctx_run0 = m->o_off[li] / 16;
  a.kv_f16 = kv->eb == 2;
  return a;
}

// Sum of the ranks' residual-stream partials (tensor parallelism) where the
// peer-memory exchange inside the GEMVs is unavailable (a rank could not
// export its buffer, or FURNACE_B200_TP_ALLREDUCE=nccl): ncclAllReduce.
void tp_allreduce_x(fz_model* m, cudaStream_t s) {
  if (m->world == 1 || m->ar_p2p) return;
  nccl_comm_check(&m->comm, nccl().AllReduce(m->x.p, m->x.p, m->cfg.hidden, ncclFloat32, ncclSum, m->comm, s),
                  "ncclAllReduce");
}

// One step as separate kernels (programmatic dependent launches): the path
// of fz_step_profile, whose per-kernel events time each op.
void record_step(fz_kv* kv, bool with_logits, cudaStream_t s, OpHook* hook = nullptr) {
  auto H = [&](int op, bool b) {
    if (hook) hook->at(op, b);
  };
  fz_model* m = kv->m;
  const fz_config& c = m->cfg;
  StepState* st = kv->state.as<StepState>();
  float* x = m->x.as<float>();
  std::vector<GemvLaunch> gl = step_gemvs(kv);
  GemvLaunch& lm = gl[4 * c.n_layers];
  size_t last = with_logits ? gl.size() - 1 : gl.size() - 2;
  for (size_t i = 0; i <= last; i++) gl[i].next = i < last ? &gl[i + 1] : &gl[0];

  H(FZ_OP_EMBED, true);
  launch_embed(m->embd, st, x, s);
  H(FZ_OP_EMBED, false);
  for (uint32_t li = 0; li < c.n_layers; li++) {
    H(FZ_OP_QKV, true);
    launch_gemv(gl[4 * li], s);
    H(FZ_OP_QKV, false);
    AttnLaunch a = layer_attention(kv, li, kv->splits);
    H(FZ_OP_ATTN, true);
    launch_attention(a, s);
    H(FZ_OP_ATTN, false);
    H(FZ_OP_OPROJ, true);
    launch_gemv(gl[4 * li + 1], s);
    tp_allreduce_x(m, s);
    H(FZ_OP_OPROJ, false);
    H(FZ_OP_GATEUP, true);
    launch_gemv(gl[4 * li + 2], s);
    H(FZ_OP_GATEUP, false);
    H(FZ_OP_DOWN, true);
    launch_gemv(gl[4 * li + 3], s);
    tp_allreduce_x(m, s);
    H(FZ_OP_DOWN, false);
  }
  if (with_logits) {
    H(FZ_OP_LMHEAD, true);
    launch_gemv(lm, s);
    // greedy pick over all ranks' vocabulary slices: max of the packed
    // (logit, index) keys, which prefers the first index on ties
    if (m->world > 1)
      nccl_comm_check(&m->comm, nccl().AllReduce(&st->argmax_key, &st->argmax_key, 1, ncclUint64, ncclMax, m->comm, s),
                 "ncclAllReduce");
    H(FZ_OP_LMHEAD, false);
  }
  H(FZ_OP_FINALIZE, true);
  const bool xch = m->world > 1 && m->ar_p2p;
  launch_finalize(st, kv->forced.as<uint32_t>(), kv->ids.as<uint32_t>(), with_logits, s,
                  xch ? m->ar_base.as<uint32_t>() : nullptr, xch ? 2 * c.n_layers : 0);
  H(FZ_OP_FINALIZE, false);
}

// ---- batched prefill on the tensor cores ------------------------------------
constexpr uint32_t PF_CHUNK = 8192;  // tokens per prefill pass (each weight is dequantized once per pass)
constexpr uint32_t PF_MIN = 8;       // shorter prompts replay the decode step

// Every GEMM's reduction width (hidden, this rank's o_proj input and FFN
// slice) must be a multiple of 64, the k-step of the panels.
bool prefill_supported(const fz_model* m) {
  if (m->cfg.hidden % 64) return false;
  for (const Layer& L : m->layers)
    if (L.wo.cols % 64 || L.wd.cols % 64) return false;
  return true;
}

void prefill_alloc(fz_model* m, uint32_t T) {
  if (m->pf_cap >= T) return;
  const fz_config& c = m->cfg;
  const uint32_t H = c.hidden, F = c.ffn, qd = m->qd_l, kd = m->kd_l;
  const uint32_t maxK = std::max(std::max(H, F), std::max(qd, m->o_w));
  uint64_t wmax = 0, rmax = 0;
  for (auto& L : m->layers) {
    wmax = std::max(wmax, wpanel_elems(L.wq.rows + L.wk.rows + L.wv.rows, H));
    wmax = std::max(wmax, wpanel_elems(L.wo.rows, L.wo.cols));
    wmax = std::max(wmax, wpanel_elems(L.wgu.rows, H));
    wmax = std::max(wmax, wpanel_elems(L.wd.rows, L.wd.cols));
    rmax = std::max<uint64_t>(rmax, std::max({L.wq.rows + L.wk.rows + L.wv.rows, L.wo.rows, L.wgu.rows, L.wd.rows}));
  }
  m->pf_x.alloc((uint64_t)T * H * 4);
  m->pf_qkv.alloc((uint64_t)T * (qd + 2 * kd) * 4);
  m->pf_ctx.alloc((uint64_t)T * std::max(qd, m->o_w) * 4);
  m->pf_h.alloc((uint64_t)T * F * 4);
  m->pf_tok.alloc((uint64_t)T * 4);
  m->pf_err.alloc(16);
  m->pf_wh.alloc(wmax * 2);
  m->pf_wl.alloc(wmax * 2);
  const uint64_t xe = xpanel_elems(T, maxK);
  m->pf_xh.alloc(xe * 2);
  m->pf_xl.alloc(xe * 2);
  // padding rows of the panels are read by the MMAs and dropped by the
  // epilogue: start them finite
  // on the model's stream: it does not wait for the legacy default stream,
  // so a cudaMemset there could still be running when the panels are written
  CK(cudaMemsetAsync(m->pf_wh.p, 0, m->pf_wh.n, m->stream));
  CK(cudaMemsetAsync(m->pf_wl.p, 0, m->pf_wl.n, m->stream));
  CK(cudaMemsetAsync(m->pf_xh.p, 0, m->pf_xh.n, m->stream));
  CK(cudaMemsetAsync(m->pf_xl.p, 0, m->pf_xl.n, m->stream));
  CK(cudaMemsetAsync(m->pf_err.p, 0, 16, m->stream));
  m->pf_rexp.alloc((rmax + 127) / 128 * 128);
  m->pf_texp.alloc(T + 16);
  CK(cudaMemsetAsync(m->pf_rexp.p, 0, m->pf_rexp.n, m->stream));
  CK(cudaMemsetAsync(m->pf_texp.p, 0, m->pf_texp.n, m->stream));
  m->pf_cap = T;
}

// Tokens [0, n) at positions pos0.. through every layer, batched
// (Model::forward_cached, src/model.rs:444-478, 579-592, without the logits):
// x rows, the KV cache rows pos0..pos0+n, nothing else.
//
// Tensor parallelism: x [T, H] is replicated; each rank projects q/k/v of its
// heads, attends over its KV heads and multiplies its o_proj columns and its
// FFN slice, so o_proj and down leave per-rank partials of the residual
// update.  Rank 0 adds its partial to x, the others to zeros, and one
// all-reduce (sum) over [T, H] restores the replicated x.
void prefill_tokens(fz_kv* kv, const uint32_t* tokens, uint32_t n, uint32_t pos0) {
  fz_model* m = kv->m;
  const fz_config& c = m->cfg;
  cudaStream_t s = m->stream;
  const uint32_t H = c.hidden, hd = c.head_dim, qd = m->qd_l, kd = m->kd_l, ldq = qd + 2 * kd;
  // ctx rows are o_proj's block-aligned input: this rank's heads start at
  // column o_off[li], the rest (a neighbour's share of a boundary block) is 0
  const uint32_t ldc = std::max(qd, m->o_w);
  prefill_init();
  prefill_alloc(m, std::min(n, PF_CHUNK));
  float* X = m->pf_x.as<float>();
  float* ctx = m->pf_ctx.as<float>();
  uint32_t* err = m->pf_err.as<uint32_t>();
  auto gemm = [&](uint32_t K, uint32_t N, uint32_t T, int epi, float* out, uint32_t ld, const float* bias) {
    QgemmLaunch q{m->pf_wh.p, m->pf_wl.p, m->pf_xh.p, m->pf_xl.p, m->pf_rexp.as<int8_t>(), m->pf_texp.as<int8_t>(),
                  K, N, T, epi, out, ld, bias, err};
    launch_qgemm(q, s);
  };
  // x += the [T, K] activations (panels built) times w (panels built), summed over ranks
  auto resid = [&](uint32_t K, uint32_t T) {
    if (m->world > 1 && m->rank != 0) CK(cudaMemsetAsync(X, 0, (size_t)T * H * 4, s));
    gemm(K, H, T, PE_RESID, X, H, nullptr);
    if (m->world > 1)
      nccl_comm_check(&m->comm, nccl().AllReduce(X, X, (size_t)T * H, ncclFloat32, ncclSum, m->comm, s),
                      "ncclAllReduce");
  };
  for (uint32_t c0 = 0; c0 < n; c0 += PF_CHUNK) {
    const uint32_t T = std::min(PF_CHUNK, n - c0);
    CK(cudaMemcpyAsync(m->pf_tok.p, tokens + c0, (size_t)T * 4, cudaMemcpyHostToDevice, s));
    launch_embed_rows(m->embd, m->pf_tok.as<uint32_t>(), T, X, H, s);
    for (uint32_t li = 0; li < c.n_layers; li++) {
      Layer& L = m->layers[li];
      const uint32_t F_l = L.wd.cols;
      // q, k, v (+ bias) of RMSNorm(x)
      launch_xpanels(X, H, T, H, L.attn_norm, c.rms_eps, m->pf_xh.p, m->pf_xl.p, m->pf_texp.as<int8_t>(), s);
      launch_wpanels(L.wq, 0, m->pf_rexp.as<int8_t>(), m->pf_wh.p, m->pf_wl.p, s);
      launch_wpanels(L.wk, L.wq.rows, m->pf_rexp.as<int8_t>(), m->pf_wh.p, m->pf_wl.p, s);
      launch_wpanels(L.wv, L.wq.rows + L.wk.rows, m->pf_rexp.as<int8_t>(), m->pf_wh.p, m->pf_wl.p, s);
      gemm(H, ldq, T, PE_STORE, m->pf_qkv.as<float>(), ldq, L.bqkv);
      // rotated k / v into the cache, causal attention per token
      if (L.wo.cols != qd) CK(cudaMemsetAsync(ctx, 0, (size_t)T * ldc * 4, s));
      launch_prefill_attention(m->pf_qkv.as<float>(), ldq, kv->rope_cs.as<float>(), kv->layer_k(li, m->nkv_l, hd),
                               kv->layer_v(li, m->nkv_l, hd), kv->eb == 2, ctx + m->o_off[li], ldc, m->nh_l,
                               m->nkv_l, hd, kv->max_ctx, pos0 + c0, T, err, s);
      // x += o_proj(ctx)
      launch_xpanels(ctx, ldc, T, L.wo.cols, nullptr, 0.f, m->pf_xh.p, m->pf_xl.p, m->pf_texp.as<int8_t>(), s);
      launch_wpanels(L.wo, 0, m->pf_rexp.as<int8_t>(), m->pf_wh.p, m->pf_wl.p, s);
      resid(L.wo.cols, T);
      // h = swiglu(gate, up)(RMSNorm(x)); x += down(h)
      launch_xpanels(X, H, T, H, L.ffn_norm, c.rms_eps, m->pf_xh.p, m->pf_xl.p, m->pf_texp.as<int8_t>(), s);
      launch_wpanels(L.wgu, 0, m->pf_rexp.as<int8_t>(), m->pf_wh.p, m->pf_wl.p, s);
      gemm(H, L.wgu.rows, T, PE_SWIGLU, m->pf_h.as<float>(), F_l, nullptr);
      launch_xpanels(m->pf_h.as<float>(), F_l, T, F_l, nullptr, 0.f, m->pf_xh.p, m->pf_xl.p, m->pf_texp.as<int8_t>(), s);
      launch_wpanels(L.wd, 0, m->pf_rexp.as<int8_t>(), m->pf_wh.p, m->pf_wl.p, s);
      resid(F_l, T);
    }
  }
  uint32_t e = 0;
  CK(cudaMemcpyAsync(&e, err, 4, cudaMemcpyDeviceToHost, s));
  CK(cudaStreamSynchronize(s));
  if (e) {
    CK(cudaMemsetAsync(err, 0, 4, s));
    fail(FZ_ETIMEOUT, "prefill: a bounded device wait ran out (code %u)", e);
  }
}


// ---- sampling (src/sampler.rs) ------------------------------------------------
// Softmax, top-p, renormalisation and the draw over candidates (id, l / temp)
// sorted by value descending, id ascending on ties: Sampler::filtered's tail
// and Sampler::sample's walk (src/sampler.rs:96-108, 126-154), in the
// reference's f32 operation order.
uint32_t sampler_finish(fz_sampler* s, std::vector<std::pair<uint32_t, float>>& c) {
  const float mx = c[0].second;
  float sum = 0.0f;
  for (auto& e : c) {
    e.second = expf(e.second - mx);
    sum += e.second;
  }
  for (auto& e : c) e.second /= sum;
  if (s->top_p < 1.0f) {
    float cum = 0.0f;
    size_t keep = c.size();
    for (size_t i = 0; i < c.size(); i++) {
      cum += c[i].second;
      if (cum >= s->top_p) {
        keep = i + 1;
        break;
      }
    }
    c.resize(keep);
    float t = 0.0f;
    for (auto& e : c) t += e.second;
    for (auto& e : c) e.second /= t;
  }
  const float u = s->next_f32();
  s->draws++;
  float cum = 0.0f;
  for (auto& e : c) {
    cum += e.second;
    if (u < cum) return e.first;
  }
  return c.back().first;
}

// Sampler::sample on host logits (src/sampler.rs:86-108).
uint32_t sample_host(fz_sampler* s, const float* logits, size_t n, const uint32_t* recent, size_t nr) {
  std::vector<float> lg(logits, logits + n);
  if (s->repeat_penalty != 1.0f) {  // apply_repeat_penalty (src/sampler.rs:39-55)
    std::vector<uint32_t> seen;
    for (size_t i = 0; i < nr; i++) {
      const uint32_t t = recent[i];
      if (t >= n || std::find(seen.begin(), seen.end(), t) != seen.end()) continue;
      seen.push_back(t);
      lg[t] = lg[t] > 0.0f ? lg[t] / s->repeat_penalty : lg[t] * s->repeat_penalty;
    }
  }
  if (s->greedy()) {  // first max (src/generate.rs:69-77)
    size_t best = 0;
    for (size_t i = 1; i < n; i++)
      if (lg[i] > lg[best]) best = i;
    return (uint32_t)best;
  }
  std::vector<std::pair<uint32_t, float>> c(n);
  for (size_t i = 0; i < n; i++) c[i] = {(uint32_t)i, lg[i] / s->temperature};
  std::stable_sort(c.begin(), c.end(), [](const auto& a, const auto& b) { return a.second > b.second; });
  if (s->top_k > 0 && s->top_k < c.size()) c.resize(s->top_k);
  return sampler_finish(s, c);
}

// Sampler::sample on the model's current logits: penalty, temperature and
// top-k on the device, only the k survivors cross to the host.
uint32_t sample_device(fz_model* m, fz_sampler* s, const uint32_t* recent, uint32_t nr) {
  const fz_config& c = m->cfg;
  cudaStream_t st = m->stream;
  const bool greedy = s->greedy();
  const uint32_t k = greedy ? 1 : s->top_k;
  if (k == 0 || k > topk_max()) {  // the whole vocabulary is a candidate: host path
    std::vector<float> lg(c.vocab);
    CK(cudaMemcpyAsync(lg.data(), m->logits.p, (size_t)c.vocab * 4, cudaMemcpyDeviceToHost, st));
    CK(cudaStreamSynchronize(st));
    return sample_host(s, lg.data(), lg.size(), recent, nr);
  }
  sampler_init();
  if (!m->smp_scratch.p) {
    m->smp_scratch.alloc(topk_scratch_bytes(c.vocab));
    m->smp_out.alloc(topk_max() * 8 + 64 * 4);
  }
  uint32_t* rdev = reinterpret_cast<uint32_t*>(m->smp_out.as<uint8_t>() + topk_max() * 8);
  if (nr) CK(cudaMemcpyAsync(rdev, recent, nr * 4, cudaMemcpyHostToDevice, st));
  launch_topk(m->logits.as<float>(), c.vocab, rdev, nr, s->repeat_penalty, greedy ? 1.0f : s->temperature, k,
              m->smp_scratch.p, m->smp_out.p, st);
  std::vector<unsigned long long> keys(k);
  CK(cudaMemcpyAsync(keys.data(), m->smp_out.p, k * 8, cudaMemcpyDeviceToHost, st));
  CK(cudaStreamSynchronize(st));
  std::vector<std::pair<uint32_t, float>> cand(k);
  for (uint32_t i = 0; i < k; i++) {
    const uint32_t ord = (uint32_t)(keys[i] >> 32), idx = 0xFFFFFFFFu - (uint32_t)(keys[i] & 0xFFFFFFFFull);
    const uint32_t bits = (ord & 0x80000000u) ? (ord & 0x7FFFFFFFu) : ~ord;
    cand[i] = {idx, __builtin_bit_cast(float, bits)};
  }
  if (greedy) return cand[0].first;
  return sampler_finish(s, cand);
}

// The step is captured as separate kernels chained by programmatic dependent
// launches: one graph with the logits (lm_head + argmax), one without.
void build_graphs(fz_kv* kv) {
  if (kv->g_full) return;
  cudaStream_t s = kv->m->stream;
  for (int variant = 0; variant < 2; variant++) {
    cudaGraph_t g;
    CK(cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal));
    try {
      record_step(kv, variant == 0, s);
    } catch (...) {
      cudaStreamEndCapture(s, &g);
      if (g) cudaGraphDestroy(g);
      throw;
    }
    CK(cudaStreamEndCapture(s, &g));
    cudaGraphExec_t ge;
    CK(cudaGraphInstantiate(&ge, g, 0));
    cudaGraphDestroy(g);
    (variant == 0 ? kv->g_full : kv->g_layers) = ge;
  }
}

// Every rank's vocabulary slice of the last logits, in place (tensor
// parallelism; slices are vocab_pad / world long and in rank order).
void tp_gather_logits(fz_model* m, cudaStream_t s) {
  if (m->world == 1) return;
  const size_t per = m->sl.vocab_pad / m->world;
  float* all = m->logits.as<float>();
  nccl_comm_check(&m->comm, nccl().AllGather(all + (size_t)m->rank * per, all, per, ncclFloat32, m->comm, s),
                  "ncclAllGather");
}

// IEEE binary16 -> binary32, exact (cached f16 KV elements read back).
float half_to_float(uint16_t h) {
  const uint32_t sign = (uint32_t)(h & 0x8000u) << 16, ex = (h >> 10) & 0x1Fu, man = h & 0x3FFu;
  uint32_t bits;
  if (ex == 0) {
    const float f = (float)man * 5.9604644775390625e-8f;  // man * 2^-24 (zero and subnormals)
    return sign ? -f : f;
  }
  if (ex == 31)
    bits = sign | 0x7F800000u | (man << 13);
  else
    bits = sign | ((ex + 112) << 23) | (man << 13);
  float f;
  memcpy(&f, &bits, 4);
  return f;
}

void set_state(fz_kv* kv, uint32_t pos, uint32_t token, uint32_t n_forced) {
  StepState st{};
  st.pos = pos;
  st.token = token;
  st.step = 0;
  st.n_forced = n_forced;
  st.argmax_key = 0;
  CK(cudaMemcpyAsync(kv->state.p, &st, sizeof st, cudaMemcpyHostToDevice, kv->m->stream));
}

void check_state(fz_kv* kv) {
  StepState st;
  CK(cudaMemcpyAsync(&st, kv->state.p, sizeof st, cudaMemcpyDeviceToHost, kv->m->stream));
  CK(cudaStreamSynchronize(kv->m->stream));
  // codes 1-2: token >= vocab, position >= max_ctx; 3-5 and 7: a bounded
  // device wait (input records, ring slot, KV tile; residual exchange) ran out
  if (st.error >= 3) fail(FZ_ETIMEOUT, "a bounded device wait ran out (code %u)", st.error);
  if (st.error) fail(FZ_EINVAL, "device step rejected its input (code %u)", st.error);
}

void use_device(const fz_model* m) { CK(cudaSetDevice(m->device)); }

// Algorithmic bytes of one decode step at position pos, per op kind:
// GGUF weight bytes, the KV rows read, the vectors read and written.
void step_bytes(const fz_model* m, const fz_kv* kv, uint64_t pos, double* bytes) {
  const fz_config& c = m->cfg;
  uint64_t H = c.hidden, F = m->sl.ffn_n, qd = m->qd_l, kd = m->kd_l;  // this rank's widths
  bytes[FZ_OP_EMBED] += m->embd.gguf_bytes / c.vocab + H * 4;
  for (auto& L : m->layers) {
    bytes[FZ_OP_QKV] += L.wq.gguf_bytes + L.wk.gguf_bytes + L.wv.gguf_bytes + (2 * H + qd + 2 * kd) * 4;
    bytes[FZ_OP_ROPE] += (qd + 2 * kd) * 4 + (qd + 2 * kd) * 4;
    bytes[FZ_OP_ATTN] += 2 * (pos + 1) * kd * kv->eb + 2 * qd * 4;
    bytes[FZ_OP_OPROJ] += L.wo.gguf_bytes + (qd + 2 * H) * 4;
    bytes[FZ_OP_GATEUP] += L.wgu.gguf_bytes + (2 * H + F) * 4;
    bytes[FZ_OP_DOWN] += L.wd.gguf_bytes + (F + 2 * H) * 4;
  }
  bytes[FZ_OP_LMHEAD] += m->lm_head.gguf_bytes + (2 * H + (uint64_t)c.vocab) * 4;
}

}  // namespace

// ===========================================================================
// C ABI
// ===========================================================================
extern "C" {

const char* fz_last_error(void) { return fz::last_error().c_str(); }
const char* fz_version(void) { return "furnace-b200 0.1 sm_100a"; }

int fz_open(const char* path, fz_file** out) {
  return guard([&] {
    need(path && out, "null argument");
    auto f = new fz_file();
    try {
      f->g = open_gguf(path);
    } catch (...) {
      delete f;
      throw;
    }
    *out = f;
  });
}

int fz_open_bytes(const void* data, size_t n, fz_file** out) {
  return guard([&] {
    need(out && (data || n == 0), "null argument");
    auto f = new fz_file();
    try {
      f->g = open_gguf_bytes(data, n);
    } catch (...) {
      delete f;
      throw;
    }
    *out = f;
  });
}

void fz_file_free(fz_file* f) { delete f; }

int fz_file_info(const fz_file* f, uint32_t* version, size_t* n_tensors, size_t* n_meta, size_t* data_start) {
  return guard([&] {
    need(f != nullptr, "null file");
    if (version) *version = f->g->version;
    if (n_tensors) *n_tensors = f->g->tensors.size();
    if (n_meta) *n_meta = f->g->meta.size();
    if (data_start) *data_start = f->g->data_start;
  });
}

static void fill_info(const GgufFile& g, const TensorEntry& t, fz_tensor_info* out) {
  out->name = t.name.c_str();
  out->dtype = t.dtype;
  out->n_dims = (uint32_t)t.dims.size();
  for (int i = 0; i < 4; i++) out->dims[i] = i < (int)t.dims.size() ? t.dims[i] : 1;
  out->offset = t.offset;
  uint32_t be, bb;
  out->nbytes = block_geom(t.dtype, &be, &bb) && t.n_elements() % be == 0 ? t.n_elements() / be * bb : 0;
  (void)g;
}

int fz_tensor_at(const fz_file* f, size_t i, fz_tensor_info* out) {
  return guard([&] {
    need(f && out, "null argument");
    need(i < f->g->tensors.size(), "tensor index %zu out of range", i);
    fill_info(*f->g, f->g->tensors[i], out);
  });
}

int fz_tensor(const fz_file* f, const char* name, fz_tensor_info* info, const void** data) {
  return guard([&] {
    need(f && name, "null argument");
    const TensorEntry* t = f->g->find(name);
    if (!t) fail(FZ_EFORMAT, "no tensor named '%s'", name);
    uint64_t nb;
    const uint8_t* d = f->g->tensor_data(*t, &nb);
    if (info) fill_info(*f->g, *t, info);
    if (data) *data = d;
  });
}

int fz_meta_u32(const fz_file* f, const char* key, uint32_t* out) {
  return guard([&] { *out = f->g->meta_u32(key); });
}
int fz_meta_f32(const fz_file* f, const char* key, float* out) {
  return guard([&] { *out = f->g->meta_f32(key); });
}
int fz_meta_str(const fz_file* f, const char* key, const char** out) {
  return guard([&] { *out = f->g->meta_str(key).c_str(); });
}
int fz_meta_array_len(const fz_file* f, const char* key, size_t* out) {
  return guard([&] { *out = f->g->meta_array_len(key); });
}

int fz_config_from_gguf(const fz_file* f, fz_config* out) {
  return guard([&] {
    need(f && out, "null argument");
    *out = config_from_gguf(*f->g);
  });
}

}  // extern "C"

namespace {

// Model::load (src/model.rs:520-552) for rank `rank` of `world`: the rank's
// slice of every matrix, uploaded raw and repacked into the device layout.
// Receive buffers of the residual exchange: every rank exports its buffer
// by CUDA IPC, the handles travel by NCCL all-gather, and each rank maps the
// others'.  Collective: every rank calls it once while loading.
void tp_p2p_setup(fz_model* m) {
  const char* e = getenv("FURNACE_B200_TP_ALLREDUCE");
  const bool want = !(e && strcmp(e, "nccl") == 0);
  const uint32_t W = (uint32_t)m->world;
  need(W <= (uint32_t)AR_MAX_RANKS, "tensor parallelism over %u ranks > %d", W, AR_MAX_RANKS);
  need(m->cfg.hidden % 4 == 0, "hidden %u not a multiple of 4", m->cfg.hidden);
  m->ar_buf.alloc(ar_buffer_bytes(m->cfg.hidden, W));
  CK(cudaMemsetAsync(m->ar_buf.p, 0, m->ar_buf.n, m->stream));
  m->ar_base.alloc(16);
  CK(cudaMemsetAsync(m->ar_base.p, 0, m->ar_base.n, m->stream));
  CK(cudaStreamSynchronize(m->stream));
  // every rank takes part in the exchange (the same collective steps on all
  // ranks); a rank that cannot export marks its handle invalid
  static_assert(sizeof(cudaIpcMemHandle_t) == 64, "IPC handle size");
  std::vector<uint8_t> mine(72, 0), all(72 * W);
  cudaIpcMemHandle_t h{};
  const bool ok = want && cudaIpcGetMemHandle(&h, m->ar_buf.p) == cudaSuccess;
  cudaGetLastError();
  memcpy(mine.data(), &h, 64);
  mine[64] = ok ? 1 : 0;
  DevBuf d(72ull * W);
  CK(cudaMemcpy(d.as<uint8_t>() + 72ull * m->rank, mine.data(), 72, cudaMemcpyHostToDevice));
  nccl_comm_check(&m->comm, nccl().AllGather(d.as<uint8_t>() + 72ull * m->rank, d.p, 72, ncclUint8, m->comm, m->stream),
             "ncclAllGather");
  CK(cudaStreamSynchronize(m->stream));
  CK(cudaMemcpy(all.data(), d.p, all.size(), cudaMemcpyDeviceToHost));
  bool all_ok = true;
  for (uint32_t q = 0; q < W; q++) all_ok = all_ok && all[72 * q + 64] == 1;
  if (!all_ok) return;  // NCCL all-reduce
  m->ar_peers.buf[m->rank] = m->ar_buf.as<float>();
  for (uint32_t q = 0; q < W; q++) {
    if (q == (uint32_t)m->rank) continue;
    cudaIpcMemHandle_t hq;
    memcpy(&hq, all.data() + 72 * q, 64);
    void* p = nullptr;
    CK(cudaIpcOpenMemHandle(&p, hq, cudaIpcMemLazyEnablePeerAccess));
    m->ar_peers.buf[q] = static_cast<float*>(p);
  }
  m->ar_p2p = true;
}

std::unique_ptr<fz_model> load_model(const fz_file* f, int rank, int world, const ncclUniqueId* id, int device) {
  need(f != nullptr, "null argument");
  const GgufFile& g = *f->g;
  auto m = std::make_unique<fz_model>();
  m->cfg = config_from_gguf(g);
  const fz_config& c = m->cfg;
  m->device = device;
  m->rank = rank;
  m->world = world;
  CK(cudaSetDevice(m->device));
  need(c.head_dim == 64 || c.head_dim == 128, "head_dim %u unsupported (64 or 128)", c.head_dim);
  need(c.n_kv_heads && c.n_heads % c.n_kv_heads == 0, "%u heads not divisible by %u kv heads", c.n_heads, c.n_kv_heads);
  need(c.n_heads / c.n_kv_heads <= 8, "GQA group %u > 8 unsupported", c.n_heads / c.n_kv_heads);
  need(c.hidden % 32 == 0 && c.ffn % 32 == 0, "hidden/ffn must be multiples of 32");
  const fz_tp_slice sl = tp_slice(c, rank, world);
  m->sl = sl;
  m->nh_l = sl.q_heads;
  m->nkv_l = sl.kv_heads;
  const uint32_t hd = c.head_dim, H = c.hidden, F = c.ffn;
  const uint32_t qd = c.n_heads * hd, kd = c.n_kv_heads * hd;
  const uint32_t qd_l = sl.q_heads * hd, kd_l = sl.kv_heads * hd, F_l = sl.ffn_n;
  m->qd_l = qd_l;
  m->kd_l = kd_l;
  CK(cudaStreamCreateWithFlags(&m->stream, cudaStreamNonBlocking));
  kernels_init();
  attention_init();

  // the matrices of this rank: rows [row0, row0 + rows) and block-aligned
  // input columns [col0, col0 + cols) of each GGUF weight
  struct Up {
    const TensorEntry* t;
    uint64_t row0;
    uint32_t col0, in_d;
    DevMat* dst;
  };
  m->layers.resize(c.n_layers);
  m->o_off.assign(c.n_layers, 0);
  std::vector<Up> ups;
  auto add = [&](const std::string& name, uint64_t out_d, uint64_t in_d, uint64_t row0, uint32_t rows, uint32_t col0,
                 uint32_t cols, DevMat* dst) {
    const TensorEntry& t = tensor2d(g, name, out_d, in_d);
    dst->dtype = t.dtype;
    dst->rows = rows;
    dst->cols = cols;
    dst->stride = dev_row_stride(t.dtype, cols);
    dst->gguf_bytes = gguf_bytes(t.dtype, rows, cols);
    ups.push_back({&t, row0, col0, (uint32_t)in_d, dst});
  };
  add("token_embd.weight", c.vocab, H, 0, c.vocab, 0, H, &m->embd);
  // lm_head: this rank's vocabulary rows (a tied model on one device reads
  // token_embd itself, src/model.rs:539-545)
  const bool tied = g.find("output.weight") == nullptr, share_embd = tied && world == 1;
  if (!share_embd)
    add(tied ? "token_embd.weight" : "output.weight", c.vocab, H, sl.vocab0, sl.vocab_n, 0, H, &m->lm_head);
  std::vector<const TensorEntry*> gates(c.n_layers), upsw(c.n_layers);
  for (uint32_t i = 0; i < c.n_layers; i++) {
    std::string p = "blk." + std::to_string(i) + ".";
    Layer& L = m->layers[i];
    add(p + "attn_q.weight", qd, H, (uint64_t)sl.q_head0 * hd, qd_l, 0, H, &L.wq);
    add(p + "attn_k.weight", kd, H, (uint64_t)sl.kv_head0 * hd, kd_l, 0, H, &L.wk);
    add(p + "attn_v.weight", kd, H, (uint64_t)sl.kv_head0 * hd, kd_l, 0, H, &L.wv);
    // o_proj: this rank's ctx columns, widened to whole blocks; the part of
    // a shared boundary block that belongs to the neighbour multiplies zeros
    const TensorEntry* to = g.find(p + "attn_output.weight");
    need(to != nullptr, "no tensor named '%s'", (p + "attn_output.weight").c_str());
    uint32_t be, bb;
    block_geom(to->dtype, &be, &bb);
    const uint32_t a0 = sl.o_col0 / be * be, a1 = (sl.o_col0 + sl.o_cols + be - 1) / be * be;
    m->o_off[i] = sl.o_col0 - a0;
    m->o_w = std::max(m->o_w, a1 - a0);
    add(p + "attn_output.weight", H, qd, 0, H, a0, a1 - a0, &L.wo);
    add(p + "ffn_down.weight", H, F, 0, H, sl.ffn0, F_l, &L.wd);
    gates[i] = &tensor2d(g, p + "ffn_gate.weight", F, H);
    upsw[i] = &tensor2d(g, p + "ffn_up.weight", F, H);
    need(gates[i]->dtype == upsw[i]->dtype, "blk.%u ffn_gate/ffn_up dtypes differ (%u vs %u)", i, gates[i]->dtype,
         upsw[i]->dtype);
    L.wgu.dtype = gates[i]->dtype;
    L.wgu.rows = 2 * F_l;
    L.wgu.cols = H;
    L.wgu.stride = dev_row_stride(L.wgu.dtype, H);
    L.wgu.gguf_bytes = 2 * gguf_bytes(L.wgu.dtype, F_l, H);
  }
  need(m->o_w % 16 == 0, "o_proj input width %u", m->o_w);
  // one pool for every matrix, 256-byte aligned, in the order a decode step
  // streams them (L2 prefetch runs from one matrix into the next)
  uint64_t total = 0;
  auto reserve = [&](DevMat& d) {
    uint64_t off = total;
    total = (total + (uint64_t)d.rows * d.stride + 255) & ~uint64_t(255);
    return off;
  };
  std::vector<std::pair<DevMat*, uint64_t>> order;
  order.push_back({&m->embd, reserve(m->embd)});
  for (uint32_t i = 0; i < c.n_layers; i++) {
    Layer& L = m->layers[i];
    for (DevMat* d : {&L.wq, &L.wk, &L.wv, &L.wo, &L.wgu, &L.wd}) order.push_back({d, reserve(*d)});
  }
  if (!share_embd) order.push_back({&m->lm_head, reserve(m->lm_head)});
  m->weights.alloc(total);
  CK(cudaMemsetAsync(m->weights.p, 0, total, m->stream));  // the uploads below run on m->stream
  uint8_t* base = m->weights.as<uint8_t>();
  for (auto& o : order) o.first->ptr = base + o.second;
  uint64_t max_raw = 0;
  for (auto& u : ups) max_raw = std::max<uint64_t>(max_raw, u.dst->gguf_bytes);
  Uploader up(m->stream, std::min<uint64_t>(max_raw + 16, 64ull << 20));
  for (auto& u : ups) {
    DevMat& d = *u.dst;
    uint64_t nb;
    const uint8_t* raw = g.tensor_data(*u.t, &nb);
    if (u.col0 == 0 && d.cols == u.in_d)
      upload_rows(d.dtype, raw + u.row0 * gguf_bytes(d.dtype, 1, u.in_d), d.rows, d.cols, d.ptr, up);
    else
      upload_cols(d.dtype, raw, d.rows, u.in_d, u.col0, d.cols, d.ptr, up);
  }
  if (share_embd) m->lm_head = m->embd;
  // gate/up interleaved by row: row 2i = gate_(ffn0+i), row 2i+1 = up_(ffn0+i)
  for (uint32_t i = 0; i < c.n_layers; i++) {
    DevMat& d = m->layers[i].wgu;
    uint64_t nb;
    const uint8_t* graw = g.tensor_data(*gates[i], &nb);
    const uint8_t* uraw = g.tensor_data(*upsw[i], &nb);
    const uint64_t rb = gguf_bytes(d.dtype, 1, H);
    const uint32_t per = (uint32_t)std::max<uint64_t>(1, up.cap / (2 * rb));
    for (uint32_t r0 = 0; r0 < F_l; r0 += per) {
      const uint32_t nr = std::min<uint32_t>(per, F_l - r0);
      std::vector<std::pair<const uint8_t*, size_t>> segs(2 * nr);
      for (uint32_t r = 0; r < nr; r++) {
        segs[2 * r] = {graw + (uint64_t)(sl.ffn0 + r0 + r) * rb, rb};
        segs[2 * r + 1] = {uraw + (uint64_t)(sl.ffn0 + r0 + r) * rb, rb};
      }
      up.push(segs, [&](const uint8_t* dv) {
        launch_repack(d.dtype, dv, d.ptr, 2 * r0, 2 * nr, d.rows, H, m->stream);
      });
    }
  }
  up.finish();
  // norms (replicated) and this rank's q/k/v bias slices
  std::vector<float> smalls;
  std::vector<std::pair<size_t, float**>> fix;
  auto push = [&](const std::vector<float>& v, float** where) {
    fix.push_back({smalls.size(), where});
    smalls.insert(smalls.end(), v.begin(), v.end());
    while (smalls.size() % 64) smalls.push_back(0.f);
  };
  for (uint32_t i = 0; i < c.n_layers; i++) {
    std::string p = "blk." + std::to_string(i) + ".";
    Layer& L = m->layers[i];
    push(vec_f32(g, p + "attn_norm.weight", H), &L.attn_norm);
    push(vec_f32(g, p + "ffn_norm.weight", H), &L.ffn_norm);
    std::vector<float> bq = vec_f32(g, p + "attn_q.bias", qd);
    std::vector<float> bk = vec_f32(g, p + "attn_k.bias", kd), bv = vec_f32(g, p + "attn_v.bias", kd);
    std::vector<float> b(bq.begin() + (size_t)sl.q_head0 * hd, bq.begin() + (size_t)sl.q_head0 * hd + qd_l);
    b.insert(b.end(), bk.begin() + (size_t)sl.kv_head0 * hd, bk.begin() + (size_t)sl.kv_head0 * hd + kd_l);
    b.insert(b.end(), bv.begin() + (size_t)sl.kv_head0 * hd, bv.begin() + (size_t)sl.kv_head0 * hd + kd_l);
    push(b, &L.bqkv);
  }
  push(vec_f32(g, "output_norm.weight", H), &m->out_norm);
  m->smalls.alloc(smalls.size() * 4);
  CK(cudaMemcpy(m->smalls.p, smalls.data(), smalls.size() * 4, cudaMemcpyHostToDevice));
  for (auto& fx : fix) *fx.second = m->smalls.as<float>() + fx.first;
  // activations
  m->x.alloc(H * 4);
  m->qkv.alloc((qd_l + 2 * kd_l) * 4);
  m->ctx.alloc(qd_l * 4);
  m->h.alloc(F_l * 4);
  m->logits.alloc((uint64_t)sl.vocab_pad * 4);
  CK(cudaMemsetAsync(m->logits.p, 0, m->logits.n, m->stream));
  auto runs = [&](DevBuf& b, uint32_t n) {
    b.alloc((uint64_t)runs_for(n) * 64);
    CK(cudaMemsetAsync(b.p, 0, b.n, m->stream));  // padding records past the vector must read as zero
  };
  std::vector<uint32_t> offs;  // distinct o_off values, in order of first use
  m->ctx_buf.assign(c.n_layers, 0);
  for (uint32_t i = 0; i < c.n_layers; i++) {
    size_t b = std::find(offs.begin(), offs.end(), m->o_off[i]) - offs.begin();
    if (b == offs.size()) {
      offs.push_back(m->o_off[i]);
      m->runs_ctx.push_back(std::make_unique<DevBuf>());
      runs(*m->runs_ctx.back(), m->o_w);
    }
    m->ctx_buf[i] = (uint32_t)b;
  }
  runs(m->runs_h, F_l);
  // byte accounting (this rank)
  m->resident = total + smalls.size() * 4;
  uint64_t per_tok = m->lm_head.gguf_bytes + m->embd.gguf_bytes / c.vocab + (uint64_t)H * 4;
  for (auto& L : m->layers)
    per_tok += L.wq.gguf_bytes + L.wk.gguf_bytes + L.wv.gguf_bytes + L.wo.gguf_bytes + L.wgu.gguf_bytes +
               L.wd.gguf_bytes + (uint64_t)(2 * H + qd_l + 2 * kd_l) * 4;
  m->streamed = per_tok;
  if (world > 1) {
    need(id != nullptr, "tensor parallelism needs an NCCL id");
    if (nccl().CommInitRankConfig) {
      // non-blocking: a peer that never joins ends in FZ_ETIMEOUT, not a hang
      ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
      cfg.blocking = 0;
      nccl_comm_check(&m->comm, nccl().CommInitRankConfig(&m->comm, world, *id, rank, &cfg),
                      "ncclCommInitRankConfig");
    } else {
      nccl_check(nccl().CommInitRank(&m->comm, world, *id, rank), "ncclCommInitRank");
    }
    tp_p2p_setup(m.get());
  }
  // optional timeline of every decode-step kernel's CTAs, written to the named
  // file by fz_model_free (the records of the last fz_decode_greedy call)
  if (const char* tp = getenv("FURNACE_B200_TRACE")) {
    const uint32_t cap = 1u << 20;
    m->trace.alloc((uint64_t)cap * sizeof(TraceRec));
    m->trace_path = tp;
    trace_install(m->trace.as<TraceRec>(), cap);
  }
  CK(cudaStreamSynchronize(m->stream));
  return m;
}

}  // namespace

extern "C" {

int fz_model_load(const fz_file* f, int tp, const int* device_ids, fz_model** out) {
  return guard([&] {
    need(f && out, "null argument");
    need(tp == 1, "fz_model_load loads one device (tp = 1); use fz_model_load_tp per rank");
    *out = load_model(f, 0, 1, nullptr, device_ids ? device_ids[0] : 0).release();
  });
}

int fz_model_load_tp(const fz_file* f, int rank, int world, const void* id, size_t n, int device, fz_model** out) {
  return guard([&] {
    need(f && out, "null argument");
    need(world >= 1 && rank >= 0 && rank < world, "rank %d of %d", rank, world);
    need(world == 1 || (id && n >= sizeof(ncclUniqueId)), "an NCCL id of %zu bytes is required", sizeof(ncclUniqueId));
    ncclUniqueId uid{};
    if (world > 1) memcpy(&uid, id, sizeof uid);
    *out = load_model(f, rank, world, world > 1 ? &uid : nullptr, device).release();
  });
}

int fz_tp_unique_id(void* id, size_t n) {
  return guard([&] {
    need(id && n >= sizeof(ncclUniqueId), "an id buffer of %zu bytes is required", sizeof(ncclUniqueId));
    ncclUniqueId uid;
    nccl_check(nccl().GetUniqueId(&uid), "ncclGetUniqueId");
    memcpy(id, &uid, sizeof uid);
  });
}

int fz_tp_slice_of(const fz_config* c, int rank, int world, fz_tp_slice* out) {
  return guard([&] {
    need(c && out, "null argument");
    *out = tp_slice(*c, rank, world);
  });
}

void fz_model_free(fz_model* m) {
  if (!m) return;
  cudaSetDevice(m->device);
  if (m->stream) {
    cudaStreamSynchronize(m->stream);
    cudaStreamDestroy(m->stream);
  }
  for (fz_kv* kv : m->caches) {
    kv->release();
    kv->m = nullptr;
  }
  if (m->ar_p2p)
    for (int q = 0; q < m->world; q++)
      if (q != m->rank && m->ar_peers.buf[q]) cudaIpcCloseMemHandle(m->ar_peers.buf[q]);
  if (m->comm) {
    try {
      nccl().CommDestroy(m->comm);
    } catch (...) {
    }
  }
  if (m->trace.p) {
    try {
      uint32_t n = std::min<uint32_t>(trace_count(), (uint32_t)(m->trace.n / sizeof(TraceRec)));
      std::vector<TraceRec> recs(n);
      if (n) CK(cudaMemcpy(recs.data(), m->trace.p, n * sizeof(TraceRec), cudaMemcpyDeviceToHost));
      if (FILE* f = fopen(m->trace_path.c_str(), "wb")) {
        if (n) fwrite(recs.data(), sizeof(TraceRec), n, f);
        fclose(f);
      }
      trace_install(nullptr, 0);
    } catch (...) {
    }
  }
  delete m;
}

int fz_model_config(const fz_model* m, fz_config* out) {
  return guard([&] {
    need(m && out, "null argument");
    *out = m->cfg;
  });
}

int fz_model_bytes(const fz_model* m, uint64_t* resident, uint64_t* streamed) {
  return guard([&] {
    need(m != nullptr, "null model");
    if (resident) *resident = m->resident;
    if (streamed) *streamed = m->streamed;
  });
}

int fz_model_stream(const fz_model* m, void** stream, int* device) {
  return guard([&] {
    need(m != nullptr, "null model");
    if (stream) *stream = (void*)m->stream;
    if (device) *device = m->device;
  });
}

int fz_kv_new(fz_model* m, uint32_t max_ctx, int kv_dtype, fz_kv** out) {
  return guard([&] {
    need(m && out, "null argument");
    need(kv_dtype == FZ_KV_F32 || kv_dtype == FZ_KV_F16, "kv dtype %d unsupported (FZ_KV_F32 or FZ_KV_F16)",
         kv_dtype);
    need(max_ctx > 0, "max_ctx must be positive");
    use_device(m);
    const fz_config& c = m->cfg;
    auto kv = std::make_unique<fz_kv>();
    kv->m = m;
    kv->max_ctx = max_ctx;
    kv->eb = kv_dtype == FZ_KV_F16 ? 2 : 4;
    uint64_t per = (uint64_t)c.n_layers * m->nkv_l * max_ctx * c.head_dim * kv->eb;  // this rank's KV heads
    kv->k.alloc(per);
    kv->v.alloc(per);
    // every user of the cache runs on the model's stream
    CK(cudaMemsetAsync(kv->k.p, 0, per, m->stream));
    CK(cudaMemsetAsync(kv->v.p, 0, per, m->stream));
    // RoPE factors with the reference's arithmetic (src/model.rs:207-210):
    // freq = theta^(-2i/hd), angle = pos * freq, (sin, cos) via libm.
    uint32_t half = c.head_dim / 2;
    std::vector<float> cs((uint64_t)max_ctx * half * 2);
    for (uint32_t i = 0; i < half; i++) {
      volatile float expo = -2.0f * (float)i / (float)c.head_dim;
      float freq = powf(c.rope_theta, expo);
      for (uint32_t p = 0; p < max_ctx; p++) {
        volatile float angle = (float)p * freq;
        cs[((uint64_t)p * half + i) * 2] = cosf(angle);
        cs[((uint64_t)p * half + i) * 2 + 1] = sinf(angle);
      }
    }
    kv->rope_cs.alloc(cs.size() * 4);
    CK(cudaMemcpy(kv->rope_cs.p, cs.data(), cs.size() * 4, cudaMemcpyHostToDevice));
    kv->splits = attention_splits(m->nkv_l);
    kv->partials.alloc(attention_partial_floats(m->nh_l, m->nkv_l, c.head_dim, kv->splits) * 4);
    // the split-padding entries of the accumulator block are never written
    // and must read as zero (they are weighted by 0 in the merge)
    CK(cudaMemsetAsync(kv->partials.p, 0, kv->partials.n, m->stream));
    kv->state.alloc(sizeof(StepState));
    CK(cudaMemsetAsync(kv->state.p, 0, sizeof(StepState), m->stream));
    kv->forced.alloc((uint64_t)max_ctx * 4 + 16);
    kv->ids.alloc((uint64_t)max_ctx * 4 + 16);
    m->caches.push_back(kv.get());
    *out = kv.release();
  });
}

void fz_kv_free(fz_kv* kv) {
  if (!kv) return;
  if (fz_model* m = kv->m) {  // else its model was freed first and took the device memory back
    cudaSetDevice(m->device);
    cudaStreamSynchronize(m->stream);
    m->caches.erase(std::remove(m->caches.begin(), m->caches.end(), kv), m->caches.end());
  }
  delete kv;
}

int fz_kv_len(const fz_kv* kv, uint32_t* len) {
  return guard([&] {
    need(kv && len, "null argument");
    *len = kv->len;
  });
}

int fz_kv_set_len(fz_kv* kv, uint32_t len) {
  return guard([&] {
    need(kv != nullptr, "null kv");
    need(kv->m != nullptr, "the cache's model has been freed");
    need(len <= kv->max_ctx, "kv len %u > max_ctx %u", len, kv->max_ctx);
    kv->len = len;
  });
}

int fz_kv_reset(fz_kv* kv) { return fz_kv_set_len(kv, 0); }

int fz_kv_bytes(const fz_kv* kv, uint64_t* bytes) {
  return guard([&] {
    need(kv && bytes, "null argument");
    need(kv->m != nullptr, "the cache's model has been freed");
    *bytes = (uint64_t)kv->k.n + kv->v.n;
  });
}

int fz_kv_read(const fz_kv* kv, uint32_t layer, int which_v, uint32_t n, float* out) {
  return guard([&] {
    need(kv && out, "null argument");
    need(kv->m != nullptr, "the cache's model has been freed");
    const fz_config& c = kv->m->cfg;
    need(layer < c.n_layers && n <= kv->max_ctx, "kv read out of range");
    use_device(kv->m);
    CK(cudaStreamSynchronize(kv->m->stream));  // the copies below run on the legacy stream
    uint32_t hd = c.head_dim;
    const uint32_t nkv = kv->m->nkv_l;  // this rank's KV heads
    const uint8_t* base = static_cast<const uint8_t*>(which_v ? kv->layer_v(layer, nkv, hd) : kv->layer_k(layer, nkv, hd));
    // device [kvh][pos][hd] -> host [pos][kvh*hd] (f16 elements widened exactly)
    const uint32_t eb = kv->eb;
    std::vector<uint8_t> raw((size_t)n * nkv * hd * eb);
    for (uint32_t h = 0; h < nkv; h++)
      CK(cudaMemcpy2D(raw.data() + (size_t)h * hd * eb, (size_t)nkv * hd * eb, base + (uint64_t)h * kv->max_ctx * hd * eb,
                      hd * eb, hd * eb, n, cudaMemcpyDeviceToHost));
    if (eb == 4) {
      memcpy(out, raw.data(), raw.size());
    } else {
      const uint16_t* r16 = reinterpret_cast<const uint16_t*>(raw.data());
      for (size_t i = 0; i < (size_t)n * nkv * hd; i++) out[i] = half_to_float(r16[i]);
    }
  });
}

int fz_forward(fz_model* m, fz_kv* kv, const uint32_t* tokens, uint32_t n, float* logits, uint32_t* argmax) {
  return guard([&] {
    need(m && kv && kv->m == m, "null or mismatched handles");
    need(tokens && n > 0, "forward with no tokens");
    need((uint64_t)kv->len + n <= kv->max_ctx, "context overflow: %u + %u > max_ctx %u", kv->len, n, kv->max_ctx);
    for (uint32_t i = 0; i < n; i++)
      need(tokens[i] < m->cfg.vocab, "token id %u out of range (vocab %u)", tokens[i], m->cfg.vocab);
    use_device(m);
    build_graphs(kv);
    cudaStream_t s = m->stream;
    uint32_t first = 0;  // tokens [0, first) go through the batched prefill
    if (n > PF_MIN && prefill_supported(m) && !getenv("FURNACE_B200_NO_PREFILL_GEMM")) {
      first = n - 1;
      prefill_tokens(kv, tokens, first, kv->len);
    }
    const uint32_t rest = n - first;
    CK(cudaMemcpyAsync(kv->forced.p, tokens + first, (size_t)rest * 4, cudaMemcpyHostToDevice, s));
    set_state(kv, kv->len + first, tokens[first], rest);
    for (uint32_t i = 0; i + 1 < rest; i++) CK(cudaGraphLaunch(kv->g_layers, s));
    CK(cudaGraphLaunch(kv->g_full, s));
    if (logits) {
      tp_gather_logits(m, s);
      CK(cudaMemcpyAsync(logits, m->logits.p, (size_t)m->cfg.vocab * 4, cudaMemcpyDeviceToHost, s));
    }
    uint32_t id = 0;
    CK(cudaMemcpyAsync(&id, kv->ids.as<uint32_t>() + (rest - 1), 4, cudaMemcpyDeviceToHost, s));
    check_state(kv);
    kv->len += n;
    if (argmax) *argmax = id;
  });
}

int fz_forward_last(fz_model* m, const uint32_t* tokens, uint32_t n, float* logits, uint32_t* argmax) {
  return guard([&] {
    need(m && tokens && n > 0, "forward_last with no tokens");
    // the uncached forward over positions 0..n-1 is the cached one from an
    // empty cache: a scratch cache of n positions, freed on every path
    fz_kv* kv = nullptr;
    int rc = fz_kv_new(m, n, 0, &kv);
    if (rc != FZ_OK) fail(rc, "%s", fz_last_error());
    std::unique_ptr<fz_kv, void (*)(fz_kv*)> hold(kv, fz_kv_free);
    rc = fz_forward(m, kv, tokens, n, logits, argmax);
    if (rc != FZ_OK) fail(rc, "%s", fz_last_error());
  });
}

int fz_decode_greedy(fz_model* m, fz_kv* kv, uint32_t first, uint32_t n_steps, const uint32_t* stop_ids,
                     uint32_t n_stop, uint32_t* ids_out, float* logits_out, uint32_t* n_out) {
  return guard([&] {
    need(m && kv && kv->m == m && ids_out, "null or mismatched handles");
    need(first < m->cfg.vocab, "token id %u out of range (vocab %u)", first, m->cfg.vocab);
    if (n_out) *n_out = 0;
    if (n_steps == 0) return;
    uint32_t fwd = n_steps - 1;
    need((uint64_t)kv->len + fwd <= kv->max_ctx, "context overflow: %u + %u > max_ctx %u", kv->len, fwd, kv->max_ctx);
    for (uint32_t i = 0; i < n_stop; i++)
      if (stop_ids[i] == first) return;  // src/generate.rs:125-127
    ids_out[0] = first;
    uint32_t written = 1;
    if (m->trace.p) trace_reset(m->stream);
    if (fwd) {
      use_device(m);
      build_graphs(kv);
      cudaStream_t s = m->stream;
      CK(cudaMemcpyAsync(kv->forced.p, &first, 4, cudaMemcpyHostToDevice, s));
      set_state(kv, kv->len, first, 1);
      for (uint32_t i = 0; i < fwd; i++) {
        CK(cudaGraphLaunch(kv->g_full, s));
        if (logits_out) {
          tp_gather_logits(m, s);
          CK(cudaMemcpyAsync(logits_out + (uint64_t)i * m->cfg.vocab, m->logits.p, (size_t)m->cfg.vocab * 4,
                             cudaMemcpyDeviceToHost, s));
        }
      }
      CK(cudaMemcpyAsync(ids_out + 1, kv->ids.p, (size_t)fwd * 4, cudaMemcpyDeviceToHost, s));
      check_state(kv);
      // Stop at the first stop id (src/generate.rs:124-127): it is not
      // emitted.  Forward i processed ids_out[i]; when ids_out[i] stops the
      // loop, forwards 0..i-1 are the ones the reference would have run.
      uint32_t used = fwd;
      for (uint32_t i = 1; i <= fwd; i++) {
        bool stop = false;
        for (uint32_t k = 0; k < n_stop; k++) stop |= ids_out[i] == stop_ids[k];
        if (stop) {
          used = i;
          break;
        }
        written++;
      }
      kv->len += used;
    }
    if (n_out) *n_out = written;
  });
}

int fz_sampler_new(float temperature, uint32_t top_k, float top_p, float repeat_penalty, uint64_t seed,
                   fz_sampler** out) {
  return guard([&] {
    need(out != nullptr, "null argument");
    need(temperature >= 0.0f && top_p > 0.0f && top_p <= 1.0f && repeat_penalty > 0.0f, "sampler settings out of range");
    auto s = std::make_unique<fz_sampler>();
    s->temperature = temperature;
    s->top_k = top_k;
    s->top_p = top_p;
    s->repeat_penalty = repeat_penalty;
    // Pcg32::new (src/sampler.rs:12-19): one step, add the seed, one step
    s->next_u32();
    s->state += seed;
    s->next_u32();
    *out = s.release();
  });
}

void fz_sampler_free(fz_sampler* s) { delete s; }

int fz_sampler_draws(const fz_sampler* s, uint64_t* draws) {
  return guard([&] {
    need(s && draws, "null argument");
    *draws = s->draws;
  });
}

int fz_sample_logits(fz_sampler* s, const float* logits, size_t n, const uint32_t* recent, size_t n_recent,
                     uint32_t* out) {
  return guard([&] {
    need(s && logits && out && n > 0 && (recent || n_recent == 0), "null argument");
    *out = sample_host(s, logits, n, recent, n_recent);
  });
}

int fz_sample(fz_model* m, fz_sampler* s, const uint32_t* recent, uint32_t n_recent, uint32_t* out) {
  return guard([&] {
    need(m && s && out && (recent || n_recent == 0), "null argument");
    need(n_recent <= 64, "at most 64 recent tokens (the reference's repeat window)");
    use_device(m);
    tp_gather_logits(m, m->stream);
    *out = sample_device(m, s, recent, n_recent);
  });
}

int fz_generate(fz_model* m, fz_kv* kv, fz_sampler* s, const uint32_t* prompt, uint32_t n_prompt, uint32_t max_new,
                const uint32_t* stop_ids, uint32_t n_stop, uint32_t* ids_out, uint32_t* n_out) {
  return guard([&] {
    need(m && kv && kv->m == m && s && prompt && n_prompt > 0 && ids_out && n_out, "null or mismatched handles");
    need(n_stop == 0 || stop_ids, "null stop ids");
    *n_out = 0;
    need((uint64_t)kv->len + n_prompt + (max_new ? max_new - 1 : 0) <= kv->max_ctx,
         "prompt (%u) + max tokens (%u) exceeds the cache (%u of %u used)", n_prompt, max_new, kv->len, kv->max_ctx);
    if (max_new == 0) return;
    auto check = [](int rc) {
      if (rc) throw Error(rc, fz::last_error());
    };
    if (s->greedy() && s->repeat_penalty == 1.0f) {
      // greedy: the device feeds each argmax back itself (fz_decode_greedy)
      uint32_t first = 0;
      check(fz_forward(m, kv, prompt, n_prompt, nullptr, &first));
      check(fz_decode_greedy(m, kv, first, max_new, stop_ids, n_stop, ids_out, nullptr, n_out));
      return;
    }
    std::vector<uint32_t> context(prompt, prompt + n_prompt);
    check(fz_forward(m, kv, prompt, n_prompt, nullptr, nullptr));
    uint32_t n = 0;
    for (uint32_t step = 0; step < max_new; step++) {
      const size_t window = context.size() > 64 ? context.size() - 64 : 0;  // repeat window (src/sampler.rs:74)
      uint32_t next = 0;
      check(fz_sample(m, s, context.data() + window, (uint32_t)(context.size() - window), &next));
      bool stop = false;
      for (uint32_t i = 0; i < n_stop; i++) stop |= stop_ids[i] == next;
      if (stop) break;
      ids_out[n++] = next;
      context.push_back(next);
      if (step + 1 == max_new) break;
      check(fz_forward(m, kv, &next, 1, nullptr, nullptr));
    }
    *n_out = n;
  });
}

int fz_step_profile(fz_model* m, fz_kv* kv, uint32_t first, uint32_t reps, double* ms, double* bytes,
                    uint32_t* launches) {
  return guard([&] {
    need(m && kv && kv->m == m && ms && bytes && launches, "null or mismatched handles");
    need(first < m->cfg.vocab, "token id %u out of range (vocab %u)", first, m->cfg.vocab);
    need((uint64_t)kv->len + reps <= kv->max_ctx, "context overflow: %u + %u > max_ctx %u", kv->len, reps, kv->max_ctx);
    use_device(m);
    cudaStream_t s = m->stream;
    struct Hook : OpHook {
      std::vector<cudaEvent_t> ev;
      std::vector<int> ops;
      cudaStream_t s;
      void at(int op, bool begin) override {
        cudaEvent_t e;
        CK(cudaEventCreate(&e));
        CK(cudaEventRecord(e, s));
        ev.push_back(e);
        if (begin) ops.push_back(op);
      }
      ~Hook() override {
        for (auto e : ev) cudaEventDestroy(e);
      }
    } hook;
    hook.s = s;
    for (int k = 0; k < FZ_OP_COUNT; k++) {
      ms[k] = 0;
      bytes[k] = 0;
      launches[k] = 0;
    }
    CK(cudaMemcpyAsync(kv->forced.p, &first, 4, cudaMemcpyHostToDevice, s));
    set_state(kv, kv->len, first, 1);
    for (uint32_t r = 0; r < reps; r++) record_step(kv, true, s, &hook);
    CK(cudaStreamSynchronize(s));
    for (size_t i = 0; i < hook.ops.size(); i++) {
      float t = 0;
      CK(cudaEventElapsedTime(&t, hook.ev[2 * i], hook.ev[2 * i + 1]));
      ms[hook.ops[i]] += t;
      launches[hook.ops[i]] += 1;
    }
    check_state(kv);
    for (uint32_t r = 0; r < reps; r++) step_bytes(m, kv, kv->len + r, bytes);
    kv->len += reps;
  });
}

int fz_selftest_exchange_timeout(int device, uint32_t limit_us) {
  return guard([&] {
    need(limit_us > 0, "zero wait limit");
    CK(cudaSetDevice(device));
    kernels_init();
    cudaStream_t s;
    CK(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking));
    struct Hold {
      cudaStream_t s;
      ~Hold() {
        cudaStreamSynchronize(s);
        cudaStreamDestroy(s);
      }
    } hold{s};
    // a 32 x 256 Q8_0 weight of zero bytes whose RMS-normalised input is the
    // exchanged residual of ranks {0, 1}; rank 1 never sends
    const uint32_t H = 256, R = 32;
    DevMat w;
    w.dtype = FZ_Q8_0;
    w.rows = R;
    w.cols = H;
    w.stride = dev_row_stride(FZ_Q8_0, H);
    DevBuf wb((uint64_t)R * w.stride + 256), xb(H * 4), nb(H * 4), yb(R * 4), arb(ar_buffer_bytes(H, 2)), base(16),
        st(sizeof(StepState));
    for (DevBuf* b : {&wb, &xb, &yb, &arb, &base, &st}) CK(cudaMemsetAsync(b->p, 0, b->n, s));
    std::vector<float> ones(H, 1.0f);
    CK(cudaMemcpyAsync(nb.p, ones.data(), H * 4, cudaMemcpyHostToDevice, s));
    w.ptr = wb.as<uint8_t>();
    GemvLaunch g;
    g.seg[0] = GemvSeg{w, nullptr, yb.as<float>()};
    g.x = xb.as<float>();
    g.norm_w = nb.as<float>();
    g.eps = 1e-6f;
    g.epilogue = EPI_STORE;
    g.state = st.as<StepState>();
    g.ar_peers.buf[0] = g.ar_peers.buf[1] = arb.as<float>();
    g.ar_w = 2;
    g.ar_rank = 0;
    g.ar_k = 0;
    g.ar_h = H;
    g.ar_base = base.as<uint32_t>();
    g.ar_pull = 1;
    g.ar_spin_ns = (uint64_t)limit_us * 1000;
    launch_gemv(g, s);
    StepState out{};
    CK(cudaMemcpyAsync(&out, st.p, sizeof out, cudaMemcpyDeviceToHost, s));
    CK(cudaStreamSynchronize(s));
    if (out.error == 7) fail(FZ_ETIMEOUT, "exchange wait ran out after %u us per word (as intended)", limit_us);
    fail(FZ_EINVAL, "the exchange wait did not run out (error word %u)", out.error);
  });
}

// ---- kernel-level entry points -------------------------------------------
int fz_weight_upload(uint32_t dtype, const void* raw, size_t nbytes, uint32_t d_out, uint32_t d_in, fz_weight** out) {
  return guard([&] {
    need(raw && out, "null argument");
    need(is_quant(dtype), "no fused matmul kernel for dtype %u", dtype);
    uint32_t be, bb;
    block_geom(dtype, &be, &bb);
    need(d_in % be == 0, "matmul: in dim %u not a multiple of %u", d_in, be);
    need(nbytes == gguf_bytes(dtype, d_out, d_in), "matmul: bad weight byte count");
    kernels_init();
    auto w = std::make_unique<fz_weight>();
    w->m.dtype = dtype;
    w->m.rows = d_out;
    w->m.cols = d_in;
    w->m.stride = dev_row_stride(dtype, d_in);
    w->m.gguf_bytes = nbytes;
    w->buf.alloc((uint64_t)d_out * w->m.stride + 256);
    CK(cudaMemset(w->buf.p, 0, w->buf.n));
    w->m.ptr = w->buf.as<uint8_t>();
    w->runs.alloc((uint64_t)runs_for(d_in) * 64);
    CK(cudaMemset(w->runs.p, 0, w->runs.n));
    {
      Uploader up(0, std::min<uint64_t>(nbytes + 16, 64ull << 20));
      upload_rows(dtype, (const uint8_t*)raw, d_out, d_in, w->m.ptr, up);
      up.finish();
    }
    *out = w.release();
  });
}

void fz_weight_free(fz_weight* w) { delete w; }

int fz_matmul_quant_dev(const fz_weight* w, const float* a_dev, uint32_t seq, float* out_dev, void* stream) {
  return guard([&] {
    need(w && a_dev && out_dev, "null argument");
    cudaStream_t s = (cudaStream_t)stream;
    if (seq >= PF_MIN && w->m.cols % 64 == 0 && !getenv("FURNACE_B200_NO_PREFILL_GEMM")) {
      // several rows: the tensor-core GEMM of the batched prefill
      prefill_init();
      const uint32_t rows = w->m.rows, cols = w->m.cols;
      DevBuf wh(wpanel_elems(rows, cols) * 2), wl(wpanel_elems(rows, cols) * 2);
      DevBuf xh(xpanel_elems(seq, cols) * 2), xl(xpanel_elems(seq, cols) * 2), err(16);
      DevBuf rexp((rows + 127) / 128 * 128), texp(seq + 16);
      for (DevBuf* b : {&wh, &wl, &xh, &xl, &err, &rexp, &texp}) CK(cudaMemsetAsync(b->p, 0, b->n, s));
      launch_wpanels(w->m, 0, rexp.as<int8_t>(), wh.p, wl.p, s);
      launch_xpanels(a_dev, cols, seq, cols, nullptr, 0.f, xh.p, xl.p, texp.as<int8_t>(), s);
      launch_qgemm(QgemmLaunch{wh.p, wl.p, xh.p, xl.p, rexp.as<int8_t>(), texp.as<int8_t>(), cols, rows, seq,
                               PE_STORE, out_dev, rows, nullptr, err.as<uint32_t>()},
                   s);
      uint32_t e = 0;
      CK(cudaMemcpyAsync(&e, err.p, 4, cudaMemcpyDeviceToHost, s));
      CK(cudaStreamSynchronize(s));
      if (e) fail(FZ_ETIMEOUT, "matmul: a bounded device wait ran out");
      return;
    }
    // widths up to 30720 convert the f32 input inside the GEMV; wider inputs
    // are converted to run records by a separate pass
    const bool direct = w->m.cols <= 30720;
    for (uint32_t i = 0; i < seq; i++) {
      GemvLaunch g;
      g.seg[0] = GemvSeg{w->m, nullptr, out_dev + (uint64_t)i * w->m.rows};
      if (direct) {
        g.x = a_dev + (uint64_t)i * w->m.cols;
      } else {
        launch_to_runs(a_dev + (uint64_t)i * w->m.cols, w->m.cols, w->runs.p, runs_for(w->m.cols), s);
        g.in_runs = w->runs.p;
      }
      g.epilogue = EPI_STORE;
      launch_gemv(g, s);
    }
  });
}

int fz_matmul_quant(const float* a, uint32_t seq, const void* raw, size_t nbytes, uint32_t d_out, uint32_t d_in,
                    uint32_t dtype, float* out) {
  fz_weight* w = nullptr;
  int rc = fz_weight_upload(dtype, raw, nbytes, d_out, d_in, &w);
  if (rc) return rc;
  rc = guard([&] {
    need(a && out, "null argument");
    DevBuf da((uint64_t)seq * d_in * 4), dout((uint64_t)seq * d_out * 4);
    CK(cudaMemcpy(da.p, a, (uint64_t)seq * d_in * 4, cudaMemcpyHostToDevice));
    int r = fz_matmul_quant_dev(w, da.as<float>(), seq, dout.as<float>(), nullptr);
    if (r) throw Error(r, fz::last_error());
    CK(cudaMemcpy(out, dout.p, (uint64_t)seq * d_out * 4, cudaMemcpyDeviceToHost));
  });
  fz_weight_free(w);
  return rc;
}

int fz_gemv(uint32_t dtype, const void* raw, uint32_t d_out, uint32_t d_in, const float* x, float* y) {
  uint64_t nbytes = 0;
  const int rc = guard([&] {
    uint32_t be, bb;
    need(block_geom(dtype, &be, &bb), "type %u is not implemented", dtype);
    need(d_in % be == 0, "d_in %u is not a multiple of the %u-element block", d_in, be);
    nbytes = gguf_bytes(dtype, d_out, d_in);
  });
  return rc ? rc : fz_matmul_quant(x, 1, raw, nbytes, d_out, d_in, dtype, y);
}

int fz_dequant(uint32_t dtype, const void* raw, size_t nbytes, size_t n, float* out) {
  return guard([&] {
    need(raw && out, "null argument");
    uint32_t be, bb;
    need(block_geom(dtype, &be, &bb), "dequantization for type %u is not implemented", dtype);
    if (dtype == FZ_F32) {
      need(nbytes == n * 4, "F32 data is %zu bytes, expected %zu", nbytes, n * 4);
      memcpy(out, raw, n * 4);
      return;
    }
    need(is_quant(dtype), "dequantization for type %u is not implemented", dtype);
    need(n % be == 0, "element count %zu is not a multiple of %u", n, be);
    need(nbytes == n / be * bb, "data is %zu bytes, expected %zu (%zu blocks of %u)", nbytes, n / be * bb, n / be, bb);
    // view the blob as rows of k blocks, k the largest divisor of the block
    // count that keeps a row within one chunk of the device layout
    uint64_t nblk = n / be, kmax = be == 256 ? 8 : 64, k = 1;
    for (uint64_t t = kmax; t >= 1; t--)
      if (nblk % t == 0) {
        k = t;
        break;
      }
    DevMat m;
    m.dtype = dtype;
    m.rows = (uint32_t)(nblk / k);
    m.cols = (uint32_t)(k * be);
    m.stride = dev_row_stride(dtype, m.cols);
    DevBuf raw_d(nbytes + 16), lay((uint64_t)m.rows * m.stride + 256), outd(n * 4 + 16);
    CK(cudaMemset(lay.p, 0, lay.n));
    CK(cudaMemcpy(raw_d.p, raw, nbytes, cudaMemcpyHostToDevice));
    launch_repack(dtype, raw_d.as<uint8_t>(), lay.as<uint8_t>(), 0, m.rows, m.rows, m.cols, 0);
    m.ptr = lay.as<uint8_t>();
    launch_dequant(m, 0, m.rows, outd.as<float>(), 0);
    CK(cudaMemcpy(out, outd.p, n * 4, cudaMemcpyDeviceToHost));
  });
}

}  // extern "C"
