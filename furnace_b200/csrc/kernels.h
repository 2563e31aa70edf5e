// Kernel launch interface (host side).  Device layouts and algorithms are
// described in kernels.cu.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>
#include <vector>

namespace fz {

// A matmul weight [rows, cols] resident in HBM in the device layout.
struct DevMat {
  uint32_t dtype = 0;
  uint32_t rows = 0, cols = 0;
  uint64_t stride = 0;      // bytes per row (multiple of 16)
  uint8_t* ptr = nullptr;   // device
  uint64_t gguf_bytes = 0;  // bytes of the same rows in GGUF encoding
};

// Device-layout row stride for `cols` elements of `dtype`.
uint64_t dev_row_stride(uint32_t dtype, uint32_t cols);

// Repack `rows` GGUF rows (raw, device memory) into the chunked device
// layout (layout.cuh) at dst.  Same bytes, different order.
// raw holds GGUF rows [r0, r0 + nrows) of a matrix of total_rows rows.
void launch_repack(uint32_t dtype, const uint8_t* raw, uint8_t* dst, uint32_t r0, uint32_t nrows, uint32_t total_rows,
                   uint32_t cols, cudaStream_t s);

// Dequantize device-layout rows [r0, r0+rows) of m to f32 [rows, cols],
// bit-exact with the reference's block decoders.
void launch_dequant(const DevMat& m, uint32_t r0, uint32_t rows, float* out, cudaStream_t s);

// Dynamic per-step scalars read by the kernels (so that one captured graph
// serves every position).
struct StepState {
  uint32_t pos;        // position of the token being processed
  uint32_t token;      // token id being processed
  uint32_t step;       // index into ids_out / forced
  uint32_t n_forced;   // tokens [0, n_forced) of `forced` are fed in order
  unsigned long long argmax_key;
  uint32_t error;      // nonzero: a kernel rejected its input (see kernels.cu)
  uint32_t pad[3];
};

enum GemvEpilogue : int { EPI_STORE = 0, EPI_RESID = 1, EPI_SWIGLU = 2, EPI_LOGITS = 3 };

// Step-kernel timeline record (see trace_install): one per CTA per launch.
enum TraceTag : uint32_t { TR_GEMV = 0, TR_ATTN = 8, TR_COMBINE = 9 };  // TR_GEMV + epilogue
struct TraceRec {
  uint32_t tag, cta, aux, pad;
  uint64_t t[6];
};
void trace_install(TraceRec* buf, uint32_t cap);
void trace_reset(cudaStream_t s);
uint32_t trace_count();

// Activation vectors travel between kernels as 64-byte run records (one per
// 16 elements, see kernels.cu); runs_for(cols) records cover `cols`.
uint32_t runs_for(uint32_t cols);
void launch_to_runs(const float* x, uint32_t cols, void* runs, uint32_t nruns, cudaStream_t s);

// Tensor-parallel exchange of the residual stream through peer memory (see
// kernels.cu): buf[q] is rank q's receive buffer of ar_buffer_bytes(H, W)
// bytes as mapped in this process (buf[rank] the local one, zeroed once).
constexpr int AR_MAX_RANKS = 8;
struct ArPeers {
  float* buf[AR_MAX_RANKS];
};
uint64_t ar_buffer_bytes(uint32_t H, uint32_t W);

// Up to 3 weight segments sharing one input vector (q|k|v).
struct GemvSeg {
  DevMat w;
  const float* bias;   // [rows] or null
  float* out;          // destination base for this segment (RESID: the residual, updated in place)
};

struct GemvLaunch {
  GemvSeg seg[3];
  int nseg = 1;
  const void* in_runs = nullptr;    // input as run records (written by the producing kernel), or
  const float* x = nullptr;         // input as f32 [cols], converted in the GEMV prologue,
  const float* norm_w = nullptr;    //   RMS-normalised with this weight when set
  float eps = 0.f;
  int epilogue = EPI_STORE;
  StepState* state = nullptr;       // EPI_LOGITS argmax key
  void* out_runs = nullptr;         // SWIGLU: records of the next GEMV's input
  const GemvLaunch* next = nullptr; // the next GEMV of the step (L2 prefetch)
  uint32_t idx_base = 0;            // EPI_LOGITS: global index of row 0 (vocab slice)
  // tensor parallelism, exchange k of the step (epoch *ar_base + k + 1):
  // ar_push: the RESID epilogue sends its rows' partial (plus x on rank 0)
  // to every rank instead of updating x; ar_pull: the f32 prologue sums the
  // W partials of every element as its input and writes its slice of x
  ArPeers ar_peers{};
  uint32_t ar_w = 0, ar_rank = 0, ar_k = 0, ar_h = 0;
  const uint32_t* ar_base = nullptr;
  int ar_push = 0, ar_pull = 0;
  uint64_t ar_spin_ns = 0;          // ar_pull wait limit (0: FURNACE_B200_WAIT_MS or 2 s)
};

void launch_gemv(const GemvLaunch& g, cudaStream_t s);
uint32_t gemv_ctas(const GemvLaunch& g);

// Embedding row of state->token dequantized to f32.
void launch_embed(const DevMat& emb, StepState* st, float* x, cudaStream_t s);

// Split-K attention over positions [0, state->pos] with RoPE on q and the new
// k, and the K/V append at pos.  Caches are laid out [n_kv][max_ctx][hd];
// rope_cs is [max_ctx][hd/2] of (cos, sin).
struct AttnLaunch {
  const float* qkv;      // [q | k | v] after bias
  const float* rope_cs;
  void* kcache;          // f32, or f16 when kv_f16
  void* vcache;
  float* ctx;            // [nh*hd]
  void* ctx_runs;        // run records of ctx (o_proj input)
  float* partials;       // attention_partial_floats(...) floats
  uint32_t n_heads, n_kv, hd, max_ctx, splits;
  StepState* state;
  uint32_t ctx_run0 = 0;  // run record index of ctx[0] in ctx_runs
  int kv_f16 = 0;         // cache elements are f16
};
void launch_attention(const AttnLaunch& a, cudaStream_t s);
uint32_t attention_splits(uint32_t n_kv);
uint64_t attention_partial_floats(uint32_t nh, uint32_t nkv, uint32_t hd, uint32_t splits);

// Step bookkeeping after the logits (argmax -> ids_out, next token, pos++;
// ar_base, when set, advances by ar_step: the step's exchanges).
void launch_finalize(StepState* st, const uint32_t* forced, uint32_t* ids_out, bool has_logits, cudaStream_t s,
                     uint32_t* ar_base = nullptr, uint32_t ar_step = 0);

int num_sms();
void kernels_init();
void attention_init();


// ---- sampling (src/sampler.rs) ------------------------------------------------
// Top k (k <= topk_max()) of the repeat-penalised, temperature-scaled logits as
// packed keys (orderable value << 32 | ~index), descending; recent: <= 64 ids.
void sampler_init();
uint32_t topk_max();
size_t topk_scratch_bytes(uint32_t V);
void launch_topk(const float* logits, uint32_t V, const uint32_t* recent, uint32_t nr, float pen, float temp,
                 uint32_t k, void* scratch, void* out, cudaStream_t s);

// ---- prefill on the tensor cores (prefill.cuh) -------------------------------
enum PrefillEpilogue : int { PE_STORE = 0, PE_RESID = 1, PE_SWIGLU = 2 };
struct QgemmLaunch {
  const void *ahi, *alo;  // weight panels (launch_wpanels)
  const void *bhi, *blo;  // token panels (launch_xpanels)
  const int8_t *rexp, *texp;  // their power-of-two row / token exponents
  uint32_t K, N, T;
  int epi;                // PE_*: out[t*ld + r] (+ bias[r]); += ; SwiGLU into out[t*ld + r/2]
  float* out;
  uint32_t ld;
  const float* bias;
  uint32_t* err;          // device word, nonzero if a bounded wait ran out
};
void prefill_init();
uint64_t wpanel_elems(uint32_t rows, uint32_t K);  // fp16 elements of one weight panel set
uint64_t xpanel_elems(uint32_t T, uint32_t K);
// rexp: one int8 exponent per panel row (rows padded to 128, padding zero)
void launch_wpanels(const DevMat& m, uint32_t row0, int8_t* rexp, void* hi, void* lo, cudaStream_t s);
void launch_xpanels(const float* x, uint32_t ld, uint32_t T, uint32_t K, const float* w, float eps, void* hi,
                    void* lo, int8_t* texp, cudaStream_t s);
void launch_qgemm(const QgemmLaunch& q, cudaStream_t s);
void launch_embed_rows(const DevMat& emb, const uint32_t* tokens, uint32_t T, float* x, uint32_t ld, cudaStream_t s);
void launch_prefill_attention(const float* qkv, uint32_t ldq, const float* rope_cs, void* kc, void* vc, bool kv_f16,
                              float* ctx, uint32_t ldc, uint32_t nh, uint32_t nkv, uint32_t hd, uint32_t max_ctx,
                              uint32_t pos0, uint32_t T, uint32_t* err, cudaStream_t s);

}  // namespace fz
