/* furnace.h -- C ABI of libfurnace_cuda.so, the B200 (sm_100a) implementation
 * of the furnace decode token loop.
 *
 * The reference (a Rust binary crate) has no FFI of its own; its internal
 * API is the boundary this library replaces.  Each entry point names the
 * reference function it stands in for (paths inside the furnace project).
 *
 * Conventions
 *   - Every call returns FZ_OK (0) or a nonzero FZ_E* status; fz_last_error()
 *     returns a thread-local message for the last failure on this thread.
 *     Where the reference panics on misuse (kv overflow, token >= vocab), the
 *     library returns FZ_EINVAL instead and leaves its state unchanged.
 *   - Handles are opaque.  The caller owns every host buffer it passes; the
 *     library owns all device memory and frees it in fz_*_free.
 *   - Matrices follow the reference convention: weights are [out, in] with
 *     each row a contiguous run of GGUF blocks, activations [seq, in] f32,
 *     outputs [seq, out] f32 (src/tensor.rs:1-10).
 *   - One model handle is used from one host thread at a time, like the
 *     reference's single caller thread (src/main.rs:162-270).
 */
#ifndef FURNACE_H
#define FURNACE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#pragma GCC visibility push(default)
#endif

enum {
  FZ_OK = 0,
  FZ_EINVAL = 1,   /* bad argument, shape or state (reference: assert!/ensure!) */
  FZ_EFORMAT = 2,  /* malformed or unsupported GGUF (reference: anyhow bail!) */
  FZ_EIO = 3,      /* cannot open / map the file */
  FZ_ECUDA = 4,    /* CUDA runtime or kernel error */
  FZ_ENOMEM = 5,   /* device allocation failed */
  FZ_ETIMEOUT = 6, /* a bounded device-side wait ran out */
  FZ_ESPACE = 7    /* output buffer too small: the size needed is reported, nothing was consumed */
};

/* ggml tensor types the decode path computes on (src/gguf.rs:180-201). */
enum { FZ_F32 = 0, FZ_F16 = 1, FZ_Q5_0 = 6, FZ_Q8_0 = 8, FZ_Q4_K = 12, FZ_Q6_K = 14 };

/* KV cache element types.  F32 is the reference's (src/model.rs:321-327);
 * F16 keeps binary16 elements, rounded to nearest even when appended (the
 * 8K-context cache of the 32B configuration: half the bytes per position). */
enum { FZ_KV_F32 = 0, FZ_KV_F16 = 1 };

typedef struct fz_file fz_file;   /* GgufFile (src/gguf.rs:297-304) */
typedef struct fz_model fz_model; /* Model (src/model.rs:511-517), resident in HBM */
typedef struct fz_kv fz_kv;       /* KvCache (src/model.rs:321-327), resident in HBM */

/* Config (src/model.rs:27-38). */
typedef struct fz_config {
  uint32_t n_layers, n_heads, n_kv_heads, hidden, ffn, head_dim;
  float rope_theta, rms_eps;
  uint32_t vocab, context_length;
} fz_config;

/* Tensor table entry (TensorInfo, src/gguf.rs:246-254). dims in ggml order. */
typedef struct fz_tensor_info {
  const char* name;
  uint32_t dtype;
  uint32_t n_dims;
  uint64_t dims[4];
  uint64_t offset;  /* relative to the data blob */
  uint64_t nbytes;  /* GGUF byte size of the tensor data */
} fz_tensor_info;

const char* fz_last_error(void);
/* Library version string, e.g. "furnace-b200 0.1 sm_100a". */
const char* fz_version(void);

/* ---- GGUF file (src/gguf.rs) ------------------------------------------ */
/* GgufFile::open (src/gguf.rs:366-380): mmap + parse with the reference's
 * checks (magic, version 2|3, bounds, power-of-two alignment). */
int fz_open(const char* path, fz_file** out);
/* Parse an in-memory GGUF image (parse, src/gguf.rs:315-363).  The bytes are
 * copied. */
int fz_open_bytes(const void* data, size_t n, fz_file** out);
void fz_file_free(fz_file* f);
/* version, tensor count, metadata count, data_start (src/gguf.rs:297-304) */
int fz_file_info(const fz_file* f, uint32_t* version, size_t* n_tensors, size_t* n_meta, size_t* data_start);
/* TensorInfo by index (src/gguf.rs:246-291). */
int fz_tensor_at(const fz_file* f, size_t i, fz_tensor_info* out);
/* GgufFile::tensor (src/gguf.rs:412-434): info plus a zero-copy pointer into
 * the mapping; fails when the data runs past the end of the file. */
int fz_tensor(const fz_file* f, const char* name, fz_tensor_info* info, const void** data);
/* meta_u32 / meta_f32 / meta_str (src/gguf.rs:382-401); meta_array length
 * (src/gguf.rs:403-408). */
int fz_meta_u32(const fz_file* f, const char* key, uint32_t* out);
int fz_meta_f32(const fz_file* f, const char* key, float* out);
int fz_meta_str(const fz_file* f, const char* key, const char** out);
int fz_meta_array_len(const fz_file* f, const char* key, size_t* out);
/* Config::from_gguf (src/model.rs:41-60). */
int fz_config_from_gguf(const fz_file* f, fz_config* out);

/* ---- Model and KV cache (src/model.rs) ----------------------------------- */
/* Model::load (src/model.rs:520-552) with use_f32 = false: uploads the raw
 * quantized blocks of every matmul weight to HBM (repacked into the
 * device layout, same byte count up to 16-byte row padding) and the norms
 * and biases as f32.  tp must be 1 in this release; device_ids may be NULL
 * (device 0). */
int fz_model_load(const fz_file* f, int tp, const int* device_ids, fz_model** out);
void fz_model_free(fz_model* m);
int fz_model_config(const fz_model* m, fz_config* out);
/* Bytes of weights resident on the device (Model::param_bytes,
 * src/model.rs:555-563), and the GGUF bytes one decode step streams. */
int fz_model_bytes(const fz_model* m, uint64_t* resident, uint64_t* streamed_per_token);
/* The CUDA stream (cudaStream_t) and device ordinal the model's work runs on,
 * so a caller can order its own work or record timing events on it. */
int fz_model_stream(const fz_model* m, void** stream, int* device);

/* ---- Tensor parallelism (one process per GPU, NCCL) ----------------------
 * No counterpart in the reference, which runs one process on one device: a
 * rank loads its share of what Model::load (src/model.rs:520-552) loads and
 * all ranks step together, each calling the same fz_forward /
 * fz_decode_greedy sequence with the same tokens.  Split (Megatron style):
 * q/k/v rows by query / KV head (attention and the KV cache stay local),
 * o_proj input columns by the rank's heads, gate/up rows and down input
 * columns by an FFN slice on 256-element boundaries, lm_head rows by
 * vocabulary slice; the residual stream is summed across ranks by an NCCL
 * all-reduce after o_proj and after down, and the greedy argmax by an
 * all-reduce (max) of the packed (logit, index) key.  Needs n_heads and
 * n_kv_heads divisible by world. */
typedef struct fz_tp_slice {
  uint32_t q_head0, q_heads;   /* query heads of this rank */
  uint32_t kv_head0, kv_heads; /* KV heads (and KV cache) of this rank */
  uint32_t o_col0, o_cols;     /* o_proj input columns = this rank's ctx */
  uint32_t ffn0, ffn_n;        /* FFN slice: gate/up rows, down input columns */
  uint32_t vocab0, vocab_n;    /* lm_head rows (all slices vocab_pad / world long) */
  uint32_t vocab_pad;
} fz_tp_slice;
int fz_tp_slice_of(const fz_config* c, int rank, int world, fz_tp_slice* out);
/* An NCCL unique id (n >= 128 bytes): made once (rank 0) and given to every
 * rank's fz_model_load_tp. */
int fz_tp_unique_id(void* id, size_t n);
/* Model::load for rank `rank` of `world` on CUDA device `device`; joins the
 * ranks' NCCL communicator (collective: every rank must call it). */
int fz_model_load_tp(const fz_file* f, int rank, int world, const void* id, size_t n, int device, fz_model** out);

/* KvCache::new (src/model.rs:330-339): max_ctx positions of kv_dtype
 * (FZ_KV_F32 or FZ_KV_F16) elements. */
int fz_kv_new(fz_model* m, uint32_t max_ctx, int kv_dtype, fz_kv** out);
/* Either order of fz_kv_free and fz_model_free is safe: freeing the model
 * releases its caches' device memory, and a cache handle of a freed model
 * then accepts only fz_kv_free and fz_kv_len (the rest return FZ_EINVAL). */
void fz_kv_free(fz_kv* kv);
/* KvCache::len (src/model.rs:324).  set_len rewinds (or restores) the
 * filled length; positions >= len are overwritten by later forwards. */
int fz_kv_len(const fz_kv* kv, uint32_t* len);
int fz_kv_set_len(fz_kv* kv, uint32_t len);
/* kv.len = 0: the cache reused for a new sequence. */
int fz_kv_reset(fz_kv* kv);
/* KvCache::bytes (src/model.rs:341-343): K and V bytes of this rank's cache. */
int fz_kv_bytes(const fz_kv* kv, uint64_t* bytes);
/* Copy layer `layer`'s cached K (which_v = 0) or V rows [0, n) to the host
 * as [n, n_kv_heads*head_dim] f32 (the reference's row layout); under tensor
 * parallelism, this rank's KV heads ([n, kv_heads*head_dim]). */
int fz_kv_read(const fz_kv* kv, uint32_t layer, int which_v, uint32_t n, float* out);

/* Model::forward_cached (src/model.rs:579-592): run the tokens at positions
 * kv.len .. kv.len+n, advance kv.len by n, and return the last position's
 * logits [vocab] (logits may be NULL) and their argmax (first max wins,
 * src/generate.rs:69-77; argmax may be NULL). */
int fz_forward(fz_model* m, fz_kv* kv, const uint32_t* tokens, uint32_t n, float* logits, uint32_t* argmax);

/* Model::forward_last (src/model.rs:569-575): the uncached forward over
 * positions 0 .. n-1 (the reference's --no-cache mode), returning the last
 * position's logits [vocab] (may be NULL) and their argmax (may be NULL).  It
 * runs forward_cached on a scratch cache of n positions, the same arithmetic
 * as the reference's full recompute up to summation order. */
int fz_forward_last(fz_model* m, const uint32_t* tokens, uint32_t n, float* logits, uint32_t* argmax);

/* Greedy decode loop of generate (src/generate.rs:122-141) at temperature 0
 * (Sampler::sample's argmax short-circuit, src/sampler.rs:92-94): starting
 * from `first` (the token sampled from the previous logits), runs up to
 * n_steps-1 decode forwards on the device with the token fed back on the
 * device, and writes the n_steps greedy ids to ids_out (ids_out[0] = first).
 * Stops early at any of stop_ids (not written), like src/generate.rs:125-127.
 * logits_out, when non-NULL, receives [n_steps-1, vocab]: the logits each
 * later id was taken from.  *n_out = ids written. */
int fz_decode_greedy(fz_model* m, fz_kv* kv, uint32_t first, uint32_t n_steps, const uint32_t* stop_ids,
                     uint32_t n_stop, uint32_t* ids_out, float* logits_out, uint32_t* n_out);

/* ---- Sampling (src/sampler.rs) and the generate loop (src/generate.rs) ---- */
typedef struct fz_sampler fz_sampler;
/* Sampler::new (src/sampler.rs:68-78): temperature (0 = greedy), top_k (0 =
 * off), top_p (1 = off), repeat_penalty (1 = off), PCG32 seed. */
int fz_sampler_new(float temperature, uint32_t top_k, float top_p, float repeat_penalty, uint64_t seed,
                   fz_sampler** out);
void fz_sampler_free(fz_sampler* s);
/* Sampler::draws (src/sampler.rs:82-84). */
int fz_sampler_draws(const fz_sampler* s, uint64_t* draws);
/* Sampler::sample (src/sampler.rs:86-108) on host logits [n] with the recent
 * context (the repeat window). */
int fz_sample_logits(fz_sampler* s, const float* logits, size_t n, const uint32_t* recent, size_t n_recent,
                     uint32_t* out);
/* Sampler::sample on the model's logits of its last forward, without copying
 * them back: penalty, temperature and top-k (k <= 64) run on the device and
 * only the k candidates reach the host, which finishes softmax, top-p and
 * the PCG32 draw in the reference's f32 order.  top_k = 0 or > 64 copies the
 * logits and samples on the host.  n_recent <= 64. */
int fz_sample(fz_model* m, fz_sampler* s, const uint32_t* recent, uint32_t n_recent, uint32_t* out);
/* generate (src/generate.rs:83-157) from kv->len: prefill the prompt, then
 * sample up to max_new ids (max_new - 1 decode forwards), stopping before any
 * stop id.  Greedy settings without a penalty use fz_decode_greedy's
 * device-fed loop.  *n_out = ids written. */
int fz_generate(fz_model* m, fz_kv* kv, fz_sampler* s, const uint32_t* prompt, uint32_t n_prompt, uint32_t max_new,
                const uint32_t* stop_ids, uint32_t n_stop, uint32_t* ids_out, uint32_t* n_out);

/* ---- Tokenizer (src/tokenizer.rs) and text helpers (src/generate.rs) -------
 * Host code.  Text is UTF-8 (len bytes, not terminated); ill-formed input
 * returns FZ_EINVAL.  Outputs go to caller buffers of `cap` elements: the
 * count or size is always reported, and FZ_ESPACE means it did not fit and
 * nothing was consumed. */
typedef struct fz_tokenizer fz_tokenizer;
/* Tokenizer::from_gguf (src/tokenizer.rs:67-90): tokenizer.ggml.model "gpt2",
 * tokenizer.ggml.pre "qwen2", tokens, token_type and merges from the file. */
int fz_tokenizer_from_gguf(const fz_file* f, fz_tokenizer** out);
/* Tokenizer::new (src/tokenizer.rs:92-138): n token strings (in the GPT-2
 * byte alphabet) with their gguf token types (3 control and 4 user-defined
 * are special), n_merges "left right" rules in rank order. */
int fz_tokenizer_new(const char* const* tokens, const int64_t* token_types, size_t n, const char* const* merges,
                     size_t n_merges, fz_tokenizer** out);
void fz_tokenizer_free(fz_tokenizer* t);
int fz_tokenizer_vocab_size(const fz_tokenizer* t, size_t* n);
/* Tokenizer::encode (src/tokenizer.rs:140-149): *n = number of ids. */
int fz_tokenizer_encode(const fz_tokenizer* t, const char* text, size_t len, uint32_t* ids, size_t cap, size_t* n);
/* Tokenizer::decode (src/tokenizer.rs:151-157): UTF-8, each maximal
 * ill-formed subsequence replaced by U+FFFD (String::from_utf8_lossy). */
int fz_tokenizer_decode(const fz_tokenizer* t, const uint32_t* ids, size_t n, char* out, size_t cap, size_t* len);
/* Tokenizer::token_bytes (src/tokenizer.rs:159-181): raw bytes of one token,
 * possibly a partial UTF-8 sequence. */
int fz_tokenizer_token_bytes(const fz_tokenizer* t, uint32_t id, char* out, size_t cap, size_t* len);
/* The qwen2 pre-tokenizer split (the pattern of src/tokenizer.rs:16, applied
 * by encode_ordinary, :215-232) alone: ends[i] = byte offset where chunk i
 * ends; *n = number of chunks. */
int fz_pretokenize(const char* text, size_t len, size_t* ends, size_t cap, size_t* n);
/* chat_template (src/generate.rs:13-21): the ChatML prompt around `prompt`. */
int fz_chat_template(const char* prompt, size_t len, char* out, size_t cap, size_t* out_len);
/* Utf8Stream (src/generate.rs:24-66): push token bytes, get the printable
 * prefix (an incomplete last character is held back); flush emits the rest
 * lossily. */
typedef struct fz_utf8_stream fz_utf8_stream;
int fz_utf8_stream_new(fz_utf8_stream** out);
void fz_utf8_stream_free(fz_utf8_stream* s);
int fz_utf8_stream_push(fz_utf8_stream* s, const void* bytes, size_t n, char* out, size_t cap, size_t* len);
int fz_utf8_stream_flush(fz_utf8_stream* s, char* out, size_t cap, size_t* len);

/* Per-op decode timings, the device counterpart of the reference's perf
 * counters (src/perf.rs:25-39, reported by `run --timings`): runs `reps`
 * greedy decode steps from kv.len WITHOUT the graph, with CUDA events around
 * every launch, and accumulates per op kind (FZ_OP_*) the milliseconds, the
 * launches and the algorithmic bytes (GGUF weight bytes, KV bytes, vectors).
 * Advances kv.len by reps like fz_decode_greedy. */
enum {
  FZ_OP_EMBED = 0, FZ_OP_QKV, FZ_OP_ROPE, FZ_OP_ATTN, FZ_OP_OPROJ, FZ_OP_GATEUP, FZ_OP_DOWN, FZ_OP_LMHEAD,
  FZ_OP_FINALIZE, FZ_OP_COUNT
};
int fz_step_profile(fz_model* m, fz_kv* kv, uint32_t first, uint32_t reps, double* ms, double* bytes,
                    uint32_t* launches);

/* ---- Kernel-level entry points (src/quant.rs) ---------------------------- */
/* quant::dequantize (src/quant.rs:261-281) on the device: raw GGUF blocks
 * -> f32, bit-exact with the reference. */
int fz_dequant(uint32_t dtype, const void* raw, size_t nbytes, size_t n, float* out);
/* quant::matmul_quant (src/quant.rs:170-193) on the device: a [seq, d_in]
 * times the quantized weight [d_out, d_in] (raw GGUF bytes) -> [seq, d_out]. */
int fz_matmul_quant(const float* a, uint32_t seq, const void* raw, size_t nbytes, uint32_t d_out, uint32_t d_in,
                    uint32_t dtype, float* out);
/* One row of quant::matmul_quant: y[d_out] = W x[d_in] with W the raw GGUF
 * blocks of a [d_out, d_in] weight (its size follows from the type). */
int fz_gemv(uint32_t dtype, const void* raw, uint32_t d_out, uint32_t d_in, const float* x, float* y);

/* ---- Failure detection self-test ---------------------------------------- */
/* No counterpart in the reference (which has no multi-rank path; it panics on
 * misuse, src/model.rs:348-352).  Runs, on `device`, one GEMV whose input is
 * the tensor-parallel exchange of a 2-rank group in which the peer never
 * writes: every word it polls stays stale, the bounded wait runs out after
 * `limit_us` microseconds per word, the kernel records error 7 and returns,
 * and this call reports FZ_ETIMEOUT (FZ_EINVAL if the wait did not run out).
 * The device stays usable.  The same limit applies to real exchanges through
 * FURNACE_B200_WAIT_MS (default 2000). */
int fz_selftest_exchange_timeout(int device, uint32_t limit_us);

/* ---- Device-resident variants (inputs already in HBM) --------------------- */
/* Same as fz_matmul_quant with device pointers and a CUDA stream
 * (cudaStream_t passed as void*).  `w_dev` must come from fz_weight_upload. */
typedef struct fz_weight fz_weight;
int fz_weight_upload(uint32_t dtype, const void* raw, size_t nbytes, uint32_t d_out, uint32_t d_in, fz_weight** out);
void fz_weight_free(fz_weight* w);
int fz_matmul_quant_dev(const fz_weight* w, const float* a_dev, uint32_t seq, float* out_dev, void* stream);

/* quant::dequantize on device buffers, allocating nothing.  No counterpart in
 * the reference (its dequantize, src/quant.rs:261-281, returns a new Vec):
 * fz_dequant allocates device buffers per call, which a caller whose device
 * memory is fully committed, or that must not stall other streams with a
 * device-wide cudaFree, cannot use.  raw_dev / out_dev are device pointers,
 * `stream` a cudaStream_t as void*; the work is queued on that stream.  The
 * repacked tensor lives in a fixed 8 MiB per-device scratch array: tensors
 * whose device layout exceeds it return FZ_EINVAL (any tensor of at most
 * 2 MiB of GGUF data fits).  Calls on one device whose work overlaps in time
 * race on the scratch.  The first call on each device looks up the scratch
 * address; make it before any stream capture begins. */
int fz_dequant_dev_noalloc(uint32_t dtype, const void* raw_dev, size_t nbytes, size_t n, float* out_dev,
                           void* stream);

#if defined(__GNUC__)
#pragma GCC visibility pop
#endif

#ifdef __cplusplus
}
#endif

#endif /* FURNACE_H */
