// Device code of the decode path (sm_100a).
//
// Weights live in the chunked device layout of layout.cuh.  The batch-1 GEMV
// streams them with the Tensor Memory Accelerator's bulk copies
// (cp.async.bulk, one elected producer thread, mbarrier completion) into a
// ring of shared-memory stages; eight consumer warps dot them with the
// activation vector.  The producer also keeps an L2 prefetch window
// (cp.async.bulk.prefetch.L2) ahead of the ring that runs on into the next
// kernel's weights, so HBM stays busy across the dependency gap between
// launches, and every launch is a programmatic dependent launch (PDL): a
// kernel's producer starts while its predecessor is still running and only
// the consumers wait (griddepcontrol.wait) for the predecessor's output.
//
// Activations enter the dot products as 24-bit fixed point: each run of 16
// elements shares one power-of-two scale and every element is split into
// three signed 8-bit limbs, so the quantized weights (4/5/6/8-bit integers)
// multiply them with dp4a.  The fixed-point rounding (<= 2^-23 of the run's
// largest magnitude) is below f32 rounding of the sums; the GEMV parity bar
// is 1e-4 relative.
//
// Dequantization (fz_dequant, the embedding row) is bit-exact with the
// reference block decoders (src/quant.rs:17-133): same integer unpack, same
// f32 products in the same order, no contraction (__fmul_rn/__fsub_rn).

#include <cuda_fp16.h>

#include <cstdio>
#include <utility>

#include "fz_internal.h"
#include "kernels.h"
#include "layout.cuh"

namespace fz {

#define CK(x)                                                                               \
  do {                                                                                      \
    cudaError_t e_ = (x);                                                                   \
    if (e_ != cudaSuccess) fail(FZ_ECUDA, "%s failed: %s", #x, cudaGetErrorString(e_));     \
  } while (0)

int num_sms() {
  static int n = 0;
  if (!n) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = 148;
  }
  return n;
}

uint64_t dev_row_stride(uint32_t dtype, uint32_t cols) { return lay_row_stride(dtype, cols); }

// ---------------------------------------------------------------------------
// small PTX helpers
// ---------------------------------------------------------------------------
__device__ __forceinline__ float h2f(uint32_t bits16) {
  return __half2float(__ushort_as_half((unsigned short)(bits16 & 0xffff)));
}
__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait: false once ~2^31 cycles (about a second) have passed.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
  if (mbar_try(bar, parity)) return true;
  long long t0 = clock64();
  while (!mbar_try(bar, parity))
    if (clock64() - t0 > (1ll << 31)) return false;
  return true;
}
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar, uint64_t pol) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(pol)
      : "memory");
}
__device__ __forceinline__ void bulk_prefetch(const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}
__device__ __forceinline__ uint64_t policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ void fence_barrier_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
__device__ __forceinline__ void named_sync(int id, int n) { asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory"); }

__device__ __forceinline__ uint4 lds128(const uint8_t* p) { return *reinterpret_cast<const uint4*>(p); }
__device__ __forceinline__ uint2 lds64(const uint8_t* p) { return *reinterpret_cast<const uint2*>(p); }
__device__ __forceinline__ uint32_t lds32(const uint8_t* p) { return *reinterpret_cast<const uint32_t*>(p); }
__device__ __forceinline__ uint32_t lds16(const uint8_t* p) { return *reinterpret_cast<const unsigned short*>(p); }

// ---------------------------------------------------------------------------
// Repack GGUF rows into the chunked layout.  One thread per (row, unit).
// ---------------------------------------------------------------------------
// raw holds GGUF rows [r0, r0 + nrows) of a matrix of total_rows rows; dst is
// the matrix base.
__global__ void k_repack(uint32_t dt, const uint8_t* __restrict__ raw, uint8_t* __restrict__ dst, uint32_t r0,
                         uint32_t nrows, uint32_t total_rows, uint32_t cols) {
  uint32_t U = (cols + 63) / 64;
  uint64_t idx = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (uint64_t)nrows * U) return;
  uint64_t r = idx / U;
  uint32_t u = (uint32_t)(idx % U);
  uint32_t c = lay_chunk_of(dt, cols, u);
  uint32_t cu0 = lay_cu0(dt, cols, c), nu = lay_cu0(dt, cols, c + 1) - cu0, lu = u - cu0;
  uint8_t* ch = dst + lay_tile_off(dt, cols, total_rows, r0 + (uint32_t)r, c);
  if (dt == FZ_Q4_K) {
    const uint8_t* src = raw + r * (cols / 256) * 144 + (uint64_t)(u >> 2) * 144;
    uint8_t* b = ch + 144 * (lu >> 2);
    uint32_t j = u & 3;  // each of the 4 units copies 36 bytes of its super-block
    for (int i = 0; i < 36; i++) b[36 * j + i] = src[36 * j + i];
  } else if (dt == FZ_Q6_K) {
    const uint8_t* src = raw + r * (cols / 256) * 210 + (uint64_t)(u >> 2) * 210;
    uint8_t* body = ch + 208 * (lu >> 2);
    uint32_t uu = u & 3, h = uu >> 1, is = uu & 1, l0 = 16 * is;
    for (int i = 0; i < 16; i++) {
      body[48 * uu + i] = src[64 * h + l0 + i];             // ql run a (groups 0, 2)
      body[48 * uu + 16 + i] = src[64 * h + 32 + l0 + i];   // ql run b (groups 1, 3)
      body[48 * uu + 32 + i] = src[128 + 32 * h + l0 + i];  // qh run
    }
    const uint8_t* sc = src + 192;
    body[192 + 4 * uu + 0] = sc[8 * h + is];      // group 0
    body[192 + 4 * uu + 1] = sc[8 * h + is + 4];  // group 2
    body[192 + 4 * uu + 2] = sc[8 * h + is + 2];  // group 1
    body[192 + 4 * uu + 3] = sc[8 * h + is + 6];  // group 3
    if (uu == 0) {
      uint8_t* d = ch + 208 * (nu >> 2) + 2 * (lu >> 2);
      d[0] = src[208];
      d[1] = src[209];
    }
  } else {
    uint32_t nb = cols / 32;
    for (uint32_t k = 0; k < 2; k++) {
      uint32_t blk = 2 * u + k;
      if (blk >= nb) break;
      if (dt == FZ_Q8_0) {
        const uint8_t* src = raw + (r * nb + blk) * 34;
        for (int i = 0; i < 32; i++) ch[64 * lu + 32 * k + i] = src[2 + i];
        ch[64 * nu + 4 * lu + 2 * k] = src[0];
        ch[64 * nu + 4 * lu + 2 * k + 1] = src[1];
      } else {
        const uint8_t* src = raw + (r * nb + blk) * 22;
        for (int i = 0; i < 16; i++) ch[32 * lu + 16 * k + i] = src[6 + i];
        for (int i = 0; i < 4; i++) ch[32 * nu + 8 * lu + 4 * k + i] = src[2 + i];
        uint32_t doff = 32 * nu + round16u(8 * nu) + 4 * lu + 2 * k;
        ch[doff] = src[0];
        ch[doff + 1] = src[1];
      }
    }
  }
}

void launch_repack(uint32_t dtype, const uint8_t* raw, uint8_t* dst, uint32_t r0, uint32_t nrows, uint32_t total_rows,
                   uint32_t cols, cudaStream_t s) {
  uint64_t n = (uint64_t)nrows * ((cols + 63) / 64);
  if (!n) return;
  k_repack<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(dtype, raw, dst, r0, nrows, total_rows, cols);
  CK(cudaGetLastError());
}

// ---------------------------------------------------------------------------
// Exact dequantization of one 64-element unit of a chunked row
// (src/quant.rs:35-39, 53-63, 78-109, 114-133).
// ---------------------------------------------------------------------------
__device__ void dequant_unit(uint32_t dt, const uint8_t* base, uint32_t rows, uint32_t r, uint32_t cols, uint32_t u,
                             float* o) {
  uint32_t c = lay_chunk_of(dt, cols, u);
  uint32_t cu0 = lay_cu0(dt, cols, c), nu = lay_cu0(dt, cols, c + 1) - cu0, lu = u - cu0;
  const uint8_t* ch = base + lay_tile_off(dt, cols, rows, r, c);
  if (dt == FZ_Q4_K) {
    uint32_t sb = u >> 2, j64 = u & 3;
    const uint8_t* blk = ch + 144 * (lu >> 2);
    float d = h2f(blk[0] | (blk[1] << 8)), dmin = h2f(blk[2] | (blk[3] << 8));
    const uint8_t* s = blk + 4;
    float scv[2], mv[2];
    for (int t = 0; t < 2; t++) {
      int j = 2 * j64 + t;
      uint32_t sc, m;
      if (j < 4) {
        sc = s[j] & 63;
        m = s[j + 4] & 63;
      } else {
        sc = (s[j + 4] & 0x0F) | ((s[j - 4] >> 6) << 4);
        m = (s[j + 4] >> 4) | ((s[j] >> 6) << 4);
      }
      scv[t] = (float)sc;
      mv[t] = (float)m;
    }
    float d1 = __fmul_rn(d, scv[0]), min1 = __fmul_rn(dmin, mv[0]);
    float d2 = __fmul_rn(d, scv[1]), min2 = __fmul_rn(dmin, mv[1]);
    const uint8_t* q = blk + 16 + 32 * j64;
    float* oa = o + 256 * sb + 64 * j64;
    for (int l = 0; l < 32; l++) {
      oa[l] = __fsub_rn(__fmul_rn(d1, (float)(q[l] & 0x0F)), min1);
      oa[32 + l] = __fsub_rn(__fmul_rn(d2, (float)(q[l] >> 4)), min2);
    }
  } else if (dt == FZ_Q6_K) {
    uint32_t sb = u >> 2, uu = u & 3, h = uu >> 1, l0 = (uu & 1) << 4;
    const uint8_t* body = ch + 208 * (lu >> 2);
    const uint8_t* dp = ch + 208 * (nu >> 2) + 2 * (lu >> 2);
    float d = h2f(dp[0] | (dp[1] << 8));
    const uint8_t* qh = body + 48 * uu + 32;
    const int scpos[4] = {0, 2, 1, 3};
    for (int g = 0; g < 4; g++) {
      const uint8_t* ql = body + 48 * uu + 16 * (g & 1);
      float sc = (float)(int8_t)body[192 + 4 * uu + scpos[g]];
      float ds = __fmul_rn(d, sc);
      int sh = g >= 2 ? 4 : 0;
      float* og = o + 256 * sb + 128 * h + 32 * g + l0;
      for (int i = 0; i < 16; i++) {
        int q = (int)(((ql[i] >> sh) & 0x0F) | (((qh[i] >> (2 * g)) & 3) << 4)) - 32;
        og[i] = __fmul_rn(ds, (float)q);
      }
    }
  } else {
    uint32_t nb = cols / 32;
    for (uint32_t k = 0; k < 2; k++) {
      uint32_t blk = 2 * u + k;
      if (blk >= nb) break;
      float* ob = o + 32 * blk;
      if (dt == FZ_Q8_0) {
        const uint8_t* dp = ch + 64 * nu + 4 * lu + 2 * k;
        float d = h2f(dp[0] | (dp[1] << 8));
        const uint8_t* q = ch + 64 * lu + 32 * k;
        for (int i = 0; i < 32; i++) ob[i] = __fmul_rn(d, (float)(int8_t)q[i]);
      } else {
        const uint8_t* qs = ch + 32 * lu + 16 * k;
        const uint8_t* hp = ch + 32 * nu + 8 * lu + 4 * k;
        uint32_t qh = hp[0] | (hp[1] << 8) | (hp[2] << 16) | ((uint32_t)hp[3] << 24);
        const uint8_t* dp = ch + 32 * nu + round16u(8 * nu) + 4 * lu + 2 * k;
        float d = h2f(dp[0] | (dp[1] << 8));
        for (int j = 0; j < 16; j++) {
          uint32_t hi0 = ((qh >> j) & 1) << 4, hi1 = ((qh >> (j + 16)) & 1) << 4;
          ob[j] = __fmul_rn(d, (float)((int)((qs[j] & 0x0F) | hi0) - 16));
          ob[j + 16] = __fmul_rn(d, (float)((int)((qs[j] >> 4) | hi1) - 16));
        }
      }
    }
  }
}

__global__ void k_dequant(uint32_t dt, const uint8_t* __restrict__ base, uint32_t total_rows, uint32_t cols, uint32_t r0,
                          uint32_t rows, float* __restrict__ out) {
  uint32_t U = (cols + 63) / 64;
  uint64_t idx = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (uint64_t)rows * U) return;
  uint64_t r = idx / U;
  uint32_t u = (uint32_t)(idx % U);
  dequant_unit(dt, base, total_rows, r0 + (uint32_t)r, cols, u, out + r * cols);
}

void launch_dequant(const DevMat& m, uint32_t r0, uint32_t rows, float* out, cudaStream_t s) {
  uint64_t n = (uint64_t)rows * ((m.cols + 63) / 64);
  if (!n) return;
  k_dequant<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(m.dtype, m.ptr, m.rows, m.cols, r0, rows, out);
  CK(cudaGetLastError());
}

// ---------------------------------------------------------------------------
// Launch helper: every kernel of the step is a programmatic dependent launch.
// ---------------------------------------------------------------------------
template <class... KArgs, class... Args>
static void launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  CK(cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...));
}

// Embedding lookup of state->token (src/model.rs:482-506): one dequantized row.
__global__ void k_embed(uint32_t dt, const uint8_t* __restrict__ base, uint32_t cols, uint32_t vocab,
                        StepState* __restrict__ st, float* __restrict__ x) {
  pdl_trigger();
  pdl_wait();
  uint32_t tok = st->token;
  uint32_t u = blockIdx.x * blockDim.x + threadIdx.x;
  if (u >= (cols + 63) / 64) return;
  if (tok >= vocab) {
    // the host validates ids before they reach the device; this is a guard
    for (uint32_t i = 64 * u; i < 64 * u + 64 && i < cols; i++) x[i] = 0.f;
    st->error = 1;
    return;
  }
  dequant_unit(dt, base, vocab, tok, cols, u, x);
}

void launch_embed(const DevMat& emb, StepState* st, float* x, cudaStream_t s) {
  uint32_t units = (emb.cols + 63) / 64;
  launch_pdl(k_embed, dim3((units + 63) / 64), dim3(64), 0, s, emb.dtype, (const uint8_t*)emb.ptr, emb.cols,
             emb.rows, st, x);
}

// ---------------------------------------------------------------------------
// GEMV
// ---------------------------------------------------------------------------
constexpr int GV_CWARPS = 15;                      // consumer warps (16 warps/CTA incl. producer)
constexpr int GV_RPW = 2;                          // rows per consumer warp per stage
constexpr int GV_ROWS = GV_CWARPS * GV_RPW;        // rows per stage
constexpr int GV_THREADS = (GV_CWARPS + 1) * 32;   // + one producer warp
constexpr int GV_MAX_SLOTS = 8;
constexpr int GV_MAX_CH = 32;                      // chunks per row (cols <= 65536)

struct GvSeg {
  const uint8_t* w;
  uint32_t rows, dtype, cols;
  const float* bias;
  float* out;
  uint32_t cta_begin, cta_end;
};

struct GvNext {
  GvSeg seg[3];
  int nseg;
  uint32_t budget;  // bytes per CTA to prefetch from the next kernel's stream
};

struct GvParams {
  GvSeg seg[3];
  int nseg;
  uint32_t cols;
  const float* x;
  const float* norm_w;
  float eps;
  int prologue, epilogue;
  StepState* state;
  uint32_t slots, slot_bytes, max_rows;
  uint32_t pf_ahead;
  GvNext next;
};

// This CTA's row range within its segment (even boundaries for gate/up pairs).
__device__ __forceinline__ void cta_rows(const GvSeg& s, uint32_t b, uint32_t* r0, uint32_t* r1) {
  uint32_t n = s.cta_end - s.cta_begin, lb = b - s.cta_begin, half = s.rows / 2;
  if (s.rows & 1) {
    *r0 = (uint32_t)((uint64_t)s.rows * lb / n);
    *r1 = (uint32_t)((uint64_t)s.rows * (lb + 1) / n);
  } else {
    *r0 = 2 * (uint32_t)((uint64_t)half * lb / n);
    *r1 = 2 * (uint32_t)((uint64_t)half * (lb + 1) / n);
  }
}

__device__ __forceinline__ int seg_of(const GvSeg* seg, int nseg, uint32_t b) {
  int i = 0;
  while (i + 1 < nseg && b >= seg[i].cta_end) i++;
  return i;
}

// The (chunk-major) stage sequence of one CTA of one GEMV launch.  Stage
// (c, k) covers chunk c of rows [r0 + k*GV_ROWS, ...): one contiguous range of
// the chunk plane.
struct StageIter {
  const GvSeg* s;
  uint32_t r0, r1, nrb, nch, cols, dt;
  uint32_t n_stages;
  __device__ void init(const GvSeg* seg, int nseg, uint32_t b) {
    n_stages = 0;
    nch = 0;
    nrb = 0;
    r0 = r1 = 0;
    s = nullptr;
    if (nseg <= 0) return;
    int si = seg_of(seg, nseg, b);
    s = &seg[si];
    if (b < s->cta_begin || b >= s->cta_end) return;
    cta_rows(*s, b, &r0, &r1);
    cols = s->cols;
    dt = s->dtype;
    nch = lay_nch(cols);
    nrb = (r1 - r0 + GV_ROWS - 1) / GV_ROWS;
    n_stages = nch * nrb;
  }
};

// Per-chunk geometry of the CTA's matrix, computed once per CTA.
struct ChunkInfo {
  uint32_t cu0, nu, tb;
  uint32_t pad;
  const uint8_t* plane;  // w + rows * chunk_off(c)
};

__device__ __forceinline__ void chunk_info(const StageIter& it, uint32_t c, ChunkInfo* ci) {
  uint32_t u0 = lay_cu0(it.dt, it.cols, c), u1 = lay_cu0(it.dt, it.cols, c + 1);
  ci->cu0 = u0;
  ci->nu = u1 - u0;
  ci->tb = lay_chunk_bytes(it.dt, u1 - u0);
  ci->plane = it.s->w + (uint64_t)it.s->rows * lay_chunk_off(it.dt, it.cols, c);
}

// ---- dot-product helpers ----------------------------------------------------
__device__ __forceinline__ int dp4a_us(uint32_t a, uint32_t b, int c) {
  int d;
  asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
__device__ __forceinline__ int dp4a_ss(uint32_t a, uint32_t b, int c) {
  int d;
  asm("dp4a.s32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

struct XRun {  // one 16-element activation run in limb form
  uint4 a, b, c;
  float scale, sum;
};

// sum_i q_i * X_i for 16 unsigned quants of <= 5 bits as one f32, the limbs
// combined in integer arithmetic (|total| < 2^31 for |limb a| <= 65).
__device__ __forceinline__ float dot_u_int(const uint32_t* q, const XRun& x) {
  int A = dp4a_us(q[0], x.a.x, 0), B = dp4a_us(q[0], x.b.x, 0), C = dp4a_us(q[0], x.c.x, 0);
  A = dp4a_us(q[1], x.a.y, A);
  B = dp4a_us(q[1], x.b.y, B);
  C = dp4a_us(q[1], x.c.y, C);
  A = dp4a_us(q[2], x.a.z, A);
  B = dp4a_us(q[2], x.b.z, B);
  C = dp4a_us(q[2], x.c.z, C);
  A = dp4a_us(q[3], x.a.w, A);
  B = dp4a_us(q[3], x.b.w, B);
  C = dp4a_us(q[3], x.c.w, C);
  return (float)(A * 65536 + B * 256 + C);
}
// Same with the limb sums combined in f32 (6- and 8-bit quants).
template <bool SIGNED>
__device__ __forceinline__ float dot_f(const uint32_t* q, const XRun& x) {
  int A, B, C;
  if (SIGNED) {
    A = dp4a_ss(q[0], x.a.x, 0);
    B = dp4a_ss(q[0], x.b.x, 0);
    C = dp4a_ss(q[0], x.c.x, 0);
    A = dp4a_ss(q[1], x.a.y, A);
    B = dp4a_ss(q[1], x.b.y, B);
    C = dp4a_ss(q[1], x.c.y, C);
    A = dp4a_ss(q[2], x.a.z, A);
    B = dp4a_ss(q[2], x.b.z, B);
    C = dp4a_ss(q[2], x.c.z, C);
    A = dp4a_ss(q[3], x.a.w, A);
    B = dp4a_ss(q[3], x.b.w, B);
    C = dp4a_ss(q[3], x.c.w, C);
  } else {
    A = dp4a_us(q[0], x.a.x, 0);
    B = dp4a_us(q[0], x.b.x, 0);
    C = dp4a_us(q[0], x.c.x, 0);
    A = dp4a_us(q[1], x.a.y, A);
    B = dp4a_us(q[1], x.b.y, B);
    C = dp4a_us(q[1], x.c.y, C);
    A = dp4a_us(q[2], x.a.z, A);
    B = dp4a_us(q[2], x.b.z, B);
    C = dp4a_us(q[2], x.c.z, C);
    A = dp4a_us(q[3], x.a.w, A);
    B = dp4a_us(q[3], x.b.w, B);
    C = dp4a_us(q[3], x.c.w, C);
  }
  return fmaf((float)A, 65536.0f, fmaf((float)B, 256.0f, (float)C));
}

// Dot of one 64-element unit of one row (tile row at `tp`, unit lu of a
// chunk of nu units) with the unit's four activation runs.
template <uint32_t DT>
__device__ __forceinline__ float unit_dot(const uint8_t* tp, uint32_t lu, uint32_t nu, const XRun* x) {
  constexpr uint32_t M4 = 0x0F0F0F0Fu, M30 = 0x30303030u;
  if (DT == FZ_Q4_K) {
    const uint8_t* blk = tp + 144 * (lu >> 2);
    uint32_t j64 = lu & 3;
    uint4 hdr = lds128(blk);
    uint4 q0 = lds128(blk + 16 + 32 * j64), q1 = lds128(blk + 32 + 32 * j64);
    // the 8 six-bit (scale, min) pairs as bytes (src/quant.rs:78-88):
    // sub-blocks 0-3 in the low 6 bits of bytes 0-3 / 4-7, sub-blocks 4-7
    // split between bytes 8-11 and the top 2 bits of bytes 0-7
    const uint32_t sc_lo = hdr.y & 0x3F3F3F3Fu, m_lo = hdr.z & 0x3F3F3F3Fu;
    const uint32_t sc_hi = (hdr.w & 0x0F0F0F0Fu) | ((hdr.y >> 2) & 0x30303030u);
    const uint32_t m_hi = ((hdr.w >> 4) & 0x0F0F0F0Fu) | ((hdr.z >> 2) & 0x30303030u);
    const uint32_t scw = j64 < 2 ? sc_lo : sc_hi, mw = j64 < 2 ? m_lo : m_hi;
    const uint32_t sh = 16 * (j64 & 1);
    const uint32_t sca = (scw >> sh) & 0xff, scb = (scw >> (sh + 8)) & 0xff;
    const uint32_t ma = (mw >> sh) & 0xff, mb = (mw >> (sh + 8)) & 0xff;
    uint32_t l0[4] = {q0.x & M4, q0.y & M4, q0.z & M4, q0.w & M4};
    uint32_t l1[4] = {q1.x & M4, q1.y & M4, q1.z & M4, q1.w & M4};
    uint32_t h0[4] = {(q0.x >> 4) & M4, (q0.y >> 4) & M4, (q0.z >> 4) & M4, (q0.w >> 4) & M4};
    uint32_t h1[4] = {(q1.x >> 4) & M4, (q1.y >> 4) & M4, (q1.z >> 4) & M4, (q1.w >> 4) & M4};
    float sa = dot_u_int(l0, x[0]) * x[0].scale + dot_u_int(l1, x[1]) * x[1].scale;
    float sbv = dot_u_int(h0, x[2]) * x[2].scale + dot_u_int(h1, x[3]) * x[3].scale;
    float d = h2f(hdr.x), dmin = h2f(hdr.x >> 16);
    return d * ((float)sca * sa + (float)scb * sbv) -
           dmin * ((float)ma * (x[0].sum + x[1].sum) + (float)mb * (x[2].sum + x[3].sum));
  } else if (DT == FZ_Q6_K) {
    const uint8_t* body = tp + 208 * (lu >> 2);
    uint32_t uu = lu & 3;
    uint4 qa = lds128(body + 48 * uu), qb = lds128(body + 48 * uu + 16), qh = lds128(body + 48 * uu + 32);
    uint32_t sc4 = lds32(body + 192 + 4 * uu);
    float d = h2f(lds16(tp + 208 * (nu >> 2) + 2 * (lu >> 2)));
    const uint32_t qav[4] = {qa.x, qa.y, qa.z, qa.w}, qbv[4] = {qb.x, qb.y, qb.z, qb.w};
    const uint32_t qhv[4] = {qh.x, qh.y, qh.z, qh.w};
    uint32_t g0[4], g1[4], g2[4], g3[4];
#pragma unroll
    for (int k = 0; k < 4; k++) {
      g0[k] = (qav[k] & M4) | ((qhv[k] << 4) & M30);
      g1[k] = (qbv[k] & M4) | ((qhv[k] << 2) & M30);
      g2[k] = ((qav[k] >> 4) & M4) | (qhv[k] & M30);
      g3[k] = ((qbv[k] >> 4) & M4) | ((qhv[k] >> 2) & M30);
    }
    float s0 = fmaf(dot_f<false>(g0, x[0]), x[0].scale, -32.0f * x[0].sum);
    float s1 = fmaf(dot_f<false>(g1, x[1]), x[1].scale, -32.0f * x[1].sum);
    float s2 = fmaf(dot_f<false>(g2, x[2]), x[2].scale, -32.0f * x[2].sum);
    float s3 = fmaf(dot_f<false>(g3, x[3]), x[3].scale, -32.0f * x[3].sum);
    float c0 = (float)(int8_t)(sc4 & 0xff), c2 = (float)(int8_t)((sc4 >> 8) & 0xff);
    float c1 = (float)(int8_t)((sc4 >> 16) & 0xff), c3 = (float)(int8_t)(sc4 >> 24);
    return d * (c0 * s0 + c1 * s1 + c2 * s2 + c3 * s3);
  } else if (DT == FZ_Q8_0) {
    const uint8_t* q = tp + 64 * lu;
    uint4 w0 = lds128(q), w1 = lds128(q + 16), w2 = lds128(q + 32), w3 = lds128(q + 48);
    uint32_t dd = lds32(tp + 64 * nu + 4 * lu);
    const uint32_t a0[4] = {w0.x, w0.y, w0.z, w0.w}, a1[4] = {w1.x, w1.y, w1.z, w1.w};
    const uint32_t a2[4] = {w2.x, w2.y, w2.z, w2.w}, a3[4] = {w3.x, w3.y, w3.z, w3.w};
    float s01 = dot_f<true>(a0, x[0]) * x[0].scale + dot_f<true>(a1, x[1]) * x[1].scale;
    float s23 = dot_f<true>(a2, x[2]) * x[2].scale + dot_f<true>(a3, x[3]) * x[3].scale;
    return h2f(dd) * s01 + h2f(dd >> 16) * s23;
  } else {  // Q5_0
    uint4 s0 = lds128(tp + 32 * lu), s1 = lds128(tp + 32 * lu + 16);
    uint2 qh = lds64(tp + 32 * nu + 8 * lu);
    uint32_t dd = lds32(tp + 32 * nu + round16u(8 * nu) + 4 * lu);
    const uint32_t sv0[4] = {s0.x, s0.y, s0.z, s0.w}, sv1[4] = {s1.x, s1.y, s1.z, s1.w};
    uint32_t c0[4], c1[4], c2[4], c3[4];
#pragma unroll
    for (int k = 0; k < 4; k++) {
      // spread 4 high bits into bit 4 of 4 bytes
      uint32_t h00 = ((((qh.x >> (4 * k)) & 15u) * 0x00204081u) & 0x01010101u) << 4;
      uint32_t h01 = ((((qh.x >> (16 + 4 * k)) & 15u) * 0x00204081u) & 0x01010101u) << 4;
      uint32_t h10 = ((((qh.y >> (4 * k)) & 15u) * 0x00204081u) & 0x01010101u) << 4;
      uint32_t h11 = ((((qh.y >> (16 + 4 * k)) & 15u) * 0x00204081u) & 0x01010101u) << 4;
      c0[k] = (sv0[k] & M4) | h00;
      c1[k] = ((sv0[k] >> 4) & M4) | h01;
      c2[k] = (sv1[k] & M4) | h10;
      c3[k] = ((sv1[k] >> 4) & M4) | h11;
    }
    float t0 = fmaf(dot_u_int(c0, x[0]), x[0].scale, -16.0f * x[0].sum);
    float t1 = fmaf(dot_u_int(c1, x[1]), x[1].scale, -16.0f * x[1].sum);
    float t2 = fmaf(dot_u_int(c2, x[2]), x[2].scale, -16.0f * x[2].sum);
    float t3 = fmaf(dot_u_int(c3, x[3]), x[3].scale, -16.0f * x[3].sum);
    return h2f(dd) * (t0 + t1) + h2f(dd >> 16) * (t2 + t3);
  }
}

__device__ __forceinline__ unsigned long long argmax_key(float v, uint32_t idx) {
  uint32_t b = __float_as_uint(v);
  uint32_t ord = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
  return ((unsigned long long)ord << 32) | (0xFFFFFFFFu - idx);
}

// Consumer side of one CTA: all stages of the CTA's rows for format DT.
// Warp w takes rows ra + w + GV_CWARPS*j (j < GV_RPW) of every stage.
template <uint32_t DT>
__device__ bool gv_consume(const GvParams& p, const StageIter& it, const ChunkInfo* chunks, uint8_t* ring,
                           uint64_t* full, uint64_t* empty, const uint8_t* limbs, const float* xsc, const float* xsum,
                           float* acc) {
  const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  uint32_t i = 0, slot = 0, phase = 0;
  for (uint32_t c = 0; c < it.nch; c++) {
    const uint32_t nu = chunks[c].nu, tb = chunks[c].tb;
    XRun xr[4];
    if (lane < nu) {
      uint32_t u = chunks[c].cu0 + lane;
#pragma unroll
      for (uint32_t j = 0; j < 4; j++) {
        uint32_t xc = x_chunk_of(DT, u, j);
        const uint8_t* lp = limbs + 48 * xc;
        xr[j].a = lds128(lp);
        xr[j].b = lds128(lp + 16);
        xr[j].c = lds128(lp + 32);
        xr[j].scale = xsc[xc];
        xr[j].sum = xsum[xc];
      }
    }
    for (uint32_t ra = it.r0; ra < it.r1; ra += GV_ROWS, i++) {
      if (!mbar_wait(&full[slot], phase)) return false;
      const uint8_t* tile = ring + (size_t)slot * p.slot_bytes;
      float v[GV_RPW];
#pragma unroll
      for (int j = 0; j < GV_RPW; j++) {
        uint32_t row = ra + warp + GV_CWARPS * j;
        v[j] = (row < it.r1 && lane < nu) ? unit_dot<DT>(tile + (row - ra) * tb, lane, nu, xr) : 0.f;
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1)
#pragma unroll
        for (int j = 0; j < GV_RPW; j++) v[j] += __shfl_xor_sync(0xffffffffu, v[j], o);
      if (lane == 0) {
#pragma unroll
        for (int j = 0; j < GV_RPW; j++) {
          uint32_t row = ra + warp + GV_CWARPS * j;
          if (row < it.r1) acc[row - it.r0] += v[j];
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[slot]);
      if (++slot == p.slots) {
        slot = 0;
        phase ^= 1;
      }
    }
  }
  return true;
}

__global__ void __launch_bounds__(GV_THREADS, 1) k_gemv(const __grid_constant__ GvParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  const uint32_t tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t U = (p.cols + 63) / 64, NX = 4 * U;
  uint8_t* ring = smem;
  uint8_t* limbs = ring + (size_t)p.slots * p.slot_bytes;
  float* xsc = reinterpret_cast<float*>(limbs + 48 * NX);
  float* xsum = xsc + NX;
  float* acc = xsum + NX;
  uint64_t* full = reinterpret_cast<uint64_t*>(((uintptr_t)(acc + p.max_rows) + 15) & ~uintptr_t(15));
  uint64_t* empty = full + GV_MAX_SLOTS;
  __shared__ float red[GV_CWARPS];
  __shared__ unsigned long long kred[GV_CWARPS];
  __shared__ ChunkInfo chunks[GV_MAX_CH];

  StageIter it;
  it.init(p.seg, p.nseg, blockIdx.x);
  if (tid < it.nch && it.n_stages) chunk_info(it, tid, &chunks[tid]);
  if (tid == 0) {
    for (uint32_t s = 0; s < p.slots; s++) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], GV_CWARPS);
    }
    fence_barrier_init();
  }
  __syncthreads();
  if (tid == 0) pdl_trigger();

  if (warp == GV_CWARPS) {
    // ---------------- producer ----------------
    if (lane != 0) return;
    const uint64_t pol = policy_evict_first();
    StageIter nx;
    nx.init(p.next.seg, p.next.nseg, blockIdx.x);
    // L2 prefetch cursors: own stages, then the next kernel's first stages
    uint32_t pc = 0, pr = it.r0;                       // own (chunk, row)
    const uint32_t nx_nch = nx.n_stages ? nx.nch : 0;   // next kernel (0: nothing to prefetch)
    uint32_t nc = 0, nr = nx.r0;
    ChunkInfo nci = {};
    if (nx_nch) chunk_info(nx, 0, &nci);
    uint64_t copied = 0, prefetched = 0, next_bytes = 0;
    uint32_t slot = 0, phase = 0, i = 0;
    for (uint32_t c = 0; c < it.nch; c++) {
      const ChunkInfo ci = chunks[c];
      for (uint32_t ra = it.r0; ra < it.r1; ra += GV_ROWS, i++) {
        if (i >= p.slots && !mbar_wait(&empty[slot], phase ^ 1)) {
          atomicExch(&p.state->error, 4u);
          return;
        }
        uint32_t bytes = (min(ra + GV_ROWS, it.r1) - ra) * ci.tb;
        mbar_expect_tx(&full[slot], bytes);
        bulk_g2s(ring + (size_t)slot * p.slot_bytes, ci.plane + (uint64_t)ra * ci.tb, bytes, &full[slot], pol);
        copied += bytes;
        if (++slot == p.slots) {
          slot = 0;
          phase ^= 1;
        }
        // keep the L2 prefetch window pf_ahead bytes in front of the copies,
        // running on into the next kernel's stream
        while (prefetched < copied + p.pf_ahead) {
          if (pc < it.nch) {
            const ChunkInfo& pci = chunks[pc];
            uint32_t rows = min(pr + GV_ROWS, it.r1) - pr;
            bulk_prefetch(pci.plane + (uint64_t)pr * pci.tb, rows * pci.tb);
            prefetched += rows * pci.tb;
            pr += GV_ROWS;
            if (pr >= it.r1) {
              pr = it.r0;
              pc++;
            }
          } else if (nc < nx_nch && next_bytes < p.next.budget) {
            uint32_t rows = min(nr + GV_ROWS, nx.r1) - nr;
            bulk_prefetch(nci.plane + (uint64_t)nr * nci.tb, rows * nci.tb);
            prefetched += rows * nci.tb;
            next_bytes += rows * nci.tb;
            nr += GV_ROWS;
            if (nr >= nx.r1) {
              nr = nx.r0;
              if (++nc < nx_nch) chunk_info(nx, nc, &nci);
            }
          } else {
            break;
          }
        }
      }
    }
    return;
  }

  // ---------------- consumers: activation prologue ----------------
  // x (optionally RMS-normalised, src/tensor.rs:164-186) -> 16-element runs
  // of three 8-bit limbs with a shared power-of-two scale.  A quad of lanes
  // converts one run: each lane owns 4 elements (one dp4a word per limb).
  pdl_wait();
  const uint32_t ctid = tid;  // 0..255
  const float4* x4 = reinterpret_cast<const float4*>(p.x);
  const float4* w4 = reinterpret_cast<const float4*>(p.norm_w);
  const uint32_t n4 = p.cols / 4;
  float inv = 1.f;
  if (p.prologue == PRO_RMSNORM) {
    float ss = 0.f;
    for (uint32_t i = ctid; i < n4; i += GV_CWARPS * 32) {
      float4 v = x4[i];
      ss = fmaf(v.x, v.x, ss);
      ss = fmaf(v.y, v.y, ss);
      ss = fmaf(v.z, v.z, ss);
      ss = fmaf(v.w, v.w, ss);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if (lane == 0) red[warp] = ss;
    named_sync(1, GV_CWARPS * 32);
    float tot = 0.f;
#pragma unroll
    for (int w = 0; w < GV_CWARPS; w++) tot += red[w];
    inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, (float)p.cols), p.eps)));
  }
  for (uint32_t base = warp * 8; base < NX; base += GV_CWARPS * 8) {
    uint32_t k = base + (lane >> 2), q = lane & 3, i4 = 4 * k + q;
    float v[4] = {0.f, 0.f, 0.f, 0.f};
    if (k < NX && i4 < n4) {
      float4 t = x4[i4];
      v[0] = t.x;
      v[1] = t.y;
      v[2] = t.z;
      v[3] = t.w;
      if (p.prologue == PRO_RMSNORM) {
        float4 wn = w4[i4];
        v[0] = __fmul_rn(__fmul_rn(v[0], inv), wn.x);
        v[1] = __fmul_rn(__fmul_rn(v[1], inv), wn.y);
        v[2] = __fmul_rn(__fmul_rn(v[2], inv), wn.z);
        v[3] = __fmul_rn(__fmul_rn(v[3], inv), wn.w);
      }
    }
    float m = fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3])));
    float sm = (v[0] + v[1]) + (v[2] + v[3]);
    m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 1));
    m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 2));
    sm += __shfl_xor_sync(0xffffffffu, sm, 1);
    sm += __shfl_xor_sync(0xffffffffu, sm, 2);
    if (k < NX) {
      int e = 0;
      if (m > 0.f) frexpf(m, &e);
      uint32_t wa = 0, wb = 0, wc = 0;
#pragma unroll
      for (int i = 0; i < 4; i++) {
        int X = __float2int_rn(ldexpf(v[i], 22 - e));
        int c = ((X + 128) & 255) - 128;
        int X1 = (X - c) >> 8;
        int b = ((X1 + 128) & 255) - 128;
        int a = (X1 - b) >> 8;
        wa |= (uint32_t)(a & 255) << (8 * i);
        wb |= (uint32_t)(b & 255) << (8 * i);
        wc |= (uint32_t)(c & 255) << (8 * i);
      }
      uint32_t* lp = reinterpret_cast<uint32_t*>(limbs + 48 * k);
      lp[q] = wa;
      lp[4 + q] = wb;
      lp[8 + q] = wc;
      if (q == 0) {
        xsc[k] = ldexpf(1.0f, e - 22);
        xsum[k] = sm;
      }
    }
  }
  for (uint32_t r = ctid; r < p.max_rows; r += GV_CWARPS * 32) acc[r] = 0.f;
  named_sync(1, GV_CWARPS * 32);

  bool ok = true;
  if (it.n_stages) {
    switch (it.dt) {
      case FZ_Q4_K: ok = gv_consume<FZ_Q4_K>(p, it, chunks, ring, full, empty, limbs, xsc, xsum, acc); break;
      case FZ_Q6_K: ok = gv_consume<FZ_Q6_K>(p, it, chunks, ring, full, empty, limbs, xsc, xsum, acc); break;
      case FZ_Q8_0: ok = gv_consume<FZ_Q8_0>(p, it, chunks, ring, full, empty, limbs, xsc, xsum, acc); break;
      case FZ_Q5_0: ok = gv_consume<FZ_Q5_0>(p, it, chunks, ring, full, empty, limbs, xsc, xsum, acc); break;
    }
  }
  if (!ok && lane == 0) atomicExch(&p.state->error, 3u);
  named_sync(1, GV_CWARPS * 32);

  // ---------------- epilogue ----------------
  if (!it.n_stages) return;
  const GvSeg& s = *it.s;
  uint32_t nrows = it.r1 - it.r0;
  unsigned long long best = 0;
  for (uint32_t i = ctid; i < nrows; i += GV_CWARPS * 32) {
    uint32_t row = it.r0 + i;
    float v = acc[i];
    if (p.epilogue == EPI_STORE) {
      s.out[row] = s.bias ? __fadd_rn(v, s.bias[row]) : v;
    } else if (p.epilogue == EPI_RESID) {
      s.out[row] = __fadd_rn(s.out[row], v);
    } else if (p.epilogue == EPI_SWIGLU) {
      if (!(i & 1)) {
        float u = acc[i + 1];
        s.out[row >> 1] = __fmul_rn(__fdiv_rn(v, __fadd_rn(1.0f, expf(-v))), u);
      }
    } else {
      s.out[row] = v;
      unsigned long long k = argmax_key(v, row);
      best = k > best ? k : best;
    }
  }
  if (p.epilogue == EPI_LOGITS) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
      best = other > best ? other : best;
    }
    if (lane == 0) kred[warp] = best;
    named_sync(1, GV_CWARPS * 32);
    if (ctid == 0) {
      unsigned long long m = 0;
      for (int w = 0; w < GV_CWARPS; w++) m = kred[w] > m ? kred[w] : m;
      atomicMax(&p.state->argmax_key, m);
    }
  }
}

// ---- host side ---------------------------------------------------------------
constexpr uint32_t GV_SMEM_2 = 110 * 1024;   // two blocks per SM (current + next kernel)
constexpr uint32_t GV_SMEM_1 = 220 * 1024;   // one block per SM
constexpr uint32_t GV_PF_AHEAD = 96 * 1024;
constexpr uint32_t GV_PF_NEXT = 64 * 1024;

void kernels_init() {
  CK(cudaFuncSetAttribute(k_gemv, cudaFuncAttributeMaxDynamicSharedMemorySize, GV_SMEM_1));
  num_sms();
}

static void fill_segs(const GemvSeg* in, int nseg, GvSeg* out, uint32_t nctas) {
  uint64_t total = 0;
  for (int i = 0; i < nseg; i++) total += (uint64_t)in[i].w.rows * in[i].w.stride;
  uint32_t begin = 0;
  for (int i = 0; i < nseg; i++) {
    const DevMat& w = in[i].w;
    uint32_t want = (uint32_t)((double)nctas * (double)((uint64_t)w.rows * w.stride) / (double)total + 0.5);
    uint32_t maxb = (w.rows + 1) / 2;
    want = want < 1 ? 1 : want > maxb ? maxb : want;
    out[i] = GvSeg{w.ptr, w.rows, w.dtype, w.cols, in[i].bias, in[i].out, begin, begin + want};
    begin += want;
  }
}

static uint32_t gemv_ctas(const GemvLaunch& g) {
  uint32_t n = (uint32_t)num_sms();
  if (g.nseg == 1) n = std::min<uint32_t>(n, (g.seg[0].w.rows + 1) / 2);
  return n;
}

void launch_gemv(const GemvLaunch& g, cudaStream_t st) {
  GvParams p{};
  uint32_t cols = g.seg[0].w.cols;
  for (int i = 0; i < g.nseg; i++)
    if (g.seg[i].w.cols != cols) fail(FZ_EINVAL, "gemv segments disagree on input width");
  uint32_t nctas = gemv_ctas(g);
  fill_segs(g.seg, g.nseg, p.seg, nctas);
  uint32_t grid = p.seg[g.nseg - 1].cta_end;
  p.nseg = g.nseg;
  p.cols = cols;
  p.x = g.x;
  p.norm_w = g.norm_w;
  p.eps = g.eps;
  p.prologue = g.prologue;
  p.epilogue = g.epilogue;
  p.state = g.state;
  // shared memory: ring + activation limbs + per-run scale/sum + row sums
  uint32_t U = (cols + 63) / 64, NX = 4 * U;
  uint32_t max_rows = 0, slot = 0;
  for (int i = 0; i < g.nseg; i++) {
    const GvSeg& s = p.seg[i];
    uint32_t n = s.cta_end - s.cta_begin;
    max_rows = std::max(max_rows, 2 * ((s.rows / 2 + n - 1) / n) + 2);
    slot = std::max(slot, GV_ROWS * lay_max_chunk_bytes(s.dtype, s.cols));
  }
  slot = (slot + 127) & ~127u;
  uint32_t fixed = 48 * NX + 8 * NX + 4 * max_rows + 16 + 16 * GV_MAX_SLOTS + 128;
  uint32_t budget = GV_SMEM_1;  // one block per SM (register file: 16 warps x up to 128 registers)
  if (fixed + 2 * slot > budget) fail(FZ_EINVAL, "gemv: input width %u too large for shared memory", cols);
  uint32_t slots = std::min<uint32_t>(GV_MAX_SLOTS, (budget - fixed) / slot);
  p.slots = slots;
  p.slot_bytes = slot;
  p.max_rows = max_rows;
  p.pf_ahead = GV_PF_AHEAD;
  if (g.next) {
    fill_segs(g.next->seg, g.next->nseg, p.next.seg, gemv_ctas(*g.next));
    p.next.nseg = g.next->nseg;
    p.next.budget = GV_PF_NEXT;
  }
  size_t smem = (size_t)slots * slot + fixed;
  launch_pdl(k_gemv, dim3(grid), dim3(GV_THREADS), smem, st, p);
}

// ---------------------------------------------------------------------------
// Attention (src/model.rs:371-438) with RoPE (src/model.rs:193-217) and the
// KV append (src/model.rs:346-356) folded in.  Grid (splits, n_kv): a block
// owns one KV head, the G = nh/nkv query heads that read it, and a slice of
// positions [0, pos].  It rotates q (and, in the slice that holds pos, the
// new k, which it also writes to the cache), bulk-copies its K and V rows
// into shared memory, and writes the slice's (max, sum, weighted V)
// partials; k_attn_combine merges the slices.  RoPE uses host-computed
// cos/sin (glibc powf/sinf/cosf: the reference's own factors) and the
// reference's uncontracted a*c - b*s / a*s + b*c.
// ---------------------------------------------------------------------------
constexpr int AT_THREADS = 256;
constexpr int AT_MAXG = 8;

template <int HD>
__global__ void __launch_bounds__(AT_THREADS) k_attn(const float* __restrict__ qkv, const float2* __restrict__ cs,
                                                      float* __restrict__ kc, float* __restrict__ vc,
                                                      float* __restrict__ partials, uint32_t nh, uint32_t nkv,
                                                      uint32_t max_ctx, uint32_t per_split, StepState* st) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ __align__(16) float qs[AT_MAXG][HD];
  __shared__ __align__(8) uint64_t bar;
  const uint32_t G = nh / nkv, kvh = blockIdx.y, split = blockIdx.x;
  const uint32_t tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const uint32_t half = HD / 2;
  if (tid == 0) {
    pdl_trigger();
    // The K/V rows of this slice below the (possibly not yet advanced)
    // position are already final: start pulling them into L2 before waiting
    // for the predecessor.
    uint32_t p0 = *((volatile uint32_t*)&st->pos);
    uint32_t a0 = split * per_split, a1 = min(min(p0, max_ctx), a0 + per_split);
    if (a1 > a0) {
      bulk_prefetch(kc + ((uint64_t)kvh * max_ctx + a0) * HD, (a1 - a0) * HD * 4);
      bulk_prefetch(vc + ((uint64_t)kvh * max_ctx + a0) * HD, (a1 - a0) * HD * 4);
    }
  }
  pdl_wait();
  const uint32_t pos = st->pos;
  if (pos >= max_ctx) {
    if (tid == 0) st->error = 2;
    return;
  }
  const uint32_t total = pos + 1;
  const uint32_t t0 = split * per_split;
  const uint32_t t1 = min(total, t0 + per_split);
  const uint32_t n = t1 > t0 ? t1 - t0 : 0;
  float* kt = reinterpret_cast<float*>(smem);     // [per_split][HD]
  float* vt = kt + (size_t)per_split * HD;         // [per_split][HD]
  float* sc = vt + (size_t)per_split * HD;         // [G][per_split]
  const float* kvk = kc + (uint64_t)kvh * max_ctx * HD;
  const float* kvv = vc + (uint64_t)kvh * max_ctx * HD;
  // cached rows [t0, min(t1, pos)) arrive by bulk copy
  const uint32_t ncached = t1 > pos ? (pos > t0 ? pos - t0 : 0) : n;
  if (tid == 0) {
    mbar_init(&bar, 1);
    fence_barrier_init();
  }
  __syncthreads();
  if (tid == 0 && ncached) {
    uint32_t bytes = ncached * HD * 4;
    mbar_expect_tx(&bar, 2 * bytes);
    uint64_t pol = policy_evict_first();
    bulk_g2s(kt, kvk + (uint64_t)t0 * HD, bytes, &bar, pol);
    bulk_g2s(vt, kvv + (uint64_t)t0 * HD, bytes, &bar, pol);
  }
  // rotated queries (the 1/sqrt(hd) scale is applied to the dot, src/model.rs:237)
  const float scale = __fdiv_rn(1.0f, __fsqrt_rn((float)HD));
  const float2* csp = cs + (uint64_t)pos * half;
  for (uint32_t idx = tid; idx < G * half; idx += AT_THREADS) {
    uint32_t h = idx / half, i = idx % half;
    const float* x = qkv + (uint64_t)(kvh * G + h) * HD;
    float a = x[i], b = x[i + half];
    float2 c = csp[i];
    qs[h][i] = __fsub_rn(__fmul_rn(a, c.x), __fmul_rn(b, c.y));
    qs[h][i + half] = __fadd_rn(__fmul_rn(a, c.y), __fmul_rn(b, c.x));
  }
  if (t1 == total && n) {
    // this slice holds pos: rotate the new k, append k and v
    const float* kx = qkv + (uint64_t)(nh + kvh) * HD;
    const float* vx = qkv + (uint64_t)(nh + nkv + kvh) * HD;
    float* kdst = kc + ((uint64_t)kvh * max_ctx + pos) * HD;
    float* vdst = vc + ((uint64_t)kvh * max_ctx + pos) * HD;
    for (uint32_t i = tid; i < half; i += AT_THREADS) {
      float a = kx[i], b = kx[i + half];
      float2 c = csp[i];
      float ra = __fsub_rn(__fmul_rn(a, c.x), __fmul_rn(b, c.y));
      float rb = __fadd_rn(__fmul_rn(a, c.y), __fmul_rn(b, c.x));
      kdst[i] = ra;
      kdst[i + half] = rb;
      kt[(size_t)(pos - t0) * HD + i] = ra;
      kt[(size_t)(pos - t0) * HD + i + half] = rb;
    }
    for (uint32_t i = tid; i < HD; i += AT_THREADS) {
      float v = vx[i];
      vdst[i] = v;
      vt[(size_t)(pos - t0) * HD + i] = v;
    }
  }
  if (ncached && !mbar_wait(&bar, 0)) {
    if (tid == 0) st->error = 5;
    return;
  }
  __syncthreads();
  // scores: one (position, head) per thread-iteration; lanes start at
  // different columns so a warp's 16-byte reads spread over the banks
  for (uint32_t idx = tid; idx < n * G; idx += AT_THREADS) {
    uint32_t t = idx % n, h = idx / n;
    const float4* kr = reinterpret_cast<const float4*>(kt + (size_t)t * HD);
    const float4* qr = reinterpret_cast<const float4*>(qs[h]);
    float s = 0.f;
#pragma unroll 8
    for (uint32_t j = 0; j < HD / 4; j++) {
      uint32_t jj = (j + t) & (HD / 4 - 1);
      float4 k4 = kr[jj], q4 = qr[jj];
      s = fmaf(q4.x, k4.x, s);
      s = fmaf(q4.y, k4.y, s);
      s = fmaf(q4.z, k4.z, s);
      s = fmaf(q4.w, k4.w, s);
    }
    sc[h * per_split + t] = __fmul_rn(s, scale);
  }
  __syncthreads();
  // per-head max / exp / sum over this slice (warp h).  Partials:
  // stats [nkv][G][S] of (max, sum), then acc [nkv][G][HD][Spad].
  const uint32_t S = gridDim.x, Spad = (S + 3) & ~3u;
  float2* stats = reinterpret_cast<float2*>(partials) + (uint64_t)kvh * G * S;
  float* pacc = partials + 2 * (uint64_t)nkv * G * S + (uint64_t)kvh * G * HD * Spad;
  if (warp < G) {
    float m = -INFINITY;
    for (uint32_t t = lane; t < n; t += 32) m = fmaxf(m, sc[warp * per_split + t]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    float l = 0.f;
    for (uint32_t t = lane; t < n; t += 32) {
      float e = expf(sc[warp * per_split + t] - m);
      sc[warp * per_split + t] = e;
      l += e;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) l += __shfl_xor_sync(0xffffffffu, l, o);
    if (lane == 0) stats[warp * S + split] = make_float2(n ? m : -INFINITY, n ? l : 0.f);
  }
  __syncthreads();
  // weighted V sum: thread per (head, dim)
  for (uint32_t idx = tid; idx < G * HD; idx += AT_THREADS) {
    uint32_t h = idx / HD, d = idx % HD;
    const float* pr = sc + h * per_split;
    float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
    uint32_t t = 0;
    for (; t + 4 <= n; t += 4) {
      a0 = fmaf(pr[t], vt[(size_t)t * HD + d], a0);
      a1 = fmaf(pr[t + 1], vt[(size_t)(t + 1) * HD + d], a1);
      a2 = fmaf(pr[t + 2], vt[(size_t)(t + 2) * HD + d], a2);
      a3 = fmaf(pr[t + 3], vt[(size_t)(t + 3) * HD + d], a3);
    }
    for (; t < n; t++) a0 = fmaf(pr[t], vt[(size_t)t * HD + d], a0);
    pacc[((uint64_t)h * HD + d) * Spad + split] = (a0 + a1) + (a2 + a3);
  }
}

// Merge the split partials: ctx[h][d] = sum_s w_s acc_s[d] / sum_s w_s l_s,
// w_s = exp(m_s - max_s m_s).  Grid nh, block hd.  Each thread reads its
// split values as consecutive float4s, all issued before they are used.
constexpr int AT_MAXS = 256;
__global__ void k_attn_combine(const float* __restrict__ partials, float* __restrict__ ctx, uint32_t nh, uint32_t nkv,
                               uint32_t hd, uint32_t S, StepState* st) {
  __shared__ float ws[AT_MAXS], ls[AT_MAXS];
  __shared__ float s_den;
  if (threadIdx.x == 0) pdl_trigger();
  pdl_wait();
  (void)st;
  const uint32_t G = nh / nkv, h = blockIdx.x, kvh = h / G, hg = h % G, d = threadIdx.x;
  const uint32_t Spad = (S + 3) & ~3u;
  const float2* stats = reinterpret_cast<const float2*>(partials) + ((uint64_t)kvh * G + hg) * S;
  const float4* acc4 =
      reinterpret_cast<const float4*>(partials + 2 * (uint64_t)nkv * G * S + (((uint64_t)h) * hd + d) * Spad);
  // all of this thread's acc values in flight at once (S <= 64 in one pass)
  float4 av[16];
#pragma unroll
  for (int k = 0; k < 16; k++) av[k] = (4u * k < Spad) ? acc4[k] : make_float4(0.f, 0.f, 0.f, 0.f);
  for (uint32_t s2 = threadIdx.x; s2 < S; s2 += blockDim.x) {
    float2 v = stats[s2];
    ws[s2] = v.x;
    ls[s2] = v.y;
  }
  for (uint32_t s2 = S + threadIdx.x; s2 < Spad; s2 += blockDim.x) ws[s2] = ls[s2] = 0.f;
  __syncthreads();
  if (threadIdx.x < 32) {
    float M = -INFINITY;
    for (uint32_t s2 = threadIdx.x; s2 < S; s2 += 32) M = fmaxf(M, ws[s2]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
    float den = 0.f;
    for (uint32_t s2 = threadIdx.x; s2 < S; s2 += 32) {
      float ms = ws[s2];
      float w = ms == -INFINITY ? 0.f : expf(ms - M);
      ws[s2] = w;
      den = fmaf(w, ls[s2], den);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) den += __shfl_xor_sync(0xffffffffu, den, o);
    if (threadIdx.x == 0) s_den = den;
  }
  __syncthreads();
  float num = 0.f;
#pragma unroll
  for (int k = 0; k < 16; k++) {
    if (4u * k >= Spad) break;
    num = fmaf(ws[4 * k], av[k].x, num);
    num = fmaf(ws[4 * k + 1], av[k].y, num);
    num = fmaf(ws[4 * k + 2], av[k].z, num);
    num = fmaf(ws[4 * k + 3], av[k].w, num);
  }
  for (uint32_t k = 16; 4 * k < Spad; k++) {
    float4 a4 = acc4[k];
    num = fmaf(ws[4 * k], a4.x, num);
    num = fmaf(ws[4 * k + 1], a4.y, num);
    num = fmaf(ws[4 * k + 2], a4.z, num);
    num = fmaf(ws[4 * k + 3], a4.w, num);
  }
  ctx[(uint64_t)h * hd + d] = __fdiv_rn(num, s_den);
}

static uint32_t attention_per_split(uint32_t hd) { return hd == 128 ? 64 : 128; }

uint32_t attention_splits(uint32_t hd, uint32_t max_ctx) {
  uint32_t per = attention_per_split(hd);
  return (max_ctx + per - 1) / per;
}

uint64_t attention_partial_floats(uint32_t nh, uint32_t nkv, uint32_t hd, uint32_t splits) {
  uint32_t G = nh / nkv, Spad = (splits + 3) & ~3u;
  return 2ull * nkv * G * splits + (uint64_t)nkv * G * hd * Spad;
}

void attention_init() {
  CK(cudaFuncSetAttribute(k_attn<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, 160 * 1024));
  CK(cudaFuncSetAttribute(k_attn<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, 160 * 1024));
}

void launch_attention(const AttnLaunch& a, cudaStream_t s) {
  uint32_t G = a.n_heads / a.n_kv;
  if (G > AT_MAXG) fail(FZ_EINVAL, "attention: GQA group %u > %d", G, AT_MAXG);
  uint32_t per = attention_per_split(a.hd);
  uint32_t splits = attention_splits(a.hd, a.max_ctx);
  if (splits > a.splits) fail(FZ_EINVAL, "attention: partials sized for %u splits, need %u", a.splits, splits);
  if (splits > AT_MAXS) fail(FZ_EINVAL, "attention: %u splits > %d (max_ctx too large)", splits, AT_MAXS);
  size_t smem = (size_t)per * a.hd * 4 * 2 + (size_t)G * per * 4;
  dim3 grid(splits, a.n_kv);
  const float2* cs = reinterpret_cast<const float2*>(a.rope_cs);
  if (a.hd == 128)
    launch_pdl(k_attn<128>, grid, dim3(AT_THREADS), smem, s, a.qkv, cs, a.kcache, a.vcache, a.partials, a.n_heads,
               a.n_kv, a.max_ctx, per, a.state);
  else if (a.hd == 64)
    launch_pdl(k_attn<64>, grid, dim3(AT_THREADS), smem, s, a.qkv, cs, a.kcache, a.vcache, a.partials, a.n_heads,
               a.n_kv, a.max_ctx, per, a.state);
  else
    fail(FZ_EINVAL, "head_dim %u unsupported (64 or 128)", a.hd);
  launch_pdl(k_attn_combine, dim3(a.n_heads), dim3(a.hd), 0, s, (const float*)a.partials, a.ctx, a.n_heads, a.n_kv,
             a.hd, splits, a.state);
}

// ---------------------------------------------------------------------------
// Step bookkeeping: the sampled id (first max, src/generate.rs:69-77), the
// next input token (forced prompt token or the id itself), pos += 1.
// ---------------------------------------------------------------------------
__global__ void k_finalize(StepState* st, const uint32_t* forced, uint32_t* ids_out, int has_logits) {
  pdl_trigger();
  pdl_wait();
  uint32_t step = st->step;
  if (has_logits) {
    uint32_t id = 0xFFFFFFFFu - (uint32_t)(st->argmax_key & 0xFFFFFFFFull);
    if (ids_out) ids_out[step] = id;
    st->token = (step + 1 < st->n_forced) ? forced[step + 1] : id;
  } else {
    st->token = (step + 1 < st->n_forced) ? forced[step + 1] : st->token;
  }
  st->argmax_key = 0;
  st->step = step + 1;
  st->pos = st->pos + 1;
}

void launch_finalize(StepState* st, const uint32_t* forced, uint32_t* ids_out, bool has_logits, cudaStream_t s) {
  launch_pdl(k_finalize, dim3(1), dim3(1), 0, s, st, forced, ids_out, has_logits ? 1 : 0);
}

}  // namespace fz
