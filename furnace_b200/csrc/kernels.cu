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
#include <cstdlib>
#include <cstring>
#include <algorithm>
#include <memory>
#include <type_traits>
#include <utility>
#include <vector>

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

// ---------------------------------------------------------------------------
// Optional per-CTA timeline of the decode-step kernels (%globaltimer, ns), recorded
// by thread 0 of every CTA while a trace buffer is installed (trace_enable):
// t[0] start, t[1] after the wait on the predecessor, t[2] input ready,
// t[3] main loop done, t[4] end.  Off (one global load per CTA) otherwise.
// ---------------------------------------------------------------------------
__device__ TraceRec* g_trace = nullptr;
__device__ uint32_t g_trace_cap = 0;
__device__ uint32_t g_trace_n = 0;

__device__ __forceinline__ uint64_t gtimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

struct Tracer {
  TraceRec* r = nullptr;
  __device__ __forceinline__ void begin(uint32_t tag, uint32_t aux) {
    TraceRec* base = g_trace;
    if (!base) return;
    const uint32_t i = atomicAdd(&g_trace_n, 1u);
    if (i >= g_trace_cap) return;
    r = base + i;
    r->tag = tag;
    r->cta = blockIdx.x | (blockIdx.y << 16);
    r->aux = aux;
    r->t[0] = gtimer();
  }
  __device__ __forceinline__ void mark(int k) {
    if (r) r->t[k] = gtimer();
  }
};
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
    // one thread per 64-element unit k of a super-block: regroup its quants
    // (src/quant.rs:114-133 gives element e = 128h + 32g + l its bits)
    const uint8_t* src = raw + r * (cols / 256) * 210 + (uint64_t)(u >> 2) * 210;
    uint8_t* body = ch + 208 * (lu >> 2);
    const uint32_t k = u & 3;
    auto q6 = [&](uint32_t e) -> uint32_t {
      uint32_t h = e >> 7, g = (e & 127) >> 5, l = e & 31;
      uint32_t b = src[64 * h + l + 32 * (g & 1)];
      uint32_t lo = g < 2 ? (b & 0x0F) : (b >> 4);
      return lo | (((src[128 + 32 * h + l] >> (2 * g)) & 3) << 4);
    };
    for (uint32_t i = 0; i < 32; i++)
      body[32 * k + i] = (uint8_t)((q6(64 * k + i) & 15) | ((q6(64 * k + 32 + i) & 15) << 4));
    for (uint32_t i = 0; i < 16; i++)
      body[128 + 16 * k + i] = (uint8_t)((q6(64 * k + i) >> 4) | ((q6(64 * k + 16 + i) >> 4) << 2) |
                                         ((q6(64 * k + 32 + i) >> 4) << 4) | ((q6(64 * k + 48 + i) >> 4) << 6));
    for (uint32_t t = 0; t < 4; t++) {
      uint32_t e = 64 * k + 16 * t, h = e >> 7, g = (e & 127) >> 5, l = e & 31;
      body[192 + 4 * k + t] = src[192 + 8 * h + l / 16 + 2 * g];
    }
    if (k == 0) {
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
// (src/quant.rs:35-39, 53-63, 78-109, 114-133) into o[0..64) (o[0..32) for
// the last unit of a row of 32 mod 64 Q8_0 / Q5_0 columns).  Inlined with
// constant indices, so o may be a register array.
// ---------------------------------------------------------------------------
// One 64-element unit's bytes in registers (fetch_unit), decoded by
// decode_unit.  Q4_K: a = the super-block's header (d, dmin, 12 scale bytes),
// b, c = the unit's 32 quant bytes.  Q6_K: a, b = nibble bytes, c = high-bit
// bytes, x0 = the unit's 4 scales, x1 = d.  Q8_0: a..d = 64 quants, x0 = the
// two blocks' d.  Q5_0: a, b = nibble bytes, x0, x1 = the two blocks' high
// bits, c.x = the two blocks' d.
struct RawUnit {
  uint4 a, b, c, d;
  uint32_t x0, x1;
};
__device__ __forceinline__ uint32_t byte_of(const uint4& v, uint32_t k) {
  const uint32_t w = k < 4 ? v.x : k < 8 ? v.y : k < 12 ? v.z : v.w;
  return (w >> (8 * (k & 3))) & 0xFFu;
}
__device__ __forceinline__ uint32_t byte_of2(const uint4& lo, const uint4& hi, uint32_t k) {
  return k < 16 ? byte_of(lo, k) : byte_of(hi, k - 16);
}

__device__ __forceinline__ RawUnit fetch_unit(uint32_t dt, const uint8_t* base, uint32_t rows, uint32_t r,
                                              uint32_t cols, uint32_t u) {
  const uint32_t c = lay_chunk_of(dt, cols, u);
  const uint32_t cu0 = lay_cu0(dt, cols, c), nu = lay_cu0(dt, cols, c + 1) - cu0, lu = u - cu0;
  const uint8_t* ch = base + lay_tile_off(dt, cols, rows, r, c);
  RawUnit w{};
  if (dt == FZ_Q4_K) {
    const uint8_t* blk = ch + 144 * (lu >> 2);
    w.a = *reinterpret_cast<const uint4*>(blk);
    w.b = *reinterpret_cast<const uint4*>(blk + 16 + 32 * (u & 3));
    w.c = *reinterpret_cast<const uint4*>(blk + 32 + 32 * (u & 3));
  } else if (dt == FZ_Q6_K) {
    const uint32_t k = u & 3;
    const uint8_t* body = ch + 208 * (lu >> 2);
    w.a = *reinterpret_cast<const uint4*>(body + 32 * k);
    w.b = *reinterpret_cast<const uint4*>(body + 32 * k + 16);
    w.c = *reinterpret_cast<const uint4*>(body + 128 + 16 * k);
    w.x0 = *reinterpret_cast<const uint32_t*>(body + 192 + 4 * k);
    w.x1 = *reinterpret_cast<const uint16_t*>(ch + 208 * (nu >> 2) + 2 * (lu >> 2));
  } else if (dt == FZ_Q8_0) {
    const uint4* q = reinterpret_cast<const uint4*>(ch + 64 * lu);
    w.a = q[0];
    w.b = q[1];
    if (2 * u + 1 < cols / 32) {  // a last half unit holds one block
      w.c = q[2];
      w.d = q[3];
    }
    w.x0 = *reinterpret_cast<const uint32_t*>(ch + 64 * nu + 4 * lu);
  } else {
    const uint4* q = reinterpret_cast<const uint4*>(ch + 32 * lu);
    w.a = q[0];
    if (2 * u + 1 < cols / 32) w.b = q[1];
    const uint2 h = *reinterpret_cast<const uint2*>(ch + 32 * nu + 8 * lu);
    w.x0 = h.x;
    w.x1 = h.y;
    w.c.x = *reinterpret_cast<const uint32_t*>(ch + 32 * nu + round16u(8 * nu) + 4 * lu);
  }
  return w;
}

// The unit's 64 values, in the reference's arithmetic (src/quant.rs:17-133).
// A last half unit (Q8_0 / Q5_0 with an odd block count) writes o[0..31] only.
__device__ __forceinline__ void decode_unit(uint32_t dt, uint32_t cols, uint32_t u, const RawUnit& w, float* o) {
  if (dt == FZ_Q4_K) {
    const uint32_t j64 = u & 3;
    const float d = h2f(w.a.x & 0xFFFFu), dmin = h2f(w.a.x >> 16);
    float scv[2], mv[2];
#pragma unroll
    for (int t = 0; t < 2; t++) {
      const uint32_t j = 2 * j64 + t;  // scale byte s[k] is header byte 4 + k
      uint32_t sc, m;
      if (j < 4) {
        sc = byte_of(w.a, 4 + j) & 63;
        m = byte_of(w.a, 8 + j) & 63;
      } else {
        sc = (byte_of(w.a, 8 + j) & 0x0F) | ((byte_of(w.a, j) >> 6) << 4);
        m = (byte_of(w.a, 8 + j) >> 4) | ((byte_of(w.a, 4 + j) >> 6) << 4);
      }
      scv[t] = (float)sc;
      mv[t] = (float)m;
    }
    const float d1 = __fmul_rn(d, scv[0]), min1 = __fmul_rn(dmin, mv[0]);
    const float d2 = __fmul_rn(d, scv[1]), min2 = __fmul_rn(dmin, mv[1]);
#pragma unroll
    for (uint32_t l = 0; l < 32; l++) {
      const uint32_t q = byte_of2(w.b, w.c, l);
      o[l] = __fsub_rn(__fmul_rn(d1, (float)(q & 0x0F)), min1);
      o[32 + l] = __fsub_rn(__fmul_rn(d2, (float)(q >> 4)), min2);
    }
  } else if (dt == FZ_Q6_K) {
    const float d = h2f(w.x1);
#pragma unroll
    for (uint32_t i = 0; i < 64; i++) {
      const uint32_t nib = (byte_of2(w.a, w.b, i & 31) >> (i < 32 ? 0 : 4)) & 15;
      const uint32_t hb = (byte_of(w.c, i & 15) >> (2 * (i >> 4))) & 3;
      const int q = (int)(nib | (hb << 4)) - 32;
      const float sc = (float)(int8_t)((w.x0 >> (8 * (i >> 4))) & 0xFFu);
      o[i] = __fmul_rn(__fmul_rn(d, sc), (float)q);  // (d * sc) * q, src/quant.rs:127-130
    }
  } else {
    const uint32_t nb = cols / 32;
#pragma unroll
    for (uint32_t k = 0; k < 2; k++) {
      if (2 * u + k >= nb) break;
      float* ob = o + 32 * k;
      if (dt == FZ_Q8_0) {
        const float d = h2f((w.x0 >> (16 * k)) & 0xFFFFu);
        const uint4& lo = k ? w.c : w.a;
        const uint4& hi = k ? w.d : w.b;
#pragma unroll
        for (uint32_t i = 0; i < 32; i++) ob[i] = __fmul_rn(d, (float)(int8_t)byte_of2(lo, hi, i));
      } else {
        const uint4& qs = k ? w.b : w.a;
        const uint32_t qh = k ? w.x1 : w.x0;
        const float d = h2f((w.c.x >> (16 * k)) & 0xFFFFu);
#pragma unroll
        for (uint32_t j = 0; j < 16; j++) {
          const uint32_t hi0 = ((qh >> j) & 1) << 4, hi1 = ((qh >> (j + 16)) & 1) << 4;
          const uint32_t qb = byte_of(qs, j);
          ob[j] = __fmul_rn(d, (float)((int)((qb & 0x0F) | hi0) - 16));
          ob[j + 16] = __fmul_rn(d, (float)((int)((qb >> 4) | hi1) - 16));
        }
      }
    }
  }
}

__device__ __forceinline__ void dequant_unit(uint32_t dt, const uint8_t* base, uint32_t rows, uint32_t r,
                                             uint32_t cols, uint32_t u, float* o) {
  decode_unit(dt, cols, u, fetch_unit(dt, base, rows, r, cols, u), o);
}

__global__ void k_dequant(uint32_t dt, const uint8_t* __restrict__ base, uint32_t total_rows, uint32_t cols, uint32_t r0,
                          uint32_t rows, float* __restrict__ out) {
  uint32_t U = (cols + 63) / 64;
  uint64_t idx = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (uint64_t)rows * U) return;
  uint64_t r = idx / U;
  uint32_t u = (uint32_t)(idx % U);
  dequant_unit(dt, base, total_rows, r0 + (uint32_t)r, cols, u, out + r * cols + 64 * u);
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

// ---------------------------------------------------------------------------
// Activation runs.  A GEMV input vector is handed between kernels as one
// 64-byte record per 16 elements: the elements as 24-bit fixed point with a
// shared power-of-two scale, split into three signed 8-bit limbs (a, b, c:
// X = a*2^16 + b*2^8 + c, x = X * scale), plus the run's f32 sum.  The
// kernel that produces a vector writes its records in its epilogue, so a
// consuming GEMV never converts activations; RMSNorm inputs are recorded as
// x (.) w_norm and the 1/rms factor is applied to each dot product at the end
// (from per-CTA sum-of-squares partials).
// ---------------------------------------------------------------------------
struct XRun {  // one 16-element activation run in limb form (== a run record)
  uint4 a, b, c;
  float scale, sum;
  uint32_t pad[2];
};
static_assert(sizeof(XRun) == 64, "run record");

// Records are stored unit by unit (4 runs = 64 elements = 256 bytes, the
// span one weight unit multiplies).  Inside a unit the sixteen 16-byte pieces
// -- run j's limbs a, b, c and then (scale, sum) -- sit at piece index
// (4j + f) ^ (unit & 7): the 8 lanes of a quarter warp, which read the same
// piece of 8 consecutive units, then hit 8 different groups of 4 banks.
__host__ __device__ __forceinline__ uint32_t run_piece_off(uint32_t run, uint32_t f) {
  const uint32_t u = run >> 2;
  return 256 * u + 16 * ((4 * (run & 3) + f) ^ (u & 7));
}

// Four consecutive lanes (a quad) convert one run, 4 elements each; every lane
// of the warp must call this (shuffles).  The record goes to run `run` of the
// record array at `base`; `base` = null for an idle quad.
__device__ __forceinline__ void quad_to_run(const float* v, uint32_t q, XRun* base, uint32_t run) {
  float m = fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3])));
  float sm = (v[0] + v[1]) + (v[2] + v[3]);
  m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 1));
  m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 2));
  sm += __shfl_xor_sync(0xffffffffu, sm, 1);
  sm += __shfl_xor_sync(0xffffffffu, sm, 2);
  if (!base) return;
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
  uint8_t* b8 = reinterpret_cast<uint8_t*>(base);
  reinterpret_cast<uint32_t*>(b8 + run_piece_off(run, 0))[q] = wa;
  reinterpret_cast<uint32_t*>(b8 + run_piece_off(run, 1))[q] = wb;
  reinterpret_cast<uint32_t*>(b8 + run_piece_off(run, 2))[q] = wc;
  if (q == 0) *reinterpret_cast<float2*>(b8 + run_piece_off(run, 3)) = make_float2(ldexpf(1.0f, e - 22), sm);
}

// Run j (< 4) of unit u from a unit-swizzled record array.
__device__ __forceinline__ XRun load_run(const XRun* base, uint32_t u, uint32_t j) {
  const uint8_t* b8 = reinterpret_cast<const uint8_t*>(base) + 256 * u;
  const uint32_t s = u & 7;
  XRun r;
  r.a = *reinterpret_cast<const uint4*>(b8 + 16 * ((4 * j) ^ s));
  r.b = *reinterpret_cast<const uint4*>(b8 + 16 * ((4 * j + 1) ^ s));
  r.c = *reinterpret_cast<const uint4*>(b8 + 16 * ((4 * j + 2) ^ s));
  const float2 ss = *reinterpret_cast<const float2*>(b8 + 16 * ((4 * j + 3) ^ s));
  r.scale = ss.x;
  r.sum = ss.y;
  return r;
}

// Records for n values (n % 16 == 0) held in shared memory, optionally scaled
// elementwise by w (global), written to runs run0 .. run0 + n/16 of the record
// array `out`.  Called by `nthreads` threads (whole warps) with thread index t.
__device__ void values_to_runs(const float* vals, uint32_t n, const float* w, XRun* out, uint32_t run0, uint32_t t,
                               uint32_t nthreads) {
  const uint32_t n4 = n / 4, iters = (n4 + nthreads - 1) / nthreads;
  for (uint32_t it = 0; it < iters; it++) {
    uint32_t i4 = t + it * nthreads;
    float v[4] = {0.f, 0.f, 0.f, 0.f};
    bool act = i4 < n4;
    if (act) {
#pragma unroll
      for (int i = 0; i < 4; i++) {
        v[i] = vals[4 * i4 + i];
        if (w) v[i] = __fmul_rn(v[i], w[4 * i4 + i]);
      }
    }
    quad_to_run(v, i4 & 3, act ? out : nullptr, run0 + (i4 >> 2));
  }
}

// f32 vector -> run records (fz_matmul_quant_dev and tests).  One warp per 8 runs.
__global__ void k_to_runs(const float* __restrict__ x, uint32_t cols, XRun* __restrict__ out, uint32_t nruns) {
  uint32_t i4 = blockIdx.x * blockDim.x + threadIdx.x;
  float v[4] = {0.f, 0.f, 0.f, 0.f};
  bool act = i4 < 4 * nruns;
  if (act)
    for (int i = 0; i < 4; i++) v[i] = 4 * i4 + i < cols ? x[4 * i4 + i] : 0.f;
  quad_to_run(v, i4 & 3, act ? out : nullptr, i4 >> 2);
}

void launch_to_runs(const float* x, uint32_t cols, void* runs, uint32_t nruns, cudaStream_t s) {
  uint32_t n4 = 4 * nruns;
  k_to_runs<<<(n4 + 255) / 256, 256, 0, s>>>(x, cols, reinterpret_cast<XRun*>(runs), nruns);
  CK(cudaGetLastError());
}

__host__ __device__ __forceinline__ uint32_t runs_for_dev(uint32_t cols) { return 4 * ((cols + 63) / 64); }
uint32_t runs_for(uint32_t cols) { return runs_for_dev(cols); }

// ---------------------------------------------------------------------------
// GEMV
// ---------------------------------------------------------------------------
constexpr int GV_CWARPS = 15;                      // consumer warps (16 warps per block with the producer)
constexpr int GV_RPW = 2;                          // rows per consumer warp per stage
#ifndef GV_PAIRS_DEF
#define GV_PAIRS_DEF 1
#endif
constexpr bool GV_PAIRS = GV_PAIRS_DEF;            // warp w: rows 2w, 2w+1 (else w, w + GV_CWARPS)
constexpr int GV_ROWS = GV_CWARPS * GV_RPW;        // rows per stage
constexpr int GV_THREADS = (GV_CWARPS + 1) * 32;   // + one producer warp
constexpr int GV_NT = GV_CWARPS * 32;              // consumer threads
constexpr int GV_MAX_SLOTS = 8;
constexpr int GV_MAX_CH = 32;                      // chunks per row (cols <= 65536)

// Chunk geometry of one matrix (layout.cuh), computed on the host: chunk c
// covers units [cu0[c], cu0[c+1]) and starts off[c] bytes into a row.
struct GvChunks {
  uint16_t cu0[GV_MAX_CH + 1];
  uint32_t off[GV_MAX_CH + 1];
};

struct GvSeg {
  const uint8_t* w;
  uint32_t rows, dtype, cols;
  const float* bias;
  float* out;
  uint32_t cta_begin, cta_end, align;
  GvChunks ch;
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
  const XRun* in_runs;   // activation as run records (one bulk copy), or
  const float* x;        // activation as f32, converted in the prologue
  const float* norm_w;   //   optionally RMS-normalised (src/tensor.rs:164-186)
  float eps;
  int epilogue;
  StepState* state;
  XRun* out_runs;        // SWIGLU: records of the next GEMV's input
  uint32_t slots, slot_bytes, max_rows, pf_ahead;
  GvNext next;
  uint32_t idx_base;     // EPI_LOGITS: global index of row 0
  uint32_t chunked_rec;  // in_runs stream per K-chunk through GV_NREC buffers (long inputs)
  // tensor-parallel exchange through peer memory (GemvLaunch::ar_*)
  ArPeers ar_peers;
  uint32_t ar_w, ar_rank, ar_k, ar_h;
  const uint32_t* ar_base;
  int ar_push, ar_pull;
  float* x_out;          // ar_pull: this CTA's slice of the summed x goes here
  uint64_t ar_spin_ns;   // ar_pull: time limit of the wait for a peer's word
};
constexpr uint32_t GV_CREC = 32 * 256;  // run records of one chunk (<= 32 units)
constexpr uint32_t GV_NREC = 4;         // chunk record buffers of a long input (copies in flight)

// This CTA's row range within its segment: whole multiples of seg.align rows
// (pairs for gate/up, 16-row runs where the epilogue writes run records).
__device__ __forceinline__ void cta_rows(const GvSeg& s, uint32_t b, uint32_t* r0, uint32_t* r1) {
  uint32_t n = s.cta_end - s.cta_begin, lb = b - s.cta_begin, units = s.rows / s.align;
  *r0 = s.align * (uint32_t)((uint64_t)units * lb / n);
  *r1 = lb + 1 == n ? s.rows : s.align * (uint32_t)((uint64_t)units * (lb + 1) / n);
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
    if (r1 <= r0) return;
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
  const GvChunks& ch = it.s->ch;
  ci->cu0 = ch.cu0[c];
  ci->nu = ch.cu0[c + 1] - ch.cu0[c];
  ci->tb = ch.off[c + 1] - ch.off[c];
  ci->plane = it.s->w + (uint64_t)it.s->rows * ch.off[c];
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
    const uint32_t k = lu & 3;
    uint4 n0 = lds128(body + 32 * k), n1 = lds128(body + 32 * k + 16), qh = lds128(body + 128 + 16 * k);
    uint32_t sc4 = lds32(body + 192 + 4 * k);
    float d = h2f(lds16(tp + 208 * (nu >> 2) + 2 * (lu >> 2)));
    const uint32_t a0[4] = {n0.x, n0.y, n0.z, n0.w}, a1[4] = {n1.x, n1.y, n1.z, n1.w};
    const uint32_t hv[4] = {qh.x, qh.y, qh.z, qh.w};
    uint32_t g0[4], g1[4], g2[4], g3[4];
#pragma unroll
    for (int w = 0; w < 4; w++) {
      g0[w] = (a0[w] & M4) | ((hv[w] << 4) & M30);
      g1[w] = (a1[w] & M4) | ((hv[w] << 2) & M30);
      g2[w] = ((a0[w] >> 4) & M4) | (hv[w] & M30);
      g3[w] = ((a1[w] >> 4) & M4) | ((hv[w] >> 2) & M30);
    }
    float s0 = fmaf(dot_f<false>(g0, x[0]), x[0].scale, -32.0f * x[0].sum);
    float s1 = fmaf(dot_f<false>(g1, x[1]), x[1].scale, -32.0f * x[1].sum);
    float s2 = fmaf(dot_f<false>(g2, x[2]), x[2].scale, -32.0f * x[2].sum);
    float s3 = fmaf(dot_f<false>(g3, x[3]), x[3].scale, -32.0f * x[3].sum);
    float c0 = (float)(int8_t)(sc4 & 0xff), c1 = (float)(int8_t)((sc4 >> 8) & 0xff);
    float c2 = (float)(int8_t)((sc4 >> 16) & 0xff), c3 = (float)(int8_t)(sc4 >> 24);
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
// Warp w takes rows ra + 2w and ra + 2w + 1 of every stage; the activation
// records of the whole input sit in shared memory (rec).
// Chunk c's input records as record buffer use c (buffer c & 1, phase c / 2
// of its mbarriers), once use c - 2 of that buffer has been released.  One
// thread; the chunked-record mode of long inputs.
__device__ __forceinline__ bool gv_issue_records(const GvParams& p, const ChunkInfo& ci, uint32_t c, uint8_t* crec,
                                                 uint64_t* recbar, uint64_t* recfree) {
  const uint32_t b = c % GV_NREC;
  if (c >= GV_NREC && !mbar_wait(&recfree[b], ((c - GV_NREC) / GV_NREC) & 1)) return false;
  asm volatile("fence.proxy.async;" ::: "memory");
  mbar_expect_tx(&recbar[b], ci.nu * 256);
  bulk_g2s(crec + b * GV_CREC, reinterpret_cast<const uint8_t*>(p.in_runs) + 256ull * ci.cu0, ci.nu * 256,
           &recbar[b], 0ull);
  return true;
}

template <uint32_t DT>
__device__ bool gv_consume(const GvParams& p, const StageIter& it, const ChunkInfo* chunks, uint8_t* ring,
                           uint64_t* full, uint64_t* empty, const XRun* rec, float* acc, uint64_t* recbar,
                           uint64_t* recfree) {
  const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  uint32_t slot = 0, phase = 0;
  for (uint32_t c = 0; c < it.nch; c++) {
    const uint32_t nu = chunks[c].nu, tb = chunks[c].tb;
    // lanes past the chunk's units, and row slots past the CTA's rows, work
    // on a clamped (valid) unit / row and drop the result: no divergence, so
    // the rows of a warp interleave
    const uint32_t lu = min(lane, nu - 1);
    const float lane_on = lane < nu ? 1.f : 0.f;
    const XRun* rb = rec;
    if (p.chunked_rec) {
      if (!mbar_wait(&recbar[c % GV_NREC], (c / GV_NREC) & 1)) return false;
      rb = reinterpret_cast<const XRun*>(reinterpret_cast<const uint8_t*>(rec) + (c % GV_NREC) * GV_CREC) -
           4 * chunks[c].cu0;
    }
    XRun xr[4];
#pragma unroll
    for (uint32_t j = 0; j < 4; j++) xr[j] = load_run(rb, chunks[c].cu0 + lu, j);
    if (p.chunked_rec) {
      __syncwarp();
      if (lane == 0) mbar_arrive(&recfree[c % GV_NREC]);
      if (threadIdx.x == 0 && c + GV_NREC < it.nch &&
          !gv_issue_records(p, chunks[c + GV_NREC], c + GV_NREC, reinterpret_cast<uint8_t*>(const_cast<XRun*>(rec)),
                            recbar, recfree))
        return false;
    }
    for (uint32_t ra = it.r0; ra < it.r1; ra += GV_ROWS) {
      if (!mbar_wait(&full[slot], phase)) return false;
      const uint8_t* tile = ring + (size_t)slot * p.slot_bytes;
      static_assert(GV_RPW == 2, "a warp takes two rows of a stage");
      // warp w takes rows 2w and 2w + 1 of the stage; a warp past the stage's
      // rows (short GEMVs: o_proj, down and qkv have 24-31 rows per CTA)
      // skips the stage (warp-uniform), and an odd last row pairs with a
      // clamped copy of itself whose sum is dropped
      const uint32_t last = it.r1 - 1 - ra;
      const uint32_t rw0 = GV_PAIRS ? 2 * warp : warp, rw1 = GV_PAIRS ? 2 * warp + 1 : warp + GV_CWARPS;
      float v[2] = {0.f, 0.f};
      if (!GV_PAIRS || rw0 <= last) {
        v[0] = lane_on * unit_dot<DT>(tile + min(rw0, last) * tb, lu, nu, xr);
        v[1] = lane_on * unit_dot<DT>(tile + min(rw1, last) * tb, lu, nu, xr);
      }
      // both sums in one butterfly: the first step leaves row 0's pairs in
      // lanes 0-15 and row 1's in lanes 16-31
      const bool up = lane & 16;
      float a = up ? v[1] : v[0];
      a += __shfl_xor_sync(0xffffffffu, up ? v[0] : v[1], 16);
#pragma unroll
      for (int o = 8; o > 0; o >>= 1) a += __shfl_xor_sync(0xffffffffu, a, o);
      if ((lane & 15) == 0) {
        const uint32_t rw = lane ? rw1 : rw0;
        if (rw <= last) acc[ra - it.r0 + rw] += a;
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

// ---- tensor-parallel exchange of the residual stream -----------------------
// After o_proj and after down every rank holds a partial of the new residual
// x (rank 0's includes the old x).  The GEMV epilogue stores each row's
// partial into the rank's slot of every rank's receive buffer as one 8-byte
// word {value, epoch} (an 8-byte store is seen whole or not at all), over
// NVLink.  The next RMS-normalised GEMV (gate_up, qkv, lm_head) polls its
// own buffer until every word of every slot carries the exchange's epoch and
// sums the W slots in rank order as its input, so every rank computes the
// identical x; each of its CTAs also writes its slice of x for the next
// residual add.  No fence or flag round trip: the data is its own flag.  A
// buffer (exported by CUDA IPC) is uint2 recv[2][W][H]; the epoch's parity
// picks the half, so a rank one exchange ahead never overwrites a slot that
// is still being read (a rank's exchange e+2 needs every rank's e+1, which
// each rank sends only after it read e).  epoch = *ar_base + k + 1, where
// ar_base advances by the step's exchange count at every step's end and k
// numbers the exchanges inside the step; all ranks run the same steps.  A
// word that does not arrive within the wait limit (GvParams::ar_spin_ns:
// FURNACE_B200_WAIT_MS, default 2 s) sets error 7.
constexpr uint64_t AR_SPIN_NS = 2000000000ull;

uint64_t ar_buffer_bytes(uint32_t H, uint32_t W) { return 2ull * W * H * 8; }

__device__ __forceinline__ void st_volatile_u2(uint2* p, uint2 v) {
  asm volatile("st.volatile.global.v2.u32 [%0], {%1, %2};" ::"l"(p), "r"(v.x), "r"(v.y) : "memory");
}
__device__ __forceinline__ uint4 ld_volatile_u4(const uint4* p) {
  uint4 v;
  asm volatile("ld.volatile.global.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p)
               : "memory");
  return v;
}

// Elements 4i..4i+3 of the exchanged x: the sum of the W ranks' words in rank
// order, each word polled until it carries epoch e.  False on the time limit.
__device__ __forceinline__ bool ar_pull4(const GvParams& p, uint32_t e, uint32_t i, float4* out) {
  const uint4* slot = reinterpret_cast<const uint4*>(p.ar_peers.buf[p.ar_rank]) + ((uint64_t)(e & 1) * p.ar_w * p.ar_h) / 2;
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  for (uint32_t q = 0; q < p.ar_w; q++) {
    const uint4* w = slot + ((uint64_t)q * p.ar_h) / 2 + 2 * i;  // words 4i, 4i+1 | 4i+2, 4i+3
    uint4 a = ld_volatile_u4(w), b = ld_volatile_u4(w + 1);
    if (a.y != e || a.w != e || b.y != e || b.w != e) {
      const uint64_t t0 = gtimer();
      while (a.y != e || a.w != e || b.y != e || b.w != e) {
        if (gtimer() - t0 > p.ar_spin_ns) return false;
        a = ld_volatile_u4(w);
        b = ld_volatile_u4(w + 1);
      }
    }
    acc.x += __uint_as_float(a.x);
    acc.y += __uint_as_float(a.z);
    acc.z += __uint_as_float(b.x);
    acc.w += __uint_as_float(b.z);
  }
  *out = acc;
  return true;
}

__global__ void __launch_bounds__(GV_THREADS, 1) k_gemv(const __grid_constant__ GvParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  const uint32_t tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t NX = runs_for_dev(p.cols);
  uint8_t* ring = smem;
  XRun* rec = reinterpret_cast<XRun*>(ring + (size_t)p.slots * p.slot_bytes);
  float* acc = p.chunked_rec ? reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(rec) + GV_NREC * GV_CREC)
                             : reinterpret_cast<float*>(rec + NX);
  __shared__ __align__(8) uint64_t crecbar[GV_NREC], crecfree[GV_NREC];
  __shared__ float red[GV_CWARPS];
  __shared__ unsigned long long kred[GV_CWARPS];
  __shared__ ChunkInfo chunks[GV_MAX_CH];
  __shared__ __align__(8) uint64_t full[GV_MAX_SLOTS], empty[GV_MAX_SLOTS], recbar;

  StageIter it;
  it.init(p.seg, p.nseg, blockIdx.x);
  if (tid < it.nch && it.n_stages) chunk_info(it, tid, &chunks[tid]);
  if (tid == 0) {
    for (uint32_t s = 0; s < p.slots; s++) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], GV_CWARPS);
    }
    mbar_init(&recbar, 1);
    for (uint32_t b = 0; b < GV_NREC; b++) {
      mbar_init(&crecbar[b], 1);
      mbar_init(&crecfree[b], GV_CWARPS);
    }
    fence_barrier_init();
  }
  __syncthreads();
  if (tid == 0) pdl_trigger();
  Tracer tr;
  if (tid == 0) tr.begin(TR_GEMV + p.epilogue, gridDim.x);

  if (warp == GV_CWARPS) {
    // ---------------- producer (weights only: no wait on the predecessor) ----
    if (lane != 0) return;
    const uint64_t pol = policy_evict_first();
    StageIter nx;
    nx.init(p.next.seg, p.next.nseg, blockIdx.x);
    // L2 prefetch cursors: own stages, then the next kernel's first stages
    uint32_t pc = 0, pr = it.r0;
    const uint32_t nx_nch = nx.n_stages ? nx.nch : 0;
    uint32_t nc = 0, nr = nx.r0;
    ChunkInfo nci = {};
    if (nx_nch) chunk_info(nx, 0, &nci);
    uint64_t copied = 0, prefetched = 0, next_bytes = 0;
    uint32_t slot = 0, phase = 0, i = 0;
    for (uint32_t c = 0; c < it.nch; c++) {
      const ChunkInfo ci = chunks[c];
      for (uint32_t ra = it.r0; ra < it.r1; ra += GV_ROWS, i++) {
        if (i >= p.slots && !mbar_wait(&empty[slot], phase ^ 1)) {
          if (p.state) atomicExch(&p.state->error, 4u);
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

  // ---------------- consumers ----------------
  const uint32_t ctid = tid;
  for (uint32_t r = ctid; r < p.max_rows; r += GV_NT) acc[r] = 0.f;
  // f32 input: x in buf[0..7] and the RMSNorm weight in buf[8..15] when
  // normalising, else x in buf[0..15] (the host bounds cols).  The weight is
  // constant: its loads are issued before the wait on the predecessor.
  const float4* x4 = reinterpret_cast<const float4*>(p.x);
  const float4* w4 = reinterpret_cast<const float4*>(p.norm_w);
  const uint32_t n4 = p.cols / 4;
  const bool norm = !p.in_runs && p.norm_w != nullptr;
  float4 buf[16];
  if (norm) {
#pragma unroll
    for (int j = 8; j < 16; j++) {
      const uint32_t i4 = ctid + GV_NT * (j - 8);
      buf[j] = i4 < n4 ? w4[i4] : make_float4(0.f, 0.f, 0.f, 0.f);
    }
  }
  pdl_wait();  // the predecessor's output (this GEMV's input) is complete
  if (ctid == 0) tr.mark(1);
  if (p.in_runs && p.chunked_rec) {
    // records of a long input stream per chunk (gv_consume): the first GV_NREC
    if (ctid == 0 && it.n_stages)
      for (uint32_t c = 0; c < GV_NREC && c < it.nch; c++)
        gv_issue_records(p, chunks[c], c, reinterpret_cast<uint8_t*>(rec), crecbar, crecfree);
  } else if (p.in_runs) {
    // records written by the producing kernel: one bulk copy
    if (ctid == 0) {
      mbar_expect_tx(&recbar, NX * 64);
      bulk_g2s(rec, p.in_runs, NX * 64, &recbar, 0ull);
    }
    if (!mbar_wait(&recbar, 0)) {
      if (lane == 0 && p.state) atomicExch(&p.state->error, 3u);
      return;
    }
  } else if (p.ar_pull) {
    // tensor parallelism: x = the sum of the ranks' exchanged partials; this
    // CTA writes its slice of x (src/model.rs:470, :477 summed over ranks)
    const uint32_t e = *p.ar_base + p.ar_k + 1;
    const uint32_t s0 = blockIdx.x * n4 / gridDim.x, s1 = (blockIdx.x + 1) * n4 / gridDim.x;
    bool okp = true;
#pragma unroll
    for (int j = 0; j < 8; j++) {
      const uint32_t i4 = ctid + GV_NT * j;
      buf[j] = make_float4(0.f, 0.f, 0.f, 0.f);
      if (i4 < n4) {
        okp = ar_pull4(p, e, i4, &buf[j]) && okp;
        if (i4 >= s0 && i4 < s1) reinterpret_cast<float4*>(p.x_out)[i4] = buf[j];
      }
    }
    if (!okp && p.state) atomicExch(&p.state->error, 7u);
  } else {
    // f32 input (RMS-normalised when norm_w is set) -> records; every x load
    // of this thread in flight at once
#pragma unroll
    for (int j = 0; j < 16; j++) {
      if (norm && j >= 8) break;
      const uint32_t i4 = ctid + GV_NT * j;
      buf[j] = i4 < n4 ? x4[i4] : make_float4(0.f, 0.f, 0.f, 0.f);
    }
  }
  if (!p.in_runs) {
    float inv = 1.f;
    if (norm) {
      float ss = 0.f;
#pragma unroll
      for (int j = 0; j < 8; j++) {
        ss = fmaf(buf[j].x, buf[j].x, ss);
        ss = fmaf(buf[j].y, buf[j].y, ss);
        ss = fmaf(buf[j].z, buf[j].z, ss);
        ss = fmaf(buf[j].w, buf[j].w, ss);
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
      if (lane == 0) red[warp] = ss;
      named_sync(1, GV_NT);
      float tot = 0.f;
#pragma unroll
      for (int w = 0; w < GV_CWARPS; w++) tot += red[w];
      inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, (float)p.cols), p.eps)));
    }
#pragma unroll
    for (int j = 0; j < 16; j++) {
      if (norm && j >= 8) break;
      if (GV_NT * j >= 4 * NX) break;  // block-uniform
      const uint32_t i4 = ctid + GV_NT * j;
      float v[4] = {buf[j].x, buf[j].y, buf[j].z, buf[j].w};
      if (norm) {
        const float4 wn = buf[j + 8];
        v[0] = __fmul_rn(__fmul_rn(v[0], inv), wn.x);
        v[1] = __fmul_rn(__fmul_rn(v[1], inv), wn.y);
        v[2] = __fmul_rn(__fmul_rn(v[2], inv), wn.z);
        v[3] = __fmul_rn(__fmul_rn(v[3], inv), wn.w);
      }
      quad_to_run(v, i4 & 3, (i4 >> 2) < NX ? rec : nullptr, i4 >> 2);
    }
  }
  named_sync(1, GV_NT);
  if (ctid == 0) tr.mark(2);

  bool ok = true;
  if (it.n_stages) {
    switch (it.dt) {
      case FZ_Q4_K: ok = gv_consume<FZ_Q4_K>(p, it, chunks, ring, full, empty, rec, acc, crecbar, crecfree); break;
      case FZ_Q6_K: ok = gv_consume<FZ_Q6_K>(p, it, chunks, ring, full, empty, rec, acc, crecbar, crecfree); break;
      case FZ_Q8_0: ok = gv_consume<FZ_Q8_0>(p, it, chunks, ring, full, empty, rec, acc, crecbar, crecfree); break;
      case FZ_Q5_0: ok = gv_consume<FZ_Q5_0>(p, it, chunks, ring, full, empty, rec, acc, crecbar, crecfree); break;
    }
  }
  if (!ok) {
    if (lane == 0 && p.state) atomicExch(&p.state->error, 3u);
    return;
  }
  named_sync(1, GV_NT);
  if (ctid == 0) tr.mark(3);

  // ---------------- epilogue ----------------
  if (!it.n_stages) return;
  const GvSeg& s = *it.s;
  const uint32_t nrows = it.r1 - it.r0;
  if (p.epilogue == EPI_STORE) {
    for (uint32_t i = ctid; i < nrows; i += GV_NT) {
      uint32_t row = it.r0 + i;
      s.out[row] = s.bias ? __fadd_rn(acc[i], s.bias[row]) : acc[i];
    }
  } else if (p.epilogue == EPI_RESID && p.ar_push) {
    // tensor parallelism: this rank's partial of x + W v (rank 0 adds x) to
    // every rank's slot (the exchange above)
    const uint32_t e = *p.ar_base + p.ar_k + 1;
    const uint64_t slot = ((uint64_t)(e & 1) * p.ar_w + p.ar_rank) * p.ar_h;
    for (uint32_t i = ctid; i < nrows; i += GV_NT) {
      const uint32_t row = it.r0 + i;
      const float v = p.ar_rank == 0 ? __fadd_rn(s.out[row], acc[i]) : acc[i];
      const uint2 w = make_uint2(__float_as_uint(v), e);
      for (uint32_t q = 0; q < p.ar_w; q++)
        st_volatile_u2(reinterpret_cast<uint2*>(p.ar_peers.buf[q]) + slot + row, w);
    }
  } else if (p.epilogue == EPI_RESID) {
    // x += W v (src/model.rs:470, :477)
    for (uint32_t i = ctid; i < nrows; i += GV_NT) {
      uint32_t row = it.r0 + i;
      s.out[row] = __fadd_rn(s.out[row], acc[i]);
    }
  } else if (p.epilogue == EPI_SWIGLU) {
    // rows interleave gate/up: h = silu(gate) * up (src/tensor.rs:213-227).
    // Thread i4 makes h of pairs 4 i4 .. 4 i4 + 3 and its quad turns them
    // into one run record (the CTA's rows are whole 32-row units, so its h
    // values are whole runs starting at run r0 / 32); warps past the CTA's
    // pairs skip, the others run every lane through the quad shuffles
    const uint32_t np = nrows / 2, n4 = np / 4;
    for (uint32_t base = 0; base < n4; base += GV_NT) {
      if (base + warp * 32 >= n4) break;  // warp-uniform
      const uint32_t i4 = base + ctid;
      const bool act = i4 < n4;
      float v[4] = {0.f, 0.f, 0.f, 0.f};
      if (act) {
#pragma unroll
        for (int q = 0; q < 4; q++) {
          const uint32_t j = 4 * i4 + q;
          const float g = acc[2 * j], u = acc[2 * j + 1];
          v[q] = __fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, expf(-g))), u);
          if (s.out) s.out[(it.r0 >> 1) + j] = v[q];
        }
      }
      if (p.out_runs) quad_to_run(v, i4 & 3, act ? p.out_runs : nullptr, it.r0 / 32 + (i4 >> 2));
    }
  } else {
    unsigned long long best = 0;
    for (uint32_t i = ctid; i < nrows; i += GV_NT) {
      uint32_t row = it.r0 + i;
      float v = acc[i];
      s.out[row] = v;
      unsigned long long k = argmax_key(v, row + p.idx_base);
      best = k > best ? k : best;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
      best = other > best ? other : best;
    }
    if (lane == 0) kred[warp] = best;
    named_sync(1, GV_NT);
    if (ctid == 0) {
      unsigned long long m = 0;
      for (int w = 0; w < GV_CWARPS; w++) m = kred[w] > m ? kred[w] : m;
      atomicMax(&p.state->argmax_key, m);
    }
  }
  if (ctid == 0) tr.mark(4);
}

// ---- host side ---------------------------------------------------------------
#ifndef GV_SMEM_KB
#define GV_SMEM_KB 200
#endif
constexpr uint32_t GV_SMEM = GV_SMEM_KB * 1024;  // one block per SM
#ifndef GV_PF_AHEAD_KB
#define GV_PF_AHEAD_KB 96
#endif
#ifndef GV_PF_NEXT_KB
#define GV_PF_NEXT_KB 64
#endif
constexpr uint32_t GV_PF_AHEAD = GV_PF_AHEAD_KB * 1024;  // L2 prefetch distance ahead of the copies
constexpr uint32_t GV_PF_NEXT = GV_PF_NEXT_KB * 1024;    // of the next kernel's stream, per CTA

// Install (cap > 0) or remove (cap == 0) the decode-step trace buffer.
void trace_install(TraceRec* buf, uint32_t cap) {
  CK(cudaMemcpyToSymbol(g_trace, &buf, sizeof buf));
  CK(cudaMemcpyToSymbol(g_trace_cap, &cap, sizeof cap));
  trace_reset(0);
}

void trace_reset(cudaStream_t s) {
  uint32_t z = 0;
  CK(cudaMemcpyToSymbolAsync(g_trace_n, &z, sizeof z, 0, cudaMemcpyHostToDevice, s));
}

uint32_t trace_count() {
  uint32_t n = 0;
  CK(cudaMemcpyFromSymbol(&n, g_trace_n, sizeof n));
  return n;
}

void kernels_init() {
  CK(cudaFuncSetAttribute(k_gemv, cudaFuncAttributeMaxDynamicSharedMemorySize, GV_SMEM));
  num_sms();
}

static uint32_t epi_align(int epi) { return epi == EPI_SWIGLU ? 32 : 1; }

// CTA ranges: one block per SM split in proportion to bytes, each segment's
// rows divided into whole `align`-row units as evenly as the count allows.
static void fill_segs(const GemvLaunch& g, GvSeg* out) {
  const uint32_t sms = (uint32_t)num_sms();
  const uint32_t align = epi_align(g.epilogue);
  uint64_t total = 0;
  for (int i = 0; i < g.nseg; i++) total += (uint64_t)g.seg[i].w.rows * dev_row_stride(g.seg[i].w.dtype, g.seg[i].w.cols);
  uint32_t begin = 0;
  for (int i = 0; i < g.nseg; i++) {
    const DevMat& w = g.seg[i].w;
    if (w.rows % align) fail(FZ_EINVAL, "gemv: %u rows not a multiple of %u", w.rows, align);
    uint32_t units = w.rows / align;
    uint32_t share = g.nseg == 1 ? sms
                                 : (uint32_t)((double)sms * (double)((uint64_t)w.rows * dev_row_stride(w.dtype, w.cols)) /
                                                  (double)total + 0.5);
    share = std::max<uint32_t>(1, std::min(share, units));
    uint32_t per = (units + share - 1) / share;
    uint32_t n = (units + per - 1) / per;
    out[i] = GvSeg{w.ptr, w.rows, w.dtype, w.cols, g.seg[i].bias, g.seg[i].out, begin, begin + n, align, {}};
    const uint32_t nch = lay_nch(w.cols);
    if (nch > GV_MAX_CH) fail(FZ_EINVAL, "gemv: input width %u too large", w.cols);
    for (uint32_t c = 0; c <= nch; c++) {
      out[i].ch.cu0[c] = (uint16_t)lay_cu0(w.dtype, w.cols, c);
      out[i].ch.off[c] = lay_chunk_off(w.dtype, w.cols, c);
    }
    begin += n;
  }
}

uint32_t gemv_ctas(const GemvLaunch& g) {
  GvSeg s[3];
  fill_segs(g, s);
  return s[g.nseg - 1].cta_end;
}

void launch_gemv(const GemvLaunch& g, cudaStream_t st) {
  GvParams p{};
  uint32_t cols = g.seg[0].w.cols;
  for (int i = 0; i < g.nseg; i++)
    if (g.seg[i].w.cols != cols) fail(FZ_EINVAL, "gemv segments disagree on input width");
  if (!g.in_runs && !g.x) fail(FZ_EINVAL, "gemv: no input activation");
  if (!g.in_runs && (cols / 4 > (g.norm_w ? 8u : 16u) * GV_NT || cols % 32))
    fail(FZ_EINVAL, "gemv: input width %u unsupported for an f32 input", cols);
  if (lay_nch(cols) > GV_MAX_CH) fail(FZ_EINVAL, "gemv: input width %u too large", cols);
  fill_segs(g, p.seg);
  uint32_t grid = p.seg[g.nseg - 1].cta_end;
  p.nseg = g.nseg;
  p.cols = cols;
  p.in_runs = reinterpret_cast<const XRun*>(g.in_runs);
  p.x = g.x;
  p.norm_w = g.norm_w;
  p.eps = g.eps;
  p.epilogue = g.epilogue;
  p.state = g.state;
  p.out_runs = reinterpret_cast<XRun*>(g.out_runs);
  p.idx_base = g.idx_base;
  if (g.ar_push || g.ar_pull) {
    if (!g.ar_base || g.ar_w < 2 || g.ar_w > (uint32_t)AR_MAX_RANKS || g.ar_h % 4 || !g.state)
      fail(FZ_EINVAL, "gemv: bad tensor-parallel exchange");
    if (g.ar_pull && (g.in_runs || !g.norm_w || cols != g.ar_h))
      fail(FZ_EINVAL, "gemv: the exchange feeds an RMS-normalised f32 input only");
    if (g.ar_push && (g.epilogue != EPI_RESID || g.seg[0].w.rows != g.ar_h))
      fail(FZ_EINVAL, "gemv: the exchange is fed by a residual epilogue only");
    p.ar_peers = g.ar_peers;
    p.ar_w = g.ar_w;
    p.ar_rank = g.ar_rank;
    p.ar_k = g.ar_k;
    p.ar_h = g.ar_h;
    p.ar_base = g.ar_base;
    p.ar_push = g.ar_push;
    p.ar_pull = g.ar_pull;
    p.x_out = const_cast<float*>(g.x);
    p.ar_spin_ns = g.ar_spin_ns ? g.ar_spin_ns : AR_SPIN_NS;
    if (const char* e = getenv("FURNACE_B200_WAIT_MS"))
      if (atof(e) > 0) p.ar_spin_ns = (uint64_t)(atof(e) * 1e6);
  }
  uint32_t max_rows = 0, slot = 0;
  for (int i = 0; i < g.nseg; i++) {
    const GvSeg& s = p.seg[i];
    uint32_t n = s.cta_end - s.cta_begin, units = s.rows / s.align;
    max_rows = std::max(max_rows, s.align * ((units + n - 1) / n) + s.align);
    slot = std::max(slot, GV_ROWS * lay_max_chunk_bytes(s.dtype, s.cols));
  }
  slot = (slot + 127) & ~127u;
  uint32_t fixed = runs_for(cols) * 64 + 4 * max_rows + 128;
  if (g.in_runs && fixed + 2 * slot > GV_SMEM) {
    // a long record input (ffn hidden of the large configs): stream it
    p.chunked_rec = 1;
    fixed = GV_NREC * GV_CREC + 4 * max_rows + 128;
  }
  if (fixed + 2 * slot > GV_SMEM) fail(FZ_EINVAL, "gemv: %u rows per block exceed shared memory", max_rows);
  uint32_t slots = std::min<uint32_t>(GV_MAX_SLOTS, (GV_SMEM - fixed) / slot);
  p.slots = slots;
  p.slot_bytes = slot;
  p.max_rows = max_rows;
  p.pf_ahead = GV_PF_AHEAD;
  if (g.next) {
    fill_segs(*g.next, p.next.seg);
    p.next.nseg = g.next->nseg;
    p.next.budget = GV_PF_NEXT;
  }
  size_t smem = (size_t)slots * slot + fixed;
  launch_pdl(k_gemv, dim3(grid), dim3(GV_THREADS), smem, st, p);
}

// Embedding lookup of state->token (src/model.rs:482-506): one dequantized row.
__global__ void k_embed(uint32_t dt, const uint8_t* __restrict__ base, uint32_t cols, uint32_t vocab,
                        StepState* __restrict__ st, float* __restrict__ x) {
  pdl_trigger();
  pdl_wait();
  const uint32_t tok = st->token, u = blockIdx.x * blockDim.x + threadIdx.x;
  if (tok >= vocab) {
    // the host validates ids before they reach the device; this is a guard
    if (u == 0) st->error = 1;
  }
  if (u < (cols + 63) / 64) dequant_unit(dt, base, vocab, tok < vocab ? tok : 0, cols, u, x + 64 * u);
}

void launch_embed(const DevMat& emb, StepState* st, float* x, cudaStream_t s) {
  uint32_t units = (emb.cols + 63) / 64;
  launch_pdl(k_embed, dim3((units + 63) / 64), dim3(64), 0, s, emb.dtype, (const uint8_t*)emb.ptr, emb.cols, emb.rows,
             st, x);
}

// ---------------------------------------------------------------------------
// Attention (src/model.rs:371-438) with RoPE (src/model.rs:193-217) and the
// KV append (src/model.rs:346-356) folded in: flash-decode.  Grid
// (S, n_kv), S = ceil(#SM / n_kv): a block owns one KV head, the G = nh/nkv
// query heads that read it, and an equal share of positions [0, pos] (sized
// from pos at run time, so every block has work at every position).  K/V
// rows stream through a 3-deep ring of 32-position tiles by bulk copy; warp
// h keeps head h's online softmax (running max, sum and weighted V).  The
// block that owns pos rotates the new k, appends k and v to the cache and
// places them in its last tile.  k_attn_combine merges the S partials.
// RoPE uses host-computed cos/sin (glibc powf/sinf/cosf: the reference's own
// factors) and the reference's uncontracted a*c - b*s / a*s + b*c.
// ---------------------------------------------------------------------------
constexpr int AT_THREADS = 256;
constexpr int AT_MAXG = 8;
constexpr int AT_TP = 32;    // positions per tile
// Build parameters: tiles in flight per block, and blocks per SM that the
// split count is sized for (3 blocks need AT_NBUF_DEF=2 to fit in shared
// memory; measured slower on C3)
#ifndef AT_NBUF_DEF
#define AT_NBUF_DEF 3
#endif
#ifndef AT_CTAS_PER_SM
#define AT_CTAS_PER_SM 2
#endif
constexpr int AT_NBUF = AT_NBUF_DEF;  // tiles in flight

// KV cache elements: f32 (the reference's KvCache) or f16 (FZ_KV_F16: values
// rounded to nearest even when appended, read back exactly).
__device__ __forceinline__ float4 kv_ld4(const float* row, uint32_t c) { return reinterpret_cast<const float4*>(row)[c]; }
__device__ __forceinline__ float4 kv_ld4(const __half* row, uint32_t c) {
  const uint2 u = reinterpret_cast<const uint2*>(row)[c];
  const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&u.x));
  const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&u.y));
  return make_float4(a.x, a.y, b.x, b.y);
}
__device__ __forceinline__ float kv_ld(const float* p) { return *p; }
__device__ __forceinline__ float kv_ld(const __half* p) { return __half2float(*p); }
// The value as stored: f32 unchanged, f16 rounded to nearest even.
template <typename KT>
__device__ __forceinline__ float kv_round(float v) {
  return sizeof(KT) == 4 ? v : __half2float(__float2half_rn(v));
}
__device__ __forceinline__ void kv_st(float* p, float v) { *p = v; }
__device__ __forceinline__ void kv_st(__half* p, float v) { *p = __float2half_rn(v); }

template <int HD, typename KT>
__global__ void __launch_bounds__(AT_THREADS) k_attn(const float* __restrict__ qkv, const float2* __restrict__ cs,
                                                      KT* __restrict__ kc, KT* __restrict__ vc,
                                                      float* __restrict__ partials, uint32_t nh, uint32_t nkv,
                                                      uint32_t max_ctx, StepState* st) {
  constexpr uint32_t EB = sizeof(KT);
  constexpr int DPL = HD / 32;
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ __align__(8) uint64_t bar[AT_NBUF];
  const uint32_t G = nh / nkv, kvh = blockIdx.y, split = blockIdx.x, S = gridDim.x;
  const uint32_t tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const uint32_t half = HD / 2;
  KT* tiles = reinterpret_cast<KT*>(smem);  // [NBUF][K|V][TP][HD]
  const KT* kvk = kc + (uint64_t)kvh * max_ctx * HD;
  const KT* kvv = vc + (uint64_t)kvh * max_ctx * HD;
  __shared__ uint32_t s_p0, s_pre;
  const uint64_t pol = policy_evict_first();
  // tile j of a block owning positions [ta, tb) while the new position is pc:
  // positions [ta + j*TP, ..) below pc come from the cache
  auto issue = [&](uint32_t j, uint32_t ta, uint32_t tb, uint32_t pc) {
    uint32_t b = j % AT_NBUF, a = ta + j * AT_TP, e = min(min(tb, a + AT_TP), pc);
    uint32_t rows = e > a ? e - a : 0;
    KT* kt = tiles + (size_t)b * 2 * AT_TP * HD;
    mbar_expect_tx(&bar[b], 2 * rows * HD * EB);
    if (rows) {
      bulk_g2s(kt, kvk + (uint64_t)a * HD, rows * HD * EB, &bar[b], pol);
      bulk_g2s(kt + AT_TP * HD, kvv + (uint64_t)a * HD, rows * HD * EB, &bar[b], pol);
    }
  };
  Tracer tr;
  if (tid == 0) {
    tr.begin(TR_ATTN, gridDim.x * gridDim.y);
    pdl_trigger();
    for (int b = 0; b < AT_NBUF; b++) mbar_init(&bar[b], 1);
    fence_barrier_init();
  }
  __syncthreads();  // barrier init visible
  if (tid == 0) {
    // Rows below the position read here are final already (it is this step's
    // position, or the previous step's if k_finalize has not published it
    // yet): the first tiles of the share that position gives this block are
    // copied before waiting for the predecessor, the rest of the share is
    // pulled into L2.  After the wait, a block whose share moved (pos != p0)
    // lets those copies land and starts over.
    const uint32_t p0 = min(*((volatile uint32_t*)&st->pos), max_ctx - 1);
    const uint32_t tot0 = p0 + 1, per0 = (tot0 + S - 1) / S;
    const uint32_t a0 = min(split * per0, tot0), b0 = min(tot0, a0 + per0);
    const uint32_t pre = min((b0 - a0 + AT_TP - 1) / AT_TP, (uint32_t)AT_NBUF);
    for (uint32_t j = 0; j < pre; j++) issue(j, a0, b0, p0);
    const uint32_t f0 = min(a0 + pre * AT_TP, p0), f1 = min(b0, p0);
    if (f1 > f0) {
      bulk_prefetch(kvk + (uint64_t)f0 * HD, (f1 - f0) * HD * EB);
      bulk_prefetch(kvv + (uint64_t)f0 * HD, (f1 - f0) * HD * EB);
    }
    s_p0 = p0;
    s_pre = pre;
  }
  pdl_wait();
  if (tid == 0) tr.mark(1);
  const uint32_t pos = st->pos;
  __syncthreads();  // s_p0, s_pre
  const uint32_t pre = s_pre;
  const bool redo = pos != s_p0;  // block-uniform
  if (redo || pos >= max_ctx) {
    // the early copies land before their buffers are reused or the block exits
    if (tid == 0)
      for (uint32_t j = 0; j < pre; j++)
        if (!mbar_wait(&bar[j], 0)) st->error = 5;
    __syncthreads();
  }
  if (pos >= max_ctx) {
    if (tid == 0) st->error = 2;
    return;
  }
  const uint32_t total = pos + 1, per = (total + S - 1) / S;
  const uint32_t t0 = min(split * per, total), t1 = min(total, t0 + per), n = t1 - t0;
  const uint32_t ntiles = (n + AT_TP - 1) / AT_TP;
  // parity of tile j's buffer: uses before it, plus the drained early copy
  auto parity = [&](uint32_t j) { return ((j / AT_NBUF) + ((redo && (j % AT_NBUF) < pre) ? 1u : 0u)) & 1u; };
  if (tid == 0)
    for (uint32_t j = redo ? 0 : pre; j < ntiles && j < (uint32_t)AT_NBUF; j++) issue(j, t0, t1, pos);
  // rotated query of warp w's head, dims lane*DPL .. lane*DPL + DPL - 1, in
  // registers: dim i < half is a*c - b*s, dim i + half is a*s + b*c, with
  // (a, b) = (q[i], q[i + half]) and (c, s) = the table's row pos, entry i
  const float2* csp = cs + (uint64_t)pos * half;
  float qv[DPL];
  if (warp < G) {
    const float* x = qkv + (uint64_t)(kvh * G + warp) * HD;
    const uint32_t i0 = lane * DPL, j0 = i0 < half ? i0 : i0 - half;
#pragma unroll
    for (int d = 0; d < DPL; d++) {
      const float a = x[j0 + d], b = x[j0 + d + half];
      const float2 c = csp[j0 + d];
      qv[d] = i0 < half ? __fsub_rn(__fmul_rn(a, c.x), __fmul_rn(b, c.y))
                        : __fadd_rn(__fmul_rn(a, c.y), __fmul_rn(b, c.x));
    }
  }
  const bool owns_pos = n && t1 == total;
  float kn[2] = {0.f, 0.f}, vn[2] = {0.f, 0.f};
  if (owns_pos && tid < half) {
    // rotate the new k, append k and v (KvCache::append)
    const float* kx = qkv + (uint64_t)(nh + kvh) * HD;
    const float* vx = qkv + (uint64_t)(nh + nkv + kvh) * HD;
    float a = kx[tid], b = kx[tid + half];
    float2 c = csp[tid];
    // the values as cached (f16: rounded), used for this position too
    kn[0] = kv_round<KT>(__fsub_rn(__fmul_rn(a, c.x), __fmul_rn(b, c.y)));
    kn[1] = kv_round<KT>(__fadd_rn(__fmul_rn(a, c.y), __fmul_rn(b, c.x)));
    vn[0] = kv_round<KT>(vx[tid]);
    vn[1] = kv_round<KT>(vx[tid + half]);
    KT* kdst = kc + ((uint64_t)kvh * max_ctx + pos) * HD;
    KT* vdst = vc + ((uint64_t)kvh * max_ctx + pos) * HD;
    kv_st(kdst + tid, kn[0]);
    kv_st(kdst + tid + half, kn[1]);
    kv_st(vdst + tid, vn[0]);
    kv_st(vdst + tid + half, vn[1]);
  }
  if (tid == 0) tr.mark(2);
  const float scale = __fdiv_rn(1.0f, __fsqrt_rn((float)HD));
  float m = -INFINITY, l = 0.f, acc[DPL];
#pragma unroll
  for (int d = 0; d < DPL; d++) acc[d] = 0.f;
  for (uint32_t j = 0; j < ntiles; j++) {
    const uint32_t b = j % AT_NBUF, a = t0 + j * AT_TP, tn = min(t1, a + AT_TP) - a;
    KT* kt = tiles + (size_t)b * 2 * AT_TP * HD;
    KT* vt = kt + AT_TP * HD;
    if (!mbar_wait(&bar[b], parity(j))) {
      if (tid == 0) st->error = 5;
      return;
    }
    if (owns_pos && pos >= a && pos < a + AT_TP) {  // block-uniform
      if (tid < half) {
        kv_st(kt + (pos - a) * HD + tid, kn[0]);
        kv_st(kt + (pos - a) * HD + tid + half, kn[1]);
        kv_st(vt + (pos - a) * HD + tid, vn[0]);
        kv_st(vt + (pos - a) * HD + tid + half, vn[1]);
      }
      __syncthreads();
    }
    if (warp < G) {
      const uint32_t t = lane;
      float s = -INFINITY;
      {
        // lane L multiplies dims L*DPL.. of every row of the tile with its
        // registers of q (each K row read once, 16 B per lane); then a
        // transpose reduction over the 32 lanes leaves position t's score
        // in lane t
        float part[AT_TP];
#pragma unroll
        for (int r = 0; r < AT_TP; r++) {
          part[r] = 0.f;
          if ((uint32_t)r < tn) {  // warp-uniform
            if constexpr (DPL == 4) {
              const float4 k4 = kv_ld4(kt + (size_t)r * HD, lane);
              part[r] = (qv[0] * k4.x + qv[1] * k4.y) + (qv[2] * k4.z + qv[3] * k4.w);
            } else {
              const KT* kr = kt + (size_t)r * HD + lane * DPL;
              part[r] = qv[0] * kv_ld(kr) + qv[1] * kv_ld(kr + 1);
            }
          }
        }
#pragma unroll
        for (int o = AT_TP / 2; o > 0; o >>= 1) {
          const bool up = lane & o;
#pragma unroll
          for (int i = 0; i < o; i++) {
            const float keep = up ? part[i + o] : part[i], send = up ? part[i] : part[i + o];
            part[i] = keep + __shfl_xor_sync(0xffffffffu, send, o);
          }
        }
        if (t < tn) s = __fmul_rn(part[0], scale);
      }
      float mt = s;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, o));
      const float mn = fmaxf(m, mt);
      const float alpha = expf(m - mn);
      const float pr = t < tn ? expf(s - mn) : 0.f;
      float ps = pr;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) ps += __shfl_xor_sync(0xffffffffu, ps, o);
      l = fmaf(l, alpha, ps);
      m = mn;
#pragma unroll
      for (int d = 0; d < DPL; d++) acc[d] *= alpha;
#pragma unroll 8
      for (uint32_t t2 = 0; t2 < tn; t2++) {
        const float pt = __shfl_sync(0xffffffffu, pr, t2);
        const KT* vr = vt + (size_t)t2 * HD + lane * DPL;
        if (DPL == 4) {  // one load per lane: consecutive lanes, no bank conflict
          const float4 v4 = kv_ld4(vt + (size_t)t2 * HD, lane);
          acc[0] = fmaf(pt, v4.x, acc[0]);
          acc[1] = fmaf(pt, v4.y, acc[1]);
          acc[2] = fmaf(pt, v4.z, acc[2]);
          acc[3] = fmaf(pt, v4.w, acc[3]);
        } else {
#pragma unroll
          for (int d = 0; d < DPL; d++) acc[d] = fmaf(pt, kv_ld(vr + d), acc[d]);
        }
      }
    }
    __syncthreads();  // buffer b free
    if (tid == 0 && j + AT_NBUF < ntiles) issue(j + AT_NBUF, t0, t1, pos);
  }
  if (tid == 0) tr.mark(3);
  // partials: stats [nkv][G][S] of (max, sum), then acc [nkv][G][S][HD]
  // (a split's weighted V is one contiguous row: coalesced stores here and
  // coalesced loads in the combine)
  if (warp < G) {
    float2* stats = reinterpret_cast<float2*>(partials) + (uint64_t)kvh * G * S;
    float* pacc = partials + ((2 * (uint64_t)nkv * G * S + 3) & ~3ull) + (((uint64_t)kvh * G + warp) * S + split) * HD;
    if (lane == 0) stats[warp * S + split] = make_float2(m, l);
    if constexpr (DPL == 4)
      reinterpret_cast<float4*>(pacc)[lane] = make_float4(acc[0], acc[1], acc[2], acc[3]);
    else
      reinterpret_cast<float2*>(pacc)[lane] = make_float2(acc[0], acc[1]);
  }
  if (tid == 0) tr.mark(4);
}

// Merge the split partials: ctx[h][d] = sum_s w_s acc_s[d] / sum_s w_s l_s,
// w_s = exp(m_s - max_s m_s).  Grid nh, block AT_CB_THREADS (4 warps).  Warp
// w takes splits w, w + 4, ...; lane L holds dims L*DPT .. L*DPT + DPT - 1
// (DPT = hd / 32), so one load instruction of a warp reads one split's
// contiguous row.  Every load of a thread -- its first AT_CB_REGS splits and,
// per warp, the head's split statistics -- is issued right after the wait,
// so the merge costs one L2 round trip; each warp reduces the statistics
// itself.  The four warps' sums meet in shared memory, added in warp order
// (split s mod 4 chains, then (c0 + c1) + (c2 + c3)).
constexpr int AT_MAXS = 256;
constexpr int AT_CB_THREADS = 128;
constexpr int AT_CB_REGS = 24;  // splits per warp whose rows are held in registers
template <int DPT>
__global__ void __launch_bounds__(AT_CB_THREADS) k_attn_combine(const float* __restrict__ partials,
                                                                 float* __restrict__ ctx, XRun* __restrict__ ctx_runs,
                                                                 uint32_t nh, uint32_t nkv, uint32_t S, StepState* st,
                                                                 uint32_t run0) {
  constexpr uint32_t HD = 32 * DPT;
  using VecT = typename std::conditional<DPT == 4, float4, float2>::type;
  __shared__ float ws[4][AT_MAXS];
  __shared__ __align__(16) float red[4][HD];
  __shared__ float sv[HD];
  Tracer tr;
  if (threadIdx.x == 0) {
    tr.begin(TR_COMBINE, gridDim.x);
    pdl_trigger();
  }
  pdl_wait();
  if (threadIdx.x == 0) tr.mark(1);
  (void)st;
  const uint32_t G = nh / nkv, h = blockIdx.x, kvh = h / G, hg = h % G;
  const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const float2* stats = reinterpret_cast<const float2*>(partials) + ((uint64_t)kvh * G + hg) * S;
  const VecT* rows = reinterpret_cast<const VecT*>(partials + ((2 * (uint64_t)nkv * G * S + 3) & ~3ull) +
                                                   (uint64_t)h * S * HD) + lane;
  VecT av[AT_CB_REGS];
#pragma unroll
  for (int k = 0; k < AT_CB_REGS; k++) {
    const uint32_t s2 = warp + 4 * k;
    if (s2 < S) av[k] = rows[(uint64_t)s2 * (HD / DPT)];
  }
  float2 sm[AT_MAXS / 32];
#pragma unroll
  for (int k = 0; k < AT_MAXS / 32; k++) {
    const uint32_t s2 = lane + 32 * k;
    sm[k] = s2 < S ? stats[s2] : make_float2(-INFINITY, 0.f);
  }
  float M = -INFINITY;
#pragma unroll
  for (int k = 0; k < AT_MAXS / 32; k++) M = fmaxf(M, sm[k].x);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
  float den = 0.f;
#pragma unroll
  for (int k = 0; k < AT_MAXS / 32; k++) {
    const float w = sm[k].x == -INFINITY ? 0.f : expf(sm[k].x - M);
    ws[warp][lane + 32 * k] = w;
    den = fmaf(w, sm[k].y, den);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) den += __shfl_xor_sync(0xffffffffu, den, o);
  __syncwarp();
  const float* w = ws[warp];
  float n[DPT];
#pragma unroll
  for (int i = 0; i < DPT; i++) n[i] = 0.f;
#pragma unroll
  for (int k = 0; k < AT_CB_REGS; k++) {
    const uint32_t s2 = warp + 4 * k;
    if (s2 >= S) break;
    const float* a = reinterpret_cast<const float*>(&av[k]);
#pragma unroll
    for (int i = 0; i < DPT; i++) n[i] = fmaf(w[s2], a[i], n[i]);
  }
  for (uint32_t s2 = warp + 4 * AT_CB_REGS; s2 < S; s2 += 4) {
    const VecT v4 = rows[(uint64_t)s2 * (HD / DPT)];
    const float* a = reinterpret_cast<const float*>(&v4);
#pragma unroll
    for (int i = 0; i < DPT; i++) n[i] = fmaf(w[s2], a[i], n[i]);
  }
#pragma unroll
  for (int i = 0; i < DPT; i++) red[warp][lane * DPT + i] = n[i];
  __syncthreads();
  // thread d < HD: the head's output element d
  const uint32_t d = threadIdx.x;
  float v = 0.f;
  if (d < HD) {
    const float num = (red[0][d] + red[1][d]) + (red[2][d] + red[3][d]);
    v = __fdiv_rn(num, den);
    ctx[(uint64_t)h * HD + d] = v;
    sv[d] = v;
  }
  if (threadIdx.x == 0) tr.mark(2);
  __syncthreads();
  // run records of ctx (the o_proj input): HD / 16 runs per head
  if (d < HD) values_to_runs(sv, HD, nullptr, ctx_runs, run0 + h * (HD / 16), d, HD);
  if (threadIdx.x == 0) tr.mark(4);
}

// AT_CTAS_PER_SM blocks per SM (2): more warps in flight hide the latency-bound tile loop.
uint32_t attention_splits(uint32_t n_kv) {
  uint32_t s = (AT_CTAS_PER_SM * (uint32_t)num_sms() + n_kv - 1) / n_kv;
  return s < 1 ? 1 : s > AT_MAXS ? AT_MAXS : s;
}

uint64_t attention_partial_floats(uint32_t nh, uint32_t nkv, uint32_t hd, uint32_t splits) {
  uint32_t G = nh / nkv;
  return ((2ull * nkv * G * splits + 3) & ~3ull) + (uint64_t)nkv * G * splits * hd;
}

static size_t attention_smem(uint32_t hd, uint32_t eb = 4) { return (size_t)AT_NBUF * 2 * AT_TP * hd * eb; }

void attention_init() {
  CK(cudaFuncSetAttribute(k_attn<128, float>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)attention_smem(128)));
  CK(cudaFuncSetAttribute(k_attn<64, float>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)attention_smem(64)));
  CK(cudaFuncSetAttribute(k_attn<128, __half>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                          (int)attention_smem(128, 2)));
  CK(cudaFuncSetAttribute(k_attn<64, __half>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)attention_smem(64, 2)));
}

void launch_attention(const AttnLaunch& a, cudaStream_t s) {
  uint32_t G = a.n_heads / a.n_kv;
  if (G > AT_MAXG) fail(FZ_EINVAL, "attention: GQA group %u > %d", G, AT_MAXG);
  uint32_t splits = a.splits;
  if (splits > AT_MAXS) fail(FZ_EINVAL, "attention: %u splits > %d", splits, AT_MAXS);
  dim3 grid(splits, a.n_kv);
  const float2* cs = reinterpret_cast<const float2*>(a.rope_cs);
  float *kf = static_cast<float*>(a.kcache), *vf = static_cast<float*>(a.vcache);
  __half *kh = static_cast<__half*>(a.kcache), *vh = static_cast<__half*>(a.vcache);
  if (a.hd == 128 && !a.kv_f16)
    launch_pdl(k_attn<128, float>, grid, dim3(AT_THREADS), attention_smem(128), s, a.qkv, cs, kf, vf, a.partials,
               a.n_heads, a.n_kv, a.max_ctx, a.state);
  else if (a.hd == 64 && !a.kv_f16)
    launch_pdl(k_attn<64, float>, grid, dim3(AT_THREADS), attention_smem(64), s, a.qkv, cs, kf, vf, a.partials,
               a.n_heads, a.n_kv, a.max_ctx, a.state);
  else if (a.hd == 128)
    launch_pdl(k_attn<128, __half>, grid, dim3(AT_THREADS), attention_smem(128, 2), s, a.qkv, cs, kh, vh,
               a.partials, a.n_heads, a.n_kv, a.max_ctx, a.state);
  else if (a.hd == 64)
    launch_pdl(k_attn<64, __half>, grid, dim3(AT_THREADS), attention_smem(64, 2), s, a.qkv, cs, kh, vh, a.partials,
               a.n_heads, a.n_kv, a.max_ctx, a.state);
  else
    fail(FZ_EINVAL, "head_dim %u unsupported (64 or 128)", a.hd);
  if (a.hd == 128)
    launch_pdl(k_attn_combine<4>, dim3(a.n_heads), dim3(AT_CB_THREADS), 0, s, (const float*)a.partials, a.ctx,
               reinterpret_cast<XRun*>(a.ctx_runs), a.n_heads, a.n_kv, splits, a.state, a.ctx_run0);
  else
    launch_pdl(k_attn_combine<2>, dim3(a.n_heads), dim3(AT_CB_THREADS), 0, s, (const float*)a.partials, a.ctx,
               reinterpret_cast<XRun*>(a.ctx_runs), a.n_heads, a.n_kv, splits, a.state, a.ctx_run0);
}

// ---------------------------------------------------------------------------
// Step bookkeeping: the sampled id (first max, src/generate.rs:69-77), the
// next input token (forced prompt token or the id itself), pos += 1.
// ---------------------------------------------------------------------------
__global__ void k_finalize(StepState* st, const uint32_t* forced, uint32_t* ids_out, int has_logits,
                           uint32_t* ar_base, uint32_t ar_step) {
  pdl_trigger();
  pdl_wait();
  if (ar_base) *ar_base += ar_step;
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

void launch_finalize(StepState* st, const uint32_t* forced, uint32_t* ids_out, bool has_logits, cudaStream_t s,
                     uint32_t* ar_base, uint32_t ar_step) {
  launch_pdl(k_finalize, dim3(1), dim3(1), 0, s, st, forced, ids_out, has_logits ? 1 : 0, ar_base, ar_step);
}

// ---------------------------------------------------------------------------
// Prefill on the tensor cores
// ---------------------------------------------------------------------------
#include "prefill.cuh"

void prefill_init() {
  CK(cudaFuncSetAttribute(k_qgemm, cudaFuncAttributeMaxDynamicSharedMemorySize, QG_SMEM));
  CK(cudaFuncSetAttribute(k_attn_prefill<128, float>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                          (int)ap_smem<128, float>()));
  CK(cudaFuncSetAttribute(k_attn_prefill<64, float>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                          (int)ap_smem<64, float>()));
  CK(cudaFuncSetAttribute(k_attn_prefill<128, __half>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                          (int)ap_smem<128, __half>()));
  CK(cudaFuncSetAttribute(k_attn_prefill<64, __half>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                          (int)ap_smem<64, __half>()));
}

uint64_t wpanel_elems(uint32_t rows, uint32_t K) { return (uint64_t)((rows + QG_M - 1) / QG_M) * QG_M * K; }
uint64_t xpanel_elems(uint32_t T, uint32_t K) { return (uint64_t)((T + QG_N - 1) / QG_N) * QG_N * K; }

void launch_wpanels(const DevMat& m, uint32_t row0, int8_t* rexp, void* hi, void* lo, cudaStream_t s) {
  if (m.cols % 64) fail(FZ_EINVAL, "prefill: %u columns not a multiple of 64", m.cols);
  k_rowexp<<<(m.rows * 32 + 255) / 256, 256, 0, s>>>(m, row0, rexp);
  CK(cudaGetLastError());
  const uint64_t n = (uint64_t)m.rows * (m.cols / 64);
  k_wpanels<<<(unsigned)((n + 127) / 128), 128, 0, s>>>(m, row0, rexp, reinterpret_cast<__half*>(hi),
                                                        reinterpret_cast<__half*>(lo));
  CK(cudaGetLastError());
}

void launch_xpanels(const float* x, uint32_t ld, uint32_t T, uint32_t K, const float* w, float eps, void* hi,
                    void* lo, int8_t* texp, cudaStream_t s) {
  if (K % 64) fail(FZ_EINVAL, "prefill: width %u not a multiple of 64", K);
  if (ld % 4) fail(FZ_EINVAL, "prefill: row stride %u not a multiple of 4", ld);
  k_xpanels<<<(T + XP_TOK - 1) / XP_TOK, 256, 0, s>>>(x, ld, T, K, w, eps, reinterpret_cast<__half*>(hi),
                                                      reinterpret_cast<__half*>(lo), texp);
  CK(cudaGetLastError());
}

void launch_qgemm(const QgemmLaunch& q, cudaStream_t s) {
  if (q.K % QG_KB || q.K == 0) fail(FZ_EINVAL, "prefill gemm: K %u not a multiple of %u", q.K, QG_KB);
  QgParams p{};
  p.ahi = reinterpret_cast<const __half*>(q.ahi);
  p.alo = reinterpret_cast<const __half*>(q.alo);
  p.bhi = reinterpret_cast<const __half*>(q.bhi);
  p.blo = reinterpret_cast<const __half*>(q.blo);
  p.K = q.K;
  p.N = q.N;
  p.T = q.T;
  p.epi = q.epi;
  p.out = q.out;
  p.ld = q.ld;
  p.bias = q.bias;
  p.err = q.err;
  p.rexp = q.rexp;
  p.texp = q.texp;
  if (!q.rexp || !q.texp) fail(FZ_EINVAL, "prefill gemm: missing row / token exponents");
  dim3 grid((q.T + QG_N - 1) / QG_N, (q.N + QG_M - 1) / QG_M);
  if (grid.y > 65535) fail(FZ_EINVAL, "prefill gemm: %u output rows", q.N);
  k_qgemm<<<grid, 128, QG_SMEM, s>>>(p);
  CK(cudaGetLastError());
}

void launch_embed_rows(const DevMat& emb, const uint32_t* tokens, uint32_t T, float* x, uint32_t ld, cudaStream_t s) {
  const uint32_t U = emb.cols / 64;
  k_embed_rows<<<dim3((U + 63) / 64, T), 64, 0, s>>>(emb, tokens, x, ld);
  CK(cudaGetLastError());
}

template <typename KT>
static void prefill_attention_t(const float* qkv, uint32_t ldq, const float2* cs, KT* kc, KT* vc, float* ctx,
                                uint32_t ldc, uint32_t nh, uint32_t nkv, uint32_t hd, uint32_t max_ctx, uint32_t pos0,
                                uint32_t T, uint32_t* err, cudaStream_t s) {
  k_kv_append<KT><<<dim3(T, nkv), 64, 0, s>>>(qkv, ldq, nh, nkv, hd, cs, kc, vc, max_ctx, pos0);
  CK(cudaGetLastError());
  const uint32_t G = nh / nkv;
  if (G == 0 || G > AP_ROWS || nh % nkv) fail(FZ_EINVAL, "prefill attention: %u heads over %u KV heads", nh, nkv);
  const dim3 grid((T + AP_ROWS / G - 1) / (AP_ROWS / G), nkv);
  if (hd == 128)
    k_attn_prefill<128, KT><<<grid, AP_THREADS, ap_smem<128, KT>(), s>>>(qkv, ldq, cs, kc, vc, ctx, ldc, nh, nkv,
                                                                        max_ctx, pos0, T, err);
  else
    k_attn_prefill<64, KT><<<grid, AP_THREADS, ap_smem<64, KT>(), s>>>(qkv, ldq, cs, kc, vc, ctx, ldc, nh, nkv,
                                                                      max_ctx, pos0, T, err);
  CK(cudaGetLastError());
}

void launch_prefill_attention(const float* qkv, uint32_t ldq, const float* rope_cs, void* kc, void* vc, bool kv_f16,
                              float* ctx, uint32_t ldc, uint32_t nh, uint32_t nkv, uint32_t hd, uint32_t max_ctx,
                              uint32_t pos0, uint32_t T, uint32_t* err, cudaStream_t s) {
  const float2* cs = reinterpret_cast<const float2*>(rope_cs);
  if (kv_f16)
    prefill_attention_t(qkv, ldq, cs, static_cast<__half*>(kc), static_cast<__half*>(vc), ctx, ldc, nh, nkv, hd,
                        max_ctx, pos0, T, err, s);
  else
    prefill_attention_t(qkv, ldq, cs, static_cast<float*>(kc), static_cast<float*>(vc), ctx, ldc, nh, nkv, hd, max_ctx,
                        pos0, T, err, s);
}

// ---------------------------------------------------------------------------
// Sampling support (src/sampler.rs:39-155): repeat penalty, temperature and
// top-k selection on the device.  Keys (orderable(l / temp) << 32 | ~index)
// sort descending by value and ascending by index on ties, the order of the
// reference's sort of (id, l / temp); the host finishes softmax, top-p and
// the draw from the k survivors.
// ---------------------------------------------------------------------------
constexpr uint32_t TK_BLOCK = 2048;  // logits per pass-1 block
constexpr uint32_t TK_MERGE = 8192;  // keys of the pass-2 sort

__device__ __forceinline__ void bitonic_desc(unsigned long long* keys, uint32_t n) {
  for (uint32_t size = 2; size <= n; size <<= 1)
    for (uint32_t stride = size >> 1; stride > 0; stride >>= 1) {
      __syncthreads();
      for (uint32_t i = threadIdx.x; i < n / 2; i += blockDim.x) {
        const uint32_t pos = 2 * i - (i & (stride - 1)), partner = pos + stride;
        const bool desc = (pos & size) == 0;
        const unsigned long long a = keys[pos], b = keys[partner];
        if ((a < b) == desc) {
          keys[pos] = b;
          keys[partner] = a;
        }
      }
    }
  __syncthreads();
}

// Pass 1: the top k of each block of TK_BLOCK logits (penalised, scaled).
__global__ void k_topk1(const float* __restrict__ logits, uint32_t V, const uint32_t* __restrict__ recent, uint32_t nr,
                        float pen, float temp, uint32_t k, unsigned long long* __restrict__ out) {
  __shared__ unsigned long long keys[TK_BLOCK];
  __shared__ uint32_t rs[64];
  if (threadIdx.x < nr) rs[threadIdx.x] = recent[threadIdx.x];
  __syncthreads();
  for (uint32_t j = threadIdx.x; j < TK_BLOCK; j += blockDim.x) {
    const uint32_t i = blockIdx.x * TK_BLOCK + j;
    unsigned long long key = 0;
    if (i < V) {
      float l = logits[i];
      if (pen != 1.0f) {  // apply_repeat_penalty (src/sampler.rs:39-55): once per distinct recent token
        bool seen = false;
        for (uint32_t r = 0; r < nr; r++) seen |= rs[r] == i;
        if (seen) l = l > 0.0f ? __fdiv_rn(l, pen) : __fmul_rn(l, pen);
      }
      key = argmax_key(__fdiv_rn(l, temp), i);
    }
    keys[j] = key;
  }
  bitonic_desc(keys, TK_BLOCK);
  for (uint32_t j = threadIdx.x; j < k; j += blockDim.x) out[(uint64_t)blockIdx.x * k + j] = keys[j];
}

// Pass 2: the top k of all blocks' survivors.
__global__ void k_topk2(const unsigned long long* __restrict__ in, uint32_t n, uint32_t k,
                        unsigned long long* __restrict__ out) {
  extern __shared__ unsigned long long mkeys[];
  uint32_t m = 2;
  while (m < n) m <<= 1;
  for (uint32_t j = threadIdx.x; j < m; j += blockDim.x) mkeys[j] = j < n ? in[j] : 0ull;
  bitonic_desc(mkeys, m);
  for (uint32_t j = threadIdx.x; j < k; j += blockDim.x) out[j] = mkeys[j];
}

uint32_t topk_max() { return 64; }

void launch_topk(const float* logits, uint32_t V, const uint32_t* recent, uint32_t nr, float pen, float temp,
                 uint32_t k, void* scratch, void* out, cudaStream_t s) {
  if (k == 0 || k > topk_max() || nr > 64) fail(FZ_EINVAL, "top-k %u / %u recent tokens unsupported on the device", k, nr);
  const uint32_t nb = (V + TK_BLOCK - 1) / TK_BLOCK;
  if (nb * k > TK_MERGE) fail(FZ_EINVAL, "top-k: vocabulary %u too large for k = %u", V, k);
  unsigned long long* mid = reinterpret_cast<unsigned long long*>(scratch);
  k_topk1<<<nb, 256, 0, s>>>(logits, V, recent, nr, pen, temp, k, mid);
  CK(cudaGetLastError());
  uint32_t m = 2;
  while (m < nb * k) m <<= 1;
  k_topk2<<<1, 1024, m * sizeof(unsigned long long), s>>>(mid, nb * k, k, reinterpret_cast<unsigned long long*>(out));
  CK(cudaGetLastError());
}

size_t topk_scratch_bytes(uint32_t V) { return (size_t)((V + TK_BLOCK - 1) / TK_BLOCK) * topk_max() * 8 + 64; }

void sampler_init() {
  CK(cudaFuncSetAttribute(k_topk2, cudaFuncAttributeMaxDynamicSharedMemorySize, TK_MERGE * 8));
}


}  // namespace fz
