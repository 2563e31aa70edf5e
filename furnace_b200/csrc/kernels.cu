// Device code of the decode path (sm_100a).
//
// Device layout of a quantized weight [rows, cols] ("DL"): rows are
// contiguous, each padded to 16 bytes, and every row holds exactly the GGUF
// bytes of that row, reordered so that the bulk data of a 32-element unit
// starts on a 16-byte boundary:
//   Q4_K  native 144-byte super-blocks (already 16-byte aligned).
//   Q6_K  [nb x 208-byte bodies][nb x f16 d]; a body is four 48-byte groups
//         (ql run a, ql run b, qh run) followed by the 16 signed scales
//         reordered so each half-group's two scales are adjacent.
//   Q8_0  [cols int8 quants][nb x f16 d].
//   Q5_0  [nb x 16 nibble bytes][nb x u32 high bits][nb x f16 d].
// Every format is consumed in units of 32 elements whose activations are
// two contiguous runs of 16 (xa, xb), so a thread keeps one unit's x in
// registers while it walks R rows.
//
// Dequantization is bit-exact with the reference block decoders
// (src/quant.rs:17-133): same integer unpack, same f32 products in the same
// order, no contraction (__fmul_rn/__fsub_rn).  The GEMV reassociates its sums
// (the parity bar for matmul outputs is 1e-4 relative).

#include <cuda_fp16.h>

#include <cstdio>

#include "fz_internal.h"
#include "kernels.h"

namespace fz {

#define CK(x)                                                                               \
  do {                                                                                      \
    cudaError_t e_ = (x);                                                                   \
    if (e_ != cudaSuccess) fail(FZ_ECUDA, "%s failed: %s", #x, cudaGetErrorString(e_));     \
  } while (0)

static inline uint64_t round16(uint64_t v) { return (v + 15) & ~uint64_t(15); }

uint64_t dev_row_stride(uint32_t dtype, uint32_t cols) {
  switch (dtype) {
    case FZ_Q4_K: return (uint64_t)(cols / 256) * 144;
    case FZ_Q6_K: return round16((uint64_t)(cols / 256) * 210);
    case FZ_Q8_0: return round16((uint64_t)cols + (cols / 32) * 2);
    case FZ_Q5_0: return round16((uint64_t)(cols / 32) * 22);
    case FZ_F32: return round16((uint64_t)cols * 4);
    default: return 0;
  }
}

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

__device__ __forceinline__ float h2f(uint32_t bits16) { return __half2float(__ushort_as_half((unsigned short)(bits16 & 0xffff))); }

__device__ __forceinline__ uint4 ldg16(const uint8_t* p) { return __ldg(reinterpret_cast<const uint4*>(p)); }
__device__ __forceinline__ uint32_t ldg_u16(const uint8_t* p) { return __ldg(reinterpret_cast<const unsigned short*>(p)); }
__device__ __forceinline__ uint32_t ldg_u32(const uint8_t* p) { return __ldg(reinterpret_cast<const unsigned int*>(p)); }

// ---------------------------------------------------------------------------
// Repack: GGUF rows -> device layout.  One thread per (row, block).
// ---------------------------------------------------------------------------
__global__ void k_repack(uint32_t dtype, const uint8_t* __restrict__ raw, uint8_t* __restrict__ dst, uint32_t rows,
                         uint32_t cols, uint64_t stride) {
  uint32_t be = (dtype == FZ_Q4_K || dtype == FZ_Q6_K) ? 256 : 32;
  uint32_t bb = dtype == FZ_Q4_K ? 144 : dtype == FZ_Q6_K ? 210 : dtype == FZ_Q8_0 ? 34 : 22;
  uint32_t nb = cols / be;
  uint64_t idx = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (uint64_t)rows * nb) return;
  uint64_t r = idx / nb;
  uint32_t b = (uint32_t)(idx % nb);
  const uint8_t* src = raw + (r * nb + b) * bb;
  uint8_t* row = dst + r * stride;
  switch (dtype) {
    case FZ_Q4_K:
      for (int i = 0; i < 144; i++) row[(uint64_t)b * 144 + i] = src[i];
      break;
    case FZ_Q6_K: {
      uint8_t* body = row + (uint64_t)b * 208;
      for (int uu = 0; uu < 4; uu++) {
        int h = uu >> 1, is = uu & 1, l0 = 16 * is;
        for (int i = 0; i < 16; i++) {
          body[48 * uu + i] = src[64 * h + l0 + i];            // ql run a
          body[48 * uu + 16 + i] = src[64 * h + 32 + l0 + i];  // ql run b
          body[48 * uu + 32 + i] = src[128 + 32 * h + l0 + i];  // qh run
        }
        const uint8_t* sc = src + 192;
        body[192 + 4 * uu + 0] = sc[8 * h + is];      // group 0 (ql a low)
        body[192 + 4 * uu + 1] = sc[8 * h + is + 4];  // group 2 (ql a high)
        body[192 + 4 * uu + 2] = sc[8 * h + is + 2];  // group 1 (ql b low)
        body[192 + 4 * uu + 3] = sc[8 * h + is + 6];  // group 3 (ql b high)
      }
      row[(uint64_t)nb * 208 + 2 * b] = src[208];
      row[(uint64_t)nb * 208 + 2 * b + 1] = src[209];
      break;
    }
    case FZ_Q8_0:
      for (int i = 0; i < 32; i++) row[32 * b + i] = src[2 + i];
      row[cols + 2 * b] = src[0];
      row[cols + 2 * b + 1] = src[1];
      break;
    case FZ_Q5_0:
      for (int i = 0; i < 16; i++) row[16 * b + i] = src[6 + i];
      for (int i = 0; i < 4; i++) row[16 * nb + 4 * b + i] = src[2 + i];
      row[20 * nb + 2 * b] = src[0];
      row[20 * nb + 2 * b + 1] = src[1];
      break;
  }
}

void launch_repack(uint32_t dtype, const uint8_t* raw, uint8_t* dst, uint32_t rows, uint32_t cols, cudaStream_t s) {
  uint32_t be, bb;
  block_geom(dtype, &be, &bb);
  uint64_t n = (uint64_t)rows * (cols / be);
  if (!n) return;
  k_repack<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(dtype, raw, dst, rows, cols, dev_row_stride(dtype, cols));
  CK(cudaGetLastError());
}

// ---------------------------------------------------------------------------
// Exact dequantization of one 32-element unit (src/quant.rs:35-39, 53-63,
// 93-109, 114-133).  `row` is a device-layout row, `o` the row's f32 output.
// ---------------------------------------------------------------------------
__device__ void dequant_unit(uint32_t dtype, const uint8_t* row, uint32_t cols, uint32_t u, float* o) {
  if (dtype == FZ_Q4_K) {
    uint32_t sb = u >> 3, k = u & 7, j64 = k >> 1, l0 = (k & 1) << 4;
    const uint8_t* blk = row + (uint64_t)sb * 144;
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
    const uint8_t* q = blk + 16 + 32 * j64 + l0;
    float* oa = o + 256 * sb + 64 * j64 + l0;
    for (int i = 0; i < 16; i++) {
      oa[i] = __fsub_rn(__fmul_rn(d1, (float)(q[i] & 0x0F)), min1);
      oa[32 + i] = __fsub_rn(__fmul_rn(d2, (float)(q[i] >> 4)), min2);
    }
  } else if (dtype == FZ_Q6_K) {
    uint32_t nb = cols / 256;
    uint32_t sb = u >> 3, v = u & 7, uu = v >> 1, half = v & 1, h = uu >> 1, l0 = (uu & 1) << 4;
    const uint8_t* body = row + (uint64_t)sb * 208;
    const uint8_t* ql = body + 48 * uu + 16 * half;
    const uint8_t* qh = body + 48 * uu + 32;
    float sclo = (float)(int8_t)body[192 + 4 * uu + 2 * half];
    float schi = (float)(int8_t)body[193 + 4 * uu + 2 * half];
    const uint8_t* dp = row + (uint64_t)nb * 208 + 2 * sb;
    float d = h2f(dp[0] | (dp[1] << 8));
    float dlo = __fmul_rn(d, sclo), dhi = __fmul_rn(d, schi);
    int shlo = 2 * half, shhi = 2 * half + 4;
    float* oa = o + 256 * sb + 128 * h + 32 * half + l0;
    for (int i = 0; i < 16; i++) {
      int qlo = (int)((ql[i] & 0x0F) | (((qh[i] >> shlo) & 3) << 4)) - 32;
      int qhi = (int)((ql[i] >> 4) | (((qh[i] >> shhi) & 3) << 4)) - 32;
      oa[i] = __fmul_rn(dlo, (float)qlo);
      oa[64 + i] = __fmul_rn(dhi, (float)qhi);
    }
  } else if (dtype == FZ_Q8_0) {
    const uint8_t* dp = row + cols + 2 * u;
    float d = h2f(dp[0] | (dp[1] << 8));
    for (int i = 0; i < 32; i++) o[32 * u + i] = __fmul_rn(d, (float)(int8_t)row[32 * u + i]);
  } else if (dtype == FZ_Q5_0) {
    uint32_t nb = cols / 32;
    const uint8_t* qs = row + 16 * u;
    const uint8_t* hp = row + 16 * nb + 4 * u;
    uint32_t qh = hp[0] | (hp[1] << 8) | (hp[2] << 16) | ((uint32_t)hp[3] << 24);
    const uint8_t* dp = row + 20 * nb + 2 * u;
    float d = h2f(dp[0] | (dp[1] << 8));
    for (int j = 0; j < 16; j++) {
      uint32_t hi0 = ((qh >> j) & 1) << 4, hi1 = ((qh >> (j + 16)) & 1) << 4;
      o[32 * u + j] = __fmul_rn(d, (float)((int)((qs[j] & 0x0F) | hi0) - 16));
      o[32 * u + j + 16] = __fmul_rn(d, (float)((int)((qs[j] >> 4) | hi1) - 16));
    }
  } else if (dtype == FZ_F32) {
    const float* f = reinterpret_cast<const float*>(row);
    for (int i = 0; i < 32; i++) o[32 * u + i] = f[32 * u + i];
  }
}

__global__ void k_dequant(uint32_t dtype, const uint8_t* __restrict__ base, uint64_t stride, uint32_t cols, uint32_t r0,
                          uint32_t rows, float* __restrict__ out) {
  uint32_t units = cols / 32;
  uint64_t idx = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (uint64_t)rows * units) return;
  uint64_t r = idx / units;
  uint32_t u = (uint32_t)(idx % units);
  dequant_unit(dtype, base + (r0 + r) * stride, cols, u, out + r * cols);
}

void launch_dequant(const DevMat& m, uint32_t r0, uint32_t rows, float* out, cudaStream_t s) {
  uint64_t n = (uint64_t)rows * (m.cols / 32);
  if (!n) return;
  k_dequant<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(m.dtype, m.ptr, m.stride, m.cols, r0, rows, out);
  CK(cudaGetLastError());
}

// Embedding lookup of state->token (src/model.rs:482-506): one dequantized row.
__global__ void k_embed(uint32_t dtype, const uint8_t* __restrict__ base, uint64_t stride, uint32_t cols, uint32_t vocab,
                        const StepState* __restrict__ st, float* __restrict__ x) {
  uint32_t tok = st->token;
  uint32_t u = blockIdx.x * blockDim.x + threadIdx.x;
  if (u >= cols / 32) return;
  if (tok >= vocab) {
    // the host validates ids before they reach the device; this is a guard
    for (int i = 0; i < 32; i++) x[32 * u + i] = 0.f;
    const_cast<StepState*>(st)->error = 1;
    return;
  }
  dequant_unit(dtype, base + (uint64_t)tok * stride, cols, u, x);
}

void launch_embed(const DevMat& emb, const StepState* st, float* x, cudaStream_t s) {
  uint32_t units = emb.cols / 32;
  k_embed<<<(units + 127) / 128, 128, 0, s>>>(emb.dtype, emb.ptr, emb.stride, emb.cols, emb.rows, st, x);
  CK(cudaGetLastError());
}

// ---------------------------------------------------------------------------
// GEMV: y[row] = sum_k W[row, k] x[k] for one activation vector.
//
// Each warp owns groups of R consecutive rows; lane l handles units
// l, l+32, ... of every row in the group, so the 32 activations of a unit
// are loaded from shared memory once and reused R times.  The activation
// vector (optionally RMS-normalised, src/tensor.rs:164-186) lives in shared
// memory.  Partial sums are reduced with warp shuffles.
// ---------------------------------------------------------------------------
constexpr int GEMV_THREADS = 256;
constexpr int GEMV_R = 4;

struct SegParams {
  const uint8_t* w;
  uint64_t stride;
  uint32_t rows, dtype;
  const float* bias;
  float* out;
  uint32_t block_begin, block_end;
};

struct GemvParams {
  SegParams seg[3];
  int nseg;
  uint32_t cols;
  const float* x;
  const float* norm_w;
  float eps;
  int prologue;
  StepState* state;
};

__device__ __forceinline__ void load_x16(const float* xs, uint32_t base, float* v) {
  const float4* p = reinterpret_cast<const float4*>(xs + base);
#pragma unroll
  for (int i = 0; i < 4; i++) {
    float4 f = p[i];
    v[4 * i] = f.x;
    v[4 * i + 1] = f.y;
    v[4 * i + 2] = f.z;
    v[4 * i + 3] = f.w;
  }
}

template <uint32_t DT>
__device__ __forceinline__ void unit_bases(uint32_t u, uint32_t* a, uint32_t* b) {
  if (DT == FZ_Q4_K) {
    uint32_t sb = u >> 3, k = u & 7;
    *a = 256 * sb + 64 * (k >> 1) + ((k & 1) << 4);
    *b = *a + 32;
  } else if (DT == FZ_Q6_K) {
    uint32_t sb = u >> 3, v = u & 7, uu = v >> 1, half = v & 1;
    *a = 256 * sb + 128 * (uu >> 1) + 32 * half + ((uu & 1) << 4);
    *b = *a + 64;
  } else {
    *a = 32 * u;
    *b = 32 * u + 16;
  }
}

__device__ __forceinline__ uint32_t byte_of(uint4 v, int i) {
  uint32_t w = i < 4 ? v.x : i < 8 ? v.y : i < 12 ? v.z : v.w;
  return (w >> (8 * (i & 3))) & 0xff;
}

// dot of one unit of one row with its activations (xa, xb: 16 each).
template <uint32_t DT>
__device__ __forceinline__ float unit_dot(const uint8_t* row, uint32_t cols, uint32_t u, const float* xa, const float* xb,
                                          float sa, float sbx) {
  if (DT == FZ_Q4_K) {
    uint32_t sb = u >> 3, k = u & 7, j64 = k >> 1, l0 = (k & 1) << 4;
    const uint8_t* blk = row + (uint64_t)sb * 144;
    uint4 hdr = ldg16(blk);
    uint4 q = ldg16(blk + 16 + 32 * j64 + l0);
    float d = h2f(hdr.x), dmin = h2f(hdr.x >> 16);
    uint32_t w1 = hdr.y, w2 = hdr.z, w3 = hdr.w;
    uint32_t sh = 16 * (j64 & 1);
    uint32_t sca, ma, scb, mb;
    if (j64 < 2) {
      sca = (w1 >> sh) & 63;
      ma = (w2 >> sh) & 63;
      scb = (w1 >> (sh + 8)) & 63;
      mb = (w2 >> (sh + 8)) & 63;
    } else {
      sca = ((w3 >> sh) & 15) | (((w1 >> (sh + 6)) & 3) << 4);
      ma = ((w3 >> (sh + 4)) & 15) | (((w2 >> (sh + 6)) & 3) << 4);
      scb = ((w3 >> (sh + 8)) & 15) | (((w1 >> (sh + 14)) & 3) << 4);
      mb = ((w3 >> (sh + 12)) & 15) | (((w2 >> (sh + 14)) & 3) << 4);
    }
    float acca = 0.f, accb = 0.f;
#pragma unroll
    for (int i = 0; i < 16; i++) {
      uint32_t byte = byte_of(q, i);
      acca = fmaf(xa[i], (float)(byte & 15), acca);
      accb = fmaf(xb[i], (float)(byte >> 4), accb);
    }
    return d * ((float)sca * acca + (float)scb * accb) - dmin * ((float)ma * sa + (float)mb * sbx);
  } else if (DT == FZ_Q6_K) {
    uint32_t nb = cols >> 8;
    uint32_t sb = u >> 3, v = u & 7, uu = v >> 1, half = v & 1;
    const uint8_t* body = row + (uint64_t)sb * 208;
    uint4 ql = ldg16(body + 48 * uu + 16 * half);
    uint4 qh = ldg16(body + 48 * uu + 32);
    uint32_t sc = ldg_u16(body + 192 + 4 * uu + 2 * half);
    float d = h2f(ldg_u16(row + (uint64_t)nb * 208 + 2 * sb));
    int shlo = 2 * half, shhi = 2 * half + 4;
    float acca = 0.f, accb = 0.f;
#pragma unroll
    for (int i = 0; i < 16; i++) {
      uint32_t l = byte_of(ql, i), h = byte_of(qh, i);
      int qlo = (int)((l & 15) | (((h >> shlo) & 3) << 4)) - 32;
      int qhi = (int)((l >> 4) | (((h >> shhi) & 3) << 4)) - 32;
      acca = fmaf(xa[i], (float)qlo, acca);
      accb = fmaf(xb[i], (float)qhi, accb);
    }
    return d * ((float)(int8_t)(sc & 0xff) * acca + (float)(int8_t)(sc >> 8) * accb);
  } else if (DT == FZ_Q8_0) {
    uint4 q0 = ldg16(row + 32 * u), q1 = ldg16(row + 32 * u + 16);
    float d = h2f(ldg_u16(row + cols + 2 * u));
    float acc = 0.f;
#pragma unroll
    for (int i = 0; i < 16; i++) {
      acc = fmaf(xa[i], (float)(int8_t)byte_of(q0, i), acc);
      acc = fmaf(xb[i], (float)(int8_t)byte_of(q1, i), acc);
    }
    return d * acc;
  } else {  // Q5_0
    uint32_t nb = cols >> 5;
    uint4 qs = ldg16(row + 16 * u);
    uint32_t qh = ldg_u32(row + 16 * nb + 4 * u);
    float d = h2f(ldg_u16(row + 20 * nb + 2 * u));
    float acc = 0.f;
#pragma unroll
    for (int i = 0; i < 16; i++) {
      uint32_t b = byte_of(qs, i);
      int q0 = (int)((b & 15) | (((qh >> i) & 1) << 4)) - 16;
      int q1 = (int)((b >> 4) | (((qh >> (i + 16)) & 1) << 4)) - 16;
      acc = fmaf(xa[i], (float)q0, acc);
      acc = fmaf(xb[i], (float)q1, acc);
    }
    return d * acc;
  }
}

__device__ __forceinline__ unsigned long long argmax_key(float v, uint32_t idx) {
  uint32_t b = __float_as_uint(v);
  uint32_t ord = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
  return ((unsigned long long)ord << 32) | (0xFFFFFFFFu - idx);
}

template <uint32_t DT, int EPI>
__device__ void gemv_seg(const GemvParams& p, const SegParams& s, const float* xs, unsigned long long* best) {
  const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const uint32_t nwarps = GEMV_THREADS / 32;
  const uint32_t units = p.cols / 32;
  const uint32_t total_warps = (s.block_end - s.block_begin) * nwarps;
  const uint32_t groups = (s.rows + GEMV_R - 1) / GEMV_R;
  for (uint32_t g = (blockIdx.x - s.block_begin) * nwarps + warp; g < groups; g += total_warps) {
    const uint32_t r0 = g * GEMV_R;
    const uint8_t* rp[GEMV_R];
#pragma unroll
    for (int r = 0; r < GEMV_R; r++) rp[r] = s.w + (uint64_t)min(r0 + r, s.rows - 1) * s.stride;
    float acc[GEMV_R];
#pragma unroll
    for (int r = 0; r < GEMV_R; r++) acc[r] = 0.f;
    for (uint32_t u = lane; u < units; u += 32) {
      uint32_t ba, bb;
      unit_bases<DT>(u, &ba, &bb);
      float xa[16], xb[16];
      load_x16(xs, ba, xa);
      load_x16(xs, bb, xb);
      float sa = 0.f, sbx = 0.f;
      if (DT == FZ_Q4_K) {
#pragma unroll
        for (int i = 0; i < 16; i++) {
          sa += xa[i];
          sbx += xb[i];
        }
      }
#pragma unroll
      for (int r = 0; r < GEMV_R; r++) acc[r] += unit_dot<DT>(rp[r], p.cols, u, xa, xb, sa, sbx);
    }
#pragma unroll
    for (int r = 0; r < GEMV_R; r++) {
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) acc[r] += __shfl_xor_sync(0xffffffffu, acc[r], o);
    }
    if (EPI == EPI_SWIGLU) {
      // rows are interleaved gate/up: out[(r0+2j)/2] = silu(gate) * up
      if (lane < GEMV_R / 2) {
        float gv = lane == 0 ? acc[0] : acc[2];
        float uv = lane == 0 ? acc[1] : acc[3];
        uint32_t row = r0 + 2 * lane;
        if (row + 1 < s.rows + 1 && row < s.rows) s.out[row >> 1] = __fmul_rn(__fdiv_rn(gv, __fadd_rn(1.0f, expf(-gv))), uv);
      }
    } else if (lane < GEMV_R) {
      float v = acc[0];
#pragma unroll
      for (int r = 1; r < GEMV_R; r++)
        if (lane == r) v = acc[r];
      uint32_t row = r0 + lane;
      if (row < s.rows) {
        if (EPI == EPI_STORE) {
          s.out[row] = s.bias ? __fadd_rn(v, s.bias[row]) : v;
        } else if (EPI == EPI_RESID) {
          s.out[row] = __fadd_rn(s.out[row], v);
        } else if (EPI == EPI_LOGITS) {
          s.out[row] = v;
          unsigned long long k = argmax_key(v, row);
          if (k > *best) *best = k;
        }
      }
    }
  }
}

template <int EPI>
__global__ void __launch_bounds__(GEMV_THREADS) k_gemv(GemvParams p) {
  extern __shared__ float4 smem4[];
  float* xs = reinterpret_cast<float*>(smem4);
  __shared__ float red[GEMV_THREADS / 32];
  __shared__ unsigned long long kred[GEMV_THREADS / 32];
  const uint32_t tid = threadIdx.x;
  // prologue: activation vector into shared memory
  float ss = 0.f;
  for (uint32_t i = tid; i < p.cols; i += GEMV_THREADS) {
    float v = p.x[i];
    xs[i] = v;
    ss = fmaf(v, v, ss);
  }
  if (p.prologue == PRO_RMSNORM) {
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if ((tid & 31) == 0) red[tid >> 5] = ss;
    __syncthreads();
    float tot = 0.f;
    for (int w = 0; w < GEMV_THREADS / 32; w++) tot += red[w];
    float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, (float)p.cols), p.eps)));
    for (uint32_t i = tid; i < p.cols; i += GEMV_THREADS) xs[i] = __fmul_rn(__fmul_rn(xs[i], inv), p.norm_w[i]);
  }
  __syncthreads();
  int si = 0;
  while (si + 1 < p.nseg && blockIdx.x >= p.seg[si].block_end) si++;
  const SegParams& s = p.seg[si];
  unsigned long long best = 0;
  switch (s.dtype) {
    case FZ_Q4_K: gemv_seg<FZ_Q4_K, EPI>(p, s, xs, &best); break;
    case FZ_Q6_K: gemv_seg<FZ_Q6_K, EPI>(p, s, xs, &best); break;
    case FZ_Q8_0: gemv_seg<FZ_Q8_0, EPI>(p, s, xs, &best); break;
    case FZ_Q5_0: gemv_seg<FZ_Q5_0, EPI>(p, s, xs, &best); break;
  }
  if (EPI == EPI_LOGITS) {
    for (int o = 16; o > 0; o >>= 1) {
      unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
      if (other > best) best = other;
    }
    if ((tid & 31) == 0) kred[tid >> 5] = best;
    __syncthreads();
    if (tid == 0) {
      unsigned long long m = 0;
      for (int w = 0; w < GEMV_THREADS / 32; w++) m = kred[w] > m ? kred[w] : m;
      atomicMax(&p.state->argmax_key, m);
    }
  }
}

constexpr size_t GEMV_MAX_SMEM = 200 * 1024;

// Opt the GEMV kernels into large dynamic shared memory (once per device,
// outside any stream capture).
void kernels_init() {
  CK(cudaFuncSetAttribute(k_gemv<EPI_STORE>, cudaFuncAttributeMaxDynamicSharedMemorySize, GEMV_MAX_SMEM));
  CK(cudaFuncSetAttribute(k_gemv<EPI_RESID>, cudaFuncAttributeMaxDynamicSharedMemorySize, GEMV_MAX_SMEM));
  CK(cudaFuncSetAttribute(k_gemv<EPI_SWIGLU>, cudaFuncAttributeMaxDynamicSharedMemorySize, GEMV_MAX_SMEM));
  CK(cudaFuncSetAttribute(k_gemv<EPI_LOGITS>, cudaFuncAttributeMaxDynamicSharedMemorySize, GEMV_MAX_SMEM));
  num_sms();
}

void launch_gemv(const GemvLaunch& g, cudaStream_t st) {
  GemvParams p{};
  uint32_t cols = g.seg[0].w.cols;
  uint64_t total_bytes = 0;
  for (int i = 0; i < g.nseg; i++) total_bytes += (uint64_t)g.seg[i].w.rows * g.seg[i].w.stride;
  // two resident blocks per SM when the activation vector fits twice
  size_t smem = (size_t)cols * 4;
  int per_sm = smem <= 100 * 1024 ? 2 : 1;
  uint32_t budget = (uint32_t)(num_sms() * per_sm);
  uint32_t begin = 0;
  for (int i = 0; i < g.nseg; i++) {
    const DevMat& w = g.seg[i].w;
    uint32_t groups = (w.rows + GEMV_R - 1) / GEMV_R;
    uint32_t want = (uint32_t)((double)budget * (double)((uint64_t)w.rows * w.stride) / (double)total_bytes + 0.5);
    uint32_t maxb = (groups + GEMV_THREADS / 32 - 1) / (GEMV_THREADS / 32);
    want = want < 1 ? 1 : want > maxb ? maxb : want;
    p.seg[i] = SegParams{w.ptr, w.stride, w.rows, w.dtype, g.seg[i].bias, g.seg[i].out, begin, begin + want};
    begin += want;
  }
  p.nseg = g.nseg;
  p.cols = cols;
  p.x = g.x;
  p.norm_w = g.norm_w;
  p.eps = g.eps;
  p.prologue = g.prologue;
  p.state = g.state;
  if (smem > GEMV_MAX_SMEM) fail(FZ_EINVAL, "gemv: %u input columns exceed the shared-memory vector", cols);
  auto run = [&](auto kern, int) { kern<<<begin, GEMV_THREADS, smem, st>>>(p); };
  switch (g.epilogue) {
    case EPI_STORE: run(k_gemv<EPI_STORE>, 0); break;
    case EPI_RESID: run(k_gemv<EPI_RESID>, 1); break;
    case EPI_SWIGLU: run(k_gemv<EPI_SWIGLU>, 2); break;
    case EPI_LOGITS: run(k_gemv<EPI_LOGITS>, 3); break;
  }
  CK(cudaGetLastError());
}

// ---------------------------------------------------------------------------
// RoPE (src/model.rs:193-217) with host-computed cos/sin (glibc powf, sinf,
// cosf, exactly the reference's factors) and K/V append at state->pos
// (KvCache::append, src/model.rs:346-356).  qkv = [q | k | v] after bias.
// ---------------------------------------------------------------------------
__global__ void k_rope_append(float* __restrict__ qkv, const float2* __restrict__ cs, uint32_t nh, uint32_t nkv,
                              uint32_t hd, float* __restrict__ kc, float* __restrict__ vc, uint32_t max_ctx,
                              StepState* __restrict__ st) {
  uint32_t h = blockIdx.x, i = threadIdx.x, half = hd / 2;
  uint32_t pos = st->pos;
  if (pos >= max_ctx) {
    if (i == 0) st->error = 2;
    return;
  }
  if (i >= half) return;
  float2 c = cs[(uint64_t)pos * half + i];  // (cos, sin)
  if (h < nh + nkv) {
    float* x = qkv + (uint64_t)h * hd;
    float a = x[i], b = x[i + half];
    float ra = __fsub_rn(__fmul_rn(a, c.x), __fmul_rn(b, c.y));
    float rb = __fadd_rn(__fmul_rn(a, c.y), __fmul_rn(b, c.x));
    if (h < nh) {
      x[i] = ra;
      x[i + half] = rb;
    } else {
      float* dst = kc + ((uint64_t)(h - nh) * max_ctx + pos) * hd;
      dst[i] = ra;
      dst[i + half] = rb;
    }
  } else {
    uint32_t kh = h - nh - nkv;
    const float* v = qkv + (uint64_t)(nh + nkv + kh) * hd;
    float* dst = vc + ((uint64_t)kh * max_ctx + pos) * hd;
    dst[i] = v[i];
    dst[i + half] = v[i + half];
  }
}

void launch_rope_append(float* qkv, const float* rope_cs, uint32_t n_heads, uint32_t n_kv, uint32_t hd, float* kcache,
                        float* vcache, uint32_t max_ctx, const StepState* st, cudaStream_t s) {
  k_rope_append<<<n_heads + 2 * n_kv, hd / 2, 0, s>>>(qkv, reinterpret_cast<const float2*>(rope_cs), n_heads, n_kv, hd,
                                                       kcache, vcache, max_ctx, const_cast<StepState*>(st));
  CK(cudaGetLastError());
}

// ---------------------------------------------------------------------------
// Split-K flash-decode attention (src/model.rs:371-438): grid (splits, n_kv).
// Each block takes one KV head, all G = nh/nkv query heads that read it, and
// a contiguous slice of positions [0, pos].  Phase 1 scores (lanes split the
// head dimension), phase 2 softmax statistics, phase 3 the weighted V sum;
// the block writes (acc, max, sum) partials and the last block of the head
// (atomic ticket) merges them into ctx.
// ---------------------------------------------------------------------------
constexpr int ATT_THREADS = 256;
constexpr int ATT_MAXG = 8;
constexpr int ATT_MAXP = 256;
constexpr int ATT_MAXS = 128;

template <int HD>
__global__ void __launch_bounds__(ATT_THREADS) k_attention(const float* __restrict__ q, const float* __restrict__ kc,
                                                           const float* __restrict__ vc, float* __restrict__ ctx,
                                                           float* __restrict__ partials, unsigned int* counters,
                                                           uint32_t nh, uint32_t nkv, uint32_t max_ctx,
                                                           const StepState* __restrict__ st) {
  constexpr int DPL = HD / 32;
  __shared__ float sc[ATT_MAXG][ATT_MAXP];
  __shared__ float sacc[ATT_THREADS / 32][ATT_MAXG][HD];
  __shared__ float sm[ATT_MAXG], sl[ATT_MAXG];
  __shared__ float wts[ATT_MAXG][ATT_MAXS];
  __shared__ int s_last;
  const uint32_t G = nh / nkv, kvh = blockIdx.y, split = blockIdx.x, S = gridDim.x;
  const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  // the host keeps pos < max_ctx; the clamp keeps every read in bounds regardless
  const uint32_t total = min(st->pos + 1, max_ctx);
  const uint32_t t0 = (uint32_t)((uint64_t)total * split / S), t1 = (uint32_t)((uint64_t)total * (split + 1) / S);
  const uint32_t n = t1 - t0;
  const float scale = __fdiv_rn(1.0f, __fsqrt_rn((float)HD));
  const float* kbase = kc + (uint64_t)kvh * max_ctx * HD;
  const float* vbase = vc + (uint64_t)kvh * max_ctx * HD;

  float qr[ATT_MAXG][DPL];
#pragma unroll
  for (int h = 0; h < ATT_MAXG; h++)
#pragma unroll
    for (int d = 0; d < DPL; d++) qr[h][d] = h < (int)G ? q[(uint64_t)(kvh * G + h) * HD + lane * DPL + d] : 0.f;

  // phase 1: scores
  for (uint32_t t = warp; t < n; t += ATT_THREADS / 32) {
    const float* kp = kbase + (uint64_t)(t0 + t) * HD + lane * DPL;
    float kv[DPL];
#pragma unroll
    for (int d = 0; d < DPL; d++) kv[d] = kp[d];
#pragma unroll
    for (int h = 0; h < ATT_MAXG; h++) {
      if (h >= (int)G) break;
      float s = 0.f;
#pragma unroll
      for (int d = 0; d < DPL; d++) s = fmaf(qr[h][d], kv[d], s);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
      if (lane == 0) sc[h][t] = __fmul_rn(s, scale);
    }
  }
  __syncthreads();
  // phase 2: per-head max and exp-sum over this slice
  if (warp < G) {
    float m = -INFINITY;
    for (uint32_t t = lane; t < n; t += 32) m = fmaxf(m, sc[warp][t]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    float l = 0.f;
    for (uint32_t t = lane; t < n; t += 32) {
      float e = expf(sc[warp][t] - m);
      sc[warp][t] = e;
      l += e;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) l += __shfl_xor_sync(0xffffffffu, l, o);
    if (lane == 0) {
      sm[warp] = m;
      sl[warp] = l;
    }
  }
  __syncthreads();
  // phase 3: weighted V sum
  float acc[ATT_MAXG][DPL];
#pragma unroll
  for (int h = 0; h < ATT_MAXG; h++)
#pragma unroll
    for (int d = 0; d < DPL; d++) acc[h][d] = 0.f;
  for (uint32_t t = warp; t < n; t += ATT_THREADS / 32) {
    const float* vp = vbase + (uint64_t)(t0 + t) * HD + lane * DPL;
    float vv[DPL];
#pragma unroll
    for (int d = 0; d < DPL; d++) vv[d] = vp[d];
#pragma unroll
    for (int h = 0; h < ATT_MAXG; h++) {
      if (h >= (int)G) break;
      float pw = sc[h][t];
#pragma unroll
      for (int d = 0; d < DPL; d++) acc[h][d] = fmaf(pw, vv[d], acc[h][d]);
    }
  }
#pragma unroll
  for (int h = 0; h < ATT_MAXG; h++)
#pragma unroll
    for (int d = 0; d < DPL; d++)
      if (h < (int)G) sacc[warp][h][lane * DPL + d] = acc[h][d];
  __syncthreads();
  float* part = partials + ((uint64_t)kvh * S + split) * G * (HD + 2);
  for (uint32_t idx = threadIdx.x; idx < G * HD; idx += ATT_THREADS) {
    uint32_t h = idx / HD, d = idx % HD;
    float s = 0.f;
    for (int w = 0; w < ATT_THREADS / 32; w++) s += sacc[w][h][d];
    part[h * (HD + 2) + d] = s;
  }
  if (threadIdx.x < G) {
    part[threadIdx.x * (HD + 2) + HD] = n ? sm[threadIdx.x] : -INFINITY;
    part[threadIdx.x * (HD + 2) + HD + 1] = n ? sl[threadIdx.x] : 0.f;
  }
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) s_last = atomicAdd(&counters[kvh], 1u) == S - 1;
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  // merge the S partials of this KV head
  const float* pk = partials + (uint64_t)kvh * S * G * (HD + 2);
  if (threadIdx.x < G) {
    uint32_t h = threadIdx.x;
    float M = -INFINITY;
    for (uint32_t s = 0; s < S; s++) M = fmaxf(M, __ldcg(pk + ((uint64_t)s * G + h) * (HD + 2) + HD));
    float den = 0.f;
    for (uint32_t s = 0; s < S; s++) {
      float ms = __ldcg(pk + ((uint64_t)s * G + h) * (HD + 2) + HD);
      float w = ms == -INFINITY ? 0.f : expf(ms - M);
      wts[h][s] = w;
      den += w * __ldcg(pk + ((uint64_t)s * G + h) * (HD + 2) + HD + 1);
    }
    sl[h] = den;
  }
  __syncthreads();
  for (uint32_t idx = threadIdx.x; idx < G * HD; idx += ATT_THREADS) {
    uint32_t h = idx / HD, d = idx % HD;
    float num = 0.f;
    for (uint32_t s = 0; s < S; s++) num = fmaf(wts[h][s], __ldcg(pk + ((uint64_t)s * G + h) * (HD + 2) + d), num);
    ctx[(uint64_t)(kvh * G + h) * HD + d] = __fdiv_rn(num, sl[h]);
  }
  if (threadIdx.x == 0) counters[kvh] = 0;
}

uint32_t attention_splits(uint32_t n_kv, uint32_t max_ctx, int sms) {
  uint32_t s = (uint32_t)((sms + n_kv - 1) / n_kv);
  uint32_t need = (max_ctx + ATT_MAXP - 1) / ATT_MAXP;
  if (s < need) s = need;
  if (s > ATT_MAXS) s = ATT_MAXS;
  return s;
}

void launch_attention(const AttnLaunch& a, cudaStream_t s) {
  uint32_t G = a.n_heads / a.n_kv;
  if (G > ATT_MAXG || a.splits > ATT_MAXS || (uint64_t)a.splits * ATT_MAXP < a.max_ctx)
    fail(FZ_EINVAL, "attention geometry unsupported (group %u, splits %u, max_ctx %u)", G, a.splits, a.max_ctx);
  dim3 grid(a.splits, a.n_kv);
  if (a.hd == 128)
    k_attention<128><<<grid, ATT_THREADS, 0, s>>>(a.q, a.kcache, a.vcache, a.ctx, a.partials, a.counters, a.n_heads,
                                                 a.n_kv, a.max_ctx, a.state);
  else if (a.hd == 64)
    k_attention<64><<<grid, ATT_THREADS, 0, s>>>(a.q, a.kcache, a.vcache, a.ctx, a.partials, a.counters, a.n_heads,
                                                a.n_kv, a.max_ctx, a.state);
  else
    fail(FZ_EINVAL, "head_dim %u unsupported (64 or 128)", a.hd);
  CK(cudaGetLastError());
}

// ---------------------------------------------------------------------------
// Step bookkeeping: the sampled id (first max, src/generate.rs:69-77), the
// next input token (forced prompt token or the id itself), pos += 1.
// ---------------------------------------------------------------------------
__global__ void k_finalize(StepState* st, const uint32_t* forced, uint32_t* ids_out, int has_logits) {
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
  k_finalize<<<1, 1, 0, s>>>(st, forced, ids_out, has_logits ? 1 : 0);
  CK(cudaGetLastError());
}

}  // namespace fz
