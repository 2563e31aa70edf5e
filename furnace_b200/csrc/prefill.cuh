// Prefill on the tensor cores: batched forward of a run of prompt tokens.
// Included by kernels.cu (shares dequant_unit and the bulk-copy / mbarrier
// helpers).
//
// Every matrix product of a prefill chunk of T tokens is Y[T, N] = X[T, K] W^T
// with W quantized.  The reference computes it in f32 (src/tensor.rs:86-136);
// here:
//   * W is dequantized exactly (dequant_unit, the reference's arithmetic) and
//     split into fp16 hi and lo' = (w - hi) * 2^11, stored as "panels";
//   * X (after RMSNorm where the layer applies one) is split the same way;
//   * tcgen05.mma (kind::f16, f32 accumulation in tensor memory) forms
//     hi.hi in one accumulator and hi.lo' + lo'.hi in another; the epilogue
//     adds them as acc1 + acc2 * 2^-11.  The dropped lo.lo term is ~2^-22 of
//     each product, so the result carries about 22 significant bits.
//
// Panel layout (UMMA K-major, no swizzle): a matrix of R rows and K columns
// (K a multiple of 64, R padded to the panel height P = 128 for weights or
// 256 for tokens) is stored as panels of P rows x 64 columns, panel (b, kb)
// at index b * (K / 64) + kb.  Inside a panel the 8-row x 8-element core
// matrix (rg, kc) sits at byte (kc * P/8 + rg) * 128 and row i of it at
// +16 i: leading-byte offset (between k-chunks) P/8 * 128, stride-byte
// offset (between row groups) 128.  One MMA (K = 16) reads k-chunks 2s and
// 2s + 1 of a panel.

constexpr uint32_t QG_M = 128;          // weight rows per CTA (UMMA M)
constexpr uint32_t QG_N = 256;          // tokens per CTA (UMMA N)
constexpr uint32_t QG_KB = 64;          // K per stage
constexpr uint32_t QG_STAGES = 2;
constexpr uint32_t QG_APANEL = QG_M * QG_KB * 2;   // bytes of one A panel (16 KB)
constexpr uint32_t QG_BPANEL = QG_N * QG_KB * 2;   // bytes of one B panel (32 KB)
constexpr uint32_t QG_STAGE = 2 * QG_APANEL + 2 * QG_BPANEL;
constexpr uint32_t QG_SMEM = QG_STAGES * QG_STAGE + 1024;
constexpr float QG_LO = 2048.0f;        // lo' = (x - hi) * QG_LO

enum : int { QE_STORE = 0, QE_RESID = 1, QE_SWIGLU = 2 };

__host__ __device__ __forceinline__ uint32_t panel_elem(uint32_t P, uint32_t rr, uint32_t k) {
  return ((k >> 3) * (P >> 3) + (rr >> 3)) * 64 + (rr & 7) * 8 + (k & 7);  // in fp16 elements
}

// Power-of-two scaling of the fp16 split: every weight row and every token
// row is multiplied by 2^e before the split, with e chosen from the row's
// largest magnitude so that it lands in [2^13, 2^14): no element overflows
// fp16 (|x| > 65504 would become inf) and small rows keep the split's full
// precision instead of falling into fp16 subnormals.  The GEMM epilogue
// multiplies by 2^-(e_row + e_token).  Power-of-two scaling is exact.
__device__ __forceinline__ int pow2_exp(float amax) {
  if (!(amax > 0.f) || !isfinite(amax)) return 0;
  int ex;
  frexpf(amax, &ex);  // amax in [2^(ex-1), 2^ex)
  return min(max(14 - ex, -100), 100);
}
__device__ __forceinline__ float exp2i(int e) { return __int_as_float((127 + e) << 23); }  // e in [-126, 127]

// Row exponents of weight rows [0, m.rows), stored at rexp[row0 + r]: one
// warp per row dequantizes it (dequant_unit) and takes the largest magnitude.
__global__ void k_rowexp(DevMat m, uint32_t row0, int8_t* __restrict__ rexp) {
  const uint32_t row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (row >= m.rows) return;  // warp-uniform
  float amax = 0.f;
  for (uint32_t u = lane; u < m.cols / 64; u += 32) {
    float v[64];
    dequant_unit(m.dtype, m.ptr, m.rows, row, m.cols, u, v);
#pragma unroll
    for (int i = 0; i < 64; i++) amax = fmaxf(amax, fabsf(v[i]));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  if (lane == 0) rexp[row0 + row] = (int8_t)pow2_exp(amax);
}

__device__ __forceinline__ void split16(float v, __half* hi, __half* lo) {
  const __half h = __float2half_rn(v);
  *hi = h;
  *lo = __float2half_rn(__fmul_rn(__fsub_rn(v, __half2float(h)), QG_LO));
}

__device__ __forceinline__ uint32_t half2_bits(__half a, __half b) {
  return (uint32_t)__half_as_ushort(a) | ((uint32_t)__half_as_ushort(b) << 16);
}

// W (chunk-planar) rows -> hi/lo panels at rows row0.. of a panel matrix of
// K = m.cols columns.  One thread per (row, 64-column unit), rows fastest:
// the 8 elements of a core-matrix row are one 16-byte store, and a warp's
// 32 rows of one core-matrix column are 512 contiguous bytes.
__global__ void k_wpanels(DevMat m, uint32_t row0, const int8_t* __restrict__ rexp, __half* __restrict__ hi,
                          __half* __restrict__ lo) {
  const uint32_t U = m.cols / 64;
  const uint64_t idx = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (uint64_t)m.rows * U) return;
  const uint32_t u = (uint32_t)(idx / m.rows), r = (uint32_t)(idx % m.rows);
  float v[64];
  dequant_unit(m.dtype, m.ptr, m.rows, r, m.cols, u, v);
  const uint32_t R = row0 + r;
  const float sc = exp2i(rexp[R]);
#pragma unroll
  for (int i = 0; i < 64; i++) v[i] = __fmul_rn(v[i], sc);
  const uint64_t pbase = ((uint64_t)(R / QG_M) * U + u) * (QG_M * QG_KB);
#pragma unroll
  for (uint32_t kc = 0; kc < 8; kc++) {
    uint32_t h[4], l[4];
#pragma unroll
    for (uint32_t i = 0; i < 4; i++) {
      __half h0, l0, h1, l1;
      split16(v[8 * kc + 2 * i], &h0, &l0);
      split16(v[8 * kc + 2 * i + 1], &h1, &l1);
      h[i] = half2_bits(h0, h1);
      l[i] = half2_bits(l0, l1);
    }
    const uint64_t e = pbase + panel_elem(QG_M, R % QG_M, 8 * kc);
    *reinterpret_cast<uint4*>(hi + e) = make_uint4(h[0], h[1], h[2], h[3]);
    *reinterpret_cast<uint4*>(lo + e) = make_uint4(l[0], l[1], l[2], l[3]);
  }
}

// X [T, K] f32 (row stride ld) -> hi/lo token panels (P = QG_N), optionally
// RMS-normalised per row with weight w (src/tensor.rs:164-186).  One block
// per 8 tokens (the 8 rows of a core matrix): warp i reduces token i's sum of
// squares, then each thread converts 8 columns of one token into one 16-byte
// store per panel, the block's 8 tokens of a column group being 128
// contiguous bytes.  Tokens T.. up to the panel padding are never written
// (zeroed once at allocation).
constexpr uint32_t XP_TOK = 8;
__global__ void __launch_bounds__(256) k_xpanels(const float* __restrict__ x, uint32_t ld, uint32_t T, uint32_t K,
                                                 const float* __restrict__ w, float eps, __half* __restrict__ hi,
                                                 __half* __restrict__ lo, int8_t* __restrict__ texp) {
  const uint32_t tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, tb0 = blockIdx.x * XP_TOK;
  __shared__ float inv_s[XP_TOK], sc_s[XP_TOK];
  {
    // warp i: token tb0 + i's sum of squares (RMSNorm) and largest |x * w|
    const uint32_t t = tb0 + warp;
    float ss = 0.f, amax = 0.f;
    if (t < T) {
      const float* row = x + (uint64_t)t * ld;
      for (uint32_t k = lane; k < K; k += 32) {
        const float v = row[k];
        ss = fmaf(v, v, ss);
        amax = fmaxf(amax, fabsf(w ? v * w[k] : v));
      }
    }
    for (int o = 16; o > 0; o >>= 1) {
      ss += __shfl_xor_sync(0xffffffffu, ss, o);
      amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    }
    if (lane == 0) {
      const float inv = w ? __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)K), eps))) : 1.0f;
      // the normalised values are (x * inv) * w: at most inv * amax up to rounding
      const int e = pow2_exp(inv * amax * 1.0001f);
      inv_s[warp] = inv;
      sc_s[warp] = exp2i(e);
      if (t < T) texp[t] = (int8_t)e;
    }
    __syncthreads();
  }
  const uint32_t U = K / 64, nk8 = K / 8;
  for (uint32_t idx = tid; idx < nk8 * XP_TOK; idx += blockDim.x) {
    const uint32_t i = idx % XP_TOK, k0 = (idx / XP_TOK) * 8, t = tb0 + i;
    if (t >= T) continue;
    const float4* src = reinterpret_cast<const float4*>(x + (uint64_t)t * ld + k0);
    const float4 a = src[0], b = src[1];
    float v[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
    if (w) {
      const float inv = inv_s[i];
#pragma unroll
      for (int j = 0; j < 8; j++) v[j] = __fmul_rn(__fmul_rn(v[j], inv), w[k0 + j]);
    }
    const float sc = sc_s[i];
#pragma unroll
    for (int j = 0; j < 8; j++) v[j] = __fmul_rn(v[j], sc);
    uint32_t h[4], l[4];
#pragma unroll
    for (int j = 0; j < 4; j++) {
      __half h0, l0, h1, l1;
      split16(v[2 * j], &h0, &l0);
      split16(v[2 * j + 1], &h1, &l1);
      h[j] = half2_bits(h0, h1);
      l[j] = half2_bits(l0, l1);
    }
    const uint64_t panel = (uint64_t)(t / QG_N) * U + k0 / 64;
    const uint64_t e = panel * (QG_N * QG_KB) + panel_elem(QG_N, t % QG_N, k0 % 64);
    *reinterpret_cast<uint4*>(hi + e) = make_uint4(h[0], h[1], h[2], h[3]);
    *reinterpret_cast<uint4*>(lo + e) = make_uint4(l[0], l[1], l[2], l[3]);
  }
}

// ---- tcgen05 helpers ----------------------------------------------------------
__device__ __forceinline__ uint64_t umma_desc(const void* smem_ptr, uint32_t lbo, uint32_t sbo) {
  const uint32_t a = smem_u32(smem_ptr);
  uint64_t d = 0;
  d |= (uint64_t)((a >> 4) & 0x3FFF);
  d |= (uint64_t)((lbo >> 4) & 0x3FFF) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFF) << 32;
  d |= (uint64_t)1 << 46;  // descriptor version (Blackwell)
  // base offset 0, leading-byte-offset mode 0, layout type 0 (no swizzle)
  return d;
}
// kind::f16, A = B = f16 (K-major), D = f32, M = 128, N = QG_N
constexpr uint32_t QG_IDESC = (1u << 4) | ((QG_N >> 3) << 17) | ((QG_M >> 4) << 24);

__device__ __forceinline__ void umma_f16(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %5, %5, %5}, p;\n}\n" ::"r"(tmem_d),
      "l"(a), "l"(b), "r"(QG_IDESC), "r"(accumulate), "r"(0u)
      : "memory");
}
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, float* v) {
  uint32_t r[8];
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
               : "r"(taddr)
               : "memory");
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 8; i++) v[i] = __uint_as_float(r[i]);
}

struct QgParams {
  const __half* ahi;  // weight panels [Np/128][K/64]
  const __half* alo;
  const __half* bhi;  // token panels [Tp/256][K/64]
  const __half* blo;
  uint32_t K, N, T;   // true weight rows N and tokens T
  int epi;
  float* out;         // STORE / RESID: out[t * ld + r]; SWIGLU: out[t * ld + r / 2]
  uint32_t ld;
  const float* bias;  // STORE: + bias[r]
  uint32_t* err;      // set nonzero if a bounded wait ran out
  const int8_t* rexp;  // power-of-two exponents of the weight rows [Np] and
  const int8_t* texp;  //   of the token rows [T] applied before the fp16 split
};

// Y^T tile [128 weight rows x 256 tokens] of one CTA.  Warp 0 lane 0 copies
// panels into a two-stage ring, warp 1 lane 0 issues the MMAs, warp 2 owns
// the tensor memory (512 columns: two f32 accumulators of 256 columns), all
// four warps read the accumulators back (warp w: rows 32w..32w+31).
__global__ void __launch_bounds__(128, 1) k_qgemm(const __grid_constant__ QgParams p) {
  extern __shared__ __align__(1024) uint8_t qsm[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(qsm) + 1023) & ~uintptr_t(1023));
  __shared__ __align__(8) uint64_t full[QG_STAGES], empty[QG_STAGES], done;
  __shared__ uint32_t tmem_base;
  __shared__ volatile uint32_t fail;
  const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // token tiles fastest: the CTAs that share a weight panel run together and
  // read it from DRAM once between them
  const uint32_t rb = blockIdx.y, tb = blockIdx.x, KB = p.K / QG_KB;
  if (threadIdx.x == 0) {
    for (uint32_t s = 0; s < QG_STAGES; s++) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(&done, 1);
    fail = 0;
    fence_barrier_init();
  }
  if (warp == 2) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;" ::"r"(smem_u32(&tmem_base))
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tm = tmem_base;

  if (warp == 0 && lane == 0) {
    // ---- producer ----
    const uint8_t* ah = reinterpret_cast<const uint8_t*>(p.ahi) + (uint64_t)rb * KB * QG_APANEL;
    const uint8_t* al = reinterpret_cast<const uint8_t*>(p.alo) + (uint64_t)rb * KB * QG_APANEL;
    const uint8_t* bh = reinterpret_cast<const uint8_t*>(p.bhi) + (uint64_t)tb * KB * QG_BPANEL;
    const uint8_t* bl = reinterpret_cast<const uint8_t*>(p.blo) + (uint64_t)tb * KB * QG_BPANEL;
    for (uint32_t kb = 0; kb < KB; kb++) {
      const uint32_t s = kb % QG_STAGES;
      if (kb >= QG_STAGES && !mbar_wait(&empty[s], ((kb / QG_STAGES) - 1) & 1)) {
        fail = 1;
        break;
      }
      uint8_t* st = sm + s * QG_STAGE;
      mbar_expect_tx(&full[s], QG_STAGE);
      bulk_g2s(st, ah + (uint64_t)kb * QG_APANEL, QG_APANEL, &full[s], 0ull);
      bulk_g2s(st + QG_APANEL, al + (uint64_t)kb * QG_APANEL, QG_APANEL, &full[s], 0ull);
      bulk_g2s(st + 2 * QG_APANEL, bh + (uint64_t)kb * QG_BPANEL, QG_BPANEL, &full[s], 0ull);
      bulk_g2s(st + 2 * QG_APANEL + QG_BPANEL, bl + (uint64_t)kb * QG_BPANEL, QG_BPANEL, &full[s], 0ull);
    }
  } else if (warp == 1 && lane == 0) {
    // ---- MMA issuer ----
    const uint32_t acc1 = tm, acc2 = tm + QG_N;
    bool ok = true;
    for (uint32_t kb = 0; kb < KB && ok; kb++) {
      const uint32_t s = kb % QG_STAGES;
      if (!mbar_wait(&full[s], (kb / QG_STAGES) & 1)) {
        fail = 1;
        ok = false;
        break;
      }
      tc_fence_after();
      const uint8_t* st = sm + s * QG_STAGE;
#pragma unroll
      for (uint32_t k = 0; k < QG_KB / 16; k++) {
        const uint64_t a_h = umma_desc(st + k * 2 * (QG_M / 8) * 128, (QG_M / 8) * 128, 128);
        const uint64_t a_l = umma_desc(st + QG_APANEL + k * 2 * (QG_M / 8) * 128, (QG_M / 8) * 128, 128);
        const uint64_t b_h = umma_desc(st + 2 * QG_APANEL + k * 2 * (QG_N / 8) * 128, (QG_N / 8) * 128, 128);
        const uint64_t b_l =
            umma_desc(st + 2 * QG_APANEL + QG_BPANEL + k * 2 * (QG_N / 8) * 128, (QG_N / 8) * 128, 128);
        const uint32_t accum = (kb > 0 || k > 0) ? 1u : 0u;
        umma_f16(acc1, a_h, b_h, accum);
        umma_f16(acc2, a_h, b_l, accum);
        umma_f16(acc2, a_l, b_h, 1u);
      }
      umma_commit(&empty[s]);  // the stage is free once these MMAs have read it
    }
    if (ok) umma_commit(&done);
  }
  __syncwarp();
  // ---- epilogue: accumulators -> outputs ----
  bool ok = mbar_wait(&done, 0) && fail == 0;
  if (!ok && threadIdx.x == 0) atomicExch(p.err, 1u);
  tc_fence_after();
  const uint32_t r = rb * QG_M + warp * 32 + lane;
  const float rsc = exp2i(-(int)p.rexp[r]);  // rows past N are zero-padded: their exponent is 0
  if (ok) {
    const uint32_t lanebase = (warp * 32) << 16;
    for (uint32_t c = 0; c < QG_N; c += 8) {
      float a1[8], a2[8];
      tmem_ld8(tm + lanebase + c, a1);
      tmem_ld8(tm + lanebase + QG_N + c, a2);
#pragma unroll
      for (int j = 0; j < 8; j++) {
        const uint32_t t = tb * QG_N + c + j;
        // undo the row and token scaling (exact powers of two)
        const float y = __fmul_rn(__fmul_rn(__fadd_rn(a1[j], __fmul_rn(a2[j], 1.0f / QG_LO)), rsc),
                                  exp2i(-(int)p.texp[min(t, p.T - 1)]));
        if (p.epi == QE_SWIGLU) {
          // rows interleave gate (even) / up (odd): h = silu(g) * u (src/tensor.rs:213-227)
          const float other = __shfl_xor_sync(0xffffffffu, y, 1);
          if ((lane & 1) == 0 && t < p.T && r < p.N) {
            const float g = y, u = other;
            p.out[(uint64_t)t * p.ld + r / 2] = __fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, expf(-g))), u);
          }
        } else if (t < p.T && r < p.N) {
          float* o = p.out + (uint64_t)t * p.ld + r;
          if (p.epi == QE_STORE)
            *o = p.bias ? __fadd_rn(y, p.bias[r]) : y;
          else
            *o = __fadd_rn(*o, y);
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 2) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 512;" ::"r"(tm) : "memory");
}

// KV append for a prefill chunk: rotated k and v of tokens t < T at
// positions pos0 + t (src/model.rs:193-217, 340-352).  Grid (T, n_kv).
template <typename KT>
__global__ void k_kv_append(const float* __restrict__ qkv, uint32_t ldq, uint32_t nh, uint32_t nkv, uint32_t hd,
                            const float2* __restrict__ cs, KT* __restrict__ kc, KT* __restrict__ vc,
                            uint32_t max_ctx, uint32_t pos0) {
  const uint32_t t = blockIdx.x, h = blockIdx.y, half = hd / 2, pos = pos0 + t;
  const float* k = qkv + (uint64_t)t * ldq + (uint64_t)nh * hd + (uint64_t)h * hd;
  const float* v = qkv + (uint64_t)t * ldq + (uint64_t)(nh + nkv) * hd + (uint64_t)h * hd;
  KT* kd = kc + ((uint64_t)h * max_ctx + pos) * hd;
  KT* vd = vc + ((uint64_t)h * max_ctx + pos) * hd;
  const float2* c = cs + (uint64_t)pos * half;
  for (uint32_t i = threadIdx.x; i < half; i += blockDim.x) {
    const float a = k[i], b = k[i + half];
    const float2 cc = c[i];
    kv_st(kd + i, __fsub_rn(__fmul_rn(a, cc.x), __fmul_rn(b, cc.y)));
    kv_st(kd + i + half, __fadd_rn(__fmul_rn(a, cc.y), __fmul_rn(b, cc.x)));
    kv_st(vd + i, v[i]);
    kv_st(vd + i + half, v[i + half]);
  }
}

// Causal attention of a prefill chunk (src/model.rs:371-438) on the CUDA
// cores in f32.  One CTA per (block of QB = 64 / G consecutive tokens, KV
// head): its query rows r = i * G + h (token t0 + i, query head kvh * G + h)
// stream the cache positions [0, pos0 + t0 + QB) in tiles of 64 through
// shared memory once per block, each row masked to its own causal limit.
// Scores: each thread holds a 4-row x 8-position tile and walks the 128-bit
// columns of q and k starting at its own rotation, so the eight rows a
// quarter-warp reads fall in distinct banks.  Online softmax per row over the
// eight threads of a row group (shuffles), probabilities through shared
// memory, then P V with an 8-row x (HD / 16)-dimension tile per thread.
constexpr uint32_t AP_ROWS = 64;     // query rows per CTA
constexpr uint32_t AP_POS = 64;      // cache positions per tile
constexpr uint32_t AP_PST = AP_POS + 4;  // row stride of the probability tile (floats)
constexpr uint32_t AP_THREADS = 128;

// Shared memory of k_attn_prefill: q rows, one K and one V tile, and the
// probability tile, which reuses the K tile's space when it fits (the next K
// tile is requested only once P V is done).
template <int HD, typename KT>
__host__ __device__ constexpr bool ap_palias() {
  return (size_t)AP_POS * HD * sizeof(KT) >= (size_t)AP_ROWS * AP_PST * 4;
}
template <int HD, typename KT>
__host__ __device__ constexpr size_t ap_smem() {
  return (size_t)AP_ROWS * HD * 4 + 2 * (size_t)AP_POS * HD * sizeof(KT) +
         (ap_palias<HD, KT>() ? 0 : (size_t)AP_ROWS * AP_PST * 4) + 2 * AP_ROWS * 4;
}

template <int HD, typename KT>
__global__ void __launch_bounds__(AP_THREADS) k_attn_prefill(const float* __restrict__ qkv, uint32_t ldq,
                                                              const float2* __restrict__ cs,
                                                              const KT* __restrict__ kc,
                                                              const KT* __restrict__ vc, float* __restrict__ ctx,
                                                              uint32_t ldc, uint32_t nh, uint32_t nkv,
                                                              uint32_t max_ctx, uint32_t pos0, uint32_t T,
                                                              uint32_t* err) {
  constexpr uint32_t C4 = HD / 4;       // 4-element columns of a row
  constexpr uint32_t EB = sizeof(KT);
  constexpr uint32_t NC = HD / 64;      // P V: 4-element columns per thread (dg, dg + 16)
  extern __shared__ __align__(128) uint8_t smem[];
  float* qsm = reinterpret_cast<float*>(smem);                         // [AP_ROWS][HD]
  KT* ksm = reinterpret_cast<KT*>(smem + (size_t)AP_ROWS * HD * 4);    // [AP_POS][HD]
  KT* vsm = ksm + AP_POS * HD;                                         // [AP_POS][HD]
  uint8_t* after = reinterpret_cast<uint8_t*>(vsm + AP_POS * HD);
  float* psm = ap_palias<HD, KT>() ? reinterpret_cast<float*>(ksm) : reinterpret_cast<float*>(after);
  float* alpha_s = reinterpret_cast<float*>(after + (ap_palias<HD, KT>() ? 0 : (size_t)AP_ROWS * AP_PST * 4));
  float* lfin = alpha_s + AP_ROWS;
  __shared__ __align__(8) uint64_t kbar, vbar;

  const uint32_t G = nh / nkv, QB = AP_ROWS / G, kvh = blockIdx.y;
  const uint32_t blk = gridDim.x - 1 - blockIdx.x;  // longest blocks first
  const uint32_t t0 = blk * QB, tq = min(QB, T - t0), R = tq * G;
  const uint32_t nmax = pos0 + t0 + tq, ntiles = (nmax + AP_POS - 1) / AP_POS;
  const uint32_t tid = threadIdx.x;
  const KT* kvk = kc + (uint64_t)kvh * max_ctx * HD;
  const KT* kvv = vc + (uint64_t)kvh * max_ctx * HD;
  auto issue = [&](uint64_t* bar, KT* dst, const KT* src, uint32_t j) {
    const uint32_t a = j * AP_POS, rows = min(nmax, a + AP_POS) - a;
    mbar_expect_tx(bar, rows * HD * EB);
    bulk_g2s(dst, src + (uint64_t)a * HD, rows * HD * EB, bar, 0ull);
  };
  if (tid == 0) {
    mbar_init(&kbar, 1);
    mbar_init(&vbar, 1);
    fence_barrier_init();
  }
  __syncthreads();
  if (tid == 0) {
    issue(&kbar, ksm, kvk, 0);
    issue(&vbar, vsm, kvv, 0);
  }
  // q rows with RoPE at each token's position (src/model.rs:193-217); rows
  // past R are zero and never written out
  constexpr uint32_t half = HD / 2;
  for (uint32_t idx = tid; idx < AP_ROWS * half; idx += AP_THREADS) {
    const uint32_t r = idx / half, i = idx % half;
    float o0 = 0.f, o1 = 0.f;
    if (r < R) {
      const uint32_t t = t0 + r / G, h = r % G;
      const float* x = qkv + (uint64_t)t * ldq + (uint64_t)(kvh * G + h) * HD;
      const float xa = x[i], xb = x[i + half];
      const float2 c = cs[(uint64_t)(pos0 + t) * half + i];
      o0 = __fsub_rn(__fmul_rn(xa, c.x), __fmul_rn(xb, c.y));
      o1 = __fadd_rn(__fmul_rn(xa, c.y), __fmul_rn(xb, c.x));
    }
    qsm[r * HD + i] = o0;
    qsm[r * HD + i + half] = o1;
  }
  __syncthreads();

  const uint32_t rg = tid >> 3, pg = tid & 7;   // scores: rows rg*4 + i, positions pg*8 + jj
  const uint32_t rp = tid >> 4, dg = tid & 15;  // P V: rows rp + 8k, columns dg (+ 16)
  const float scale = __fdiv_rn(1.0f, __fsqrt_rn((float)HD));
  float m[4], l[4];
  uint32_t lim[4];  // last position row rg*4 + i may attend to
#pragma unroll
  for (int i = 0; i < 4; i++) {
    m[i] = -INFINITY;
    l[i] = 0.f;
    lim[i] = pos0 + t0 + min((rg * 4 + i) / G, tq - 1);
  }
  float4 o[8][NC];
#pragma unroll
  for (int k = 0; k < 8; k++)
#pragma unroll
    for (int c = 0; c < (int)NC; c++) o[k][c] = make_float4(0.f, 0.f, 0.f, 0.f);

  bool ok = true;
  for (uint32_t j = 0; j < ntiles; j++) {
    const uint32_t a = j * AP_POS, tn = min(nmax, a + AP_POS) - a;
    if (!mbar_wait(&kbar, j & 1)) {
      ok = false;
      break;
    }
    float sc[4][8];
#pragma unroll
    for (int i = 0; i < 4; i++)
#pragma unroll
      for (int jj = 0; jj < 8; jj++) sc[i][jj] = 0.f;
#pragma unroll 2
    for (uint32_t c = 0; c < C4; c++) {
      const uint32_t cc = (c + pg) & (C4 - 1);
      float4 q4[4], k4[8];
#pragma unroll
      for (int i = 0; i < 4; i++) q4[i] = reinterpret_cast<const float4*>(qsm + (rg * 4 + i) * HD)[cc];
#pragma unroll
      for (int jj = 0; jj < 8; jj++) k4[jj] = kv_ld4(ksm + (pg * 8 + jj) * HD, cc);
#pragma unroll
      for (int i = 0; i < 4; i++)
#pragma unroll
        for (int jj = 0; jj < 8; jj++) {
          sc[i][jj] = fmaf(q4[i].x, k4[jj].x, sc[i][jj]);
          sc[i][jj] = fmaf(q4[i].y, k4[jj].y, sc[i][jj]);
          sc[i][jj] = fmaf(q4[i].z, k4[jj].z, sc[i][jj]);
          sc[i][jj] = fmaf(q4[i].w, k4[jj].w, sc[i][jj]);
        }
    }
    __syncthreads();  // K tile read by every thread (its space may now hold P)
    // causal mask, scale and the online softmax of each row
#pragma unroll
    for (int i = 0; i < 4; i++) {
      float mt = -INFINITY;
#pragma unroll
      for (int jj = 0; jj < 8; jj++) {
        const uint32_t pp = pg * 8 + jj;
        sc[i][jj] = (pp < tn && a + pp <= lim[i]) ? __fmul_rn(sc[i][jj], scale) : -INFINITY;
        mt = fmaxf(mt, sc[i][jj]);
      }
      mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 1));
      mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 2));
      mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 4));
      const float mn = fmaxf(m[i], mt);
      const float al = expf(m[i] - mn);
      float ps = 0.f;
#pragma unroll
      for (int jj = 0; jj < 8; jj++) {
        sc[i][jj] = expf(sc[i][jj] - mn);
        ps += sc[i][jj];
      }
      ps += __shfl_xor_sync(0xffffffffu, ps, 1);
      ps += __shfl_xor_sync(0xffffffffu, ps, 2);
      ps += __shfl_xor_sync(0xffffffffu, ps, 4);
      l[i] = fmaf(l[i], al, ps);
      m[i] = mn;
      float4* pr = reinterpret_cast<float4*>(psm + (rg * 4 + i) * AP_PST + pg * 8);
      pr[0] = make_float4(sc[i][0], sc[i][1], sc[i][2], sc[i][3]);
      pr[1] = make_float4(sc[i][4], sc[i][5], sc[i][6], sc[i][7]);
      if (pg == 0) alpha_s[rg * 4 + i] = al;
    }
    __syncthreads();  // P and the rescale factors are complete
    if (!mbar_wait(&vbar, j & 1)) {
      ok = false;
      break;
    }
#pragma unroll
    for (int k = 0; k < 8; k++) {
      const float al = alpha_s[rp + 8 * k];
#pragma unroll
      for (int c = 0; c < (int)NC; c++) {
        o[k][c].x *= al;
        o[k][c].y *= al;
        o[k][c].z *= al;
        o[k][c].w *= al;
      }
    }
    for (uint32_t pp = 0; pp < tn; pp++) {
      float4 v4[NC];
#pragma unroll
      for (int c = 0; c < (int)NC; c++) v4[c] = kv_ld4(vsm + pp * HD, dg + 16 * c);
#pragma unroll
      for (int k = 0; k < 8; k++) {
        const float pv = psm[(rp + 8 * k) * AP_PST + pp];
#pragma unroll
        for (int c = 0; c < (int)NC; c++) {
          o[k][c].x = fmaf(pv, v4[c].x, o[k][c].x);
          o[k][c].y = fmaf(pv, v4[c].y, o[k][c].y);
          o[k][c].z = fmaf(pv, v4[c].z, o[k][c].z);
          o[k][c].w = fmaf(pv, v4[c].w, o[k][c].w);
        }
      }
    }
    __syncthreads();  // P and the V tile consumed
    if (tid == 0 && j + 1 < ntiles) {
      // the bulk copies overwrite what this CTA's threads wrote (P) and read
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      issue(&kbar, ksm, kvk, j + 1);
      issue(&vbar, vsm, kvv, j + 1);
    }
  }
  if (!ok) {
    if (tid == 0) atomicExch(err, 2u);
    return;
  }
  if (pg == 0)
#pragma unroll
    for (int i = 0; i < 4; i++) lfin[rg * 4 + i] = l[i];
  __syncthreads();
#pragma unroll
  for (int k = 0; k < 8; k++) {
    const uint32_t r = rp + 8 * k;
    if (r < R) {
      const float lr = lfin[r];
      float4* out = reinterpret_cast<float4*>(ctx + (uint64_t)(t0 + r / G) * ldc + (uint64_t)(kvh * G + r % G) * HD);
#pragma unroll
      for (int c = 0; c < (int)NC; c++)
        out[dg + 16 * c] = make_float4(__fdiv_rn(o[k][c].x, lr), __fdiv_rn(o[k][c].y, lr), __fdiv_rn(o[k][c].z, lr),
                                       __fdiv_rn(o[k][c].w, lr));
    }
  }
}

// x[t] += embedding rows: x[t] = dequant row(tokens[t]) (src/model.rs:482-506).
__global__ void k_embed_rows(DevMat emb, const uint32_t* __restrict__ tokens, float* __restrict__ x, uint32_t ld) {
  const uint32_t t = blockIdx.y, U = emb.cols / 64, u = blockIdx.x * blockDim.x + threadIdx.x;
  if (u >= U) return;
  const uint32_t tok = tokens[t];
  if (tok >= emb.rows) return;  // the host validates ids
  dequant_unit(emb.dtype, emb.ptr, emb.rows, tok, emb.cols, u, x + (uint64_t)t * ld + 64 * u);
}
