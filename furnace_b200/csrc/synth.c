// synth.c -- seeded synthetic GGUF tensor data (fills the data blob of a file
// whose header furnace_b200/synth.py has written).
//
// Values: a counter-based generator (splitmix64 of seed and element index)
// feeds an Irwin-Hall(4) approximation of a normal draw, so element i of a
// tensor depends only on (seed, i): output is independent of the thread
// count.  Quantizers are written from the block layouts the reference
// decodes (src/quant.rs:3-6, :44-52, :65-72, :111-113); they choose scales by
// plain min/max rules, which is all a synthetic weight file needs.

#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <string.h>

enum { T_F32 = 0, T_Q5_0 = 6, T_Q8_0 = 8, T_Q4_K = 12, T_Q6_K = 14 };

static inline uint64_t splitmix64(uint64_t x) {
  x += 0x9E3779B97F4A7C15ull;
  x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
  x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
  return x ^ (x >> 31);
}

// Approximately N(0, 1): sum of four 16-bit uniforms, standardised.
static inline float gauss(uint64_t seed, uint64_t i) {
  uint64_t r = splitmix64(seed ^ (i * 0xD1B54A32D192ED03ull));
  float s = (float)(r & 0xFFFF) + (float)((r >> 16) & 0xFFFF) + (float)((r >> 32) & 0xFFFF) + (float)(r >> 48);
  // mean 4 * 32767.5, variance 4 * (65536^2 - 1) / 12
  return (s - 131070.0f) * (1.0f / 37837.2f);
}

static uint16_t f32_to_f16(float f) {
  uint32_t x;
  memcpy(&x, &f, 4);
  uint32_t sign = (x >> 16) & 0x8000;
  int32_t e = (int32_t)((x >> 23) & 0xFF) - 127 + 15;
  uint32_t m = x & 0x7FFFFF;
  if (((x >> 23) & 0xFF) == 0xFF) return (uint16_t)(sign | 0x7C00 | (m ? 0x200 : 0));
  if (e >= 31) return (uint16_t)(sign | 0x7C00);
  if (e <= 0) {
    if (e < -10) return (uint16_t)sign;
    m |= 0x800000;
    uint32_t shift = (uint32_t)(14 - e);
    uint32_t h = m >> shift;
    uint32_t rem = m & ((1u << shift) - 1), half = 1u << (shift - 1);
    if (rem > half || (rem == half && (h & 1))) h++;
    return (uint16_t)(sign | h);
  }
  uint32_t h = ((uint32_t)e << 10) | (m >> 13);
  uint32_t rem = m & 0x1FFF;
  if (rem > 0x1000 || (rem == 0x1000 && (h & 1))) h++;
  return (uint16_t)(sign | h);
}

static float f16_to_f32(uint16_t h) {
  uint32_t sign = (uint32_t)(h >> 15) << 31, e = (h >> 10) & 0x1F, m = h & 0x3FF, bits;
  if (e == 0) {
    if (!m) bits = sign;
    else {
      int k = -1;
      do { m <<= 1; k++; } while (!(m & 0x400));
      bits = sign | ((uint32_t)(112 - k) << 23) | ((m & 0x3FF) << 13);
    }
  } else if (e == 31) bits = sign | 0x7F800000 | (m << 13);
  else bits = sign | ((e + 112) << 23) | (m << 13);
  float f;
  memcpy(&f, &bits, 4);
  return f;
}

static void put16(uint8_t* p, uint16_t v) { p[0] = (uint8_t)v; p[1] = (uint8_t)(v >> 8); }

static int iround(float x) { return (int)lrintf(x); }
static int clampi(int v, int lo, int hi) { return v < lo ? lo : v > hi ? hi : v; }

static void quant_q8_0(const float* x, uint8_t* b) {
  float amax = 0;
  for (int i = 0; i < 32; i++) amax = fmaxf(amax, fabsf(x[i]));
  uint16_t dh = f32_to_f16(amax / 127.0f);
  float d = f16_to_f32(dh), id = d != 0 ? 1.0f / d : 0.0f;
  put16(b, dh);
  for (int i = 0; i < 32; i++) b[2 + i] = (uint8_t)(int8_t)clampi(iround(x[i] * id), -127, 127);
}

static void quant_q5_0(const float* x, uint8_t* b) {
  float mx = 0, amax = 0;
  for (int i = 0; i < 32; i++)
    if (fabsf(x[i]) > amax) { amax = fabsf(x[i]); mx = x[i]; }
  uint16_t dh = f32_to_f16(mx / -16.0f);
  float d = f16_to_f32(dh), id = d != 0 ? 1.0f / d : 0.0f;
  put16(b, dh);
  uint32_t qh = 0;
  uint8_t* qs = b + 6;
  for (int j = 0; j < 16; j++) {
    int q0 = clampi(iround(x[j] * id) + 16, 0, 31), q1 = clampi(iround(x[j + 16] * id) + 16, 0, 31);
    qs[j] = (uint8_t)((q0 & 0xF) | ((q1 & 0xF) << 4));
    qh |= (uint32_t)(q0 >> 4) << j;
    qh |= (uint32_t)(q1 >> 4) << (j + 16);
  }
  memcpy(b + 2, &qh, 4);
}

static void quant_q4_k(const float* x, uint8_t* b) {
  float scale[8], mins[8], smax = 0, mmax = 0;
  for (int j = 0; j < 8; j++) {
    float lo = 0, hi = 0;
    for (int i = 0; i < 32; i++) {
      lo = fminf(lo, x[32 * j + i]);
      hi = fmaxf(hi, x[32 * j + i]);
    }
    scale[j] = (hi - lo) / 15.0f;
    mins[j] = -lo;
    smax = fmaxf(smax, scale[j]);
    mmax = fmaxf(mmax, mins[j]);
  }
  uint16_t dh = f32_to_f16(smax / 63.0f), mh = f32_to_f16(mmax / 63.0f);
  float d = f16_to_f32(dh), dmin = f16_to_f32(mh);
  int sc[8], m[8];
  for (int j = 0; j < 8; j++) {
    sc[j] = d > 0 ? clampi(iround(scale[j] / d), 0, 63) : 0;
    m[j] = dmin > 0 ? clampi(iround(mins[j] / dmin), 0, 63) : 0;
  }
  put16(b, dh);
  put16(b + 2, mh);
  uint8_t* s = b + 4;
  for (int j = 0; j < 4; j++) {
    s[j] = (uint8_t)((sc[j] & 63) | ((sc[j + 4] >> 4) << 6));
    s[j + 4] = (uint8_t)((m[j] & 63) | ((m[j + 4] >> 4) << 6));
    s[j + 8] = (uint8_t)((sc[j + 4] & 0xF) | ((m[j + 4] & 0xF) << 4));
  }
  uint8_t q[256];
  for (int j = 0; j < 8; j++) {
    float ds = d * (float)sc[j], dm = dmin * (float)m[j];
    for (int i = 0; i < 32; i++) q[32 * j + i] = (uint8_t)(ds > 0 ? clampi(iround((x[32 * j + i] + dm) / ds), 0, 15) : 0);
  }
  uint8_t* qs = b + 16;
  for (int j64 = 0; j64 < 4; j64++)
    for (int l = 0; l < 32; l++) qs[32 * j64 + l] = (uint8_t)(q[64 * j64 + l] | (q[64 * j64 + 32 + l] << 4));
}

static void quant_q6_k(const float* x, uint8_t* b) {
  float sub[16], amax = 0;
  for (int s = 0; s < 16; s++) {
    float mx = 0, am = 0;
    for (int i = 0; i < 16; i++)
      if (fabsf(x[16 * s + i]) > am) { am = fabsf(x[16 * s + i]); mx = x[16 * s + i]; }
    sub[s] = mx / -32.0f;
    amax = fmaxf(amax, fabsf(sub[s]));
  }
  uint16_t dh = f32_to_f16(amax / 127.0f);
  float d = f16_to_f32(dh);
  int sc[16];
  int q[256];
  for (int s = 0; s < 16; s++) {
    sc[s] = d > 0 ? clampi(iround(sub[s] / d), -127, 127) : 0;
    float ds = d * (float)sc[s];
    for (int i = 0; i < 16; i++) q[16 * s + i] = ds != 0 ? clampi(iround(x[16 * s + i] / ds), -32, 31) + 32 : 32;
  }
  memset(b, 0, 210);
  for (int half = 0; half < 2; half++) {
    uint8_t* ql = b + 64 * half;
    uint8_t* qh = b + 128 + 32 * half;
    const int* y = q + 128 * half;
    for (int l = 0; l < 32; l++) {
      int q1 = y[l], q2 = y[l + 32], q3 = y[l + 64], q4 = y[l + 96];
      ql[l] = (uint8_t)((q1 & 0xF) | ((q3 & 0xF) << 4));
      ql[l + 32] = (uint8_t)((q2 & 0xF) | ((q4 & 0xF) << 4));
      qh[l] = (uint8_t)((q1 >> 4) | ((q2 >> 4) << 2) | ((q3 >> 4) << 4) | ((q4 >> 4) << 6));
    }
    for (int k = 0; k < 8; k++) b[192 + 8 * half + k] = (uint8_t)(int8_t)sc[8 * half + k];
  }
  put16(b + 208, dh);
}

typedef struct {
  uint8_t* dst;
  uint32_t dtype;
  uint64_t rows, cols, r0, r1;
  float mean, std;
  uint64_t seed;
} Job;

static void* run(void* arg) {
  Job* j = (Job*)arg;
  float buf[256];
  uint64_t be = j->dtype == T_Q4_K || j->dtype == T_Q6_K ? 256 : j->dtype == T_F32 ? 1 : 32;
  uint64_t bb = j->dtype == T_Q8_0 ? 34 : j->dtype == T_Q5_0 ? 22 : j->dtype == T_Q4_K ? 144 : j->dtype == T_Q6_K ? 210 : 4;
  uint64_t row_bytes = j->cols / be * bb;
  for (uint64_t r = j->r0; r < j->r1; r++) {
    uint8_t* row = j->dst + r * row_bytes;
    for (uint64_t c0 = 0; c0 < j->cols; c0 += be) {
      for (uint64_t i = 0; i < be; i++) buf[i] = j->mean + j->std * gauss(j->seed, r * j->cols + c0 + i);
      uint8_t* blk = row + c0 / be * bb;
      switch (j->dtype) {
        case T_F32: memcpy(blk, buf, 4); break;
        case T_Q8_0: quant_q8_0(buf, blk); break;
        case T_Q5_0: quant_q5_0(buf, blk); break;
        case T_Q4_K: quant_q4_k(buf, blk); break;
        case T_Q6_K: quant_q6_k(buf, blk); break;
      }
    }
  }
  return 0;
}

// Fill `dst` with a [rows, cols] tensor of `dtype` drawn from N(mean, std).
// Returns 0, or 1 for an unsupported dtype / shape.
int fzs_fill(uint8_t* dst, uint32_t dtype, uint64_t rows, uint64_t cols, float mean, float std, uint64_t seed,
             int threads) {
  uint64_t be = dtype == T_Q4_K || dtype == T_Q6_K ? 256 : dtype == T_F32 ? 1 : 32;
  if (!(dtype == T_F32 || dtype == T_Q8_0 || dtype == T_Q5_0 || dtype == T_Q4_K || dtype == T_Q6_K)) return 1;
  if (cols % be) return 1;
  if (threads < 1) threads = 1;
  if ((uint64_t)threads > rows) threads = (int)(rows ? rows : 1);
  if (threads > 256) threads = 256;
  pthread_t th[256];
  Job jobs[256];
  for (int t = 0; t < threads; t++) {
    jobs[t] = (Job){dst, dtype, rows, cols, rows * (uint64_t)t / threads, rows * (uint64_t)(t + 1) / threads, mean, std, seed};
    if (t) pthread_create(&th[t], 0, run, &jobs[t]);
  }
  run(&jobs[0]);
  for (int t = 1; t < threads; t++) pthread_join(th[t], 0);
  return 0;
}

// Quantize caller-provided f32 values (used by tests to build exact cases).
int fzs_quantize(const float* x, uint64_t rows, uint64_t cols, uint32_t dtype, uint8_t* dst) {
  uint64_t be = dtype == T_Q4_K || dtype == T_Q6_K ? 256 : 32;
  uint64_t bb = dtype == T_Q8_0 ? 34 : dtype == T_Q5_0 ? 22 : dtype == T_Q4_K ? 144 : dtype == T_Q6_K ? 210 : 0;
  if (!bb || cols % be) return 1;
  for (uint64_t r = 0; r < rows; r++)
    for (uint64_t c = 0; c < cols; c += be) {
      uint8_t* blk = dst + (r * (cols / be) + c / be) * bb;
      const float* v = x + r * cols + c;
      switch (dtype) {
        case T_Q8_0: quant_q8_0(v, blk); break;
        case T_Q5_0: quant_q5_0(v, blk); break;
        case T_Q4_K: quant_q4_k(v, blk); break;
        case T_Q6_K: quant_q6_k(v, blk); break;
      }
    }
  return 0;
}
