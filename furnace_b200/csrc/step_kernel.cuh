// Persistent decode step: one launch per token.  Included by kernels.cu,
// whose device helpers (bulk copies, mbarriers, run records, unit_dot,
// StageIter) it uses.
//
// One CTA per SM runs every phase of a token in order:
//   embed -> per layer [qkv GEMV -> attention -> o_proj -> gate_up -> down]
//   -> lm_head (argmax) -> step bookkeeping,
// the same computation as Model::forward_cached for one token
// (src/model.rs:444-478, 579-600) followed by the greedy pick
// (src/generate.rs:69-77).
//
// Warp roles.  The last warp is the producer.  Weights do not depend on
// activations, so its lane 0 walks the weight stages of all of this CTA's
// GEMV phases (the same chunk-major stage order as k_gemv) and keeps a byte
// ring of shared memory filled with cp.async.bulk copies, plus an L2
// prefetch window ahead of the copies.  It never waits for a phase barrier:
// the weight stream runs on through attention and through the barriers.  The
// other 15 warps are consumers.  They pass a grid-wide barrier between
// phases, because each phase reads the whole output of the previous one.
//
// Cross-CTA data (x, qkv, partials, run records) is read with L2-only loads
// or bulk copies after the barrier's acquire.  Every wait is bounded: a wait
// that runs out records an error code in StepState and the CTA returns.

constexpr int SK_ND = 16;                    // ring stage descriptors
constexpr int SK_TP = 16;                    // attention positions per tile
constexpr int SK_NBUF = 3;                   // attention tiles in flight
constexpr uint32_t SK_CREC = 32 * 256;       // run records of one chunk (<= 32 units)
constexpr uint32_t SK_ACC = 8 * 1024;        // row accumulators of one GEMV phase
constexpr uint32_t SK_SMEM = 218 * 1024;     // dynamic shared memory per CTA (+ ~8 KB static)
constexpr long long SK_SPIN_NS = 2000000000ll;  // grid barrier wait limit (2 s)
#ifndef SK_PF_AHEAD_KB
#define SK_PF_AHEAD_KB 96
#endif
constexpr uint32_t SK_PF_AHEAD = SK_PF_AHEAD_KB * 1024;  // L2 prefetch window ahead of the ring copies

enum : uint32_t { PH_EMBED = 0, PH_GEMV = 1, PH_ATTN = 2 };
enum : uint32_t { ERR_BARRIER = 6, ERR_RING = 7, ERR_RECORDS = 8, ERR_KV = 9 };

// What one CTA does in one phase (host-built, [phase][CTA], 160 bytes): read
// by one bulk copy a phase ahead, so no phase starts with dependent global
// loads.  GEMV: rows [r0, r1) of the phase's matrix (`active` when non-empty),
// input x (+ norm_w) or run records, epilogue outputs.  Attention: item
// (kvh, split) when active.
struct PhaseRec {
  uint32_t kind, dt, epi, cols;
  uint32_t r0, r1, nch, active;
  const float* x;
  const float* norm_w;
  const XRun* in_runs;
  XRun* out_runs;
  float* out;
  const float* bias;
  float eps;
  uint32_t nh, nkv, hd;
  uint32_t S, kvh, split, pad_;
  const float* qkv;
  float* kc;
  float* vc;
  float* ctx;
  XRun* ctx_runs;
  uint64_t pad2_;
};
static_assert(sizeof(PhaseRec) == 160, "phase record");

// One weight stage of one CTA (host-built): a contiguous range of a chunk
// plane.  A CTA's list ends with bytes == 0.
struct StageRec {
  const uint8_t* src;
  uint32_t bytes;
  uint32_t pad_;
};
static_assert(sizeof(StageRec) == 16, "stage record");
constexpr int SL_BLK = 32;  // stage records per block copy
constexpr int SL_NB = 4;    // blocks resident

struct SkParams {
  const PhaseRec* rec;         // [nph][grid]
  const StageRec* stages;      // every CTA's list, each padded to whole blocks
  const uint32_t* stage_first; // [grid] index of the CTA's first record
  uint32_t nph;
  uint32_t ring_bytes, u_bytes;  // dynamic shared memory carve-up
  uint32_t pf_ahead;
  StepState* st;
  uint32_t* bar;       // grid barrier counter, zeroed before each launch
  uint32_t* attn_cnt;  // per-KV-head arrivals, zero between phases
  float* partials;
  const float2* rope_cs;
  uint32_t max_ctx;
  const uint8_t* emb;  // token_embd in the chunked layout
  uint32_t emb_dt, emb_rows, emb_cols;
  float* x;
  const uint32_t* forced;
  uint32_t* ids_out;
  int has_logits;
};

// ---- consumer-side state (identical in every consumer thread) ----------------
// Sequence counters instead of per-buffer arrays, so that the state stays in
// registers: use q of a rotating buffer set of N buffers sits in buffer q % N
// and completes phase q / N of that buffer's mbarrier.
struct SkCons {
  uint8_t* ring;
  uint64_t* full;
  uint64_t* empty;
  const uint32_t* off;
  uint8_t* crec;
  uint64_t* recbar;   // [2] chunk-record copies landed
  uint64_t* recfree;  // [2] every consumer warp has taken its records
  uint32_t s;         // weight stages consumed so far
  uint32_t q;         // chunk-record uses so far
};

__device__ __forceinline__ uint32_t ld_acquire(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Consumer-only grid barrier (the k-th of this launch).
__device__ bool sk_grid_sync(const SkParams& P, uint32_t k, uint32_t ctid, volatile uint32_t* fail) {
  named_sync(1, GV_NT);
  if (ctid == 0) {
    __threadfence();
    atomicAdd(P.bar, 1u);
    const uint32_t target = k * gridDim.x;
    if (ld_acquire(P.bar) < target) {
      const uint64_t t0 = gtimer();
      while (ld_acquire(P.bar) < target) {
        if (gtimer() - t0 > (uint64_t)SK_SPIN_NS) {
          atomicExch(&P.st->error, ERR_BARRIER);
          *fail = 1;
          break;
        }
      }
    }
  }
  named_sync(1, GV_NT);
  return *fail == 0;
}

// Copy the run records of chunk ci (units [cu0, cu0 + nu)) as record use q,
// once use q - 2 of the same buffer has been released.  One thread.
__device__ __forceinline__ bool sk_issue_records(SkCons& S, const XRun* in_runs, const ChunkInfo& ci, uint32_t q) {
  const uint32_t b = q & 1;
  if (q >= 2 && !mbar_wait(&S.recfree[b], ((q - 2) >> 1) & 1)) return false;
  // order the records' generic-proxy writes (other CTAs, before the barrier)
  // and this buffer's earlier generic use before the async-proxy copy
  asm volatile("fence.proxy.async;" ::: "memory");
  mbar_expect_tx(&S.recbar[b], ci.nu * 256);
  bulk_g2s(S.crec + b * SK_CREC, reinterpret_cast<const uint8_t*>(in_runs) + 256ull * ci.cu0, ci.nu * 256,
           &S.recbar[b], 0ull);
  return true;
}

template <uint32_t DT>
__device__ bool sk_consume(const PhaseRec& R, const ChunkInfo* chunks, SkCons& S, const XRun* rec_full, float* acc,
                           uint32_t ctid) {
  const uint32_t lane = ctid & 31, warp = ctid >> 5;
  const bool chunked = rec_full == nullptr;
  const uint32_t r0 = R.r0, r1 = R.r1, nch = R.nch;
  for (uint32_t c = 0; c < nch; c++) {
    const uint32_t nu = chunks[c].nu, tb = chunks[c].tb, cu0 = chunks[c].cu0;
    const uint32_t lu = min(lane, nu - 1);
    const float lane_on = lane < nu ? 1.f : 0.f;
    const XRun* rb = rec_full;
    const uint32_t q = S.q + c, b = q & 1;  // record use of chunk c
    if (chunked) {
      if (!mbar_wait(&S.recbar[b], (q >> 1) & 1)) return false;
      rb = reinterpret_cast<const XRun*>(S.crec + b * SK_CREC) - 4 * cu0;
    }
    XRun xr[4];
#pragma unroll
    for (uint32_t j = 0; j < 4; j++) xr[j] = load_run(rb, cu0 + lu, j);
    if (chunked) {
      __syncwarp();
      if (lane == 0) mbar_arrive(&S.recfree[b]);
      if (ctid == 0 && c + 2 < nch && !sk_issue_records(S, R.in_runs, chunks[c + 2], q + 2)) return false;
    }
    for (uint32_t ra = r0; ra < r1; ra += GV_ROWS) {
      const uint32_t d = S.s % SK_ND;
      if (!mbar_wait(&S.full[d], (S.s / SK_ND) & 1)) return false;
      const uint8_t* tile = S.ring + S.off[d];
      const uint32_t last = r1 - 1 - ra;
      float v[GV_RPW];
#pragma unroll
      for (int j = 0; j < GV_RPW; j++) {
        const uint32_t rr = min(warp + GV_CWARPS * j, last);
        v[j] = lane_on * unit_dot<DT>(tile + rr * tb, lu, nu, xr);
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1)
#pragma unroll
        for (int j = 0; j < GV_RPW; j++) v[j] += __shfl_xor_sync(0xffffffffu, v[j], o);
      if (lane == 0) {
#pragma unroll
        for (int j = 0; j < GV_RPW; j++) {
          const uint32_t row = ra + warp + GV_CWARPS * j;
          if (row < r1) acc[row - r0] += v[j];
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&S.empty[d]);
      S.s++;
    }
  }
  if (chunked) S.q += nch;
  return true;
}

// f32 input (RMS-normalised when norm_w is set) -> run records in shared
// memory; the same arithmetic as k_gemv's prologue, with L2-only loads.
__device__ void sk_prologue_f32(const PhaseRec& g, XRun* rec, float* red, uint32_t ctid) {
  const uint32_t lane = ctid & 31, warp = ctid >> 5;
  const uint32_t NX = runs_for_dev(g.cols), n4 = g.cols / 4;
  const float4* x4 = reinterpret_cast<const float4*>(g.x);
  const float4* w4 = reinterpret_cast<const float4*>(g.norm_w);
  const bool norm = g.norm_w != nullptr;
  float4 buf[16];
#pragma unroll
  for (int j = 0; j < 16; j++) {
    const bool isw = norm && j >= 8;
    const uint32_t i4 = ctid + GV_NT * (isw ? j - 8 : j);
    buf[j] = i4 < n4 ? (isw ? __ldg(w4 + i4) : __ldcg(x4 + i4)) : make_float4(0.f, 0.f, 0.f, 0.f);
  }
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
    inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, (float)g.cols), g.eps)));
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

// Epilogues (same as k_gemv's): bias store, residual add, SwiGLU with run
// records of h, logits with the argmax key.
__device__ void sk_epilogue(const PhaseRec& g, float* acc, unsigned long long* kred, StepState* st, uint32_t ctid) {
  const uint32_t lane = ctid & 31, warp = ctid >> 5;
  const uint32_t r0 = g.r0, nrows = g.r1 - g.r0;
  float* out = g.out;
  if (g.epi == EPI_STORE) {
    for (uint32_t i = ctid; i < nrows; i += GV_NT) {
      const uint32_t row = r0 + i;
      out[row] = g.bias ? __fadd_rn(acc[i], __ldg(g.bias + row)) : acc[i];
    }
  } else if (g.epi == EPI_RESID) {
    for (uint32_t i = ctid; i < nrows; i += GV_NT) {
      const uint32_t row = r0 + i;
      out[row] = __fadd_rn(__ldcg(out + row), acc[i]);
    }
  } else if (g.epi == EPI_SWIGLU) {
    float hv[4];
    const uint32_t np = nrows / 2;
    for (uint32_t k = 0; k < 4; k++) {
      const uint32_t j = ctid + k * GV_NT;
      hv[k] = 0.f;
      if (j < np) {
        const float gt = acc[2 * j], u = acc[2 * j + 1];
        hv[k] = __fmul_rn(__fdiv_rn(gt, __fadd_rn(1.0f, expf(-gt))), u);
        if (out) out[(r0 >> 1) + j] = hv[k];
      }
    }
    named_sync(1, GV_NT);
    for (uint32_t k = 0; k < 4; k++) {
      const uint32_t j = ctid + k * GV_NT;
      if (j < np) acc[j] = hv[k];
    }
    named_sync(1, GV_NT);
    values_to_runs(acc, np, nullptr, g.out_runs, r0 / 32, ctid, GV_NT);
  } else {
    unsigned long long best = 0;
    for (uint32_t i = ctid; i < nrows; i += GV_NT) {
      const uint32_t row = r0 + i;
      const float v = acc[i];
      out[row] = v;
      const unsigned long long k = argmax_key(v, row);
      best = k > best ? k : best;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
      best = other > best ? other : best;
    }
    if (lane == 0) kred[warp] = best;
    named_sync(1, GV_NT);
    if (ctid == 0) {
      unsigned long long m = 0;
      for (int w = 0; w < GV_CWARPS; w++) m = kred[w] > m ? kred[w] : m;
      atomicMax(&st->argmax_key, m);
    }
  }
}

// ---- attention phase -----------------------------------------------------------
// Item (kvh, split): positions [t0, t1) of KV head kvh for its G query heads
// (src/model.rs:371-438).  Tiles of SK_TP positions stream in through
// SK_NBUF bulk-copy buffers; every step of a tile uses all consumer warps:
//   scores  s[h][p] = q_h . k_p / sqrt(hd)   (4 threads per (h, p))
//   softmax online per head                    (one warp per head)
//   values  acc[h][d] = acc*alpha + sum_p p[h][p] v[p][d]  (thread per (h, d))
// The last split of a KV head to finish merges all splits' partials
// (k_attn_combine's math) and writes ctx and its run records.
constexpr int SK_AO = 3;  // outputs (h, d) per consumer thread: G * hd <= 3 * GV_NT
template <int HD>
__device__ bool sk_attention(const SkParams& P, const PhaseRec& D, float* tiles, float (*qs)[128], uint64_t* abar,
                             uint32_t& aseq, float* scr, uint32_t ctid) {
  const uint32_t lane = ctid & 31, warp = ctid >> 5;
  const uint32_t G = D.nh / D.nkv, S = D.S, half = HD / 2;
  if (!D.active) return true;
  const uint32_t kvh = D.kvh, split = D.split;
  const uint32_t max_ctx = P.max_ctx;
  const float* kvk = D.kc + (uint64_t)kvh * max_ctx * HD;
  const float* kvv = D.vc + (uint64_t)kvh * max_ctx * HD;
  const uint32_t pos = __ldcg(&P.st->pos);
  if (pos >= max_ctx) {
    if (ctid == 0) P.st->error = 2;
    return false;
  }
  const uint32_t total = pos + 1, per = (total + S - 1) / S;
  const uint32_t t0 = min(split * per, total), t1 = min(total, t0 + per), n = t1 - t0;
  const uint32_t ntiles = (n + SK_TP - 1) / SK_TP;
  const uint64_t pol = policy_evict_first();
  // tile j is tile use aseq + j of the rotating tile buffers
  auto issue = [&](uint32_t j) {
    const uint32_t b = (aseq + j) % SK_NBUF, a = t0 + j * SK_TP, e = min(min(t1, a + SK_TP), pos);
    const uint32_t rows = e > a ? e - a : 0;
    float* kt = tiles + (size_t)b * 2 * SK_TP * HD;
    asm volatile("fence.proxy.async;" ::: "memory");  // after generic writes to the tile buffers
    mbar_expect_tx(&abar[b], 2 * rows * HD * 4);
    if (rows) {
      bulk_g2s(kt, kvk + (uint64_t)a * HD, rows * HD * 4, &abar[b], pol);
      bulk_g2s(kt + SK_TP * HD, kvv + (uint64_t)a * HD, rows * HD * 4, &abar[b], pol);
    }
  };
  if (ctid == 0)
    for (uint32_t j = 0; j < ntiles && j < (uint32_t)SK_NBUF; j++) issue(j);
  // shared scratch: scores / probabilities [G][SK_TP], per-head alpha [G]
  float* sc = scr;
  float* alph = scr + AT_MAXG * SK_TP;
  // rotated queries (src/model.rs:193-217, half-split pairs)
  const float2* csp = P.rope_cs + (uint64_t)pos * half;
  for (uint32_t idx = ctid; idx < G * half; idx += GV_NT) {
    const uint32_t h = idx / half, i = idx % half;
    const float* x = D.qkv + (uint64_t)(kvh * G + h) * HD;
    const float a = __ldcg(x + i), bb = __ldcg(x + i + half);
    const float2 c = csp[i];
    qs[h][i] = __fsub_rn(__fmul_rn(a, c.x), __fmul_rn(bb, c.y));
    qs[h][i + half] = __fadd_rn(__fmul_rn(a, c.y), __fmul_rn(bb, c.x));
  }
  // the split holding `pos` appends this token's rotated k and its v
  const bool owns_pos = pos >= t0 && pos < t1;
  float kn[2] = {0.f, 0.f}, vn[2] = {0.f, 0.f};
  if (owns_pos && ctid < half) {
    const float* kx = D.qkv + (uint64_t)D.nh * HD + (uint64_t)kvh * HD;
    const float* vx = D.qkv + (uint64_t)(D.nh + D.nkv) * HD + (uint64_t)kvh * HD;
    const float2 c = csp[ctid];
    const float a = __ldcg(kx + ctid), bb = __ldcg(kx + ctid + half);
    kn[0] = __fsub_rn(__fmul_rn(a, c.x), __fmul_rn(bb, c.y));
    kn[1] = __fadd_rn(__fmul_rn(a, c.y), __fmul_rn(bb, c.x));
    vn[0] = __ldcg(vx + ctid);
    vn[1] = __ldcg(vx + ctid + half);
    float* kdst = D.kc + ((uint64_t)kvh * max_ctx + pos) * HD;
    float* vdst = D.vc + ((uint64_t)kvh * max_ctx + pos) * HD;
    kdst[ctid] = kn[0];
    kdst[ctid + half] = kn[1];
    vdst[ctid] = vn[0];
    vdst[ctid + half] = vn[1];
  }
  named_sync(1, GV_NT);
  const float scale = __fdiv_rn(1.0f, __fsqrt_rn((float)HD));
  float m = -INFINITY, l = 0.f;  // online softmax state of head `warp` (warps < G)
  float acc[SK_AO];
#pragma unroll
  for (int k = 0; k < SK_AO; k++) acc[k] = 0.f;
  for (uint32_t j = 0; j < ntiles; j++) {
    const uint32_t u = aseq + j, b = u % SK_NBUF, a = t0 + j * SK_TP, tn = min(t1, a + SK_TP) - a;
    float* kt = tiles + (size_t)b * 2 * SK_TP * HD;
    float* vt = kt + SK_TP * HD;
    if (!mbar_wait(&abar[b], (u / SK_NBUF) & 1)) {
      if (ctid == 0) P.st->error = ERR_KV;
      return false;
    }
    if (owns_pos && pos >= a && pos < a + SK_TP) {  // block-uniform
      if (ctid < half) {
        kt[(pos - a) * HD + ctid] = kn[0];
        kt[(pos - a) * HD + ctid + half] = kn[1];
        vt[(pos - a) * HD + ctid] = vn[0];
        vt[(pos - a) * HD + ctid + half] = vn[1];
      }
      named_sync(1, GV_NT);
    }
    // scores: thread w -> pair w / 4 = (h, p), quarter w % 4 of the dims; the
    // float4 order is rotated by p and the quarter so that the 8 lanes of a
    // quarter warp hit 8 bank groups
    for (uint32_t w0 = 0; w0 < G * SK_TP * 4; w0 += GV_NT) {
      const uint32_t w = w0 + ctid, pair = w >> 2, qq = w & 3, h = pair / SK_TP, p = pair % SK_TP;
      const bool on = pair < G * SK_TP && p < tn;
      float dsum = 0.f;
      if (on) {
        const float4* kr = reinterpret_cast<const float4*>(kt + (size_t)p * HD) + qq * (HD / 16);
        const float4* qr = reinterpret_cast<const float4*>(qs[h]) + qq * (HD / 16);
#pragma unroll
        for (uint32_t c = 0; c < HD / 16; c++) {
          const uint32_t cc = (c + p + 2 * qq) & (HD / 16 - 1);
          const float4 k4 = kr[cc], q4 = qr[cc];
          dsum = fmaf(q4.x, k4.x, dsum);
          dsum = fmaf(q4.y, k4.y, dsum);
          dsum = fmaf(q4.z, k4.z, dsum);
          dsum = fmaf(q4.w, k4.w, dsum);
        }
      }
      dsum += __shfl_xor_sync(0xffffffffu, dsum, 1);
      dsum += __shfl_xor_sync(0xffffffffu, dsum, 2);
      if (qq == 0 && pair < G * SK_TP) sc[pair] = on ? __fmul_rn(dsum, scale) : -INFINITY;
    }
    named_sync(1, GV_NT);
    // online softmax per head (lanes < SK_TP hold the tile's positions)
    if (warp < G) {
      const float sv = lane < SK_TP ? sc[warp * SK_TP + lane] : -INFINITY;
      float mt = sv;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, o));
      const float mn = fmaxf(m, mt);
      const float al = expf(m - mn);
      const float pr = (lane < SK_TP && lane < tn) ? expf(sv - mn) : 0.f;
      float ps = pr;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) ps += __shfl_xor_sync(0xffffffffu, ps, o);
      l = fmaf(l, al, ps);
      m = mn;
      if (lane < SK_TP) sc[warp * SK_TP + lane] = pr;
      if (lane == 0) alph[warp] = al;
    }
    named_sync(1, GV_NT);
    // values: output o = (h, d)
#pragma unroll
    for (int k = 0; k < SK_AO; k++) {
      const uint32_t o = ctid + k * GV_NT;
      if (o < G * HD) {
        const uint32_t h = o / HD, d = o % HD;
        float av = acc[k] * alph[h];
        const float* pr = sc + h * SK_TP;
        for (uint32_t p = 0; p < tn; p++) av = fmaf(pr[p], vt[(size_t)p * HD + d], av);
        acc[k] = av;
      }
    }
    named_sync(1, GV_NT);  // buffer b and the score scratch are free
    if (ctid == 0 && j + SK_NBUF < ntiles) issue(j + SK_NBUF);
  }
  aseq += ntiles;
  // partials: stats [nkv][G][S] of (max, sum), then acc [nkv][G][HD][Spad]
  const uint32_t Spad = (S + 3) & ~3u;
  float* pacc_base = P.partials + ((2 * (uint64_t)D.nkv * G * S + 3) & ~3ull);
  float2* stats = reinterpret_cast<float2*>(P.partials) + (uint64_t)kvh * G * S;
  if (warp < G && lane == 0) stats[warp * S + split] = make_float2(m, l);
#pragma unroll
  for (int k = 0; k < SK_AO; k++) {
    const uint32_t o = ctid + k * GV_NT;
    if (o < G * HD) pacc_base[((uint64_t)kvh * G * HD + o) * Spad + split] = acc[k];
  }
  // the last split of this KV head merges
  __shared__ uint32_t s_last;
  named_sync(1, GV_NT);
  if (ctid == 0) {
    __threadfence();
    const uint32_t prev = atomicAdd(&P.attn_cnt[kvh], 1u);
    s_last = prev == S - 1;
    if (s_last) {
      __threadfence();
      P.attn_cnt[kvh] = 0;  // every split has arrived: ready for the next layer
    }
  }
  named_sync(1, GV_NT);
  if (!s_last) return true;
  // merge: stage the splits' (m, l) in shared memory, turn them into weights
  // w_s = exp(m_s - M) and den = sum_s w_s l_s per head, then each output is
  // sum_s w_s acc_s / den over its consecutive split values
  float* ws = tiles;                       // [G][Spad]
  float* ls = tiles + AT_MAXG * 160;       // [G][Spad]
  float* den = tiles + 2 * AT_MAXG * 160;  // [G]
  for (uint32_t i = ctid; i < G * Spad; i += GV_NT) {
    const uint32_t hg = i / Spad, s2 = i % Spad;
    float2 v = make_float2(-INFINITY, 0.f);
    if (s2 < S) v = __ldcg(&stats[hg * S + s2]);
    ws[i] = v.x;
    ls[i] = v.y;
  }
  named_sync(1, GV_NT);
  if (warp < G) {
    float M = -INFINITY;
    for (uint32_t s2 = lane; s2 < S; s2 += 32) M = fmaxf(M, ws[warp * Spad + s2]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
    float dn = 0.f;
    for (uint32_t s2 = lane; s2 < Spad; s2 += 32) {
      const float ms = ws[warp * Spad + s2];
      const float w = ms == -INFINITY ? 0.f : expf(ms - M);
      ws[warp * Spad + s2] = w;
      dn = fmaf(w, ls[warp * Spad + s2], dn);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) dn += __shfl_xor_sync(0xffffffffu, dn, o);
    if (lane == 0) den[warp] = dn;
  }
  named_sync(1, GV_NT);
  float* sv = scr;  // ctx values of the group, for the run records
  for (uint32_t idx = ctid; idx < G * HD; idx += GV_NT) {
    const uint32_t hg = idx / HD;
    const float4* pa = reinterpret_cast<const float4*>(pacc_base + ((uint64_t)kvh * G * HD + idx) * Spad);
    const float* w = ws + hg * Spad;
    float num = 0.f;
    for (uint32_t k0 = 0; 4 * k0 < Spad; k0 += 8) {
      float4 av[8];
#pragma unroll
      for (int k = 0; k < 8; k++) av[k] = 4 * (k0 + k) < Spad ? __ldcg(pa + k0 + k) : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int k = 0; k < 8; k++) {
        const uint32_t s4 = 4 * (k0 + k);
        if (s4 >= Spad) break;
        num = fmaf(w[s4], av[k].x, num);
        num = fmaf(w[s4 + 1], av[k].y, num);
        num = fmaf(w[s4 + 2], av[k].z, num);
        num = fmaf(w[s4 + 3], av[k].w, num);
      }
    }
    const float v = __fdiv_rn(num, den[hg]);
    D.ctx[(uint64_t)kvh * G * HD + idx] = v;
    sv[idx] = v;
  }
  named_sync(1, GV_NT);
  values_to_runs(sv, G * HD, nullptr, D.ctx_runs, kvh * G * HD / 16, ctid, GV_NT);
  return true;
}

__global__ void __launch_bounds__(GV_THREADS, 1) k_step(const __grid_constant__ SkParams P) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ __align__(8) uint64_t full[SK_ND], empty[SK_ND], recbar[2], recfree[2], abar[SK_NBUF], slbar[SL_NB],
      prbar[2];
  __shared__ __align__(16) StageRec sl[SL_NB * SL_BLK];
  __shared__ __align__(16) PhaseRec prs[2];
  __shared__ uint32_t stage_off[SK_ND];
  __shared__ ChunkInfo chunks[GV_MAX_CH];
  __shared__ float red[GV_CWARPS];
  __shared__ unsigned long long kred[GV_CWARPS];
  __shared__ __align__(16) float qs[AT_MAXG][128];
  __shared__ volatile uint32_t s_fail;
  __shared__ volatile uint32_t s_issued;  // stages the producer has issued (trace)
  const uint32_t tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  uint8_t* ring = smem;
  uint8_t* ureg = smem + P.ring_bytes;  // run records of an f32 input, or attention tiles
  uint8_t* crec = ureg + P.u_bytes;     // two chunk-record buffers
  float* acc = reinterpret_cast<float*>(crec + 2 * SK_CREC);
  // phase record p of this CTA -> prs[p % 2] (phase p / 2 of prbar[p % 2])
  auto issue_rec = [&](uint32_t p) {
    asm volatile("fence.proxy.async;" ::: "memory");
    mbar_expect_tx(&prbar[p & 1], sizeof(PhaseRec));
    bulk_g2s(&prs[p & 1], P.rec + (uint64_t)p * gridDim.x + blockIdx.x, sizeof(PhaseRec), &prbar[p & 1], 0ull);
  };
  if (tid == 0) {
    for (int i = 0; i < SK_ND; i++) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], GV_CWARPS);
    }
    for (int i = 0; i < 2; i++) {
      mbar_init(&recbar[i], 1);
      mbar_init(&recfree[i], GV_CWARPS);
      mbar_init(&prbar[i], 1);
    }
    for (int i = 0; i < SK_NBUF; i++) mbar_init(&abar[i], 1);
    for (int i = 0; i < SL_NB; i++) mbar_init(&slbar[i], 1);
    s_fail = 0;
    s_issued = 0;
    fence_barrier_init();
  }
  __syncthreads();

  if (warp == GV_CWARPS) {
    // ---------------- producer: this CTA's weight stages, in order ------------
    if (lane != 0) return;
    const uint64_t pol = policy_evict_first();
    const StageRec* L = P.stages + P.stage_first[blockIdx.x];
    // stage records stream through SL_NB blocks of SL_BLK: block k sits in
    // buffer k % SL_NB and completes phase k / SL_NB of slbar[k % SL_NB]
    uint32_t loaded = 0, ready = 0;
    auto load_block = [&](uint32_t k) {
      mbar_expect_tx(&slbar[k % SL_NB], SL_BLK * sizeof(StageRec));
      bulk_g2s(&sl[(k % SL_NB) * SL_BLK], L + (uint64_t)k * SL_BLK, SL_BLK * sizeof(StageRec), &slbar[k % SL_NB],
               0ull);
    };
    auto entry = [&](uint32_t i, StageRec* e) -> bool {
      while (ready <= i / SL_BLK) {
        if (!mbar_wait(&slbar[ready % SL_NB], (ready / SL_NB) & 1)) return false;
        ready++;
      }
      *e = sl[(i / SL_BLK) % SL_NB * SL_BLK + i % SL_BLK];
      return true;
    };
    for (; loaded < (uint32_t)SL_NB; loaded++) load_block(loaded);
    const uint32_t RB = P.ring_bytes;
    uint64_t head = 0, tail = 0, copied = 0, prefetched = 0;
    uint64_t q_end[SK_ND];
    uint32_t s = 0, oldest = 0, j = 0;
    bool pf_done = false;
    for (;;) {
      StageRec e;
      if (!entry(s, &e)) break;
      if (e.bytes == 0) break;
      const uint32_t B = e.bytes;
      if (head % RB + B > RB) head += RB - head % RB;  // wrap: skip the ring's tail
      while (s - oldest >= (uint32_t)SK_ND || head + B - tail > RB) {
        if (oldest == s || !mbar_wait(&empty[oldest % SK_ND], (oldest / SK_ND) & 1)) {
          atomicExch(&P.st->error, ERR_RING);
          return;
        }
        tail = q_end[oldest % SK_ND];
        oldest++;
      }
      const uint32_t d = s % SK_ND;
      stage_off[d] = (uint32_t)(head % RB);
      mbar_expect_tx(&full[d], B);
      bulk_g2s(ring + head % RB, e.src, B, &full[d], pol);
      q_end[d] = head + B;
      head += B;
      s++;
      s_issued = s;
      copied += B;
      // stage records: keep SL_NB blocks loaded from the copy cursor's block on
      while (loaded < s / SL_BLK + SL_NB) load_block(loaded++);
      // L2 prefetch window ahead of the copies, within the loaded blocks
      if (j < s) j = s;
      while (!pf_done && j < loaded * SL_BLK && prefetched < copied + P.pf_ahead) {
        StageRec f;
        if (!entry(j, &f)) break;
        if (f.bytes == 0) {
          pf_done = true;
          break;
        }
        bulk_prefetch(f.src, f.bytes);
        prefetched += f.bytes;
        j++;
      }
    }
    return;
  }

  // ---------------- consumers ----------------
  const uint32_t ctid = tid;
  SkCons S;
  S.ring = ring;
  S.full = full;
  S.empty = empty;
  S.off = stage_off;
  S.crec = crec;
  S.recbar = recbar;
  S.recfree = recfree;
  S.s = 0;
  S.q = 0;
  uint32_t aseq = 0;
  uint32_t nbar = 0;
  Tracer tr;
  if (ctid == 0) issue_rec(0);
  for (uint32_t pi = 0; pi < P.nph; pi++) {
    if (pi > 0 && !sk_grid_sync(P, ++nbar, ctid, &s_fail)) return;
    if (!mbar_wait(&prbar[pi & 1], (pi >> 1) & 1)) {
      if (ctid == 0) atomicExch(&P.st->error, ERR_RECORDS);
      return;  // every consumer thread times out the same way
    }
    const PhaseRec& R = prs[pi & 1];
    if (ctid == 0) {
      if (pi + 1 < P.nph) issue_rec(pi + 1);
      tr.begin(TR_STEP + R.kind, pi);
      if (tr.r) tr.r->t[5] = s_issued - S.s;  // stages issued ahead of the consumers
    }
    if (R.kind == PH_EMBED) {
      // x = token_embd row of the step's token (src/model.rs:482-506)
      const uint32_t tok = __ldcg(&P.st->token), U = (P.emb_cols + 63) / 64;
      if (tok >= P.emb_rows) {
        if (blockIdx.x == 0 && ctid == 0) P.st->error = 1;
      } else {
        for (uint32_t u = blockIdx.x * GV_NT + ctid; u < U; u += gridDim.x * GV_NT)
          dequant_unit(P.emb_dt, P.emb, P.emb_rows, tok, P.emb_cols, u, P.x);
      }
    } else if (R.kind == PH_ATTN) {
      bool ok = R.hd == 128 ? sk_attention<128>(P, R, reinterpret_cast<float*>(ureg), qs, abar, aseq,
                                                reinterpret_cast<float*>(crec), ctid)
                            : sk_attention<64>(P, R, reinterpret_cast<float*>(ureg), qs, abar, aseq,
                                               reinterpret_cast<float*>(crec), ctid);
      if (!ok) s_fail = 1;
      named_sync(1, GV_NT);
      if (s_fail) return;
    } else if (R.active) {
      const uint32_t dt = R.dt, cols = R.cols;
      if (ctid < R.nch) {
        const uint32_t u0 = lay_cu0(dt, cols, ctid), u1 = lay_cu0(dt, cols, ctid + 1);
        chunks[ctid].cu0 = u0;
        chunks[ctid].nu = u1 - u0;
        chunks[ctid].tb = lay_chunk_bytes(dt, u1 - u0);
      }
      for (uint32_t r = ctid; r < SK_ACC / 4; r += GV_NT) acc[r] = 0.f;
      const XRun* rec_full = nullptr;
      if (R.x) {
        sk_prologue_f32(R, reinterpret_cast<XRun*>(ureg), red, ctid);
        rec_full = reinterpret_cast<const XRun*>(ureg);
      }
      named_sync(1, GV_NT);
      if (ctid == 0) tr.mark(1);
      if (!R.x && ctid == 0) {
        // the first two chunks' input records
        for (uint32_t c = 0; c < 2 && c < R.nch; c++) {
          if (!sk_issue_records(S, R.in_runs, chunks[c], S.q + c)) {
            atomicExch(&P.st->error, ERR_RECORDS);
            s_fail = 1;
            break;
          }
        }
      }
      bool ok = s_fail == 0;
      if (ok) {
        switch (dt) {
          case FZ_Q4_K: ok = sk_consume<FZ_Q4_K>(R, chunks, S, rec_full, acc, ctid); break;
          case FZ_Q6_K: ok = sk_consume<FZ_Q6_K>(R, chunks, S, rec_full, acc, ctid); break;
          case FZ_Q8_0: ok = sk_consume<FZ_Q8_0>(R, chunks, S, rec_full, acc, ctid); break;
          case FZ_Q5_0: ok = sk_consume<FZ_Q5_0>(R, chunks, S, rec_full, acc, ctid); break;
        }
      }
      if (!ok) {
        if (ctid == 0) atomicExch(&P.st->error, ERR_RING);
        s_fail = 1;
      }
      named_sync(1, GV_NT);
      if (ctid == 0) tr.mark(2);
      if (s_fail) return;
      sk_epilogue(R, acc, kred, P.st, ctid);
    }
    if (ctid == 0) {
      tr.mark(3);
      // the next phase's record has landed by now as a rule; if it is an
      // attention item, pull this CTA's share of its K/V rows into L2
      if (pi + 1 < P.nph && mbar_wait(&prbar[(pi + 1) & 1], ((pi + 1) >> 1) & 1)) {
        const PhaseRec& A = prs[(pi + 1) & 1];
        if (A.kind == PH_ATTN && A.active) {
          const uint32_t pos = min(__ldcg(&P.st->pos), P.max_ctx - 1), per = (pos + 1 + A.S - 1) / A.S;
          const uint32_t a0 = min(A.split * per, pos), a1 = min(pos, a0 + per);
          if (a1 > a0) {
            const uint64_t off = ((uint64_t)A.kvh * P.max_ctx + a0) * A.hd;
            bulk_prefetch(A.kc + off, (a1 - a0) * A.hd * 4);
            bulk_prefetch(A.vc + off, (a1 - a0) * A.hd * 4);
          }
        }
      }
    }
  }
  // step bookkeeping once every CTA's argmax candidate is in (src/generate.rs:69-77)
  if (!sk_grid_sync(P, ++nbar, ctid, &s_fail)) return;
  if (blockIdx.x == 0 && ctid == 0) {
    StepState* st = P.st;
    const uint32_t step = st->step;
    if (P.has_logits) {
      const uint32_t id = 0xFFFFFFFFu - (uint32_t)(__ldcg(&st->argmax_key) & 0xFFFFFFFFull);
      if (P.ids_out) P.ids_out[step] = id;
      st->token = (step + 1 < st->n_forced) ? P.forced[step + 1] : id;
    } else {
      st->token = (step + 1 < st->n_forced) ? P.forced[step + 1] : st->token;
    }
    st->argmax_key = 0;
    st->step = step + 1;
    st->pos = st->pos + 1;
  }
}
