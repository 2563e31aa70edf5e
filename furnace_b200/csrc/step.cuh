// The whole decode step as one persistent kernel (included by kernels.cu,
// after the GEMV and attention code whose device functions it reuses).
//
// One CTA per SM runs every phase of the step -- per layer the q|k|v GEMV,
// attention, o_proj, gate/up and down, then lm_head (src/model.rs:444-478,
// 594-600) -- from a list of phase descriptors built on the host.  Warp 15 is
// the producer: it walks the same list and bulk-copies this CTA's share of
// every phase's bytes (weight tiles; for attention the cached K/V rows of its
// split of the context) into a byte ring of shared memory.  It never waits
// for activations, only for ring space, so HBM keeps streaming the next
// phases' weights while the consumers synchronise.
//
// Warps 0-14 consume the ring in the same order.  Stage n occupies ring
// slot n mod MK_NSLOT (its full / empty mbarriers) and a byte range that
// both sides compute the same way from the stage sizes (ring_alloc).  Phase
// descriptors reach shared memory by bulk copy, two phases ahead of use, so
// neither side waits on descriptor loads.
//
// Phases hand data to each other through global memory and arrival counters:
// a phase's CTAs add one to its counter when their outputs are written (proxy
// fence, fence, atomic add), and the next phase's consumers poll the counter
// with acquire loads before they read.  Reads of data written by other CTAs
// of this launch go to L2 (ld.cg, acquire loads, or bulk copies after a proxy
// fence).
//
// Attention (src/model.rs:371-438) is split-K over the context: CTA b takes
// KV head g = b / S and positions [t0, t1) of split s = b % S, and stores
// the partial softmax state of that head's query heads.  The S CTAs of a KV
// head then wait for each other and each merges its share of the head
// group's 16-element output runs, written as run records for o_proj.
//
// Every wait is bounded (about a second, or earlier once another CTA has set
// the error word): on expiry the CTA records an error code in the step state
// and stops, the producer waits for its copies in flight, and the host
// reports FZ_ETIMEOUT.  The counters are returned to zero by the last CTA to
// finish, so the captured launch can be replayed.

constexpr int MK_THREADS = 512;
constexpr int MK_CWARPS = 15;
constexpr int MK_NT = MK_CWARPS * 32;
#ifndef MK_RPW
#define MK_RPW 2  // rows per consumer warp and ring stage
#endif
constexpr int MK_ROWS = MK_CWARPS * MK_RPW;
#ifndef MK_NOINLINE
#define MK_NOINLINE
#endif
constexpr uint32_t MK_NSLOT = 8;   // stages in flight at most
constexpr uint32_t MK_NREC = 4;    // record chunks in flight (long inputs)
constexpr long long MK_SPIN_NS = 1000000000ll;

struct MkParams {
  const MkPhase* ph;
  uint32_t nph;
  uint32_t* sync;
  uint32_t nsync, done_ctr;
  StepState* st;
  float eps;
  const float* qkv;
  const float2* rope_cs;
  float* partials;
  float* ctx;
  uint32_t nh, nkv, hd, max_ctx, splits;
  int kv_f16;
  uint32_t ring_bytes, rec_bytes, acc_floats;
};

__device__ __forceinline__ uint32_t ld_acquire_u32(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ uint32_t ld_volatile_u32(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.volatile.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void fence_proxy_async_global() { asm volatile("fence.proxy.async.global;" ::: "memory"); }
__device__ __forceinline__ void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// Poll sync[i] until it reaches target; false (with the error word set) when
// the wait runs out or another CTA reported an error.
__device__ bool mk_poll(const MkParams& p, uint32_t i, uint32_t target) {
  const uint32_t* c = p.sync + i;
  if (ld_acquire_u32(c) >= target) return true;
  const uint64_t t0 = gtimer();
  for (;;) {
    if (ld_acquire_u32(c) >= target) return true;
    if (ld_volatile_u32(&p.st->error)) return false;
    if (gtimer() - t0 > (uint64_t)MK_SPIN_NS) {
      atomicCAS(&p.st->error, 0u, 8u);
      return false;
    }
  }
}

// mbarrier wait that also gives up once the error word is set.
__device__ __forceinline__ bool mk_mbar_wait(uint64_t* bar, uint32_t parity, const uint32_t* err) {
  if (mbar_try(bar, parity)) return true;
  const long long t0 = clock64();
  uint32_t n = 0;
  while (!mbar_try(bar, parity)) {
    if ((++n & 63) == 0 && ld_volatile_u32(err)) return false;
    if (clock64() - t0 > (1ll << 31)) return false;
  }
  return true;
}

// Consumer-side barrier of the 15 consumer warps.
__device__ __forceinline__ void mk_csync() { named_sync(1, MK_NT); }

// All of this CTA's outputs of the phase are written: publish them.
__device__ void mk_arrive(const MkParams& p, uint32_t ctr) {
  mk_csync();
  if (threadIdx.x == 0) {
    fence_proxy_async_global();  // generic-proxy writes, read later by bulk copies
    __threadfence();
    atomicAdd(p.sync + ctr, 1u);
  }
}

// Wait until sync[ctr] >= target: one thread polls, then every consumer
// thread proceeds.  Returns false on error (block-uniform).
__device__ bool mk_wait(const MkParams& p, uint32_t ctr, uint32_t target, volatile uint32_t* flag) {
  if (threadIdx.x == 0) *flag = target == 0 || mk_poll(p, ctr, target) ? 1u : 0u;
  mk_csync();
  return *flag != 0;
}

// This CTA's attention work: KV head g and positions [t0, t1) of [0, pos].
__device__ __forceinline__ bool mk_att_range(const MkParams& p, uint32_t pos, uint32_t* g, uint32_t* t0,
                                             uint32_t* t1) {
  const uint32_t S = p.splits, b = blockIdx.x;
  if (b >= p.nkv * S) return false;
  *g = b / S;
  const uint32_t s = b % S, total = pos + 1, per = (total + S - 1) / S;
  *t0 = min(s * per, total);
  *t1 = min(total, *t0 + per);
  return true;
}

// Byte range of the next stage: FIFO through the ring, restarting at 0 when
// the stage does not fit before the end.  Producer and consumers call it
// with the same sizes in the same order.
__device__ __forceinline__ uint32_t ring_alloc(uint32_t& head, uint32_t bytes, uint32_t ring_bytes) {
  if (head + bytes > ring_bytes) head = 0;
  const uint32_t off = head;
  head += bytes;
  return off;
}

// Bytes of one attention stage: a K tile and a V tile of AT_TP positions.
__device__ __forceinline__ uint32_t mk_kv_stage(const MkParams& p) { return 2u * AT_TP * p.hd * (p.kv_f16 ? 2u : 4u); }

// ---------------------------------------------------------------------------
// producer: every phase's bytes for this CTA, in consumption order
// ---------------------------------------------------------------------------
struct MkProd {
  uint8_t* ring;
  uint64_t *full, *empty;
  const uint32_t* err;
  uint64_t pol;
  uint32_t n = 0, rel = 0, head = 0;  // stages issued, stages known released, ring head
  // byte ranges of the stages in flight by slot, kept in registers: every
  // index below is a compile-time constant after unrolling
  uint32_t soff[MK_NSLOT], send[MK_NSLOT], live = 0;
  uint64_t waited = 0;  // ns spent waiting for ring space (timeline trace)
  bool ok = true, reserve_ok = true;

  // Room for a stage of `bytes`: its slot and its byte range free.
  __device__ bool reserve(uint32_t bytes, uint32_t ring_bytes, uint32_t* off) {
    const uint32_t o = ring_alloc(head, bytes, ring_bytes), e = o + bytes;
    for (;;) {
      bool clash = n - rel >= MK_NSLOT;
#pragma unroll
      for (uint32_t j = 0; j < MK_NSLOT; j++) clash |= ((live >> j) & 1) && o < send[j] && soff[j] < e;
      if (!clash) break;
      const uint64_t tw = gtimer();
      const bool got = mk_mbar_wait(&empty[rel % MK_NSLOT], (rel / MK_NSLOT) & 1, err);
      waited += gtimer() - tw;
      if (!got) return reserve_ok = false;
      live &= ~(1u << (rel % MK_NSLOT));
      rel++;
    }
    const uint32_t sl = n % MK_NSLOT;
#pragma unroll
    for (uint32_t j = 0; j < MK_NSLOT; j++)
      if (j == sl) {
        soff[j] = o;
        send[j] = e;
      }
    live |= 1u << sl;
    *off = o;
    return true;
  }
};

// One stage of the producer's walk: up to two copies (attention: K and V)
// into one ring range of `size` bytes.
struct MkStage {
  const uint8_t* src[2];
  uint32_t nb[2], off1, size;
};

// Walks this CTA's stages of phases [k, kend) in consumption order.  The
// producer runs one walker that issues the copies and a second one ahead of
// it that only prefetches into L2 (cp.async.bulk.prefetch.L2), so more bytes
// are requested from HBM than the ring can hold.
struct MkWalk {
  uint32_t k = 0, c = 0, ra = 0, a = 0, t1 = 0;
  uint32_t sk = 0;  // phase of the stage returned last
  bool open = false;
  bool fetches = false;  // the copying walk refills a descriptor buffer as it leaves a phase
  StageIter it;
  const uint8_t *kb = nullptr, *vb = nullptr;

  __device__ void leave(const MkParams& p, MkPhase* desc, uint64_t* dbar) {
    if (fetches && k + 2 < p.nph) {
      // phase k's descriptor is not read again: its buffer takes phase k + 2
      fence_proxy_async_smem();
      mbar_expect_tx(&dbar[k & 1], sizeof(MkPhase));
      bulk_g2s(&desc[k & 1], &p.ph[k + 2], sizeof(MkPhase), &dbar[k & 1], 0ull);
    }
    k++;
    open = false;
  }

  // 1: *st is the next stage; 0: phase kend reached; -1: phase k's
  // descriptor has not landed yet (only when !block); -2: a wait ran out.
  __device__ int next(const MkParams& p, MkPhase* desc, uint64_t* dbar, uint32_t kend, bool block, uint32_t pos,
                      MkStage* st) {
    for (;;) {
      if (k >= kend) return 0;
      const MkPhase& ph = desc[k & 1];
      if (!open) {
        if (block) {
          if (!mk_mbar_wait(&dbar[k & 1], (k >> 1) & 1, &p.st->error)) return -2;
        } else if (!mbar_try(&dbar[k & 1], (k >> 1) & 1)) {
          return -1;
        }
        open = true;
        if (ph.kind == MK_GEMV) {
          it.init(ph.seg, ph.nseg, blockIdx.x);
          c = 0;
          ra = it.r0;
        } else {
          uint32_t g, t0;
          a = t1 = 0;
          if (pos < p.max_ctx && mk_att_range(p, pos, &g, &t0, &t1)) {
            const uint32_t rowb = p.hd * (p.kv_f16 ? 2u : 4u);
            kb = static_cast<const uint8_t*>(ph.kc) + (uint64_t)g * p.max_ctx * rowb;
            vb = static_cast<const uint8_t*>(ph.vc) + (uint64_t)g * p.max_ctx * rowb;
            a = t0;
          }
        }
      }
      // the walk leaves a phase as soon as its last stage is handed out, so
      // the phase's descriptor is not read again after that
      sk = k;
      if (ph.kind == MK_GEMV) {
        if (c < it.nch) {
          ChunkInfo ci;
          chunk_info(it, c, &ci);
          const uint32_t nr = min(ra + ph.rs, it.r1) - ra;
          st->src[0] = ci.plane + (uint64_t)ra * ci.tb;
          st->nb[0] = nr * ci.tb;
          st->src[1] = nullptr;
          st->nb[1] = 0;
          st->off1 = 0;
          st->size = st->nb[0];
          ra += ph.rs;
          if (ra >= it.r1) {
            ra = it.r0;
            c++;
          }
          if (c >= it.nch) leave(p, desc, dbar);
          return 1;
        }
      } else if (a < t1) {
        // rows below pos are final; row pos is this step's and is patched in
        const uint32_t rowb = p.hd * (p.kv_f16 ? 2u : 4u);
        const uint32_t e = min(min(t1, a + AT_TP), pos), rows = e > a ? e - a : 0;
        st->src[0] = kb + (uint64_t)a * rowb;
        st->src[1] = vb + (uint64_t)a * rowb;
        st->nb[0] = st->nb[1] = rows * rowb;
        st->off1 = AT_TP * rowb;
        st->size = mk_kv_stage(p);
        a += AT_TP;
        if (a >= t1) leave(p, desc, dbar);
        return 1;
      }
      leave(p, desc, dbar);  // a phase without stages for this CTA
    }
  }
};

constexpr uint32_t MK_PF_AHEAD = 128 * 1024;  // bytes requested ahead of the ring's copies

MK_NOINLINE __device__ void mk_producer(const MkParams& p, uint8_t* ring, uint64_t* full, uint64_t* empty, MkPhase* desc,
                            uint64_t* dbar) {
  MkProd pr;
  pr.ring = ring;
  pr.full = full;
  pr.empty = empty;
  pr.err = &p.st->error;
  pr.pol = policy_evict_first();
  const uint32_t pos = p.st->pos;  // written before this launch (stream order)
  auto fetch_desc = [&](uint32_t k) {
    mbar_expect_tx(&dbar[k & 1], sizeof(MkPhase));
    bulk_g2s(&desc[k & 1], &p.ph[k], sizeof(MkPhase), &dbar[k & 1], 0ull);
  };
  fetch_desc(0);
  if (p.nph > 1) fetch_desc(1);
  MkWalk w, pf;
  w.fetches = true;
  uint64_t copied = 0, prefetched = 0;
  MkStage st, sp;
  Tracer tr;  // per phase: t[0] first copy issued, t[1] last, t[2] ns waiting for ring space
  uint32_t tk = ~0u;
  uint64_t w0 = 0;
  for (;;) {
    const int r = w.next(p, desc, dbar, p.nph, true, pos, &st);
    if (r == 1 && w.sk != tk) {
      if (tr.r) tr.r->t[2] = pr.waited - w0;
      tr = Tracer();
      tr.begin(TR_STEP + 8, w.sk);
      tk = w.sk;
      w0 = pr.waited;
    }
    if (r == 0) break;
    if (r < 0) {
      pr.ok = false;
      break;
    }
    uint32_t off;
    if (!pr.reserve(st.size, p.ring_bytes, &off)) break;
    uint64_t* fb = &full[pr.n % MK_NSLOT];
    mbar_expect_tx(fb, st.nb[0] + st.nb[1]);
    if (st.nb[0]) bulk_g2s(ring + off, st.src[0], st.nb[0], fb, pr.pol);
    if (st.nb[1]) bulk_g2s(ring + off + st.off1, st.src[1], st.nb[1], fb, pr.pol);
    pr.n++;
    copied += st.size;
    tr.mark(1);
    // keep the L2 prefetch walk MK_PF_AHEAD bytes in front, at most into the
    // phase after the one being copied (whose descriptor is resident)
    if (prefetched < copied) {
      pf = w;
      pf.fetches = false;
      prefetched = copied;
    }
    while (prefetched < copied + MK_PF_AHEAD) {
      const int q = pf.next(p, desc, dbar, min(p.nph, w.k + 2), false, pos, &sp);
      if (q <= 0) break;
      if (sp.nb[0]) bulk_prefetch(sp.src[0], sp.nb[0]);
      if (sp.nb[1]) bulk_prefetch(sp.src[1], sp.nb[1]);
      prefetched += sp.size;
    }
  }
  if (tr.r) tr.r->t[2] = pr.waited - w0;
  if (!pr.ok || !pr.reserve_ok) {
    atomicCAS(&p.st->error, 0u, 4u);
    // descriptors up to two phases past the walk may still be in flight
    for (uint32_t j = w.k; j < w.k + 2 && j < p.nph; j++) mbar_wait(&dbar[j & 1], (j >> 1) & 1);
    // the copies already issued land in this CTA's shared memory: wait for
    // them (bounded) before this thread, possibly the CTA's last, exits
    for (uint32_t j = pr.n > MK_NSLOT ? pr.n - MK_NSLOT : 0; j < pr.n; j++)
      mbar_wait(&full[j % MK_NSLOT], (j / MK_NSLOT) & 1);
  }
}

// ---------------------------------------------------------------------------
// consumers
// ---------------------------------------------------------------------------
struct MkCons {
  uint8_t* ring;
  uint64_t *full, *empty;
  const uint32_t* err;
  uint32_t n = 0, head = 0;  // stages consumed, ring head (mirrors the producer)
  // the next stage: wait until it has landed; returns its bytes in the ring
  uint64_t waited = 0;  // ns this thread spent waiting for stages (timeline trace)
  __device__ const uint8_t* acquire(uint32_t bytes, uint32_t ring_bytes) {
    const uint32_t off = ring_alloc(head, bytes, ring_bytes);
    uint64_t* b = &full[n % MK_NSLOT];
    const uint32_t par = (n / MK_NSLOT) & 1;
    if (!mbar_try(b, par)) {
      const uint64_t t = gtimer();
      const bool ok = mk_mbar_wait(b, par, err);
      waited += gtimer() - t;
      if (!ok) return nullptr;
    }
    return ring + off;
  }
  // every consumer warp calls this once per stage
  __device__ void release() {
    __syncwarp();
    if ((threadIdx.x & 31) == 0) mbar_arrive(&empty[n % MK_NSLOT]);
    n++;
  }
};

struct MkRec {  // streamed input records of long vectors (MK_NREC buffers)
  uint64_t *bar, *free;
  uint32_t use = 0;
};

template <uint32_t DT>
__device__ bool mk_gemv_body(const MkParams& p, const MkPhase& ph, const StageIter& it, const ChunkInfo* chunks,
                             MkCons& cs, uint8_t* rec, float* acc, MkRec& rr) {
  const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const bool chunked = ph.in_kind == MK_IN_RUNS_CHUNKED;
  const uint32_t use0 = rr.use;
  auto issue_rec = [&](uint32_t c) -> bool {  // thread 0: chunk c's records into buffer (use0 + c) % MK_NREC
    const uint32_t u = use0 + c, b = u % MK_NREC;
    if (u >= MK_NREC && !mk_mbar_wait(&rr.free[b], ((u - MK_NREC) / MK_NREC) & 1, cs.err)) return false;
    fence_proxy_async_global();
    mbar_expect_tx(&rr.bar[b], chunks[c].nu * 256);
    bulk_g2s(rec + b * GV_CREC, reinterpret_cast<const uint8_t*>(ph.in_runs) + 256ull * chunks[c].cu0,
             chunks[c].nu * 256, &rr.bar[b], 0ull);
    return true;
  };
  if (chunked && threadIdx.x == 0)
    for (uint32_t c = 0; c < MK_NREC && c < it.nch; c++)
      if (!issue_rec(c)) return false;
  for (uint32_t c = 0; c < it.nch; c++) {
    const uint32_t nu = chunks[c].nu, tb = chunks[c].tb;
    const uint32_t lu = min(lane, nu - 1);
    const float lane_on = lane < nu ? 1.f : 0.f;
    const XRun* rb = reinterpret_cast<const XRun*>(rec);
    if (chunked) {
      const uint32_t u = use0 + c;
      if (!mk_mbar_wait(&rr.bar[u % MK_NREC], (u / MK_NREC) & 1, cs.err)) return false;
      rb = reinterpret_cast<const XRun*>(rec + (u % MK_NREC) * GV_CREC) - 4 * chunks[c].cu0;
    }
    XRun xr[4];
#pragma unroll
    for (uint32_t j = 0; j < 4; j++) xr[j] = load_run(rb, chunks[c].cu0 + lu, j);
    if (chunked) {
      __syncwarp();
      if (lane == 0) mbar_arrive(&rr.free[(use0 + c) % MK_NREC]);
      if (threadIdx.x == 0 && c + MK_NREC < it.nch && !issue_rec(c + MK_NREC)) return false;
    }
    for (uint32_t ra = it.r0; ra < it.r1; ra += ph.rs) {
      const uint32_t nr = min(ra + ph.rs, it.r1) - ra;
      const uint8_t* tile = cs.acquire(nr * tb, p.ring_bytes);
      if (!tile) return false;
      const uint32_t last = nr - 1;
      float v[MK_RPW];
#pragma unroll
      for (int j = 0; j < MK_RPW; j++) {
        const uint32_t r = min(warp + MK_CWARPS * j, last);
        v[j] = lane_on * unit_dot<DT>(tile + r * tb, lu, nu, xr);
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1)
#pragma unroll
        for (int j = 0; j < MK_RPW; j++) v[j] += __shfl_xor_sync(0xffffffffu, v[j], o);
      if (lane == 0) {
#pragma unroll
        for (int j = 0; j < MK_RPW; j++) {
          const uint32_t r = warp + MK_CWARPS * j;
          if (r <= last) acc[ra + r - it.r0] += v[j];
        }
      }
      cs.release();
    }
  }
  if (chunked) rr.use = use0 + it.nch;
  return true;
}

__device__ bool mk_gemv(const MkParams& p, const MkPhase& ph, MkCons& cs, uint8_t* rec, float* acc, uint64_t* rbar,
                        uint32_t& ruse, MkRec& rr, ChunkInfo* chunks, float* red, unsigned long long* kred,
                        volatile uint32_t* flag, Tracer& tr) {
  const uint32_t ctid = threadIdx.x, warp = ctid >> 5, lane = ctid & 31;
  StageIter it;
  it.init(ph.seg, ph.nseg, blockIdx.x);
  if (ctid < it.nch && it.n_stages) chunk_info(it, ctid, &chunks[ctid]);
  for (uint32_t r = ctid; r < ph.max_rows; r += MK_NT) acc[r] = 0.f;
  // the RMSNorm weight does not depend on the predecessor: load it first
  const uint32_t n4 = ph.cols / 4, NX = runs_for_dev(ph.cols);
  const bool norm = ph.in_kind == MK_IN_NORM;
  float4 buf[16];
  if (norm && it.n_stages) {
    const float4* w4 = reinterpret_cast<const float4*>(ph.norm_w);
#pragma unroll
    for (int j = 8; j < 16; j++) {
      const uint32_t i4 = ctid + MK_NT * (j - 8);
      buf[j] = i4 < n4 ? w4[i4] : make_float4(0.f, 0.f, 0.f, 0.f);
    }
  }
  if (!mk_wait(p, ph.wait_ctr, ph.wait_target, flag)) return false;
  if (ctid == 0) tr.mark(1);
  if (it.n_stages) {
    if (ph.in_kind == MK_IN_RUNS) {
      // records written by other CTAs (the attention merges): one bulk copy
      if (ctid == 0) {
        fence_proxy_async_global();
        mbar_expect_tx(rbar, NX * 64);
        bulk_g2s(rec, ph.in_runs, NX * 64, rbar, 0ull);
      }
      if (!mk_mbar_wait(rbar, ruse & 1, cs.err)) *flag = 0;
      ruse++;
    } else if (norm) {
      // x (updated by other CTAs: read through L2), RMS-normalised
      // (src/tensor.rs:164-186), to records
      const float4* x4 = reinterpret_cast<const float4*>(ph.x);
#pragma unroll
      for (int j = 0; j < 8; j++) {
        const uint32_t i4 = ctid + MK_NT * j;
        buf[j] = i4 < n4 ? __ldcg(x4 + i4) : make_float4(0.f, 0.f, 0.f, 0.f);
      }
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
      mk_csync();
      float tot = 0.f;
#pragma unroll
      for (int w = 0; w < MK_CWARPS; w++) tot += red[w];
      const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, (float)ph.cols), p.eps)));
#pragma unroll
      for (int j = 0; j < 8; j++) {
        if (MK_NT * j >= 4 * NX) break;  // block-uniform
        const uint32_t i4 = ctid + MK_NT * j;
        const float4 wn = buf[j + 8];
        float v[4] = {buf[j].x, buf[j].y, buf[j].z, buf[j].w};
        v[0] = __fmul_rn(__fmul_rn(v[0], inv), wn.x);
        v[1] = __fmul_rn(__fmul_rn(v[1], inv), wn.y);
        v[2] = __fmul_rn(__fmul_rn(v[2], inv), wn.z);
        v[3] = __fmul_rn(__fmul_rn(v[3], inv), wn.w);
        quad_to_run(v, i4 & 3, (i4 >> 2) < NX ? reinterpret_cast<XRun*>(rec) : nullptr, i4 >> 2);
      }
    }
  }
  mk_csync();
  if (*flag == 0) return false;  // a wait above ran out (block-uniform after the barrier)
  if (ctid == 0) tr.mark(2);
  bool ok = true;
  if (it.n_stages) {
    switch (it.dt) {
      case FZ_Q4_K: ok = mk_gemv_body<FZ_Q4_K>(p, ph, it, chunks, cs, rec, acc, rr); break;
      case FZ_Q6_K: ok = mk_gemv_body<FZ_Q6_K>(p, ph, it, chunks, cs, rec, acc, rr); break;
      case FZ_Q8_0: ok = mk_gemv_body<FZ_Q8_0>(p, ph, it, chunks, cs, rec, acc, rr); break;
      case FZ_Q5_0: ok = mk_gemv_body<FZ_Q5_0>(p, ph, it, chunks, cs, rec, acc, rr); break;
    }
  }
  // a failed wait is block-uniform only after this vote
  if (lane == 0 && !ok) *flag = 0;
  mk_csync();
  if (*flag == 0) return false;
  if (ctid == 0) tr.mark(3);
  if (!it.n_stages) return true;
  const GvSeg& s = *it.s;
  const uint32_t nrows = it.r1 - it.r0;
  if (ph.epilogue == EPI_STORE) {
    for (uint32_t i = ctid; i < nrows; i += MK_NT) {
      const uint32_t row = it.r0 + i;
      s.out[row] = s.bias ? __fadd_rn(acc[i], s.bias[row]) : acc[i];
    }
  } else if (ph.epilogue == EPI_RESID) {
    // x += W v (src/model.rs:470, :477); x was last written by another CTA
    for (uint32_t i = ctid; i < nrows; i += MK_NT) {
      const uint32_t row = it.r0 + i;
      s.out[row] = __fadd_rn(__ldcg(s.out + row), acc[i]);
    }
  } else if (ph.epilogue == EPI_SWIGLU) {
    // rows interleave gate/up: h = silu(gate) * up (src/tensor.rs:213-227)
    const uint32_t np = nrows / 2;
    float hv[4];
#pragma unroll
    for (uint32_t k = 0; k < 4; k++) {
      const uint32_t j = ctid + k * MK_NT;
      hv[k] = 0.f;
      if (j < np) {
        const float g = acc[2 * j], u = acc[2 * j + 1];
        hv[k] = __fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, expf(-g))), u);
      }
    }
    mk_csync();
#pragma unroll
    for (uint32_t k = 0; k < 4; k++) {
      const uint32_t j = ctid + k * MK_NT;
      if (j < np) acc[j] = hv[k];
    }
    mk_csync();
    values_to_runs(acc, np, nullptr, ph.out_runs, it.r0 / 32, ctid, MK_NT);
  } else {
    unsigned long long best = 0;
    for (uint32_t i = ctid; i < nrows; i += MK_NT) {
      const uint32_t row = it.r0 + i;
      const float v = acc[i];
      s.out[row] = v;
      const unsigned long long k = argmax_key(v, row + ph.idx_base);
      best = k > best ? k : best;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
      best = other > best ? other : best;
    }
    if (lane == 0) kred[warp] = best;
    mk_csync();
    if (ctid == 0) {
      unsigned long long m = 0;
      for (int w = 0; w < MK_CWARPS; w++) m = kred[w] > m ? kred[w] : m;
      atomicMax(&p.st->argmax_key, m);
    }
  }
  return true;
}

// Attention of one layer: this CTA's split, then its share of the merge.
template <int HD, typename KT>
MK_NOINLINE __device__ bool mk_attn(const MkParams& p, const MkPhase& ph, MkCons& cs, uint8_t* scratch, volatile uint32_t* flag,
                        Tracer& tr) {
  constexpr int DPL = HD / 32;
  const uint32_t tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const uint32_t G = p.nh / p.nkv, half = HD / 2, S = p.splits;
  const uint32_t pos = ld_volatile_u32(&p.st->pos);
  uint32_t g = 0, t0 = 0, t1 = 0;
  const bool work = pos < p.max_ctx && mk_att_range(p, pos, &g, &t0, &t1);
  if (!mk_wait(p, ph.wait_ctr, ph.wait_target, flag)) return false;
  if (tid == 0) tr.mark(1);
  if (!work) {
    if (pos >= p.max_ctx && tid == 0) atomicCAS(&p.st->error, 0u, 2u);
    return pos < p.max_ctx;
  }
  // shared scratch (the records region, unused by attention):
  // q[AT_MAXG][HD] | knew[HD] | vnew[HD] | per-warp (m, l) | per-warp acc[HD];
  // the merge reuses it from the start once the partials are stored
  float* qs = reinterpret_cast<float*>(scratch);
  float* knew = qs + AT_MAXG * HD;
  float* vnew = knew + HD;
  float2* wml = reinterpret_cast<float2*>(vnew + HD);
  float* wacc = reinterpret_cast<float*>(wml + MK_CWARPS);
  const float2* csp = p.rope_cs + (uint64_t)pos * half;
  for (uint32_t idx = tid; idx < G * half; idx += MK_NT) {
    const uint32_t h = idx / half, i = idx % half;
    const float* xq = p.qkv + (uint64_t)(g * G + h) * HD;
    const float a = __ldcg(xq + i), b = __ldcg(xq + i + half);
    const float2 c = csp[i];
    qs[h * HD + i] = __fsub_rn(__fmul_rn(a, c.x), __fmul_rn(b, c.y));
    qs[h * HD + i + half] = __fadd_rn(__fmul_rn(a, c.y), __fmul_rn(b, c.x));
  }
  const bool owns_pos = t1 > t0 && t1 == pos + 1;
  if (owns_pos && tid < half) {
    // rotate the new k, append k and v (KvCache::append, src/model.rs:346-356);
    // the values as cached (f16: rounded) serve this position too
    const float* kx = p.qkv + (uint64_t)(p.nh + g) * HD;
    const float* vx = p.qkv + (uint64_t)(p.nh + p.nkv + g) * HD;
    const float a = __ldcg(kx + tid), b = __ldcg(kx + tid + half);
    const float2 c = csp[tid];
    const float k0 = kv_round<KT>(__fsub_rn(__fmul_rn(a, c.x), __fmul_rn(b, c.y)));
    const float k1 = kv_round<KT>(__fadd_rn(__fmul_rn(a, c.y), __fmul_rn(b, c.x)));
    const float v0 = kv_round<KT>(__ldcg(vx + tid)), v1 = kv_round<KT>(__ldcg(vx + tid + half));
    knew[tid] = k0;
    knew[tid + half] = k1;
    vnew[tid] = v0;
    vnew[tid + half] = v1;
    KT* kdst = static_cast<KT*>(ph.kc) + ((uint64_t)g * p.max_ctx + pos) * HD;
    KT* vdst = static_cast<KT*>(ph.vc) + ((uint64_t)g * p.max_ctx + pos) * HD;
    kv_st(kdst + tid, k0);
    kv_st(kdst + tid + half, k1);
    kv_st(vdst + tid, v0);
    kv_st(vdst + tid + half, v1);
  }
  mk_csync();
  if (tid == 0) tr.mark(2);
  // warps per query head: 15 / G (at least 1); warp w serves head w / wph and
  // tiles j = w % wph (mod wph)
  const uint32_t wph = max(1u, MK_CWARPS / G);
  const uint32_t hh = warp / wph, sub = warp % wph;
  const bool active = hh < G;
  const float scale = __fdiv_rn(1.0f, __fsqrt_rn((float)HD));
  float m = -INFINITY, l = 0.f, acc[DPL];
#pragma unroll
  for (int d = 0; d < DPL; d++) acc[d] = 0.f;
  const uint32_t ntiles = (t1 - t0 + AT_TP - 1) / AT_TP;
  for (uint32_t j = 0; j < ntiles; j++) {
    const uint32_t a = t0 + j * AT_TP, tn = min(t1, a + AT_TP) - a;
    KT* kt = reinterpret_cast<KT*>(const_cast<uint8_t*>(cs.acquire(mk_kv_stage(p), p.ring_bytes)));
    if (!kt && lane == 0) *flag = 0;
    mk_csync();
    if (*flag == 0) return false;  // block-uniform after the barrier
    KT* vt = kt + AT_TP * HD;
    if (owns_pos && pos >= a && pos < a + AT_TP) {  // block-uniform
      if (tid < HD) {
        kv_st(kt + (pos - a) * HD + tid, knew[tid]);
        kv_st(vt + (pos - a) * HD + tid, vnew[tid]);
      }
      mk_csync();
    }
    if (active && j % wph == sub) {
      const uint32_t t = lane;
      float s = -INFINITY;
      if (t < tn) {
        const KT* kr = kt + (size_t)t * HD;
        const float4* qr = reinterpret_cast<const float4*>(qs + hh * HD);
        float d0 = 0.f, d1 = 0.f, d2 = 0.f, d3 = 0.f;
#pragma unroll 8
        for (uint32_t c = 0; c < HD / 4; c++) {
          const uint32_t cc = (c + t) & (HD / 4 - 1);
          const float4 k4 = kv_ld4(kr, cc), q4 = qr[cc];
          d0 = fmaf(q4.x, k4.x, d0);
          d1 = fmaf(q4.y, k4.y, d1);
          d2 = fmaf(q4.z, k4.z, d2);
          d3 = fmaf(q4.w, k4.w, d3);
        }
        s = __fmul_rn((d0 + d1) + (d2 + d3), scale);
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
        if (DPL == 4) {
          const float4 v4 = kv_ld4(vt + (size_t)t2 * HD, lane);
          acc[0] = fmaf(pt, v4.x, acc[0]);
          acc[1] = fmaf(pt, v4.y, acc[1]);
          acc[2] = fmaf(pt, v4.z, acc[2]);
          acc[3] = fmaf(pt, v4.w, acc[3]);
        } else {
          const KT* vr = vt + (size_t)t2 * HD + lane * DPL;
#pragma unroll
          for (int d = 0; d < DPL; d++) acc[d] = fmaf(pt, kv_ld(vr + d), acc[d]);
        }
      }
    }
    cs.release();
  }
  // merge the wph warps of each head, then store this split's partial:
  // stats [nkv][G][S] of (max, sum), acc [nkv][G][HD][Spad]
  if (active) {
    if (lane == 0) wml[warp] = make_float2(m, l);
#pragma unroll
    for (int d = 0; d < DPL; d++) wacc[warp * HD + lane * DPL + d] = acc[d];
  }
  mk_csync();
  const uint32_t Spad = (S + 3) & ~3u, s_idx = blockIdx.x % S;
  float2* stats = reinterpret_cast<float2*>(p.partials) + (uint64_t)g * G * S;
  float* pacc = p.partials + ((2 * (uint64_t)p.nkv * G * S + 3) & ~3ull) + (uint64_t)g * G * HD * Spad;
  for (uint32_t idx = tid; idx < G * HD; idx += MK_NT) {
    const uint32_t h = idx / HD, d = idx % HD;
    float M = -INFINITY;
    for (uint32_t w = 0; w < wph; w++) M = fmaxf(M, wml[h * wph + w].x);
    float L = 0.f, A = 0.f;
    for (uint32_t w = 0; w < wph; w++) {
      const float2 ml = wml[h * wph + w];
      const float f = ml.x == -INFINITY ? 0.f : expf(ml.x - M);
      L = fmaf(ml.y, f, L);
      A = fmaf(wacc[(h * wph + w) * HD + d], f, A);
    }
    if (d == 0) stats[h * S + s_idx] = make_float2(M, L);
    pacc[((uint64_t)h * HD + d) * Spad + s_idx] = A;
  }
  if (tid == 0) tr.mark(3);
  // every split of this KV head has stored its partial: merge this CTA's share
  // of the group's runs, ctx[h][d] = sum_s w_s acc_s[d] / sum_s w_s l_s with
  // w_s = exp(m_s - max m)
  mk_arrive(p, ph.att_ctr0 + g);
  if (!mk_wait(p, ph.att_ctr0 + g, S, flag)) return false;
  const uint32_t R = G * HD / 16, r0 = s_idx * R / S, r1 = (s_idx + 1) * R / S;
  const uint32_t e0 = 16 * r0, ne = 16 * (r1 - r0);  // elements [e0, e0 + ne) of the group
  float* vals = reinterpret_cast<float*>(scratch);   // [ne] merged values
  float* ws = vals + 16 * ((R + S - 1) / S);         // per head touched: [Spad] weights
  __shared__ float den[2];
  const uint32_t h0 = e0 / HD, nhd = ne ? (e0 + ne - 1) / HD - h0 + 1 : 0;  // heads touched (<= 2)
  for (uint32_t hi = warp; hi < nhd; hi += MK_CWARPS) {
    const uint32_t h = h0 + hi;
    float M = -INFINITY;
    for (uint32_t s2 = lane; s2 < S; s2 += 32) M = fmaxf(M, __ldcg(&stats[h * S + s2].x));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
    float dsum = 0.f;
    for (uint32_t s2 = lane; s2 < Spad; s2 += 32) {
      float w = 0.f;
      if (s2 < S) {
        const float2 ml = __ldcg(&stats[h * S + s2]);
        w = ml.x == -INFINITY ? 0.f : expf(ml.x - M);
        dsum = fmaf(w, ml.y, dsum);
      }
      ws[hi * Spad + s2] = w;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) dsum += __shfl_xor_sync(0xffffffffu, dsum, o);
    if (lane == 0) den[hi] = dsum;
  }
  mk_csync();
  // one quarter warp per element: the Spad / 4 float4 of its accumulators
  // (the loop bound is block-uniform: every lane takes part in the shuffles)
  const uint32_t q = tid & 7;
  for (uint32_t i0 = 0; i0 < ne; i0 += MK_NT / 8) {
    const uint32_t idx = i0 + tid / 8, e = e0 + min(idx, ne - 1), h = e / HD, d = e % HD;
    const float4* a4 = reinterpret_cast<const float4*>(pacc + ((uint64_t)h * HD + d) * Spad);
    const float* w = ws + (h - h0) * Spad;
    float num = 0.f;
    for (uint32_t k = q; 4 * k < Spad; k += 8) {
      const float4 v = __ldcg(a4 + k);
      num = fmaf(w[4 * k], v.x, num);
      num = fmaf(w[4 * k + 1], v.y, num);
      num = fmaf(w[4 * k + 2], v.z, num);
      num = fmaf(w[4 * k + 3], v.w, num);
    }
    num += __shfl_xor_sync(0xffffffffu, num, 1);
    num += __shfl_xor_sync(0xffffffffu, num, 2);
    num += __shfl_xor_sync(0xffffffffu, num, 4);
    if (q == 0 && idx < ne) {
      const float v = __fdiv_rn(num, den[h - h0]);
      vals[idx] = v;
      if (p.ctx) p.ctx[(uint64_t)g * G * HD + e] = v;
    }
  }
  mk_csync();
  if (ne) values_to_runs(vals, ne, nullptr, ph.out_runs, ph.ctx_run0 + g * R + r0, tid, MK_NT);
  mk_arrive(p, ph.arrive_ctr);
  return true;
}

__global__ void __launch_bounds__(MK_THREADS, 1) k_step(const __grid_constant__ MkParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  uint8_t* ring = smem;
  uint8_t* rec = ring + p.ring_bytes;
  float* acc = reinterpret_cast<float*>(rec + p.rec_bytes);
  MkPhase* pdesc = reinterpret_cast<MkPhase*>(reinterpret_cast<uint8_t*>(acc) + ((p.acc_floats * 4 + 127) & ~127u));
  MkPhase* cdesc = pdesc + 2;
  __shared__ __align__(8) uint64_t full[MK_NSLOT], empty[MK_NSLOT], rbar, crecbar[MK_NREC], crecfree[MK_NREC],
      pdbar[2], cdbar[2];
  __shared__ ChunkInfo chunks[GV_MAX_CH];
  __shared__ float red[MK_CWARPS];
  __shared__ unsigned long long kred[MK_CWARPS];
  __shared__ volatile uint32_t flag;
  const uint32_t tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (tid == 0) {
    for (uint32_t s = 0; s < MK_NSLOT; s++) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], MK_CWARPS);
    }
    mbar_init(&rbar, 1);
    for (uint32_t b = 0; b < MK_NREC; b++) {
      mbar_init(&crecbar[b], 1);
      mbar_init(&crecfree[b], MK_CWARPS);
    }
    for (int b = 0; b < 2; b++) {
      mbar_init(&pdbar[b], 1);
      mbar_init(&cdbar[b], 1);
    }
    fence_barrier_init();
  }
  __syncthreads();
  if (warp == MK_CWARPS) {
    if (lane == 0) mk_producer(p, ring, full, empty, pdesc, pdbar);
    return;
  }
  MkCons cs;
  cs.ring = ring;
  cs.full = full;
  cs.empty = empty;
  cs.err = &p.st->error;
  MkRec rr;
  rr.bar = crecbar;
  rr.free = crecfree;
  uint32_t ruse = 0;
  auto fetch_desc = [&](uint32_t k) {  // thread 0
    mbar_expect_tx(&cdbar[k & 1], sizeof(MkPhase));
    bulk_g2s(&cdesc[k & 1], &p.ph[k], sizeof(MkPhase), &cdbar[k & 1], 0ull);
  };
  if (tid == 0) {
    fetch_desc(0);
    if (p.nph > 1) fetch_desc(1);
  }
  bool ok = true;
  uint32_t k = 0;
  for (; k < p.nph && ok; k++) {
    if (tid == 0) flag = 1;
    mk_csync();
    if (!mk_mbar_wait(&cdbar[k & 1], (k >> 1) & 1, cs.err)) flag = 0;
    mk_csync();
    if (flag == 0) {  // block-uniform after the barrier
      ok = false;
      break;
    }
    const MkPhase& ph = cdesc[k & 1];
    Tracer tr;
    if (tid == 0) tr.begin(TR_STEP + (ph.kind == MK_ATTN ? 4 : ph.epilogue), k);
    if (ph.kind == MK_GEMV) {
      ok = mk_gemv(p, ph, cs, rec, acc, &rbar, ruse, rr, chunks, red, kred, &flag, tr);
      if (ok) mk_arrive(p, ph.arrive_ctr);
    } else if (p.hd == 128) {
      ok = p.kv_f16 ? mk_attn<128, __half>(p, ph, cs, rec, &flag, tr) : mk_attn<128, float>(p, ph, cs, rec, &flag, tr);
    } else {
      ok = p.kv_f16 ? mk_attn<64, __half>(p, ph, cs, rec, &flag, tr) : mk_attn<64, float>(p, ph, cs, rec, &flag, tr);
    }
    mk_csync();
    if (tid == 0) {
      tr.mark(4);
      if (tr.r) tr.r->t[5] = cs.waited;  // cumulative ns warp 0 waited for stages
      // every consumer thread is done with this descriptor: refill its buffer
      if (ok && k + 2 < p.nph) {
        fence_proxy_async_smem();
        fetch_desc(k + 2);
      }
    }
  }
  if (!ok) {
    // stopped in phase k - 1 (or waiting for descriptor k): the copies of
    // descriptors k - 1 .. k may still be landing in this CTA's shared memory
    if (tid == 0) {
      atomicCAS(&p.st->error, 0u, 3u);
      const uint32_t k0 = k > 0 ? k - 1 : 0;
      for (uint32_t j = k0; j < k0 + 2 && j < p.nph; j++) mbar_wait(&cdbar[j & 1], (j >> 1) & 1);
    }
    return;
  }
  // the last CTA to finish returns every counter to zero for the next launch
  if (tid == 0) {
    __threadfence();
    if (atomicAdd(p.sync + p.done_ctr, 1u) == gridDim.x - 1) {
      for (uint32_t i = 0; i < p.nsync; i++) p.sync[i] = 0;
      __threadfence();
    }
  }
}
