// Batch execution on warps: every warp of the grid works through its share of
// a batch's chunks straight from HBM, with no staging or hand-off between
// warps.
//
//  * The host cuts each request into chunks and the batch into granules of
//    `gran` consecutive chunks; for every granule it stores the request that
//    owns the granule's first chunk (and that request's first chunk).  Warp g
//    of W takes the contiguous granule range [g G / W, (g + 1) G / W) (no
//    atomics), walks forward through the requests of its granules, and
//    decodes each request's record once.
//  * Aligned elementwise chunks run the vector body (ew_vec: 128-bit loads,
//    up to 8 groups of 4 elements per lane in flight); strided views and
//    reductions run the general warp bodies of executor.cuh.
//  * Completion: in the persistent worker each warp fences its stores, the
//    CTA adds its chunk count to the batch's done counter once, and the CTA
//    that completes the batch posts the completion word; the last CTA to leave
//    the batch marks its payload reusable (retired).  A stream-mode launch of a
//    batch without stage barriers has no such protocol: the event recorded
//    after it completes the batch, and a warp that meets an error posts it.
//  * A batch with stage barriers (a request that depends on an earlier one)
//    hands granules out in order with an atomic instead, counts chunks one by
//    one, and a chunk of a later stage waits (bounded) until every chunk of
//    the earlier stages is done.  Claims in order mean that an earlier stage
//    is always held by a running warp, whether or not the grid is resident.
//
// Every wait is bounded by %globaltimer.
#pragma once
#include "executor.cuh"

namespace gpuos {

static constexpr int kWarpsPerCta = 8;
static constexpr int kCtaThreads = 32 * kWarpsPerCta;
static constexpr int kMinCtasPerSm = 2;

// Stage waits of one CTA share one poller: the warp that takes `poller`
// reads the batch's done counter (acquire) and leaves the largest value seen
// in `seen`; the CTA's other waiting warps watch `seen` in shared memory, so a
// stage hop costs at most one poll round trip and the counter sees one poller
// per CTA instead of one per warp.  Both are zero when a batch starts.
struct StageSync {
  uint32_t seen;
  int32_t poller;
};

struct CtaSmem {
  StageSync ss;              // stage waits (batches with stage barriers)
  ExtRec ext[kWarpsPerCta];  // per warp: the strided request's dims and strides
  BatchHdr hdr;              // persistent worker: the current batch's header
  uint32_t chunks;           // chunks this CTA finished in the current batch
  int32_t go;                // persistent worker: a batch is ready
  uint32_t off;              // persistent worker: its offset in the arena
  uint32_t pad;
};

// The decoded request a warp is working on: the vector view of an aligned
// elementwise request, or just its record for the other kinds (reloaded per
// chunk, which keeps the vector path's registers free).
struct Cur {
  VecView u;
  const Req* rec;
  int v;
  float p0, p1;
  bool vec;
};

// The record carries the operator the request's slot named when it was
// flushed (the host resolves the jump table), and its parameters.  A strided
// (or more-operand) request's ExtRec is copied from the arena to the warp's
// shared-memory slot.
// `words`: the record as load_req_words returned it (loaded ahead of time).
__device__ __forceinline__ void decode(Cur& cur, const Exec& ex, const Req* rec, uint4 words,
                                       ExtRec* xs) {
  const ReqView q = decode_req(words);
  cur.rec = rec;
  cur.v = q.op == kOpNone ? V_NONE : q.op;
  cur.p0 = q.p0;
  cur.p1 = q.p1;
  if ((q.flags & RF_SLOT) && ex.tab) {
    // the persistent worker resolves a slot when it starts the request:
    // alias, then the physical slot's operator and parameters, with acquire
    // loads (the reference's g_op_alias -> g_op_table read,
    // src/persistent_kernel.cu:168-175), so a hot swap reaches batches that
    // are published but not yet started
    const int phys = q.op < kMaxSlots ? ld_acquire_s32(&ex.tab->alias[q.op]) : -1;
    if (phys >= 0 && phys < kMaxSlots) {
      const SlotEntry* e = &ex.tab->slot[phys];
      cur.v = ld_acquire_s32(&e->variant);
      cur.p0 = __int_as_float(ld_acquire_s32(reinterpret_cast<const int32_t*>(&e->p0)));
      cur.p1 = __int_as_float(ld_acquire_s32(reinterpret_cast<const int32_t*>(&e->p1)));
    } else {
      cur.v = V_NONE;
    }
  }
  cur.vec = q.kind == RK_EW && (q.flags & RF_VEC) && !(q.flags & RF_NARY) &&
            q.layout != EL_STRIDED && ew_vec_known(cur.v);
  if (cur.vec) {
    cur.u = vec_view(q);
  } else if ((q.kind == RK_EW && (q.layout == EL_STRIDED || (q.flags & RF_NARY))) ||
             (q.kind == RK_RED && q.layout == RL_GENERIC)) {
    static_assert(sizeof(ExtRec) % 16 == 0, "ExtRec is copied in 16-byte words");
    const uint4* src = reinterpret_cast<const uint4*>(ex.base + q.ext);
    uint4* dst = reinterpret_cast<uint4*>(xs);
    for (uint32_t i = ex.lane; i < sizeof(ExtRec) / 16; i += 32) dst[i] = __ldcg(src + i);
    __syncwarp();
  }
}

template <int BODIES>
__device__ __forceinline__ void run_chunk(const Exec& ex, Cur& cur, uint32_t k,
                                          const ExtRec* xs) {
  if constexpr (!(BODIES & BODY_EW)) cur.vec = false;
  if (cur.vec) {
    if (ex.flags & BF_STAGED) {
      // a scalar operand can be the output of an earlier stage: read it after
      // this chunk's stage wait, not when the record was decoded
      if (cur.u.ma == OM_SCALAR) cur.u.As = ld1(cur.u.a, cur.u.dta, 0);
      if (cur.u.mb == OM_SCALAR && (cur.u.flags & RF_HAS_B)) cur.u.Bs = ld1(cur.u.b, cur.u.dtb, 0);
    }
    const int64_t e0 = (int64_t)k * cur.u.chunk;
    int64_t n = cur.u.numel - e0;
    if (n > (int64_t)cur.u.chunk) n = cur.u.chunk;
    ew_vec_dispatch(cur.v, cur.u, cur.p0, cur.p1, e0, n, ex.lane);
  } else {
    process_chunk<BODIES>(ex, load_req(cur.rec, ex.lane), cur.v, cur.p0, cur.p1, k, xs);
  }
}

// One warp's share of a batch: warp gw of W.  Returns the chunks it ran that
// are still to be counted (all of them, unless the batch counts chunk by chunk).
template <int BODIES = BODY_ALL>
__device__ __forceinline__ uint32_t warp_batch(const Exec& ex, uint32_t gw, uint32_t W,
                                               ExtRec* xs, StageSync* ss) {
  const int lane = ex.lane;
  const uint32_t nchunk = ex.nchunk;
  const bool staged = ex.flags & BF_STAGED;
  const bool dyn = ex.flags & (BF_STAGED | BF_CLAIM);  // granules claimed one at a time
  const uint32_t G = ex.gran;
  const uint32_t ngran = G ? (nchunk + G - 1) / G : 0u;
  auto claim = [&]() -> uint32_t {
    uint32_t x = 0;
    if (lane == 0) x = atomicAdd(&ex.st->claim, 1u);
    return __shfl_sync(GPUOS_FULL, x, 0);
  };
  // Otherwise warp gw takes granules gw, gw + W, gw + 2 W, ...: the warps of
  // a CTA run neighbouring granules, and each warp's share samples the whole
  // batch, which evens out chunks of different costs better than contiguous
  // ranges (measured on the broadcast stream: 0.185 of HBM against 0.119).
  uint32_t j;
  const uint32_t jend = ngran;
  if (dyn) {
    j = claim();
  } else {
    j = gw;
  }
  auto next_of = [&](uint32_t x) -> uint32_t { return x + W < ngran ? x + W : ngran; };
  uint32_t count = 0, waited = 0;
  int r = -1;
  uint32_t rbase = 0, rend = 0;
  Cur cur;
  // granule j's entry, its first request's record words and end, loaded ahead
  uint2 g = make_uint2(0u, 0u);
  uint4 gw_rec = make_uint4(0u, 0u, 0u, 0u);
  uint32_t g_end = 0;
  // static order: the entry of the granule after the next one is loaded an
  // iteration ahead, so that the next granule's record load never waits on it
  uint2 gq = make_uint2(0u, 0u);
  if (j < jend) {
    g = __ldcg(ex.gtab + j);
    if (!dyn) {
      const uint32_t jq = next_of(j);
      if (jq < ngran) gq = __ldcg(ex.gtab + jq);
    }
    gw_rec = load_req_words(ex.recs + g.x, lane);
    g_end = __ldcg(ex.gcb + g.x + 1);
  }
  while (j < jend) {
    const uint32_t jn = dyn ? claim() : next_of(j);  // the next granule, known ahead
    uint2 gn;
    if (dyn) {
      gn = jn < ngran ? __ldcg(ex.gtab + jn) : make_uint2(0u, 0u);
    } else {
      gn = gq;
      const uint32_t jq = jn < ngran ? next_of(jn) : ngran;
      gq = jq < ngran ? __ldcg(ex.gtab + jq) : make_uint2(0u, 0u);
    }
    uint32_t c = j * G;
    const uint32_t cend = min(c + G, nchunk);
    if ((int)g.x != r) {
      r = (int)g.x;
      rbase = g.y;
      rend = g_end;
      decode(cur, ex, ex.recs + r, gw_rec, xs);
    }
    // the next granule's record is in flight while this one runs
    uint4 n_rec = make_uint4(0u, 0u, 0u, 0u);
    uint32_t n_end = 0;
    if (jn < ngran) {
      n_rec = load_req_words(ex.recs + gn.x, lane);
      n_end = __ldcg(ex.gcb + gn.x + 1);
    }
    for (; c < cend; ++c) {
      if (c >= rend) {
        do {
          ++r;
          rbase = rend;
          rend = __ldcg(ex.gcb + r + 1);
        } while (c >= rend);
        decode(cur, ex, ex.recs + r, load_req_words(ex.recs + r, lane), xs);
      }
      if (staged) {
        const uint32_t w = __ldcg(ex.req_wait + r);
        if (w > waited) {
          // every chunk of the earlier stages must be done first
          if (lane == 0) {
            volatile uint32_t* seen = &ss->seen;
            if (*seen < w) {
              const uint64_t t0 = globaltimer();
              while (true) {
                if (atomicCAS(&ss->poller, 0, 1) == 0) {
                  // this warp polls for the CTA
                  const uint32_t d = ld_acquire_u32(&ex.st->done);
                  __threadfence_block();
                  atomicMax(&ss->seen, d);
                  atomicExch(&ss->poller, 0);
                  if (d >= w) break;
                  __nanosleep(32);
                } else {
                  __nanosleep(32);
                }
                if (*seen >= w) break;
                if (globaltimer() - t0 > ex.wait_limit_ns) {
                  atomicOr(&ex.st->err, ERR_STAGE_TIMEOUT);
                  break;
                }
              }
            }
            // order this warp's loads after the acquire another warp may have made
            __threadfence_block();
          }
          waited = w;
          __syncwarp();
        }
      }
      run_chunk<BODIES>(ex, cur, c - rbase, xs);
      if (staged) {
        __threadfence();  // release this chunk's stores before it is counted
        __syncwarp();
        if (lane == 0) {
          const uint32_t d = atomicAdd(&ex.st->done, 1u) + 1u;
          if (d == nchunk) finish_batch(ex);
        }
      } else {
        ++count;
      }
    }
    j = jn;
    g = gn;
    gw_rec = n_rec;
    g_end = n_end;
  }
  return count;
}

// ---- chain batches ---------------------------------------------------------
// A stream-mode batch with stage barriers that is small (a dependent chain of
// small requests, e.g. a decode step at batch 1) runs on one thread-block
// cluster instead of the whole GPU: the cluster's warps split each stage's
// chunks (warp g of W takes chunks g, g + W, ... of the stage), and a cluster
// barrier with release / acquire semantics separates the stages.  A stage hop
// then costs one hardware barrier instead of a fence, an atomic and a polled
// counter in global memory.  Every CTA of the cluster runs every stage, so
// the barrier needs no bound.
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\t"
               "barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

__device__ __forceinline__ uint32_t cluster_size() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_nctarank;" : "=r"(r));
  return r;
}

// The first request of [r0, nreq) whose req_wait differs from r0's (the end
// of r0's stage).
__device__ __forceinline__ uint32_t chain_stage_end(const Exec& ex, uint32_t r0, uint32_t nreq) {
  const uint32_t w0 = __ldcg(ex.req_wait + r0);
  uint32_t r1 = r0 + 1;
  while (r1 < nreq && __ldcg(ex.req_wait + r1) == w0) ++r1;
  return r1;
}

// Returns the chunks this warp ran.  The stages are the runs of requests
// with equal req_wait (their stage's first chunk); requests are in stage
// order.  The batch's records do not depend on the data, so each warp loads
// the record of its first chunk of the next stage before the barrier, and a
// request that is not on the vector path runs from the record words already
// in registers: after a barrier a chunk's first global load is its data.
template <int BODIES>
__device__ __forceinline__ uint32_t chain_batch(const Exec& ex, uint32_t nreq, ExtRec* xs) {
  const uint32_t W = cluster_size() * kWarpsPerCta;
  const uint32_t gw = cluster_rank() * kWarpsPerCta + (threadIdx.x >> 5);
  uint32_t count = 0;
  Cur cur;
  uint32_t r0 = 0, r1 = nreq ? chain_stage_end(ex, 0, nreq) : 0;
  // this warp's first chunk of the stage, its request and record words
  uint32_t cf = 0, rf = 0;
  uint4 wf = make_uint4(0u, 0u, 0u, 0u);
  auto ahead = [&]() {
    cf = __ldcg(ex.gcb + r0) + gw;
    rf = r0;
    if (cf < __ldcg(ex.gcb + r1)) {
      while (__ldcg(ex.gcb + rf + 1) <= cf) ++rf;
      wf = load_req_words(ex.recs + rf, ex.lane);
    }
  };
  if (nreq) ahead();
  while (r0 < nreq) {
    const uint32_t s1 = __ldcg(ex.gcb + r1);
    uint32_t r = rf, rbase = __ldcg(ex.gcb + rf), rend = __ldcg(ex.gcb + rf + 1);
    uint4 words = wf;
    bool have = true;  // `words` are request r's
    int decoded = -1;
    for (uint32_t c = cf; c < s1; c += W) {
      while (c >= rend) {
        ++r;
        rbase = rend;
        rend = __ldcg(ex.gcb + r + 1);
        have = false;
      }
      if ((int)r != decoded) {
        if (!have) words = load_req_words(ex.recs + r, ex.lane);
        have = true;
        decode(cur, ex, ex.recs + r, words, xs);
        decoded = (int)r;
      }
      if constexpr ((BODIES & BODY_EW) != 0) {
        if (cur.vec) {
          run_chunk<BODIES>(ex, cur, c - rbase, xs);
          ++count;
          continue;
        }
      }
      process_chunk<BODIES>(ex, decode_req(words), cur.v, cur.p0, cur.p1, c - rbase, xs);
      ++count;
    }
    r0 = r1;
    if (r0 < nreq) {
      r1 = chain_stage_end(ex, r0, nreq);
      ahead();
    }
    cluster_sync_all();
  }
  return count;
}

// All threads of the CTA, after warp_batch: count the CTA's chunks into the
// batch (completing it if they are the last), then leave the batch.  The last
// of `nctas` CTAs to leave zeroes the batch's counters for the slot's next use
// and, in the persistent worker, marks the payload reusable (retired); a
// stream-mode payload is reusable once its kernel has completed.
__device__ __forceinline__ void cta_leave_batch(const Exec& ex, uint32_t* cta_chunks,
                                                uint32_t count, uint32_t nctas,
                                                volatile uint64_t* retired_ring) {
  __threadfence();  // each warp releases its stores
  if (ex.lane == 0 && count) atomicAdd(cta_chunks, count);
  __syncthreads();
  if (threadIdx.x == 0) {
    const uint32_t add = *cta_chunks;
    *cta_chunks = 0;
    if (add) {
      const uint32_t d = atomicAdd(&ex.st->done, add) + add;
      if (d == ex.nchunk) finish_batch(ex);
    }
    __threadfence();
    const uint32_t left = atomicAdd(&ex.st->ctas_left, 1u) + 1u;
    if (left == nctas) {
      __threadfence();
      ex.st->claim = 0;
      ex.st->done = 0;
      ex.st->err = 0;
      ex.st->nt0 = 0;
      ex.st->ctas_left = 0;
      if (retired_ring) st_release_sys_u64(&retired_ring[ex.seq % kDoneRing], ex.seq + 1);
    }
  }
  __syncthreads();
}

// Thread 0, before a batch with BF_AFTER_PREV: wait (bounded) until every
// batch in [wait_from, seq) has completed.
__device__ __forceinline__ void wait_prev_batches(const Exec& ex) {
  const uint64_t t0 = globaltimer();
  for (uint64_t j = ex.wait_from; j < ex.seq; ++j) {
    while ((ld_acquire_u64(&ex.done_dev[j % kDoneRing]) & ((1ull << 48) - 1)) != j + 1) {
      __nanosleep(256);
      if (globaltimer() - t0 > ex.wait_limit_ns) {
        atomicOr(&ex.st->err, ERR_STAGE_TIMEOUT);
        return;
      }
    }
  }
}

}  // namespace gpuos
