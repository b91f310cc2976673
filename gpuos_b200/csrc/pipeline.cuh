// CTA pipeline of the batch executor: one producer warp stages work, eight
// consumer warps compute it.
//
//  producer (warp 0)  works through its granules of the current batch, eight
//                     chunks a round, one chunk per lane: each lane decodes its
//                     chunk's request record and fills one shared-memory
//                     stage.  For an aligned elementwise chunk it copies the
//                     contiguous operand ranges into the stage with
//                     cp.async.bulk (the SM's copy engine: no registers or
//                     threads tied up while the bytes are in flight).  Other
//                     chunks (strided views, reductions) are handed over as
//                     (request, chunk) for a consumer warp to run from HBM.
//  consumers (1..8)   each takes the next stage in ring order (a shared
//                     counter), waits on its mbarrier, computes it and stores
//                     straight to HBM, then releases the stage.  Eight stages
//                     are computed at once, one per warp, while the rest land.
//
// With 12 stages of 16 KB, up to ~190 KB of operands per SM are in flight.
// Every wait is bounded by %globaltimer; on expiry the CTA records an error,
// lets its bulk copies land and exits.  No copy uses cluster multicast.
#pragma once
#include "executor.cuh"

namespace gpuos {

static constexpr int kConsumers = 8;                 // consumer warps per CTA
static constexpr int kStages = 12;                   // shared-memory stages
static constexpr int kUnit = 2048;                   // elements per staged chunk
static constexpr int kStageBytes = 8192;             // bytes per staged operand
static constexpr int kCtaThreads = 32 * (1 + kConsumers);

enum StageType : uint32_t { ST_VEC = 1, ST_CHUNK = 2, ST_END = 3, ST_STOP = 4 };
enum OperandMode : int32_t { OM_STAGED = 0, OM_LINEAR = 1, OM_ROW = 2, OM_ROWSPLAT = 3, OM_SCALAR = 4 };

struct alignas(16) StageHdr {
  uint32_t type;
  uint32_t nchunk;       // chunks to add to the batch's done count when the stage completes
  uint32_t c;            // ST_CHUNK: chunk index within its request
  int32_t r;             // ST_CHUNK: request index
  const uint8_t* payload;
  uint64_t seq;          // batch of the stage (payload memory is reused across batches)
  // ST_VEC
  uint64_t a, b, o;
  int64_t e0, n;
  int64_t inner, sa_row, sb_row, so_row;
  int32_t v, flags, dta, dtb, dto, ma, mb, mo;
  float p0, p1;
  uint32_t fdiv_m, fdiv_s, na, nb;  // na/nb: elements staged in shared memory
};

struct PipeSmem {
  StageHdr hdr[kStages];
  uint64_t full[kStages];
  uint64_t empty[kStages];
  uint32_t sdone[kStages];  // per slot: 1 + index of the last stage completed in it
  uint32_t take;            // next stage index a consumer warp takes
  int32_t abort;
  int32_t pad[2];
  Tables tab;
};

// dynamic shared memory: PipeSmem, then kStages x (A, B) operand buffers
__host__ __device__ constexpr size_t pipe_buf_offset() {
  return (sizeof(PipeSmem) + 127) / 128 * 128;
}
__host__ __device__ constexpr size_t pipe_smem_bytes() {
  return pipe_buf_offset() + (size_t)kStages * 2 * kStageBytes;
}

// ---- PTX wrappers ------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ uint32_t lds_acquire_u32(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.cta.shared::cta.u32 %0, [%1];" : "=r"(v) : "r"(smem_u32(p)) : "memory");
  return v;
}

__device__ __forceinline__ void sts_release_u32(uint32_t* p, uint32_t v) {
  asm volatile("st.release.cta.shared::cta.u32 [%0], %1;" ::"r"(smem_u32(p)), "r"(v) : "memory");
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_fence_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  uint64_t state;
  asm volatile("mbarrier.arrive.shared::cta.b64 %0, [%1];" : "=l"(state) : "r"(smem_u32(bar)) : "memory");
  (void)state;
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  uint64_t state;
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 %0, [%1], %2;"
               : "=l"(state) : "r"(smem_u32(bar)), "r"(bytes) : "memory");
  (void)state;
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok) : "r"(smem_u32(bar)), "r"(parity) : "memory");
  return ok != 0;
}

// Bounded wait on one phase of an mbarrier; false on timeout or abort.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, uint64_t limit_ns,
                                          volatile int32_t* abort) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer();
  unsigned ns = 32;
  while (!mbar_try_wait(bar, parity)) {
    if (*abort) return false;
    if (globaltimer() - t0 > limit_ns) return false;
    __nanosleep(ns);
    if (ns < 256) ns <<= 1;
  }
  return true;
}

// bulk global -> shared copy completing on `bar` (no multicast)
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
      ::"r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// order earlier generic-proxy writes to global memory (made visible to this
// thread by an acquire) before later bulk copies read them
__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}

// ---- shared-memory operand loads ---------------------------------------------
__device__ __forceinline__ void lds4(const uint8_t* buf, int dt, int64_t i, float* v) {
  if (dt == kF32) {
    const float4 x = *reinterpret_cast<const float4*>(buf + i * 4);
    v[0] = x.x; v[1] = x.y; v[2] = x.z; v[3] = x.w;
  } else {
    const uint2 u = *reinterpret_cast<const uint2*>(buf + i * 2);
    if (dt == kF16) {
      float2 f = __half22float2(*reinterpret_cast<const __half2*>(&u.x));
      v[0] = f.x; v[1] = f.y;
      f = __half22float2(*reinterpret_cast<const __half2*>(&u.y));
      v[2] = f.x; v[3] = f.y;
    } else {
      bf2_to_f(u.x, v[0], v[1]);
      bf2_to_f(u.y, v[2], v[3]);
    }
  }
}

__device__ __forceinline__ float lds1(const uint8_t* buf, int dt, int64_t i) {
  if (dt == kF32) return reinterpret_cast<const float*>(buf)[i];
  if (dt == kF16) return __half2float(reinterpret_cast<const __half*>(buf)[i]);
  return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(buf)[i]);
}

// ---- consumer side of a staged elementwise chunk ------------------------------
struct UnitView {
  uint64_t a, b, o;
  int64_t e0, n, inner, sa_row, sb_row, so_row;
  int ma, mb, mo, dta, dtb, dto, flags;
  float As, Bs;
  uint32_t fdiv_m, fdiv_s, na, nb;
};

__device__ __forceinline__ int64_t unit_row(const UnitView& u, int64_t e) {
  if (u.flags & RF_BIG) return e / u.inner;
  return (int64_t)fdiv_u32((uint32_t)e, u.fdiv_m, u.fdiv_s);
}

// 4 values of one operand for the group at unit index i (linear element e)
__device__ __forceinline__ void unit_opnd4(int mode, const uint8_t* buf, int64_t nstaged,
                                           uint64_t p, int dt, float sc, int64_t i, int64_t e,
                                           int64_t rowoff, int64_t c, float* v) {
  if (mode == OM_STAGED && i + 4 <= nstaged) {
    lds4(buf, dt, i, v);
  } else if (mode == OM_STAGED || mode == OM_LINEAR) {
    ld4(p, dt, e, v);
  } else if (mode == OM_ROW) {
    ld4(p, dt, rowoff + c, v);
  } else if (mode == OM_ROWSPLAT) {
    const float x = ld1(p, dt, rowoff);
#pragma unroll
    for (int k = 0; k < 4; ++k) v[k] = x;
  } else {
#pragma unroll
    for (int k = 0; k < 4; ++k) v[k] = sc;
  }
}

__device__ __forceinline__ float unit_opnd1(int mode, const uint8_t* buf, int64_t nstaged,
                                            uint64_t p, int dt, float sc, int64_t i, int64_t e,
                                            int64_t rowoff, int64_t c) {
  if (mode == OM_STAGED && i < nstaged) return lds1(buf, dt, i);
  if (mode == OM_STAGED || mode == OM_LINEAR) return ld1(p, dt, e);
  if (mode == OM_ROW) return ld1(p, dt, rowoff + c);
  if (mode == OM_ROWSPLAT) return ld1(p, dt, rowoff);
  return sc;
}

// The 32 lanes of one consumer warp split the unit into groups of 4.
template <int V>
__device__ __forceinline__ void unit_vec(const UnitView& u, const uint8_t* bufA,
                                         const uint8_t* bufB, float p0, float p1, int L) {
  const bool rows = (u.ma == OM_ROW || u.ma == OM_ROWSPLAT || u.mb == OM_ROW ||
                     u.mb == OM_ROWSPLAT || u.mo != 0);
  for (int64_t i = 4 * (int64_t)L; i < u.n; i += 4 * 32) {
    const int64_t e = u.e0 + i;
    if (i + 4 <= u.n) {
      int64_t r = 0, c = e;
      if (rows) {
        r = unit_row(u, e);
        c = e - r * u.inner;
      }
      float A[4], B[4], R[4];
      unit_opnd4(u.ma, bufA, u.na, u.a, u.dta, u.As, i, e, r * u.sa_row, c, A);
      unit_opnd4(u.mb, bufB, u.nb, u.b, u.dtb, u.Bs, i, e, r * u.sb_row, c, B);
      op4<V>(A, B, R, p0, p1);
      st4(u.o, u.dto, u.mo ? r * u.so_row + c : e, R);
    } else {
      // ragged end of a contiguous request: fewer than 4 elements
      for (int64_t k = 0; k < u.n - i; ++k) {
        const int64_t ek = e + k, ik = i + k;
        int64_t r = 0, c = ek;
        if (rows) {
          r = unit_row(u, ek);
          c = ek - r * u.inner;
        }
        const float A = unit_opnd1(u.ma, bufA, u.na, u.a, u.dta, u.As, ik, ek, r * u.sa_row, c);
        const float B = unit_opnd1(u.mb, bufB, u.nb, u.b, u.dtb, u.Bs, ik, ek, r * u.sb_row, c);
        st1(u.o, u.dto, u.mo ? r * u.so_row + c : ek, op1<V>(A, B, p0, p1));
      }
    }
  }
}

#define GPUOS_UNIT_CASE(V) case V: unit_vec<V>(u, bufA, bufB, p0, p1, L); return;

__device__ __forceinline__ void unit_dispatch(int v, const UnitView& u, const uint8_t* bufA,
                                              const uint8_t* bufB, float p0, float p1, int L) {
  switch (v) {
    GPUOS_ALL_EW(GPUOS_UNIT_CASE)
    GPUOS_JIT_UNIT_CASES
    default: return;
  }
}

// ---- producer helpers ------------------------------------------------------------
__device__ __forceinline__ int resolve_smem(const ReqView& q, const Tables& tab, float& p0,
                                            float& p1) {
  p0 = q.p0;
  p1 = q.p1;
  if (!(q.flags & RF_SLOT)) return q.op;
  const int s = q.op;
  if (s < 0 || s >= kMaxSlots) return V_NONE;
  const int phys = tab.alias[s];
  if (phys < 0 || phys >= kMaxSlots) return V_NONE;
  p0 = tab.slot[phys].p0;
  p1 = tab.slot[phys].p1;
  return tab.slot[phys].variant;
}

__device__ __forceinline__ int esz_of(int dt) { return dt == kF32 ? 4 : 2; }

// Everything the producer warp of one CTA needs while it works through
// batches.  All 32 lanes hold the same copy: `it` and `dead` change only in
// warp-uniform code.
struct Producer {
  PipeSmem* sm;
  uint8_t* bufs;
  uint64_t seq;           // batch being produced
  uint32_t it;            // stages published so far
  uint64_t limit_ns;      // bound of every wait
  bool dead;              // a wait expired: stop producing
};

// Bounded wait until the consumers released the previous use of stage `it`.
__device__ __forceinline__ bool wait_stage_free(PipeSmem* sm, uint32_t it, uint64_t limit_ns) {
  const uint32_t use = it / kStages;
  if (use == 0) return true;
  return mbar_wait(&sm->empty[it % kStages], (use - 1) & 1u, limit_ns, &sm->abort);
}

// A header-only stage (END, STOP) published by lane 0; warp-uniform.
__device__ __forceinline__ void publish_plain_warp(Producer& P, uint32_t type, uint32_t nchunk,
                                                   const uint8_t* payload, int lane) {
  if (P.dead) return;
  uint32_t ok = 1;
  if (lane == 0) {
    ok = wait_stage_free(P.sm, P.it, P.limit_ns) ? 1u : 0u;
    if (ok) {
      StageHdr& H = P.sm->hdr[P.it % kStages];
      H.type = type;
      H.nchunk = nchunk;
      H.payload = payload;
      H.seq = P.seq;
      mbar_arrive(&P.sm->full[P.it % kStages]);
    } else {
      P.sm->abort = 1;
    }
  }
  ok = __shfl_sync(GPUOS_FULL, ok, 0);
  if (ok) ++P.it;
  else P.dead = true;
}

// Fill stage `it` (already free) with one aligned elementwise chunk: the
// header plus bulk copies of the contiguous operand ranges into the stage's
// buffers.  Called by one lane per stage.
__device__ __forceinline__ void fill_vec(Producer& P, uint32_t it, const uint8_t* payload,
                                         const ReqView& q, int v, float p0, float p1,
                                         uint32_t k, bool count_now) {
  const int s = (int)(it % kStages);
  StageHdr& H = P.sm->hdr[s];
  const bool row2d = q.layout == EL_ROW2D;
  const bool hasb = q.flags & RF_HAS_B;
  const int64_t e0 = (int64_t)k * q.chunk;
  int64_t n = q.numel - e0;
  if (n > (int64_t)q.chunk) n = q.chunk;
  auto mode = [&](bool scalar, int64_t srow, int64_t sin) -> int {
    if (scalar) return OM_SCALAR;
    if (!row2d) return OM_LINEAR;
    if (sin == 0) return OM_ROWSPLAT;
    return srow == q.inner ? OM_LINEAR : OM_ROW;
  };
  int ma = mode(q.flags & RF_A_SCALAR, q.sa_row, q.sa_in);
  int mb = hasb ? mode(q.flags & RF_B_SCALAR, q.sb_row, q.sb_in) : OM_SCALAR;
  uint8_t* bufA = P.bufs + (size_t)s * 2 * kStageBytes;
  uint8_t* bufB = bufA + kStageBytes;
  uint32_t na = 0, nb = 0, bytes = 0;
  const uint8_t* srcA = nullptr;
  const uint8_t* srcB = nullptr;
  if (ma == OM_LINEAR) {
    const int es = esz_of(q.dta);
    srcA = reinterpret_cast<const uint8_t*>(q.a) + e0 * es;
    const uint32_t bb = (uint32_t)((n * es) & ~(int64_t)15);
    if ((reinterpret_cast<uint64_t>(srcA) & 15) == 0 && bb > 0 && bb <= kStageBytes) {
      ma = OM_STAGED;
      na = bb / es;
      bytes += bb;
    }
  }
  if (mb == OM_LINEAR) {
    const int es = esz_of(q.dtb);
    srcB = reinterpret_cast<const uint8_t*>(q.b) + e0 * es;
    const uint32_t bb = (uint32_t)((n * es) & ~(int64_t)15);
    if ((reinterpret_cast<uint64_t>(srcB) & 15) == 0 && bb > 0 && bb <= kStageBytes) {
      mb = OM_STAGED;
      nb = bb / es;
      bytes += bb;
    }
  }
  H.type = ST_VEC;
  H.nchunk = count_now ? 1u : 0u;
  H.payload = payload;
  H.seq = P.seq;
  H.a = q.a;
  H.b = q.b;
  H.o = q.o;
  H.e0 = e0;
  H.n = n;
  H.inner = q.inner;
  H.sa_row = q.sa_row;
  H.sb_row = q.sb_row;
  H.so_row = q.so_row;
  H.v = v;
  H.flags = q.flags;
  H.dta = q.dta;
  H.dtb = q.dtb;
  H.dto = q.dto;
  H.ma = ma;
  H.mb = mb;
  H.mo = (!row2d || q.so_row == q.inner) ? 0 : 1;
  H.p0 = p0;
  H.p1 = p1;
  H.fdiv_m = q.fdiv_m;
  H.fdiv_s = q.fdiv_s;
  H.na = na;
  H.nb = nb;
  if (bytes) {
    mbar_arrive_expect_tx(&P.sm->full[s], bytes);
    if (na) bulk_g2s(bufA, srcA, na * esz_of(q.dta), &P.sm->full[s]);
    if (nb) bulk_g2s(bufB, srcB, nb * esz_of(q.dtb), &P.sm->full[s]);
  } else {
    mbar_arrive(&P.sm->full[s]);
  }
}

// Chunks one round of the producer warp handles (one per lane and stage).  A
// round publishes at most kRound stages, fewer than kStages, so that every
// lane of a round waits on a different stage.
static constexpr uint32_t kRound = 8;
static_assert(kRound < (uint32_t)kStages, "round size");

// The producer warp works through one batch in granules of `gran` consecutive
// chunks.  The host stores, per granule, the request that owns its first
// chunk.  Each round, lane l takes chunk c0 + l: the lanes find their
// requests from the chunk prefix of the (at most kRound + 1) requests that
// follow, decode their records and fill stage it + l in parallel.
// Without stage barriers CTA b takes granules b, b + nctas, ... (no atomics;
// the next granule's entry is loaded ahead).  A batch with stage barriers
// hands granules out in order with an atomic instead, so that an earlier
// stage is always held by a running CTA.
__device__ void produce_batch(Producer& P, const uint8_t* payload, const Tables* jtab,
                              const uint64_t* done_dev, uint32_t cta, uint32_t nctas, int lane) {
  PipeSmem* sm = P.sm;
  const BatchHdr* h = reinterpret_cast<const BatchHdr*>(payload);
  BatchState* st = reinterpret_cast<BatchState*>(const_cast<uint8_t*>(payload) + sizeof(BatchHdr));
  const uint32_t nreq = __ldcg(&h->nreq);
  const uint32_t nchunk = __ldcg(&h->nchunk);
  const uint32_t flags = __ldcg(&h->flags);
  P.seq = __ldcg(&h->seq);
  if ((flags & BF_AFTER_PREV) && done_dev && lane == 0) {
    // a hazard with an earlier batch: wait (bounded) until every batch in
    // [wait_from, seq) has completed
    const uint64_t seq = P.seq;
    const uint64_t t0 = globaltimer();
    for (uint64_t j = __ldcg(&h->wait_from); j < seq; ++j) {
      while ((ld_acquire_u64(&done_dev[j % kDoneRing]) & ((1ull << 48) - 1)) != j + 1) {
        __nanosleep(256);
        if (globaltimer() - t0 > P.limit_ns) {
          atomicOr(&st->err, ERR_STAGE_TIMEOUT);
          break;
        }
      }
    }
  }
  {
    const uint4* tsrc = reinterpret_cast<const uint4*>(jtab);
    uint4* tdst = reinterpret_cast<uint4*>(&sm->tab);
    constexpr uint32_t kTab16 = sizeof(Tables) / 16;
#pragma unroll
    for (uint32_t i0 = 0; i0 < kTab16; i0 += 32) {
      if (i0 + lane < kTab16) tdst[i0 + lane] = __ldcg(tsrc + i0 + lane);
    }
  }
  __syncwarp();
  fence_proxy_async_global();
  const bool staged = flags & BF_STAGED;
  const Req* recs = reinterpret_cast<const Req*>(payload + __ldcg(&h->rec_off));
  const uint32_t* gcb = reinterpret_cast<const uint32_t*>(payload + __ldcg(&h->cb_off));
  const uint32_t* grq = reinterpret_cast<const uint32_t*>(payload + __ldcg(&h->gtab_off));
  const uint32_t G = __ldcg(&h->gran);
  const uint32_t ngran = G ? (nchunk + G - 1) / G : 0u;
  const uint32_t* req_wait = staged ? grq + ngran : nullptr;
  const uint32_t lt = (1u << lane) - 1u;
  auto next_granule = [&](uint32_t j) -> uint32_t {
    uint32_t x = 0;
    if (staged) {
      if (lane == 0) x = atomicAdd(&st->claim, 1u);
      return __shfl_sync(GPUOS_FULL, x, 0);
    }
    return j + nctas;
  };
  uint32_t issued = 0, waited = 0;
  uint32_t j = staged ? next_granule(0) : cta;
  if (j == 0 && lane == 0) st->t_first = globaltimer();
  uint32_t jr = j < ngran ? __ldcg(grq + j) : 0u;
  while (j < ngran && !P.dead) {
    uint32_t c0 = j * G;
    const uint32_t gend = min(c0 + G, nchunk);
    uint32_t r0 = jr;
    const uint32_t jn = next_granule(j);
    const uint32_t jnr = jn < ngran ? __ldcg(grq + jn) : 0u;
    while (c0 < gend && !P.dead) {
      const uint32_t cnt = min(gend - c0, kRound);
      // the chunk prefix of requests r0 .. r0 + kRound: lane m holds the first
      // chunk and the end of request r0 + m
      uint32_t s = 0, e = 0xffffffffu;
      if (lane <= (int)kRound && r0 + lane < nreq) {
        s = __ldcg(gcb + r0 + lane);
        e = __ldcg(gcb + r0 + lane + 1);
      }
      // lane l <= kRound: chunk c0 + l belongs to request r0 + m (m <= l, as
      // every request of a batch has at least one chunk)
      const uint32_t c = c0 + lane;
      uint32_t m = 0;
#pragma unroll
      for (int i = 0; i <= (int)kRound; ++i) m += __shfl_sync(GPUOS_FULL, e, i) <= c ? 1u : 0u;
      m = min(m, kRound);
      const uint32_t r = r0 + m;
      const uint32_t k = c - __shfl_sync(GPUOS_FULL, s, (int)m);
      uint32_t take = cnt;
      uint32_t w = 0;
      if (staged && lane < (int)cnt) w = __ldcg(req_wait + r);
      if (staged) {
        // a chunk of a later stage waits until the earlier stage is done
        uint32_t d = 0;
        if (lane == 0) d = ld_acquire_u32(&st->done);
        d = __shfl_sync(GPUOS_FULL, d, 0);
        const uint32_t blocked =
            __ballot_sync(GPUOS_FULL, lane < (int)cnt && w > waited && d < w);
        if (blocked) {
          const int f = __ffs(blocked) - 1;
          if (f == 0) {
            const uint32_t w0 = __shfl_sync(GPUOS_FULL, w, 0);
            if (lane == 0) {
              const uint64_t t0 = globaltimer();
              while (ld_acquire_u32(&st->done) < w0) {
                __nanosleep(128);
                if (globaltimer() - t0 > P.limit_ns) {
                  atomicOr(&st->err, ERR_STAGE_TIMEOUT);
                  break;
                }
              }
            }
            waited = w0;
            __syncwarp();
            fence_proxy_async_global();
            continue;
          }
          take = (uint32_t)f;
        }
      }
      const bool act = lane < (int)take;
      ReqView q;
      int v = V_NONE;
      float p0 = 0.f, p1 = 0.f;
      if (act) {
        q = load_req(recs + r);
        v = resolve_smem(q, sm->tab, p0, p1);
      }
      const bool vec = act && q.kind == RK_EW && (q.flags & RF_VEC) && q.layout != EL_STRIDED &&
                       ew_known(v);
      // lane l fills stage P.it + l
      const uint32_t its = P.it + (uint32_t)lane;
      bool ok = true;
      if (act) {
        ok = wait_stage_free(sm, its, P.limit_ns);
        if (ok && vec) {
          fill_vec(P, its, payload, q, v, p0, p1, k, staged);
        } else if (ok) {
          StageHdr& H = sm->hdr[its % kStages];
          H.type = ST_CHUNK;
          H.nchunk = staged ? 1u : 0u;
          H.c = k;
          H.r = (int32_t)r;
          H.payload = payload;
          H.seq = P.seq;
          mbar_arrive(&sm->full[its % kStages]);
        }
      }
      if (__any_sync(GPUOS_FULL, !ok)) {
        P.dead = true;
        if (lane == 0) sm->abort = 1;
        break;
      }
      P.it += take;
      issued += take;
      // lane `take` found the request of the round's next chunk
      r0 = __shfl_sync(GPUOS_FULL, r, (int)take);
      c0 += take;
    }
    j = jn;
    jr = jnr;
  }
  // end-of-batch marker: the consumers count this CTA's chunks (unless they
  // were counted stage by stage) and count the CTA out of the batch
  publish_plain_warp(P, ST_END, staged ? 0u : issued, payload, lane);
}

// Producer exit (warp-uniform): publish one STOP per consumer warp; if a wait
// expired, let the copies in flight land (bounded) before the CTA leaves.
__device__ __forceinline__ void produce_stop(Producer& P, int lane) {
  for (int i = 0; i < kConsumers; ++i) publish_plain_warp(P, ST_STOP, 0u, nullptr, lane);
  if (!P.dead || lane != 0) return;
  const uint32_t from = P.it > (uint32_t)kStages ? P.it - kStages : 0u;
  for (uint32_t j = from; j < P.it; ++j) {
    volatile int32_t never = 0;
    mbar_wait(&P.sm->full[j % kStages], (j / kStages) & 1u, P.limit_ns, &never);
  }
}

// Bounded wait until every stage before `it` of this CTA has completed.
// Stages before it - kStages + 1 completed before their slots were reused.
__device__ __forceinline__ bool wait_earlier_stages(PipeSmem* sm, uint32_t it,
                                                    uint64_t limit_ns) {
  const uint32_t from = it > (uint32_t)kStages - 1u ? it - ((uint32_t)kStages - 1u) : 0u;
  const uint64_t t0 = globaltimer();
  for (uint32_t j = from; j < it; ++j) {
    while (lds_acquire_u32(&sm->sdone[j % kStages]) < j + 1u) {
      if (sm->abort || globaltimer() - t0 > limit_ns) return false;
      __nanosleep(64);
    }
  }
  return true;
}

// A consumer warp: take the next stage (in ring order) until a STOP.
__device__ void consume(PipeSmem* sm, uint8_t* bufs, const Tables* gtab,
                        volatile uint64_t* done_ring, uint64_t* done_dev,
                        volatile uint64_t* retired_ring, uint32_t nctas, uint64_t limit_ns) {
  const int lane = threadIdx.x & 31;
  const uint8_t* cur = nullptr;
  uint64_t cur_seq = ~0ull;
  Exec ex;
  for (;;) {
    uint32_t it = 0;
    if (lane == 0) it = atomicAdd(&sm->take, 1u);
    it = __shfl_sync(GPUOS_FULL, it, 0);
    const int s = (int)(it % kStages);
    // A warp can take stage it before the slot's previous use (it - kStages)
    // was even published; a parity wait would then see that older phase as
    // complete.  Wait for the previous use to finish first.
    if (it >= (uint32_t)kStages) {
      uint32_t ok = 1;
      if (lane == 0) {
        const uint64_t t0 = globaltimer();
        while (lds_acquire_u32(&sm->sdone[s]) < it - (uint32_t)kStages + 1u) {
          if (sm->abort || globaltimer() - t0 > limit_ns) {
            ok = 0;
            break;
          }
          __nanosleep(64);
        }
      }
      if (!__shfl_sync(GPUOS_FULL, ok, 0)) {
        sm->abort = 1;
        return;
      }
    }
    if (!mbar_wait(&sm->full[s], (it / kStages) & 1u, limit_ns, &sm->abort)) {
      sm->abort = 1;
      return;
    }
    const StageHdr& H = sm->hdr[s];
    const uint32_t type = H.type;
    if (type == ST_STOP) return;
    const uint8_t* payload = H.payload;
    if (payload != cur || H.seq != cur_seq) {
      ex = bind_batch(payload, gtab, done_ring, done_dev, limit_ns);
      cur = payload;
      cur_seq = H.seq;
    }
    const uint32_t add = H.nchunk;
    if (type == ST_VEC) {
      UnitView u;
      u.a = H.a; u.b = H.b; u.o = H.o;
      u.e0 = H.e0; u.n = H.n; u.inner = H.inner;
      u.sa_row = H.sa_row; u.sb_row = H.sb_row; u.so_row = H.so_row;
      u.ma = H.ma; u.mb = H.mb; u.mo = H.mo;
      u.dta = H.dta; u.dtb = H.dtb; u.dto = H.dto; u.flags = H.flags;
      u.fdiv_m = H.fdiv_m; u.fdiv_s = H.fdiv_s; u.na = H.na; u.nb = H.nb;
      u.As = u.ma == OM_SCALAR ? ld1(u.a, u.dta, 0) : 0.f;
      u.Bs = (u.mb == OM_SCALAR && (u.flags & RF_HAS_B)) ? ld1(u.b, u.dtb, 0) : 0.f;
      const uint8_t* bufA = bufs + (size_t)s * 2 * kStageBytes;
      unit_dispatch(H.v, u, bufA, bufA + kStageBytes, H.p0, H.p1, lane);
    } else if (type == ST_CHUNK) {
      const ReqView q = load_req(ex.recs + H.r);
      process_chunk(ex, q, H.c);
    } else if (type == ST_END) {
      // this CTA leaves the batch once all its earlier stages are done; it
      // counts the chunks it issued (unless they were counted stage by stage)
      const bool ok = lane == 0 ? wait_earlier_stages(sm, it, limit_ns) : true;
      if (!__all_sync(GPUOS_FULL, ok)) {
        if (lane == 0) {
          atomicOr(&ex.st->err, ERR_STAGE_TIMEOUT);
          sm->abort = 1;
        }
        return;
      }
      if (lane == 0) {
        __threadfence();  // release the CTA's stores (observed through sdone)
        if (add) {
          const uint32_t d = atomicAdd(&ex.st->done, add) + add;
          if (d == ex.nchunk) finish_batch(ex);
        }
        __threadfence();
        const uint32_t left = atomicAdd(&ex.st->ctas_left, 1u) + 1u;
        if (left == nctas && retired_ring) {
          __threadfence_system();
          const uint64_t seq = ex.seq;
          st_release_sys_u64(&retired_ring[seq % kDoneRing], seq + 1);
        }
      }
    }
    if (add && type != ST_END) {
      // counted stage by stage (batches with stage barriers)
      __threadfence();
      __syncwarp();
      if (lane == 0) {
        const uint32_t d = atomicAdd(&ex.st->done, add) + add;
        if (d == ex.nchunk) finish_batch(ex);
      }
    }
    __syncwarp();
    if (lane == 0) {
      sts_release_u32(&sm->sdone[s], it + 1u);
      mbar_arrive(&sm->empty[s]);
    }
  }
}

// Shared-memory setup of a pipeline CTA.
__device__ __forceinline__ PipeSmem* pipe_init(uint8_t* smem) {
  PipeSmem* sm = reinterpret_cast<PipeSmem*>(smem);
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&sm->full[s], 1);
      mbar_init(&sm->empty[s], 1);
      sm->sdone[s] = 0;
    }
    sm->take = 0;
    sm->abort = 0;
    mbar_fence_init();
  }
  __syncthreads();
  return sm;
}

}  // namespace gpuos
