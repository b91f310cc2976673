// Batch executor building blocks: request records, jump-table resolution,
// and the per-warp chunk processors (strided elementwise, reductions).  The
// CTA pipeline that feeds them, and the staged vector path, are in
// pipeline.cuh.
//
// Replaces the reference's op_batch (src/persistent_kernel.cu:81-112), which
// walks the sub-tasks of a 512-task shard one after another inside a single
// CTA with int64 div/mod index math per element, and the NVRTC operators of
// pytorch_ext/gpuos_ext.cpp:625-679 (elementwise) and 726-806 (reduce), which
// run one request per CTA.  Here every request is split into chunks and the
// chunks of a batch are spread over every SM.
//
// Chunks that are not staged through shared memory (misaligned views,
// arbitrary strides up to 8 dims, reductions) run here, one warp per chunk.
// A request record is decoded from eight 16-byte loads straight into
// registers.
//
// Compiled by nvcc into the library and by NVRTC for custom expressions.
#pragma once
#include "gpuos_abi.h"
#include "ops.cuh"

namespace gpuos {

#define GPUOS_FULL 0xffffffffu

#ifndef GPUOS_JIT_KNOWN
#define GPUOS_JIT_KNOWN(v) false
#endif
#ifndef GPUOS_JIT_UNIT_CASES
#define GPUOS_JIT_UNIT_CASES
#endif

__device__ __forceinline__ bool ew_known(int v) {
  return (v >= 0 && v < V_NUM_EW) || GPUOS_JIT_KNOWN(v);
}

__device__ __forceinline__ uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint32_t ld_acquire_u32(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ uint64_t ld_acquire_u64(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ uint64_t ld_acquire_sys_u64(const volatile uint64_t* p) {
  uint64_t v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_release_sys_u64(volatile uint64_t* p, uint64_t v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__device__ __forceinline__ void st_release_gpu_u64(uint64_t* p, uint64_t v) {
  asm volatile("st.release.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

// n / d for n < 2^31 with a precomputed multiplier (Granlund & Montgomery,
// "Division by invariant integers using multiplication", PLDI 1994).
__device__ __forceinline__ uint32_t fdiv_u32(uint32_t n, uint32_t m, uint32_t s) {
  return (__umulhi(n, m) + n) >> s;
}

// A request record in registers (fields as in struct Req).
struct ReqView {
  uint64_t a, b, o;
  int64_t numel, inner, sa_row, sb_row, so_row, sa_in, sb_in;
  uint32_t chunk, nseg, ext, part, cnt, fdiv_m, fdiv_s, rg;
  int op, kind, layout, dta, dtb, dto, flags;
  float p0, p1;
};

__device__ __forceinline__ uint64_t u64of(uint32_t lo, uint32_t hi) {
  return ((uint64_t)hi << 32) | lo;
}

// Decode the 128-byte record from eight uniform 16-byte loads (L2, so that a
// record restaged by the persistent worker is never read stale from L1).
__device__ __forceinline__ ReqView load_req(const Req* g) {
  const uint4* s = reinterpret_cast<const uint4*>(g);
  const uint4 w0 = __ldcg(s + 0), w1 = __ldcg(s + 1), w2 = __ldcg(s + 2), w3 = __ldcg(s + 3);
  const uint4 w4 = __ldcg(s + 4), w5 = __ldcg(s + 5), w6 = __ldcg(s + 6), w7 = __ldcg(s + 7);
  ReqView q;
  q.op = (int)(w0.x & 0xffffu);
  q.kind = (int)((w0.x >> 16) & 0xffu);
  q.layout = (int)(w0.x >> 24);
  q.dta = (int)(w0.y & 0xffu);
  q.dtb = (int)((w0.y >> 8) & 0xffu);
  q.dto = (int)((w0.y >> 16) & 0xffu);
  q.flags = (int)(w0.y >> 24);
  q.p0 = __uint_as_float(w0.z);
  q.p1 = __uint_as_float(w0.w);
  q.chunk = w1.x;
  q.nseg = w1.y;
  q.numel = (int64_t)u64of(w1.z, w1.w);
  q.a = u64of(w2.x, w2.y);
  q.b = u64of(w2.z, w2.w);
  q.o = u64of(w3.x, w3.y);
  q.inner = (int64_t)u64of(w3.z, w3.w);
  q.sa_row = (int64_t)u64of(w4.x, w4.y);
  q.sb_row = (int64_t)u64of(w4.z, w4.w);
  q.so_row = (int64_t)u64of(w5.x, w5.y);
  q.sa_in = (int64_t)u64of(w5.z, w5.w);
  q.sb_in = (int64_t)u64of(w6.x, w6.y);
  q.ext = w6.z;
  q.part = w6.w;
  q.cnt = w7.x;
  q.fdiv_m = w7.y;
  q.fdiv_s = w7.z;
  q.rg = w7.w;
  return q;
}

__device__ __forceinline__ int64_t row_of(const ReqView& q, int64_t e) {
  if (q.flags & RF_BIG) return e / q.inner;
  return (int64_t)fdiv_u32((uint32_t)e, q.fdiv_m, q.fdiv_s);
}

// Execution context of one warp inside one batch.
struct Exec {
  const uint8_t* base;          // batch payload in device memory
  const BatchHdr* h;
  BatchState* st;
  const Req* recs;
  const uint32_t* req_wait;     // per-request chunk count that must be done first (0: none)
  const Tables* tab;
  float* scratch;               // partial sums of split reductions
  uint32_t* counters;           // self-cleaning combine counters
  volatile uint64_t* done_ring; // completion words in mapped host memory (may be null)
  uint64_t* done_dev;           // device copy of the completion words (worker only)
  uint64_t wait_limit_ns;
  uint64_t seq;                 // batch sequence number
  uint32_t nchunk;              // chunks in the batch
  int lane;
};

__device__ __forceinline__ void set_err(const Exec& ex, uint32_t bits) {
  atomicOr(&ex.st->err, bits);
}

// Jump-table resolution (alias -> physical slot -> variant + parameters).
// The tables are read with plain volatile loads: the worker acquires at the
// batch boundary, a launched kernel starts after the host's table writes.
__device__ __forceinline__ int resolve(const ReqView& q, const Tables* tab, float& p0, float& p1) {
  p0 = q.p0;
  p1 = q.p1;
  if (!(q.flags & RF_SLOT)) return q.op;
  const int s = q.op;
  if (s < 0 || s >= kMaxSlots) return V_NONE;
  const volatile int32_t* al = tab->alias;
  const int phys = al[s];
  if (phys < 0 || phys >= kMaxSlots) return V_NONE;
  const volatile SlotEntry* se = &tab->slot[phys];
  const int v = se->variant;
  p0 = se->p0;
  p1 = se->p1;
  return v;
}

// ---------------------------------------------------------------------------
// Elementwise generic path (one shared body): misaligned views, arbitrary
// inner strides, and general strided requests of up to 8 dims.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void ew_generic(const ReqView& q, const ExtRec* x, int v, float p0,
                                           float p1, int64_t e0, int64_t e1, int lane) {
  const bool hasb = q.flags & RF_HAS_B;
  const int lay = q.layout;
  const int64_t N = q.inner;
  for (int64_t e = e0 + lane; e < e1; e += 32) {
    int64_t oa, ob, oo;
    if (lay == EL_CONTIG) {
      oa = (q.flags & RF_A_SCALAR) ? 0 : e;
      ob = (q.flags & RF_B_SCALAR) ? 0 : e;
      oo = e;
    } else if (lay == EL_ROW2D) {
      const int64_t r = row_of(q, e), c = e - r * N;
      oa = r * q.sa_row + c * q.sa_in;
      ob = r * q.sb_row + c * q.sb_in;
      oo = r * q.so_row + c;
    } else {
      int64_t rem = e;
      oa = ob = oo = 0;
      for (int d = __ldcg(&x->ndim) - 1; d >= 0; --d) {
        const int64_t sz = __ldcg(&x->sizes[d]);
        const int64_t i = rem % sz;
        rem /= sz;
        oa += i * __ldcg(&x->sa[d]);
        ob += i * __ldcg(&x->sb[d]);
        oo += i * __ldcg(&x->so[d]);
      }
    }
    const float A = ld1(q.a, q.dta, oa);
    const float B = hasb ? ld1(q.b, q.dtb, ob) : 0.f;
    float R = 0.f;
    ew_apply1(v, A, B, R, p0, p1);
    st1(q.o, q.dto, oo, R);
  }
}

// ---------------------------------------------------------------------------
// Reductions (sum / mean over the reduced columns), fp32 accumulation.
// ---------------------------------------------------------------------------
__device__ __forceinline__ float red_finish(float s, bool mean, int64_t C) {
  return mean ? s / (float)C : s;
}

// Combine the partial sums of one output (or a group of outputs) once every
// segment is in.  The warp that brings the counter to nseg sums the partials
// in segment order, so the result does not depend on which warp came last.
__device__ __forceinline__ bool combine_arrive(const Exec& ex, uint32_t* cnt, uint32_t nseg) {
  __threadfence();  // every lane releases its partial-sum store
  __syncwarp();
  uint32_t last = 0;
  if (ex.lane == 0) last = (atomicAdd(cnt, 1u) == nseg - 1) ? 1u : 0u;
  last = __shfl_sync(GPUOS_FULL, last, 0);
  if (last) __threadfence();
  return last != 0;
}

// Rows contiguous: a lane group of q.rg lanes sums one row (nseg == 1), or the
// whole warp sums one segment of a long row (nseg > 1).
__device__ __forceinline__ void red_rows(const Exec& ex, const ReqView& q, bool mean, uint32_t k) {
  const int lane = ex.lane;
  const int64_t C = q.inner;
  const bool vec = q.flags & RF_VEC;
  if (q.nseg == 1) {
    const int G = (int)q.rg;                   // lanes per row (power of two)
    const int per = 32 / G;                    // rows per warp step
    const int sub = lane / G, li = lane % G;
    const int64_t r0 = (int64_t)k * q.chunk;
    int64_t r1 = r0 + q.chunk;
    if (r1 > q.numel) r1 = q.numel;
    for (int64_t rb = r0; rb < r1; rb += per) {
      const int64_t r = rb + sub;
      const bool valid = r < r1;
      float acc0 = 0.f, acc1 = 0.f;
      if (valid) {
        const int64_t base = r * q.sa_row;
        if (vec) {
          const int64_t C8 = C & ~(int64_t)7;
          int64_t c = 8 * li;
          for (; c + 8 * G < C8; c += 16 * G) {
            float x[8], y[8];
            ld8(q.a, q.dta, base + c, x);
            ld8(q.a, q.dta, base + c + 8 * G, y);
#pragma unroll
            for (int t = 0; t < 8; ++t) { acc0 += x[t]; acc1 += y[t]; }
          }
          if (c < C8) {
            float x[8];
            ld8(q.a, q.dta, base + c, x);
#pragma unroll
            for (int t = 0; t < 8; ++t) acc0 += x[t];
          }
          for (int64_t t = C8 + li; t < C; t += G) acc1 += ld1(q.a, q.dta, base + t);
        } else {
          int64_t c = li;
          for (; c + G < C; c += 2 * G) {
            acc0 += ld1(q.a, q.dta, base + c);
            acc1 += ld1(q.a, q.dta, base + c + G);
          }
          if (c < C) acc0 += ld1(q.a, q.dta, base + c);
        }
      }
      float acc = acc0 + acc1;
      for (int off = G >> 1; off > 0; off >>= 1) acc += __shfl_xor_sync(GPUOS_FULL, acc, off);
      if (valid && li == 0) st1(q.o, q.dto, r * q.so_row, red_finish(acc, mean, C));
    }
    return;
  }
  // long rows: one warp per (row, segment)
  const uint32_t nseg = q.nseg;
  const int64_t r = k / nseg;
  const uint32_t seg = k % nseg;
  const int64_t c0 = (int64_t)seg * q.chunk;
  int64_t c1 = c0 + q.chunk;
  if (c1 > C) c1 = C;
  const int64_t base = r * q.sa_row;
  float acc0 = 0.f, acc1 = 0.f;
  if (vec) {  // c0 is a multiple of 8 (chunk is), c1 may end ragged on the last segment
    const int64_t c8 = c0 + ((c1 - c0) & ~(int64_t)7);
    int64_t c = c0 + 8 * lane;
    for (; c + 256 < c8; c += 512) {
      float x[8], y[8];
      ld8(q.a, q.dta, base + c, x);
      ld8(q.a, q.dta, base + c + 256, y);
#pragma unroll
      for (int t = 0; t < 8; ++t) { acc0 += x[t]; acc1 += y[t]; }
    }
    if (c < c8) {
      float x[8];
      ld8(q.a, q.dta, base + c, x);
#pragma unroll
      for (int t = 0; t < 8; ++t) acc0 += x[t];
    }
    for (int64_t t = c8 + lane; t < c1; t += 32) acc1 += ld1(q.a, q.dta, base + t);
  } else {
    for (int64_t c = c0 + lane; c < c1; c += 32) acc0 += ld1(q.a, q.dta, base + c);
  }
  float acc = acc0 + acc1;
  for (int off = 16; off > 0; off >>= 1) acc += __shfl_xor_sync(GPUOS_FULL, acc, off);
  float* part = ex.scratch + q.part + r * nseg;
  if (lane == 0) part[seg] = acc;
  uint32_t* cnt = ex.counters + q.cnt + r;
  if (combine_arrive(ex, cnt, nseg)) {
    float s = 0.f;
    for (uint32_t i = lane; i < nseg; i += 32) s += __ldcg(part + i);
    for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(GPUOS_FULL, s, off);
    if (lane == 0) {
      st1(q.o, q.dto, r * q.so_row, red_finish(s, mean, C));
      *cnt = 0u;  // leave the counter clean for the next batch
    }
  }
}

// Rows adjacent in memory (a transposed view): lanes own rows, so every step
// of the column loop reads rg adjacent rows of cl columns.
__device__ __forceinline__ void red_cols(const Exec& ex, const ReqView& q, bool mean, uint32_t k) {
  const int lane = ex.lane;
  const int64_t C = q.inner, R = q.numel;
  const int rg = (int)q.rg, cl = 32 / rg;
  const int rl = lane % rg, ci = lane / rg;
  const uint32_t nseg = q.nseg;
  const int64_t gi = k / nseg;
  const uint32_t seg = k % nseg;
  const int64_t r = gi * rg + rl;
  const bool valid = r < R;
  const int64_t c0 = (int64_t)seg * q.chunk;
  int64_t c1 = c0 + q.chunk;
  if (c1 > C) c1 = C;
  float acc0 = 0.f, acc1 = 0.f;
  if (valid) {
    const int64_t rb = r * q.sa_row;
    const int64_t sc = q.sa_in;
    int64_t c = c0 + ci;
    for (; c + 3 * cl < c1; c += 4 * cl) {
      const float x0 = ld1(q.a, q.dta, rb + c * sc);
      const float x1 = ld1(q.a, q.dta, rb + (c + cl) * sc);
      const float x2 = ld1(q.a, q.dta, rb + (c + 2 * cl) * sc);
      const float x3 = ld1(q.a, q.dta, rb + (c + 3 * cl) * sc);
      acc0 += x0; acc1 += x1; acc0 += x2; acc1 += x3;
    }
    for (; c < c1; c += cl) acc0 += ld1(q.a, q.dta, rb + c * sc);
  }
  float acc = acc0 + acc1;
  for (int off = rg; off < 32; off <<= 1) acc += __shfl_xor_sync(GPUOS_FULL, acc, off);
  if (nseg == 1) {
    if (valid && ci == 0) st1(q.o, q.dto, r * q.so_row, red_finish(acc, mean, C));
    return;
  }
  float* part = ex.scratch + q.part + (gi * nseg) * rg;
  if (ci == 0) part[seg * rg + rl] = acc;
  uint32_t* cnt = ex.counters + q.cnt + gi;
  if (combine_arrive(ex, cnt, nseg)) {
    if (ci == 0) {
      float s = 0.f;
      for (uint32_t i = 0; i < nseg; ++i) s += __ldcg(part + i * rg + rl);
      if (valid) st1(q.o, q.dto, r * q.so_row, red_finish(s, mean, C));
    }
    if (lane == 0) *cnt = 0u;
  }
}

// Anything else: one lane per output element, serial over the reduced
// elements with the first reduced axis varying fastest (the order of the
// reference's generic path, pytorch_ext/gpuos_ext.cpp:794-798).
__device__ __forceinline__ void red_generic(const Exec& ex, const ReqView& q, const ExtRec* x,
                                            bool mean, uint32_t k) {
  const int64_t o0 = (int64_t)k * q.chunk;
  int64_t o1 = o0 + q.chunk;
  if (o1 > q.numel) o1 = q.numel;
  const int nd = __ldcg(&x->ndim), rd = __ldcg(&x->rdim);
  for (int64_t oi = o0 + ex.lane; oi < o1; oi += 32) {
    int64_t rem = oi, ib = 0, ob = 0;
    for (int d = nd - 1; d >= 0; --d) {
      const int64_t sz = __ldcg(&x->sizes[d]);
      const int64_t i = rem % sz;
      rem /= sz;
      ib += i * __ldcg(&x->sa[d]);
      ob += i * __ldcg(&x->so[d]);
    }
    float acc = 0.f;
    for (int64_t rv = 0; rv < q.inner; ++rv) {
      int64_t t = rv, off = 0;
      for (int j = 0; j < rd; ++j) {
        const int64_t sz = __ldcg(&x->rsizes[j]);
        off += (t % sz) * __ldcg(&x->rstrides[j]);
        t /= sz;
      }
      acc += ld1(q.a, q.dta, ib + off);
    }
    st1(q.o, q.dto, ob, red_finish(acc, mean, q.inner));
  }
}

// ---------------------------------------------------------------------------
// One chunk of one request.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void process_chunk(const Exec& ex, const ReqView& q, uint32_t k) {
  float p0, p1;
  const int v = resolve(q, ex.tab, p0, p1);
  if (q.kind == RK_EW) {
    if (!ew_known(v)) {
      if (ex.lane == 0) set_err(ex, ERR_BAD_OP);
      return;
    }
    const int64_t e0 = (int64_t)k * q.chunk;
    int64_t e1 = e0 + q.chunk;
    if (e1 > q.numel) e1 = q.numel;
    ew_generic(q, reinterpret_cast<const ExtRec*>(ex.base + q.ext), v, p0, p1, e0, e1, ex.lane);
    return;
  }
  if (v != V_SUM && v != V_MEAN) {
    if (ex.lane == 0) set_err(ex, v < 0 ? ERR_BAD_OP : ERR_BAD_KIND);
    return;
  }
  const bool mean = (v == V_MEAN);
  if (q.layout == RL_ROWS) red_rows(ex, q, mean, k);
  else if (q.layout == RL_COLS) red_cols(ex, q, mean, k);
  else red_generic(ex, q, reinterpret_cast<const ExtRec*>(ex.base + q.ext), mean, k);
}

// Lane 0 waits (bounded) until `target` chunks of the batch are done.
__device__ __forceinline__ bool wait_chunks_done(const Exec& ex, uint32_t target) {
  uint32_t ok = 1;
  if (ex.lane == 0) {
    if (ld_acquire_u32(&ex.st->done) < target) {
      const uint64_t t0 = globaltimer();
      unsigned ns = 32;
      while (ld_acquire_u32(&ex.st->done) < target) {
        __nanosleep(ns);
        if (ns < 1024) ns <<= 1;
        if (globaltimer() - t0 > ex.wait_limit_ns) { ok = 0; break; }
      }
    }
  }
  ok = __shfl_sync(GPUOS_FULL, ok, 0);
  return ok != 0;
}

// Called by the warp that finished the last chunk of the batch.  The
// completion word is seq + 1 with the batch's error bits in bits 48..55.
__device__ __forceinline__ void finish_batch(const Exec& ex) {
  __threadfence();
  ex.st->t_last = globaltimer();
  const uint64_t seq = ex.seq;
  const uint32_t err = atomicOr(&ex.st->err, 0u);
  const uint64_t word = (seq + 1) | ((uint64_t)(err & 0xffu) << 48);
  if (ex.done_dev) st_release_gpu_u64(&ex.done_dev[seq % kDoneRing], word);
  if (ex.done_ring) {
    __threadfence_system();
    st_release_sys_u64(&ex.done_ring[seq % kDoneRing], word);
  }
}

// Bind the execution context of one batch payload.
__device__ __forceinline__ Exec bind_batch(const uint8_t* payload, const Tables* tab,
                                           volatile uint64_t* done_ring, uint64_t* done_dev,
                                           uint64_t wait_limit_ns) {
  // the header is read through L2: the persistent worker reuses payload memory
  const BatchHdr* h = reinterpret_cast<const BatchHdr*>(payload);
  Exec ex;
  ex.base = payload;
  ex.h = h;
  ex.st = reinterpret_cast<BatchState*>(const_cast<uint8_t*>(payload) + sizeof(BatchHdr));
  ex.recs = reinterpret_cast<const Req*>(payload + __ldcg(&h->rec_off));
  const uint32_t flags = __ldcg(&h->flags);
  const uint32_t gran = __ldcg(&h->gran), nch = __ldcg(&h->nchunk);
  ex.req_wait = (flags & BF_STAGED)
                    ? reinterpret_cast<const uint32_t*>(payload + __ldcg(&h->gtab_off)) +
                          (nch + gran - 1) / gran
                    : nullptr;
  ex.tab = tab;
  ex.scratch = reinterpret_cast<float*>(__ldcg(&h->scratch));
  ex.counters = reinterpret_cast<uint32_t*>(__ldcg(&h->counters));
  ex.seq = __ldcg(&h->seq);
  ex.nchunk = __ldcg(&h->nchunk);
  ex.done_ring = done_ring;
  ex.done_dev = done_dev;
  ex.wait_limit_ns = wait_limit_ns;
  ex.lane = threadIdx.x & 31;
  return ex;
}

}  // namespace gpuos
