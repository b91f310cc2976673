// Batch executor: warps claim fixed-size chunks of a batch with one atomic
// each and run the chunk through a layout-specific processor.
//
// Replaces the reference's op_batch (src/persistent_kernel.cu:81-112), which
// walks the sub-tasks of a 512-task shard one after another inside a single
// CTA with int64 div/mod index math per element, and the NVRTC operators of
// pytorch_ext/gpuos_ext.cpp:625-679 (elementwise) and 726-806 (reduce), which
// run one request per CTA.  Here every request is split into chunks and all
// chunks of a batch are spread over every SM; contiguous and row-broadcast
// requests move 16 bytes per lane per access.
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

__device__ __forceinline__ int64_t row_of(const Req& q, int64_t e) {
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
  int lane;
};

__device__ __forceinline__ void set_err(const Exec& ex, uint32_t bits) {
  atomicOr(&ex.st->err, bits);
}

// Jump-table resolution (alias -> physical slot -> variant + parameters).
// The tables are read with plain volatile loads: the worker acquires at the
// batch boundary, a launched kernel starts after the host's table writes.
__device__ __forceinline__ int resolve(const Req& q, const Tables* tab, float& p0, float& p1) {
  p0 = q.p0;
  p1 = q.p1;
  if (!(q.flags & RF_SLOT)) return q.op;
  int s = q.op;
  if (s < 0 || s >= kMaxSlots) return V_NONE;
  const volatile int32_t* al = tab->alias;
  int phys = al[s];
  if (phys < 0 || phys >= kMaxSlots) return V_NONE;
  const volatile SlotEntry* se = &tab->slot[phys];
  int v = se->variant;
  p0 = se->p0;
  p1 = se->p1;
  return v;
}

// ---------------------------------------------------------------------------
// Elementwise, every operand contiguous over numel (or a broadcast scalar).
// ---------------------------------------------------------------------------
__device__ __noinline__ void ew_contig(const Req& q, int v, float p0, float p1,
                                       int64_t e0, int64_t e1, int lane) {
  const bool hasb = q.flags & RF_HAS_B;
  const bool asc = q.flags & RF_A_SCALAR;
  const bool bsc = q.flags & RF_B_SCALAR;
  const float As = asc ? ld1(q.a, q.dta, 0) : 0.f;
  const float Bs = (hasb && bsc) ? ld1(q.b, q.dtb, 0) : 0.f;
  if (q.flags & RF_VEC) {
    const int64_t eend = e1 & ~(int64_t)7;
    int64_t e = e0 + 8 * lane;
    for (; e + 256 < eend; e += 512) {
      float A0[8], A1[8], B0[8], B1[8], R0[8], R1[8];
      if (asc) {
#pragma unroll
        for (int k = 0; k < 8; ++k) { A0[k] = As; A1[k] = As; }
      } else {
        ld8(q.a, q.dta, e, A0);
        ld8(q.a, q.dta, e + 256, A1);
      }
      if (hasb && !bsc) {
        ld8(q.b, q.dtb, e, B0);
        ld8(q.b, q.dtb, e + 256, B1);
      } else {
#pragma unroll
        for (int k = 0; k < 8; ++k) { B0[k] = Bs; B1[k] = Bs; }
      }
      ew_apply8(v, A0, B0, R0, p0, p1);
      ew_apply8(v, A1, B1, R1, p0, p1);
      st8(q.o, q.dto, e, R0);
      st8(q.o, q.dto, e + 256, R1);
    }
    if (e < eend) {
      float A0[8], B0[8], R0[8];
      if (asc) {
#pragma unroll
        for (int k = 0; k < 8; ++k) A0[k] = As;
      } else {
        ld8(q.a, q.dta, e, A0);
      }
      if (hasb && !bsc) {
        ld8(q.b, q.dtb, e, B0);
      } else {
#pragma unroll
        for (int k = 0; k < 8; ++k) B0[k] = Bs;
      }
      ew_apply8(v, A0, B0, R0, p0, p1);
      st8(q.o, q.dto, e, R0);
    }
    const int64_t t = eend + lane;
    if (t < e1) {
      float A = asc ? As : ld1(q.a, q.dta, t);
      float B = (hasb && !bsc) ? ld1(q.b, q.dtb, t) : Bs;
      float r = 0.f;
      ew_apply1(v, A, B, r, p0, p1);
      st1(q.o, q.dto, t, r);
    }
    return;
  }
  // scalar path: 4 elements per lane per iteration, loads issued first
  int64_t e = e0 + lane;
  for (; e + 96 < e1; e += 128) {
    float A[4], B[4], R[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      A[k] = asc ? As : ld1(q.a, q.dta, e + 32 * k);
      B[k] = (hasb && !bsc) ? ld1(q.b, q.dtb, e + 32 * k) : Bs;
    }
#pragma unroll
    for (int k = 0; k < 4; ++k) ew_apply1(v, A[k], B[k], R[k], p0, p1);
#pragma unroll
    for (int k = 0; k < 4; ++k) st1(q.o, q.dto, e + 32 * k, R[k]);
  }
  for (; e < e1; e += 32) {
    float A = asc ? As : ld1(q.a, q.dta, e);
    float B = (hasb && !bsc) ? ld1(q.b, q.dtb, e) : Bs;
    float r = 0.f;
    ew_apply1(v, A, B, r, p0, p1);
    st1(q.o, q.dto, e, r);
  }
}

// ---------------------------------------------------------------------------
// Elementwise over [rows, inner]: out(r, c) = o[r*so_row + c]; each input
// x(r, c) = x[r*sx_row + c*sx_in].  Covers [B,N] op [N], [B,N] op [B,1],
// transposed 2-D views and every request that collapses to two dims.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void ld8_or_splat(uint64_t p, int dt, int64_t row_off, int64_t col,
                                             int64_t s_in, bool scalar, float sc, float* v) {
  if (scalar) {
#pragma unroll
    for (int k = 0; k < 8; ++k) v[k] = sc;
  } else if (s_in == 0) {
    float x = ld1(p, dt, row_off);
#pragma unroll
    for (int k = 0; k < 8; ++k) v[k] = x;
  } else {
    ld8(p, dt, row_off + col, v);
  }
}

__device__ __noinline__ void ew_row2d(const Req& q, int v, float p0, float p1,
                                      int64_t e0, int64_t e1, int lane) {
  const bool hasb = q.flags & RF_HAS_B;
  const bool asc = q.flags & RF_A_SCALAR;
  const bool bsc = q.flags & RF_B_SCALAR;
  const float As = asc ? ld1(q.a, q.dta, 0) : 0.f;
  const float Bs = (hasb && bsc) ? ld1(q.b, q.dtb, 0) : 0.f;
  const int64_t N = q.inner;
  if (q.flags & RF_VEC) {  // N % 8 == 0, so an 8-group never straddles rows
    int64_t e = e0 + 8 * lane;
    for (; e + 256 < e1; e += 512) {
      const int64_t r0 = row_of(q, e), c0 = e - r0 * N;
      const int64_t r1 = row_of(q, e + 256), c1 = e + 256 - r1 * N;
      float A0[8], A1[8], B0[8], B1[8], R0[8], R1[8];
      ld8_or_splat(q.a, q.dta, r0 * q.sa_row, c0, q.sa_in, asc, As, A0);
      ld8_or_splat(q.a, q.dta, r1 * q.sa_row, c1, q.sa_in, asc, As, A1);
      if (hasb) {
        ld8_or_splat(q.b, q.dtb, r0 * q.sb_row, c0, q.sb_in, bsc, Bs, B0);
        ld8_or_splat(q.b, q.dtb, r1 * q.sb_row, c1, q.sb_in, bsc, Bs, B1);
      } else {
#pragma unroll
        for (int k = 0; k < 8; ++k) { B0[k] = 0.f; B1[k] = 0.f; }
      }
      ew_apply8(v, A0, B0, R0, p0, p1);
      ew_apply8(v, A1, B1, R1, p0, p1);
      st8(q.o, q.dto, r0 * q.so_row + c0, R0);
      st8(q.o, q.dto, r1 * q.so_row + c1, R1);
    }
    if (e < e1) {
      const int64_t r0 = row_of(q, e), c0 = e - r0 * N;
      float A0[8], B0[8], R0[8];
      ld8_or_splat(q.a, q.dta, r0 * q.sa_row, c0, q.sa_in, asc, As, A0);
      if (hasb) {
        ld8_or_splat(q.b, q.dtb, r0 * q.sb_row, c0, q.sb_in, bsc, Bs, B0);
      } else {
#pragma unroll
        for (int k = 0; k < 8; ++k) B0[k] = 0.f;
      }
      ew_apply8(v, A0, B0, R0, p0, p1);
      st8(q.o, q.dto, r0 * q.so_row + c0, R0);
    }
    return;
  }
  int64_t e = e0 + lane;
  for (; e + 96 < e1; e += 128) {
    float A[4], B[4], R[4];
    int64_t oo[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int64_t ek = e + 32 * k;
      const int64_t r = row_of(q, ek), c = ek - r * N;
      A[k] = asc ? As : ld1(q.a, q.dta, r * q.sa_row + c * q.sa_in);
      B[k] = hasb ? (bsc ? Bs : ld1(q.b, q.dtb, r * q.sb_row + c * q.sb_in)) : 0.f;
      oo[k] = r * q.so_row + c;
    }
#pragma unroll
    for (int k = 0; k < 4; ++k) ew_apply1(v, A[k], B[k], R[k], p0, p1);
#pragma unroll
    for (int k = 0; k < 4; ++k) st1(q.o, q.dto, oo[k], R[k]);
  }
  for (; e < e1; e += 32) {
    const int64_t r = row_of(q, e), c = e - r * N;
    float A = asc ? As : ld1(q.a, q.dta, r * q.sa_row + c * q.sa_in);
    float B = hasb ? (bsc ? Bs : ld1(q.b, q.dtb, r * q.sb_row + c * q.sb_in)) : 0.f;
    float R = 0.f;
    ew_apply1(v, A, B, R, p0, p1);
    st1(q.o, q.dto, r * q.so_row + c, R);
  }
}

// ---------------------------------------------------------------------------
// Elementwise, general strides over up to 8 dims (extension record).
// ---------------------------------------------------------------------------
__device__ __noinline__ void ew_strided(const Req& q, const ExtRec* x, int v, float p0, float p1,
                                        int64_t e0, int64_t e1, int lane) {
  const bool hasb = q.flags & RF_HAS_B;
  const int nd = x->ndim;
  for (int64_t e = e0 + lane; e < e1; e += 32) {
    int64_t rem = e, oa = 0, ob = 0, oo = 0;
    for (int d = nd - 1; d >= 0; --d) {
      const int64_t sz = x->sizes[d];
      const int64_t i = rem % sz;
      rem /= sz;
      oa += i * x->sa[d];
      ob += i * x->sb[d];
      oo += i * x->so[d];
    }
    float A = ld1(q.a, q.dta, oa);
    float B = hasb ? ld1(q.b, q.dtb, ob) : 0.f;
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
__device__ __noinline__ void red_rows(const Exec& ex, const Req& q, bool mean, uint32_t k) {
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
__device__ __noinline__ void red_cols(const Exec& ex, const Req& q, bool mean, uint32_t k) {
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
__device__ __noinline__ void red_generic(const Exec& ex, const Req& q, const ExtRec* x, bool mean,
                                         uint32_t k) {
  const int64_t o0 = (int64_t)k * q.chunk;
  int64_t o1 = o0 + q.chunk;
  if (o1 > q.numel) o1 = q.numel;
  const int nd = x->ndim, rd = x->rdim;
  for (int64_t oi = o0 + ex.lane; oi < o1; oi += 32) {
    int64_t rem = oi, ib = 0, ob = 0;
    for (int d = nd - 1; d >= 0; --d) {
      const int64_t sz = x->sizes[d];
      const int64_t i = rem % sz;
      rem /= sz;
      ib += i * x->sa[d];
      ob += i * x->so[d];
    }
    float acc = 0.f;
    for (int64_t rv = 0; rv < q.inner; ++rv) {
      int64_t t = rv, off = 0;
      for (int j = 0; j < rd; ++j) {
        const int64_t sz = x->rsizes[j];
        off += (t % sz) * x->rstrides[j];
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
__device__ __forceinline__ void process_chunk(const Exec& ex, const Req& q, uint32_t k) {
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
    if (q.layout == EL_CONTIG) ew_contig(q, v, p0, p1, e0, e1, ex.lane);
    else if (q.layout == EL_ROW2D) ew_row2d(q, v, p0, p1, e0, e1, ex.lane);
    else ew_strided(q, reinterpret_cast<const ExtRec*>(ex.base + q.ext), v, p0, p1, e0, e1, ex.lane);
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

__device__ __forceinline__ void load_req(const Req* src, Req& dst) {
  const uint4* s = reinterpret_cast<const uint4*>(src);
  uint4* d = reinterpret_cast<uint4*>(&dst);
#pragma unroll
  for (int i = 0; i < 8; ++i) d[i] = __ldcg(s + i);
}

// index of the request that owns chunk c: s_cb[r] <= c < s_cb[r + 1]
__device__ __forceinline__ int find_req(const uint32_t* s_cb, int nreq, uint32_t c) {
  int lo = 0, hi = nreq - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (s_cb[mid] <= c) lo = mid; else hi = mid - 1;
  }
  return lo;
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
// completion word is seq + 1 with the batch's error bits in the top byte.
__device__ __forceinline__ void finish_batch(const Exec& ex) {
  __threadfence();
  ex.st->t_last = globaltimer();
  const uint64_t seq = ex.h->seq;
  const uint32_t err = atomicOr(&ex.st->err, 0u);
  const uint64_t word = (seq + 1) | ((uint64_t)(err & 0xffu) << 56);
  if (ex.done_dev) st_release_gpu_u64(&ex.done_dev[seq % kDoneRing], word);
  if (ex.done_ring) {
    __threadfence_system();
    st_release_sys_u64(&ex.done_ring[seq % kDoneRing], word);
  }
}

// Count `n` finished chunks.  Every lane releases its stores first, so a warp
// that sees the count (a stage waiter, the finisher) also sees the data.
__device__ __forceinline__ void arrive_done(const Exec& ex, uint32_t n) {
  __threadfence();
  __syncwarp();
  if (ex.lane == 0 && n != 0u) {
    const uint32_t d = atomicAdd(&ex.st->done, n) + n;
    if (d == ex.h->nchunk) finish_batch(ex);
  }
}

// The claim loop of one warp over one batch.  s_cb is the CTA's shared copy of
// the chunk prefix array.  Without stage barriers a warp reports its finished
// chunks once, when it runs out of work; with them it reports every chunk, so
// that warps waiting on an earlier stage are never waiting on it.
__device__ void run_batch_warp(const Exec& ex, const uint32_t* s_cb) {
  const uint32_t nchunk = ex.h->nchunk;
  const int nreq = (int)ex.h->nreq;
  const int lane = ex.lane;
  const bool staged = ex.req_wait != nullptr;
  uint32_t c = 0;
  if (lane == 0) {
    c = atomicAdd(&ex.st->claim, 1u);
    if (c == 0) ex.st->t_first = globaltimer();
  }
  c = __shfl_sync(GPUOS_FULL, c, 0);
  int r = -1;
  uint32_t rbase = 0, rend = 0, mine = 0;
  Req q;
  while (c < nchunk) {
    uint32_t cn = 0;
    if (lane == 0) cn = atomicAdd(&ex.st->claim, 1u);
    if (r < 0 || c >= rend || c < rbase) {
      r = find_req(s_cb, nreq, c);
      rbase = s_cb[r];
      rend = s_cb[r + 1];
      load_req(ex.recs + r, q);
    }
    bool run = true;
    if (staged) {
      const uint32_t w = __ldcg(ex.req_wait + r);
      if (w != 0u && !wait_chunks_done(ex, w)) {
        if (lane == 0) set_err(ex, ERR_STAGE_TIMEOUT);
        run = false;
      }
    }
    if (run) process_chunk(ex, q, c - rbase);
    if (staged) arrive_done(ex, 1u);
    else ++mine;
    c = __shfl_sync(GPUOS_FULL, cn, 0);
  }
  if (!staged) arrive_done(ex, mine);
}

// Bind the execution context of one batch payload.
__device__ __forceinline__ Exec bind_batch(const uint8_t* payload, const Tables* tab,
                                           volatile uint64_t* done_ring, uint64_t* done_dev,
                                           uint64_t wait_limit_ns) {
  const BatchHdr* h = reinterpret_cast<const BatchHdr*>(payload);
  Exec ex;
  ex.base = payload;
  ex.h = h;
  ex.st = reinterpret_cast<BatchState*>(const_cast<uint8_t*>(payload) + sizeof(BatchHdr));
  ex.recs = reinterpret_cast<const Req*>(payload + h->rec_off);
  ex.req_wait = (h->flags & BF_STAGED)
                    ? reinterpret_cast<const uint32_t*>(payload + h->cb_off) + (h->nreq + 1)
                    : nullptr;
  ex.tab = tab;
  ex.scratch = reinterpret_cast<float*>(h->scratch);
  ex.counters = reinterpret_cast<uint32_t*>(h->counters);
  ex.done_ring = done_ring;
  ex.done_dev = done_dev;
  ex.wait_limit_ns = wait_limit_ns;
  ex.lane = threadIdx.x & 31;
  return ex;
}

// CTA-level entry for one batch: copy the chunk prefix into shared memory,
// run every warp's claim loop, then count this CTA out of the batch.  The CTA
// that leaves last retires the batch: nobody reads its payload any more, so
// the host may reuse the memory.
__device__ __forceinline__ void run_batch_cta(const uint8_t* payload, const Tables* tab,
                                              volatile uint64_t* done_ring, uint64_t* done_dev,
                                              volatile uint64_t* retired_ring, uint32_t nctas,
                                              uint64_t wait_limit_ns, uint32_t* s_cb) {
  const BatchHdr* h = reinterpret_cast<const BatchHdr*>(payload);
  const uint32_t nreq = h->nreq;
  const uint32_t* cb = reinterpret_cast<const uint32_t*>(payload + h->cb_off);
  for (uint32_t i = threadIdx.x; i <= nreq; i += blockDim.x) s_cb[i] = __ldcg(cb + i);
  __syncthreads();
  Exec ex = bind_batch(payload, tab, done_ring, done_dev, wait_limit_ns);
  run_batch_warp(ex, s_cb);
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const uint32_t left = atomicAdd(&ex.st->ctas_left, 1u) + 1u;
    if (left == nctas && retired_ring) {
      __threadfence_system();
      const uint64_t seq = h->seq;
      st_release_sys_u64(&retired_ring[seq % kDoneRing], seq + 1);
    }
  }
}

}  // namespace gpuos
