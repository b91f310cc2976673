// The lean batch kernel: stream-mode batches of contiguous, aligned fp32
// elementwise requests of the precompiled operators, with the whole batch in
// the kernel's parameters (struct LeanBatch, gpuos_abi.h).
//
// Why it exists: such batches are the mixed-operator and add/mul streams.
// The general batch kernel carries every body (strided views, per-row
// operands, 16-bit types, reductions, stage barriers) and needs 128 registers
// per thread, so an SM holds 16 warps, and neighbouring warps run different
// operator bodies out of one large kernel: a third of the stall cycles were
// instruction fetch.  Here:
//   * one CTA of 512 threads per SM at 64 registers per thread (16 warps):
//     half the SM's registers, so the next batch's CTA fits beside it;
//   * warp g of W runs the contiguous chunk range [g n / W, (g + 1) n / W):
//     the host sorts a batch's requests by operator, so the warps of an SM
//     run one or two operator bodies;
//   * the CTA copies the chunk prefix from parameter space into shared
//     memory (one element per thread), each warp finds its first request by
//     a binary search there and reads its records from parameter space: no
//     staging copy of the batch, no granule table, no global load before the
//     first data load;
//   * programmatic dependent launch: a batch launches while the previous one
//     drains and does its parameter-only set-up meanwhile.  It waits for the
//     previous grid before touching global memory when the host says so
//     (LEAN_WAIT_FIRST: the first batch of a flush, or a hazard with an
//     earlier batch of the same flush), lets the next batch launch at once,
//     and waits for the previous grid before it exits, so that batches
//     complete in stream order.
//   * completion: the last CTA posts the batch's completion word (seq + 1)
//     to mapped host memory.
// A batch of up to 1024 requests of one shape (LeanUniBatch: the add/mul
// stream's 1024 x 4096 in one launch instead of two) has no chunk prefix:
// chunk c belongs to request c / kpr.
#pragma once
#include "executor.cuh"

namespace gpuos {

__device__ __forceinline__ void gdc_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void gdc_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// 4-element groups per lane in flight per round: GL for the light operators,
// GL / 2 for those with a division, a square root or a transcendental function.
template <int V, int GL>
__device__ __forceinline__ constexpr int lean_groups() {
  return op_unroll<V>() == 2 ? GL : GL / 2;
}

struct LeanCur {
  const float* a;
  const float* b;
  float* o;
  uint32_t numel, chunk;
  int op, pidx;
};

// elements [e0, e0 + n) of one request, n > 0 (unary operators ignore b)
template <int V, int GL>
__device__ __forceinline__ void lean_chunk(const LeanCur& u, const LeanHdr& h, uint32_t e0,
                                           uint32_t n, int lane) {
  constexpr int kG = lean_groups<V, GL>();
  constexpr bool kBin = V == V_ADD || V == V_MUL || V == V_SUB || V == V_DIV0 || V == V_DIV ||
                        V == V_MAX || V == V_MIN || V == V_POW;
  const float p0 = h.par[u.pidx][0], p1 = h.par[u.pidx][1];
  const uint32_t nq = n >> 2;
  const float4* A = reinterpret_cast<const float4*>(u.a + e0);
  const float4* B = reinterpret_cast<const float4*>(u.b + e0);
  float4* O = reinterpret_cast<float4*>(u.o + e0);
#pragma unroll 1
  for (uint32_t q0 = lane; q0 < nq; q0 += 32 * kG) {
    float4 a[kG], b[kG];
#pragma unroll
    for (int g = 0; g < kG; ++g) {
      a[g] = make_float4(0.f, 0.f, 0.f, 0.f);
      b[g] = make_float4(0.f, 0.f, 0.f, 0.f);
      if (q0 + 32 * g < nq) {
        a[g] = A[q0 + 32 * g];
        if (kBin) b[g] = B[q0 + 32 * g];
      }
    }
#pragma unroll
    for (int g = 0; g < kG; ++g) {
      if (q0 + 32 * g < nq) {
        float4 r;
        r.x = op1<V>(a[g].x, b[g].x, p0, p1);
        r.y = op1<V>(a[g].y, b[g].y, p0, p1);
        r.z = op1<V>(a[g].z, b[g].z, p0, p1);
        r.w = op1<V>(a[g].w, b[g].w, p0, p1);
        O[q0 + 32 * g] = r;
      }
    }
  }
  if (lane < (int)(n & 3u)) {
    const uint32_t e = e0 + 4 * nq + lane;
    u.o[e] = op1<V>(u.a[e], kBin ? u.b[e] : 0.f, p0, p1);
  }
}

#define GPUOS_LEAN_CASE(V) case V: lean_chunk<V, GL>(u, h, e0, n, lane); return;

template <int GL>
__device__ __forceinline__ void lean_dispatch(const LeanCur& u, const LeanHdr& h, uint32_t e0,
                                              uint32_t n, int lane) {
  switch (u.op) {
    GPUOS_ALL_EW(GPUOS_LEAN_CASE)
    default: return;
  }
}

// End of a lean batch: every CTA releases its stores, the last one posts the
// batch's duration and completion word; the grid completes only after the
// previous grid in the stream has (stream order).
__device__ __forceinline__ void lean_finish(const LeanHdr& h, BatchState* st) {
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const uint32_t left = atomicAdd(&st->ctas_left, 1u) + 1u;
    if (left == gridDim.x) {
      __threadfence();
      const uint64_t nt0 = *reinterpret_cast<volatile uint64_t*>(&st->nt0);
      st->nt0 = 0ull;
      st->ctas_left = 0u;
      reinterpret_cast<volatile uint64_t*>(h.dur_ring)[h.seq % kDoneRing] =
          nt0 ? globaltimer() - ~nt0 : 0ull;
      volatile uint64_t* dr = reinterpret_cast<volatile uint64_t*>(h.done_ring);
      st_release_sys_u64(&dr[h.seq % kDoneRing], h.seq + 1);
    }
  }
  gdc_wait();
}

template <int N>
__device__ __forceinline__ void lean_decode(LeanCur& u, const LeanBatch<N>& bt, uint32_t r) {
  const LeanRec& q = bt.rec[r];
  u.a = reinterpret_cast<const float*>(q.a);
  u.b = reinterpret_cast<const float*>(q.b);
  u.o = reinterpret_cast<float*>(q.o);
  u.numel = q.numel;
  u.chunk = q.chunk;
  u.op = q.op;
  u.pidx = q.pidx;
}

template <int N, int THREADS, int GL>
__device__ __forceinline__ void lean_batch(const LeanBatch<N>& bt) {
  __shared__ uint32_t s_cb[N + 1];
  const LeanHdr& h = bt.h;
  gdc_launch_dependents();
  BatchState* st = reinterpret_cast<BatchState*>(h.st);
  if (threadIdx.x == 0) atomicMax(reinterpret_cast<unsigned long long*>(&st->nt0), ~globaltimer());
  // the chunk prefix into shared memory, one element per thread: every warp
  // then searches it there instead of through dependent parameter reads
  const uint32_t nreq = h.nreq;
  for (uint32_t i = threadIdx.x; i <= nreq; i += blockDim.x) s_cb[i] = bt.cb[i];
  __syncthreads();
  const int lane = threadIdx.x & 31;
  constexpr uint32_t kWarps = THREADS / 32;
  const uint64_t W = (uint64_t)gridDim.x * kWarps;
  const uint64_t gw = (uint64_t)blockIdx.x * kWarps + (threadIdx.x >> 5);
  const uint32_t nchunk = h.nchunk;
  const uint32_t c0 = (uint32_t)(gw * nchunk / W);
  const uint32_t c1 = (uint32_t)((gw + 1) * nchunk / W);
  // the request holding chunk c0: s_cb[lo] <= c0 < s_cb[lo + 1]
  uint32_t lo = 0, hi = nreq;
  while (hi - lo > 1) {
    const uint32_t mid = (lo + hi) >> 1;
    if (s_cb[mid] <= c0) lo = mid;
    else hi = mid;
  }
  uint32_t r = lo;
  LeanCur u;
  lean_decode(u, bt, r);
  // everything above reads parameters and shared memory only; memory the
  // previous grid may write is touched from here on
  if (h.flags & LEAN_WAIT_FIRST) gdc_wait();
  uint32_t rbase = s_cb[r], rend = s_cb[r + 1];
  for (uint32_t c = c0; c < c1; ++c) {
    if (c >= rend) {
      do {
        ++r;
        rbase = rend;
        rend = s_cb[r + 1];
      } while (c >= rend);
      lean_decode(u, bt, r);
    }
    const uint32_t e0 = (c - rbase) * u.chunk;
    const uint32_t n = min(u.chunk, u.numel - e0);
    lean_dispatch<GL>(u, h, e0, n, lane);
  }
  lean_finish(h, st);
}

// A batch of requests of one shape (LeanUniBatch): chunk c is chunk
// c mod kpr of request c / kpr; otherwise as lean_batch.
template <int THREADS, int GL>
__device__ __forceinline__ void lean_uni_batch(const LeanUniBatch& bt) {
  const LeanHdr& h = bt.h;
  gdc_launch_dependents();
  BatchState* st = reinterpret_cast<BatchState*>(h.st);
  if (threadIdx.x == 0) atomicMax(reinterpret_cast<unsigned long long*>(&st->nt0), ~globaltimer());
  const int lane = threadIdx.x & 31;
  constexpr uint32_t kWarps = THREADS / 32;
  const uint64_t W = (uint64_t)gridDim.x * kWarps;
  const uint64_t gw = (uint64_t)blockIdx.x * kWarps + (threadIdx.x >> 5);
  const uint32_t nchunk = h.nchunk, kpr = bt.kpr;
  const uint32_t c0 = (uint32_t)(gw * nchunk / W);
  const uint32_t c1 = (uint32_t)((gw + 1) * nchunk / W);
  if (h.flags & LEAN_WAIT_FIRST) gdc_wait();
  LeanCur u;
  u.numel = bt.numel;
  u.chunk = bt.chunk;
  uint32_t r = c0 / kpr, k = c0 - r * kpr;
  for (uint32_t c = c0; c < c1; ++c) {
    u.a = reinterpret_cast<const float*>(bt.a[r]);
    u.b = reinterpret_cast<const float*>(bt.b[r]);
    u.o = reinterpret_cast<float*>(bt.o[r]);
    u.op = bt.op[r];
    u.pidx = bt.pidx[r];
    const uint32_t e0 = k * u.chunk;
    lean_dispatch<GL>(u, h, e0, min(u.chunk, u.numel - e0), lane);
    if (++k == kpr) {
      k = 0;
      ++r;
    }
  }
  lean_finish(h, st);
}


}  // namespace gpuos
