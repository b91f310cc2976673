// Kernels of the aggregated small-op path for sm_100a.
//
//  gpuos_batch_kernel   one launch per batch, stream-ordered with the caller's
//                       CUDA stream (the mode that interoperates with torch
//                       streams and CUDA graphs).  Every warp runs its share of
//                       the batch's chunks (batch.cuh).
//  gpuos_worker_kernel  the persistent worker: CTA 0 polls the doorbell in
//                       mapped host memory and stages published batches into
//                       the device ring; every other CTA walks the staged
//                       batches in order, its warps running their share of
//                       each.  Replaces persistent_worker
//                       (src/persistent_kernel.cu:133-200), whose thread 0
//                       CAS-claims one 496-byte Task per CTA.
//
// Every wait in these kernels is bounded by %globaltimer.
#include "batch.cuh"
#include "lean.cuh"

namespace gpuos {

// Lean batches (lean.cuh): the whole batch is the kernel's parameter block,
// in three sizes so that a small batch does not ship 22 KB of parameters.
// One CTA of 512 threads per SM at 64 registers: half the SM's registers,
// so that the next batch's CTA fits beside it and starts (programmatic
// dependent launch) while this one drains.  Measured against one CTA of 1024
// threads (no room beside it), 512 threads with 8 groups in flight at 105
// registers, and 256 threads with 8 groups: 8.0 us per mixed-stream batch
// against 11.0, 11.5 and 10.5.
template <int N>
__global__ void __launch_bounds__(kLeanThreads, 2)
gpuos_lean_kernel(const __grid_constant__ LeanBatch<N> bt) {
  lean_batch<N, kLeanThreads, 4>(bt);
}

// Up to 1024 requests of one shape in one parameter block (LeanUniBatch).
__global__ void __launch_bounds__(kLeanThreads, 2)
gpuos_lean_uni_kernel(const __grid_constant__ LeanUniBatch bt) {
  lean_uni_batch<kLeanThreads, 4>(bt);
}

// The batch's descriptors are in the device staging ring (payload); its
// counters are `st`, one slot of a device array.  BODIES selects the chunk
// bodies the kernel carries (process_chunk).
template <int BODIES>
__device__ __forceinline__ void batch_body(const uint8_t* payload, const BatchHdr& hdr,
                                           BatchState* st, volatile uint64_t* done_ring,
                                           uint64_t wait_limit_ns) {
  __shared__ ExtRec ext[kWarpsPerCta];
  __shared__ uint32_t cta_chunks;
  __shared__ StageSync ss;
  if (threadIdx.x == 0) {
    cta_chunks = 0;
    ss.seen = 0;
    ss.poller = 0;
  }
  __syncthreads();
  const Exec ex = bind_batch(payload, hdr, st, done_ring, nullptr, wait_limit_ns);
  const int warp = threadIdx.x >> 5;
  const uint32_t count = warp_batch<BODIES>(ex, blockIdx.x * kWarpsPerCta + warp,
                                            gridDim.x * kWarpsPerCta, &ext[warp], &ss);
  // without stage barriers nothing waits on the batch's counters: the kernel's
  // completion completes the batch, and its warps leave as soon as they are done
  if (posts_own_errors(ex)) return;
  cta_leave_batch(ex, &cta_chunks, count, gridDim.x, nullptr);
}

extern "C" __global__ void __launch_bounds__(kCtaThreads, kMinCtasPerSm)
gpuos_batch_kernel(const uint8_t* payload, const BatchHdr hdr, BatchState* st,
                   volatile uint64_t* done_ring, uint64_t wait_limit_ns) {
  batch_body<BODY_ALL>(payload, hdr, st, done_ring, wait_limit_ns);
}

// Batches of only elementwise requests (that the lean kernel does not take)
// and of only reductions: the same loop with one class of bodies (less code
// to fetch).  Both at 2 CTAs per SM: at 3 the reduction bodies spill (80
// registers), and the spill-free 128-register form measured faster.
extern "C" __global__ void __launch_bounds__(kCtaThreads, kMinCtasPerSm)
gpuos_batch_ew_kernel(const uint8_t* payload, const BatchHdr hdr, BatchState* st,
                      volatile uint64_t* done_ring, uint64_t wait_limit_ns) {
  batch_body<BODY_EW>(payload, hdr, st, done_ring, wait_limit_ns);
}

extern "C" __global__ void __launch_bounds__(kCtaThreads, kMinCtasPerSm)
gpuos_batch_red_kernel(const uint8_t* payload, const BatchHdr hdr, BatchState* st,
                       volatile uint64_t* done_ring, uint64_t wait_limit_ns) {
  batch_body<BODY_RED>(payload, hdr, st, done_ring, wait_limit_ns);
}

// A small batch with stage barriers on one thread-block cluster (chain_batch
// in batch.cuh); launched with a cluster dimension equal to the grid.
extern "C" __global__ void __launch_bounds__(kCtaThreads, 1)
gpuos_chain_kernel(const uint8_t* payload, const BatchHdr hdr, BatchState* st,
                   volatile uint64_t* done_ring, uint64_t wait_limit_ns) {
  __shared__ ExtRec ext[kWarpsPerCta];
  __shared__ uint32_t cta_chunks;
  if (threadIdx.x == 0) cta_chunks = 0;
  __syncthreads();
  const Exec ex = bind_batch(payload, hdr, st, done_ring, nullptr, wait_limit_ns);
  const uint32_t count = chain_batch<BODY_ALL>(ex, hdr.nreq, &ext[threadIdx.x >> 5]);
  cta_leave_batch(ex, &cta_chunks, count, gridDim.x, nullptr);
}

// Copy `bytes` (multiple of 16, both ends 16-byte aligned) from mapped host
// memory to device memory: 16-byte loads that bypass the caches (ld.cv),
// 8 of them in flight per thread.
__device__ __forceinline__ void stage_copy(uint8_t* dst, const uint8_t* src, uint32_t bytes) {
  const uint32_t n = bytes >> 4;
  const uint4* s = reinterpret_cast<const uint4*>(src);
  uint4* d = reinterpret_cast<uint4*>(dst);
  const uint32_t stride = blockDim.x;
  uint32_t i = threadIdx.x;
  for (; i + 7 * stride < n; i += 8 * stride) {
    uint4 v[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) v[k] = __ldcv(s + i + k * stride);
#pragma unroll
    for (int k = 0; k < 8; ++k) d[i + k * stride] = v[k];
  }
  for (; i < n; i += stride) d[i] = __ldcv(s + i);
}

// CTA 0: doorbell poller and stager.
__device__ void ingest_loop(const WorkerArgs& w) {
  __shared__ uint64_t s_tail, s_quit, s_yield;
  __shared__ int s_stop;
  uint64_t s = w.start_seq;
  uint64_t staged_here = 0;
  uint64_t idle_since = globaltimer();
  unsigned backoff = 64;
  while (true) {
    if (threadIdx.x == 0) {
      s_tail = ld_acquire_sys_u64(&w.hctrl->tail);
      s_quit = w.hctrl->quit;
      s_yield = w.hctrl->yield_every;
      s_stop = 0;
    }
    __syncthreads();
    const uint64_t tail = s_tail;
    if (s < tail) {
      const volatile Pub* p = &w.pub[s % kDoneRing];
      const uint32_t off = p->off, bytes = p->bytes;
      stage_copy(w.ring + off, w.arena + off, bytes);
      __syncthreads();
      if (threadIdx.x == 0) {
        __threadfence();
        w.dctrl->ready_off[s % kDoneRing] = off;
        st_release_gpu_u64(&w.dctrl->ready, s + 1);
        w.hctrl->staged = s + 1;
      }
      ++s;
      ++staged_here;
      idle_since = globaltimer();
      backoff = 64;
      continue;
    }
    if (threadIdx.x == 0) {
      const uint64_t now = globaltimer();
      const bool yield = s_yield != 0 && staged_here >= s_yield;
      const bool idle = now - idle_since > w.idle_ns;
      if (s_quit || yield || idle) {
        // announce the stop, then look at the doorbell once more so that a
        // batch published in between is not stranded
        w.hctrl->running = 0u;
        __threadfence_system();
        if (ld_acquire_sys_u64(&w.hctrl->tail) > s && !s_quit && !yield) {
          w.hctrl->running = 1u;
        } else {
          w.hctrl->exit_reason = s_quit ? 1u : (yield ? 2u : 3u);
          st_release_gpu_u64(&w.dctrl->stop_at, s);
          s_stop = 1;
        }
      } else {
        w.hctrl->heartbeat = w.hctrl->heartbeat + 1;
        __nanosleep(backoff);
        if (backoff < 4096) backoff <<= 1;
      }
    }
    __syncthreads();
    if (s_stop) return;
  }
}

// CTAs 1..n: run the staged batches in order.
__device__ __forceinline__ void worker_loop(const WorkerArgs& w, CtaSmem* sm) {
  const uint32_t nproc = gridDim.x - 1;
  const uint32_t gw = (blockIdx.x - 1) * kWarpsPerCta + (threadIdx.x >> 5);
  // the ingest stops the worker after idle_ns without work, so waiting much
  // longer than that for the next batch means it is gone
  const uint64_t idle_limit = w.idle_ns + 2000000000ull;
  if (threadIdx.x == 0) sm->chunks = 0;
  for (uint64_t s = w.start_seq;; ++s) {
    if (threadIdx.x == 0) {
      int go = 0;
      const uint64_t t0 = globaltimer();
      unsigned backoff = 32;
      while (true) {
        if (ld_acquire_u64(&w.dctrl->ready) > s) { go = 1; break; }
        if (ld_acquire_u64(&w.dctrl->stop_at) <= s) break;
        if (globaltimer() - t0 > idle_limit) {
          w.hctrl->err = w.hctrl->err | ERR_IDLE_EXIT;
          break;
        }
        __nanosleep(backoff);
        if (backoff < 2048) backoff <<= 1;
      }
      sm->go = go;
      if (go) sm->off = *reinterpret_cast<volatile uint32_t*>(&w.dctrl->ready_off[s % kDoneRing]);
    }
    __syncthreads();
    if (!sm->go) return;
    const uint8_t* payload = w.ring + sm->off;
    if (threadIdx.x < sizeof(BatchHdr) / 16) {
      // the header through L2: the ring is reused, and the ingest CTA wrote it
      reinterpret_cast<uint4*>(&sm->hdr)[threadIdx.x] =
          __ldcg(reinterpret_cast<const uint4*>(payload) + threadIdx.x);
    }
    __syncthreads();
    const Exec ex = bind_batch(payload, sm->hdr, &w.states[s % kDoneRing], w.done_ring,
                               w.dctrl->done_dev, w.wait_limit_ns, w.dur_ring, w.tab);
    if (threadIdx.x == 0)
      atomicMax(reinterpret_cast<unsigned long long*>(&ex.st->nt0), ~globaltimer());
    if (threadIdx.x == 0) {
      sm->ss.seen = 0;
      sm->ss.poller = 0;
      if (ex.flags & BF_AFTER_PREV) wait_prev_batches(ex);
    }
    __syncthreads();
    const uint32_t count = warp_batch<BODY_ALL>(ex, gw, nproc * kWarpsPerCta,
                                                &sm->ext[threadIdx.x >> 5], &sm->ss);
    cta_leave_batch(ex, &sm->chunks, count, nproc, w.retired_ring);
  }
}

extern "C" __global__ void __launch_bounds__(kCtaThreads, kMinCtasPerSm)
gpuos_worker_kernel(WorkerArgs w) {
  __shared__ CtaSmem sm;
  if (blockIdx.x == 0) ingest_loop(w);
  else worker_loop(w, &sm);
}

}  // namespace gpuos

// ---- launch wrappers used by the host runtime ------------------------------
extern "C" int gpuos_cta_threads() { return gpuos::kCtaThreads; }

extern "C" cudaError_t gpuos_launch_batch(const uint8_t* payload, const gpuos::BatchHdr* hdr,
                                          gpuos::BatchState* st, volatile uint64_t* done_ring,
                                          uint64_t wait_limit_ns, int grid, cudaStream_t stream,
                                          int bodies) {
  if (bodies == gpuos::BODY_EW)
    gpuos::gpuos_batch_ew_kernel<<<grid, gpuos::kCtaThreads, 0, stream>>>(payload, *hdr, st,
                                                                          done_ring, wait_limit_ns);
  else if (bodies == gpuos::BODY_RED)
    gpuos::gpuos_batch_red_kernel<<<grid, gpuos::kCtaThreads, 0, stream>>>(payload, *hdr, st,
                                                                           done_ring, wait_limit_ns);
  else
    gpuos::gpuos_batch_kernel<<<grid, gpuos::kCtaThreads, 0, stream>>>(payload, *hdr, st, done_ring,
                                                                       wait_limit_ns);
  return cudaGetLastError();
}

// One cluster of `ctas` CTAs (at most 8, the portable cluster size).
extern "C" cudaError_t gpuos_launch_chain(const uint8_t* payload, const gpuos::BatchHdr* hdr,
                                          gpuos::BatchState* st, volatile uint64_t* done_ring,
                                          uint64_t wait_limit_ns, int ctas, cudaStream_t stream) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)ctas);
  cfg.blockDim = dim3(gpuos::kCtaThreads);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = stream;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = (unsigned)ctas;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, gpuos::gpuos_chain_kernel, payload, *hdr, st, done_ring,
                            wait_limit_ns);
}

extern "C" cudaError_t gpuos_launch_worker(const void* args, int grid, cudaStream_t stream) {
  const gpuos::WorkerArgs* w = static_cast<const gpuos::WorkerArgs*>(args);
  gpuos::gpuos_worker_kernel<<<grid, gpuos::kCtaThreads, 0, stream>>>(*w);
  return cudaGetLastError();
}

// Launch a lean batch (`params` points at a LeanBatch<32>, <128> or <512>, by
// size_class 0, 1, 2) on `grid` CTAs, with programmatic dependent launch.
extern "C" cudaError_t gpuos_launch_lean(const void* params, int size_class, int grid,
                                         cudaStream_t stream) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)grid);
  cfg.blockDim = dim3(gpuos::kLeanThreads);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = stream;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  switch (size_class) {
    case 0:
      return cudaLaunchKernelEx(&cfg, gpuos::gpuos_lean_kernel<32>,
                                *static_cast<const gpuos::LeanBatch<32>*>(params));
    case 1:
      return cudaLaunchKernelEx(&cfg, gpuos::gpuos_lean_kernel<128>,
                                *static_cast<const gpuos::LeanBatch<128>*>(params));
    case 2:
      return cudaLaunchKernelEx(&cfg, gpuos::gpuos_lean_kernel<gpuos::kLeanMaxReq>,
                                *static_cast<const gpuos::LeanBatch<gpuos::kLeanMaxReq>*>(params));
    case 3:
      return cudaLaunchKernelEx(&cfg, gpuos::gpuos_lean_uni_kernel,
                                *static_cast<const gpuos::LeanUniBatch*>(params));
    default:
      return cudaErrorInvalidValue;
  }
}

extern "C" size_t gpuos_lean_params_size(int size_class) {
  switch (size_class) {
    case 0: return sizeof(gpuos::LeanBatch<32>);
    case 1: return sizeof(gpuos::LeanBatch<128>);
    case 2: return sizeof(gpuos::LeanBatch<gpuos::kLeanMaxReq>);
    case 3: return sizeof(gpuos::LeanUniBatch);
    default: return 0;
  }
}

// Resident blocks per SM of the two kernels (the persistent grid must be
// fully resident).
extern "C" cudaError_t gpuos_occupancy(int* batch_blocks_per_sm, int* worker_blocks_per_sm,
                                       int* ew_blocks_per_sm, int* red_blocks_per_sm) {
  cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(
      batch_blocks_per_sm, gpuos::gpuos_batch_kernel, gpuos::kCtaThreads, 0);
  if (e != cudaSuccess) return e;
  e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(ew_blocks_per_sm, gpuos::gpuos_batch_ew_kernel,
                                                    gpuos::kCtaThreads, 0);
  if (e != cudaSuccess) return e;
  e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(red_blocks_per_sm, gpuos::gpuos_batch_red_kernel,
                                                    gpuos::kCtaThreads, 0);
  if (e != cudaSuccess) return e;
  return cudaOccupancyMaxActiveBlocksPerMultiprocessor(
      worker_blocks_per_sm, gpuos::gpuos_worker_kernel, gpuos::kCtaThreads, 0);
}

extern "C" size_t gpuos_worker_args_size() { return sizeof(gpuos::WorkerArgs); }
