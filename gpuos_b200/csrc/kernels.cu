// Kernels of the aggregated small-op path for sm_100a.
//
//  gpuos_batch_kernel   one launch per batch, stream-ordered with the caller's
//                       CUDA stream (the mode that interoperates with torch
//                       streams and CUDA graphs).  One pipeline CTA per SM
//                       (pipeline.cuh).
//  gpuos_worker_kernel  the persistent worker: CTA 0 polls the doorbell in
//                       mapped host memory and stages published batches into
//                       the device ring; every other CTA is a pipeline that
//                       walks the batches in order, its producer warp moving
//                       from one batch to the next without draining.  Replaces
//                       persistent_worker (src/persistent_kernel.cu:133-200),
//                       whose thread 0 CAS-claims one 496-byte Task per CTA.
//
// Every wait in these kernels is bounded by %globaltimer.
#include "pipeline.cuh"

namespace gpuos {

extern "C" __global__ void __launch_bounds__(kCtaThreads, 1)
gpuos_batch_kernel(const uint8_t* payload, const Tables* tab, volatile uint64_t* done_ring,
                   volatile uint64_t* retired_ring, uint64_t wait_limit_ns) {
  extern __shared__ __align__(128) uint8_t smem[];
  PipeSmem* sm = pipe_init(smem);
  uint8_t* bufs = smem + pipe_buf_offset();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (warp == 0) {
    Producer P{sm, bufs, 0, 0, wait_limit_ns, false};
    produce_batch(P, payload, tab, nullptr, blockIdx.x, gridDim.x, lane);
    produce_stop(P, lane);
  } else {
    consume(sm, bufs, tab, done_ring, nullptr, retired_ring, gridDim.x, wait_limit_ns);
  }
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

// CTAs 1..n: a pipeline over the staged batches, in order.
__device__ void pipeline_loop(const WorkerArgs& w, uint8_t* smem) {
  PipeSmem* sm = pipe_init(smem);
  uint8_t* bufs = smem + pipe_buf_offset();
  const uint32_t nproc = gridDim.x - 1;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // the ingest stops the worker after idle_ns without work, so waiting much
  // longer than that for the next batch means it is gone
  const uint64_t idle_limit = w.idle_ns + 2000000000ull;
  if (warp != 0) {
    consume(sm, bufs, w.tab, w.done_ring, w.dctrl->done_dev, w.retired_ring, nproc,
            idle_limit + w.wait_limit_ns);
    return;
  }
  Producer P{sm, bufs, 0, 0, w.wait_limit_ns, false};
  for (uint64_t s = w.start_seq;; ++s) {
    int go = 0;
    uint32_t off = 0;
    if (lane == 0) {
      const uint64_t t0 = globaltimer();
      unsigned backoff = 32;
      while (!P.dead) {
        if (ld_acquire_u64(&w.dctrl->ready) > s) { go = 1; break; }
        if (ld_acquire_u64(&w.dctrl->stop_at) <= s) break;
        if (globaltimer() - t0 > idle_limit) {
          w.hctrl->err = w.hctrl->err | ERR_IDLE_EXIT;
          break;
        }
        __nanosleep(backoff);
        if (backoff < 2048) backoff <<= 1;
      }
      if (go) off = *reinterpret_cast<volatile uint32_t*>(&w.dctrl->ready_off[s % kDoneRing]);
    }
    go = __shfl_sync(GPUOS_FULL, go, 0);
    off = __shfl_sync(GPUOS_FULL, off, 0);
    if (!go) break;
    produce_batch(P, w.ring + off, w.tab, w.dctrl->done_dev, blockIdx.x - 1, nproc, lane);
    const int dead = __shfl_sync(GPUOS_FULL, P.dead ? 1 : 0, 0);
    if (dead) break;
  }
  produce_stop(P, lane);
}

extern "C" __global__ void __launch_bounds__(kCtaThreads, 1) gpuos_worker_kernel(WorkerArgs w) {
  extern __shared__ __align__(128) uint8_t smem[];
  if (blockIdx.x == 0) ingest_loop(w);
  else pipeline_loop(w, smem);
}

}  // namespace gpuos

// ---- launch wrappers used by the host runtime ------------------------------
extern "C" size_t gpuos_pipe_smem_bytes() { return gpuos::pipe_smem_bytes(); }
extern "C" int gpuos_cta_threads() { return gpuos::kCtaThreads; }
extern "C" int gpuos_unit_elems() { return gpuos::kUnit; }

// Opt in to the dynamic shared memory of a pipeline CTA (current device).
extern "C" cudaError_t gpuos_kernel_setup() {
  const int bytes = (int)gpuos::pipe_smem_bytes();
  cudaError_t e = cudaFuncSetAttribute(gpuos::gpuos_batch_kernel,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e != cudaSuccess) return e;
  return cudaFuncSetAttribute(gpuos::gpuos_worker_kernel,
                              cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
}

extern "C" cudaError_t gpuos_launch_batch(const uint8_t* payload, const gpuos::Tables* tab,
                                          volatile uint64_t* done_ring,
                                          volatile uint64_t* retired_ring, uint64_t wait_limit_ns,
                                          int grid, int block, cudaStream_t stream) {
  (void)block;
  gpuos::gpuos_batch_kernel<<<grid, gpuos::kCtaThreads, gpuos::pipe_smem_bytes(), stream>>>(
      payload, tab, done_ring, retired_ring, wait_limit_ns);
  return cudaGetLastError();
}

extern "C" cudaError_t gpuos_launch_worker(const void* args, int grid, int block,
                                           cudaStream_t stream) {
  (void)block;
  const gpuos::WorkerArgs* w = static_cast<const gpuos::WorkerArgs*>(args);
  gpuos::gpuos_worker_kernel<<<grid, gpuos::kCtaThreads, gpuos::pipe_smem_bytes(), stream>>>(*w);
  return cudaGetLastError();
}

extern "C" cudaError_t gpuos_occupancy(int block, int* batch_blocks_per_sm,
                                       int* worker_blocks_per_sm) {
  (void)block;
  const size_t smem = gpuos::pipe_smem_bytes();
  cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(
      batch_blocks_per_sm, gpuos::gpuos_batch_kernel, gpuos::kCtaThreads, smem);
  if (e != cudaSuccess) return e;
  return cudaOccupancyMaxActiveBlocksPerMultiprocessor(
      worker_blocks_per_sm, gpuos::gpuos_worker_kernel, gpuos::kCtaThreads, smem);
}

extern "C" size_t gpuos_worker_args_size() { return sizeof(gpuos::WorkerArgs); }
