// Kernels of the aggregated small-op path for sm_100a.
//
//  gpuos_batch_kernel   one launch per batch, stream-ordered with the caller's
//                       CUDA stream (the mode that interoperates with torch
//                       streams and CUDA graphs).
//  gpuos_worker_kernel  the persistent worker: CTA 0 polls the doorbell in
//                       mapped host memory and stages published batches into
//                       the device ring; every other CTA walks the batches in
//                       order and claims chunks warp by warp.  Replaces
//                       persistent_worker (src/persistent_kernel.cu:133-200),
//                       whose thread 0 CAS-claims one 496-byte Task per CTA.
//
// Every wait in these kernels is bounded by %globaltimer.
#include "executor.cuh"

namespace gpuos {

static constexpr int kBlockMax = 1024;

extern "C" __global__ void __launch_bounds__(kBlockMax)
gpuos_batch_kernel(const uint8_t* payload, const Tables* tab, volatile uint64_t* done_ring,
                   volatile uint64_t* retired_ring, uint64_t wait_limit_ns) {
  __shared__ uint32_t s_cb[kMaxReqPerBatch + 1];
  run_batch_cta(payload, tab, done_ring, nullptr, retired_ring, gridDim.x, wait_limit_ns, s_cb);
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

// CTAs 1..n: walk the staged batches in order.
__device__ void process_loop(const WorkerArgs& w, uint32_t* s_cb) {
  __shared__ int s_go;
  __shared__ uint32_t s_off;
  const uint32_t nproc = gridDim.x - 1;
  // bound for waiting on the next batch: the ingest stops the worker after
  // idle_ns without work, so waiting much longer than that means it is gone
  const uint64_t limit = w.idle_ns + 2000000000ull;
  for (uint64_t s = w.start_seq;; ++s) {
    if (threadIdx.x == 0) {
      int go = 0;
      const uint64_t t0 = globaltimer();
      unsigned backoff = 32;
      while (true) {
        if (ld_acquire_u64(&w.dctrl->ready) > s) { go = 1; break; }
        if (ld_acquire_u64(&w.dctrl->stop_at) <= s) break;
        if (globaltimer() - t0 > limit) {
          w.hctrl->err = w.hctrl->err | ERR_IDLE_EXIT;
          break;
        }
        __nanosleep(backoff);
        if (backoff < 2048) backoff <<= 1;
      }
      s_go = go;
      if (go) s_off = *reinterpret_cast<volatile uint32_t*>(&w.dctrl->ready_off[s % kDoneRing]);
    }
    __syncthreads();
    if (!s_go) return;
    const uint8_t* payload = w.ring + s_off;
    const BatchHdr* h = reinterpret_cast<const BatchHdr*>(payload);
    if (h->flags & BF_AFTER_PREV) {
      // a hazard with an earlier batch: wait (bounded) until every batch in
      // [wait_from, s) has completed
      if (threadIdx.x == 0) {
        const uint64_t t0 = globaltimer();
        for (uint64_t j = h->wait_from; j < s; ++j) {
          while ((ld_acquire_u64(&w.dctrl->done_dev[j % kDoneRing]) & ((1ull << 56) - 1)) != j + 1) {
            __nanosleep(256);
            if (globaltimer() - t0 > w.wait_limit_ns) break;
          }
        }
      }
      __syncthreads();
    }
    run_batch_cta(payload, w.tab, w.done_ring, w.dctrl->done_dev, w.retired_ring, nproc,
                  w.wait_limit_ns, s_cb);
    __syncthreads();
  }
}

extern "C" __global__ void __launch_bounds__(kBlockMax) gpuos_worker_kernel(WorkerArgs w) {
  __shared__ uint32_t s_cb[kMaxReqPerBatch + 1];
  if (blockIdx.x == 0) ingest_loop(w);
  else process_loop(w, s_cb);
}

}  // namespace gpuos

// ---- launch wrappers used by the host runtime ------------------------------
extern "C" cudaError_t gpuos_launch_batch(const uint8_t* payload, const gpuos::Tables* tab,
                                          volatile uint64_t* done_ring,
                                          volatile uint64_t* retired_ring, uint64_t wait_limit_ns,
                                          int grid, int block, cudaStream_t stream) {
  gpuos::gpuos_batch_kernel<<<grid, block, 0, stream>>>(payload, tab, done_ring, retired_ring,
                                                        wait_limit_ns);
  return cudaGetLastError();
}

extern "C" cudaError_t gpuos_launch_worker(const void* args, int grid, int block,
                                           cudaStream_t stream) {
  const gpuos::WorkerArgs* w = static_cast<const gpuos::WorkerArgs*>(args);
  gpuos::gpuos_worker_kernel<<<grid, block, 0, stream>>>(*w);
  return cudaGetLastError();
}

extern "C" cudaError_t gpuos_occupancy(int block, int* batch_blocks_per_sm,
                                       int* worker_blocks_per_sm) {
  cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(
      batch_blocks_per_sm, gpuos::gpuos_batch_kernel, block, 0);
  if (e != cudaSuccess) return e;
  return cudaOccupancyMaxActiveBlocksPerMultiprocessor(worker_blocks_per_sm,
                                                       gpuos::gpuos_worker_kernel, block, 0);
}

extern "C" size_t gpuos_worker_args_size() { return sizeof(gpuos::WorkerArgs); }
