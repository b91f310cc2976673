// The batch kernel for batches with custom expressions, built relocatable
// (-rdc): the operators of slots V_JIT_BASE + 0..15 are the external device
// functions gpuos_jit_op0..15, which the runtime compiles from the registered
// expression strings with NVRTC and links to this code with the driver's
// linker (runtime.cpp, JitOps).  Same batch format, chunking and completion
// as gpuos_batch_kernel, and every body of it as well, so that a batch that
// mixes custom expressions with precompiled operators and reductions runs in
// one launch.
#define GPUOS_JIT_LINK 1
#include "batch.cuh"

namespace gpuos {

extern "C" __global__ void __launch_bounds__(kCtaThreads, kMinCtasPerSm)
gpuos_jit_batch_kernel(const uint8_t* payload, const BatchHdr hdr, BatchState* st,
                       volatile uint64_t* done_ring, uint64_t wait_limit_ns) {
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
  const uint32_t count = warp_batch(ex, blockIdx.x * kWarpsPerCta + warp,
                                    gridDim.x * kWarpsPerCta, &ext[warp], &ss);
  // without stage barriers nothing waits on the batch's counters: the kernel's
  // completion completes the batch, and its warps leave as soon as they are done
  if (posts_own_errors(ex)) return;
  cta_leave_batch(ex, &cta_chunks, count, gridDim.x, nullptr);
}

}  // namespace gpuos
