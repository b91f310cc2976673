// Launcher for the reference's own op_batch device function — PARITY CHECKER
// ONLY (test infrastructure; nothing in gpuos_b200/ links or loads it).
//
// oracle/build_ref.py compiles this file with nvcc against the reference's
// sources where they lie: src/persistent_kernel.cu is included as a
// translation-unit source (the include path points at the reference's src/),
// so op_batch (src/persistent_kernel.cu:81-112) is compiled exactly as the
// reference's extension build compiles it (pytorch_ext/setup.py:17-33 nvcc
// flags, with the B200 gencode).  The output, oracle/_ref/libref_opbatch.so,
// stays out of git and is used only by tests/golden/gen_ref_fixtures.py to
// record the reference's outputs on a B200.
//
// The reference runs each batch Task on one CTA of its persistent worker
// (src/persistent_kernel.cu:133-200: thread 0 claims the Task, every thread
// of the CTA calls the operator).  Here one CTA per shard Task calls op_batch
// directly: no persistent kernel, no queue, no device function pointers.
#include "persistent_kernel.cu"

extern "C" __global__ void gpuos_ref_op_batch_kernel(const Task* shards) {
  op_batch(shards[blockIdx.x]);
}

// shards: device array of `n` batch Tasks (op 10, numel = sub-task count,
// in0.data = device array of sub-Tasks).  Returns a cudaError_t.
extern "C" int gpuos_ref_launch_op_batch(const void* shards, int n, int threads, void* stream) {
  if (n <= 0) return 0;
  gpuos_ref_op_batch_kernel<<<n, threads, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const Task*>(shards));
  return static_cast<int>(cudaGetLastError());
}

extern "C" int gpuos_ref_task_size() { return static_cast<int>(sizeof(Task)); }
