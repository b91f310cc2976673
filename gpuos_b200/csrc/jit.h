// Custom expressions compiled at run time (jit.cpp).
#pragma once
#include <cstdint>
#include <string>
#include <vector>

#include "gpuos_abi.h"

namespace gpuos {

static constexpr int kJitSlots = 16;  // gpuos_jit_op0..15 (ops.cuh kJitOps)

struct JitKernel {
  void* module = nullptr;    // CUmodule
  void* function = nullptr;  // CUfunction of gpuos_jit_batch_kernel
};

// NVRTC: the device functions gpuos_jit_op<k> for exprs[k] (the rest return
// A), as a relocatable cubin.  Throws GError (GPUOS_ENVRTC with the compiler
// log, GPUOS_EUNSUPPORTED without NVRTC, GPUOS_EINVAL for a malformed string).
std::vector<char> jit_compile(const std::vector<std::string>& exprs);

// Link them to the embedded batch kernel and load the result into the
// current context.
JitKernel jit_link(const std::vector<char>& ops_cubin);

// Launch the linked batch kernel (the arguments of gpuos_batch_kernel).
void jit_launch(const JitKernel& k, int grid, int block, void* stream, const void* payload,
                const BatchHdr& hdr, BatchState* st, volatile uint64_t* done_ring,
                uint64_t wait_limit_ns);

void jit_unload(JitKernel& k);

void set_last_error(const char* msg);

}  // namespace gpuos
