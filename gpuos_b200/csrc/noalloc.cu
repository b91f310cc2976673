// gpuos_reduce_rows_noalloc: a sum / mean over the last dimension of a
// row-major [rows, cols] tensor for callers that cannot allocate device memory.
//
// It runs the executor's row-reduction body (red_rows, the code the batch
// kernel runs for a contiguous last-dim reduction) in a kernel of its own, and
// plans rows exactly as the executor does, so its results are those of
// gpuos_submit_reduce on the same input.  Rows longer than 8192 columns are
// split into segments whose partial sums and combine counters live in
// g_noalloc_scratch below, a file-scope device array of 1 MiB that every GPU
// loading this library holds until the process exits.  Nothing is allocated:
// no cudaMalloc, no cudaFree, no allocating library routine.
//
//  * limits: at most 65,536 split rows and 196,608 (row, segment) partial sums
//    per call (rows x ceil(cols / 8192) when cols > 8192); larger calls
//    return GPUOS_EINVAL before any device work.  Rows of at most 8192 columns
//    use no scratch and have no such limit.
//  * set-up: the first call on a device (the current device) looks up the
//    array's device address with cudaGetSymbolAddress, once per device, and
//    caches it; make that first call before any stream capture.
//  * sharing: every call uses the same array, which keeps the last call's
//    contents.  The combine counters must start at zero, so each call clears
//    the ones it uses with cudaMemsetAsync on its stream before the kernel.
//    Calls that overlap on the GPU (different streams, or concurrent threads)
//    race on the array; serialise them.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdio>
#include <mutex>
#include <string>

#include "../../include/gpuos_b200.h"
#include "executor.cuh"

namespace gpuos {
void set_last_error(const char* msg);  // runtime.cpp: message for gpuos_last_error()
}

namespace {

using namespace gpuos;

constexpr uint32_t kNaCounters = 65536;    // split rows per call
constexpr uint32_t kNaPartials = 196608;   // (row, segment) partial sums per call
constexpr size_t kNaBytes = (size_t)kNaCounters * 4 + (size_t)kNaPartials * 4;  // 1 MiB
constexpr int64_t kSeg = 8192;             // columns per segment (the executor's split)
constexpr int kNaThreads = 256;
constexpr int kMaxDevices = 64;

// In host code this name is only a handle for cudaGetSymbolAddress, not a
// device address.
static __device__ __align__(256) uint8_t g_noalloc_scratch[kNaBytes];

std::mutex g_na_mu;
uint8_t* g_na_base[kMaxDevices];  // device address of g_noalloc_scratch, per device
int g_na_sms[kMaxDevices];

__global__ void __launch_bounds__(kNaThreads)
gpuos_rows_noalloc_kernel(ReqView q, float* partials, uint32_t* counters, uint32_t nchunk,
                          int mean) {
  Exec ex{};
  ex.scratch = partials;
  ex.counters = counters;
  ex.lane = threadIdx.x & 31;
  const uint32_t warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const uint32_t nwarps = (gridDim.x * blockDim.x) >> 5;
  for (uint32_t k = warp; k < nchunk; k += nwarps) red_rows(ex, q, mean != 0, k);
}

int32_t fail(int32_t code, const std::string& msg) {
  set_last_error(("gpuos_reduce_rows_noalloc: " + msg).c_str());
  return code;
}

int esz(int32_t dt) { return dt == kF32 ? 4 : 2; }

uint32_t pow2_ceil(uint64_t x) {
  uint32_t p = 1;
  while (p < x && p < (1u << 30)) p <<= 1;
  return p;
}

}  // namespace

extern "C" int32_t gpuos_reduce_rows_noalloc(int32_t variant, const void* x, int32_t x_dtype,
                                             int64_t rows, int64_t cols, int64_t row_stride,
                                             void* out, int32_t out_dtype, void* stream) {
  if (variant != V_SUM && variant != V_MEAN)
    return fail(GPUOS_EINVAL, "variant must be sum or mean");
  auto dt_ok = [](int32_t d) { return d == kF32 || d == kF16 || d == kBF16; };
  if (!dt_ok(x_dtype) || !dt_ok(out_dtype))
    return fail(GPUOS_EINVAL, "dtype must be f32, f16 or bf16");
  if (rows < 0 || cols < 0) return fail(GPUOS_EINVAL, "negative shape");
  if (rows > 1 && row_stride < cols) return fail(GPUOS_EINVAL, "row_stride < cols");
  if (rows == 0) return GPUOS_OK;
  if (!out || (cols > 0 && !x)) return fail(GPUOS_EINVAL, "NULL data pointer");

  // the executor's plan for a contiguous last-dim reduction
  ReqView q{};
  q.a = reinterpret_cast<uint64_t>(x);
  q.o = reinterpret_cast<uint64_t>(out);
  q.numel = rows;
  q.inner = cols;
  q.sa_row = row_stride;
  q.so_row = 1;
  q.sa_in = 1;
  q.op = variant;
  q.kind = RK_RED;
  q.layout = RL_ROWS;
  q.dta = q.dtb = x_dtype;
  q.dto = out_dtype;
  q.nseg = 1;
  if ((q.a & 15) == 0 && (rows == 1 || ((row_stride * esz(x_dtype)) & 15) == 0)) q.flags |= RF_VEC;
  uint64_t nchunk = 0;
  if (cols <= kSeg) {
    const uint32_t G = std::min<uint32_t>(32, pow2_ceil((uint64_t)std::max<int64_t>(1, (cols + 15) / 16)));
    const uint32_t per = 32 / G;
    uint64_t rpc = (uint64_t)std::max<int64_t>(1, kSeg / std::max<int64_t>(cols, 1));
    rpc = std::max<uint64_t>(per, rpc / per * per);
    q.rg = G;
    q.chunk = (uint32_t)rpc;
    nchunk = ((uint64_t)rows + rpc - 1) / rpc;
  } else {
    q.rg = 32;
    q.chunk = (uint32_t)kSeg;
    q.nseg = (uint32_t)((cols + kSeg - 1) / kSeg);
    if ((uint64_t)rows > kNaCounters || (uint64_t)rows * q.nseg > kNaPartials) {
      char buf[256];
      std::snprintf(buf, sizeof(buf),
                    "%lld rows x %u segments exceed the static scratch (at most %u split rows "
                    "and %u partial sums per call)",
                    (long long)rows, q.nseg, kNaCounters, kNaPartials);
      return fail(GPUOS_EINVAL, buf);
    }
    nchunk = (uint64_t)rows * q.nseg;
  }
  if (nchunk > 0x7fffffffull) return fail(GPUOS_EINVAL, "too many rows");

  // set-up, once per device: the device address of the scratch array
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(GPUOS_ECUDA, std::string("cudaGetDevice: ") + cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices) return fail(GPUOS_EINVAL, "device index out of range");
  uint8_t* base = nullptr;
  int sms = 0;
  {
    std::lock_guard<std::mutex> lk(g_na_mu);
    if (!g_na_base[dev]) {
      void* p = nullptr;
      e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
      if (e != cudaSuccess)
        return fail(GPUOS_ECUDA, std::string("cudaGetSymbolAddress: ") + cudaGetErrorString(e));
      int n = 0;
      e = cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
      if (e != cudaSuccess)
        return fail(GPUOS_ECUDA, std::string("cudaDeviceGetAttribute: ") + cudaGetErrorString(e));
      g_na_sms[dev] = n;
      g_na_base[dev] = static_cast<uint8_t*>(p);
    }
    base = g_na_base[dev];
    sms = g_na_sms[dev];
  }
  uint32_t* counters = reinterpret_cast<uint32_t*>(base);
  float* partials = reinterpret_cast<float*>(base + (size_t)kNaCounters * 4);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (q.nseg > 1) {
    e = cudaMemsetAsync(counters, 0, (size_t)rows * 4, s);
    if (e != cudaSuccess)
      return fail(GPUOS_ECUDA, std::string("cudaMemsetAsync: ") + cudaGetErrorString(e));
  }
  const uint64_t warps_per_cta = kNaThreads / 32;
  uint64_t grid = (nchunk + warps_per_cta - 1) / warps_per_cta;
  grid = std::min<uint64_t>(grid, (uint64_t)std::max(sms, 1) * 8);
  gpuos_rows_noalloc_kernel<<<(unsigned)grid, kNaThreads, 0, s>>>(q, partials, counters,
                                                                  (uint32_t)nchunk,
                                                                  variant == V_MEAN ? 1 : 0);
  e = cudaGetLastError();
  if (e != cudaSuccess) return fail(GPUOS_ECUDA, std::string("launch: ") + cudaGetErrorString(e));
  return GPUOS_OK;
}
