// Custom expressions: NVRTC compiles the registered expression strings into
// the device functions gpuos_jit_op0..15, and the driver's linker joins them
// to the prebuilt relocatable batch kernel (jit_kernel.cu, embedded in this
// library as gpuos_jit_cubin).  Replaces the reference's per-expression NVRTC
// kernels (pytorch_ext/gpuos_ext.cpp:625-692), which it installs one Task per
// request; here custom requests are batched like every other request.
//
// NVRTC is loaded with dlopen and the driver entry points through the
// runtime (cudaGetDriverEntryPoint), so the library links against neither.
#include "jit.h"

#include <cuda.h>
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nvrtc.h>

#include <cstdlib>
#include <mutex>
#include <string>
#include <vector>

#include "runtime.h"

extern "C" const unsigned char gpuos_jit_cubin[];
extern "C" const unsigned long long gpuos_jit_cubin_size;

namespace gpuos {
namespace {

struct Nvrtc {
  void* h = nullptr;
  decltype(&::nvrtcCreateProgram) create = nullptr;
  decltype(&::nvrtcCompileProgram) compile = nullptr;
  decltype(&::nvrtcGetProgramLogSize) log_size = nullptr;
  decltype(&::nvrtcGetProgramLog) log = nullptr;
  decltype(&::nvrtcGetCUBINSize) cubin_size = nullptr;
  decltype(&::nvrtcGetCUBIN) cubin = nullptr;
  decltype(&::nvrtcDestroyProgram) destroy = nullptr;
  decltype(&::nvrtcGetErrorString) err = nullptr;
  std::string why;  // why NVRTC is unavailable
};

Nvrtc& nvrtc() {
  static Nvrtc n;
  static std::once_flag once;
  std::call_once(once, [] {
    std::vector<std::string> names = {"libnvrtc.so.12", "libnvrtc.so"};
    const char* home = std::getenv("CUDA_HOME");
    names.push_back(std::string(home ? home : "/usr/local/cuda") + "/lib64/libnvrtc.so.12");
    for (const auto& nm : names) {
      n.h = dlopen(nm.c_str(), RTLD_NOW | RTLD_LOCAL);
      if (n.h) break;
    }
    if (!n.h) {
      n.why = "NVRTC (libnvrtc.so.12) is not available";
      return;
    }
    auto sym = [&](const char* s) { return dlsym(n.h, s); };
    n.create = reinterpret_cast<decltype(n.create)>(sym("nvrtcCreateProgram"));
    n.compile = reinterpret_cast<decltype(n.compile)>(sym("nvrtcCompileProgram"));
    n.log_size = reinterpret_cast<decltype(n.log_size)>(sym("nvrtcGetProgramLogSize"));
    n.log = reinterpret_cast<decltype(n.log)>(sym("nvrtcGetProgramLog"));
    n.cubin_size = reinterpret_cast<decltype(n.cubin_size)>(sym("nvrtcGetCUBINSize"));
    n.cubin = reinterpret_cast<decltype(n.cubin)>(sym("nvrtcGetCUBIN"));
    n.destroy = reinterpret_cast<decltype(n.destroy)>(sym("nvrtcDestroyProgram"));
    n.err = reinterpret_cast<decltype(n.err)>(sym("nvrtcGetErrorString"));
    if (!n.create || !n.compile || !n.log_size || !n.log || !n.cubin_size || !n.cubin ||
        !n.destroy || !n.err) {
      n.why = "NVRTC library lacks an entry point";
      n.h = nullptr;
    }
  });
  return n;
}

// An expression is spliced into `return (float)(<expr>);`: keep it one
// expression.
void check_expression(const std::string& e) {
  if (e.empty()) throw GError(GPUOS_EINVAL, "empty expression");
  for (char c : e)
    if (c == ';' || c == '{' || c == '}' || c == '#' || c == '\\' || c == '"' || c == '\'')
      throw GError(GPUOS_EINVAL, std::string("expression may not contain '") + c + "': " + e);
  if (e.find("//") != std::string::npos || e.find("/*") != std::string::npos)
    throw GError(GPUOS_EINVAL, "expression may not contain comments: " + e);
}

std::string ops_source(const std::vector<std::string>& exprs) {
  // gpuos_keep_f32 / _f16 / _bf16: the value a fused chain's intermediate
  // result would have had in memory.  fp32: an add of -0.0 (exact for every
  // value) with an explicit rounding mode, which the code generator never
  // contracts with the multiply that produced the value, so the product is
  // rounded on its own as in the unfused chain; fp16 / bf16: the rounding of
  // the store (cvt.rn).
  std::string s =
      "// custom expressions of one executor, A..D the operands\n"
      "#define INFINITY __int_as_float(0x7f800000)\n"
      "#define NAN __int_as_float(0x7fffffff)\n"
      "static __device__ __forceinline__ float gpuos_keep_f32(float x) {\n"
      "  float y; asm(\"add.rn.f32 %0, %1, 0f80000000;\" : \"=f\"(y) : \"f\"(x)); return y;\n}\n"
      "static __device__ __forceinline__ float gpuos_keep_f16(float x) {\n"
      "  float y; asm(\"{ .reg .b16 h; cvt.rn.f16.f32 h, %1; cvt.f32.f16 %0, h; }\" "
      ": \"=f\"(y) : \"f\"(x)); return y;\n}\n"
      "static __device__ __forceinline__ float gpuos_keep_bf16(float x) {\n"
      "  unsigned u; asm(\"{ .reg .b16 h, z; cvt.rn.bf16.f32 h, %1; mov.b16 z, 0; "
      "mov.b32 %0, {z, h}; }\" : \"=r\"(u) : \"f\"(x)); return __uint_as_float(u);\n}\n";
  for (int k = 0; k < kJitSlots; ++k) {
    s += "extern \"C\" __device__ float gpuos_jit_op" + std::to_string(k) +
         "(float A, float B, float C, float D, float p0, float p1) {\n"
         "  (void)A; (void)B; (void)C; (void)D; (void)p0; (void)p1;\n"
         "  return (float)(";
    s += k < (int)exprs.size() ? exprs[k] : std::string("A");
    s += ");\n}\n";
  }
  return s;
}

template <class F>
F driver_fn(const char* name) {
  void* p = nullptr;
  cudaDriverEntryPointQueryResult q;
  cudaError_t e = cudaGetDriverEntryPoint(name, &p, cudaEnableDefault, &q);
  if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || !p)
    throw GError(GPUOS_ECUDA, std::string("driver entry point not found: ") + name);
  return reinterpret_cast<F>(p);
}

void cu_check(CUresult r, const char* what) {
  if (r == CUDA_SUCCESS) return;
  const char* msg = nullptr;
  auto get = driver_fn<CUresult (*)(CUresult, const char**)>("cuGetErrorString");
  get(r, &msg);
  throw GError(GPUOS_ECUDA, std::string(what) + ": " + (msg ? msg : "CUDA driver error"));
}

}  // namespace

std::vector<char> jit_compile(const std::vector<std::string>& exprs) {
  Nvrtc& n = nvrtc();
  if (!n.h) throw GError(GPUOS_EUNSUPPORTED, n.why);
  if ((int)exprs.size() > kJitSlots)
    throw GError(GPUOS_EINVAL, "at most " + std::to_string(kJitSlots) + " custom expressions");
  for (const auto& e : exprs) check_expression(e);
  const std::string src = ops_source(exprs);
  nvrtcProgram prog;
  nvrtcResult r = n.create(&prog, src.c_str(), "gpuos_jit_ops.cu", 0, nullptr, nullptr);
  if (r != NVRTC_SUCCESS) throw GError(GPUOS_ENVRTC, std::string("nvrtc: ") + n.err(r));
  const char* opts[] = {"--gpu-architecture=sm_100a", "--relocatable-device-code=true",
                        "--std=c++17"};
  r = n.compile(prog, 3, opts);
  if (r != NVRTC_SUCCESS) {
    size_t ls = 0;
    n.log_size(prog, &ls);
    std::string log(ls, '\0');
    if (ls) n.log(prog, &log[0]);
    n.destroy(&prog);
    throw GError(GPUOS_ENVRTC, "nvrtc could not compile the expression: " + log);
  }
  size_t cs = 0;
  n.cubin_size(prog, &cs);
  std::vector<char> cubin(cs);
  n.cubin(prog, cubin.data());
  n.destroy(&prog);
  return cubin;
}

JitKernel jit_link(const std::vector<char>& ops_cubin) {
  auto linkCreate = driver_fn<CUresult (*)(unsigned, CUjit_option*, void**, CUlinkState*)>(
      "cuLinkCreate");
  auto linkAddData = driver_fn<CUresult (*)(CUlinkState, CUjitInputType, void*, size_t,
                                            const char*, unsigned, CUjit_option*, void**)>(
      "cuLinkAddData");
  auto linkComplete = driver_fn<CUresult (*)(CUlinkState, void**, size_t*)>("cuLinkComplete");
  auto linkDestroy = driver_fn<CUresult (*)(CUlinkState)>("cuLinkDestroy");
  auto moduleLoad = driver_fn<CUresult (*)(CUmodule*, const void*)>("cuModuleLoadData");
  auto getFunction = driver_fn<CUresult (*)(CUfunction*, CUmodule, const char*)>(
      "cuModuleGetFunction");
  CUlinkState ls = nullptr;
  cu_check(linkCreate(0, nullptr, nullptr, &ls), "cuLinkCreate");
  JitKernel k;
  try {
    cu_check(linkAddData(ls, CU_JIT_INPUT_CUBIN, const_cast<unsigned char*>(gpuos_jit_cubin),
                         (size_t)gpuos_jit_cubin_size, "gpuos_jit_kernel", 0, nullptr, nullptr),
             "cuLinkAddData (batch kernel)");
    cu_check(linkAddData(ls, CU_JIT_INPUT_CUBIN, const_cast<char*>(ops_cubin.data()),
                         ops_cubin.size(), "gpuos_jit_ops", 0, nullptr, nullptr),
             "cuLinkAddData (expressions)");
    void* out = nullptr;
    size_t outsz = 0;
    cu_check(linkComplete(ls, &out, &outsz), "cuLinkComplete");
    CUmodule mod = nullptr;
    cu_check(moduleLoad(&mod, out), "cuModuleLoadData");
    k.module = mod;
    CUfunction fn = nullptr;
    cu_check(getFunction(&fn, mod, "gpuos_jit_batch_kernel"), "cuModuleGetFunction");
    k.function = fn;
  } catch (...) {
    if (k.module) driver_fn<CUresult (*)(CUmodule)>("cuModuleUnload")(static_cast<CUmodule>(k.module));
    linkDestroy(ls);
    throw;
  }
  linkDestroy(ls);
  return k;
}

void jit_launch(const JitKernel& k, int grid, int block, void* stream, const void* payload,
                const BatchHdr& hdr, BatchState* st, volatile uint64_t* done_ring,
                uint64_t wait_limit_ns) {
  auto launch = driver_fn<CUresult (*)(CUfunction, unsigned, unsigned, unsigned, unsigned,
                                       unsigned, unsigned, unsigned, CUstream, void**, void**)>(
      "cuLaunchKernel");
  BatchHdr h = hdr;
  const void* p = payload;
  void* args[] = {&p, &h, &st, &done_ring, &wait_limit_ns};
  cu_check(launch(static_cast<CUfunction>(k.function), (unsigned)grid, 1, 1, (unsigned)block, 1, 1,
                  0, static_cast<CUstream>(stream), args, nullptr),
           "cuLaunchKernel (custom expressions)");
}

void jit_unload(JitKernel& k) {
  if (!k.module) return;
  auto unload = driver_fn<CUresult (*)(CUmodule)>("cuModuleUnload");
  unload(static_cast<CUmodule>(k.module));
  k.module = nullptr;
  k.function = nullptr;
}

}  // namespace gpuos

// Compile `expr` with NVRTC only (no GPU needed): GPUOS_OK, GPUOS_ENVRTC with
// the compiler's log, or GPUOS_EUNSUPPORTED when NVRTC is not installed.
extern "C" int32_t gpuos_jit_check(const char* expr, int32_t arity) {
  try {
    if (!expr) throw gpuos::GError(GPUOS_EINVAL, "expression is NULL");
    if (arity < 1 || arity > 4) throw gpuos::GError(GPUOS_EINVAL, "arity must be 1 to 4");
    gpuos::jit_compile({std::string(expr)});
    return GPUOS_OK;
  } catch (const gpuos::GError& e) {
    gpuos::set_last_error(e.what());
    return e.code;
  } catch (const std::exception& e) {
    gpuos::set_last_error(e.what());
    return GPUOS_EINVAL;
  }
}
