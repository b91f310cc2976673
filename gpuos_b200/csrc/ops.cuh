// Builtin micro-op expressions, dtype load/store and 8-wide vector helpers.
//
// Every builtin elementwise op is the fp32 expression the reference evaluates
// for it, written with the same operators in the same order, so that the
// compiler's default contraction of a*b+c into fma (on in both nvcc and
// NVRTC, which the reference uses without flags) gives the same rounding:
//   add/mul/sub and the B==0 division rule: op_batch,
//     src/persistent_kernel.cu:101-106
//   the other ops: the expression strings of pytorch_ext/scheduler.py:145-153,
//     192-205, 244-290, with the literal parameters replaced by p0/p1.
// Loads widen fp16/bf16 exactly; stores round to nearest even
// (ld_as_float / st_from_float, src/persistent_kernel.cu:60-78).
#pragma once
#include "gpuos_abi.h"
#include <cuda_fp16.h>
#include <cuda_bf16.h>

namespace gpuos {

// Custom expressions (variants V_JIT_BASE + k): in the relocatable batch
// kernel for custom expressions (GPUOS_JIT_LINK) these are external device
// functions, compiled from the expression strings by NVRTC and linked in at
// run time.
static constexpr int kJitOps = 16;
#ifdef GPUOS_JIT_LINK
extern "C" {
#define GPUOS_JIT_DECL(k) \
  __device__ float gpuos_jit_op##k(float A, float B, float C, float D, float p0, float p1);
GPUOS_JIT_DECL(0) GPUOS_JIT_DECL(1) GPUOS_JIT_DECL(2) GPUOS_JIT_DECL(3)
GPUOS_JIT_DECL(4) GPUOS_JIT_DECL(5) GPUOS_JIT_DECL(6) GPUOS_JIT_DECL(7)
GPUOS_JIT_DECL(8) GPUOS_JIT_DECL(9) GPUOS_JIT_DECL(10) GPUOS_JIT_DECL(11)
GPUOS_JIT_DECL(12) GPUOS_JIT_DECL(13) GPUOS_JIT_DECL(14) GPUOS_JIT_DECL(15)
#undef GPUOS_JIT_DECL
}
template <int K>
__device__ __forceinline__ float jit_op(float A, float B, float C, float D, float p0, float p1) {
#define GPUOS_JIT_CALL(k) if constexpr (K == k) return gpuos_jit_op##k(A, B, C, D, p0, p1);
  GPUOS_JIT_CALL(0) GPUOS_JIT_CALL(1) GPUOS_JIT_CALL(2) GPUOS_JIT_CALL(3)
  GPUOS_JIT_CALL(4) GPUOS_JIT_CALL(5) GPUOS_JIT_CALL(6) GPUOS_JIT_CALL(7)
  GPUOS_JIT_CALL(8) GPUOS_JIT_CALL(9) GPUOS_JIT_CALL(10) GPUOS_JIT_CALL(11)
  GPUOS_JIT_CALL(12) GPUOS_JIT_CALL(13) GPUOS_JIT_CALL(14) GPUOS_JIT_CALL(15)
#undef GPUOS_JIT_CALL
  return A;
}
#endif

template <int V>
__device__ __forceinline__ float op1(float A, float B, float p0, float p1) {
#ifdef GPUOS_JIT_LINK
  if constexpr (V >= V_JIT_BASE && V < V_JIT_BASE + kJitOps)
    return jit_op<V - V_JIT_BASE>(A, B, 0.f, 0.f, p0, p1);
  else
#endif
  if constexpr (V == V_ADD) return A + B;
  else if constexpr (V == V_MUL) return A * B;
  else if constexpr (V == V_SUB) return A - B;
  else if constexpr (V == V_DIV0) return (B != 0.f) ? (A / B) : 0.f;
  else if constexpr (V == V_DIV) return (A / B);
  else if constexpr (V == V_MAX) return (A > B ? A : B);
  else if constexpr (V == V_MIN) return (A < B ? A : B);
  else if constexpr (V == V_POW) return powf(A, B);
  else if constexpr (V == V_RELU) return (A > 0.f ? A : 0.f);
  else if constexpr (V == V_SIGMOID) return 1.f / (1.f + expf(-A));
  else if constexpr (V == V_TANH) return tanhf(A);
  else if constexpr (V == V_EXP) return expf(A);
  else if constexpr (V == V_LOG) return logf(A);
  else if constexpr (V == V_SQRT) return sqrtf(A);
  else if constexpr (V == V_ABS) return fabsf(A);
  else if constexpr (V == V_HARDSIGMOID) return fminf(fmaxf(0.2f * A + 0.5f, 0.f), 1.f);
  else if constexpr (V == V_HARDSWISH) return A * fminf(fmaxf(A / 6.f + 0.5f, 0.f), 1.f);
  else if constexpr (V == V_GELU)
    return 0.5f * A * (1.f + tanhf(0.79788456f * (A + 0.044715f * A * A * A)));
  else if constexpr (V == V_SIN) return sinf(A);
  else if constexpr (V == V_COS) return cosf(A);
  else if constexpr (V == V_LEAKY_RELU) return (A >= 0.f ? A : p0 * A);
  else if constexpr (V == V_CLAMP) return fminf(fmaxf(A, p0), p1);
  else if constexpr (V == V_ELU) return (A > 0.f ? A : p0 * (expf(A) - 1.f));
  else if constexpr (V == V_SOFTPLUS) return (log1pf(expf(p0 * A)) / p0);
  else if constexpr (V == V_CLAMP_MIN) return fmaxf(A, p0);
  else if constexpr (V == V_CLAMP_MAX) return fminf(A, p0);
  else return A;  // V_COPY
}

#define GPUOS_CASE1(V) case V: r = op1<V>(A, B, p0, p1); return true;
// The elementwise variants a kernel instantiates.  GPUOS_ALL_EW gets the
// vector bodies: the precompiled operators, or in the kernel linked with
// custom expressions the custom slots.  GPUOS_APPLY_EW is the per-element
// switch of the general and 2-D tile bodies: in the linked kernel the custom
// slots and the precompiled operators, so that a batch mixing both runs in
// one launch (its precompiled requests through those bodies).
#define GPUOS_BUILTIN_EW(M) \
  M(V_ADD) M(V_MUL) M(V_SUB) M(V_DIV0) M(V_DIV) M(V_MAX) M(V_MIN) M(V_POW) \
  M(V_RELU) M(V_SIGMOID) M(V_TANH) M(V_EXP) M(V_LOG) M(V_SQRT) M(V_ABS) \
  M(V_HARDSIGMOID) M(V_HARDSWISH) M(V_GELU) M(V_SIN) M(V_COS) M(V_LEAKY_RELU) \
  M(V_CLAMP) M(V_ELU) M(V_SOFTPLUS) M(V_CLAMP_MIN) M(V_CLAMP_MAX) M(V_COPY)
#ifdef GPUOS_JIT_LINK
#define GPUOS_JIT_EW(M) \
  M(V_JIT_BASE + 0) M(V_JIT_BASE + 1) M(V_JIT_BASE + 2) M(V_JIT_BASE + 3) \
  M(V_JIT_BASE + 4) M(V_JIT_BASE + 5) M(V_JIT_BASE + 6) M(V_JIT_BASE + 7) \
  M(V_JIT_BASE + 8) M(V_JIT_BASE + 9) M(V_JIT_BASE + 10) M(V_JIT_BASE + 11) \
  M(V_JIT_BASE + 12) M(V_JIT_BASE + 13) M(V_JIT_BASE + 14) M(V_JIT_BASE + 15)
#define GPUOS_ALL_EW(M) GPUOS_JIT_EW(M)
#define GPUOS_APPLY_EW(M) GPUOS_BUILTIN_EW(M) GPUOS_JIT_EW(M)
#else
#define GPUOS_ALL_EW(M) GPUOS_BUILTIN_EW(M)
#define GPUOS_APPLY_EW(M) GPUOS_BUILTIN_EW(M)
#endif

__device__ __forceinline__ bool ew_apply1(int v, float A, float B, float& r, float p0, float p1) {
  switch (v) {
    GPUOS_APPLY_EW(GPUOS_CASE1)
    default: return false;
  }
}

#ifdef GPUOS_JIT_LINK
// A custom expression of up to four operands (RF_NARY requests).
#define GPUOS_CASE4(V) case V: r = jit_op<V - V_JIT_BASE>(A, B, C, D, p0, p1); return true;
__device__ __forceinline__ bool ew_apply4(int v, float A, float B, float C, float D, float& r,
                                          float p0, float p1) {
  switch (v) {
    GPUOS_JIT_EW(GPUOS_CASE4)
    default: return false;
  }
}
#undef GPUOS_CASE4
#endif

// Groups of 4 elements each lane handles per iteration of the vector loop
// (the loop keeps the next iteration's loads in flight while it computes the
// current one, so twice this many groups are live): 2 for the cheap,
// memory-bound operators, 1 for those with a division, square root or
// transcendental (compute heavy: a smaller body keeps the instruction cache
// warm and the register budget low).
template <int V>
__device__ __forceinline__ constexpr int op_unroll() {
  return (V >= V_JIT_BASE || V == V_POW || V == V_SIGMOID || V == V_TANH || V == V_EXP || V == V_LOG ||
          V == V_GELU || V == V_SIN || V == V_COS || V == V_ELU || V == V_SOFTPLUS ||
          V == V_DIV || V == V_DIV0 || V == V_SQRT || V == V_HARDSWISH)
             ? 1
             : 2;
}

template <int V>
__device__ __forceinline__ void op4(const float* A, const float* B, float* R, float p0, float p1) {
#pragma unroll
  for (int k = 0; k < 4; ++k) R[k] = op1<V>(A[k], B[k], p0, p1);
}

// ---- scalar load / store (element offsets) -------------------------------
__device__ __forceinline__ float ld1(uint64_t base, int dt, int64_t off) {
  if (dt == kF32) return reinterpret_cast<const float*>(base)[off];
  if (dt == kF16) return __half2float(reinterpret_cast<const __half*>(base)[off]);
  return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(base)[off]);
}

__device__ __forceinline__ void st1(uint64_t base, int dt, int64_t off, float v) {
  if (dt == kF32) reinterpret_cast<float*>(base)[off] = v;
  else if (dt == kF16) reinterpret_cast<__half*>(base)[off] = __float2half_rn(v);
  else reinterpret_cast<__nv_bfloat16*>(base)[off] = __float2bfloat16(v);
}

// ---- raw loads: the bits of 4 (or 1) elements, with nothing computed from
// them, so that every load of a round is issued before the first one is
// waited on (a conversion right after each load would wait a full memory
// round trip per load); cvt4 / cvt1 turn the bits into floats where they are
// used.  A 16-bit type fills the low two words (or the low 16 bits).
__device__ __forceinline__ uint4 ld4_raw(uint64_t base, int dt, int64_t e) {
  if (dt == kF32) return *reinterpret_cast<const uint4*>(reinterpret_cast<const float*>(base) + e);
  const uint2 u = *reinterpret_cast<const uint2*>(reinterpret_cast<const uint16_t*>(base) + e);
  return make_uint4(u.x, u.y, 0u, 0u);
}

__device__ __forceinline__ uint32_t ld1_raw(uint64_t base, int dt, int64_t off) {
  if (dt == kF32) return reinterpret_cast<const uint32_t*>(base)[off];
  return reinterpret_cast<const uint16_t*>(base)[off];
}

__device__ __forceinline__ float cvt1(uint32_t r, int dt) {
  if (dt == kF32) return __uint_as_float(r);
  if (dt == kF16) return __half2float(__ushort_as_half((unsigned short)r));
  return __uint_as_float(r << 16);
}

__device__ __forceinline__ void bf2_to_f(uint32_t u, float& lo, float& hi);

__device__ __forceinline__ void cvt4(uint4 r, int dt, float* v) {
  if (dt == kF32) {
    v[0] = __uint_as_float(r.x); v[1] = __uint_as_float(r.y);
    v[2] = __uint_as_float(r.z); v[3] = __uint_as_float(r.w);
  } else if (dt == kF16) {
    float2 f = __half22float2(*reinterpret_cast<const __half2*>(&r.x));
    v[0] = f.x; v[1] = f.y;
    f = __half22float2(*reinterpret_cast<const __half2*>(&r.y));
    v[2] = f.x; v[3] = f.y;
  } else {
    bf2_to_f(r.x, v[0], v[1]);
    bf2_to_f(r.y, v[2], v[3]);
  }
}

__device__ __forceinline__ void bf2_to_f(uint32_t u, float& lo, float& hi) {
  lo = __uint_as_float(u << 16);
  hi = __uint_as_float(u & 0xffff0000u);
}

// 4-element vector load / store: `e` is a multiple of 4 and the address is
// aligned to 4 elements (16 bytes for fp32, 8 for fp16 / bf16).
__device__ __forceinline__ void ld4(uint64_t base, int dt, int64_t e, float* v) {
  if (dt == kF32) {
    const float4 x = *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(base) + e);
    v[0] = x.x; v[1] = x.y; v[2] = x.z; v[3] = x.w;
  } else {
    const uint2 u = *reinterpret_cast<const uint2*>(reinterpret_cast<const uint16_t*>(base) + e);
    if (dt == kF16) {
      float2 f = __half22float2(*reinterpret_cast<const __half2*>(&u.x));
      v[0] = f.x; v[1] = f.y;
      f = __half22float2(*reinterpret_cast<const __half2*>(&u.y));
      v[2] = f.x; v[3] = f.y;
    } else {
      bf2_to_f(u.x, v[0], v[1]);
      bf2_to_f(u.y, v[2], v[3]);
    }
  }
}

__device__ __forceinline__ uint32_t f2_to_h2(float a, float b);
__device__ __forceinline__ uint32_t f2_to_bf2(float a, float b);

__device__ __forceinline__ void st4(uint64_t base, int dt, int64_t e, const float* v) {
  if (dt == kF32) {
    *reinterpret_cast<float4*>(reinterpret_cast<float*>(base) + e) = make_float4(v[0], v[1], v[2], v[3]);
  } else {
    uint2 u;
    if (dt == kF16) {
      u.x = f2_to_h2(v[0], v[1]);
      u.y = f2_to_h2(v[2], v[3]);
    } else {
      u.x = f2_to_bf2(v[0], v[1]);
      u.y = f2_to_bf2(v[2], v[3]);
    }
    *reinterpret_cast<uint2*>(reinterpret_cast<uint16_t*>(base) + e) = u;
  }
}

__device__ __forceinline__ uint32_t f2_to_h2(float a, float b) {
  __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}
__device__ __forceinline__ uint32_t f2_to_bf2(float a, float b) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

}  // namespace gpuos
