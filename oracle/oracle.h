/* oracle.h — CPU restatement of the reference's aggregated small-op path.
 *
 * TEST INFRASTRUCTURE ONLY.  Only tests/, __graft_entry__.smoke() and the
 * cpu_baseline / --impl reference legs of bench.py use this library, always as
 * the checker or the timed CPU baseline, never as part of the product path.
 *
 * What it restates (paths relative to the Multi-V-VM/GPUOS repository):
 *   loads / stores         ld_as_float, st_from_float   src/persistent_kernel.cu:60-78
 *   op_batch op codes      add/mul/sub/div(B!=0)        src/persistent_kernel.cu:101-106
 *   elementwise formulas   the scheduler's JIT strings  pytorch_ext/scheduler.py:145-153,192-205,244-290
 *   reduce, last axis      thread-strided partial sums + smem tree   pytorch_ext/gpuos_ext.cpp:731-775
 *   reduce, generic        serial, first reduced axis fastest        pytorch_ext/gpuos_ext.cpp:777-805
 *   index decomposition    linear_to_offset             src/persistent_kernel.cu:20-31
 *                          (oracle_ew_refindex reproduces the reference's
 *                          broadcast defect for [B,1] operands; oracle_ew uses
 *                          torch broadcasting)
 *
 * Parity pins: the known-answer inputs of the reference's own tests
 * (src/host.cpp:219, test/online_switch.cpp:156, test/dual_slot_switch.cpp:138)
 * and the golden fixtures under tests/golden/.
 */
#ifndef GPUOS_ORACLE_H
#define GPUOS_ORACLE_H
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* same layout as gpuos_tensor / the reference TensorRef */
typedef struct or_tensor {
  void* data;
  int32_t dtype; /* 0 f32, 1 f16, 2 bf16, 4 f64 (exact mode only) */
  int32_t ndim;
  int64_t sizes[8];
  int64_t strides[8];
} or_tensor;

/* variant ids: the same numbering as the executor's operator ids */
enum {
  OR_ADD = 0, OR_MUL = 1, OR_SUB = 2, OR_DIV0 = 3, OR_DIV = 4, OR_MAX = 5, OR_MIN = 6,
  OR_POW = 7, OR_RELU = 8, OR_SIGMOID = 9, OR_TANH = 10, OR_EXP = 11, OR_LOG = 12,
  OR_SQRT = 13, OR_ABS = 14, OR_HARDSIGMOID = 15, OR_HARDSWISH = 16, OR_GELU = 17,
  OR_SIN = 18, OR_COS = 19, OR_LEAKY_RELU = 20, OR_CLAMP = 21, OR_ELU = 22,
  OR_SOFTPLUS = 23, OR_CLAMP_MIN = 24, OR_CLAMP_MAX = 25, OR_COPY = 26,
  OR_SUM = 32, OR_MEAN = 33
};

float oracle_op1(int variant, float a, float b, float p0, float p1);
uint16_t oracle_f32_to_f16(float x);
uint16_t oracle_f32_to_bf16(float x);
float oracle_f16_to_f32(uint16_t h);
float oracle_bf16_to_f32(uint16_t h);

/* out = op(a[, b]); a and b broadcast onto out's shape the torch way.
 * Returns 0, or -1 on a shape error. */
int oracle_ew(int variant, float p0, float p1, const or_tensor* a, const or_tensor* b,
              const or_tensor* out);

/* The same formulas in double precision, out must be float64 (dtype code 4,
 * the reference's kF64): the exact values fp32 results are measured against. */
double oracle_op1_exact(int variant, double a, double b, double p0, double p1);
int oracle_ew_exact(int variant, float p0, float p1, const or_tensor* a, const or_tensor* b,
                    const or_tensor* out);

/* The same with the reference's own index decomposition: every operand's
 * offset is decomposed over that operand's own (right-aligned) sizes, as
 * linear_to_offset does after fill_tensorref (gpuos_ext.cpp:147-165). */
int oracle_ew_refindex(int variant, float p0, float p1, const or_tensor* a, const or_tensor* b,
                       const or_tensor* out);

/* sum (mean != 0: mean) of x over axes into out, in the reference's
 * accumulation order; `threads` is the CTA size of the fast path (256). */
int oracle_reduce(int mean, const or_tensor* x, const or_tensor* out, const int32_t* axes,
                  int naxes, int keepdim, int threads);

/* one request of a stream, for the CPU baseline */
typedef struct or_req {
  int32_t kind; /* 0 elementwise, 1 reduce */
  int32_t variant;
  float p0, p1;
  int32_t has_b;
  int32_t naxes;
  int32_t keepdim;
  int32_t axes[8];
  int32_t pad;
  or_tensor a, b, out;
} or_req;

/* run n requests with up to nthreads threads (<= 0: all cores);
 * returns the number of threads used */
int oracle_run(const or_req* reqs, int n, int nthreads);

#ifdef __cplusplus
}
#endif
#endif
