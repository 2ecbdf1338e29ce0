// Shared host/device definitions for the b2msl kernels (status codes, dtype
// tags, per-thread error text, the device status word every bounded wait writes).
#pragma once
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <cstdint>
#include <cstdio>
#include <string>

#include "../../include/b2msl.h"

namespace b2 {

// Thread-local text behind b2_last_error(); set by every failing entry point.
void set_error(const char* fmt, ...);
void clear_error();

// Streaming-multiprocessor count of the current device, cached per device
// ordinal behind std::call_once (safe from several host threads). 148 on B200.
int device_sm_count();

// Device status bits, OR-ed into a per-module __device__ word by kernels and
// read back with b2_device_status().
enum : uint32_t {
  DEV_OK = 0u,
  DEV_TIMEOUT_TMA = 1u << 0,    // a consumer waited too long for a TMA fill
  DEV_TIMEOUT_MMA = 1u << 1,    // a waiter gave up on a tensor-core commit
  DEV_TIMEOUT_EPI = 1u << 2,    // an epilogue/softmax waiter gave up
  DEV_TIMEOUT_SLOT = 1u << 3,   // a producer gave up waiting for a free slot
};

// Upper bound on any single spin inside a kernel. Every legitimate wait in
// these kernels is microseconds; one second means the pipeline is wedged.
constexpr unsigned long long kWaitLimitNs = 1000ull * 1000ull * 1000ull;

inline int dtype_size(int dt) {
  switch (dt) {
    case B2_F32: return 4;
    case B2_F16: return 2;
    case B2_BF16: return 2;
    case B2_I64: return 8;
    default: return 0;
  }
}

inline const char* dtype_name(int dt) {
  switch (dt) {
    case B2_F32: return "f32";
    case B2_F16: return "f16";
    case B2_BF16: return "bf16";
    case B2_I64: return "i64";
    default: return "?";
  }
}

// Converters used by every kernel family: load any of the three float types
// as fp32, store fp32 as any of them (round-to-nearest-even).
template <typename T> __device__ __forceinline__ float to_f32(T v);
template <> __device__ __forceinline__ float to_f32<float>(float v) { return v; }
template <> __device__ __forceinline__ float to_f32<__half>(__half v) { return __half2float(v); }
template <> __device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }

template <typename T> __device__ __forceinline__ T from_f32(float v);
template <> __device__ __forceinline__ float from_f32<float>(float v) { return v; }
template <> __device__ __forceinline__ __half from_f32<__half>(float v) { return __float2half_rn(v); }
template <> __device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }

// Epilogue activations shared by the GEMM kernels. ReLU propagates NaN, as
// torch.relu does (the reference's epilogue maps tl.maximum to a NaN-propagating max).
__device__ __forceinline__ float apply_act(float x, int act) {
  switch (act) {
    case B2_ACT_RELU: return (x > 0.f || x != x) ? x : 0.f;
    case B2_ACT_GELU: return 0.5f * x * (1.f + erff(x * 0.70710678118654752f));
    case B2_ACT_GELU_TANH: {
      const float k0 = 0.7978845608028654f, k1 = 0.044715f;
      return 0.5f * x * (1.f + tanhf(k0 * (x + k1 * x * x * x)));
    }
    case B2_ACT_SILU: return x / (1.f + __expf(-x));
    default: return x;
  }
}

// ---- general epilogue chains (b2_gemm_epilogue)
// Internal activation code that selects the chain in every GEMM kernel.
constexpr int kActChain = 6;
constexpr int kMaxEpiOps = B2_EPI_MAX_OPS;
// Passed by value as a kernel parameter.
struct EpiProgram {
  int n;
  int code[kMaxEpiOps];
  float a[kMaxEpiOps];
  float b[kMaxEpiOps];
};
// The chain of the b2_gemm_epilogue call running on this host thread (n = 0
// otherwise); every GEMM launch copies it into its kernel's parameters.
const EpiProgram& epi_program();
void set_epi_program(const EpiProgram* p);

__device__ __forceinline__ float epi_op(float x, int code, float a, float b, float bias) {
  switch (code) {
    case B2_EPI_ADD: return x + a;
    case B2_EPI_SUB: return x - a;
    case B2_EPI_RSUB: return a - x;
    case B2_EPI_MUL: return x * a;
    case B2_EPI_DIV: return x / a;
    case B2_EPI_RDIV: return a / x;
    case B2_EPI_ADD_BIAS: return x + bias;
    case B2_EPI_MUL_BIAS: return x * bias;
    case B2_EPI_MAX: return (x != x || a != a) ? __int_as_float(0x7fffffff) : fmaxf(x, a);
    case B2_EPI_MIN: return (x != x || a != a) ? __int_as_float(0x7fffffff) : fminf(x, a);
    case B2_EPI_MAXNUM: return fmaxf(x, a);
    case B2_EPI_MINNUM: return fminf(x, a);
    case B2_EPI_CLAMP: return x != x ? x : fminf(fmaxf(x, a), b);
    case B2_EPI_CLAMPNUM: return fminf(fmaxf(x, a), b);
    case B2_EPI_NEG: return -x;
    case B2_EPI_EXP: return expf(x);
    case B2_EPI_EXP2: return exp2f(x);
    case B2_EPI_LOG: return logf(x);
    case B2_EPI_LOG2: return log2f(x);
    case B2_EPI_SQRT: return sqrtf(x);
    case B2_EPI_RSQRT: return rsqrtf(x);
    case B2_EPI_SIN: return sinf(x);
    case B2_EPI_COS: return cosf(x);
    case B2_EPI_ERF: return erff(x);
    case B2_EPI_TANH: return tanhf(x);
    case B2_EPI_FLOOR: return floorf(x);
    case B2_EPI_CEIL: return ceilf(x);
    case B2_EPI_ABS: return fabsf(x);
    case B2_EPI_RELU: return apply_act(x, B2_ACT_RELU);
    case B2_EPI_GELU: return apply_act(x, B2_ACT_GELU);
    case B2_EPI_GELU_TANH: return apply_act(x, B2_ACT_GELU_TANH);
    case B2_EPI_SILU: return x / (1.f + expf(-x));
    case B2_EPI_SIGMOID: return 1.f / (1.f + expf(-x));
    case B2_EPI_FMA: return fmaf(x, a, b);
    default: return x;
  }
}

// A chain over N values of one output row chunk: one branch per op, then a
// straight loop over the chunk (a per-element branch over 34 cases costs the
// epilogue warps far more than the arithmetic).
template <int N>
__device__ __forceinline__ void epi_chain_chunk(float (&f)[N], const float (&bv)[N], const EpiProgram& p) {
#define B2_EPI_CASE(CODE, EXPR)   \
  case CODE:                      \
    _Pragma("unroll")             \
    for (int j = 0; j < N; ++j) { \
      const float x = f[j];       \
      (void)x;                    \
      f[j] = (EXPR);              \
    }                             \
    break;
#pragma unroll 1
  for (int o = 0; o < p.n; ++o) {
    const float a = p.a[o], b = p.b[o];
    switch (p.code[o]) {
      B2_EPI_CASE(B2_EPI_ADD, x + a)
      B2_EPI_CASE(B2_EPI_SUB, x - a)
      B2_EPI_CASE(B2_EPI_RSUB, a - x)
      B2_EPI_CASE(B2_EPI_MUL, x * a)
      B2_EPI_CASE(B2_EPI_DIV, x / a)
      B2_EPI_CASE(B2_EPI_RDIV, a / x)
      B2_EPI_CASE(B2_EPI_ADD_BIAS, x + bv[j])
      B2_EPI_CASE(B2_EPI_MUL_BIAS, x * bv[j])
      B2_EPI_CASE(B2_EPI_FMA, fmaf(x, a, b))
      B2_EPI_CASE(B2_EPI_RELU, apply_act(x, B2_ACT_RELU))
      B2_EPI_CASE(B2_EPI_GELU, apply_act(x, B2_ACT_GELU))
      B2_EPI_CASE(B2_EPI_GELU_TANH, apply_act(x, B2_ACT_GELU_TANH))
      B2_EPI_CASE(B2_EPI_CLAMP, x != x ? x : fminf(fmaxf(x, a), b))
      B2_EPI_CASE(B2_EPI_CLAMPNUM, fminf(fmaxf(x, a), b))
      B2_EPI_CASE(B2_EPI_MAX, (x != x || a != a) ? __int_as_float(0x7fffffff) : fmaxf(x, a))
      B2_EPI_CASE(B2_EPI_MIN, (x != x || a != a) ? __int_as_float(0x7fffffff) : fminf(x, a))
      B2_EPI_CASE(B2_EPI_MAXNUM, fmaxf(x, a))
      B2_EPI_CASE(B2_EPI_MINNUM, fminf(x, a))
      B2_EPI_CASE(B2_EPI_NEG, -x)
      B2_EPI_CASE(B2_EPI_EXP, expf(x))
      B2_EPI_CASE(B2_EPI_EXP2, exp2f(x))
      B2_EPI_CASE(B2_EPI_LOG, logf(x))
      B2_EPI_CASE(B2_EPI_LOG2, log2f(x))
      B2_EPI_CASE(B2_EPI_SQRT, sqrtf(x))
      B2_EPI_CASE(B2_EPI_RSQRT, rsqrtf(x))
      B2_EPI_CASE(B2_EPI_SIN, sinf(x))
      B2_EPI_CASE(B2_EPI_COS, cosf(x))
      B2_EPI_CASE(B2_EPI_ERF, erff(x))
      B2_EPI_CASE(B2_EPI_TANH, tanhf(x))
      B2_EPI_CASE(B2_EPI_FLOOR, floorf(x))
      B2_EPI_CASE(B2_EPI_CEIL, ceilf(x))
      B2_EPI_CASE(B2_EPI_ABS, fabsf(x))
      B2_EPI_CASE(B2_EPI_SILU, x / (1.f + expf(-x)))
      B2_EPI_CASE(B2_EPI_SIGMOID, 1.f / (1.f + expf(-x)))
      default:
        break;
    }
  }
#undef B2_EPI_CASE
}

__device__ __forceinline__ float epi_chain(float x, float bias, const EpiProgram& p) {
#pragma unroll 1
  for (int o = 0; o < p.n; ++o) x = epi_op(x, p.code[o], p.a[o], p.b[o], bias);
  return x;
}

}  // namespace b2

#define B2_CUDA_TRY(expr)                                                        \
  do {                                                                           \
    cudaError_t _e = (expr);                                                     \
    if (_e != cudaSuccess) {                                                     \
      ::b2::set_error("%s failed: %s (%s:%d)", #expr, cudaGetErrorString(_e),    \
                      __FILE__, __LINE__);                                       \
      return B2_ELAUNCH;                                                         \
    }                                                                            \
  } while (0)

#define B2_CHECK_LAUNCH()                                                        \
  do {                                                                           \
    cudaError_t _e = cudaGetLastError();                                         \
    if (_e != cudaSuccess) {                                                     \
      ::b2::set_error("kernel launch failed: %s (%s:%d)", cudaGetErrorString(_e),\
                      __FILE__, __LINE__);                                       \
      return B2_ELAUNCH;                                                         \
    }                                                                            \
  } while (0)
