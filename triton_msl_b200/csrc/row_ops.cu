// Row-reduction family for sm_100a: softmax, LayerNorm, RMSNorm, sum, max,
// min, argmax, argmin over x[rows, cols].
//
// Reference semantics (triton-msl):
//   softmax      _lowerer_templates.py:992-1167 (exp(x - max) / sum), prebuilt
//                make_softmax_kernel _msl_templates.py:365-449
//   LayerNorm    make_layer_norm_kernel _msl_templates.py:1010-1090 (two-pass
//                mean / variance, * gamma + beta)
//   RMSNorm      make_rms_norm_kernel _msl_templates.py:888-951
//                (x * rsqrt(mean(x^2) + eps) * w)
//   sum/max      make_row_reduce_kernel _msl_templates.py:259-310 and the
//                NaN-propagating tt.reduce lowering _lowerer_reduce.py:773-1010
//   argmax       _lowerer_reduce.py:1223-1333 (ties -> lower index)
//
// B200 design: HBM-bound, so each row is read exactly once with 16-byte
// streaming loads into registers (up to 32 elements per thread), reduced with
// warp shuffles (+ one shared-memory hop across warps), and written once with
// 16-byte streaming stores. Rows up to 32768 elements stay register
// resident. Longer or unaligned rows take a strided path that re-reads the row
// (second read mostly hits L2). Few-but-long rows for the scalar reductions are
// split across CTAs, with partials in caller-provided workspace.
#include "b2_common.cuh"

#include <cfloat>
#include <mutex>

namespace b2 {
namespace {

__device__ uint32_t g_row_status;

constexpr float kLog2e = 1.4426950408889634f;

// ---------------------------------------------------------------- combiners
__device__ __forceinline__ float nan_max(float a, float b) {
  return (a > b || a != a) ? a : b;
}
__device__ __forceinline__ float nan_min(float a, float b) {
  return (a < b || a != a) ? a : b;
}
// true if (a, ia) beats (b, ib) for argmax (MAXI) / argmin (!MAXI): NaN is the
// extreme value, ties and NaN-vs-NaN go to the lower index (torch semantics).
template <bool MAXI, typename I>
__device__ __forceinline__ bool arg_better(float a, I ia, float b, I ib) {
  const bool an = a != a, bn = b != b;
  if (an || bn) return an && (!bn || ia < ib);
  if (MAXI) return a > b || (a == b && ia < ib);
  return a < b || (a == b && ia < ib);
}

// ------------------------------------------------------- group reductions
// Reductions over a group of G consecutive lanes (G <= 32) inside a warp.
template <int G>
__device__ __forceinline__ float group_sum(float v) {
#pragma unroll
  for (int o = G / 2; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o, G);
  return v;
}
template <int G>
__device__ __forceinline__ float group_max(float v) {
#pragma unroll
  for (int o = G / 2; o > 0; o >>= 1) v = nan_max(v, __shfl_xor_sync(0xffffffffu, v, o, G));
  return v;
}
template <int G>
__device__ __forceinline__ float group_min(float v) {
#pragma unroll
  for (int o = G / 2; o > 0; o >>= 1) v = nan_min(v, __shfl_xor_sync(0xffffffffu, v, o, G));
  return v;
}
template <int G, bool MAXI, typename I>
__device__ __forceinline__ void group_arg(float& v, I& i) {
#pragma unroll
  for (int o = G / 2; o > 0; o >>= 1) {
    float ov = __shfl_xor_sync(0xffffffffu, v, o, G);
    I oi = __shfl_xor_sync(0xffffffffu, i, o, G);
    if (arg_better<MAXI>(ov, oi, v, i)) { v = ov; i = oi; }
  }
}

// 2^x on the MUFU alone (results below 2^-126 flush to zero, far under every
// tolerance here). Against exp2f, measured on B200: fp16 softmax +4-7 %,
// bf16 +2-3 %, fp32 unchanged.
__device__ __forceinline__ float ex2_fast(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

enum RedKind { RK_SUM, RK_MAX, RK_MIN };

// Reduce across a row handled by TPR threads. TPR <= 32: pure shuffles inside
// the lane group. TPR > 32: the block is one row; shuffles then one smem hop.
template <int TPR, int KIND>
__device__ __forceinline__ float row_reduce(float v, float* red_smem) {
  auto op_warp = [](float x) {
    if (KIND == RK_SUM) return group_sum<(TPR < 32 ? TPR : 32)>(x);
    if (KIND == RK_MAX) return group_max<(TPR < 32 ? TPR : 32)>(x);
    return group_min<(TPR < 32 ? TPR : 32)>(x);
  };
  v = op_warp(v);
  if constexpr (TPR > 32) {
    constexpr int NW = TPR / 32;
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    __syncthreads();  // red_smem may still be read by a previous reduction
    if (lane == 0) red_smem[wid] = v;
    __syncthreads();
    float t = lane < NW ? red_smem[lane] : (KIND == RK_SUM ? 0.f : red_smem[0]);
    if (KIND == RK_SUM) t = group_sum<32>(t);
    else if (KIND == RK_MAX) t = group_max<32>(t);
    else t = group_min<32>(t);
    v = t;
  }
  return v;
}

template <int TPR, bool MAXI, typename I>
__device__ __forceinline__ void row_reduce_arg(float& v, I& i, float* red_v, I* red_i) {
  group_arg<(TPR < 32 ? TPR : 32), MAXI>(v, i);
  if constexpr (TPR > 32) {
    constexpr int NW = TPR / 32;
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    if (lane == 0) { red_v[wid] = v; red_i[wid] = i; }
    __syncthreads();
    float tv = lane < NW ? red_v[lane] : red_v[0];
    I ti = lane < NW ? red_i[lane] : red_i[0];
    group_arg<32, MAXI>(tv, ti);
    v = tv; i = ti;
  }
}

// -------------------------------------------------------- vector load/store
template <typename T> struct Vec;  // 16-byte vectors of T
template <> struct Vec<float> { static constexpr int N = 4; };
template <> struct Vec<__half> { static constexpr int N = 8; };
template <> struct Vec<__nv_bfloat16> { static constexpr int N = 8; };

template <typename T>
__device__ __forceinline__ void ld_vec(const T* p, float* f) {
  const uint4 u = __ldcs(reinterpret_cast<const uint4*>(p));
  if constexpr (sizeof(T) == 4) {
    f[0] = __uint_as_float(u.x); f[1] = __uint_as_float(u.y);
    f[2] = __uint_as_float(u.z); f[3] = __uint_as_float(u.w);
  } else {
    const T* h = reinterpret_cast<const T*>(&u);
#pragma unroll
    for (int j = 0; j < 8; ++j) f[j] = to_f32<T>(h[j]);
  }
}
// Parameters (gamma/beta/weight) are re-read by every row: keep them cached.
template <typename T>
__device__ __forceinline__ void ld_vec_cached(const T* p, float* f) {
  const uint4 u = __ldg(reinterpret_cast<const uint4*>(p));
  if constexpr (sizeof(T) == 4) {
    f[0] = __uint_as_float(u.x); f[1] = __uint_as_float(u.y);
    f[2] = __uint_as_float(u.z); f[3] = __uint_as_float(u.w);
  } else {
    const T* h = reinterpret_cast<const T*>(&u);
#pragma unroll
    for (int j = 0; j < 8; ++j) f[j] = to_f32<T>(h[j]);
  }
}
template <typename T>
__device__ __forceinline__ void st_vec(T* p, const float* f) {
  uint4 u;
  if constexpr (sizeof(T) == 4) {
    u.x = __float_as_uint(f[0]); u.y = __float_as_uint(f[1]);
    u.z = __float_as_uint(f[2]); u.w = __float_as_uint(f[3]);
  } else {
    T* h = reinterpret_cast<T*>(&u);
#pragma unroll
    for (int j = 0; j < 8; ++j) h[j] = from_f32<T>(f[j]);
  }
  __stcs(reinterpret_cast<uint4*>(p), u);
}

// ------------------------------------------------- register-resident kernel
// TPR threads per row, VPT 16-byte vectors per thread, block = max(TPR, 256)
// threads (several rows per block when TPR < 256... only for TPR <= 32).
// Requires cols % Vec<T>::N == 0, 16-byte aligned rows, cols <= TPR*VPT*EPV.
template <typename T, int OP, int TPR, int VPT>
__global__ void __launch_bounds__(TPR > 32 ? TPR : 256)
row_reg_kernel(const T* __restrict__ x, const T* __restrict__ w, const T* __restrict__ bvec,
               void* __restrict__ out, long long rows, int cols, long long ldx, long long ldo,
               float eps) {
  constexpr int EPV = Vec<T>::N;
  constexpr int BLOCK = TPR > 32 ? TPR : 256;
  constexpr int RPB = BLOCK / TPR;  // rows per block
  static_assert(TPR <= 32 || RPB == 1, "multi-row blocks need TPR <= 32");
  __shared__ float red_v[32];
  __shared__ float red_av[2][32];  // argmax / argmin: one buffer per row parity,
  __shared__ int red_ai[2][32];    // so consecutive rows need no extra barrier

  const int sub = threadIdx.x % TPR;          // thread index inside the row
  const int rloc = threadIdx.x / TPR;         // row slot inside the block
  const float inv_cols = 1.f / (float)cols;

  int parity = 0;
  for (long long row0 = (long long)blockIdx.x * RPB; row0 < rows; row0 += (long long)gridDim.x * RPB, parity ^= 1) {
    const long long row = row0 + rloc;
    const bool row_ok = row < rows;
    const T* xr = x + (row_ok ? row : 0) * ldx;
    // argmax / argmin over 16-bit inputs compare the raw pairs (see below)
    constexpr bool PACKED_ARG = (OP == B2_ROW_ARGMAX || OP == B2_ROW_ARGMIN) && sizeof(T) == 2;
    float v[VPT][EPV];
    uint4 raw[PACKED_ARG ? VPT : 1];
    bool ok[VPT];
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int c = (sub + i * TPR) * EPV;
      ok[i] = row_ok && c < cols;
      if (ok[i]) {
        if constexpr (PACKED_ARG) raw[i] = __ldcs(reinterpret_cast<const uint4*>(xr + c));
        else ld_vec<T>(xr + c, v[i]);
      }
    }

    if constexpr (OP == B2_ROW_SUM || OP == B2_ROW_MAX || OP == B2_ROW_MIN) {
      float a = OP == B2_ROW_SUM ? 0.f : (OP == B2_ROW_MAX ? -INFINITY : INFINITY);
#pragma unroll
      for (int i = 0; i < VPT; ++i)
        if (ok[i]) {
#pragma unroll
          for (int j = 0; j < EPV; ++j) {
            if (OP == B2_ROW_SUM) a += v[i][j];
            else if (OP == B2_ROW_MAX) a = nan_max(a, v[i][j]);
            else a = nan_min(a, v[i][j]);
          }
        }
      a = row_reduce<TPR, OP == B2_ROW_SUM ? RK_SUM : (OP == B2_ROW_MAX ? RK_MAX : RK_MIN)>(a, red_v);
      if (row_ok && sub == 0) reinterpret_cast<T*>(out)[row] = from_f32<T>(a);
    } else if constexpr (PACKED_ARG) {
      // 16-bit inputs: four chains of value pairs per thread, compared two at a
      // time in the inputs' own type (exact: no conversion is needed to order
      // them) with bitwise selects of the values and of 16-bit column indices
      // (register-path rows have < 2^15 columns). The per-pair rule is the
      // scalar chains' rule below: take x when !(x <= best) and best is not
      // NaN, so ties keep the earlier column and the first NaN wins.
      constexpr bool MAXI = OP == B2_ROW_ARGMAX;
      using T2 = typename std::conditional<std::is_same<T, __half>::value, __half2, __nv_bfloat162>::type;
      auto as2 = [](uint32_t u) { T2 r; memcpy(&r, &u, 4); return r; };
      const uint32_t inf2 = std::is_same<T, __half>::value ? (MAXI ? 0xFC00FC00u : 0x7C007C00u)
                                                           : (MAXI ? 0xFF80FF80u : 0x7F807F80u);
      uint32_t cv[EPV / 2], ck[EPV / 2];
#pragma unroll
      for (int p = 0; p < EPV / 2; ++p) {
        const uint32_t c0 = (uint32_t)(sub * EPV + 2 * p);
        cv[p] = ok[0] ? (&raw[0].x)[p] : inf2;
        ck[p] = ok[0] ? (c0 | ((c0 + 1) << 16)) : 0xFFFFFFFFu;
      }
#pragma unroll
      for (int i = 1; i < VPT; ++i)
        if (ok[i]) {
#pragma unroll
          for (int p = 0; p < EPV / 2; ++p) {
            const uint32_t xv = (&raw[i].x)[p];
            const uint32_t notbetter = MAXI ? __hle2_mask(as2(xv), as2(cv[p])) : __hge2_mask(as2(xv), as2(cv[p]));
            const uint32_t take = ~notbetter & __heq2_mask(as2(cv[p]), as2(cv[p]));
            const uint32_t c0 = (uint32_t)((sub + i * TPR) * EPV + 2 * p);
            cv[p] = (cv[p] & ~take) | (xv & take);
            ck[p] = (ck[p] & ~take) | ((c0 | ((c0 + 1) << 16)) & take);
          }
        }
      float bv = MAXI ? -INFINITY : INFINITY;
      int bi = 0x7fffffff;
#pragma unroll
      for (int p = 0; p < EPV / 2; ++p) {
#pragma unroll
        for (int hsel = 0; hsel < 2; ++hsel) {
          const uint16_t hb = (uint16_t)(hsel ? cv[p] >> 16 : cv[p] & 0xFFFFu);
          T hv;
          memcpy(&hv, &hb, 2);
          const uint32_t ix = hsel ? ck[p] >> 16 : ck[p] & 0xFFFFu;
          const int ii = ix == 0xFFFFu ? 0x7fffffff : (int)ix;
          const float fv = to_f32<T>(hv);
          if (arg_better<MAXI>(fv, ii, bv, bi)) { bv = fv; bi = ii; }
        }
      }
      row_reduce_arg<TPR, MAXI>(bv, bi, red_av[parity], red_ai[parity]);
      if (row_ok && sub == 0) reinterpret_cast<long long*>(out)[row] = (long long)bi;
    } else if constexpr (OP == B2_ROW_ARGMAX || OP == B2_ROW_ARGMIN) {
      constexpr bool MAXI = OP == B2_ROW_ARGMAX;
      // One independent scan per vector lane j (EPV chains, so the compare /
      // select latency overlaps); each chain visits its columns in increasing
      // order, so a strict comparison keeps the earliest of equal values and
      // the first NaN, and arg_better (ties -> lower index) merges the chains
      // exactly. 32-bit indices (rows are < 2^31 columns) until the int64 store.
      float cv[EPV];
      int ck[EPV];
#pragma unroll
      for (int j = 0; j < EPV; ++j) {
        cv[j] = MAXI ? -INFINITY : INFINITY;
        ck[j] = 0x7fffffff;
      }
      // columns grow with i, so a thread without a first vector has none
      if (ok[0]) {
#pragma unroll
        for (int j = 0; j < EPV; ++j) {
          cv[j] = v[0][j];
          ck[j] = sub * EPV + j;
        }
      }
#pragma unroll
      for (int i = 1; i < VPT; ++i)
        if (ok[i]) {
#pragma unroll
          for (int j = 0; j < EPV; ++j) {
            const float x = v[i][j];
            const int ci = (sub + i * TPR) * EPV + j;
            // x beats the chain's best: strictly better, or a NaN against a
            // number (NaN is the extreme value)
            const bool take = (MAXI ? !(x <= cv[j]) : !(x >= cv[j])) && cv[j] == cv[j];
            cv[j] = take ? x : cv[j];
            ck[j] = take ? ci : ck[j];
          }
        }
      float bv = cv[0];
      int bi = ck[0];
#pragma unroll
      for (int j = 1; j < EPV; ++j)
        if (arg_better<MAXI>(cv[j], ck[j], bv, bi)) { bv = cv[j]; bi = ck[j]; }
      row_reduce_arg<TPR, MAXI>(bv, bi, red_av[parity], red_ai[parity]);
      if (row_ok && sub == 0) reinterpret_cast<long long*>(out)[row] = (long long)bi;
    } else if constexpr (OP == B2_ROW_SOFTMAX) {
      float m = -INFINITY;
#pragma unroll
      for (int i = 0; i < VPT; ++i)
        if (ok[i]) {
#pragma unroll
          for (int j = 0; j < EPV; ++j) m = nan_max(m, v[i][j]);
        }
      m = row_reduce<TPR, RK_MAX>(m, red_v);
      const float ms = m * kLog2e;
      float s = 0.f;
#pragma unroll
      for (int i = 0; i < VPT; ++i)
        if (ok[i]) {
#pragma unroll
          for (int j = 0; j < EPV; ++j) {
            v[i][j] = ex2_fast(fmaf(v[i][j], kLog2e, -ms));
            s += v[i][j];
          }
        }
      s = row_reduce<TPR, RK_SUM>(s, red_v);
      const float inv = 1.f / s;
      T* o = reinterpret_cast<T*>(out) + (row_ok ? row : 0) * ldo;
#pragma unroll
      for (int i = 0; i < VPT; ++i)
        if (ok[i]) {
#pragma unroll
          for (int j = 0; j < EPV; ++j) v[i][j] *= inv;
          st_vec<T>(o + (sub + i * TPR) * EPV, v[i]);
        }
    } else if constexpr (OP == B2_ROW_LAYERNORM) {
      float s = 0.f;
#pragma unroll
      for (int i = 0; i < VPT; ++i)
        if (ok[i]) {
#pragma unroll
          for (int j = 0; j < EPV; ++j) s += v[i][j];
        }
      const float mean = row_reduce<TPR, RK_SUM>(s, red_v) * inv_cols;
      float q = 0.f;
#pragma unroll
      for (int i = 0; i < VPT; ++i)
        if (ok[i]) {
#pragma unroll
          for (int j = 0; j < EPV; ++j) {
            const float d = v[i][j] - mean;
            q = fmaf(d, d, q);
          }
        }
      const float var = row_reduce<TPR, RK_SUM>(q, red_v) * inv_cols;
      const float rstd = rsqrtf(var + eps);
      T* o = reinterpret_cast<T*>(out) + (row_ok ? row : 0) * ldo;
#pragma unroll
      for (int i = 0; i < VPT; ++i)
        if (ok[i]) {
          const int c = (sub + i * TPR) * EPV;
          float g[EPV], bb[EPV];
          if (w) ld_vec_cached<T>(w + c, g);
          else {
#pragma unroll
            for (int j = 0; j < EPV; ++j) g[j] = 1.f;
          }
          if (bvec) ld_vec_cached<T>(bvec + c, bb);
          else {
#pragma unroll
            for (int j = 0; j < EPV; ++j) bb[j] = 0.f;
          }
#pragma unroll
          for (int j = 0; j < EPV; ++j) v[i][j] = fmaf((v[i][j] - mean) * rstd, g[j], bb[j]);
          st_vec<T>(o + c, v[i]);
        }
    } else if constexpr (OP == B2_ROW_RMSNORM) {
      float q = 0.f;
#pragma unroll
      for (int i = 0; i < VPT; ++i)
        if (ok[i]) {
#pragma unroll
          for (int j = 0; j < EPV; ++j) q = fmaf(v[i][j], v[i][j], q);
        }
      const float ms = row_reduce<TPR, RK_SUM>(q, red_v) * inv_cols;
      const float r = rsqrtf(ms + eps);
      T* o = reinterpret_cast<T*>(out) + (row_ok ? row : 0) * ldo;
#pragma unroll
      for (int i = 0; i < VPT; ++i)
        if (ok[i]) {
          const int c = (sub + i * TPR) * EPV;
          float g[EPV];
          if (w) ld_vec_cached<T>(w + c, g);
          else {
#pragma unroll
            for (int j = 0; j < EPV; ++j) g[j] = 1.f;
          }
#pragma unroll
          for (int j = 0; j < EPV; ++j) v[i][j] = v[i][j] * r * g[j];
          st_vec<T>(o + c, v[i]);
        }
    }
  }
}

// ------------------------------------------------------------ strided kernel
// Any cols / alignment: one row per block, scalar loads, the row is re-read
// once per pass.
template <typename T, int OP>
__global__ void __launch_bounds__(512)
row_generic_kernel(const T* __restrict__ x, const T* __restrict__ w, const T* __restrict__ bvec,
                   void* __restrict__ out, long long rows, long long cols, long long ldx,
                   long long ldo, float eps) {
  constexpr int TPR = 512;
  __shared__ float red_v[32];
  __shared__ long long red_i[32];
  for (long long row = blockIdx.x; row < rows; row += gridDim.x) {
    const T* xr = x + row * ldx;
    if constexpr (OP == B2_ROW_SUM || OP == B2_ROW_MAX || OP == B2_ROW_MIN) {
      float a = OP == B2_ROW_SUM ? 0.f : (OP == B2_ROW_MAX ? -INFINITY : INFINITY);
      for (long long c = threadIdx.x; c < cols; c += TPR) {
        const float t = to_f32<T>(xr[c]);
        if (OP == B2_ROW_SUM) a += t;
        else if (OP == B2_ROW_MAX) a = nan_max(a, t);
        else a = nan_min(a, t);
      }
      a = row_reduce<TPR, OP == B2_ROW_SUM ? RK_SUM : (OP == B2_ROW_MAX ? RK_MAX : RK_MIN)>(a, red_v);
      if (threadIdx.x == 0) reinterpret_cast<T*>(out)[row] = from_f32<T>(a);
    } else if constexpr (OP == B2_ROW_ARGMAX || OP == B2_ROW_ARGMIN) {
      constexpr bool MAXI = OP == B2_ROW_ARGMAX;
      float bv = MAXI ? -INFINITY : INFINITY;
      long long bi = 0x7fffffffffffffffLL;
      for (long long c = threadIdx.x; c < cols; c += TPR) {
        const float t = to_f32<T>(xr[c]);
        if (arg_better<MAXI>(t, c, bv, bi)) { bv = t; bi = c; }
      }
      __syncthreads();
      row_reduce_arg<TPR, MAXI>(bv, bi, red_v, red_i);
      if (threadIdx.x == 0) reinterpret_cast<long long*>(out)[row] = bi;
      __syncthreads();
    } else {
      T* o = reinterpret_cast<T*>(out) + row * ldo;
      const float inv_cols = 1.f / (float)cols;
      if constexpr (OP == B2_ROW_SOFTMAX) {
        float m = -INFINITY;
        for (long long c = threadIdx.x; c < cols; c += TPR) m = nan_max(m, to_f32<T>(xr[c]));
        m = row_reduce<TPR, RK_MAX>(m, red_v);
        const float ms = m * kLog2e;
        float s = 0.f;
        for (long long c = threadIdx.x; c < cols; c += TPR) s += exp2f(fmaf(to_f32<T>(xr[c]), kLog2e, -ms));
        s = row_reduce<TPR, RK_SUM>(s, red_v);
        const float inv = 1.f / s;
        for (long long c = threadIdx.x; c < cols; c += TPR)
          o[c] = from_f32<T>(exp2f(fmaf(to_f32<T>(xr[c]), kLog2e, -ms)) * inv);
      } else if constexpr (OP == B2_ROW_LAYERNORM) {
        float s = 0.f;
        for (long long c = threadIdx.x; c < cols; c += TPR) s += to_f32<T>(xr[c]);
        const float mean = row_reduce<TPR, RK_SUM>(s, red_v) * inv_cols;
        float q = 0.f;
        for (long long c = threadIdx.x; c < cols; c += TPR) {
          const float d = to_f32<T>(xr[c]) - mean;
          q = fmaf(d, d, q);
        }
        const float rstd = rsqrtf(row_reduce<TPR, RK_SUM>(q, red_v) * inv_cols + eps);
        for (long long c = threadIdx.x; c < cols; c += TPR) {
          const float g = w ? to_f32<T>(w[c]) : 1.f, bb = bvec ? to_f32<T>(bvec[c]) : 0.f;
          o[c] = from_f32<T>(fmaf((to_f32<T>(xr[c]) - mean) * rstd, g, bb));
        }
      } else if constexpr (OP == B2_ROW_RMSNORM) {
        float q = 0.f;
        for (long long c = threadIdx.x; c < cols; c += TPR) {
          const float t = to_f32<T>(xr[c]);
          q = fmaf(t, t, q);
        }
        const float r = rsqrtf(row_reduce<TPR, RK_SUM>(q, red_v) * inv_cols + eps);
        for (long long c = threadIdx.x; c < cols; c += TPR) {
          const float g = w ? to_f32<T>(w[c]) : 1.f;
          o[c] = from_f32<T>(to_f32<T>(xr[c]) * r * g);
        }
      }
    }
  }
}

// ------------------------------------------------------------ long rows
// Rows too long for the register-resident kernel (cols > 32K, 16-byte aligned):
// one 512-thread CTA per row, two CTAs per SM, 16-byte loads with four in
// flight per thread. Pass 1 reads the row once and keeps per-thread running
// statistics (online max and sum of exponentials for softmax, sums shifted by
// the thread's first element for LayerNorm, the sum of squares for RMSNorm;
// sum / max / min / argmax / argmin finish here). Pass 2 re-reads the row,
// which the ~300 rows in flight leave in L2 for rows up to ~100K fp32
// columns, and writes the output.
// Measured on B200 (4096 x 65536 and 512 x 524288 fp32): two CTAs per SM with
// four 16-byte loads in flight per thread beat one CTA per SM with four or
// eight by 5-30 %.
constexpr int kLongTPR = 512, kLongU = 4, kLongCtas = 2;

// (m, s): running max m (NaN-propagating) and sum s of 2^((x - m) * log2 e)
__device__ __forceinline__ void sm_combine(float& m, float& s, float m2, float s2) {
  const float mm = nan_max(m, m2);
  const float a = (m == mm) ? s : s * exp2f((m - mm) * kLog2e);
  const float b = (m2 == mm) ? s2 : s2 * exp2f((m2 - mm) * kLog2e);
  m = mm;
  s = a + b;
}
// (n, mean, M2) of two disjoint sets (Chan et al.'s pairwise update)
__device__ __forceinline__ void mv_combine(float& n, float& mean, float& m2, float nb, float meanb,
                                           float m2b) {
  if (nb == 0.f) return;
  if (n == 0.f) { n = nb; mean = meanb; m2 = m2b; return; }
  const float nt = n + nb, d = meanb - mean;
  mean = fmaf(d, nb / nt, mean);
  m2 = m2 + m2b + d * d * (n * nb / nt);
  n = nt;
}

template <typename T, int OP>
__global__ void __launch_bounds__(kLongTPR, kLongCtas)
row_long_kernel(const T* __restrict__ x, const T* __restrict__ w, const T* __restrict__ bvec,
                void* __restrict__ out, long long rows, int cols, long long ldx, long long ldo,
                float eps) {
  constexpr int EPV = Vec<T>::N, TPR = kLongTPR, NW = TPR / 32;
  constexpr int U = sizeof(T) == 4 ? kLongU : kLongU / 2;  // 16-bit types: 8 values per vector
  __shared__ float red_a[NW], red_b[NW], red_c[NW];
  __shared__ int red_i[NW];
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  const int nvec = cols / EPV;
  // Two-pass ops read pass 1 with an L2 evict-last policy, so the row is
  // still in L2 when pass 2 (streaming, evict-first loads) reads it again
  // (B200: fp16 / bf16 LayerNorm +6-7 %, the other ops within 1 %).
  constexpr bool TWO_PASS = (OP == B2_ROW_SOFTMAX || OP == B2_ROW_LAYERNORM || OP == B2_ROW_RMSNORM);
  uint64_t keep = 0;
  if constexpr (TWO_PASS) asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(keep));
  for (long long row = blockIdx.x; row < rows; row += gridDim.x) {
    const T* xr = x + row * ldx;
    // pass 1
    float a0, a1 = 0.f, a2 = 0.f;  // per-op running statistics
    int ai = 0x7fffffff;
    float shift = 0.f;
    if constexpr (OP == B2_ROW_SUM || OP == B2_ROW_RMSNORM) a0 = 0.f;
    else if constexpr (OP == B2_ROW_MAX || OP == B2_ROW_ARGMAX || OP == B2_ROW_SOFTMAX) a0 = -INFINITY;
    else if constexpr (OP == B2_ROW_MIN || OP == B2_ROW_ARGMIN) a0 = INFINITY;
    else a0 = 0.f;  // LayerNorm: a0 = count, a1 = sum of (x - shift), a2 = sum of squares
    if constexpr (OP == B2_ROW_LAYERNORM) {
      if (tid < nvec) shift = to_f32<T>(xr[tid * EPV]);
    }
    for (int k0 = tid; k0 < nvec; k0 += TPR * U) {
      float v[U][EPV];
#pragma unroll
      for (int u = 0; u < U; ++u)
        if (k0 + u * TPR < nvec) {
          uint4 q;
          const T* src = xr + (long long)(k0 + u * TPR) * EPV;
          if constexpr (TWO_PASS)
            asm volatile("ld.global.L2::cache_hint.v4.u32 {%0, %1, %2, %3}, [%4], %5;"
                         : "=r"(q.x), "=r"(q.y), "=r"(q.z), "=r"(q.w) : "l"(src), "l"(keep));
          else
            q = *reinterpret_cast<const uint4*>(src);
          if constexpr (sizeof(T) == 4) {
            v[u][0] = __uint_as_float(q.x); v[u][1] = __uint_as_float(q.y);
            v[u][2] = __uint_as_float(q.z); v[u][3] = __uint_as_float(q.w);
          } else {
            const T* h = reinterpret_cast<const T*>(&q);
#pragma unroll
            for (int j = 0; j < EPV; ++j) v[u][j] = to_f32<T>(h[j]);
          }
        }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        if (k0 + u * TPR >= nvec) break;
        if constexpr (OP == B2_ROW_SUM) {
#pragma unroll
          for (int j = 0; j < EPV; ++j) a0 += v[u][j];
        } else if constexpr (OP == B2_ROW_MAX) {
#pragma unroll
          for (int j = 0; j < EPV; ++j) a0 = nan_max(a0, v[u][j]);
        } else if constexpr (OP == B2_ROW_MIN) {
#pragma unroll
          for (int j = 0; j < EPV; ++j) a0 = nan_min(a0, v[u][j]);
        } else if constexpr (OP == B2_ROW_ARGMAX || OP == B2_ROW_ARGMIN) {
          // elements arrive in ascending column order: a tie keeps the earlier
          // column, the first NaN is kept
          const int c = (k0 + u * TPR) * EPV;
#pragma unroll
          for (int j = 0; j < EPV; ++j) {
            const float f = v[u][j];
            const bool better = (OP == B2_ROW_ARGMAX ? f > a0 : f < a0) || (f != f && a0 == a0) ||
                                ai == 0x7fffffff;
            a0 = better ? f : a0;
            ai = better ? c + j : ai;
          }
        } else if constexpr (OP == B2_ROW_SOFTMAX) {
          float mv = a0;
#pragma unroll
          for (int j = 0; j < EPV; ++j) mv = nan_max(mv, v[u][j]);
          if (mv != a0) {  // the max grew (or turned NaN): rescale the sum
            a1 = (a0 == -INFINITY) ? 0.f : a1 * exp2f((a0 - mv) * kLog2e);
            a0 = mv;
          }
          const float ms = a0 == -INFINITY ? 0.f : a0 * kLog2e;
#pragma unroll
          for (int j = 0; j < EPV; ++j) a1 += ex2_fast(fmaf(v[u][j], kLog2e, -ms));
        } else if constexpr (OP == B2_ROW_LAYERNORM) {
#pragma unroll
          for (int j = 0; j < EPV; ++j) {
            const float d = v[u][j] - shift;
            a1 += d;
            a2 = fmaf(d, d, a2);
          }
          a0 += (float)EPV;
        } else {  // RMSNorm
#pragma unroll
          for (int j = 0; j < EPV; ++j) a0 = fmaf(v[u][j], v[u][j], a0);
        }
      }
    }
    // combine across the CTA: warp shuffles, then one value per warp in shared
    // memory, folded in warp order by every thread
    if constexpr (OP == B2_ROW_LAYERNORM) {
      // (count, sum of x - shift, sum of squares) -> (count, mean, M2)
      float n = a0, mean = a0 > 0.f ? shift + a1 / a0 : 0.f;
      float m2 = a0 > 0.f ? fmaxf(a2 - a1 * a1 / a0, 0.f) : 0.f;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float nb = __shfl_xor_sync(0xffffffffu, n, o), mb = __shfl_xor_sync(0xffffffffu, mean, o),
                    qb = __shfl_xor_sync(0xffffffffu, m2, o);
        mv_combine(n, mean, m2, nb, mb, qb);
      }
      __syncthreads();
      if (lane == 0) { red_a[wid] = n; red_b[wid] = mean; red_c[wid] = m2; }
      __syncthreads();
      n = red_a[0]; mean = red_b[0]; m2 = red_c[0];
      for (int i = 1; i < NW; ++i) mv_combine(n, mean, m2, red_a[i], red_b[i], red_c[i]);
      a1 = mean;
      a2 = rsqrtf(m2 / (float)cols + eps);
    } else if constexpr (OP == B2_ROW_SOFTMAX) {
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float mb = __shfl_xor_sync(0xffffffffu, a0, o), sb = __shfl_xor_sync(0xffffffffu, a1, o);
        sm_combine(a0, a1, mb, sb);
      }
      __syncthreads();
      if (lane == 0) { red_a[wid] = a0; red_b[wid] = a1; }
      __syncthreads();
      a0 = red_a[0]; a1 = red_b[0];
      for (int i = 1; i < NW; ++i) sm_combine(a0, a1, red_a[i], red_b[i]);
    } else if constexpr (OP == B2_ROW_ARGMAX || OP == B2_ROW_ARGMIN) {
      constexpr bool MAXI = OP == B2_ROW_ARGMAX;
      __syncthreads();
      row_reduce_arg<TPR, MAXI>(a0, ai, red_a, red_i);
      if (tid == 0) reinterpret_cast<long long*>(out)[row] = (long long)ai;
      continue;
    } else {
      constexpr int KIND = (OP == B2_ROW_SUM || OP == B2_ROW_RMSNORM) ? RK_SUM
                         : (OP == B2_ROW_MAX ? RK_MAX : RK_MIN);
      a0 = row_reduce<TPR, KIND>(a0, red_a);
      if constexpr (OP == B2_ROW_SUM || OP == B2_ROW_MAX || OP == B2_ROW_MIN) {
        if (tid == 0) reinterpret_cast<T*>(out)[row] = from_f32<T>(a0);
        continue;
      }
    }
    // pass 2: normalise and write
    T* o = reinterpret_cast<T*>(out) + row * ldo;
    float ms = 0.f, inv = 0.f;
    if constexpr (OP == B2_ROW_SOFTMAX) {
      ms = a0 == -INFINITY ? 0.f : a0 * kLog2e;
      inv = 1.f / a1;
    } else if constexpr (OP == B2_ROW_RMSNORM) {
      inv = rsqrtf(a0 / (float)cols + eps);
    }
    // last chunk first: the most recently read part of the row is the most
    // likely to be still in L2
    for (int kb = ((nvec - 1) / (TPR * U)) * (TPR * U); kb >= 0; kb -= TPR * U) {
      const int k0 = kb + tid;
      float v[U][EPV];
#pragma unroll
      for (int u = 0; u < U; ++u)
        if (k0 + u * TPR < nvec) ld_vec<T>(xr + (long long)(k0 + u * TPR) * EPV, v[u]);
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int k = k0 + u * TPR;
        if (k >= nvec) break;
        if constexpr (OP == B2_ROW_SOFTMAX) {
#pragma unroll
          for (int j = 0; j < EPV; ++j) v[u][j] = ex2_fast(fmaf(v[u][j], kLog2e, -ms)) * inv;
        } else if constexpr (OP == B2_ROW_LAYERNORM) {
          float g[EPV], bb[EPV];
          if (w) ld_vec_cached<T>(w + (long long)k * EPV, g);
          else {
#pragma unroll
            for (int j = 0; j < EPV; ++j) g[j] = 1.f;
          }
          if (bvec) ld_vec_cached<T>(bvec + (long long)k * EPV, bb);
          else {
#pragma unroll
            for (int j = 0; j < EPV; ++j) bb[j] = 0.f;
          }
#pragma unroll
          for (int j = 0; j < EPV; ++j) v[u][j] = fmaf((v[u][j] - a1) * a2, g[j], bb[j]);
        } else {
          float g[EPV];
          if (w) ld_vec_cached<T>(w + (long long)k * EPV, g);
          else {
#pragma unroll
            for (int j = 0; j < EPV; ++j) g[j] = 1.f;
          }
#pragma unroll
          for (int j = 0; j < EPV; ++j) v[u][j] = v[u][j] * inv * g[j];
        }
        st_vec<T>(o + (long long)k * EPV, v[u]);
      }
    }
  }
}

// ---------------------------------------------------- split-row reduction
// Few long rows: grid (splits, rows). Each CTA reduces one chunk into the
// workspace; a second launch folds the partials in chunk order.
struct Partial {
  float v;
  int pad;
  long long i;
};

template <typename T, int OP>
__global__ void __launch_bounds__(512)
row_split_partial_kernel(const T* __restrict__ x, long long cols, long long ldx, long long chunk,
                         Partial* __restrict__ ws) {
  constexpr int TPR = 512;
  __shared__ float red_v[32];
  __shared__ long long red_i[32];
  const long long row = blockIdx.y;
  const long long c0 = (long long)blockIdx.x * chunk;
  const long long c1 = c0 + chunk < cols ? c0 + chunk : cols;
  const T* xr = x + row * ldx;
  Partial p;
  p.pad = 0;
  const bool vec_ok = (sizeof(T) == 4) && ((reinterpret_cast<uintptr_t>(xr + c0) & 15) == 0);
  if constexpr (OP == B2_ROW_ARGMAX || OP == B2_ROW_ARGMIN) {
    constexpr bool MAXI = OP == B2_ROW_ARGMAX;
    float bv = MAXI ? -INFINITY : INFINITY;
    long long bi = 0x7fffffffffffffffLL;
    for (long long c = c0 + threadIdx.x; c < c1; c += TPR) {
      const float t = to_f32<T>(xr[c]);
      if (arg_better<MAXI>(t, c, bv, bi)) { bv = t; bi = c; }
    }
    row_reduce_arg<TPR, MAXI>(bv, bi, red_v, red_i);
    p.v = bv; p.i = bi;
  } else {
    constexpr int KIND = OP == B2_ROW_SUM ? RK_SUM : (OP == B2_ROW_MAX ? RK_MAX : RK_MIN);
    float a = KIND == RK_SUM ? 0.f : (KIND == RK_MAX ? -INFINITY : INFINITY);
    long long c = c0;
    if (vec_ok) {
      const long long nv = (c1 - c0) / 4;
      const float4* xv = reinterpret_cast<const float4*>(xr + c0);
      for (long long k = threadIdx.x; k < nv; k += TPR) {
        const float4 f = __ldcs(xv + k);
        if (KIND == RK_SUM) a += (f.x + f.y) + (f.z + f.w);
        else if (KIND == RK_MAX) a = nan_max(nan_max(a, f.x), nan_max(nan_max(f.y, f.z), f.w));
        else a = nan_min(nan_min(a, f.x), nan_min(nan_min(f.y, f.z), f.w));
      }
      c = c0 + nv * 4;
    }
    for (long long cc = c + threadIdx.x; cc < c1; cc += TPR) {
      const float t = to_f32<T>(xr[cc]);
      if (KIND == RK_SUM) a += t;
      else if (KIND == RK_MAX) a = nan_max(a, t);
      else a = nan_min(a, t);
    }
    a = row_reduce<TPR, KIND>(a, red_v);
    p.v = a; p.i = 0;
  }
  if (threadIdx.x == 0) ws[row * gridDim.x + blockIdx.x] = p;
}

template <typename T, int OP>
__global__ void __launch_bounds__(32)
row_split_final_kernel(const Partial* __restrict__ ws, int splits, void* __restrict__ out) {
  const long long row = blockIdx.x;
  const Partial* pr = ws + row * splits;
  const int lane = threadIdx.x;
  if constexpr (OP == B2_ROW_ARGMAX || OP == B2_ROW_ARGMIN) {
    constexpr bool MAXI = OP == B2_ROW_ARGMAX;
    float bv = MAXI ? -INFINITY : INFINITY;
    long long bi = 0x7fffffffffffffffLL;
    for (int s = lane; s < splits; s += 32)
      if (arg_better<MAXI>(pr[s].v, pr[s].i, bv, bi)) { bv = pr[s].v; bi = pr[s].i; }
    group_arg<32, MAXI>(bv, bi);
    if (lane == 0) reinterpret_cast<long long*>(out)[row] = bi;
  } else {
    float a = OP == B2_ROW_SUM ? 0.f : (OP == B2_ROW_MAX ? -INFINITY : INFINITY);
    for (int s = lane; s < splits; s += 32) {
      if (OP == B2_ROW_SUM) a += pr[s].v;
      else if (OP == B2_ROW_MAX) a = nan_max(a, pr[s].v);
      else a = nan_min(a, pr[s].v);
    }
    if (OP == B2_ROW_SUM) a = group_sum<32>(a);
    else if (OP == B2_ROW_MAX) a = group_max<32>(a);
    else a = group_min<32>(a);
    if (lane == 0) reinterpret_cast<T*>(out)[row] = from_f32<T>(a);
  }
}

// -------------------------------------------------------------- dispatch
int num_sms() { return device_sm_count(); }

template <typename T, int OP, int TPR, int VPT>
int launch_reg(const void* x, const void* w, const void* b, void* out, long long rows, int cols,
               long long ldx, long long ldo, float eps, cudaStream_t st) {
  constexpr int BLOCK = TPR > 32 ? TPR : 256;
  constexpr int RPB = BLOCK / TPR;
  long long blocks = (rows + RPB - 1) / RPB;
  const long long cap = (long long)num_sms() * 64;
  if (blocks > cap) blocks = cap;
  row_reg_kernel<T, OP, TPR, VPT><<<(unsigned)blocks, BLOCK, 0, st>>>(
      (const T*)x, (const T*)w, (const T*)b, out, rows, cols, ldx, ldo, eps);
  B2_CHECK_LAUNCH();
  return B2_OK;
}

// Pick threads-per-row so each thread holds 16 elements (32 for the longest rows).
template <typename T, int OP>
int dispatch_reg(const void* x, const void* w, const void* b, void* out, long long rows, int cols,
                 long long ldx, long long ldo, float eps, cudaStream_t st) {
  constexpr int EPV = Vec<T>::N;
  constexpr int V16 = 16 / EPV;  // vectors per thread for 16 elements
  const int per16 = (cols + 15) / 16;
  if constexpr ((OP == B2_ROW_ARGMAX || OP == B2_ROW_ARGMIN) && sizeof(T) == 2) {
    // packed 16-bit compares make each element cheap, so the per-row
    // cross-thread reduction dominates: 64 elements per thread (B200, fp16 /
    // bf16 argmax: 768 columns 1666 -> 3448 GB/s, 1024 2351 -> 4948, 4096
    // 3604 -> 4110 against 16-32 elements per thread)
    const int per64 = (cols + 63) / 64;
    if (per64 <= 8) return launch_reg<T, OP, 8, 4 * V16>(x, w, b, out, rows, cols, ldx, ldo, eps, st);
    if (per64 <= 16) return launch_reg<T, OP, 16, 4 * V16>(x, w, b, out, rows, cols, ldx, ldo, eps, st);
    if (per64 <= 32) return launch_reg<T, OP, 32, 4 * V16>(x, w, b, out, rows, cols, ldx, ldo, eps, st);
    if (per64 <= 64) return launch_reg<T, OP, 64, 4 * V16>(x, w, b, out, rows, cols, ldx, ldo, eps, st);
    if (per64 <= 128) return launch_reg<T, OP, 128, 4 * V16>(x, w, b, out, rows, cols, ldx, ldo, eps, st);
    if (per64 <= 256) return launch_reg<T, OP, 256, 4 * V16>(x, w, b, out, rows, cols, ldx, ldo, eps, st);
    return launch_reg<T, OP, 512, 4 * V16>(x, w, b, out, rows, cols, ldx, ldo, eps, st);
  }
  if constexpr (OP == B2_ROW_ARGMAX || OP == B2_ROW_ARGMIN) {
    // index tracking doubles the cross-thread reduction: 32 elements per
    // thread halve the threads per row (65536x4096 fp32 on B200: 0.86 -> 0.96
    // of the measured HBM copy bandwidth)
    if (per16 > 64 && per16 <= 2048) {
      const int per32 = (cols + 31) / 32;
      if (per32 <= 64) return launch_reg<T, OP, 64, 2 * V16>(x, w, b, out, rows, cols, ldx, ldo, eps, st);
      if (per32 <= 128) return launch_reg<T, OP, 128, 2 * V16>(x, w, b, out, rows, cols, ldx, ldo, eps, st);
      if (per32 <= 256) return launch_reg<T, OP, 256, 2 * V16>(x, w, b, out, rows, cols, ldx, ldo, eps, st);
      if (per32 <= 512) return launch_reg<T, OP, 512, 2 * V16>(x, w, b, out, rows, cols, ldx, ldo, eps, st);
      return launch_reg<T, OP, 1024, 2 * V16>(x, w, b, out, rows, cols, ldx, ldo, eps, st);
    }
  }
  if constexpr (OP == B2_ROW_SOFTMAX || OP == B2_ROW_LAYERNORM || OP == B2_ROW_RMSNORM ||
                OP == B2_ROW_ARGMAX || OP == B2_ROW_ARGMIN) {
    // 32 elements per thread above 512 columns: half the threads per row, so
    // a row of <= 1024 elements is one warp (no shared-memory hop) and long
    // rows need fewer barriers per reduction. Measured on B200 against 16 per
    // thread: fp32 softmax 1024 columns 4946 -> 6402 GB/s, 16384 columns
    // 4262 -> 6473; fp16 softmax 768 columns 4011 -> 5008; bf16 LayerNorm 8192
    // columns 3987 -> 4569; 256 columns lose (LayerNorm 6251 -> 5606), and
    // fp32 rows of 4096 lose 1-3 % (softmax 6449 -> 6392, LayerNorm 6416 ->
    // 6251), so short rows and fp32 rows of 1K-8K columns keep 16.
    const bool e32 = cols > 512 && (sizeof(T) == 2 || cols <= 1024 || cols > 8192);
    if (e32) {
      const int per32 = (cols + 31) / 32;
      if (per32 <= 32) return launch_reg<T, OP, 32, 2 * V16>(x, w, b, out, rows, cols, ldx, ldo, eps, st);
      if (per32 <= 64) return launch_reg<T, OP, 64, 2 * V16>(x, w, b, out, rows, cols, ldx, ldo, eps, st);
      if (per32 <= 128) return launch_reg<T, OP, 128, 2 * V16>(x, w, b, out, rows, cols, ldx, ldo, eps, st);
      if (per32 <= 256) return launch_reg<T, OP, 256, 2 * V16>(x, w, b, out, rows, cols, ldx, ldo, eps, st);
      if (per32 <= 512) return launch_reg<T, OP, 512, 2 * V16>(x, w, b, out, rows, cols, ldx, ldo, eps, st);
      return launch_reg<T, OP, 1024, 2 * V16>(x, w, b, out, rows, cols, ldx, ldo, eps, st);
    }
  }
  if (per16 <= 8) return launch_reg<T, OP, 8, V16>(x, w, b, out, rows, cols, ldx, ldo, eps, st);
  if (per16 <= 16) return launch_reg<T, OP, 16, V16>(x, w, b, out, rows, cols, ldx, ldo, eps, st);
  if (per16 <= 32) return launch_reg<T, OP, 32, V16>(x, w, b, out, rows, cols, ldx, ldo, eps, st);
  if (per16 <= 64) return launch_reg<T, OP, 64, V16>(x, w, b, out, rows, cols, ldx, ldo, eps, st);
  if (per16 <= 128) return launch_reg<T, OP, 128, V16>(x, w, b, out, rows, cols, ldx, ldo, eps, st);
  if (per16 <= 256) return launch_reg<T, OP, 256, V16>(x, w, b, out, rows, cols, ldx, ldo, eps, st);
  if (per16 <= 512) return launch_reg<T, OP, 512, V16>(x, w, b, out, rows, cols, ldx, ldo, eps, st);
  if (per16 <= 1024) return launch_reg<T, OP, 1024, V16>(x, w, b, out, rows, cols, ldx, ldo, eps, st);
  return launch_reg<T, OP, 1024, 2 * V16>(x, w, b, out, rows, cols, ldx, ldo, eps, st);
}

constexpr long long kSplitChunk = 1 << 16;  // elements per CTA on the split path

bool use_split(int op, long long rows, long long cols) {
  const bool scalar_op = op == B2_ROW_SUM || op == B2_ROW_MAX || op == B2_ROW_MIN ||
                         op == B2_ROW_ARGMAX || op == B2_ROW_ARGMIN;
  return scalar_op && cols >= 4 * kSplitChunk && rows < 2LL * num_sms();
}

template <typename T, int OP>
int dispatch_op(const void* x, const void* w, const void* b, void* out, long long rows,
                long long cols, long long ldx, long long ldo, float eps, void* ws, size_t ws_bytes,
                cudaStream_t st) {
  constexpr int EPV = Vec<T>::N;
  if (use_split(OP, rows, cols)) {
    const long long splits = (cols + kSplitChunk - 1) / kSplitChunk;
    const size_t need = (size_t)(rows * splits) * sizeof(Partial);
    if (ws == nullptr || ws_bytes < need) {
      set_error("b2_row_op: split-row path needs %zu workspace bytes, got %zu", need, ws_bytes);
      return B2_EINVAL;
    }
    if ((reinterpret_cast<uintptr_t>(ws) & 15) != 0) {
      set_error("b2_row_op: workspace must be 16-byte aligned");
      return B2_EINVAL;
    }
    dim3 grid((unsigned)splits, (unsigned)rows);
    row_split_partial_kernel<T, OP><<<grid, 512, 0, st>>>((const T*)x, cols, ldx, kSplitChunk,
                                                          (Partial*)ws);
    B2_CHECK_LAUNCH();
    row_split_final_kernel<T, OP><<<(unsigned)rows, 32, 0, st>>>((const Partial*)ws, (int)splits, out);
    B2_CHECK_LAUNCH();
    return B2_OK;
  }
  const bool row_out = OP == B2_ROW_SOFTMAX || OP == B2_ROW_LAYERNORM || OP == B2_ROW_RMSNORM;
  auto al16 = [](const void* p) { return p == nullptr || (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  const bool aligned = cols % EPV == 0 && ldx % EPV == 0 && al16(x) && al16(w) && al16(b) &&
                       (!row_out || (ldo % EPV == 0 && al16(out)));
  if (aligned && cols <= 32 * 1024 && cols > 0) {
    return dispatch_reg<T, OP>(x, w, b, out, rows, (int)cols, ldx, ldo, eps, st);
  }
  if (aligned && cols < (1LL << 31)) {
    long long blocks = rows;
    const long long cap = (long long)num_sms() * kLongCtas;
    if (blocks > cap) blocks = cap;
    row_long_kernel<T, OP><<<(unsigned)blocks, kLongTPR, 0, st>>>((const T*)x, (const T*)w, (const T*)b,
                                                                 out, rows, (int)cols, ldx, ldo, eps);
    B2_CHECK_LAUNCH();
    return B2_OK;
  }
  long long blocks = rows;
  const long long cap = (long long)num_sms() * 16;
  if (blocks > cap) blocks = cap;
  row_generic_kernel<T, OP><<<(unsigned)blocks, 512, 0, st>>>((const T*)x, (const T*)w,
                                                               (const T*)b, out, rows, cols, ldx,
                                                               ldo, eps);
  B2_CHECK_LAUNCH();
  return B2_OK;
}

template <typename T>
int dispatch_type(int op, const void* x, const void* w, const void* b, void* out, long long rows,
                  long long cols, long long ldx, long long ldo, float eps, void* ws,
                  size_t ws_bytes, cudaStream_t st) {
  switch (op) {
#define B2_ROW_CASE(OPV) \
  case OPV: return dispatch_op<T, OPV>(x, w, b, out, rows, cols, ldx, ldo, eps, ws, ws_bytes, st);
    B2_ROW_CASE(B2_ROW_SOFTMAX)
    B2_ROW_CASE(B2_ROW_LAYERNORM)
    B2_ROW_CASE(B2_ROW_RMSNORM)
    B2_ROW_CASE(B2_ROW_SUM)
    B2_ROW_CASE(B2_ROW_MAX)
    B2_ROW_CASE(B2_ROW_ARGMAX)
    B2_ROW_CASE(B2_ROW_MIN)
    B2_ROW_CASE(B2_ROW_ARGMIN)
#undef B2_ROW_CASE
    default:
      set_error("b2_row_op: unknown op %d", op);
      return B2_EINVAL;
  }
}

// ------------------------------------------------ reduction over a middle axis
// rows unrolled per thread, and target CTAs per SM (measured on B200 for
// sum over dim 0 of [65536, 4096] and dim 1 of [16, 4096, 4096]: 4-16 rows and
// 4 CTAs/SM within 2 %, 8 CTAs/SM 10-20 % slower)
constexpr int kAxisUnroll = 8, kAxisWant = 4;
// x[outer, R, inner] (contiguous) -> out[outer, inner], reducing over R
// (torch's sum / amax / amin / argmax / argmin along a dim that is not the last:
// the reference fuzzer's 2d_sum_ax0 / 3d_sum_ax0 forms, tests/test_fuzz_reduce.py:88-139).
// A thread owns VEC consecutive inner elements (consecutive threads, consecutive
// addresses: every warp load is coalesced) and walks its R range; grid.z splits R
// when the (inner, outer) grid alone would not fill the SMs, partials to the
// workspace and a second pass folds them in split order.
template <typename T, int OP, int VEC, typename IDX>
__global__ void __launch_bounds__(256)
axis_reduce_kernel(const T* __restrict__ x, long long outer, long long R, long long inner,
                   long long r_chunk, int splits, Partial* __restrict__ ws, void* __restrict__ out) {
  const long long i0 = ((long long)blockIdx.x * blockDim.x + threadIdx.x) * VEC;
  if (i0 >= inner) return;
  const long long r0 = (long long)blockIdx.z * r_chunk;
  const long long r1 = r0 + r_chunk < R ? r0 + r_chunk : R;
  if (r0 >= r1) return;
  constexpr bool ARG = OP == B2_ROW_ARGMAX || OP == B2_ROW_ARGMIN;
  constexpr bool MAXI = OP == B2_ROW_ARGMAX;
  // one row's VEC elements of this thread as fp32
  auto load = [&](const T* xo, long long r, float (&f)[VEC]) {
    if constexpr (VEC == 4 && sizeof(T) == 4) {
      const float4 q = __ldcs(reinterpret_cast<const float4*>(xo + r * inner));
      f[0] = q.x; f[1] = q.y; f[2] = q.z; f[3] = q.w;
    } else {
#pragma unroll
      for (int e = 0; e < VEC; ++e) f[e] = (i0 + e < inner) ? to_f32<T>(xo[r * inner + e]) : 0.f;
    }
  };
  // Fold one later row into the running value. Rows arrive in ascending order,
  // so for argmax/argmin a tie keeps the earlier row (the lower index) and the
  // first NaN, once taken, is never replaced. IDX is the row offset from r0.
  auto fold = [&](float& a, IDX& ia, float f, IDX rf) {
    if constexpr (ARG) {
      const bool better = (MAXI ? f > a : f < a) || (f != f && a == a);
      a = better ? f : a;
      ia = better ? rf : ia;
    } else if constexpr (OP == B2_ROW_SUM) {
      a += f;
    } else if constexpr (OP == B2_ROW_MAX) {
      a = nan_max(a, f);
    } else {
      a = nan_min(a, f);
    }
  };
  for (long long o = blockIdx.y; o < outer; o += gridDim.y) {
    const T* xo = x + o * R * inner + i0;
    float acc[VEC];
    IDX idx[VEC];
    load(xo, r0, acc);
#pragma unroll
    for (int e = 0; e < VEC; ++e) idx[e] = 0;
    long long r = r0 + 1;
    // kAxisUnroll rows' loads issued before any of them is folded
    for (; r + kAxisUnroll <= r1; r += kAxisUnroll) {
      float f[kAxisUnroll][VEC];
#pragma unroll
      for (int u = 0; u < kAxisUnroll; ++u) load(xo, r + u, f[u]);
#pragma unroll
      for (int u = 0; u < kAxisUnroll; ++u)
#pragma unroll
        for (int e = 0; e < VEC; ++e) fold(acc[e], idx[e], f[u][e], (IDX)(r + u - r0));
    }
    for (; r < r1; ++r) {
      float f[VEC];
      load(xo, r, f);
#pragma unroll
      for (int e = 0; e < VEC; ++e) fold(acc[e], idx[e], f[e], (IDX)(r - r0));
    }
#pragma unroll
    for (int e = 0; e < VEC; ++e) {
      if (i0 + e >= inner) break;
      const long long oi = o * inner + i0 + e;
      if (splits > 1) {
        Partial p;
        p.v = acc[e];
        p.pad = 0;
        p.i = r0 + (long long)idx[e];
        ws[(long long)blockIdx.z * outer * inner + oi] = p;
      } else if (ARG) {
        reinterpret_cast<long long*>(out)[oi] = r0 + (long long)idx[e];
      } else {
        reinterpret_cast<T*>(out)[oi] = from_f32<T>(acc[e]);
      }
    }
  }
}

template <typename T, int OP>
__global__ void __launch_bounds__(256)
axis_reduce_final_kernel(const Partial* __restrict__ ws, long long n, int splits, void* __restrict__ out) {
  constexpr bool ARG = OP == B2_ROW_ARGMAX || OP == B2_ROW_ARGMIN;
  constexpr bool MAXI = OP == B2_ROW_ARGMAX;
  for (long long k = (long long)blockIdx.x * blockDim.x + threadIdx.x; k < n;
       k += (long long)gridDim.x * blockDim.x) {
    Partial p = ws[k];
    float a = p.v;
    long long ai = p.i;
#pragma unroll 8
    for (int sp = 1; sp < splits; ++sp) {
      const Partial q = ws[(long long)sp * n + k];
      if (ARG) {
        if (arg_better<MAXI>(q.v, q.i, a, ai)) { a = q.v; ai = q.i; }
      } else if (OP == B2_ROW_SUM) {
        a += q.v;
      } else if (OP == B2_ROW_MAX) {
        a = nan_max(a, q.v);
      } else {
        a = nan_min(a, q.v);
      }
    }
    if (ARG) reinterpret_cast<long long*>(out)[k] = ai;
    else reinterpret_cast<T*>(out)[k] = from_f32<T>(a);
  }
}

struct AxisPlan {
  int vec = 1, splits = 1;
  long long r_chunk = 0, xblocks = 0;
  size_t ws = 0;
};

AxisPlan axis_plan(long long outer, long long R, long long inner, bool vec4) {
  AxisPlan p;
  p.vec = vec4 ? 4 : 1;
  p.xblocks = (inner + 256LL * p.vec - 1) / (256LL * p.vec);
  const long long blocks = p.xblocks * outer;
  // enough CTAs for every SM to hold several (memory-level parallelism), each
  // still reading at least 128 rows
  const long long want = (long long)kAxisWant * num_sms();
  long long sp = 1;
  if (blocks < want && R >= 256) {
    sp = (want + blocks - 1) / blocks;
    if (sp > R / 128) sp = R / 128;
    if (sp > 256) sp = 256;
    if (sp < 1) sp = 1;
  }
  p.r_chunk = (R + sp - 1) / sp;
  p.splits = (int)((R + p.r_chunk - 1) / p.r_chunk);
  if (p.splits > 1) p.ws = (size_t)p.splits * (size_t)outer * (size_t)inner * sizeof(Partial);
  return p;
}

template <typename T, int OP>
int axis_launch(const void* x, void* out, long long outer, long long R, long long inner, void* ws,
                size_t ws_bytes, cudaStream_t st) {
  const bool vec4 = sizeof(T) == 4 && inner % 4 == 0 && (reinterpret_cast<uintptr_t>(x) & 15) == 0;
  AxisPlan p = axis_plan(outer, R, inner, vec4);
  if (p.splits > 1 && (ws == nullptr || ws_bytes < p.ws || (reinterpret_cast<uintptr_t>(ws) & 15))) {
    // without the workspace: one pass (correct, fewer CTAs)
    p.splits = 1;
    p.r_chunk = R;
  }
  const dim3 grid((unsigned)p.xblocks, (unsigned)(outer < 65535 ? outer : 65535), (unsigned)p.splits);
  // row offsets within a split as int32 unless a split spans 2^31 rows
  const bool wide = p.r_chunk > 0x7fffffffLL;
  if (p.vec == 4 && !wide)
    axis_reduce_kernel<T, OP, 4, int><<<grid, 256, 0, st>>>((const T*)x, outer, R, inner, p.r_chunk,
                                                            p.splits, (Partial*)ws, out);
  else if (p.vec == 4)
    axis_reduce_kernel<T, OP, 4, long long><<<grid, 256, 0, st>>>((const T*)x, outer, R, inner, p.r_chunk,
                                                                  p.splits, (Partial*)ws, out);
  else if (!wide)
    axis_reduce_kernel<T, OP, 1, int><<<grid, 256, 0, st>>>((const T*)x, outer, R, inner, p.r_chunk,
                                                            p.splits, (Partial*)ws, out);
  else
    axis_reduce_kernel<T, OP, 1, long long><<<grid, 256, 0, st>>>((const T*)x, outer, R, inner, p.r_chunk,
                                                                  p.splits, (Partial*)ws, out);
  B2_CHECK_LAUNCH();
  if (p.splits > 1) {
    const long long n = outer * inner;
    long long blocks = (n + 255) / 256;
    if (blocks > 16LL * num_sms()) blocks = 16LL * num_sms();
    axis_reduce_final_kernel<T, OP><<<(unsigned)blocks, 256, 0, st>>>((const Partial*)ws, n, p.splits, out);
    B2_CHECK_LAUNCH();
  }
  return B2_OK;
}

template <typename T>
int axis_dispatch(int op, const void* x, void* out, long long outer, long long R, long long inner,
                  void* ws, size_t ws_bytes, cudaStream_t st) {
  switch (op) {
    case B2_ROW_SUM: return axis_launch<T, B2_ROW_SUM>(x, out, outer, R, inner, ws, ws_bytes, st);
    case B2_ROW_MAX: return axis_launch<T, B2_ROW_MAX>(x, out, outer, R, inner, ws, ws_bytes, st);
    case B2_ROW_MIN: return axis_launch<T, B2_ROW_MIN>(x, out, outer, R, inner, ws, ws_bytes, st);
    case B2_ROW_ARGMAX: return axis_launch<T, B2_ROW_ARGMAX>(x, out, outer, R, inner, ws, ws_bytes, st);
    case B2_ROW_ARGMIN: return axis_launch<T, B2_ROW_ARGMIN>(x, out, outer, R, inner, ws, ws_bytes, st);
  }
  set_error("b2_reduce_axis: op %d is not sum/max/min/argmax/argmin", op);
  return B2_EINVAL;
}

}  // namespace

size_t axis_reduce_workspace(long long outer, long long R, long long inner) {
  if (outer <= 0 || R <= 0 || inner <= 0) return 0;
  return axis_plan(outer, R, inner, true).ws > axis_plan(outer, R, inner, false).ws
             ? axis_plan(outer, R, inner, true).ws
             : axis_plan(outer, R, inner, false).ws;
}

int axis_reduce_launch(int op, const void* x, void* out, long long outer, long long R, long long inner,
                       int dtype, void* ws, size_t ws_bytes, cudaStream_t st) {
  switch (dtype) {
    case B2_F32: return axis_dispatch<float>(op, x, out, outer, R, inner, ws, ws_bytes, st);
    case B2_F16: return axis_dispatch<__half>(op, x, out, outer, R, inner, ws, ws_bytes, st);
    case B2_BF16: return axis_dispatch<__nv_bfloat16>(op, x, out, outer, R, inner, ws, ws_bytes, st);
  }
  set_error("b2_reduce_axis: unsupported dtype %d", dtype);
  return B2_EINVAL;
}

size_t row_op_workspace(int op, long long rows, long long cols) {
  if (rows <= 0 || cols <= 0 || !use_split(op, rows, cols)) return 0;
  const long long splits = (cols + kSplitChunk - 1) / kSplitChunk;
  return (size_t)(rows * splits) * sizeof(Partial);
}

int row_op_launch(int op, const void* x, const void* w, const void* b, void* out, long long rows,
                  long long cols, long long ldx, long long ldo, float eps, int dtype, void* ws,
                  size_t ws_bytes, cudaStream_t st) {
  switch (dtype) {
    case B2_F32: return dispatch_type<float>(op, x, w, b, out, rows, cols, ldx, ldo, eps, ws, ws_bytes, st);
    case B2_F16: return dispatch_type<__half>(op, x, w, b, out, rows, cols, ldx, ldo, eps, ws, ws_bytes, st);
    case B2_BF16: return dispatch_type<__nv_bfloat16>(op, x, w, b, out, rows, cols, ldx, ldo, eps, ws, ws_bytes, st);
    default:
      set_error("b2_row_op: unsupported dtype %d", dtype);
      return B2_EINVAL;
  }
}

uint32_t row_read_status(bool clear) {
  uint32_t s = 0;
  cudaMemcpyFromSymbol(&s, g_row_status, sizeof(s));
  if (clear) {
    const uint32_t z = 0;
    cudaMemcpyToSymbol(g_row_status, &z, sizeof(z));
  }
  return s;
}

}  // namespace b2

// ---------------------------------------------------------------------------
// Allocation-free variant of the split-row reduction.
//
// Some callers cannot allocate device memory at the point where they reduce:
// code running inside a custom allocator or an out-of-memory handler, a
// library that must not touch the process's CUDA memory pool, or a host
// runtime that forbids cudaMalloc after start-up. For them the split path's
// scratch lives in a fixed array in this library's device image instead of a
// caller-provided workspace. Every GPU that loads the library reserves it
// until the process exits.
namespace b2 {
namespace {

constexpr long long kNoAllocMaxPartials = 16384;  // 16384 x 16 B = 256 KiB per device
static __device__ __align__(256) Partial g_row_noalloc_scratch[kNoAllocMaxPartials];

// Device address of the array per device ordinal, looked up with that device
// current (host code only sees a host-side stand-in under the array's name).
// A successful lookup is cached; a failed one is not, so the next call tries
// again. The mutex makes the first lookup safe from several host threads.
constexpr int kNoAllocMaxDev = 64;
Partial* g_noalloc_ptr[kNoAllocMaxDev];
std::mutex g_noalloc_mu;

cudaError_t noalloc_scratch(int dev, Partial** out) {
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (g_noalloc_ptr[dev] == nullptr) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_row_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr) {
      *out = nullptr;
      return e != cudaSuccess ? e : cudaErrorInvalidSymbol;
    }
    g_noalloc_ptr[dev] = static_cast<Partial*>(p);
  }
  *out = g_noalloc_ptr[dev];
  return cudaSuccess;
}

template <typename T, int OP>
int noalloc_launch(const void* x, void* out, long long rows, long long cols, long long ldx,
                   Partial* scratch, long long splits, cudaStream_t st) {
  dim3 grid((unsigned)splits, (unsigned)rows);
  row_split_partial_kernel<T, OP><<<grid, 512, 0, st>>>((const T*)x, cols, ldx, kSplitChunk, scratch);
  B2_CHECK_LAUNCH();
  row_split_final_kernel<T, OP><<<(unsigned)rows, 32, 0, st>>>(scratch, (int)splits, out);
  B2_CHECK_LAUNCH();
  return B2_OK;
}

template <typename T>
int noalloc_dispatch(int op, const void* x, void* out, long long rows, long long cols,
                     long long ldx, Partial* scratch, long long splits, cudaStream_t st) {
  switch (op) {
    case B2_ROW_SUM: return noalloc_launch<T, B2_ROW_SUM>(x, out, rows, cols, ldx, scratch, splits, st);
    case B2_ROW_MAX: return noalloc_launch<T, B2_ROW_MAX>(x, out, rows, cols, ldx, scratch, splits, st);
    case B2_ROW_MIN: return noalloc_launch<T, B2_ROW_MIN>(x, out, rows, cols, ldx, scratch, splits, st);
    case B2_ROW_ARGMAX: return noalloc_launch<T, B2_ROW_ARGMAX>(x, out, rows, cols, ldx, scratch, splits, st);
    case B2_ROW_ARGMIN: return noalloc_launch<T, B2_ROW_ARGMIN>(x, out, rows, cols, ldx, scratch, splits, st);
  }
  set_error("b2_row_reduce_noalloc: op %d is not a scalar reduction (sum/max/min/argmax/argmin)", op);
  return B2_EINVAL;
}

}  // namespace
}  // namespace b2

extern "C" __attribute__((visibility("default")))
int b2_row_reduce_noalloc(int op, const void* x, void* out, int64_t rows, int64_t cols,
                          int64_t ld_x, int dtype, void* stream) {
  using namespace b2;
  clear_error();
  if (op != B2_ROW_SUM && op != B2_ROW_MAX && op != B2_ROW_MIN && op != B2_ROW_ARGMAX &&
      op != B2_ROW_ARGMIN) {
    set_error("b2_row_reduce_noalloc: op %d is not a scalar reduction (sum/max/min/argmax/argmin)", op);
    return B2_EINVAL;
  }
  if (dtype != B2_F32 && dtype != B2_F16 && dtype != B2_BF16) {
    set_error("b2_row_reduce_noalloc: unsupported dtype %d", dtype);
    return B2_EINVAL;
  }
  if (rows < 0 || cols <= 0 || ld_x < cols) {
    set_error("b2_row_reduce_noalloc: invalid shape rows=%lld cols=%lld ld_x=%lld (cols must be > 0)",
              (long long)rows, (long long)cols, (long long)ld_x);
    return B2_EINVAL;
  }
  if (rows == 0) return B2_OK;
  if (!x || !out) {
    set_error("b2_row_reduce_noalloc: null pointer argument");
    return B2_EINVAL;
  }
  const long long splits = (cols + kSplitChunk - 1) / kSplitChunk;
  if (rows > kNoAllocMaxPartials || rows * splits > kNoAllocMaxPartials) {
    set_error("b2_row_reduce_noalloc: rows * ceil(cols / %lld) = %lld exceeds the fixed scratch of "
              "%lld partials; use b2_row_op with a workspace instead",
              kSplitChunk, rows * splits, kNoAllocMaxPartials);
    return B2_EINVAL;
  }
  int dev = 0;
  B2_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kNoAllocMaxDev) {
    set_error("b2_row_reduce_noalloc: device ordinal %d out of range", dev);
    return B2_EINVAL;
  }
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (st != nullptr) {
    // The array's address is per device: the stream must belong to the
    // current device, or the kernels would write another GPU's copy.
    int sdev = dev;
    if (cudaStreamGetDevice(st, &sdev) == cudaSuccess && sdev != dev) {
      set_error("b2_row_reduce_noalloc: stream belongs to device %d but device %d is current", sdev, dev);
      return B2_EINVAL;
    }
    cudaGetLastError();
  }
  // First call on this device: resolve the array's device address (the
  // current device is the one being set up). A failure is reported and
  // retried on the next call.
  Partial* scratch = nullptr;
  const cudaError_t le = noalloc_scratch(dev, &scratch);
  if (le != cudaSuccess) {
    cudaGetLastError();
    set_error("b2_row_reduce_noalloc: cudaGetSymbolAddress failed on device %d: %s", dev,
              cudaGetErrorString(le));
    return B2_ELAUNCH;
  }
  switch (dtype) {
    case B2_F32: return noalloc_dispatch<float>(op, x, out, rows, cols, ld_x, scratch, splits, st);
    case B2_F16: return noalloc_dispatch<__half>(op, x, out, rows, cols, ld_x, scratch, splits, st);
    default: return noalloc_dispatch<__nv_bfloat16>(op, x, out, rows, cols, ld_x, scratch, splits, st);
  }
}
