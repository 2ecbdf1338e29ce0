// GEMM with fused epilogue, CUDA-core (FFMA) variant.
//
// Serves fp32 inputs (the reference's fp32 fast-matmul config, checked at
// 1e-4 max-abs: plain TF32 tensor cores cannot meet it) and any operand whose
// strides the TMA path cannot describe (non-unit inner stride, unaligned rows).
// It plays the role of the reference's stride-aware generic matmul
// (_lowerer_templates.py:128-258 `_lower_strided_scalar_matmul`) and of the
// fp32 fast template (_msl_templates.py:4134-4255), with the epilogue of
// _lowerer_templates.py:1515-1855 (column bias, activation) fused.
//
// Tiling: 128x128 C tile, K step 8, 256 threads, 8x8 outputs per thread split
// into four 4x4 quadrants (conflict-free float4 shared-memory reads), global
// loads for step k+1 issued before the FMAs of step k.
#include "b2_common.cuh"

namespace b2 {
namespace {

constexpr int BM = 128, BN = 128, BK = 8, NT = 256;

template <typename TI, typename TO, typename TB>
__global__ void __launch_bounds__(NT)
gemm_simt_kernel(const TI* __restrict__ A, const TI* __restrict__ B, const TB* __restrict__ bias,
                 TO* __restrict__ C, int M, int N, int K, long long sam, long long sak,
                 long long sbk, long long sbn, long long scm, long long scn, float alpha, int act,
                 const EpiProgram prog) {
  __shared__ __align__(16) float As[2][BK][BM];
  __shared__ __align__(16) float Bs[2][BK][BN];
  const int tid = threadIdx.x;
  const int m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;
  const int tx = tid & 15, ty = tid >> 4;

  // Loader mapping: A tile 128x8 -> each thread loads 4 (rows a_r, k a_k..a_k+3)
  const int a_r = tid >> 1, a_k = (tid & 1) * 4;
  // B tile 8x128 -> each thread loads 4 (k b_k, cols b_n..b_n+3)
  const int b_k = tid >> 5, b_n = (tid & 31) * 4;

  float ra[4], rb[4];
  auto load_regs = [&](int k0) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int m = m0 + a_r, kk = k0 + a_k + j;
      ra[j] = (m < M && kk < K) ? to_f32<TI>(A[m * sam + kk * sak]) : 0.f;
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int kk = k0 + b_k, n = n0 + b_n + j;
      rb[j] = (kk < K && n < N) ? to_f32<TI>(B[kk * sbk + n * sbn]) : 0.f;
    }
  };
  auto store_smem = [&](int buf) {
#pragma unroll
    for (int j = 0; j < 4; ++j) As[buf][a_k + j][a_r] = ra[j];
    *reinterpret_cast<float4*>(&Bs[buf][b_k][b_n]) = make_float4(rb[0], rb[1], rb[2], rb[3]);
  };

  float acc[8][8];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[i][j] = 0.f;

  load_regs(0);
  store_smem(0);
  __syncthreads();
  int buf = 0;
  for (int k0 = 0; k0 < K; k0 += BK) {
    const bool more = k0 + BK < K;
    if (more) load_regs(k0 + BK);
#pragma unroll
    for (int kk = 0; kk < BK; ++kk) {
      const float4 a0 = *reinterpret_cast<const float4*>(&As[buf][kk][ty * 4]);
      const float4 a1 = *reinterpret_cast<const float4*>(&As[buf][kk][64 + ty * 4]);
      const float4 b0 = *reinterpret_cast<const float4*>(&Bs[buf][kk][tx * 4]);
      const float4 b1 = *reinterpret_cast<const float4*>(&Bs[buf][kk][64 + tx * 4]);
      const float av[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
      const float bv[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
    }
    if (more) {
      store_smem(buf ^ 1);
      __syncthreads();
      buf ^= 1;
    }
  }

#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int m = m0 + (i < 4 ? ty * 4 + i : 64 + ty * 4 + (i - 4));
    if (m >= M) continue;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int n = n0 + (j < 4 ? tx * 4 + j : 64 + tx * 4 + (j - 4));
      if (n >= N) continue;
      float c = acc[i][j] * alpha;
      if (act == kActChain) {
        C[m * scm + n * scn] = from_f32<TO>(epi_chain(c, bias ? to_f32<TB>(bias[n]) : 0.f, prog));
        continue;
      }
      if (bias) c += to_f32<TB>(bias[n]);
      C[m * scm + n * scn] = from_f32<TO>(apply_act(c, act));
    }
  }
}

template <typename TI, typename TO, typename TB>
int launch3(const void* A, const void* B, const void* bias, void* C, long long M, long long N,
            long long K, const int64_t* s, float alpha, int act, cudaStream_t st) {
  dim3 grid((unsigned)((N + BN - 1) / BN), (unsigned)((M + BM - 1) / BM));
  gemm_simt_kernel<TI, TO, TB><<<grid, NT, 0, st>>>((const TI*)A, (const TI*)B, (const TB*)bias,
                                                    (TO*)C, (int)M, (int)N, (int)K, s[0], s[1],
                                                    s[2], s[3], s[4], s[5], alpha, act, epi_program());
  B2_CHECK_LAUNCH();
  return B2_OK;
}

template <typename TI, typename TO>
int launch2(const void* A, const void* B, const void* bias, int bias_dt, void* C, long long M,
            long long N, long long K, const int64_t* s, float alpha, int act, cudaStream_t st) {
  switch (bias_dt) {
    case B2_F32: return launch3<TI, TO, float>(A, B, bias, C, M, N, K, s, alpha, act, st);
    case B2_F16: return launch3<TI, TO, __half>(A, B, bias, C, M, N, K, s, alpha, act, st);
    case B2_BF16: return launch3<TI, TO, __nv_bfloat16>(A, B, bias, C, M, N, K, s, alpha, act, st);
  }
  set_error("b2_gemm: unsupported bias dtype %d", bias_dt);
  return B2_EINVAL;
}

template <typename TI>
int launch1(const void* A, const void* B, const void* bias, int bias_dt, void* C, int out_dt,
            long long M, long long N, long long K, const int64_t* s, float alpha, int act,
            cudaStream_t st) {
  switch (out_dt) {
    case B2_F32: return launch2<TI, float>(A, B, bias, bias_dt, C, M, N, K, s, alpha, act, st);
    case B2_F16: return launch2<TI, __half>(A, B, bias, bias_dt, C, M, N, K, s, alpha, act, st);
    case B2_BF16: return launch2<TI, __nv_bfloat16>(A, B, bias, bias_dt, C, M, N, K, s, alpha, act, st);
  }
  set_error("b2_gemm: unsupported out dtype %d", out_dt);
  return B2_EINVAL;
}

}  // namespace

int gemm_simt_launch(const void* A, const void* B, const void* bias, void* C, long long M,
                     long long N, long long K, const int64_t* strides, float alpha, int act,
                     int in_dt, int bias_dt, int out_dt, cudaStream_t st) {
  if (M >= (1LL << 31) || N >= (1LL << 31) || K >= (1LL << 31)) {
    set_error("b2_gemm: dims must be < 2^31");
    return B2_EINVAL;
  }
  if (bias == nullptr) bias_dt = B2_F32;
  switch (in_dt) {
    case B2_F32: return launch1<float>(A, B, bias, bias_dt, C, out_dt, M, N, K, strides, alpha, act, st);
    case B2_F16: return launch1<__half>(A, B, bias, bias_dt, C, out_dt, M, N, K, strides, alpha, act, st);
    case B2_BF16: return launch1<__nv_bfloat16>(A, B, bias, bias_dt, C, out_dt, M, N, K, strides, alpha, act, st);
  }
  set_error("b2_gemm: unsupported input dtype %d", in_dt);
  return B2_EINVAL;
}

}  // namespace b2
