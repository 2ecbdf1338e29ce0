// FlashAttention forward, CUDA-core (FFMA) variant.
//
// Serves what the tcgen05 kernel does not: fp32 inputs (the reference's fp32
// config, checked at 1e-4 max-abs, which TF32 tensor cores cannot meet),
// non-unit inner strides, and head dims outside {32, 64, 128}.
//
// Semantics follow the reference's canonical kernel `_flash_attn_fwd`
// (tests/test_flash_attention.py:35-118): q is multiplied by the scale before
// Q.K^T, online max / exp / sum per BLOCK_N keys, causal keep iff key <= query
// with the key loop bounded by the end of the query block, acc / l at the end.
// Rows whose keys are all masked return 0 (reference oracle nan_to_num,
// tests/test_flash_attention.py:124-135).
//
// Tiling: 16*RPT query rows x 64 keys per step, 256 threads; thread (rg, cg)
// owns rows RPT*rg..RPT*rg+RPT-1 and columns cg + 16*j. RPT = 4 (64-row tiles)
// normally; RPT = 1 (16-row tiles, four times the CTAs) when 64-row tiles would
// leave most SMs idle (the fp32 [1,4,256,64] configuration: 64 CTAs instead of
// 16). Q, K, V, P staged in shared memory as fp32 (padded rows, conflict-free).
#include "b2_common.cuh"

namespace b2 {
namespace {

constexpr int kBN = 64, kThreads = 256;

template <typename T, int DMAX, int RPT>
__global__ void __launch_bounds__(kThreads)
fa_simt_kernel(const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ v,
               T* __restrict__ o, int H, int S, int D, const long long* __restrict__ st_dev,
               long long sqz, long long sqh, long long sqm, long long sqk,
               long long skz, long long skh, long long skn, long long skk,
               long long svz, long long svh, long long svn, long long svk,
               long long soz, long long soh, long long som, long long sok,
               float scale, int causal) {
  constexpr int kBM = 16 * RPT;
  extern __shared__ float smem[];
  constexpr int DP = DMAX + 1;
  float* Qs = smem;                 // [kBM][DP]
  float* Ks = Qs + kBM * DP;        // [kBN][DP]
  float* Vs = Ks + kBN * DP;        // [kBN][DMAX]
  float* Ps = Vs + kBN * DMAX;      // [kBM][kBN + 1]
  (void)st_dev;

  const int qblk = blockIdx.x;
  const int zh = blockIdx.y;
  const int z = zh / H, h = zh % H;
  const int m0 = qblk * kBM;
  const T* qb = q + z * sqz + h * sqh;
  const T* kb = k + z * skz + h * skh;
  const T* vb = v + z * svz + h * svh;
  T* ob = o + z * soz + h * soh;

  const int tid = threadIdx.x;
  const int rg = tid >> 4, cg = tid & 15;
  constexpr int NJ = DMAX / 16;

  // Stage q * scale (the reference scales q before the dot).
  {
    constexpr int PQ = (kBM * DMAX + kThreads - 1) / kThreads;
    float qr[PQ];
#pragma unroll
    for (int it = 0; it < PQ; ++it) {
      const int idx = tid + it * kThreads;
      const int r = idx / D, d = idx % D;
      const int m = m0 + r;
      qr[it] = (idx < kBM * D && m < S) ? to_f32<T>(qb[(long long)m * sqm + d * sqk]) * scale : 0.f;
    }
#pragma unroll
    for (int it = 0; it < PQ; ++it) {
      const int idx = tid + it * kThreads;
      if (idx < kBM * D) Qs[(idx / D) * DP + idx % D] = qr[it];
    }
  }

  float acc[RPT][NJ];
  float mrow[RPT], lrow[RPT];
#pragma unroll
  for (int i = 0; i < RPT; ++i) {
    mrow[i] = -INFINITY;
    lrow[i] = 0.f;
#pragma unroll
    for (int j = 0; j < NJ; ++j) acc[i][j] = 0.f;
  }

  int hi = S;
  if (causal) hi = min(m0 + kBM, S);
  // K and V of the next block are loaded into registers while the current one
  // is computed (all of a thread's elements in flight together), then stored to
  // shared memory at the top of the next iteration.
  constexpr int PER = kBN * DMAX / kThreads;
  float kr[PER], vr[PER];
  auto load_kv = [&](int nb) {
#pragma unroll
    for (int it = 0; it < PER; ++it) {
      const int idx = tid + it * kThreads;
      const int r = idx / D, d = idx % D;
      const int n = nb + r;
      const bool ok = idx < kBN * D && n < S;
      kr[it] = ok ? to_f32<T>(kb[(long long)n * skn + d * skk]) : 0.f;
      vr[it] = ok ? to_f32<T>(vb[(long long)n * svn + d * svk]) : 0.f;
    }
  };
  // (head dims up to 64; at 128 the second set of registers would spill, so
  // the block's own loads are issued at the top of its iteration instead)
  constexpr bool kPipe = DMAX <= 64;
  if (kPipe && hi > 0) load_kv(0);
  for (int n0 = 0; n0 < hi; n0 += kBN) {
    if (!kPipe) load_kv(n0);
    __syncthreads();
#pragma unroll
    for (int it = 0; it < PER; ++it) {
      const int idx = tid + it * kThreads;
      if (idx < kBN * D) {
        const int r = idx / D, d = idx % D;
        Ks[r * DP + d] = kr[it];
        Vs[r * DMAX + d] = vr[it];
      }
    }
    __syncthreads();
    if (kPipe && n0 + kBN < hi) load_kv(n0 + kBN);

    float s[RPT][4];
#pragma unroll
    for (int i = 0; i < RPT; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) s[i][j] = 0.f;
    for (int d = 0; d < D; ++d) {
      float qv[RPT], kv[4];
#pragma unroll
      for (int i = 0; i < RPT; ++i) qv[i] = Qs[(rg * RPT + i) * DP + d];
#pragma unroll
      for (int j = 0; j < 4; ++j) kv[j] = Ks[(cg + 16 * j) * DP + d];
#pragma unroll
      for (int i = 0; i < RPT; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) s[i][j] = fmaf(qv[i], kv[j], s[i][j]);
    }

#pragma unroll
    for (int i = 0; i < RPT; ++i) {
      const int m = m0 + rg * RPT + i;
      float tmax = -INFINITY;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int n = n0 + cg + 16 * j;
        if (n >= S || (causal && n > m)) s[i][j] = -INFINITY;
        tmax = fmaxf(tmax, s[i][j]);
      }
#pragma unroll
      for (int off = 8; off > 0; off >>= 1) tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, off, 16));
      const float mnew = fmaxf(mrow[i], tmax);
      const float muse = mnew == -INFINITY ? 0.f : mnew;
      const float alpha = expf(mrow[i] - muse);
      float psum = 0.f;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float p = expf(s[i][j] - muse);
        psum += p;
        Ps[(rg * RPT + i) * (kBN + 1) + cg + 16 * j] = p;
      }
#pragma unroll
      for (int off = 8; off > 0; off >>= 1) psum += __shfl_xor_sync(0xffffffffu, psum, off, 16);
      lrow[i] = lrow[i] * alpha + psum;
      mrow[i] = mnew;
#pragma unroll
      for (int j = 0; j < NJ; ++j) acc[i][j] *= alpha;
    }
    __syncthreads();
    const int nlim = min(kBN, S - n0);
    for (int c = 0; c < nlim; ++c) {
      float pv[RPT];
#pragma unroll
      for (int i = 0; i < RPT; ++i) pv[i] = Ps[(rg * RPT + i) * (kBN + 1) + c];
#pragma unroll
      for (int j = 0; j < NJ; ++j) {
        const int d = cg + 16 * j;
        const float vv = Vs[c * DMAX + d];
#pragma unroll
        for (int i = 0; i < RPT; ++i) acc[i][j] = fmaf(pv[i], vv, acc[i][j]);
      }
    }
  }

#pragma unroll
  for (int i = 0; i < RPT; ++i) {
    const int m = m0 + rg * RPT + i;
    if (m >= S) continue;
    const float inv = lrow[i] > 0.f ? 1.f / lrow[i] : 0.f;
#pragma unroll
    for (int j = 0; j < NJ; ++j) {
      const int d = cg + 16 * j;
      if (d < D) ob[m * som + d * sok] = from_f32<T>(acc[i][j] * inv);
    }
  }
}

template <typename T, int DMAX, int RPT>
int launch_r(const void* q, const void* k, const void* v, void* o, long long B, long long H,
             long long S, long long D, const int64_t* s, float scale, int causal, cudaStream_t st) {
  constexpr int kBM = 16 * RPT;
  const size_t smem = sizeof(float) * (kBM * (DMAX + 1) + kBN * (DMAX + 1) + kBN * DMAX + kBM * (kBN + 1));
  auto kern = fa_simt_kernel<T, DMAX, RPT>;
  B2_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  dim3 grid((unsigned)((S + kBM - 1) / kBM), (unsigned)(B * H));
  kern<<<grid, kThreads, smem, st>>>((const T*)q, (const T*)k, (const T*)v, (T*)o, (int)H, (int)S,
                                     (int)D, nullptr, s[0], s[1], s[2], s[3], s[4], s[5], s[6],
                                     s[7], s[8], s[9], s[10], s[11], s[12], s[13], s[14], s[15],
                                     scale, causal);
  B2_CHECK_LAUNCH();
  return B2_OK;
}

template <typename T, int DMAX>
int launch_t(const void* q, const void* k, const void* v, void* o, long long B, long long H,
             long long S, long long D, const int64_t* s, float scale, int causal, cudaStream_t st) {
  const long long ctas64 = ((S + 63) / 64) * B * H;
  if (ctas64 < device_sm_count())
    return launch_r<T, DMAX, 1>(q, k, v, o, B, H, S, D, s, scale, causal, st);
  return launch_r<T, DMAX, 4>(q, k, v, o, B, H, S, D, s, scale, causal, st);
}

template <typename T>
int launch_d(const void* q, const void* k, const void* v, void* o, long long B, long long H,
             long long S, long long D, const int64_t* s, float scale, int causal, cudaStream_t st) {
  if (D <= 32) return launch_t<T, 32>(q, k, v, o, B, H, S, D, s, scale, causal, st);
  if (D <= 64) return launch_t<T, 64>(q, k, v, o, B, H, S, D, s, scale, causal, st);
  return launch_t<T, 128>(q, k, v, o, B, H, S, D, s, scale, causal, st);
}

}  // namespace

int fa_simt_launch(const void* q, const void* k, const void* v, void* o, long long B, long long H,
                   long long S, long long D, const int64_t* strides, float scale, int causal,
                   int dtype, cudaStream_t st) {
  if (D > 128) {
    set_error("b2_fa_fwd: head_dim %lld > 128 is not supported", D);
    return B2_EUNSUPPORTED;
  }
  switch (dtype) {
    case B2_F32: return launch_d<float>(q, k, v, o, B, H, S, D, strides, scale, causal, st);
    case B2_F16: return launch_d<__half>(q, k, v, o, B, H, S, D, strides, scale, causal, st);
    case B2_BF16: return launch_d<__nv_bfloat16>(q, k, v, o, B, H, S, D, strides, scale, causal, st);
    default:
      set_error("b2_fa_fwd: unsupported dtype %d", dtype);
      return B2_EINVAL;
  }
}

}  // namespace b2
