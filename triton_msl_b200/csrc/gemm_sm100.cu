// GEMM with fused bias/activation epilogue on 5th-generation tensor cores.
//
// Replaces the reference's fast matmul (`make_simdgroup_matmul_kernel_fast`,
// triton_msl/codegen/_msl_templates.py:4134-4255: fp32 accumulate, cast out)
// and its staged epilogue (`_lower_matmul_softmax_template` /
// `_emit_matmul_epilogue_loop`, _lowerer_templates.py:1515-1855: column bias
// folded into the accumulator, then the activation, then the store). The
// reference refuses a K-looped matmul with an epilogue; here the epilogue is
// fused into every tile.
//
// Design (one CTA per SM, persistent):
//  * C tile 128 x 256, K step 64 (one 128-byte swizzle atom), 4-stage
//    TMA -> shared-memory ring (48 KB per stage).
//  * warp 0: TMA producer; warp 1: TMEM allocation + single-thread tcgen05.mma
//    issue (M=128, N=256, K=16 per instruction); warps 2-5: epilogue.
//  * Two 256-column fp32 accumulators in TMEM (all 512 columns), so the
//    epilogue of tile i overlaps the main loop of tile i+1.
//  * A is K-major ([M,K] row-major). B is either MN-major ([K,N] row-major, the
//    reference `A @ B` layout) or K-major ([N,K] row-major, `x @ w.t()`); the
//    instruction descriptor's B-major bit selects it, no transpose pass.
//  * Epilogue: tcgen05.ld 32 columns at a time, alpha, + bias[n], activation,
//    convert, 16-byte stores.
//  * Every mbarrier wait is bounded (see sm100.cuh).
#include <cstdlib>
#include <cstring>

#include "sm100.cuh"

namespace b2 {
namespace {

using namespace sm100;

__device__ uint32_t g_gemm_status;

constexpr int kBM = 128, kBK = 64, kMaxStages = 6;
constexpr int kThreads = 192;
constexpr uint32_t kABytes = kBM * kBK * 2;   // 16 KB
#ifndef B2_GEMM_GROUP_M
#define B2_GEMM_GROUP_M 16
#endif
constexpr int kGroupM = B2_GEMM_GROUP_M;      // raster: M-tiles per group
// Per tile width BN (256, or 128 when that fills the SMs better): B stage
// bytes, and two BN-column fp32 accumulators in TMEM.
// Epilogue staging: per epilogue warp two 32x32 output blocks, written
// swizzled and sent to global memory with TMA tensor stores, plus two bias
// tiles. The operand ring takes what is left of 227 KB of shared memory:
// 4 stages (3 with fp32 output) at BN=256, 6 (5) at BN=128.
template <typename TO, int BN> struct EpiCfg {
  static constexpr uint32_t kBBytes = BN * kBK * 2;
  static constexpr uint32_t kStageBytes = kABytes + kBBytes;
  static constexpr uint32_t kTmemCols = 2 * BN;
  static constexpr int kRing = BN == 256 ? (sizeof(TO) == 4 ? 3 : 4) : (sizeof(TO) == 4 ? 5 : 6);
  static constexpr uint32_t kOutBytes = 32 * 32 * sizeof(TO);
  static constexpr uint32_t kEpiSmem = 4 * 2 * kOutBytes + 2 * BN * 4;
  static_assert(kRing <= kMaxStages, "ring deeper than the barrier arrays");
};

struct __align__(8) GemmBarriers {
  uint64_t full[kMaxStages];
  uint64_t empty[kMaxStages];
  uint64_t acc_full[2];
  uint64_t acc_empty[2];
  uint64_t done;
  uint32_t tmem_base;
  int abort_flag;
};

__device__ __forceinline__ float bias_at(const void* b, int dt, int n) {
  if (dt == B2_F32) return __ldg(reinterpret_cast<const float*>(b) + n);
  if (dt == B2_F16) return __half2float(reinterpret_cast<const __half*>(b)[n]);
  return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(b)[n]);
}

__device__ __forceinline__ void tile_coords(int t, int num_m, int num_n, int& mb, int& nb) {
  const int per_group = kGroupM * num_n;
  const int g = t / per_group;
  const int first_m = g * kGroupM;
  const int gsize = min(num_m - first_m, kGroupM);
  const int r = t % per_group;
  mb = first_m + r % gsize;
  nb = r / gsize;
}

// TF32: operands are fp32 hi/lo splits laid out by tf32_split_kernel (both
// K-major), 32 elements per 128-byte row, consumed by kind::tf32 MMAs.
// alpha * acc + bias, then the activation, for one 32-column chunk. The
// activation is a template argument so the chunk holds no per-element branch
// (a runtime switch inside the unrolled loop measured ~25 us per 128x256 tile:
// branch resolution and instruction-cache misses over 32 inlined copies).
template <int ACT>
__device__ __forceinline__ void act_chunk(float (&f)[32], const uint32_t (&r)[32], const float (&bv)[32],
                                          float alpha) {
#pragma unroll
  for (int j = 0; j < 32; ++j) f[j] = apply_act(fmaf(__uint_as_float(r[j]), alpha, bv[j]), ACT);
}

// Split-K (few output tiles, long K): tile index t covers (output tile
// t / splits, K range t % splits); each K range holds kb_per_split K blocks.
// A split's raw fp32 accumulator goes to rows [split * m_pad, ...) of the
// workspace matrix that tmC then describes; gemm_splitk_reduce_kernel sums the
// splits and applies the epilogue.
template <typename TO, bool B_MN, bool TF32, int BN>
__global__ void __launch_bounds__(kThreads, 1)
gemm_sm100_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                  const __grid_constant__ CUtensorMap tmC, int use_tma_store,
                  const void* __restrict__ bias, int bias_dt, TO* __restrict__ C, int M, int N,
                  int K, long long ldc, float alpha, int act, uint32_t idesc, int vec_ok,
                  unsigned long long wait_ns, int stall_producer, int splits, int kb_per_split,
                  int m_pad, int tf32_kp_blocks, const EpiProgram prog) {
  using Cfg = EpiCfg<TO, BN>;
  constexpr int kBN = BN;
  constexpr int kRing = Cfg::kRing;
  constexpr uint32_t kBBytes = Cfg::kBBytes;
  constexpr uint32_t kStageBytes = Cfg::kStageBytes;
  constexpr uint32_t kTmemCols = Cfg::kTmemCols;
  constexpr uint32_t kStageOutBytes = Cfg::kOutBytes;
  constexpr uint32_t kEpiSmem = Cfg::kEpiSmem;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + kRing * kABytes;
  uint8_t* sOut = smem + kRing * kStageBytes;
  float* sBias = reinterpret_cast<float*>(sOut + 4 * 2 * kStageOutBytes);  // [2][kBN]
  GemmBarriers* bars = reinterpret_cast<GemmBarriers*>(smem + kRing * kStageBytes + kEpiSmem);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int num_m = (M + kBM - 1) / kBM, num_n = (N + kBN - 1) / kBN;
  const int tiles = num_m * num_n * splits;
  static_assert(!(TF32 && B_MN), "tf32 operands are K-major");
  constexpr int kKE = TF32 ? 32 : kBK;  // K elements per 128-byte swizzle row
  const int nk_all = (K + kKE - 1) / kKE;
  // K blocks [kb_lo, kb_hi) of tile index t
  auto k_range = [&](int t, int& kb_lo, int& kb_hi) {
    const int sp = t % splits;
    kb_lo = sp * kb_per_split;
    kb_hi = min(nk_all, kb_lo + kb_per_split);
  };
  volatile int* abort_flag = &bars->abort_flag;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kRing; ++s) {
      mbar_init(&bars->full[s], 1);
      mbar_init(&bars->empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&bars->acc_full[a], 1);
      mbar_init(&bars->acc_empty[a], 4);
    }
    mbar_init(&bars->done, 1);
    bars->abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(&bars->tmem_base, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem_base;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t filled = 0;  // stages filled at least once
      bool ok = true;
      // stall_producer (failure-path test only): issue no loads, so the MMA
      // warp's first wait on a full stage runs out after wait_ns.
      for (int t = blockIdx.x; t < tiles && ok && !stall_producer; t += gridDim.x) {
        int mb, nb, kb_lo, kb_hi;
        tile_coords(t / splits, num_m, num_n, mb, nb);
        k_range(t, kb_lo, kb_hi);
        for (int kb = kb_lo; kb < kb_hi; ++kb) {
          if (!mbar_wait(&bars->empty[stage], phase ^ 1u, abort_flag, &g_gemm_status, DEV_TIMEOUT_SLOT, wait_ns)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&bars->full[stage], kStageBytes);
          int xa = kb * kKE, xb = kb * kKE;
          if constexpr (TF32) {
            // tripled K = [hi.hi | hi.lo | lo.hi] over operands stored as [hi | lo]
            const int seg = kb / tf32_kp_blocks, off = (kb - seg * tf32_kp_blocks) * kKE;
            const int kp = tf32_kp_blocks * kKE;
            xa = off + (seg == 2 ? kp : 0);
            xb = off + (seg == 1 ? kp : 0);
          }
          tma_load_2d(sA + stage * kABytes, &tmA, &bars->full[stage], xa, mb * kBM);
          if (B_MN) {
#pragma unroll
            for (int j = 0; j < kBN / 64; ++j)
              tma_load_2d(sB + stage * kBBytes + j * (64 * kBK * 2), &tmB, &bars->full[stage],
                          nb * kBN + j * 64, kb * kBK);
          } else {
            tma_load_2d(sB + stage * kBBytes, &tmB, &bars->full[stage], xb, nb * kBN);
          }
          filled |= 1u << stage;
          if (++stage == kRing) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      // Never leave with bulk copies in flight into this CTA's shared memory:
      // wait (bounded) for the latest fill of every stage to land.
      for (int s = 0; s < kRing; ++s) {
        if (!(filled & (1u << s))) continue;
        // the latest fill of stage s used parity (phase of that round)
        const uint32_t par = (s < stage) ? phase : (phase ^ 1u);
        const unsigned long long t0 = globaltimer();
        while (!mbar_test(smem_addr(&bars->full[s]), par)) {
          if (globaltimer() - t0 > kWaitLimitNs) {
            atomicOr(&g_gemm_status, DEV_TIMEOUT_TMA);
            break;
          }
        }
      }
    }
  } else if (warp == 1) {
    // ----------------------------------------------------------- MMA issue
    // Whole warp runs the loop (warp-uniform operands); one elected lane issues.
    {
      const bool leader = elect_one();
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      bool issued = false;
      for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x) {
        if (!mbar_wait(&bars->acc_empty[acc], acc_phase ^ 1u, abort_flag, &g_gemm_status, DEV_TIMEOUT_EPI, wait_ns)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem + acc * kBN;
        int kb_lo, kb_hi;
        k_range(t, kb_lo, kb_hi);
        for (int kb = kb_lo; kb < kb_hi; ++kb) {
          if (!mbar_wait(&bars->full[stage], phase, abort_flag, &g_gemm_status, DEV_TIMEOUT_TMA, wait_ns)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a0 = smem_addr(sA + stage * kABytes);
          const uint32_t b0 = smem_addr(sB + stage * kBBytes);
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k) {
            const uint64_t ad = sdesc(a0 + k * 32, 16, 1024, kSwizzle128);
            const uint64_t bd = B_MN ? sdesc(b0 + k * 16 * 128, 64 * kBK * 2, 1024, kSwizzle128)
                                     : sdesc(b0 + k * 32, 16, 1024, kSwizzle128);
            // 32 bytes of K per instruction: K=16 (f16/bf16) or K=8 (tf32)
            if (leader) {
              const uint32_t accum = (kb != kb_lo || k != 0) ? 1u : 0u;
              if (TF32) mma_tf32_ss(d_tmem, ad, bd, idesc, accum);
              else mma_f16_ss(d_tmem, ad, bd, idesc, accum);
            }
          }
          issued = true;
          if (leader) mma_commit(&bars->empty[stage]);
          if (++stage == kRing) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        if (leader) mma_commit(&bars->acc_full[acc]);
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1u;
        }
      }
      // Drain: all MMAs issued by this thread have retired before TMEM is freed.
      if (issued) {
        if (leader) mma_commit(&bars->done);
        const unsigned long long t0 = globaltimer();
        while (!mbar_test(smem_addr(&bars->done), 0)) {
          if (globaltimer() - t0 > kWaitLimitNs) {
            atomicOr(&g_gemm_status, DEV_TIMEOUT_MMA);
            break;
          }
        }
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int quarter = warp & 3;  // TMEM lanes this warp may access
    int acc = 0;
    uint32_t acc_phase = 0;
    int tile_iter = 0;
    for (int t = blockIdx.x; t < tiles; t += gridDim.x) {
      int mb, nb;
      tile_coords(t / splits, num_m, num_n, mb, nb);
      const int row_off = (t % splits) * m_pad;  // split-K: this split's rows of the workspace
      // This tile's bias columns into shared memory (double-buffered by tile
      // parity), loaded while the accumulator is still being computed.
      float* tb_bias = sBias + (tile_iter & 1) * kBN;
      if (bias != nullptr) {
        const int et = threadIdx.x - 64;  // 0..127 over the four epilogue warps
        for (int cidx = et; cidx < kBN; cidx += 128) {
          const int n = nb * kBN + cidx;
          tb_bias[cidx] = n < N ? bias_at(bias, bias_dt, n) : 0.f;
        }
        asm volatile("bar.sync 1, 128;" ::: "memory");
      }
      ++tile_iter;
      // In the stall test only the MMA warp's wait is shortened; this one keeps
      // the full limit and leaves on the abort flag the MMA warp sets.
      if (!mbar_wait(&bars->acc_full[acc], acc_phase, abort_flag, &g_gemm_status, DEV_TIMEOUT_MMA,
                     stall_producer ? kWaitLimitNs : wait_ns))
        break;
      tc_fence_after();
      const int row = mb * kBM + quarter * 32 + lane;
      const uint32_t tbase = tmem + ((uint32_t)(quarter * 32) << 16) + acc * kBN;
      TO* crow = C + (long long)row * ldc;
      // Row-softmax epilogue (N <= kBN, so this tile holds whole rows): two
      // read passes over the accumulator for the row max and the sum of
      // exponentials, then the chunk loop below writes exp(x - max) / sum.
      float sm_max = 0.f, sm_inv = 0.f;
      if (act == B2_ACT_SOFTMAX) {
        constexpr float kLog2e = 1.4426950408889634f;
        float mloc = -INFINITY;
#pragma unroll 1
        for (int c = 0; c < kBN / 32 && c * 32 < N; ++c) {
          uint32_t r[32];
          tmem_ld32(tbase + c * 32, r);
          tmem_ld_wait();
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const float x = fmaf(__uint_as_float(r[j]), alpha, bias ? tb_bias[c * 32 + j] : 0.f);
            if (c * 32 + j < N) mloc = fmaxf(mloc, x);
          }
        }
        float l = 0.f;
#pragma unroll 1
        for (int c = 0; c < kBN / 32 && c * 32 < N; ++c) {
          uint32_t r[32];
          tmem_ld32(tbase + c * 32, r);
          tmem_ld_wait();
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const float x = fmaf(__uint_as_float(r[j]), alpha, bias ? tb_bias[c * 32 + j] : 0.f);
            if (c * 32 + j < N) l += exp2f((x - mloc) * kLog2e);
          }
        }
        sm_max = mloc;
        sm_inv = 1.f / l;
      }
#pragma unroll 1
      for (int c = 0; c < kBN / 32; ++c) {
        uint32_t r[32];
        tmem_ld32(tbase + c * 32, r);
        tmem_ld_wait();
        const int n0 = nb * kBN + c * 32;
        if (n0 >= N) continue;  // warp-uniform
        float bv[32];
        if (bias != nullptr) {
#pragma unroll
          for (int v = 0; v < 8; ++v) {
            const float4 q = *reinterpret_cast<const float4*>(tb_bias + c * 32 + 4 * v);
            bv[4 * v] = q.x; bv[4 * v + 1] = q.y; bv[4 * v + 2] = q.z; bv[4 * v + 3] = q.w;
          }
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j) bv[j] = 0.f;
        }
        float f[32];
        switch (act) {  // warp-uniform
          case B2_ACT_RELU: act_chunk<B2_ACT_RELU>(f, r, bv, alpha); break;
          case B2_ACT_GELU: act_chunk<B2_ACT_GELU>(f, r, bv, alpha); break;
          case B2_ACT_GELU_TANH: act_chunk<B2_ACT_GELU_TANH>(f, r, bv, alpha); break;
          case B2_ACT_SILU: act_chunk<B2_ACT_SILU>(f, r, bv, alpha); break;
          case kActChain:
#pragma unroll
            for (int j = 0; j < 32; ++j) f[j] = __uint_as_float(r[j]) * alpha;
            epi_chain_chunk<32>(f, bv, prog);
            break;
          default: act_chunk<B2_ACT_NONE>(f, r, bv, alpha); break;
        }
        if (act == B2_ACT_SOFTMAX) {
#pragma unroll
          for (int j = 0; j < 32; ++j) f[j] = exp2f((f[j] - sm_max) * 1.4426950408889634f) * sm_inv;
        }
        if (use_tma_store) {
          // Row `lane` of a 32x32 block -> swizzled staging -> one TMA store
          // per warp (rows >= M and columns >= N are clipped by the TMA unit).
          constexpr int RB = 32 * (int)sizeof(TO);  // staging row bytes: 64 or 128
          uint8_t* stg = sOut + ((warp - 2) * 2 + (c & 1)) * kStageOutBytes;
          if (lane == 0) bulk_wait_group_read<1>();
          __syncwarp();
          const int swz = ((lane * RB) >> 7) & (RB / 16 - 1);
#pragma unroll
          for (int ch = 0; ch < RB / 16; ++ch) {
            uint4 u;
            if constexpr (sizeof(TO) == 2) {
              TO* h = reinterpret_cast<TO*>(&u);
#pragma unroll
              for (int e = 0; e < 8; ++e) h[e] = from_f32<TO>(f[ch * 8 + e]);
            } else {
              u = make_uint4(__float_as_uint(f[ch * 4]), __float_as_uint(f[ch * 4 + 1]),
                             __float_as_uint(f[ch * 4 + 2]), __float_as_uint(f[ch * 4 + 3]));
            }
            *reinterpret_cast<uint4*>(stg + lane * RB + ((ch ^ swz) * 16)) = u;
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            tma_store_2d(stg, &tmC, n0, row_off + mb * kBM + quarter * 32);
            bulk_commit_group();
          }
          continue;
        }
        if (row >= M) continue;
        if (vec_ok && n0 + 32 <= N) {
          if constexpr (sizeof(TO) == 2) {
            uint4* dst = reinterpret_cast<uint4*>(crow + n0);
#pragma unroll
            for (int v = 0; v < 4; ++v) {
              uint4 u;
              TO* h = reinterpret_cast<TO*>(&u);
#pragma unroll
              for (int j = 0; j < 8; ++j) h[j] = from_f32<TO>(f[v * 8 + j]);
              dst[v] = u;
            }
          } else {
            float4* dst = reinterpret_cast<float4*>(crow + n0);
#pragma unroll
            for (int v = 0; v < 8; ++v)
              dst[v] = make_float4(f[v * 4], f[v * 4 + 1], f[v * 4 + 2], f[v * 4 + 3]);
          }
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j)
            if (n0 + j < N) crow[n0 + j] = from_f32<TO>(f[j]);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->acc_empty[acc]);
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1u;
      }
    }
    // Output stores still in flight must finish before the CTA exits.
    if (use_tma_store && lane == 0) bulk_wait_group<0>();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// ---------------------------------------------------------------- 3xTF32
// fp32 GEMM on the tf32 tensor path with fp32-level accuracy: x = hi + lo with
// hi = tf32(x) and lo = tf32(x - hi), and
//   A.B ~= A_hi.B_hi + A_hi.B_lo + A_lo.B_hi
// (the dropped A_lo.B_lo is ~2^-22 relative). The three products are one GEMM
// over a tripled K' = 3 Kp (Kp = K rounded up to 32, zero-padded): each split
// operand row holds [hi | lo] (B transposed to K-major), and the TMA producer
// reads K' segment 0/1/2 from A's hi/hi/lo and B's hi/lo/hi halves.
__device__ __forceinline__ float tf32_rna(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return __uint_as_float(r);
}

// A[r, k] (M rows) and B^T[n, k] (N rows) -> [hi | lo] rows of 2*Kp floats
// (Kp = K rounded up to 32, zero padded), both operands in one launch
// (blockIdx.y below mblocks: A, else B). 32x32 tiles through shared memory so
// both a row-major A and a [K, N] B read and write coalesced.
__global__ void __launch_bounds__(256)
tf32_split_kernel(const float* __restrict__ A, long long M, long long sar, long long sak,
                  const float* __restrict__ B, long long N, long long sbr, long long sbk, long long K,
                  float* __restrict__ dA, float* __restrict__ dB, long long Kp, int mblocks) {
  __shared__ float tile[32][33];
  const bool isA = (int)blockIdx.y < mblocks;
  const float* src = isA ? A : B;
  const long long R = isA ? M : N, sr = isA ? sar : sbr, sk = isA ? sak : sbk;
  float* dst = isA ? dA : dB;
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
  const long long r0 = (long long)(isA ? blockIdx.y : blockIdx.y - mblocks) * 32, k0 = (long long)blockIdx.x * 32;
  if (sk == 1) {
#pragma unroll
    for (int i = ty; i < 32; i += 8) {
      const long long r = r0 + i, k = k0 + tx;
      tile[i][tx] = (r < R && k < K) ? src[r * sr + k] : 0.f;
    }
  } else {
#pragma unroll
    for (int i = ty; i < 32; i += 8) {
      const long long r = r0 + tx, k = k0 + i;
      tile[tx][i] = (r < R && k < K) ? src[r * sr + k * sk] : 0.f;
    }
  }
  __syncthreads();
#pragma unroll
  for (int i = ty; i < 32; i += 8) {
    const long long r = r0 + i;
    if (r >= R) continue;
    const float x = tile[i][tx];
    const float hi = tf32_rna(x);
    float* d = dst + r * 2 * Kp + k0 + tx;
    d[0] = hi;
    d[Kp] = tf32_rna(x - hi);
  }
}

// Launch parameters beyond the operands: tile width, split-K layout and the
// failure-path test knobs.
struct LaunchOpts {
  int bn = 256;
  int splits = 1, kb_per_split = 0, m_pad = 0;
  int tf32_kp_blocks = 1;  // 3xTF32: 32-element K blocks per hi / lo segment
  unsigned long long wait_ns = kWaitLimitNs;
  int stall_producer = 0;
};

template <typename TO, bool B_MN, bool TF32, int BN>
int launch_bn(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tc, int use_tma,
              const void* bias, int bias_dt, void* C, long long M, long long N, long long K,
              long long ldc, float alpha, int act, uint32_t idesc, int vec_ok, cudaStream_t st,
              const LaunchOpts& o) {
  using Cfg = EpiCfg<TO, BN>;
  auto kern = gemm_sm100_kernel<TO, B_MN, TF32, BN>;
  const size_t smem = 1024 + Cfg::kRing * Cfg::kStageBytes + Cfg::kEpiSmem + sizeof(GemmBarriers);
  static_assert(1024 + Cfg::kRing * Cfg::kStageBytes + Cfg::kEpiSmem + sizeof(GemmBarriers) <= 227 * 1024,
                "shared memory per CTA exceeded");
  B2_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  const int sms = device_sm_count();
  const long long tiles = ((M + kBM - 1) / kBM) * ((N + BN - 1) / BN) * o.splits;
  const int grid = (int)(tiles < sms ? tiles : sms);
  const int kbs = o.splits > 1 ? o.kb_per_split : (int)((K + 31) / 32);  // >= every K-block count
  kern<<<grid, kThreads, smem, st>>>(ta, tb, tc, use_tma, bias, bias_dt, (TO*)C, (int)M, (int)N, (int)K, ldc,
                                      alpha, act, idesc, vec_ok, o.wait_ns, o.stall_producer, o.splits,
                                      kbs, o.m_pad, o.tf32_kp_blocks, epi_program());
  B2_CHECK_LAUNCH();
  return B2_OK;
}

template <typename TO, bool B_MN, bool TF32 = false>
int launch(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tc, int use_tma,
           const void* bias, int bias_dt, void* C, long long M, long long N, long long K,
           long long ldc, float alpha, int act, uint32_t idesc, int vec_ok, cudaStream_t st,
           const LaunchOpts& o = LaunchOpts()) {
  if constexpr (!TF32) {
    if (o.bn == 128)
      return launch_bn<TO, B_MN, TF32, 128>(ta, tb, tc, use_tma, bias, bias_dt, C, M, N, K, ldc, alpha, act,
                                            idesc, vec_ok, st, o);
  }
  return launch_bn<TO, B_MN, TF32, 256>(ta, tb, tc, use_tma, bias, bias_dt, C, M, N, K, ldc, alpha, act,
                                        idesc, vec_ok, st, o);
}

}  // namespace

struct GemmPlan {
  int bn = 256;
  int splits = 1, kb_per_split = 0;
  long long m_pad = 0, np = 0;
  size_t ws = 0;
};

namespace {

// Split-K epilogue: C[m, n] = act(alpha * sum_s W[s * m_pad + m, n] + bias[n]),
// four columns per thread (W's row pitch np is a multiple of 4 floats), the
// splits summed in order (deterministic).
template <typename TO, int ACT>
__global__ void __launch_bounds__(256)
gemm_splitk_reduce_kernel(const float* __restrict__ W, int splits, long long m_pad, long long np,
                          const void* __restrict__ bias, int bias_dt, TO* __restrict__ C, long long ldc,
                          int M, int N, float alpha, const EpiProgram prog) {
  const long long n4 = (N + 3) / 4;
  const long long total = (long long)M * n4;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const long long m = i / n4;
    const int n = (int)(i % n4) * 4;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int sp = 0; sp < splits; ++sp) {
      const float4 w = *reinterpret_cast<const float4*>(W + ((long long)sp * m_pad + m) * np + n);
      acc.x += w.x; acc.y += w.y; acc.z += w.z; acc.w += w.w;
    }
    const float a[4] = {acc.x, acc.y, acc.z, acc.w};
    TO* crow = C + m * ldc;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      if (n + e >= N) break;
      const float bv = bias ? bias_at(bias, bias_dt, n + e) : 0.f;
      crow[n + e] = from_f32<TO>(ACT == kActChain ? epi_chain(a[e] * alpha, bv, prog)
                                                  : apply_act(fmaf(a[e], alpha, bv), ACT));
    }
  }
}

template <typename TO>
int splitk_reduce(const float* W, int splits, long long m_pad, long long np, const void* bias, int bias_dt,
                  void* C, long long ldc, long long M, long long N, float alpha, int act, cudaStream_t st) {
  const long long total = M * ((N + 3) / 4);
  long long blocks = (total + 255) / 256;
  const long long cap = (long long)device_sm_count() * 16;
  if (blocks > cap) blocks = cap;
  TO* c = reinterpret_cast<TO*>(C);
  switch (act) {
#define B2_SPLITK_CASE(A) \
  case A: gemm_splitk_reduce_kernel<TO, A><<<(unsigned)blocks, 256, 0, st>>>(W, splits, m_pad, np, bias, bias_dt, c, ldc, (int)M, (int)N, alpha, epi_program()); break;
    B2_SPLITK_CASE(B2_ACT_RELU)
    B2_SPLITK_CASE(B2_ACT_GELU)
    B2_SPLITK_CASE(B2_ACT_GELU_TANH)
    B2_SPLITK_CASE(B2_ACT_SILU)
    B2_SPLITK_CASE(kActChain)
    default:
      gemm_splitk_reduce_kernel<TO, B2_ACT_NONE><<<(unsigned)blocks, 256, 0, st>>>(W, splits, m_pad, np, bias,
                                                                                 bias_dt, c, ldc, (int)M, (int)N, alpha,
                                                                                 epi_program());
#undef B2_SPLITK_CASE
  }
  B2_CHECK_LAUNCH();
  return B2_OK;
}

}  // namespace

// True when the tensor-core path can describe these operands with TMA.
bool gemm_sm100_eligible(const void* A, const void* B, long long M, long long N, long long K,
                         const int64_t* s, int in_dt) {
  if (in_dt != B2_F16 && in_dt != B2_BF16) return false;
  if (M <= 0 || N <= 0 || K <= 0) return false;
  if (M >= (1LL << 31) || N >= (1LL << 31) || K >= (1LL << 31)) return false;
  auto al16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  if (!al16(A) || !al16(B)) return false;
  // A: unit K stride, row pitch a multiple of 16 bytes
  if (s[1] != 1 || (s[0] * 2) % 16 != 0 || s[0] < K) return false;
  const bool b_mn = s[3] == 1, b_k = s[2] == 1;
  if (b_mn && (s[2] * 2) % 16 == 0 && s[2] >= N) return true;
  if (b_k && (s[3] * 2) % 16 == 0 && s[3] >= K) return true;
  return false;
}

// Tile width and split-K choice for an fp16/bf16 GEMM (the reference's tile
// choice with its occupancy gate, triton_msl/autotuning/matmul_tuner.py:76-104,
// restated for a persistent kernel on the SM count):
//  * BN = 128 instead of 256 when ceil(tiles / SMs) x tile cost is lower,
//    with a 128-wide tile costing 1.25x half a wide one (measured on B200: the
//    narrow tile moves 33 % more operand bytes per MMA cycle and loses
//    15-30 % at full occupancy, so it only pays when it turns idle SMs into
//    busy ones, e.g. 512 x 4096 but not 2048 x 2048);
//  * split-K when even 128-wide tiles fill at most half the SMs and K has at
//    least 8 blocks of 64: the K blocks are divided into up to 32 ranges of at
//    least 4 blocks, one CTA per (tile, range), partial sums in the workspace,
//    and a reduce kernel applies alpha, bias and the activation. Not for the
//    row-softmax epilogue (it needs whole rows in one tile).
// B2MSL_GEMM_TILE=256|128|splitk|pair (read once) forces a tile choice where it
// applies: a tuning and diagnostic override, unset in normal use.
int tile_override() {
  static const int v = [] {
    const char* e = getenv("B2MSL_GEMM_TILE");
    if (!e) return 0;
    if (!strcmp(e, "256")) return 256;
    if (!strcmp(e, "128")) return 128;
    if (!strcmp(e, "splitk")) return 1;
    if (!strcmp(e, "pair")) return 2;
    return 0;
  }();
  return v;
}

bool gemm_pair_wanted(long long M, long long N, long long K, const int64_t* s, const void* C, int out_dt,
                      int act, bool forced);
int gemm_pair_launch(const void* A, const void* B, const void* bias, void* C, long long M, long long N,
                     long long K, const int64_t* s, float alpha, int act, int in_dt, int bias_dt, int out_dt,
                     cudaStream_t st);

GemmPlan gemm_plan(long long M, long long N, long long K, int act) {
  GemmPlan p;
  if (M <= 0 || N <= 0 || K <= 0) return p;
  const int force = tile_override();
  if (force == 256 || force == 2 || (force == 128 && act != B2_ACT_SOFTMAX)) {
    p.bn = force == 128 ? 128 : 256;
    return p;
  }
  const long long sms = device_sm_count();
  auto tiles = [&](long long bn) { return ((M + kBM - 1) / kBM) * ((N + bn - 1) / bn); };
  if (act == B2_ACT_SOFTMAX) return p;  // whole rows (N <= 256) in one 256-wide tile
  // waves x tile width, the narrow tile weighted by its measured 1.25x cost
  // per output column
  auto cost = [&](long long bn) { return ((tiles(bn) + sms - 1) / sms) * (bn == 128 ? 160 : 256); };
  if (cost(128) < cost(256)) p.bn = 128;
  const long long nk = (K + kBK - 1) / kBK;
  const long long t128 = tiles(128);
  if (act != B2_ACT_SOFTMAX && ((2 * t128 <= sms && nk >= 8) || (force == 1 && nk >= 8))) {
    long long sp = force == 1 ? (sms + t128 - 1) / t128 : sms / t128;
    if (sp > nk / 4) sp = nk / 4;
    if (sp > 32) sp = 32;
    if (sp >= 2) {
      const long long kbs = (nk + sp - 1) / sp;
      p.bn = 128;
      p.splits = (int)((nk + kbs - 1) / kbs);
      p.kb_per_split = (int)kbs;
      p.m_pad = (M + kBM - 1) / kBM * kBM;
      p.np = (N + 3) / 4 * 4;
      p.ws = (size_t)p.splits * (size_t)p.m_pad * (size_t)p.np * sizeof(float);
    }
  }
  return p;
}

int gemm_sm100_launch(const void* A, const void* B, const void* bias, void* C, long long M,
                      long long N, long long K, const int64_t* s, float alpha, int act, int in_dt,
                      int bias_dt, int out_dt, void* workspace, size_t ws_bytes, cudaStream_t st,
                      int* variant) {
  const CUtensorMapDataType tdt =
      in_dt == B2_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  if (s[5] != 1) {
    set_error("b2_gemm: tensor-core path needs unit column stride in C");
    return B2_EUNSUPPORTED;
  }
  GemmPlan plan = gemm_plan(M, N, K, act);
  const bool split = plan.splits > 1 && workspace != nullptr && ws_bytes >= plan.ws &&
                     (reinterpret_cast<uintptr_t>(workspace) & 15) == 0 && plan.m_pad * plan.splits < (1LL << 31);
  LaunchOpts o;
  o.bn = plan.bn;
  if (split) {
    o.splits = plan.splits;
    o.kb_per_split = plan.kb_per_split;
    o.m_pad = (int)plan.m_pad;
  }
  const int BN = o.bn;
  if (!split && tile_override() != 256 && tile_override() != 128 &&
      gemm_pair_wanted(M, N, K, s, C, out_dt, act, tile_override() == 2)) {
    if (variant) *variant = 3;
    return gemm_pair_launch(A, B, bias, C, M, N, K, s, alpha, act, in_dt, bias_dt, out_dt, st);
  }
  if (variant) *variant = split ? 2 : (BN == 128 ? 1 : 0);
  CUtensorMap ta, tb;
  {
    const uint64_t dims[2] = {(uint64_t)K, (uint64_t)M};
    const uint64_t strides[1] = {(uint64_t)s[0] * 2};
    const uint32_t box[2] = {kBK, kBM};
    if (!encode_tmap(&ta, tdt, 2, A, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B)) return B2_ELAUNCH;
  }
  const bool b_mn = s[3] == 1 && (s[2] * 2) % 16 == 0 && s[2] >= N;
  if (b_mn) {
    const uint64_t dims[2] = {(uint64_t)N, (uint64_t)K};
    const uint64_t strides[1] = {(uint64_t)s[2] * 2};
    const uint32_t box[2] = {64, kBK};
    if (!encode_tmap(&tb, tdt, 2, B, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B)) return B2_ELAUNCH;
  } else {
    const uint64_t dims[2] = {(uint64_t)K, (uint64_t)N};
    const uint64_t strides[1] = {(uint64_t)s[3] * 2};
    const uint32_t box[2] = {kBK, (uint32_t)BN};
    if (!encode_tmap(&tb, tdt, 2, B, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B)) return B2_ELAUNCH;
  }
  const uint32_t idesc = idesc_f16(kBM, BN, in_dt == B2_BF16, false, b_mn);
  if (bias == nullptr) bias_dt = B2_F32;
  if (split) {
    // partial sums: fp32 [splits * m_pad, N] (row pitch np) through TMA stores
    CUtensorMap tw;
    const uint64_t dims[2] = {(uint64_t)N, (uint64_t)(plan.splits * plan.m_pad)};
    const uint64_t strides[1] = {(uint64_t)plan.np * 4};
    const uint32_t box[2] = {32, 32};
    if (!encode_tmap(&tw, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, workspace, dims, strides, box,
                     CU_TENSOR_MAP_SWIZZLE_128B))
      return B2_ELAUNCH;
    int rc = b_mn ? launch<float, true>(ta, tb, tw, 1, nullptr, B2_F32, workspace, M, N, K, plan.np, 1.f,
                                        B2_ACT_NONE, idesc, 1, st, o)
                  : launch<float, false>(ta, tb, tw, 1, nullptr, B2_F32, workspace, M, N, K, plan.np, 1.f,
                                         B2_ACT_NONE, idesc, 1, st, o);
    if (rc != B2_OK) return rc;
    const float* W = reinterpret_cast<const float*>(workspace);
    switch (out_dt) {
      case B2_F16: return splitk_reduce<__half>(W, plan.splits, plan.m_pad, plan.np, bias, bias_dt, C, s[4], M, N, alpha, act, st);
      case B2_BF16: return splitk_reduce<__nv_bfloat16>(W, plan.splits, plan.m_pad, plan.np, bias, bias_dt, C, s[4], M, N, alpha, act, st);
      default: return splitk_reduce<float>(W, plan.splits, plan.m_pad, plan.np, bias, bias_dt, C, s[4], M, N, alpha, act, st);
    }
  }
  const int osz = dtype_size(out_dt);
  const int vec_ok = (reinterpret_cast<uintptr_t>(C) & 15) == 0 && ((s[4] * osz) % 16) == 0;
  // Output through TMA tensor stores when C's base and row pitch allow it.
  CUtensorMap tc;
  int use_tma = 0;
  if (vec_ok && s[4] >= N) {
    const CUtensorMapDataType cdt = out_dt == B2_F32    ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                    : out_dt == B2_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                        : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    const uint64_t dims[2] = {(uint64_t)N, (uint64_t)M};
    const uint64_t strides[1] = {(uint64_t)s[4] * osz};
    const uint32_t box[2] = {32, 32};
    use_tma = encode_tmap(&tc, cdt, 2, C, dims, strides, box,
                          osz == 2 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_128B) ? 1 : 0;
    clear_error();
  }
  if (!use_tma) memset(&tc, 0, sizeof(tc));
  switch (out_dt) {
    case B2_F16:
      return b_mn ? launch<__half, true>(ta, tb, tc, use_tma, bias, bias_dt, C, M, N, K, s[4], alpha, act, idesc, vec_ok, st, o)
                  : launch<__half, false>(ta, tb, tc, use_tma, bias, bias_dt, C, M, N, K, s[4], alpha, act, idesc, vec_ok, st, o);
    case B2_BF16:
      return b_mn ? launch<__nv_bfloat16, true>(ta, tb, tc, use_tma, bias, bias_dt, C, M, N, K, s[4], alpha, act, idesc, vec_ok, st, o)
                  : launch<__nv_bfloat16, false>(ta, tb, tc, use_tma, bias, bias_dt, C, M, N, K, s[4], alpha, act, idesc, vec_ok, st, o);
    case B2_F32:
      return b_mn ? launch<float, true>(ta, tb, tc, use_tma, bias, bias_dt, C, M, N, K, s[4], alpha, act, idesc, vec_ok, st, o)
                  : launch<float, false>(ta, tb, tc, use_tma, bias, bias_dt, C, M, N, K, s[4], alpha, act, idesc, vec_ok, st, o);
  }
  set_error("b2_gemm: unsupported out dtype %d", out_dt);
  return B2_EINVAL;
}

size_t gemm_f16_workspace(long long M, long long N, long long K, int act) {
  return gemm_plan(M, N, K, act).ws;
}


// Split-K plan of the 3xTF32 GEMM (one 128x256 tile per CTA): when the tiles
// fill at most half the SMs (2048^3 has 64 tiles), the tripled K loop is split
// like the fp16 path's (gemm_plan) so every SM works; not with the row-softmax
// epilogue.
struct Tf32Plan {
  int splits = 1, kb_per_split = 0;
  long long m_pad = 0, np = 0;
  size_t ws = 0;
};

Tf32Plan tf32_plan(long long M, long long N, long long K, int act) {
  Tf32Plan p;
  if (M <= 0 || N <= 0 || K <= 0 || act == B2_ACT_SOFTMAX) return p;
  const long long sms = device_sm_count();
  const long long tiles = ((M + kBM - 1) / kBM) * ((N + 255) / 256);
  const long long nk = 3 * ((K + 31) / 32);  // 32-element K blocks over the tripled K
  if (2 * tiles <= sms && nk >= 8) {
    long long sp = sms / tiles;
    if (sp > nk / 4) sp = nk / 4;
    if (sp > 32) sp = 32;
    if (sp >= 2) {
      const long long kbs = (nk + sp - 1) / sp;
      p.splits = (int)((nk + kbs - 1) / kbs);
      p.kb_per_split = (int)kbs;
      p.m_pad = (M + kBM - 1) / kBM * kBM;
      p.np = (N + 3) / 4 * 4;
      p.ws = (size_t)p.splits * (size_t)p.m_pad * (size_t)p.np * sizeof(float);
    }
  }
  return p;
}

size_t tf32_operand_bytes(long long M, long long N, long long K) {
  const long long Kp = (K + 31) / 32 * 32;
  return ((size_t)(M + N) * 2 * (size_t)Kp * sizeof(float) + 255) / 256 * 256;
}

size_t gemm_tf32x3_workspace(long long M, long long N, long long K) {
  if (M <= 0 || N <= 0 || K <= 0) return 0;
  return tf32_operand_bytes(M, N, K) + tf32_plan(M, N, K, B2_ACT_NONE).ws;
}

int gemm_tf32x3_launch(const float* A, const float* B, const void* bias, void* C, long long M,
                       long long N, long long K, const int64_t* s, float alpha, int act,
                       int bias_dt, int out_dt, void* workspace, cudaStream_t st) {
  if (M >= (1LL << 31) || N >= (1LL << 31) || 3 * ((K + 31) / 32 * 32) >= (1LL << 31)) {
    set_error("b2_gemm: dims too large for the 3xTF32 path");
    return B2_EINVAL;
  }
  if (s[5] != 1) {
    set_error("b2_gemm: tensor-core path needs unit column stride in C");
    return B2_EUNSUPPORTED;
  }
  const long long Kp = (K + 31) / 32 * 32, K3 = 3 * Kp;
  float* Ap = reinterpret_cast<float*>(workspace);
  float* Bp = Ap + (size_t)M * 2 * Kp;
  {
    // B[k, n] at B + k*s[2] + n*s[3]: rows of the split operand are n
    const int mblocks = (int)((M + 31) / 32);
    tf32_split_kernel<<<dim3((unsigned)(Kp / 32), (unsigned)(mblocks + (N + 31) / 32)), 256, 0, st>>>(
        A, M, s[0], s[1], B, N, s[3], s[2], K, Ap, Bp, Kp, mblocks);
    B2_CHECK_LAUNCH();
  }
  CUtensorMap ta, tb;
  {
    const uint64_t dims[2] = {(uint64_t)(2 * Kp), (uint64_t)M};
    const uint64_t strides[1] = {(uint64_t)(2 * Kp) * 4};
    const uint32_t box[2] = {32, kBM};
    if (!encode_tmap(&ta, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, Ap, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B))
      return B2_ELAUNCH;
  }
  {
    const uint64_t dims[2] = {(uint64_t)(2 * Kp), (uint64_t)N};
    const uint64_t strides[1] = {(uint64_t)(2 * Kp) * 4};
    const uint32_t box[2] = {32, 256};
    if (!encode_tmap(&tb, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, Bp, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B))
      return B2_ELAUNCH;
  }
  const uint32_t idesc = idesc_tf32(kBM, 256);
  const int osz = dtype_size(out_dt);
  const int vec_ok = (reinterpret_cast<uintptr_t>(C) & 15) == 0 && ((s[4] * osz) % 16) == 0;
  if (bias == nullptr) bias_dt = B2_F32;
  const Tf32Plan plan = tf32_plan(M, N, K, act);
  if (plan.splits > 1 && plan.m_pad * plan.splits < (1LL << 31)) {
    float* W = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(workspace) + tf32_operand_bytes(M, N, K));
    CUtensorMap tw;
    const uint64_t dims[2] = {(uint64_t)N, (uint64_t)(plan.splits * plan.m_pad)};
    const uint64_t strides[1] = {(uint64_t)plan.np * 4};
    const uint32_t box[2] = {32, 32};
    if (!encode_tmap(&tw, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, W, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B))
      return B2_ELAUNCH;
    LaunchOpts o;
    o.splits = plan.splits;
    o.kb_per_split = plan.kb_per_split;
    o.m_pad = (int)plan.m_pad;
    o.tf32_kp_blocks = (int)(Kp / 32);
    const int rc = launch<float, false, true>(ta, tb, tw, 1, nullptr, B2_F32, W, M, N, K3, plan.np, 1.f,
                                              B2_ACT_NONE, idesc, 1, st, o);
    if (rc != B2_OK) return rc;
    switch (out_dt) {
      case B2_F16: return splitk_reduce<__half>(W, plan.splits, plan.m_pad, plan.np, bias, bias_dt, C, s[4], M, N, alpha, act, st);
      case B2_BF16: return splitk_reduce<__nv_bfloat16>(W, plan.splits, plan.m_pad, plan.np, bias, bias_dt, C, s[4], M, N, alpha, act, st);
      default: return splitk_reduce<float>(W, plan.splits, plan.m_pad, plan.np, bias, bias_dt, C, s[4], M, N, alpha, act, st);
    }
  }
  LaunchOpts ot;
  ot.tf32_kp_blocks = (int)(Kp / 32);
  CUtensorMap tc;
  int use_tma = 0;
  if (vec_ok && s[4] >= N) {
    const CUtensorMapDataType cdt = out_dt == B2_F32    ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                    : out_dt == B2_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                        : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    const uint64_t dims[2] = {(uint64_t)N, (uint64_t)M};
    const uint64_t strides[1] = {(uint64_t)s[4] * osz};
    const uint32_t box[2] = {32, 32};
    use_tma = encode_tmap(&tc, cdt, 2, C, dims, strides, box,
                          osz == 2 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_128B) ? 1 : 0;
    clear_error();
  }
  if (!use_tma) memset(&tc, 0, sizeof(tc));
  switch (out_dt) {
    case B2_F16:
      return launch<__half, false, true>(ta, tb, tc, use_tma, bias, bias_dt, C, M, N, K3, s[4], alpha, act, idesc, vec_ok, st, ot);
    case B2_BF16:
      return launch<__nv_bfloat16, false, true>(ta, tb, tc, use_tma, bias, bias_dt, C, M, N, K3, s[4], alpha, act, idesc, vec_ok, st, ot);
    case B2_F32:
      return launch<float, false, true>(ta, tb, tc, use_tma, bias, bias_dt, C, M, N, K3, s[4], alpha, act, idesc, vec_ok, st, ot);
  }
  set_error("b2_gemm: unsupported out dtype %d", out_dt);
  return B2_EINVAL;
}

// Failure-path test: one fp16 tile GEMM (K-major A and B, fp16 C) whose TMA
// producer is told to load nothing, with every wait bounded by wait_ns. The
// MMA warp's wait for the first stage runs out, sets the CTA abort flag and
// DEV_TIMEOUT_TMA in the status word; the epilogue leaves on the flag; TMEM is
// freed and the kernel returns. Nothing is left in flight.
int gemm_stall_test_launch(const void* A, const void* B, void* C, long long M, long long N,
                           long long K, unsigned long long wait_ns, cudaStream_t st) {
  CUtensorMap ta, tb, tc;
  {
    const uint64_t dims[2] = {(uint64_t)K, (uint64_t)M};
    const uint64_t strides[1] = {(uint64_t)K * 2};
    const uint32_t box[2] = {kBK, kBM};
    if (!encode_tmap(&ta, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, A, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B))
      return B2_ELAUNCH;
  }
  {
    const uint64_t dims[2] = {(uint64_t)K, (uint64_t)N};
    const uint64_t strides[1] = {(uint64_t)K * 2};
    const uint32_t box[2] = {kBK, 256};
    if (!encode_tmap(&tb, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, B, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B))
      return B2_ELAUNCH;
  }
  memset(&tc, 0, sizeof(tc));
  const uint32_t idesc = idesc_f16(kBM, 256, false, false, false);
  LaunchOpts o;
  o.wait_ns = wait_ns;
  o.stall_producer = 1;
  return launch<__half, false>(ta, tb, tc, 0, nullptr, B2_F32, C, M, N, K, N, 1.f, B2_ACT_NONE, idesc,
                               0, st, o);
}

uint32_t gemm_read_status(bool clear) {
  uint32_t v = 0;
  cudaMemcpyFromSymbol(&v, g_gemm_status, sizeof(v));
  if (clear) {
    const uint32_t z = 0;
    cudaMemcpyToSymbol(g_gemm_status, &z, sizeof(z));
  }
  return v;
}

}  // namespace b2
