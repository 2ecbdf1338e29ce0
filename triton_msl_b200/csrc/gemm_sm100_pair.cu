// GEMM with fused bias/activation epilogue on CTA pairs (tcgen05 cta_group::2).
//
// Same contract as gemm_sm100.cu (C = act(alpha * A.B + bias), fp32
// accumulate; the reference's fast matmul, triton_msl/codegen/_msl_templates.py:4134-4255,
// with the epilogue of _lowerer_templates.py:1515-1855), for shapes with at
// least one full wave of output tiles and at most 4e12 FLOP. Two CTAs on two SMs (a cluster of 2)
// compute one 256 x 256 output tile with M=256 MMAs issued by rank 0:
//  * each CTA loads its own 128 rows of A and its own 128 columns of B (K step
//    64) into its own shared memory; the pair's tensor cores share the B
//    halves, so every SM fills 32 KB of operands per 512 MMA cycles instead of
//    48 KB for a 128 x 256 tile on one SM;
//  * the TMA byte counts of both CTAs complete on rank 0's stage barrier; the
//    MMA commits signal the stage-free and accumulator-full barriers of both
//    CTAs;
//  * each CTA's TMEM holds its 128 rows of the two 256-column accumulators,
//    and its four epilogue warps store them (alpha, bias, activation, cast,
//    swizzled staging, TMA tensor stores) and report to rank 0's
//    accumulator-free barrier.
// Last wave: when the tiles left over after the full waves fill at most half
// of the pairs, each of them is computed as two 256 x 128 halves on two pairs
// (M=256, N=128 MMAs; each CTA loads 64 columns of B), so the last wave runs
// about half as long; no partial sums, so no reduction or workspace.
// Every wait is bounded (sm100.cuh); the CTAs meet at a cluster barrier before
// the TMEM is freed.
#include <cstdlib>
#include <cstring>

#include "sm100.cuh"

namespace b2 {
namespace {

using namespace sm100;

__device__ uint32_t g_pair_status;

constexpr int kPM = 256, kBN = 256, kBK = 64, kHalf = 128;
constexpr int kThreads = 192;
constexpr int kMaxRing = 6;
constexpr uint32_t kABytes = kHalf * kBK * 2;  // 16 KB: this CTA's A rows
constexpr uint32_t kBBytes = kHalf * kBK * 2;  // 16 KB: this CTA's B columns
constexpr uint32_t kStageBytes = kABytes + kBBytes;
constexpr uint32_t kTmemCols = 2 * kBN;
#ifndef B2_GEMM_PAIR_GROUP_M
#define B2_GEMM_PAIR_GROUP_M 8
#endif
// raster: 256-row blocks per group. Measured on 8192^3 (DRAM read bytes / TFLOP/s):
// 4: 1.73 GB / 1297, 8: 1.10 / 1384, 16: 1.23 / 1378, 32 and 64: 2.32 / 1265 --
// 74 concurrent pair tiles keep a ~9 x 8 window (A rows + B columns, ~70 MB at
// K = 8192) hottest in L2 with 8.
constexpr int kGroupM = B2_GEMM_PAIR_GROUP_M;

template <typename TO> struct PairCfg {
  static constexpr int kRing = sizeof(TO) == 4 ? 5 : 6;
  static constexpr uint32_t kOutBytes = 32 * 32 * sizeof(TO);
  static constexpr uint32_t kEpiSmem = 4 * 2 * kOutBytes + 2 * kBN * 4;
};

struct __align__(8) PairBarriers {
  uint64_t full[kMaxRing];   // rank 0: both CTAs' bytes of a stage landed
  uint64_t empty[kMaxRing];  // each CTA: the MMAs reading a stage retired
  uint64_t acc_full[2];      // each CTA: accumulator complete
  uint64_t acc_empty[2];     // rank 0: all 8 epilogue warps read the accumulator
  uint64_t done;
  uint32_t tmem_base;
  int abort_flag;
};

__device__ __forceinline__ float bias_at(const void* b, int dt, int n) {
  if (dt == B2_F32) return __ldg(reinterpret_cast<const float*>(b) + n);
  if (dt == B2_F16) return __half2float(reinterpret_cast<const __half*>(b)[n]);
  return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(b)[n]);
}

__device__ __forceinline__ void pair_tile_coords(int t, int num_m, int num_n, int& mb, int& nb) {
  const int per_group = kGroupM * num_n;
  const int g = t / per_group;
  const int first_m = g * kGroupM;
  const int gsize = min(num_m - first_m, kGroupM);
  const int r = t % per_group;
  mb = first_m + r % gsize;
  nb = r / gsize;
}

// Work unit u of the persistent loop: whole tile u below tail_start, else
// half (u - tail_start) & 1 (columns 0-127 or 128-255) of tile
// tail_start + (u - tail_start) / 2.
__device__ __forceinline__ void pair_unit(int u, int tail_start, int& t, int& half) {
  if (u < tail_start) {
    t = u;
    half = -1;
  } else {
    t = tail_start + ((u - tail_start) >> 1);
    half = (u - tail_start) & 1;
  }
}

template <int ACT>
__device__ __forceinline__ void pair_act_chunk(float (&f)[32], const uint32_t (&r)[32], const float* bv,
                                               float alpha) {
#pragma unroll
  for (int j = 0; j < 32; ++j) f[j] = apply_act(fmaf(__uint_as_float(r[j]), alpha, bv[j]), ACT);
}

template <typename TO, bool B_MN>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
gemm_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                 const __grid_constant__ CUtensorMap tmBh, const __grid_constant__ CUtensorMap tmC,
                 const void* __restrict__ bias, int bias_dt, int M, int N, int K, float alpha, int act,
                 uint32_t idesc, uint32_t idesc_half, int tail_start, const EpiProgram prog) {
  constexpr int kRing = PairCfg<TO>::kRing;
  constexpr uint32_t kStageOutBytes = PairCfg<TO>::kOutBytes;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + kRing * kABytes;
  uint8_t* sOut = smem + kRing * kStageBytes;
  float* sBias = reinterpret_cast<float*>(sOut + 4 * 2 * kStageOutBytes);  // [2][kBN]
  PairBarriers* bars = reinterpret_cast<PairBarriers*>(smem + kRing * kStageBytes + PairCfg<TO>::kEpiSmem);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
  const int num_m = (M + kPM - 1) / kPM, num_n = (N + kBN - 1) / kBN;
  const int tiles = num_m * num_n;
  const int units = tail_start + 2 * (tiles - tail_start);
  const int nk = (K + kBK - 1) / kBK;
  volatile int* abort_flag = &bars->abort_flag;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kRing; ++s) {
      mbar_init(&bars->full[s], 1);
      mbar_init(&bars->empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&bars->acc_full[a], 1);
      mbar_init(&bars->acc_empty[a], 8);
    }
    mbar_init(&bars->done, 1);
    bars->abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    if (!B_MN) tma_prefetch_desc(&tmBh);
    tma_prefetch_desc(&tmC);
  }
  if (warp == 1) {
    tmem_alloc_pair(&bars->tmem_base, kTmemCols);
    tmem_relinquish_pair();
  }
  // barriers initialised and TMEM allocated in both CTAs before any use
  tc_fence_before();
  cluster_sync();
  tc_fence_after();
  const uint32_t tmem = bars->tmem_base;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      const uint32_t full0 = mapa_shared(&bars->full[0], 0);  // rank 0's stage barriers
      int stage = 0;
      uint32_t phase = 0;
      uint32_t filled = 0;
      bool ok = true;
      for (int u = pair; u < units && ok; u += npairs) {
        int t, half, mb, nb;
        pair_unit(u, tail_start, t, half);
        pair_tile_coords(t, num_m, num_n, mb, nb);
        // this CTA's B columns: 128 of the tile, or 64 of the tile's half
        const int bcols = half < 0 ? kHalf : kHalf / 2;
        const int bcol0 = nb * kBN + (half < 0 ? rank * kHalf : half * kHalf + rank * (kHalf / 2));
        const uint32_t stage_tx = 2 * (kABytes + (uint32_t)bcols * kBK * 2);
        for (int kb = 0; kb < nk; ++kb) {
          if (!mbar_wait(&bars->empty[stage], phase ^ 1u, abort_flag, &g_pair_status, DEV_TIMEOUT_SLOT)) {
            ok = false;
            break;
          }
          if (rank == 0) mbar_arrive_expect_tx(&bars->full[stage], stage_tx);
          const uint32_t fb = full0 + stage * 8;
          tma_load_2d_pair(sA + stage * kABytes, &tmA, fb, kb * kBK, mb * kPM + rank * kHalf);
          if (B_MN) {
            for (int j = 0; j < bcols / 64; ++j)
              tma_load_2d_pair(sB + stage * kBBytes + j * (64 * kBK * 2), &tmB, fb, bcol0 + j * 64, kb * kBK);
          } else {
            tma_load_2d_pair(sB + stage * kBBytes, half < 0 ? &tmB : &tmBh, fb, kb * kBK, bcol0);
          }
          filled |= 1u << stage;
          if (++stage == kRing) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (rank == 0) {
        // Both CTAs' latest fills of every stage count on rank 0's barriers:
        // wait (bounded) for them to land before leaving.
        for (int s = 0; s < kRing; ++s) {
          if (!(filled & (1u << s))) continue;
          const uint32_t par = (s < stage) ? phase : (phase ^ 1u);
          const unsigned long long t0 = globaltimer();
          while (!mbar_test(smem_addr(&bars->full[s]), par)) {
            if (globaltimer() - t0 > kWaitLimitNs) {
              atomicOr(&g_pair_status, DEV_TIMEOUT_TMA);
              break;
            }
          }
        }
      }
    }
  } else if (warp == 1) {
    // ----------------------------------------------------------- MMA issue
    if (rank == 0) {
      const bool leader = elect_one();
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true, issued = false;
      for (int u = pair; u < units && ok; u += npairs) {
        const uint32_t id = u < tail_start ? idesc : idesc_half;
        if (!mbar_wait(&bars->acc_empty[acc], acc_phase ^ 1u, abort_flag, &g_pair_status, DEV_TIMEOUT_EPI)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem + acc * kBN;
        for (int kb = 0; kb < nk; ++kb) {
          if (!mbar_wait(&bars->full[stage], phase, abort_flag, &g_pair_status, DEV_TIMEOUT_TMA)) {
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
            if (leader) mma_f16_ss_pair(d_tmem, ad, bd, id, (kb | k) != 0 ? 1u : 0u);
          }
          issued = true;
          if (leader) mma_commit_pair(&bars->empty[stage], 0x3);
          if (++stage == kRing) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        if (leader) mma_commit_pair(&bars->acc_full[acc], 0x3);
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1u;
        }
      }
      if (issued) {
        if (leader) mma_commit_pair(&bars->done, 0x1);
        const unsigned long long t0 = globaltimer();
        while (!mbar_test(smem_addr(&bars->done), 0)) {
          if (globaltimer() - t0 > kWaitLimitNs) {
            atomicOr(&g_pair_status, DEV_TIMEOUT_MMA);
            break;
          }
        }
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int quarter = warp & 3;
    const uint32_t acc_empty0 = mapa_shared(&bars->acc_empty[0], 0);
    int acc = 0;
    uint32_t acc_phase = 0;
    int tile_iter = 0;
    for (int u = pair; u < units; u += npairs) {
      int t, half, mb, nb;
      pair_unit(u, tail_start, t, half);
      pair_tile_coords(t, num_m, num_n, mb, nb);
      const int col0 = half < 0 ? 0 : half * kHalf;  // first tile column of this unit
      const int nchunks = half < 0 ? kBN / 32 : kHalf / 32;
      float* tb_bias = sBias + (tile_iter & 1) * kBN;
      if (bias != nullptr) {
        const int et = threadIdx.x - 64;
        for (int cidx = et; cidx < kBN; cidx += 128) {
          const int n = nb * kBN + cidx;
          tb_bias[cidx] = n < N ? bias_at(bias, bias_dt, n) : 0.f;
        }
        asm volatile("bar.sync 1, 128;" ::: "memory");
      }
      ++tile_iter;
      if (!mbar_wait(&bars->acc_full[acc], acc_phase, abort_flag, &g_pair_status, DEV_TIMEOUT_MMA)) break;
      tc_fence_after();
      const int row0 = mb * kPM + rank * kHalf + quarter * 32;
      const uint32_t tbase = tmem + ((uint32_t)(quarter * 32) << 16) + acc * kBN;
#pragma unroll 1
      for (int c = 0; c < nchunks; ++c) {
        uint32_t r[32];
        tmem_ld32(tbase + c * 32, r);
        tmem_ld_wait();
        const int n0 = nb * kBN + col0 + c * 32;
        if (n0 >= N) continue;  // warp-uniform
        float bv[32];
        if (bias != nullptr) {
#pragma unroll
          for (int v = 0; v < 8; ++v) {
            const float4 q = *reinterpret_cast<const float4*>(tb_bias + col0 + c * 32 + 4 * v);
            bv[4 * v] = q.x; bv[4 * v + 1] = q.y; bv[4 * v + 2] = q.z; bv[4 * v + 3] = q.w;
          }
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j) bv[j] = 0.f;
        }
        float f[32];
        switch (act) {  // warp-uniform
          case B2_ACT_RELU: pair_act_chunk<B2_ACT_RELU>(f, r, bv, alpha); break;
          case B2_ACT_GELU: pair_act_chunk<B2_ACT_GELU>(f, r, bv, alpha); break;
          case B2_ACT_GELU_TANH: pair_act_chunk<B2_ACT_GELU_TANH>(f, r, bv, alpha); break;
          case B2_ACT_SILU: pair_act_chunk<B2_ACT_SILU>(f, r, bv, alpha); break;
          case kActChain:
#pragma unroll
            for (int j = 0; j < 32; ++j) f[j] = __uint_as_float(r[j]) * alpha;
            epi_chain_chunk<32>(f, bv, prog);
            break;
          default: pair_act_chunk<B2_ACT_NONE>(f, r, bv, alpha); break;
        }
        constexpr int RB = 32 * (int)sizeof(TO);
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
          tma_store_2d(stg, &tmC, n0, row0);
          bulk_commit_group();
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(acc_empty0 + acc * 8);
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1u;
      }
    }
    if (lane == 0) bulk_wait_group<0>();
  }

  tc_fence_before();
  cluster_sync();  // no CTA frees TMEM or leaves while its peer may still signal it
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem, kTmemCols);
  }
}

// B2MSL_GEMM_PAIR_HALVES=0 (read once) keeps the last wave in whole tiles: a
// tuning and diagnostic override, unset in normal use.
bool pair_halves_off() {
  static const bool off = [] {
    const char* e = getenv("B2MSL_GEMM_PAIR_HALVES");
    return e != nullptr && !strcmp(e, "0");
  }();
  return off;
}

template <typename TO, bool B_MN>
int launch_pair(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tbh, const CUtensorMap& tc,
                const void* bias, int bias_dt, long long M, long long N, long long K, float alpha, int act,
                uint32_t idesc, uint32_t idesc_half, cudaStream_t st) {
  auto kern = gemm_pair_kernel<TO, B_MN>;
  constexpr size_t smem = 1024 + PairCfg<TO>::kRing * kStageBytes + PairCfg<TO>::kEpiSmem + sizeof(PairBarriers);
  static_assert(smem <= 227 * 1024, "shared memory per CTA exceeded");
  B2_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  const int sms = device_sm_count();
  const long long tiles = ((M + kPM - 1) / kPM) * ((N + kBN - 1) / kBN);
  const long long pairs = tiles < sms / 2 ? tiles : sms / 2;
  // last wave in halves when it fills at most half of the pairs
  const long long rem = tiles % pairs;
  const long long tail_start = (rem > 0 && 2 * rem <= pairs && !pair_halves_off()) ? tiles - rem : tiles;
  kern<<<(unsigned)(2 * pairs), kThreads, smem, st>>>(ta, tb, tbh, tc, bias, bias_dt, (int)M, (int)N, (int)K,
                                                      alpha, act, idesc, idesc_half, (int)tail_start,
                                                      epi_program());
  B2_CHECK_LAUNCH();
  return B2_OK;
}

}  // namespace

// True when the pair kernel serves this call: fp16/bf16 in, no row-softmax
// epilogue, C describable by a TMA map (16-byte aligned base and row pitch,
// unit column stride), at least one full wave of 256 x 256 tiles, and a
// problem short enough to run at burst clocks (<= 4e12 FLOP).
bool gemm_pair_wanted(long long M, long long N, long long K, const int64_t* s, const void* C, int out_dt,
                      int act, bool forced) {
  if (act == B2_ACT_SOFTMAX || K <= 0) return false;
  const int osz = dtype_size(out_dt);
  if (s[5] != 1 || (reinterpret_cast<uintptr_t>(C) & 15) != 0 || (s[4] * osz) % 16 != 0 || s[4] < N) return false;
  if (forced) return true;
  const long long tiles = ((M + kPM - 1) / kPM) * ((N + kBN - 1) / kBN);
  // Measured on B200 (bf16, L2 flushed): pairs win 7-12 % at 4096^3..8192^3
  // (1300 / 1590 vs 1150 / 1475 TFLOP/s), but on a 35-TFLOP problem that runs
  // tens of ms under the 1 kW power cap the one-SM kernel sustained
  // 1220 vs 1050-1180; pairs are used up to 4e12 FLOP per call.
  return 2 * tiles >= device_sm_count() && 2.0 * (double)M * (double)N * (double)K <= 4e12;
}

int gemm_pair_launch(const void* A, const void* B, const void* bias, void* C, long long M, long long N,
                     long long K, const int64_t* s, float alpha, int act, int in_dt, int bias_dt, int out_dt,
                     cudaStream_t st) {
  const CUtensorMapDataType tdt =
      in_dt == B2_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUtensorMap ta, tb, tbh, tc;
  {
    const uint64_t dims[2] = {(uint64_t)K, (uint64_t)M};
    const uint64_t strides[1] = {(uint64_t)s[0] * 2};
    const uint32_t box[2] = {kBK, kHalf};
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
    const uint32_t box[2] = {kBK, kHalf};
    if (!encode_tmap(&tb, tdt, 2, B, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B)) return B2_ELAUNCH;
    const uint32_t box_half[2] = {kBK, kHalf / 2};  // 64 columns of B per CTA in a half tile
    if (!encode_tmap(&tbh, tdt, 2, B, dims, strides, box_half, CU_TENSOR_MAP_SWIZZLE_128B)) return B2_ELAUNCH;
  }
  if (b_mn) tbh = tb;
  {
    const int osz = dtype_size(out_dt);
    const CUtensorMapDataType cdt = out_dt == B2_F32    ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                    : out_dt == B2_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                        : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    const uint64_t dims[2] = {(uint64_t)N, (uint64_t)M};
    const uint64_t strides[1] = {(uint64_t)s[4] * osz};
    const uint32_t box[2] = {32, 32};
    if (!encode_tmap(&tc, cdt, 2, C, dims, strides, box,
                     osz == 2 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_128B))
      return B2_ELAUNCH;
  }
  const uint32_t idesc = idesc_f16(kPM, kBN, in_dt == B2_BF16, false, b_mn);
  const uint32_t idesc_half = idesc_f16(kPM, kBN / 2, in_dt == B2_BF16, false, b_mn);
  if (bias == nullptr) bias_dt = B2_F32;
  switch (out_dt) {
    case B2_F16:
      return b_mn ? launch_pair<__half, true>(ta, tb, tbh, tc, bias, bias_dt, M, N, K, alpha, act, idesc, idesc_half, st)
                  : launch_pair<__half, false>(ta, tb, tbh, tc, bias, bias_dt, M, N, K, alpha, act, idesc, idesc_half, st);
    case B2_BF16:
      return b_mn ? launch_pair<__nv_bfloat16, true>(ta, tb, tbh, tc, bias, bias_dt, M, N, K, alpha, act, idesc, idesc_half, st)
                  : launch_pair<__nv_bfloat16, false>(ta, tb, tbh, tc, bias, bias_dt, M, N, K, alpha, act, idesc, idesc_half, st);
    case B2_F32:
      return b_mn ? launch_pair<float, true>(ta, tb, tbh, tc, bias, bias_dt, M, N, K, alpha, act, idesc, idesc_half, st)
                  : launch_pair<float, false>(ta, tb, tbh, tc, bias, bias_dt, M, N, K, alpha, act, idesc, idesc_half, st);
  }
  set_error("b2_gemm: unsupported out dtype %d", out_dt);
  return B2_EINVAL;
}

uint32_t pair_read_status(bool clear) {
  uint32_t v = 0;
  cudaMemcpyFromSymbol(&v, g_pair_status, sizeof(v));
  if (clear) {
    const uint32_t z = 0;
    cudaMemcpyToSymbol(g_pair_status, &z, sizeof(z));
  }
  return v;
}

}  // namespace b2
