// FlashAttention forward on 5th-generation tensor cores (fp16 / bf16 in,
// fp32 accumulate), head_dim 32, 64 or 128.
//
// Replaces the reference's simdgroup-MMA template
// `make_flash_attention_kernel_simdgroup` (triton_msl/codegen/_msl_templates.py:1833-2070),
// with the semantics of the canonical kernel `_flash_attn_fwd`
// (tests/test_flash_attention.py:35-118): online max / exp / sum per block of
// keys, causal keep iff key <= query with the key loop bounded by the query
// block, O / l at the end.
//
// One CTA owns 256 query rows (two 128-row tiles Q0, Q1) of one (batch, head):
//  * warp 0: TMA producer (Q0, Q1 once; K_j, V_j through 2-deep rings).
//  * warp 1: TMEM allocation and the single issuing thread of tcgen05.mma.
//  * warps 4-7: softmax + O correction for Q0; warps 8-11: the same for Q1.
// TMEM (512 columns): S0 | S1 (128 fp32 columns each) | O0 | O1 (D each).
// The softmax warps read S_t row-per-thread, write P_t as packed fp16/bf16
// over the first 64 columns of S_t, and the MMA warp consumes P_t straight
// from TMEM (tcgen05.mma with A in tensor memory), so P never touches shared
// memory. MMA issue order per key block j:
//     PV0_j, S0_{j+1}, PV1_j, S1_{j+1}
// so while one softmax warpgroup works on S_t the tensor core runs the other
// tile's GEMMs. A commit after S_t_{j+1} also covers PV_t_j (commits track all
// earlier MMAs), which is what lets the softmax warps rescale O_t safely.
// O is only rescaled when a row max grows by more than 2^8 (the stale max is
// used consistently for P and l, so the result is exact up to rounding).
// For D <= 64, where TMEM has columns to spare, the row sums l come from the
// tensor core too: after each P_t.V an N=16 MMA of P_t with a ones tile
// accumulates l_t into 16 TMEM columns L_t beside O (every column holds the
// row sum), so the softmax warps issue no per-score additions; L_t is
// rescaled with O_t and read once per unit.
#include "sm100.cuh"

namespace b2 {
namespace {

using namespace sm100;

__device__ uint32_t g_fa_status;

constexpr int kBM = 128;      // query rows per tile
constexpr int kBN = 128;      // keys per block
constexpr int kThreads = 384; // 12 warps
// Register split (setmaxnreg): warpgroup 0 (TMA, MMA, two idle warps) gives
// registers to the two softmax warpgroups, which hold a 128-key row of S and
// its packed P per thread. The sum must fit the block's launch allocation,
// kThreads x kLaunchRegs; the host checks the compiled register count.
constexpr int kRegsProducer = 56, kRegsSoftmax = 224, kLaunchRegs = 168;
static_assert(128 * (kRegsProducer + 2 * kRegsSoftmax) <= kThreads * kLaunchRegs,
              "register split exceeds the launch allocation");
constexpr uint32_t kTmemCols = 512;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kRescaleThreshold = 8.0f;  // log2 units

struct __align__(8) FaBarriers {
  uint64_t q_full;
  uint64_t k_full[2], k_empty[2];
  uint64_t v_full[2], v_empty[2];
  uint64_t s_full[2];
  uint64_t p_full[2];
  uint64_t o_full[2], o_empty[2];  // per tile: O_t complete / O_t read out
  uint64_t q_empty;
  uint64_t done;
  uint32_t tmem_base;
  int abort_flag;
};

template <int D>
struct FaCfg {
  static constexpr int kAtom = D >= 64 ? 64 : 32;           // elements per swizzle atom row
  static constexpr int kAtomBytes = kAtom * 2;              // 128 or 64
  static constexpr uint32_t kSwz = D >= 64 ? kSwizzle128 : kSwizzle64;
  static constexpr int kNumAtoms = D / kAtom;
  static constexpr uint32_t kTileBytes = 128 * D * 2;       // one 128-row tile
  static constexpr uint32_t kAtomTileBytes = 128 * kAtomBytes;
  static constexpr uint32_t kSBO = 8 * kAtomBytes;          // 8-row group pitch
  // output staging: per softmax warp one 32-row x atom-wide block
  static constexpr uint32_t kOutStageBytes = 32 * kAtomBytes;
  // row sums on the tensor core (TMEM: 2 x (128 + D + 16) columns <= 512)
  static constexpr bool kSumMma = D <= 64;
  static constexpr uint32_t kOnesBytes = kSumMma ? 1024 : 0;  // ones tile, B of the l MMA
  static constexpr size_t kSmem =
      1024 + 6 * kTileBytes + 8 * kOutStageBytes + kOnesBytes + sizeof(FaBarriers);
  // TMEM: S0 | S1 (128 columns each) | O0 | O1 (D each) | L0 | L1 (16 each, D <= 64)
  static_assert(2 * (kBN + D + (kSumMma ? 16 : 0)) <= (int)kTmemCols, "TMEM columns exceeded");
  static_assert(kSmem <= 227 * 1024, "shared memory per CTA exceeded");
};

// Of every 8 key pairs, how many take their exponentials on the MUFU (the
// rest use exp2_poly2 on the FMA pipe).
#ifndef B2_FA_MUFU8_D128
#define B2_FA_MUFU8_D128 5
#endif
#ifndef B2_FA_MUFU8_SMALL
#define B2_FA_MUFU8_SMALL 4
#endif
template <int D>
__device__ __forceinline__ constexpr bool on_mufu(int i) {
  return D == 128 ? ((i & 7) < B2_FA_MUFU8_D128)
                  : (B2_FA_MUFU8_SMALL == 4 ? ((i & 1) == 0) : ((i & 7) < B2_FA_MUFU8_SMALL));
}

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// ---- packed fp32x2 arithmetic (one issue slot for two lanes' worth of work)
typedef unsigned long long f2_t;
__device__ __forceinline__ f2_t f2_pack(float a, float b) {
  f2_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ void f2_unpack(f2_t v, float& a, float& b) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(v));
}
__device__ __forceinline__ f2_t f2_fma(f2_t a, f2_t b, f2_t c) {
  f2_t r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}
__device__ __forceinline__ f2_t f2_add(f2_t a, f2_t b) {
  f2_t r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ f2_t f2_add_rm(f2_t a, f2_t b) {
  f2_t r;
  asm("add.rm.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

// 2^x for two lanes on the FMA pipe, x clamped to [-126, 126].
// Range reduction: t = x + 1.5*2^23 rounded toward -inf holds floor(x) in the
// low mantissa bits of t; f = x - floor(x) lies in [0, 1); 2^f comes from a
// cubic p(f) = 1 + f*(c1 + f*(c2 + f*c3)) whose coefficients are this file's
// own weighted least-squares fit of 2^f on [0, 1] with p(0) = 1 and p(1) = 2
// (max relative error 1.03e-4, below the fp16 / bf16 rounding of P); floor(x)
// is then added into the exponent field.
__device__ __forceinline__ void exp2_poly2(float x0, float x1, float& y0, float& y1) {
  constexpr float kMagic = 12582912.0f;  // 1.5 * 2^23
  constexpr float c1 = 0.6954244f, c2 = 0.22630768f, c3 = 0.07826797f;
  x0 = fmaxf(x0, -126.f);
  x1 = fmaxf(x1, -126.f);
  const f2_t x = f2_pack(x0, x1);
  const f2_t t = f2_add_rm(x, f2_pack(kMagic, kMagic));
  const f2_t xi = f2_add(t, f2_pack(-kMagic, -kMagic));
  const f2_t f = f2_fma(xi, f2_pack(-1.f, -1.f), x);
  f2_t p = f2_fma(f, f2_pack(c3, c3), f2_pack(c2, c2));
  p = f2_fma(f, p, f2_pack(c1, c1));
  p = f2_fma(f, p, f2_pack(1.f, 1.f));
  float p0, p1, t0, t1;
  f2_unpack(p, p0, p1);
  f2_unpack(t, t0, t1);
  // bits(t) << 23 == floor(x) << 23 (mod 2^32): the magic's own bits shift out.
  y0 = __int_as_float(__float_as_int(p0) + (__float_as_int(t0) << 23));
  y1 = __int_as_float(__float_as_int(p1) + (__float_as_int(t1) << 23));
}

template <int D, bool BF16>
__global__ void __launch_bounds__(kThreads, 1)
fa_sm100_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmO,
                int H, int BH, int S, int num_qblk, float scale_log2,
                int causal) {
  using Cfg = FaCfg<D>;
  using T = typename std::conditional<BF16, __nv_bfloat16, __half>::type;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;                              // 2 tiles
  uint8_t* sK = smem + 2 * Cfg::kTileBytes;        // 2 stages
  uint8_t* sV = smem + 4 * Cfg::kTileBytes;        // 2 stages
  uint8_t* sO = smem + 6 * Cfg::kTileBytes;        // output staging, 8 warps
  uint8_t* sOnes = sO + 8 * Cfg::kOutStageBytes;  // kOnesBytes of 1.0 (D <= 64)
  FaBarriers* bars = reinterpret_cast<FaBarriers*>(sOnes + Cfg::kOnesBytes);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int num_units = num_qblk * BH;
  const int nkv_all = (S + kBN - 1) / kBN;
  // Unit u -> (query block, batch*head); heaviest query blocks first (causal
  // work grows with the block index). CTA i takes, in round r, unit
  // r*G + i (even r) or r*G + G-1-i (odd r): the serpentine order pairs heavy
  // and light units, matching a longest-first dynamic schedule without any
  // global counter.
  auto unit_at = [&](uint32_t r) -> int {
    const long long base = (long long)r * gridDim.x;
    const long long u = base + ((r & 1) ? (gridDim.x - 1 - blockIdx.x) : blockIdx.x);
    return u > 0x7fffffffLL ? 0x7fffffff : (int)u;
  };
  auto decode = [&](int u, int& b, int& h, int& m0, int& n0, int& n1) {
    const int qblk = num_qblk - 1 - u / BH;
    const int bh = u % BH;
    b = bh / H;
    h = bh % H;
    m0 = qblk * 2 * kBM;
    n1 = nkv_all;
    n0 = nkv_all;
    if (causal) {
      n1 = min((m0 + 2 * kBM + kBN - 1) / kBN, nkv_all);
      n0 = min((m0 + kBM + kBN - 1) / kBN, nkv_all);
    }
  };
  volatile int* abort_flag = &bars->abort_flag;

  if (threadIdx.x == 0) {
    mbar_init(&bars->q_full, 1);
    mbar_init(&bars->q_empty, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bars->k_full[i], 1);
      mbar_init(&bars->k_empty[i], 1);
      mbar_init(&bars->v_full[i], 1);
      mbar_init(&bars->v_empty[i], 1);
      mbar_init(&bars->s_full[i], 1);
      mbar_init(&bars->p_full[i], 4);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bars->o_full[i], 1);
      mbar_init(&bars->o_empty[i], 4);
    }
    mbar_init(&bars->done, 1);
    bars->abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
    tma_prefetch_desc(&tmO);
  }
  if (warp == 1) {
    tmem_alloc(&bars->tmem_base, kTmemCols);
    tmem_relinquish();
  }
  if constexpr (Cfg::kSumMma) {
    // 1.0 in every element (fp16 0x3C00, bf16 0x3F80); the tensor core reads
    // the tile through the async proxy.
    if (threadIdx.x < Cfg::kOnesBytes / 16) {
      const uint32_t w = BF16 ? 0x3F803F80u : 0x3C003C00u;
      reinterpret_cast<uint4*>(sOnes)[threadIdx.x] = make_uint4(w, w, w, w);
      fence_proxy_async_smem();
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem_base;
  const uint32_t tS[2] = {tmem, tmem + 128};
  const uint32_t tO[2] = {tmem + 256, tmem + 256 + D};
  const uint32_t tL[2] = {tmem + 256 + 2 * D, tmem + 256 + 2 * D + 16};  // D <= 64 only

  // Each role branch executes its own setmaxnreg, so the compiler sees one
  // register budget per region.
  if (warp == 0) {
    // ---------------------------------------------------------------- TMA
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kRegsProducer));
    if (lane == 0) {
      bool ok = true;
      uint32_t g = 0;   // K/V blocks issued by this CTA (ring position)
      uint32_t ui = 0;  // units started
      for (;; ++ui) {
        const int u = unit_at(ui);
        if (u >= num_units || !ok) break;
        int b, h, m0, n0, n1;
        decode(u, b, h, m0, n0, n1);
        // Q of the previous unit is free once its last Q.K^T has been issued.
        if (!mbar_wait(&bars->q_empty, (ui & 1) ^ 1u, abort_flag, &g_fa_status, DEV_TIMEOUT_SLOT)) { ok = false; break; }
        mbar_arrive_expect_tx(&bars->q_full, 2 * Cfg::kTileBytes);
        for (int t = 0; t < 2; ++t)
          for (int a = 0; a < Cfg::kNumAtoms; ++a)
            tma_load_4d(sQ + t * Cfg::kTileBytes + a * Cfg::kAtomTileBytes, &tmQ, &bars->q_full,
                        a * Cfg::kAtom, m0 + t * kBM, h, b);
        for (int j = 0; j < n1; ++j, ++g) {
          const int s = g & 1;
          const uint32_t par = ((g >> 1) & 1) ^ 1u;
          if (!mbar_wait(&bars->k_empty[s], par, abort_flag, &g_fa_status, DEV_TIMEOUT_SLOT)) { ok = false; break; }
          mbar_arrive_expect_tx(&bars->k_full[s], Cfg::kTileBytes);
          for (int a = 0; a < Cfg::kNumAtoms; ++a)
            tma_load_4d(sK + s * Cfg::kTileBytes + a * Cfg::kAtomTileBytes, &tmK, &bars->k_full[s],
                        a * Cfg::kAtom, j * kBN, h, b);
          if (!mbar_wait(&bars->v_empty[s], par, abort_flag, &g_fa_status, DEV_TIMEOUT_SLOT)) { ok = false; ++g; break; }
          mbar_arrive_expect_tx(&bars->v_full[s], Cfg::kTileBytes);
          for (int a = 0; a < Cfg::kNumAtoms; ++a)
            tma_load_4d(sV + s * Cfg::kTileBytes + a * Cfg::kAtomTileBytes, &tmV, &bars->v_full[s],
                        a * Cfg::kAtom, j * kBN, h, b);
        }
      }
      // Bounded drain of copies still in flight into this CTA's shared memory:
      // the latest fill of each ring slot and of Q.
      const unsigned long long t0 = globaltimer();
      auto drain = [&](uint64_t* bar, uint32_t par) {
        while (!mbar_test(smem_addr(bar), par)) {
          if (globaltimer() - t0 > kWaitLimitNs) { atomicOr(&g_fa_status, DEV_TIMEOUT_TMA); return; }
        }
      };
      if (ui > 0) drain(&bars->q_full, (ui - 1) & 1);
      for (uint32_t j = (g > 2 ? g - 2 : 0); j < g; ++j) {
        drain(&bars->k_full[j & 1], (j >> 1) & 1);
        drain(&bars->v_full[j & 1], (j >> 1) & 1);
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kRegsProducer));
    // The whole warp runs the issue loop (so loop-invariant operands stay
    // warp-uniform) and one elected lane issues each tcgen05 instruction.
    {
      const bool leader = elect_one();
      constexpr uint32_t idS = idesc_f16(kBM, kBN, BF16, false, false);  // Q K^T: both K-major
      constexpr uint32_t idO = idesc_f16(kBM, D, BF16, false, true);     // P V: V is MN-major
      const uint32_t q0 = smem_addr(sQ), k0 = smem_addr(sK), v0 = smem_addr(sV);
      bool ok = true;
      bool issued = false;
      // Base descriptors per buffer, computed once: each MMA issue below is a
      // 64-bit add of a compile-time offset plus the tcgen05.mma itself.
      const uint64_t dq0 = sdesc(q0, 16, Cfg::kSBO, Cfg::kSwz);
      const uint64_t dq1 = sdesc(q0 + Cfg::kTileBytes, 16, Cfg::kSBO, Cfg::kSwz);
      const uint64_t dk0 = sdesc(k0, 16, Cfg::kSBO, Cfg::kSwz);
      const uint64_t dk1 = sdesc(k0 + Cfg::kTileBytes, 16, Cfg::kSBO, Cfg::kSwz);
      const uint64_t dv0 = sdesc(v0, Cfg::kAtomTileBytes, Cfg::kSBO, Cfg::kSwz);
      const uint64_t dv1 = sdesc(v0 + Cfg::kTileBytes, Cfg::kAtomTileBytes, Cfg::kSBO, Cfg::kSwz);
      auto qk = [&](int t, int ks) {
        const uint64_t da = t ? dq1 : dq0, db = ks ? dk1 : dk0;
        const uint32_t d = t ? tS[1] : tS[0];
#pragma unroll
        for (int k = 0; k < D / 16; ++k) {
          const uint32_t off16 =
              ((k * 16 / Cfg::kAtom) * Cfg::kAtomTileBytes + (k * 16 % Cfg::kAtom) * 2) >> 4;
          if (leader) mma_f16_ss(d, da + off16, db + off16, idS, k > 0 ? 1u : 0u);
        }
      };
      auto pv = [&](int t, int vs, bool accumulate) {
        const uint64_t db = vs ? dv1 : dv0;
        const uint32_t d = t ? tO[1] : tO[0], pa = t ? tS[1] : tS[0];
        const uint32_t acc0 = accumulate ? 1u : 0u;
#pragma unroll
        for (int k = 0; k < kBN / 16; ++k) {
          // A = P_t: 16 keys = 8 packed TMEM columns per step.
          // B = V: MN-major, 16 key rows = 16 * atom-row bytes per step,
          //        64-wide D chunks kAtomTileBytes apart (the LBO).
          if (leader) mma_f16_ts(d, pa + k * 8, db + ((k * 16 * Cfg::kAtomBytes) >> 4), idO, k > 0 ? 1u : acc0);
        }
      };
      // l_t += P_t . ones (D <= 64): one K=16 slice of the ones tile serves
      // every key step, since all its elements are equal. No swizzle; the
      // K-major core matrices lie within the tile's first 512 bytes.
      constexpr uint32_t idL = idesc_f16(kBM, 16, BF16, false, false);
      const uint64_t dones = sdesc(smem_addr(sOnes), 128, 256, 0);
      auto pl = [&](int t, bool accumulate) {
        if constexpr (Cfg::kSumMma) {
          const uint32_t pa = t ? tS[1] : tS[0];
#pragma unroll
          for (int k = 0; k < kBN / 16; ++k)
            if (leader) mma_f16_ts(tL[t], pa + k * 8, dones, idL, (k > 0 || accumulate) ? 1u : 0u);
        }
      };
      (void)dones;
      uint32_t g = 0;             // K/V ring position
      uint32_t gs0 = 0, gs1 = 0;  // P blocks consumed per tile (p_full parity)
      uint32_t ui = 0;
      for (;; ++ui) {
        const int u = unit_at(ui);
        if (u >= num_units || !ok) break;
        int b, h, m0, n0, n1;
        decode(u, b, h, m0, n0, n1);
        const int n = n1;
        (void)b; (void)h; (void)m0;
        if (!mbar_wait(&bars->q_full, ui & 1, abort_flag, &g_fa_status, DEV_TIMEOUT_TMA)) { ok = false; break; }
        if (!mbar_wait(&bars->k_full[g & 1], (g >> 1) & 1, abort_flag, &g_fa_status, DEV_TIMEOUT_TMA)) { ok = false; break; }
        tc_fence_after();
        // S of this unit's first block; S_t's TMEM held the previous unit's last
        // P_t, whose P.V was issued earlier (tcgen05.mma executes in order).
        if (n0 > 0) { qk(0, g & 1); if (leader) mma_commit(&bars->s_full[0]); }
        qk(1, g & 1);
        if (leader) mma_commit(&bars->s_full[1]);
        if (leader) mma_commit(&bars->k_empty[g & 1]);
        if (n == 1 && leader) mma_commit(&bars->q_empty);
        issued = true;
        for (int j = 0; j < n; ++j) {
          const uint32_t gj = g + j;
          const int vs = gj & 1;
          const uint32_t vph = (gj >> 1) & 1;
          if (!mbar_wait(&bars->v_full[vs], vph, abort_flag, &g_fa_status, DEV_TIMEOUT_TMA)) { ok = false; break; }
          if (j < n0) {
            // O_0 holds the previous unit's result until tile 0's softmax warps
            // have read it out
            if (j == 0 && !mbar_wait(&bars->o_empty[0], (ui & 1) ^ 1u, abort_flag, &g_fa_status, DEV_TIMEOUT_EPI)) { ok = false; break; }
            if (!mbar_wait(&bars->p_full[0], gs0 & 1, abort_flag, &g_fa_status, DEV_TIMEOUT_EPI)) { ok = false; break; }
            tc_fence_after();
            pv(0, vs, j > 0);
            pl(0, j > 0);
            ++gs0;
            // causal: tile 0 ends a block before tile 1, and its output is
            // stored while tile 1 works on its diagonal block
            if (j == n0 - 1 && leader) mma_commit(&bars->o_full[0]);
          }
          const uint32_t gk = gj + 1;
          const int ks = gk & 1;
          if (j + 1 < n) {
            if (!mbar_wait(&bars->k_full[ks], (gk >> 1) & 1, abort_flag, &g_fa_status, DEV_TIMEOUT_TMA)) { ok = false; break; }
            tc_fence_after();
            if (j + 1 < n0) { qk(0, ks); if (leader) mma_commit(&bars->s_full[0]); }
          }
          if (j == 0 && !mbar_wait(&bars->o_empty[1], (ui & 1) ^ 1u, abort_flag, &g_fa_status, DEV_TIMEOUT_EPI)) { ok = false; break; }
          if (!mbar_wait(&bars->p_full[1], gs1 & 1, abort_flag, &g_fa_status, DEV_TIMEOUT_EPI)) { ok = false; break; }
          tc_fence_after();
          pv(1, vs, j > 0);
          pl(1, j > 0);
          ++gs1;
          if (j == n - 1 && leader) mma_commit(&bars->o_full[1]);
          if (leader) mma_commit(&bars->v_empty[vs]);
          if (j + 1 < n) {
            qk(1, ks);
            if (leader) mma_commit(&bars->s_full[1]);
            if (leader) mma_commit(&bars->k_empty[ks]);
            if (j + 2 == n && leader) mma_commit(&bars->q_empty);  // last Q.K^T of the unit
          }
        }
        if (!ok) break;
        g += n;
      }
      if (issued) {
        if (leader) mma_commit(&bars->done);
        const unsigned long long t0 = globaltimer();
        while (!mbar_test(smem_addr(&bars->done), 0)) {
          if (globaltimer() - t0 > kWaitLimitNs) { atomicOr(&g_fa_status, DEV_TIMEOUT_MMA); break; }
        }
      }
    }
  } else if (warp >= 4) {
    // ------------------------------------------------- softmax / correction
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kRegsSoftmax));
    const int t = (warp >= 8) ? 1 : 0;
    const int quarter = warp & 3;
    const int row_in_tile = quarter * 32 + lane;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    bool ok = true;
    uint32_t gs = 0;  // S blocks of this tile seen (s_full parity)
    uint32_t ui = 0;
    for (;; ++ui) {
    const int u = unit_at(ui);
    if (u >= num_units || !ok) break;
    int b, h, m0, n0, n1;
    decode(u, b, h, m0, n0, n1);
    const int qrow = m0 + t * kBM + row_in_tile;
    const int n_t = t == 0 ? n0 : n1;
    float m_run = -INFINITY;  // running max in log2 units (possibly stale)
    float l_run = 0.f;
    for (int j = 0; j < n_t; ++j) {
      if (!mbar_wait(&bars->s_full[t], gs & 1, abort_flag, &g_fa_status, DEV_TIMEOUT_MMA)) { ok = false; break; }
      ++gs;
      tc_fence_after();
      // All four 32-column loads in flight, then one wait; the empty asm
      // statements pin every use of the loaded registers after the wait.
      uint32_t sr[kBN];
#pragma unroll
      for (int c = 0; c < kBN / 32; ++c)
        tmem_ld32(tS[t] + lane_off + c * 32, *reinterpret_cast<uint32_t(*)[32]>(&sr[c * 32]));
      tmem_ld_wait();
#pragma unroll
      for (int i = 0; i < kBN; ++i) asm volatile("" : "+r"(sr[i]));
      float s[kBN];
#pragma unroll
      for (int i = 0; i < kBN; ++i) s[i] = __uint_as_float(sr[i]);
      const int kbase = j * kBN;
      const bool need_mask = (kbase + kBN > S) || (causal && kbase + kBN - 1 > m0 + t * kBM);
      if (need_mask) {
        const int lim = min(S - kbase, causal ? qrow - kbase + 1 : kBN);  // keys [0, lim) kept
        if constexpr (D < 128) {
          // Per 32-key chunk, warp-uniform: chunks every lane keeps are skipped
          // (on the causal diagonal only the warp's own 32x32 square and the
          // chunks after it need the per-key comparison). Measured: +6..10 %
          // for D=32 causal; at D=128 the branches cost the softmax warps
          // register spills and the plain per-key mask is faster.
          const int lim_lo = __reduce_min_sync(0xffffffffu, lim);
#pragma unroll
          for (int c = 0; c < kBN / 32; ++c) {
            if (lim_lo < 32 * (c + 1)) {
#pragma unroll
              for (int e = 0; e < 32; ++e)
                if (32 * c + e >= lim) s[32 * c + e] = -INFINITY;
            }
          }
        } else {
#pragma unroll
          for (int i = 0; i < kBN; ++i)
            if (i >= lim) s[i] = -INFINITY;
        }
      }
      // Row max: four independent 3-input max chains.
      float mq[4] = {s[0], s[1], s[2], s[3]};
#pragma unroll
      for (int i = 4; i < kBN; i += 8) {
        mq[0] = fmax3(mq[0], s[i], s[i + 1]);
        mq[1] = fmax3(mq[1], s[i + 2], s[i + 3]);
        mq[2] = fmax3(mq[2], i + 4 < kBN ? s[i + 4] : -INFINITY, i + 5 < kBN ? s[i + 5] : -INFINITY);
        mq[3] = fmax3(mq[3], i + 6 < kBN ? s[i + 6] : -INFINITY, i + 7 < kBN ? s[i + 7] : -INFINITY);
      }
      const float mx = fmaxf(fmaxf(mq[0], mq[1]), fmaxf(mq[2], mq[3])) * scale_log2;
      // Rescale only when some row of this warp grew its max by > 2^8.
      const bool grow = mx > m_run + kRescaleThreshold;
      const bool warp_rescale = __any_sync(0xffffffffu, grow);
      float alpha = 1.f;
      if (warp_rescale) {
        const float m_new = fmaxf(m_run, mx);
        alpha = (m_run == -INFINITY) ? 0.f : ex2(m_run - m_new);
        m_run = m_new;
      }
      const float m_use = m_run == -INFINITY ? 0.f : m_run;
      // p = 2^(s*scale_log2 - m). Measured on B200, per warp instruction per SM
      // sub-partition: MUFU ex2 8 cycles on its own pipe; f32x2 FMA/ADD 2 cycles
      // (yet a scalar-FFMA version of this loop measured 10 % slower), max / cvt
      // 2 on the ALU pipe. All
      // exponentials on the MUFU would take as long as the tensor core's work
      // per key block; the FMA-pipe cubic costs ~9 issue slots per score. Share
      // on the MUFU measured best: 5/8 of the key pairs at D=128, 1/2 (every
      // other pair) at D <= 64.
      const f2_t sc2 = f2_pack(scale_log2, scale_log2), nm2 = f2_pack(-m_use, -m_use);
      f2_t acc2[4] = {0ull, 0ull, 0ull, 0ull};
      uint32_t p[kBN / 2];
#pragma unroll
      for (int i = 0; i < kBN / 2; ++i) {
        const f2_t x2 = f2_fma(f2_pack(s[2 * i], s[2 * i + 1]), sc2, nm2);
        float x0, x1, p0, p1;
        f2_unpack(x2, x0, x1);
        if (on_mufu<D>(i)) {
          p0 = ex2(x0);
          p1 = ex2(x1);
        } else {
          exp2_poly2(x0, x1, p0, p1);
        }
        if constexpr (!Cfg::kSumMma) acc2[i & 3] = f2_add(acc2[i & 3], f2_pack(p0, p1));
        p[i] = BF16 ? pack_bf162(p0, p1) : pack_half2(p0, p1);
      }
      if constexpr (!Cfg::kSumMma) {
        const f2_t a01 = f2_add(acc2[0], acc2[1]), a23 = f2_add(acc2[2], acc2[3]);
        float u0, u1;
        f2_unpack(f2_add(a01, a23), u0, u1);
        l_run = l_run * alpha + (u0 + u1);
      }
#pragma unroll
      for (int c = 0; c < kBN / 2 / 32; ++c) {
        uint32_t r[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) r[i] = p[c * 32 + i];
        tmem_st32(tS[t] + lane_off + c * 32, r);
      }
      if (warp_rescale && j > 0) {
#pragma unroll
        for (int c = 0; c < D / 32; ++c) {
          uint32_t r[32];
          tmem_ld32(tO[t] + lane_off + c * 32, r);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 32; ++i) r[i] = __float_as_uint(__uint_as_float(r[i]) * alpha);
          tmem_st32(tO[t] + lane_off + c * 32, r);
        }
        if constexpr (Cfg::kSumMma) {
          const uint32_t lc = tmem_ld1(tL[t] + lane_off);
          tmem_ld_wait();
          tmem_st1(tL[t] + lane_off, __float_as_uint(__uint_as_float(lc) * alpha));
        }
      }
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->p_full[t]);
    }
    if (!ok || !mbar_wait(&bars->o_full[t], ui & 1, abort_flag, &g_fa_status, DEV_TIMEOUT_MMA)) {
      ok = false;
      break;
    }
    {
      tc_fence_after();
      if constexpr (Cfg::kSumMma) {
        l_run = __uint_as_float(tmem_ld1(tL[t] + lane_off));
        tmem_ld_wait();
      }
      const float inv = l_run > 0.f ? 1.f / l_run : 0.f;
      // O rows -> swizzled staging (one atom-wide 32-row block per warp) -> TMA
      // store; rows >= S are clipped by the TMA unit. One atom at a time.
      uint8_t* stg = sO + (warp - 4) * Cfg::kOutStageBytes;
      const int swz = ((lane * Cfg::kAtomBytes) >> 7) & (Cfg::kAtomBytes / 16 - 1);
#pragma unroll
      for (int at = 0; at < Cfg::kNumAtoms; ++at) {
        if (lane == 0) bulk_wait_group_read<0>();  // previous store has read the buffer
        __syncwarp();
#pragma unroll
        for (int c = 0; c < Cfg::kAtom / 32; ++c) {
          uint32_t r[32];
          tmem_ld32(tO[t] + lane_off + at * Cfg::kAtom + c * 32, r);
          tmem_ld_wait();
#pragma unroll
          for (int v = 0; v < 4; ++v) {
            uint32_t w[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const float f0 = __uint_as_float(r[v * 8 + 2 * e]) * inv;
              const float f1 = __uint_as_float(r[v * 8 + 2 * e + 1]) * inv;
              w[e] = BF16 ? pack_bf162(f0, f1) : pack_half2(f0, f1);
            }
            *reinterpret_cast<uint4*>(stg + lane * Cfg::kAtomBytes + (((c * 4 + v) ^ swz) * 16)) =
                make_uint4(w[0], w[1], w[2], w[3]);
          }
        }
        if (at == Cfg::kNumAtoms - 1) {
          // every TMEM read of O is done: the next unit's first P.V may overwrite it
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&bars->o_empty[t]);
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          tma_store_4d(stg, &tmO, at * Cfg::kAtom, m0 + t * kBM + quarter * 32, h, b);
          bulk_commit_group();
        }
      }
    }
    }
    if (lane == 0) bulk_wait_group<0>();  // output stores complete before the CTA exits
  } else {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kRegsProducer));
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

template <int D, bool BF16>
int launch(const void* q, const void* k, const void* v, void* o, long long B, long long H,
           long long S, const int64_t* s, float sm_scale, int causal, cudaStream_t st) {
  using Cfg = FaCfg<D>;
  const CUtensorMapDataType tdt = BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  const CUtensorMapSwizzle swz = D >= 64 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B;
  CUtensorMap tm[3];
  const void* ptrs[3] = {q, k, v};
  for (int i = 0; i < 3; ++i) {
    const int64_t* st4 = s + 4 * i;  // z, h, m, d strides
    const uint64_t dims[4] = {(uint64_t)D, (uint64_t)S, (uint64_t)H, (uint64_t)B};
    const uint64_t strides[3] = {(uint64_t)st4[2] * 2, (uint64_t)st4[1] * 2, (uint64_t)st4[0] * 2};
    const uint32_t box[4] = {(uint32_t)Cfg::kAtom, 128, 1, 1};
    if (!encode_tmap(&tm[i], tdt, 4, ptrs[i], dims, strides, box, swz)) return B2_ELAUNCH;
  }
  CUtensorMap tmo;
  {
    const uint64_t dims[4] = {(uint64_t)D, (uint64_t)S, (uint64_t)H, (uint64_t)B};
    const uint64_t strides[3] = {(uint64_t)s[14] * 2, (uint64_t)s[13] * 2, (uint64_t)s[12] * 2};
    const uint32_t box[4] = {(uint32_t)Cfg::kAtom, 32, 1, 1};
    if (!encode_tmap(&tmo, tdt, 4, o, dims, strides, box, swz)) return B2_ELAUNCH;
  }
  auto kern = fa_sm100_kernel<D, BF16>;
  B2_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)Cfg::kSmem));
  {
    // setmaxnreg.inc waits until the block's register pool can serve it, so
    // only launch when the compiled allocation covers the split.
    cudaFuncAttributes fa;
    B2_CUDA_TRY(cudaFuncGetAttributes(&fa, kern));
    if (fa.numRegs < kLaunchRegs) {
      set_error("b2_fa_fwd: kernel compiled with %d registers/thread, register split needs %d",
                fa.numRegs, kLaunchRegs);
      return B2_ELAUNCH;
    }
  }
  const int num_qblk = (int)((S + 2 * kBM - 1) / (2 * kBM));
  const long long units = (long long)num_qblk * B * H;
  const int sms = device_sm_count();
  const long long grid = units < sms ? units : sms;  // persistent: one CTA per SM
  if (units >= (1LL << 31)) {
    set_error("b2_fa_fwd: grid too large");
    return B2_EINVAL;
  }
  kern<<<(unsigned)grid, kThreads, Cfg::kSmem, st>>>(tm[0], tm[1], tm[2], tmo, (int)H, (int)(B * H), (int)S, num_qblk,
                                                      sm_scale * kLog2e, causal);
  B2_CHECK_LAUNCH();
  return B2_OK;
}

}  // namespace

bool fa_sm100_eligible(const void* q, const void* k, const void* v, const void* o, long long D,
                       const int64_t* s, int dtype) {
  if (dtype != B2_F16 && dtype != B2_BF16) return false;
  if (D != 32 && D != 64 && D != 128) return false;
  const void* p[4] = {q, k, v, o};
  for (int i = 0; i < 4; ++i) {
    if ((reinterpret_cast<uintptr_t>(p[i]) & 15) != 0) return false;
    if (s[4 * i + 3] != 1) return false;
    for (int j = 0; j < 3; ++j)
      if ((s[4 * i + j] * 2) % 16 != 0) return false;
  }
  return true;
}

int fa_sm100_launch(const void* q, const void* k, const void* v, void* o, long long B, long long H,
                    long long S, long long D, const int64_t* s, float sm_scale, int causal,
                    int dtype, cudaStream_t st) {
  const bool bf = dtype == B2_BF16;
  switch (D) {
    case 32: return bf ? launch<32, true>(q, k, v, o, B, H, S, s, sm_scale, causal, st)
                       : launch<32, false>(q, k, v, o, B, H, S, s, sm_scale, causal, st);
    case 64: return bf ? launch<64, true>(q, k, v, o, B, H, S, s, sm_scale, causal, st)
                       : launch<64, false>(q, k, v, o, B, H, S, s, sm_scale, causal, st);
    case 128: return bf ? launch<128, true>(q, k, v, o, B, H, S, s, sm_scale, causal, st)
                        : launch<128, false>(q, k, v, o, B, H, S, s, sm_scale, causal, st);
  }
  set_error("b2_fa_fwd: tensor-core path supports head_dim 32/64/128, got %lld", D);
  return B2_EUNSUPPORTED;
}

uint32_t fa_read_status(bool clear) {
  uint32_t v = 0;
  cudaMemcpyFromSymbol(&v, g_fa_status, sizeof(v));
  if (clear) {
    const uint32_t z = 0;
    cudaMemcpyToSymbol(g_fa_status, &z, sizeof(z));
  }
  return v;
}

}  // namespace b2
