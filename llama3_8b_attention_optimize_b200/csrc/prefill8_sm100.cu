// prefill8_sm100.cu -- fused causal GQA prefill, four softmax threads per row in one warp.
//
// Same computation and interface as prefill_sm100.cu (the golden's RoPE -> QK^T/sqrt(d)
// -> causal mask -> softmax -> PV -> bf16, llama3_attention_golden_model.py:162-190),
// organised so that no thread waits on another warp for a row statistic:
//
//   * each Q tile (128 rows = 4 heads x 32 positions) has 8 softmax warps; a warp reads
//     16 rows of S with the 16x256b TMEM shape, so 4 neighbouring lanes share a row (32
//     of its 128 keys each, two rows per thread) and the row max and sum are combined
//     with two warp shuffles -- no shared memory, no barrier;
//   * p (bf16) is written back into TMEM over the row's scores, and O_t += P_t V runs
//     with P_t as the TMEM operand (tcgen05.mma A from tensor memory) and V from shared
//     memory: no shared-memory traffic for P;
//   * the tensor core alternates the two tiles -- PV0(j) QK0(j+1) PV1(j) QK1(j+1) -- so
//     each tile's softmax for K tile j+1 runs while the other tile's PV and QK^T execute;
//   * the shared memory freed from P holds a 4-stage K/V ring and one O staging tile.
//
// Work units, unit order, Q prefetch / rotation between units and the epilogue follow
// prefill_sm100.cu.  Warps: 0-7 softmax tile 0, 8-15 softmax tile 1, 16 TMA producer,
// 17 MMA issuer (+ TMEM allocator), 18-19 RoPE of K tiles (FLAG_ROPE_K).
// TMEM (512 columns): S0 [0,128) (P0 over [0,64)), S1 [128,256), O0 [256,384), O1 [384,512).
#include <cuda.h>

#include "attn_common.cuh"
#include "common.cuh"
#include "gqa_internal.h"

namespace gqa {
namespace prefill8 {

using namespace attn;

constexpr int kD = 128;
constexpr int kG = 4;
constexpr int kBM = 128;
constexpr int kRowsPerHead = kBM / kG;        // 32
constexpr int kPosPerCta = 2 * kRowsPerHead;  // 64
constexpr int kBN = 128;                      // keys per K/V tile
constexpr int kStages = 4;                    // K/V ring stages
constexpr int kTileBytes = 128 * 128 * 2;     // Q, K, V and O tiles: 32 KB
constexpr int kHalf = kHalfTile;
constexpr float kRescaleLog2 = 16.0f;
constexpr int kWarpProducer = 16;
constexpr int kWarpMma = 17;
constexpr int kWarpRope0 = 18;
constexpr int kThreads = 640;
constexpr int kTileThreads = 256;  // softmax threads per Q tile
// Register split (setmaxnreg): launch kRegsLaunch per thread; the helper warpgroup
// (warps 16-19) drops to kRegsHelper, the four softmax warpgroups rise to kRegsSoftmax.
// The host checks the compiled launch count before every launch (an over-budget
// setmaxnreg.inc would never complete).
constexpr int kRegsLaunch = 96;
constexpr int kRegsHelper = 64;
constexpr int kRegsSoftmax = 104;
static_assert(4 * 128 * kRegsSoftmax + 128 * kRegsHelper <= kThreads * kRegsLaunch, "register split over budget");
// Emulated exponentials: pairs k with (k & kEmuMask) == kEmuMask of fully visible tiles
// run on the FMA pipe (3: a quarter), 0 = none (measured fastest here: the FMA-pipe cubic costs more issue
// slots than the MUFU time it saves).
constexpr int kEmuMask = 0;
// One mbarrier arrival per softmax warp (after __syncwarp) instead of one per thread.
constexpr bool kWarpArrive = true;
constexpr int kHandoffCount = kWarpArrive ? kTileThreads / 32 : kTileThreads;

constexpr int kOffQ = 0;
constexpr int kOffKV = kOffQ + 2 * kTileBytes;
constexpr int kOffStage = kOffKV + kStages * kTileBytes;  // O staging tile (the two tiles take turns)
constexpr int kOffBar = kOffStage + kTileBytes;
constexpr int kNumBars = 32;
constexpr int kOffTmemPtr = kOffBar + kNumBars * 8;
constexpr int kSmemBytes = kOffTmemPtr + 16;
static_assert(kSmemBytes <= 232448, "shared memory over the per-block limit");

enum : int {
  B_QFULL = 0,     // [2]  TMA Q tile t of the current unit landed
  B_QREADY = 2,    // [2]  Q tile t rotated (256 arrivals)
  B_QEMPTY = 4,    // [1]  the unit's last QK^T done: Q tiles may be reloaded
  B_KVFULL = 5,    // [4]  TMA K/V stage landed
  B_KVEMPTY = 9,   // [4]  MMAs reading the stage completed
  B_KREADY = 13,   // [4]  K tile rotated (slot k % 4), 64 arrivals
  B_SFULL = 17,    // [2]  S_t = Q_t K^T complete (and so every earlier MMA of the CTA)
  B_PREADY = 19,   // [2]  P_t written into TMEM, O_t rescaled (256 arrivals)
  B_PVDONE = 21,   // [2]  O_t += P_t V complete
  B_OSTAGE = 23,   // [2]  the O staging tile is free for tile t
  B_DRAIN = 25,    // [1]  every MMA of the CTA complete
};
constexpr int kKReadySlots = 4;

enum : int {  // error sites
  SITE_PRODUCER = 0x131,
  SITE_MMA = 0x132,
  SITE_SOFTMAX = 0x133,
  SITE_ROPEK = 0x134,
  SITE_EPILOGUE = 0x135,
  SITE_DRAIN = 0x136,
  SITE_SMEM_ALIGN = 0x137,
};

struct Params {
  int B, S, Hq, Hkv, kv_begin, kv_count, n_qblocks, n_units;
  int flags;
  float scale_log2;
  const uint16_t* cos;  // [>= S][128] bf16
  const uint16_t* sin;
  long long* trace;  // diagnostic clock64 trace of one CTA (nullptr = off)
  int trace_block;
};

constexpr int kTraceIters = 128;
constexpr int kTraceEv = 8;
#define P8_TRACE(role, it, ev)                                                                             \
  do {                                                                                                     \
    if (kTrace && tr) tr[((role) * kTraceIters + min(static_cast<int>(it), kTraceIters - 1)) * kTraceEv + (ev)] = clock64(); \
  } while (0)

struct Unit {
  int p0, n_kv, zq, zk;
};

__device__ __forceinline__ uint32_t colS(int t) { return static_cast<uint32_t>(t * 128); }
__device__ __forceinline__ uint32_t colO(int t) { return static_cast<uint32_t>(256 + t * 128); }

// The 16 rows x 128 keys of S this warp reads (16x256b: rows ra, ra + 8, keys 8k + 2t0,
// 8k + 2t0 + 1), with keys past each row's causal limit set to -inf.
__device__ __forceinline__ void load_scores(uint32_t tS, bool ok, int rela, int relb, int t0, uint32_t (&s)[64]) {
  if (ok) {
    tc_fence_after();
    tmem_ld16x256_x16(tS, s);
    tmem_wait_ld_dep64(s);
  } else {
#pragma unroll
    for (int k = 0; k < 64; ++k) s[k] = 0xFF800000u;
  }
  if (rela < kBN - 1) {
#pragma unroll
    for (int k = 0; k < 16; ++k) {
      const int key = 8 * k + 2 * t0;
      if (key > rela) s[4 * k] = 0xFF800000u;
      if (key + 1 > rela) s[4 * k + 1] = 0xFF800000u;
      if (key > relb) s[4 * k + 2] = 0xFF800000u;
      if (key + 1 > relb) s[4 * k + 3] = 0xFF800000u;
    }
  }
}

// p = 2^(s * scale_log2 - m) for both rows, packed to bf16 pairs in 16x128b store order,
// and the row sums of the packed values.
__device__ __forceinline__ void exp_rows(const uint32_t (&s)[64], float sl2, float ma, float mb, bool emu,
                                         uint32_t (&pw)[32], float2& suma, float2& sumb) {
  const float2 sc2 = make_float2(sl2, sl2), na2 = make_float2(-ma, -ma), nb2 = make_float2(-mb, -mb);
#pragma unroll
  for (int k = 0; k < 16; ++k) {
    const float2 xa = __ffma2_rn(make_float2(__uint_as_float(s[4 * k]), __uint_as_float(s[4 * k + 1])), sc2, na2);
    const float2 xb = __ffma2_rn(make_float2(__uint_as_float(s[4 * k + 2]), __uint_as_float(s[4 * k + 3])), sc2, nb2);
    float2 ya, yb;
    if (kEmuMask != 0 && emu && (k & kEmuMask) == kEmuMask) {
      ya = exp2_poly2(xa);
      yb = exp2_poly2(xb);
    } else {
      ya = make_float2(ex2_approx(xa.x), ex2_approx(xa.y));
      yb = make_float2(ex2_approx(xb.x), ex2_approx(xb.y));
    }
    pw[2 * k] = pack_bf16x2(ya.x, ya.y);
    pw[2 * k + 1] = pack_bf16x2(yb.x, yb.y);
    add_bf16x2_to_f32(suma, pw[2 * k]);
    add_bf16x2_to_f32(sumb, pw[2 * k + 1]);
  }
}

template <bool kTrace>
__global__ void __launch_bounds__(kThreads, 1)
    prefill8_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                    const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmO,
                    const Params p) {
  extern __shared__ __align__(1024) uint8_t smem[];
  if (smem_u32(smem) & 1023u) {
    if (threadIdx.x == 0) record_error(SITE_SMEM_ALIGN);
    return;
  }
  const uint32_t sbase = smem_u32(smem);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  auto bar = [&](int i) -> uint32_t { return sbase + kOffBar + 8 * i; };

  const bool causal = (p.flags & GQA_FLAG_CAUSAL) != 0;
  const bool rope_q = (p.flags & GQA_FLAG_ROPE_Q) != 0;
  const bool rope_k = (p.flags & GQA_FLAG_ROPE_K) != 0;
  const int n_kv_all = (p.S + kBN - 1) / kBN;
  const int n_ctas = static_cast<int>(gridDim.x);
  const int n_rounds = (p.n_units + n_ctas - 1) / n_ctas;
  auto unit_of = [&](int i) -> int {  // snake order over the heaviest-first list; -1 if none
    const int c = (i & 1) ? n_ctas - 1 - static_cast<int>(blockIdx.x) : static_cast<int>(blockIdx.x);
    const int u = i * n_ctas + c;
    return u < p.n_units ? u : -1;
  };
  auto decode = [&](int u) -> Unit {
    const int per_qb = p.B * p.kv_count;
    const int qb = p.n_qblocks - 1 - u / per_qb;
    const int rem = u % per_qb;
    const int b = rem / p.kv_count;
    const int kvh = p.kv_begin + rem % p.kv_count;
    Unit x;
    x.p0 = qb * kPosPerCta;
    x.n_kv = causal ? min(n_kv_all, (x.p0 + kPosPerCta - 1) / kBN + 1) : n_kv_all;
    x.zq = b * p.Hq + kvh * kG;
    x.zk = b * p.Hkv + kvh;
    return x;
  };

  if (threadIdx.x == 0) {
    for (int t = 0; t < 2; ++t) {
      mbar_init(bar(B_QFULL + t), 1);
      mbar_init(bar(B_QREADY + t), kHandoffCount);
      mbar_init(bar(B_SFULL + t), 1);
      mbar_init(bar(B_PREADY + t), kHandoffCount);
      mbar_init(bar(B_PVDONE + t), 1);
      mbar_init(bar(B_OSTAGE + t), 1);
    }
    mbar_init(bar(B_QEMPTY), 1);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(bar(B_KVFULL + s), 1);
      mbar_init(bar(B_KVEMPTY + s), 1);
    }
    for (int k = 0; k < kKReadySlots; ++k) mbar_init(bar(B_KREADY + k), 64);
    mbar_init(bar(B_DRAIN), 1);
    fence_mbar_init();
  }
  if (warp == kWarpMma) {
    tmem_alloc(sbase + kOffTmemPtr, 512);
    tmem_relinquish();
  }
  if (warp == kWarpProducer && lane == 0) {
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
    tma_prefetch_desc(&tmO);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(smem + kOffTmemPtr);
  long long* tr = (kTrace && static_cast<int>(blockIdx.x) == p.trace_block) ? p.trace : nullptr;
  if (threadIdx.x == 0) P8_TRACE(5, 0, 0);

  if (warp == kWarpProducer) {
    // ------------------------------------------------------------ TMA producer
    regs_dec<kRegsHelper>();
    if (lane == 0) {
      bool ok = true;
      uint32_t L = 0;
      int uc = 0;
      for (int i = 0; ok && i < n_rounds; ++i) {
        const int u = unit_of(i);
        if (u < 0) continue;
        const Unit x = decode(u);
        if (uc > 0 && !(ok = mbar_wait(bar(B_QEMPTY), (uc - 1) & 1, SITE_PRODUCER))) break;
        for (int t = 0; t < 2; ++t) {
          const uint32_t dst = sbase + kOffQ + t * kTileBytes;
          mbar_expect_tx(bar(B_QFULL + t), kTileBytes);
          tma_load_3d(dst, &tmQ, bar(B_QFULL + t), 0, x.p0 + t * kRowsPerHead, x.zq);
          tma_load_3d(dst + kHalf, &tmQ, bar(B_QFULL + t), 64, x.p0 + t * kRowsPerHead, x.zq);
        }
        const int un = unit_of(i + 1);
        const int nloads = 2 * x.n_kv;
        for (int li = 0; li < nloads; ++li) {
          if (un >= 0 && li == max(0, nloads - 16)) {  // warm L2 with the next unit's Q
            const Unit y = decode(un);
            for (int t = 0; t < 2; ++t) {
              tma_prefetch_l2_3d(&tmQ, 0, y.p0 + t * kRowsPerHead, y.zq);
              tma_prefetch_l2_3d(&tmQ, 64, y.p0 + t * kRowsPerHead, y.zq);
            }
          }
          const int s = static_cast<int>(L % kStages);
          const uint32_t r = L / kStages;
          if (r > 0 && !(ok = mbar_wait(bar(B_KVEMPTY + s), (r - 1) & 1u, SITE_PRODUCER))) break;
          const bool is_v = (li == nloads - 1) || (li >= 2 && (li & 1) == 0);
          const int j = li == 0 ? 0 : (is_v ? (li == nloads - 1 ? x.n_kv - 1 : (li - 2) >> 1) : (li + 1) >> 1);
          const void* map = is_v ? static_cast<const void*>(&tmV) : static_cast<const void*>(&tmK);
          const uint32_t dst = sbase + kOffKV + s * kTileBytes;
          mbar_expect_tx(bar(B_KVFULL + s), kTileBytes);
          tma_load_3d(dst, map, bar(B_KVFULL + s), 0, j * kBN, x.zk);
          tma_load_3d(dst + kHalf, map, bar(B_KVFULL + s), 64, j * kBN, x.zk);
          ++L;
        }
        ++uc;
      }
      for (uint32_t i = L > static_cast<uint32_t>(kStages) ? L - kStages : 0u; i < L; ++i)
        mbar_wait_drain(bar(B_KVFULL + static_cast<int>(i % kStages)), (i / kStages) & 1u, SITE_DRAIN);
      if (uc > 0) {
        mbar_wait_drain(bar(B_QFULL + 0), (uc - 1) & 1, SITE_DRAIN);
        mbar_wait_drain(bar(B_QFULL + 1), (uc - 1) & 1, SITE_DRAIN);
      }
    }
    __syncwarp();
  } else if (warp == kWarpMma) {
    // ------------------------------------------------------------ MMA issuer
    regs_dec<kRegsHelper>();
    if (lane == 0) {
      constexpr uint32_t kIdQK = idesc_bf16_f32(128, kBN, false);
      constexpr uint32_t kIdPV = idesc_bf16_f32(128, kD, true);  // B (V) MN-major
      constexpr uint32_t kHi = sdesc_hi_sw128(1024);
      const uint32_t q_lo = sdesc_lo(sbase + kOffQ, 16);
      const uint32_t kv_lo = sdesc_lo(sbase + kOffKV, 16);
      const uint32_t v_lo = sdesc_lo(sbase + kOffKV, kHalf);
      constexpr uint32_t kTile16 = kTileBytes / 16;
      auto issue_qk = [&](int t, int s) {  // S_t = Q_t K^T
        const uint32_t a0 = q_lo + t * kTile16, b0 = kv_lo + s * kTile16;
        const uint32_t d = tmem + colS(t);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint32_t off = ((kk >> 2) * kHalf + (kk & 3) * 32) / 16;
          umma_ss_lohi(d, a0 + off, b0 + off, kHi, kIdQK, kk > 0 ? 1u : 0u);
        }
      };
      auto issue_pv = [&](int t, int s, uint32_t acc) {  // O_t (+)= P_t V, P_t in TMEM over S_t
        const uint32_t a = tmem + colS(t), b0 = v_lo + s * kTile16;
        const uint32_t d = tmem + colO(t);
        umma_ts_lohi(d, a, b0, kHi, kIdPV, acc);
#pragma unroll
        for (int kk = 1; kk < 8; ++kk) umma_ts_lohi(d, a + 8u * kk, b0 + kk * (2048 / 16), kHi, kIdPV, 1u);
      };
      bool ok = true;
      uint32_t L = 0, Gb = 0, Kb = 0;
      int uc = 0;
      for (int i = 0; ok && i < n_rounds; ++i) {
        const int u = unit_of(i);
        if (u < 0) continue;
        const int n = decode(u).n_kv;
        auto wait_k = [&](int j) -> bool {
          if (rope_k) {
            const uint32_t kk = Kb + j;
            return mbar_wait_spin(bar(B_KREADY + kk % kKReadySlots), (kk / kKReadySlots) & 1u, SITE_MMA);
          }
          const uint32_t ii = L + load_idx_k(j);
          return mbar_wait_spin(bar(B_KVFULL + ii % kStages), (ii / kStages) & 1u, SITE_MMA);
        };
        // A unit's first QK^T overwrites S_t, which the previous unit's last PV_t read as
        // P_t: both are issued by this thread, and the tensor core runs them in order.
        ok = mbar_wait_spin(bar(B_QREADY + 0), uc & 1, SITE_MMA) && mbar_wait_spin(bar(B_QREADY + 1), uc & 1, SITE_MMA) &&
             wait_k(0);
        if (!ok) break;
        {
          const int sk = static_cast<int>((L + load_idx_k(0)) % kStages);
          tc_fence_after();
          issue_qk(0, sk);
          umma_commit(bar(B_SFULL + 0));
          issue_qk(1, sk);
          umma_commit(bar(B_SFULL + 1));
          umma_commit(bar(B_KVEMPTY + sk));
          if (n == 1) umma_commit(bar(B_QEMPTY));
        }
        for (int j = 0; ok && j < n; ++j) {
          const uint32_t g = Gb + j;
          const uint32_t iv = L + load_idx_v(j, n);
          const int sv = static_cast<int>(iv % kStages);
          const int sk = static_cast<int>((L + load_idx_k(j + 1)) % kStages);  // used when j + 1 < n
          // tile 0: PV0(j), then QK0(j+1) over the same TMEM columns
          P8_TRACE(1, g, 0);
          ok = mbar_wait_spin(bar(B_KVFULL + sv), (iv / kStages) & 1u, SITE_MMA) &&
               mbar_wait_spin(bar(B_PREADY + 0), g & 1u, SITE_MMA);
          if (!ok) break;
          P8_TRACE(1, g, 1);
          tc_fence_after();
          issue_pv(0, sv, j > 0 ? 1u : 0u);
          umma_commit(bar(B_PVDONE + 0));
          if (j + 1 < n) {
            if (!(ok = wait_k(j + 1))) break;
            tc_fence_after();
            issue_qk(0, sk);
            umma_commit(bar(B_SFULL + 0));
          }
          P8_TRACE(1, g, 2);
          // tile 1: PV1(j), then QK1(j+1)
          if (!(ok = mbar_wait_spin(bar(B_PREADY + 1), g & 1u, SITE_MMA))) break;
          P8_TRACE(1, g, 3);
          tc_fence_after();
          issue_pv(1, sv, j > 0 ? 1u : 0u);
          umma_commit(bar(B_PVDONE + 1));
          umma_commit(bar(B_KVEMPTY + sv));
          if (j + 1 < n) {
            issue_qk(1, sk);
            umma_commit(bar(B_SFULL + 1));
            umma_commit(bar(B_KVEMPTY + sk));
            if (j + 1 == n - 1) umma_commit(bar(B_QEMPTY));
          }
          P8_TRACE(1, g, 4);
        }
        L += 2 * n;
        Gb += n;
        Kb += n;
        ++uc;
      }
      umma_commit(bar(B_DRAIN));
      mbar_wait_drain(bar(B_DRAIN), 0, SITE_DRAIN);
    }
    __syncwarp();
  } else if (warp >= kWarpRope0) {
    // ------------------------------------------------------------ RoPE of K tiles
    regs_dec<kRegsHelper>();
    const int tid = threadIdx.x - kWarpRope0 * 32;  // 0..63
    bool ok = true;
    uint32_t L = 0, Kb = 0;
    for (int i = 0; rope_k && i < n_rounds; ++i) {
      const int u = unit_of(i);
      if (u < 0) continue;
      const Unit x = decode(u);
      for (int j = 0; j < x.n_kv; ++j) {
        const uint32_t ii = L + load_idx_k(j);
        const int s = static_cast<int>(ii % kStages);
        if (ok) ok = mbar_wait(bar(B_KVFULL + s), (ii / kStages) & 1u, SITE_ROPEK);
        if (ok) {
          uint8_t* tile = smem + kOffKV + s * kTileBytes;
#pragma unroll 1
          for (int rr = tid; rr < kBN; rr += 64) {
            const int key = j * kBN + rr;
            if (key < p.S)
              rope_row_smem(tile, kHalf, rr, p.cos + static_cast<size_t>(key) * kD,
                            p.sin + static_cast<size_t>(key) * kD);
          }
        }
        fence_proxy_async_smem();
        mbar_arrive(bar(B_KREADY + (Kb + j) % kKReadySlots));
      }
      L += 2 * x.n_kv;
      Kb += x.n_kv;
    }
  } else {
    // ------------------------------------------------------------ softmax: 4 lanes per row
    regs_inc<kRegsSoftmax>();
    const int t = warp >> 3;                               // Q tile
    const int wt = warp & 7;                               // warp within the tile
    const int lb = 32 * (warp & 3) + 16 * ((wt >> 2) & 1);  // first TMEM lane of this warp's 16
    const int t0 = lane & 3, t1 = lane >> 2;
    const int ra = lb + t1;                                // rows ra and ra + 8 of the tile
    const uint32_t lane_bits = static_cast<uint32_t>(lb) << 16;
    const uint32_t tS = tmem + lane_bits + colS(t);
    const uint32_t tO = tmem + lane_bits + colO(t);
    const int tid = wt * 32 + lane;                        // 0..255 within the tile
    const float sl2 = p.scale_log2;
    bool ok = true;
    bool store_pending = false;  // this thread's TMA store of O may still read the staging tile
    uint32_t Gb = 0;
    int uc = 0;
    // Q tile t of unit y landed: rotate half a row (4 of the 8 chunk pairs), release it
    auto prepare_q = [&](const Unit& y, int parity) {
      if (ok) ok = __all_sync(0xffffffffu, mbar_wait(bar(B_QFULL + t), parity, SITE_SOFTMAX));
      const int row = tid & 127;
      const int pos = y.p0 + t * kRowsPerHead + (row & (kRowsPerHead - 1));
      if (ok && rope_q && pos < p.S)
        rope_row_smem_part(smem + kOffQ + t * kTileBytes, kHalf, row, p.cos + static_cast<size_t>(pos) * kD,
                           p.sin + static_cast<size_t>(pos) * kD, 4 * (tid >> 7));
      fence_proxy_async_smem();
      if (kWarpArrive) {
        __syncwarp();
        if (lane == 0) mbar_arrive(bar(B_QREADY + t));
      } else {
        mbar_arrive(bar(B_QREADY + t));
      }
    };
    {
      const int u0 = unit_of(0);
      if (u0 >= 0) prepare_q(decode(u0), 0);
    }
    for (int i = 0; i < n_rounds; ++i) {
      const int u = unit_of(i);
      if (u < 0) continue;
      const Unit x = decode(u);
      const int n_kv = x.n_kv;
      // row ra: position qa (row ra + 8 is position qa + 8 of the same head)
      const int qa = x.p0 + t * kRowsPerHead + (ra & (kRowsPerHead - 1));
      const int lima = causal ? min(qa, p.S - 1) : p.S - 1;
      const int limb = causal ? min(qa + 8, p.S - 1) : p.S - 1;
      int inext = i + 1;
      while (inext < n_rounds && unit_of(inext) < 0) ++inext;
      float m_a = -INFINITY, m_b = -INFINITY, l_a = 0.0f, l_b = 0.0f;  // this thread's part of l
      for (int j = 0; j < n_kv; ++j) {
        const uint32_t gi = Gb + j;
        if (j == n_kv - 1 && inext < n_rounds && rope_q) {  // the next unit's cos/sin row into L1
          const int pos = decode(unit_of(inext)).p0 + t * kRowsPerHead + ((tid & 127) & (kRowsPerHead - 1));
          if (pos < p.S) {
            prefetch_l1(p.cos + static_cast<size_t>(pos) * kD + 32 * (tid >> 7));
            prefetch_l1(p.sin + static_cast<size_t>(pos) * kD + 32 * (tid >> 7));
          }
        }
        if (ok) ok = __all_sync(0xffffffffu, mbar_wait(bar(B_SFULL + t), gi & 1u, SITE_SOFTMAX));
        if (lane == 0 && wt == 0) P8_TRACE(2 + t, gi, 0);
        const int rela = lima - j * kBN, relb = limb - j * kBN;  // keys > rel are masked
        const bool emu = kEmuMask != 0 && rela >= kBN - 1;       // the whole tile is visible to both rows
        // s[4k+0..1]: row ra keys 8k+2t0, 8k+2t0+1; s[4k+2..3]: row ra+8, same keys
        uint32_t s[64];
        load_scores(tS, ok, rela, relb, t0, s);
        if (lane == 0 && wt == 0) P8_TRACE(2 + t, gi, 4);
        uint32_t pw[32];  // 16x128b order: pw[2k] = row ra, P column 4k+t0; pw[2k+1] = row ra+8
        float2 suma = make_float2(0.f, 0.f), sumb = make_float2(0.f, 0.f);
        float alpha_a = 1.0f, alpha_b = 1.0f;
        {
          float mxa = -INFINITY, mxb = -INFINITY;
#pragma unroll
          for (int k = 0; k < 16; ++k) {
            mxa = fmax3(mxa, __uint_as_float(s[4 * k]), __uint_as_float(s[4 * k + 1]));
            mxb = fmax3(mxb, __uint_as_float(s[4 * k + 2]), __uint_as_float(s[4 * k + 3]));
          }
          // the row's 4 lanes are consecutive: combine their maxima
          mxa = fmaxf(mxa, __shfl_xor_sync(0xffffffffu, mxa, 1));
          mxb = fmaxf(mxb, __shfl_xor_sync(0xffffffffu, mxb, 1));
          mxa = fmaxf(mxa, __shfl_xor_sync(0xffffffffu, mxa, 2));
          mxb = fmaxf(mxb, __shfl_xor_sync(0xffffffffu, mxb, 2));
          if (lane == 0 && wt == 0) P8_TRACE(2 + t, gi, 1);
          const float mna = fmaxf(m_a, mxa * sl2), mnb = fmaxf(m_b, mxb * sl2);
          const bool needa = mna > m_a + kRescaleLog2, needb = mnb > m_b + kRescaleLog2;
          alpha_a = needa ? ex2_approx(m_a - mna) : 1.0f;
          alpha_b = needb ? ex2_approx(m_b - mnb) : 1.0f;
          if (needa) m_a = mna;
          if (needb) m_b = mnb;
          // O_t rescale (rows whose max rose): PV_t(j-1) completed before S_t(j) did
          if (ok && j > 0 && __any_sync(0xffffffffu, needa || needb)) {
#pragma unroll 1
            for (int c = 0; c < 4; ++c) {
              uint32_t o[16];
              tmem_ld16x256_x4(tO + 32 * c, o);
              tmem_wait_ld_dep16(o);
#pragma unroll
              for (int k = 0; k < 4; ++k) {
                o[4 * k] = __float_as_uint(__uint_as_float(o[4 * k]) * alpha_a);
                o[4 * k + 1] = __float_as_uint(__uint_as_float(o[4 * k + 1]) * alpha_a);
                o[4 * k + 2] = __float_as_uint(__uint_as_float(o[4 * k + 2]) * alpha_b);
                o[4 * k + 3] = __float_as_uint(__uint_as_float(o[4 * k + 3]) * alpha_b);
              }
              tmem_st16x256_x4(tO + 32 * c, o);
            }
          }
          exp_rows(s, sl2, m_a == -INFINITY ? 0.0f : m_a, m_b == -INFINITY ? 0.0f : m_b, emu, pw, suma, sumb);
        }
        if (ok) {
          tmem_st16x128_x16(tS, pw);  // P over the scores: P columns 4k + t0
          if (lane == 0 && wt == 0) P8_TRACE(2 + t, gi, 2);
          tmem_wait_st();
          tc_fence_before();
          if (kWarpArrive) {
            __syncwarp();
            if (lane == 0) mbar_arrive(bar(B_PREADY + t));
          } else {
            mbar_arrive(bar(B_PREADY + t));
          }
          if (lane == 0 && wt == 0) P8_TRACE(2 + t, gi, 3);
        }
        l_a = l_a * alpha_a + (suma.x + suma.y);
        l_b = l_b * alpha_b + (sumb.x + sumb.y);
      }
      // The next unit's Q was loaded once this unit's last QK^T finished: rotate and
      // release it now, so its first QK^T overlaps this unit's epilogue.
      if (inext < n_rounds) prepare_q(decode(unit_of(inext)), (uc + 1) & 1);

      // ---- epilogue: O / l -> bf16 -> staging tile (the tiles take turns) -> TMA store
      l_a += __shfl_xor_sync(0xffffffffu, l_a, 1);
      l_b += __shfl_xor_sync(0xffffffffu, l_b, 1);
      l_a += __shfl_xor_sync(0xffffffffu, l_a, 2);
      l_b += __shfl_xor_sync(0xffffffffu, l_b, 2);
      const uint32_t last = Gb + n_kv - 1;
      if (ok) ok = __all_sync(0xffffffffu, mbar_wait(bar(B_PVDONE + t), last & 1u, SITE_EPILOGUE));
      // staging free for this tile: tile 0 after tile 1's previous store, tile 1 after tile 0's
      if (t == 0 && uc > 0 && ok) ok = __all_sync(0xffffffffu, mbar_wait(bar(B_OSTAGE + 0), (uc - 1) & 1, SITE_EPILOGUE));
      if (t == 1 && ok) ok = __all_sync(0xffffffffu, mbar_wait(bar(B_OSTAGE + 1), uc & 1, SITE_EPILOGUE));
      uint8_t* stg = smem + kOffStage;
      if (ok) {
        tc_fence_after();
        const float ia = l_a > 0.0f ? 1.0f / l_a : 0.0f, ib = l_b > 0.0f ? 1.0f / l_b : 0.0f;
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {  // dims 32c .. 32c+31
          uint32_t o[16];
          tmem_ld16x256_x4(tO + 32 * c, o);
          tmem_wait_ld_dep16(o);
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const int d = 32 * c + 8 * k + 2 * t0;  // dims d, d+1 of rows ra and ra+8
            const int off = (d & 7) * 2;
            *reinterpret_cast<uint32_t*>(stg + sw128_chunk(ra, d >> 3) + off) =
                pack_bf16x2(__uint_as_float(o[4 * k]) * ia, __uint_as_float(o[4 * k + 1]) * ia);
            *reinterpret_cast<uint32_t*>(stg + sw128_chunk(ra + 8, d >> 3) + off) =
                pack_bf16x2(__uint_as_float(o[4 * k + 2]) * ib, __uint_as_float(o[4 * k + 3]) * ib);
          }
        }
        tc_fence_before();  // O_t may be overwritten by the next unit's first PV
      }
      fence_proxy_async_smem();
      named_bar_sync(1 + t, kTileThreads);
      const int p0 = x.p0 + t * kRowsPerHead;
      if (tid == 0) {
        if (ok && p0 < p.S) {
          tma_store_3d(&tmO, sbase + kOffStage, 0, p0, x.zq);
          tma_store_3d(&tmO, sbase + kOffStage + kHalf, 64, p0, x.zq);
          bulk_commit();
          store_pending = true;
        }
        if (store_pending) bulk_wait_read0();  // the other tile may write the staging tile once it is read
        mbar_arrive(bar(B_OSTAGE + (1 - t)));
      }
      Gb += n_kv;
      ++uc;
    }
    if (tid == 0 && store_pending) bulk_wait0();
  }

  // ---- teardown
  tc_fence_before();
  named_bar_sync(5, kThreads);
  if (warp == kWarpMma) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace prefill8

int launch_prefill8(const void* q, const void* k, const void* v, void* o, const void* cos, const void* sin, int B,
                    int S, int Hq, int Hkv, int kv_begin, int kv_count, float scale, int flags, cudaStream_t stream,
                    long long* trace, int trace_block) {
  using namespace prefill8;
  const long long n_qblocks = (S + kPosPerCta - 1) / kPosPerCta;
  const long long n_units = n_qblocks * B * kv_count;
  if (n_units > 0x7FFFFFFFLL || static_cast<long long>(B) * Hq > 0x7FFFFFFFLL) return GQA_ERR_UNSUPPORTED;
  CUtensorMap tmQ, tmK, tmV, tmO;
  int rc;
  if ((rc = make_tmap_3d_bf16(&tmQ, q, kD, S, static_cast<long long>(B) * Hq, 64, kRowsPerHead, kG)) != GQA_OK)
    return rc;
  if ((rc = make_tmap_3d_bf16(&tmK, k, kD, S, static_cast<long long>(B) * Hkv, 64, kBN, 1)) != GQA_OK) return rc;
  if ((rc = make_tmap_3d_bf16(&tmV, v, kD, S, static_cast<long long>(B) * Hkv, 64, kBN, 1)) != GQA_OK) return rc;
  if ((rc = make_tmap_3d_bf16(&tmO, o, kD, S, static_cast<long long>(B) * Hq, 64, kRowsPerHead, kG)) != GQA_OK)
    return rc;
  static std::atomic<uint64_t> attr_done{0}, attr_done_tr{0};
  if ((rc = ensure_smem_attr(prefill8_kernel<false>, kSmemBytes, attr_done)) != GQA_OK) return rc;
  if (trace && (rc = ensure_smem_attr(prefill8_kernel<true>, kSmemBytes, attr_done_tr)) != GQA_OK) return rc;
  static std::atomic<int> regs_ok{0};
  if (regs_ok.load(std::memory_order_acquire) == 0) {
    cudaFuncAttributes fa, fb;
    if (cudaFuncGetAttributes(&fa, prefill8_kernel<false>) != cudaSuccess ||
        cudaFuncGetAttributes(&fb, prefill8_kernel<true>) != cudaSuccess)
      return GQA_ERR_CUDA;
    regs_ok.store(fa.numRegs == kRegsLaunch && fb.numRegs == kRegsLaunch ? 1 : -1, std::memory_order_release);
  }
  if (regs_ok.load(std::memory_order_acquire) < 0) return GQA_ERR_UNSUPPORTED;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  Params p;
  p.B = B;
  p.S = S;
  p.Hq = Hq;
  p.Hkv = Hkv;
  p.kv_begin = kv_begin;
  p.kv_count = kv_count;
  p.n_qblocks = static_cast<int>(n_qblocks);
  p.n_units = static_cast<int>(n_units);
  p.flags = flags;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.cos = static_cast<const uint16_t*>(cos);
  p.sin = static_cast<const uint16_t*>(sin);
  p.trace = trace;
  p.trace_block = trace_block;
  const int grid = static_cast<int>(n_units < sms ? n_units : sms);
  if (trace)
    prefill8_kernel<true><<<grid, kThreads, kSmemBytes, stream>>>(tmQ, tmK, tmV, tmO, p);
  else
    prefill8_kernel<false><<<grid, kThreads, kSmemBytes, stream>>>(tmQ, tmK, tmV, tmO, p);
  return cudaGetLastError() == cudaSuccess ? GQA_OK : GQA_ERR_CUDA;
}

GQA_ERROR_FLAG_ACCESSOR(error_flag_prefill8)

}  // namespace gqa
