// prefill7_sm100.cu -- fused causal GQA prefill with one softmax thread per row.
//
// Same computation and interface as prefill_sm100.cu (the golden's RoPE -> QK^T/sqrt(d)
// -> causal mask -> softmax -> PV -> bf16, llama3_attention_golden_model.py:162-190),
// organised so that no thread waits on another for a row statistic:
//
//   * each Q tile (128 rows = 4 heads x 32 positions) has one softmax warpgroup; thread r
//     owns row r (TMEM lane r) and reads all 128 scores of its row from TMEM, so the row
//     max and sum never cross threads;
//   * p (bf16) is written back into TMEM over the row's scores, and O_t += P_t V runs
//     with P_t as the TMEM operand (tcgen05.mma A from tensor memory) and V from shared
//     memory: no shared-memory traffic for P;
//   * the tensor core alternates the two tiles -- PV0(j) QK0(j+1) PV1(j) QK1(j+1) -- so
//     each tile's softmax for K tile j+1 runs while the other tile's PV and QK^T execute;
//   * the shared memory freed from P holds a 4-stage K/V ring and one O staging tile.
//
// Work units, unit order, Q prefetch / rotation between units and the epilogue follow
// prefill_sm100.cu.  Warps: 0-3 softmax tile 0, 4-7 softmax tile 1, 8 TMA producer,
// 9 MMA issuer (+ TMEM allocator), 10-11 RoPE of K tiles (FLAG_ROPE_K).
// TMEM (512 columns): S0 [0,128) (P0 over [0,64)), S1 [128,256), O0 [256,384), O1 [384,512).
#include <cuda.h>

#include "attn_common.cuh"
#include "common.cuh"
#include "gqa_internal.h"

namespace gqa {
namespace prefill7 {

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
constexpr int kWarpProducer = 8;
constexpr int kWarpMma = 9;
constexpr int kWarpRope0 = 10;
constexpr int kThreads = 384;
// Register split (setmaxnreg): launch kRegsLaunch per thread; the helper warpgroup
// (warps 8-11) drops to kRegsHelper, the two softmax warpgroups rise to kRegsSoftmax.
// The host checks the compiled launch count before every launch (an over-budget
// setmaxnreg.inc would never complete).
constexpr int kRegsLaunch = 168;
constexpr int kRegsHelper = 88;
constexpr int kRegsSoftmax = 208;
static_assert(2 * 128 * kRegsSoftmax + 128 * kRegsHelper <= kThreads * kRegsLaunch, "register split over budget");

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
  B_QREADY = 2,    // [2]  Q tile t rotated (128 arrivals)
  B_QEMPTY = 4,    // [1]  the unit's last QK^T done: Q tiles may be reloaded
  B_KVFULL = 5,    // [4]  TMA K/V stage landed
  B_KVEMPTY = 9,   // [4]  MMAs reading the stage completed
  B_KREADY = 13,   // [4]  K tile rotated (slot k % 4), 64 arrivals
  B_SFULL = 17,    // [2]  S_t = Q_t K^T complete (and so every earlier MMA of the CTA)
  B_PREADY = 19,   // [2]  P_t written into TMEM, O_t rescaled (128 arrivals)
  B_PVDONE = 21,   // [2]  O_t += P_t V complete
  B_OSTAGE = 23,   // [2]  the O staging tile is free for tile t
  B_DRAIN = 25,    // [1]  every MMA of the CTA complete
};
constexpr int kKReadySlots = 4;

enum : int {  // error sites
  SITE_PRODUCER = 0x121,
  SITE_MMA = 0x122,
  SITE_SOFTMAX = 0x123,
  SITE_ROPEK = 0x124,
  SITE_EPILOGUE = 0x125,
  SITE_DRAIN = 0x126,
  SITE_SMEM_ALIGN = 0x127,
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
#define P7_TRACE(role, it, ev)                                                                             \
  do {                                                                                                     \
    if (kTrace && tr) tr[((role) * kTraceIters + min(static_cast<int>(it), kTraceIters - 1)) * kTraceEv + (ev)] = clock64(); \
  } while (0)

struct Unit {
  int p0, n_kv, zq, zk;
};

__device__ __forceinline__ uint32_t colS(int t) { return static_cast<uint32_t>(t * 128); }
__device__ __forceinline__ uint32_t colO(int t) { return static_cast<uint32_t>(256 + t * 128); }

// 32 scores (one 32-key chunk of the row) -> 16 packed bf16 pairs of p = 2^(s*sl2 - m),
// acc += the bf16-rounded p.  With kEmulate a quarter of the pairs run on the FMA pipe.
template <bool kEmulate>
__device__ __forceinline__ void exp_chunk(const uint32_t (&s)[32], uint32_t (&w)[16], float2 sc2, float2 nm2,
                                          float2& acc) {
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const float2 x = __ffma2_rn(make_float2(__uint_as_float(s[2 * i]), __uint_as_float(s[2 * i + 1])), sc2, nm2);
    float2 y;
    if (kEmulate && (i & 3) == 3) {
      y = exp2_poly2(x);
    } else {
      y.x = ex2_approx(x.x);
      y.y = ex2_approx(x.y);
    }
    w[i] = pack_bf16x2(y.x, y.y);
    add_bf16x2_to_f32(acc, w[i]);
  }
}

template <bool kTrace>
__global__ void __launch_bounds__(kThreads, 1)
    prefill7_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
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
      mbar_init(bar(B_QREADY + t), 128);
      mbar_init(bar(B_SFULL + t), 1);
      mbar_init(bar(B_PREADY + t), 128);
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
  if (threadIdx.x == 0) P7_TRACE(5, 0, 0);

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
          P7_TRACE(1, g, 0);
          ok = mbar_wait_spin(bar(B_KVFULL + sv), (iv / kStages) & 1u, SITE_MMA) &&
               mbar_wait_spin(bar(B_PREADY + 0), g & 1u, SITE_MMA);
          if (!ok) break;
          P7_TRACE(1, g, 1);
          tc_fence_after();
          issue_pv(0, sv, j > 0 ? 1u : 0u);
          umma_commit(bar(B_PVDONE + 0));
          if (j + 1 < n) {
            if (!(ok = wait_k(j + 1))) break;
            tc_fence_after();
            issue_qk(0, sk);
            umma_commit(bar(B_SFULL + 0));
          }
          P7_TRACE(1, g, 2);
          // tile 1: PV1(j), then QK1(j+1)
          if (!(ok = mbar_wait_spin(bar(B_PREADY + 1), g & 1u, SITE_MMA))) break;
          P7_TRACE(1, g, 3);
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
          P7_TRACE(1, g, 4);
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
    // ------------------------------------------------------------ softmax: thread = row
    regs_inc<kRegsSoftmax>();
    const int t = warp >> 2;           // Q tile
    const int r = threadIdx.x & 127;   // row in tile == TMEM lane
    const uint32_t lane_off = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const uint32_t tS = tmem + lane_off + colS(t);
    const uint32_t tO = tmem + lane_off + colO(t);
    const float sl2 = p.scale_log2;
    bool ok = true;
    bool store_pending = false;  // this thread's TMA store of O may still read the staging tile
    uint32_t Gb = 0;
    int uc = 0;
    auto prepare_q = [&](const Unit& y, int parity) {  // rotate row r of Q tile t, release it
      if (ok) ok = __all_sync(0xffffffffu, mbar_wait(bar(B_QFULL + t), parity, SITE_SOFTMAX));
      const int pos = y.p0 + t * kRowsPerHead + (r & (kRowsPerHead - 1));
      if (ok && rope_q && pos < p.S)
        rope_row_smem(smem + kOffQ + t * kTileBytes, kHalf, r, p.cos + static_cast<size_t>(pos) * kD,
                      p.sin + static_cast<size_t>(pos) * kD);
      fence_proxy_async_smem();
      mbar_arrive(bar(B_QREADY + t));
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
      const int qpos = x.p0 + t * kRowsPerHead + (r & (kRowsPerHead - 1));
      const int lim = causal ? min(qpos, p.S - 1) : p.S - 1;  // last key this row attends
      int inext = i + 1;
      while (inext < n_rounds && unit_of(inext) < 0) ++inext;
      float m_run = -INFINITY, l_run = 0.0f;
      for (int j = 0; j < n_kv; ++j) {
        const uint32_t gi = Gb + j;
        if (j == n_kv - 1 && inext < n_rounds && rope_q) {  // the next unit's cos/sin rows into L1
          const int pos = decode(unit_of(inext)).p0 + t * kRowsPerHead + (r & (kRowsPerHead - 1));
          if (pos < p.S) {
            prefetch_l1(p.cos + static_cast<size_t>(pos) * kD);
            prefetch_l1(p.cos + static_cast<size_t>(pos) * kD + 64);
            prefetch_l1(p.sin + static_cast<size_t>(pos) * kD);
            prefetch_l1(p.sin + static_cast<size_t>(pos) * kD + 64);
          }
        }
        if (ok) ok = __all_sync(0xffffffffu, mbar_wait(bar(B_SFULL + t), gi & 1u, SITE_SOFTMAX));
        if (r == 0) P7_TRACE(2 + t, gi, 0);
        uint32_t s[4][32];
        if (ok) {
          tc_fence_after();
          tmem_ld32(tS + 0, s[0]);
          tmem_ld32(tS + 32, s[1]);
          tmem_ld32(tS + 64, s[2]);
          tmem_ld32(tS + 96, s[3]);
          tmem_wait_ld_dep(s[0]);
          reg_dep(s[1]);
          reg_dep(s[2]);
          reg_dep(s[3]);
        } else {
#pragma unroll
          for (int c = 0; c < 4; ++c)
#pragma unroll
            for (int k = 0; k < 32; ++k) s[c][k] = 0xFF800000u;
        }
        const int rel = lim - j * kBN;  // keys > rel are masked
        if (rel < kBN - 1) {
#pragma unroll
          for (int c = 0; c < 4; ++c)
#pragma unroll
            for (int k = 0; k < 32; ++k)
              if (32 * c + k > rel) s[c][k] = 0xFF800000u;
        }
        float mx[4];
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          mx[c] = -INFINITY;
#pragma unroll
          for (int k = 0; k < 32; k += 2) mx[c] = fmax3(mx[c], __uint_as_float(s[c][k]), __uint_as_float(s[c][k + 1]));
        }
        const float m_tile = fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])) * sl2;
        if (r == 0) P7_TRACE(2 + t, gi, 1);
        const float m_new = fmaxf(m_run, m_tile);
        const bool need = m_new > m_run + kRescaleLog2;
        const float m_use = need ? m_new : m_run;
        const float alpha = need ? ex2_approx(m_run - m_new) : 1.0f;
        const float moff = (m_use == -INFINITY) ? 0.0f : m_use;
        // O_t rescale: PV_t(j-1) completed before S_t(j) (issued after it, in order)
        if (ok && j > 0 && __any_sync(0xffffffffu, need)) {
#pragma unroll 1
          for (int c = 0; c < 4; ++c) {
            uint32_t o[32];
            tmem_ld32(tO + 32 * c, o);
            tmem_wait_ld_dep(o);
#pragma unroll
            for (int k = 0; k < 32; ++k) o[k] = __float_as_uint(__uint_as_float(o[k]) * alpha);
            tmem_st32(tO + 32 * c, o);
          }
        }
        float2 sum = make_float2(0.f, 0.f);
        if (ok) {
          const float2 sc2 = make_float2(sl2, sl2), nm2 = make_float2(-moff, -moff);
          float2 part[4];
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            uint32_t w[16];
            part[c] = make_float2(0.f, 0.f);  // one accumulator per chunk: short add chains
            // chunks with no masked key evaluate a quarter of the exponentials on the FMA pipe
            if (32 * c + 31 <= rel)
              exp_chunk<true>(s[c], w, sc2, nm2, part[c]);
            else
              exp_chunk<false>(s[c], w, sc2, nm2, part[c]);
            tmem_st16(tS + 16 * c, w);  // P over this row's scores: keys 32c..32c+31
          }
          sum = __fadd2_rn(__fadd2_rn(part[0], part[1]), __fadd2_rn(part[2], part[3]));
          if (r == 0) P7_TRACE(2 + t, gi, 2);
          tmem_wait_st();
          tc_fence_before();
          mbar_arrive(bar(B_PREADY + t));
          if (r == 0) P7_TRACE(2 + t, gi, 3);
        }
        l_run = l_run * alpha + (sum.x + sum.y);
        m_run = m_use;
      }
      // The next unit's Q was loaded once this unit's last QK^T finished: rotate and
      // release it now, so its first QK^T overlaps this unit's epilogue.
      if (inext < n_rounds) prepare_q(decode(unit_of(inext)), (uc + 1) & 1);

      // ---- epilogue: O / l -> bf16 -> staging tile (the tiles take turns) -> TMA store
      const uint32_t last = Gb + n_kv - 1;
      if (ok) ok = __all_sync(0xffffffffu, mbar_wait(bar(B_PVDONE + t), last & 1u, SITE_EPILOGUE));
      // staging free for this tile: tile 0 after tile 1's previous store, tile 1 after tile 0's
      if (t == 0 && uc > 0 && ok) ok = __all_sync(0xffffffffu, mbar_wait(bar(B_OSTAGE + 0), (uc - 1) & 1, SITE_EPILOGUE));
      if (t == 1 && ok) ok = __all_sync(0xffffffffu, mbar_wait(bar(B_OSTAGE + 1), uc & 1, SITE_EPILOGUE));
      uint8_t* stg = smem + kOffStage;
      if (ok) {
        tc_fence_after();
        const float inv_l = l_run > 0.0f ? 1.0f / l_run : 0.0f;
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          uint32_t o[32];
          tmem_ld32(tO + 32 * c, o);
          tmem_wait_ld_dep(o);
#pragma unroll
          for (int q = 0; q < 4; ++q) {  // 8 dims per 16-byte chunk
            uint4 v;
            v.x = pack_bf16x2(__uint_as_float(o[q * 8 + 0]) * inv_l, __uint_as_float(o[q * 8 + 1]) * inv_l);
            v.y = pack_bf16x2(__uint_as_float(o[q * 8 + 2]) * inv_l, __uint_as_float(o[q * 8 + 3]) * inv_l);
            v.z = pack_bf16x2(__uint_as_float(o[q * 8 + 4]) * inv_l, __uint_as_float(o[q * 8 + 5]) * inv_l);
            v.w = pack_bf16x2(__uint_as_float(o[q * 8 + 6]) * inv_l, __uint_as_float(o[q * 8 + 7]) * inv_l);
            *reinterpret_cast<uint4*>(stg + sw128_chunk(r, 4 * c + q)) = v;
          }
        }
        tc_fence_before();  // O_t may be overwritten by the next unit's first PV
      }
      fence_proxy_async_smem();
      named_bar_sync(1 + t, 128);
      const int p0 = x.p0 + t * kRowsPerHead;
      if (r == 0) {
        if (ok && p0 < p.S) {
          tma_store_3d(&tmO, sbase + kOffStage, 0, p0, x.zq);
          tma_store_3d(&tmO, sbase + kOffStage + kHalf, 64, p0, x.zq);
          bulk_commit();
          store_pending = true;
        }
        if (store_pending) {  // the other tile may write the staging tile once it is read
          bulk_wait_read0();
        }
        mbar_arrive(bar(B_OSTAGE + (1 - t)));
      }
      Gb += n_kv;
      ++uc;
    }
    if (r == 0 && store_pending) bulk_wait0();
  }

  // ---- teardown
  tc_fence_before();
  named_bar_sync(5, kThreads);
  if (warp == kWarpMma) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace prefill7

int launch_prefill7(const void* q, const void* k, const void* v, void* o, const void* cos, const void* sin, int B,
                    int S, int Hq, int Hkv, int kv_begin, int kv_count, float scale, int flags, cudaStream_t stream,
                    long long* trace, int trace_block) {
  using namespace prefill7;
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
  if ((rc = ensure_smem_attr(prefill7_kernel<false>, kSmemBytes, attr_done)) != GQA_OK) return rc;
  if (trace && (rc = ensure_smem_attr(prefill7_kernel<true>, kSmemBytes, attr_done_tr)) != GQA_OK) return rc;
  static std::atomic<int> regs_ok{0};
  if (regs_ok.load(std::memory_order_acquire) == 0) {
    cudaFuncAttributes fa, fb;
    if (cudaFuncGetAttributes(&fa, prefill7_kernel<false>) != cudaSuccess ||
        cudaFuncGetAttributes(&fb, prefill7_kernel<true>) != cudaSuccess)
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
    prefill7_kernel<true><<<grid, kThreads, kSmemBytes, stream>>>(tmQ, tmK, tmV, tmO, p);
  else
    prefill7_kernel<false><<<grid, kThreads, kSmemBytes, stream>>>(tmQ, tmK, tmV, tmO, p);
  return cudaGetLastError() == cudaSuccess ? GQA_OK : GQA_ERR_CUDA;
}

GQA_ERROR_FLAG_ACCESSOR(error_flag_prefill7)

}  // namespace gqa
