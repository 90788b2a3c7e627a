// prefill_sm100.cu -- fused causal GQA prefill on the sm_100a tensor core.
//
// Computes, per query head h (kv head h/4) and position i,
//   O[h,i,:] = softmax_j( (rope(q)[h,i] . rope(k)[h/4,j]) * scale , j <= i ) . V[h/4,:,:]
// i.e. stages RoPE -> QK^T/sqrt(d) -> causal mask -> softmax -> PV -> bf16 of the
// reference's golden model (llama3_attention_golden_model.py:162-190) and the fp32
// core of CPU_Baseline (CPU_Baseline/cpu_baseline/attention.py:60-84), without
// materialising the S x S score matrix.
//
// Work unit: batch b, kv head g, a block of 64 query positions, held as two 128-row
// Q tiles; each tile packs the 4 query heads of group g x 32 positions (row r =
// head_in_group*32 + position_offset), so one K/V tile in shared memory serves all 4
// heads of the group (GQA by address, no KV duplication).
//
// Persistent CTAs (one per SM) walk the units heaviest-first (causal: most K tiles
// first; in bands of 16 query blocks that keep the CTAs reading one K/V head together
// when many (sequence, kv head) pairs share a round) in snake order over the rounds, so
// each SM gets a balanced share.  Nothing
// drains between units: the K/V ring and every barrier phase run on across them, the
// next unit's Q is prefetched into L2 and loaded as soon as the last QK^T of the
// current unit is done, the softmax threads rotate it before the current unit's
// epilogue, and its first QK^T overlaps that epilogue (O is normalised from TMEM into
// the tile's P buffer and written out by TMA).
//
// Pipeline: each softmax thread copies its row of S_t (128 keys) from TMEM into
// registers and releases S_t at once, so the tensor core computes S_t for the next
// K tile while the softmax works; P_t (bf16) goes to shared memory and O_t += P_t V
// runs with both operands in shared memory.  Softmax and both GEMMs overlap.
//
// Warp roles (20 warps):
//   warps 0-15 four softmax warpgroups; warpgroup g serves Q tile g/2 and key/dim half
//              g%2 (thread r owns TMEM lane / row r; the two halves of a row exchange
//              their partial row max through shared memory)
//   warp 16    TMA producer (Q tiles of each unit, then K0 K1 V0 K2 V1 ... into a
//              3-stage ring)
//   warps 17-18 tcgen05.mma issuers, one per Q tile (lane 0 issues QK_t and PV_t);
//              warp 17 also allocates TMEM.  A single thread can start a 128x128x16
//              MMA only every ~85-90 cycles against 64 cycles of tensor work (measured
//              on B200), so one issuer would cap the tensor pipe near 70 %; two issue
//              streams interleave and keep it fed.
//   warp 19    RoPE of K tiles in shared memory (FLAG_ROPE_K); Q tiles are rotated
//              by the softmax threads (FLAG_ROPE_Q), the next unit's before the
//              current unit's epilogue
// TMEM (512 columns x 128 lanes, fp32): S0 [0,128) S1 [128,256) O0 [256,384) O1 [384,512).
//
// Online softmax in the log2 domain: p = 2^(s*scale*log2e - m); the running max m is
// only raised (and O rescaled) when a tile's max exceeds it by more than kRescaleLog2,
// so p <= 2^16: with |v| < 2^16 and at most 2^17 keys, O stays below 2^49 (fp32-safe).
#include <cuda.h>

#include "attn_common.cuh"
#include "common.cuh"
#include "gqa_internal.h"

namespace gqa {
namespace prefill {

using namespace attn;

constexpr int kD = 128;
constexpr int kG = 4;
constexpr int kBM = 128;
constexpr int kRowsPerHead = kBM / kG;        // 32
constexpr int kPosPerCta = 2 * kRowsPerHead;  // 64
constexpr int kBN = 128;                      // keys per K/V tile
constexpr int kStages = 3;                    // K/V ring stages
constexpr int kBand = 16;                     // query blocks per band of the unit order (when banded)
constexpr int kTileBytes = 128 * 128 * 2;     // Q, P, K and V tiles: 32 KB
constexpr int kHalf = kTileBytes / 2;         // one 64-column swizzle block of 128 rows
constexpr int kSoftmaxThreads = 512;  // warps 0-15
constexpr float kRescaleLog2 = 16.0f;
constexpr int kWarpProducer = 16;
constexpr int kWarpMma = 17;   // issues the MMAs of Q tile 0
constexpr int kWarpMma1 = 18;  // issues the MMAs of Q tile 1
constexpr int kWarpRope0 = 19;
constexpr int kThreads = 640;
// Register split (setmaxnreg): the launch gives every thread kRegsLaunch registers; the
// helper warpgroup (warps 16-19) gives some back and the four softmax warpgroups take
// them.  The sum must stay within the launch allocation, or setmaxnreg.inc would wait
// forever; the host checks the compiled register count before every launch.
constexpr int kRegsLaunch = 96;
constexpr int kRegsHelper = 64;
constexpr int kRegsSoftmax = 104;
static_assert(4 * 128 * kRegsSoftmax + 128 * kRegsHelper <= kThreads * kRegsLaunch, "register split over budget");

// The 1024-byte-aligned tiles come first; the dynamic shared-memory base is
// 1024-byte aligned (checked at run time), so no alignment slack is allocated.
constexpr int kOffQ = 0;
constexpr int kOffP = kOffQ + 2 * kTileBytes;
constexpr int kOffKV = kOffP + 2 * kTileBytes;
constexpr int kOffBar = kOffKV + kStages * kTileBytes;
constexpr int kNumBars = 32;
constexpr int kOffX = kOffBar + kNumBars * 8;        // row-max / row-sum exchange [2 tiles][2 halves][128]
constexpr int kOffTmemPtr = kOffX + 2 * 2 * 128 * 4;
constexpr int kSmemBytes = kOffTmemPtr + 16;
static_assert(kSmemBytes <= 232448, "shared memory over the per-block limit");

enum : int {
  B_QFULL = 0,     // [2]  TMA Q tile t of the current unit landed
  B_QREADY = 2,    // [2]  Q tile t (rotated) visible to the tensor core, 256 arrivals
  B_QEMPTY = 4,    // [1]  last QK^T of both tiles complete (one arrival per issuer)
  B_KVFULL = 5,    // [3]  TMA K/V stage landed
  B_KVEMPTY = 8,   // [3]  MMAs reading the stage completed (one arrival per issuer)
  B_KREADY = 11,   // [4]  K tile rotated (slot k % 4), 32 arrivals
  B_SFULL = 15,    // [2]  S_t = Q_t K^T complete
  B_SFREE = 17,    // [2]  S_t copied to registers
  B_PREADY = 19,   // [2]  P_t in shared memory, O_t rescaled
  B_PVDONE = 21,   // [2]  O_t += P_t V complete (P_t buffer free)
  B_DRAIN = 23,    // [2]  every MMA of issuer t complete
};
constexpr int kHandoffThreads = kSoftmaxThreads / 2;  // per-tile hand-offs: one tile's 256 threads
// Exponentials of unmasked chunks partly on the FMA pipe (a cubic fit of 2^f, a quarter
// of the pairs): with the bf16-consistent row sums below the kernel is MUFU-bound enough
// for this to pay (about 10 % measured).
constexpr bool kEmulateExp = true;
__device__ __forceinline__ int sfree_bar(int t) { return B_SFREE + t; }
__device__ __forceinline__ int pready_bar(int t) { return B_PREADY + t; }
constexpr int kKReadySlots = 4;

enum : int {  // error sites reported through g_gqa_dev_error
  SITE_PRODUCER = 0x101,
  SITE_MMA = 0x102,
  SITE_SOFTMAX = 0x103,
  SITE_ROPEK = 0x104,
  SITE_EPILOGUE = 0x105,
  SITE_DRAIN = 0x106,
  SITE_SMEM_ALIGN = 0x107,
};

struct Params {
  int B, S, Hq, Hkv, kv_begin, kv_count, n_qblocks, n_units;
  int band;  // query blocks per band of the unit order: kBand or 1 (see launch_prefill)
  int flags;
  float scale_log2;
  const uint16_t* cos;  // [>= S][128] bf16 (cat(freqs, freqs) layout)
  const uint16_t* sin;
};

__device__ __forceinline__ uint32_t colS(int t) { return static_cast<uint32_t>(t * 128); }
__device__ __forceinline__ uint32_t colO(int t) { return static_cast<uint32_t>(256 + t * 128); }

// One 32-column chunk of S -> p = 2^(s*scale_log2 - m) as bf16, stored straight into
// the K-major SW128 P tile (row r, 16-byte chunks c0..c0+3); acc += the bf16-rounded p.
template <bool kEmulate>
__device__ __forceinline__ void exp_chunk_store(const uint32_t (&s)[32], uint8_t* ptile, int r, int c0, float2 sc2,
                                                float2 nm2, float2& acc) {
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    uint32_t w[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int i = 4 * c + e;
      const float2 x = __ffma2_rn(make_float2(__uint_as_float(s[2 * i]), __uint_as_float(s[2 * i + 1])), sc2, nm2);
      float2 y;
      if (kEmulate && e == 3) {
        y = exp2_poly2(x);
      } else {
        y.x = ex2_approx(x.x);
        y.y = ex2_approx(x.y);
      }
      w[e] = pack_bf16x2(y.x, y.y);
      // The row sum adds the bf16 values PV multiplies, so O / l is a weighted mean with
      // weights summing to exactly 1.  (Summing the unrounded fp32 p saves ~1 instruction
      // per score but lets the weights' rounding bias O by up to 2^-8 relative, which
      // exceeds the 1e-2 absolute tolerance for |O| near 2.)
      add_bf16x2_to_f32(acc, w[e]);
    }
    *reinterpret_cast<uint4*>(ptile + sw128_chunk(r, c0 + c)) = make_uint4(w[0], w[1], w[2], w[3]);
  }
}

struct Unit {
  int p0, n_kv, zq, zk;
};

__global__ void __launch_bounds__(kThreads, 1)
    prefill_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                   const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmO,
                   const Params p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  if (smem_u32(smem_raw) & 1023u) {  // uniform across the CTA: leave before any barrier
    if (threadIdx.x == 0) record_error(SITE_SMEM_ALIGN);
    return;
  }
  uint8_t* smem = smem_raw;
  const uint32_t sbase = smem_u32(smem);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  auto bar = [&](int i) -> uint32_t { return sbase + kOffBar + 8 * i; };
  // softmax hand-off: every thread arrives (one arrival per warp after __syncwarp
  // measured no faster)
  auto warp_arrive = [&](uint32_t b) { mbar_arrive(b); };

  const bool causal = (p.flags & GQA_FLAG_CAUSAL) != 0;
  const bool rope_q = (p.flags & GQA_FLAG_ROPE_Q) != 0;
  const bool rope_k = (p.flags & GQA_FLAG_ROPE_K) != 0;
  const int n_kv_all = (p.S + kBN - 1) / kBN;
  const int n_ctas = static_cast<int>(gridDim.x);
  const int n_rounds = (p.n_units + n_ctas - 1) / n_ctas;
  // Unit of round i for this CTA (snake order over the heaviest-first list), -1 if none.
  auto unit_of = [&](int i) -> int {
    const int c = (i & 1) ? n_ctas - 1 - static_cast<int>(blockIdx.x) : static_cast<int>(blockIdx.x);
    const int u = i * n_ctas + c;
    return u < p.n_units ? u : -1;
  };
  // Unit order: bands of p.band query blocks, heaviest band first; inside a band the blocks
  // of one (sequence, kv head) are consecutive.  With 32 (sequence, kv head) pairs a round
  // of 148 CTAs then streams the K/V of ~9 pairs, each read by ~16 CTAs at nearly the same
  // time, instead of 32 pairs read by ~4.6 CTAs each: more K/V tile loads hit in L2 (+2.8 %
  // measured at seq 8192, batch 4).  p.band = 1 is plain heaviest-first order.
  auto decode = [&](int u) -> Unit {
    const int per_qb = p.B * p.kv_count;
    const int band_units = p.band * per_qb;
    const int band = u / band_units;
    const int nb = min(p.band, p.n_qblocks - band * p.band);  // the last band may be partial
    const int rem = u - band * band_units;
    const int pair = rem / nb;
    const int qb = p.n_qblocks - 1 - (band * p.band + rem % nb);
    const int b = pair / p.kv_count;
    const int kvh = p.kv_begin + pair % p.kv_count;
    Unit x;
    x.p0 = qb * kPosPerCta;
    x.n_kv = causal ? min(n_kv_all, (x.p0 + kPosPerCta - 1) / kBN + 1) : n_kv_all;
    x.zq = b * p.Hq + kvh * kG;  // first Q/O head row of the group
    x.zk = b * p.Hkv + kvh;
    return x;
  };

  if (threadIdx.x == 0) {
    for (int t = 0; t < 2; ++t) {
      mbar_init(bar(B_QFULL + t), 1);
      mbar_init(bar(B_QREADY + t), 256);
      mbar_init(bar(B_SFULL + t), 1);
      mbar_init(bar(B_PVDONE + t), 1);
    }
    mbar_init(bar(B_QEMPTY), 2);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(bar(B_KVFULL + s), 1);
      mbar_init(bar(B_KVEMPTY + s), 2);
    }
    for (int k = 0; k < kKReadySlots; ++k) mbar_init(bar(B_KREADY + k), 32);
    for (int t = 0; t < 2; ++t) {
      mbar_init(bar(B_SFREE + t), kHandoffThreads);
      mbar_init(bar(B_PREADY + t), kHandoffThreads);
    }
    mbar_init(bar(B_DRAIN), 1);
    mbar_init(bar(B_DRAIN + 1), 1);
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

  if (warp == kWarpProducer) {
    // ------------------------------------------------------------ TMA producer
    regs_dec<kRegsHelper>();
    if (lane == 0) {
      bool ok = true;
      uint32_t L = 0;  // K/V loads issued by this CTA (ring position)
      int uc = 0;      // units started
      for (int i = 0; ok && i < n_rounds; ++i) {
        const int u = unit_of(i);
        if (u < 0) continue;
        const Unit x = decode(u);
        // The Q tiles are reused once the previous unit's last QK^T is done.
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
          // Warm L2 with the next unit's Q about eight K tiles before it is loaded (early
          // enough to hide HBM latency, late enough not to be evicted by the K/V stream).
          if (un >= 0 && li == max(0, nloads - 16)) {
            const Unit y = decode(un);
            for (int t = 0; t < 2; ++t) {
              tma_prefetch_l2_3d(&tmQ, 0, y.p0 + t * kRowsPerHead, y.zq);
              tma_prefetch_l2_3d(&tmQ, 64, y.p0 + t * kRowsPerHead, y.zq);
            }
          }
          const int s = static_cast<int>(L % kStages);
          const uint32_t r = L / kStages;
          if (r > 0 && !(ok = mbar_wait(bar(B_KVEMPTY + s), (r - 1) & 1u, SITE_PRODUCER))) break;
          // li -> (tile, K or V) in the K-ahead order
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
      // Drain: every load this thread issued must land before the CTA may exit.
      for (uint32_t i = L > static_cast<uint32_t>(kStages) ? L - kStages : 0u; i < L; ++i)
        mbar_wait_drain(bar(B_KVFULL + static_cast<int>(i % kStages)), (i / kStages) & 1u, SITE_DRAIN);
      if (uc > 0) {
        mbar_wait_drain(bar(B_QFULL + 0), (uc - 1) & 1, SITE_DRAIN);
        mbar_wait_drain(bar(B_QFULL + 1), (uc - 1) & 1, SITE_DRAIN);
      }
    }
    __syncwarp();
  } else if (warp == kWarpMma || warp == kWarpMma1) {
    // ------------------------------------------------------------ MMA issuers
    // One issuing thread can start a 128x128x16 tcgen05.mma only every ~85 cycles, a
    // third slower than the tensor core runs it, so each Q tile has its own issuer: warp
    // kWarpMma + t issues QK_t and PV_t, and the two streams interleave in the pipe.
    regs_dec<kRegsHelper>();
    const int tq = warp - kWarpMma;  // Q tile of this issuer
    if (lane == 0) {
      constexpr uint32_t kIdQK = idesc_bf16_f32(128, kBN, false);
      constexpr uint32_t kIdPV = idesc_bf16_f32(128, kD, true);
      constexpr uint32_t kHi = sdesc_hi_sw128(1024);
      const uint32_t q_lo = sdesc_lo(sbase + kOffQ + tq * kTileBytes, 16);
      const uint32_t p_lo = sdesc_lo(sbase + kOffP + tq * kTileBytes, 16);
      const uint32_t kv_lo = sdesc_lo(sbase + kOffKV, 16);
      const uint32_t v_lo = sdesc_lo(sbase + kOffKV, kHalf);
      constexpr uint32_t kTile16 = kTileBytes / 16;
      const uint32_t dS = tmem + colS(tq), dO = tmem + colO(tq);
      // S_t = Q_t K^T over d = 128 (8 k-steps of 16; both operands K-major SW128)
      auto issue_qk = [&](int s) {
        const uint32_t b0 = kv_lo + s * kTile16;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint32_t off = ((kk >> 2) * kHalf + (kk & 3) * 32) / 16;
          umma_ss_lohi(dS, q_lo + off, b0 + off, kHi, kIdQK, kk > 0 ? 1u : 0u);
        }
      };
      // O_t (+)= P_t V over 128 keys (8 k-steps; P K-major SW128, V MN-major SW128)
      auto issue_pv = [&](int s, uint32_t acc) {
        const uint32_t b0 = v_lo + s * kTile16;
        umma_ss_lohi(dO, p_lo, b0, kHi, kIdPV, acc);
#pragma unroll
        for (int kk = 1; kk < 8; ++kk) {
          const uint32_t off = ((kk >> 2) * kHalf + (kk & 3) * 32) / 16;
          umma_ss_lohi(dO, p_lo + off, b0 + kk * (2048 / 16), kHi, kIdPV, 1u);
        }
      };
      bool ok = true;
      uint32_t L = 0, Gb = 0, Kb = 0;  // ring position, global iteration, K tiles consumed
      int uc = 0;
      for (int i = 0; ok && i < n_rounds; ++i) {
        const int u = unit_of(i);
        if (u < 0) continue;
        const int n = decode(u).n_kv;
        auto wait_k = [&](int j) -> bool {  // K tile j of this unit landed (and rotated)
          if (rope_k) {
            const uint32_t kk = Kb + j;
            return mbar_wait_spin(bar(B_KREADY + kk % kKReadySlots), (kk / kKReadySlots) & 1u, SITE_MMA);
          }
          const uint32_t ii = L + load_idx_k(j);
          return mbar_wait_spin(bar(B_KVFULL + ii % kStages), (ii / kStages) & 1u, SITE_MMA);
        };
        // Q tile of this unit ready, and S_t released by the previous unit's softmax
        ok = mbar_wait_spin(bar(B_QREADY + tq), uc & 1, SITE_MMA) && wait_k(0) &&
             (Gb == 0 || mbar_wait_spin(bar(sfree_bar(tq)), (Gb - 1) & 1u, SITE_MMA));
        if (!ok) break;
        {
          const int sk = static_cast<int>((L + load_idx_k(0)) % kStages);
          tc_fence_after();
          issue_qk(sk);
          umma_commit(bar(B_SFULL + tq));
          umma_commit(bar(B_KVEMPTY + sk));
          if (n == 1) umma_commit(bar(B_QEMPTY));
        }
        for (int j = 0; ok && j < n; ++j) {
          const uint32_t g = Gb + j;
          const uint32_t iv = L + load_idx_v(j, n);
          const int sv = static_cast<int>(iv % kStages);
          if (j + 1 < n) {
            // next S as soon as this tile's softmax holds S(j) in registers
            const int sk = static_cast<int>((L + load_idx_k(j + 1)) % kStages);
            ok = wait_k(j + 1) && mbar_wait_spin(bar(sfree_bar(tq)), g & 1u, SITE_MMA);
            if (!ok) break;
            tc_fence_after();
            issue_qk(sk);
            umma_commit(bar(B_SFULL + tq));
            umma_commit(bar(B_KVEMPTY + sk));
            if (j + 1 == n - 1) umma_commit(bar(B_QEMPTY));
          }
          ok = mbar_wait_spin(bar(B_KVFULL + sv), (iv / kStages) & 1u, SITE_MMA) &&
               mbar_wait_spin(bar(pready_bar(tq)), g & 1u, SITE_MMA);
          if (!ok) break;
          tc_fence_after();
          issue_pv(sv, j > 0 ? 1u : 0u);
          umma_commit(bar(B_PVDONE + tq));
          umma_commit(bar(B_KVEMPTY + sv));
        }
        L += 2 * n;
        Gb += n;
        Kb += n;
        ++uc;
      }
      umma_commit(bar(B_DRAIN + tq));
      mbar_wait_drain(bar(B_DRAIN + tq), 0, SITE_DRAIN);
    }
    __syncwarp();
  } else if (warp >= kWarpRope0) {
    // ------------------------------------------------------------ RoPE helpers (K tiles)
    regs_dec<kRegsHelper>();
    const int tid = threadIdx.x - kWarpRope0 * 32;  // 0..31
    bool ok = true;
    uint32_t L = 0, Kb = 0;
    int uc = 0;
    for (int i = 0; rope_k && i < n_rounds; ++i) {
      const int u = unit_of(i);
      if (u < 0) continue;
      const Unit x = decode(u);
      if (rope_k) {
        for (int j = 0; j < x.n_kv; ++j) {
          const uint32_t ii = L + load_idx_k(j);
          const int s = static_cast<int>(ii % kStages);
          if (ok) ok = mbar_wait(bar(B_KVFULL + s), (ii / kStages) & 1u, SITE_ROPEK);
          if (ok) {
            uint8_t* tile = smem + kOffKV + s * kTileBytes;
#pragma unroll 1
            for (int rr = tid; rr < kBN; rr += 32) {
              const int key = j * kBN + rr;
              if (key < p.S)
                rope_row_smem(tile, kHalf, rr, p.cos + static_cast<size_t>(key) * kD,
                              p.sin + static_cast<size_t>(key) * kD);
            }
          }
          fence_proxy_async_smem();
          mbar_arrive(bar(B_KREADY + (Kb + j) % kKReadySlots));
        }
      }
      L += 2 * x.n_kv;
      Kb += x.n_kv;
      ++uc;
    }
  } else {
    // ------------------------------------------------------------ softmax warpgroups
    regs_inc<kRegsSoftmax>();
    const int g = warp >> 2;             // warpgroup 0..3
    const int t = g >> 1;                // Q tile
    const int h = g & 1;                 // keys [64h, 64h+64) of each K tile; O dims [64h, 64h+64)
    const int r = threadIdx.x & 127;     // row in tile == TMEM lane
    const uint32_t lane_off = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const uint32_t tS = tmem + lane_off + colS(t) + 64 * h;
    const uint32_t tO = tmem + lane_off + colO(t) + 64 * h;
    uint8_t* ptile = smem + kOffP + t * kTileBytes;
    float* xchg = reinterpret_cast<float*>(smem + kOffX) + t * 256;  // [half][row]
    const int bar_x = 1 + t;     // named barrier: both halves of tile t (256 threads)
    const int bar_free = 3 + t;  // named barrier: exchange slots may be rewritten
    const float sl2 = p.scale_log2;
    bool ok = true;
    bool store_pending = false;  // this thread's TMA store of O may still read P_t
    uint32_t Gb = 0;             // global iteration of this unit's first K tile
    int uc = 0;                  // units started
    // Q tile t of unit y landed: rotate this thread's half of row r in place (each half
    // rotates 4 of the row's 8 chunk pairs), then release it to the tensor core.
    auto prepare_q = [&](const Unit& y, int parity, int unit_no) {
      if (ok) ok = __all_sync(0xffffffffu, mbar_wait(bar(B_QFULL + t), parity, SITE_SOFTMAX));
      const int pos = y.p0 + t * kRowsPerHead + (r & (kRowsPerHead - 1));
      if (ok && rope_q && pos < p.S)
        rope_row_smem_part(smem + kOffQ + t * kTileBytes, kHalf, r, p.cos + static_cast<size_t>(pos) * kD,
                           p.sin + static_cast<size_t>(pos) * kD, 4 * h);
      fence_proxy_async_smem();
      warp_arrive(bar(B_QREADY + t));
    };
    {
      const int u0 = unit_of(0);
      if (u0 >= 0) prepare_q(decode(u0), 0, 0);
    }

    // Every warp of the tile runs every iteration of every unit and meets every named
    // barrier, even after a bounded wait failed (ok == false only skips the work), so
    // the two halves of a tile can never wait on each other forever.
    for (int i = 0; i < n_rounds; ++i) {
      const int u = unit_of(i);
      if (u < 0) continue;
      const Unit x = decode(u);
      const int n_kv = x.n_kv;
      const int qpos = x.p0 + t * kRowsPerHead + (r & (kRowsPerHead - 1));
      // last key this row may attend
      const int lim = causal ? min(qpos, p.S - 1) : p.S - 1;
      float m_run = -INFINITY, l_run = 0.0f;
      // the next unit, whose Q this thread rotates before this unit's epilogue
      int inext = i + 1;
      while (inext < n_rounds && unit_of(inext) < 0) ++inext;
      for (int j = 0; j < n_kv; ++j) {
        const uint32_t gi = Gb + j;
        if (j == n_kv - 1 && inext < n_rounds && rope_q) {
          // pull this row's cos/sin chunks of the next unit into L1 now, so the rotation
          // between the units does not wait on L2
          const int pos = decode(unit_of(inext)).p0 + t * kRowsPerHead + (r & (kRowsPerHead - 1));
          if (pos < p.S) {
            prefetch_l1(p.cos + static_cast<size_t>(pos) * kD + 32 * h);
            prefetch_l1(p.sin + static_cast<size_t>(pos) * kD + 32 * h);
          }
        }
        if (ok) ok = __all_sync(0xffffffffu, mbar_wait(bar(B_SFULL + t), gi & 1u, SITE_SOFTMAX));
        uint32_t s0[32], s1[32];
        if (ok) {
          tc_fence_after();
          tmem_ld32(tS + 0, s0);
          tmem_ld32(tS + 32, s1);
          tmem_wait_ld_dep(s0);
          reg_dep(s1);
          tc_fence_before();
          warp_arrive(bar(sfree_bar(t)));  // S_t may now be overwritten by the next QK^T
        } else {
#pragma unroll
          for (int k = 0; k < 32; ++k) s0[k] = s1[k] = 0xFF800000u;
        }

        const int rel = lim - j * kBN - 64 * h;  // columns (of this half) > rel are masked
        if (rel < 63) {
#pragma unroll
          for (int k = 0; k < 32; ++k) {
            if (k > rel) s0[k] = 0xFF800000u;
            if (k + 32 > rel) s1[k] = 0xFF800000u;
          }
        }
        float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
        for (int k = 0; k < 32; k += 2) {
          mx0 = fmax3(mx0, __uint_as_float(s0[k]), __uint_as_float(s0[k + 1]));
          mx1 = fmax3(mx1, __uint_as_float(s1[k]), __uint_as_float(s1[k + 1]));
        }
        // The previous unit's O went out through P_t: the tile writes P_t only after this
        // barrier, which the storing thread reaches once the stores have read it.
        if (store_pending) {
          bulk_wait_read0();
          store_pending = false;
        }
        // row max over both halves: slot [h][r] <-> [1-h][r]
        named_bar_sync(bar_free, 256);  // everyone has read the previous exchange's slots
        xchg[h * 128 + r] = fmaxf(mx0, mx1);
        named_bar_sync(bar_x, 256);
        const float m_tile = fmaxf(fmaxf(mx0, mx1), xchg[(1 - h) * 128 + r]) * sl2;
        const float m_new = fmaxf(m_run, m_tile);
        const bool need = m_new > m_run + kRescaleLog2;
        const float m_use = need ? m_new : m_run;
        const float alpha = need ? ex2_approx(m_run - m_new) : 1.0f;
        const float moff = (m_use == -INFINITY) ? 0.0f : m_use;

        // P_t's buffer (and O_t) are free once the previous PV of this unit finished (the
        // previous unit's last PV was waited for by its epilogue).  That PV ran while this
        // iteration loaded S and exchanged the row max, so the wait is normally short, and
        // p can then go to shared memory as it is computed.
        if (ok && j > 0) ok = __all_sync(0xffffffffu, mbar_wait(bar(B_PVDONE + t), (gi - 1) & 1u, SITE_SOFTMAX));
        float2 sum = make_float2(0.f, 0.f), sumb = make_float2(0.f, 0.f);
        if (ok) {
          const float2 sc2 = make_float2(sl2, sl2), nm2 = make_float2(-moff, -moff);
          // Chunks with no masked entry may evaluate part of the exponentials on the FMA
          // pipe (kEmulateExp); masked chunks use ex2 only, so masked entries stay zero.
          if (rel >= 63) {
            exp_chunk_store<kEmulateExp>(s0, ptile, r, 8 * h, sc2, nm2, sum);
            exp_chunk_store<kEmulateExp>(s1, ptile, r, 8 * h + 4, sc2, nm2, sumb);
          } else {
            exp_chunk_store<false>(s0, ptile, r, 8 * h, sc2, nm2, sum);
            exp_chunk_store<false>(s1, ptile, r, 8 * h + 4, sc2, nm2, sumb);
          }
          fence_proxy_async_smem();
          if (j > 0 && __any_sync(0xffffffffu, need)) {
            tc_fence_after();
#pragma unroll 1
            for (int c = 0; c < 2; ++c) {
              uint32_t o[32];
              tmem_ld32(tO + 32 * c, o);
              tmem_wait_ld_dep(o);
#pragma unroll
              for (int k = 0; k < 32; ++k) o[k] = __float_as_uint(__uint_as_float(o[k]) * alpha);
              tmem_st32(tO + 32 * c, o);
            }
            tmem_wait_st();
          }
          tc_fence_before();
          warp_arrive(bar(pready_bar(t)));
        }
        l_run = l_run * alpha + ((sum.x + sum.y) + (sumb.x + sumb.y));
        m_run = m_use;
      }

      // The next unit's Q was loaded once this unit's last QK^T finished: rotate and
      // release it now, so its first QK^T overlaps this unit's epilogue.
      if (inext < n_rounds) prepare_q(decode(unit_of(inext)), (uc + 1) & 1, uc + 1);
      // ---- epilogue: O / l -> bf16 -> P_t's buffer (free once the last PV is done) ->
      // one TMA store per 64-dim half of the tile
      const uint32_t last = Gb + n_kv - 1;
      if (ok) ok = __all_sync(0xffffffffu, mbar_wait(bar(B_PVDONE + t), last & 1u, SITE_EPILOGUE));
      named_bar_sync(bar_free, 256);
      xchg[h * 128 + r] = l_run;
      named_bar_sync(bar_x, 256);
      const float l_tot = l_run + xchg[(1 - h) * 128 + r];
      if (ok) {
        tc_fence_after();
        const float inv_l = l_tot > 0.0f ? 1.0f / l_tot : 0.0f;
#pragma unroll 1
        for (int c = 0; c < 2; ++c) {
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
            *reinterpret_cast<uint4*>(ptile + sw128_chunk(r, 8 * h + c * 4 + q)) = v;
          }
        }
        tc_fence_before();  // O_t may be overwritten by the next unit's first PV
      }
      fence_proxy_async_smem();
      named_bar_sync(bar_x, 256);
      const int p0 = x.p0 + t * kRowsPerHead;
      if (ok && h == 0 && r == 0 && p0 < p.S) {  // a tile starting past the sequence has nothing to store
        const uint32_t src = sbase + kOffP + t * kTileBytes;
        tma_store_3d(&tmO, src, 0, p0, x.zq);
        tma_store_3d(&tmO, src + kHalf, 64, p0, x.zq);
        bulk_commit();
        store_pending = true;
      }
      Gb += n_kv;
      ++uc;
    }
    if (h == 0 && r == 0) bulk_wait0();
  }

  // ---- teardown: everyone done with TMEM and shared memory
  tc_fence_before();
  named_bar_sync(5, kThreads);
  if (warp == kWarpMma) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace prefill

// ------------------------------------------------------------------ host side
int launch_prefill(const void* q, const void* k, const void* v, void* o, const void* cos, const void* sin, int B, int S,
                   int Hq, int Hkv, int head_dim, int kv_begin, int kv_count, float scale, int flags,
                   cudaStream_t stream) {
  using namespace prefill;
  if (!q || !k || !v || !o) return GQA_ERR_INVALID_ARGUMENT;
  if (B <= 0 || S <= 0 || Hq <= 0 || Hkv <= 0) return GQA_ERR_INVALID_ARGUMENT;
  if (head_dim != kD || Hq != kG * Hkv) return GQA_ERR_UNSUPPORTED;
  if (kv_begin < 0 || kv_count <= 0 || kv_begin + kv_count > Hkv) return GQA_ERR_INVALID_ARGUMENT;
  if (!(scale > 0.0f) || !(scale < 1e30f)) return GQA_ERR_INVALID_ARGUMENT;
  if ((flags & ~(GQA_FLAG_CAUSAL | GQA_FLAG_ROPE_Q | GQA_FLAG_ROPE_K)) != 0) return GQA_ERR_INVALID_ARGUMENT;
  if ((flags & (GQA_FLAG_ROPE_Q | GQA_FLAG_ROPE_K)) && (!cos || !sin)) return GQA_ERR_INVALID_ARGUMENT;
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(o)) return GQA_ERR_MISALIGNED;
  if ((flags & (GQA_FLAG_ROPE_Q | GQA_FLAG_ROPE_K)) && (!aligned16(cos) || !aligned16(sin))) return GQA_ERR_MISALIGNED;
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

  static std::atomic<uint64_t> attr_done{0};
  if ((rc = ensure_smem_attr(prefill_kernel, kSmemBytes, attr_done)) != GQA_OK) return rc;
  // The register split assumes the kernel was compiled to kRegsLaunch registers per thread.
  static std::atomic<int> regs_ok{0};
  if (regs_ok.load(std::memory_order_acquire) == 0) {
    cudaFuncAttributes fa;
    if (cudaFuncGetAttributes(&fa, prefill_kernel) != cudaSuccess) return GQA_ERR_CUDA;
    regs_ok.store(fa.numRegs == kRegsLaunch ? 1 : -1, std::memory_order_release);
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
  const int grid = static_cast<int>(n_units < sms ? n_units : sms);
  // Bands only pay when the (sequence, kv head) pairs outnumber what a round shares by
  // itself (grid / pairs query blocks of each pair per round, fewer than kBand), and when
  // there are enough rounds that bands of unequal units still balance across the SMs.
  // Batch 1 with 8 kv heads (each K/V stream already read by ~18 CTAs per round) or a
  // problem of a few rounds keeps the plain heaviest-first order: at seq 2048 the bands
  // would leave the busiest SM with 1.43x the mean work instead of 1.09x.
  const long long pairs = static_cast<long long>(B) * kv_count;
  p.band = (pairs * kBand > grid && n_units >= 8LL * grid) ? kBand : 1;
  prefill_kernel<<<grid, kThreads, kSmemBytes, stream>>>(tmQ, tmK, tmV, tmO, p);
  return cudaGetLastError() == cudaSuccess ? GQA_OK : GQA_ERR_CUDA;
}

}  // namespace gqa

namespace gqa {
GQA_ERROR_FLAG_ACCESSOR(error_flag_prefill)
}  // namespace gqa
