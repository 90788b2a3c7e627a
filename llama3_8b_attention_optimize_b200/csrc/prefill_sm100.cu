// prefill_sm100.cu -- fused causal GQA prefill on the sm_100a tensor core.
//
// Computes, per query head h (kv head h/4) and position i,
//   O[h,i,:] = softmax_j( (rope(q)[h,i] . rope(k)[h/4,j]) * scale , j <= i ) . V[h/4,:,:]
// i.e. stages RoPE -> QK^T/sqrt(d) -> causal mask -> softmax -> PV -> bf16 of the
// reference's golden model (llama3_attention_golden_model.py:162-190) and the fp32
// core of CPU_Baseline (CPU_Baseline/cpu_baseline/attention.py:60-84), without
// materialising the S x S score matrix.
//
// Work unit (one CTA): batch b, kv head g, a block of 64 query positions.  The CTA
// holds two 128-row Q tiles; each tile packs the 4 query heads of group g x 32
// positions (row r = head_in_group*32 + position_offset), so one K/V tile in shared
// memory serves all 4 heads of the group (GQA by address, no KV duplication).
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
//   warp 16    TMA producer (Q tiles, then K0 K1 V0 K2 V1 ... into a 3-stage ring)
//   warp 17    tcgen05.mma issuer (one elected thread) + TMEM allocator
//   warps 18-19 RoPE of K tiles in shared memory (when FLAG_ROPE_K)
// TMEM (512 columns x 128 lanes, fp32): S0 [0,128) S1 [128,256) O0 [256,384) O1 [384,512).
//
// Online softmax in the log2 domain: p = 2^(s*scale*log2e - m); the running max m is
// only raised (and O rescaled) when a tile's max exceeds it by more than kRescaleLog2,
// so p <= 2^16: with |v| < 2^16 and at most 2^17 keys, O stays below 2^49 (fp32-safe).
#include <cuda.h>

#include "common.cuh"
#include "gqa_internal.h"

namespace gqa {
namespace prefill {

constexpr int kD = 128;
constexpr int kG = 4;
constexpr int kBM = 128;
constexpr int kRowsPerHead = kBM / kG;        // 32
constexpr int kPosPerCta = 2 * kRowsPerHead;  // 64
constexpr int kBN = 128;                      // keys per K/V tile
constexpr int kStages = 3;                    // K/V ring stages
constexpr int kTileBytes = 128 * 128 * 2;     // Q, P, K and V tiles: 32 KB
constexpr int kHalf = kTileBytes / 2;         // one 64-column swizzle block of 128 rows
constexpr int kSoftmaxThreads = 512;  // warps 0-15
constexpr float kRescaleLog2 = 16.0f;
constexpr int kWarpProducer = 16;
constexpr int kWarpMma = 17;
constexpr int kWarpRope0 = 18;
constexpr int kThreads = 640;

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
  B_QFULL = 0,     // [2]  TMA Q landed
  B_QREADY = 2,    // [2]  Q (rotated) visible to the tensor core, 128 arrivals
  B_KVFULL = 4,    // [3]  TMA K/V stage landed
  B_KVEMPTY = 7,   // [3]  MMAs reading the stage completed
  B_KREADY = 10,   // [4]  K tile j rotated (slot j % 4), 64 arrivals
  B_SFULL = 14,    // [2]  S_t = Q_t K^T complete
  B_SFREE = 16,    // [1]  S_0 and S_1 copied to registers (512 arrivals)
  B_PREADY = 18,   // [1]  P_0 and P_1 in shared memory, O rescaled (512 arrivals)
  B_PVDONE = 20,   // [2]  O_t += P_t V complete (P_t buffer free)
  B_DRAIN = 22,    // [1]  every MMA of the CTA complete
};
constexpr int kKReadySlots = 4;

// Load order of the K/V ring: K0, K1, V0, K2, V1, ..., K(n-1), V(n-2), V(n-1).  With K
// one tile ahead, every stage a load reuses was released an iteration earlier (K(j+1)
// reuses V(j-2)'s stage, V(j) reuses K(j)'s), so a 3-stage ring never stalls the MMAs.
__device__ __forceinline__ int load_idx_k(int j) { return j == 0 ? 0 : 2 * j - 1; }
__device__ __forceinline__ int load_idx_v(int j, int n) { return j + 1 < n ? 2 * j + 2 : 2 * n - 1; }

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
  int B, S, Hq, Hkv, kv_begin, kv_count, n_qblocks;
  int flags;
  float scale_log2;
  const uint16_t* cos;  // [>= S][128] bf16 (cat(freqs, freqs) layout)
  const uint16_t* sin;
  long long* trace;  // diagnostic event trace of one CTA (nullptr = off)
  int trace_block;
};

// Diagnostic trace: clock64 stamps [role][iteration][event] for CTA trace_block.
constexpr int kTraceIters = 128;
constexpr int kTraceRoles = 6;
constexpr int kTraceEv = 8;
#define PF_TRACE(role, it, ev)                                                                        \
  do {                                                                                                \
    if (kTrace && tr) tr[((role) * kTraceIters + min((it), kTraceIters - 1)) * kTraceEv + (ev)] = clock64(); \
  } while (0)

__device__ __forceinline__ uint32_t colS(int t) { return static_cast<uint32_t>(t * 128); }
__device__ __forceinline__ uint32_t colO(int t) { return static_cast<uint32_t>(256 + t * 128); }

// Byte offset of 16-byte chunk c (elements 8c..8c+7) of row r in a 128x128 bf16
// K-major SWIZZLE_128B tile (two 64-column blocks of 128 rows x 128 B).
__device__ __forceinline__ int sw128_chunk(int r, int c) {
  return (c >> 3) * kHalf + r * 128 + (((c & 7) ^ (r & 7)) << 4);
}

__device__ __forceinline__ void rope_pair(uint32_t& xa, uint32_t& xb, uint32_t c, uint32_t s) {
  // y[d] = x[d]*cos - x[d+64]*sin ; y[d+64] = x[d+64]*cos + x[d]*sin (products are exact)
  const float x0l = bf16_lo(xa), x0h = bf16_hi(xa), x1l = bf16_lo(xb), x1h = bf16_hi(xb);
  const float cl = bf16_lo(c), chh = bf16_hi(c), sl = bf16_lo(s), shh = bf16_hi(s);
  const float y0l = __fadd_rn(__fmul_rn(x0l, cl), -__fmul_rn(x1l, sl));
  const float y0h = __fadd_rn(__fmul_rn(x0h, chh), -__fmul_rn(x1h, shh));
  const float y1l = __fadd_rn(__fmul_rn(x1l, cl), __fmul_rn(x0l, sl));
  const float y1h = __fadd_rn(__fmul_rn(x1h, chh), __fmul_rn(x0h, shh));
  xa = pack_bf16x2(y0l, y0h);
  xb = pack_bf16x2(y1l, y1h);
}

// Rotate chunk pairs [c0, c0+4) of one row (half of the row's 8 pairs).
__device__ __forceinline__ void rope_row_smem_part(uint8_t* tile, int half, int row, const uint16_t* cos_row,
                                                   const uint16_t* sin_row, int c0) {
#pragma unroll 2
  for (int ch = c0; ch < c0 + 4; ++ch) {
    const int off = row * 128 + ((ch ^ (row & 7)) << 4);
    uint4* pa = reinterpret_cast<uint4*>(tile + off);
    uint4* pb = reinterpret_cast<uint4*>(tile + half + off);
    uint4 a = *pa, b = *pb;
    const uint4 c = __ldg(reinterpret_cast<const uint4*>(cos_row + ch * 8));
    const uint4 s = __ldg(reinterpret_cast<const uint4*>(sin_row + ch * 8));
    rope_pair(a.x, b.x, c.x, s.x);
    rope_pair(a.y, b.y, c.y, s.y);
    rope_pair(a.z, b.z, c.z, s.z);
    rope_pair(a.w, b.w, c.w, s.w);
    *pa = a;
    *pb = b;
  }
}

// Rotate one 128-element row held in a K-major SWIZZLE_128B tile made of two
// 64-dim blocks `half` bytes apart (dims d and d+64 sit at the same offset in the
// two blocks).
__device__ __forceinline__ void rope_row_smem(uint8_t* tile, int half, int row, const uint16_t* cos_row,
                                              const uint16_t* sin_row) {
#pragma unroll 2
  for (int ch = 0; ch < 8; ++ch) {
    const int off = row * 128 + ((ch ^ (row & 7)) << 4);
    uint4* pa = reinterpret_cast<uint4*>(tile + off);
    uint4* pb = reinterpret_cast<uint4*>(tile + half + off);
    uint4 a = *pa, b = *pb;
    const uint4 c = __ldg(reinterpret_cast<const uint4*>(cos_row + ch * 8));
    const uint4 s = __ldg(reinterpret_cast<const uint4*>(sin_row + ch * 8));
    rope_pair(a.x, b.x, c.x, s.x);
    rope_pair(a.y, b.y, c.y, s.y);
    rope_pair(a.z, b.z, c.z, s.z);
    rope_pair(a.w, b.w, c.w, s.w);
    *pa = a;
    *pb = b;
  }
}

__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// 2^x on the FMA pipe for a pair: x = n + f with n = round(x) (added-constant trick,
// exact for |x| < 2^22), 2^f by a cubic on [-1/2, 1/2] (relative error 7.5e-5, a
// near-minimax fit of 2^f made for this kernel), and 2^n added to the exponent
// field.  x is clamped to >= -126 so the result stays a normal number.
__device__ __forceinline__ float2 exp2_poly2(float2 x) {
  constexpr float kRound = 12582912.0f;  // 1.5 * 2^23
  constexpr float c0 = 0.99992806f, c1 = 0.69326097f, c2 = 0.24261114f, c3 = 0.05517167f;
  x.x = fmaxf(x.x, -126.0f);
  x.y = fmaxf(x.y, -126.0f);
  const float2 t = __fadd2_rn(x, make_float2(kRound, kRound));
  const float2 n = __fadd2_rn(t, make_float2(-kRound, -kRound));
  const float2 f = __ffma2_rn(n, make_float2(-1.0f, -1.0f), x);
  float2 q = __ffma2_rn(make_float2(c3, c3), f, make_float2(c2, c2));
  q = __ffma2_rn(q, f, make_float2(c1, c1));
  q = __ffma2_rn(q, f, make_float2(c0, c0));
  return make_float2(__int_as_float(__float_as_int(q.x) + (__float_as_int(t.x) << 23)),
                     __int_as_float(__float_as_int(q.y) + (__float_as_int(t.y) << 23)));
}

// One 32-column chunk of S -> 16 packed bf16 pairs of p = 2^(s*scale_log2 - m) at
// out[base..base+16); acc += the bf16-rounded p.
template <bool kEmulate>
__device__ __forceinline__ void exp_chunk(const uint32_t (&s)[32], uint32_t (&out)[32], int base, float2 sc2,
                                          float2 nm2, float2& acc) {
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const float2 x = __ffma2_rn(make_float2(__uint_as_float(s[2 * i]), __uint_as_float(s[2 * i + 1])), sc2, nm2);
    float2 e;
    if (kEmulate && (i & 3) == 3) {
      e = exp2_poly2(x);
    } else {
      e.x = ex2_approx(x.x);
      e.y = ex2_approx(x.y);
    }
    const uint32_t w = pack_bf16x2(e.x, e.y);
    out[base + i] = w;
    // the row sum uses the bf16 values PV multiplies, so O / l normalises exactly them
    acc = __fadd2_rn(acc, make_float2(bf16_lo(w), bf16_hi(w)));
  }
}

template <bool kTrace>
__global__ void __launch_bounds__(kThreads, 1)
    prefill_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                   const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmO, const Params p) {
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

  // ---- work unit (heaviest causal blocks first)
  const int per_qb = p.B * p.kv_count;
  const int qb = p.n_qblocks - 1 - static_cast<int>(blockIdx.x) / per_qb;
  const int rem = static_cast<int>(blockIdx.x) % per_qb;
  const int b = rem / p.kv_count;
  const int kvh = p.kv_begin + rem % p.kv_count;
  const int cta_p0 = qb * kPosPerCta;
  const bool causal = (p.flags & GQA_FLAG_CAUSAL) != 0;
  const bool rope_q = (p.flags & GQA_FLAG_ROPE_Q) != 0;
  const bool rope_k = (p.flags & GQA_FLAG_ROPE_K) != 0;
  const int n_kv_all = (p.S + kBN - 1) / kBN;
  const int n_kv = causal ? min(n_kv_all, (cta_p0 + kPosPerCta - 1) / kBN + 1) : n_kv_all;
  const int zq = b * p.Hq + kvh * kG;  // first Q/O head row of the group
  const int zk = b * p.Hkv + kvh;

  if (threadIdx.x == 0) {
    for (int t = 0; t < 2; ++t) {
      mbar_init(bar(B_QFULL + t), 1);
      mbar_init(bar(B_QREADY + t), 256);
      mbar_init(bar(B_SFULL + t), 1);

      mbar_init(bar(B_PVDONE + t), 1);
    }
    for (int s = 0; s < kStages; ++s) {
      mbar_init(bar(B_KVFULL + s), 1);
      mbar_init(bar(B_KVEMPTY + s), 1);
    }
    for (int k = 0; k < kKReadySlots; ++k) mbar_init(bar(B_KREADY + k), 64);
    mbar_init(bar(B_SFREE), kSoftmaxThreads);
    mbar_init(bar(B_PREADY), kSoftmaxThreads);
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
  if (threadIdx.x == 0) PF_TRACE(5, 0, 0);

  if (warp == kWarpProducer) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      for (int t = 0; t < 2; ++t) {
        const uint32_t dst = sbase + kOffQ + t * kTileBytes;
        mbar_expect_tx(bar(B_QFULL + t), kTileBytes);
        tma_load_3d(dst, &tmQ, bar(B_QFULL + t), 0, cta_p0 + t * kRowsPerHead, zq);
        tma_load_3d(dst + kHalf, &tmQ, bar(B_QFULL + t), 64, cta_p0 + t * kRowsPerHead, zq);
      }
      const int nloads = 2 * n_kv;
      int issued = 0;
      bool ok = true;
      for (int i = 0; i < nloads; ++i) {
        const int s = i % kStages, r = i / kStages;
        if (r > 0) ok = mbar_wait(bar(B_KVEMPTY + s), (r - 1) & 1, SITE_PRODUCER);
        if (!ok) break;
        // i -> (tile, K or V) in the K-ahead order
        const bool is_v = (i == nloads - 1) || (i >= 2 && (i & 1) == 0);
        const int j = i == 0 ? 0 : (is_v ? (i == nloads - 1 ? n_kv - 1 : (i - 2) >> 1) : (i + 1) >> 1);
        const void* map = is_v ? static_cast<const void*>(&tmV) : static_cast<const void*>(&tmK);
        const uint32_t dst = sbase + kOffKV + s * kTileBytes;
        mbar_expect_tx(bar(B_KVFULL + s), kTileBytes);
        tma_load_3d(dst, map, bar(B_KVFULL + s), 0, j * kBN, zk);
        tma_load_3d(dst + kHalf, map, bar(B_KVFULL + s), 64, j * kBN, zk);
        PF_TRACE(0, j, is_v ? 1 : 0);
        issued = i + 1;
      }
      // Drain: every load this thread issued must land before the CTA may exit.
      for (int i = max(0, issued - kStages); i < issued; ++i)
        mbar_wait(bar(B_KVFULL + i % kStages), (i / kStages) & 1, SITE_DRAIN);
      mbar_wait(bar(B_QFULL + 0), 0, SITE_DRAIN);
      mbar_wait(bar(B_QFULL + 1), 0, SITE_DRAIN);
    }
    __syncwarp();
  } else if (warp == kWarpMma) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t kIdQK = idesc_bf16_f32(128, kBN, false);
      constexpr uint32_t kIdPV = idesc_bf16_f32(128, kD, true);
      // Descriptor halves computed once; each MMA adds a compile-time offset (in
      // 16-byte units) to the low word.  K-major operands (Q, K, P): LBO unused;
      // V is MN-major with its two 64-dim blocks kHalf apart (LBO = kHalf).
      constexpr uint32_t kHi = sdesc_hi_sw128(1024);
      const uint32_t q_lo = sdesc_lo(sbase + kOffQ, 16);
      const uint32_t p_lo = sdesc_lo(sbase + kOffP, 16);
      const uint32_t kv_lo = sdesc_lo(sbase + kOffKV, 16);
      const uint32_t v_lo = sdesc_lo(sbase + kOffKV, kHalf);
      constexpr uint32_t kTile16 = kTileBytes / 16;
      // S_t = Q_t K^T over d = 128 (8 k-steps of 16; both operands K-major SW128)
      auto issue_qk = [&](int t, int s) {
        const uint32_t a0 = q_lo + t * kTile16, b0 = kv_lo + s * kTile16;
        const uint32_t d = tmem + colS(t);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint32_t off = ((kk >> 2) * kHalf + (kk & 3) * 32) / 16;
          umma_ss_lohi(d, a0 + off, b0 + off, kHi, kIdQK, kk > 0 ? 1u : 0u);
        }
      };
      // O_t (+)= P_t V over 128 keys (8 k-steps; P K-major SW128, V MN-major SW128)
      auto issue_pv = [&](int t, int s, uint32_t acc) {
        const uint32_t a0 = p_lo + t * kTile16, b0 = v_lo + s * kTile16;
        const uint32_t d = tmem + colO(t);
        umma_ss_lohi(d, a0, b0, kHi, kIdPV, acc);
#pragma unroll
        for (int kk = 1; kk < 8; ++kk) {
          const uint32_t off = ((kk >> 2) * kHalf + (kk & 3) * 32) / 16;
          umma_ss_lohi(d, a0 + off, b0 + kk * (2048 / 16), kHi, kIdPV, 1u);
        }
      };
      auto wait_k = [&](int j) -> bool {  // K tile j landed (and rotated)
        if (rope_k) return mbar_wait_spin(bar(B_KREADY + j % kKReadySlots), (j / kKReadySlots) & 1, SITE_MMA);
        const int i = load_idx_k(j);
        return mbar_wait_spin(bar(B_KVFULL + i % kStages), (i / kStages) & 1, SITE_MMA);
      };
      bool ok = mbar_wait_spin(bar(B_QREADY + 0), 0, SITE_MMA) && mbar_wait_spin(bar(B_QREADY + 1), 0, SITE_MMA) &&
                wait_k(0);
      if (ok) {
        tc_fence_after();
        issue_qk(0, 0);
        umma_commit(bar(B_SFULL + 0));
        issue_qk(1, 0);
        umma_commit(bar(B_SFULL + 1));
        umma_commit(bar(B_KVEMPTY + 0));
      }
      for (int j = 0; ok && j < n_kv; ++j) {
        PF_TRACE(1, j, 0);
        if (j + 1 < n_kv) {
          // next S as soon as the softmax warps hold S(j) in registers
          const int sk = load_idx_k(j + 1) % kStages;
          ok = wait_k(j + 1) && mbar_wait_spin(bar(B_SFREE), j & 1, SITE_MMA);
          if (!ok) break;
          PF_TRACE(1, j, 1);
          tc_fence_after();
          issue_qk(0, sk);
          umma_commit(bar(B_SFULL + 0));
          PF_TRACE(1, j, 2);
          issue_qk(1, sk);
          umma_commit(bar(B_SFULL + 1));
          umma_commit(bar(B_KVEMPTY + sk));
          PF_TRACE(1, j, 3);
        }
        const int iv = load_idx_v(j, n_kv), sv = iv % kStages;
        ok = mbar_wait_spin(bar(B_KVFULL + sv), (iv / kStages) & 1, SITE_MMA) &&
             mbar_wait_spin(bar(B_PREADY), j & 1, SITE_MMA);
        if (!ok) break;
        PF_TRACE(1, j, 4);
        tc_fence_after();
        issue_pv(0, sv, j > 0 ? 1u : 0u);
        umma_commit(bar(B_PVDONE + 0));
        PF_TRACE(1, j, 5);
        PF_TRACE(1, j, 6);
        tc_fence_after();
        issue_pv(1, sv, j > 0 ? 1u : 0u);
        umma_commit(bar(B_PVDONE + 1));
        umma_commit(bar(B_KVEMPTY + sv));
        PF_TRACE(1, j, 7);
      }
      umma_commit(bar(B_DRAIN));
      mbar_wait(bar(B_DRAIN), 0, SITE_DRAIN);
    }
    __syncwarp();
  } else if (warp >= kWarpRope0) {
    // ------------------------------------------------------------ RoPE of K tiles
    if (rope_k) {
      const int tid = threadIdx.x - kWarpRope0 * 32;  // 0..63
      for (int j = 0; j < n_kv; ++j) {
        const int i = load_idx_k(j), s = i % kStages, r = i / kStages;
        if (!mbar_wait(bar(B_KVFULL + s), r & 1, SITE_ROPEK)) break;
        if (tid == 0) PF_TRACE(4, j, 0);
        uint8_t* tile = smem + kOffKV + s * kTileBytes;
#pragma unroll 1
        for (int rr = tid; rr < kBN; rr += 64) {
          const int key = j * kBN + rr;
          if (key < p.S)
            rope_row_smem(tile, kHalf, rr, p.cos + static_cast<size_t>(key) * kD, p.sin + static_cast<size_t>(key) * kD);
        }
        fence_proxy_async_smem();
        if (tid == 0) PF_TRACE(4, j, 1);
        mbar_arrive(bar(B_KREADY + j % kKReadySlots));
      }
    }
  } else {
    // ------------------------------------------------------------ softmax warpgroups
    const int g = warp >> 2;             // warpgroup 0..3
    const int t = g >> 1;                // Q tile
    const int h = g & 1;                 // keys [64h, 64h+64) of each K tile; O dims [64h, 64h+64)
    const int r = threadIdx.x & 127;     // row in tile == TMEM lane
    const uint32_t lane_off = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const uint32_t tS = tmem + lane_off + colS(t) + 64 * h;
    const uint32_t tO = tmem + lane_off + colO(t) + 64 * h;
    const int p0 = cta_p0 + t * kRowsPerHead;
    const int qpos = p0 + (r & (kRowsPerHead - 1));
    uint8_t* qtile = smem + kOffQ + t * kTileBytes;
    uint8_t* ptile = smem + kOffP + t * kTileBytes;
    float* xchg = reinterpret_cast<float*>(smem + kOffX) + t * 256;  // [half][row]
    const int bar_x = 1 + t;     // named barrier: both halves of tile t (256 threads)
    const int bar_free = 3 + t;  // named barrier: exchange slots may be rewritten
    const float sl2 = p.scale_log2;

    bool ok = mbar_wait(bar(B_QFULL + t), 0, SITE_SOFTMAX);
    if (ok && rope_q && qpos < p.S)  // each half rotates 4 of the row's 8 chunk pairs
      rope_row_smem_part(qtile, kHalf, r, p.cos + static_cast<size_t>(qpos) * kD,
                         p.sin + static_cast<size_t>(qpos) * kD, 4 * h);
    fence_proxy_async_smem();
    mbar_arrive(bar(B_QREADY + t));
    ok = __all_sync(0xffffffffu, ok);

    // last key this row may attend
    const int lim = causal ? min(qpos, p.S - 1) : p.S - 1;
    float m_run = -INFINITY, l_run = 0.0f;
    // Every warp of the tile runs all n_kv iterations and meets every named barrier,
    // even after a bounded wait failed (ok == false only skips the work), so the two
    // halves of a tile can never wait on each other forever.
    for (int j = 0; j < n_kv; ++j) {
      if (ok) ok = __all_sync(0xffffffffu, mbar_wait(bar(B_SFULL + t), j & 1, SITE_SOFTMAX));
      if (r == 0 && h == 0) PF_TRACE(2 + t, j, 0);
      uint32_t s0[32], s1[32];
      if (ok) {
        tc_fence_after();
        tmem_ld32(tS + 0, s0);
        tmem_ld32(tS + 32, s1);
        tmem_wait_ld_dep(s0);
        reg_dep(s1);
        tc_fence_before();
        mbar_arrive(bar(B_SFREE));  // S_t may now be overwritten by the next QK^T
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
      // row max over both halves: slot [h][r] <-> [1-h][r]
      named_bar_sync(bar_free, 256);  // everyone has read the previous iteration's slots
      xchg[h * 128 + r] = fmaxf(mx0, mx1);
      named_bar_sync(bar_x, 256);
      const float m_tile = fmaxf(fmaxf(mx0, mx1), xchg[(1 - h) * 128 + r]) * sl2;
      if (r == 0 && h == 0) PF_TRACE(2 + t, j, 1);
      const float m_new = fmaxf(m_run, m_tile);
      const bool need = m_new > m_run + kRescaleLog2;
      const float m_use = need ? m_new : m_run;
      const float alpha = need ? ex2_approx(m_run - m_new) : 1.0f;
      const float moff = (m_use == -INFINITY) ? 0.0f : m_use;

      uint32_t pw[32];
      float2 sum = make_float2(0.f, 0.f), sumb = make_float2(0.f, 0.f);
      const float2 sc2 = make_float2(sl2, sl2), nm2 = make_float2(-moff, -moff);
      // Chunks with no masked entry evaluate a quarter of the exponentials on the FMA
      // pipe; masked chunks use ex2 only, so masked entries stay exactly zero.
      if (rel >= 63) {
        exp_chunk<true>(s0, pw, 0, sc2, nm2, sum);
        exp_chunk<true>(s1, pw, 16, sc2, nm2, sumb);
      } else {
        exp_chunk<false>(s0, pw, 0, sc2, nm2, sum);
        exp_chunk<false>(s1, pw, 16, sc2, nm2, sumb);
      }

      // P_t's buffer (and O_t) are free once the previous PV finished.
      if (ok && j > 0) ok = __all_sync(0xffffffffu, mbar_wait(bar(B_PVDONE + t), (j - 1) & 1, SITE_SOFTMAX));
      if (r == 0 && h == 0) PF_TRACE(2 + t, j, 2);
      if (ok) {
#pragma unroll
        for (int c = 0; c < 8; ++c)
          *reinterpret_cast<uint4*>(ptile + sw128_chunk(r, 8 * h + c)) =
              make_uint4(pw[4 * c], pw[4 * c + 1], pw[4 * c + 2], pw[4 * c + 3]);
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
        mbar_arrive(bar(B_PREADY));
      }
      l_run = l_run * alpha + ((sum.x + sum.y) + (sumb.x + sumb.y));
      m_run = m_use;
      if (r == 0 && h == 0) PF_TRACE(2 + t, j, 3);
    }

    // ---- epilogue: O / l -> bf16 -> (reuse the Q tile smem) -> TMA store
    if (ok) ok = __all_sync(0xffffffffu, mbar_wait(bar(B_PVDONE + t), (n_kv - 1) & 1, SITE_EPILOGUE));
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
          *reinterpret_cast<uint4*>(qtile + sw128_chunk(r, 8 * h + c * 4 + q)) = v;
        }
      }
    }
    fence_proxy_async_smem();
    named_bar_sync(bar_x, 256);
    if (ok && h == 0 && r == 0 && p0 < p.S) {  // a tile starting past the sequence has nothing to store
      const uint32_t src = sbase + kOffQ + t * kTileBytes;
      tma_store_3d(&tmO, src, 0, p0, zq);
      tma_store_3d(&tmO, src + kHalf, 64, p0, zq);
      bulk_commit();
      bulk_wait0();
    }
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
                   cudaStream_t stream, long long* trace, int trace_block) {
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
  const long long grid = n_qblocks * B * kv_count;
  if (grid > 0x7FFFFFFFLL || static_cast<long long>(B) * Hq > 0x7FFFFFFFLL) return GQA_ERR_UNSUPPORTED;

  CUtensorMap tmQ, tmK, tmV, tmO;
  int rc;
  if ((rc = make_tmap_3d_bf16(&tmQ, q, kD, S, static_cast<long long>(B) * Hq, 64, kRowsPerHead, kG)) != GQA_OK)
    return rc;
  if ((rc = make_tmap_3d_bf16(&tmK, k, kD, S, static_cast<long long>(B) * Hkv, 64, kBN, 1)) != GQA_OK) return rc;
  if ((rc = make_tmap_3d_bf16(&tmV, v, kD, S, static_cast<long long>(B) * Hkv, 64, kBN, 1)) != GQA_OK) return rc;
  if ((rc = make_tmap_3d_bf16(&tmO, o, kD, S, static_cast<long long>(B) * Hq, 64, kRowsPerHead, kG)) != GQA_OK)
    return rc;

  static std::atomic<uint64_t> attr_done{0}, attr_done_tr{0};
  if ((rc = ensure_smem_attr(prefill_kernel<false>, kSmemBytes, attr_done)) != GQA_OK) return rc;
  if (trace && (rc = ensure_smem_attr(prefill_kernel<true>, kSmemBytes, attr_done_tr)) != GQA_OK) return rc;
  Params p;
  p.B = B;
  p.S = S;
  p.Hq = Hq;
  p.Hkv = Hkv;
  p.kv_begin = kv_begin;
  p.kv_count = kv_count;
  p.n_qblocks = static_cast<int>(n_qblocks);
  p.flags = flags;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.cos = static_cast<const uint16_t*>(cos);
  p.sin = static_cast<const uint16_t*>(sin);
  p.trace = trace;
  p.trace_block = trace_block;
  if (trace)
    prefill_kernel<true><<<static_cast<unsigned>(grid), kThreads, kSmemBytes, stream>>>(tmQ, tmK, tmV, tmO, p);
  else
    prefill_kernel<false><<<static_cast<unsigned>(grid), kThreads, kSmemBytes, stream>>>(tmQ, tmK, tmV, tmO, p);
  return cudaGetLastError() == cudaSuccess ? GQA_OK : GQA_ERR_CUDA;
}

}  // namespace gqa
