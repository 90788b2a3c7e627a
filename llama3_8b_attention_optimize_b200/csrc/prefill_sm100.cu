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
// Warp roles (12 warps):
//   warps 0-3  softmax warpgroup for Q tile 0 (thread r owns TMEM lane / row r)
//   warps 4-7  softmax warpgroup for Q tile 1
//   warp 8     TMA producer (Q tiles, then K0 V0 K1 V1 ... into a 4-stage ring)
//   warp 9     tcgen05.mma issuer (one elected thread) + TMEM allocator
//   warps 10-11 RoPE of K tiles in shared memory (when FLAG_ROPE_K)
// TMEM (512 columns x 128 lanes, fp32): S0 [0,128) S1 [128,256) O0 [256,384) O1 [384,512);
// P_t (bf16 pairs) overwrites the first 64 columns of S_t and feeds PV as the A operand.
//
// Online softmax in the log2 domain: p = 2^(s*scale*log2e - m); the running max m is
// only raised (and O rescaled) when a tile's max exceeds it by more than 8, so p <= 256.
#include <cuda.h>

#include "common.cuh"
#include "gqa_internal.h"

namespace gqa {
namespace prefill {

constexpr int kD = 128;
constexpr int kG = 4;
constexpr int kBM = 128;
constexpr int kRowsPerHead = kBM / kG;  // 32
constexpr int kPosPerCta = 2 * kRowsPerHead;  // 64
constexpr int kBN = 128;
constexpr int kStages = 4;
constexpr int kTileBytes = 128 * 128 * 2;
constexpr int kHalfBytes = kTileBytes / 2;
constexpr int kThreads = 384;

constexpr int kOffQ = 0;
constexpr int kOffKV = kOffQ + 2 * kTileBytes;
constexpr int kOffBar = kOffKV + kStages * kTileBytes;
constexpr int kNumBars = 24;
constexpr int kOffTmemPtr = kOffBar + kNumBars * 8;
constexpr int kSmemBytes = kOffTmemPtr + 16 + 1024;

enum : int {
  B_QFULL = 0,     // [2]  TMA Q landed
  B_QREADY = 2,    // [2]  Q (rotated) visible to the tensor core, 128 arrivals
  B_KVFULL = 4,    // [4]  TMA K/V stage landed
  B_KVEMPTY = 8,   // [4]  MMAs reading the stage completed
  B_KREADY = 12,   // [4]  K stage rotated, 64 arrivals
  B_SFULL = 16,    // [2]  S_t = Q_t K^T complete
  B_PREADY = 18,   // [2]  P_t in TMEM (and O_t rescaled), 128 arrivals
  B_ODONE = 20,    // [2]  O_t += P_t V complete
  B_DRAIN = 22,    // [1]  every MMA of the CTA complete
};

enum : int {  // error sites reported through g_gqa_dev_error
  SITE_PRODUCER = 0x101,
  SITE_MMA = 0x102,
  SITE_SOFTMAX = 0x103,
  SITE_ROPEK = 0x104,
  SITE_EPILOGUE = 0x105,
  SITE_DRAIN = 0x106,
};

struct Params {
  int B, S, Hq, Hkv, kv_begin, kv_count, n_qblocks;
  int flags;
  float scale_log2;
  const uint16_t* cos;  // [>= S][128] bf16 (cat(freqs, freqs) layout)
  const uint16_t* sin;
};

__device__ __forceinline__ uint32_t colS(int t) { return static_cast<uint32_t>(t * 128); }
__device__ __forceinline__ uint32_t colO(int t) { return static_cast<uint32_t>(256 + t * 128); }

// Rotate one 128-element row held in a K-major SWIZZLE_128B tile (two 64-column
// blocks 16 KB apart; dims d and d+64 sit at the same offset in the two blocks).
__device__ __forceinline__ void rope_row_smem(uint8_t* tile, int row, const uint16_t* cos_row,
                                              const uint16_t* sin_row) {
#pragma unroll
  for (int ch = 0; ch < 8; ++ch) {
    const int off = row * 128 + ((ch ^ (row & 7)) << 4);
    uint4* pa = reinterpret_cast<uint4*>(tile + off);
    uint4* pb = reinterpret_cast<uint4*>(tile + kHalfBytes + off);
    uint4 a = *pa, b = *pb;
    const uint4 c = __ldg(reinterpret_cast<const uint4*>(cos_row + ch * 8));
    const uint4 s = __ldg(reinterpret_cast<const uint4*>(sin_row + ch * 8));
    uint32_t* aw = reinterpret_cast<uint32_t*>(&a);
    uint32_t* bw = reinterpret_cast<uint32_t*>(&b);
    const uint32_t* cw = reinterpret_cast<const uint32_t*>(&c);
    const uint32_t* sw = reinterpret_cast<const uint32_t*>(&s);
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      float x0l = bf16_lo(aw[w]), x0h = bf16_hi(aw[w]);
      float x1l = bf16_lo(bw[w]), x1h = bf16_hi(bw[w]);
      float cl = bf16_lo(cw[w]), chh = bf16_hi(cw[w]);
      float sl = bf16_lo(sw[w]), shh = bf16_hi(sw[w]);
      // y[d] = x[d]*cos - x[d+64]*sin ; y[d+64] = x[d+64]*cos + x[d]*sin (products are exact)
      float y0l = __fadd_rn(__fmul_rn(x0l, cl), -__fmul_rn(x1l, sl));
      float y0h = __fadd_rn(__fmul_rn(x0h, chh), -__fmul_rn(x1h, shh));
      float y1l = __fadd_rn(__fmul_rn(x1l, cl), __fmul_rn(x0l, sl));
      float y1h = __fadd_rn(__fmul_rn(x1h, chh), __fmul_rn(x0h, shh));
      aw[w] = pack_bf16x2(y0l, y0h);
      bw[w] = pack_bf16x2(y1l, y1h);
    }
    *pa = a;
    *pb = b;
  }
}

__global__ void __launch_bounds__(kThreads, 1)
    prefill_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                   const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmO, const Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
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
    mbar_init(bar(B_QFULL + 0), 1);
    mbar_init(bar(B_QFULL + 1), 1);
    mbar_init(bar(B_QREADY + 0), 128);
    mbar_init(bar(B_QREADY + 1), 128);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(bar(B_KVFULL + s), 1);
      mbar_init(bar(B_KVEMPTY + s), 1);
      mbar_init(bar(B_KREADY + s), 64);
    }
    for (int t = 0; t < 2; ++t) {
      mbar_init(bar(B_SFULL + t), 1);
      mbar_init(bar(B_PREADY + t), 128);
      mbar_init(bar(B_ODONE + t), 1);
    }
    mbar_init(bar(B_DRAIN), 1);
    fence_mbar_init();
  }
  if (warp == 9) {
    tmem_alloc(sbase + kOffTmemPtr, 512);
    tmem_relinquish();
  }
  if (warp == 8 && lane == 0) {
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
    tma_prefetch_desc(&tmO);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(smem + kOffTmemPtr);

  if (warp == 8) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      for (int t = 0; t < 2; ++t) {
        const uint32_t dst = sbase + kOffQ + t * kTileBytes;
        mbar_expect_tx(bar(B_QFULL + t), kTileBytes);
        tma_load_3d(dst, &tmQ, bar(B_QFULL + t), 0, cta_p0 + t * kRowsPerHead, zq);
        tma_load_3d(dst + kHalfBytes, &tmQ, bar(B_QFULL + t), 64, cta_p0 + t * kRowsPerHead, zq);
      }
      const int nloads = 2 * n_kv;
      int issued = 0;
      bool ok = true;
      for (int i = 0; i < nloads; ++i) {
        const int s = i % kStages, r = i / kStages;
        if (r > 0) ok = mbar_wait(bar(B_KVEMPTY + s), (r - 1) & 1, SITE_PRODUCER);
        if (!ok) break;
        const int j = i >> 1;
        const void* map = (i & 1) ? static_cast<const void*>(&tmV) : static_cast<const void*>(&tmK);
        const uint32_t dst = sbase + kOffKV + s * kTileBytes;
        mbar_expect_tx(bar(B_KVFULL + s), kTileBytes);
        tma_load_3d(dst, map, bar(B_KVFULL + s), 0, j * kBN, zk);
        tma_load_3d(dst + kHalfBytes, map, bar(B_KVFULL + s), 64, j * kBN, zk);
        issued = i + 1;
      }
      // Drain: every load this thread issued must land before the CTA may exit.
      for (int i = max(0, issued - kStages); i < issued; ++i)
        mbar_wait(bar(B_KVFULL + i % kStages), (i / kStages) & 1, SITE_DRAIN);
      mbar_wait(bar(B_QFULL + 0), 0, SITE_DRAIN);
      mbar_wait(bar(B_QFULL + 1), 0, SITE_DRAIN);
    }
    __syncwarp();
  } else if (warp == 9) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t kIdQK = idesc_bf16_f32(128, 128, false);
      constexpr uint32_t kIdPV = idesc_bf16_f32(128, 128, true);
      auto issue_qk = [&](int t, int s) {
        const uint32_t qa = sbase + kOffQ + t * kTileBytes;
        const uint32_t ka = sbase + kOffKV + s * kTileBytes;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint32_t off = (kk >> 2) * kHalfBytes + (kk & 3) * 32;
          umma_ss(tmem + colS(t), sdesc_sw128(qa + off, 16, 1024), sdesc_sw128(ka + off, 16, 1024), kIdQK,
                  kk > 0 ? 1u : 0u);
        }
      };
      auto issue_pv = [&](int t, int s, bool acc) {
        const uint32_t va = sbase + kOffKV + s * kTileBytes;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          umma_ts(tmem + colO(t), tmem + colS(t) + kk * 8, sdesc_sw128(va + kk * 2048, kHalfBytes, 1024), kIdPV,
                  (acc || kk > 0) ? 1u : 0u);
        }
      };
      auto wait_k = [&](int i) -> bool {
        const int s = i % kStages, r = i / kStages;
        return mbar_wait(bar((rope_k ? B_KREADY : B_KVFULL) + s), r & 1, SITE_MMA);
      };
      bool ok = mbar_wait(bar(B_QREADY + 0), 0, SITE_MMA) && mbar_wait(bar(B_QREADY + 1), 0, SITE_MMA);
      if (ok) ok = wait_k(0);
      if (ok) {
        tc_fence_after();
        issue_qk(0, 0);
        umma_commit(bar(B_SFULL + 0));
        issue_qk(1, 0);
        umma_commit(bar(B_SFULL + 1));
        umma_commit(bar(B_KVEMPTY + 0));
      }
      for (int j = 0; ok && j < n_kv; ++j) {
        const int iv = 2 * j + 1, sv = iv % kStages;
        const int ik = 2 * j + 2, sk = ik % kStages;
        const bool more = (j + 1) < n_kv;
        ok = mbar_wait(bar(B_KVFULL + sv), (iv / kStages) & 1, SITE_MMA) &&
             mbar_wait(bar(B_PREADY + 0), j & 1, SITE_MMA);
        if (!ok) break;
        tc_fence_after();
        issue_pv(0, sv, j > 0);
        umma_commit(bar(B_ODONE + 0));
        if (more) {
          ok = wait_k(ik);
          if (!ok) break;
          tc_fence_after();
          issue_qk(0, sk);
          umma_commit(bar(B_SFULL + 0));
        }
        ok = mbar_wait(bar(B_PREADY + 1), j & 1, SITE_MMA);
        if (!ok) break;
        tc_fence_after();
        issue_pv(1, sv, j > 0);
        umma_commit(bar(B_ODONE + 1));
        umma_commit(bar(B_KVEMPTY + sv));
        if (more) {
          issue_qk(1, sk);
          umma_commit(bar(B_SFULL + 1));
          umma_commit(bar(B_KVEMPTY + sk));
        }
      }
      umma_commit(bar(B_DRAIN));
      mbar_wait(bar(B_DRAIN), 0, SITE_DRAIN);
    }
    __syncwarp();
  } else if (warp >= 10) {
    // ------------------------------------------------------------ RoPE of K tiles
    if (rope_k) {
      const int tid = threadIdx.x - 320;  // 0..63
      for (int j = 0; j < n_kv; ++j) {
        const int i = 2 * j, s = i % kStages, r = i / kStages;
        if (!mbar_wait(bar(B_KVFULL + s), r & 1, SITE_ROPEK)) break;
        uint8_t* tile = smem + kOffKV + s * kTileBytes;
#pragma unroll 1
        for (int rr = tid; rr < kBN; rr += 64) {
          const int key = j * kBN + rr;
          if (key < p.S) rope_row_smem(tile, rr, p.cos + static_cast<size_t>(key) * kD, p.sin + static_cast<size_t>(key) * kD);
        }
        fence_proxy_async_smem();
        mbar_arrive(bar(B_KREADY + s));
      }
    }
  } else {
    // ------------------------------------------------------------ softmax warpgroups
    const int t = warp >> 2;             // Q tile
    const int r = threadIdx.x & 127;     // row in tile == TMEM lane
    const uint32_t lane_off = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const uint32_t tS = tmem + lane_off + colS(t);
    const uint32_t tO = tmem + lane_off + colO(t);
    const int p0 = cta_p0 + t * kRowsPerHead;
    const int qpos = p0 + (r & (kRowsPerHead - 1));
    uint8_t* qtile = smem + kOffQ + t * kTileBytes;
    const float sl2 = p.scale_log2;

    bool ok = mbar_wait(bar(B_QFULL + t), 0, SITE_SOFTMAX);
    if (ok && rope_q && qpos < p.S)
      rope_row_smem(qtile, r, p.cos + static_cast<size_t>(qpos) * kD, p.sin + static_cast<size_t>(qpos) * kD);
    fence_proxy_async_smem();
    mbar_arrive(bar(B_QREADY + t));
    ok = __all_sync(0xffffffffu, ok);

    // last key this row may attend
    const int lim = causal ? min(qpos, p.S - 1) : p.S - 1;
    float m_run = -INFINITY, l_run = 0.0f;
    for (int j = 0; ok && j < n_kv; ++j) {
      ok = __all_sync(0xffffffffu, mbar_wait(bar(B_SFULL + t), j & 1, SITE_SOFTMAX));
      if (!ok) break;
      tc_fence_after();
      uint32_t s0[32], s1[32], s2[32], s3[32];
      tmem_ld32(tS + 0, s0);
      tmem_ld32(tS + 32, s1);
      tmem_ld32(tS + 64, s2);
      tmem_ld32(tS + 96, s3);
      tmem_wait_ld_dep(s0);
      reg_dep(s1);
      reg_dep(s2);
      reg_dep(s3);
      const int key0 = j * kBN;
      const int rel = lim - key0;  // columns > rel are masked
      if (rel < kBN - 1) {
#pragma unroll
        for (int k = 0; k < 32; ++k) {
          if (k > rel) s0[k] = 0xFF800000u;
          if (k + 32 > rel) s1[k] = 0xFF800000u;
          if (k + 64 > rel) s2[k] = 0xFF800000u;
          if (k + 96 > rel) s3[k] = 0xFF800000u;
        }
      }
      float mx0 = -INFINITY, mx1 = -INFINITY, mx2 = -INFINITY, mx3 = -INFINITY;
#pragma unroll
      for (int k = 0; k < 32; ++k) {
        mx0 = fmaxf(mx0, __uint_as_float(s0[k]));
        mx1 = fmaxf(mx1, __uint_as_float(s1[k]));
        mx2 = fmaxf(mx2, __uint_as_float(s2[k]));
        mx3 = fmaxf(mx3, __uint_as_float(s3[k]));
      }
      const float m_tile = fmaxf(fmaxf(mx0, mx1), fmaxf(mx2, mx3)) * sl2;
      const float m_new = fmaxf(m_run, m_tile);
      const bool need = m_new > m_run + 8.0f;
      const float m_use = need ? m_new : m_run;
      const float alpha = need ? ex2_approx(m_run - m_new) : 1.0f;
      const float moff = (m_use == -INFINITY) ? 0.0f : m_use;

      uint32_t pa[32], pb[32];
      float sum0 = 0.f, sum1 = 0.f, sum2 = 0.f, sum3 = 0.f;
#pragma unroll
      for (int k = 0; k < 32; k += 2) {
        float e0 = ex2_approx(fmaf(__uint_as_float(s0[k]), sl2, -moff));
        float e1 = ex2_approx(fmaf(__uint_as_float(s0[k + 1]), sl2, -moff));
        float e2 = ex2_approx(fmaf(__uint_as_float(s1[k]), sl2, -moff));
        float e3 = ex2_approx(fmaf(__uint_as_float(s1[k + 1]), sl2, -moff));
        float e4 = ex2_approx(fmaf(__uint_as_float(s2[k]), sl2, -moff));
        float e5 = ex2_approx(fmaf(__uint_as_float(s2[k + 1]), sl2, -moff));
        float e6 = ex2_approx(fmaf(__uint_as_float(s3[k]), sl2, -moff));
        float e7 = ex2_approx(fmaf(__uint_as_float(s3[k + 1]), sl2, -moff));
        const uint32_t w0 = pack_bf16x2(e0, e1), w1 = pack_bf16x2(e2, e3);
        const uint32_t w2 = pack_bf16x2(e4, e5), w3 = pack_bf16x2(e6, e7);
        pa[k >> 1] = w0;
        pa[16 + (k >> 1)] = w1;
        pb[k >> 1] = w2;
        pb[16 + (k >> 1)] = w3;
        // the row sum uses the bf16 values PV multiplies, so O / l normalises exactly them
        sum0 += bf16_lo(w0) + bf16_hi(w0);
        sum1 += bf16_lo(w1) + bf16_hi(w1);
        sum2 += bf16_lo(w2) + bf16_hi(w2);
        sum3 += bf16_lo(w3) + bf16_hi(w3);
      }
      tmem_st32(tS + 0, pa);
      tmem_st32(tS + 32, pb);

      if (j > 0 && __any_sync(0xffffffffu, need)) {
        // O_t must be quiescent: PV of the previous tile finished.
        ok = __all_sync(0xffffffffu, mbar_wait(bar(B_ODONE + t), (j - 1) & 1, SITE_SOFTMAX));
        if (ok) {
          tc_fence_after();
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
      }
      tmem_wait_st();
      l_run = l_run * alpha + ((sum0 + sum1) + (sum2 + sum3));
      m_run = m_use;
      tc_fence_before();
      mbar_arrive(bar(B_PREADY + t));
    }

    // ---- epilogue: O / l -> bf16 -> (reuse the Q tile smem) -> TMA store
    if (ok) ok = __all_sync(0xffffffffu, mbar_wait(bar(B_ODONE + t), (n_kv - 1) & 1, SITE_EPILOGUE));
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
          const int dc = c * 4 + q;    // chunk index over d (0..15)
          uint4 v;
          v.x = pack_bf16x2(__uint_as_float(o[q * 8 + 0]) * inv_l, __uint_as_float(o[q * 8 + 1]) * inv_l);
          v.y = pack_bf16x2(__uint_as_float(o[q * 8 + 2]) * inv_l, __uint_as_float(o[q * 8 + 3]) * inv_l);
          v.z = pack_bf16x2(__uint_as_float(o[q * 8 + 4]) * inv_l, __uint_as_float(o[q * 8 + 5]) * inv_l);
          v.w = pack_bf16x2(__uint_as_float(o[q * 8 + 6]) * inv_l, __uint_as_float(o[q * 8 + 7]) * inv_l);
          const int cb = dc >> 3, ch = dc & 7;
          *reinterpret_cast<uint4*>(qtile + cb * kHalfBytes + r * 128 + ((ch ^ (r & 7)) << 4)) = v;
        }
      }
    }
    fence_proxy_async_smem();
    named_bar_sync(1 + t, 128);
    if (ok && r == 0 && p0 < p.S) {  // a tile starting past the sequence has nothing to store
      const uint32_t src = sbase + kOffQ + t * kTileBytes;
      tma_store_3d(&tmO, src, 0, p0, zq);
      tma_store_3d(&tmO, src + kHalfBytes, 64, p0, zq);
      bulk_commit();
      bulk_wait0();
    }
  }

  // ---- teardown: everyone done with TMEM and shared memory
  tc_fence_before();
  named_bar_sync(3, kThreads);
  if (warp == 9) {
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
  const long long grid = n_qblocks * B * kv_count;
  if (grid > 0x7FFFFFFFLL || static_cast<long long>(B) * Hq > 0x7FFFFFFFLL) return GQA_ERR_UNSUPPORTED;

  CUtensorMap tmQ, tmK, tmV, tmO;
  int rc;
  if ((rc = make_tmap_3d_bf16(&tmQ, q, kD, S, static_cast<long long>(B) * Hq, 64, kRowsPerHead, kG)) != GQA_OK) return rc;
  if ((rc = make_tmap_3d_bf16(&tmK, k, kD, S, static_cast<long long>(B) * Hkv, 64, kBN, 1)) != GQA_OK) return rc;
  if ((rc = make_tmap_3d_bf16(&tmV, v, kD, S, static_cast<long long>(B) * Hkv, 64, kBN, 1)) != GQA_OK) return rc;
  if ((rc = make_tmap_3d_bf16(&tmO, o, kD, S, static_cast<long long>(B) * Hq, 64, kRowsPerHead, kG)) != GQA_OK) return rc;

  static std::atomic<uint64_t> attr_done{0};
  if ((rc = ensure_smem_attr(prefill_kernel, kSmemBytes, attr_done)) != GQA_OK) return rc;
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
  prefill_kernel<<<static_cast<unsigned>(grid), kThreads, kSmemBytes, stream>>>(tmQ, tmK, tmV, tmO, p);
  return cudaGetLastError() == cudaSuccess ? GQA_OK : GQA_ERR_CUDA;
}

}  // namespace gqa
