// decode_sm100.cu -- split-KV GQA decode on the sm_100a tensor core (persistent CTAs).
//
// out[b,h,:] = softmax_j(q[b,h] . K[b,h/4,j] * scale, j < lens[b]) . V[b,h/4,:,:]
// This is the single-query-row case of the reference's core
// (CPU_Baseline/cpu_baseline/attention.py:60-84); the reference has no decode
// function of its own.  The path is HBM-bound: every K/V byte is read once.
//
// Work items: (sequence b, kv head g, segment of split_len keys).  One CTA per SM
// walks items blockIdx.x, blockIdx.x + gridDim.x, ...; inside an item the keys are
// consumed in 128-key chunks that a TMA producer streams through a 3-stage ring
// (K and V of a chunk: 64 KB per stage).  Per chunk the tensor core computes
//   S^T[key][head] = K_chunk . Q^T      (M = 128 keys, N = 16: the group's 4 heads, rest 0)
//   O^T[dim][head] += V_chunk^T . P     (M = 128 dims, V as an MN-major operand)
// in TMEM; one softmax warpgroup (thread = key for S^T, = dim for O^T) keeps the
// per-head running max / sum (lazy rescaling) and writes P (bf16) to shared memory.
// Each item leaves (O unnormalised, m, l) per head in the workspace; a second kernel
// merges an item's segments with a log-sum-exp combine.
#include <cuda.h>

#include "common.cuh"
#include "gqa_internal.h"

namespace gqa {
namespace decode2 {

constexpr int kD = 128;
constexpr int kG = 4;
constexpr int kChunk = 128;                    // keys per chunk
constexpr int kStages = 3;
constexpr int kHalfBytes = kChunk * 64 * 2;    // one 64-dim block of a K or V chunk: 16 KB
constexpr int kKVBytes = 2 * kHalfBytes;       // K (or V) chunk: 32 KB
constexpr int kStageBytes = 2 * kKVBytes;      // K + V
constexpr int kNPad = 16;                      // MMA N: 4 heads padded to 16
constexpr int kSmallHalf = kNPad * 128;        // 16 rows x 128 B: one 64-column block of Q^T / P
constexpr int kSmallBytes = 2 * kSmallHalf;    // 4 KB
constexpr int kThreads = 256;                  // warp 0 producer, warp 1 MMA, warps 4-7 softmax
constexpr float kRescaleLog2 = 16.0f;

constexpr int kOffKV = 0;
constexpr int kOffQ = kOffKV + kStages * kStageBytes;
constexpr int kOffP = kOffQ + kSmallBytes;             // [2] buffers
constexpr int kOffBar = kOffP + 2 * kSmallBytes;
constexpr int kNumBars = 24;
constexpr int kOffRed = kOffBar + kNumBars * 8;        // [2][4 warps][4 heads] floats
constexpr int kOffTmemPtr = kOffRed + 2 * 4 * 4 * 4;
constexpr int kSmemBytes = kOffTmemPtr + 16;
static_assert(kSmemBytes <= 232448, "shared memory over the per-block limit");

enum : int {
  B_KVFULL = 0,   // [3]
  B_KVEMPTY = 3,  // [3]
  B_QREADY = 6,   // [1] q of the current item in smem (128 arrivals)
  B_SFULL = 7,    // [2] S^T buffer complete
  B_SFREE = 9,    // [2] S^T buffer copied to registers (128 arrivals)
  B_PREADY = 11,  // [2] P buffer written (and O rescaled) (128 arrivals)
  B_PVDONE = 13,  // [2] PV that read P buffer complete
  B_DRAIN = 15,
};

enum : int {
  SITE_PRODUCER = 0x201,
  SITE_MMA = 0x202,
  SITE_SOFTMAX = 0x203,
  SITE_DRAIN = 0x204,
  SITE_SMEM_ALIGN = 0x205,
  SITE_BAD_PAGE = 0x601,  // a block-table entry outside [0, num_pages) (input error)
};

struct Params {
  const uint16_t* q;
  const int32_t* lens;
  const int32_t* q_pos;
  const uint16_t* cos;
  const uint16_t* sin;
  float* ws_o;   // [B][Hq][n_splits][128]
  float* ws_ml;  // [B][Hq][n_splits][2]
  uint16_t* out; // [B][Hq][128]
  // Paged cache (table != nullptr): K/V pages [num_pages][Hkv][page_size][128]; key j of
  // sequence b lives in page table[b * max_pages + j / page_size], row j % page_size.
  const int32_t* table;
  int page_size, max_pages, num_pages;
  int B, Lmax, Hq, Hkv, kv_begin, kv_count, n_splits, split_len, flags;
  float scale_log2;
};

__device__ __forceinline__ void tmem_ld4(uint32_t taddr, uint32_t (&r)[4]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait_ld4(uint32_t (&r)[4]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;" : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3])::"memory");
}
__device__ __forceinline__ void tmem_st4(uint32_t taddr, const uint32_t (&r)[4]) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x4.b32 [%0], {%1,%2,%3,%4};" ::"r"(taddr), "r"(r[0]), "r"(r[1]),
               "r"(r[2]), "r"(r[3])
               : "memory");
}

// Byte offset of element (row, col) in a [16 rows][128 cols] bf16 K-major SW128 tile.
__device__ __forceinline__ int small_off(int row, int col) {
  return (col >> 6) * kSmallHalf + row * 128 + ((((col & 63) >> 3) ^ (row & 7)) << 4) + (col & 7) * 2;
}

struct Item {
  int b, g, seg, k0, k1, nchunks;
};

// Decode work item `it` (b-major, then kv head, then segment); nchunks = 0 if empty.
__device__ __forceinline__ Item item_of(const Params& p, long long it) {
  Item x;
  x.seg = static_cast<int>(it % p.n_splits);
  const long long bg = it / p.n_splits;
  x.g = p.kv_begin + static_cast<int>(bg % p.kv_count);
  x.b = static_cast<int>(bg / p.kv_count);
  const int len = min(max(p.lens[x.b], 0), p.Lmax);
  x.k0 = x.seg * p.split_len;
  x.k1 = min(x.k0 + p.split_len, len);
  x.nchunks = x.k1 > x.k0 ? (x.k1 - x.k0 + kChunk - 1) / kChunk : 0;
  return x;
}

__global__ void __launch_bounds__(kThreads, 1)
    decode_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV, const Params p) {
  extern __shared__ __align__(1024) uint8_t smem[];
  if (smem_u32(smem) & 1023u) {
    if (threadIdx.x == 0) record_error(SITE_SMEM_ALIGN);
    return;
  }
  const uint32_t sbase = smem_u32(smem);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  auto bar = [&](int i) -> uint32_t { return sbase + kOffBar + 8 * i; };
  const long long n_items = static_cast<long long>(p.B) * p.kv_count * p.n_splits;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(bar(B_KVFULL + s), 1);
      mbar_init(bar(B_KVEMPTY + s), 1);
    }
    mbar_init(bar(B_QREADY), 128);
    for (int b = 0; b < 2; ++b) {
      mbar_init(bar(B_SFULL + b), 1);
      mbar_init(bar(B_SFREE + b), 128);
      mbar_init(bar(B_PREADY + b), 128);
      mbar_init(bar(B_PVDONE + b), 1);
    }
    mbar_init(bar(B_DRAIN), 1);
    fence_mbar_init();
  }
  // Q^T and both P tiles start as zeros: rows 4..15 (padding heads) stay zero.
  for (int i = threadIdx.x; i < 3 * kSmallBytes / 16; i += kThreads)
    reinterpret_cast<uint4*>(smem + kOffQ)[i] = make_uint4(0, 0, 0, 0);
  fence_proxy_async_smem();
  if (warp == 1) {
    tmem_alloc(sbase + kOffTmemPtr, 64);
    tmem_relinquish();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(smem + kOffTmemPtr);
  // TMEM columns: S^T buffers at 0 and 16 (16 each), O^T at 32
  constexpr uint32_t kColO = 32u;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      bool ok = true;
      long long c = 0;  // global chunk counter of this CTA
      for (long long it = blockIdx.x; ok && it < n_items; it += gridDim.x) {
        const Item x = item_of(p, it);
        for (int ch = 0; ch < x.nchunks; ++ch, ++c) {
          const int s = static_cast<int>(c % kStages);
          const long long r = c / kStages;
          if (r > 0) ok = mbar_wait(bar(B_KVEMPTY + s), static_cast<uint32_t>((r - 1) & 1), SITE_PRODUCER);
          if (!ok) break;
          const uint32_t dst = sbase + kOffKV + s * kStageBytes;
          int key0 = x.k0 + ch * kChunk;
          int z = x.b * p.Hkv + x.g;
          if (p.table) {  // 128-key chunks never straddle a page (page_size, split % 128 == 0)
            int page = __ldg(p.table + static_cast<size_t>(x.b) * p.max_pages + key0 / p.page_size);
            if (page < 0 || page >= p.num_pages) {
              record_input_error(SITE_BAD_PAGE);
              page = 0;  // keep the pipeline flowing; the call reports the input error
            }
            z = page * p.Hkv + x.g;
            key0 %= p.page_size;
          }
          mbar_expect_tx(bar(B_KVFULL + s), kStageBytes);
          tma_load_3d(dst, &tmK, bar(B_KVFULL + s), 0, key0, z);
          tma_load_3d(dst + kHalfBytes, &tmK, bar(B_KVFULL + s), 64, key0, z);
          tma_load_3d(dst + kKVBytes, &tmV, bar(B_KVFULL + s), 0, key0, z);
          tma_load_3d(dst + kKVBytes + kHalfBytes, &tmV, bar(B_KVFULL + s), 64, key0, z);
        }
      }
      // drain: every issued load must land before the CTA exits
      for (long long i = c > kStages ? c - kStages : 0; i < c; ++i)
        mbar_wait_drain(bar(B_KVFULL + static_cast<int>(i % kStages)), static_cast<uint32_t>((i / kStages) & 1), SITE_DRAIN);
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t kIdQK = idesc_bf16_f32(128, kNPad, false);
      constexpr uint32_t kIdPV = idesc_bf16_f32(128, kNPad, false) | (1u << 15);  // A (V^T) MN-major
      constexpr uint32_t kHi = sdesc_hi_sw128(1024);
      const uint32_t kv_lo = sdesc_lo(sbase + kOffKV, 16);
      const uint32_t vt_lo = sdesc_lo(sbase + kOffKV + kKVBytes, kHalfBytes);
      const uint32_t q_lo = sdesc_lo(sbase + kOffQ, 16);
      const uint32_t p_lo = sdesc_lo(sbase + kOffP, 16);
      auto issue_qk = [&](int s, int bb) {  // S^T[bb] = K_s . Q^T
        const uint32_t a0 = kv_lo + s * (kStageBytes / 16);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          umma_ss_lohi(tmem + 16u * bb, a0 + ((kk >> 2) * kHalfBytes + (kk & 3) * 32) / 16,
                       q_lo + ((kk >> 2) * kSmallHalf + (kk & 3) * 32) / 16, kHi, kIdQK, kk > 0 ? 1u : 0u);
      };
      auto issue_pv = [&](int s, int bb, uint32_t acc) {  // O^T (+)= V_s^T . P[bb]
        const uint32_t a0 = vt_lo + s * (kStageBytes / 16);
        const uint32_t b0 = p_lo + bb * (kSmallBytes / 16);
        umma_ss_lohi(tmem + kColO, a0, b0, kHi, kIdPV, acc);
#pragma unroll
        for (int kk = 1; kk < 8; ++kk)
          umma_ss_lohi(tmem + kColO, a0 + kk * (2048 / 16), b0 + ((kk >> 2) * kSmallHalf + (kk & 3) * 32) / 16, kHi,
                       kIdPV, 1u);
      };
      bool ok = true;
      long long c = 0, item_idx = 0;
      int pend_s = -1, pend_b = 0;  // PV of the previous chunk, not yet issued
      uint32_t pend_acc = 0;
      long long pend_c = -1;
      auto flush_pv = [&]() -> bool {
        if (pend_s < 0) return true;
        if (!mbar_wait_spin(bar(B_PREADY + pend_b), static_cast<uint32_t>((pend_c >> 1) & 1), SITE_MMA)) return false;
        tc_fence_after();
        issue_pv(pend_s, pend_b, pend_acc);
        umma_commit(bar(B_PVDONE + pend_b));
        umma_commit(bar(B_KVEMPTY + pend_s));
        pend_s = -1;
        return true;
      };
      for (long long it = blockIdx.x; ok && it < n_items; it += gridDim.x) {
        const Item x = item_of(p, it);
        if (x.nchunks == 0) continue;
        // close the previous item first: its epilogue (and the new q) wait on this PV
        ok = flush_pv() && mbar_wait_spin(bar(B_QREADY), static_cast<uint32_t>(item_idx & 1), SITE_MMA);
        ++item_idx;
        for (int ch = 0; ok && ch < x.nchunks; ++ch, ++c) {
          const int s = static_cast<int>(c % kStages), bb = static_cast<int>(c & 1);
          ok = mbar_wait_spin(bar(B_KVFULL + s), static_cast<uint32_t>((c / kStages) & 1), SITE_MMA);
          if (ok && c >= 2) ok = mbar_wait_spin(bar(B_SFREE + bb), static_cast<uint32_t>(((c - 2) >> 1) & 1), SITE_MMA);
          if (!ok) break;
          tc_fence_after();
          issue_qk(s, bb);
          umma_commit(bar(B_SFULL + bb));
          ok = flush_pv();  // PV of the previous chunk overlaps this chunk's softmax
          pend_s = s;
          pend_b = bb;
          pend_acc = ch > 0 ? 1u : 0u;
          pend_c = c;
        }
      }
      if (ok) flush_pv();
      umma_commit(bar(B_DRAIN));
      mbar_wait_drain(bar(B_DRAIN), 0, SITE_DRAIN);
    }
    __syncwarp();
  } else if (warp >= 4) {
    // ------------------------------------------------------------ softmax warpgroup
    const int i = threadIdx.x - 128;  // key lane of S^T, dim lane of O^T
    const uint32_t lane_off = static_cast<uint32_t>((warp & 3) * 32) << 16;
    float* red = reinterpret_cast<float*>(smem + kOffRed);  // [2][4 warps][4 heads]
    const int wq = warp & 3;
    const float sl2 = p.scale_log2;
    bool ok = true;
    long long c = 0;
    int red_par = 0;
    for (long long it = blockIdx.x; it < n_items; it += gridDim.x) {
      const Item x = item_of(p, it);
      if (x.nchunks == 0) continue;
      // ---- q of the group's 4 heads -> Q^T tile (optionally rotated at q_pos[b])
      if (i < 64) {
        const size_t qbase = (static_cast<size_t>(x.b) * p.Hq + x.g * kG) * kD;
        const size_t row = (p.flags & GQA_FLAG_ROPE_Q) ? static_cast<size_t>(min(max(p.q_pos[x.b], 0), p.Lmax)) * kD : 0;
#pragma unroll
        for (int h = 0; h < kG; ++h) {
          const uint16_t* qr = p.q + qbase + h * kD;
          uint16_t y0 = qr[i], y1 = qr[i + 64];
          if (p.flags & GQA_FLAG_ROPE_Q) {
            const float x0 = bf2f_bits(y0), x1 = bf2f_bits(y1);
            const float cs = bf2f_bits(p.cos[row + i]), sn = bf2f_bits(p.sin[row + i]);
            y0 = f2bf_bits(__fadd_rn(__fmul_rn(x0, cs), __fmul_rn(-x1, sn)));
            y1 = f2bf_bits(__fadd_rn(__fmul_rn(x1, cs), __fmul_rn(x0, sn)));
          }
          *reinterpret_cast<uint16_t*>(smem + kOffQ + small_off(h, i)) = y0;
          *reinterpret_cast<uint16_t*>(smem + kOffQ + small_off(h, i + 64)) = y1;
        }
      }
      fence_proxy_async_smem();
      mbar_arrive(bar(B_QREADY));

      float m_run[kG], l_part[kG];
#pragma unroll
      for (int h = 0; h < kG; ++h) {
        m_run[h] = -INFINITY;
        l_part[h] = 0.0f;
      }
      long long c_last = c;
      for (int ch = 0; ch < x.nchunks; ++ch, ++c) {
        const int bb = static_cast<int>(c & 1);
        uint32_t sv[4] = {0xFF800000u, 0xFF800000u, 0xFF800000u, 0xFF800000u};
        if (ok) ok = __all_sync(0xffffffffu, mbar_wait(bar(B_SFULL + bb), static_cast<uint32_t>((c >> 1) & 1), SITE_SOFTMAX));
        if (ok) {
          tc_fence_after();
          tmem_ld4(tmem + lane_off + 16u * bb, sv);
          tmem_wait_ld4(sv);
          tc_fence_before();
          mbar_arrive(bar(B_SFREE + bb));
        }
        const int key = x.k0 + ch * kChunk + i;
        float sc[kG], mw[kG];
#pragma unroll
        for (int h = 0; h < kG; ++h) {
          sc[h] = key < x.k1 ? __uint_as_float(sv[h]) : -INFINITY;
          float v = sc[h];
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
          mw[h] = v;
        }
        if (lane == 0) {
#pragma unroll
          for (int h = 0; h < kG; ++h) red[(red_par * 4 + wq) * 4 + h] = mw[h];
        }
        named_bar_sync(1, 128);
        float alpha[kG], moff[kG];
        bool need_any = false;
#pragma unroll
        for (int h = 0; h < kG; ++h) {
          const float* rr = red + red_par * 16;
          const float mt = fmaxf(fmaxf(rr[h], rr[4 + h]), fmaxf(rr[8 + h], rr[12 + h])) * sl2;
          const float m_new = fmaxf(m_run[h], mt);
          const bool need = m_new > m_run[h] + kRescaleLog2;  // CTA-uniform
          const float m_use = need ? m_new : m_run[h];
          alpha[h] = need ? ex2_approx(m_run[h] - m_new) : 1.0f;
          moff[h] = (m_use == -INFINITY) ? 0.0f : m_use;
          m_run[h] = m_use;
          need_any |= need && ch > 0;
        }
        red_par ^= 1;
        // P buffer bb is free once the PV of chunk c-2 finished
        if (ok && c - c_last >= 2)
          ok = __all_sync(0xffffffffu, mbar_wait(bar(B_PVDONE + bb), static_cast<uint32_t>(((c - 2) >> 1) & 1), SITE_SOFTMAX));
        if (ok && x.k0 + (ch + 1) * kChunk > x.k1) {
          // Partial chunk: rows of V past the segment end get P = 0, but 0 * NaN would
          // still poison O (a cache is not required to hold finite values past lens[b]),
          // so those rows are zeroed before the PV reads them.  Waiting on the stage's
          // full barrier makes the TMA bytes visible to this thread first; the stage
          // cannot be refilled before PREADY of this chunk, so the parity is unambiguous.
          const int s = static_cast<int>(c % kStages);
          ok = __all_sync(0xffffffffu, mbar_wait(bar(B_KVFULL + s), static_cast<uint32_t>((c / kStages) & 1),
                                                 SITE_SOFTMAX));
          if (ok && key >= x.k1) {
            uint4* v0 = reinterpret_cast<uint4*>(smem + kOffKV + s * kStageBytes + kKVBytes + i * 128);
            uint4* v1 = reinterpret_cast<uint4*>(smem + kOffKV + s * kStageBytes + kKVBytes + kHalfBytes + i * 128);
#pragma unroll
            for (int k = 0; k < 8; ++k) {
              v0[k] = make_uint4(0u, 0u, 0u, 0u);
              v1[k] = make_uint4(0u, 0u, 0u, 0u);
            }
          }
        }
        if (ok) {
#pragma unroll
          for (int h = 0; h < kG; ++h) {
            const float e = ex2_approx(fmaf(sc[h], sl2, -moff[h]));
            const uint16_t w = f2bf_bits(e);
            l_part[h] = l_part[h] * alpha[h] + bf2f_bits(w);
            *reinterpret_cast<uint16_t*>(smem + kOffP + bb * kSmallBytes + small_off(h, i)) = w;
          }
          fence_proxy_async_smem();
          if (need_any) {  // O^T row i (dim i) *= alpha per head, after the PV of chunk c-1
            ok = __all_sync(0xffffffffu, mbar_wait(bar(B_PVDONE + (bb ^ 1)), static_cast<uint32_t>(((c - 1) >> 1) & 1),
                                                   SITE_SOFTMAX));
            if (ok) {
              tc_fence_after();
              uint32_t o[4];
              tmem_ld4(tmem + lane_off + kColO, o);
              tmem_wait_ld4(o);
#pragma unroll
              for (int h = 0; h < kG; ++h) o[h] = __float_as_uint(__uint_as_float(o[h]) * alpha[h]);
              tmem_st4(tmem + lane_off + kColO, o);
              tmem_wait_st();
            }
          }
          tc_fence_before();
          mbar_arrive(bar(B_PREADY + bb));
        } else {
#pragma unroll
          for (int h = 0; h < kG; ++h) l_part[h] *= alpha[h];
        }
      }
      // ---- item epilogue: wait for the last PV, reduce l, write the partial
      const long long cl = c - 1;
      if (ok) ok = __all_sync(0xffffffffu, mbar_wait(bar(B_PVDONE + static_cast<int>(cl & 1)),
                                                      static_cast<uint32_t>((cl >> 1) & 1), SITE_SOFTMAX));
      float lw[kG];
#pragma unroll
      for (int h = 0; h < kG; ++h) {
        float v = l_part[h];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        lw[h] = v;
      }
      if (lane == 0) {
#pragma unroll
        for (int h = 0; h < kG; ++h) red[(red_par * 4 + wq) * 4 + h] = lw[h];
      }
      named_bar_sync(1, 128);
      uint32_t o[4] = {0u, 0u, 0u, 0u};
      if (ok) {
        tc_fence_after();
        tmem_ld4(tmem + lane_off + kColO, o);
        tmem_wait_ld4(o);
      }
      const float* rr = red + red_par * 16;
#pragma unroll
      for (int h = 0; h < kG; ++h) {
        const size_t slot = (static_cast<size_t>(x.b) * p.Hq + x.g * kG + h) * p.n_splits + x.seg;
        p.ws_o[slot * kD + i] = __uint_as_float(o[h]);
        if (i == 0) {
          p.ws_ml[slot * 2 + 0] = m_run[h];
          p.ws_ml[slot * 2 + 1] = rr[h] + rr[4 + h] + rr[8 + h] + rr[12 + h];
        }
      }
      red_par ^= 1;
      tc_fence_before();
    }
  }

  // ---- teardown
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 64);
  }
}

// grid = (kv_count*4 heads, B); block = 128 threads (thread = dim).
__global__ void __launch_bounds__(kD) combine_kernel(const Params p) {
  const int b = blockIdx.y;
  const int h = p.kv_begin * kG + static_cast<int>(blockIdx.x);
  const int len = min(max(p.lens[b], 0), p.Lmax);
  const int ns = (len + p.split_len - 1) / p.split_len;
  const size_t base = (static_cast<size_t>(b) * p.Hq + h) * p.n_splits;
  float M = -INFINITY;
  for (int s = 0; s < ns; ++s) M = fmaxf(M, p.ws_ml[(base + s) * 2]);
  float L = 0.0f, acc = 0.0f;
  for (int s = 0; s < ns; ++s) {
    const float m = p.ws_ml[(base + s) * 2];
    const float w = (m == -INFINITY) ? 0.0f : ex2_approx(m - M);
    L += p.ws_ml[(base + s) * 2 + 1] * w;
    acc += p.ws_o[(base + s) * kD + threadIdx.x] * w;
  }
  p.out[(static_cast<size_t>(b) * p.Hq + h) * kD + threadIdx.x] = f2bf_bits(L > 0.0f ? acc / L : 0.0f);
}

}  // namespace decode2

int launch_decode_tc(const void* q, const void* kcache, const void* vcache, const int32_t* lens, const int32_t* q_pos,
                     const void* cos, const void* sin, void* o, float* ws, int B, int max_len, int Hq, int Hkv,
                     int kv_begin, int kv_count, int split_len, int n_splits, float scale, int flags,
                     cudaStream_t stream, const int32_t* table, int page_size, int max_pages, int num_pages) {
  using namespace decode2;
  CUtensorMap tmK, tmV;
  int rc;
  // contiguous: rows (B*Hkv) x max_len keys; paged: rows (num_pages*Hkv) x page_size keys
  const int rows_per_z = table ? page_size : max_len;
  const long long nz = table ? static_cast<long long>(num_pages) * Hkv : static_cast<long long>(B) * Hkv;
  if ((rc = make_tmap_3d_bf16(&tmK, kcache, kD, rows_per_z, nz, 64, kChunk, 1)) != GQA_OK) return rc;
  if ((rc = make_tmap_3d_bf16(&tmV, vcache, kD, rows_per_z, nz, 64, kChunk, 1)) != GQA_OK) return rc;
  static std::atomic<uint64_t> attr_done{0};
  if ((rc = ensure_smem_attr(decode_kernel, kSmemBytes, attr_done)) != GQA_OK) return rc;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  Params p;
  p.q = static_cast<const uint16_t*>(q);
  p.lens = lens;
  p.q_pos = q_pos;
  p.cos = static_cast<const uint16_t*>(cos);
  p.sin = static_cast<const uint16_t*>(sin);
  const size_t n_slots = static_cast<size_t>(B) * Hq * n_splits;
  p.ws_o = ws;
  p.ws_ml = ws + n_slots * kD;
  p.out = static_cast<uint16_t*>(o);
  p.table = table;
  p.page_size = page_size;
  p.max_pages = max_pages;
  p.num_pages = num_pages;
  p.B = B;
  p.Lmax = max_len;
  p.Hq = Hq;
  p.Hkv = Hkv;
  p.kv_begin = kv_begin;
  p.kv_count = kv_count;
  p.n_splits = n_splits;
  p.split_len = split_len;
  p.flags = flags;
  p.scale_log2 = scale * 1.4426950408889634f;
  const long long n_items = static_cast<long long>(B) * kv_count * n_splits;
  const int grid = static_cast<int>(n_items < sms ? n_items : sms);
  decode_kernel<<<grid, kThreads, kSmemBytes, stream>>>(tmK, tmV, p);
  if (cudaGetLastError() != cudaSuccess) return GQA_ERR_CUDA;
  combine_kernel<<<dim3(kv_count * kG, B), kD, 0, stream>>>(p);
  return cudaGetLastError() == cudaSuccess ? GQA_OK : GQA_ERR_CUDA;
}

}  // namespace gqa

namespace gqa {
GQA_ERROR_FLAG_ACCESSOR(error_flag_decode_tc)
}  // namespace gqa
