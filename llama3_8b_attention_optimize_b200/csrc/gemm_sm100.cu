// gemm_sm100.cu -- the attention layer's projections on the sm_100a tensor core.
//
//   C[m, n] = sum_k A[m, k] * W[n, k]        (y = x W^T, HF [out, in] weights)
//
// Used for q/k/v = to_bf16(h @ W^T) (llama3_attention_golden_model.py:149-151) and
// final = to_bf16(attn @ o_proj^T) (:193-194): bf16 operands, fp32 accumulation in
// TMEM, one round-to-nearest-even to bf16 at the end -- or an fp32 result, for the
// row-parallel partial sums that are all-reduced across GPUs before that rounding.
//
// Persistent CTAs (one per SM) walk 128 x BN output tiles, or persistent pairs of CTAs
// (a cluster of two) walk 256 x BN tiles with tcgen05.mma.cta_group::2: each CTA loads
// its 128 rows of A and half of W, the even CTA issues the MMAs, and every MMA commit
// is sent to the barrier of each CTA of the pair.  Warp roles:
//   warp 0     TMA producer: A (128 x 64) and W (BN x 64, pair: BN/2 x 64) k-blocks
//              into a ring (pair: both CTAs' loads complete on the even CTA's barrier)
//   warp 1     MMA issuer: 4 x tcgen05.mma (M=128 or 256, N=BN, K=16) per k-block into
//              one of two TMEM accumulators (the epilogue drains one while the next
//              tile accumulates into the other)
//   warps 2-5  epilogue: tcgen05.ld -> bf16 (or fp32) -> swizzled staging -> TMA store
//
// All global tensors are addressed through 4-D tensor maps (inner, s, outer, batch), so
// one kernel serves three layouts without a transpose pass:
//   row-major A [M][K] and C [M][N];
//   head-major A [B][H][S][128] (the attention output, k = h*128 + d: the
//     transpose(0,1).view(S, -1) of :193 is folded into the load coordinates);
//   head-major outputs [B][H][S][128] (the .view(S,H,128).transpose(0,1) of
//     :153-155), with q/k rotated in the epilogue after the bf16 rounding
//     (to_bf16(apply_rope(to_bf16(h @ W^T))), :149-164).
// The N axis may be split into up to three regions (q, k, v), each with its own
// weight tensor and output map, so the fused projection is a single launch.
#include <cuda.h>

#include "common.cuh"
#include "gqa_internal.h"

namespace gqa {
namespace gemm {

constexpr int kBM = 128;
constexpr int kBK = 64;
constexpr int kThreads = 192;
constexpr int kMaxRegions = 3;
constexpr int kMaxDest = 8;

// kPair: a cluster of two CTAs computes one 256 x BN tile with tcgen05.mma.cta_group::2
// (M = 256): each CTA holds its own 128 rows of A and half (BN / 2 rows) of W's k-block,
// the even CTA issues the MMAs, and each CTA's TMEM receives its 128 rows of the result.
template <int BN, bool kPair>
struct Cfg {
  static constexpr int kWRows = kPair ? BN / 2 : BN;  // W rows this CTA loads per k-block
  static constexpr int kTileM = kPair ? 2 * kBM : kBM;
  static constexpr int kStages = kPair ? 6 : (BN == 256 ? 4 : 6);
  static constexpr int kABytes = kBM * kBK * 2;
  static constexpr int kWBytes = kWRows * kBK * 2;
  static constexpr int kStageBytes = kABytes + kWBytes;
  static constexpr int kBoxBytes = kBM * 128;  // one 128-row x 128-byte store box
  static constexpr int kOffStaging = kStages * kStageBytes;
  static constexpr int kOffBar = kOffStaging + 2 * kBoxBytes;
  static constexpr int kNumBars = 2 * kStages + 4;
  static constexpr int kOffTmemPtr = kOffBar + kNumBars * 8;
  static constexpr int kSmemBytes = kOffTmemPtr + 16;
  static constexpr int kTmemCols = 2 * BN;
  static_assert(kSmemBytes <= 232448, "shared memory over the per-block limit");
  static_assert(kTmemCols <= 512, "two accumulators must fit in TMEM");
};

enum : int {
  SITE_PRODUCER = 0x301,
  SITE_MMA = 0x302,
  SITE_EPILOGUE = 0x303,
  SITE_SMEM_ALIGN = 0x305,
};

struct Region {
  int n0, n1;      // GEMM columns [n0, n1) (multiples of BN, except n1 of the last region)
  int head_major;  // output [B][heads][S][128] (else row-major [M][n1 - n0])
  int rope;        // rotate pairs (d, d + 64) at position pos0 + s after the bf16 rounding
};

struct Params {
  int M, N, K, S;  // rows m = b * S + s
  int a_kin;       // extent of the A map's innermost dimension (K, or 128 for head-major A)
  int tiles_m, tiles_n, n_tiles, n_kb;
  int out_f32;     // fp32 row-major output (one region, no rope)
  int n_regions;
  Region reg[kMaxRegions];
  const uint16_t* cos;  // [pos0 + S][128] bf16 (rope regions only)
  const uint16_t* sin;
  int pos0;
  // Scatter epilogue (scatter_rows > 0, fp32 only): row m goes to dst[m / scatter_rows] +
  // (m % scatter_rows) * N by direct stores (dst may be NVLink peer memory); when the grid
  // is done, the last CTA raises sig_flag[q] = sig_epoch at every destination q.
  int scatter_rows, n_dest;
  float* dst[kMaxDest];
  uint32_t* sig_flag[kMaxDest];
  uint32_t* sig_counter;  // zero between launches
  uint32_t sig_epoch;
};

struct Maps {
  CUtensorMap a;
  CUtensorMap w[kMaxRegions];
  CUtensorMap c[kMaxRegions];
};

__device__ __forceinline__ int region_of(const Params& p, int n0) {
  int r = 0;
  if (p.n_regions > 1 && n0 >= p.reg[1].n0) r = 1;
  if (p.n_regions > 2 && n0 >= p.reg[2].n0) r = 2;
  return r;
}

// Region r without a dynamically indexed parameter array (which would go to local memory).
__device__ __forceinline__ Region region_at(const Params& p, int r) {
  return r == 0 ? p.reg[0] : (r == 1 ? p.reg[1] : p.reg[2]);
}

__device__ __forceinline__ float* dst_at(const Params& p, int q) {
  switch (q) {
    case 0: return p.dst[0];
    case 1: return p.dst[1];
    case 2: return p.dst[2];
    case 3: return p.dst[3];
    case 4: return p.dst[4];
    case 5: return p.dst[5];
    case 6: return p.dst[6];
    default: return p.dst[7];
  }
}
__device__ __forceinline__ uint32_t* flag_at(const Params& p, int q) {
  switch (q) {
    case 0: return p.sig_flag[0];
    case 1: return p.sig_flag[1];
    case 2: return p.sig_flag[2];
    case 3: return p.sig_flag[3];
    case 4: return p.sig_flag[4];
    case 5: return p.sig_flag[5];
    case 6: return p.sig_flag[6];
    default: return p.sig_flag[7];
  }
}

__device__ __forceinline__ const CUtensorMap* pick(const CUtensorMap* m0, const CUtensorMap* m1,
                                                   const CUtensorMap* m2, int r) {
  return r == 0 ? m0 : (r == 1 ? m1 : m2);
}

// ---- CTA-pair helpers (cluster of two CTAs along x)
__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// Address of the same shared-memory location in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t map_to_rank(uint32_t saddr, uint32_t rank) {
  uint32_t d;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(d) : "r"(saddr), "r"(rank));
  return d;
}
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
// Arrive on an mbarrier (any CTA of the pair) once this thread's earlier pair MMAs are done.
__device__ __forceinline__ void umma_commit_pair(uint32_t cluster_addr) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(cluster_addr)
               : "memory");
}
__device__ __forceinline__ void umma_ss_pair(uint32_t d_tmem, uint32_t a_lo, uint32_t b_lo, uint32_t hi,
                                             uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t.reg .b64 da, db;\n\t"
      "mov.b64 da, {%1, %3};\n\t"
      "mov.b64 db, {%2, %3};\n\t"
      "setp.ne.b32 p, %5, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], da, db, %4, p;\n\t}" ::"r"(d_tmem),
      "r"(a_lo), "r"(b_lo), "r"(hi), "r"(idesc), "r"(accumulate)
      : "memory");
}
// 4-D tiled load into this CTA's shared memory whose completion is counted on the
// mbarrier at `bar_cluster` (the even CTA's barrier: the pair's loads share one count).
__device__ __forceinline__ void tma_load_4d_pair(uint32_t dst, const void* map, uint32_t bar_cluster, int c0, int c1,
                                                 int c2, int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, "
      "%5, %6}], [%2];" ::"r"(dst),
      "l"(map), "r"(bar_cluster), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
      : "memory");
}
template <bool kPair>
__device__ __forceinline__ void tmem_alloc_g(uint32_t dst_smem, uint32_t ncols) {
  if (kPair)
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem), "r"(ncols)
                 : "memory");
  else
    tmem_alloc(dst_smem, ncols);
}
template <bool kPair>
__device__ __forceinline__ void tmem_relinquish_g() {
  if (kPair)
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
  else
    tmem_relinquish();
}
template <bool kPair>
__device__ __forceinline__ void tmem_dealloc_g(uint32_t taddr, uint32_t ncols) {
  if (kPair)
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
  else
    tmem_dealloc(taddr, ncols);
}

// Byte offset of 16-byte unit j of row `row` in a 128-row x 128-byte SW128 box.
__device__ __forceinline__ uint32_t box_unit(int row, int j) {
  return static_cast<uint32_t>(row * 128 + ((j ^ (row & 7)) << 4));
}

template <int BN, bool kPair>
__global__ void __launch_bounds__(kThreads, 1) gemm_kernel(const __grid_constant__ Maps maps, const Params p) {
  using C = Cfg<BN, kPair>;
  extern __shared__ __align__(1024) uint8_t smem[];
  if (smem_u32(smem) & 1023u) {
    if (threadIdx.x == 0) record_error(SITE_SMEM_ALIGN);
    return;
  }
  const uint32_t sbase = smem_u32(smem);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  auto bar_full = [&](int s) -> uint32_t { return sbase + C::kOffBar + 8 * s; };
  auto bar_empty = [&](int s) -> uint32_t { return sbase + C::kOffBar + 8 * (C::kStages + s); };
  auto bar_acc_full = [&](int b) -> uint32_t { return sbase + C::kOffBar + 8 * (2 * C::kStages + b); };
  auto bar_acc_empty = [&](int b) -> uint32_t { return sbase + C::kOffBar + 8 * (2 * C::kStages + 2 + b); };

  // Pair: rank 0 issues the MMAs; tiles are walked per cluster.
  const uint32_t rank = kPair ? cluster_rank() : 0u;
  const int unit = kPair ? static_cast<int>(blockIdx.x >> 1) : static_cast<int>(blockIdx.x);
  const int n_units = kPair ? static_cast<int>(gridDim.x >> 1) : static_cast<int>(gridDim.x);
  if (threadIdx.x == 0) {
    for (int s = 0; s < C::kStages; ++s) {
      mbar_init(bar_full(s), 1);
      mbar_init(bar_empty(s), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(bar_acc_full(b), 1);
      mbar_init(bar_acc_empty(b), kPair ? 256 : 128);  // pair: both CTAs' epilogue threads
    }
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc_g<kPair>(sbase + C::kOffTmemPtr, C::kTmemCols);
    tmem_relinquish_g<kPair>();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&maps.a);
    for (int r = 0; r < p.n_regions; ++r) {
      tma_prefetch_desc(pick(&maps.w[0], &maps.w[1], &maps.w[2], r));
      tma_prefetch_desc(pick(&maps.c[0], &maps.c[1], &maps.c[2], r));
    }
  }
  tc_fence_before();
  if (kPair)
    cluster_sync_all();  // both CTAs' barriers initialised before either signals the other
  else
    __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(smem + C::kOffTmemPtr);

  if (warp == 0) {
    // ---------------------------------------------------------------- producer
    if (lane == 0) {
      bool ok = true;
      uint32_t it = 0;
      for (int tile = unit; ok && tile < p.n_tiles; tile += n_units) {
        const int m0 = (tile % p.tiles_m) * C::kTileM + static_cast<int>(rank) * kBM;  // this CTA's rows
        const int n0 = (tile / p.tiles_m) * BN;
        const int r = region_of(p, n0);
        const CUtensorMap* wm = pick(&maps.w[0], &maps.w[1], &maps.w[2], r);
        const int b = m0 / p.S, s0 = m0 - b * p.S;
        const int wn = n0 - region_at(p, r).n0 + static_cast<int>(rank) * C::kWRows;
        for (int kb = 0; kb < p.n_kb; ++kb, ++it) {
          const int s = static_cast<int>(it % C::kStages);
          const uint32_t round = it / C::kStages;
          if (round > 0 && !(ok = mbar_wait(bar_empty(s), (round - 1) & 1u, SITE_PRODUCER))) break;
          const uint32_t dst = sbase + s * C::kStageBytes;
          const int k0 = kb * kBK;
          if (kPair) {
            // both CTAs' loads complete on the even CTA's barrier, which expects them all
            const uint32_t full0 = map_to_rank(bar_full(s), 0);
            if (rank == 0) mbar_expect_tx(bar_full(s), 2 * C::kStageBytes);
            tma_load_4d_pair(dst, &maps.a, full0, k0 % p.a_kin, s0, k0 / p.a_kin, b);
            tma_load_4d_pair(dst + C::kABytes, wm, full0, k0, wn, 0, 0);
          } else {
            mbar_expect_tx(bar_full(s), C::kStageBytes);
            tma_load_4d(dst, &maps.a, bar_full(s), k0 % p.a_kin, s0, k0 / p.a_kin, b);
            tma_load_4d(dst + C::kABytes, wm, bar_full(s), k0, wn, 0, 0);
          }
        }
      }
      // every issued load lands before the CTA exits (pair: the even CTA's MMA waited for
      // all of them, and both CTAs meet at the cluster barrier before exiting)
      if (!kPair) {
        const uint32_t first = it > static_cast<uint32_t>(C::kStages) ? it - C::kStages : 0u;
        for (uint32_t i = first; i < it; ++i)
          mbar_wait(bar_full(static_cast<int>(i % C::kStages)), (i / C::kStages) & 1u, SITE_PRODUCER);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0 && rank == 0) {
      constexpr uint32_t kId = idesc_bf16_f32(C::kTileM, BN, false);
      constexpr uint32_t kHi = sdesc_hi_sw128(1024);
      const uint32_t lo0 = sdesc_lo(sbase, 16);
      // pair: a barrier in each CTA is told when the pair's MMAs are done
      auto commit = [&](uint32_t bar) {
        if (kPair) {
          umma_commit_pair(map_to_rank(bar, 0));
          umma_commit_pair(map_to_rank(bar, 1));
        } else {
          umma_commit(bar);
        }
      };
      bool ok = true;
      uint32_t it = 0, t_iter = 0;
      for (int tile = unit; ok && tile < p.n_tiles; tile += n_units, ++t_iter) {
        const int ab = static_cast<int>(t_iter & 1u);
        const uint32_t use = t_iter >> 1;
        if (use > 0 && !(ok = mbar_wait_spin(bar_acc_empty(ab), (use - 1) & 1u, SITE_MMA))) break;
        tc_fence_after();
        const uint32_t d = tmem + static_cast<uint32_t>(ab * BN);
        for (int kb = 0; kb < p.n_kb; ++kb, ++it) {
          const int s = static_cast<int>(it % C::kStages);
          if (!(ok = mbar_wait_spin(bar_full(s), (it / C::kStages) & 1u, SITE_MMA))) break;
          tc_fence_after();
          const uint32_t a_lo = lo0 + static_cast<uint32_t>(s * C::kStageBytes) / 16u;
          const uint32_t w_lo = a_lo + C::kABytes / 16u;
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk) {
            if (kPair)
              umma_ss_pair(d, a_lo + 2u * kk, w_lo + 2u * kk, kHi, kId, (kb | kk) ? 1u : 0u);
            else
              umma_ss_lohi(d, a_lo + 2u * kk, w_lo + 2u * kk, kHi, kId, (kb | kk) ? 1u : 0u);
          }
          commit(bar_empty(s));
        }
        if (ok) commit(bar_acc_full(ab));
      }
    }
    __syncwarp();
  } else {
    // ---------------------------------------------------------------- epilogue (warps 2-5)
    const int quarter = warp & 3;            // TMEM lanes this warp may access
    const int row = quarter * 32 + lane;     // output row within the tile
    const int et = threadIdx.x - 64;         // 0..127
    const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
    const uint32_t stg0 = sbase + C::kOffStaging, stg1 = stg0 + C::kBoxBytes;
    uint8_t* const stg0_p = smem + C::kOffStaging;
    uint8_t* const stg1_p = stg0_p + C::kBoxBytes;
    bool ok = true;
    uint32_t t_iter = 0;
    for (int tile = unit; tile < p.n_tiles; tile += n_units, ++t_iter) {
      const int m0 = (tile % p.tiles_m) * C::kTileM + static_cast<int>(rank) * kBM;  // this CTA's rows
      const int n0 = (tile / p.tiles_m) * BN;
      const int r = region_of(p, n0);
      const Region rg = region_at(p, r);
      const CUtensorMap* cm = pick(&maps.c[0], &maps.c[1], &maps.c[2], r);
      const int b = m0 / p.S, s0 = m0 - b * p.S;
      const int ab = static_cast<int>(t_iter & 1u);
      if (ok) ok = __all_sync(0xffffffffu, mbar_wait(bar_acc_full(ab), (t_iter >> 1) & 1u, SITE_EPILOGUE));
      tc_fence_after();
      const uint32_t acc = tmem + lane_off + static_cast<uint32_t>(ab * BN);
      // Each cycle fills both staging boxes (128 rows x 128 B each) and stores them.
      constexpr int kCycles = BN / 64;  // fp32: 2 x 32 columns; bf16: 2 x 64 columns per 2 cycles
      const int n_cycles = p.out_f32 ? kCycles : kCycles / 2;
      for (int cyc = 0; cyc < n_cycles; ++cyc) {
        if (et == 0) bulk_wait_read0();  // the previous cycle's stores have read the staging boxes
        named_bar_sync(1, 128);
        if (p.out_f32) {
#pragma unroll
          for (int hb = 0; hb < 2; ++hb) {
            uint32_t x[32];
            if (ok) {
              tmem_ld32(acc + static_cast<uint32_t>(cyc * 64 + hb * 32), x);
              tmem_wait_ld_dep(x);
            }
            uint8_t* box = hb ? stg1_p : stg0_p;
#pragma unroll
            for (int j = 0; j < 8; ++j)
              *reinterpret_cast<uint4*>(box + box_unit(row, j)) = make_uint4(x[4 * j], x[4 * j + 1], x[4 * j + 2],
                                                                             x[4 * j + 3]);
          }
        } else {
          // one 128-column group (a head): staging box 0 = dims 0..63, box 1 = dims 64..127
          const int pos = p.pos0 + s0 + row;
          const bool rot = rg.rope && (s0 + row) < p.S;
#pragma unroll
          for (int c = 0; c < 64; c += 32) {
            uint32_t x0[32], x1[32];
            if (ok) {
              tmem_ld32(acc + static_cast<uint32_t>(cyc * 128 + c), x0);
              tmem_ld32(acc + static_cast<uint32_t>(cyc * 128 + 64 + c), x1);
              tmem_wait_ld_dep(x0);
              tmem_wait_ld_dep(x1);
            }
            uint32_t w0[16], w1[16];
            if (rot) {
              const uint4* cr = reinterpret_cast<const uint4*>(p.cos + static_cast<size_t>(pos) * 128 + c);
              const uint4* sr = reinterpret_cast<const uint4*>(p.sin + static_cast<size_t>(pos) * 128 + c);
#pragma unroll
              for (int u = 0; u < 4; ++u) {
                const uint4 c0 = __ldg(cr + u), c1 = __ldg(cr + 8 + u);  // dims c+8u.., 64+c+8u..
                const uint4 s0v = __ldg(sr + u), s1v = __ldg(sr + 8 + u);
                const uint32_t cw0[4] = {c0.x, c0.y, c0.z, c0.w}, cw1[4] = {c1.x, c1.y, c1.z, c1.w};
                const uint32_t sw0[4] = {s0v.x, s0v.y, s0v.z, s0v.w}, sw1[4] = {s1v.x, s1v.y, s1v.z, s1v.w};
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                  const int j = 8 * u + 2 * e;  // columns j, j+1 of this 32-column slice
                  float a0[2], a1[2], yv0[2], yv1[2];
#pragma unroll
                  for (int t = 0; t < 2; ++t) {
                    a0[t] = bf2f_bits(f2bf_bits(__uint_as_float(x0[j + t])));
                    a1[t] = bf2f_bits(f2bf_bits(__uint_as_float(x1[j + t])));
                    const float cl = t ? bf16_hi(cw0[e]) : bf16_lo(cw0[e]);
                    const float ch = t ? bf16_hi(cw1[e]) : bf16_lo(cw1[e]);
                    const float sl = t ? bf16_hi(sw0[e]) : bf16_lo(sw0[e]);
                    const float sh = t ? bf16_hi(sw1[e]) : bf16_lo(sw1[e]);
                    yv0[t] = __fadd_rn(__fmul_rn(a0[t], cl), __fmul_rn(-a1[t], sl));
                    yv1[t] = __fadd_rn(__fmul_rn(a1[t], ch), __fmul_rn(a0[t], sh));
                  }
                  w0[j / 2] = static_cast<uint32_t>(f2bf_bits(yv0[0])) | (static_cast<uint32_t>(f2bf_bits(yv0[1])) << 16);
                  w1[j / 2] = static_cast<uint32_t>(f2bf_bits(yv1[0])) | (static_cast<uint32_t>(f2bf_bits(yv1[1])) << 16);
                }
              }
            } else {
#pragma unroll
              for (int j = 0; j < 16; ++j) {
                w0[j] = static_cast<uint32_t>(f2bf_bits(__uint_as_float(x0[2 * j]))) |
                        (static_cast<uint32_t>(f2bf_bits(__uint_as_float(x0[2 * j + 1]))) << 16);
                w1[j] = static_cast<uint32_t>(f2bf_bits(__uint_as_float(x1[2 * j]))) |
                        (static_cast<uint32_t>(f2bf_bits(__uint_as_float(x1[2 * j + 1]))) << 16);
              }
            }
#pragma unroll
            for (int u = 0; u < 4; ++u) {
              *reinterpret_cast<uint4*>(stg0_p + box_unit(row, c / 8 + u)) =
                  make_uint4(w0[4 * u], w0[4 * u + 1], w0[4 * u + 2], w0[4 * u + 3]);
              *reinterpret_cast<uint4*>(stg1_p + box_unit(row, c / 8 + u)) =
                  make_uint4(w1[4 * u], w1[4 * u + 1], w1[4 * u + 2], w1[4 * u + 3]);
            }
          }
        }
        if (cyc == n_cycles - 1) {  // accumulator fully read: the MMA may reuse it
          tc_fence_before();
          if (kPair)
            mbar_arrive_cluster(map_to_rank(bar_acc_empty(ab), 0));
          else
            mbar_arrive(bar_acc_empty(ab));
        }
        fence_proxy_async_smem();
        named_bar_sync(1, 128);
        if (p.scatter_rows > 0) {
          // rows go to their owner (possibly NVLink peer memory) by plain stores, 8
          // consecutive threads per 128-byte row segment so every line is written whole
          const int q = m0 / p.scatter_rows;  // a tile never straddles two owners
          float* dbase = dst_at(p, q) + static_cast<size_t>(m0 - q * p.scatter_rows) * p.N + n0 + cyc * 64;
#pragma unroll 4
          for (int idx = et; idx < 2 * 128 * 8; idx += 128) {
            const int box = idx >> 10, rr = (idx >> 3) & 127, j = idx & 7;
            const uint4 v = *reinterpret_cast<const uint4*>((box ? stg1_p : stg0_p) + box_unit(rr, j));
            if (ok && m0 + rr < p.M)
              *reinterpret_cast<uint4*>(dbase + static_cast<size_t>(rr) * p.N + box * 32 + 4 * j) = v;
          }
          named_bar_sync(1, 128);  // staging free again (the next cycle refills it)
        } else if (et == 0 && ok) {
          if (p.out_f32) {
            const int nc = n0 - rg.n0 + cyc * 64;
            tma_store_4d(cm, stg0, nc, m0, 0, 0);
            tma_store_4d(cm, stg1, nc + 32, m0, 0, 0);
          } else if (rg.head_major) {
            const int h = (n0 - rg.n0) / 128 + cyc;
            tma_store_4d(cm, stg0, 0, s0, h, b);
            tma_store_4d(cm, stg1, 64, s0, h, b);
          } else {
            const int nc = n0 - rg.n0 + cyc * 128;
            tma_store_4d(cm, stg0, nc, m0, 0, 0);
            tma_store_4d(cm, stg1, nc + 64, m0, 0, 0);
          }
          bulk_commit();
        }
      }
    }
    if (et == 0) bulk_wait0();
    if (p.scatter_rows > 0) __threadfence_system();  // this thread's direct stores, before the signal
  }

  // ---- teardown
  tc_fence_before();
  if (kPair)
    cluster_sync_all();  // neither CTA leaves while the other may still signal it
  else
    __syncthreads();
  if (p.scatter_rows > 0 && threadIdx.x == 0) {
    // The last CTA to finish tells every destination that its rows are complete, unless
    // a wait of this grid gave up (a CTA that failed skipped its stores): then no flag is
    // raised, the owners' bounded waits expire and they report the timeout too, instead
    // of reducing slots that still hold the previous step's rows.  The fences order every
    // CTA's error record (made before the block barrier above) before its arrival.
    __threadfence();
    if (atomicAdd(p.sig_counter, 1u) + 1u == gridDim.x) {
      __threadfence();
      *p.sig_counter = 0u;
      __threadfence_system();
      if (!error_pending())
        for (int q = 0; q < p.n_dest; ++q)
          asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(flag_at(p, q)), "r"(p.sig_epoch) : "memory");
    }
  }
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_g<kPair>(tmem, C::kTmemCols);
  }
}

// Host-side description of one launch.
struct Launch {
  // A: 4-D (inner, s, outer, batch) view
  const void* a;
  long long a_dims[4];
  long long a_strides[3];  // bytes, dims 1..3
  int a_kin;
  int M, N, K, S;
  int out_f32;
  int n_regions;
  Region reg[kMaxRegions];
  const void* w[kMaxRegions];
  int ldw[kMaxRegions];
  void* c[kMaxRegions];
  long long c_dims[kMaxRegions][4];
  long long c_strides[kMaxRegions][3];
  const void* cos;
  const void* sin;
  int pos0;
  int max_ctas;  // persistent grid cap (0 = one CTA per SM), e.g. to leave SMs to a collective
  int scatter_rows, n_dest;  // scatter epilogue (see Params)
  float* dst[kMaxDest];
  uint32_t* sig_flag[kMaxDest];
  uint32_t* sig_counter;
  uint32_t sig_epoch;
};

template <int BN, bool kPair>
int launch_bn(const Launch& L, cudaStream_t stream) {
  using C = Cfg<BN, kPair>;
  Maps maps;
  int rc;
  const int box_a[4] = {kBK, kBM, 1, 1};
  if ((rc = make_tmap_4d(&maps.a, L.a, 2, L.a_dims, L.a_strides, box_a)) != GQA_OK) return rc;
  for (int r = 0; r < kMaxRegions; ++r) {
    const int rr = r < L.n_regions ? r : 0;  // unused slots repeat region 0
    const long long wd[4] = {L.K, L.reg[rr].n1 - L.reg[rr].n0, 1, 1};
    const long long ws[3] = {static_cast<long long>(L.ldw[rr]) * 2, static_cast<long long>(L.ldw[rr]) * 2 * wd[1],
                             static_cast<long long>(L.ldw[rr]) * 2 * wd[1]};
    const int box_w[4] = {kBK, C::kWRows, 1, 1};
    if ((rc = make_tmap_4d(&maps.w[r], L.w[rr], 2, wd, ws, box_w)) != GQA_OK) return rc;
    const int box_c[4] = {L.out_f32 ? 32 : 64, kBM, 1, 1};
    if ((rc = make_tmap_4d(&maps.c[r], L.c[rr], L.out_f32 ? 4 : 2, L.c_dims[rr], L.c_strides[rr], box_c)) != GQA_OK)
      return rc;
  }
  static std::atomic<uint64_t> attr_done{0};
  if ((rc = ensure_smem_attr(gemm_kernel<BN, kPair>, C::kSmemBytes, attr_done)) != GQA_OK) return rc;
  Params p;
  p.M = L.M;
  p.N = L.N;
  p.K = L.K;
  p.S = L.S;
  p.a_kin = L.a_kin;
  p.tiles_m = (L.M + C::kTileM - 1) / C::kTileM;
  p.tiles_n = (L.N + BN - 1) / BN;
  p.n_tiles = p.tiles_m * p.tiles_n;
  p.n_kb = (L.K + kBK - 1) / kBK;
  p.out_f32 = L.out_f32;
  p.n_regions = L.n_regions;
  for (int r = 0; r < kMaxRegions; ++r) p.reg[r] = L.reg[r < L.n_regions ? r : 0];
  p.cos = static_cast<const uint16_t*>(L.cos);
  p.sin = static_cast<const uint16_t*>(L.sin);
  p.pos0 = L.pos0;
  p.scatter_rows = L.scatter_rows;
  p.n_dest = L.n_dest;
  for (int q = 0; q < kMaxDest; ++q) {
    p.dst[q] = L.dst[q];
    p.sig_flag[q] = L.sig_flag[q];
  }
  p.sig_counter = L.sig_counter;
  p.sig_epoch = L.sig_epoch;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int cap = L.max_ctas > 0 && L.max_ctas < sms ? L.max_ctas : sms;
  if (!kPair) {
    const int grid = p.n_tiles < cap ? p.n_tiles : cap;
    gemm_kernel<BN, false><<<grid, kThreads, C::kSmemBytes, stream>>>(maps, p);
    return cudaGetLastError() == cudaSuccess ? GQA_OK : GQA_ERR_CUDA;
  }
  // one cluster of two CTAs per tile slot; at most as many clusters as fit at once
  static std::atomic<int> max_clusters{0};
  int mc = max_clusters.load(std::memory_order_acquire);
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = C::kSmemBytes;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (mc == 0) {
    cfg.gridDim = dim3(sms & ~1);
    if (cudaOccupancyMaxActiveClusters(&mc, gemm_kernel<BN, true>, &cfg) != cudaSuccess || mc <= 0) return GQA_ERR_CUDA;
    max_clusters.store(mc, std::memory_order_release);
  }
  int clusters = cap / 2 < mc ? cap / 2 : mc;
  if (clusters > p.n_tiles) clusters = p.n_tiles;
  if (clusters < 1) clusters = 1;
  cfg.gridDim = dim3(2 * clusters);
  if (cudaLaunchKernelEx(&cfg, gemm_kernel<BN, true>, maps, p) != cudaSuccess) return GQA_ERR_CUDA;
  return cudaGetLastError() == cudaSuccess ? GQA_OK : GQA_ERR_CUDA;
}

// 128 x 256 tiles: a 128 x 128 tile reads as many operand bytes per flop again and
// runs at about two thirds of the rate (measured at 4096^3).  128-wide tiles are used
// when a region boundary needs them, or when even they fill no more than one wave
// (small problems: twice the CTAs in flight).
int pick_bn(const Launch& L, int sms) {
  for (int r = 1; r < L.n_regions; ++r)
    if (L.reg[r].n0 % 256) return 128;
  if (L.out_f32 == 0)
    for (int r = 0; r < L.n_regions; ++r)
      if (L.reg[r].head_major && (L.reg[r].n1 - L.reg[r].n0) % 256) return 128;
  const long long tm = (L.M + kBM - 1) / kBM;
  const long long t128 = tm * ((L.N + 127) / 128);
  return t128 <= sms ? 128 : 256;
}

int launch(const Launch& L, cudaStream_t stream) {
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int bn = pick_bn(L, sms);
  // CTA pairs (256-row tiles, W rows split between the two CTAs) wherever the rows
  // divide into pair tiles; the scatter epilogue keeps single CTAs.  Pairs compute the
  // same sums in the same order (bit-identical results) with half of W per CTA: 1.28
  // against 1.23 PFLOP/s at 4096^3 (bf16 out), the rest of the gap to cuBLAS being the
  // 3.46 waves of 256 x 256 tiles on 74 pairs and the power cap.
  const bool pair = L.scatter_rows == 0 && L.M % (2 * kBM) == 0;
  if (pair) return bn == 256 ? launch_bn<256, true>(L, stream) : launch_bn<128, true>(L, stream);
  return bn == 256 ? launch_bn<256, false>(L, stream) : launch_bn<128, false>(L, stream);
}

}  // namespace gemm
}  // namespace gqa

using namespace gqa;

namespace {

bool bad16(const void* p) { return p == nullptr || !aligned16(p); }

}  // namespace

extern "C" int gqa_gemm_bf16(const void* a, const void* w, void* c, int M, int N, int K, int lda, int ldw, int ldc,
                             int flags, gqa_stream_t stream) {
  if (!a || !w || !c || M <= 0 || N <= 0 || K <= 0) return GQA_ERR_INVALID_ARGUMENT;
  if (flags & ~GQA_GEMM_OUT_F32) return GQA_ERR_INVALID_ARGUMENT;
  if (lda < K || ldw < K || ldc < N) return GQA_ERR_INVALID_ARGUMENT;
  const bool f32 = (flags & GQA_GEMM_OUT_F32) != 0;
  if (bad16(a) || bad16(w) || bad16(c)) return GQA_ERR_MISALIGNED;
  if (lda % 8 || ldw % 8 || (f32 ? ldc % 4 : ldc % 8)) return GQA_ERR_MISALIGNED;  // 16-byte row strides
  gemm::Launch L{};
  L.a = a;
  L.a_dims[0] = K;
  L.a_dims[1] = M;
  L.a_dims[2] = 1;
  L.a_dims[3] = 1;
  L.a_strides[0] = static_cast<long long>(lda) * 2;
  L.a_strides[1] = L.a_strides[0] * M;
  L.a_strides[2] = L.a_strides[1];
  L.a_kin = K;
  L.M = M;
  L.N = N;
  L.K = K;
  L.S = M;
  L.out_f32 = f32 ? 1 : 0;
  L.n_regions = 1;
  L.reg[0] = gemm::Region{0, N, 0, 0};
  L.w[0] = w;
  L.ldw[0] = ldw;
  L.c[0] = c;
  const long long esz = f32 ? 4 : 2;
  L.c_dims[0][0] = N;
  L.c_dims[0][1] = M;
  L.c_dims[0][2] = 1;
  L.c_dims[0][3] = 1;
  L.c_strides[0][0] = static_cast<long long>(ldc) * esz;
  L.c_strides[0][1] = L.c_strides[0][0] * M;
  L.c_strides[0][2] = L.c_strides[0][1];
  return gemm::launch(L, static_cast<cudaStream_t>(stream));
}

extern "C" int gqa_qkv_proj_bf16(const void* h, const void* wq, const void* wk, const void* wv, void* q, void* k,
                                 void* v, const void* cos, const void* sin, int B, int S, int hidden, int Hq, int Hkv,
                                 int head_dim, int pos0, int flags, gqa_stream_t stream) {
  if (!h || !wq || !wk || !wv || !q || !k || !v || B <= 0 || S <= 0 || hidden <= 0 || Hq <= 0 || Hkv <= 0 || pos0 < 0)
    return GQA_ERR_INVALID_ARGUMENT;
  if (flags & ~(GQA_FLAG_ROPE_Q | GQA_FLAG_ROPE_K)) return GQA_ERR_INVALID_ARGUMENT;
  if ((flags & (GQA_FLAG_ROPE_Q | GQA_FLAG_ROPE_K)) && (!cos || !sin)) return GQA_ERR_INVALID_ARGUMENT;
  if (head_dim != 128) return GQA_ERR_UNSUPPORTED;
  if (B > 1 && S % gemm::kBM) return GQA_ERR_UNSUPPORTED;  // a row tile must not straddle two sequences
  if (bad16(h) || bad16(wq) || bad16(wk) || bad16(wv) || bad16(q) || bad16(k) || bad16(v)) return GQA_ERR_MISALIGNED;
  if ((cos && bad16(cos)) || (sin && bad16(sin)) || hidden % 8) return GQA_ERR_MISALIGNED;
  gemm::Launch L{};
  const long long M = static_cast<long long>(B) * S;
  L.a = h;  // [B][S][hidden] viewed as (hidden, s, 1, b): row tile (b, s0) reads rows b*S + s0 ..
  L.a_dims[0] = hidden;
  L.a_dims[1] = S;
  L.a_dims[2] = 1;
  L.a_dims[3] = B;
  L.a_strides[0] = static_cast<long long>(hidden) * 2;
  L.a_strides[1] = L.a_strides[0] * S;
  L.a_strides[2] = L.a_strides[1];
  L.a_kin = hidden;
  L.M = static_cast<int>(M);
  L.K = hidden;
  L.S = S;
  const int nq = Hq * 128, nkv = Hkv * 128;
  L.N = nq + 2 * nkv;
  L.n_regions = 3;
  L.reg[0] = gemm::Region{0, nq, 1, (flags & GQA_FLAG_ROPE_Q) ? 1 : 0};
  L.reg[1] = gemm::Region{nq, nq + nkv, 1, (flags & GQA_FLAG_ROPE_K) ? 1 : 0};
  L.reg[2] = gemm::Region{nq + nkv, nq + 2 * nkv, 1, 0};
  const void* ws[3] = {wq, wk, wv};
  void* outs[3] = {q, k, v};
  const int heads[3] = {Hq, Hkv, Hkv};
  for (int r = 0; r < 3; ++r) {
    L.w[r] = ws[r];
    L.ldw[r] = hidden;
    L.c[r] = outs[r];
    L.c_dims[r][0] = 128;
    L.c_dims[r][1] = S;
    L.c_dims[r][2] = heads[r];
    L.c_dims[r][3] = B;
    L.c_strides[r][0] = 256;
    L.c_strides[r][1] = 256LL * S;
    L.c_strides[r][2] = 256LL * S * heads[r];
  }
  L.cos = cos;
  L.sin = sin;
  L.pos0 = pos0;
  return gemm::launch(L, static_cast<cudaStream_t>(stream));
}

extern "C" int gqa_o_proj_bf16(const void* attn, const void* wo, void* out, int B, int S, int Hq, int head_dim, int N,
                               int ldw, int flags, gqa_stream_t stream) {
  if (!attn || !wo || !out || B <= 0 || S <= 0 || Hq <= 0 || N <= 0) return GQA_ERR_INVALID_ARGUMENT;
  if (flags & ~GQA_GEMM_OUT_F32) return GQA_ERR_INVALID_ARGUMENT;
  if (head_dim != 128) return GQA_ERR_UNSUPPORTED;
  if (ldw < Hq * 128) return GQA_ERR_INVALID_ARGUMENT;
  if (B > 1 && S % gemm::kBM) return GQA_ERR_UNSUPPORTED;
  const bool f32 = (flags & GQA_GEMM_OUT_F32) != 0;
  if (bad16(attn) || bad16(wo) || bad16(out)) return GQA_ERR_MISALIGNED;
  if (ldw % 8 || (f32 ? N % 4 : N % 8)) return GQA_ERR_MISALIGNED;
  gemm::Launch L{};
  L.a = attn;  // [B][Hq][S][128]: k = h * 128 + d
  L.a_dims[0] = 128;
  L.a_dims[1] = S;
  L.a_dims[2] = Hq;
  L.a_dims[3] = B;
  L.a_strides[0] = 256;
  L.a_strides[1] = 256LL * S;
  L.a_strides[2] = 256LL * S * Hq;
  L.a_kin = 128;
  L.M = B * S;
  L.N = N;
  L.K = Hq * 128;
  L.S = S;
  L.out_f32 = f32 ? 1 : 0;
  L.n_regions = 1;
  L.reg[0] = gemm::Region{0, N, 0, 0};
  L.w[0] = wo;
  L.ldw[0] = ldw;
  L.c[0] = out;
  const long long esz = f32 ? 4 : 2;
  L.c_dims[0][0] = N;
  L.c_dims[0][1] = static_cast<long long>(B) * S;
  L.c_dims[0][2] = 1;
  L.c_dims[0][3] = 1;
  L.c_strides[0][0] = N * esz;
  L.c_strides[0][1] = L.c_strides[0][0] * B * S;
  L.c_strides[0][2] = L.c_strides[0][1];
  return gemm::launch(L, static_cast<cudaStream_t>(stream));
}

// Rows [s0, s0 + s_count) of the o_proj output of one sequence (B = 1): attn [Hq][S][128]
// head-major, out [S][N] (only the chunk's rows written).  Lets a caller overlap the
// reduction of finished rows with the GEMM of the next ones; max_ctas caps the
// persistent grid so that a collective running beside it finds free SMs.
extern "C" int gqa_o_proj_rows_bf16(const void* attn, const void* wo, void* out, int S, int s0, int s_count, int Hq,
                                    int head_dim, int N, int ldw, int max_ctas, int flags, gqa_stream_t stream) {
  if (!attn || !wo || !out || S <= 0 || Hq <= 0 || N <= 0 || s_count <= 0) return GQA_ERR_INVALID_ARGUMENT;
  if (s0 < 0 || s0 + s_count > S || max_ctas < 0) return GQA_ERR_INVALID_ARGUMENT;
  if (flags & ~GQA_GEMM_OUT_F32) return GQA_ERR_INVALID_ARGUMENT;
  if (head_dim != 128) return GQA_ERR_UNSUPPORTED;
  if (ldw < Hq * 128) return GQA_ERR_INVALID_ARGUMENT;
  const bool f32 = (flags & GQA_GEMM_OUT_F32) != 0;
  const long long esz = f32 ? 4 : 2;
  if (bad16(attn) || bad16(wo) || bad16(out)) return GQA_ERR_MISALIGNED;
  if (ldw % 8 || (f32 ? N % 4 : N % 8)) return GQA_ERR_MISALIGNED;
  gemm::Launch L{};
  L.a = static_cast<const uint16_t*>(attn) + static_cast<size_t>(s0) * 128;  // token s0 of head 0
  L.a_dims[0] = 128;
  L.a_dims[1] = s_count;
  L.a_dims[2] = Hq;
  L.a_dims[3] = 1;
  L.a_strides[0] = 256;
  L.a_strides[1] = 256LL * S;
  L.a_strides[2] = 256LL * S * Hq;
  L.a_kin = 128;
  L.M = s_count;
  L.N = N;
  L.K = Hq * 128;
  L.S = s_count;
  L.out_f32 = f32 ? 1 : 0;
  L.n_regions = 1;
  L.reg[0] = gemm::Region{0, N, 0, 0};
  L.w[0] = wo;
  L.ldw[0] = ldw;
  L.c[0] = static_cast<uint8_t*>(out) + static_cast<size_t>(s0) * N * esz;
  L.c_dims[0][0] = N;
  L.c_dims[0][1] = s_count;
  L.c_dims[0][2] = 1;
  L.c_dims[0][3] = 1;
  L.c_strides[0][0] = N * esz;
  L.c_strides[0][1] = L.c_strides[0][0] * s_count;
  L.c_strides[0][2] = L.c_strides[0][1];
  L.max_ctas = max_ctas;
  return gemm::launch(L, static_cast<cudaStream_t>(stream));
}

namespace gqa {
// o_proj (B = 1) whose fp32 rows go straight to their owners: row m to dst[m / (S / world)]
// + (m % (S / world)) * N, then the grid's last CTA raises flags[q] = epoch for every q.
// `local` is a buffer of this GPU holding at least S / world x N fp32.
int launch_o_proj_scatter(const void* attn, const void* wo, int S, int Hq, int N, int ldw, float* const* dst,
                          uint32_t* const* flags, int world, uint32_t* counter, uint32_t epoch, float* local,
                          cudaStream_t stream) {
  if (!attn || !wo || !dst || !flags || !counter || !local || world < 1 || world > gemm::kMaxDest)
    return GQA_ERR_INVALID_ARGUMENT;
  if (bad16(local)) return GQA_ERR_MISALIGNED;
  if (S <= 0 || Hq <= 0 || N <= 0 || S % world || (S / world) % gemm::kBM || N % 256) return GQA_ERR_UNSUPPORTED;
  if (ldw < Hq * 128 || ldw % 8) return GQA_ERR_INVALID_ARGUMENT;
  if (bad16(attn) || bad16(wo)) return GQA_ERR_MISALIGNED;
  for (int q = 0; q < world; ++q)
    if (!dst[q] || bad16(dst[q]) || !flags[q]) return GQA_ERR_INVALID_ARGUMENT;
  gemm::Launch L{};
  L.a = attn;
  L.a_dims[0] = 128;
  L.a_dims[1] = S;
  L.a_dims[2] = Hq;
  L.a_dims[3] = 1;
  L.a_strides[0] = 256;
  L.a_strides[1] = 256LL * S;
  L.a_strides[2] = 256LL * S * Hq;
  L.a_kin = 128;
  L.M = S;
  L.N = N;
  L.K = Hq * 128;
  L.S = S;
  L.out_f32 = 1;
  L.n_regions = 1;
  L.reg[0] = gemm::Region{0, N, 0, 0};
  L.w[0] = wo;
  L.ldw[0] = ldw;
  // The staging / TMA-store map is built but never used in scatter mode.  It covers the
  // caller's local buffer (at least S / world rows of N fp32), so no tensor map of the
  // multi-GPU path describes another GPU's memory.
  L.c[0] = local;
  L.c_dims[0][0] = N;
  L.c_dims[0][1] = S / world;
  L.c_dims[0][2] = 1;
  L.c_dims[0][3] = 1;
  L.c_strides[0][0] = static_cast<long long>(N) * 4;
  L.c_strides[0][1] = L.c_strides[0][0] * (S / world);
  L.c_strides[0][2] = L.c_strides[0][1];
  L.scatter_rows = S / world;
  L.n_dest = world;
  for (int q = 0; q < gemm::kMaxDest; ++q) {
    L.dst[q] = dst[q < world ? q : 0];
    L.sig_flag[q] = flags[q < world ? q : 0];
  }
  L.sig_counter = counter;
  L.sig_epoch = epoch;
  return gemm::launch(L, stream);
}
}  // namespace gqa

namespace {
__global__ void cast_f32_bf16_kernel(const float* __restrict__ src, uint16_t* __restrict__ dst, long long n) {
  const long long n4 = n >> 2;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n4;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const float4 v = reinterpret_cast<const float4*>(src)[i];
    uint2 o;
    o.x = static_cast<uint32_t>(f2bf_bits(v.x)) | (static_cast<uint32_t>(f2bf_bits(v.y)) << 16);
    o.y = static_cast<uint32_t>(f2bf_bits(v.z)) | (static_cast<uint32_t>(f2bf_bits(v.w)) << 16);
    reinterpret_cast<uint2*>(dst)[i] = o;
  }
  for (long long i = (n4 << 2) + blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<long long>(gridDim.x) * blockDim.x)
    dst[i] = f2bf_bits(src[i]);
}
}  // namespace

extern "C" int gqa_cast_f32_bf16(const void* src, void* dst, long long n, gqa_stream_t stream) {
  if (!src || !dst || n < 0) return GQA_ERR_INVALID_ARGUMENT;
  if (n == 0) return GQA_OK;
  if (bad16(src) || (reinterpret_cast<uintptr_t>(dst) & 7u)) return GQA_ERR_MISALIGNED;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const long long want = (n / 4 + 255) / 256;
  const int grid = static_cast<int>(want < 8LL * sms ? (want > 0 ? want : 1) : 8LL * sms);
  cast_f32_bf16_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(static_cast<const float*>(src),
                                                                           static_cast<uint16_t*>(dst), n);
  return cudaGetLastError() == cudaSuccess ? GQA_OK : GQA_ERR_CUDA;
}

namespace gqa {
GQA_ERROR_FLAG_ACCESSOR(error_flag_gemm)

int gemm_error_word(const int** out) {
  constexpr int kMaxDevices = 64;
  static std::atomic<const int*> cache[kMaxDevices];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return GQA_ERR_NO_DEVICE;
  if (dev < 0 || dev >= kMaxDevices) return GQA_ERR_UNSUPPORTED;
  const int* a = cache[dev].load(std::memory_order_acquire);
  if (a == nullptr) {
    void* addr = nullptr;
    if (cudaGetSymbolAddress(&addr, g_gqa_dev_error) != cudaSuccess || addr == nullptr) return GQA_ERR_CUDA;
    a = static_cast<const int*>(addr);
    cache[dev].store(a, std::memory_order_release);
  }
  *out = a;
  return GQA_OK;
}
}  // namespace gqa
