// attn_common.cuh -- device helpers shared by the sm_100a prefill kernels: the K/V
// ring's load order, the SW128 tile layout, RoPE of rows held in shared memory, and the
// exponential evaluated on the FMA pipe.
#pragma once

#include <cstdint>

#include "common.cuh"

namespace gqa {
namespace attn {

constexpr int kHalfTile = 128 * 64 * 2;  // one 64-column SW128 block of a 128-row bf16 tile

// Load order of the K/V ring: K0, K1, V0, K2, V1, ..., K(n-1), V(n-2), V(n-1).  With K
// one tile ahead, every stage a load reuses was released an iteration earlier (K(j+1)
// reuses V(j-2)'s stage, V(j) reuses K(j)'s), so a 3-stage ring never stalls the MMAs.
__device__ __forceinline__ int load_idx_k(int j) { return j == 0 ? 0 : 2 * j - 1; }
__device__ __forceinline__ int load_idx_v(int j, int n) { return j + 1 < n ? 2 * j + 2 : 2 * n - 1; }

// Byte offset of 16-byte chunk c (elements 8c..8c+7) of row r in a 128x128 bf16
// K-major SWIZZLE_128B tile (two 64-column blocks of 128 rows x 128 B).
__device__ __forceinline__ int sw128_chunk(int r, int c) {
  return (c >> 3) * kHalfTile + r * 128 + (((c & 7) ^ (r & 7)) << 4);
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

}  // namespace attn
}  // namespace gqa
