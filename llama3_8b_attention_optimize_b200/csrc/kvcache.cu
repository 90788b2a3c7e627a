// kvcache.cu -- append new tokens' K/V to a decode cache, rotating K on the way in.
//
// For each sequence b, head h and new token i (position pos = lens[b] + i):
//   K cache row  <- RoPE(k_new[b][h][i], cos[pos], sin[pos])   (GQA_FLAG_ROPE_K; else a copy)
//   V cache row  <- v_new[b][h][i]
// The rotation is the golden model's apply_rope (llama3_attention_golden_model.py:133-139,
// pairs (d, d + 64), fp32 products and sum, one RNE to bf16), so a cache filled token by
// token holds exactly the rotated K that the golden model computes for the whole prompt.
//
// Cache layouts:
//   contiguous (block_table == NULL): [B][Hkv][max_len][128]
//   paged: pages [num_pages][Hkv][page_size][128]; position pos of sequence b is row
//          pos % page_size of page block_table[b][pos / page_size].
// Device-side checks (pos beyond the cache, a block-table entry outside the pool) skip
// the row and record an input error that gqa_device_check reports.
//
// One warp per (b, h, token) row; lane l moves dims (2l, 2l+1) and (2l+64, 2l+65), the
// RoPE pairs, as 32-bit words.  HBM-bound: 2 x 256 B read and written per row.
#include "attn_common.cuh"
#include "common.cuh"
#include "gqa_internal.h"

namespace gqa {
namespace kvcache {

constexpr int kD = 128;
constexpr int kWarps = 8;

enum : int {
  SITE_CAPACITY = 0x602,  // lens[b] + i beyond the cache
  SITE_BAD_PAGE = 0x603,  // block-table entry outside [0, num_pages)
};

struct Params {
  const uint16_t* k_new;  // [B][Hkv][n_new][128]
  const uint16_t* v_new;
  uint16_t* kc;
  uint16_t* vc;
  const int32_t* table;  // [B][max_pages] or nullptr
  const int32_t* lens;   // [B]
  const uint16_t* cos;   // [>= capacity][128]
  const uint16_t* sin;
  long long rows;  // B * Hkv * n_new
  int Hkv, n_new, max_len, page_size, max_pages, num_pages, flags;
};

__global__ void __launch_bounds__(kWarps * 32) append_kernel(const Params p) {
  const long long row = static_cast<long long>(blockIdx.x) * kWarps + (threadIdx.x >> 5);
  if (row >= p.rows) return;
  const int lane = threadIdx.x & 31;
  const int i = static_cast<int>(row % p.n_new);
  const long long bh = row / p.n_new;
  const int h = static_cast<int>(bh % p.Hkv);
  const int b = static_cast<int>(bh / p.Hkv);
  const long long pos = static_cast<long long>(__ldg(p.lens + b)) + i;
  const long long capacity = p.table ? static_cast<long long>(p.max_pages) * p.page_size : p.max_len;
  if (pos < 0 || pos >= capacity) {
    if (lane == 0) record_input_error(SITE_CAPACITY);
    return;
  }
  size_t dst;
  if (p.table) {
    const int page = __ldg(p.table + static_cast<size_t>(b) * p.max_pages + pos / p.page_size);
    if (page < 0 || page >= p.num_pages) {
      if (lane == 0) record_input_error(SITE_BAD_PAGE);
      return;
    }
    dst = ((static_cast<size_t>(page) * p.Hkv + h) * p.page_size + static_cast<size_t>(pos % p.page_size)) * kD;
  } else {
    dst = ((static_cast<size_t>(b) * p.Hkv + h) * p.max_len + static_cast<size_t>(pos)) * kD;
  }
  const size_t src = static_cast<size_t>(row) * kD;
  const int d = 2 * lane;
  uint32_t ka = *reinterpret_cast<const uint32_t*>(p.k_new + src + d);
  uint32_t kb = *reinterpret_cast<const uint32_t*>(p.k_new + src + d + 64);
  if (p.flags & GQA_FLAG_ROPE_K) {
    const size_t t = static_cast<size_t>(pos) * kD + d;  // cos[d] == cos[d + 64]: one word serves both
    attn::rope_pair(ka, kb, *reinterpret_cast<const uint32_t*>(p.cos + t), *reinterpret_cast<const uint32_t*>(p.sin + t));
  }
  *reinterpret_cast<uint32_t*>(p.kc + dst + d) = ka;
  *reinterpret_cast<uint32_t*>(p.kc + dst + d + 64) = kb;
  *reinterpret_cast<uint32_t*>(p.vc + dst + d) = *reinterpret_cast<const uint32_t*>(p.v_new + src + d);
  *reinterpret_cast<uint32_t*>(p.vc + dst + d + 64) = *reinterpret_cast<const uint32_t*>(p.v_new + src + d + 64);
}

// lens_out[b] = lens[b] + n (a separate launch, so lens_out may alias lens)
__global__ void advance_lens_kernel(const int32_t* lens, int32_t* lens_out, int B, int n) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b < B) lens_out[b] = lens[b] + n;
}

}  // namespace kvcache

GQA_ERROR_FLAG_ACCESSOR(error_flag_kvcache)

}  // namespace gqa

extern "C" int gqa_kv_append_bf16(const void* k_new, const void* v_new, void* kcache, void* vcache,
                                  const int32_t* block_table, int max_pages_per_seq, int page_size, int num_pages,
                                  const int32_t* lens, int32_t* lens_out, const void* cos, const void* sin, int B,
                                  int Hkv, int n_new, int head_dim, int max_len, int flags, gqa_stream_t stream) {
  using namespace gqa;
  using namespace gqa::kvcache;
  if (!k_new || !v_new || !kcache || !vcache || !lens) return GQA_ERR_INVALID_ARGUMENT;
  if (B <= 0 || Hkv <= 0 || n_new <= 0) return GQA_ERR_INVALID_ARGUMENT;
  if (head_dim != kD) return GQA_ERR_UNSUPPORTED;
  if (flags & ~GQA_FLAG_ROPE_K) return GQA_ERR_INVALID_ARGUMENT;
  if ((flags & GQA_FLAG_ROPE_K) && (!cos || !sin)) return GQA_ERR_INVALID_ARGUMENT;
  if (block_table) {
    if (max_pages_per_seq <= 0 || page_size <= 0 || num_pages <= 0) return GQA_ERR_INVALID_ARGUMENT;
  } else if (max_len <= 0) {
    return GQA_ERR_INVALID_ARGUMENT;
  }
  // word (4-byte) accesses throughout
  auto al4 = [](const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 3u) == 0; };
  if (!al4(k_new) || !al4(v_new) || !al4(kcache) || !al4(vcache)) return GQA_ERR_MISALIGNED;
  if ((flags & GQA_FLAG_ROPE_K) && (!al4(cos) || !al4(sin))) return GQA_ERR_MISALIGNED;
  Params p;
  p.k_new = static_cast<const uint16_t*>(k_new);
  p.v_new = static_cast<const uint16_t*>(v_new);
  p.kc = static_cast<uint16_t*>(kcache);
  p.vc = static_cast<uint16_t*>(vcache);
  p.table = block_table;
  p.lens = lens;
  p.cos = static_cast<const uint16_t*>(cos);
  p.sin = static_cast<const uint16_t*>(sin);
  p.rows = static_cast<long long>(B) * Hkv * n_new;
  p.Hkv = Hkv;
  p.n_new = n_new;
  p.max_len = max_len;
  p.page_size = page_size;
  p.max_pages = max_pages_per_seq;
  p.num_pages = num_pages;
  p.flags = flags;
  const long long blocks = (p.rows + kWarps - 1) / kWarps;
  if (blocks > 0x7FFFFFFFLL) return GQA_ERR_UNSUPPORTED;
  append_kernel<<<static_cast<unsigned>(blocks), kWarps * 32, 0, stream>>>(p);
  if (cudaGetLastError() != cudaSuccess) return GQA_ERR_CUDA;
  if (lens_out) {
    advance_lens_kernel<<<(B + 255) / 256, 256, 0, stream>>>(lens, lens_out, B, n_new);
    if (cudaGetLastError() != cudaSuccess) return GQA_ERR_CUDA;
  }
  return GQA_OK;
}
