// decode.cu -- split-KV GQA decode (one query token per sequence) on sm_100a.
//
// out[b,h,:] = softmax_j(q[b,h] . K[b,h/4,j] * scale, j < lens[b]) . V[b,h/4,:,:]
// This is the single-query-row case of the reference's core
// (CPU_Baseline/cpu_baseline/attention.py:60-84); the reference has no decode
// function of its own.  The path is HBM-bound: every K/V byte is read once.
//
// Pass 1 (decode_split_kernel): CTA = (key chunk, kv head, sequence), 4 warps.
//   The chunk's K/V rows are streamed once for all 4 query heads of the group.
//   Each warp walks 32-key groups: lane = key for q.k (16 x 128-bit loads of its
//   K row, q broadcast from shared memory), an online softmax per head, then
//   half-warp = key for p.V (128-bit loads of V rows, p broadcast by shuffle).
//   The warps' (max, sum, O) states merge in shared memory and the chunk's
//   partial (O unnormalised, running max m, sum l) goes to the workspace.
// Pass 2 (decode_combine_kernel): log-sum-exp merge of a sequence's chunks,
//   O = sum_s 2^(m_s - M) O_s / sum_s 2^(m_s - M) l_s, written as bf16.
#include "common.cuh"
#include "gqa_internal.h"

#include <cstdlib>

namespace gqa {
namespace decode {

constexpr int kD = 128;
constexpr int kG = 4;
constexpr int kWarps = 4;
constexpr int kThreads = kWarps * 32;
constexpr int kDefaultSplit = 2048;

struct Params {
  const uint16_t* q;
  const uint16_t* k;
  const uint16_t* v;
  const int32_t* lens;
  const int32_t* q_pos;
  const uint16_t* cos;
  const uint16_t* sin;
  float* ws_o;   // [B][Hq][n_splits][128]
  float* ws_ml;  // [B][Hq][n_splits][2]
  uint16_t* out; // [B][Hq][128]
  int B, Lmax, Hq, Hkv, kv_begin, n_splits, split_len, flags;
  float scale_log2;
};

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__global__ void __launch_bounds__(kThreads) decode_split_kernel(const Params p) {
  __shared__ float q_s[kG][kD];
  __shared__ float m_s[kWarps][kG], l_s[kWarps][kG];
  __shared__ float o_s[kWarps][kG][kD];

  const int split = blockIdx.x, g = p.kv_begin + static_cast<int>(blockIdx.y), b = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int len = min(max(p.lens[b], 0), p.Lmax);
  const int k0 = split * p.split_len;
  if (k0 >= len) return;  // chunk past the end of this sequence
  const int k1 = min(k0 + p.split_len, len);

  // ---- q (4 heads of group g) -> shared fp32, optionally rotated at q_pos[b]
  {
    const int h = threadIdx.x >> 5;  // 4 warps <-> 4 heads
    const uint16_t* qr = p.q + (static_cast<size_t>(b) * p.Hq + g * kG + h) * kD;
#pragma unroll
    for (int e = lane; e < kD / 2; e += 32) {
      float x0 = bf2f_bits(qr[e]), x1 = bf2f_bits(qr[e + kD / 2]);
      if (p.flags & GQA_FLAG_ROPE_Q) {
        const size_t row = static_cast<size_t>(min(max(p.q_pos[b], 0), p.Lmax)) * kD;  // table has Lmax+1 rows
        const float c = bf2f_bits(p.cos[row + e]), s = bf2f_bits(p.sin[row + e]);
        const float y0 = __fadd_rn(__fmul_rn(x0, c), __fmul_rn(-x1, s));
        const float y1 = __fadd_rn(__fmul_rn(x1, c), __fmul_rn(x0, s));
        x0 = bf2f_bits(f2bf_bits(y0));
        x1 = bf2f_bits(f2bf_bits(y1));
      }
      q_s[h][e] = x0;
      q_s[h][e + kD / 2] = x1;
    }
  }
  __syncthreads();

  const size_t kv_base = (static_cast<size_t>(b) * p.Hkv + g) * static_cast<size_t>(p.Lmax) * kD;
  const uint16_t* K = p.k + kv_base;
  const uint16_t* V = p.v + kv_base;
  const float sl2 = p.scale_log2;

  float m_run[kG], l_part[kG], o[kG][8];
#pragma unroll
  for (int h = 0; h < kG; ++h) {
    m_run[h] = -INFINITY;
    l_part[h] = 0.0f;
#pragma unroll
    for (int e = 0; e < 8; ++e) o[h][e] = 0.0f;
  }
  const int half = lane >> 4;      // which key of a pair this half-warp handles in p.V
  const int dchunk = lane & 15;    // 8 dims [8*dchunk, 8*dchunk+8)

  for (int gk = k0 + warp * 32; gk < k1; gk += kWarps * 32) {
    // ---- q.k, lane = key
    const int key = gk + lane;
    float s[kG];
#pragma unroll
    for (int h = 0; h < kG; ++h) s[h] = 0.0f;
    if (key < k1) {
      const uint4* kr = reinterpret_cast<const uint4*>(K + static_cast<size_t>(key) * kD);
      uint4 kv[16];
#pragma unroll
      for (int c = 0; c < 16; ++c) kv[c] = __ldg(kr + c);
#pragma unroll
      for (int c = 0; c < 16; ++c) {
        const uint32_t w[4] = {kv[c].x, kv[c].y, kv[c].z, kv[c].w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float k_lo = bf16_lo(w[e]), k_hi = bf16_hi(w[e]);
#pragma unroll
          for (int h = 0; h < kG; ++h) {
            const float2 qq = *reinterpret_cast<const float2*>(&q_s[h][c * 8 + e * 2]);
            s[h] = fmaf(qq.x, k_lo, s[h]);
            s[h] = fmaf(qq.y, k_hi, s[h]);
          }
        }
      }
    }
    // ---- online softmax per head over this 32-key group
    float pk[kG];
#pragma unroll
    for (int h = 0; h < kG; ++h) {
      const float x = key < k1 ? s[h] * sl2 : -INFINITY;
      const float m_new = fmaxf(m_run[h], warp_max(x));  // finite: the group has >= 1 valid key
      const float alpha = ex2_approx(m_run[h] - m_new);
      pk[h] = ex2_approx(x - m_new);
      l_part[h] = l_part[h] * alpha + pk[h];
#pragma unroll
      for (int e = 0; e < 8; ++e) o[h][e] *= alpha;
      m_run[h] = m_new;
    }
    // ---- p.V, half-warp = key (2 keys per step)
    const int nk = min(32, k1 - gk);
    for (int e = 0; e < nk; e += 2) {
      const int src = e + half;
      float pp[kG];
#pragma unroll
      for (int h = 0; h < kG; ++h) pp[h] = __shfl_sync(0xffffffffu, pk[h], src);
      if (src < nk) {
        const uint4 vv = __ldg(reinterpret_cast<const uint4*>(V + static_cast<size_t>(gk + src) * kD) + dchunk);
        const uint32_t w[4] = {vv.x, vv.y, vv.z, vv.w};
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float v_lo = bf16_lo(w[q]), v_hi = bf16_hi(w[q]);
#pragma unroll
          for (int h = 0; h < kG; ++h) {
            o[h][2 * q] = fmaf(pp[h], v_lo, o[h][2 * q]);
            o[h][2 * q + 1] = fmaf(pp[h], v_hi, o[h][2 * q + 1]);
          }
        }
      }
    }
  }

  // ---- per-warp reduction: halves hold different keys for the same dims
#pragma unroll
  for (int h = 0; h < kG; ++h) {
    const float lsum = warp_sum(l_part[h]);
#pragma unroll
    for (int e = 0; e < 8; ++e) o[h][e] += __shfl_xor_sync(0xffffffffu, o[h][e], 16);
    if (lane == 0) {
      m_s[warp][h] = m_run[h];
      l_s[warp][h] = lsum;
    }
    if (lane < 16) {
#pragma unroll
      for (int e = 0; e < 8; ++e) o_s[warp][h][dchunk * 8 + e] = o[h][e];
    }
  }
  __syncthreads();

  // ---- merge the 4 warps; thread = (head, 32 dims)
  {
    const int h = threadIdx.x >> 5;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) M = fmaxf(M, m_s[w][h]);
    float L = 0.0f, sc[kWarps];
#pragma unroll
    for (int w = 0; w < kWarps; ++w) {
      sc[w] = (m_s[w][h] == -INFINITY) ? 0.0f : ex2_approx(m_s[w][h] - M);
      L += l_s[w][h] * sc[w];
    }
    const size_t slot = (static_cast<size_t>(b) * p.Hq + g * kG + h) * p.n_splits + split;
#pragma unroll
    for (int e = lane; e < kD; e += 32) {
      float acc = 0.0f;
#pragma unroll
      for (int w = 0; w < kWarps; ++w) acc += o_s[w][h][e] * sc[w];
      p.ws_o[slot * kD + e] = acc;
    }
    if (lane == 0) {
      p.ws_ml[slot * 2 + 0] = M;
      p.ws_ml[slot * 2 + 1] = L;
    }
  }
}

// grid = (kv_count*4 heads, B); block = 128 threads (thread = dim).
__global__ void __launch_bounds__(kD) decode_combine_kernel(const Params p) {
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

inline int effective_split(int max_len, int split_len) {
  if (split_len > 0) return split_len;
  return kDefaultSplit;
}

// The tcgen05 split-KV kernel (decode_sm100.cu) is the default; GQA_DECODE_CUDA_CORES=1
// selects the CUDA-core kernel above (kept as a cross-check of the tensor-core path).
inline bool use_tensor_core_decode() {
  static const bool tc = [] {
    const char* e = getenv("GQA_DECODE_CUDA_CORES");
    return !(e && e[0] == '1');
  }();
  return tc;
}

}  // namespace decode
}  // namespace gqa

using namespace gqa;

extern "C" size_t gqa_decode_workspace_size(int B, int Hq, int max_len, int split_len) {
  if (B <= 0 || Hq <= 0 || max_len <= 0 || split_len < 0) return 0;
  const int sl = decode::effective_split(max_len, split_len);
  const size_t ns = (static_cast<size_t>(max_len) + sl - 1) / sl;
  return static_cast<size_t>(B) * Hq * ns * (decode::kD + 2) * sizeof(float);
}

extern "C" int gqa_decode_bf16(const void* q, const void* kcache, const void* vcache, const int32_t* lens,
                               const int32_t* q_pos, const void* cos, const void* sin, void* o, void* workspace,
                               size_t workspace_bytes, int B, int max_len, int Hq, int Hkv, int head_dim,
                               int kv_head_begin, int kv_head_count, int split_len, float scale, int flags,
                               gqa_stream_t stream) {
  using namespace decode;
  if (!q || !kcache || !vcache || !lens || !o) return GQA_ERR_INVALID_ARGUMENT;
  if (B <= 0 || max_len <= 0 || Hq <= 0 || Hkv <= 0 || split_len < 0) return GQA_ERR_INVALID_ARGUMENT;
  if (head_dim != kD || Hq != kG * Hkv) return GQA_ERR_UNSUPPORTED;
  if (kv_head_begin < 0 || kv_head_count <= 0 || kv_head_begin + kv_head_count > Hkv) return GQA_ERR_INVALID_ARGUMENT;
  if (split_len % 64) return GQA_ERR_INVALID_ARGUMENT;
  if (!(scale > 0.0f) || !(scale < 1e30f)) return GQA_ERR_INVALID_ARGUMENT;
  if (flags & ~(GQA_FLAG_ROPE_Q)) return GQA_ERR_INVALID_ARGUMENT;
  if ((flags & GQA_FLAG_ROPE_Q) && (!cos || !sin || !q_pos)) return GQA_ERR_INVALID_ARGUMENT;
  if (!aligned16(q) || !aligned16(kcache) || !aligned16(vcache) || !aligned16(o)) return GQA_ERR_MISALIGNED;
  const size_t need = gqa_decode_workspace_size(B, Hq, max_len, split_len);
  if (!workspace || workspace_bytes < need) return GQA_ERR_WORKSPACE;
  if (!aligned16(workspace)) return GQA_ERR_MISALIGNED;
  const int sl = effective_split(max_len, split_len);
  const int ns = (max_len + sl - 1) / sl;
  if (ns > 65535 || B > 65535) return GQA_ERR_UNSUPPORTED;

  Params p;
  p.q = static_cast<const uint16_t*>(q);
  p.k = static_cast<const uint16_t*>(kcache);
  p.v = static_cast<const uint16_t*>(vcache);
  p.lens = lens;
  p.q_pos = q_pos;
  p.cos = static_cast<const uint16_t*>(cos);
  p.sin = static_cast<const uint16_t*>(sin);
  float* ws = static_cast<float*>(workspace);
  const size_t n_slots = static_cast<size_t>(B) * Hq * ns;
  p.ws_o = ws;
  p.ws_ml = ws + n_slots * kD;
  p.out = static_cast<uint16_t*>(o);
  p.B = B;
  p.Lmax = max_len;
  p.Hq = Hq;
  p.Hkv = Hkv;
  p.kv_begin = kv_head_begin;
  p.n_splits = ns;
  p.split_len = sl;
  p.flags = flags;
  p.scale_log2 = scale * 1.4426950408889634f;
  if (use_tensor_core_decode())
    return launch_decode_tc(q, kcache, vcache, lens, q_pos, cos, sin, o, ws, B, max_len, Hq, Hkv, kv_head_begin,
                            kv_head_count, sl, ns, scale, flags, stream);
  decode_split_kernel<<<dim3(ns, kv_head_count, B), kThreads, 0, stream>>>(p);
  if (cudaGetLastError() != cudaSuccess) return GQA_ERR_CUDA;
  decode_combine_kernel<<<dim3(kv_head_count * kG, B), kD, 0, stream>>>(p);
  return cudaGetLastError() == cudaSuccess ? GQA_OK : GQA_ERR_CUDA;
}

// ---------------------------------------------------------------------------
// Decode over a paged K/V cache: the same tensor-core split-KV kernel, its TMA
// producer resolving each 128-key chunk through the block table.
extern "C" int gqa_decode_paged_bf16(const void* q, const void* kpages, const void* vpages, const int32_t* block_table,
                                     int max_pages_per_seq, int page_size, int num_pages, const int32_t* lens,
                                     const int32_t* q_pos, const void* cos, const void* sin, void* o, void* workspace,
                                     size_t workspace_bytes, int B, int Hq, int Hkv, int head_dim, int kv_head_begin,
                                     int kv_head_count, int split_len, float scale, int flags, gqa_stream_t stream) {
  using namespace decode;
  if (!q || !kpages || !vpages || !block_table || !lens || !o) return GQA_ERR_INVALID_ARGUMENT;
  if (B <= 0 || Hq <= 0 || Hkv <= 0 || split_len < 0) return GQA_ERR_INVALID_ARGUMENT;
  if (max_pages_per_seq <= 0 || page_size <= 0 || num_pages <= 0) return GQA_ERR_INVALID_ARGUMENT;
  if (head_dim != kD || Hq != kG * Hkv) return GQA_ERR_UNSUPPORTED;
  // chunks of 128 keys must not straddle pages, and splits must start on a chunk
  if (page_size % 128 || split_len % 128) return GQA_ERR_UNSUPPORTED;
  const long long capacity = static_cast<long long>(max_pages_per_seq) * page_size;
  if (capacity > (1LL << 30) || static_cast<long long>(num_pages) * Hkv > (1LL << 31) - 1 || page_size > (1 << 20))
    return GQA_ERR_UNSUPPORTED;
  if (kv_head_begin < 0 || kv_head_count <= 0 || kv_head_begin + kv_head_count > Hkv) return GQA_ERR_INVALID_ARGUMENT;
  if (!(scale > 0.0f) || !(scale < 1e30f)) return GQA_ERR_INVALID_ARGUMENT;
  if (flags & ~(GQA_FLAG_ROPE_Q)) return GQA_ERR_INVALID_ARGUMENT;
  if ((flags & GQA_FLAG_ROPE_Q) && (!cos || !sin || !q_pos)) return GQA_ERR_INVALID_ARGUMENT;
  if (!aligned16(q) || !aligned16(kpages) || !aligned16(vpages) || !aligned16(o)) return GQA_ERR_MISALIGNED;
  const int max_len = static_cast<int>(capacity);
  const size_t need = gqa_decode_workspace_size(B, Hq, max_len, split_len);
  if (!workspace || workspace_bytes < need) return GQA_ERR_WORKSPACE;
  if (!aligned16(workspace)) return GQA_ERR_MISALIGNED;
  const int sl = effective_split(max_len, split_len);
  const int ns = (max_len + sl - 1) / sl;
  if (ns > 65535 || B > 65535) return GQA_ERR_UNSUPPORTED;
  return launch_decode_tc(q, kpages, vpages, lens, q_pos, cos, sin, o, static_cast<float*>(workspace), B, max_len, Hq,
                          Hkv, kv_head_begin, kv_head_count, sl, ns, scale, flags, stream, block_table, page_size,
                          max_pages_per_seq, num_pages);
}

// ---------------------------------------------------------------------------
// Allocation-free variant of gqa_decode_bf16.
//
// Some callers cannot allocate device memory: a plugin host that hands the
// library only its own input and output buffers and owns every other byte of
// device memory, a serving loop that must not call cudaMalloc/cudaFree because
// those calls synchronise the device, or a process whose memory pool was
// reserved in full before the model started.  For them the split-KV partials
// live in a fixed scratch array compiled into this library instead of a
// caller-provided workspace.
//
// Limits and sharing rules:
//  - The scratch holds kNoAllocScratchBytes (16 MiB) per GPU; every GPU that
//    loads the library keeps it for the life of the process.  A request whose
//    partials need more (gqa_decode_workspace_size(B, Hq, max_len, split_len))
//    is rejected with GQA_ERR_WORKSPACE before anything is launched.
//  - All calls on a device share the one array, and it keeps the previous
//    call's contents.  Nothing in it has to start at zero: every slot the
//    combine step reads is written earlier in the same call.  Two calls whose
//    kernels overlap on the GPU (different streams, no ordering between them)
//    race on the array and produce wrong results; order them on one stream.
//  - The first call on each device looks up the array's device address with
//    cudaGetSymbolAddress (with that device current); make that first call
//    before any stream capture begins.
namespace gqa {
namespace decode {

constexpr size_t kNoAllocScratchBytes = 16u << 20;
static __device__ __align__(256) float g_decode_scratch[kNoAllocScratchBytes / sizeof(float)];

constexpr int kMaxDevices = 64;
std::atomic<float*> g_scratch_ptr[kMaxDevices];

// Device address of g_decode_scratch on the current device (looked up once).
// In host code the symbol name is only a host-side handle; kernels must be given
// the address returned by cudaGetSymbolAddress.
int scratch_address(float** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return GQA_ERR_NO_DEVICE;
  if (dev < 0 || dev >= kMaxDevices) return GQA_ERR_UNSUPPORTED;
  float* p = g_scratch_ptr[dev].load(std::memory_order_acquire);
  if (p == nullptr) {
    void* addr = nullptr;
    if (cudaGetSymbolAddress(&addr, g_decode_scratch) != cudaSuccess || addr == nullptr) return GQA_ERR_CUDA;
    p = static_cast<float*>(addr);
    g_scratch_ptr[dev].store(p, std::memory_order_release);
  }
  *out = p;
  return GQA_OK;
}

}  // namespace decode
}  // namespace gqa

extern "C" size_t gqa_decode_noalloc_scratch_bytes(void) { return gqa::decode::kNoAllocScratchBytes; }

extern "C" int gqa_decode_bf16_noalloc(const void* q, const void* kcache, const void* vcache, const int32_t* lens,
                                       const int32_t* q_pos, const void* cos, const void* sin, void* o, int B,
                                       int max_len, int Hq, int Hkv, int head_dim, int kv_head_begin,
                                       int kv_head_count, int split_len, float scale, int flags,
                                       gqa_stream_t stream) {
  using namespace gqa::decode;
  if (B <= 0 || Hq <= 0 || max_len <= 0 || split_len < 0) return GQA_ERR_INVALID_ARGUMENT;
  const size_t need = gqa_decode_workspace_size(B, Hq, max_len, split_len);
  if (need == 0) return GQA_ERR_INVALID_ARGUMENT;
  if (need > kNoAllocScratchBytes) return GQA_ERR_WORKSPACE;
  float* scratch = nullptr;
  const int rc = scratch_address(&scratch);
  if (rc != GQA_OK) return rc;
  return gqa_decode_bf16(q, kcache, vcache, lens, q_pos, cos, sin, o, scratch, kNoAllocScratchBytes, B, max_len, Hq,
                         Hkv, head_dim, kv_head_begin, kv_head_count, split_len, scale, flags, stream);
}

namespace gqa {
GQA_ERROR_FLAG_ACCESSOR(error_flag_decode)
}  // namespace gqa
