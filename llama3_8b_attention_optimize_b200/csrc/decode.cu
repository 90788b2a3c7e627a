// decode.cu -- host entry points of the split-KV GQA decode (one query token per
// sequence): argument checks, workspace sizing and the allocation-free variant.
//
// out[b,h,:] = softmax_j(q[b,h] . K[b,h/4,j] * scale, j < lens[b]) . V[b,h/4,:,:]
// This is the single-query-row case of the reference's core
// (CPU_Baseline/cpu_baseline/attention.py:60-84); the reference has no decode
// function of its own.  The kernels (tcgen05 split pass and log-sum-exp combine)
// live in decode_sm100.cu.
#include "common.cuh"
#include "gqa_internal.h"

namespace gqa {
namespace decode {

constexpr int kD = 128;
constexpr int kG = 4;
constexpr int kDefaultSplit = 2048;

inline int effective_split(int max_len, int split_len) {
  (void)max_len;
  return split_len > 0 ? split_len : kDefaultSplit;
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

  return launch_decode_tc(q, kcache, vcache, lens, q_pos, cos, sin, o, static_cast<float*>(workspace), B, max_len, Hq,
                          Hkv, kv_head_begin, kv_head_count, sl, ns, scale, flags, stream);
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

