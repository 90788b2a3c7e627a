// gqa_internal.h -- host-side helpers shared by the kernel translation units.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <atomic>
#include <cstdint>

#include "../../include/gqa_b200.h"

namespace gqa {

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Encode a 3-D bf16 tensor map over a contiguous [dim2][dim1][dim0] array with a
// (box0, box1, box2) box and 128-byte swizzle (box0 * 2 bytes must be <= 128).
int make_tmap_3d_bf16(CUtensorMap* map, const void* base, long long dim0, long long dim1, long long dim2, int box0,
                      int box1, int box2);

// Encode a 4-D tensor map (bf16 or fp32 elements) with 128-byte swizzle: dims are
// innermost first, strides (bytes) belong to dims 1..3, box[0] * elem_bytes <= 128.
int make_tmap_4d(CUtensorMap* map, const void* base, int elem_bytes, const long long dims[4],
                 const long long strides[3], const int box[4]);

// Set cudaFuncAttributeMaxDynamicSharedMemorySize once per device for `func`.
template <typename F>
int ensure_smem_attr(F func, int bytes, std::atomic<uint64_t>& done_mask) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return GQA_ERR_NO_DEVICE;
  const uint64_t bit = 1ull << (dev & 63);
  if (done_mask.load(std::memory_order_acquire) & bit) return GQA_OK;
  if (cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) != cudaSuccess)
    return GQA_ERR_CUDA;
  done_mask.fetch_or(bit, std::memory_order_acq_rel);
  return GQA_OK;
}

// Per-file device error words (see GQA_ERROR_FLAG_ACCESSOR): value, optionally cleared.
int error_flag_stages(bool clear);
int error_flag_prefill(bool clear);
int error_flag_decode_tc(bool clear);
int error_flag_gemm(bool clear);
int error_flag_kvcache(bool clear);
int error_flag_peer(bool clear);

int launch_prefill(const void* q, const void* k, const void* v, void* o, const void* cos, const void* sin, int B, int S,
                   int Hq, int Hkv, int head_dim, int kv_begin, int kv_count, float scale, int flags,
                   cudaStream_t stream);

int launch_o_proj_scatter(const void* attn, const void* wo, int S, int Hq, int N, int ldw, float* const* dst,
                          uint32_t* const* flags, int world, uint32_t* counter, uint32_t epoch, float* local,
                          cudaStream_t stream);

// Device address of the GEMM file's sticky error word on the current device (looked up
// once per device), so kernels of other files can refuse to signal after a failed GEMM.
int gemm_error_word(const int** out);

int launch_decode_tc(const void* q, const void* kcache, const void* vcache, const int32_t* lens, const int32_t* q_pos,
                     const void* cos, const void* sin, void* o, float* ws, int B, int max_len, int Hq, int Hkv,
                     int kv_begin, int kv_count, int split_len, int n_splits, float scale, int flags,
                     cudaStream_t stream, const int32_t* table = nullptr, int page_size = 0, int max_pages = 0,
                     int num_pages = 0);

}  // namespace gqa
