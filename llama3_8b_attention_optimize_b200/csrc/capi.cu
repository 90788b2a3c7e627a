// capi.cu -- C-ABI glue: status strings, device-error readback, TMA descriptor
// encoding, and the extern "C" entry of the fused prefill kernel.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "common.cuh"
#include "gqa_internal.h"

namespace gqa {

namespace {

PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::once_flag g_encode_once;

void resolve_encode() {
  void* fn = nullptr;
  cudaDriverEntryPointQueryResult q;
  if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &fn, 12000, cudaEnableDefault, &q) == cudaSuccess &&
      q == cudaDriverEntryPointSuccess)
    g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
}

}  // namespace

int make_tmap_3d_bf16(CUtensorMap* map, const void* base, long long dim0, long long dim1, long long dim2, int box0,
                      int box1, int box2) {
  std::call_once(g_encode_once, resolve_encode);
  if (!g_encode) return GQA_ERR_NO_DEVICE;
  if (box0 * 2 > 128 || box0 <= 0 || box1 <= 0 || box2 <= 0 || box1 > 256 || box2 > 256) return GQA_ERR_UNSUPPORTED;
  cuuint64_t gdim[3] = {static_cast<cuuint64_t>(dim0), static_cast<cuuint64_t>(dim1), static_cast<cuuint64_t>(dim2)};
  cuuint64_t gstride[2] = {static_cast<cuuint64_t>(dim0) * 2, static_cast<cuuint64_t>(dim0 * dim1) * 2};
  cuuint32_t box[3] = {static_cast<cuuint32_t>(box0), static_cast<cuuint32_t>(box1), static_cast<cuuint32_t>(box2)};
  cuuint32_t estride[3] = {1, 1, 1};
  CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), gdim, gstride, box, estride,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? GQA_OK : GQA_ERR_UNSUPPORTED;
}

int make_tmap_4d(CUtensorMap* map, const void* base, int elem_bytes, const long long dims[4],
                 const long long strides[3], const int box[4]) {
  std::call_once(g_encode_once, resolve_encode);
  if (!g_encode) return GQA_ERR_NO_DEVICE;
  if (elem_bytes != 2 && elem_bytes != 4) return GQA_ERR_UNSUPPORTED;
  if (box[0] * elem_bytes > 128 || (box[0] * elem_bytes) % 16) return GQA_ERR_UNSUPPORTED;
  cuuint64_t gdim[4];
  cuuint64_t gstride[3];
  cuuint32_t bx[4], estride[4] = {1, 1, 1, 1};
  for (int i = 0; i < 4; ++i) {
    if (dims[i] <= 0 || box[i] <= 0 || box[i] > 256) return GQA_ERR_UNSUPPORTED;
    gdim[i] = static_cast<cuuint64_t>(dims[i]);
    bx[i] = static_cast<cuuint32_t>(box[i]);
  }
  for (int i = 0; i < 3; ++i) {
    if (strides[i] <= 0 || strides[i] % 16) return GQA_ERR_MISALIGNED;
    gstride[i] = static_cast<cuuint64_t>(strides[i]);
  }
  CUresult r = g_encode(map, elem_bytes == 2 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4,
                        const_cast<void*>(base), gdim, gstride, bx, estride, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? GQA_OK : GQA_ERR_UNSUPPORTED;
}

}  // namespace gqa

using namespace gqa;

extern "C" const char* gqa_strerror(int code) {
  switch (code) {
    case GQA_OK: return "ok";
    case GQA_ERR_INVALID_ARGUMENT: return "invalid argument (null pointer, size or flag)";
    case GQA_ERR_UNSUPPORTED: return "unsupported shape (head_dim must be 128 and Hq = 4*Hkv)";
    case GQA_ERR_MISALIGNED: return "pointer not 16-byte aligned";
    case GQA_ERR_CUDA: return "CUDA error";
    case GQA_ERR_DEVICE_TIMEOUT: return "a kernel's bounded wait expired (device error flag set)";
    case GQA_ERR_WORKSPACE: return "workspace missing or too small";
    case GQA_ERR_NO_DEVICE: return "no usable sm_100 device / driver entry point";
    case GQA_ERR_DEVICE_INPUT: return "a kernel found invalid device-side input (page index or cache capacity)";
    default: return "unknown status";
  }
}

extern "C" int gqa_version(void) { return 1 * 10000 + 0 * 100 + 0; }

extern "C" int gqa_device_check(gqa_stream_t stream, int* site) {
  if (site) *site = 0;
  if (cudaStreamSynchronize(stream) != cudaSuccess) return GQA_ERR_CUDA;
  int (*const readers[])(bool) = {error_flag_stages, error_flag_prefill, error_flag_decode_tc,
                                   error_flag_gemm,   error_flag_kvcache, error_flag_peer};
  int first = 0;
  for (auto rd : readers) {  // read and clear every file's word; report the first set one
    const int v = rd(true);
    if (v < 0) return GQA_ERR_CUDA;
    if (first == 0) first = v;
  }
  if (first == 0) return GQA_OK;
  if (site) *site = first;
  // sites 0x600-0x6ff are checks of device-side input data, the rest are bounded waits
  return (first >= 0x600 && first < 0x700) ? GQA_ERR_DEVICE_INPUT : GQA_ERR_DEVICE_TIMEOUT;
}

extern "C" int gqa_prefill_bf16(const void* q, const void* k, const void* v, void* o, const void* cos, const void* sin,
                                int B, int seq_len, int Hq, int Hkv, int head_dim, int kv_head_begin,
                                int kv_head_count, float scale, int flags, gqa_stream_t stream) {
  return launch_prefill(q, k, v, o, cos, sin, B, seq_len, Hq, Hkv, head_dim, kv_head_begin, kv_head_count, scale,
                        flags, stream);
}
