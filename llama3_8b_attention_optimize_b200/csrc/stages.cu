// stages.cu -- RoPE and the per-stage (debug-dump) kernels.
//
// These reproduce each stage of the golden model with its bf16 boundary
// rounding (llama3_attention_golden_model.py:124-190):
//   rope_cache_kernel  build_rope_cache   :124-130
//   rope_kernel        apply_rope          :133-139 (used :162-164); rope128_kernel is its
//                      16-byte vectorised form for head_dim 128
//   scores_kernel      to_bf16(q k^T * s)  :175-176
//   mask_kernel        to_bf16(s + triu)   :180-181
//   word_mask_kernel   HLS attention_mask  attention_mask_module/src/attention_mask.cpp:3-58
//   softmax_kernel     to_bf16(softmax)    :185
//   pv_kernel          to_bf16(p v)        :189
// Dot products and sums run in fp32 in index order, so results equal the CPU
// restatement of the golden arithmetic bit for bit.  They materialise S x S
// tensors and are meant for the debug dump at small sequence lengths; the fused
// path is gqa_prefill_bf16.
#include "common.cuh"
#include "gqa_internal.h"

namespace gqa {

GQA_ERROR_FLAG_ACCESSOR(error_flag_stages)

namespace {

__global__ void rope_cache_kernel(uint16_t* cos, uint16_t* sin, int S, int D, int pos0, double theta) {
  const int half = D >> 1;
  const long long n = static_cast<long long>(S) * half;
  for (long long idx = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; idx < n;
       idx += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int s = static_cast<int>(idx / half), i = static_cast<int>(idx % half);
    // inv_freq = fl32(1 / fl32(theta ** fl32(2i/d)))
    const float e = __fdiv_rn(static_cast<float>(2 * i), static_cast<float>(D));
    const float pw = static_cast<float>(pow(theta, static_cast<double>(e)));
    const float inv = __fdiv_rn(1.0f, pw);
    const float ang = __fmul_rn(static_cast<float>(pos0 + s), inv);
    const uint16_t c = f2bf_bits(static_cast<float>(::cos(static_cast<double>(ang))));
    const uint16_t sn = f2bf_bits(static_cast<float>(::sin(static_cast<double>(ang))));
    const long long row = static_cast<long long>(s) * D;
    cos[row + i] = c;
    cos[row + i + half] = c;
    sin[row + i] = sn;
    sin[row + i + half] = sn;
  }
}

// One thread per (row, pair d / d+half).
__global__ void rope_kernel(const uint16_t* x, uint16_t* y, const uint16_t* cos, const uint16_t* sin, int H, int S,
                            int D, int pos0) {
  const int half = D >> 1;
  const long long n = static_cast<long long>(H) * S * half;
  for (long long idx = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; idx < n;
       idx += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long row = idx / half;
    const int d = static_cast<int>(idx % half);
    const int s = static_cast<int>(row % S);
    const uint16_t* xr = x + row * D;
    const long long trow = static_cast<long long>(pos0 + s) * D;
    const float x0 = bf2f_bits(xr[d]), x1 = bf2f_bits(xr[d + half]);
    const float c0 = bf2f_bits(cos[trow + d]), s0 = bf2f_bits(sin[trow + d]);
    const float c1 = bf2f_bits(cos[trow + d + half]), s1 = bf2f_bits(sin[trow + d + half]);
    const float y0 = __fadd_rn(__fmul_rn(x0, c0), __fmul_rn(-x1, s0));
    const float y1 = __fadd_rn(__fmul_rn(x1, c1), __fmul_rn(x0, s1));
    y[row * D + d] = f2bf_bits(y0);
    y[row * D + d + half] = f2bf_bits(y1);
  }
}

// rope_kernel's arithmetic for two adjacent pairs packed in bf16x2 words: xa holds
// x[d], x[d+1], xb holds x[d+64], x[d+65]; ca/sa the table words at d, cb/sb at d+64.
__device__ __forceinline__ void rope_words(uint32_t xa, uint32_t xb, uint32_t ca, uint32_t cb, uint32_t sa,
                                           uint32_t sb, uint32_t& ya, uint32_t& yb) {
  uint32_t out_a = 0, out_b = 0;
#pragma unroll
  for (int k = 0; k < 2; ++k) {
    const int sh = 16 * k;
    const float x0 = bf2f_bits(static_cast<uint16_t>(xa >> sh)), x1 = bf2f_bits(static_cast<uint16_t>(xb >> sh));
    const float c0 = bf2f_bits(static_cast<uint16_t>(ca >> sh)), s0 = bf2f_bits(static_cast<uint16_t>(sa >> sh));
    const float c1 = bf2f_bits(static_cast<uint16_t>(cb >> sh)), s1 = bf2f_bits(static_cast<uint16_t>(sb >> sh));
    const float y0 = __fadd_rn(__fmul_rn(x0, c0), __fmul_rn(-x1, s0));
    const float y1 = __fadd_rn(__fmul_rn(x1, c1), __fmul_rn(x0, s1));
    out_a |= static_cast<uint32_t>(f2bf_bits(y0)) << sh;
    out_b |= static_cast<uint32_t>(f2bf_bits(y1)) << sh;
  }
  ya = out_a;
  yb = out_b;
}

// head_dim 128 with 16-byte aligned tensors: one thread per (row, 8 consecutive pairs),
// 16-byte loads and stores, the same per-element arithmetic as rope_kernel (bit-identical).
// This is the K pre-pass of the prefill step, so it runs at HBM speed instead of
// element by element.
__global__ void rope128_kernel(const uint4* x, uint4* y, const uint4* cos, const uint4* sin, int rows, int S,
                               int pos0) {
  const int n = rows * 8;  // 8 chunks of 8 pairs per row; each row is 16 uint4
  for (int idx = blockIdx.x * blockDim.x + threadIdx.x; idx < n; idx += gridDim.x * blockDim.x) {
    const int row = idx >> 3, c = idx & 7;
    const long long xo = static_cast<long long>(row) * 16 + c;
    const long long to = static_cast<long long>(pos0 + row % S) * 16 + c;
    const uint4 a = x[xo], b = x[xo + 8];
    const uint4 ca = __ldg(cos + to), cb = __ldg(cos + to + 8), sa = __ldg(sin + to), sb = __ldg(sin + to + 8);
    uint4 ya, yb;
    rope_words(a.x, b.x, ca.x, cb.x, sa.x, sb.x, ya.x, yb.x);
    rope_words(a.y, b.y, ca.y, cb.y, sa.y, sb.y, ya.y, yb.y);
    rope_words(a.z, b.z, ca.z, cb.z, sa.z, sb.z, ya.z, yb.z);
    rope_words(a.w, b.w, ca.w, cb.w, sa.w, sb.w, ya.w, yb.w);
    y[xo] = ya;
    y[xo + 8] = yb;
  }
}

// One thread per score element; q row cached in shared memory per block row.
__global__ void scores_kernel(const uint16_t* q, const uint16_t* k, uint16_t* out, int Hq, int Hkv, int S, int D,
                              float scale) {
  extern __shared__ float qs[];
  const long long qrow = blockIdx.y;  // over B*Hq*S
  const int G = Hq / Hkv;
  const long long bh = qrow / S;      // b*Hq + h
  const int h = static_cast<int>(bh % Hq);
  const long long b = bh / Hq;
  for (int d = threadIdx.x; d < D; d += blockDim.x) qs[d] = bf2f_bits(q[qrow * D + d]);
  __syncthreads();
  const int j = blockIdx.x * blockDim.x + threadIdx.x;
  if (j >= S) return;
  const uint16_t* kr = k + ((b * Hkv + h / G) * S + j) * static_cast<long long>(D);
  float acc = 0.0f;
  for (int d = 0; d < D; ++d) acc = __fadd_rn(acc, __fmul_rn(qs[d], bf2f_bits(kr[d])));
  out[qrow * S + j] = f2bf_bits(__fmul_rn(acc, scale));
}

__global__ void mask_kernel(const uint16_t* in, uint16_t* out, long long n, int S, int causal) {
  for (long long idx = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; idx < n;
       idx += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int j = static_cast<int>(idx % S);
    const int i = static_cast<int>((idx / S) % S);
    const float m = (causal && j > i) ? -INFINITY : 0.0f;
    out[idx] = f2bf_bits(__fadd_rn(bf2f_bits(in[idx]), m));
  }
}

__global__ void word_mask_kernel(const uint16_t* raw, uint16_t* out, long long n, int S, int causal, uint16_t mv) {
  for (long long idx = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; idx < n;
       idx += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int kt = static_cast<int>(idx % S);
    const int qt = static_cast<int>((idx / S) % S);
    out[idx] = (causal && kt > qt) ? mv : raw[idx];
  }
}

// One thread per row, sequential fp32 max / sum (the golden rounding makes the
// sum order invisible at bf16 except in rare ties; this keeps it bit-exact with
// the restatement).  exp is evaluated in double and rounded to fp32.
__global__ void softmax_kernel(const uint16_t* in, uint16_t* out, long long rows, int cols) {
  for (long long r = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; r < rows;
       r += static_cast<long long>(gridDim.x) * blockDim.x) {
    const uint16_t* x = in + r * cols;
    uint16_t* y = out + r * cols;
    float mx = -INFINITY;
    for (int j = 0; j < cols; ++j) mx = fmaxf(mx, bf2f_bits(x[j]));
    float sum = 0.0f;
    for (int j = 0; j < cols; ++j) sum = __fadd_rn(sum, static_cast<float>(::exp(static_cast<double>(__fsub_rn(bf2f_bits(x[j]), mx)))));
    for (int j = 0; j < cols; ++j) {
      const float e = static_cast<float>(::exp(static_cast<double>(__fsub_rn(bf2f_bits(x[j]), mx))));
      y[j] = f2bf_bits(__fdiv_rn(e, sum));
    }
  }
}

// One thread per output element, fp32 accumulation in key order.
__global__ void pv_kernel(const uint16_t* p, const uint16_t* v, uint16_t* out, long long n, int Hq, int Hkv, int S,
                          int D) {
  const int G = Hq / Hkv;
  for (long long idx = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; idx < n;
       idx += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int d = static_cast<int>(idx % D);
    const long long row = idx / D;        // over B*Hq*S
    const long long bh = row / S;
    const int h = static_cast<int>(bh % Hq);
    const long long b = bh / Hq;
    const uint16_t* pr = p + row * S;
    const uint16_t* vb = v + (b * Hkv + h / G) * static_cast<long long>(S) * D + d;
    float acc = 0.0f;
    for (int j = 0; j < S; ++j) acc = __fadd_rn(acc, __fmul_rn(bf2f_bits(pr[j]), bf2f_bits(vb[static_cast<long long>(j) * D])));
    out[idx] = f2bf_bits(acc);
  }
}

inline unsigned grid_for(long long n, int block) {
  long long g = (n + block - 1) / block;
  if (g > 148LL * 64) g = 148LL * 64;
  return static_cast<unsigned>(g < 1 ? 1 : g);
}

inline int launch_status() { return cudaGetLastError() == cudaSuccess ? GQA_OK : GQA_ERR_CUDA; }

}  // namespace
}  // namespace gqa

using namespace gqa;

extern "C" int gqa_rope_cache_bf16(void* cos, void* sin, int seq_len, int head_dim, int pos0, double theta,
                                   gqa_stream_t stream) {
  if (!cos || !sin || seq_len <= 0 || head_dim <= 0 || (head_dim & 1) || pos0 < 0 || !(theta > 0.0))
    return GQA_ERR_INVALID_ARGUMENT;
  if (head_dim > 1024) return GQA_ERR_UNSUPPORTED;
  const long long n = static_cast<long long>(seq_len) * (head_dim / 2);
  rope_cache_kernel<<<grid_for(n, 256), 256, 0, stream>>>(static_cast<uint16_t*>(cos), static_cast<uint16_t*>(sin),
                                                          seq_len, head_dim, pos0, theta);
  return launch_status();
}

extern "C" int gqa_rope_bf16(const void* x, void* y, const void* cos, const void* sin, int num_heads, int seq_len,
                             int head_dim, int pos0, gqa_stream_t stream) {
  if (!x || !y || !cos || !sin || num_heads <= 0 || seq_len <= 0 || head_dim <= 0 || (head_dim & 1) || pos0 < 0)
    return GQA_ERR_INVALID_ARGUMENT;
  const long long n = static_cast<long long>(num_heads) * seq_len * (head_dim / 2);
  const auto a16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
  if (head_dim == 128 && a16(x) && a16(y) && a16(cos) && a16(sin) &&
      static_cast<long long>(num_heads) * seq_len * 8 <= (1LL << 30)) {
    const int rows = num_heads * seq_len;
    rope128_kernel<<<grid_for(static_cast<long long>(rows) * 8, 256), 256, 0, stream>>>(
        static_cast<const uint4*>(x), static_cast<uint4*>(y), static_cast<const uint4*>(cos),
        static_cast<const uint4*>(sin), rows, seq_len, pos0);
    return launch_status();
  }
  rope_kernel<<<grid_for(n, 256), 256, 0, stream>>>(static_cast<const uint16_t*>(x), static_cast<uint16_t*>(y),
                                                    static_cast<const uint16_t*>(cos),
                                                    static_cast<const uint16_t*>(sin), num_heads, seq_len, head_dim,
                                                    pos0);
  return launch_status();
}

extern "C" int gqa_scores_bf16(const void* q, const void* k, void* scores, int B, int Hq, int Hkv, int seq_len,
                               int head_dim, float scale, gqa_stream_t stream) {
  if (!q || !k || !scores || B <= 0 || Hq <= 0 || Hkv <= 0 || seq_len <= 0 || head_dim <= 0 || Hq % Hkv)
    return GQA_ERR_INVALID_ARGUMENT;
  const long long rows = static_cast<long long>(B) * Hq * seq_len;
  if (rows > 65535 || head_dim > 4096) return GQA_ERR_UNSUPPORTED;  // debug-size path
  dim3 grid((seq_len + 127) / 128, static_cast<unsigned>(rows));
  scores_kernel<<<grid, 128, head_dim * sizeof(float), stream>>>(static_cast<const uint16_t*>(q),
                                                                  static_cast<const uint16_t*>(k),
                                                                  static_cast<uint16_t*>(scores), Hq, Hkv, seq_len,
                                                                  head_dim, scale);
  return launch_status();
}

extern "C" int gqa_mask_bf16(const void* scores, void* masked, int num_heads, int seq_len, int causal,
                             gqa_stream_t stream) {
  if (!scores || !masked || num_heads <= 0 || seq_len <= 0) return GQA_ERR_INVALID_ARGUMENT;
  const long long n = static_cast<long long>(num_heads) * seq_len * seq_len;
  mask_kernel<<<grid_for(n, 256), 256, 0, stream>>>(static_cast<const uint16_t*>(scores),
                                                    static_cast<uint16_t*>(masked), n, seq_len, causal ? 1 : 0);
  return launch_status();
}

extern "C" int gqa_attention_mask_bf16(const void* raw_scores, void* masked_scores, int q_heads, int seq_len,
                                       int causal, uint16_t mask_value, gqa_stream_t stream) {
  if (!raw_scores || !masked_scores || q_heads <= 0 || seq_len <= 0) return GQA_ERR_INVALID_ARGUMENT;
  const long long n = static_cast<long long>(q_heads) * seq_len * seq_len;
  word_mask_kernel<<<grid_for(n, 256), 256, 0, stream>>>(static_cast<const uint16_t*>(raw_scores),
                                                         static_cast<uint16_t*>(masked_scores), n, seq_len,
                                                         causal ? 1 : 0, mask_value);
  return launch_status();
}

extern "C" int gqa_softmax_bf16(const void* scores, void* probs, long long rows, int cols, gqa_stream_t stream) {
  if (!scores || !probs || rows <= 0 || cols <= 0) return GQA_ERR_INVALID_ARGUMENT;
  softmax_kernel<<<grid_for(rows, 128), 128, 0, stream>>>(static_cast<const uint16_t*>(scores),
                                                          static_cast<uint16_t*>(probs), rows, cols);
  return launch_status();
}

extern "C" int gqa_pv_bf16(const void* probs, const void* v, void* out, int B, int Hq, int Hkv, int seq_len,
                           int head_dim, gqa_stream_t stream) {
  if (!probs || !v || !out || B <= 0 || Hq <= 0 || Hkv <= 0 || seq_len <= 0 || head_dim <= 0 || Hq % Hkv)
    return GQA_ERR_INVALID_ARGUMENT;
  const long long n = static_cast<long long>(B) * Hq * seq_len * head_dim;
  pv_kernel<<<grid_for(n, 256), 256, 0, stream>>>(static_cast<const uint16_t*>(probs),
                                                  static_cast<const uint16_t*>(v), static_cast<uint16_t*>(out), n, Hq,
                                                  Hkv, seq_len, head_dim);
  return launch_status();
}
