// peer.cu -- tensor-parallel o_proj reduction over NVLink peer memory (no NCCL).
//
// Row-parallel o_proj leaves every rank with an fp32 partial [S][N] of the same output;
// the layer's result is bf16(sum over ranks).  Each rank exports one buffer
//   [partial fp32 S x N][out bf16 S x N][flags]
// through CUDA IPC and maps its peers' buffers.  One step (epoch e) is three launches per
// rank after the o_proj GEMM has written the local partial:
//   1. signal: raise this rank's "partial ready" flag to e;
//   2. tp_reduce: wait until every rank's "partial ready" flag is e, then sum the rank's
//      own row block of all partials in rank order by P2P loads over NVLink, round once
//      to bf16, store into the local out; the last block to finish raises this rank's
//      "block done" flag to e;
//   3. tp_gather: wait until every rank's "block done" flag is e, then copy the other
//      ranks' bf16 row blocks from their out buffers (P2P loads) into the local out.
// Flags are raised with a system-scope release after a system-scope fence and read with
// system-scope acquire loads; every wait is bounded (2 s) and records an error site.
// Ordering across steps: a rank starts the next step's GEMM (overwriting its partial)
// only after its gather of this step saw every owner's "done" flag, i.e. after every
// owner finished reading its partial; an owner overwrites its out block only after every
// rank raised the next "ready" flag, i.e. after every rank finished its gather.
// The waiting kernels run on different GPUs (one rank per GPU), never two on one GPU.
#include <cstring>

#include "common.cuh"
#include "gqa_internal.h"

namespace gqa {
namespace peer {

constexpr int kMaxRanks = 8;
constexpr int kThreads = 256;
constexpr int kUnroll = 4;

enum : int {
  SITE_READY = 0x401,
  SITE_DONE = 0x402,
};

struct Ptrs {
  const float* partial[kMaxRanks];  // each rank's fp32 partial [S][N]
  const uint16_t* out[kMaxRanks];   // each rank's bf16 out [S][N]
  uint32_t* ready[kMaxRanks];       // each rank's "partial ready" flag
  uint32_t* done[kMaxRanks];        // each rank's "block done" flag
};

struct Params {
  Ptrs p;
  uint16_t* out_local;
  uint32_t* counter;  // local arrival counter of tp_reduce's blocks (zero between launches)
  int world, rank, S, N;
  uint32_t epoch;
};

__device__ __forceinline__ void st_release_sys(uint32_t* a, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(a), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* a) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(a) : "memory");
  return v;
}

// Bounded wait until *flag (a peer's or our own) reaches epoch (flags only increase).
__device__ bool wait_flag(const uint32_t* flag, uint32_t epoch, int site) {
  const unsigned long long t0 = globaltimer_ns();
  for (uint32_t it = 0;; ++it) {
    if (static_cast<int32_t>(ld_acquire_sys(flag) - epoch) >= 0) return true;
    if ((it & 255u) == 255u) {
      if (error_pending()) return false;
      if (globaltimer_ns() - t0 > kWaitTimeoutNs) {
        record_error(site);
        return false;
      }
    }
  }
}

// This rank's partial (written by the preceding GEMM launch) is ready.  Not raised when
// that GEMM or an earlier exchange kernel on this GPU gave up a wait: the peers' bounded
// waits then expire and they report the timeout too, instead of summing a stale partial.
__global__ void signal_kernel(uint32_t* flag, uint32_t epoch, const int* gemm_error) {
  __threadfence_system();
  if (*reinterpret_cast<const volatile int*>(gemm_error) == 0 && !error_pending()) st_release_sys(flag, epoch);
}

__global__ void __launch_bounds__(kThreads) tp_reduce_kernel(const Params prm) {
  __shared__ int ok_s;
  if (threadIdx.x == 0) {
    bool ok = true;
    for (int r = 0; r < prm.world && ok; ++r) ok = wait_flag(prm.p.ready[r], prm.epoch, SITE_READY);
    ok_s = ok ? 1 : 0;
  }
  __syncthreads();
  const int rows = prm.S / prm.world;
  const long long n4 = static_cast<long long>(rows) * prm.N / 4;  // float4 units of the block
  const long long base = static_cast<long long>(prm.rank) * rows * prm.N;
  if (ok_s) {
    // kUnroll independent float4 units per thread per round, all loads issued before the
    // adds: remote (NVLink) loads need many bytes in flight
    const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
    for (long long i0 = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i0 < n4;
         i0 += kUnroll * stride) {
      float4 acc[kUnroll];
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        const long long i = i0 + u * stride;
        // peer data is read past L1 (__ldcg): it changes between launches
        acc[u] = i < n4 ? __ldcg(reinterpret_cast<const float4*>(prm.p.partial[0] + base) + i)
                        : make_float4(0.f, 0.f, 0.f, 0.f);
      }
      for (int r = 1; r < prm.world; ++r) {  // rank order: the same sums on every owner
        float4 x[kUnroll];
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
          const long long i = i0 + u * stride;
          x[u] = i < n4 ? __ldcg(reinterpret_cast<const float4*>(prm.p.partial[r] + base) + i)
                        : make_float4(0.f, 0.f, 0.f, 0.f);
        }
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
          acc[u].x += x[u].x;
          acc[u].y += x[u].y;
          acc[u].z += x[u].z;
          acc[u].w += x[u].w;
        }
      }
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        const long long i = i0 + u * stride;
        if (i < n4) {
          uint2 w;
          w.x = static_cast<uint32_t>(f2bf_bits(acc[u].x)) | (static_cast<uint32_t>(f2bf_bits(acc[u].y)) << 16);
          w.y = static_cast<uint32_t>(f2bf_bits(acc[u].z)) | (static_cast<uint32_t>(f2bf_bits(acc[u].w)) << 16);
          reinterpret_cast<uint2*>(prm.out_local + base)[i] = w;
        }
      }
    }
  }
  // the last block to finish announces this rank's block (all blocks' stores fenced first)
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    const uint32_t arrived = atomicAdd(prm.counter, 1u) + 1u;
    if (arrived == gridDim.x) {
      *prm.counter = 0u;
      __threadfence_system();
      // every block's wait result is recorded before its arrival: one that gave up
      // leaves the error word set, and then no block is announced
      if (ok_s && !error_pending()) st_release_sys(prm.p.done[prm.rank], prm.epoch);
    }
  }
}

__global__ void __launch_bounds__(kThreads) tp_gather_kernel(const Params prm) {
  __shared__ int ok_s;
  if (threadIdx.x == 0) {
    bool ok = true;
    for (int r = 0; r < prm.world && ok; ++r) ok = wait_flag(prm.p.done[r], prm.epoch, SITE_DONE);
    ok_s = ok ? 1 : 0;
  }
  __syncthreads();
  if (!ok_s) return;
  const int rows = prm.S / prm.world;
  const long long blk16 = static_cast<long long>(rows) * prm.N * 2 / 16;  // uint4 units per block
  const long long total = blk16 * (prm.world - 1);
  const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
  for (long long i0 = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i0 < total;
       i0 += kUnroll * stride) {
    uint4 v[kUnroll];
    long long dst[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const long long i = i0 + u * stride;
      dst[u] = -1;
      if (i < total) {
        int q = static_cast<int>(i / blk16);
        q += (q >= prm.rank);  // the other ranks' blocks
        const long long off = static_cast<long long>(q) * blk16 + i % blk16;
        v[u] = __ldcg(reinterpret_cast<const uint4*>(prm.p.out[q]) + off);
        dst[u] = off;
      }
    }
#pragma unroll
    for (int u = 0; u < kUnroll; ++u)
      if (dst[u] >= 0) reinterpret_cast<uint4*>(prm.out_local)[dst[u]] = v[u];
  }
}

// ---------------------------------------------------------------- push variant
// The o_proj GEMM itself stores each row of its fp32 partial into the owner's buffer:
// rank r's rows of owner q's block land in q's slot r (the buffer's fp32 region read as
// [world][S / world][N]); its last CTA raises flagA[r] = e at every owner.  Then:
//   tp_reduce_push: wait until flagA[0..world) of the local buffer are e, sum the local
//     slots in rank order, round once, store the bf16 block into every rank's out (P2P
//     stores), and the last block raises flagB[rank] = e at every rank;
//   tp_wait: wait until flagB[0..world) of the local buffer are e.
// All peer traffic is stores, issued while the GEMM is still computing other tiles.
struct PushParams {
  uint16_t* out[kMaxRanks];         // each rank's bf16 out [S][N]
  uint32_t* flag_b[kMaxRanks];      // flagB[rank] in each rank's buffer
  const float* slots;               // local [world][S / world][N]
  const uint32_t* local_a;          // local flagA[world]
  const uint32_t* local_b;          // local flagB[world]
  uint32_t* counter;                // local block counter
  int world, rank, S, N;
  uint32_t epoch;
};

__device__ __forceinline__ uint16_t* out_at(const PushParams& p, int q) {
  switch (q) {
    case 0: return p.out[0];
    case 1: return p.out[1];
    case 2: return p.out[2];
    case 3: return p.out[3];
    case 4: return p.out[4];
    case 5: return p.out[5];
    case 6: return p.out[6];
    default: return p.out[7];
  }
}

__global__ void __launch_bounds__(kThreads) tp_reduce_push_kernel(const PushParams prm) {
  __shared__ int ok_s;
  if (threadIdx.x == 0) {
    bool ok = true;
    for (int r = 0; r < prm.world && ok; ++r) ok = wait_flag(prm.local_a + r, prm.epoch, SITE_READY);
    ok_s = ok ? 1 : 0;
  }
  __syncthreads();
  const int rows = prm.S / prm.world;
  const long long n4 = static_cast<long long>(rows) * prm.N / 4;
  const long long out_base = static_cast<long long>(prm.rank) * rows * prm.N;  // elements
  if (ok_s) {
    const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n4; i += stride) {
      // slots were written by other GPUs: read past L1
      float4 acc = __ldcg(reinterpret_cast<const float4*>(prm.slots) + i);
      for (int r = 1; r < prm.world; ++r) {
        const float4 x = __ldcg(reinterpret_cast<const float4*>(prm.slots + static_cast<size_t>(r) * rows * prm.N) + i);
        acc.x += x.x;
        acc.y += x.y;
        acc.z += x.z;
        acc.w += x.w;
      }
      uint2 w;
      w.x = static_cast<uint32_t>(f2bf_bits(acc.x)) | (static_cast<uint32_t>(f2bf_bits(acc.y)) << 16);
      w.y = static_cast<uint32_t>(f2bf_bits(acc.z)) | (static_cast<uint32_t>(f2bf_bits(acc.w)) << 16);
      for (int q = 0; q < prm.world; ++q) reinterpret_cast<uint2*>(out_at(prm, q) + out_base)[i] = w;
    }
  }
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    if (atomicAdd(prm.counter, 1u) + 1u == gridDim.x) {
      *prm.counter = 0u;
      __threadfence_system();
      if (ok_s && !error_pending())
        for (int q = 0; q < prm.world; ++q) st_release_sys(prm.flag_b[q], prm.epoch);
    }
  }
}

__global__ void tp_wait_kernel(const PushParams prm) {
  if (threadIdx.x == 0)
    for (int q = 0; q < prm.world; ++q)
      if (!wait_flag(prm.local_b + q, prm.epoch, SITE_DONE)) break;
}

}  // namespace peer

GQA_ERROR_FLAG_ACCESSOR(error_flag_peer)

}  // namespace gqa

// ------------------------------------------------------------------ C ABI
extern "C" int gqa_peer_alloc(size_t bytes, void** dev_ptr, void* ipc_handle) {
  if (!dev_ptr || !ipc_handle || bytes == 0) return GQA_ERR_INVALID_ARGUMENT;
  *dev_ptr = nullptr;
  void* p = nullptr;
  if (cudaMalloc(&p, bytes) != cudaSuccess) return GQA_ERR_CUDA;
  if (cudaMemset(p, 0, bytes) != cudaSuccess || cudaDeviceSynchronize() != cudaSuccess) {
    cudaFree(p);
    return GQA_ERR_CUDA;
  }
  cudaIpcMemHandle_t h;
  if (cudaIpcGetMemHandle(&h, p) != cudaSuccess) {
    cudaFree(p);
    return GQA_ERR_CUDA;
  }
  memcpy(ipc_handle, &h, sizeof(h));
  *dev_ptr = p;
  return GQA_OK;
}

extern "C" size_t gqa_peer_handle_bytes(void) { return sizeof(cudaIpcMemHandle_t); }

extern "C" int gqa_peer_open(const void* ipc_handle, void** peer_ptr) {
  if (!ipc_handle || !peer_ptr) return GQA_ERR_INVALID_ARGUMENT;
  *peer_ptr = nullptr;
  cudaIpcMemHandle_t h;
  memcpy(&h, ipc_handle, sizeof(h));
  return cudaIpcOpenMemHandle(peer_ptr, h, cudaIpcMemLazyEnablePeerAccess) == cudaSuccess ? GQA_OK : GQA_ERR_CUDA;
}

extern "C" int gqa_peer_close(void* peer_ptr) {
  if (!peer_ptr) return GQA_ERR_INVALID_ARGUMENT;
  return cudaIpcCloseMemHandle(peer_ptr) == cudaSuccess ? GQA_OK : GQA_ERR_CUDA;
}

extern "C" int gqa_peer_free(void* dev_ptr) {
  if (!dev_ptr) return GQA_ERR_INVALID_ARGUMENT;
  return cudaFree(dev_ptr) == cudaSuccess ? GQA_OK : GQA_ERR_CUDA;
}

extern "C" int gqa_tp_reduce_gather_bf16(const void* const* bases, int world, int rank, int S, int N,
                                         unsigned int epoch, gqa_stream_t stream) {
  using namespace gqa;
  using namespace gqa::peer;
  if (!bases || world < 2 || world > kMaxRanks || rank < 0 || rank >= world) return GQA_ERR_INVALID_ARGUMENT;
  if (S <= 0 || N <= 0 || S % world || N % 8 || epoch == 0) return GQA_ERR_INVALID_ARGUMENT;
  Params prm{};
  const size_t part_bytes = static_cast<size_t>(S) * N * 4, out_bytes = static_cast<size_t>(S) * N * 2;
  for (int r = 0; r < world; ++r) {
    const uint8_t* b = static_cast<const uint8_t*>(bases[r]);
    if (!b || (reinterpret_cast<uintptr_t>(b) & 255u)) return GQA_ERR_MISALIGNED;
    prm.p.partial[r] = reinterpret_cast<const float*>(b);
    prm.p.out[r] = reinterpret_cast<const uint16_t*>(b + part_bytes);
    prm.p.ready[r] = reinterpret_cast<uint32_t*>(const_cast<uint8_t*>(b + part_bytes + out_bytes));
    prm.p.done[r] = prm.p.ready[r] + 1;
  }
  prm.out_local = const_cast<uint16_t*>(prm.p.out[rank]);
  prm.counter = prm.p.ready[rank] + 2;
  prm.world = world;
  prm.rank = rank;
  prm.S = S;
  prm.N = N;
  prm.epoch = epoch;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int* gemm_err = nullptr;
  const int rc = gemm_error_word(&gemm_err);
  if (rc != GQA_OK) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  signal_kernel<<<1, 1, 0, st>>>(prm.p.ready[rank], epoch, gemm_err);
  if (cudaGetLastError() != cudaSuccess) return GQA_ERR_CUDA;
  tp_reduce_kernel<<<2 * sms, kThreads, 0, st>>>(prm);
  if (cudaGetLastError() != cudaSuccess) return GQA_ERR_CUDA;
  tp_gather_kernel<<<2 * sms, kThreads, 0, st>>>(prm);
  return cudaGetLastError() == cudaSuccess ? GQA_OK : GQA_ERR_CUDA;
}

// [partial fp32 S x N][out bf16 S x N][flags 256 B]; flags: pull variant ready @0,
// done @4, counter @8; push variant flagA[8] @64, flagB[8] @96, reduce counter @128,
// GEMM counter @132.
extern "C" size_t gqa_tp_buffer_bytes(int S, int N) {
  if (S <= 0 || N <= 0) return 0;
  return static_cast<size_t>(S) * N * 6 + 256;
}

extern "C" int gqa_tp_o_proj_exchange_bf16(const void* attn, const void* wo, int ldw, const void* const* bases,
                                           int world, int rank, int S, int Hq, int head_dim, int N,
                                           unsigned int epoch, gqa_stream_t stream) {
  using namespace gqa;
  using namespace gqa::peer;
  if (!attn || !wo || !bases || world < 2 || world > kMaxRanks || rank < 0 || rank >= world)
    return GQA_ERR_INVALID_ARGUMENT;
  if (head_dim != 128) return GQA_ERR_UNSUPPORTED;
  if (S <= 0 || N <= 0 || Hq <= 0 || epoch == 0) return GQA_ERR_INVALID_ARGUMENT;
  if (S % world || (S / world) % 128 || N % 256) return GQA_ERR_UNSUPPORTED;
  const size_t slot_bytes = static_cast<size_t>(S / world) * N * 4;
  const size_t part_bytes = static_cast<size_t>(S) * N * 4, out_bytes = static_cast<size_t>(S) * N * 2;
  float* dst[kMaxRanks];
  uint32_t* flag_a[kMaxRanks];
  PushParams pp{};
  for (int q = 0; q < world; ++q) {
    uint8_t* b = static_cast<uint8_t*>(const_cast<void*>(bases[q]));
    if (!b || (reinterpret_cast<uintptr_t>(b) & 255u)) return GQA_ERR_MISALIGNED;
    uint8_t* flags = b + part_bytes + out_bytes;
    dst[q] = reinterpret_cast<float*>(b + static_cast<size_t>(rank) * slot_bytes);  // my slot at owner q
    flag_a[q] = reinterpret_cast<uint32_t*>(flags + 64) + rank;
    pp.out[q] = reinterpret_cast<uint16_t*>(b + part_bytes);
    pp.flag_b[q] = reinterpret_cast<uint32_t*>(flags + 96) + rank;
  }
  uint8_t* mine = static_cast<uint8_t*>(const_cast<void*>(bases[rank]));
  uint8_t* mflags = mine + part_bytes + out_bytes;
  pp.slots = reinterpret_cast<const float*>(mine);
  pp.local_a = reinterpret_cast<const uint32_t*>(mflags + 64);
  pp.local_b = reinterpret_cast<const uint32_t*>(mflags + 96);
  pp.counter = reinterpret_cast<uint32_t*>(mflags + 128);
  pp.world = world;
  pp.rank = rank;
  pp.S = S;
  pp.N = N;
  pp.epoch = epoch;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int rc = launch_o_proj_scatter(attn, wo, S, Hq, N, ldw, dst, flag_a, world, reinterpret_cast<uint32_t*>(mflags + 132),
                                 epoch, reinterpret_cast<float*>(mine), st);
  if (rc != GQA_OK) return rc;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  tp_reduce_push_kernel<<<2 * sms, kThreads, 0, st>>>(pp);
  if (cudaGetLastError() != cudaSuccess) return GQA_ERR_CUDA;
  tp_wait_kernel<<<1, 32, 0, st>>>(pp);
  return cudaGetLastError() == cudaSuccess ? GQA_OK : GQA_ERR_CUDA;
}
