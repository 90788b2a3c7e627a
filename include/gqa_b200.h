/*
 * gqa_b200.h -- C ABI of libgqa_b200.so, the sm_100a (B200) GQA attention core.
 *
 * The reference (xuanhaozhang883/Llama3-8B-Attention-Optimize) computes this path
 * in Python: the bf16-staged golden model llama3_attention_golden_model.py and the
 * fp32 NumPy CPU_Baseline.  Its only native interface is the HLS C++ mask kernel
 *   extern "C" void attention_mask(const score_t raw[], score_t masked[],
 *                                  int q_heads, int seq_len, bool causal,
 *                                  score_t mask_value)
 * (attention_mask_module/src/attention_mask.hpp:31-39).  Each entry point below
 * names the reference function it replaces.
 *
 * Conventions for every entry point:
 *  - All tensors are caller-owned DEVICE buffers of raw bf16 words (uint16),
 *    contiguous, 16-byte aligned.  The compute entry points allocate no device
 *    memory.  Two exceptions: gqa_peer_alloc (the one call that allocates: an
 *    exchange buffer for the tensor-parallel o_proj) and a fixed 16 MiB scratch
 *    array per GPU compiled into the library for gqa_decode_bf16_noalloc.
 *  - Layouts follow the golden model: per-head [head][token][dim]; a batch adds a
 *    leading axis: Q/O [B][Hq][S][d], K/V [B][Hkv][S][d].  GQA maps query head h to
 *    kv head h / (Hq/Hkv) by address (no KV duplication).
 *  - Calls are asynchronous on `stream` (a cudaStream_t; NULL = legacy default
 *    stream) and return a status: 0 = GQA_OK, negative = error (see gqa_strerror).
 *    Arguments are validated on the host before any launch; nothing aborts.
 *  - Kernels bound every internal wait; a wait that gives up records a sticky
 *    device error that gqa_device_check() reports (GQA_ERR_DEVICE_TIMEOUT).
 *  - Thread-safe.  Global state: per-device launch attributes and looked-up
 *    device addresses, one sticky error word per kernel file and GPU, and the
 *    no-alloc decode's scratch array (shared by every call on a GPU).
 */
#ifndef GQA_B200_H_
#define GQA_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* gqa_stream_t; /* == cudaStream_t */

#define GQA_OK 0
#define GQA_ERR_INVALID_ARGUMENT (-1) /* null pointer, bad size, bad flag */
#define GQA_ERR_UNSUPPORTED (-2)      /* shape outside what the kernels implement */
#define GQA_ERR_MISALIGNED (-3)       /* pointer not 16-byte aligned */
#define GQA_ERR_CUDA (-4)             /* CUDA runtime / driver error at launch */
#define GQA_ERR_DEVICE_TIMEOUT (-5)   /* a kernel's bounded wait expired */
#define GQA_ERR_WORKSPACE (-6)        /* workspace missing or too small */
#define GQA_ERR_NO_DEVICE (-7)        /* no usable sm_100 device */
#define GQA_ERR_DEVICE_INPUT (-8)     /* a kernel found invalid device-side input data */

#define GQA_FLAG_CAUSAL 1 /* mask keys j > i (golden :180-181) */
#define GQA_FLAG_ROPE_Q 2 /* rotate Q in the kernel (golden apply_rope :162-163) */
#define GQA_FLAG_ROPE_K 4 /* rotate K in the kernel (golden apply_rope :164) */

#define GQA_MASK_NEG_INF_BF16 0xFF80 /* attention_mask.hpp:16 */

/* Human-readable text for a status code. */
const char* gqa_strerror(int code);

/* Library ABI version (major*10000 + minor*100 + patch). */
int gqa_version(void);

/* Synchronize `stream`, then report (and clear) the sticky device error:
 * GQA_OK, GQA_ERR_DEVICE_TIMEOUT (a bounded wait gave up), GQA_ERR_DEVICE_INPUT (a
 * device-side check of input data failed: block-table entry or cache capacity), with
 * the site code in *site if non-NULL, or GQA_ERR_CUDA. */
int gqa_device_check(gqa_stream_t stream, int* site);

/* ---------------------------------------------------------------- RoPE
 * Replaces build_rope_cache (llama3_attention_golden_model.py:124-130):
 * cos/sin [seq_len][head_dim] bf16 for positions pos0..pos0+seq_len-1 with
 * emb = cat(freqs, freqs), freqs = fp32(pos * fp32(1/theta^(2i/d))).          */
int gqa_rope_cache_bf16(void* cos, void* sin, int seq_len, int head_dim, int pos0, double theta,
                        gqa_stream_t stream);

/* Replaces rotate_half/apply_rope (:133-139, used :162-164):
 * y = bf16(x*cos + rotate_half(x)*sin), x/y [num_heads][seq_len][head_dim]
 * (num_heads = B*H for batched buffers), table rows pos0..pos0+seq_len-1.
 * y may alias x.                                                               */
int gqa_rope_bf16(const void* x, void* y, const void* cos, const void* sin, int num_heads, int seq_len, int head_dim,
                  int pos0, gqa_stream_t stream);

/* ---------------------------------------------------------------- debug stages
 * Per-stage kernels of the golden model's dump mode (:157-190); each is
 * bit-exact with the golden's bf16 boundary rounding.                          */

/* scores_before_mask (:175-176): bf16(fp32(q.k) * scale), [B][Hq][S][S]. */
int gqa_scores_bf16(const void* q, const void* k, void* scores, int B, int Hq, int Hkv, int seq_len, int head_dim,
                    float scale, gqa_stream_t stream);

/* scores_after_mask (:180-181): bf16(score + (j > i ? -inf : +0)), [rows=B*Hq][S][S]. */
int gqa_mask_bf16(const void* scores, void* masked, int num_heads, int seq_len, int causal, gqa_stream_t stream);

/* Replaces the HLS kernel attention_mask (attention_mask.cpp:3-58): raw 16-bit
 * word pass-through, `mask_value` where causal && k_token > q_token.  Unlike the
 * HLS kernel (which returns silently), invalid sizes return an error.          */
int gqa_attention_mask_bf16(const void* raw_scores, void* masked_scores, int q_heads, int seq_len, int causal,
                            uint16_t mask_value, gqa_stream_t stream);

/* softmax_weights (:185): bf16(softmax(x)) over the last axis of [rows][cols]. */
int gqa_softmax_bf16(const void* scores, void* probs, long long rows, int cols, gqa_stream_t stream);

/* attn_out_per_head (:189): bf16(sum_j fp32 p*v), p [B][Hq][S][S], v [B][Hkv][S][d]. */
int gqa_pv_bf16(const void* probs, const void* v, void* out, int B, int Hq, int Hkv, int seq_len, int head_dim,
                gqa_stream_t stream);

/* ---------------------------------------------------------------- fused prefill
 * Replaces the core of run_full_attention (:162-190) and gqa_attention_cpu
 * (CPU_Baseline/cpu_baseline/attention.py:60-84) in one tcgen05 kernel:
 *   O = softmax(mask(rope(Q) rope(K)^T * scale)) V, bf16 out [B][Hq][S][d].
 * Processes kv heads [kv_head_begin, kv_head_begin+kv_head_count) of buffers
 * holding Hq / Hkv heads (the KV-head shard of one GPU).  Requires head_dim=128,
 * Hq = 4*Hkv.  cos/sin [>= S][128] (from gqa_rope_cache_bf16) are read when
 * GQA_FLAG_ROPE_Q / GQA_FLAG_ROPE_K are set; Q/K buffers are never modified.    */
int gqa_prefill_bf16(const void* q, const void* k, const void* v, void* o, const void* cos, const void* sin, int B,
                     int seq_len, int Hq, int Hkv, int head_dim, int kv_head_begin, int kv_head_count, float scale,
                     int flags, gqa_stream_t stream);

/* ---------------------------------------------------------------- split-KV decode
 * One query token per sequence against a KV cache (no reference function; the
 * single-row case of attention.py:60-84).  q/o [B][Hq][d]; kcache/vcache
 * [B][Hkv][max_len][d] (RoPE already applied); lens [B] int32 on the device:
 * sequence b attends keys [0, lens[b]) (lens clamped to [0, max_len]).  With
 * GQA_FLAG_ROPE_Q, q is rotated at position q_pos[b] (device int32 [B], clamped to
 * [0, max_len]) using cos/sin tables of at least max_len+1 rows.  Work is split along the
 * keys into chunks of `split_len` keys (multiple of 64, 0 = automatic); partial
 * results go to `workspace` (gqa_decode_workspace_size bytes) and a log-sum-exp
 * combine writes o.                                                            */
size_t gqa_decode_workspace_size(int B, int Hq, int max_len, int split_len);
int gqa_decode_bf16(const void* q, const void* kcache, const void* vcache, const int32_t* lens, const int32_t* q_pos,
                    const void* cos, const void* sin, void* o, void* workspace, size_t workspace_bytes, int B,
                    int max_len, int Hq, int Hkv, int head_dim, int kv_head_begin, int kv_head_count, int split_len,
                    float scale, int flags, gqa_stream_t stream);

/* ---------------------------------------------------------------- allocation-free decode
 * No counterpart in the reference: an addition for callers that cannot allocate
 * device memory -- a plugin host that passes the library only its input and
 * output buffers and owns all other device memory, a serving loop that must not
 * call cudaMalloc/cudaFree (they synchronise the device), or a process whose
 * memory pool is reserved in full up front.
 * Same arguments and result as gqa_decode_bf16 minus the workspace: the split-KV
 * partials go to a 16 MiB scratch array built into the library (one per GPU,
 * held until the process exits; gqa_decode_noalloc_scratch_bytes() returns the
 * size).  A request needing more than that (gqa_decode_workspace_size) returns
 * GQA_ERR_WORKSPACE without launching.  Calls share the array: calls whose
 * kernels overlap on the GPU race and give wrong results, so order them on one
 * stream.  The first call on each device resolves the array's address; make it
 * before any stream capture starts.                                            */
size_t gqa_decode_noalloc_scratch_bytes(void);
int gqa_decode_bf16_noalloc(const void* q, const void* kcache, const void* vcache, const int32_t* lens,
                            const int32_t* q_pos, const void* cos, const void* sin, void* o, int B, int max_len,
                            int Hq, int Hkv, int head_dim, int kv_head_begin, int kv_head_count, int split_len,
                            float scale, int flags, gqa_stream_t stream);

/* ---------------------------------------------------------------- tensor-parallel o_proj over NVLink
 * The row-parallel o_proj leaves each rank an fp32 partial of the same [S][N] output; the
 * layer output is bf16(sum over ranks), the reference's single rounding (:193-194).
 * Instead of an NCCL all-reduce, ranks exchange through CUDA IPC peer memory:
 *  - gqa_tp_buffer_bytes(S, N) bytes per rank, allocated with gqa_peer_alloc (the one
 *    device allocation this library makes: IPC needs a cudaMalloc base) and laid out as
 *    [partial fp32 S x N][out bf16 S x N][flags]; its handle (gqa_peer_handle_bytes()
 *    bytes) goes to every other rank, which maps it with gqa_peer_open;
 *  - each step the caller writes its partial (e.g. gqa_o_proj_bf16 with
 *    GQA_GEMM_OUT_F32 into the buffer's start), then calls gqa_tp_reduce_gather_bf16
 *    with bases[r] = rank r's buffer as mapped in this process (its own for r = rank)
 *    and an epoch that increases by one per step (starting at 1, the same on every
 *    rank).  It sums its S/world-row block over all ranks by P2P loads in rank order,
 *    rounds once, and gathers the other blocks: the buffer's out holds the full bf16
 *    result when the stream reaches that point.  S % world == 0, N % 8 == 0, world <= 8.
 * Waits on peers are bounded; a missing peer is reported by gqa_device_check.         */
size_t gqa_tp_buffer_bytes(int S, int N);
size_t gqa_peer_handle_bytes(void);
int gqa_peer_alloc(size_t bytes, void** dev_ptr, void* ipc_handle);
int gqa_peer_open(const void* ipc_handle, void** peer_ptr);
int gqa_peer_close(void* peer_ptr);
int gqa_peer_free(void* dev_ptr);
int gqa_tp_reduce_gather_bf16(const void* const* bases, int world, int rank, int S, int N, unsigned int epoch,
                              gqa_stream_t stream);
/* The same exchange fused into the o_proj (one sequence): the GEMM of attn [Hq][S][128]
 * against wo (ldw, the shard's columns) stores each fp32 row straight into the owning
 * rank's buffer (NVLink peer stores while other tiles still compute) and signals the
 * owners when its grid is done; each owner sums its block, rounds once and stores the
 * bf16 block into every rank's out.  The buffer's out holds the full result when the
 * stream reaches that point.  (S / world) % 128 == 0, N % 256 == 0.                   */
int gqa_tp_o_proj_exchange_bf16(const void* attn, const void* wo, int ldw, const void* const* bases, int world,
                                int rank, int S, int Hq, int head_dim, int N, unsigned int epoch,
                                gqa_stream_t stream);

/* ---------------------------------------------------------------- paged K/V cache
 * The step after decode (the reference has no serving cache): append each step's new
 * K/V rows to the cache, rotating K at its position, and decode over a paged cache.
 *
 * Paged layout: K and V page pools [num_pages][Hkv][page_size][head_dim] bf16; token j
 * of sequence b is row j % page_size of page block_table[b * max_pages_per_seq +
 * j / page_size] (int32, device).  page_size must be a multiple of 128 for decode.
 *
 * gqa_kv_append_bf16: k_new/v_new [B][Hkv][n_new][128]; token i of sequence b goes to
 * position lens[b] + i.  block_table == NULL selects the contiguous cache
 * [B][Hkv][max_len][128] (max_len used only then).  GQA_FLAG_ROPE_K rotates K with
 * cos/sin rows [pos] (tables of >= capacity rows, as gqa_rope_cache_bf16 builds them),
 * bit-identical to gqa_rope_bf16 / the golden apply_rope.  If lens_out is non-NULL a
 * second launch writes lens_out[b] = lens[b] + n_new (lens_out may equal lens).
 * Positions past the cache or block-table entries outside [0, num_pages) skip their
 * row and set GQA_ERR_DEVICE_INPUT for gqa_device_check.
 *
 * gqa_decode_paged_bf16: gqa_decode_bf16 over the paged cache (capacity
 * max_pages_per_seq * page_size keys per sequence, lens[b] <= capacity); split_len a
 * multiple of 128 (0 = default); workspace = gqa_decode_workspace_size(B, Hq,
 * capacity, split_len).  Results are bit-identical to gqa_decode_bf16 on a contiguous
 * cache holding the same rows.                                                    */
int gqa_kv_append_bf16(const void* k_new, const void* v_new, void* kcache, void* vcache, const int32_t* block_table,
                       int max_pages_per_seq, int page_size, int num_pages, const int32_t* lens, int32_t* lens_out,
                       const void* cos, const void* sin, int B, int Hkv, int n_new, int head_dim, int max_len,
                       int flags, gqa_stream_t stream);
int gqa_decode_paged_bf16(const void* q, const void* kpages, const void* vpages, const int32_t* block_table,
                          int max_pages_per_seq, int page_size, int num_pages, const int32_t* lens,
                          const int32_t* q_pos, const void* cos, const void* sin, void* o, void* workspace,
                          size_t workspace_bytes, int B, int Hq, int Hkv, int head_dim, int kv_head_begin,
                          int kv_head_count, int split_len, float scale, int flags, gqa_stream_t stream);

/* ---------------------------------------------------------------- projections
 * The full layer's linear maps (golden run_full_attention,
 * llama3_attention_golden_model.py:149-151 and :193-194): y = x W^T with W in the
 * HF [out][in] layout, bf16 operands, fp32 accumulation, one round-to-nearest-even
 * to bf16 -- or, with GQA_GEMM_OUT_F32, the fp32 sums (row-parallel partials that
 * are all-reduced before the rounding).  Row strides (elements) must keep rows
 * 16-byte aligned.                                                              */
#define GQA_GEMM_OUT_F32 1

/* c[M][ldc] = a[M][lda] . w[N][ldw]^T over the first K columns.
 * Replaces `hidden_states @ q_proj.T` etc. (:149-151, :194).                   */
int gqa_gemm_bf16(const void* a, const void* w, void* c, int M, int N, int K, int lda, int ldw, int ldc, int flags,
                  gqa_stream_t stream);

/* Fused q/k/v projection, one launch: h [B][S][hidden]; wq [Hq*128][hidden],
 * wk / wv [Hkv*128][hidden]; outputs head-major q [B][Hq][S][128], k / v
 * [B][Hkv][S][128] (the .view().transpose(0,1) of :153-155).  GQA_FLAG_ROPE_Q /
 * GQA_FLAG_ROPE_K rotate q / k at positions pos0 + s after the bf16 rounding, as
 * to_bf16(apply_rope(to_bf16(h @ W^T))) (:149-164); cos/sin hold >= pos0 + S rows.
 * B > 1 needs S % 128 == 0.  For a kv-head shard pass the weight rows of the
 * shard's heads (wq + 512*g0*hidden, wk/wv + 128*g0*hidden).                    */
int gqa_qkv_proj_bf16(const void* h, const void* wq, const void* wk, const void* wv, void* q, void* k, void* v,
                      const void* cos, const void* sin, int B, int S, int hidden, int Hq, int Hkv, int head_dim,
                      int pos0, int flags, gqa_stream_t stream);

/* o_proj from the head-major attention output attn [B][Hq][S][128]:
 * out[B*S][N] = concat_h(attn[:, h]) . wo[N][ldw]^T over columns [0, Hq*128) of
 * wo (the transpose(0,1).view(S,-1) of :193 is folded into the loads).  A shard
 * owning q heads [h0, h0+Hq) passes wo + h0*128 with ldw = the full width and
 * GQA_GEMM_OUT_F32; the partials are summed across shards (all-reduce) and
 * rounded with gqa_cast_f32_bf16.  B > 1 needs S % 128 == 0.                   */
int gqa_o_proj_bf16(const void* attn, const void* wo, void* out, int B, int S, int Hq, int head_dim, int N, int ldw,
                    int flags, gqa_stream_t stream);

/* Rows [s0, s0 + s_count) of gqa_o_proj_bf16's result for one sequence (B = 1):
 * attn [Hq][S][128], out [S][N] of which only the chunk's rows are written.  For
 * overlapping the reduction of finished rows with the next chunk's GEMM (tensor-parallel
 * o_proj); max_ctas > 0 caps the persistent grid (leaving SMs free for a collective).
 * Every row is bit-identical to the full call's.                                     */
int gqa_o_proj_rows_bf16(const void* attn, const void* wo, void* out, int S, int s0, int s_count, int Hq,
                         int head_dim, int N, int ldw, int max_ctas, int flags, gqa_stream_t stream);

/* dst[i] = bf16_rne(src[i]) for n fp32 values (src 16-byte aligned, dst 8-byte). */
int gqa_cast_f32_bf16(const void* src, void* dst, long long n, gqa_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* GQA_B200_H_ */
