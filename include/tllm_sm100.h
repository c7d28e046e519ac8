/*
 * tllm_sm100.h -- C ABI of libtllm_sm100a.so, the B200 (sm_100a) implementation of the
 * four operators exported by triton_llm.ops (xdlhzdh/TritonLLMCompiler).
 *
 * Conventions (modelled on mlir/runtime/cutlass_c_api.h:4-25 of the reference: extern "C",
 * int status with 0 = success, int64_t sizes), extended for a device-pointer hot path:
 *   - every tensor pointer is a DEVICE pointer to fp16 or bf16 data (dtype: 0 = fp16,
 *     1 = bf16); indices (block tables, context lengths) are int32 device pointers;
 *   - strides are in ELEMENTS, innermost dimension last, exactly as torch reports them;
 *   - work is enqueued on `stream` (a cudaStream_t); no entry point allocates, frees or
 *     synchronises the device;
 *   - a non-zero return means nothing was launched; tllm_last_error() then describes why
 *     (thread-local string, valid until the next call on the same thread).
 * The Python package (tritonllmcompiler_b200.ops) is the only caller in this repository;
 * it maps a non-zero status to RuntimeError(tllm_last_error()).
 */
#ifndef TLLM_SM100_H_
#define TLLM_SM100_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define TLLM_API __attribute__((visibility("default")))
#else
#define TLLM_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define TLLM_OK 0
#define TLLM_ERR_INVALID 1   /* bad shape, stride, dtype or alignment */
#define TLLM_ERR_CUDA 2      /* a CUDA runtime / driver call failed */
#define TLLM_ERR_WORKSPACE 3 /* workspace pointer null or too small */

#define TLLM_DTYPE_F16 0
#define TLLM_DTYPE_BF16 1

/* Library version string ("0.2.0", the reference package's __version__). */
TLLM_API const char *tllm_version(void);

/* Human-readable description of the last failure on the calling thread ("" if none). */
TLLM_API const char *tllm_last_error(void);

/* Reads and clears the device-side error word of the current device: 0 = no kernel has
 * reported a problem; otherwise a TLLM_DEV_* code from a bounded wait that gave up.
 * Synchronises the current device (a debugging aid, not part of the hot path). */
TLLM_API int tllm_debug_status(int *out);

/* Failure-detection self-test: enqueues a one-warp kernel that waits on an mbarrier nothing
 * arrives on. The bounded wait gives up after about 10 ms and records 0x17F
 * (TLLM_DEV_WAIT_TIMEOUT + 0x7F), which tllm_debug_status then returns; the context stays
 * usable. No counterpart in the reference (its CUDA helper exits the process on errors,
 * common/cuda_utils.cuh:10-18). */
TLLM_API int tllm_selftest_bounded_wait(void *stream);

/*
 * FlashAttention forward: o = softmax(q k^T * sm_scale [+ causal mask]) v per (b, h).
 * Replaces flash_attention() in python/triton_llm/ops/flash_attention.py:107-133 and its
 * Triton kernel _flash_attn_fwd (:17-104). The causal mask is top-left aligned: query row i
 * sees key columns j <= i (:74-79). q is [B,H,Sq,D], k/v are [B,H,Sk,D] with strides
 * sq/sk/sv (4 entries each, elements), o is [B,H,Sq,D] with strides so. D in {16,32,64,128}.
 * The innermost stride must be 1 and the other strides multiples of 8 elements (16 bytes).
 */
TLLM_API int tllm_flash_attn_fwd(const void *q, const void *k, const void *v, void *o,
                        int64_t B, int64_t H, int64_t Sq, int64_t Sk, int64_t D,
                        const int64_t *sq, const int64_t *sk, const int64_t *sv,
                        const int64_t *so, float sm_scale, int causal, int dtype,
                        void *stream);

/* Same as tllm_flash_attn_fwd with an explicit kernel choice, for cross-checking the
 * implementations against each other: variant 0 = two 128-row query tiles per CTA with
 * ping-pong softmax warpgroups and work stealing (the default), 1 = one query tile per CTA,
 * 2 = variant 0 with one work item per CTA, 3 = variant 0 with P passed to P V through shared
 * memory instead of tensor memory (K and V tiles in one ring). */
TLLM_API int tllm_flash_attn_fwd_variant(const void *q, const void *k, const void *v, void *o,
                                int64_t B, int64_t H, int64_t Sq, int64_t Sk, int64_t D,
                                const int64_t *sq, const int64_t *sk, const int64_t *sv,
                                const int64_t *so, float sm_scale, int causal, int dtype,
                                int variant, void *stream);

/*
 * Bytes of device workspace tllm_paged_attn_decode needs for this problem (the split-KV
 * partial results). Replaces nothing in the reference (its kernel runs one CTA per (b, h)
 * and needs none); the Python wrapper allocates this from the torch caching allocator.
 */
TLLM_API size_t tllm_paged_attn_workspace_size(int64_t B, int64_t H, int64_t D,
                                      int64_t block_size, int64_t max_blocks);

/*
 * Paged-KV decode attention: for each (b, h), attention of the single query q[b,h,0,:]
 * over tokens 0..context_lens[b]-1, token t living at
 * k_cache[block_tables[b, t / block_size], t % block_size, h, :] (same for v_cache).
 * Replaces paged_attention() in python/triton_llm/ops/paged_attention.py:92-128 and its
 * kernel _paged_attn_kernel (:11-89). Like that kernel, at most max_blocks table entries of
 * a row are read (tokens past max_blocks * block_size are ignored) and a context length of
 * 0 yields NaN. Unlike it, no host synchronisation happens (the reference reads
 * context_lens.max() on the host, :113).
 *   q [B,H,1,D] strides sq (4), caches [num_blocks, block_size, H, D] strides skc/svc (4),
 *   block_tables [B, max_blocks] strides sbt (2), context_lens [B] contiguous,
 *   o [B,H,1,D] strides so (4). D in {16,32,64,128}; block_size in {16,32,64}.
 * workspace must hold tllm_paged_attn_workspace_size(...) bytes, 256-byte aligned.
 */
TLLM_API int tllm_paged_attn_decode(const void *q, const void *k_cache, const void *v_cache,
                           const int32_t *block_tables, const int32_t *context_lens,
                           void *o, void *workspace, size_t workspace_bytes,
                           int64_t B, int64_t H, int64_t D, int64_t block_size,
                           int64_t max_blocks, int64_t num_blocks,
                           const int64_t *sq, const int64_t *skc, const int64_t *svc,
                           const int64_t *sbt, const int64_t *so, float sm_scale,
                           int dtype, void *stream);

/* Size of the fixed device array tllm_paged_attn_decode_noalloc keeps its split-KV
 * partials in (32 MiB per GPU that loads the library). */
#define TLLM_PAGED_NOALLOC_SCRATCH_BYTES (32u << 20)

/*
 * Same operation as tllm_paged_attn_decode, for callers that cannot allocate device memory
 * (engines that reserve all device memory at start-up and forbid later cudaMalloc, or
 * foreign-language hosts without a device allocator). It has no counterpart in the
 * reference. It allocates nothing: the split-KV partials go to a fixed array inside the
 * library of TLLM_PAGED_NOALLOC_SCRATCH_BYTES bytes; a problem whose partials need more
 * (tllm_paged_attn_workspace_size above that limit) is rejected with TLLM_ERR_WORKSPACE and
 * nothing is launched. The caller still provides every input and the output.
 *   - Each call looks up the array's device address with the caller's device current
 *     (cudaGetSymbolAddress, so the address stays right after a cudaDeviceReset); the first
 *     call on a device also loads the library's device code there, so make that first call
 *     before any stream capture.
 *   - Dimensions are checked (TLLM_ERR_INVALID) before the scratch size is planned.
 *   - All calls share the one array and it keeps the last call's contents. Calls whose
 *     kernels can overlap on the GPU (different streams, no ordering between them) race on
 *     it and may return wrong results; order such calls on one stream or with events.
 */
TLLM_API int tllm_paged_attn_decode_noalloc(const void *q, const void *k_cache,
                                   const void *v_cache, const int32_t *block_tables,
                                   const int32_t *context_lens, void *o, int64_t B,
                                   int64_t H, int64_t D, int64_t block_size,
                                   int64_t max_blocks, int64_t num_blocks,
                                   const int64_t *sq, const int64_t *skc,
                                   const int64_t *svc, const int64_t *sbt,
                                   const int64_t *so, float sm_scale, int dtype,
                                   void *stream);

/*
 * Fused RMSNorm + rotate-half RoPE:
 *   r = rsqrt(mean(x^2) + eps); y = round_to_dtype(x * r * w);
 *   out[:D/2] = y1*cos[:D/2] - y2*sin[:D/2]; out[D/2:] = y2*cos[D/2:] + y1*sin[D/2:]
 * with cos/sin indexed by the sequence position s. Replaces rmsnorm_rope() in
 * python/triton_llm/ops/rmsnorm_rope.py:51-75 (kernel :9-48). The intermediate rounding of
 * y to the I/O dtype follows the reference's oracle (python/triton_llm/reference/
 * norm_rope.py:12-15). x/out [B,S,H,D] strides sx/so (4), w [D] stride sw, cos/sin [S,D]
 * strides scos/ssin (2). D in {16,32,64,128}.
 */
TLLM_API int tllm_rmsnorm_rope(const void *x, const void *w, const void *cos, const void *sin,
                      void *out, int64_t B, int64_t S, int64_t H, int64_t D,
                      const int64_t *sx, int64_t sw, const int64_t *scos,
                      const int64_t *ssin, const int64_t *so, float eps, int dtype,
                      void *stream);

/*
 * SwiGLU dual GEMM: out = silu(x @ w1) * (x @ w3), fp32 accumulation, one store in the
 * I/O dtype. Replaces swiglu() in python/triton_llm/ops/swiglu.py:54-76 (kernel :11-51)
 * and the fp32 C-ABI cutlass_gemm_swiglu / cutlass_gemm_swiglu_sm90 of
 * mlir/runtime/cutlass_c_api.h:10-18. x [M,K] row stride lda, w1/w3 [K,N] row strides
 * ldb1/ldb3, out [M,N] row stride ldo (all elements; inner strides are 1).
 * Performance limit: the tensor-core kernels need K, N, lda, ldb1 and ldb3 multiples of 8
 * and x, w1, w3 16-byte aligned (what a TMA descriptor can describe); other shapes run on a
 * CUDA-core kernel with the same results at roughly 1/50 of the speed.
 */
TLLM_API int tllm_swiglu(const void *x, const void *w1, const void *w3, void *out, int64_t M,
                int64_t N, int64_t K, int64_t lda, int64_t ldb1, int64_t ldb3,
                int64_t ldo, int dtype, void *stream);

/*
 * Column-sharded SwiGLU for one node (no counterpart in the reference, which is single-GPU):
 * computes silu(x @ w1) * (x @ w3) for this rank's column slices w1/w3 [K, N] (N = this
 * rank's share of the columns) and writes the [M, N] result at column offset col_off of
 * EVERY buffer in dsts[0..ndst) (row stride ldo): this rank's [M, N_total] output and the
 * peers' outputs mapped into this process (tllm_ipc_open). The GEMM epilogue stores straight
 * over NVLink, so the all-gather costs no separate pass. The caller orders the call after
 * every peer has finished reading its previous output and before any rank reads the new one
 * (for example a small NCCL all-reduce before and after). ndst <= 8; K, N, the leading
 * dimensions and col_off multiples of 8.
 */
TLLM_API int tllm_swiglu_colshard(const void *x, const void *w1, const void *w3,
                                  void *const *dsts, int ndst, int64_t col_off, int64_t M,
                                  int64_t N, int64_t K, int64_t lda, int64_t ldb1, int64_t ldb3,
                                  int64_t ldo, int dtype, void *stream);

/* Flag words per rank of tllm_swiglu_colshard_peers (uint32, zero before the first call). */
#define TLLM_SWIGLU_PEER_FLAG_WORDS 16

/*
 * Column-sharded SwiGLU whose output all-gather and its synchronisation both live in the
 * kernel (no counterpart in the reference, which is single-GPU). Rank `rank` of `ndst`
 * (one process per GPU of one node) computes silu(x @ w1) * (x @ w3) for its column slices
 * w1/w3 [K, N] and stores the [M, N] result at column offset rank * N of every rank's
 * [M, ndst * N] output dsts[0..ndst) (row stride ldo; the peers' buffers mapped into this
 * process with tllm_ipc_open) over NVLink, tile by tile as the GEMM finishes them.
 *   flags[d]: rank d's TLLM_SWIGLU_PEER_FLAG_WORDS words (mapped likewise), zeroed before
 *     the first call; done: one uint32 of this rank's device memory, zeroed likewise; epoch:
 *     1 on the first call with these buffers, +1 on every later one, the same on every rank.
 *   At its start a launch tells every peer it has begun (its stream's earlier work, reads of
 *   the previous output included, is complete); a CTA stores into a peer only once that
 *   peer has begun; the launch ends only after every peer has reported its stores into this
 *   rank complete. No host-side barrier is needed between calls, and a call's output is
 *   complete when the launch ends on this rank's stream. Every rank must make every call.
 *   Waits are bounded (about 2 s); a peer that never starts or finishes is reported through
 *   tllm_debug_status (TLLM_DEV_WAIT_TIMEOUT + 5 or + 6) instead of hanging.
 *   variant: 0 automatic (the CTA-pair kernel with tensor stores from M >= 256 when N % 128
 *   == 0 and ldo, N and the buffers allow 16-byte-aligned slices), 1 the one-CTA kernel,
 *   2 the CTA-pair kernel, 3 the CTA-pair kernel storing each row as one 256-byte span (3-D
 *   boxes); all give the same result. ndst <= 8; K, N and the leading dimensions multiples
 *   of 8.
 */
TLLM_API int tllm_swiglu_colshard_peers(const void *x, const void *w1, const void *w3,
                                        void *const *dsts, uint32_t *const *flags, int ndst,
                                        int rank, uint32_t *done, uint32_t epoch, int64_t M,
                                        int64_t N, int64_t K, int64_t lda, int64_t ldb1,
                                        int64_t ldb3, int64_t ldo, int dtype, int variant,
                                        void *stream);

/*
 * tllm_swiglu_colshard_peers with the output written through an NVLink multicast address
 * (no counterpart in the reference, which is single-GPU): mc is the multicast address of the
 * outputs dsts[0..ndst), i.e. the same byte offsets of every rank's buffer bound to one
 * multicast object (for example torch symmetric memory's multicast_ptr). The CTA-pair kernel
 * (M >= 256, N % 128 == 0) then stores each output block once and the NVSwitch writes it into
 * every rank's buffer, so a rank's NVLink egress is its own [M, N] slice instead of ndst - 1
 * copies of it; other shapes run the one-CTA kernel, which stores into each of dsts as
 * tllm_swiglu_colshard_peers does. flags, done, epoch and the handshake as there; the kernel
 * choice is automatic. mc 16-byte aligned.
 */
TLLM_API int tllm_swiglu_colshard_multicast(const void *x, const void *w1, const void *w3,
                                            void *const *dsts, void *mc,
                                            uint32_t *const *flags, int ndst, int rank,
                                            uint32_t *done, uint32_t epoch, int64_t M, int64_t N,
                                            int64_t K, int64_t lda, int64_t ldb1, int64_t ldb3,
                                            int64_t ldo, int dtype, void *stream);

/* CUDA IPC set-up helpers for tllm_swiglu_colshard's peer buffers: a 64-byte handle and
 * byte offset for a device pointer, opening a peer's handle in this process, and closing it.
 * Not on the hot path. */
TLLM_API int tllm_ipc_get_handle(const void *ptr, void *handle_out, uint64_t *offset_out);
TLLM_API int tllm_ipc_open(const void *handle, uint64_t offset, void **ptr_out, void **base_out);
TLLM_API int tllm_ipc_close(void *base);

/* Asynchronous 2-D copy (height rows of width bytes, row pitches in bytes) between any two of
 * host (pinned) and device memory on `stream`: one DMA request for a column block of a
 * row-major matrix. Used by the host-memory pipelines of the Python package
 * (ops/host_pipeline.py), which overlap the transfer of one block with the kernel on the
 * previous one; no counterpart in the reference. */
TLLM_API int tllm_copy2d_async(void *dst, size_t dpitch, const void *src, size_t spitch,
                               size_t width, size_t height, void *stream);

/*
 * Operators either side of decode (no counterpart in the reference, which only decodes from a
 * paged cache: python/triton_llm/ops/paged_attention.py:92-128). They use its cache layout:
 * token t of sequence b at cache[block_tables[b, t / block_size], t % block_size, h, :]
 * (python/triton_llm/reference/paged_attention.py:29-37).
 *
 * tllm_paged_kv_append writes k_new/v_new [B, T, H, D] (strides skn/svn) into the caches
 * [num_blocks, block_size, H, D] (strides skc/svc): token t of sequence b goes to position
 * start_pos[b] + t, for t < n_new[b] (every t < T when n_new is NULL). block_tables is
 * [B, max_blocks] int32 (strides sbt), start_pos and n_new are [B] int32, all on the device.
 * A position past the block table or a table entry outside [0, num_blocks) is skipped and
 * reported through tllm_debug_status (TLLM_DEV_BAD_INDEX). Inner strides must be 1, other
 * strides multiples of 8 elements, pointers 16-byte aligned.
 */
TLLM_API int tllm_paged_kv_append(const void *k_new, const void *v_new, void *k_cache,
                                  void *v_cache, const int32_t *block_tables,
                                  const int32_t *start_pos, const int32_t *n_new, int64_t B,
                                  int64_t T, int64_t H, int64_t D, int64_t block_size,
                                  int64_t max_blocks, int64_t num_blocks, const int64_t *skn,
                                  const int64_t *svn, const int64_t *skc, const int64_t *svc,
                                  const int64_t *sbt, int dtype, void *stream);

/*
 * tllm_paged_kv_append with K passed through the fused RMSNorm + RoPE of tllm_rmsnorm_rope
 * first (weight [D]; cos/sin [rope_rows, D] with row strides scos/ssin). The RoPE row of
 * token t of sequence b is its absolute position start_pos[b] + t; a position at or past
 * rope_rows is skipped and reported like a bad block index. The cache receives exactly
 * what tllm_rmsnorm_rope returns for that row.
 */
TLLM_API int tllm_paged_kv_append_rope(const void *k_new, const void *v_new, const void *weight,
                                       const void *cos, const void *sin, int64_t rope_rows,
                                       int64_t scos, int64_t ssin, void *k_cache,
                                       void *v_cache, const int32_t *block_tables,
                                       const int32_t *start_pos, const int32_t *n_new,
                                       int64_t B, int64_t T, int64_t H, int64_t D,
                                       int64_t block_size, int64_t max_blocks,
                                       int64_t num_blocks, const int64_t *skn,
                                       const int64_t *svn, const int64_t *skc,
                                       const int64_t *svc, const int64_t *sbt, float eps,
                                       int dtype, void *stream);

/*
 * Attention of Sq >= 1 new query tokens per sequence over the paged cache, with grouped query
 * heads: q [B, Hq, Sq, D] (strides sq), caches [num_blocks, block_size, Hkv, D] with
 * Hq % Hkv == 0 (query head h reads KV head h / (Hq / Hkv)), output o [B, Hq, Sq, D]
 * (strides so). context_lens[b] counts the new tokens (they are already in the cache); query
 * token s sits at position context_lens[b] - Sq + s and, when causal != 0, sees the keys at
 * positions <= its own (all context_lens[b] keys otherwise). A query that sees no key gives
 * NaN. With Sq = 1 and Hq = Hkv this is tllm_paged_attn_decode; otherwise, with at most 16
 * query rows per KV head ((Hq / Hkv) * Sq <= 16) and D in {64, 128}, a grouped-query split
 * kernel reads each K/V row once for those rows (the workspace size entry accounts for it);
 * larger calls run the tensor-core prefill kernel. Requirements as for
 * tllm_paged_attn_decode (block_size in {16,32,64}, D in {16,32,64,128}, unit inner strides,
 * 16-byte alignment); the workspace (256-byte aligned) holds split-KV partials when a launch
 * splits the keys (tllm_paged_prefill_workspace_size, 0 when it does not).
 */
TLLM_API size_t tllm_paged_prefill_workspace_size(int64_t B, int64_t Hq, int64_t Hkv, int64_t Sq,
                                                  int64_t D, int64_t block_size,
                                                  int64_t max_blocks);
TLLM_API int tllm_paged_prefill(const void *q, const void *k_cache, const void *v_cache,
                                const int32_t *block_tables, const int32_t *context_lens,
                                void *o, void *workspace, size_t workspace_bytes, int64_t B,
                                int64_t Hq, int64_t Hkv, int64_t Sq, int64_t D,
                                int64_t block_size, int64_t max_blocks, int64_t num_blocks,
                                const int64_t *sq, const int64_t *skc, const int64_t *svc,
                                const int64_t *sbt, const int64_t *so, float sm_scale,
                                int causal, int dtype, void *stream);

/*
 * Variable-length (packed) flash attention forward. No counterpart in the reference, whose
 * flash_attention (python/triton_llm/ops/flash_attention.py:107-133) takes padded
 * [B, H, S, D] tensors: here q/o are [total_q, H, D] and k/v [total_k, Hkv, D] with strides
 * {row, head, 1} (sq/sk/sv/so hold 3 entries), H % Hkv == 0, and sequence b is rows
 * [cu_seqlens_q[b], cu_seqlens_q[b+1]) of q/o and [cu_seqlens_k[b], cu_seqlens_k[b+1]) of
 * k/v (int32 arrays of B + 1 entries on the device). Every sequence is computed as
 * tllm_flash_attn_fwd would compute it alone (top-left causal mask), query head h reading
 * key/value head h / (H / Hkv). max_seqlen_q/k must bound every sequence's lengths.
 */
TLLM_API int tllm_flash_attn_varlen_fwd(const void *q, const void *k, const void *v, void *o,
                                        const int *cu_seqlens_q, const int *cu_seqlens_k,
                                        int64_t B, int64_t H, int64_t Hkv, int64_t total_q,
                                        int64_t total_k, int64_t max_seqlen_q,
                                        int64_t max_seqlen_k, int64_t D, const int64_t *sq,
                                        const int64_t *sk, const int64_t *sv, const int64_t *so,
                                        float sm_scale, int causal, int dtype, void *stream);

/*
 * FlashAttention backward. No counterpart in the reference, which has the forward only
 * (python/triton_llm/ops/flash_attention.py:1-7); the function differentiated is its
 * flash_attention (top-left causal mask). tllm_flash_attn_fwd_lse is tllm_flash_attn_fwd
 * that also writes lse [B, H, Sq] (fp32, contiguous): log2 of each row's softmax normaliser
 * in units of s * sm_scale * log2(e). tllm_flash_attn_bwd takes q, k, v, the forward's output
 * o and lse, and dout (all [B, H, S, D] with the layout rules of tllm_flash_attn_fwd, D 64 or
 * 128) and writes dq, dk, dv ([B, H, S, D], any strides). The workspace (16-byte aligned,
 * tllm_flash_attn_bwd_workspace_size bytes) holds the fp32 dq accumulator and the per-row
 * rowsum(dout * o); the call clears what it uses.
 */
TLLM_API int tllm_flash_attn_fwd_lse(const void *q, const void *k, const void *v, void *o,
                                     float *lse, int64_t B, int64_t H, int64_t Sq, int64_t Sk,
                                     int64_t D, const int64_t *sq, const int64_t *sk,
                                     const int64_t *sv, const int64_t *so, float sm_scale,
                                     int causal, int dtype, void *stream);
TLLM_API size_t tllm_flash_attn_bwd_workspace_size(int64_t B, int64_t H, int64_t Sq, int64_t D);
TLLM_API int tllm_flash_attn_bwd(const void *q, const void *k, const void *v, const void *o,
                                 const void *dout, const float *lse, void *dq, void *dk, void *dv,
                                 void *workspace, size_t workspace_bytes, int64_t B, int64_t H,
                                 int64_t Sq, int64_t Sk, int64_t D, const int64_t *sq,
                                 const int64_t *sk, const int64_t *sv, const int64_t *so,
                                 const int64_t *sdo, const int64_t *sdq, const int64_t *sdk,
                                 const int64_t *sdv, float sm_scale, int causal, int dtype,
                                 void *stream);

/* Same as tllm_swiglu with an explicit kernel choice, for cross-checking: 0 = automatic (the
 * CTA-pair kernel when M >= 256 and N % 128 == 0), 1 = one CTA per 128 x 128 output tile,
 * 2 = the CTA-pair kernel (two CTAs on two SMs share 256 x 128 output tiles through
 * tcgen05.mma.cta_group::2; N % 128 == 0). M, N, K > 0. */
TLLM_API int tllm_swiglu_variant(const void *x, const void *w1, const void *w3, void *out,
                                 int64_t M, int64_t N, int64_t K, int64_t lda, int64_t ldb1,
                                 int64_t ldb3, int64_t ldo, int dtype, int variant, void *stream);

/*
 * FP8 SwiGLU: out = silu(scale_x*scale_w1 * x@w1) * (scale_x*scale_w3 * x@w3) with e4m3 inputs
 * and per-tensor scales, fp32 accumulation, fp16/bf16 output. An extension of tllm_swiglu
 * (python/triton_llm/ops/swiglu.py:54-76 is fp16) on the tcgen05 kind::f8f6f4 path. x is
 * [M, K] (lda), the weights are given transposed: w1t, w3t [N, K] (ldb1, ldb3), K contiguous;
 * K and the input leading dimensions must be multiples of 16, inputs 16-byte aligned.
 */
TLLM_API int tllm_swiglu_fp8(const void *x, const void *w1t, const void *w3t, void *out,
                             int64_t M, int64_t N, int64_t K, int64_t lda, int64_t ldb1,
                             int64_t ldb3, int64_t ldo, float scale_x, float scale_w1,
                             float scale_w3, int out_dtype, void *stream);

/* Same as tllm_swiglu_fp8 with an explicit kernel choice, for cross-checking: 0 = automatic
 * (the CTA-pair kernel when M >= 256), 1 = one CTA per 128 x 128 output tile, 2 = the
 * CTA-pair kernel (two CTAs on two SMs share 256 x 128 output tiles through
 * tcgen05.mma.cta_group::2). */
TLLM_API int tllm_swiglu_fp8_variant(const void *x, const void *w1t, const void *w3t, void *out,
                                     int64_t M, int64_t N, int64_t K, int64_t lda, int64_t ldb1,
                                     int64_t ldb3, int64_t ldo, float scale_x, float scale_w1,
                                     float scale_w3, int out_dtype, int variant, void *stream);

/*
 * FP8 flash attention forward: softmax(sm_scale * (scale_q q)(scale_k k)^T) (scale_v v) with
 * e4m3 inputs and per-tensor scales, on the tcgen05 kind::f8f6f4 path; an extension of
 * tllm_flash_attn_fwd (python/triton_llm/ops/flash_attention.py:107-133 is fp16/bf16), with the
 * same top-left causal mask. q [B, H, Sq, D], k [B, H, Sk, D], and V transposed: vt
 * [B, H, D, Sk] (keys contiguous); D 64 or 128; strides in elements, innermost 1, the others
 * multiples of 16; inputs 16-byte aligned. o [B, H, Sq, D] in out_dtype (fp16 or bf16), any
 * strides. P is rounded to e4m3 for the P V product; the row sums use it unrounded.
 */
TLLM_API int tllm_flash_attn_fp8_fwd(const void *q, const void *k, const void *vt, void *o,
                                     int64_t B, int64_t H, int64_t Sq, int64_t Sk, int64_t D,
                                     const int64_t *sq, const int64_t *sk, const int64_t *svt,
                                     const int64_t *so, float sm_scale, float scale_q,
                                     float scale_k, float scale_v, int causal, int out_dtype,
                                     void *stream);

/*
 * QKV projection with RMSNorm + RoPE fused into its epilogue. No counterpart in the reference,
 * which runs rmsnorm_rope (python/triton_llm/ops/rmsnorm_rope.py:51-75) as a separate pass over
 * projected q/k. out [M, N] = x [M, K] @ w [K, N] with N = (Hq + 2*Hkv) * D laid out as
 * [q heads | k heads | v heads] (D = 128); every q head (RMSNorm weight wq [D]) and k head
 * (wk [D]) of token row m goes through tllm_rmsnorm_rope's arithmetic on the projection
 * rounded to the I/O dtype, with cos/sin row positions[m] (cos/sin [rope_rows, D], row strides
 * scos/ssin; positions int32 [M] on the device, clamped to the table); v heads are stored
 * as projected. K and the leading dimensions must be multiples of 8, pointers 16-byte aligned.
 */
TLLM_API int tllm_qkv_norm_rope(const void *x, const void *w, const void *wq, const void *wk,
                                const void *cos, const void *sin, int64_t rope_rows,
                                int64_t scos, int64_t ssin, const int32_t *positions, void *out,
                                int64_t M, int64_t K, int64_t Hq, int64_t Hkv, int64_t D,
                                int64_t lda, int64_t ldw, int64_t ldo, float eps, int dtype,
                                void *stream);

#ifdef __cplusplus
}
#endif

#endif /* TLLM_SM100_H_ */
