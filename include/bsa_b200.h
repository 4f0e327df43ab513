/*
 * bsa_b200.h -- C ABI of the B200 block-sparse attention (BSA) engine.
 *
 * Every entry point takes plain device pointers, sizes and a CUDA stream (as void*), launches
 * asynchronously on that stream and returns a status code (BSA_OK == 0).  Nothing here
 * allocates device memory: outputs and scratch are owned by the caller.  Inputs are borrowed
 * read-only.  The error message of the last failing call on the calling host thread is
 * available from bsa_last_error().  Every entry point checks all of its arguments (and builds
 * every TMA descriptor it needs) before it queues its first kernel: a call that returns an
 * argument error (SHAPE, DTYPE, ALIGN, ARG) has launched nothing.
 *
 * Tensor conventions (the reference's, longcat_video/models/block_sparse_attention.py):
 *   q, k, v, out : [B, H, S, D] with element strides (sb, sh, ss) and d contiguous,
 *                  S = T * Hl * Wl tokens in t-major (t, h, w) order (:74-76)
 *   blocks       : chunk_thw = (cT, cH, cW) voxels, cT*cH*cW tokens each, numbered in
 *                  (bt, bh, bw) block-major order (:98-104, :137-159).  A contiguous
 *                  64-token block is shape (1, 1, S) with chunk (1, 1, 64).
 *   pooled       : [B*H, nb, D] fp32, nb = S / (cT*cH*cW)
 *   block index  : [B, H, nb, topk] int32, each row sorted ascending
 */
#ifndef BSA_B200_H
#define BSA_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* status codes */
#define BSA_OK 0
#define BSA_ERR_SHAPE 1       /* shape / chunk divisibility / size limits          */
#define BSA_ERR_DTYPE 2       /* unsupported dtype for this entry point            */
#define BSA_ERR_ALIGN 3       /* pointer or stride alignment (TMA needs 16 bytes)  */
#define BSA_ERR_INDEX 4       /* block index out of range (device-side check)      */
#define BSA_ERR_CUDA 5        /* CUDA runtime / driver error                       */
#define BSA_ERR_TIMEOUT 6     /* a bounded device wait expired                     */
#define BSA_ERR_ARG 7         /* null pointer / bad argument                       */

/* dtype codes */
#define BSA_DTYPE_F32 0
#define BSA_DTYPE_F16 1
#define BSA_DTYPE_BF16 2

/* Library version (major*10000 + minor*100 + patch). */
int bsa_version(void);

/* Copies the last error message of this host thread into buf (NUL terminated); returns its
 * length. */
int bsa_last_error(char* buf, int n);

/* Reads (and optionally clears) the sticky device-side error code written by the kernels
 * (BSA_ERR_INDEX for an out-of-range block id, an internal wait-site code >= 100 for a
 * bounded wait that expired).  Synchronises the device. */
int bsa_device_error(int clear);

/* mean_pool_blocks_3d -- longcat_video/models/block_sparse_attention.py:67-104.
 * pooled[bh, blk, d] = mean over the block's tokens of x[b, h, token, d], in fp32 with a fixed
 * summation order: a pairwise tree over the block's rows in token order ((r0 + r1) + (r2 + r3)) + ...,
 * then * 1/n; n = cT*cH*cW (a power of two, at most 64).  With rope != NULL the 3-D RoPE of longcat_video/models/rope_3d.py:107-128 is
 * applied first (fp32, rounded back to the input dtype, written to x_rot, contiguous
 * [B,H,S,D]) and the rotated values are pooled.  rope holds per-axis tables, one angle per
 * rotated pair, over the RoPE grid (rope_T, rope_H, rope_W) (token s at t = s / (H*W),
 * h = (s / W) % H, w = s % W; this grid may differ from the block geometry, e.g. contiguous
 * 64-token blocks over a 24x45x80 latent): cos_t[rope_T][dt/2], sin_t[rope_T][dt/2],
 * cos_h[rope_H][dh/2], sin_h, cos_w[rope_W][dw/2], sin_w, concatenated in that order. */
int bsa_mean_pool(const void* x, int dtype, int B, int H, int S, int D, int64_t sb, int64_t sh, int64_t ss,
                  int T, int Hl, int Wl, int cT, int cH, int cW, const float* rope, int rope_dt, int rope_dh,
                  int rope_dw, int rope_T, int rope_H, int rope_W, void* x_rot, float* pooled, void* stream);

/* bsa_mean_pool with the q/k RMSNorm of the DiT attention fused in front of the RoPE --
 * RMSNorm_FP32 (longcat_video/models/blocks.py:55-73) applied as attention.py:195-196 does, then
 * rope_3d.py:107-128, then block_sparse_attention.py:67-104.  Per token row: x * rsqrt(mean(x^2) + eps) in
 * fp32 (the sum of squares in a fixed order; rsqrt to within its hardware error), rounded to the input
 * dtype, times norm_weight (input dtype, [D], 16-byte aligned) rounded again; then the optional RoPE.
 * The transformed rows are written to x_rot (required) and pooled. */
int bsa_mean_pool_norm(const void* x, int dtype, int B, int H, int S, int D, int64_t sb, int64_t sh, int64_t ss,
                       int T, int Hl, int Wl, int cT, int cH, int cW, const float* rope, int rope_dt, int rope_dh,
                       int rope_dw, int rope_T, int rope_H, int rope_W, const void* norm_weight, float norm_eps,
                       void* x_rot, float* pooled, void* stream);

/* block_routing_scores + topk_block_indices -- block_sparse_attention.py:107-134.
 * score[i][j] = fp32 fma chain over d = 0..D-1 of q_pooled[i][d] * k_pooled[j][d]; each row
 * keeps the topk largest scores (ties: smaller block id first) and writes their block ids
 * sorted ascending.  scores (required, caller-owned, 16-byte aligned) receives the full
 * [BH, nb, nb] fp32 score matrix that the selection reads.  D must be a multiple of 8. */
int bsa_score_topk(const float* q_pooled, const float* k_pooled, int BH, int nb, int D, int topk,
                   int32_t* block_indices, float* scores, void* stream);

/* block_routing_scores + topk_block_indices without the score matrix -- block_sparse_attention.py:107-134.
 * Same indices as bsa_score_topk (the k largest exact fp32 scores, each one fma chain over d; ties to the
 * smaller block id; ids ascending), computed from tensor-core approximate scores with an error bound and
 * exact scores for the blocks near each row's threshold.  scratch: bsa_route_scratch_bytes(BH, nb, D)
 * bytes of caller-owned device memory, 256-byte aligned (bf16 copies of the pooled blocks, their norms
 * and 16-bit score keys [BH, nb, round_up(nb, 8)]).  nb <= 3072; bsa_route_scratch_bytes returns 0 for
 * sizes it does not serve. */
int64_t bsa_route_scratch_bytes(int BH, int nb, int D);
int bsa_route_topk(const float* q_pooled, const float* k_pooled, int BH, int nb, int D, int topk,
                   int32_t* block_indices, void* scratch, void* stream);

/* block_routing_scores alone (block_sparse_attention.py:107-112): scores[BH, nq, nk] fp32. */
int bsa_block_scores(const float* q_pooled, const float* k_pooled, int BH, int nq, int nk, int D, float* scores,
                     void* stream);

/* topk_block_indices on a given score matrix (block_sparse_attention.py:115-134): scores
 * [rows, nk] fp32 -> block_indices [rows, topk], same selection rule as bsa_score_topk. */
int bsa_topk_from_scores(const float* scores, int rows, int nk, int topk, int32_t* block_indices, void* stream);

/* Sparse attention over given block indices -- the kernel-level entry of the reference
 * (bsa_attention_metal*(q, k, v, block_indices, chunk_thw, shape),
 * longcat_video/models/block_sparse_attention_metal.py:224-295, 484-548, 729-810, 985-1046).
 * out[b,h,s,:] = softmax over the tokens of the selected KV blocks of s's block.
 * dtype: BSA_DTYPE_F16 or BSA_DTYPE_BF16; D <= 128 and D % 8 == 0; block size 64.
 * q/k/v strides: element strides of [B,H,S,D] (d contiguous); b and h must merge
 * (sb == H*sh) unless B == 1.  Block ids are range-checked on the device. */
int bsa_attention_indices(const void* q, const void* k, const void* v, const int32_t* block_indices, int dtype,
                          int B, int H, int S, int D, const int64_t* q_strides, const int64_t* k_strides,
                          const int64_t* v_strides, int T, int Hl, int Wl, int cT, int cH, int cW, int topk,
                          float sm_scale, void* out, const int64_t* out_strides, void* stream);

/* Full BSA call -- bsa_attention(q, k, v, shape, sparsity, chunk_thw, sm_scale),
 * block_sparse_attention.py:201-250: pool Q and K, score, top-k, sparse attention.
 * scratch: caller-provided device memory of bsa_forward_scratch_bytes() bytes, 256-byte aligned
 * (pooled fp32 Q/K, [B*H, nb, D] each, then the routing scratch of bsa_route_topk; for nb > 3072 the
 * fp32 block-score matrix [B*H, nb, nb] with rows padded to a multiple of 4 instead).  block_indices
 * receives the routing ([B,H,nb,topk]).  With rope != NULL, q and k are
 * pre-RoPE and q_rot / k_rot (contiguous [B,H,S,D]) receive the rotated tensors that the
 * attention then reads. */
int64_t bsa_forward_scratch_bytes(int B, int H, int S, int D, int cT, int cH, int cW);
int bsa_forward(const void* q, const void* k, const void* v, int dtype, int B, int H, int S, int D,
                const int64_t* q_strides, const int64_t* k_strides, const int64_t* v_strides, int T, int Hl, int Wl,
                int cT, int cH, int cW, int topk, float sm_scale, const float* rope, int rope_dt, int rope_dh,
                int rope_dw, int rope_T, int rope_H, int rope_W, void* q_rot, void* k_rot, void* scratch,
                int32_t* block_indices, void* out, const int64_t* out_strides, void* stream);

/* The same two calls with `sm_reserve`: the persistent attention kernel then runs on (SM count -
 * sm_reserve) CTAs (at least 1), leaving sm_reserve SMs free for kernels on other streams -- the
 * all-to-all of a sequence-parallel job, whose kernels could not start next to an attention kernel
 * that holds every SM.  sm_reserve = 0 is the plain call. */
int bsa_attention_indices_ex(const void* q, const void* k, const void* v, const int32_t* block_indices, int dtype,
                             int B, int H, int S, int D, const int64_t* q_strides, const int64_t* k_strides,
                             const int64_t* v_strides, int T, int Hl, int Wl, int cT, int cH, int cW, int topk,
                             float sm_scale, void* out, const int64_t* out_strides, int sm_reserve, void* stream);
int bsa_forward_ex(const void* q, const void* k, const void* v, int dtype, int B, int H, int S, int D,
                   const int64_t* q_strides, const int64_t* k_strides, const int64_t* v_strides, int T, int Hl,
                   int Wl, int cT, int cH, int cW, int topk, float sm_scale, const float* rope, int rope_dt,
                   int rope_dh, int rope_dw, int rope_T, int rope_H, int rope_W, void* q_rot, void* k_rot,
                   void* scratch, int32_t* block_indices, void* out, const int64_t* out_strides, int sm_reserve,
                   void* stream);

/* bsa_forward_ex on the raw q/k of the attention's QKV projection: the q/k RMSNorm
 * (attention.py:195-196, blocks.py:55-73; q_norm_weight / k_norm_weight in the input dtype, [D]) runs
 * fused with the optional RoPE and the pooling (bsa_mean_pool_norm), q_rot / k_rot receive the
 * normalised (and rotated) tensors, and the attention reads them. */
int bsa_forward_qknorm(const void* q, const void* k, const void* v, int dtype, int B, int H, int S, int D,
                       const int64_t* q_strides, const int64_t* k_strides, const int64_t* v_strides, int T, int Hl,
                       int Wl, int cT, int cH, int cW, int topk, float sm_scale, const float* rope, int rope_dt,
                       int rope_dh, int rope_dw, int rope_T, int rope_H, int rope_W, const void* q_norm_weight,
                       const void* k_norm_weight, float norm_eps, void* q_rot, void* k_rot, void* scratch,
                       int32_t* block_indices, void* out, const int64_t* out_strides, int sm_reserve, void* stream);

/* bsa_set_phase_event: profiling hook, no counterpart in the reference.  `event` (a cudaEvent_t, or NULL to
 * stop) is recorded on the call's stream between the routing launches and the attention launch of every
 * later bsa_forward* call made by the calling host thread, so a caller can time the two phases of one
 * call with CUDA events.  The event must outlive those calls. */
int bsa_set_phase_event(void* event);

/* bsa_forward without caller-provided scratch -- no counterpart in the reference (MLX manages
 * memory itself); it exists for callers that cannot allocate device memory where they call
 * attention (a region whose memory is fixed in advance, an embedder that owns the whole device
 * budget, a host binding without a device allocator).  Same arguments and results as bsa_forward
 * minus `scratch`: the pooled Q/K and routing scratch comes from an array compiled into the library, of
 * BSA_NOALLOC_SCRATCH_BYTES per GPU that loads the library, held until the process exits.
 * Calls that would need more (bsa_forward_scratch_bytes() > BSA_NOALLOC_SCRATCH_BYTES) return
 * BSA_ERR_SHAPE.  Nothing is allocated: no cudaMalloc, cudaFree or allocating library routine.
 * The first call on a device resolves the array's device address (cudaGetSymbolAddress, with that
 * device current) and keeps it for the life of the process; make that first call before any stream
 * capture.  A device reset (cudaDeviceReset) is not supported: the cached address would be stale.
 * Every call on a device shares the one array: calls whose kernels overlap on the GPU (different
 * streams, or concurrent host threads) race on it and must be serialised by the caller.  The array
 * serves calls with bsa_forward_scratch_bytes(B, H, S, D, cT, cH, cW) <= BSA_NOALLOC_SCRATCH_BYTES, i.e.
 * small shapes (about B*H*nb*(8*D + 2*nb + 1100) bytes, nb = S/64); the 720p benchmark shapes need far
 * more and are refused. */
#define BSA_NOALLOC_SCRATCH_BYTES (16u << 20)
int bsa_forward_noalloc(const void* q, const void* k, const void* v, int dtype, int B, int H, int S, int D,
                        const int64_t* q_strides, const int64_t* k_strides, const int64_t* v_strides, int T, int Hl,
                        int Wl, int cT, int cH, int cW, int topk, float sm_scale, const float* rope, int rope_dt,
                        int rope_dh, int rope_dw, int rope_T, int rope_H, int rope_W, void* q_rot, void* k_rot,
                        int32_t* block_indices, void* out, const int64_t* out_strides, void* stream);

/* ---- peer exchange helpers (sequence-parallel all-to-all over NVLink by the copy engines) ----
 * No counterpart in the reference (the MLX port has no multi-GPU path; the upstream PyTorch model
 * used NCCL all-to-all).  These are the only allocating entry points: the exchange owns a few
 * persistent buffers per process group and shape, which other processes of the node map.
 * bsa_ipc_alloc: cudaMalloc `bytes` and export it; `handle` receives BSA_IPC_HANDLE_BYTES bytes.
 * bsa_ipc_open : map a buffer exported by another process of the node (peer access enabled);
 *                bsa_ipc_close unmaps it, bsa_ipc_free frees a buffer of bsa_ipc_alloc.
 * bsa_copy_2d  : `height` rows of `width` bytes, pitches in bytes, any mix of local and mapped peer
 *                memory, asynchronous on `stream` (copy engine). */
#define BSA_IPC_HANDLE_BYTES 64
int bsa_ipc_alloc(int64_t bytes, void** ptr, unsigned char* handle);
int bsa_ipc_free(void* ptr);
int bsa_ipc_open(const unsigned char* handle, void** ptr);
int bsa_ipc_close(void* ptr);
int bsa_copy_2d(void* dst, int64_t dpitch, const void* src, int64_t spitch, int64_t width, int64_t height,
                void* stream);
/* bsa_copy_3d  : `depth` slices of `height` rows of `width` bytes; row pitches dpitch / spitch and slice
 *                pitches dslice / sslice in bytes (a slice pitch is a multiple of its row pitch and holds
 *                `height` rows).  The copy engine pays a fixed cost per call (about 11 us measured on
 *                B200 over NVLink, against 4 us for moving 2.6 MiB), so one call should move as much as
 *                the layouts allow: the exchange moves q, k and v of a head group from a peer in one call.
 * bsa_copy_3d_list: n bsa_copy_3d calls in order on one stream, from desc[9*i .. 9*i+8] = (dst, dpitch,
 *                dslice, src, spitch, sslice, width, height, depth) -- one host call for an exchange's whole
 *                copy plan of a head group. */
int bsa_copy_3d(void* dst, int64_t dpitch, int64_t dslice, const void* src, int64_t spitch, int64_t sslice,
                int64_t width, int64_t height, int64_t depth, void* stream);
int bsa_copy_3d_list(const int64_t* desc, int n, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* BSA_B200_H */
