// C ABI of the BSA engine (declared in include/bsa_b200.h): argument validation, TMA tensor-map
// construction and kernel composition.  No entry point allocates device memory.
//
// Every entry point validates all of its arguments -- and builds every tensor map it will use --
// before it queues its first kernel: a call that returns an error has launched nothing.  The work of
// an entry point is therefore split into a plan (checks, maps, kernel arguments; host only) and a
// run (the launches).
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>
#include "bsa_kernels.h"

namespace {

thread_local char g_msg[512] = {0};

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_msg, sizeof(g_msg), fmt, ap);
  va_end(ap);
  return code;
}

int cuda_fail(const char* what) {
  const cudaError_t e = cudaGetLastError();
  return fail(BSA_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

int elt_bytes(int dtype) { return dtype == BSA_DTYPE_F32 ? 4 : 2; }

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Shared geometry checks of block_sparse_attention.py:86-96 (same wording as the reference).
int check_geometry(int S, int T, int Hl, int Wl, int cT, int cH, int cW) {
  if (cT <= 0 || cH <= 0 || cW <= 0 || T <= 0 || Hl <= 0 || Wl <= 0)
    return fail(BSA_ERR_SHAPE, "shape and chunk_thw must be positive");
  if (T % cT || Hl % cH || Wl % cW)
    return fail(BSA_ERR_SHAPE,
                "Latent shape (%d, %d, %d) must be a multiple of chunk_thw (%d, %d, %d); refinement padding should "
                "guarantee this.",
                T, Hl, Wl, cT, cH, cW);
  if (static_cast<long long>(T) * Hl * Wl != S)
    return fail(BSA_ERR_SHAPE, "S=%d doesn't match T*H*W=%lld for shape (%d, %d, %d)", S,
                static_cast<long long>(T) * Hl * Wl, T, Hl, Wl);
  return BSA_OK;
}

// A block of chunk_thw voxels is one contiguous run of tokens (in t-major order) when it spans whole
// rows below its first partial axis: blocks are then numbered in token order, block b starting at
// token b * cT*cH*cW.  The benchmark's 64-token blocks (shape (1, 1, S), chunk (1, 1, 64)) are.
bool contiguous_blocks(int Hl, int Wl, int cT, int cH, int cW) {
  return (cT == 1 || (cH == Hl && cW == Wl)) && (cH == 1 || cW == Wl);
}

// Tiled map over one of q/k/v, 128B swizzle, 64-element d halves.  Contiguous blocks: 3-D (d, s, b*h),
// box (64, n, 1), addressed by the block's first token; other voxel blocks: 5-D (d, w, h, t, b*h), box
// (64, cW, cH, cT, 1), addressed by the block's (t, h, w) origin.  Both move the same bytes at the same
// rate (16 KB blocks gathered from L2: 13.4 TB/s either way); the 3-D form spares the issuing threads
// the two integer divisions of the block origin.  Out-of-range d (D < 128) reads as zero, which pads
// the head dimension for the MMA.  *map3 (nullable) receives which form was built.
int make_map(CUtensorMap* m, const void* base, int dtype, int B, int H, int D, const int64_t* st, int T, int Hl,
             int Wl, int cT, int cH, int cW, const char* name, int* map3 = nullptr) {
  auto enc = encode_fn();
  if (!enc) return fail(BSA_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  const int e = elt_bytes(dtype);
  const int64_t sb = st[0], sh = st[1], ss = st[2];
  if (!aligned16(base)) return fail(BSA_ERR_ALIGN, "%s: base pointer must be 16-byte aligned", name);
  if ((ss * e) % 16 || (sh * e) % 16 || (B > 1 && (sb * e) % 16))
    return fail(BSA_ERR_ALIGN, "%s: strides must be multiples of 16 bytes (got sb=%lld sh=%lld ss=%lld elements)",
                name, (long long)sb, (long long)sh, (long long)ss);
  if (B > 1 && sb != static_cast<int64_t>(H) * sh)
    return fail(BSA_ERR_SHAPE, "%s: batch and head strides must merge (sb == H*sh) when B > 1", name);
  const bool c3 = contiguous_blocks(Hl, Wl, cT, cH, cW);
  const cuuint64_t S = static_cast<cuuint64_t>(T) * Hl * Wl;
  cuuint64_t dims[5], strides[4];
  cuuint32_t box[5];
  cuuint32_t es[5] = {1, 1, 1, 1, 1};
  cuuint32_t rank;
  if (c3) {
    rank = 3;
    dims[0] = static_cast<cuuint64_t>(D); dims[1] = S; dims[2] = static_cast<cuuint64_t>(B) * H;
    strides[0] = static_cast<cuuint64_t>(ss * e); strides[1] = static_cast<cuuint64_t>(sh * e);
    box[0] = 64; box[1] = static_cast<cuuint32_t>(cT * cH * cW); box[2] = 1;
  } else {
    rank = 5;
    dims[0] = static_cast<cuuint64_t>(D); dims[1] = static_cast<cuuint64_t>(Wl); dims[2] = static_cast<cuuint64_t>(Hl);
    dims[3] = static_cast<cuuint64_t>(T); dims[4] = static_cast<cuuint64_t>(B) * H;
    strides[0] = static_cast<cuuint64_t>(ss * e); strides[1] = static_cast<cuuint64_t>(ss * e * Wl);
    strides[2] = static_cast<cuuint64_t>(ss * e * Wl * Hl); strides[3] = static_cast<cuuint64_t>(sh * e);
    box[0] = 64; box[1] = static_cast<cuuint32_t>(cW); box[2] = static_cast<cuuint32_t>(cH);
    box[3] = static_cast<cuuint32_t>(cT); box[4] = 1;
  }
  const CUtensorMapDataType dt =
      dtype == BSA_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  const CUresult r = enc(m, dt, rank, const_cast<void*>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                         CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (map3) *map3 = c3 ? 1 : 0;
  if (r != CUDA_SUCCESS) return fail(BSA_ERR_ARG, "%s: cuTensorMapEncodeTiled failed (%d)", name, static_cast<int>(r));
  return BSA_OK;
}

// 3-D map over one bf16 pair array of the routing scratch: (d = 128, block = nb, b*h = BH), box (64, 128, 1).
int make_pair_map(CUtensorMap* m, const void* base, int nb, int BH) {
  auto enc = encode_fn();
  if (!enc) return fail(BSA_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  cuuint64_t dims[3] = {128, static_cast<cuuint64_t>(nb), static_cast<cuuint64_t>(BH)};
  cuuint64_t strides[2] = {256, static_cast<cuuint64_t>(nb) * 256};
  cuuint32_t box[3] = {64, 128, 1};
  cuuint32_t es[3] = {1, 1, 1};
  const CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, es,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(BSA_ERR_ARG, "routing pair map: cuTensorMapEncodeTiled failed (%d)", static_cast<int>(r));
  return BSA_OK;
}

// ------------------------------------------------------------------ plans: validated, ready to launch
// Profiling hook of bsa_set_phase_event: recorded between the routing and the attention launches of
// the forward calls made by this host thread.
thread_local cudaEvent_t t_phase_event = nullptr;

struct PoolPlan {
  bsa::PoolArgs a;
  CUtensorMap map;
  bool has_map = false;
};

int pool_plan(PoolPlan& pl, const void* x, int dtype, int B, int H, int S, int D, int64_t sb, int64_t sh, int64_t ss,
              int T, int Hl, int Wl, int cT, int cH, int cW, const float* rope, int rope_dt, int rope_dh, int rope_dw,
              int rope_T, int rope_H, int rope_W, void* x_rot, float* pooled, const void* norm_w = nullptr,
              float norm_eps = 0.f) {
  if (!x || !pooled) return fail(BSA_ERR_ARG, "null pointer");
  if (dtype != BSA_DTYPE_F32 && dtype != BSA_DTYPE_F16 && dtype != BSA_DTYPE_BF16)
    return fail(BSA_ERR_DTYPE, "unsupported dtype code %d", dtype);
  if (B <= 0 || H <= 0 || S <= 0 || D <= 0) return fail(BSA_ERR_SHAPE, "empty tensor");
  int rc = check_geometry(S, T, Hl, Wl, cT, cH, cW);
  if (rc) return rc;
  const int n = cT * cH * cW;
  if (n & (n - 1) || n > 64) return fail(BSA_ERR_SHAPE, "block size %d must be a power of two <= 64", n);
  if (D % 8 || D > 128) return fail(BSA_ERR_SHAPE, "head_dim D=%d must be a multiple of 8 and <= 128", D);
  const int e = elt_bytes(dtype);
  if (!aligned16(x) || (ss * e) % 16 || (sh * e) % 16 || (sb * e) % 16)
    return fail(BSA_ERR_ALIGN, "x must be 16-byte aligned with 16-byte-multiple strides");
  if (!aligned16(pooled)) return fail(BSA_ERR_ALIGN, "pooled must be 16-byte aligned");
  if (norm_w) {
    if (!x_rot) return fail(BSA_ERR_ARG, "x_rot is required with a norm weight");
    if (!aligned16(norm_w)) return fail(BSA_ERR_ALIGN, "the norm weight must be 16-byte aligned");
    if (!(norm_eps >= 0.f)) return fail(BSA_ERR_ARG, "norm eps must be >= 0");
    if (!aligned16(x_rot)) return fail(BSA_ERR_ALIGN, "x_rot must be 16-byte aligned");
  }
  if (rope) {
    if (!x_rot) return fail(BSA_ERR_ARG, "x_rot is required with rope tables");
    if (!aligned16(x_rot)) return fail(BSA_ERR_ALIGN, "x_rot must be 16-byte aligned");
    if (rope_dt + rope_dh + rope_dw != D || (rope_dt | rope_dh | rope_dw) & 1 || rope_dt < 0 || rope_dh < 0 ||
        rope_dw < 0)
      return fail(BSA_ERR_SHAPE, "rope dims (%d, %d, %d) must be even and sum to D=%d", rope_dt, rope_dh, rope_dw, D);
    if (rope_T <= 0 || rope_H <= 0 || rope_W <= 0 || static_cast<long long>(rope_T) * rope_H * rope_W != S)
      return fail(BSA_ERR_SHAPE, "rope grid (%d, %d, %d) does not cover S=%d", rope_T, rope_H, rope_W, S);
  }
  bsa::PoolArgs& a = pl.a;
  a.x = x; a.dtype = dtype; a.B = B; a.H = H; a.S = S; a.D = D; a.sb = sb; a.sh = sh; a.ss = ss;
  a.T = T; a.Hl = Hl; a.Wl = Wl; a.cT = cT; a.cH = cH; a.cW = cW;
  a.rope = rope; a.rope_dt = rope_dt; a.rope_dh = rope_dh; a.rope_dw = rope_dw;
  a.rope_T = rope_T; a.rope_H = rope_H; a.rope_W = rope_W;
  a.x_rot = x_rot; a.pooled = pooled;
  a.norm_w = norm_w; a.norm_eps = norm_eps;
  a.tmap = nullptr;
  a.map3 = 0;
  pl.has_map = false;
  // bf16/fp16 blocks of 64 d-wide halves stream through a TMA ring; the map needs mergeable batch
  // and head strides, which the register kernel does not
  if (dtype != BSA_DTYPE_F32 && !rope && !norm_w && (B == 1 || sb == static_cast<int64_t>(H) * sh)) {
    // a map that cannot be built only selects the register kernel: keep the caller's last message
    char saved[sizeof(g_msg)];
    memcpy(saved, g_msg, sizeof(g_msg));
    const int64_t st[3] = {sb, sh, ss};
    if (make_map(&pl.map, x, dtype, B, H, D, st, T, Hl, Wl, cT, cH, cW, "x", &a.map3) == BSA_OK) pl.has_map = true;
    else memcpy(g_msg, saved, sizeof(g_msg));
  }
  return BSA_OK;
}

int pool_run(PoolPlan& pl, void* stream) {
  pl.a.tmap = pl.has_map ? &pl.map : nullptr;
  const int rc = bsa::launch_pool(pl.a, static_cast<cudaStream_t>(stream));
  if (rc == BSA_ERR_CUDA) return cuda_fail("pool kernel launch");
  if (rc) return fail(rc, "pool: unsupported configuration");
  return BSA_OK;
}

struct AttnPlan {
  CUtensorMap mq, mk, mv;
  bsa::AttnArgs a;
};

int attn_plan(AttnPlan& pl, const void* q, const void* k, const void* v, const int32_t* block_indices, int dtype,
              int B, int H, int S, int D, const int64_t* q_strides, const int64_t* k_strides, const int64_t* v_strides,
              int T, int Hl, int Wl, int cT, int cH, int cW, int topk, float sm_scale, void* out,
              const int64_t* out_strides, int sm_reserve) {
  if (sm_reserve < 0) return fail(BSA_ERR_ARG, "sm_reserve=%d must be >= 0", sm_reserve);
  if (!q || !k || !v || !block_indices || !out || !q_strides || !k_strides || !v_strides || !out_strides)
    return fail(BSA_ERR_ARG, "null pointer");
  if (dtype != BSA_DTYPE_F16 && dtype != BSA_DTYPE_BF16)
    return fail(BSA_ERR_DTYPE, "sparse attention supports fp16 and bf16 inputs (dtype code %d)", dtype);
  if (B <= 0 || H <= 0 || S <= 0) return fail(BSA_ERR_SHAPE, "empty tensor");
  int rc = check_geometry(S, T, Hl, Wl, cT, cH, cW);
  if (rc) return rc;
  if (cT * cH * cW != 64)
    return fail(BSA_ERR_SHAPE, "block size must be 64 tokens (chunk_thw product), got %d", cT * cH * cW);
  if (D % 8 || D < 8 || D > 128) return fail(BSA_ERR_SHAPE, "head_dim D=%d must be a multiple of 8 in [8, 128]", D);
  const int nb = S / 64;
  if (topk < 1 || topk > nb) return fail(BSA_ERR_SHAPE, "topk=%d out of range for %d KV blocks", topk, nb);
  if (!aligned16(block_indices)) return fail(BSA_ERR_ALIGN, "block_indices must be 16-byte aligned");
  if ((rc = make_map(&pl.mq, q, dtype, B, H, D, q_strides, T, Hl, Wl, cT, cH, cW, "q", &pl.a.map3))) return rc;
  if ((rc = make_map(&pl.mk, k, dtype, B, H, D, k_strides, T, Hl, Wl, cT, cH, cW, "k"))) return rc;
  if ((rc = make_map(&pl.mv, v, dtype, B, H, D, v_strides, T, Hl, Wl, cT, cH, cW, "v"))) return rc;
  bsa::AttnArgs& a = pl.a;  // a.map3 was set by make_map (the same form for q, k and v)
  a.idx = block_indices; a.out = out;
  a.B = B; a.H = H; a.S = S; a.D = D; a.nb = nb; a.topk = topk;
  a.Hl = Hl; a.Wl = Wl; a.cT = cT; a.cH = cH; a.cW = cW;
  a.out_sb = out_strides[0]; a.out_sh = out_strides[1]; a.out_ss = out_strides[2];
  a.sm_scale = sm_scale;
  a.is_bf16 = dtype == BSA_DTYPE_BF16;
  a.sm_reserve = sm_reserve;
  return BSA_OK;
}

int attn_run(AttnPlan& pl, void* stream) {
  const int rc = bsa::launch_attn(&pl.mq, &pl.mk, &pl.mv, pl.a, static_cast<cudaStream_t>(stream));
  if (rc == BSA_ERR_CUDA) return cuda_fail("attention kernel launch");
  return rc;
}

int64_t score_ld(int nb) { return (static_cast<int64_t>(nb) + 3) & ~int64_t(3); }

}  // namespace

namespace bsa {
int set_error(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_msg, sizeof(g_msg), fmt, ap);
  va_end(ap);
  return code;
}
}  // namespace bsa

extern "C" {

int bsa_version(void) { return 100; }

int bsa_last_error(char* buf, int n) {
  const int len = static_cast<int>(strlen(g_msg));
  if (buf && n > 0) {
    strncpy(buf, g_msg, n - 1);
    buf[n - 1] = 0;
  }
  return len;
}

int bsa_device_error(int clear) {
  if (cudaDeviceSynchronize() != cudaSuccess) return cuda_fail("cudaDeviceSynchronize");
  const int a = bsa::attn_device_error(clear);
  const int s = bsa::score_device_error(clear);
  const int r = bsa::route_device_error(clear);
  return a ? a : (s ? s : r);
}

int bsa_mean_pool(const void* x, int dtype, int B, int H, int S, int D, int64_t sb, int64_t sh, int64_t ss, int T,
                  int Hl, int Wl, int cT, int cH, int cW, const float* rope, int rope_dt, int rope_dh, int rope_dw,
                  int rope_T, int rope_H, int rope_W, void* x_rot, float* pooled, void* stream) {
  PoolPlan pl;
  const int rc = pool_plan(pl, x, dtype, B, H, S, D, sb, sh, ss, T, Hl, Wl, cT, cH, cW, rope, rope_dt, rope_dh,
                           rope_dw, rope_T, rope_H, rope_W, x_rot, pooled);
  if (rc) return rc;
  return pool_run(pl, stream);
}

int bsa_mean_pool_norm(const void* x, int dtype, int B, int H, int S, int D, int64_t sb, int64_t sh, int64_t ss, int T,
                       int Hl, int Wl, int cT, int cH, int cW, const float* rope, int rope_dt, int rope_dh,
                       int rope_dw, int rope_T, int rope_H, int rope_W, const void* norm_weight, float norm_eps,
                       void* x_rot, float* pooled, void* stream) {
  if (!norm_weight) return fail(BSA_ERR_ARG, "null pointer");
  PoolPlan pl;
  const int rc = pool_plan(pl, x, dtype, B, H, S, D, sb, sh, ss, T, Hl, Wl, cT, cH, cW, rope, rope_dt, rope_dh,
                           rope_dw, rope_T, rope_H, rope_W, x_rot, pooled, norm_weight, norm_eps);
  if (rc) return rc;
  return pool_run(pl, stream);
}

int bsa_score_topk(const float* q_pooled, const float* k_pooled, int BH, int nb, int D, int topk,
                   int32_t* block_indices, float* scores, void* stream) {
  if (!q_pooled || !k_pooled || !block_indices || !scores) return fail(BSA_ERR_ARG, "null pointer");
  if (BH <= 0 || nb <= 0 || D <= 0 || D > 128 || D % 8)
    return fail(BSA_ERR_SHAPE, "bad sizes BH=%d nb=%d D=%d (D must be a multiple of 8, at most 128)", BH, nb, D);
  if (reinterpret_cast<uintptr_t>(scores) & 15u) return fail(BSA_ERR_ALIGN, "scores must be 16-byte aligned");
  if ((reinterpret_cast<uintptr_t>(q_pooled) | reinterpret_cast<uintptr_t>(k_pooled)) & 15u)
    return fail(BSA_ERR_ALIGN, "pooled blocks must be 16-byte aligned");
  if (topk < 1 || topk > nb) return fail(BSA_ERR_SHAPE, "topk=%d out of range for %d KV blocks", topk, nb);
  bsa::ScoreArgs a;
  a.qp = q_pooled; a.kp = k_pooled; a.BH = BH; a.nq = nb; a.nk = nb; a.D = D; a.topk = topk;
  a.idx = block_indices; a.scores = scores; a.ldc = nb;
  const int rc = bsa::launch_score_topk(a, static_cast<cudaStream_t>(stream));
  if (rc == BSA_ERR_CUDA) return cuda_fail("score/top-k kernel launch");
  if (rc) return fail(rc, "score/top-k: unsupported sizes (nb=%d)", nb);
  return BSA_OK;
}

int64_t bsa_route_scratch_bytes(int BH, int nb, int D) {
  if (BH <= 0 || !bsa::route_supported(nb, D)) return 0;
  return bsa::route_scratch_bytes(BH, nb);
}

int bsa_route_topk(const float* q_pooled, const float* k_pooled, int BH, int nb, int D, int topk,
                   int32_t* block_indices, void* scratch, void* stream) {
  if (!q_pooled || !k_pooled || !block_indices || !scratch) return fail(BSA_ERR_ARG, "null pointer");
  if (BH <= 0 || !bsa::route_supported(nb, D))
    return fail(BSA_ERR_SHAPE, "bad sizes BH=%d nb=%d D=%d (nb at most 3072; D a multiple of 8, at most 128)", BH,
                nb, D);
  if ((reinterpret_cast<uintptr_t>(q_pooled) | reinterpret_cast<uintptr_t>(k_pooled)) & 15u)
    return fail(BSA_ERR_ALIGN, "pooled blocks must be 16-byte aligned");
  if (reinterpret_cast<uintptr_t>(scratch) & 255u) return fail(BSA_ERR_ALIGN, "scratch must be 256-byte aligned");
  if (topk < 1 || topk > nb) return fail(BSA_ERR_SHAPE, "topk=%d out of range for %d KV blocks", topk, nb);
  bsa::RouteArgs a;
  a.qp = q_pooled; a.kp = k_pooled; a.BH = BH; a.nb = nb; a.D = D; a.topk = topk;
  a.idx = block_indices; a.scratch = scratch; a.make_pair_map = make_pair_map;
  const int rc = bsa::launch_route(a, static_cast<cudaStream_t>(stream));
  if (rc == BSA_ERR_CUDA) return cuda_fail("routing kernel launch");
  return rc;
}

int bsa_block_scores(const float* q_pooled, const float* k_pooled, int BH, int nq, int nk, int D, float* scores,
                     void* stream) {
  if (!q_pooled || !k_pooled || !scores) return fail(BSA_ERR_ARG, "null pointer");
  if (BH <= 0 || nq <= 0 || nk <= 0 || D <= 0 || D > 128 || D % 8)
    return fail(BSA_ERR_SHAPE, "bad sizes BH=%d nq=%d nk=%d D=%d (D must be a multiple of 8, at most 128)", BH, nq,
                nk, D);
  if ((reinterpret_cast<uintptr_t>(q_pooled) | reinterpret_cast<uintptr_t>(k_pooled)) & 15u)
    return fail(BSA_ERR_ALIGN, "pooled blocks must be 16-byte aligned");
  bsa::ScoreArgs a;
  a.qp = q_pooled; a.kp = k_pooled; a.BH = BH; a.nq = nq; a.nk = nk; a.D = D; a.topk = 1;
  a.idx = nullptr; a.scores = scores; a.ldc = nk;
  const int rc = bsa::launch_scores_only(a, static_cast<cudaStream_t>(stream));
  if (rc == BSA_ERR_CUDA) return cuda_fail("score kernel launch");
  if (rc) return fail(rc, "scores: unsupported sizes (nq=%d nk=%d)", nq, nk);
  return BSA_OK;
}

int bsa_topk_from_scores(const float* scores, int rows, int nk, int topk, int32_t* block_indices, void* stream) {
  if (!scores || !block_indices) return fail(BSA_ERR_ARG, "null pointer");
  if (rows <= 0 || nk <= 0) return fail(BSA_ERR_SHAPE, "bad sizes rows=%d nk=%d", rows, nk);
  if (topk < 1 || topk > nk) return fail(BSA_ERR_SHAPE, "topk=%d out of range for %d KV blocks", topk, nk);
  const int rc = bsa::launch_topk(scores, rows, nk, nk, topk, block_indices, static_cast<cudaStream_t>(stream));
  if (rc == BSA_ERR_CUDA) return cuda_fail("top-k kernel launch");
  if (rc) return fail(rc, "top-k: unsupported sizes (nk=%d)", nk);
  return BSA_OK;
}

int bsa_attention_indices(const void* q, const void* k, const void* v, const int32_t* block_indices, int dtype,
                          int B, int H, int S, int D, const int64_t* q_strides, const int64_t* k_strides,
                          const int64_t* v_strides, int T, int Hl, int Wl, int cT, int cH, int cW, int topk,
                          float sm_scale, void* out, const int64_t* out_strides, void* stream) {
  return bsa_attention_indices_ex(q, k, v, block_indices, dtype, B, H, S, D, q_strides, k_strides, v_strides, T, Hl,
                                  Wl, cT, cH, cW, topk, sm_scale, out, out_strides, 0, stream);
}

int bsa_attention_indices_ex(const void* q, const void* k, const void* v, const int32_t* block_indices, int dtype,
                             int B, int H, int S, int D, const int64_t* q_strides, const int64_t* k_strides,
                             const int64_t* v_strides, int T, int Hl, int Wl, int cT, int cH, int cW, int topk,
                             float sm_scale, void* out, const int64_t* out_strides, int sm_reserve, void* stream) {
  AttnPlan pl;
  const int rc = attn_plan(pl, q, k, v, block_indices, dtype, B, H, S, D, q_strides, k_strides, v_strides, T, Hl, Wl,
                           cT, cH, cW, topk, sm_scale, out, out_strides, sm_reserve);
  if (rc) return rc;
  return attn_run(pl, stream);
}

// Scratch of bsa_forward: pooled Q and K (fp32, [B*H, nb, D] each, padded to 256 bytes), then the
// routing scratch (bsa_route_topk) where routing supports the size, else the fp32 score matrix.
int bsa_set_phase_event(void* event) {
  t_phase_event = static_cast<cudaEvent_t>(event);
  return BSA_OK;
}

int64_t bsa_forward_scratch_bytes(int B, int H, int S, int D, int cT, int cH, int cW) {
  const int n = cT * cH * cW;
  if (n <= 0 || B <= 0 || H <= 0 || S <= 0 || D <= 0) return 0;
  const int64_t nb = S / n;
  const int64_t pooled = (2ll * B * H * nb * D * 4 + 255) & ~int64_t(255);
  if (bsa::route_supported(static_cast<int>(nb), D))
    return pooled + bsa::route_scratch_bytes(B * H, static_cast<int>(nb));
  return pooled + static_cast<int64_t>(B) * H * nb * score_ld(static_cast<int>(nb)) * 4;
}

int bsa_forward(const void* q, const void* k, const void* v, int dtype, int B, int H, int S, int D,
                const int64_t* q_strides, const int64_t* k_strides, const int64_t* v_strides, int T, int Hl, int Wl,
                int cT, int cH, int cW, int topk, float sm_scale, const float* rope, int rope_dt, int rope_dh,
                int rope_dw, int rope_T, int rope_H, int rope_W, void* q_rot, void* k_rot, void* scratch,
                int32_t* block_indices, void* out, const int64_t* out_strides, void* stream) {
  return bsa_forward_ex(q, k, v, dtype, B, H, S, D, q_strides, k_strides, v_strides, T, Hl, Wl, cT, cH, cW, topk,
                        sm_scale, rope, rope_dt, rope_dh, rope_dw, rope_T, rope_H, rope_W, q_rot, k_rot, scratch,
                        block_indices, out, out_strides, 0, stream);
}

}  // extern "C"

namespace {
int forward_impl(const void* q, const void* k, const void* v, int dtype, int B, int H, int S, int D,
                 const int64_t* q_strides, const int64_t* k_strides, const int64_t* v_strides, int T, int Hl, int Wl,
                 int cT, int cH, int cW, int topk, float sm_scale, const float* rope, int rope_dt, int rope_dh,
                 int rope_dw, int rope_T, int rope_H, int rope_W, const void* q_norm_w, const void* k_norm_w,
                 float norm_eps, void* q_rot, void* k_rot, void* scratch, int32_t* block_indices, void* out,
                 const int64_t* out_strides, int sm_reserve, void* stream) {
  // ---- every check first: nothing is queued unless the whole call is valid
  if (sm_reserve < 0) return fail(BSA_ERR_ARG, "sm_reserve=%d must be >= 0", sm_reserve);
  if (!q || !k || !v || !scratch || !block_indices || !out || !q_strides || !k_strides || !v_strides || !out_strides)
    return fail(BSA_ERR_ARG, "null pointer");
  if (reinterpret_cast<uintptr_t>(scratch) & 255u) return fail(BSA_ERR_ALIGN, "scratch must be 256-byte aligned");
  if (dtype != BSA_DTYPE_F16 && dtype != BSA_DTYPE_BF16)
    return fail(BSA_ERR_DTYPE, "sparse attention supports fp16 and bf16 inputs (dtype code %d)", dtype);
  if (B <= 0 || H <= 0 || S <= 0 || D <= 0) return fail(BSA_ERR_SHAPE, "empty tensor");
  int rc = check_geometry(S, T, Hl, Wl, cT, cH, cW);
  if (rc) return rc;
  const int n = cT * cH * cW;
  if (n != 64) return fail(BSA_ERR_SHAPE, "block size must be 64 tokens (chunk_thw product), got %d", n);
  const int nb = S / 64;
  if (D % 8 || D > 128) return fail(BSA_ERR_SHAPE, "head_dim D=%d must be a multiple of 8 in [8, 128]", D);
  if (topk < 1 || topk > nb) return fail(BSA_ERR_SHAPE, "topk=%d out of range for %d KV blocks", topk, nb);
  float* qp = static_cast<float*>(scratch);
  float* kp = qp + static_cast<int64_t>(B) * H * nb * D;
  if ((q_norm_w != nullptr) != (k_norm_w != nullptr)) return fail(BSA_ERR_ARG, "q and k norm weights come together");
  PoolPlan pq, pk;
  if ((rc = pool_plan(pq, q, dtype, B, H, S, D, q_strides[0], q_strides[1], q_strides[2], T, Hl, Wl, cT, cH, cW, rope,
                      rope_dt, rope_dh, rope_dw, rope_T, rope_H, rope_W, q_rot, qp, q_norm_w, norm_eps)))
    return rc;
  if ((rc = pool_plan(pk, k, dtype, B, H, S, D, k_strides[0], k_strides[1], k_strides[2], T, Hl, Wl, cT, cH, cW, rope,
                      rope_dt, rope_dh, rope_dw, rope_T, rope_H, rope_W, k_rot, kp, k_norm_w, norm_eps)))
    return rc;
  void* rest = static_cast<uint8_t*>(scratch) + ((2ll * B * H * nb * D * 4 + 255) & ~int64_t(255));
  const bool route = bsa::route_supported(nb, D);
  bsa::RouteArgs ra;
  ra.qp = qp; ra.kp = kp; ra.BH = B * H; ra.nb = nb; ra.D = D; ra.topk = topk;
  ra.idx = block_indices; ra.scratch = rest; ra.make_pair_map = make_pair_map;
  __nv_bfloat16* split_hl = nullptr;
  float* split_nrm = nullptr;
  float* split_nkmax = nullptr;
  bsa::ScoreArgs sa;
  sa.qp = qp; sa.kp = kp; sa.BH = B * H; sa.nq = nb; sa.nk = nb; sa.D = D; sa.topk = topk;
  sa.idx = block_indices; sa.ldc = static_cast<int>(score_ld(nb));
  sa.scores = static_cast<float*>(rest);
  AttnPlan pa;
  if (rope || q_norm_w) {
    // the attention reads the transformed tensors the pool kernels write (contiguous [B,H,S,D])
    const int64_t cst[3] = {static_cast<int64_t>(H) * S * D, static_cast<int64_t>(S) * D, D};
    rc = attn_plan(pa, q_rot, k_rot, v, block_indices, dtype, B, H, S, D, cst, cst, v_strides, T, Hl, Wl, cT, cH, cW,
                   topk, sm_scale, out, out_strides, sm_reserve);
  } else {
    rc = attn_plan(pa, q, k, v, block_indices, dtype, B, H, S, D, q_strides, k_strides, v_strides, T, Hl, Wl, cT, cH,
                   cW, topk, sm_scale, out, out_strides, sm_reserve);
  }
  if (rc) return rc;
  // ---- launches
  if (route) {
    // the pool kernels also write the routing's split (bf16 pairs, norm bounds) while each pooled row is
    // in registers; the per-head maximum key norm and the fallback count start at 0 before the pool of K
    if (bsa::route_split_targets(rest, B * H, nb, &split_hl, &split_nrm, &split_nkmax,
                                 static_cast<cudaStream_t>(stream)) != BSA_OK)
      return cuda_fail("routing scratch reset");
    pq.a.split_hl = pk.a.split_hl = split_hl;
    pq.a.split_nrm = pk.a.split_nrm = split_nrm;
    pq.a.split_nkmax = pk.a.split_nkmax = split_nkmax;
    pq.a.split_which = 0;
    pk.a.split_which = 1;
    ra.split_done = 1;
  }
  if ((rc = pool_run(pq, stream))) return rc;
  if ((rc = pool_run(pk, stream))) return rc;
  rc = route ? bsa::launch_route(ra, static_cast<cudaStream_t>(stream))
             : bsa::launch_score_topk(sa, static_cast<cudaStream_t>(stream));
  if (rc == BSA_ERR_CUDA) return cuda_fail("routing kernel launch");
  if (rc) return rc == BSA_ERR_ARG ? rc : fail(rc, "routing: unsupported sizes (nb=%d)", nb);
  if (t_phase_event && cudaEventRecord(t_phase_event, static_cast<cudaStream_t>(stream)) != cudaSuccess)
    return cuda_fail("phase event record");
  return attn_run(pa, stream);
}
}  // namespace

extern "C" {

int bsa_forward_ex(const void* q, const void* k, const void* v, int dtype, int B, int H, int S, int D,
                   const int64_t* q_strides, const int64_t* k_strides, const int64_t* v_strides, int T, int Hl,
                   int Wl, int cT, int cH, int cW, int topk, float sm_scale, const float* rope, int rope_dt,
                   int rope_dh, int rope_dw, int rope_T, int rope_H, int rope_W, void* q_rot, void* k_rot,
                   void* scratch, int32_t* block_indices, void* out, const int64_t* out_strides, int sm_reserve,
                   void* stream) {
  return forward_impl(q, k, v, dtype, B, H, S, D, q_strides, k_strides, v_strides, T, Hl, Wl, cT, cH, cW, topk,
                      sm_scale, rope, rope_dt, rope_dh, rope_dw, rope_T, rope_H, rope_W, nullptr, nullptr, 0.f, q_rot,
                      k_rot, scratch, block_indices, out, out_strides, sm_reserve, stream);
}

int bsa_forward_qknorm(const void* q, const void* k, const void* v, int dtype, int B, int H, int S, int D,
                       const int64_t* q_strides, const int64_t* k_strides, const int64_t* v_strides, int T, int Hl,
                       int Wl, int cT, int cH, int cW, int topk, float sm_scale, const float* rope, int rope_dt,
                       int rope_dh, int rope_dw, int rope_T, int rope_H, int rope_W, const void* q_norm_weight,
                       const void* k_norm_weight, float norm_eps, void* q_rot, void* k_rot, void* scratch,
                       int32_t* block_indices, void* out, const int64_t* out_strides, int sm_reserve, void* stream) {
  if (!q_norm_weight || !k_norm_weight) return fail(BSA_ERR_ARG, "null pointer");
  return forward_impl(q, k, v, dtype, B, H, S, D, q_strides, k_strides, v_strides, T, Hl, Wl, cT, cH, cW, topk,
                      sm_scale, rope, rope_dt, rope_dh, rope_dw, rope_T, rope_H, rope_W, q_norm_weight, k_norm_weight,
                      norm_eps, q_rot, k_rot, scratch, block_indices, out, out_strides, sm_reserve, stream);
}

}  // extern "C"
