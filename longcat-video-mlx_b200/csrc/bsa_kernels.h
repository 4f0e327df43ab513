// Internal interface between the C-ABI layer (bsa_capi.cu) and the kernels.
#pragma once
#include <cstdint>
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include "../../include/bsa_b200.h"

namespace bsa {

// ------------------------------------------------------------------ pooling (+ fused RoPE)
struct PoolArgs {
  const void* x;         // [B,H,S,D] with strides sb, sh, ss (elements), d contiguous
  int dtype;             // BSA_DTYPE_*
  int B, H, S, D;
  long long sb, sh, ss;
  int T, Hl, Wl, cT, cH, cW;
  // optional fused 3-D RoPE (rope_3d.py:107-128): per-axis tables, fp32, one entry per pair
  const float* rope;     // nullable: [cos_t | sin_t | cos_h | sin_h | cos_w | sin_w]
  int rope_dt, rope_dh, rope_dw;
  int rope_T, rope_H, rope_W;  // RoPE grid; token s sits at (s / (H*W), (s / W) % H, s % W)
  void* x_rot;           // [B,H,S,D] contiguous, same dtype as x (required when rope != null)
  float* pooled;         // [B*H, nb, D] fp32
  const CUtensorMap* tmap;  // nullable: block map over x (bf16/fp16); selects the TMA-ring kernel
  int map3;                 // tmap is 3-D (d, s, b*h) (contiguous blocks), else 5-D (d, w, h, t, b*h)
  // optional fused RMSNorm_FP32 (blocks.py:55-73) before the RoPE: weight [D] in x's dtype (nullable)
  const void* norm_w;
  float norm_eps;
  // optional fused routing split (the work of the routing's split step, done while the pooled row is in
  // registers): bf16 hi/lo pairs [4][B*H*nb][128], row norm bounds [2][B*H*nb], per-head max key norm
  __nv_bfloat16* split_hl = nullptr;  // nullable
  float* split_nrm = nullptr;
  float* split_nkmax = nullptr;
  int split_which = 0;                // 0: this is Q, 1: this is K
};
int launch_pool(const PoolArgs& a, cudaStream_t stream);

// ------------------------------------------------------------------ block scores + top-k
struct ScoreArgs {
  const float* qp;       // [BH, nq, D] fp32
  const float* kp;       // [BH, nk, D] fp32
  int BH, nq, nk, D, topk;
  int32_t* idx;          // [BH, nq, topk], ascending block ids
  float* scores;         // [BH, nq, ldc] fp32 (output of the score GEMM, input of the top-k)
  int ldc;               // row stride of `scores` (>= nk)
};
int launch_score_topk(const ScoreArgs& a, cudaStream_t stream);
int launch_scores_only(const ScoreArgs& a, cudaStream_t stream);
int launch_topk(const float* scores, int rows, int nk, int ldc, int topk, int32_t* idx, cudaStream_t stream);

// ------------------------------------------------------------------ routing without the score matrix
// (bsa_route.cu): the same indices as launch_score_topk, from tensor-core approximate scores and exact
// fp32 scores for the blocks near each row's threshold.
struct RouteArgs {
  const float* qp;       // [BH, nb, D] fp32
  const float* kp;       // [BH, nb, D] fp32
  int BH, nb, D, topk;
  int32_t* idx;          // [BH, nb, topk], ascending block ids
  void* scratch;         // route_scratch_bytes(BH, nb), 256-byte aligned
  // builds a 3-D bf16 map (d = 128, block = nb, b*h = BH) with 64 x 128 boxes over one pair array
  int (*make_pair_map)(CUtensorMap* m, const void* base, int nb, int BH);
  int split_done = 0;    // the pool kernels already wrote the split (route_split_targets)
};
// Where the split step writes inside the routing scratch; zeroes the per-head max key norm and the
// fallback-row count on `stream` (they must start at 0 before the pool of K runs).
int route_split_targets(void* scratch, int BH, int nb, __nv_bfloat16** hl, float** nrm, float** nkmax,
                        cudaStream_t stream);
bool route_supported(int nb, int D);
int64_t route_scratch_bytes(int BH, int nb);
int launch_route(const RouteArgs& a, cudaStream_t stream);
int route_device_error(int clear);

// ------------------------------------------------------------------ sparse attention
struct AttnArgs {
  const int32_t* idx;
  void* out;
  int B, H, S, D, nb, topk;
  int Hl, Wl, cT, cH, cW;
  long long out_sb, out_sh, out_ss;
  float sm_scale;
  int is_bf16;
  int sm_reserve;  // SMs left free for concurrent kernels (the persistent grid covers the rest)
  int map3;        // the tensor maps are 3-D (d, s, b*h): blocks are contiguous 64-token runs
};
int launch_attn(const CUtensorMap* tm_q, const CUtensorMap* tm_k, const CUtensorMap* tm_v, const AttnArgs& a,
                cudaStream_t stream);
int attn_device_error(int clear);
int score_device_error(int clear);

// Record the calling host thread's error message (read back by bsa_last_error); returns `code`.
int set_error(int code, const char* fmt, ...);

}  // namespace bsa
