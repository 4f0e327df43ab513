// Block routing on sm_100a: block mean-pooling (optionally after fused 3-D RoPE), fp32 block
// scores, and per-row top-k selection.
//
//   pool       : block_sparse_attention.py:67-104 (+ rope_3d.py:107-128 when fused)
//   score      : block_sparse_attention.py:107-112
//   top-k      : block_sparse_attention.py:115-134 with an explicit rule -- the k largest scores,
//                ties to the smaller block id, ids written in ascending order
//
// Both orders of fp32 arithmetic are fixed so that the CPU oracle (oracle/bsa_oracle.c) can
// reproduce every pooled value and score bit for bit:
//   pooling : fold-halves over the n tokens of a block: x[r] + x[r + n/2], recursively, then * 1/n
//   score   : one fma chain per score over d = 0..D-1 (fmaf(q[d], k[d], acc), acc starting at 0)
// The pool kernel is HBM-bound (one read of Q and K); the score kernel is FMA/shared-memory
// bound and keeps each score row on chip for the selection.
#include <algorithm>
#include <cstdint>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include "bsa_kernels.h"

namespace bsa {

__device__ int g_score_err;

// ======================================================================== pooling
namespace pool {
constexpr int kThreads = 256;

template <typename T>
struct Vec8;  // 8 elements = 16 bytes (16-bit types) or 32 bytes (fp32)

__device__ __forceinline__ void load8(const __nv_bfloat16* p, float (&v)[8]) {
  const uint4 u = __ldg(reinterpret_cast<const uint4*>(p));
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    v[2 * i] = __uint_as_float(w[i] << 16);
    v[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
  }
}
__device__ __forceinline__ void load8(const __half* p, float (&v)[8]) {
  const uint4 u = __ldg(reinterpret_cast<const uint4*>(p));
  const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __half22float2(h[i]);
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}
__device__ __forceinline__ void load8(const float* p, float (&v)[8]) {
  const float4 a = __ldg(reinterpret_cast<const float4*>(p));
  const float4 b = __ldg(reinterpret_cast<const float4*>(p) + 1);
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
  v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}

// round an fp32 value to T and back (RoPE output is stored in the input dtype and pooled from there)
__device__ __forceinline__ float round_to(float x, const __nv_bfloat16*) { return __bfloat162float(__float2bfloat16_rn(x)); }
__device__ __forceinline__ float round_to(float x, const __half*) { return __half2float(__float2half_rn(x)); }
__device__ __forceinline__ float round_to(float x, const float*) { return x; }

__device__ __forceinline__ void store8(__nv_bfloat16* p, const float (&v)[8]) {
  uint32_t w[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
    w[i] = *reinterpret_cast<const uint32_t*>(&h);
  }
  *reinterpret_cast<uint4*>(p) = make_uint4(w[0], w[1], w[2], w[3]);
}
__device__ __forceinline__ void store8(__half* p, const float (&v)[8]) {
  uint32_t w[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const __half2 h = __floats2half2_rn(v[2 * i], v[2 * i + 1]);
    w[i] = *reinterpret_cast<const uint32_t*>(&h);
  }
  *reinterpret_cast<uint4*>(p) = make_uint4(w[0], w[1], w[2], w[3]);
}
__device__ __forceinline__ void store8(float* p, const float (&v)[8]) {
  reinterpret_cast<float4*>(p)[0] = make_float4(v[0], v[1], v[2], v[3]);
  reinterpret_cast<float4*>(p)[1] = make_float4(v[4], v[5], v[6], v[7]);
}

struct Geo {
  int B, H, S, D, nb, n;
  long long sb, sh, ss;
  int Hl, Wl, cT, cH, cW, Bh, Bw;
  int tpr, rpp, np;            // threads per token row (D/8), rows per pass, passes (n / rpp)
  const float* rope;
  int rdt, rdh, rdw, rT, rH, rW;
};

// One CTA iteration pools one (b, h, block).  Thread (g, c): row group g < rpp, 8-element chunk
// c < tpr.  It holds rows g, g+rpp, ..., g+(NP-1)*rpp and folds them in registers (token strides
// n/2 .. rpp); the remaining fold levels (strides rpp/2 .. 1) run in place in shared memory.
template <typename T, bool kRope, int NP>
__global__ void __launch_bounds__(kThreads)
    pool_kernel(const T* __restrict__ x, T* xr, float* pooled, Geo g) {
  __shared__ __align__(16) float part[64 * 128];  // [rpp][D] fold partials
  const int tid = threadIdx.x;
  const int grp = tid / g.tpr;
  const int c = tid - grp * g.tpr;
  const bool active = grp < g.rpp;
  const long long total = static_cast<long long>(g.B) * g.H * g.nb;
  const int cHW = g.cH * g.cW;
  const float inv_n = 1.0f / static_cast<float>(g.n);
  for (long long item = blockIdx.x; item < total; item += gridDim.x) {
    const int blk = static_cast<int>(item % g.nb);
    const long long bh = item / g.nb;
    const int b = static_cast<int>(bh / g.H);
    const int h = static_cast<int>(bh - static_cast<long long>(b) * g.H);
    const int per_t = g.Bh * g.Bw;
    const int bt = blk / per_t;
    const int rr = blk - bt * per_t;
    const int bhh = rr / g.Bw;
    const int bw = rr - bhh * g.Bw;
    const int t0 = bt * g.cT, h0 = bhh * g.cH, w0 = bw * g.cW;
    if (active) {
      float acc[NP][8];
      long long toks[NP];
#pragma unroll
      for (int i = 0; i < NP; ++i) {
        const int r = grp + i * g.rpp;  // row inside the block, (ct, ch, cw) order
        const int ct = r / cHW;
        const int rem = r - ct * cHW;
        const int ch = rem / g.cW;
        const int cw = rem - ch * g.cW;
        toks[i] = (static_cast<long long>(t0 + ct) * g.Hl + (h0 + ch)) * g.Wl + (w0 + cw);
        load8(x + b * g.sb + h * g.sh + toks[i] * g.ss + c * 8, acc[i]);
      }
      if (kRope) {
        const int ht = g.rdt >> 1, hh2 = g.rdh >> 1, hw2 = g.rdw >> 1;
        const float* tab_t = g.rope;
        const float* tab_h = tab_t + 2 * g.rT * ht;
        const float* tab_w = tab_h + 2 * g.rH * hh2;
        const int rhw = g.rH * g.rW;
#pragma unroll
        for (int i = 0; i < NP; ++i) {
          // token position on the RoPE grid (t-major flat order, same as the attention layout)
          const long long tok = toks[i];
          const int pt = static_cast<int>(tok / rhw);
          const int prem = static_cast<int>(tok - static_cast<long long>(pt) * rhw);
          const int ph = prem / g.rW;
          const int pw = prem - ph * g.rW;
          // rotate 4 pairs: (x0, x1) -> (x0*cos - x1*sin, x1*cos + x0*sin), fp32, no fma
#pragma unroll
          for (int pr = 0; pr < 4; ++pr) {
            const int d = c * 8 + 2 * pr;
            float cs, sn;
            if (d < g.rdt) {
              const int i2 = d >> 1;
              cs = __ldg(tab_t + pt * ht + i2);
              sn = __ldg(tab_t + g.rT * ht + pt * ht + i2);
            } else if (d < g.rdt + g.rdh) {
              const int i2 = (d - g.rdt) >> 1;
              cs = __ldg(tab_h + ph * hh2 + i2);
              sn = __ldg(tab_h + g.rH * hh2 + ph * hh2 + i2);
            } else {
              const int i2 = (d - g.rdt - g.rdh) >> 1;
              cs = __ldg(tab_w + pw * hw2 + i2);
              sn = __ldg(tab_w + g.rW * hw2 + pw * hw2 + i2);
            }
            const float a = acc[i][2 * pr], bb = acc[i][2 * pr + 1];
            acc[i][2 * pr] = __fadd_rn(__fmul_rn(a, cs), __fmul_rn(-bb, sn));
            acc[i][2 * pr + 1] = __fadd_rn(__fmul_rn(bb, cs), __fmul_rn(a, sn));
          }
#pragma unroll
          for (int e = 0; e < 8; ++e) acc[i][e] = round_to(acc[i][e], x);
          store8(xr + ((static_cast<long long>(b) * g.H + h) * g.S + tok) * g.D + c * 8, acc[i]);
        }
      }
      // register fold levels: rows i and i + half (token strides n/2 .. rpp)
#pragma unroll
      for (int half = NP / 2; half >= 1; half >>= 1) {
#pragma unroll
        for (int i = 0; i < half; ++i)
#pragma unroll
          for (int e = 0; e < 8; ++e) acc[i][e] = __fadd_rn(acc[i][e], acc[i + half][e]);
      }
      *reinterpret_cast<float4*>(&part[grp * g.D + c * 8]) = make_float4(acc[0][0], acc[0][1], acc[0][2], acc[0][3]);
      *reinterpret_cast<float4*>(&part[grp * g.D + c * 8 + 4]) = make_float4(acc[0][4], acc[0][5], acc[0][6], acc[0][7]);
    }
    __syncthreads();
    // shared-memory fold levels (strides rpp/2 .. 1), in place
    for (int half = g.rpp >> 1; half >= 1; half >>= 1) {
      for (int e = tid; e < half * g.D; e += kThreads) part[e] = __fadd_rn(part[e], part[e + half * g.D]);
      __syncthreads();
    }
    if (tid < g.D) pooled[(bh * g.nb + blk) * g.D + tid] = __fmul_rn(part[tid], inv_n);
    __syncthreads();
  }
}
}  // namespace pool

int launch_pool(const PoolArgs& a, cudaStream_t stream) {
  using namespace pool;
  const int n = a.cT * a.cH * a.cW;
  pool::Geo g;
  g.B = a.B; g.H = a.H; g.S = a.S; g.D = a.D; g.nb = a.S / n; g.n = n;
  g.sb = a.sb; g.sh = a.sh; g.ss = a.ss;
  g.Hl = a.Hl; g.Wl = a.Wl; g.cT = a.cT; g.cH = a.cH; g.cW = a.cW;
  g.Bh = a.Hl / a.cH; g.Bw = a.Wl / a.cW;
  g.tpr = a.D / 8;
  int rpp = 1;
  while (rpp * 2 <= kThreads / g.tpr && rpp * 2 <= n) rpp *= 2;
  g.rpp = rpp;
  g.np = n / rpp;
  g.rope = a.rope; g.rdt = a.rope_dt; g.rdh = a.rope_dh; g.rdw = a.rope_dw;
  g.rT = a.rope_T; g.rH = a.rope_H; g.rW = a.rope_W;
  if (g.np > 4 || g.np * g.rpp != n) return BSA_ERR_SHAPE;
  int dev = 0, sms = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const long long total = static_cast<long long>(a.B) * a.H * g.nb;
  long long grid = static_cast<long long>(sms) * 6;
  if (grid > total) grid = total;
  if (grid < 1) return BSA_OK;
  dim3 gd(static_cast<unsigned>(grid), 1, 1);
  const bool rope = a.rope != nullptr;
#define BSA_POOL_LAUNCH_NP(TT, NP)                                                                                 \
  do {                                                                                                             \
    if (rope)                                                                                                      \
      pool_kernel<TT, true, NP><<<gd, kThreads, 0, stream>>>(static_cast<const TT*>(a.x), static_cast<TT*>(a.x_rot), \
                                                             a.pooled, g);                                         \
    else                                                                                                           \
      pool_kernel<TT, false, NP><<<gd, kThreads, 0, stream>>>(static_cast<const TT*>(a.x), nullptr, a.pooled, g);    \
  } while (0)
#define BSA_POOL_LAUNCH(TT)                        \
  do {                                             \
    if (g.np == 1) BSA_POOL_LAUNCH_NP(TT, 1);      \
    else if (g.np == 2) BSA_POOL_LAUNCH_NP(TT, 2); \
    else BSA_POOL_LAUNCH_NP(TT, 4);                \
  } while (0)
  if (a.dtype == BSA_DTYPE_BF16) BSA_POOL_LAUNCH(__nv_bfloat16);
  else if (a.dtype == BSA_DTYPE_F16) BSA_POOL_LAUNCH(__half);
  else if (a.dtype == BSA_DTYPE_F32) BSA_POOL_LAUNCH(float);
  else return BSA_ERR_DTYPE;
#undef BSA_POOL_LAUNCH_NP
#undef BSA_POOL_LAUNCH
  return cudaGetLastError() == cudaSuccess ? BSA_OK : BSA_ERR_CUDA;
}

// ======================================================================== scores + top-k
namespace score {
constexpr int kThreads = 256;
constexpr int kJT = 64;          // key blocks per shared-memory chunk
constexpr int kMaxD = 128;

__device__ __forceinline__ uint32_t ordered_key(float s) {
  // -0.0 and +0.0 are one score; NaN sorts below everything
  if (s != s) return 0u;
  const uint32_t u = __float_as_uint(s == 0.0f ? 0.0f : s);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

struct Args {
  const float* sin;  // when set: select from these scores [BH, nq, nk] instead of computing them
  const float* qp;
  const float* kp;
  int BH, nq, nk, D, topk, QT;
  int32_t* idx;
  float* scores;
  int select;  // 0: write scores only
};

// smem: [QT][nk] scores | union{ qT[D][QT] + kT[D][kJT] , per-warp histograms 8 x 256 }
__global__ void __launch_bounds__(kThreads) score_topk_kernel(Args a) {
  extern __shared__ __align__(16) float sm[];
  float* srow = sm;                                             // QT * nk
  float* qT = sm + static_cast<size_t>(a.QT) * a.nk;            // D * QT
  float* kT = qT + kMaxD * a.QT;                                // D * kJT
  uint32_t* hist = reinterpret_cast<uint32_t*>(qT);             // 8 * 256 (after scoring)
  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const int tiles_per_head = (a.nq + a.QT - 1) / a.QT;
  const int bh = blockIdx.x / tiles_per_head;
  const int q0 = (blockIdx.x - bh * tiles_per_head) * a.QT;
  const int qn = min(a.QT, a.nq - q0);
  const float* qp = a.qp + (static_cast<long long>(bh) * a.nq + q0) * a.D;
  const float* kp = a.kp + static_cast<long long>(bh) * a.nk * a.D;
  if (a.sin) {
    for (int e = tid; e < qn * a.nk; e += kThreads) {
      const int i = e / a.nk, j = e - i * a.nk;
      srow[static_cast<size_t>(i) * a.nk + j] = a.sin[(static_cast<long long>(bh) * a.nq + q0 + i) * a.nk + j];
    }
  } else {
    // ---- stage the q tile transposed: qT[d][i ^ qswz(d)] (coalesced float4 reads; the XOR
    //      keeps groups of 4 queries contiguous and spreads the transposed stores over banks)
    const int D4 = a.D >> 2;
    const int qmask = (a.QT >> 2) - 1;
    for (int e = tid; e < a.QT * D4; e += kThreads) {
      const int i = e / D4, d4 = e - i * D4;
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
      if (i < qn) v = __ldg(reinterpret_cast<const float4*>(qp + static_cast<long long>(i) * a.D) + d4);
      const int col = i ^ ((d4 & qmask) << 2);
      qT[(4 * d4 + 0) * a.QT + col] = v.x;
      qT[(4 * d4 + 1) * a.QT + col] = v.y;
      qT[(4 * d4 + 2) * a.QT + col] = v.z;
      qT[(4 * d4 + 3) * a.QT + col] = v.w;
    }
    // thread tile: 4 query rows x 2 key blocks
    const int ngroups = a.QT / 4;
    const int qg = tid / 32;         // query group (4 rows)
    const int jp = tid & 31;         // key pair inside the chunk
    const bool active = qg < ngroups;
    for (int j0 = 0; j0 < a.nk; j0 += kJT) {
      const int jn = min(kJT, a.nk - j0);
      __syncthreads();
      // kT[d][j ^ kswz(d)], kswz even so key pairs (2p, 2p+1) stay contiguous
      for (int e = tid; e < kJT * D4; e += kThreads) {
        const int j = e / D4, d4 = e - j * D4;
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if (j < jn) v = __ldg(reinterpret_cast<const float4*>(kp + static_cast<long long>(j0 + j) * a.D) + d4);
        const int col = j ^ ((d4 & 15) << 1);
        kT[(4 * d4 + 0) * kJT + col] = v.x;
        kT[(4 * d4 + 1) * kJT + col] = v.y;
        kT[(4 * d4 + 2) * kJT + col] = v.z;
        kT[(4 * d4 + 3) * kJT + col] = v.w;
      }
      __syncthreads();
      if (active) {
        float acc[4][2];
  #pragma unroll
        for (int i = 0; i < 4; ++i) acc[i][0] = acc[i][1] = 0.f;
  #pragma unroll 8
        for (int d = 0; d < a.D; ++d) {
          const int d4 = d >> 2;
          const float4 qv = *reinterpret_cast<const float4*>(qT + d * a.QT + ((qg * 4) ^ ((d4 & qmask) << 2)));
          const float2 kv = *reinterpret_cast<const float2*>(kT + d * kJT + ((jp * 2) ^ ((d4 & 15) << 1)));
          acc[0][0] = __fmaf_rn(qv.x, kv.x, acc[0][0]);
          acc[0][1] = __fmaf_rn(qv.x, kv.y, acc[0][1]);
          acc[1][0] = __fmaf_rn(qv.y, kv.x, acc[1][0]);
          acc[1][1] = __fmaf_rn(qv.y, kv.y, acc[1][1]);
          acc[2][0] = __fmaf_rn(qv.z, kv.x, acc[2][0]);
          acc[2][1] = __fmaf_rn(qv.z, kv.y, acc[2][1]);
          acc[3][0] = __fmaf_rn(qv.w, kv.x, acc[3][0]);
          acc[3][1] = __fmaf_rn(qv.w, kv.y, acc[3][1]);
        }
  #pragma unroll
        for (int i = 0; i < 4; ++i)
  #pragma unroll
          for (int jj = 0; jj < 2; ++jj) {
            const int j = jp * 2 + jj;
            if (j < jn) srow[static_cast<size_t>(qg * 4 + i) * a.nk + j0 + j] = acc[i][jj];
          }
      }
    }
  }
  __syncthreads();
  if (a.scores) {
    for (int e = tid; e < qn * a.nk; e += kThreads) {
      const int i = e / a.nk, j = e - i * a.nk;
      a.scores[(static_cast<long long>(bh) * a.nq + q0 + i) * a.nk + j] = srow[static_cast<size_t>(i) * a.nk + j];
    }
  }
  if (!a.select) return;
  // ---- top-k per row: radix select on ordered keys (4 x 8-bit digits), one warp per row
  uint32_t* h = hist + warp * 256;
  const uint32_t lt_mask = (1u << lane) - 1u;
  for (int i = warp; i < qn; i += kThreads / 32) {
    const float* row = srow + static_cast<size_t>(i) * a.nk;
    uint32_t prefix = 0, pmask = 0;
    int need = a.topk;  // keys still to take among those matching prefix
#pragma unroll 1
    for (int shift = 24; shift >= 0; shift -= 8) {
#pragma unroll
      for (int e = 0; e < 8; ++e) h[lane * 8 + e] = 0;
      __syncwarp();
      for (int j = lane; j < a.nk; j += 32) {
        const uint32_t u = ordered_key(row[j]);
        if ((u & pmask) == prefix) atomicAdd(&h[(u >> shift) & 255u], 1u);
      }
      __syncwarp();
      // lane L owns digits 8L .. 8L+7; suffix sums from the top digit down
      uint32_t cnt[8];
      uint32_t tot = 0;
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        cnt[e] = h[lane * 8 + e];
        tot += cnt[e];
      }
      // inclusive suffix scan over lanes (lanes above contribute)
      uint32_t suf = tot;
#pragma unroll
      for (int off = 1; off < 32; off <<= 1) {
        const uint32_t v = __shfl_down_sync(0xffffffffu, suf, off);
        if (lane + off < 32) suf += v;
      }
      const uint32_t above = suf - tot;  // keys with digit in lanes > L
      // the digit lane: above < need <= suf
      const bool mine = above < static_cast<uint32_t>(need) && static_cast<uint32_t>(need) <= suf;
      int digit = 0;
      uint32_t gt = 0;
      if (mine) {
        uint32_t run = above;
#pragma unroll
        for (int e = 7; e >= 0; --e) {
          if (run + cnt[e] >= static_cast<uint32_t>(need)) {
            digit = lane * 8 + e;
            gt = run;
            break;
          }
          run += cnt[e];
        }
      }
      const uint32_t ball = __ballot_sync(0xffffffffu, mine);
      const int src = __ffs(ball) - 1;
      digit = __shfl_sync(0xffffffffu, digit, src);
      gt = __shfl_sync(0xffffffffu, gt, src);
      prefix |= static_cast<uint32_t>(digit) << shift;
      pmask |= 255u << shift;
      need -= static_cast<int>(gt);
      __syncwarp();
    }
    // prefix is now the key of the k-th largest score; take every key above it and the first
    // `need` keys equal to it in ascending block order
    int32_t* out = a.idx + (static_cast<long long>(bh) * a.nq + q0 + i) * a.topk;
    int taken = 0, ties = 0;
    for (int j0 = 0; j0 < a.nk; j0 += 32) {
      const int j = j0 + lane;
      const uint32_t u = j < a.nk ? ordered_key(row[j]) : 0u;
      const bool valid = j < a.nk;
      const bool eq = valid && u == prefix;
      const uint32_t eqb = __ballot_sync(0xffffffffu, eq);
      const int rank = ties + __popc(eqb & lt_mask);
      const bool sel = valid && (u > prefix || (eq && rank < need));
      const uint32_t sb = __ballot_sync(0xffffffffu, sel);
      if (sel) out[taken + __popc(sb & lt_mask)] = j;
      taken += __popc(sb);
      ties += __popc(eqb);
    }
    if (lane == 0 && taken != a.topk) atomicCAS(&g_score_err, 0, 201);
  }
}

int pick_qt(int nk, int nq) {
  const int budget = 232448 - 2048;
  int qt = 32;
  while (qt > 4) {
    const size_t bytes = static_cast<size_t>(qt) * nk * 4 + static_cast<size_t>(kMaxD) * (qt + kJT) * 4;
    if (bytes <= static_cast<size_t>(budget)) break;
    qt >>= 1;
  }
  (void)nq;
  return qt;
}

int launch(const ScoreArgs& s, int select, cudaStream_t stream) {
  Args a;
  const int nq = s.nq;
  a.sin = s.scores_in;
  a.qp = s.qp; a.kp = s.kp; a.BH = s.BH; a.nq = nq; a.nk = s.nk; a.D = s.D; a.topk = s.topk;
  a.idx = s.idx; a.scores = s.scores; a.select = select;
  if (!s.scores_in && (s.D > kMaxD || s.D < 1)) return BSA_ERR_SHAPE;
  a.QT = pick_qt(a.nk, nq);
  const size_t smem = static_cast<size_t>(a.QT) * a.nk * 4 +
                      std::max(static_cast<size_t>(kMaxD) * (a.QT + kJT) * 4, static_cast<size_t>(8 * 256 * 4));
  if (smem > 232448 - 1024) return BSA_ERR_SHAPE;
  static bool configured[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !configured[dev]) {
    if (cudaFuncSetAttribute(score_topk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 232448 - 1024) !=
        cudaSuccess)
      return BSA_ERR_CUDA;
    configured[dev] = true;
  }
  const int tiles = (nq + a.QT - 1) / a.QT;
  const long long grid = static_cast<long long>(s.BH) * tiles;
  if (grid < 1) return BSA_OK;
  score_topk_kernel<<<static_cast<unsigned>(grid), kThreads, smem, stream>>>(a);
  return cudaGetLastError() == cudaSuccess ? BSA_OK : BSA_ERR_CUDA;
}
}  // namespace score

int launch_score_topk(const ScoreArgs& a, cudaStream_t stream) { return score::launch(a, 1, stream); }

int launch_scores_only(const ScoreArgs& a, cudaStream_t stream) { return score::launch(a, 0, stream); }

int score_device_error(int clear) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_score_err, sizeof(int)) != cudaSuccess) return BSA_ERR_CUDA;
  if (clear && v) {
    int z = 0;
    cudaMemcpyToSymbol(g_score_err, &z, sizeof(int));
  }
  return v;
}

}  // namespace bsa
