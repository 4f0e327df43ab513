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
//   pooling : pairwise tree over the n tokens of a block in token order ((r0 + r1) + (r2 + r3)) + ...,
//             then * 1/n
//   score   : one fma chain per score over d = 0..D-1 (fmaf(q[d], k[d], acc), acc starting at 0)
// Pooling is HBM-bound (one read of Q and K; bf16/fp16 blocks stream through a TMA ring). The score
// kernel is FMA-bound and writes the score matrix to the caller's scratch. The top-k kernel reads it
// back one row per warp.
#include <algorithm>
#include <cstdint>
#include <mutex>
#include <type_traits>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include "bsa_kernels.h"
#include "bsa_ptx.cuh"
#include "bsa_select.cuh"

namespace bsa {

__device__ int g_score_err;

// ======================================================================== pooling
namespace pool {
constexpr int kThreads = 256;

// round an fp32 value to T and back (RoPE output is stored in the input dtype and pooled from there)
__device__ __forceinline__ float round_to(float x, const __nv_bfloat16*) { return __bfloat162float(__float2bfloat16_rn(x)); }
__device__ __forceinline__ float round_to(float x, const __half*) { return __half2float(__float2half_rn(x)); }
__device__ __forceinline__ float round_to(float x, const float*) { return x; }

struct Geo {
  int B, H, S, D, nb, n;
  long long sb, sh, ss;
  int Hl, Wl, cT, cH, cW, Bh, Bw;
  const float* rope;
  int rdt, rdh, rdw, rT, rH, rW;
  int map3;  // the TMA-ring kernel's map is 3-D (d, s, b*h): blocks are contiguous token runs
  const void* nw;  // nullable: RMSNorm weight [D] in the input dtype (fused q/k norm)
  float eps;
  __nv_bfloat16* hl;  // nullable: fused routing split (see split_row)
  float* nrm;
  float* nkmax;
  int which;          // 0: Q, 1: K
};

// The routing's split step for one pooled row, done while the row is in registers (route::split_kernel in
// bsa_route.cu does the same from memory when the pool kernels do not): bf16 pairs hi = bf16(x),
// lo = bf16(x - hi) padded to 128 columns, an upper bound of the row's l2 norm (+inf for values the
// routing's error bound does not cover: non-finite, above 2^60 or below 2^-60 in magnitude), and for K the
// per-head maximum of those bounds.  One warp per row; lane l holds d = 4l .. 4l+3 (zeros past D).
__device__ __forceinline__ void split_row(const Geo& g, int bh, int blk, const float (&x)[4], int lane) {
  const long long rows = static_cast<long long>(g.B) * g.H * g.nb;
  const long long row = static_cast<long long>(bh) * g.nb + blk;
  __nv_bfloat16 hi[4], lo[4];
  float n2 = 0.f;
  bool extreme = false;
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    hi[e] = __float2bfloat16_rn(x[e]);
    lo[e] = __float2bfloat16_rn(__fsub_rn(x[e], __bfloat162float(hi[e])));
    n2 = fmaf(x[e], x[e], n2);
    const float a = fabsf(x[e]);
    extreme |= !(a <= 1.152921504606847e18f) || (a != 0.f && a < 8.673617379884035e-19f);  // 2^60, 2^-60
  }
  __nv_bfloat16* dh = g.hl + (static_cast<long long>(2 * g.which) * rows + row) * 128 + 4 * lane;
  __nv_bfloat16* dl = g.hl + (static_cast<long long>(2 * g.which + 1) * rows + row) * 128 + 4 * lane;
  *reinterpret_cast<uint2*>(dh) = *reinterpret_cast<const uint2*>(hi);
  *reinterpret_cast<uint2*>(dl) = *reinterpret_cast<const uint2*>(lo);
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) n2 += __shfl_xor_sync(0xffffffffu, n2, off);
  extreme = __any_sync(0xffffffffu, extreme);
  if (lane == 0) {
    // sqrt of an fp32 sum of 128 squares: relative error far below 2^-10, so the bound holds
    const float n = extreme ? INFINITY : __fmul_ru(sqrtf(n2), 1.0009765625f);
    g.nrm[static_cast<long long>(g.which) * rows + row] = n;
    if (g.which) atomicMax(reinterpret_cast<int*>(g.nkmax) + bh, __float_as_int(n));  // n >= 0
  }
}

// Four consecutive d values of one token row: 8 bytes (fp16/bf16) or 16 bytes (fp32).
__device__ __forceinline__ void load4(const __nv_bfloat16* p, float (&v)[4]) {
  const uint2 u = __ldg(reinterpret_cast<const uint2*>(p));
  v[0] = __uint_as_float(u.x << 16);
  v[1] = __uint_as_float(u.x & 0xffff0000u);
  v[2] = __uint_as_float(u.y << 16);
  v[3] = __uint_as_float(u.y & 0xffff0000u);
}
__device__ __forceinline__ void load4(const __half* p, float (&v)[4]) {
  const uint2 u = __ldg(reinterpret_cast<const uint2*>(p));
  const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&u.x));
  const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&u.y));
  v[0] = a.x; v[1] = a.y; v[2] = b.x; v[3] = b.y;
}
__device__ __forceinline__ void load4(const float* p, float (&v)[4]) {
  const float4 a = __ldg(reinterpret_cast<const float4*>(p));
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
}
__device__ __forceinline__ void store4(__nv_bfloat16* p, const float (&v)[4]) {
  const __nv_bfloat162 a = __floats2bfloat162_rn(v[0], v[1]);
  const __nv_bfloat162 b = __floats2bfloat162_rn(v[2], v[3]);
  *reinterpret_cast<uint2*>(p) = make_uint2(*reinterpret_cast<const uint32_t*>(&a), *reinterpret_cast<const uint32_t*>(&b));
}
__device__ __forceinline__ void store4(__half* p, const float (&v)[4]) {
  const __half2 a = __floats2half2_rn(v[0], v[1]);
  const __half2 b = __floats2half2_rn(v[2], v[3]);
  *reinterpret_cast<uint2*>(p) = make_uint2(*reinterpret_cast<const uint32_t*>(&a), *reinterpret_cast<const uint32_t*>(&b));
}
__device__ __forceinline__ void store4(float* p, const float (&v)[4]) {
  *reinterpret_cast<float4*>(p) = make_float4(v[0], v[1], v[2], v[3]);
}

// One warp pools one (b, h, block) at a time; lane l holds d values 4l .. 4l+3 of every row.
// Rows are read in token order, 8 at a time (all 8 loads in flight before the first is used), and
// summed as a pairwise tree over adjacent rows: (r0 + r1), (r2 + r3), then ((r0+r1) + (r2+r3)), ...
// kept as a binary counter of partial sums (level L holds the sum of the last complete run of 2^L
// rows), so the order is fixed and needs no shared memory or barrier.  Each row's token offset
// inside a block is the same for every block and is tabled once per CTA.
template <typename T, bool kRope>
__global__ void __launch_bounds__(kThreads, kRope ? 2 : 4)
    pool_kernel(const T* __restrict__ x, T* xr, float* pooled, Geo g) {
  __shared__ long long roff[64];  // token offset of row r from the block's first token, (ct, ch, cw) order
  const int tid = threadIdx.x;
  if (tid < g.n) {
    const int cHW = g.cH * g.cW;
    const int ct = tid / cHW;
    const int rem = tid - ct * cHW;
    const int ch = rem / g.cW;
    const int cw = rem - ch * g.cW;
    roff[tid] = (static_cast<long long>(ct) * g.Hl + ch) * g.Wl + cw;
  }
  __syncthreads();
  const int lane = tid & 31;
  const int d0 = lane * 4;
  const bool dact = d0 < g.D;
  const int total = g.B * g.H * g.nb;
  const int per_t = g.Bh * g.Bw;
  const float inv_n = 1.0f / static_cast<float>(g.n);
  const int nwarps = gridDim.x * (kThreads / 32);
  // RoPE: each of this lane's two pairs reads one axis table (t, h or w) at a fixed column
  const float* rcos[2] = {nullptr, nullptr};
  const float* rsin[2] = {nullptr, nullptr};
  int rstride[2] = {0, 0}, rax[2] = {0, 0};
  if (kRope && g.rope) {
    const int ht = g.rdt >> 1, hh2 = g.rdh >> 1, hw2 = g.rdw >> 1;
    const float* tab_t = g.rope;
    const float* tab_h = tab_t + 2 * g.rT * ht;
    const float* tab_w = tab_h + 2 * g.rH * hh2;
#pragma unroll
    for (int pr = 0; pr < 2; ++pr) {
      const int d = d0 + 2 * pr;
      if (d < g.rdt) {
        rax[pr] = 0; rstride[pr] = ht; rcos[pr] = tab_t + (d >> 1); rsin[pr] = rcos[pr] + g.rT * ht;
      } else if (d < g.rdt + g.rdh) {
        rax[pr] = 1; rstride[pr] = hh2; rcos[pr] = tab_h + ((d - g.rdt) >> 1); rsin[pr] = rcos[pr] + g.rH * hh2;
      } else {
        rax[pr] = 2; rstride[pr] = hw2; rcos[pr] = tab_w + ((d - g.rdt - g.rdh) >> 1); rsin[pr] = rcos[pr] + g.rW * hw2;
      }
    }
  }
  for (int item = blockIdx.x * (kThreads / 32) + (tid >> 5); item < total; item += nwarps) {
    const int blk = item % g.nb;
    const int bh = item / g.nb;
    const int b = bh / g.H;
    const int h = bh - b * g.H;
    const int bt = blk / per_t;
    const int rr = blk - bt * per_t;
    const int bhh = rr / g.Bw;
    const int bw = rr - bhh * g.Bw;
    const long long tok0 = (static_cast<long long>(bt * g.cT) * g.Hl + bhh * g.cH) * g.Wl + bw * g.cW;
    const T* base = x + b * g.sb + h * g.sh + d0;
    // RoPE grid positions of rows `lane` and `lane + 32` (token s at t = s / (H*W), h = (s / W) % H,
    // w = s % W), packed as (t) and (h << 16 | w) and handed to the other lanes by shuffle
    int posA0 = 0, posB0 = 0, posA1 = 0, posB1 = 0;
    if (kRope && g.rope) {
      const int rhw = g.rH * g.rW;
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {
        const int r = lane + 32 * hf;
        if (r < g.n) {
          const long long tok = tok0 + roff[r];
          const int pt = static_cast<int>(tok / rhw);
          const int prem = static_cast<int>(tok - static_cast<long long>(pt) * rhw);
          const int ph = prem / g.rW;
          const int pw = prem - ph * g.rW;
          if (hf == 0) { posA0 = pt; posB0 = (ph << 16) | pw; }
          else { posA1 = pt; posB1 = (ph << 16) | pw; }
        }
      }
    }
    float lvl[7][4];  // partial sums by tree level
    float tot[4] = {0.f, 0.f, 0.f, 0.f};
    for (int r0 = 0; r0 < g.n; r0 += 8) {
      float v[8][4];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        if (r0 + i < g.n && dact) load4(base + (tok0 + roff[r0 + i]) * g.ss, v[i]);
        else v[i][0] = v[i][1] = v[i][2] = v[i][3] = 0.f;
      }
      // this group's RoPE table entries, all loads issued before the first use (one latency per 8 rows)
      float rc[8][2], rsn[8][2];
      if (kRope && g.rope) {
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int r = r0 + i;
          // this row's position on the RoPE grid, computed by lane r % 32 at the start of the block
          const int src = r & 31;
          const int pt = __shfl_sync(0xffffffffu, r < 32 ? posA0 : posA1, src);
          const int pb = __shfl_sync(0xffffffffu, r < 32 ? posB0 : posB1, src);
          const int pax[3] = {pt, pb >> 16, pb & 0xffff};
#pragma unroll
          for (int pr = 0; pr < 2; ++pr) {
            const int pos = pax[rax[pr]];
            const bool live = dact && r < g.n;
            rc[i][pr] = live ? __ldg(rcos[pr] + pos * rstride[pr]) : 0.f;
            rsn[i][pr] = live ? __ldg(rsin[pr] + pos * rstride[pr]) : 0.f;
          }
        }
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int r = r0 + i;
        if (r >= g.n) break;
        if (kRope) {
          // the row's transform, written to x_rot and pooled from there: optional RMSNorm_FP32
          // (blocks.py:55-73), then optional 3-D RoPE (rope_3d.py:120-128)
          if (g.nw) {
            // fp32 mean of squares: each lane ((v0^2 + v1^2) + (v2^2 + v3^2)), then a butterfly over
            // the lanes (every lane ends with the same sum); lanes past D hold zeros
            float ss = __fadd_rn(__fadd_rn(__fmul_rn(v[i][0], v[i][0]), __fmul_rn(v[i][1], v[i][1])),
                                 __fadd_rn(__fmul_rn(v[i][2], v[i][2]), __fmul_rn(v[i][3], v[i][3])));
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) ss = __fadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, off));
            const float rs = rsqrtf(__fadd_rn(__fdiv_rn(ss, static_cast<float>(g.D)), g.eps));
            if (dact) {
              float wv[4];
              load4(static_cast<const T*>(g.nw) + d0, wv);
              // x * rsqrt in fp32, cast to the input dtype, times the weight in the input dtype
#pragma unroll
              for (int e = 0; e < 4; ++e) v[i][e] = round_to(__fmul_rn(round_to(__fmul_rn(v[i][e], rs), x), wv[e]), x);
            }
          }
          if (g.rope) {
            if (dact) {
              // rotate 2 pairs: (x0, x1) -> (x0*cos - x1*sin, x1*cos + x0*sin), fp32, no fma
#pragma unroll
              for (int pr = 0; pr < 2; ++pr) {
                const float cs = rc[i][pr];
                const float sn = rsn[i][pr];
                const float a = v[i][2 * pr], bb = v[i][2 * pr + 1];
                v[i][2 * pr] = __fadd_rn(__fmul_rn(a, cs), __fmul_rn(-bb, sn));
                v[i][2 * pr + 1] = __fadd_rn(__fmul_rn(bb, cs), __fmul_rn(a, sn));
              }
#pragma unroll
              for (int e = 0; e < 4; ++e) v[i][e] = round_to(v[i][e], x);
            }
          }
          if (dact) store4(xr + (static_cast<long long>(bh) * g.S + tok0 + roff[r]) * g.D + d0, v[i]);
        }
        // insert row r into the binary counter: merge with every complete run that ends at r
        float c[4] = {v[i][0], v[i][1], v[i][2], v[i][3]};
#pragma unroll
        for (int L = 0; L < 7; ++L) {
          if (((r >> L) & 1) == 0) {
#pragma unroll
            for (int e = 0; e < 4; ++e) lvl[L][e] = c[e];
            break;
          }
#pragma unroll
          for (int e = 0; e < 4; ++e) c[e] = __fadd_rn(lvl[L][e], c[e]);
          if (r + 1 == g.n && (1 << (L + 1)) == g.n) {
#pragma unroll
            for (int e = 0; e < 4; ++e) tot[e] = c[e];
          }
        }
      }
    }
    if (g.n == 1) {
#pragma unroll
      for (int e = 0; e < 4; ++e) tot[e] = lvl[0][e];
    }
    const float out[4] = {dact ? __fmul_rn(tot[0], inv_n) : 0.f, dact ? __fmul_rn(tot[1], inv_n) : 0.f,
                          dact ? __fmul_rn(tot[2], inv_n) : 0.f, dact ? __fmul_rn(tot[3], inv_n) : 0.f};
    if (dact) store4(pooled + (static_cast<long long>(bh) * g.nb + blk) * g.D + d0, out);
    if (g.hl) split_row(g, bh, blk, out, lane);
  }
}
// ------------------------------------------------------------------------ pooling through a TMA ring
// The same pooling (without RoPE) for bf16/fp16 inputs, with the blocks streamed into shared memory by
// TMA: one producer lane keeps up to kRing blocks (16 KB each) in flight per SM, and kConsumers warps
// reduce them.  Row order and the fp32 pairwise tree are those of pool_kernel, so results are identical.
//
// Consumer warp c takes the CTA's blocks c, c + kConsumers, ... and owns slots 2c and 2c + 1, which it
// uses alternately: every full/empty phase of a slot is then produced and consumed in order by one
// producer and one consumer.  (Round-robin blocks over a shared ring let a consumer reach its wait
// before the slot's previous block had landed -- TMA loads may complete out of issue order -- and a
// parity wait one phase ahead of its barrier reads the phase before as complete.)
constexpr int kConsumers = 6;
constexpr int kSlotsPerConsumer = 2;
constexpr int kTmaThreads = 32 * (kConsumers + 1);
constexpr int kRing = kConsumers * kSlotsPerConsumer;
constexpr int kSlotBytes = 16384;  // two 8 KB d-halves of up to 64 rows x 128 B, 128B-swizzled
struct RingSmem {
  uint64_t full[kRing];
  uint64_t empty[kRing];
  int abort_flag;
};
constexpr int kTmaSmemBytes = 1024 + kRing * kSlotBytes + static_cast<int>(sizeof(RingSmem));

// Four consecutive d values (lane's d0 .. d0+3) of row r from a 128B-swizzled block slot.
template <typename T>
__device__ __forceinline__ void slot_load4(const uint8_t* slot, int r, int lane, float (&v)[4]) {
  const uint8_t* p = slot + (lane >> 4) * 8192 + sw128_offset(static_cast<uint32_t>(r), (lane & 15) >> 1) + 8 * (lane & 1);
  const uint2 u = *reinterpret_cast<const uint2*>(p);
  if constexpr (sizeof(T) == 2 && std::is_same<T, __nv_bfloat16>::value) {
    v[0] = __uint_as_float(u.x << 16);
    v[1] = __uint_as_float(u.x & 0xffff0000u);
    v[2] = __uint_as_float(u.y << 16);
    v[3] = __uint_as_float(u.y & 0xffff0000u);
  } else {
    const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&u.x));
    const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&u.y));
    v[0] = a.x; v[1] = a.y; v[2] = b.x; v[3] = b.y;
  }
}

template <typename T>
__global__ void __launch_bounds__(kTmaThreads, 1)
    pool_tma_kernel(const __grid_constant__ CUtensorMap tm, float* pooled, Geo g) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* ring = smem_raw + ((1024u - (static_cast<uint32_t>(__cvta_generic_to_shared(smem_raw)) & 1023u)) & 1023u);
  RingSmem& rs = *reinterpret_cast<RingSmem*>(ring + kRing * kSlotBytes);
  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  if (tid == 0) {
    for (int i = 0; i < kRing; ++i) {
      mbar_init(&rs.full[i], 1);
      mbar_init(&rs.empty[i], 1);
    }
    rs.abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();
  volatile int* abort_flag = &rs.abort_flag;
  const int total = g.B * g.H * g.nb;
  const int per_t = g.Bh * g.Bw;
  const int G = gridDim.x;
  const int cnt = total > static_cast<int>(blockIdx.x) ? (total - 1 - static_cast<int>(blockIdx.x)) / G + 1 : 0;
  const uint32_t box_bytes = static_cast<uint32_t>(g.n) * 128u;
  if (warp == kConsumers) {
    // ---------------------------------------------------------------- producer
    if (lane == 0) {
      prefetch_tmap(&tm);
      int i = 0;
      for (; i < cnt; ++i) {
        // block i -> consumer i % kConsumers, its (i / kConsumers)-th block, slot 2c + (m & 1), fill m / 2
        const int m = i / kConsumers;
        const int slot = (i - m * kConsumers) * kSlotsPerConsumer + (m & 1);
        const int fill = m >> 1;
        if (fill >= 1 &&
            !mbar_wait(&rs.empty[slot], static_cast<uint32_t>((fill - 1) & 1), abort_flag, &g_score_err, 301))
          break;
        const int item = static_cast<int>(blockIdx.x) + i * G;
        const int blk = item % g.nb;
        const int bh = item / g.nb;
        const int bt = blk / per_t;
        const int rr = blk - bt * per_t;
        const int bhh = rr / g.Bw;
        const int bw = rr - bhh * g.Bw;
        uint8_t* dst = ring + slot * kSlotBytes;
        mbar_arrive_expect_tx(&rs.full[slot], 2u * box_bytes);
        if (g.map3) {  // contiguous blocks: token blk * n of the (d, s, b*h) map
          tma_load_3d(dst, &tm, &rs.full[slot], 0, blk * g.n, bh);
          tma_load_3d(dst + 8192, &tm, &rs.full[slot], 64, blk * g.n, bh);
        } else {
          tma_load_5d(dst, &tm, &rs.full[slot], 0, bw * g.cW, bhh * g.cH, bt * g.cT, bh);
          tma_load_5d(dst + 8192, &tm, &rs.full[slot], 64, bw * g.cW, bhh * g.cH, bt * g.cT, bh);
        }
      }
      // teardown: no TMA write into this CTA's shared memory may still be in flight.  The last block
      // issued into each slot is its latest fill; its phase is the newest one of that barrier.
      const uint64_t t0 = globaltimer_ns();
      for (int j = (i > kRing ? i - kRing : 0); j < i; ++j) {
        const int m = j / kConsumers;
        const int slot = (j - m * kConsumers) * kSlotsPerConsumer + (m & 1);
        while (!mbar_try_wait(&rs.full[slot], static_cast<uint32_t>((m >> 1) & 1)) &&
               globaltimer_ns() - t0 < kWaitLimitNs) {
        }
      }
    }
    __syncwarp();
  } else {
    // ---------------------------------------------------------------- consumers: warp c takes blocks c, c+6, ...
    const int d0 = lane * 4;
    const bool dact = d0 < g.D;
    const float inv_n = 1.0f / static_cast<float>(g.n);
    int m = 0;  // this warp's blocks so far
    for (int i = warp; i < cnt; i += kConsumers, ++m) {
      const int slot = warp * kSlotsPerConsumer + (m & 1);
      bool ok = mbar_wait(&rs.full[slot], static_cast<uint32_t>((m >> 1) & 1), abort_flag, &g_score_err, 302);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      const uint8_t* sl = ring + slot * kSlotBytes;
      const int item = static_cast<int>(blockIdx.x) + i * G;
      const int blk = item % g.nb;
      const int bh = item / g.nb;
      // Pairwise tree in token order: each group of 8 rows is summed as its own subtree
      // ((r0 + r1) + (r2 + r3)) + ((r4 + r5) + (r6 + r7)) in registers, and the 8-row sums are
      // carried up a 3-level binary counter (warp-uniform branches, no dynamic indexing), which
      // is the same sequence of fp32 additions as inserting the rows one by one.
      float up0[4], up1[4], up2[4];
      float tot[4] = {0.f, 0.f, 0.f, 0.f};
      for (int r0 = 0; r0 < g.n; r0 += 8) {
        float v[8][4];
#pragma unroll
        for (int ii = 0; ii < 8; ++ii) {
          if (r0 + ii < g.n) slot_load4<T>(sl, r0 + ii, lane, v[ii]);
          else v[ii][0] = v[ii][1] = v[ii][2] = v[ii][3] = 0.f;
        }
        if (g.n < 8) {  // n = 1, 2 or 4: the whole tree is in this group
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float p01 = __fadd_rn(v[0][e], v[1][e]);
            tot[e] = g.n == 1 ? v[0][e] : (g.n == 2 ? p01 : __fadd_rn(p01, __fadd_rn(v[2][e], v[3][e])));
          }
          break;
        }
        float c[4];
#pragma unroll
        for (int e = 0; e < 4; ++e)
          c[e] = __fadd_rn(__fadd_rn(__fadd_rn(v[0][e], v[1][e]), __fadd_rn(v[2][e], v[3][e])),
                           __fadd_rn(__fadd_rn(v[4][e], v[5][e]), __fadd_rn(v[6][e], v[7][e])));
        const int q = r0 >> 3;  // index of this 8-row group
        if ((q & 1) == 0) {
#pragma unroll
          for (int e = 0; e < 4; ++e) up0[e] = c[e];
        } else {
#pragma unroll
          for (int e = 0; e < 4; ++e) c[e] = __fadd_rn(up0[e], c[e]);
          if ((q & 2) == 0) {
#pragma unroll
            for (int e = 0; e < 4; ++e) up1[e] = c[e];
          } else {
#pragma unroll
            for (int e = 0; e < 4; ++e) c[e] = __fadd_rn(up1[e], c[e]);
            if ((q & 4) == 0) {
#pragma unroll
              for (int e = 0; e < 4; ++e) up2[e] = c[e];
            } else {
#pragma unroll
              for (int e = 0; e < 4; ++e) c[e] = __fadd_rn(up2[e], c[e]);
            }
          }
        }
        if (r0 + 8 == g.n) {
#pragma unroll
          for (int e = 0; e < 4; ++e) tot[e] = c[e];
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&rs.empty[slot]);  // the slot's rows are in registers / written out
      const float out[4] = {dact ? __fmul_rn(tot[0], inv_n) : 0.f, dact ? __fmul_rn(tot[1], inv_n) : 0.f,
                            dact ? __fmul_rn(tot[2], inv_n) : 0.f, dact ? __fmul_rn(tot[3], inv_n) : 0.f};
      if (dact) store4(pooled + (static_cast<long long>(bh) * g.nb + blk) * g.D + d0, out);
      if (g.hl) split_row(g, bh, blk, out, lane);
    }
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
  g.rope = a.rope; g.rdt = a.rope_dt; g.rdh = a.rope_dh; g.rdw = a.rope_dw;
  g.rT = a.rope_T; g.rH = a.rope_H; g.rW = a.rope_W;
  g.map3 = a.map3;
  g.nw = a.norm_w; g.eps = a.norm_eps;
  g.hl = a.split_hl; g.nrm = a.split_nrm; g.nkmax = a.split_nkmax; g.which = a.split_which;
  if (n < 1 || n > 64 || (n & (n - 1)) || a.D > 128 || a.D % 4) return BSA_ERR_SHAPE;
  int dev = 0, sms = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const long long total = static_cast<long long>(a.B) * a.H * g.nb;
  long long grid = static_cast<long long>(sms) * 8;
  const long long need = (total + kThreads / 32 - 1) / (kThreads / 32);
  if (grid > need) grid = need;
  if (grid < 1) return BSA_OK;
  dim3 gd(static_cast<unsigned>(grid), 1, 1);
  const bool rope = a.rope != nullptr || a.norm_w != nullptr;  // a transform: the register kernel writes x_rot
  if (a.tmap && !rope && (a.dtype == BSA_DTYPE_BF16 || a.dtype == BSA_DTYPE_F16)) {
    // TMA ring: one persistent CTA per SM.  With fused RoPE the register kernel stays faster (its 32
    // warps per SM hide the per-row table loads and the rotated-row stores; 1.77 vs 2.22 ms of routing)
    // the shared-memory opt-in is per device; first calls from several host threads may race here
    static std::mutex mu;
    static bool configured[64][2] = {};
    const int ti = a.dtype == BSA_DTYPE_BF16 ? 0 : 1;
    {
      std::lock_guard<std::mutex> lock(mu);
      if (dev >= 64 || !configured[dev][ti]) {
        const cudaError_t e =
            ti == 0 ? cudaFuncSetAttribute(pool_tma_kernel<__nv_bfloat16>,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize, kTmaSmemBytes)
                    : cudaFuncSetAttribute(pool_tma_kernel<__half>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           kTmaSmemBytes);
        if (e != cudaSuccess) return BSA_ERR_CUDA;
        if (dev < 64) configured[dev][ti] = true;
      }
    }
    const dim3 tgd(static_cast<unsigned>(total < sms ? total : sms), 1, 1);
    if (ti == 0) pool_tma_kernel<__nv_bfloat16><<<tgd, kTmaThreads, kTmaSmemBytes, stream>>>(*a.tmap, a.pooled, g);
    else pool_tma_kernel<__half><<<tgd, kTmaThreads, kTmaSmemBytes, stream>>>(*a.tmap, a.pooled, g);
    return cudaGetLastError() == cudaSuccess ? BSA_OK : BSA_ERR_CUDA;
  }
#define BSA_POOL_LAUNCH(TT)                                                                                      \
  do {                                                                                                           \
    if (rope)                                                                                                    \
      pool_kernel<TT, true><<<gd, kThreads, 0, stream>>>(static_cast<const TT*>(a.x), static_cast<TT*>(a.x_rot),   \
                                                         a.pooled, g);                                           \
    else                                                                                                         \
      pool_kernel<TT, false><<<gd, kThreads, 0, stream>>>(static_cast<const TT*>(a.x), nullptr, a.pooled, g);      \
  } while (0)
  if (a.dtype == BSA_DTYPE_BF16) BSA_POOL_LAUNCH(__nv_bfloat16);
  else if (a.dtype == BSA_DTYPE_F16) BSA_POOL_LAUNCH(__half);
  else if (a.dtype == BSA_DTYPE_F32) BSA_POOL_LAUNCH(float);
  else return BSA_ERR_DTYPE;
#undef BSA_POOL_LAUNCH
  return cudaGetLastError() == cudaSuccess ? BSA_OK : BSA_ERR_CUDA;
}

// ======================================================================== block scores
// score[bh][i][j] = fp32 fma chain over d = 0..D-1 of qp[bh][i][d] * kp[bh][j][d], starting at 0.
// SGEMM-style tiling: a 128x128 tile per CTA, 8x8 scores per thread (two 4x4 quadrants), K in
// chunks of 8 through double-buffered shared memory.  Each score still accumulates over d in
// ascending order, so it is the same fp32 value the oracle computes with C fmaf.
namespace gemm {
constexpr int kThreads = 256;
constexpr int kTile = 128;
constexpr int kBK = 8;
constexpr int kLd = kTile + 4;  // padded smem row (floats)

struct Args {
  const float* qp;   // [BH, nq, D]
  const float* kp;   // [BH, nk, D]
  float* scores;     // [BH, nq, ldc]
  int nq, nk, D, ldc;
};

__global__ void __launch_bounds__(kThreads, 2) score_gemm_kernel(Args a) {
  __shared__ __align__(16) float As[2][kBK][kLd];
  __shared__ __align__(16) float Bs[2][kBK][kLd];
  const int tid = threadIdx.x;
  const int tx = tid & 15, ty = tid >> 4;
  const int bh = blockIdx.z;
  const int i0 = blockIdx.y * kTile, j0 = blockIdx.x * kTile;
  const float* qp = a.qp + static_cast<long long>(bh) * a.nq * a.D;
  const float* kp = a.kp + static_cast<long long>(bh) * a.nk * a.D;
  // global -> smem staging map: thread stages row (tid >> 1), d4 = (tid & 1) of each operand
  const int srow = tid >> 1, sd4 = tid & 1;
  const bool qv = i0 + srow < a.nq, kv = j0 + srow < a.nk;
  const float* qsrc = qp + static_cast<long long>(i0 + srow) * a.D + 4 * sd4;
  const float* ksrc = kp + static_cast<long long>(j0 + srow) * a.D + 4 * sd4;
  // accumulators in f32x2 pairs: acc2[r][p] holds scores (r, 2p) and (r, 2p+1)
  unsigned long long acc2[8][4];
#pragma unroll
  for (int r = 0; r < 8; ++r)
#pragma unroll
    for (int c = 0; c < 4; ++c) acc2[r][c] = 0ull;
  const int nchunks = a.D / kBK;
  float4 qn = qv ? __ldg(reinterpret_cast<const float4*>(qsrc)) : make_float4(0.f, 0.f, 0.f, 0.f);
  float4 kn = kv ? __ldg(reinterpret_cast<const float4*>(ksrc)) : make_float4(0.f, 0.f, 0.f, 0.f);
  for (int ch = 0; ch < nchunks; ++ch) {
    const int buf = ch & 1;
    As[buf][4 * sd4 + 0][srow] = qn.x;
    As[buf][4 * sd4 + 1][srow] = qn.y;
    As[buf][4 * sd4 + 2][srow] = qn.z;
    As[buf][4 * sd4 + 3][srow] = qn.w;
    Bs[buf][4 * sd4 + 0][srow] = kn.x;
    Bs[buf][4 * sd4 + 1][srow] = kn.y;
    Bs[buf][4 * sd4 + 2][srow] = kn.z;
    Bs[buf][4 * sd4 + 3][srow] = kn.w;
    __syncthreads();
    if (ch + 1 < nchunks) {  // prefetch the next chunk while this one is multiplied
      qn = qv ? __ldg(reinterpret_cast<const float4*>(qsrc + (ch + 1) * kBK)) : make_float4(0.f, 0.f, 0.f, 0.f);
      kn = kv ? __ldg(reinterpret_cast<const float4*>(ksrc + (ch + 1) * kBK)) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
#pragma unroll
    for (int d = 0; d < kBK; ++d) {
      const float4 a0 = *reinterpret_cast<const float4*>(&As[buf][d][ty * 4]);
      const float4 a1 = *reinterpret_cast<const float4*>(&As[buf][d][64 + ty * 4]);
      const ulonglong2 b0 = *reinterpret_cast<const ulonglong2*>(&Bs[buf][d][tx * 4]);
      const ulonglong2 b1 = *reinterpret_cast<const ulonglong2*>(&Bs[buf][d][64 + tx * 4]);
      const float av[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
      const unsigned long long bp[4] = {b0.x, b0.y, b1.x, b1.y};  // (b[2p], b[2p+1]) pairs
#pragma unroll
      for (int r = 0; r < 8; ++r) {
        unsigned long long ap;  // (a[r], a[r])
        asm("mov.b64 %0, {%1, %1};" : "=l"(ap) : "f"(av[r]));
#pragma unroll
        for (int c = 0; c < 4; ++c)
          // two independent round-to-nearest fp32 FMAs: the same values as two fmaf calls
          asm("fma.rn.f32x2 %0, %1, %2, %0;" : "+l"(acc2[r][c]) : "l"(ap), "l"(bp[c]));
      }
    }
  }
  float acc[8][8];
#pragma unroll
  for (int r = 0; r < 8; ++r)
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      acc[r][2 * c] = __uint_as_float(static_cast<uint32_t>(acc2[r][c]));
      acc[r][2 * c + 1] = __uint_as_float(static_cast<uint32_t>(acc2[r][c] >> 32));
    }
  float* out = a.scores + static_cast<long long>(bh) * a.nq * a.ldc;
  const bool vec = (a.ldc & 3) == 0;
#pragma unroll
  for (int r = 0; r < 8; ++r) {
    const int i = i0 + (r < 4 ? ty * 4 + r : 64 + ty * 4 + (r - 4));
    if (i >= a.nq) continue;
    float* orow = out + static_cast<long long>(i) * a.ldc;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int j = j0 + h * 64 + tx * 4;
      if (vec && j + 3 < a.nk) {
        *reinterpret_cast<float4*>(orow + j) =
            make_float4(acc[r][4 * h], acc[r][4 * h + 1], acc[r][4 * h + 2], acc[r][4 * h + 3]);
      } else {
#pragma unroll
        for (int c = 0; c < 4; ++c)
          if (j + c < a.nk) orow[j + c] = acc[r][4 * h + c];
      }
    }
  }
}
}  // namespace gemm

// ======================================================================== top-k per row
// One warp per score row.  The k-th largest key T is found over 32-bit order-preserving keys: by a
// radix select (8-bit digits counted in a per-warp shared histogram) for rows that fit in registers
// (up to 3,072 keys), by a binary search over the key range for longer rows, which are re-read
// from memory.  The row is then scanned in ascending block order taking every key above T and the
// first `need` keys equal to T.
namespace topk {
constexpr int kThreads = 256;

struct Args {
  const float* scores;  // rows of length nk, stride ldc
  int rows, nk, ldc, topk;
  int32_t* idx;         // [rows, topk]
};

// PL > 0: the row lives in registers (PL keys per lane, nk <= 32*PL) and goes through select_emit
// (bsa_select.cuh); PL == 0: rows too long for registers are re-read from memory.
template <int PL>
__global__ void __launch_bounds__(kThreads, 4) topk_kernel(Args a) {
  const int lane = threadIdx.x & 31;
  const int row = blockIdx.x * (kThreads / 32) + (threadIdx.x >> 5);
  if (row >= a.rows) return;
  const float* src = a.scores + static_cast<long long>(row) * a.ldc;
  const int nk = a.nk, k = a.topk;
  int32_t* out = a.idx + static_cast<long long>(row) * k;
  int taken = 0;
  if constexpr (PL > 0) {
    __shared__ __align__(16) uint32_t hist_all[kThreads / 32][256];
    __shared__ uint32_t cand_all[kThreads / 32][kCand];
    uint32_t key[PL];
#pragma unroll
    for (int e = 0; e < PL; ++e) {
      const int j = lane + 32 * e;
      key[e] = j < nk ? ordered_key(__ldg(src + j)) : 0u;
    }
    taken = select_emit<PL>(key, nk, k, lane, hist_all[threadIdx.x >> 5], cand_all[threadIdx.x >> 5], out);
  } else {
    // binary search for the largest T with #(key >= T) >= k (every real key is >= 1)
    auto count_ge = [&](uint32_t t) -> int {
      int c = 0;
      for (int j = lane; j < nk; j += 32) c += ordered_key(__ldg(src + j)) >= t ? 1 : 0;
      return __reduce_add_sync(0xffffffffu, c);
    };
    uint32_t lo = 1u, hi = 0xffffffffu;
    while (lo < hi) {
      const uint32_t mid = lo + ((hi - lo) >> 1) + 1u;
      if (count_ge(mid) >= k) lo = mid;
      else hi = mid - 1u;
    }
    const uint32_t T = lo;
    const int need = k - count_ge(T + (T != 0xffffffffu ? 1u : 0u)) * (T != 0xffffffffu ? 1 : 0);
    const uint32_t lt_mask = (1u << lane) - 1u;
    int ties = 0;
    for (int j0 = 0; j0 < nk; j0 += 32) {
      const int j = j0 + lane;
      const uint32_t u = j < nk ? ordered_key(__ldg(src + j)) : 0u;
      const bool valid = j < nk;
      const bool eq = valid && u == T;
      const uint32_t eqb = __ballot_sync(0xffffffffu, eq);
      const int rank = ties + __popc(eqb & lt_mask);
      const bool sel = valid && (u > T || (eq && rank < need));
      const uint32_t sb = __ballot_sync(0xffffffffu, sel);
      if (sel) out[taken + __popc(sb & lt_mask)] = j;
      taken += __popc(sb);
      ties += __popc(eqb);
    }
  }
  if (lane == 0 && taken != k) atomicCAS(&g_score_err, 0, 201);
}
}  // namespace topk

int launch_scores_only(const ScoreArgs& s, cudaStream_t stream) {
  if (s.D % gemm::kBK || s.D <= 0 || !s.scores) return BSA_ERR_SHAPE;
  gemm::Args a;
  a.qp = s.qp; a.kp = s.kp; a.scores = s.scores; a.nq = s.nq; a.nk = s.nk; a.D = s.D; a.ldc = s.ldc;
  dim3 grid((s.nk + gemm::kTile - 1) / gemm::kTile, (s.nq + gemm::kTile - 1) / gemm::kTile, s.BH);
  if (grid.y > 65535u || grid.z > 65535u) return BSA_ERR_SHAPE;
  gemm::score_gemm_kernel<<<grid, gemm::kThreads, 0, stream>>>(a);
  return cudaGetLastError() == cudaSuccess ? BSA_OK : BSA_ERR_CUDA;
}

int launch_topk(const float* scores, int rows, int nk, int ldc, int topk_, int32_t* idx, cudaStream_t stream) {
  topk::Args a;
  a.scores = scores; a.rows = rows; a.nk = nk; a.ldc = ldc; a.topk = topk_; a.idx = idx;
  const unsigned grid = static_cast<unsigned>((rows + 7) / 8);
  if (grid == 0) return BSA_OK;
  if (nk <= 32 * 48) topk::topk_kernel<48><<<grid, topk::kThreads, 0, stream>>>(a);
  else if (nk <= 32 * 96) topk::topk_kernel<96><<<grid, topk::kThreads, 0, stream>>>(a);
  else topk::topk_kernel<0><<<grid, topk::kThreads, 0, stream>>>(a);
  return cudaGetLastError() == cudaSuccess ? BSA_OK : BSA_ERR_CUDA;
}

int launch_score_topk(const ScoreArgs& s, cudaStream_t stream) {
  int rc = launch_scores_only(s, stream);
  if (rc) return rc;
  return launch_topk(s.scores, s.BH * s.nq, s.nk, s.ldc, s.topk, s.idx, stream);
}

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
