// Block routing (block_routing_scores + topk_block_indices, block_sparse_attention.py:107-134) without
// the block-score matrix.  The selected indices are exactly those of the exact fp32 scores (one fma
// chain over d = 0..D-1 per score, as in bsa_score.cu and the CPU oracle) followed by top-k with ties
// to the smaller block id; the score matrix itself is never written.
//
//   1. split  : pooled fp32 Q/K rows -> bf16 pairs (hi = bf16(x), lo = bf16(x - hi)), zero padded to
//               128 columns, and an upper bound of each row's l2 norm (+inf for values this bound does
//               not cover: non-finite, above 2^60 or below 2^-60 in magnitude).
//   2. keys   : tcgen05 approximate scores a = qh.kh + qh.kl + ql.kh (fp32 accumulation in TMEM), 128
//               query blocks x 128 key blocks per step, written as 16-bit keys: the top half of the
//               score's order-preserving 32-bit pattern (so a key names an interval of fp32 scores).
//   3. select : one warp per row.  With T = the k-th largest key of the row, the exact k-th largest
//               score s_(k) lies in [L, U] = [low(T) - e, high(T) + e] (e bounds |a - s|, below).  A
//               block whose interval lies above U is selected, one below L is not; only the blocks
//               whose interval meets the band get the exact score, and the top of those fills the
//               remaining places (ties to the smaller id).  Rows whose band holds more than kMaxBand
//               blocks, or whose bound is not finite, are scored exactly in full (same result).
//
// Error bound.  With x = hi + lo + r, |r| <= 2^-18 |x| (two round-to-nearest bf16 steps), the three
// products drop lo*lo and the r terms: at most ~3.1 * 2^-18 sum_d |q_d k_d|.  bf16 products are exact
// in fp32; the tensor core's fp32 accumulation of 3 x 128 terms adds at most ~2^-14.3 sum_d |q_d k_d|
// even with truncation at every addition, and the exact fma chain itself is within 128 * 2^-24 of the
// real dot product.  So |a - s| <= 2^-13.9 sum_d |q_d k_d| <= 2^-13.9 |q| |k|, and e = 2^-12 |q| max|k|
// (with |q|, |k| rounded up) leaves a margin of about 3.7x.
#include <cstdint>
#include <mutex>
#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include "bsa_kernels.h"
#include "bsa_ptx.cuh"
#include "bsa_select.cuh"

namespace bsa {

__device__ int g_route_err;

namespace route {
constexpr int kDP = 128;                 // padded head dim of the bf16 pairs
constexpr float kErrC = 1.0f / 4096.0f;  // e = kErrC * |q| * max|k|
constexpr int kMaxBand = 64;             // blocks per row scored exactly on the fast path

// ------------------------------------------------------------------ 1. split
// One warp per pooled row (Q rows then K rows); lane l holds d = 4l .. 4l+3.
__global__ void __launch_bounds__(256) split_kernel(const float* __restrict__ qp, const float* __restrict__ kp,
                                                    int rows, int nb, int D, __nv_bfloat16* hl, float* nrm,
                                                    float* nkmax) {
  const int lane = threadIdx.x & 31;
  const int nw = gridDim.x * (blockDim.x >> 5);
  for (int r = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); r < 2 * rows; r += nw) {
    const int which = r >= rows;  // 0: Q, 1: K
    const int row = r - which * rows;
    const float* src = (which ? kp : qp) + static_cast<long long>(row) * D;
    const int d0 = 4 * lane;
    float x[4] = {0.f, 0.f, 0.f, 0.f};
    if (d0 < D) {
      const float4 v = __ldg(reinterpret_cast<const float4*>(src + d0));
      x[0] = v.x; x[1] = v.y; x[2] = v.z; x[3] = v.w;
    }
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
    __nv_bfloat16* dh = hl + (static_cast<long long>(2 * which) * rows + row) * kDP + d0;
    __nv_bfloat16* dl = hl + (static_cast<long long>(2 * which + 1) * rows + row) * kDP + d0;
    *reinterpret_cast<uint2*>(dh) = *reinterpret_cast<const uint2*>(hi);
    *reinterpret_cast<uint2*>(dl) = *reinterpret_cast<const uint2*>(lo);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) n2 += __shfl_xor_sync(0xffffffffu, n2, off);
    extreme = __any_sync(0xffffffffu, extreme);
    if (lane == 0) {
      // sqrt of an fp32 sum of 128 squares: relative error far below 2^-10, so the bound holds
      const float n = extreme ? INFINITY : __fmul_ru(sqrtf(n2), 1.0009765625f);
      nrm[static_cast<long long>(which) * rows + row] = n;
      if (which) atomicMax(reinterpret_cast<int*>(nkmax) + row / nb, __float_as_int(n));  // n >= 0
    }
  }
}

// ------------------------------------------------------------------ 2. keys (tcgen05)
constexpr int kTile = 128;                          // query blocks per CTA, key blocks per step
constexpr int kArrBytes = kTile * kDP * 2;          // 32 KB: one bf16 array tile (two 16 KB d-halves)
constexpr int kKeyThreads = 320;                    // warp 0 TMA, warp 1 MMA, warps 2-9 epilogue
struct KeySmem {
  uint64_t a_full;
  uint64_t b_full[2], b_empty[2];
  uint64_t acc_full[2], acc_empty[2];
  uint64_t drain;
  uint32_t tmem_base;
  int abort_flag;
};
constexpr int kKeyTiles = 2 * kArrBytes + 2 * 2 * kArrBytes;  // A (qh, ql) + two B stages (kh, kl)
constexpr int kKeySmemBytes = 1024 + kKeyTiles + static_cast<int>(sizeof(KeySmem));

__device__ __forceinline__ uint32_t key16(float a) {
  if (a != a) return 1u;  // NaN: the lowest real key (its interval bounds are NaN: never outside a band)
  return topk::ordered_key(a) >> 16;
}

__global__ void __launch_bounds__(kKeyThreads, 1)
    key_kernel(const __grid_constant__ CUtensorMap m_qh, const __grid_constant__ CUtensorMap m_ql,
               const __grid_constant__ CUtensorMap m_kh, const __grid_constant__ CUtensorMap m_kl, int nb, int ldk,
               uint16_t* keys) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* sm = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint8_t* sA = sm;                       // qh | ql
  uint8_t* sB = sm + 2 * kArrBytes;       // stage s: kh | kl at sB + s * 2 * kArrBytes
  KeySmem& ks = *reinterpret_cast<KeySmem*>(sm + kKeyTiles);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int bh = blockIdx.y;
  const int i0 = blockIdx.x * kTile;
  // this CTA's key-block steps: chunk z of gridDim.z of the row's ceil(nb / 128) steps
  const int nall = (nb + kTile - 1) / kTile;
  const int cbeg = static_cast<int>(static_cast<long long>(nall) * blockIdx.z / gridDim.z);
  const int nch = static_cast<int>(static_cast<long long>(nall) * (blockIdx.z + 1) / gridDim.z) - cbeg;
  if (threadIdx.x == 0) {
    mbar_init(&ks.a_full, 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&ks.b_full[s], 1);
      mbar_init(&ks.b_empty[s], 1);
      mbar_init(&ks.acc_full[s], 1);
      mbar_init(&ks.acc_empty[s], 8);
    }
    mbar_init(&ks.drain, 1);
    ks.abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(&ks.tmem_base, 256);
    tmem_relinquish();
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = ks.tmem_base;
  volatile int* abort_flag = &ks.abort_flag;
  int* err = &g_route_err;
  if (warp == 0) {
    if (lane == 0) {
      mbar_arrive_expect_tx(&ks.a_full, 2 * kArrBytes);
      for (int hh = 0; hh < 2; ++hh) {
        tma_load_3d(sA + hh * 16384, &m_qh, &ks.a_full, 64 * hh, i0, bh);
        tma_load_3d(sA + kArrBytes + hh * 16384, &m_ql, &ks.a_full, 64 * hh, i0, bh);
      }
      int c = 0;
      for (; c < nch; ++c) {
        const int s = c & 1;
        if (c >= 2 && !mbar_wait(&ks.b_empty[s], static_cast<uint32_t>(((c >> 1) - 1) & 1), abort_flag, err, 401))
          break;
        uint8_t* dst = sB + s * 2 * kArrBytes;
        mbar_arrive_expect_tx(&ks.b_full[s], 2 * kArrBytes);
        for (int hh = 0; hh < 2; ++hh) {
          tma_load_3d(dst + hh * 16384, &m_kh, &ks.b_full[s], 64 * hh, (cbeg + c) * kTile, bh);
          tma_load_3d(dst + kArrBytes + hh * 16384, &m_kl, &ks.b_full[s], 64 * hh, (cbeg + c) * kTile, bh);
        }
      }
      // teardown: every TMA write into shared memory has landed
      const uint64_t t0 = globaltimer_ns();
      for (int cc = (c > 2 ? c - 2 : 0); cc < c; ++cc)
        while (!mbar_try_wait(&ks.b_full[cc & 1], static_cast<uint32_t>((cc >> 1) & 1)) &&
               globaltimer_ns() - t0 < kWaitLimitNs) {
        }
      while (!mbar_try_wait(&ks.a_full, 0) && globaltimer_ns() - t0 < kWaitLimitNs) {
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = idesc_f16(128, 128, 1, 0, 0);
      bool ok = mbar_wait(&ks.a_full, 0, abort_flag, err, 402);
      for (int c = 0; c < nch && ok; ++c) {
        const int s = c & 1;
        ok = mbar_wait(&ks.b_full[s], static_cast<uint32_t>((c >> 1) & 1), abort_flag, err, 403);
        if (ok && c >= 2)
          ok = mbar_wait(&ks.acc_empty[s], static_cast<uint32_t>(((c >> 1) - 1) & 1), abort_flag, err, 404);
        if (!ok) break;
        tc_fence_after();
        const uint32_t d = tmem + static_cast<uint32_t>(s * kTile);
        const uint32_t aq = smem_u32(sA), bq = smem_u32(sB + s * 2 * kArrBytes);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint32_t off = (kk >> 2) * 16384 + (kk & 3) * 32;
          const uint64_t a_hi = sdesc_sw128(aq + off, 16, 1024), a_lo = sdesc_sw128(aq + kArrBytes + off, 16, 1024);
          const uint64_t b_hi = sdesc_sw128(bq + off, 16, 1024), b_lo = sdesc_sw128(bq + kArrBytes + off, 16, 1024);
          umma_ss(d, a_hi, b_hi, idesc, kk > 0 ? 1u : 0u);
          umma_ss(d, a_hi, b_lo, idesc, 1u);
          umma_ss(d, a_lo, b_hi, idesc, 1u);
        }
        umma_commit(&ks.acc_full[s]);
        umma_commit(&ks.b_empty[s]);
      }
      umma_commit(&ks.drain);
      const uint64_t t0 = globaltimer_ns();
      while (!mbar_try_wait(&ks.drain, 0) && globaltimer_ns() - t0 < kWaitLimitNs) {
      }
    }
    __syncwarp();
  } else {
    // epilogue: warp w reads TMEM lane quarter w % 4 (query blocks 32q .. 32q+31 of the tile) and
    // columns [64ch, 64ch + 64) of each 128-column step
    const int q = warp & 3;
    const int ch = (warp - 2) >> 2;
    const int i = i0 + 32 * q + lane;
    uint16_t* krow = keys + (static_cast<long long>(bh) * nb + (i < nb ? i : 0)) * ldk;
    for (int c = 0; c < nch; ++c) {
      const int s = c & 1;
      bool ok = mbar_wait(&ks.acc_full[s], static_cast<uint32_t>((c >> 1) & 1), abort_flag, err, 405);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      tc_fence_after();
#pragma unroll 1
      for (int part = 0; part < 2; ++part) {
        uint32_t r[32];
        tmem_ld32(tmem + (static_cast<uint32_t>(32 * q) << 16) + static_cast<uint32_t>(s * kTile + 64 * ch + 32 * part),
                  r);
        tmem_ld_wait();
        const int j0 = (cbeg + c) * kTile + 64 * ch + 32 * part;
        if (i < nb) {
#pragma unroll
          for (int e8 = 0; e8 < 4; ++e8) {
            if (j0 + 8 * e8 < ldk) {  // ldk is a multiple of 8; the select clears the keys past nb
              uint4 w;
              w.x = key16(__uint_as_float(r[8 * e8 + 0])) | (key16(__uint_as_float(r[8 * e8 + 1])) << 16);
              w.y = key16(__uint_as_float(r[8 * e8 + 2])) | (key16(__uint_as_float(r[8 * e8 + 3])) << 16);
              w.z = key16(__uint_as_float(r[8 * e8 + 4])) | (key16(__uint_as_float(r[8 * e8 + 5])) << 16);
              w.w = key16(__uint_as_float(r[8 * e8 + 6])) | (key16(__uint_as_float(r[8 * e8 + 7])) << 16);
              *reinterpret_cast<uint4*>(krow + j0 + 8 * e8) = w;
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&ks.acc_empty[s]);
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) tmem_dealloc(tmem, 256);
}

// ------------------------------------------------------------------ 3. select (one warp per row)
constexpr int kSelThreads = 256;
constexpr int kSelWarps = kSelThreads / 32;
// Per-warp shared state of select_kernel; two key-row buffers of 128 * words bytes follow it (the next
// row's keys and q row land by cp.async while this row is processed).
struct SelWarp {
  uint32_t hist[256];
  float q[2][kDP];
  uint32_t band_key[kMaxBand];  // exact scores of the band, order-preserving
  int32_t band_id[kMaxBand];
  uint8_t band_sel[kMaxBand];
};
constexpr int kSelFixedBytes = (static_cast<int>(sizeof(SelWarp)) + 127) & ~127;
__host__ __device__ constexpr int sel_warp_bytes(int words) { return kSelFixedBytes + 2 * 128 * words; }

__device__ __forceinline__ void cp_async16(void* sdst, const void* gsrc) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(smem_u32(sdst)), "l"(gsrc) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_prev() { asm volatile("cp.async.wait_group 1;\n" ::: "memory"); }

// fp32 value of an order-preserving bit pattern
__device__ __forceinline__ float from_ordered(uint32_t o) {
  return __uint_as_float((o & 0x80000000u) ? (o & 0x7fffffffu) : ~o);
}
// the fp32 interval a 16-bit key stands for
__device__ __forceinline__ float key_low(uint32_t key) { return from_ordered(key << 16); }
__device__ __forceinline__ float key_high(uint32_t key) { return from_ordered((key << 16) | 0xffffu); }

// exact score: one fp32 fma chain over d = 0..D-1, starting at 0 (block_routing_scores, in the order
// the CPU oracle uses)
__device__ __forceinline__ float exact_score(const float* q, const float* __restrict__ krow, int D) {
  float acc = 0.f;
  for (int d = 0; d < D; d += 4) {
    const float4 kv = __ldg(reinterpret_cast<const float4*>(krow + d));
    acc = fmaf(q[d], kv.x, acc);
    acc = fmaf(q[d + 1], kv.y, acc);
    acc = fmaf(q[d + 2], kv.z, acc);
    acc = fmaf(q[d + 3], kv.w, acc);
  }
  return acc;
}

// The same chain for two rows at once (row1 may be null), 16 d values per round: every load of a
// round is issued before its first fma, so a round costs one L2 latency instead of four.  q is a 16-byte
// aligned row in shared memory.
__device__ __forceinline__ void exact_score2(const float* q, const float* __restrict__ r0, const float* __restrict__ r1,
                                             int D, float& s0, float& s1) {
  float a0 = 0.f, a1 = 0.f;
  for (int d0 = 0; d0 < D; d0 += 16) {
    float4 k0[4], k1[4];
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const int d = d0 + 4 * c;
      k0[c] = d < D ? __ldg(reinterpret_cast<const float4*>(r0 + d)) : make_float4(0.f, 0.f, 0.f, 0.f);
      k1[c] = (r1 && d < D) ? __ldg(reinterpret_cast<const float4*>(r1 + d)) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const int d = d0 + 4 * c;
      if (d < D) {
        const float4 qv = *reinterpret_cast<const float4*>(q + d);  // q: 16-byte aligned shared memory
        a0 = fmaf(qv.x, k0[c].x, a0); a0 = fmaf(qv.y, k0[c].y, a0);
        a0 = fmaf(qv.z, k0[c].z, a0); a0 = fmaf(qv.w, k0[c].w, a0);
        a1 = fmaf(qv.x, k1[c].x, a1); a1 = fmaf(qv.y, k1[c].y, a1);
        a1 = fmaf(qv.z, k1[c].z, a1); a1 = fmaf(qv.w, k1[c].w, a1);
      }
    }
  }
  s0 = a0;
  s1 = a1;
}

// One byte of a radix select over the row's 16-bit keys (two per word, word e of lane l at kw[32e + l];
// key 0 marks a slot past nb, as no score maps to 0): counts the byte `shift` of the keys whose bits
// above it equal `prefix`, then finds the value of that byte holding the need-th largest key.  Updates
// prefix (the key bits found so far) and need.
__device__ __forceinline__ void key_radix_byte(const uint32_t* kw, int words, uint32_t* h, int lane, int shift,
                                               uint32_t& prefix, int& need) {
  reinterpret_cast<uint4*>(h)[lane * 2] = make_uint4(0u, 0u, 0u, 0u);
  reinterpret_cast<uint4*>(h)[lane * 2 + 1] = make_uint4(0u, 0u, 0u, 0u);
  __syncwarp();
  const uint32_t hi_mask = shift == 8 ? 0u : 0xff00u;  // bits above the counted byte that must match
#pragma unroll 4
  for (int e = 0; e < words; ++e) {
    const uint32_t w = kw[32 * e + lane];
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      const uint32_t key = half ? (w >> 16) : (w & 0xffffu);
      if (key != 0u && (key & hi_mask) == (prefix & hi_mask)) atomicAdd(&h[(key >> shift) & 0xffu], 1u);
    }
  }
  __syncwarp();
  const uint4 c0 = reinterpret_cast<const uint4*>(h)[lane * 2];
  const uint4 c1 = reinterpret_cast<const uint4*>(h)[lane * 2 + 1];
  const uint32_t cnt[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
  uint32_t tot = 0;
#pragma unroll
  for (int b = 0; b < 8; ++b) tot += cnt[b];
  uint32_t suf = tot;  // inclusive suffix sum over lanes >= this lane
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const uint32_t o = __shfl_down_sync(0xffffffffu, suf, off);
    if (lane + off < 32) suf += o;
  }
  const uint32_t above = suf - tot;
  const bool mine = above < static_cast<uint32_t>(need) && static_cast<uint32_t>(need) <= suf;
  int digit = 0;
  uint32_t gt = 0;
  if (mine) {
    uint32_t run = above;
#pragma unroll
    for (int b = 7; b >= 0; --b) {
      if (run + cnt[b] >= static_cast<uint32_t>(need)) {
        digit = lane * 8 + b;
        gt = run;
        break;
      }
      run += cnt[b];
    }
  }
  const int src = __ffs(__ballot_sync(0xffffffffu, mine)) - 1;
  digit = __shfl_sync(0xffffffffu, digit, src);
  gt = __shfl_sync(0xffffffffu, gt, src);
  prefix |= static_cast<uint32_t>(digit) << shift;
  need -= static_cast<int>(gt);
  __syncwarp();
}

// The k-th largest key when it lies within 255 of the row's largest key (the common case: key space is
// logarithmic, 128 keys per factor of 2, and the top k of a row seldom spans a factor of 4): one
// histogram of d = max - key over d < 256, where only the keys of that window count, so the bulk of
// the row (far below) costs a compare and no shared-memory atomic.  Returns false when fewer than k
// keys lie in the window; T is then unchanged.  Key 0 marks a slot past nb (no score maps to 0).
__device__ __forceinline__ bool key_window_select(const uint32_t* kw, int words, uint32_t* h, int lane, int k,
                                                  uint32_t& T) {
  uint32_t mx = 0;
#pragma unroll 4
  for (int e = 0; e < words; ++e) {
    const uint32_t w = kw[32 * e + lane];
    mx = max(mx, max(w & 0xffffu, w >> 16));
  }
  mx = __reduce_max_sync(0xffffffffu, mx);
  const uint32_t lim = min(256u, mx);  // d < mx excludes the key-0 slots
  reinterpret_cast<uint4*>(h)[lane * 2] = make_uint4(0u, 0u, 0u, 0u);
  reinterpret_cast<uint4*>(h)[lane * 2 + 1] = make_uint4(0u, 0u, 0u, 0u);
  __syncwarp();
#pragma unroll 4
  for (int e = 0; e < words; ++e) {
    const uint32_t w = kw[32 * e + lane];
    const uint32_t d0 = mx - (w & 0xffffu), d1 = mx - (w >> 16);
    if (d0 < lim) atomicAdd(&h[d0], 1u);
    if (d1 < lim) atomicAdd(&h[d1], 1u);
  }
  __syncwarp();
  // bins 8l .. 8l+7 on lane l, in order of decreasing key; inclusive prefix over the lanes
  const uint4 c0 = reinterpret_cast<const uint4*>(h)[lane * 2];
  const uint4 c1 = reinterpret_cast<const uint4*>(h)[lane * 2 + 1];
  const uint32_t cnt[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
  uint32_t tot = 0;
#pragma unroll
  for (int b = 0; b < 8; ++b) tot += cnt[b];
  uint32_t pre = tot;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const uint32_t o = __shfl_up_sync(0xffffffffu, pre, off);
    if (lane >= off) pre += o;
  }
  const uint32_t kk = static_cast<uint32_t>(k);
  const bool mine = pre - tot < kk && kk <= pre;
  uint32_t dk = 0;
  if (mine) {
    uint32_t run = pre - tot;
#pragma unroll
    for (int b = 0; b < 8; ++b) {
      run += cnt[b];
      if (run >= kk) {
        dk = 8u * static_cast<uint32_t>(lane) + static_cast<uint32_t>(b);
        break;
      }
    }
  }
  const uint32_t bal = __ballot_sync(0xffffffffu, mine);
  __syncwarp();
  if (!bal) return false;
  dk = __shfl_sync(0xffffffffu, dk, __ffs(bal) - 1);
  T = mx - dk;
  return true;
}

// Smallest key whose interval minus e lies above U (keys at or above it are sure), and largest finite
// key whose interval plus e lies below L (finite keys at or below it are out).  Both predicates are
// monotone over the finite keys [0x80, 0xff80]; the 32 lanes probe 32 keys next to the k-th key at
// once and a binary search covers the rare wider bands.
__device__ __forceinline__ void band_keys(uint32_t T, float L, float U, float e, int lane, uint32_t& ks, uint32_t& ko) {
  {
    const uint32_t c = T + 1u + static_cast<uint32_t>(lane);
    const bool p = c <= 0xff80u && __fsub_rd(key_low(c), e) > U;
    const uint32_t b = __ballot_sync(0xffffffffu, p);
    if (b) {
      ks = T + 1u + static_cast<uint32_t>(__ffs(b) - 1);
    } else {
      uint32_t lo = T + 33u, hi = 0xff81u;  // 0xff81: no key is sure
      if (lo > hi) lo = hi;
      while (lo < hi) {
        const uint32_t mid = (lo + hi) >> 1;
        if (__fsub_rd(key_low(mid), e) > U) hi = mid;
        else lo = mid + 1u;
      }
      ks = lo;
    }
  }
  {
    const int c = static_cast<int>(T) - 1 - lane;
    const bool p = c >= 0x80 && __fadd_ru(key_high(static_cast<uint32_t>(c)), e) < L;
    const uint32_t b = __ballot_sync(0xffffffffu, p);
    if (b) {
      ko = T - 1u - static_cast<uint32_t>(__ffs(b) - 1);
    } else {
      int lo = 0x7f, hi = static_cast<int>(T) - 33;  // 0x7f: no key is out
      if (hi < lo) hi = lo;
      while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (__fadd_ru(key_high(static_cast<uint32_t>(mid)), e) < L) lo = mid;
        else hi = mid - 1;
      }
      ko = static_cast<uint32_t>(lo);
    }
  }
}

// A key the bound does not decide: below the sure keys and above the out keys, or non-finite (1 .. 0x7f:
// NaN, -inf); key 0 is an empty slot.
__device__ __forceinline__ bool in_band(uint32_t key, uint32_t ks, uint32_t ko) {
  return key < ks && (key > ko || key - 1u < 0x7fu);
}

// One warp per row; the row's keys sit in shared memory as `words` 32-bit words per lane (lane l holds
// keys 64e + 2l and 64e + 2l + 1 in word e).  Dynamic shared memory: kSelWarps * sel_warp_bytes(words).
__global__ void __launch_bounds__(kSelThreads, 3)
    select_kernel(const uint16_t* __restrict__ keys, int ldk, const float* __restrict__ qp,
                  const float* __restrict__ kp, const float* __restrict__ nrm, const float* __restrict__ nkmax, int rows,
                  int nb, int D, int k, int32_t* idx, int* fb_count, int* fb_rows) {
  extern __shared__ __align__(128) uint8_t sel_smem[];
  const int lane = threadIdx.x & 31;
  const int words = (nb + 63) >> 6;
  uint8_t* wbase = sel_smem + static_cast<size_t>(threadIdx.x >> 5) * sel_warp_bytes(words);
  SelWarp& sw = *reinterpret_cast<SelWarp*>(wbase);
  uint32_t* kbuf = reinterpret_cast<uint32_t*>(wbase + kSelFixedBytes);  // [2][32 * words]
  const uint32_t lt = (1u << lane) - 1u;
  const int nw = gridDim.x * kSelWarps;
  int row = blockIdx.x * kSelWarps + (threadIdx.x >> 5);
  if (k == nb) {  // every block: the ids in order
    for (; row < rows; row += nw)
      for (int j = lane; j < nb; j += 32) idx[static_cast<long long>(row) * k + j] = j;
    return;
  }
  // slots from nb up to 64 * words hold key 0 (no score maps to 0): the ones no copy reaches are set
  // once here, the padding slots nb .. ldk-1 that a copy brings are cleared after each row lands
  for (int b = 0; b < 2; ++b) {
    uint16_t* kb = reinterpret_cast<uint16_t*>(kbuf + b * 32 * words);
    for (int j = ldk + lane; j < 64 * words; j += 32) kb[j] = 0;
  }
  const int kchunks = ldk >> 3, qchunks = D >> 2;  // 16-byte pieces of a key row and of a q row
  auto fetch = [&](int r, int b) {
    const uint8_t* src = reinterpret_cast<const uint8_t*>(keys + static_cast<long long>(r) * ldk);
    uint8_t* dst = reinterpret_cast<uint8_t*>(kbuf + b * 32 * words);
    for (int c = lane; c < kchunks; c += 32) cp_async16(dst + 16 * c, src + 16 * c);
    const float* qs = qp + static_cast<long long>(r) * D;
    for (int c = lane; c < qchunks; c += 32) cp_async16(sw.q[b] + 4 * c, qs + 4 * c);
  };
  if (row < rows) fetch(row, 0);
  cp_async_commit();
  for (int b = 0; row < rows; row += nw, b ^= 1) {
    if (row + nw < rows) fetch(row + nw, b ^ 1);
    cp_async_commit();
    cp_async_wait_prev();  // this row's group has landed (the next row's may still be in flight)
    __syncwarp();
    const uint32_t* kw = kbuf + b * 32 * words;
    if (lane < ldk - nb) reinterpret_cast<uint16_t*>(kbuf + b * 32 * words)[nb + lane] = 0;
    __syncwarp();
    const float* q = sw.q[b];
    const int bh = row / nb;
    int32_t* out = idx + static_cast<long long>(row) * k;
    const float ebound = __fmul_ru(__fmul_ru(kErrC, __ldg(nrm + row)), __ldg(nkmax + bh));
    // the k-th largest key T: a window below the row's largest key, else a radix select (high byte,
    // then low byte)
    uint32_t T = 0;
    if (!key_window_select(kw, words, sw.hist, lane, k, T)) {
      int need = k;
      key_radix_byte(kw, words, sw.hist, lane, 8, T, need);
      key_radix_byte(kw, words, sw.hist, lane, 0, T, need);
    }
    // s_(k) in [L, U]
    const float L = __fsub_rd(key_low(T), ebound);
    const float U = __fadd_ru(key_high(T), ebound);
    uint32_t ks = 0xff81u, ko = 0x7fu;
    if (ebound < INFINITY) band_keys(T, L, U, ebound, lane, ks, ko);
    // classes: sure (key >= ks), out (0x80 <= key <= ko), band (the other keys but 0); band ids ascending
    int n_sure = 0, pos = 0;
#pragma unroll 2
    for (int e = 0; e < words; ++e) {
      const uint32_t w = kw[32 * e + lane];
      const uint32_t k0 = w & 0xffffu, k1 = w >> 16;
      n_sure += (k0 >= ks) + (k1 >= ks);
      const bool b0 = in_band(k0, ks, ko), b1 = in_band(k1, ks, ko);
      const uint32_t m0 = __ballot_sync(0xffffffffu, b0), m1 = __ballot_sync(0xffffffffu, b1);
      const int p0 = pos + __popc(m0 & lt) + __popc(m1 & lt);
      if (b0 && p0 < kMaxBand) sw.band_id[p0] = 64 * e + 2 * lane;
      if (b1 && p0 + b0 < kMaxBand) sw.band_id[p0 + b0] = 64 * e + 2 * lane + 1;
      pos += __popc(m0) + __popc(m1);
    }
    n_sure = __reduce_add_sync(0xffffffffu, n_sure);
    const int n_band = pos;
    const bool fast = ebound < INFINITY && n_band <= kMaxBand && n_sure <= k && n_sure + n_band >= k;
    if (!fast) {  // scored exactly in full by fallback_kernel
      if (lane == 0) fb_rows[atomicAdd(fb_count, 1)] = row;
      __syncwarp();
      continue;
    }
    __syncwarp();
    // exact scores of the band (two per lane at most)
    const float* kbase = kp + static_cast<long long>(bh) * nb * D;
    if (lane < n_band) {
      float s0, s1;
      const float* r1 = lane + 32 < n_band ? kbase + static_cast<long long>(sw.band_id[lane + 32]) * D : nullptr;
      exact_score2(q, kbase + static_cast<long long>(sw.band_id[lane]) * D, r1, D, s0, s1);
      sw.band_key[lane] = topk::ordered_key(s0);
      if (r1) sw.band_key[lane + 32] = topk::ordered_key(s1);
    }
    __syncwarp();
    // the `rest` largest of the band, ties to the smaller id: rank by comparison (the band is short)
    const int rest = k - n_sure;
#pragma unroll
    for (int t = 0; t < 2; ++t) {
      const int b2 = lane + 32 * t;
      if (b2 < n_band) {
        const uint32_t mk = sw.band_key[b2];
        int rank = 0;
        for (int u = 0; u < n_band; ++u) {
          const uint32_t o = sw.band_key[u];
          rank += (o > mk || (o == mk && u < b2)) ? 1 : 0;
        }
        sw.band_sel[b2] = rank < rest;
      }
    }
    __syncwarp();
    // ascending emission: sure blocks and the chosen band blocks
    int taken = 0, bpos = 0;
#pragma unroll 2
    for (int e = 0; e < words; ++e) {
      const uint32_t w = kw[32 * e + lane];
      const uint32_t k0 = w & 0xffffu, k1 = w >> 16;
      const bool b0 = in_band(k0, ks, ko), b1 = in_band(k1, ks, ko);
      const uint32_t m0 = __ballot_sync(0xffffffffu, b0), m1 = __ballot_sync(0xffffffffu, b1);
      const int p0 = bpos + __popc(m0 & lt) + __popc(m1 & lt);
      const bool s0 = k0 >= ks || (b0 && sw.band_sel[p0]);
      const bool s1 = k1 >= ks || (b1 && sw.band_sel[p0 + b0]);
      const uint32_t t0 = __ballot_sync(0xffffffffu, s0), t1 = __ballot_sync(0xffffffffu, s1);
      const int q0 = taken + __popc(t0 & lt) + __popc(t1 & lt);
      if (s0) out[q0] = 64 * e + 2 * lane;
      if (s1) out[q0 + s0] = 64 * e + 2 * lane + 1;
      taken += __popc(t0) + __popc(t1);
      bpos += __popc(m0) + __popc(m1);
    }
    if (lane == 0 && taken != k) atomicCAS(&g_route_err, 0, 410);
    __syncwarp();
  }
  asm volatile("cp.async.wait_all;\n" ::: "memory");
}

// Rows the fast path could not bound: every score exact (one warp per row), then the register radix
// select of the top-k kernel.  The row list comes from select_kernel.
template <int PL>
__global__ void __launch_bounds__(kSelThreads, 2)
    fallback_kernel(const float* __restrict__ qp, const float* __restrict__ kp, int nb, int D, int k, int32_t* idx,
                    const int* fb_count, const int* fb_rows) {
  __shared__ __align__(16) uint32_t hist_all[kSelThreads / 32][256];
  __shared__ uint32_t cand_all[kSelThreads / 32][topk::kCand];
  __shared__ float q_all[kSelThreads / 32][kDP];
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int n = *fb_count;
  for (int i = blockIdx.x * (kSelThreads / 32) + w; i < n; i += gridDim.x * (kSelThreads / 32)) {
    const int row = fb_rows[i];
    const int bh = row / nb;
    __syncwarp();
    for (int d = lane; d < D; d += 32) q_all[w][d] = __ldg(qp + static_cast<long long>(row) * D + d);
    __syncwarp();
    const float* kbase = kp + static_cast<long long>(bh) * nb * D;
    uint32_t key[PL];
#pragma unroll
    for (int e = 0; e < PL; ++e) {
      const int j = lane + 32 * e;
      key[e] = j < nb ? topk::ordered_key(exact_score(q_all[w], kbase + static_cast<long long>(j) * D, D)) : 0u;
    }
    const int taken = topk::select_emit<PL>(key, nb, k, lane, hist_all[w], cand_all[w],
                                            idx + static_cast<long long>(row) * k);
    if (lane == 0 && taken != k) atomicCAS(&g_route_err, 0, 411);
  }
}

}  // namespace route

// Scratch layout: bf16 pairs [4][rows][128] | norms [2][rows] | per-head max key norm [BH] and the
// fallback row count (zeroed together) | fallback row list [rows] | keys [rows][round_up(nb, 8)].
namespace {
int64_t up256(int64_t b) { return (b + 255) & ~int64_t(255); }
}  // namespace

int64_t route_scratch_bytes(int BH, int nb) {
  const int64_t rows = static_cast<int64_t>(BH) * nb;
  const int64_t ldk = (static_cast<int64_t>(nb) + 7) & ~int64_t(7);
  return up256(4 * rows * route::kDP * 2) + up256(2 * rows * 4) + up256((static_cast<int64_t>(BH) + 4) * 4) +
         up256(rows * 4) + up256(rows * ldk * 2);
}

bool route_supported(int nb, int D) { return nb >= 1 && nb <= 3072 && D >= 8 && D <= 128 && D % 8 == 0; }

namespace {
struct RouteLayout {
  __nv_bfloat16* hl;
  float* nrm;
  float* nkmax;  // [BH], then the fallback-row count
  int* fb_count;
  int* fb_rows;
  uint16_t* keys;
};
RouteLayout route_layout(void* scratch, int BH, int nb) {
  const int64_t rows = static_cast<int64_t>(BH) * nb;
  RouteLayout l;
  uint8_t* base = static_cast<uint8_t*>(scratch);
  l.hl = reinterpret_cast<__nv_bfloat16*>(base);
  base += up256(4ll * rows * route::kDP * 2);
  l.nrm = reinterpret_cast<float*>(base);
  base += up256(2ll * rows * 4);
  l.nkmax = reinterpret_cast<float*>(base);
  l.fb_count = reinterpret_cast<int*>(l.nkmax + BH);
  base += up256((static_cast<int64_t>(BH) + 4) * 4);
  l.fb_rows = reinterpret_cast<int*>(base);
  base += up256(rows * 4);
  l.keys = reinterpret_cast<uint16_t*>(base);
  return l;
}
}  // namespace

int route_split_targets(void* scratch, int BH, int nb, __nv_bfloat16** hl, float** nrm, float** nkmax,
                        cudaStream_t stream) {
  const RouteLayout l = route_layout(scratch, BH, nb);
  *hl = l.hl;
  *nrm = l.nrm;
  *nkmax = l.nkmax;
  return cudaMemsetAsync(l.nkmax, 0, (static_cast<size_t>(BH) + 4) * 4, stream) == cudaSuccess ? BSA_OK
                                                                                                : BSA_ERR_CUDA;
}

int launch_route(const RouteArgs& a, cudaStream_t stream) {
  using namespace route;
  if (!route_supported(a.nb, a.D) || !a.scratch) return BSA_ERR_SHAPE;
  const int rows = a.BH * a.nb;
  const int64_t ldk = (static_cast<int64_t>(a.nb) + 7) & ~int64_t(7);
  const RouteLayout lay = route_layout(a.scratch, a.BH, a.nb);
  __nv_bfloat16* hl = lay.hl;
  float* nrm = lay.nrm;
  float* nkmax = lay.nkmax;
  int* fb_count = lay.fb_count;
  int* fb_rows = lay.fb_rows;
  uint16_t* keys = lay.keys;
  int dev = 0, sms = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return BSA_ERR_CUDA;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  // 1. split (+ the per-head maximum key norm and the fallback count, which start at 0), unless the pool
  //    kernels did it
  if (!a.split_done) {
    if (cudaMemsetAsync(nkmax, 0, (static_cast<size_t>(a.BH) + 4) * 4, stream) != cudaSuccess) return BSA_ERR_CUDA;
    long long grid = (2ll * rows + 7) / 8;
    if (grid > static_cast<long long>(sms) * 16) grid = static_cast<long long>(sms) * 16;
    split_kernel<<<static_cast<unsigned>(grid), 256, 0, stream>>>(a.qp, a.kp, rows, a.nb, a.D, hl, nrm, nkmax);
  }
  // 2. keys: four 3-D maps (d, block, b*h) over the bf16 arrays, 64 x 128 boxes
  {
    CUtensorMap maps[4];
    for (int m = 0; m < 4; ++m) {
      const int rc = a.make_pair_map(&maps[m], hl + static_cast<long long>(m) * rows * kDP, a.nb, a.BH);
      if (rc) return rc;
    }
    static std::mutex mu;
    static bool configured[64] = {};
    {
      std::lock_guard<std::mutex> lock(mu);
      if (dev >= 64 || !configured[dev]) {
        if (cudaFuncSetAttribute(key_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kKeySmemBytes) != cudaSuccess)
          return BSA_ERR_CUDA;
        if (dev < 64) configured[dev] = true;
      }
    }
    // key-block steps split over gridDim.z CTAs when the (query tile, head) grid alone would leave SMs
    // idle or a large last wave: the split minimising waves x (steps + one A load) per CTA
    const int gx = (a.nb + kTile - 1) / kTile;
    int split = 1;
    long long best = -1;
    for (int z = 1; z <= gx && z <= 16; ++z) {
      const long long ctas = static_cast<long long>(gx) * a.BH * z;
      const long long cost = ((ctas + sms - 1) / sms) * ((gx + z - 1) / z + 1);
      if (best < 0 || cost < best) {
        best = cost;
        split = z;
      }
    }
    const dim3 grid(gx, a.BH, split);
    if (grid.y > 65535u) return BSA_ERR_SHAPE;
    key_kernel<<<grid, kKeyThreads, kKeySmemBytes, stream>>>(maps[0], maps[1], maps[2], maps[3], a.nb,
                                                             static_cast<int>(ldk), keys);
  }
  // 3. select (grid: as many CTAs as fit on the SMs), then the exact full-row path for the rows the
  //    band could not settle
  {
    const int words = (a.nb + 63) / 64;
    const int sel_smem = kSelWarps * sel_warp_bytes(words);
    // the attribute only grows (a concurrent launch with a larger row never sees it lowered); the
    // occupancy of the last row length is kept per device
    static std::mutex mu;
    static int attr_bytes[64] = {}, occ_bytes[64] = {}, occ_ctas[64] = {};
    int per_sm = 0;
    {
      std::lock_guard<std::mutex> lock(mu);
      const bool cached = dev < 64 && occ_bytes[dev] == sel_smem;
      if (dev >= 64 || attr_bytes[dev] < sel_smem) {
        if (cudaFuncSetAttribute(select_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, sel_smem) != cudaSuccess)
          return BSA_ERR_CUDA;
        if (dev < 64) attr_bytes[dev] = sel_smem;
      }
      if (cached) {
        per_sm = occ_ctas[dev];
      } else {
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, select_kernel, kSelThreads, sel_smem) !=
                cudaSuccess ||
            per_sm < 1)
          return BSA_ERR_CUDA;
        if (dev < 64) {
          occ_bytes[dev] = sel_smem;
          occ_ctas[dev] = per_sm;
        }
      }
    }
    long long grid = (static_cast<long long>(rows) + kSelWarps - 1) / kSelWarps;
    if (grid > static_cast<long long>(sms) * per_sm) grid = static_cast<long long>(sms) * per_sm;
    select_kernel<<<static_cast<unsigned>(grid), kSelThreads, sel_smem, stream>>>(
        keys, static_cast<int>(ldk), a.qp, a.kp, nrm, nkmax, rows, a.nb, a.D, a.topk, a.idx, fb_count, fb_rows);
    const unsigned fgrid = static_cast<unsigned>(sms) * 2;
    if (a.nb <= 64 * 24)
      fallback_kernel<48><<<fgrid, kSelThreads, 0, stream>>>(a.qp, a.kp, a.nb, a.D, a.topk, a.idx, fb_count, fb_rows);
    else
      fallback_kernel<96><<<fgrid, kSelThreads, 0, stream>>>(a.qp, a.kp, a.nb, a.D, a.topk, a.idx, fb_count, fb_rows);
  }
  return cudaGetLastError() == cudaSuccess ? BSA_OK : BSA_ERR_CUDA;
}

int route_device_error(int clear) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_route_err, sizeof(int)) != cudaSuccess) return BSA_ERR_CUDA;
  if (clear && v) {
    int z = 0;
    cudaMemcpyToSymbol(g_route_err, &z, sizeof(int));
  }
  return v;
}

}  // namespace bsa
