// Top-k selection from order-preserving 32-bit keys held in registers, one warp per row (shared by the
// top-k kernel of bsa_score.cu and the routing kernels of bsa_route.cu).
//
// Rule (topk_block_indices, block_sparse_attention.py:115-134, with the tie rule the reference leaves
// open): the k largest keys, ties to the smaller index, indices written in ascending order.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

namespace bsa {
namespace topk {

__device__ __forceinline__ uint32_t ordered_key(float s) {
  // -0.0 and +0.0 are one score; NaN sorts below every number (key 1); key 0 marks padding
  if (s != s) return 1u;
  const uint32_t u = __float_as_uint(s == 0.0f ? 0.0f : s);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}


constexpr int kCand = 64;  // threshold candidates kept after the first radix digit

// One radix digit (up to 8 bits below `shift`) over NK keys per lane: histogram of the keys that
// match `prefix` above `shift`, then the digit whose bin holds the need-th largest key.  Updates
// shift, prefix and need (keys still to take at or below the new prefix); `bincnt` receives the
// count of the chosen bin (after the last digit: the number of keys equal to the threshold).
template <int NK>
__device__ __forceinline__ void radix_pass(const uint32_t (&key)[NK], uint32_t* h, int lane, int& shift,
                                           uint32_t& prefix, int& need, uint32_t& bincnt) {
  const int w = shift < 8 ? shift : 8;
  const int hi_bits = shift;  // keys must match `prefix` above bit `shift`
  shift -= w;
  const uint32_t dmask = (1u << w) - 1u;
  reinterpret_cast<uint4*>(h)[lane * 2] = make_uint4(0u, 0u, 0u, 0u);
  reinterpret_cast<uint4*>(h)[lane * 2 + 1] = make_uint4(0u, 0u, 0u, 0u);
  __syncwarp();
#pragma unroll
  for (int e = 0; e < NK; ++e) {
    const uint32_t u = key[e];
    const bool match = u != 0u && (hi_bits >= 32 || (u >> hi_bits) == (prefix >> hi_bits));
    if (match) atomicAdd(&h[(u >> shift) & dmask], 1u);
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
  uint32_t gt = 0, bc = 0;
  if (mine) {
    uint32_t run = above;
#pragma unroll
    for (int b = 7; b >= 0; --b) {
      if (run + cnt[b] >= static_cast<uint32_t>(need)) {
        digit = lane * 8 + b;
        gt = run;
        bc = cnt[b];
        break;
      }
      run += cnt[b];
    }
  }
  const int src = __ffs(__ballot_sync(0xffffffffu, mine)) - 1;
  digit = __shfl_sync(0xffffffffu, digit, src);
  gt = __shfl_sync(0xffffffffu, gt, src);
  bincnt = __shfl_sync(0xffffffffu, bc, src);
  prefix |= static_cast<uint32_t>(digit) << shift;
  need -= static_cast<int>(gt);
  __syncwarp();
}


// The k-th largest of the row's keys (key[e] belongs to index lane + 32e; keys of 0 are padding).
// Returns it; need receives how many keys equal to it belong to the k largest, eqc how many keys equal
// it.  h: a per-warp 256-word shared histogram, cand: a per-warp list of kCand words.
//
// Radix select: 8-bit digits, starting below the bits that every key of the row shares (from the row's
// min and max key), counted in the per-warp histogram.  After the first digit only the keys of the
// chosen bin can still be the threshold; for rows of up to 48 keys per lane with at most kCand such
// keys, they are compacted (in index order) and the later digits run on those alone.
template <int PL>
__device__ __forceinline__ uint32_t kth_largest(const uint32_t (&key)[PL], int nk, int k, int lane, uint32_t* h,
                                                uint32_t* cand, int& need, uint32_t& eqc) {
  uint32_t kmin = 0xffffffffu, kmax = 0u;
#pragma unroll
  for (int e = 0; e < PL; ++e) {
    if (key[e] != 0u) {
      kmin = min(kmin, key[e]);
      kmax = max(kmax, key[e]);
    }
  }
  kmin = __reduce_min_sync(0xffffffffu, kmin);
  kmax = __reduce_max_sync(0xffffffffu, kmax);
  int shift = 32 - __clz(kmin ^ kmax);  // low bits that still vary across the row
  uint32_t prefix = shift >= 32 ? 0u : (kmax & ~((1u << shift) - 1u));
  need = k;
  eqc = static_cast<uint32_t>(nk);  // every key is equal when no bit varies
  if (shift > 0) {
    radix_pass<PL>(key, h, lane, shift, prefix, need, eqc);
    if (PL <= 48 && shift > 0 && eqc <= static_cast<uint32_t>(kCand)) {  // measured: no gain at 96 keys
      const uint32_t lt = (1u << lane) - 1u;
      int pos = 0;
#pragma unroll
      for (int e = 0; e < PL; ++e) {
        const uint32_t u = key[e];
        const bool m = u != 0u && (u >> shift) == (prefix >> shift);
        const uint32_t mb = __ballot_sync(0xffffffffu, m);
        if (m) cand[pos + __popc(mb & lt)] = u;
        pos += __popc(mb);
      }
      __syncwarp();
      uint32_t ck[kCand / 32];
#pragma unroll
      for (int c = 0; c < kCand / 32; ++c) ck[c] = lane + 32 * c < pos ? cand[lane + 32 * c] : 0u;
      __syncwarp();
      while (shift > 0) radix_pass<kCand / 32>(ck, h, lane, shift, prefix, need, eqc);
    } else {
      while (shift > 0) radix_pass<PL>(key, h, lane, shift, prefix, need, eqc);
    }
  }
  return prefix;
}

// The k largest of the row's keys written to out[0..k) in ascending index order (ties to the smaller
// index).  Returns the number of indices written (k unless the keys are inconsistent).
template <int PL>
__device__ __forceinline__ int select_emit(const uint32_t (&key)[PL], int nk, int k, int lane, uint32_t* h,
                                           uint32_t* cand, int32_t* out) {
  int need;
  uint32_t eqc;
  const uint32_t T = kth_largest<PL>(key, nk, k, lane, h, cand, need, eqc);
  const uint32_t lt_mask = (1u << lane) - 1u;
  int taken = 0, ties = 0;
  if (need == static_cast<int>(eqc)) {
    // every key equal to T is taken: one ballot per 32 keys
#pragma unroll
    for (int e = 0; e < PL; ++e) {
      if (32 * e >= nk) break;  // warp-uniform
      const int j = lane + 32 * e;
      const bool sel = j < nk && key[e] >= T;
      const uint32_t sb = __ballot_sync(0xffffffffu, sel);
      if (sel) out[taken + __popc(sb & lt_mask)] = j;
      taken += __popc(sb);
    }
  } else {
#pragma unroll
    for (int e = 0; e < PL; ++e) {
      if (32 * e >= nk) break;  // warp-uniform
      const int j = lane + 32 * e;
      const uint32_t u = key[e];
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
  return taken;
}

}  // namespace topk
}  // namespace bsa
