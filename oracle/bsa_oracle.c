/*
 * CPU restatement of the BSA routing arithmetic -- TEST INFRASTRUCTURE ONLY (the checker, never
 * the product).  Built by oracle/bsa_oracle.py:build_oracle_lib() with gcc -ffp-contract=off so
 * that each operation below is one IEEE-754 fp32 operation with round-to-nearest-even.
 *
 * Reference semantics (xocialize/longcat-video-mlx):
 *   oracle_pool   -- mean_pool_blocks_3d, longcat_video/models/block_sparse_attention.py:67-104
 *   oracle_scores -- block_routing_scores, block_sparse_attention.py:107-112
 *   oracle_topk   -- topk_block_indices, block_sparse_attention.py:115-134 (selection rule made
 *                    explicit: score descending, then block id ascending; output ascending ids)
 *
 * The reference leaves the fp32 summation order to MLX; the engine fixes one and this file
 * restates exactly that order so indices can be compared bit-exactly:
 *   pooling: pairwise tree over the n tokens of a block in token order, ((r0 + r1) + (r2 + r3)) + ...,
 *            then * (1/n)
 *   scores : one fma chain per score, acc = fmaf(q[d], k[d], acc) for d = 0..D-1, acc0 = 0
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

/* x: [BH, S, D] fp32 t-major over the (T, Hl, Wl) grid; out: [BH, nb, D] */
void oracle_pool(const float* x, int BH, int S, int D, int T, int Hl, int Wl, int cT, int cH, int cW, float* out) {
  const int n = cT * cH * cW;
  const int Bh = Hl / cH, Bw = Wl / cW, Bt = T / cT;
  const int nb = Bt * Bh * Bw;
  float* buf = (float*)malloc(sizeof(float) * (size_t)n);
  (void)S;
  for (int bh = 0; bh < BH; ++bh) {
    for (int blk = 0; blk < nb; ++blk) {
      const int bt = blk / (Bh * Bw), bhh = (blk / Bw) % Bh, bw = blk % Bw;
      for (int d = 0; d < D; ++d) {
        for (int r = 0; r < n; ++r) {
          const int ct = r / (cH * cW), ch = (r / cW) % cH, cw = r % cW;
          const long tok = ((long)(bt * cT + ct) * Hl + (bhh * cH + ch)) * Wl + (bw * cW + cw);
          buf[r] = x[((long)bh * S + tok) * D + d];
        }
        /* pairwise tree over adjacent rows: (r0 + r1), (r2 + r3), ... then pairs of those */
        for (int stride = 1; stride < n; stride *= 2)
          for (int r = 0; r + stride < n; r += 2 * stride) buf[r] = buf[r] + buf[r + stride];
        out[((long)bh * nb + blk) * D + d] = buf[0] * (1.0f / (float)n);
      }
    }
  }
  free(buf);
}

/* qb: [BH, nq, D], kb: [BH, nk, D] -> score: [BH, nq, nk] */
void oracle_scores(const float* qb, const float* kb, int BH, int nq, int nk, int D, float* score) {
  for (int bh = 0; bh < BH; ++bh)
    for (int i = 0; i < nq; ++i) {
      const float* q = qb + ((long)bh * nq + i) * D;
      for (int j = 0; j < nk; ++j) {
        const float* k = kb + ((long)bh * nk + j) * D;
        float acc = 0.0f;
        for (int d = 0; d < D; ++d) acc = fmaf(q[d], k[d], acc);
        score[((long)bh * nq + i) * nk + j] = acc;
      }
    }
}

/* order-preserving key: larger score -> larger key; -0 == +0; NaN lowest */
static uint32_t okey(float s) {
  uint32_t u;
  if (s != s) return 0u;
  if (s == 0.0f) s = 0.0f;
  memcpy(&u, &s, 4);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

/* score: [rows, nk] -> idx: [rows, k] ascending block ids of the k largest (ties: smaller id) */
void oracle_topk(const float* score, int rows, int nk, int k, int32_t* idx) {
  uint32_t* keys = (uint32_t*)malloc(sizeof(uint32_t) * (size_t)nk);
  for (int r = 0; r < rows; ++r) {
    const float* s = score + (long)r * nk;
    for (int j = 0; j < nk; ++j) keys[j] = okey(s[j]);
    /* k-th largest key by counting: smallest key T with #(key > T) < k <= #(key >= T) */
    /* binary search over the 32-bit key space */
    uint32_t lo = 0, hi = 0xFFFFFFFFu; /* answer in [lo, hi] */
    while (lo < hi) {
      const uint32_t mid = lo + (hi - lo) / 2 + 1; /* upper mid */
      int ge = 0;
      for (int j = 0; j < nk; ++j) ge += keys[j] >= mid;
      if (ge >= k) lo = mid; else hi = mid - 1;
    }
    const uint32_t T = lo;
    int gt = 0;
    for (int j = 0; j < nk; ++j) gt += keys[j] > T;
    int need = k - gt, taken = 0;
    for (int j = 0; j < nk; ++j) {
      if (keys[j] > T) idx[(long)r * k + taken++] = j;
      else if (keys[j] == T && need > 0) { idx[(long)r * k + taken++] = j; --need; }
    }
  }
  free(keys);
}
