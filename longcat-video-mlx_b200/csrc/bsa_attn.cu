// Block-sparse attention forward on sm_100a (tcgen05 + TMA + TMEM).
//
// Semantics: reference Tier B kernels (longcat_video/models/block_sparse_attention_metal.py:75-164
// and the phase 2-4 bodies) -- for every query block, an fp32 online softmax over exactly the
// tokens of its selected key/value blocks, then out = o / l (0 when l == 0, :160-163).
//
// Formulation (B200-first, not a translation): the 64 query rows of one block are the N side
// of the MMA, two selected 64-token KV blocks are stacked on the M side, so every MMA is the
// full-rate M=128 shape:
//     S^T[128 kv x 64 q]  = Kpair[128 x D] . Q^T          (A = K, K-major; B = Q, K-major)
//     O^T[128 d  x 64 q] += Vpair^T[D x 128] . P^T        (A = V^T, MN-major; B = P^T, MN-major)
// Both accumulators live in TMEM; O^T is split into two accumulation chains (one per KV block)
// so consecutive PV MMAs do not wait on each other.
//
// Softmax: column-wise (per query) online softmax with a lazy running max.  A softmax group (4
// warps, one per TMEM lane quarter) owns 16 query columns; every thread forms
// x = S*scale*log2(e) - m with one FMA against the group's running maxima; the max is only raised
// (and O^T / the row sums rescaled) when some x exceeds 2^8, which one predicate-OR barrier per
// step detects.  Row sums stay per thread and are reduced once per query block.
//
// The kernel needs every (q-block, kv-block) pair's own 32 KB of K and V from L2, so the roles
// are decoupled so that no load waits behind an unrelated one:
//   warp 0      : Q tiles (two buffers) + K pairs (3-slot ring of 32 KB pairs, a slot is freed when its
//                 QK completes)
//   warp 1      : QK^T MMA issuer (one thread)
//   warp 2      : V blocks (4-slot ring of 16 KB blocks, a slot is freed when its PV completes)
//   warp 3      : PV MMA issuer (one thread)
//   warps 4-19  : softmax groups 0..3 -- query columns 16g..16g+15 (thread t <-> TMEM lane t); P^T is
//                 double-buffered so the softmax of step g+1 does not wait for the PV of step g, and
//                 each softmax warp arrives once (after a warp sync) on the hand-off barriers
// One CTA per SM, persistent over (head, q-block) units in head-major order so a head's K/V stays
// resident in L2.  Every mbarrier wait is bounded (bsa_ptx.cuh); a timeout records an error code
// and the CTA winds down.
#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>
#include "bsa_ptx.cuh"
#include "bsa_kernels.h"

namespace bsa {

namespace attn {
constexpr int kBlock = 64;                          // tokens per block
constexpr int kDP = 128;                            // head dim in shared memory (zero padded)
#ifndef BSA_KSTAGES
#define BSA_KSTAGES 3
#endif
#ifndef BSA_VSLOTS
#define BSA_VSLOTS 4
#endif
#ifndef BSA_QBUFS
#define BSA_QBUFS 2
#endif
constexpr int kKStages = BSA_KSTAGES;               // K pairs
constexpr int kQBufs = BSA_QBUFS;                   // Q tiles (2: the next unit's Q loads early)
constexpr int kVSlots = BSA_VSLOTS;                 // V single blocks
constexpr int kQBytes = kBlock * kDP * 2;           // 16 KB
constexpr int kPBytes = 2 * kBlock * 64 * 2;        // 16 KB: P^T [128 kv][64 q] (two buffers)
constexpr int kPairBytes = 2 * kBlock * kDP * 2;    // 32 KB: K of a block pair
constexpr int kVBlockBytes = kBlock * kDP * 2;      // 16 KB: V of one block
constexpr int kOffQ = 0;
constexpr int kOffP = kOffQ + kQBufs * kQBytes;
constexpr int kOffK = kOffP + 2 * kPBytes;
constexpr int kOffV = kOffK + kKStages * kPairBytes;
constexpr int kTileBytes = kOffV + kVSlots * kVBlockBytes;
#ifndef BSA_GROUP_COLS
#define BSA_GROUP_COLS 16
#endif
constexpr int kCols = BSA_GROUP_COLS;               // query columns per softmax group
constexpr int kGroups = 64 / kCols;                 // softmax groups (4 warps each)
constexpr int kSoftmaxThreads = 128 * kGroups;
constexpr int kThreads = 128 + kSoftmaxThreads;
static_assert(kCols == 16 || kCols == 32, "softmax group width");
constexpr float kRescaleThreshold = 8.0f;           // log2 units: P <= 2^8 between rescales

// TMEM columns: S^T double buffer (64 columns each), O^T in two KV-block halves (64 columns each).
// A softmax group owns 32 of the 64 columns of each.
constexpr uint32_t kTmemCols = 256;
__host__ __device__ constexpr uint32_t col_s(int buf) { return buf * 64; }
constexpr uint32_t kColO = 128;

struct SmallSmem {
  uint64_t k_full[kKStages];
  uint64_t k_empty[kKStages];
  uint64_t v_full[kVSlots];
  uint64_t v_empty[kVSlots];
  uint64_t s_full[2];     // QK issuer -> softmax: S^T ready
  uint64_t s_empty[2];    // softmax -> QK issuer: S^T read (one arrival per softmax warp)
  uint64_t p_full[2];     // softmax -> PV issuer: P^T of step g written into buffer g%2 (one per warp)
  uint64_t p_empty[2];    // PV issuer -> softmax: PV of step g done (buffer g%2 free, O^T up to date)
  uint64_t q_full[2];
  uint64_t q_empty[2];
  uint64_t o_empty;       // softmax -> PV issuer: O^T read by the epilogue (one arrival per softmax warp)
  uint64_t drain[2];
  uint32_t tmem_base;
  int abort_flag;
  alignas(16) float red[4][64];  // per-warp column partials (max on the slow path, sums at the end)
  alignas(16) float colv[64];    // per-column broadcast (max shift on the slow path, 1/l at the end)
  alignas(16) float mcol[64];    // running max per query column (log2 domain)
};
// The whole 227 KB opt-in: tiles, small state, and what is left as slack to align the tiles to
// 1024 bytes (checked at run time against the actual dynamic shared-memory base).
constexpr int kSmemBytes = 232448;
constexpr int kAlignSlack = kSmemBytes - kTileBytes - static_cast<int>(sizeof(SmallSmem));
static_assert(kAlignSlack >= 0, "tiles and small state fit in 227 KB");

struct Params {
  const int32_t* idx;   // [BH, nqb, topk]
  void* out;            // [B,H,S,D] with the strides below (elements)
  int BH, H, nqb, topk, nsteps, D;
  int Hl, Wl, cT, cH, cW, Bh, Bw;
  long long out_sb, out_sh, out_ss;
  float scale_log2;
  int total_units;
};

__device__ int g_attn_err;

#ifdef BSA_PROFILE
// Profiling builds only: per CTA and warp, cycles spent in up to 7 wait sites + the role's total.
__device__ long long g_bsa_prof[1024][24][8];
#define PACC(i) (&pacc[i])
#define PTS_START() pts_last = clock64()
#define PTS(i)                        \
  do {                                \
    const long long now_ = clock64(); \
    pacc[i] += now_ - pts_last;       \
    pts_last = now_;                  \
  } while (0)
#else
#define PACC(i) nullptr
#define PTS_START() \
  do {              \
  } while (0)
#define PTS(i) \
  do {         \
  } while (0)
#endif

__device__ __forceinline__ void block_origin(const Params& p, int b, int& t0, int& h0, int& w0) {
  const int per_t = p.Bh * p.Bw;
  const int bt = b / per_t;
  const int r = b - bt * per_t;
  const int bh = r / p.Bw;
  const int bw = r - bh * p.Bw;
  t0 = bt * p.cT;
  h0 = bh * p.cH;
  w0 = bw * p.cW;
}

__device__ __forceinline__ void named_bar_sync(int id, int n) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory");
}

// barrier over `n` threads on barrier `id` that also ORs a predicate across them
__device__ __forceinline__ int named_bar_or(int id, int n, int pred) {
  int r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.b32 p, %3, 0;\n\t"
      "bar.red.or.pred q, %1, %2, p;\n\t"
      "selp.b32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"(id), "r"(n), "r"(pred)
      : "memory");
  return r;
}

// Transposed warp reduction over N columns (N = 16 or 32): lane L holds v[0..N-1] (one value per
// column) for its own key row; afterwards lane L holds the reduction over all 32 lanes of column
// L % N.  N-1 shuffles halve the columns held per lane; for N < 32 the remaining lane halves are
// then combined.
template <bool kMax, int N>
__device__ __forceinline__ float transpose_reduce(float (&v)[N], int lane) {
#pragma unroll
  for (int lvl = N / 2; lvl >= 1; lvl >>= 1) {
    const bool up = (lane & lvl) != 0;
#pragma unroll
    for (int i = 0; i < lvl; ++i) {
      const float send = up ? v[i] : v[i + lvl];
      const float keep = up ? v[i + lvl] : v[i];
      const float recv = __shfl_xor_sync(0xffffffffu, send, lvl);
      v[i] = kMax ? fmaxf(keep, recv) : keep + recv;
    }
  }
  float r = v[0];
#pragma unroll
  for (int off = N; off < 32; off <<= 1) {
    const float o = __shfl_xor_sync(0xffffffffu, r, off);
    r = kMax ? fmaxf(r, o) : r + o;
  }
  return r;
}

// Block ids of step j of a unit (the second id duplicates the first for an odd tail; those rows
// are masked in the softmax).  Out-of-range ids are reported and replaced by block 0.
__device__ __forceinline__ void step_blocks(const int32_t* idx, int j, int k, int nb, int* err, int& b0, int& b1) {
  b0 = __ldg(idx + 2 * j);
  b1 = (2 * j + 1 < k) ? __ldg(idx + 2 * j + 1) : b0;
  if (static_cast<unsigned>(b0) >= static_cast<unsigned>(nb) || static_cast<unsigned>(b1) >= static_cast<unsigned>(nb)) {
    atomicCAS(err, 0, BSA_ERR_INDEX);
    b0 = static_cast<unsigned>(b0) >= static_cast<unsigned>(nb) ? 0 : b0;
    b1 = static_cast<unsigned>(b1) >= static_cast<unsigned>(nb) ? 0 : b1;
  }
}

template <bool kBF16>
__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  return kBF16 ? pack_bf16x2(lo, hi) : pack_f16x2(lo, hi);
}

template <bool kBF16>
__global__ void __launch_bounds__(kThreads, 1)
    bsa_attn_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                    const __grid_constant__ CUtensorMap tm_v, const Params p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  const uint32_t pad = (1024u - (smem_u32(smem_raw) & 1023u)) & 1023u;
  if (pad > static_cast<uint32_t>(kAlignSlack)) {  // uniform across the CTA: nothing is set up yet
    if (threadIdx.x == 0) atomicCAS(&g_attn_err, 0, 199);
    return;
  }
  uint8_t* smem = smem_raw + pad;
  uint8_t* sQ = smem + kOffQ;
  uint8_t* sP = smem + kOffP;
  uint8_t* sK = smem + kOffK;
  uint8_t* sV = smem + kOffV;
  SmallSmem& ss = *reinterpret_cast<SmallSmem*>(smem + kTileBytes);

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;

  if (tid == 0) {
    for (int s = 0; s < kKStages; ++s) {
      mbar_init(&ss.k_full[s], 1);
      mbar_init(&ss.k_empty[s], 1);
    }
    for (int s = 0; s < kVSlots; ++s) {
      mbar_init(&ss.v_full[s], 1);
      mbar_init(&ss.v_empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&ss.s_full[i], 1);
      mbar_init(&ss.s_empty[i], kSoftmaxThreads / 32);
      mbar_init(&ss.q_full[i], 1);
      mbar_init(&ss.q_empty[i], 1);
      mbar_init(&ss.drain[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&ss.p_full[i], kSoftmaxThreads / 32);
      mbar_init(&ss.p_empty[i], 1);
    }
    mbar_init(&ss.o_empty, kSoftmaxThreads / 32);
    ss.abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(&ss.tmem_base, kTmemCols);
    tmem_relinquish();
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = ss.tmem_base;
#ifdef BSA_PROFILE
  const long long prof_t0 = clock64();
  long long pacc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  long long pts_last = 0;
#endif
  volatile int* abort_flag = &ss.abort_flag;
  int* err = &g_attn_err;

  const int G = gridDim.x;
  const int nsteps = p.nsteps;
  const int k = p.topk;

  if (warp == 0) {
    // ------------------------------------------------------------------ Q + K producer
    if (lane == 0) {
      prefetch_tmap(&tm_q);
      prefetch_tmap(&tm_k);
      long long g = 0;
      int n = 0;
      bool ok = true;
      for (int unit = blockIdx.x; unit < p.total_units && ok; unit += G, ++n) {
        const int bh = unit / p.nqb;
        const int qblk = unit - bh * p.nqb;
        const int32_t* idx = p.idx + (static_cast<long long>(bh) * p.nqb + qblk) * k;
        int nb0, nb1;
        step_blocks(idx, 0, k, p.nqb, err, nb0, nb1);
        const int qb = n % kQBufs;
        if (n >= kQBufs) ok = mbar_wait(&ss.q_empty[qb], ((n - kQBufs) / kQBufs) & 1, abort_flag, err, 101, PACC(0));
        if (!ok) break;
        {
          int t0, h0, w0;
          block_origin(p, qblk, t0, h0, w0);
          mbar_arrive_expect_tx(&ss.q_full[qb], kQBytes);
          uint8_t* dst = sQ + qb * kQBytes;
          tma_load_5d(dst, &tm_q, &ss.q_full[qb], 0, w0, h0, t0, bh);
          tma_load_5d(dst + kQBytes / 2, &tm_q, &ss.q_full[qb], 64, w0, h0, t0, bh);
        }
        for (int j = 0; j < nsteps && ok; ++j, ++g) {
          const int b0 = nb0, b1 = nb1;
          if (j + 1 < nsteps) step_blocks(idx, j + 1, k, p.nqb, err, nb0, nb1);  // prefetch next ids
          const int ks = static_cast<int>(g % kKStages);
          if (g >= kKStages)
            ok = mbar_wait(&ss.k_empty[ks], static_cast<uint32_t>((g / kKStages - 1) & 1), abort_flag, err, 102,
                           PACC(1));
          if (!ok) break;
          uint8_t* dst = sK + ks * kPairBytes;
          mbar_arrive_expect_tx(&ss.k_full[ks], kPairBytes);
#pragma unroll
          for (int bi = 0; bi < 2; ++bi) {
            int t0, h0, w0;
            block_origin(p, bi ? b1 : b0, t0, h0, w0);
#pragma unroll
            for (int hh = 0; hh < 2; ++hh)
              tma_load_5d(dst + hh * 16384 + bi * 8192, &tm_k, &ss.k_full[ks], hh * 64, w0, h0, t0, bh);
          }
        }
      }
      // teardown: no TMA write into this CTA's shared memory may still be in flight
      const uint64_t t0 = globaltimer_ns();
      for (long long gg = (g > kKStages ? g - kKStages : 0); gg < g; ++gg)
        while (!mbar_try_wait(&ss.k_full[gg % kKStages], static_cast<uint32_t>((gg / kKStages) & 1)) &&
               globaltimer_ns() - t0 < kWaitLimitNs) {
        }
    }
    __syncwarp();
  } else if (warp == 2) {
    // ------------------------------------------------------------------ V producer
    if (lane == 0) {
      prefetch_tmap(&tm_v);
      long long gb = 0;  // V blocks issued
      bool ok = true;
      for (int unit = blockIdx.x; unit < p.total_units && ok; unit += G) {
        const int bh = unit / p.nqb;
        const int qblk = unit - bh * p.nqb;
        const int32_t* idx = p.idx + (static_cast<long long>(bh) * p.nqb + qblk) * k;
        int nb0, nb1;
        step_blocks(idx, 0, k, p.nqb, err, nb0, nb1);
        for (int j = 0; j < nsteps && ok; ++j) {
          const int b0 = nb0, b1 = nb1;
          if (j + 1 < nsteps) step_blocks(idx, j + 1, k, p.nqb, err, nb0, nb1);
#pragma unroll
          for (int bi = 0; bi < 2 && ok; ++bi, ++gb) {
            const int vs = static_cast<int>(gb % kVSlots);
            if (gb >= kVSlots)
              ok = mbar_wait(&ss.v_empty[vs], static_cast<uint32_t>((gb / kVSlots - 1) & 1), abort_flag, err, 103,
                             PACC(0));
            if (!ok) break;
            int t0, h0, w0;
            block_origin(p, bi ? b1 : b0, t0, h0, w0);
            uint8_t* dst = sV + vs * kVBlockBytes;
            mbar_arrive_expect_tx(&ss.v_full[vs], kVBlockBytes);
            tma_load_5d(dst, &tm_v, &ss.v_full[vs], 0, w0, h0, t0, bh);
            tma_load_5d(dst + kVBlockBytes / 2, &tm_v, &ss.v_full[vs], 64, w0, h0, t0, bh);
          }
        }
      }
      const uint64_t t0 = globaltimer_ns();
      for (long long gg = (gb > kVSlots ? gb - kVSlots : 0); gg < gb; ++gg)
        while (!mbar_try_wait(&ss.v_full[gg % kVSlots], static_cast<uint32_t>((gg / kVSlots) & 1)) &&
               globaltimer_ns() - t0 < kWaitLimitNs) {
        }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------------ QK^T issuer
    if (lane == 0) {
      const uint32_t idesc = idesc_f16(128, 64, kBF16 ? 1 : 0, 0, 0);
      long long g = 0;
      int n = 0;
      bool ok = true;
      for (int unit = blockIdx.x; unit < p.total_units && ok; unit += G, ++n) {
        const int qb = n % kQBufs;
        const uint32_t qpar = static_cast<uint32_t>((n / kQBufs) & 1);
        for (int j = 0; j < nsteps && ok; ++j, ++g) {
          const int ks = static_cast<int>(g % kKStages);
          const int sb = static_cast<int>(g & 1);
          ok = mbar_wait(&ss.k_full[ks], static_cast<uint32_t>((g / kKStages) & 1), abort_flag, err, 113, PACC(0));
          if (ok && g >= 2)
            ok = mbar_wait(&ss.s_empty[sb], static_cast<uint32_t>(((g >> 1) - 1) & 1), abort_flag, err, 114, PACC(1));
          if (ok && j == 0) ok = mbar_wait(&ss.q_full[qb], qpar, abort_flag, err, 115, PACC(2));
          if (!ok) break;
          tc_fence_after();
          const uint32_t kb = smem_u32(sK + ks * kPairBytes);
          const uint32_t qbase = smem_u32(sQ + qb * kQBytes);
#pragma unroll
          for (int kk = 0; kk < 8; ++kk) {
            const int half = kk >> 2, i = kk & 3;
            const uint64_t ad = sdesc_sw128(kb + half * 16384 + i * 32, 16, 1024);
            const uint64_t bd = sdesc_sw128(qbase + half * 8192 + i * 32, 16, 1024);
            umma_ss(tmem + col_s(sb), ad, bd, idesc, kk > 0 ? 1u : 0u);
          }
          umma_commit(&ss.s_full[sb]);
          umma_commit(&ss.k_empty[ks]);
          if (j == nsteps - 1) umma_commit(&ss.q_empty[qb]);
        }
      }
      umma_commit(&ss.drain[0]);  // teardown: this thread's MMAs complete before TMEM is released
      const uint64_t t0 = globaltimer_ns();
      while (!mbar_try_wait(&ss.drain[0], 0) && globaltimer_ns() - t0 < kWaitLimitNs) {
      }
    }
    __syncwarp();
  } else if (warp == 3) {
    // ------------------------------------------------------------------ PV issuer
    if (lane == 0) {
      const uint32_t idesc = idesc_f16(128, 64, kBF16 ? 1 : 0, 1, 1);
      long long g = 0;
      int n = 0;
      bool ok = true;
      const uint32_t pbase = smem_u32(sP);
      for (int unit = blockIdx.x; unit < p.total_units && ok; unit += G, ++n) {
        for (int j = 0; j < nsteps && ok; ++j, ++g) {
          const long long gb0 = 2 * g;
          const int vs0 = static_cast<int>(gb0 % kVSlots);
          const int vs1 = static_cast<int>((gb0 + 1) % kVSlots);
          ok = mbar_wait(&ss.v_full[vs0], static_cast<uint32_t>((gb0 / kVSlots) & 1), abort_flag, err, 116, PACC(0));
          if (ok) ok = mbar_wait(&ss.v_full[vs1], static_cast<uint32_t>(((gb0 + 1) / kVSlots) & 1), abort_flag, err, 117, PACC(1));
          const int pb = static_cast<int>(g & 1);
          if (ok) ok = mbar_wait(&ss.p_full[pb], static_cast<uint32_t>((g >> 1) & 1), abort_flag, err, 111, PACC(2));
          if (ok && j == 0 && n >= 1) ok = mbar_wait(&ss.o_empty, static_cast<uint32_t>((n - 1) & 1), abort_flag, err, 112, PACC(3));
          if (!ok) break;
          tc_fence_after();
          const uint32_t vb0 = smem_u32(sV + vs0 * kVBlockBytes);
          const uint32_t vb1 = smem_u32(sV + vs1 * kVBlockBytes);
#pragma unroll
          for (int i = 0; i < 4; ++i) {
#pragma unroll
            for (int half = 0; half < 2; ++half) {
              const int kk = half * 4 + i;
              const uint64_t ad = sdesc_sw128((half ? vb1 : vb0) + i * 2048, kVBlockBytes / 2, 1024);
              const uint64_t bd = sdesc_sw128(pbase + pb * kPBytes + kk * 2048, 16384, 1024);
              umma_ss(tmem + kColO + half * 64, ad, bd, idesc, (j > 0 || i > 0) ? 1u : 0u);
            }
          }
          umma_commit(&ss.v_empty[vs0]);
          umma_commit(&ss.v_empty[vs1]);
          umma_commit(&ss.p_empty[pb]);
        }
      }
      umma_commit(&ss.drain[1]);
      const uint64_t t0 = globaltimer_ns();
      while (!mbar_try_wait(&ss.drain[1], 0) && globaltimer_ns() - t0 < kWaitLimitNs) {
      }
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------------ softmax groups
    {
      const int grp = (warp - 4) >> 2;        // group g owns query columns [g*kCols, (g+1)*kCols)
      const int wq = warp & 3;                // TMEM lane quarter
      const int t = wq * 32 + lane;           // TMEM lane == key row (S^T) == d row (O^T)
      const int c0 = grp * kCols;             // first query column of this group
      const int bar_id = 1 + grp;
      const uint32_t lane_base = static_cast<uint32_t>(wq * 32) << 16;
      const float scale_log2 = p.scale_log2;
      const bool odd_tail = (k & 1) != 0;
      long long g = 0;
      int n = 0;
      bool ok = true;
      for (int unit = blockIdx.x; unit < p.total_units && ok; unit += G, ++n) {
        const int bh = unit / p.nqb;
        const int qblk = unit - bh * p.nqb;
        // mcol[c0 + q]: running max of query column c0+q (log2 domain), shared by the group
        float l_part[kCols];
#pragma unroll
        for (int q = 0; q < kCols; ++q) l_part[q] = 0.f;
        if (t < kCols) ss.mcol[c0 + t] = 0.f;
        named_bar_sync(bar_id, 128);
        const float4* mvec = reinterpret_cast<const float4*>(&ss.mcol[c0]);
        for (int j = 0; j < nsteps && ok; ++j, ++g) {
          const int sb = static_cast<int>(g & 1);
          ok = mbar_wait(&ss.s_full[sb], static_cast<uint32_t>((g >> 1) & 1), abort_flag, err, 121, PACC(0));
          ok = __all_sync(0xffffffffu, ok);  // leave the loop warp-uniformly
          if (!ok) break;
          PTS_START();
          tc_fence_after();
          const bool masked = odd_tail && j == nsteps - 1 && t >= 64;
          float x[kCols];  // x = S*scale*log2e - m
          {
            uint32_t r[kCols];
            if (kCols == 32) tmem_ld32(tmem + lane_base + col_s(sb) + c0, r);
            else tmem_ld16(tmem + lane_base + col_s(sb) + c0, r);
            tmem_ld_wait();
#pragma unroll
            for (int q4 = 0; q4 < kCols / 4; ++q4) {
              const float4 mv = mvec[q4];
              const float mq[4] = {mv.x, mv.y, mv.z, mv.w};
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const int q = 4 * q4 + e;
                x[q] = masked ? -INFINITY : fmaf(__uint_as_float(r[q]), scale_log2, -mq[e]);
              }
            }
          }
          PTS(4);
          // ---- lazy running max: does any key of the group exceed m + threshold?
          float mx = x[0];
#pragma unroll
          for (int q = 1; q < kCols; ++q) mx = fmaxf(mx, x[q]);
          const int over = named_bar_or(bar_id, 128, (j == 0 || mx > kRescaleThreshold) ? 1 : 0);
          if (over) {
            // slow path (first step of a block, or a large jump of the max): exact column max,
            // reduced in place, then x is reloaded from TMEM (S is released only after this)
            const float cmax = transpose_reduce<true, kCols>(x, lane);
            if (lane < kCols) ss.red[wq][c0 + lane] = cmax;
            {
              uint32_t r[kCols];
              if (kCols == 32) tmem_ld32(tmem + lane_base + col_s(sb) + c0, r);
              else tmem_ld16(tmem + lane_base + col_s(sb) + c0, r);
              tmem_ld_wait();
#pragma unroll
              for (int q = 0; q < kCols; ++q)
                x[q] = masked ? -INFINITY : fmaf(__uint_as_float(r[q]), scale_log2, -ss.mcol[c0 + q]);
            }
            named_bar_sync(bar_id, 128);
            if (t < kCols) {
              const int c = c0 + t;
              const float cm = fmaxf(fmaxf(ss.red[0][c], ss.red[1][c]), fmaxf(ss.red[2][c], ss.red[3][c]));
              // shift of column c: the new max on the first step, else only when it jumps by > 2^8
              const float d = (j == 0 || cm > kRescaleThreshold) ? cm : 0.f;
              ss.colv[c] = d;
              ss.mcol[c] += d;
            }
            const int need = named_bar_or(bar_id, 128, (t < kCols && j > 0 && ss.colv[c0 + t] != 0.f) ? 1 : 0);
#pragma unroll
            for (int q = 0; q < kCols; ++q) x[q] -= ss.colv[c0 + q];
            if (need) {
              // O^T columns of this group must be rescaled: the previous step's PV must be complete
              ok = mbar_wait(&ss.p_empty[(g - 1) & 1], static_cast<uint32_t>(((g - 1) >> 1) & 1), abort_flag, err, 122,
                             PACC(3));
          ok = __all_sync(0xffffffffu, ok);  // leave the loop warp-uniformly
              if (!ok) break;
              tc_fence_after();
#pragma unroll
              for (int half = 0; half < 2; ++half) {
#pragma unroll
                for (int c = 0; c < kCols; c += 16) {
                  uint32_t r[16];
                  const uint32_t a = tmem + lane_base + kColO + half * 64 + c0 + c;
                  tmem_ld16(a, r);
                  tmem_ld_wait();
#pragma unroll
                  for (int q = 0; q < 16; ++q)
                    r[q] = __float_as_uint(__uint_as_float(r[q]) * ex2_approx(-ss.colv[c0 + c + q]));
                  tmem_st16(a, r);
                }
              }
              tmem_st_wait();
#pragma unroll
              for (int q = 0; q < kCols; ++q) l_part[q] *= ex2_approx(-ss.colv[c0 + q]);
            }
            named_bar_sync(bar_id, 128);  // colv is rewritten by the next slow path
          }
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&ss.s_empty[sb]);  // one arrival per warp
          PTS(5);
          // ---- probabilities, row-sum partials, P^T row into the P buffer
          uint32_t packed[kCols / 2];
#pragma unroll
          for (int q = 0; q < kCols; q += 2) {
            const float p0 = ex2_approx(x[q]);
            const float p1 = ex2_approx(x[q + 1]);
            l_part[q] += p0;
            l_part[q + 1] += p1;
            packed[q >> 1] = pack2<kBF16>(p0, p1);
          }
          PTS(6);
          if (g >= 2) {  // the PV of step g-2 must be done reading this P buffer
            ok = mbar_wait(&ss.p_empty[g & 1], static_cast<uint32_t>(((g - 2) >> 1) & 1), abort_flag, err, 124,
                           PACC(1));
          ok = __all_sync(0xffffffffu, ok);  // leave the loop warp-uniformly
            if (!ok) break;
          }
          uint8_t* sPg = sP + (g & 1) * kPBytes;
          PTS_START();
#pragma unroll
          for (int c = 0; c < kCols / 8; ++c) {
            const uint4 v = make_uint4(packed[4 * c], packed[4 * c + 1], packed[4 * c + 2], packed[4 * c + 3]);
            *reinterpret_cast<uint4*>(sPg + sw128_offset(static_cast<uint32_t>(t), static_cast<uint32_t>(c0 / 8 + c))) = v;
          }
          fence_proxy_async_smem();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&ss.p_full[g & 1]);
          PTS(3);
        }
        if (!ok) break;
        // ---- epilogue: row sums, O^T / l -> out (this group's query rows)
        {
          const float lsum = transpose_reduce<false, kCols>(l_part, lane);
          if (lane < kCols) ss.red[wq][c0 + lane] = lsum;
        }
        ok = mbar_wait(&ss.p_empty[(g - 1) & 1], static_cast<uint32_t>(((g - 1) >> 1) & 1), abort_flag, err, 123,
                       PACC(2));
          ok = __all_sync(0xffffffffu, ok);  // leave the loop warp-uniformly
        if (!ok) break;
        tc_fence_after();
        float o[kCols];
#pragma unroll
        for (int c = 0; c < kCols; c += 16) {
          uint32_t ra[16], rb[16];
          tmem_ld16(tmem + lane_base + kColO + c0 + c, ra);
          tmem_ld16(tmem + lane_base + kColO + 64 + c0 + c, rb);
          tmem_ld_wait();
#pragma unroll
          for (int q = 0; q < 16; ++q) o[c + q] = __uint_as_float(ra[q]) + __uint_as_float(rb[q]);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&ss.o_empty);
        named_bar_sync(bar_id, 128);
        if (t < kCols) {
          const int c = c0 + t;
          const float l = ss.red[0][c] + ss.red[1][c] + ss.red[2][c] + ss.red[3][c];
          ss.colv[c] = l > 0.f ? 1.f / l : 0.f;
        }
        named_bar_sync(bar_id, 128);
        if (t < p.D) {
          int t0, h0, w0;
          block_origin(p, qblk, t0, h0, w0);
          const int b = bh / p.H;
          const int h = bh - b * p.H;
          const long long base = b * p.out_sb + h * p.out_sh + t;
          const int cHW = p.cH * p.cW;
#pragma unroll
          for (int q = 0; q < kCols; ++q) {
            const int r = c0 + q;
            const int ct = r / cHW;
            const int rem = r - ct * cHW;
            const int ch = rem / p.cW;
            const int cw = rem - ch * p.cW;
            const long long tok = (static_cast<long long>(t0 + ct) * p.Hl + (h0 + ch)) * p.Wl + (w0 + cw);
            const float val = o[q] * ss.colv[r];
            if (kBF16)
              reinterpret_cast<__nv_bfloat16*>(p.out)[base + tok * p.out_ss] = __float2bfloat16_rn(val);
            else
              reinterpret_cast<__half*>(p.out)[base + tok * p.out_ss] = __float2half_rn(val);
          }
        }
        named_bar_sync(bar_id, 128);
      }
    }
  }
  // ------------------------------------------------------------------ teardown
#ifdef BSA_PROFILE
  pacc[7] = clock64() - prof_t0;
  if (lane == 0 && blockIdx.x < 1024)
    for (int i = 0; i < 8; ++i) g_bsa_prof[blockIdx.x][warp][i] = pacc[i];
#endif
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) tmem_dealloc(tmem, kTmemCols);
}

}  // namespace attn

// -------------------------------------------------------------------------------- host side
int launch_attn(const CUtensorMap* tm_q, const CUtensorMap* tm_k, const CUtensorMap* tm_v, const AttnArgs& a,
                cudaStream_t stream) {
  using namespace attn;
  static bool configured[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !configured[dev]) {
    if (cudaFuncSetAttribute(bsa_attn_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes) !=
            cudaSuccess ||
        cudaFuncSetAttribute(bsa_attn_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes) !=
            cudaSuccess)
      return BSA_ERR_CUDA;
    configured[dev] = true;
  }
  int sms = 0;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  Params p;
  p.idx = a.idx;
  p.out = a.out;
  p.BH = a.B * a.H;
  p.H = a.H;
  p.nqb = a.nb;
  p.topk = a.topk;
  p.nsteps = (a.topk + 1) / 2;
  p.D = a.D;
  p.Hl = a.Hl;
  p.Wl = a.Wl;
  p.cT = a.cT;
  p.cH = a.cH;
  p.cW = a.cW;
  p.Bh = a.Hl / a.cH;
  p.Bw = a.Wl / a.cW;
  p.out_sb = a.out_sb;
  p.out_sh = a.out_sh;
  p.out_ss = a.out_ss;
  p.scale_log2 = a.sm_scale * 1.4426950408889634f;
  p.total_units = p.BH * a.nb;
  int ctas = sms - a.sm_reserve;
  if (ctas < 1) ctas = 1;
  const int grid = p.total_units < ctas ? p.total_units : ctas;
  if (grid <= 0) return BSA_OK;
  if (a.is_bf16)
    bsa_attn_kernel<true><<<grid, kThreads, kSmemBytes, stream>>>(*tm_q, *tm_k, *tm_v, p);
  else
    bsa_attn_kernel<false><<<grid, kThreads, kSmemBytes, stream>>>(*tm_q, *tm_k, *tm_v, p);
  return cudaGetLastError() == cudaSuccess ? BSA_OK : BSA_ERR_CUDA;
}

#ifdef BSA_PROFILE
extern "C" int bsa_prof_read(long long* out, int clear) {
  (void)clear;
  if (cudaDeviceSynchronize() != cudaSuccess) return BSA_ERR_CUDA;
  if (cudaMemcpyFromSymbol(out, attn::g_bsa_prof, sizeof(attn::g_bsa_prof)) != cudaSuccess) return BSA_ERR_CUDA;
  return BSA_OK;
}
#endif

int attn_device_error(int clear) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, attn::g_attn_err, sizeof(int)) != cudaSuccess) return BSA_ERR_CUDA;
  if (clear && v) {
    int z = 0;
    cudaMemcpyToSymbol(attn::g_attn_err, &z, sizeof(int));
  }
  return v;
}

}  // namespace bsa
