// Block-sparse attention forward on sm_100a (tcgen05 + TMA + TMEM).
//
// Semantics: reference Tier B kernels (longcat_video/models/block_sparse_attention_metal.py:75-164
// and the phase 2-4 bodies) -- for every query block, an fp32 online softmax over exactly the
// tokens of its selected key/value blocks, then out = o / l (0 when l == 0, :160-163).
//
// Formulation: row-wise, M = 64 query rows, with both A operands in tensor memory so that shared
// memory carries only the K/V tiles (TMA writes + one MMA read each):
//     S[64 q x 128 kv]  = Q[64 x D] . Kpair^T        (A = Q in TMEM, B = K pair, K-major)
//     O[64 q x 128 d]  += P[64 x 128 kv] . Vpair      (A = P in TMEM, B = V pair, MN-major)
// An M = 64 accumulator occupies 16 of the 32 lanes of each TMEM lane quarter.  The two lane
// halves (lanes 0-15 and 16-31 of every quarter) hold two independent pipelines over the same
// columns: half 0 takes the even KV steps of a query block, half 1 the odd ones, each with its
// own Q copy, S, P (double buffered) and O, and its own running max.  The epilogue merges the
// two partial softmax states (m, l, O) of each row.
//
// Roles (384 threads, one CTA per SM, persistent over (head, q-block) units in head-major order so a
// head's K/V stays resident in L2):
//   warp 0      : Q tiles (two shared-memory buffers) + K pairs (ring of 2 x 32 KB pairs)
//   warp 1      : QK issuer (one thread), steps in order, S into the step's lane half
//   warp 2      : V blocks (ring of 8 x 16 KB blocks; V is consumed after the softmax, so it needs
//                 the deeper ring)
//   warp 3      : PV issuer (one thread)
//   warps 4-7   : softmax of lane half 0 (warp w <-> TMEM lane quarter w % 4; 16 rows each)
//   warps 8-11  : softmax of lane half 1
// Ring positions advance incrementally (RingPos): a 64-bit modulo per step on the single issuing
// threads cost 15 % at ring sizes that are not powers of two.
// A softmax thread owns half of one query row per step (64 keys): threads t and t+16 of a warp
// share a row, so the row max and row sum need one shuffle and no cross-warp barrier.  The max is
// lazy: it is raised (and O / l rescaled) only when a score exceeds it by more than 2^8.  The step
// body is kept small for the instruction cache: packed f32x2 arithmetic, and the rare or per-unit
// paths (O rescale, Q copy, epilogue stores, the spin of a wait) are out of line.
// Every mbarrier wait is bounded (bsa_ptx.cuh); a timeout records an error code and the CTA winds
// down.
#include <cstdint>
#include <mutex>
#include <cuda.h>
#include <cuda_runtime.h>
#include "bsa_ptx.cuh"
#include "bsa_kernels.h"

namespace bsa {

namespace attn {
constexpr int kBlock = 64;                          // tokens per block
constexpr int kDP = 128;                            // head dim in shared memory (zero padded)
#ifndef BSA_KSTAGES
#define BSA_KSTAGES 2
#endif
#ifndef BSA_VSLOTS
#define BSA_VSLOTS 8
#endif
constexpr int kKStages = BSA_KSTAGES;               // K pairs
constexpr int kVSlots = BSA_VSLOTS;                 // V single blocks
#ifndef BSA_QBUFS
#define BSA_QBUFS 2
#endif
constexpr int kQBufs = BSA_QBUFS;                   // Q tiles in shared memory (copied into TMEM once per unit)
constexpr int kQBytes = kBlock * kDP * 2;           // 16 KB
constexpr int kPairBytes = 2 * kBlock * kDP * 2;    // 32 KB: K of a block pair
constexpr int kVBlockBytes = kBlock * kDP * 2;      // 16 KB: V of one block
constexpr int kOffQ = 0;
constexpr int kOffK = kOffQ + kQBufs * kQBytes;
constexpr int kOffV = kOffK + kKStages * kPairBytes;
constexpr int kTileBytes = kOffV + kVSlots * kVBlockBytes;
constexpr int kSoftmaxWarps = 8;
constexpr int kThreads = 128 + 32 * kSoftmaxWarps;
constexpr float kRescaleThreshold = 8.0f;           // log2 units: P <= 2^8 between rescales

// TMEM columns, identical for both lane halves.
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColS = 0;                       // S: 128 fp32 columns
constexpr uint32_t kColO = 128;                     // O: 128 fp32 columns
__host__ __device__ constexpr uint32_t col_p(int b) { return 256u + 64u * static_cast<uint32_t>(b); }  // P: 64 x 2
constexpr uint32_t kColQ = 384;                     // Q: 64 columns (bf16/fp16 pairs)
__host__ __device__ constexpr uint32_t half_lanes(int h) { return static_cast<uint32_t>(16 * h) << 16; }

struct SmallSmem {
  uint64_t k_full[kKStages];
  uint64_t k_empty[kKStages];
  uint64_t v_full[kVSlots];
  uint64_t v_empty[kVSlots];
  uint64_t s_full[2];     // per half: QK issuer -> softmax, S ready
  uint64_t s_empty[2];    // per half: softmax -> QK issuer, S read (one arrival per warp of the half)
  uint64_t p_full[2][2];  // [half][buf]: softmax -> PV issuer, P written (one arrival per warp)
  uint64_t p_empty[2][2]; // [half][buf]: PV done (P buffer free, O of the half up to date)
  uint64_t q_full[kQBufs];   // TMA: Q tile landed in shared memory
  uint64_t q_empty[kQBufs];  // softmax warps: Q tile copied into TMEM (shared buffer free)
  uint64_t q_ready[2];       // per half: Q of the unit is in TMEM (one arrival per warp of the half)
  uint64_t o_empty;          // epilogue read O (one arrival per softmax warp)
  uint64_t ep[4];            // per lane quarter: both halves' row statistics written, their PVs done
  uint64_t drain[2];
  uint32_t tmem_base;
  int abort_flag;
  alignas(16) float st_m[2][2][64];  // [unit parity][half][row]: running max (log2 domain)
  alignas(16) float st_l[2][2][64];  // [unit parity][half][row]: row sum
};
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
  int vec_out;          // out rows may be written with 16-byte stores
  int map3;             // blocks are contiguous 64-token runs: q/k/v maps are 3-D (d, s, b*h)
};

__device__ int g_attn_err;

// Position in a ring of N slots: the slot and the phase bit of its current fill, advanced by one
// increment per fill (no division on the issuing threads' critical path).
template <int N>
struct RingPos {
  int slot = 0;
  uint32_t phase = 0;
  __device__ __forceinline__ void next() {
    if (++slot == N) {
      slot = 0;
      phase ^= 1u;
    }
  }
};

#ifdef BSA_PROFILE
// Profiling builds only: per CTA and warp, cycles spent in up to 7 sites + the role's total.
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

// One 64-wide d-half (c0 = 0 or 64) of block b of (b, h) slice bh into shared memory.  Blocks that are
// contiguous runs of 64 tokens are read through a 3-D map (d, s, b*h) at token 64*b, which spares the
// single issuing thread the divisions of the block's (t, h, w) origin; voxel blocks use the 5-D map.
__device__ __forceinline__ void tma_block(const Params& p, void* dst, const CUtensorMap* m, uint64_t* bar, int c0,
                                          int b, int bh);

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

__device__ __forceinline__ void tma_block(const Params& p, void* dst, const CUtensorMap* m, uint64_t* bar, int c0,
                                          int b, int bh) {
  if (p.map3) {
    tma_load_3d(dst, m, bar, c0, b * kBlock, bh);
  } else {
    int t0, h0, w0;
    block_origin(p, b, t0, h0, w0);
    tma_load_5d(dst, m, bar, c0, w0, h0, t0, bh);
  }
}

// Block ids of step j of a unit (the second id duplicates the first for an odd tail; those keys
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
__device__ __forceinline__ void store_row8(void* out, long long off, const float* v, int vec) {
  if (vec) {
    uint4 u;
    u.x = pack2<kBF16>(v[0], v[1]);
    u.y = pack2<kBF16>(v[2], v[3]);
    u.z = pack2<kBF16>(v[4], v[5]);
    u.w = pack2<kBF16>(v[6], v[7]);
    *reinterpret_cast<uint4*>(reinterpret_cast<uint16_t*>(out) + off) = u;
  } else {
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      if (kBF16)
        reinterpret_cast<__nv_bfloat16*>(out)[off + e] = __float2bfloat16_rn(v[e]);
      else
        reinterpret_cast<__half*>(out)[off + e] = __float2half_rn(v[e]);
    }
  }
}

// O rows of one lane half times f (per row; threads t and t + 16 hold the two column halves).  Rare:
// kept out of line so the softmax loop stays compact in the instruction cache.
__device__ __noinline__ void rescale_o(uint32_t la, float f) {
#pragma unroll
  for (int c = 0; c < 2; ++c) {
    uint32_t r[32];
    tmem_ld_16x2_x32(la + kColO + 64 * c, r);
    tmem_ld_wait();
#pragma unroll
    for (int e = 0; e < 32; ++e) r[e] = __float_as_uint(__uint_as_float(r[e]) * f);
    tmem_st_16x2_x32(la + kColO + 64 * c, r);
  }
  tmem_st_wait();
}

// One row half of a 128B-swizzled K-major Q tile (64 bf16/fp16 values, already in (even, odd) pairs)
// into 32 TMEM columns of this thread's lane; threads t and t + 16 take the two halves of row t.
__device__ __noinline__ void copy_q_tile(const uint8_t* src, int row, uint32_t dst) {
  uint32_t r[32];
#pragma unroll
  for (int c = 0; c < 8; ++c) {
    const uint4 v = *reinterpret_cast<const uint4*>(src + sw128_offset(static_cast<uint32_t>(row), c));
    r[4 * c] = v.x;
    r[4 * c + 1] = v.y;
    r[4 * c + 2] = v.z;
    r[4 * c + 3] = v.w;
  }
  tmem_st_16x2_x32(dst, r);
  tmem_st_wait();
}

// Epilogue of one warp: head-dim columns [64h, 64h + 64) of its 16 rows, 32 columns per pass.  Thread t
// (< 16) reads half 0's O of row t, thread t + 16 half 1's (32x32b shape over the whole lane quarter);
// they swap 16 columns so each ends with 16 merged columns of row t: a0 * O_0 + a1 * O_1.
template <bool kBF16>
__device__ __noinline__ void store_rows(uint32_t tq, int h, int cs, float a0, float a1, bool two_halves, void* out,
                                        long long orow, int D, int vec) {
#pragma unroll 1
  for (int c = 0; c < 2; ++c) {
    const uint32_t col = kColO + 64 * h + 32 * c;
    uint32_t r[32];
    tmem_ld32(tq + col, r);
    tmem_ld_wait();
    float o[16];
#pragma unroll
    for (int e = 0; e < 16; ++e) {
      const float keep = __uint_as_float(cs == 0 ? r[e] : r[16 + e]);
      const float send = __uint_as_float(cs == 0 ? r[16 + e] : r[e]);
      const float recv = __shfl_xor_sync(0xffffffffu, send, 16);
      const float o0 = cs == 0 ? keep : recv;
      const float o1 = cs == 0 ? recv : keep;
      o[e] = two_halves ? fmaf(a1, o1, a0 * o0) : a0 * o0;
    }
    const int d0 = 64 * h + 32 * c + 16 * cs;
#pragma unroll
    for (int e8 = 0; e8 < 2; ++e8)
      if (d0 + 8 * e8 < D) store_row8<kBF16>(out, orow + d0 + 8 * e8, o + 8 * e8, vec);
  }
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
  uint8_t* sK = smem + kOffK;
  uint8_t* sV = smem + kOffV;
  SmallSmem& ss = *reinterpret_cast<SmallSmem*>(smem + kTileBytes);

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int nsteps = p.nsteps;
  const bool two_halves = nsteps >= 2;  // half 1 takes the odd steps; it has none when nsteps == 1
  const int copy_warps = two_halves ? 8 : 4;

  if (tid == 0) {
    for (int s = 0; s < kKStages; ++s) {
      mbar_init(&ss.k_full[s], 1);
      mbar_init(&ss.k_empty[s], 1);
    }
    for (int s = 0; s < kVSlots; ++s) {
      mbar_init(&ss.v_full[s], 1);
      mbar_init(&ss.v_empty[s], 1);
    }
    for (int h = 0; h < 2; ++h) {
      mbar_init(&ss.s_full[h], 1);
      mbar_init(&ss.s_empty[h], 4);
      mbar_init(&ss.q_ready[h], 4);
      for (int b = 0; b < 2; ++b) {
        mbar_init(&ss.p_full[h][b], 4);
        mbar_init(&ss.p_empty[h][b], 1);
      }
    }
    for (int i = 0; i < kQBufs; ++i) {
      mbar_init(&ss.q_full[i], 1);
      mbar_init(&ss.q_empty[i], copy_warps);
    }
    for (int i = 0; i < 4; ++i) mbar_init(&ss.ep[i], 2);
    mbar_init(&ss.o_empty, kSoftmaxWarps);
    mbar_init(&ss.drain[0], 1);
    mbar_init(&ss.drain[1], 1);
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
  const int k = p.topk;

  if (warp == 0) {
    // ------------------------------------------------------------------ Q + K producer
    if (lane == 0) {
      prefetch_tmap(&tm_q);
      prefetch_tmap(&tm_k);
      // Q tile of unit u, the nn-th unit of this CTA, into buffer nn % kQBufs
      auto load_q = [&](int u, int nn) -> bool {
        const int qb = nn % kQBufs;
        if (nn >= kQBufs &&
            !mbar_wait(&ss.q_empty[qb], static_cast<uint32_t>(((nn - kQBufs) / kQBufs) & 1), abort_flag, err, 101,
                       PACC(0)))
          return false;
        const int bh = u / p.nqb;
        const int qblk = u - bh * p.nqb;
        mbar_arrive_expect_tx(&ss.q_full[qb], kQBytes);
        uint8_t* dst = sQ + qb * kQBytes;
        tma_block(p, dst, &tm_q, &ss.q_full[qb], 0, qblk, bh);
        tma_block(p, dst + kQBytes / 2, &tm_q, &ss.q_full[qb], 64, qblk, bh);
        return true;
      };
      long long g = 0;
      RingPos<kKStages> kp;
      int n = 0;
      int nq = 0;  // Q tiles issued
      bool ok = true;
      for (int unit = blockIdx.x; unit < p.total_units && ok; unit += G, ++n) {
        const int bh = unit / p.nqb;
        const int qblk = unit - bh * p.nqb;
        const int32_t* idx = p.idx + (static_cast<long long>(bh) * p.nqb + qblk) * k;
        int nb0, nb1;
        step_blocks(idx, 0, k, p.nqb, err, nb0, nb1);
        // this unit's Q tile, at most kKStages steps before its first QK (a Q tile issued a whole unit
        // early measured 30 % slower: more K/V reads went to DRAM)
        ok = load_q(unit, n);
        if (!ok) break;
        nq = n + 1;
        for (int j = 0; j < nsteps && ok; ++j, ++g) {
          const int b0 = nb0, b1 = nb1;
          if (j + 1 < nsteps) step_blocks(idx, j + 1, k, p.nqb, err, nb0, nb1);  // prefetch next ids
          const int ks = kp.slot;
          if (g >= kKStages) ok = mbar_wait(&ss.k_empty[ks], kp.phase ^ 1u, abort_flag, err, 102, PACC(1));
          if (!ok) break;
          kp.next();
          uint8_t* dst = sK + ks * kPairBytes;
          mbar_arrive_expect_tx(&ss.k_full[ks], kPairBytes);
#pragma unroll
          for (int bi = 0; bi < 2; ++bi)
#pragma unroll
            for (int hh = 0; hh < 2; ++hh)
              tma_block(p, dst + hh * 16384 + bi * 8192, &tm_k, &ss.k_full[ks], hh * 64, bi ? b1 : b0, bh);
        }
      }
      // teardown: no TMA write into this CTA's shared memory may still be in flight
      const uint64_t t0 = globaltimer_ns();
      for (long long gg = (g > kKStages ? g - kKStages : 0); gg < g; ++gg)
        while (!mbar_try_wait(&ss.k_full[gg % kKStages], static_cast<uint32_t>((gg / kKStages) & 1)) &&
               globaltimer_ns() - t0 < kWaitLimitNs) {
        }
      for (int nn = (nq > kQBufs ? nq - kQBufs : 0); nn < nq; ++nn)
        while (!mbar_try_wait(&ss.q_full[nn % kQBufs], static_cast<uint32_t>((nn / kQBufs) & 1)) &&
               globaltimer_ns() - t0 < kWaitLimitNs) {
        }
    }
    __syncwarp();
  } else if (warp == 2) {
    // ------------------------------------------------------------------ V producer
    if (lane == 0) {
      prefetch_tmap(&tm_v);
      long long gb = 0;  // V blocks issued
      RingPos<kVSlots> vp;
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
            const int vs = vp.slot;
            if (gb >= kVSlots) ok = mbar_wait(&ss.v_empty[vs], vp.phase ^ 1u, abort_flag, err, 103, PACC(0));
            if (!ok) break;
            vp.next();
            uint8_t* dst = sV + vs * kVBlockBytes;
            mbar_arrive_expect_tx(&ss.v_full[vs], kVBlockBytes);
            tma_block(p, dst, &tm_v, &ss.v_full[vs], 0, bi ? b1 : b0, bh);
            tma_block(p, dst + kVBlockBytes / 2, &tm_v, &ss.v_full[vs], 64, bi ? b1 : b0, bh);
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
    // ------------------------------------------------------------------ QK issuer
    if (lane == 0) {
      const uint32_t idesc = idesc_f16(64, 128, kBF16 ? 1 : 0, 0, 0);
      long long i0 = 0, i1 = 0;  // steps issued per half
      RingPos<kKStages> kp;
      int n = 0;
      bool ok = true;
      for (int unit = blockIdx.x; unit < p.total_units && ok; unit += G, ++n) {
        for (int j = 0; j < nsteps && ok; ++j) {
          const int h = j & 1;
          const long long i = h ? i1 : i0;  // step of the half
          const int ks = kp.slot;
          ok = mbar_wait(&ss.k_full[ks], kp.phase, abort_flag, err, 113, PACC(0));
          if (ok && i >= 1)
            ok = mbar_wait(&ss.s_empty[h], static_cast<uint32_t>((i - 1) & 1), abort_flag, err, 114, PACC(1));
          if (ok && j == h) ok = mbar_wait(&ss.q_ready[h], static_cast<uint32_t>(n & 1), abort_flag, err, 115, PACC(2));
          if (!ok) break;
          tc_fence_after();
          const uint32_t kb = smem_u32(sK + ks * kPairBytes);
          const uint32_t hl = half_lanes(h);
#pragma unroll
          for (int kk = 0; kk < 8; ++kk) {
            const uint64_t bd = sdesc_sw128(kb + (kk >> 2) * 16384 + (kk & 3) * 32, 16, 1024);
            umma_ts(tmem + hl + kColS, tmem + hl + kColQ + 8 * kk, bd, idesc, kk > 0 ? 1u : 0u);
          }
          umma_commit(&ss.s_full[h]);
          umma_commit(&ss.k_empty[ks]);
          kp.next();
          if (h) ++i1; else ++i0;
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
      const uint32_t idesc = idesc_f16(64, 128, kBF16 ? 1 : 0, 0, 1);
      long long i0 = 0, i1 = 0;  // steps issued per half
      RingPos<kVSlots> vp;
      int n = 0;
      bool ok = true;
      for (int unit = blockIdx.x; unit < p.total_units && ok; unit += G, ++n) {
        for (int j = 0; j < nsteps && ok; ++j) {
          const int h = j & 1;
          const long long i = h ? i1 : i0;  // step of the half
          const int pb = static_cast<int>(i & 1);
          const int vs0 = vp.slot;
          ok = mbar_wait(&ss.v_full[vs0], vp.phase, abort_flag, err, 116, PACC(0));
          vp.next();
          const int vs1 = vp.slot;
          if (ok) ok = mbar_wait(&ss.v_full[vs1], vp.phase, abort_flag, err, 117, PACC(1));
          vp.next();
          if (ok) ok = mbar_wait(&ss.p_full[h][pb], static_cast<uint32_t>((i >> 1) & 1), abort_flag, err, 111, PACC(2));
          if (ok && j == 0 && n >= 1) ok = mbar_wait(&ss.o_empty, static_cast<uint32_t>((n - 1) & 1), abort_flag, err, 112, PACC(3));
          if (!ok) break;
          tc_fence_after();
          const uint32_t vb0 = smem_u32(sV + vs0 * kVBlockBytes);
          const uint32_t vb1 = smem_u32(sV + vs1 * kVBlockBytes);
          const uint32_t hl = half_lanes(h);
#pragma unroll
          for (int kk = 0; kk < 8; ++kk) {
            const uint64_t bd = sdesc_sw128((kk < 4 ? vb0 : vb1) + (kk & 3) * 2048, kVBlockBytes / 2, 1024);
            umma_ts(tmem + hl + kColO, tmem + hl + col_p(pb) + 8 * kk, bd, idesc, (j >= 2 || kk > 0) ? 1u : 0u);
          }
          umma_commit(&ss.v_empty[vs0]);
          umma_commit(&ss.v_empty[vs1]);
          umma_commit(&ss.p_empty[h][pb]);
          if (h) ++i1; else ++i0;
        }
      }
      umma_commit(&ss.drain[1]);
      const uint64_t t0 = globaltimer_ns();
      while (!mbar_try_wait(&ss.drain[1], 0) && globaltimer_ns() - t0 < kWaitLimitNs) {
      }
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------------ softmax, one lane half
    const int h = (warp - 4) >> 2;               // lane half: 0 = even steps, 1 = odd steps
    const int qq = warp & 3;                     // TMEM lane quarter
    const int cs = lane >> 4;                    // column side: keys 0-63 (0) or 64-127 (1) of a step
    const int row = 16 * qq + (lane & 15);       // query row of the block
    const uint32_t la = tmem + (static_cast<uint32_t>(32 * qq + 16 * h) << 16);  // this warp's 16 lanes
    const float scale_log2 = p.scale_log2;
    const bool odd_tail = (k & 1) != 0;
    const bool active = h == 0 || two_halves;    // half 1 has no steps when nsteps == 1
    const int hsteps = (nsteps + 1 - h) >> 1;    // steps of this half per unit
    long long i = 0;                             // steps of this half processed so far
    int n = 0;
    bool ok = true;

    // Q tile of unit n (shared memory, 128B-swizzled K-major) -> this half's Q columns in TMEM.
    auto copy_q = [&](int nn) -> bool {
      const int qb = nn % kQBufs;
      bool w = mbar_wait(&ss.q_full[qb], static_cast<uint32_t>((nn / kQBufs) & 1), abort_flag, err, 131);
      w = __all_sync(0xffffffffu, w);
      if (!w) return false;
      copy_q_tile(sQ + qb * kQBytes + cs * (kQBytes / 2), row, la + kColQ);
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&ss.q_ready[h]);
        mbar_arrive(&ss.q_empty[qb]);
      }
      return true;
    };

    if (active && blockIdx.x < p.total_units) ok = copy_q(0);
    for (int unit = blockIdx.x; unit < p.total_units && ok; unit += G, ++n) {
      const int bh = unit / p.nqb;
      const int qblk = unit - bh * p.nqb;
      float m_run = 0.f;  // running max of this row and half (log2 domain), same in threads t and t^16
      uint64_t l2 = f2_pack(0.f, 0.f);  // this thread's share of the row sum, two partial sums
      if (active) {
        for (int s = 0; s < hsteps; ++s, ++i) {
          const int j = 2 * s + h;
          ok = mbar_wait(&ss.s_full[h], static_cast<uint32_t>(i & 1), abort_flag, err, 121, PACC(0));
          ok = __all_sync(0xffffffffu, ok);  // leave the loop warp-uniformly
          if (!ok) break;
          PTS_START();
          tc_fence_after();
          uint32_t r[64];
          tmem_ld_16x2_x64(la + kColS, r);
          tmem_ld_wait();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&ss.s_empty[h]);  // S may be overwritten by the next QK of this half
          PTS(4);
          const bool masked = odd_tail && j == nsteps - 1 && cs == 1;
          // row max of the raw scores (tree), then of the pair of threads sharing the row
          float mv[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) mv[e] = __uint_as_float(r[e]);
#pragma unroll
          for (int c = 8; c < 64; c += 8)
#pragma unroll
            for (int e = 0; e < 8; ++e) mv[e] = fmaxf(mv[e], __uint_as_float(r[c + e]));
          float smax = fmaxf(fmaxf(fmaxf(mv[0], mv[1]), fmaxf(mv[2], mv[3])), fmaxf(fmaxf(mv[4], mv[5]), fmaxf(mv[6], mv[7])));
          if (masked) smax = -INFINITY;
          smax = fmaxf(smax, __shfl_xor_sync(0xffffffffu, smax, 16));
          // first step of the block: take the row max; later: raise it only on a jump above 2^8
          const float mx = fmaf(smax, scale_log2, -m_run);
          const float d = (s == 0 || mx > kRescaleThreshold) ? mx : 0.f;
          m_run += d;
          const bool rescale = s > 0 && d != 0.f;
          if (__any_sync(0xffffffffu, rescale)) {
            // O rows of this half must be rescaled: the previous PV of this half must be complete
            ok = mbar_wait(&ss.p_empty[h][(i - 1) & 1], static_cast<uint32_t>(((i - 1) >> 1) & 1), abort_flag, err,
                           122);
            ok = __all_sync(0xffffffffu, ok);
            if (!ok) break;
            tc_fence_after();
            const float f = rescale ? ex2_approx(-d) : 1.f;
            l2 = f2_mul(l2, f2_pack(f, f));
            rescale_o(la, f);
          }
          PTS(5);
          // x = s * scale - m (masked keys: 0 * s - inf), P = 2^x, row-sum pair, P row half to TMEM
          const float sc = masked ? 0.f : scale_log2;
          const float nm = masked ? -INFINITY : -m_run;
          const uint64_t sc2 = f2_pack(sc, sc);
          const uint64_t nm2 = f2_pack(nm, nm);
          uint32_t packed[32];
#pragma unroll
          for (int c = 0; c < 32; ++c) {
            float x0, x1;
            f2_unpack(f2_fma(f2_pack(__uint_as_float(r[2 * c]), __uint_as_float(r[2 * c + 1])), sc2, nm2), x0, x1);
            const float p0 = ex2_approx(x0);
            const float p1 = ex2_approx(x1);
            l2 = f2_add(l2, f2_pack(p0, p1));
            packed[c] = pack2<kBF16>(p0, p1);
          }
          PTS(6);
          if (i >= 2) {  // the PV two steps back (same half) must be done reading this P buffer
            ok = mbar_wait(&ss.p_empty[h][i & 1], static_cast<uint32_t>(((i - 2) >> 1) & 1), abort_flag, err, 124,
                           PACC(1));
            ok = __all_sync(0xffffffffu, ok);
            if (!ok) break;
            tc_fence_after();
          }
          PTS_START();
          tmem_st_16x2_x32(la + col_p(static_cast<int>(i & 1)), packed);
          tmem_st_wait();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&ss.p_full[h][i & 1]);
          PTS(3);
        }
        if (!ok) break;
        // the next unit's Q first, so its QK can start while this epilogue runs
        if (unit + G < p.total_units) {
          ok = copy_q(n + 1);
          if (!ok) break;
        }
      }
      // ---- epilogue: merge the two halves' (m, l, O) of each row, out = O / l
      PTS_START();
      const int ub = n & 1;
      {
        float la0, la1;
        f2_unpack(l2, la0, la1);
        const float l_run = la0 + la1;
        const float l_half = l_run + __shfl_xor_sync(0xffffffffu, l_run, 16);
        if (cs == 0) {
          ss.st_m[ub][h][row] = active ? m_run : -INFINITY;
          ss.st_l[ub][h][row] = active ? l_half : 0.f;
        }
      }
      // both halves' last PVs of this unit must be complete before O is read.  Each warp waits for its
      // own half's last PV only (i - 1: steps of this half so far), in order; the ep handshake below
      // carries the other half's.  Waiting on the other half's barrier here could run a whole phase
      // ahead of it (that half may still be two PVs behind), which a parity wait misreads as done.
      bool w = true;
      if (active) {
        const long long last = i - 1;
        w = mbar_wait(&ss.p_empty[h][last & 1], static_cast<uint32_t>((last >> 1) & 1), abort_flag, err, 125);
      }
      __syncwarp();
      if (lane == 0 && w) mbar_arrive(&ss.ep[qq]);
      if (w) w = mbar_wait(&ss.ep[qq], static_cast<uint32_t>(n & 1), abort_flag, err, 127);
      ok = __all_sync(0xffffffffu, w);
      if (!ok) break;
      tc_fence_after();
      float a0, a1;
      {
        const int r = row;
        const float m0 = ss.st_m[ub][0][r], m1 = ss.st_m[ub][1][r];
        const float l0 = ss.st_l[ub][0][r], l1 = ss.st_l[ub][1][r];
        const float m = fmaxf(m0, m1);
        const float e0 = ex2_approx(m0 - m);
        const float e1 = two_halves ? ex2_approx(m1 - m) : 0.f;
        const float l = l0 * e0 + l1 * e1;
        const float inv = l > 0.f ? 1.f / l : 0.f;
        a0 = e0 * inv;
        a1 = e1 * inv;
      }
      int t0, h0, w0;
      block_origin(p, qblk, t0, h0, w0);
      const int b = bh / p.H;
      const int hh = bh - b * p.H;
      long long orow;
      {
        const int cHW = p.cH * p.cW;
        const int ct = row / cHW;
        const int rem = row - ct * cHW;
        const int ch = rem / p.cW;
        const int cw = rem - ch * p.cW;
        const long long tok = (static_cast<long long>(t0 + ct) * p.Hl + (h0 + ch)) * p.Wl + (w0 + cw);
        orow = b * p.out_sb + hh * p.out_sh + tok * p.out_ss;
      }
      store_rows<kBF16>(tmem + (static_cast<uint32_t>(32 * qq) << 16), h, cs, a0, a1, two_halves, p.out, orow, p.D,
                        p.vec_out);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&ss.o_empty);
      PTS(2);
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
  // the shared-memory opt-in is per device; first calls from several host threads may race here
  static std::mutex mu;
  static bool configured[64] = {false};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return BSA_ERR_CUDA;
  {
    std::lock_guard<std::mutex> lock(mu);
    if (dev >= 64 || !configured[dev]) {
      if (cudaFuncSetAttribute(bsa_attn_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes) !=
              cudaSuccess ||
          cudaFuncSetAttribute(bsa_attn_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes) !=
              cudaSuccess)
        return BSA_ERR_CUDA;
      if (dev < 64) configured[dev] = true;
    }
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
  p.map3 = a.map3;
  p.vec_out = ((reinterpret_cast<uintptr_t>(a.out) & 15u) == 0 && (a.out_ss * 2) % 16 == 0 &&
               (a.out_sh * 2) % 16 == 0 && (a.out_sb * 2) % 16 == 0)
                  ? 1
                  : 0;
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
