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
// Both accumulators live in TMEM.  The column-wise (per query) online softmax uses a lazy
// running max: it is only raised when a score exceeds it by more than 2^8, so the common step
// needs no cross-thread max; the row sums are kept per thread and reduced once per block.
//
// Roles (256 threads, one CTA per SM, persistent over (head, q-block) units in head-major
// order so a head's K/V stays resident in L2):
//   warp 0     : TMA producer (Q tiles, K/V block pairs into a 3-stage ring)
//   warp 1     : MMA issuer (one thread)
//   warps 4-7  : softmax / correction / epilogue warpgroup (thread t <-> TMEM lane t)
// Every mbarrier wait is bounded (bsa_ptx.cuh); a timeout records an error code and the CTA
// winds down.
#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>
#include "bsa_ptx.cuh"
#include "bsa_kernels.h"

namespace bsa {

namespace attn {
constexpr int kBlock = 64;            // tokens per block
constexpr int kDP = 128;              // head dim as laid out in shared memory (zero padded)
constexpr int kStages = 3;
constexpr int kQBytes = kBlock * kDP * 2;          // 16 KB
constexpr int kPairBytes = 2 * kBlock * kDP * 2;   // 32 KB (one operand of a block pair)
constexpr int kStageBytes = 2 * kPairBytes;        // K pair + V pair = 64 KB
constexpr int kTileBytes = 2 * kQBytes + kStages * kStageBytes;  // 224 KB
constexpr int kThreads = 256;
constexpr float kRescaleThreshold = 8.0f;          // log2 units: P <= 2^8 between rescales

// TMEM column map (512 allocated): S^T double buffer, each split in two d-halves, and O^T
// split in two kv-halves (independent accumulation chains hide the tensor-pipe latency).
constexpr uint32_t kTmemCols = 512;
__host__ __device__ constexpr uint32_t col_s(int buf, int half) { return buf * 128 + half * 64; }
constexpr uint32_t kColO = 256;  // O^T.a at 256, O^T.b at 320

struct SmallSmem {
  uint64_t full[kStages];    // TMA -> MMA: stage loaded
  uint64_t empty[kStages];   // MMA -> TMA: stage's PV done (stage free)
  uint64_t s_full[2];        // MMA -> softmax: S^T ready
  uint64_t s_empty[2];       // softmax -> MMA: S^T read
  uint64_t p_full[2];        // softmax -> MMA: P^T written
  uint64_t q_full[2];        // TMA -> MMA: Q tile loaded
  uint64_t q_empty[2];       // MMA -> TMA: last QK of the unit done
  uint64_t o_empty;          // softmax -> MMA: O^T read by the epilogue
  uint64_t drain;            // teardown: all MMAs complete
  uint32_t tmem_base;
  int abort_flag;
  uint32_t flags[2][4][2];   // per-warp overflow bitmasks, double-buffered by step parity
  alignas(16) float m[64];               // running max per query column (log2 domain)
  alignas(16) float mthr[64];            // m + threshold
  alignas(16) float alpha[64];           // rescale factors of the last max update; 1/l in the epilogue
  alignas(16) float red[4][64];          // per-warp column partials (max or sum)
};
constexpr int kSmemBytes = kTileBytes + 2048 + 1024;  // tiles + small + alignment slack
static_assert(sizeof(SmallSmem) <= 2048, "small smem");
static_assert(kSmemBytes <= 232448, "fits in 227 KB");

struct Params {
  const int32_t* idx;   // [BH, nqb, topk]
  void* out;            // [B,H,S,D] with the strides below (elements)
  int BH, H, nqb, topk, nsteps, D;
  int Hl, Wl, cT, cH, cW, Bh, Bw;
  long long out_sb, out_sh, out_ss;
  float scale_log2;
  int is_bf16;
  int total_units;
};

__device__ int g_attn_err;

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

// Transposed warp reduction: each lane holds v[0..63] (one value per query column) for its own
// key row; afterwards lane L holds the reduction over the 32 lanes of columns
// col(L, 0) and col(L, 1) where col(L, i) = 32*b4 + 16*b3 + 8*b2 + 4*b1 + 2*b0 + i (bK = bit K
// of L).  62 shuffles instead of 64 x 5.
template <bool kMax>
__device__ __forceinline__ void transpose_reduce(float (&v)[64], float& r0, float& r1, int lane) {
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    const bool up = lane & 16;
    float send = up ? v[i] : v[i + 32];
    float keep = up ? v[i + 32] : v[i];
    float recv = __shfl_xor_sync(0xffffffffu, send, 16);
    v[i] = kMax ? fmaxf(keep, recv) : keep + recv;
  }
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const bool up = lane & 8;
    float send = up ? v[i] : v[i + 16];
    float keep = up ? v[i + 16] : v[i];
    float recv = __shfl_xor_sync(0xffffffffu, send, 8);
    v[i] = kMax ? fmaxf(keep, recv) : keep + recv;
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const bool up = lane & 4;
    float send = up ? v[i] : v[i + 8];
    float keep = up ? v[i + 8] : v[i];
    float recv = __shfl_xor_sync(0xffffffffu, send, 4);
    v[i] = kMax ? fmaxf(keep, recv) : keep + recv;
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const bool up = lane & 2;
    float send = up ? v[i] : v[i + 4];
    float keep = up ? v[i + 4] : v[i];
    float recv = __shfl_xor_sync(0xffffffffu, send, 2);
    v[i] = kMax ? fmaxf(keep, recv) : keep + recv;
  }
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const bool up = lane & 1;
    float send = up ? v[i] : v[i + 2];
    float keep = up ? v[i + 2] : v[i];
    float recv = __shfl_xor_sync(0xffffffffu, send, 1);
    v[i] = kMax ? fmaxf(keep, recv) : keep + recv;
  }
  r0 = v[0];
  r1 = v[1];
}

__device__ __forceinline__ int transpose_col(int lane, int i) {
  return ((lane >> 4) & 1) * 32 + ((lane >> 3) & 1) * 16 + ((lane >> 2) & 1) * 8 + ((lane >> 1) & 1) * 4 +
         (lane & 1) * 2 + i;
}

__global__ void __launch_bounds__(kThreads, 1)
    bsa_attn_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                    const __grid_constant__ CUtensorMap tm_v, const Params p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;                           // 2 x 16 KB
  uint8_t* sStage = smem + 2 * kQBytes;         // 3 x 64 KB: [K pair 32 KB | V pair 32 KB]
  SmallSmem& ss = *reinterpret_cast<SmallSmem*>(smem + kTileBytes);

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;

  if (tid == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&ss.full[s], 1);
      mbar_init(&ss.empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&ss.s_full[i], 1);
      mbar_init(&ss.s_empty[i], 128);
      mbar_init(&ss.p_full[i], 128);
      mbar_init(&ss.q_full[i], 1);
      mbar_init(&ss.q_empty[i], 1);
    }
    mbar_init(&ss.o_empty, 128);
    mbar_init(&ss.drain, 1);
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
  volatile int* abort_flag = &ss.abort_flag;
  int* err = &g_attn_err;

  const int G = gridDim.x;
  const int nsteps = p.nsteps;
  const int k = p.topk;

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      prefetch_tmap(&tm_q);
      prefetch_tmap(&tm_k);
      prefetch_tmap(&tm_v);
    }
    long long g = 0;
    int n = 0;
    bool ok = true;
    for (int unit = blockIdx.x; unit < p.total_units && ok; unit += G, ++n) {
      const int bh = unit / p.nqb;
      const int qblk = unit - bh * p.nqb;
      const int32_t* idx = p.idx + (static_cast<long long>(bh) * p.nqb + qblk) * k;
      if (lane == 0) {
        const int qb = n & 1;
        if (n >= 2) ok = mbar_wait(&ss.q_empty[qb], ((n - 2) >> 1) & 1, abort_flag, err, 101);
        if (ok) {
          int t0, h0, w0;
          block_origin(p, qblk, t0, h0, w0);
          mbar_arrive_expect_tx(&ss.q_full[qb], kQBytes);
          uint8_t* dst = sQ + qb * kQBytes;
          tma_load_5d(dst, &tm_q, &ss.q_full[qb], 0, w0, h0, t0, bh);
          tma_load_5d(dst + kQBytes / 2, &tm_q, &ss.q_full[qb], 64, w0, h0, t0, bh);
        }
      }
      ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
      int nb0 = 0, nb1 = 0;
      if (lane == 0) {
        nb0 = __ldg(idx);
        nb1 = (1 < k) ? __ldg(idx + 1) : nb0;
      }
      for (int j = 0; j < nsteps && ok; ++j, ++g) {
        if (lane == 0) {
          int b0 = nb0, b1 = nb1;
          if (j + 1 < nsteps) {  // prefetch the next pair while this step waits for a free stage
            nb0 = __ldg(idx + 2 * j + 2);
            nb1 = (2 * j + 3 < k) ? __ldg(idx + 2 * j + 3) : nb0;
          }
          const int s = static_cast<int>(g % kStages);
          if (g >= kStages) ok = mbar_wait(&ss.empty[s], static_cast<uint32_t>((g / kStages - 1) & 1), abort_flag, err, 102);
          if (ok) {
            if (static_cast<unsigned>(b0) >= static_cast<unsigned>(p.nqb) ||
                static_cast<unsigned>(b1) >= static_cast<unsigned>(p.nqb)) {
              atomicCAS(err, 0, BSA_ERR_INDEX);
              b0 = static_cast<unsigned>(b0) >= static_cast<unsigned>(p.nqb) ? 0 : b0;
              b1 = static_cast<unsigned>(b1) >= static_cast<unsigned>(p.nqb) ? 0 : b1;
            }
            uint8_t* st = sStage + s * kStageBytes;
            mbar_arrive_expect_tx(&ss.full[s], kStageBytes);
#pragma unroll
            for (int bi = 0; bi < 2; ++bi) {
              int t0, h0, w0;
              block_origin(p, bi ? b1 : b0, t0, h0, w0);
#pragma unroll
              for (int hh = 0; hh < 2; ++hh) {
                tma_load_5d(st + hh * 16384 + bi * 8192, &tm_k, &ss.full[s], hh * 64, w0, h0, t0, bh);
                tma_load_5d(st + kPairBytes + hh * 16384 + bi * 8192, &tm_v, &ss.full[s], hh * 64, w0, h0, t0, bh);
              }
            }
          }
        }
        ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
      }
    }
    // teardown: make sure no TMA write into this CTA's shared memory is still in flight
    if (lane == 0 && g > 0) {
      const long long first = g > kStages ? g - kStages : 0;
      for (long long gg = first; gg < g; ++gg) {
        const int s = static_cast<int>(gg % kStages);
        const uint64_t t0 = globaltimer_ns();
        while (!mbar_try_wait(&ss.full[s], static_cast<uint32_t>((gg / kStages) & 1)) &&
               globaltimer_ns() - t0 < kWaitLimitNs) {
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    const uint32_t id_qk = idesc_f16(128, 64, p.is_bf16, 0, 0);
    const uint32_t id_pv = idesc_f16(128, 64, p.is_bf16, 1, 1);
    long long g = 0;
    int n = 0;
    bool ok = true;
    bool have_prev = false;
    long long prev_g = 0;
    int prev_j = 0, prev_n = 0;
    auto issue_pv = [&](long long gp, int jp, int np) -> bool {
      const int s = static_cast<int>(gp % kStages);
      const int pb = static_cast<int>(gp & 1);
      if (!mbar_wait(&ss.p_full[pb], static_cast<uint32_t>((gp >> 1) & 1), abort_flag, err, 111)) return false;
      if (jp == 0 && np >= 1) {
        if (!mbar_wait(&ss.o_empty, static_cast<uint32_t>((np - 1) & 1), abort_flag, err, 112)) return false;
      }
      tc_fence_after();
      if (lane == 0) {
        const uint32_t vb = smem_u32(sStage + s * kStageBytes + kPairBytes);
        const uint32_t pbase = smem_u32(sStage + s * kStageBytes);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
#pragma unroll
          for (int half = 0; half < 2; ++half) {
            const int kk = half * 4 + i;
            const uint64_t ad = sdesc_sw128(vb + kk * 2048, 16384, 1024);
            const uint64_t bd = sdesc_sw128(pbase + kk * 2048, 16384, 1024);
            umma_ss(tmem + kColO + half * 64, ad, bd, id_pv, (jp > 0 || i > 0) ? 1u : 0u);
          }
        }
        umma_commit(&ss.empty[s]);
      }
      __syncwarp();
      return true;
    };
    for (int unit = blockIdx.x; unit < p.total_units && ok; unit += G, ++n) {
      const int qb = n & 1;
      for (int j = 0; j < nsteps && ok; ++j, ++g) {
        const int s = static_cast<int>(g % kStages);
        const int sb = static_cast<int>(g & 1);
        ok = mbar_wait(&ss.full[s], static_cast<uint32_t>((g / kStages) & 1), abort_flag, err, 113);
        if (ok && g >= 2) ok = mbar_wait(&ss.s_empty[sb], static_cast<uint32_t>(((g >> 1) - 1) & 1), abort_flag, err, 114);
        if (ok && j == 0) ok = mbar_wait(&ss.q_full[qb], static_cast<uint32_t>((n >> 1) & 1), abort_flag, err, 115);
        if (!ok) break;
        tc_fence_after();
        if (lane == 0) {
          const uint32_t kb = smem_u32(sStage + s * kStageBytes);
          const uint32_t qbase = smem_u32(sQ + qb * kQBytes);
#pragma unroll
          for (int i = 0; i < 4; ++i) {
#pragma unroll
            for (int half = 0; half < 2; ++half) {
              const uint64_t ad = sdesc_sw128(kb + half * 16384 + i * 32, 16, 1024);
              const uint64_t bd = sdesc_sw128(qbase + half * 8192 + i * 32, 16, 1024);
              umma_ss(tmem + col_s(sb, half), ad, bd, id_qk, i > 0 ? 1u : 0u);
            }
          }
          umma_commit(&ss.s_full[sb]);
          if (j == nsteps - 1) umma_commit(&ss.q_empty[qb]);
        }
        __syncwarp();
        if (have_prev) ok = issue_pv(prev_g, prev_j, prev_n);
        have_prev = true;
        prev_g = g;
        prev_j = j;
        prev_n = n;
      }
    }
    if (ok && have_prev) ok = issue_pv(prev_g, prev_j, prev_n);
    // teardown: wait until every issued MMA has completed before TMEM is released
    if (lane == 0) {
      umma_commit(&ss.drain);
      const uint64_t t0 = globaltimer_ns();
      while (!mbar_try_wait(&ss.drain, 0) && globaltimer_ns() - t0 < kWaitLimitNs) {
      }
    }
    __syncwarp();
  } else if (warp >= 4) {
    // ------------------------------------------------------------------ softmax warpgroup
    const int t = tid - 128;               // TMEM lane == key row (S^T) == d row (O^T)
    const int wq = warp - 4;               // warp quarter
    const uint32_t lane_base = static_cast<uint32_t>(wq * 32) << 16;
    const float scale_log2 = p.scale_log2;
    const bool odd_tail = (k & 1) != 0;
    long long g = 0;
    int n = 0;
    bool ok = true;
    for (int unit = blockIdx.x; unit < p.total_units && ok; unit += G, ++n) {
      const int bh = unit / p.nqb;
      const int qblk = unit - bh * p.nqb;
      if (t < 64) {
        ss.m[t] = -INFINITY;
        ss.mthr[t] = -INFINITY;
      }
      float l_part[64];
#pragma unroll
      for (int q = 0; q < 64; ++q) l_part[q] = 0.f;
      named_bar_sync(1, 128);
      for (int j = 0; j < nsteps && ok; ++j, ++g) {
        const int s = static_cast<int>(g % kStages);
        const int sb = static_cast<int>(g & 1);
        ok = mbar_wait(&ss.s_full[sb], static_cast<uint32_t>((g >> 1) & 1), abort_flag, err, 121);
        if (!ok) break;
        tc_fence_after();
        float x[64];
        {
          uint32_t ra[32], rb[32];
#pragma unroll
          for (int c = 0; c < 2; ++c) {
            tmem_ld32(tmem + lane_base + col_s(sb, 0) + c * 32, ra);
            tmem_ld32(tmem + lane_base + col_s(sb, 1) + c * 32, rb);
            tmem_ld_wait();
#pragma unroll
            for (int q = 0; q < 32; ++q)
              x[c * 32 + q] = (__uint_as_float(ra[q]) + __uint_as_float(rb[q])) * scale_log2;
          }
        }
        tc_fence_before();
        mbar_arrive(&ss.s_empty[sb]);
        if (odd_tail && j == nsteps - 1 && t >= 64) {
#pragma unroll
          for (int q = 0; q < 64; ++q) x[q] = -INFINITY;
        }
        // ---- lazy running max: find columns where some key exceeds m + threshold
        uint32_t bits0 = 0, bits1 = 0;
#pragma unroll
        for (int q = 0; q < 32; ++q) bits0 |= (x[q] > ss.mthr[q] ? 1u : 0u) << q;
#pragma unroll
        for (int q = 0; q < 32; ++q) bits1 |= (x[q + 32] > ss.mthr[q + 32] ? 1u : 0u) << q;
        bits0 = __reduce_or_sync(0xffffffffu, bits0);
        bits1 = __reduce_or_sync(0xffffffffu, bits1);
        if (lane == 0) {
          ss.flags[sb][wq][0] = bits0;
          ss.flags[sb][wq][1] = bits1;
        }
        named_bar_sync(1, 128);
        bits0 = ss.flags[sb][0][0] | ss.flags[sb][1][0] | ss.flags[sb][2][0] | ss.flags[sb][3][0];
        bits1 = ss.flags[sb][0][1] | ss.flags[sb][1][1] | ss.flags[sb][2][1] | ss.flags[sb][3][1];
        if ((bits0 | bits1) != 0u) {
          // exact column max over the 128 keys of this step, then raise m where needed
          float tmp[64];
#pragma unroll
          for (int q = 0; q < 64; ++q) tmp[q] = x[q];
          float r0, r1;
          transpose_reduce<true>(tmp, r0, r1, lane);
          ss.red[wq][transpose_col(lane, 0)] = r0;
          ss.red[wq][transpose_col(lane, 1)] = r1;
          named_bar_sync(1, 128);
          bool any_rescale = false;
          if (t < 64) {
            const float mo = ss.m[t];
            const float cm = fmaxf(fmaxf(ss.red[0][t], ss.red[1][t]), fmaxf(ss.red[2][t], ss.red[3][t]));
            float mn = mo, a = 1.f;
            if (cm > ss.mthr[t]) {
              mn = fmaxf(mo, cm);
              a = (mo == -INFINITY) ? 0.f : ex2_approx(mo - mn);
            }
            ss.m[t] = mn;
            ss.mthr[t] = mn + kRescaleThreshold;
            ss.alpha[t] = a;
            any_rescale = a != 1.f;
          }
          const int need = named_bar_or(1, 128, any_rescale ? 1 : 0);
          if (need && j > 0) {
            // O^T columns must be rescaled: wait for the previous step's PV, then load/scale/store
            const long long gp = g - 1;
            ok = mbar_wait(&ss.empty[gp % kStages], static_cast<uint32_t>((gp / kStages) & 1), abort_flag, err, 122);
            if (!ok) break;
            tc_fence_after();
#pragma unroll
            for (int half = 0; half < 2; ++half) {
#pragma unroll
              for (int c = 0; c < 4; ++c) {
                uint32_t r[16];
                const uint32_t a = tmem + lane_base + kColO + half * 64 + c * 16;
                tmem_ld16(a, r);
                tmem_ld_wait();
#pragma unroll
                for (int q = 0; q < 16; ++q) r[q] = __float_as_uint(__uint_as_float(r[q]) * ss.alpha[c * 16 + q]);
                tmem_st16(a, r);
              }
            }
            tmem_st_wait();
          }
          if (need) {
#pragma unroll
            for (int q = 0; q < 64; ++q) l_part[q] *= ss.alpha[q];
          }
        }
        // ---- probabilities, row-sum partials, P^T row into the consumed K slot of this stage
        uint32_t packed[32];
#pragma unroll
        for (int q = 0; q < 64; q += 2) {
          const float p0 = ex2_approx(x[q] - ss.m[q]);
          const float p1 = ex2_approx(x[q + 1] - ss.m[q + 1]);
          l_part[q] += p0;
          l_part[q + 1] += p1;
          packed[q >> 1] = p.is_bf16 ? pack_bf16x2(p0, p1) : pack_f16x2(p0, p1);
        }
        uint8_t* prow = sStage + s * kStageBytes;
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          uint4 v = make_uint4(packed[4 * c], packed[4 * c + 1], packed[4 * c + 2], packed[4 * c + 3]);
          *reinterpret_cast<uint4*>(prow + sw128_offset(static_cast<uint32_t>(t), static_cast<uint32_t>(c))) = v;
        }
        fence_proxy_async_smem();
        tc_fence_before();
        mbar_arrive(&ss.p_full[sb]);
      }
      if (!ok) break;
      // ---- epilogue: row sums, O^T / l -> out
      {
        float r0, r1;
        transpose_reduce<false>(l_part, r0, r1, lane);
        ss.red[wq][transpose_col(lane, 0)] = r0;
        ss.red[wq][transpose_col(lane, 1)] = r1;
      }
      const long long gl = g - 1;
      ok = mbar_wait(&ss.empty[gl % kStages], static_cast<uint32_t>((gl / kStages) & 1), abort_flag, err, 123);
      if (!ok) break;
      tc_fence_after();
      float o[64];
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t ra[16], rb[16];
        tmem_ld16(tmem + lane_base + kColO + c * 16, ra);
        tmem_ld16(tmem + lane_base + kColO + 64 + c * 16, rb);
        tmem_ld_wait();
#pragma unroll
        for (int q = 0; q < 16; ++q) o[c * 16 + q] = __uint_as_float(ra[q]) + __uint_as_float(rb[q]);
      }
      tc_fence_before();
      mbar_arrive(&ss.o_empty);
      named_bar_sync(1, 128);
      if (t < 64) {
        const float l = ss.red[0][t] + ss.red[1][t] + ss.red[2][t] + ss.red[3][t];
        ss.alpha[t] = l > 0.f ? 1.f / l : 0.f;
      }
      named_bar_sync(1, 128);
      if (t < p.D) {
        int t0, h0, w0;
        block_origin(p, qblk, t0, h0, w0);
        const int b = bh / p.H;
        const int h = bh - b * p.H;
        const long long base = b * p.out_sb + h * p.out_sh + t;
        const int cHW = p.cH * p.cW;
#pragma unroll
        for (int q = 0; q < 64; ++q) {
          const int ct = q / cHW;
          const int rem = q - ct * cHW;
          const int ch = rem / p.cW;
          const int cw = rem - ch * p.cW;
          const long long tok = (static_cast<long long>(t0 + ct) * p.Hl + (h0 + ch)) * p.Wl + (w0 + cw);
          const float val = o[q] * ss.alpha[q];
          if (p.is_bf16)
            reinterpret_cast<__nv_bfloat16*>(p.out)[base + tok * p.out_ss] = __float2bfloat16_rn(val);
          else
            reinterpret_cast<__half*>(p.out)[base + tok * p.out_ss] = __float2half_rn(val);
        }
      }
      named_bar_sync(1, 128);
    }
  }
  // ------------------------------------------------------------------ teardown
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
    if (cudaFuncSetAttribute(bsa_attn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes) !=
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
  p.is_bf16 = a.is_bf16;
  p.total_units = p.BH * a.nb;
  const int grid = p.total_units < sms ? p.total_units : sms;
  if (grid <= 0) return BSA_OK;
  bsa_attn_kernel<<<grid, kThreads, kSmemBytes, stream>>>(*tm_q, *tm_k, *tm_v, p);
  return cudaGetLastError() == cudaSuccess ? BSA_OK : BSA_ERR_CUDA;
}

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
