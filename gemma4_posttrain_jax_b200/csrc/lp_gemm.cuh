// Persistent, warp-specialised tcgen05 GEMM for sm_100a with pluggable epilogues.
//
//   D[M, N] = A[M, K] . B[N, K]^T       (bf16 operands, f32 accumulation in TMEM)
//
// CG = 1: one CTA per SM computes 128x256 tiles (tcgen05.mma.cta_group::1, M=128 N=256).
// CG = 2: a cluster of two CTAs on two SMs computes 256x256 tiles with one
//         tcgen05.mma.cta_group::2 (M=256 N=256) issued by the pair leader. Each CTA stages
//         its own 128 rows of A and its own half (128 rows) of B, so per SM the operand
//         traffic per MMA-FLOP drops by a third and the smem ring gets 6 stages instead of 4.
//         Each CTA's TMEM holds the accumulator rows of its half of the M tile.
//
// Persistent CTAs (CG = 2: CTA pairs) claim work units dynamically, in unit order, from an
// atomic counter (so the units in flight form a compact window of the order, which keeps
// the operands they share in L2). A unit is one M tile (128*CG rows), a run of consecutive
// 256-column N tiles and a range of 64-deep K blocks.
//
//   warp 0      : TMA producer (one thread)  -> NUM_STAGES-deep smem ring
//   warp 1      : TMEM allocator + MMA issuer (one thread; in the pair leader only)
//   warps 2..9  : epilogue; warp w reads TMEM lanes 32*(w%4).. (its 32 rows of the tile) and
//                 one half (128 columns) of the tile; two epilogue warps per SM sub-partition
//
// The two 256-column f32 accumulators (512 TMEM columns) are double-buffered, so the
// epilogue of tile i overlaps the MMAs of tile i+1. Operands are K-major or MN-major,
// staged by TMA with 128-byte swizzle.
//
// Epilogues:
//   EPI_FWD_LSE : softcap + running (max, sum-exp) per row in base 2 + target pick, never
//                 writing logits; one (max, sum) partial per row per unit and column half.
//   EPI_BWD_DZ  : recompute path; dZ = g * (onehot - softmax) * softcap' written as bf16
//                 through swizzled smem staging + TMA store.
//   EPI_STORE   : plain f32 / bf16 store or f32 TMA reduce-add of the accumulator.
//   EPI_HEAD    : sampler head: softcapped logits stored as f32 (optional), running
//                 (max, sum-exp) per row in base 2 and the first column of the row maximum;
//                 one partial of each per row per unit and column half.
//
// Synchronisation (all waits bounded, see lp_ptx.cuh):
//   full[s]   : TMA -> MMA. CG=2: lives in the leader, counts both CTAs' bytes.
//   empty[s]  : MMA -> TMA, in every CTA; CG=2: one multicast commit arrives on both copies.
//   tfull[b]  : MMA -> epilogue, in every CTA (CG=2: one multicast commit).
//   tempty[b] : epilogue -> MMA, in the leader; every epilogue warp of the pair arrives.
#pragma once

#include "lp_ptx.cuh"

// Shared-memory ring depth per CTA group: the largest that fits 227 KB with the epilogue
// staging (single CTAs: 4 x 48 KB; pairs: 6 x 32 KB, or 5 x 32 KB beside the 64 KB of
// 128-byte store staging of the plain-store GEMMs). Measured (pipeline counters, config-2
// workload): the single-CTA forward waits 639 / 207 / 103 cycles per K block for its loads
// with 2 / 3 / 4 stages. Pairs, per K block: the forward waits 98 / 94 / 146 cycles with
// 5 / 6 / 7 stages (7 x 32 KB fit without store staging; with 7 it runs 6 % slower: more
// loads in flight only queue longer), the dZ GEMM 140 / 122 with 5 / 6, dH and dW 125 / 88 and
// 169 / 124 with 4 / 5: the defaults are the best depth each way. Overridable at build time
// for tuning.
#ifndef LP_STAGES_CG1
#define LP_STAGES_CG1 4
#endif
#ifndef LP_STAGES_CG2
#define LP_STAGES_CG2 6
#endif
// 1: the pair's MMA thread signals a barrier in both CTAs with one multicast commit; 0: one
// commit per CTA.
#ifndef LP_PAIR_COMMIT_BOTH
#define LP_PAIR_COMMIT_BOTH 1
#endif
#ifndef LP_STAGES_CG2_STORE
#define LP_STAGES_CG2_STORE 5
#endif
#ifndef LP_STAGES_CG2_FWD
#define LP_STAGES_CG2_FWD LP_STAGES_CG2
#endif

namespace lpk {

constexpr int BN = 256;
constexpr int BK = 64;
constexpr int EPI_WARPS = 8;
constexpr int NUM_THREADS = 64 + 32 * EPI_WARPS;
constexpr int TMEM_COLS = 2 * BN;
constexpr int A_STAGE_BYTES = 128 * BK * 2;                // 16 KB: 128 rows of A per CTA
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

enum : int { EPI_FWD_LSE = 0, EPI_BWD_DZ = 1, EPI_STORE = 2, EPI_HEAD = 3 };
enum : int { STORE_BF16 = 0, STORE_F32 = 1, STORE_F32_ADD = 2 };

template <int CG>
struct Cfg {
  static constexpr int BM = 128 * CG;                      // rows of one M tile (the pair's for CG=2)
  static constexpr int B_ROWS = BN / CG;                   // rows of B staged by each CTA
  static constexpr int B_STAGE_BYTES = B_ROWS * BK * 2;    // 32 KB (CG=1) / 16 KB (CG=2)
  static constexpr int STAGE_BYTES = A_STAGE_BYTES + B_STAGE_BYTES;
};

// Epilogue TMA store box: 32 rows x store_row_bytes (64 B with 64-byte swizzle, or 128 B
// with 128-byte swizzle). The plain-store pair GEMMs (dH, dW) use 128-byte rows: half the
// store instructions per tile and whole 128-byte lines per row; the others keep 64-byte
// rows, which leave room for a deeper operand ring.
template <int CG, int EPI>
__host__ __device__ constexpr int store_row_bytes() {
  return (EPI == EPI_STORE && CG == 2) ? 128 : 64;
}

template <int CG, int EPI>
__host__ __device__ constexpr int staging_buf_bytes() {
  return 32 * store_row_bytes<CG, EPI>();
}

template <int CG, int EPI>
__host__ __device__ constexpr int num_stages() {
  return CG == 1 ? LP_STAGES_CG1
                 : (EPI == EPI_STORE ? LP_STAGES_CG2_STORE : (EPI == EPI_FWD_LSE ? LP_STAGES_CG2_FWD : LP_STAGES_CG2));
}

struct GemmSched {
  int M, N, K;
  int tiles_m, tiles_n, k_blocks;
  int n_group, n_groups;  // N tiles per unit, number of N groups
  int k_splits, kb_per_split;
  int num_units;
  int n_fast;  // 1: consecutive units step through N groups first (share the A tile)
  int bm;      // rows per M tile (128 * CG)
  int m_chunk; // > 0 (with n_fast = 0): units walk M in chunks of m_chunk tiles, all N groups
               // of a chunk before the next chunk, so the A rows CTAs re-read stay in L2
  // > 0: cross-rank sum of the output (n_fast, one tile per unit, no K split). The work list
  // holds one reduce item per M tile after the tiles: the reduce item of row block b follows
  // the tiles of row block b + red_lag, so the block is normally complete on every rank by
  // the time a CTA takes it.
  int red_lag;
};

struct EpiParams {
  const int32_t* y;      // [M] target ids (global vocabulary ids)
  long long v_off;       // first vocabulary id held by this shard
  float softcap;         // <= 0 means no softcap
  float2* part;          // FWD: [n_groups][M] (running max in base 2, running sum)
  float* tgt;            // FWD: [M] target logit (natural units), written by the owning tile
  float2* best;          // HEAD: [n_groups][M] (largest logit, its column as int bits)
  int store_logits;      // HEAD: store the logits through tmO (else only the row statistics)
  const float* g;        // DZ : [M] upstream d logp
  const float* stats;    // DZ : [2][stats_ld] global (max, sum) in natural units
  long long stats_ld;    // DZ : row stride of stats
  int store_mode;        // STORE: STORE_BF16 / STORE_F32 / STORE_F32_ADD
  // Cross-rank sum (sched red_lag > 0, STORE_BF16 into symmetric memory): every rank stores
  // its partial tiles locally and counts them on the row block's counter in all ranks' copies
  // (multimem.red); rank r then reduces its share of each block's rows (ld_reduce over all
  // copies through the NVSwitch, f32 accumulation) and stores the sum to all copies.
  __nv_bfloat16* sum_mc;        // multicast address of the output (row 0 of this launch)
  __nv_bfloat16* sum_local;     // this rank's address of the same rows (NaN-filled on a timeout)
  long long sum_ld;             // output row stride (elements, multiple of 8)
  unsigned* cnt_local;          // this rank's copy of the per-128-row-block tile counters
  unsigned* cnt_mc;             // their multicast address
  unsigned cnt_target;          // counter value of a complete block: world * tiles_n * EPI_WARPS * CG
  int sum_rank, sum_world;
  unsigned long long peer_limit_ns;  // bound of a wait for the other ranks' tiles
  int split_rows;        // STORE: output-row offset between K splits (partials)
  int a_l2, b_l2;        // L2 eviction priority of the A / B loads (L2_NORMAL / _EVICT_FIRST / _EVICT_LAST)
};

struct GemmParams {
  GemmSched s;
  EpiParams e;
  // Optional pipeline counters (nullptr = off), 8 per CTA, accumulated with atomicAdd:
  // [0] producer cycles waiting for a free stage, [1] MMA cycles waiting for loaded stages,
  // [2] MMA cycles waiting for a free accumulator, [3] epilogue-warp cycles waiting for a
  // full accumulator (warp 2), [4] MMA-thread cycles from start to drain, [5] K blocks
  // issued, [6] epilogue-warp cycles from accumulator ready to hand-back (warp 2), [7] tiles.
  unsigned long long* dbg;
  // Dynamic work distribution: units are claimed in order with atomicAdd on this counter
  // (zero at launch), so the units in flight always form a compact window of the unit order.
  unsigned int* sched;
  // MN-major operands with 3-D tensor maps (64 columns, K, 64-column chunks): the CTA's
  // tile of that operand is one TMA instruction instead of one per 64-column chunk.
  int a_mn3d, b_mn3d;
};

__device__ __forceinline__ unsigned long long clk64() { return (unsigned long long)clock64(); }

struct Unit {
  int m_tile, group, split;
  int n_begin, n_count;
  int kb_begin, kb_count;
  int red_block;  // >= 0: a reduce item of this row block (no tiles)
};

__host__ __device__ __forceinline__ Unit get_unit(const GemmSched& s, int u) {
  int m, g, ks;
  if (s.red_lag > 0) {
    // tiles and reduce items interleaved (see red_lag); tiles in n_fast order
    const int tn = s.tiles_n, lag = s.red_lag;
    int tile = -1, rb = -1;
    if (u < lag * tn) {
      tile = u;
    } else {
      const int j = u - lag * tn;
      const int q = j / (tn + 1), r = j % (tn + 1);
      if (q < s.tiles_m - lag) {
        if (r < tn) tile = (q + lag) * tn + r; else rb = q;
      } else {
        rb = (s.tiles_m - lag) + (j - (s.tiles_m - lag) * (tn + 1));
      }
    }
    Unit x;
    x.split = 0;
    x.kb_begin = 0;
    x.kb_count = s.k_blocks;
    if (tile >= 0) {
      x.m_tile = tile / tn;
      x.group = tile % tn;
      x.n_begin = x.group;
      x.n_count = 1;
      x.red_block = -1;
    } else {
      x.m_tile = rb;
      x.group = 0;
      x.n_begin = 0;
      x.n_count = 0;
      x.red_block = rb;
    }
    return x;
  }
  if (!s.n_fast && s.m_chunk > 0) {
    // chunk-major: (chunk, N group, M tile within the chunk); the last chunk may be short
    const int mc = s.m_chunk;
    const int full = s.tiles_m / mc;
    const int per_chunk = mc * s.n_groups;
    if (u < full * per_chunk) {
      const int c = u / per_chunk, r = u % per_chunk;
      g = r / mc;
      m = c * mc + r % mc;
    } else {
      const int lm = s.tiles_m - full * mc;
      const int r = u - full * per_chunk;
      g = r / lm;
      m = full * mc + r % lm;
    }
    ks = 0;
  } else if (s.n_fast) {
    g = u % s.n_groups;
    const int r = u / s.n_groups;
    m = r % s.tiles_m;
    ks = r / s.tiles_m;
  } else {
    m = u % s.tiles_m;
    const int r = u / s.tiles_m;
    g = r % s.n_groups;
    ks = r / s.n_groups;
  }
  Unit x;
  x.m_tile = m;
  x.group = g;
  x.split = ks;
  x.n_begin = g * s.n_group;
  x.n_count = min(s.n_group, s.tiles_n - x.n_begin);
  x.kb_begin = ks * s.kb_per_split;
  x.kb_count = min(s.kb_per_split, s.k_blocks - x.kb_begin);
  x.red_block = -1;
  return x;
}

template <int CG, int EPI>
__host__ __device__ constexpr int staging_bytes() {
  // double-buffered box per epilogue warp
  return EPI == EPI_FWD_LSE ? 0 : EPI_WARPS * 2 * staging_buf_bytes<CG, EPI>();
}

template <int CG, int EPI>
__host__ __device__ constexpr int gemm_smem_bytes() {
  // 1 KB alignment slack + stages + staging + barriers, work-unit ring, TMEM slot, abort flag
  return 1024 + num_stages<CG, EPI>() * Cfg<CG>::STAGE_BYTES + staging_bytes<CG, EPI>() + 512;
}

// Every kernel variant fits the 227 KB of dynamic shared memory a CTA may use.
static_assert(gemm_smem_bytes<1, EPI_FWD_LSE>() <= 232448 && gemm_smem_bytes<1, EPI_BWD_DZ>() <= 232448 &&
                  gemm_smem_bytes<1, EPI_STORE>() <= 232448 && gemm_smem_bytes<1, EPI_HEAD>() <= 232448 &&
                  gemm_smem_bytes<2, EPI_FWD_LSE>() <= 232448 && gemm_smem_bytes<2, EPI_BWD_DZ>() <= 232448 &&
                  gemm_smem_bytes<2, EPI_STORE>() <= 232448 && gemm_smem_bytes<2, EPI_HEAD>() <= 232448,
              "GEMM shared memory above 227 KB");

// Byte offset of 16-byte chunk c (0..3) of row r in a 64-byte-swizzled box of 64-byte rows
// (the TMA SWIZZLE_64B pattern: address bits [4,6) ^= bits [7,9)); 512-byte aligned box.
__device__ __forceinline__ uint32_t sw64_offset(int r, int c) { return (uint32_t)(r * 64 + ((c ^ ((r >> 1) & 3)) << 4)); }

// The same for chunk c (0..7) of a 128-byte-swizzled box of 128-byte rows (SWIZZLE_128B:
// address bits [4,7) ^= bits [7,10)); 1024-byte aligned box. Eight consecutive rows put a
// given chunk in eight different bank groups, so a warp's 16-byte stores do not conflict.
__device__ __forceinline__ uint32_t sw128_offset(int r, int c) { return (uint32_t)(r * 128 + ((c ^ (r & 7)) << 4)); }

template <int RB>
__device__ __forceinline__ uint32_t staging_offset(int r, int c) {
  if constexpr (RB == 128) return sw128_offset(r, c);
  else return sw64_offset(r, c);
}

// ----------------------------------------------------------------------------- kernel
template <int CG, int EPI, bool A_MN, bool B_MN, bool HAS_CAP>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    tc_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const __grid_constant__ CUtensorMap tmO, const GemmParams P) {
  using C = Cfg<CG>;
  constexpr int NS = num_stages<CG, EPI>();
  constexpr int SBUF = staging_buf_bytes<CG, EPI>();  // one staging box
  constexpr int RB = store_row_bytes<CG, EPI>();
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* stages = smem;
  uint8_t* staging = smem + NS * C::STAGE_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(staging + staging_bytes<CG, EPI>());
  uint64_t* full_bar = bars;             // [NS]
  uint64_t* empty_bar = bars + NS;       // [NS]
  uint64_t* tfull_bar = bars + 2 * NS;   // [2]
  uint64_t* tempty_bar = tfull_bar + 2;  // [2]
  uint64_t* done_bar = tempty_bar + 2;   // [1]
  // work-unit ring: the (pair leader's) producer claims units and publishes them here
  constexpr int SR = 8;
  uint64_t* sfull_bar = done_bar + 1;     // [SR] unit id written
  uint64_t* sempty_bar = sfull_bar + SR;  // [SR] every consumer has read it (leader's copy counts)
  volatile int* sched_u = reinterpret_cast<volatile int*>(sempty_bar + SR);  // [SR]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(const_cast<int*>(sched_u) + SR);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const GemmSched& S = P.s;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = CG == 2 ? cluster_ctarank() : 0u;  // position in the pair
  const bool leader = rank == 0;
  // consumers of a ring entry: the MMA thread and the epilogue warps (+ the peer's
  // producer and epilogue warps for a pair)
  constexpr int kRingConsumers = CG == 1 ? 1 + EPI_WARPS : 2 * (1 + EPI_WARPS);

  if (threadIdx.x == 0) {
    for (int s = 0; s < NS; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull_bar[b], 1);
      mbar_init(&tempty_bar[b], EPI_WARPS * CG);
    }
    mbar_init(done_bar, 1);
    for (int i = 0; i < SR; ++i) {
      mbar_init(&sfull_bar[i], 1);
      mbar_init(&sempty_bar[i], kRingConsumers);
    }
    *abort_flag = 0;
    fence_mbar_init();
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmB);
    if (EPI != EPI_FWD_LSE) prefetch_tmap(&tmO);
  }
  if (warp == 1) {
    if (CG == 2) {
      tmem_alloc_pair(tmem_slot, TMEM_COLS);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(tmem_slot, TMEM_COLS);
      tmem_relinquish();
    }
  }
  tc_fence_before();
  if (CG == 2) cluster_sync(); else __syncthreads();  // barriers initialised in both CTAs
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      // plain loads unless a priority was asked for (an explicit evict_normal policy is not
      // the same as no hint)
      const bool hint_a = P.e.a_l2 != L2_NORMAL, hint_b = P.e.b_l2 != L2_NORMAL;
      const uint64_t pol_a = hint_a ? make_l2_policy(P.e.a_l2) : 0;
      const uint64_t pol_b = hint_b ? make_l2_policy(P.e.b_l2) : 0;
      auto ld1 = [&](void* dst, const CUtensorMap* m, uint64_t* bar, int x, int y, bool h, uint64_t pol) {
        if (h) tma_load_2d_hint(dst, m, bar, x, y, pol); else tma_load_2d(dst, m, bar, x, y);
      };
      auto ld2 = [&](void* dst, const CUtensorMap* m, uint32_t bar, int x, int y, bool h, uint64_t pol) {
        if (h) tma_load_2d_pair_hint(dst, m, bar, x, y, pol); else tma_load_2d_pair(dst, m, bar, x, y);
      };
      uint32_t it = 0;
      unsigned long long dbg_wait_prod = 0;
      int last_stage_phase[NS];
#pragma unroll
      for (int s = 0; s < NS; ++s) last_stage_phase[s] = -1;
      bool ok = true;
      for (int i = 0; ok; ++i) {
        const int slot = i % SR;
        const uint32_t sph = (i / SR) & 1;
        int u;
        if (leader) {
          // claim the next unit and publish it (to the peer CTA too)
          const bool free_slot = CG == 1
                                     ? mbar_wait_bounded(&sempty_bar[slot], sph ^ 1, abort_flag, DEV_TIMEOUT_PRODUCER)
                                     : mbar_wait_bounded_cluster(&sempty_bar[slot], sph ^ 1, abort_flag,
                                                                 DEV_TIMEOUT_PRODUCER);
          if (!free_slot) break;
          const unsigned claimed = atomicAdd(P.sched, 1u);
          u = claimed < (unsigned)S.num_units ? (int)claimed : -1;
          sched_u[slot] = u;
          if constexpr (CG == 2) {
            st_shared_cluster_u32(mapa_shared(smem_u32(const_cast<int*>(&sched_u[slot])), 1), (uint32_t)u);
            mbar_arrive_remote(mapa_shared(smem_u32(&sfull_bar[slot]), 1));
          }
          mbar_arrive(&sfull_bar[slot]);
        } else {
          if (!mbar_wait_bounded_cluster(&sfull_bar[slot], sph, abort_flag, DEV_TIMEOUT_PRODUCER)) break;
          u = sched_u[slot];
          mbar_arrive_remote(mapa_shared(smem_u32(&sempty_bar[slot]), 0));
        }
        if (u < 0) break;
        const Unit un = get_unit(S, u);
        const int a_row = un.m_tile * C::BM + (int)rank * 128;
        for (int nt = un.n_begin; ok && nt < un.n_begin + un.n_count; ++nt) {
          const int b_row = nt * BN + (int)rank * C::B_ROWS;
          for (int kb = un.kb_begin; kb < un.kb_begin + un.kb_count; ++kb, ++it) {
            const int s = it % NS;
            const uint32_t ph = (it / NS) & 1;
            const unsigned long long w0 = P.dbg ? clk64() : 0ull;
            if (!mbar_wait_bounded(&empty_bar[s], ph ^ 1, abort_flag, DEV_TIMEOUT_PRODUCER)) {
              ok = false;
              break;
            }
            if (P.dbg) dbg_wait_prod += clk64() - w0;
            last_stage_phase[s] = (int)ph;
            uint8_t* a = stages + s * C::STAGE_BYTES;
            uint8_t* b = a + A_STAGE_BYTES;
            const int k0 = kb * BK;
            if constexpr (CG == 1) {
              mbar_arrive_expect_tx(&full_bar[s], C::STAGE_BYTES);
              if (!A_MN) {
                ld1(a, &tmA, &full_bar[s], k0, a_row, hint_a, pol_a);
              } else if (P.a_mn3d) {
                tma_load_3d(a, &tmA, &full_bar[s], 0, k0, a_row / 64);
              } else {
                ld1(a, &tmA, &full_bar[s], a_row, k0, hint_a, pol_a);
                ld1(a + 8192, &tmA, &full_bar[s], a_row + 64, k0, hint_a, pol_a);
              }
              if (!B_MN) {
                ld1(b, &tmB, &full_bar[s], k0, b_row, hint_b, pol_b);
              } else if (P.b_mn3d) {
                tma_load_3d(b, &tmB, &full_bar[s], 0, k0, b_row / 64);
              } else {
#pragma unroll
                for (int j = 0; j < C::B_ROWS / 64; ++j)
                  ld1(b + 8192 * j, &tmB, &full_bar[s], b_row + 64 * j, k0, hint_b, pol_b);
              }
            } else {
              // both CTAs' bytes land on the leader's full barrier
              if (leader) mbar_arrive_expect_tx(&full_bar[s], 2 * C::STAGE_BYTES);
              const uint32_t fb = mapa_shared(smem_u32(&full_bar[s]), 0);
              if (!A_MN) {
                ld2(a, &tmA, fb, k0, a_row, hint_a, pol_a);
              } else if (P.a_mn3d) {
                tma_load_3d_pair(a, &tmA, fb, 0, k0, a_row / 64);
              } else {
                ld2(a, &tmA, fb, a_row, k0, hint_a, pol_a);
                ld2(a + 8192, &tmA, fb, a_row + 64, k0, hint_a, pol_a);
              }
              if (!B_MN) {
                ld2(b, &tmB, fb, k0, b_row, hint_b, pol_b);
              } else if (P.b_mn3d) {
                tma_load_3d_pair(b, &tmB, fb, 0, k0, b_row / 64);
              } else {
#pragma unroll
                for (int j = 0; j < C::B_ROWS / 64; ++j) ld2(b + 8192 * j, &tmB, fb, b_row + 64 * j, k0, hint_b, pol_b);
              }
            }
          }
        }
      }
      if (P.dbg) atomicAdd(&P.dbg[blockIdx.x * 8 + 0], dbg_wait_prod);
      // Never leave with TMA writes in flight into this CTA's shared memory. The leader's
      // full barriers count both CTAs' bytes; in a healthy run every load was consumed by
      // an MMA (so these waits return at once), and after a timeout the wait limit is
      // orders of magnitude longer than any load.
      if (leader) {
        for (int s = 0; s < NS; ++s) {
          if (last_stage_phase[s] < 0) continue;
          const uint64_t t0 = globaltimer_ns();
          while (!mbar_try_wait(&full_bar[s], (uint32_t)last_stage_phase[s])) {
            if (globaltimer_ns() - t0 > kWaitLimitNs) {
              record_device_error(DEV_TIMEOUT_DRAIN);
              break;
            }
          }
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0 && leader) {
      constexpr uint32_t idesc = make_idesc_bf16(C::BM, BN, A_MN, B_MN);
      uint32_t it = 0, tc = 0;
      bool ok = true;
      const unsigned long long t_start = P.dbg ? clk64() : 0ull;
      unsigned long long dbg_full = 0, dbg_tempty = 0, dbg_kb = 0, dbg_tiles = 0;
      for (int i = 0; ok; ++i) {
        const int slot = i % SR;
        if (!mbar_wait_bounded(&sfull_bar[slot], (i / SR) & 1, abort_flag, DEV_TIMEOUT_MMA)) break;
        const int u = sched_u[slot];
        mbar_arrive(&sempty_bar[slot]);
        if (u < 0) break;
        const Unit un = get_unit(S, u);
        for (int nt = un.n_begin; ok && nt < un.n_begin + un.n_count; ++nt, ++tc) {
          const int buf = tc & 1;
          const uint32_t tph = (tc >> 1) & 1;
          const unsigned long long w0 = P.dbg ? clk64() : 0ull;
          if (!mbar_wait_bounded(&tempty_bar[buf], tph ^ 1, abort_flag, DEV_TIMEOUT_MMA)) {
            ok = false;
            break;
          }
          if (P.dbg) {
            dbg_tempty += clk64() - w0;
            dbg_tiles += 1;
          }
          tc_fence_after();
          const uint32_t d_tmem = tmem_base + (uint32_t)(buf * BN);
          // Peek at the next stage's barrier (non-blocking) before issuing this stage's MMAs,
          // so a stage that has already landed costs no blocking wait.
          bool ready = mbar_test_wait(&full_bar[it % NS], (it / NS) & 1);
          for (int kb = 0; kb < un.kb_count; ++kb, ++it) {
            const int s = it % NS;
            const uint32_t ph = (it / NS) & 1;
            const unsigned long long w1 = P.dbg ? clk64() : 0ull;
            if (!ready && !mbar_wait_bounded(&full_bar[s], ph, abort_flag, DEV_TIMEOUT_MMA)) {
              ok = false;
              break;
            }
            ready = kb + 1 < un.kb_count && mbar_test_wait(&full_bar[(it + 1) % NS], ((it + 1) / NS) & 1);
            if (P.dbg) {
              dbg_full += clk64() - w1;
              dbg_kb += 1;
            }
            tc_fence_after();
            const uint32_t a_addr = smem_u32(stages + s * C::STAGE_BYTES);
            const uint32_t b_addr = a_addr + A_STAGE_BYTES;
#pragma unroll
            for (int kk = 0; kk < BK / 16; ++kk) {
              const uint64_t ad =
                  A_MN ? smem_desc_sw128(a_addr + kk * 2048, 8192, 1024) : smem_desc_sw128(a_addr + kk * 32, 16, 1024);
              const uint64_t bd =
                  B_MN ? smem_desc_sw128(b_addr + kk * 2048, 8192, 1024) : smem_desc_sw128(b_addr + kk * 32, 16, 1024);
              if constexpr (CG == 1)
                mma_bf16_ss(d_tmem, ad, bd, idesc, (kb > 0 || kk > 0) ? 1u : 0u);
              else
                mma_bf16_ss_pair(d_tmem, ad, bd, idesc, (kb > 0 || kk > 0) ? 1u : 0u);
            }
            // free the smem stage (in every CTA of the pair) once these MMAs have read it
            if constexpr (CG == 1) {
              mma_commit(&empty_bar[s]);
            } else if (LP_PAIR_COMMIT_BOTH) {
              mma_commit_pair_both(smem_u32(&empty_bar[s]), 0x3);
            } else {
              const uint32_t eb = smem_u32(&empty_bar[s]);
              mma_commit_pair(mapa_shared(eb, 0));
              mma_commit_pair(mapa_shared(eb, 1));
            }
          }
          if (!ok) break;
          // accumulator ready for the epilogue warps (of every CTA of the pair)
          if constexpr (CG == 1) {
            mma_commit(&tfull_bar[buf]);
          } else if (LP_PAIR_COMMIT_BOTH) {
            mma_commit_pair_both(smem_u32(&tfull_bar[buf]), 0x3);
          } else {
            const uint32_t fb = smem_u32(&tfull_bar[buf]);
            mma_commit_pair(mapa_shared(fb, 0));
            mma_commit_pair(mapa_shared(fb, 1));
          }
        }
      }
      if (P.dbg) {
        unsigned long long* d = &P.dbg[blockIdx.x * 8];
        atomicAdd(d + 1, dbg_full);
        atomicAdd(d + 2, dbg_tempty);
        atomicAdd(d + 4, clk64() - t_start);
        atomicAdd(d + 5, dbg_kb);
        atomicAdd(d + 7, dbg_tiles);
      }
      // Drain: every MMA issued by this thread completes before TMEM is released.
      if constexpr (CG == 1) mma_commit(done_bar); else mma_commit_pair(mapa_shared(smem_u32(done_bar), 0));
      const uint64_t t0 = globaltimer_ns();
      while (!mbar_try_wait(done_bar, 0)) {
        if (globaltimer_ns() - t0 > kWaitLimitNs) {
          record_device_error(DEV_TIMEOUT_DRAIN);
          break;
        }
      }
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------------ epilogue warps
    // Two warps per TMEM lane quarter: warp 2+e (e = 0..7) reads lanes 32*(warp%4).. and
    // columns [128*h, 128*h + 128) of every tile, h = e / 4.
    const int q = warp & 3;
    const int ew = warp - 2;
    const int h = ew / 4;
    const uint32_t lane_base = (uint32_t)(q * 32) << 16;
    uint8_t* my_staging = staging + ew * 2 * SBUF;
    int sb = 0;
    uint32_t tc = 0;
    const EpiParams& E = P.e;
    const float cap = E.softcap;
    const float k1 = HAS_CAP ? 2.0f * kLog2e / cap : 0.f;  // x -> 2x/c in base 2
    const float c2 = HAS_CAP ? cap * kLog2e : 0.f;        // c in base 2
    bool ok = true;
    const bool dbg_warp = P.dbg != nullptr && warp == 2 && lane == 0;
    unsigned long long dbg_wait = 0, dbg_busy = 0, dbg_t = 0;

    for (int i = 0; ok; ++i) {
      const int slot = i % SR;
      const uint32_t sph = (i / SR) & 1;
      const bool got = CG == 1 || leader
                           ? mbar_wait_bounded(&sfull_bar[slot], sph, abort_flag, DEV_TIMEOUT_EPILOGUE)
                           : mbar_wait_bounded_cluster(&sfull_bar[slot], sph, abort_flag, DEV_TIMEOUT_EPILOGUE);
      if (!__all_sync(0xffffffffu, got)) break;
      const int u = sched_u[slot];
      __syncwarp();
      if (lane == 0) {
        if (CG == 1 || leader)
          mbar_arrive(&sempty_bar[slot]);
        else
          mbar_arrive_remote(mapa_shared(smem_u32(&sempty_bar[slot]), 0));
      }
      if (u < 0) break;
      const Unit un = get_unit(S, u);
      const int row_base = un.m_tile * C::BM + (int)rank * 128 + q * 32;  // first row of this warp
      const int row = row_base + lane;
      const bool row_ok = row < S.M;

      // per-row state
      int yl = -1;
      float run_m = -INFINITY, run_s = 0.f;
      float best_z = -INFINITY;  // HEAD: largest logit so far (natural units) and its column
      int best_i = -1;
      float gv = 0.f, l2 = 0.f;
      if (EPI == EPI_FWD_LSE) {
        if (row_ok) {
          const long long t = (long long)E.y[row] - E.v_off;
          yl = (t >= 0 && t < (long long)S.N) ? (int)t : -1;
        }
      } else if (EPI == EPI_BWD_DZ) {
        if (row_ok) {
          const long long t = (long long)E.y[row] - E.v_off;
          yl = (t >= 0 && t < (long long)S.N) ? (int)t : -1;
          gv = E.g[row];
          l2 = E.stats[row] * kLog2e + log2f(E.stats[E.stats_ld + row]);
        }
      }
      const float ng = -gv, ng4 = -4.f * gv;  // dZ of a non-target column, without / with softcap
      const float c2ml2 = c2 - l2;

      for (int nt = un.n_begin; nt < un.n_begin + un.n_count; ++nt, ++tc) {
        const int buf = tc & 1;
        const uint32_t tph = (tc >> 1) & 1;
        if (dbg_warp) dbg_t = clk64();
        // warp-uniform decision: tcgen05.ld below is .sync.aligned
        if (!__all_sync(0xffffffffu, mbar_wait_bounded(&tfull_bar[buf], tph, abort_flag, DEV_TIMEOUT_EPILOGUE))) {
          ok = false;
          break;
        }
        if (dbg_warp) {
          const unsigned long long now = clk64();
          dbg_wait += now - dbg_t;
          dbg_t = now;
        }
        tc_fence_after();
        const uint32_t taddr = tmem_base + lane_base + (uint32_t)(buf * BN + h * (BN / 2));
        const int colh = nt * BN + h * (BN / 2);  // first column of this warp's half

        if constexpr (EPI == EPI_FWD_LSE) {
#pragma unroll 1
          for (int c = 0; c < BN / 64; ++c) {
            uint32_t r[32];
            __syncwarp();
            tmem_ld32(taddr + c * 32, r);
            tmem_wait_ld(r);
            const int col0 = colh + c * 32;
            const int nvalid = S.N - col0;  // columns >= nvalid are vocabulary padding (warp-uniform)
            if (nvalid <= 0) continue;
            float mx0 = -INFINITY, mx1 = -INFINITY;
            if (nvalid >= 32) {
#pragma unroll
              for (int j = 0; j < 32; ++j) {
                const float x = __uint_as_float(r[j]);
                const float z = HAS_CAP ? fmaf(-2.f * c2, fast_rcp(1.f + fast_ex2(x * k1)), c2) : x * kLog2e;
                r[j] = __float_as_uint(z);
                if (j & 1) mx1 = fmaxf(mx1, z); else mx0 = fmaxf(mx0, z);
              }
            } else {
#pragma unroll
              for (int j = 0; j < 32; ++j) {
                const float x = __uint_as_float(r[j]);
                float z = HAS_CAP ? fmaf(-2.f * c2, fast_rcp(1.f + fast_ex2(x * k1)), c2) : x * kLog2e;
                z = (j < nvalid) ? z : -INFINITY;
                r[j] = __float_as_uint(z);
                if (j & 1) mx1 = fmaxf(mx1, z); else mx0 = fmaxf(mx0, z);
              }
            }
            const int tj = yl - col0;
            if ((unsigned)tj < 32u) {
              float tv = 0.f;
#pragma unroll
              for (int j = 0; j < 32; ++j) tv = (j == tj) ? __uint_as_float(r[j]) : tv;
              E.tgt[row] = tv * kLn2;
            }
            const float nm = fmaxf(run_m, fmaxf(mx0, mx1));
            const float scale = (nm == run_m) ? 1.f : fast_ex2(run_m - nm);
            float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
#pragma unroll
            for (int j = 0; j < 32; j += 4) {
              s0 += fast_ex2(__uint_as_float(r[j + 0]) - nm);
              s1 += fast_ex2(__uint_as_float(r[j + 1]) - nm);
              s2 += fast_ex2(__uint_as_float(r[j + 2]) - nm);
              s3 += fast_ex2(__uint_as_float(r[j + 3]) - nm);
            }
            run_s = fmaf(run_s, scale, (s0 + s1) + (s2 + s3));
            run_m = nm;
          }
        } else if constexpr (EPI == EPI_BWD_DZ) {
#pragma unroll 1
          for (int pc = 0; pc < BN / 64; ++pc) {
            uint32_t r[32];
            __syncwarp();
            tmem_ld32(taddr + pc * 32, r);
            tmem_wait_ld(r);
            const int col0 = colh + pc * 32;
            const int tj = yl - col0;
            // dZ = g * (onehot - p) * (1 - tanh^2) with p = 2^(z2 - l2). Per column, without the
            // one-hot term: with r = 1 / (1 + e^(2x/c)), z2 = c2 - 2 c2 r, 1 - tanh^2 = 4 r (1 - r),
            //   dZ = (-4 g) * r * (1 - r) * 2^(fma(-2 c2, r, c2 - l2)).
            // The target column (at most one per row) adds g * (1 - tanh^2) afterwards.
            float v[32];
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              const float x = __uint_as_float(r[j]);
              if (HAS_CAP) {
                const float rr = fast_rcp(1.f + fast_ex2(x * k1));
                const float p = fast_ex2(fmaf(-2.f * c2, rr, c2ml2));
                v[j] = ng4 * rr * (1.f - rr) * p;
              } else {
                v[j] = ng * fast_ex2(fmaf(x, kLog2e, -l2));
              }
            }
            if ((unsigned)tj < 32u) {
#pragma unroll
              for (int j = 0; j < 32; ++j) {
                if (j == tj) {
                  const float x = __uint_as_float(r[j]);
                  float chain = 1.f;
                  if (HAS_CAP) {
                    const float rr = fast_rcp(1.f + fast_ex2(x * k1));
                    chain = 4.f * rr * (1.f - rr);
                  }
                  v[j] += gv * chain;
                }
              }
            }
            uint32_t pk[16];
#pragma unroll
            for (int j = 0; j < 16; ++j) pk[j] = pack_bf16x2(v[2 * j], v[2 * j + 1]);
            if (lane == 0) bulk_wait_read<1>();
            __syncwarp();
            uint8_t* buf_s = my_staging + sb * SBUF;
            const uint32_t sbase = smem_u32(buf_s);
#pragma unroll
            for (int c = 0; c < 4; ++c)
              st_shared_v4(sbase + sw64_offset(lane, c), pk[4 * c], pk[4 * c + 1], pk[4 * c + 2], pk[4 * c + 3]);
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
              tma_store_2d(&tmO, buf_s, col0, row_base);
              bulk_commit();
            }
            sb ^= 1;
          }
        } else if constexpr (EPI == EPI_HEAD) {
          // z = c * tanh(x / c) = c * (1 - 2 r), r = 1 / (1 + 2^(2x log2(e) / c)), or z = x
#pragma unroll 1
          for (int pc = 0; pc < BN / 32; ++pc) {
            uint32_t r[16];
            __syncwarp();
            tmem_ld16(taddr + pc * 16, r);
            tmem_wait_ld16(r);
            const int col0 = colh + pc * 16;
            const int nvalid = S.N - col0;  // columns >= nvalid are vocabulary padding (warp-uniform)
            float mx = -INFINITY;
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              const float x = __uint_as_float(r[j]);
              const float z = HAS_CAP ? fmaf(-2.f * cap, fast_rcp(1.f + fast_ex2(x * k1)), cap) : x;
              r[j] = __float_as_uint(z);
              if (j < nvalid) {
                if (z > best_z) {  // strict: the first column of a tie is kept
                  best_z = z;
                  best_i = col0 + j;
                }
                mx = fmaxf(mx, z);
              }
            }
            if (nvalid > 0) {
              const float nm = fmaxf(run_m, mx * kLog2e);
              const float scale = (nm == run_m) ? 1.f : fast_ex2(run_m - nm);
              float s0 = 0.f, s1 = 0.f;
#pragma unroll
              for (int j = 0; j < 16; j += 2) {
                if (j < nvalid) s0 += fast_ex2(fmaf(__uint_as_float(r[j]), kLog2e, -nm));
                if (j + 1 < nvalid) s1 += fast_ex2(fmaf(__uint_as_float(r[j + 1]), kLog2e, -nm));
              }
              run_s = fmaf(run_s, scale, s0 + s1);
              run_m = nm;
            }
            if (E.store_logits && nvalid > 0) {
              if (lane == 0) bulk_wait_read<1>();
              __syncwarp();
              uint8_t* buf_s = my_staging + sb * SBUF;
              const uint32_t sbase = smem_u32(buf_s);
#pragma unroll
              for (int c = 0; c < 4; ++c)
                st_shared_v4(sbase + sw64_offset(lane, c), r[4 * c], r[4 * c + 1], r[4 * c + 2], r[4 * c + 3]);
              fence_proxy_async_smem();
              __syncwarp();
              if (lane == 0) {
                tma_store_2d(&tmO, buf_s, col0, row_base);
                bulk_commit();
              }
              sb ^= 1;
            }
          }
        } else {  // EPI_STORE
          const int row0 = un.split * E.split_rows + row_base;
          if (E.store_mode == STORE_BF16) {
            constexpr int COLS = RB / 2;  // bf16 columns per box
#pragma unroll 1
            for (int pc = 0; pc < (BN / 2) / COLS; ++pc) {
              uint32_t pk[COLS / 2];
#pragma unroll
              for (int q = 0; q < COLS / 32; ++q) {
                uint32_t r[32];
                __syncwarp();
                tmem_ld32(taddr + pc * COLS + q * 32, r);
                tmem_wait_ld(r);
#pragma unroll
                for (int j = 0; j < 16; ++j)
                  pk[q * 16 + j] = pack_bf16x2(__uint_as_float(r[2 * j]), __uint_as_float(r[2 * j + 1]));
              }
              if (lane == 0) bulk_wait_read<1>();
              __syncwarp();
              uint8_t* buf_s = my_staging + sb * SBUF;
              const uint32_t sbase = smem_u32(buf_s);
#pragma unroll
              for (int c = 0; c < RB / 16; ++c)
                st_shared_v4(sbase + staging_offset<RB>(lane, c), pk[4 * c], pk[4 * c + 1], pk[4 * c + 2],
                             pk[4 * c + 3]);
              fence_proxy_async_smem();
              __syncwarp();
              if (lane == 0) {
                tma_store_2d(&tmO, buf_s, colh + pc * COLS, row0);
                bulk_commit();
              }
              sb ^= 1;
            }
          } else {
            constexpr int COLS = RB / 4;  // f32 columns per box
#pragma unroll 1
            for (int pc = 0; pc < (BN / 2) / COLS; ++pc) {
              uint32_t r[COLS];
              __syncwarp();
              if constexpr (COLS == 32) {
                tmem_ld32(taddr + pc * COLS, r);
                tmem_wait_ld(r);
              } else {
                tmem_ld16(taddr + pc * COLS, r);
                tmem_wait_ld16(r);
              }
              if (lane == 0) bulk_wait_read<1>();
              __syncwarp();
              uint8_t* buf_s = my_staging + sb * SBUF;
              const uint32_t sbase = smem_u32(buf_s);
#pragma unroll
              for (int c = 0; c < RB / 16; ++c)
                st_shared_v4(sbase + staging_offset<RB>(lane, c), r[4 * c], r[4 * c + 1], r[4 * c + 2], r[4 * c + 3]);
              fence_proxy_async_smem();
              __syncwarp();
              if (lane == 0) {
                if (E.store_mode == STORE_F32_ADD)
                  tma_reduce_add_2d(&tmO, buf_s, colh + pc * COLS, row0);
                else
                  tma_store_2d(&tmO, buf_s, colh + pc * COLS, row0);
                bulk_commit();
              }
              sb ^= 1;
            }
          }
        }

        // hand the accumulator back to the MMA warp (in the leader for CG = 2)
        tc_fence_before();
        __syncwarp();
        if (dbg_warp) dbg_busy += clk64() - dbg_t;
        if (lane == 0) {
          if constexpr (CG == 1)
            mbar_arrive(&tempty_bar[buf]);
          else
            mbar_arrive_remote(mapa_shared(smem_u32(&tempty_bar[buf]), 0));
        }
        if (EPI == EPI_STORE && E.cnt_mc != nullptr) {
          // this warp's rows of the partial tile are in this rank's memory: count them on the
          // row block's counter in every rank's copy
          if (lane == 0) {
            bulk_wait<0>();
            fence_proxy_async_global();
            multimem_red_add_release_u32(E.cnt_mc + (size_t)un.m_tile * (C::BM / 128), 1u);
          }
          __syncwarp();
        }
      }
      if (!ok) break;

      if (EPI == EPI_STORE && un.red_block >= 0) {
        // Reduce item: once every rank has stored all tiles of the row block, sum this rank's
        // share of its rows over all ranks' copies (ld_reduce through the NVSwitch) and store
        // the sum to every copy. The pair's CTAs split the share.
        const int b = un.red_block;
        const int lo = b * C::BM + (E.sum_rank * C::BM) / E.sum_world;
        const int hi = b * C::BM + ((E.sum_rank + 1) * C::BM) / E.sum_world;
        const int r0 = lo + ((hi - lo) * (int)rank) / CG;
        const int r1 = min(lo + ((hi - lo) * ((int)rank + 1)) / CG, S.M);
        const int vpr = S.N >> 3;  // 16-byte vectors per row
        const int nv = r0 < r1 ? (r1 - r0) * vpr : 0;
        constexpr int NT = EPI_WARPS * 32;
        bool ready = true;
        if (lane == 0)
          ready = wait_counter_bounded(E.cnt_local + (size_t)b * (C::BM / 128), E.cnt_target, abort_flag,
                                       E.peer_limit_ns);
        if (!__shfl_sync(0xffffffffu, (int)ready, 0)) {
          // another rank's tiles never arrived: this share of the sum does not exist, so its
          // rows in this rank's copy get bf16 NaN rather than this rank's partial alone
          const uint4 nan8 = make_uint4(0x7fc07fc0u, 0x7fc07fc0u, 0x7fc07fc0u, 0x7fc07fc0u);
          for (int v = ew * 32 + lane; v < nv; v += NT)
            *reinterpret_cast<uint4*>(E.sum_local + (size_t)(r0 + v / vpr) * E.sum_ld + (v % vpr) * 8) = nan8;
          ok = false;
          break;
        }
        for (int v0 = ew * 32 + lane; v0 < nv; v0 += 4 * NT) {
          uint4 acc[4];
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const int v = v0 + k * NT;
            if (v < nv) acc[k] = multimem_ld_reduce_bf16x8(E.sum_mc + (size_t)(r0 + v / vpr) * E.sum_ld + (v % vpr) * 8);
          }
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const int v = v0 + k * NT;
            if (v < nv) multimem_st_bf16x8(E.sum_mc + (size_t)(r0 + v / vpr) * E.sum_ld + (v % vpr) * 8, acc[k]);
          }
        }
      }

      if constexpr (EPI == EPI_FWD_LSE || EPI == EPI_HEAD) {
        // one (max, sum) partial per unit and column half
        if (row_ok) E.part[(size_t)(un.group * 2 + h) * S.M + row] = make_float2(run_m, run_s);
      }
      if constexpr (EPI == EPI_HEAD) {
        if (row_ok) E.best[(size_t)(un.group * 2 + h) * S.M + row] = make_float2(best_z, __int_as_float(best_i));
      }
    }
    if (EPI != EPI_FWD_LSE) {
      if (lane == 0) bulk_wait<0>();  // all TMA stores of this warp complete before exit
      // the multicast stores are performed at system scope before the kernel ends, so a
      // peer barrier after this launch publishes them
      if (E.cnt_mc != nullptr) fence_sys();
      __syncwarp();
    }
    if (dbg_warp) {
      atomicAdd(&P.dbg[blockIdx.x * 8 + 3], dbg_wait);
      atomicAdd(&P.dbg[blockIdx.x * 8 + 6], dbg_busy);
    }
  }

  tc_fence_before();
  if (CG == 2) cluster_sync(); else __syncthreads();  // the pair's MMAs and loads are done
  if (warp == 1) {
    tc_fence_after();
    if (CG == 2) tmem_dealloc_pair(tmem_base, TMEM_COLS); else tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

}  // namespace lpk
