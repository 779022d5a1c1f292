// Host-side planning of the library's launches: the forward's tile plan, the split-K plan
// of the plain GEMMs, the backward's token chunks and workspace layout, and the widening of
// the forward's vocabulary groups for the fixed-scratch entry point. Pure functions of the
// problem sizes (and of a few LP_B200_* tuning variables), so the CPU tests check them
// without a GPU (tests/sched/plan_check.cu).
#pragma once

#include <algorithm>
#include <cstdint>
#include <cstdlib>

#include "../../include/lp_logprob.h"
#include "lp_gemm.cuh"

namespace lpk {

inline int64_t cdiv(int64_t a, int64_t b) { return (a + b - 1) / b; }
inline size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

// Forward plan. The forward reads every H row block once per vocabulary tile, so the H rows
// that concurrent CTAs re-read must stay in L2: units walk the tokens in chunks of about
// 12288 rows (48 MB of bf16 H at d = 2048), and within a chunk all vocabulary groups
// before the next chunk. Each unit covers G consecutive vocabulary tiles; G keeps the
// per-row (max, sum) partials ([n_groups, T] float2) under ~128 MB.
inline GemmSched plan_fwd(int64_t T, int64_t Vs, int64_t d, int workers, int bm) {
  GemmSched s{};
  s.bm = bm;
  s.M = (int)T;
  s.N = (int)Vs;
  s.K = (int)d;
  s.tiles_m = (int)cdiv(T, bm);
  s.tiles_n = (int)cdiv(Vs, BN);
  s.k_blocks = (int)cdiv(d, BK);
  s.k_splits = 1;
  s.kb_per_split = s.k_blocks;
  s.n_fast = 0;
  static const char* chunk_env = getenv("LP_B200_FWD_CHUNK_MB");  // tuning: H chunk size
  const int64_t chunk_mb = (chunk_env != nullptr && atoi(chunk_env) > 0) ? atoi(chunk_env) : 48;
  const int64_t chunk_rows = std::max<int64_t>(bm, (chunk_mb << 20) / std::max<int64_t>(2 * d, 1));
  s.m_chunk = (int)std::max<int64_t>(1, chunk_rows / bm);
  static const char* no_chunk = getenv("LP_B200_FWD_NO_CHUNK");  // tuning: plain M-fast order
  if (no_chunk != nullptr && no_chunk[0] == '1') s.m_chunk = 0;
  const int64_t part_cap = int64_t(128) << 20;
  int g = 1;
  while (g < s.tiles_n && 2 * cdiv(s.tiles_n, g) * T * 8 > part_cap) g *= 2;
  // at least a few tiles per unit so the per-unit epilogue state amortises, unless that
  // leaves fewer than four units per worker (few tokens: T = 256 has two M tiles)
  const int g_part = g;
  g = std::max(g, std::min(4, s.tiles_n));
  while (g > g_part && (int64_t)s.tiles_m * cdiv(s.tiles_n, g) < 4 * (int64_t)std::max(workers, 1)) g /= 2;
  static const char* force_g = getenv("LP_B200_FWD_GROUP");  // tuning: tiles per unit
  if (force_g != nullptr && atoi(force_g) > 0) g = std::min(atoi(force_g), s.tiles_n);
  s.n_group = g;
  s.n_groups = (int)cdiv(s.tiles_n, g);
  s.num_units = s.tiles_m * s.n_groups;
  return s;
}

// Plain GEMM with optional split-K: pick S in [1, 16] minimising the critical path,
// keeping at least 8 K blocks per split; ties prefer fewer splits.
inline GemmSched plan_gemm(int64_t M, int64_t N, int64_t K, int sms, bool allow_split, int n_fast, int bm) {
  GemmSched s{};
  s.bm = bm;
  s.M = (int)M;
  s.N = (int)N;
  s.K = (int)K;
  s.tiles_m = (int)cdiv(M, bm);
  s.tiles_n = (int)cdiv(N, BN);
  s.k_blocks = (int)cdiv(K, BK);
  s.n_group = 1;
  s.n_groups = s.tiles_n;
  s.n_fast = n_fast;
  const int64_t tiles = (int64_t)s.tiles_m * s.tiles_n;
  int best_s = 1;
  double best = 1e300;
  const int smax = allow_split ? 64 : 1;
  // Concurrent units stream shared operands through L2; a unit longer than ~1024 K blocks
  // lets CTAs drift apart by more than L2 holds, so long K ranges are split.
  const int64_t kb_cap = 1024;
  // A split writes f32 partials that a separate pass reads back: S * M * N * 4 bytes each way,
  // charged in units of one K block's time on one worker (~512 cycles, in which the GPU
  // moves ~2 MB through HBM).
  const double reduce_units_per_split = (double)M * (double)N * 8.0 / (2.0 * 1024 * 1024);
  for (int sp = 1; sp <= smax; ++sp) {
    const int64_t kb = cdiv(s.k_blocks, sp);
    if (sp > 1 && kb < 8) break;
    if (allow_split && kb > kb_cap) continue;
    const int64_t real_splits = cdiv(s.k_blocks, kb);
    if (real_splits != sp) continue;
    const double c = (double)cdiv(tiles * sp, sms) * kb * (1.0 + 0.02 * (sp > 1)) +
                     (sp > 1 ? sp * reduce_units_per_split : 0.0);
    if (c < best * 0.995) {
      best = c;
      best_s = sp;
    }
  }
  s.kb_per_split = (int)cdiv(s.k_blocks, best_s);
  s.k_splits = (int)cdiv(s.k_blocks, s.kb_per_split);
  s.num_units = (int)(tiles * s.k_splits);
  return s;
}

// Plan of the dZ recompute GEMM (M = tokens of the chunk, N = the shard's vocabulary, K = d):
// every vocabulary tile re-reads the chunk's hidden rows, so the units walk the tokens in
// chunks of ~48 MB of hidden rows (LP_B200_DZ_MCHUNK_MB, 0 = plain M-fast order), all
// vocabulary tiles of a chunk before the next, as the forward does: the rows the CTAs in
// flight re-read stay in L2 however many tokens the backward chunk holds.
inline GemmSched plan_dz(int64_t M, int64_t Vs, int64_t d, int workers, int bm) {
  GemmSched s = plan_gemm(M, Vs, d, workers, false, 0, bm);
  static const int64_t mb = [] {
    const char* e = getenv("LP_B200_DZ_MCHUNK_MB");
    return (e != nullptr) ? (int64_t)atoll(e) : (int64_t)48;
  }();
  if (mb > 0) s.m_chunk = (int)std::max<int64_t>(1, (mb << 20) / std::max<int64_t>(2 * d, 1) / bm);
  return s;
}

// Backward token chunk: dZ (bf16 [chunk, Vs]) is the backward's only [T, V]-shaped buffer,
// and at most 4 GiB of it (LP_B200_DZ_CHUNK_MB) is kept: larger chunks at Vs = 262144 drew
// more power for no gain (16 GiB: 263.7k tokens/s at 1290 MHz vs 293.4k at 1395). The
// hidden rows a chunk's dZ GEMM re-reads stay in L2 through its M-chunked unit order
// (plan_dz), whatever the chunk size. Chunks are of equal size on 256-row boundaries: a
// short last chunk leaves most SMs idle at the end of each of its three GEMMs.
inline int64_t default_token_chunk(int64_t T, int64_t Vs, int64_t d) {
  (void)d;
  static const int64_t budget = [] {
    const char* e = getenv("LP_B200_DZ_CHUNK_MB");
    const long long mb = (e != nullptr && atoll(e) > 0) ? atoll(e) : 4096;
    return (int64_t)mb << 20;
  }();
  const int64_t ldz = (Vs + 7) / 8 * 8;
  const int64_t cap = std::max<int64_t>(256, budget / (ldz * 2) / 256 * 256);
  if (T <= cap) return std::max<int64_t>(T, 1);
  const int64_t chunks = cdiv(T, cap);
  return std::min<int64_t>(cap, cdiv(cdiv(T, chunks), 256) * 256);
}

struct BwdLayout {
  int64_t tc, chunks, ldz;
  size_t dz_off, part_off, dwacc_off, total;
  int max_splits;
  int64_t mpad;
};

inline BwdLayout bwd_layout(int64_t T, int64_t d, int64_t Vs, int64_t token_chunk, int flags, int sms, int bm) {
  BwdLayout L{};
  L.tc = token_chunk > 0 ? std::min<int64_t>(token_chunk, std::max<int64_t>(T, 1)) : default_token_chunk(T, Vs, d);
  L.chunks = T > 0 ? cdiv(T, L.tc) : 0;
  L.ldz = (Vs + 7) / 8 * 8;
  L.mpad = cdiv(L.tc, bm) * bm;
  // the largest split-K of any chunk (the first chunk is the largest)
  L.max_splits = 1;
  if (!(flags & LP_BWD_NO_DH) && T > 0) {
    GemmSched s = plan_gemm(L.tc, d, Vs, sms, true, 1, bm);
    L.max_splits = s.k_splits;
    // a shorter last chunk may choose more splits
    const int64_t last = T - (L.chunks - 1) * L.tc;
    GemmSched s2 = plan_gemm(last, d, Vs, sms, true, 1, bm);
    L.max_splits = std::max(L.max_splits, s2.k_splits);
  }
  size_t off = 0;
  L.dz_off = off;
  off += align_up((size_t)L.tc * L.ldz * 2, 1024);
  L.part_off = off;
  if (L.max_splits > 1) off += align_up((size_t)L.max_splits * L.mpad * d * 4, 1024);
  L.dwacc_off = off;
  if (!(flags & LP_BWD_NO_DW) && (flags & LP_BWD_DW_BF16) && L.chunks > 1) off += align_up((size_t)Vs * d * 4, 1024);
  L.total = off;
  return L;
}

// Scratch bytes of the forward's partials and target logits for plan `s` ([2 * n_groups, T]
// float2 + [T] f32, each 256-byte aligned); *part_bytes receives the first part.
inline size_t fwd_scratch_bytes(const GemmSched& s, int64_t T, size_t* part_bytes) {
  *part_bytes = align_up((size_t)2 * s.n_groups * T * 8, 256);
  return *part_bytes + align_up((size_t)T * 4, 256);
}

// Widens the vocabulary groups of forward plan `s` (doubling the tiles per unit) until its
// scratch fits `limit` bytes or there is one group; returns the scratch bytes of the result
// (which may still exceed `limit` when one group is not enough).
inline size_t widen_fwd_groups(GemmSched* s, int64_t T, size_t limit, size_t* part_bytes) {
  while (fwd_scratch_bytes(*s, T, part_bytes) > limit && s->n_group < s->tiles_n) {
    s->n_group = std::min(s->tiles_n, s->n_group * 2);
    s->n_groups = (int)cdiv(s->tiles_n, s->n_group);
    s->num_units = s->tiles_m * s->n_groups;
  }
  return fwd_scratch_bytes(*s, T, part_bytes);
}

}  // namespace lpk
