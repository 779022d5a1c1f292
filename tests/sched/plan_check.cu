// Host-side checks of the launch planning in lp_plan.cuh (compiled with nvcc as a host
// program and run on the CPU by tests/test_plan.py): backward token chunks, split-K choices,
// the forward's vocabulary groups and their widening for the fixed-scratch forward.
#include <cstdio>

#include "../../gemma4_posttrain_jax_b200/csrc/lp_plan.cuh"

static int failures = 0;
#define CHECK(cond)                                                   \
  do {                                                                \
    if (!(cond)) {                                                    \
      std::printf("FAILED %s:%d: %s\n", __FILE__, __LINE__, #cond); \
      ++failures;                                                     \
    }                                                                 \
  } while (0)

int main() {
  using namespace lpk;
  const int pairs = 74, sms = 148;

  // config 2 (97,703 backward rows): 4 GiB of dZ is 8192 rows at V = 262144 (12 chunks);
  // at 32768 rows per shard (8 GPUs) it would be 65536, so two equal chunks of 48896
  CHECK(default_token_chunk(97703, 262144, 2048) == 8192);
  CHECK(default_token_chunk(97703, 32768, 2048) == 48896);
  CHECK(default_token_chunk(97703, 131072, 2048) == 16384);
  CHECK(default_token_chunk(256, 262144, 2048) == 256);
  CHECK(default_token_chunk(32768, 65536, 3840) == 32768);  // config 4 at 4 GPUs: one chunk
  // chunks are equal up to the 256-row rounding: no short tail
  for (int64_t T : {20000, 97703, 100001, 262144}) {
    for (int64_t Vs : {32768, 65536, 262144}) {
      const int64_t tc = default_token_chunk(T, Vs, 2048);
      const int64_t chunks = cdiv(T, tc);
      const int64_t last = T - (chunks - 1) * tc;
      CHECK(tc % 256 == 0 || tc == T);
      CHECK(chunks == 1 || last > tc - 256 * chunks);
      CHECK((size_t)tc * Vs * 2 <= (size_t(4) << 30) || tc == 256);
    }
  }

  // split-K of the dH GEMM (pairs, 256-row tiles, K = the shard's vocabulary)
  {
    const GemmSched s = plan_gemm(8192, 2048, 262144, pairs, true, 1, 256);  // config 2 at one GPU
    CHECK(s.k_splits >= 4 && s.kb_per_split <= 1024);
    const GemmSched t = plan_gemm(15783, 2048, 32768, pairs, true, 1, 256);  // last chunk at 8 GPUs
    CHECK(t.k_splits == 1);  // the partials' round trip outweighs the wave tail
    const GemmSched u = plan_gemm(256, 2048, 262144, pairs, true, 1, 256);  // config 1: 8 tiles only
    CHECK(u.k_splits > 8 && u.kb_per_split >= 8);
    for (int64_t M : {256, 1000, 8192, 16384}) {
      const GemmSched g = plan_gemm(M, 2048, 32768, pairs, true, 1, 256);
      CHECK(g.k_splits == 1 || g.kb_per_split >= 8);
      CHECK((int64_t)g.k_splits * g.kb_per_split >= g.k_blocks);
      CHECK((int64_t)(g.k_splits - 1) * g.kb_per_split < g.k_blocks);
      CHECK(g.num_units == g.tiles_m * g.tiles_n * g.k_splits);
    }
    const GemmSched n = plan_gemm(8192, 2048, 262144, pairs, false, 1, 256);  // mesh sum: no split
    CHECK(n.k_splits == 1);
  }

  // dZ recompute: no split, token chunks of 12288 rows (48 MB of hidden rows) walked chunk by
  // chunk, every vocabulary tile of a chunk before the next
  {
    const GemmSched z = plan_dz(48896, 32768, 2048, sms, 128);
    CHECK(z.k_splits == 1 && z.n_fast == 0 && z.m_chunk == 96);
    CHECK(z.num_units == z.tiles_m * z.tiles_n);
  }

  // forward plan of config 2 at one GPU: 16 vocabulary tiles per unit (the partials stay
  // under 128 MB), 12288-row H chunks
  {
    const GemmSched f = plan_fwd(108376, 262144, 2048, sms, 128);
    CHECK(f.n_group == 16 && f.n_groups == 64 && f.m_chunk == 96);
    CHECK(f.num_units == f.tiles_m * f.n_groups);
    size_t part = 0;
    CHECK(fwd_scratch_bytes(f, 108376, &part) <= (size_t(129) << 20));
  }

  // few tokens (config 1, T = 256: two M tiles): smaller groups, so the forward has at least
  // four units per SM
  {
    const GemmSched f = plan_fwd(256, 262144, 2048, sms, 128);
    CHECK(f.n_group == 2 && f.num_units == 1024);
    const GemmSched h = plan_fwd(4096, 262144, 2048, sms, 128);  // 32 M tiles: the default 4 tiles
    CHECK(h.n_group == 4);
  }

  // fixed-scratch forward: groups widen until the partials fit 8 MiB
  {
    const size_t limit = size_t(8) << 20;
    GemmSched s = plan_fwd(60000, 70000, 64, sms, 128);
    CHECK(s.n_group == 4 && s.n_groups == 69);
    size_t part = 0;
    CHECK(fwd_scratch_bytes(s, 60000, &part) > limit);
    const size_t need = widen_fwd_groups(&s, 60000, limit, &part);
    CHECK(need <= limit && s.n_group == 64 && s.n_groups == 5 && s.num_units == s.tiles_m * 5);
    GemmSched big = plan_fwd(419424, 262144, 2048, sms, 128);
    CHECK(widen_fwd_groups(&big, 419424, limit, &part) <= limit && big.n_groups == 1);
    GemmSched over = plan_fwd(419425, 262144, 2048, sms, 128);
    CHECK(widen_fwd_groups(&over, 419425, limit, &part) > limit);
    GemmSched two = plan_fwd(233016, 262144, 2048, sms, 128);
    widen_fwd_groups(&two, 233016, limit, &part);
    CHECK(two.n_groups == 2);
  }

  // backward workspace: dZ chunk + the largest split's partials + the f32 dW accumulator
  {
    const BwdLayout L = bwd_layout(97703, 2048, 262144, 0, LP_BWD_DW_BF16, pairs, 256);
    CHECK(L.tc == 8192 && L.chunks == 12);
    CHECK(L.part_off >= (size_t)8192 * 262144 * 2);
    CHECK(L.max_splits >= 4);
    CHECK(L.total >= L.dwacc_off + (size_t)262144 * 2048 * 4);
    const BwdLayout M = bwd_layout(97703, 2048, 32768, 0, LP_BWD_DW_BF16, pairs, 256);
    CHECK(M.tc == 48896 && M.chunks == 2 && M.max_splits == 1);
    const BwdLayout F = bwd_layout(256, 2048, 262144, 0, LP_BWD_DW_BF16, pairs, 256);
    CHECK(F.chunks == 1 && F.dwacc_off == F.total);  // one chunk: dW stored as bf16 directly
  }

  if (failures == 0) std::printf("plan: ok\n");
  return failures == 0 ? 0 : 1;
}
