// Host-side check of the GEMM work-unit map (lpk::get_unit): every tile / K range is
// produced by exactly one unit for the forward's chunk-major order (short last chunk
// included), the N-fast and M-fast orders with split-K, and the interleaved tile / reduce-
// item order of the cross-rank dH sum, where each reduce item must come after every tile of
// its row block. Runs on the CPU; exit status 0 = all shapes pass.
#include <cstdio>
#include <vector>

#include "../../gemma4_posttrain_jax_b200/csrc/lp_gemm.cuh"

using namespace lpk;

static int failures = 0;
#define CHECK(cond, ...)                  \
  do {                                    \
    if (!(cond)) {                        \
      if (failures < 20) {                \
        std::printf("FAIL: " __VA_ARGS__); \
        std::printf("\n");                \
      }                                   \
      ++failures;                         \
    }                                     \
  } while (0)

static GemmSched base(int tiles_m, int tiles_n, int n_group, int k_blocks, int k_splits) {
  GemmSched s{};
  s.tiles_m = tiles_m;
  s.tiles_n = tiles_n;
  s.n_group = n_group;
  s.n_groups = (tiles_n + n_group - 1) / n_group;
  s.k_blocks = k_blocks;
  s.kb_per_split = (k_blocks + k_splits - 1) / k_splits;
  s.k_splits = (k_blocks + s.kb_per_split - 1) / s.kb_per_split;
  s.num_units = tiles_m * s.n_groups * s.k_splits;
  return s;
}

// Every (M tile, N tile, K block) is computed exactly once.
static void check_cover(const GemmSched& s, const char* what) {
  std::vector<int> seen((size_t)s.tiles_m * s.tiles_n * s.k_blocks, 0);
  for (int u = 0; u < s.num_units; ++u) {
    const Unit x = get_unit(s, u);
    CHECK(x.red_block < 0, "%s: unexpected reduce item at unit %d", what, u);
    CHECK(x.m_tile >= 0 && x.m_tile < s.tiles_m, "%s: m_tile %d out of range", what, x.m_tile);
    CHECK(x.n_count > 0 && x.n_begin >= 0 && x.n_begin + x.n_count <= s.tiles_n, "%s: bad N run", what);
    CHECK(x.kb_count > 0 && x.kb_begin >= 0 && x.kb_begin + x.kb_count <= s.k_blocks, "%s: bad K range", what);
    if (x.m_tile < 0 || x.m_tile >= s.tiles_m || x.n_begin < 0 || x.n_begin + x.n_count > s.tiles_n ||
        x.kb_begin < 0 || x.kb_begin + x.kb_count > s.k_blocks)
      continue;
    for (int n = x.n_begin; n < x.n_begin + x.n_count; ++n)
      for (int k = x.kb_begin; k < x.kb_begin + x.kb_count; ++k)
        ++seen[((size_t)x.m_tile * s.tiles_n + n) * s.k_blocks + k];
  }
  for (size_t i = 0; i < seen.size(); ++i) CHECK(seen[i] == 1, "%s: (tile, K block) %zu computed %d times", what, i, seen[i]);
}

// The cross-rank dH sum: tiles (one N tile, full K) and one reduce item per row block.
static void check_reduce_order(int tiles_m, int tiles_n, int lag) {
  GemmSched s = base(tiles_m, tiles_n, 1, 7, 1);
  s.n_fast = 1;
  s.red_lag = lag;
  s.num_units = tiles_m * tiles_n + tiles_m;
  std::vector<int> tile_seen((size_t)tiles_m * tiles_n, 0), red_seen(tiles_m, 0);
  std::vector<int> last_tile_pos(tiles_m, -1), red_pos(tiles_m, -1);
  for (int u = 0; u < s.num_units; ++u) {
    const Unit x = get_unit(s, u);
    if (x.red_block >= 0) {
      CHECK(x.red_block < tiles_m && x.n_count == 0, "reduce item %d bad (tiles_m %d)", x.red_block, tiles_m);
      if (x.red_block < tiles_m) {
        ++red_seen[x.red_block];
        red_pos[x.red_block] = u;
      }
    } else {
      CHECK(x.m_tile < tiles_m && x.n_count == 1 && x.n_begin < tiles_n && x.kb_count == 7, "tile unit %d bad", u);
      if (x.m_tile < tiles_m && x.n_begin < tiles_n) {
        ++tile_seen[(size_t)x.m_tile * tiles_n + x.n_begin];
        last_tile_pos[x.m_tile] = u;
      }
    }
  }
  for (size_t i = 0; i < tile_seen.size(); ++i)
    CHECK(tile_seen[i] == 1, "reduce order %dx%d lag %d: tile %zu seen %d times", tiles_m, tiles_n, lag, i, tile_seen[i]);
  for (int b = 0; b < tiles_m; ++b) {
    CHECK(red_seen[b] == 1, "reduce order %dx%d lag %d: block %d reduced %d times", tiles_m, tiles_n, lag, b, red_seen[b]);
    CHECK(red_pos[b] > last_tile_pos[b], "reduce order %dx%d lag %d: block %d reduced before its last tile", tiles_m,
          tiles_n, lag, b);
  }
}

int main() {
  const int tms[] = {1, 2, 5, 95, 96, 97, 200, 847};
  const int tns[] = {1, 3, 12, 64, 1024};
  // forward: chunk-major (m_chunk > 0, N-group order within a chunk), groups of N tiles
  for (int tm : tms)
    for (int tn : tns)
      for (int g : {1, 4, 16})
        for (int mc : {1, 7, 96}) {
          if (g > tn) continue;
          GemmSched s = base(tm, tn, g, 3, 1);
          s.m_chunk = mc;
          check_cover(s, "chunk-major");
        }
  // N-fast (dH, dW) and M-fast (dZ) orders, with split-K
  for (int tm : tms)
    for (int tn : {1, 8, 15})
      for (int ks : {1, 2, 4, 7}) {
        GemmSched s = base(tm, tn, 1, 29, ks);
        s.n_fast = 1;
        check_cover(s, "n-fast");
        s.n_fast = 0;
        s.m_chunk = 0;
        check_cover(s, "m-fast");
      }
  // the cross-rank dH sum's tile / reduce-item interleaving (lag clipped to tiles_m)
  for (int tm : {1, 2, 3, 5, 32, 40, 257})
    for (int tn : {1, 8, 15})
      for (int lag : {1, 2, 5, 30})
        if (lag <= tm) check_reduce_order(tm, tn, lag);
  if (failures == 0) std::printf("unit map: ok\n");
  return failures == 0 ? 0 : 1;
}
