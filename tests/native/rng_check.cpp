// Host check of fusesampleagg_b200/csrc/fsa_rng.cuh (compiled with g++ by
// tests/test_rng_host.py): reads "state steps" / "draw value bound" queries
// on stdin and prints the header's jump-ahead / bounded-draw results.
#include <cstdio>
#include <cstring>

#include "fsa_rng.cuh"

static const fsa::JumpTables kTables = fsa::make_jump_tables();
static const fsa::LaneTables kLanes1 = fsa::make_lane_tables(fsa::kChunkLog2);
static const fsa::LaneTables kLanes2 = fsa::make_lane_tables(fsa::kChunkLog2 + 5);
static const fsa::LaneTablesT kLanes1T = fsa::transpose_lane_tables(kLanes1);

// Start state of chunk j as the 2-hop draw kernel forms it: the transposed
// one-chunk table (entry [p][nib][j % 32]), then the 32-chunk table and the
// jump matrices.
static uint64_t chunk_start_transposed(uint64_t s0, uint64_t j) {
  uint64_t s = 0;
  for (int p = 0; p < 16; ++p) s ^= kLanes1T.v[p][(s0 >> (4 * p)) & 15][j % fsa::kLaneTables];
  s = fsa::apply_nibbles(kLanes2.v[(j / fsa::kLaneTables) % fsa::kLaneTables], s);
  uint64_t hi = j / (fsa::kLaneTables * fsa::kLaneTables);
  for (int b = 0; hi != 0; ++b, hi >>= 1) {
    if (hi & 1) s = fsa::apply_nibbles(kTables.v[fsa::kChunkLog2 + 10 + b], s);
  }
  return s;
}

int main() {
  char op[16];
  unsigned long long a = 0, b = 0;
  while (std::scanf("%15s %llu %llu", op, &a, &b) == 3) {
    if (std::strcmp(op, "jump") == 0) {
      std::printf("%llu\n", static_cast<unsigned long long>(fsa::jump_host(kTables, a, b)));
    } else if (std::strcmp(op, "chunk") == 0) {
      // start state of chunk b of a row with initial state a
      std::printf("%llu\n", static_cast<unsigned long long>(
                                 fsa::chunk_start_host(kTables, kLanes1, kLanes2, a, b)));
    } else if (std::strcmp(op, "chunkt") == 0) {
      std::printf("%llu\n", static_cast<unsigned long long>(chunk_start_transposed(a, b)));
    } else if (std::strcmp(op, "draw") == 0) {
      std::printf("%u\n", fsa::bounded_draw(a, static_cast<uint32_t>(b)));
    } else if (std::strcmp(op, "seed") == 0) {
      // a = base, b = root; hop 1, pos 3 (fixed) and hop 0, pos b
      std::printf("%llu %llu\n",
                  static_cast<unsigned long long>(fsa::row_state(a, b, 1, 3)),
                  static_cast<unsigned long long>(fsa::row_state(a, b, 0, b)));
    }
  }
  return 0;
}
