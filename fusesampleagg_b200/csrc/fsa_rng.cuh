// Counter-seeded random streams of the FuseSampleAgg sampler, plus GF(2)
// jump-ahead so that one reservoir stream can be split across many threads.
//
// Stream definition (must match the reference bit for bit):
//   * splitmix64 finaliser ............ fuseop/fused_sample_agg.cu:14-19
//   * xorshift64* generator ........... fuseop/fused_sample_agg.cu:21-26
//   * multiply-high bounded draw ...... fuseop/fused_sample_agg.cu:28-31
//   * per-(seed, root, hop, pos) seed .. fuseop/fused_sample_agg.cu:33-38
//   * zero seed -> golden-ratio state .. fuseop/fused_sample_agg.cu:46
//
// The xorshift64 state update (three shift-xor steps) is linear over GF(2)^64,
// so k steps are one 64x64 bit-matrix T^k.  `JumpTables` holds T^(2^j) for
// j < kJumpBits, each stored as 16 nibble tables: T^(2^j) * s is the XOR of
// one 64-bit entry per 4-bit nibble of s.  The tables are built at compile
// time (constexpr repeated squaring) and placed in device global memory, so
// the library has no run-time initialisation step.
//
// This header compiles as plain C++17 as well (host unit tests).
#pragma once

#include <stdint.h>

#if defined(__CUDACC__)
#define FSA_HD __host__ __device__ __forceinline__
#else
#define FSA_HD inline
#endif

namespace fsa {

constexpr uint64_t kGoldenGamma = 0x9E3779B97F4A7C15ULL;
constexpr uint64_t kMixMul1 = 0xBF58476D1CE4E5B9ULL;
constexpr uint64_t kMixMul2 = 0x94D049BB133111EBULL;
constexpr uint64_t kStarMul = 2685821657736338717ULL;

// Number of jump matrices: jumps of up to 2^31 - 1 steps (any int32 degree).
constexpr int kJumpBits = 31;

FSA_HD constexpr uint64_t splitmix64(uint64_t v) {
  v += kGoldenGamma;
  v = (v ^ (v >> 30)) * kMixMul1;
  v = (v ^ (v >> 27)) * kMixMul2;
  return v ^ (v >> 31);
}

// One xorshift64 state transition (the linear part of xorshift64*).
FSA_HD constexpr uint64_t xorshift_step(uint64_t s) {
  s ^= s >> 12;
  s ^= s << 25;
  s ^= s >> 27;
  return s;
}

// Initial reservoir state for row (root, hop, pos).  1-hop rows and the
// first hop of 2-hop use hop=0, pos=global batch index; second-hop rows use
// hop=1, pos=first-hop slot.  A zero seed is replaced by the golden gamma
// because xorshift would stay at zero forever.
FSA_HD constexpr uint64_t row_state(uint64_t base, uint64_t root, uint64_t hop,
                                    uint64_t pos) {
  const uint64_t s = splitmix64(base ^ splitmix64(root) ^ splitmix64(hop) ^
                                splitmix64(pos));
  return s == 0 ? kGoldenGamma : s;
}

// floor(r * bound / 2^64) for bound < 2^32, from two 32x32->64 products.
// Equal to the high word of the full 64x64 product, i.e. the reference's
// multiply-shift draw in [0, bound).
FSA_HD uint32_t bounded_draw(uint64_t r, uint32_t bound) {
  const uint64_t lo = static_cast<uint64_t>(static_cast<uint32_t>(r)) * bound;
  const uint64_t mid =
      static_cast<uint64_t>(static_cast<uint32_t>(r >> 32)) * bound + (lo >> 32);
  return static_cast<uint32_t>(mid >> 32);
}

struct JumpTables {
  uint64_t v[kJumpBits][16][16];
};

constexpr JumpTables make_jump_tables() {
  JumpTables t{};
  uint64_t cols[64] = {};  // column k = T^(2^j) applied to bit k
  for (int k = 0; k < 64; ++k) cols[k] = xorshift_step(uint64_t{1} << k);
  for (int j = 0; j < kJumpBits; ++j) {
    for (int p = 0; p < 16; ++p) {
      for (int nib = 0; nib < 16; ++nib) {
        uint64_t acc = 0;
        for (int b = 0; b < 4; ++b) {
          if ((nib >> b) & 1) acc ^= cols[4 * p + b];
        }
        t.v[j][p][nib] = acc;
      }
    }
    // Square: T^(2^(j+1)) e_k = T^(2^j) (T^(2^j) e_k).
    uint64_t sq[64] = {};
    for (int k = 0; k < 64; ++k) {
      const uint64_t x = cols[k];
      uint64_t acc = 0;
      for (int b = 0; b < 64; ++b) {
        if ((x >> b) & 1) acc ^= cols[b];
      }
      sq[k] = acc;
    }
    for (int k = 0; k < 64; ++k) cols[k] = sq[k];
  }
  return t;
}

// Draws are handed out in chunks of 2^kChunkLog2 positions aligned to the
// start of each row; a warp takes 32 consecutive chunks.  LaneTables holds
// T^(l * 2^step_log2) for l < 32 in the same nibble form.  With one set for
// step 2^kChunkLog2 (one chunk) and one for 32 chunks, the start state of
// chunk j of a row is  K1[j % 32] * K2[(j / 32) % 32] * T^(...) s0: one or
// two table products per lane, plus one jump matrix per set bit of j / 1024
// (rows of more than 2^(kChunkLog2 + 10) draws only).  64-draw chunks were
// the fastest of 32/64/128 on the 2-hop power-law workload.
constexpr int kChunkLog2 = 6;
constexpr int kLaneTables = 32;

struct LaneTables {
  uint64_t v[kLaneTables][16][16];
};

constexpr uint64_t apply_nibbles(const uint64_t (&tab)[16][16], uint64_t s) {
  uint64_t acc = 0;
  for (int p = 0; p < 16; ++p) acc ^= tab[p][(s >> (4 * p)) & 15];
  return acc;
}

constexpr LaneTables make_lane_tables(int step_log2) {
  const JumpTables jt = make_jump_tables();
  LaneTables t{};
  // Identity for l = 0.
  for (int p = 0; p < 16; ++p) {
    for (int nib = 0; nib < 16; ++nib) t.v[0][p][nib] = static_cast<uint64_t>(nib) << (4 * p);
  }
  uint64_t step_cols[64] = {};  // columns of T^(2^step_log2)
  for (int k = 0; k < 64; ++k) step_cols[k] = apply_nibbles(jt.v[step_log2], uint64_t{1} << k);
  for (int l = 1; l < kLaneTables; ++l) {
    uint64_t cols[64] = {};  // columns of T^(l * step) = T^((l-1) * step) * T^step
    for (int k = 0; k < 64; ++k) cols[k] = apply_nibbles(t.v[l - 1], step_cols[k]);
    for (int p = 0; p < 16; ++p) {
      for (int nib = 0; nib < 16; ++nib) {
        uint64_t acc = 0;
        for (int b = 0; b < 4; ++b) {
          if ((nib >> b) & 1) acc ^= cols[4 * p + b];
        }
        t.v[l][p][nib] = acc;
      }
    }
  }
  return t;
}

// The same tables with the lane index innermost: v[p][nib][l].  Threads
// that apply different lane tables to different states read entry
// [p][nib][l] -- in shared memory that is a different bank pair for every l
// of a half-warp, whatever the nibbles.
struct LaneTablesT {
  uint64_t v[16][16][kLaneTables];
};

constexpr LaneTablesT transpose_lane_tables(const LaneTables& t) {
  LaneTablesT o{};
  for (int l = 0; l < kLaneTables; ++l) {
    for (int p = 0; p < 16; ++p) {
      for (int nib = 0; nib < 16; ++nib) o.v[p][nib][l] = t.v[l][p][nib];
    }
  }
  return o;
}

// Host-side evaluation of T^n s (tests and host tools).
inline uint64_t jump_host(const JumpTables& t, uint64_t s, uint64_t n) {
  for (int j = 0; j < kJumpBits && n != 0; ++j, n >>= 1) {
    if (n & 1) {
      uint64_t acc = 0;
      for (int p = 0; p < 16; ++p) acc ^= t.v[j][p][(s >> (4 * p)) & 15];
      s = acc;
    }
  }
  return s;
}

// Host-side start state of chunk j of a row (the device uses the same
// decomposition).
inline uint64_t chunk_start_host(const JumpTables& jt, const LaneTables& k1,
                                 const LaneTables& k2, uint64_t s0, uint64_t j) {
  uint64_t s = apply_nibbles(k1.v[j % kLaneTables], s0);
  s = apply_nibbles(k2.v[(j / kLaneTables) % kLaneTables], s);
  uint64_t hi = j / (kLaneTables * kLaneTables);
  for (int b = 0; hi != 0; ++b, hi >>= 1) {
    if (hi & 1) s = apply_nibbles(jt.v[kChunkLog2 + 10 + b], s);
  }
  return s;
}

}  // namespace fsa
