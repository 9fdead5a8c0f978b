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

}  // namespace fsa
