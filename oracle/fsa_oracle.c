/*
 * ORACLE - test infrastructure, not product code.
 *
 * A plain-C, sequential restatement of the reference FuseSampleAgg operator
 * (fuseop/fused_sample_agg.cu), used only as the checker: by tests/, by
 * __graft_entry__.smoke() and by bench.py's CPU-baseline leg.  The product
 * path (fusesampleagg_b200) never loads this library.
 *
 * It follows the reference's serial semantics line by line: one reservoir
 * per row in draw order, one thread per feature, sums in the reference's
 * j-then-i order, IEEE single-precision division.  Forward outputs and
 * sampled ids are therefore bit-identical to the reference on the same
 * inputs; the backward accumulates in a fixed (root, slot, leaf) order, so
 * it differs from the reference's atomics only by fp32 rounding order.
 *
 * Parity pin: tests/golden/ holds ids, outputs and gradients produced by the
 * reference's own CUDA op on a B200 (tests/golden/make_golden.py); the CPU
 * test suite checks this file against them bit for bit.
 *
 * Roots are independent, so sampling and forward loops take an OpenMP
 * thread count (results do not depend on it).
 */
#include <stdint.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

#define ORACLE_API __attribute__((visibility("default")))

/* fused_sample_agg.cu:14-19 */
static uint64_t splitmix64(uint64_t v) {
  v += 0x9E3779B97F4A7C15ULL;
  v = (v ^ (v >> 30)) * 0xBF58476D1CE4E5B9ULL;
  v = (v ^ (v >> 27)) * 0x94D049BB133111EBULL;
  return v ^ (v >> 31);
}

/* fused_sample_agg.cu:21-26 (xorshift64*) */
static uint64_t next_random(uint64_t* state) {
  uint64_t s = *state;
  s ^= s >> 12;
  s ^= s << 25;
  s ^= s >> 27;
  *state = s;
  return s * 2685821657736338717ULL;
}

/* fused_sample_agg.cu:28-31: high 64 bits of the 64x64 product */
static uint32_t bounded_random(uint64_t* state, uint32_t bound) {
  unsigned __int128 p = (unsigned __int128)next_random(state) * (unsigned __int128)bound;
  return (uint32_t)(p >> 64);
}

/* fused_sample_agg.cu:33-38 */
static uint64_t make_seed(uint64_t base, uint64_t root, uint64_t hop, uint64_t pos) {
  return splitmix64(base ^ splitmix64(root) ^ splitmix64(hop) ^ splitmix64(pos));
}

/* fused_sample_agg.cu:40-56: Vitter's Algorithm R with -1 padding */
static void reservoir_sample(const int32_t* nbr, int degree, int fanout, uint64_t seed,
                             int32_t* out) {
  const int take = degree < fanout ? degree : fanout;
  for (int i = 0; i < take; ++i) out[i] = nbr[i];
  uint64_t state = seed == 0 ? 0x9E3779B97F4A7C15ULL : seed;
  for (int i = take; i < degree; ++i) {
    const uint32_t sel = bounded_random(&state, (uint32_t)(i + 1));
    if (sel < (uint32_t)take) out[sel] = nbr[i];
  }
  for (int i = take < 0 ? 0 : take; i < fanout; ++i) out[i] = -1;
}

static void set_threads(int nthreads) {
#ifdef _OPENMP
  omp_set_num_threads(nthreads > 0 ? nthreads : 1);
#else
  (void)nthreads;
#endif
}

/* 1-hop sampling, fused_sample_agg.cu:75-92.  batch_offset is added to the
 * batch index of the seed (a slice of a larger batch). */
ORACLE_API void fsa_oracle_sample_1hop(const int32_t* rowptr, const int32_t* col,
                                       const int32_t* frontier, int64_t batch_size,
                                       int64_t batch_offset, int fanout, uint64_t seed,
                                       int32_t* samples, int32_t* takes, int nthreads) {
  set_threads(nthreads);
#pragma omp parallel for schedule(dynamic, 16)
  for (int64_t b = 0; b < batch_size; ++b) {
    const int32_t root = frontier[b];
    const int32_t begin = rowptr[root];
    const int32_t degree = rowptr[root + 1] - begin;
    reservoir_sample(col + begin, degree, fanout,
                     make_seed(seed, (uint64_t)root, 0, (uint64_t)(b + batch_offset)),
                     samples + b * fanout);
    takes[b] = degree < fanout ? degree : fanout;
  }
}

/* 1-hop mean, fused_sample_agg.cu:96-103 (per feature, i in order). */
ORACLE_API void fsa_oracle_forward_1hop(const float* x, int64_t feature_dim,
                                        const int32_t* samples, const int32_t* takes,
                                        int64_t batch_size, int fanout, float* out,
                                        int nthreads) {
  set_threads(nthreads);
#pragma omp parallel for schedule(static)
  for (int64_t b = 0; b < batch_size; ++b) {
    const int take = takes[b];
    for (int64_t f = 0; f < feature_dim; ++f) {
      float sum = 0.0F;
      for (int i = 0; i < take; ++i) {
        sum += x[(int64_t)samples[b * fanout + i] * feature_dim + f];
      }
      out[b * feature_dim + f] = take > 0 ? sum / (float)take : 0.0F;
    }
  }
}

/* 2-hop sampling, fused_sample_agg.cu:149-185. */
ORACLE_API void fsa_oracle_sample_2hop(const int32_t* rowptr, const int32_t* col,
                                       const int32_t* frontier, int64_t batch_size,
                                       int64_t batch_offset, int fanout1, int fanout2,
                                       uint64_t seed, int32_t* samples1, int32_t* samples2,
                                       int nthreads) {
  set_threads(nthreads);
#pragma omp parallel for schedule(dynamic, 1)
  for (int64_t b = 0; b < batch_size; ++b) {
    const int32_t root = frontier[b];
    int32_t* s1 = samples1 + b * fanout1;
    int32_t* s2 = samples2 + b * (int64_t)fanout1 * fanout2;
    const int32_t begin = rowptr[root];
    const int32_t degree = rowptr[root + 1] - begin;
    reservoir_sample(col + begin, degree, fanout1,
                     make_seed(seed, (uint64_t)root, 0, (uint64_t)(b + batch_offset)), s1);
    for (int i = 0; i < fanout1; ++i) {
      const int32_t middle = s1[i];
      int32_t* hop2 = s2 + (int64_t)i * fanout2;
      if (middle < 0) {
        for (int j = 0; j < fanout2; ++j) hop2[j] = -1;
      } else {
        const int32_t mb = rowptr[middle];
        const int32_t md = rowptr[middle + 1] - mb;
        reservoir_sample(col + mb, md, fanout2,
                         make_seed(seed, (uint64_t)root, 1, (uint64_t)i), hop2);
      }
    }
  }
}

/* 2-hop nested mean, fused_sample_agg.cu:189-213. */
ORACLE_API void fsa_oracle_forward_2hop(const float* x, int64_t feature_dim,
                                        const int32_t* samples2, int64_t batch_size,
                                        int fanout1, int fanout2, float* out, int nthreads) {
  set_threads(nthreads);
#pragma omp parallel for schedule(static)
  for (int64_t b = 0; b < batch_size; ++b) {
    const int32_t* s2 = samples2 + b * (int64_t)fanout1 * fanout2;
    for (int64_t f = 0; f < feature_dim; ++f) {
      float outer_sum = 0.0F;
      int nonempty = 0;
      for (int i = 0; i < fanout1; ++i) {
        float inner_sum = 0.0F;
        int valid = 0;
        for (int j = 0; j < fanout2; ++j) {
          const int32_t leaf = s2[i * fanout2 + j];
          if (leaf >= 0) {
            inner_sum += x[(int64_t)leaf * feature_dim + f];
            ++valid;
          }
        }
        if (valid > 0) {
          outer_sum += inner_sum / (float)valid;
          ++nonempty;
        }
      }
      out[b * feature_dim + f] = nonempty > 0 ? outer_sum / (float)nonempty : 0.0F;
    }
  }
}

/* 1-hop backward, fused_sample_agg.cu:119-131, sequential (grad_x pre-zeroed). */
ORACLE_API void fsa_oracle_backward_1hop(const int32_t* samples, const int32_t* takes,
                                         const float* grad_out, int64_t batch_size,
                                         int64_t feature_dim, int fanout, float* grad_x) {
  for (int64_t b = 0; b < batch_size; ++b) {
    const int take = takes[b];
    if (take == 0) continue;
    for (int64_t f = 0; f < feature_dim; ++f) {
      const float contribution = grad_out[b * feature_dim + f] / (float)take;
      for (int i = 0; i < take; ++i) {
        const int32_t nbr = samples[b * fanout + i];
        grad_x[(int64_t)nbr * feature_dim + f] += contribution;
      }
    }
  }
}

/* 2-hop backward, fused_sample_agg.cu:227-270, sequential. */
ORACLE_API void fsa_oracle_backward_2hop(const float* grad_out, const int32_t* samples1,
                                         const int32_t* samples2, int64_t batch_size,
                                         int64_t feature_dim, int fanout1, int fanout2,
                                         float* grad_x) {
  for (int64_t b = 0; b < batch_size; ++b) {
    const int64_t first = b * fanout1;
    const int64_t second = first * fanout2;
    int nonempty = 0;
    for (int i = 0; i < fanout1; ++i) {
      if (samples1[first + i] < 0) continue;
      for (int j = 0; j < fanout2; ++j) {
        if (samples2[second + (int64_t)i * fanout2 + j] >= 0) {
          ++nonempty;
          break;
        }
      }
    }
    if (nonempty == 0) continue;
    for (int64_t f = 0; f < feature_dim; ++f) {
      const float outer = grad_out[b * feature_dim + f] / (float)nonempty;
      for (int i = 0; i < fanout1; ++i) {
        int valid = 0;
        for (int j = 0; j < fanout2; ++j) {
          valid += samples2[second + (int64_t)i * fanout2 + j] >= 0 ? 1 : 0;
        }
        if (valid == 0) continue;
        const float inner = outer / (float)valid;
        for (int j = 0; j < fanout2; ++j) {
          const int32_t leaf = samples2[second + (int64_t)i * fanout2 + j];
          if (leaf >= 0) grad_x[(int64_t)leaf * feature_dim + f] += inner;
        }
      }
    }
  }
}

/* Serial xorshift64 state after n steps (checks GPU jump-ahead tables). */
ORACLE_API uint64_t fsa_oracle_xorshift_advance(uint64_t state, uint64_t n) {
  for (uint64_t k = 0; k < n; ++k) (void)next_random(&state);
  return state;
}

/* Reference seed derivation incl. zero substitution (fused_sample_agg.cu:46). */
ORACLE_API uint64_t fsa_oracle_row_state(uint64_t base, uint64_t root, uint64_t hop,
                                         uint64_t pos) {
  const uint64_t s = make_seed(base, root, hop, pos);
  return s == 0 ? 0x9E3779B97F4A7C15ULL : s;
}

ORACLE_API uint32_t fsa_oracle_bounded(uint64_t state, uint32_t bound) {
  return bounded_random(&state, bound);
}
