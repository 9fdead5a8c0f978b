// Fused reservoir-sample + mean-aggregate kernels for B200 (sm_100a) and the
// C ABI declared in include/fsa_sm100.h.
//
// Design (see the reference kernels at fuseop/fused_sample_agg.cu:58-271):
//
//   * One CTA per root.  The reference runs Algorithm R on a single thread
//     per row (fused_sample_agg.cu:40-56), which for power-law graphs means
//     tens of thousands of dependent xorshift steps per root while the rest
//     of the CTA idles.  Here the draws of a row are split into contiguous
//     per-thread chunks; a thread reaches the first state of its chunk with
//     a GF(2) jump (fsa_rng.cuh) and records, for every reservoir slot, the
//     largest draw index that replaced it (shared-memory atomicMax).  The
//     slot's final neighbour is col[winner] or, if never replaced,
//     col[slot] -- exactly what the serial loop leaves behind, so sampled
//     ids are bit-identical.
//   * 2-hop: the draws of all fanout1 second-hop rows of a root form one
//     concatenated sequence that the whole CTA splits evenly, so a hub
//     middle does not serialise the root.
//   * Gather: every (first-hop slot, feature vector) pair is one work item
//     that sums its valid leaf rows with 128-bit (or 64/32-bit, by feature
//     width) non-allocating loads in the reference's j order and divides by
//     the valid count; the per-slot means are then summed in i order.  The
//     arithmetic order equals the reference's, so forward outputs are
//     bit-identical too.
//   * Backward: red.global.add.v4.f32 (v2/scalar for narrow rows) of
//     (grad/nonempty)/valid into grad_x, one CTA per root.
//   * No kernel allocates, synchronises or spins.  Out-of-range ids are never
//     dereferenced: they are skipped and reported in a per-device status word.
#include <cuda_runtime.h>

#include <atomic>
#include <cstdint>

#include "fsa_rng.cuh"
#include "fsa_sm100.h"

namespace {

using fsa::JumpTables;

__device__ constexpr JumpTables g_jump = fsa::make_jump_tables();
__device__ unsigned int g_status;

constexpr int kThreads1Hop = 128;
constexpr int kThreads2Hop = 256;
constexpr int kThreadsBwd = 256;
constexpr int kThreadsFill = 256;
// Fewest draws a thread is given before more threads join a row: below this
// the jump to the chunk start costs more than the draws it parallelises.
constexpr long long kMinChunk = 64;
// Shared-memory budget for the per-slot partial means of one feature tile.
constexpr int kInnerBudgetBytes = 24 * 1024;
constexpr int kMaxSmemBytes = 227 * 1024;
constexpr int64_t kMaxGrid = int64_t{1} << 20;

std::atomic<uint64_t> g_launches{0};
thread_local int t_last_cuda_error = 0;

// ---------------------------------------------------------------------------
// Device helpers
// ---------------------------------------------------------------------------

__device__ __forceinline__ void flag_status(unsigned int bits) {
  atomicOr(&g_status, bits);
}

// T^n s: one nibble-table product per set bit of n.
__device__ __forceinline__ uint64_t jump_ahead(uint64_t s, uint32_t n) {
#pragma unroll 1
  while (n != 0) {
    const int j = __ffs(n) - 1;
    n &= n - 1;
    const uint64_t* tab = &g_jump.v[j][0][0];
    uint64_t acc = 0;
#pragma unroll
    for (int p = 0; p < 16; ++p) {
      acc ^= __ldg(tab + p * 16 + static_cast<int>((s >> (4 * p)) & 15));
    }
    s = acc;
  }
  return s;
}

// Draws [t_begin, t_end) of one row whose reservoir holds `take` slots.
// Draw t is row position take + t, uses the state after t + 1 steps and the
// bound take + t + 1; a hit records position take + t in win[slot].
__device__ __forceinline__ void run_draws(uint64_t s0, uint32_t t_begin,
                                          uint32_t t_end, int take, int* win) {
  uint64_t s = jump_ahead(s0, t_begin);
  const uint32_t utake = static_cast<uint32_t>(take);
#pragma unroll 2
  for (uint32_t t = t_begin; t < t_end; ++t) {
    s = fsa::xorshift_step(s);
    const uint32_t slot = fsa::bounded_draw(s * fsa::kStarMul, utake + t + 1u);
    if (slot < utake) atomicMax(&win[slot], static_cast<int>(utake + t));
  }
}

// Splits the `ndraws` draws of a single row over the CTA.
__device__ __forceinline__ void block_draws_one_row(uint64_t s0, int take,
                                                    long long ndraws, int* win) {
  const long long per = (ndraws + blockDim.x - 1) / blockDim.x;
  const long long chunk = per > kMinChunk ? per : kMinChunk;
  const long long g0 = static_cast<long long>(threadIdx.x) * chunk;
  if (g0 >= ndraws) return;
  const long long g1 = g0 + chunk < ndraws ? g0 + chunk : ndraws;
  run_draws(s0, static_cast<uint32_t>(g0), static_cast<uint32_t>(g1), take, win);
}

// Reads row r of the CSR with validation.  Returns false (and flags) when the
// row range is not inside [0, num_edges].
__device__ __forceinline__ bool read_row(const int32_t* __restrict__ rowptr,
                                         int64_t num_edges, int32_t r,
                                         int32_t& begin, int32_t& degree) {
  const int32_t b = rowptr[r];
  const int32_t e = rowptr[r + 1];
  if (b < 0 || e < b || static_cast<int64_t>(e) > num_edges) {
    begin = 0;
    degree = 0;
    return false;
  }
  begin = b;
  degree = e - b;
  return true;
}

template <int V>
struct VecF {
  float v[V];
};

template <int V>
__device__ __forceinline__ void vzero(VecF<V>& a) {
#pragma unroll
  for (int k = 0; k < V; ++k) a.v[k] = 0.0F;
}

template <int V>
__device__ __forceinline__ VecF<V> load_stream(const float* p);

template <>
__device__ __forceinline__ VecF<4> load_stream<4>(const float* p) {
  VecF<4> r;
  asm("ld.global.nc.L1::no_allocate.v4.f32 {%0,%1,%2,%3}, [%4];"
      : "=f"(r.v[0]), "=f"(r.v[1]), "=f"(r.v[2]), "=f"(r.v[3])
      : "l"(p));
  return r;
}

template <>
__device__ __forceinline__ VecF<2> load_stream<2>(const float* p) {
  VecF<2> r;
  asm("ld.global.nc.L1::no_allocate.v2.f32 {%0,%1}, [%2];"
      : "=f"(r.v[0]), "=f"(r.v[1])
      : "l"(p));
  return r;
}

template <>
__device__ __forceinline__ VecF<1> load_stream<1>(const float* p) {
  VecF<1> r;
  asm("ld.global.nc.L1::no_allocate.f32 %0, [%1];" : "=f"(r.v[0]) : "l"(p));
  return r;
}

template <int V>
__device__ __forceinline__ void red_add(float* p, const VecF<V>& a);

template <>
__device__ __forceinline__ void red_add<4>(float* p, const VecF<4>& a) {
  asm volatile("red.global.add.v4.f32 [%0], {%1,%2,%3,%4};" ::"l"(p),
               "f"(a.v[0]), "f"(a.v[1]), "f"(a.v[2]), "f"(a.v[3])
               : "memory");
}

template <>
__device__ __forceinline__ void red_add<2>(float* p, const VecF<2>& a) {
  asm volatile("red.global.add.v2.f32 [%0], {%1,%2};" ::"l"(p), "f"(a.v[0]),
               "f"(a.v[1])
               : "memory");
}

template <>
__device__ __forceinline__ void red_add<1>(float* p, const VecF<1>& a) {
  asm volatile("red.global.add.f32 [%0], %1;" ::"l"(p), "f"(a.v[0]) : "memory");
}

template <int V>
__device__ __forceinline__ void store_vec(float* p, const VecF<V>& a) {
#pragma unroll
  for (int k = 0; k < V; ++k) p[k] = a.v[k];
}

template <int V>
__device__ __forceinline__ VecF<V> load_vec(const float* p) {
  VecF<V> r;
#pragma unroll
  for (int k = 0; k < V; ++k) r.v[k] = p[k];
  return r;
}

// ---------------------------------------------------------------------------
// 1-hop forward: fuseop/fused_sample_agg.cu:58-104
// ---------------------------------------------------------------------------

struct Fwd1Args {
  const int32_t* rowptr;
  const int32_t* col;
  const float* x;
  int64_t num_nodes;
  int64_t num_edges;
  int64_t feature_dim;
  const int32_t* frontier;
  int64_t batch_size;
  int64_t batch_offset;
  int fanout;
  uint64_t seed;
  float* out;
  int32_t* samples;
  int32_t* takes;
};

template <int V>
__global__ void __launch_bounds__(kThreads1Hop)
    fsa_1hop_forward_kernel(const Fwd1Args a) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  int* slots = reinterpret_cast<int*>(smem_raw);  // winners, then sample ids
  const int k = a.fanout;
  const int tid = threadIdx.x;
  const int nthreads = blockDim.x;
  const int64_t dvec = a.feature_dim / V;

  for (int64_t b = blockIdx.x; b < a.batch_size; b += gridDim.x) {
    const int32_t root = a.frontier[b];
    int32_t begin = 0, degree = 0;
    if (root >= 0 && root < a.num_nodes) {
      if (!read_row(a.rowptr, a.num_edges, root, begin, degree) && tid == 0) {
        flag_status(FSA_STATUS_BAD_ROW);
      }
    } else if (tid == 0) {
      flag_status(FSA_STATUS_BAD_ROOT);
    }
    const int take = degree < k ? degree : k;
    for (int i = tid; i < k; i += nthreads) slots[i] = -1;
    __syncthreads();
    if (degree > take) {
      const uint64_t s0 = fsa::row_state(a.seed, static_cast<uint64_t>(root), 0,
                                         static_cast<uint64_t>(b + a.batch_offset));
      block_draws_one_row(s0, take, static_cast<long long>(degree - take), slots);
    }
    __syncthreads();
    for (int i = tid; i < k; i += nthreads) {
      int32_t id = -1;
      if (i < take) {
        const int w = slots[i];
        id = a.col[static_cast<int64_t>(begin) + (w >= 0 ? w : i)];
      }
      slots[i] = id;
      if (a.samples != nullptr) a.samples[b * k + i] = id;
    }
    if (tid == 0 && a.takes != nullptr) a.takes[b] = take;
    __syncthreads();
    for (int64_t v = tid; v < dvec; v += nthreads) {
      VecF<V> acc;
      vzero(acc);
      for (int i = 0; i < take; ++i) {
        const int32_t leaf = slots[i];
        if (leaf >= 0 && leaf < a.num_nodes) {
          const VecF<V> r = load_stream<V>(a.x + static_cast<int64_t>(leaf) * a.feature_dim + v * V);
#pragma unroll
          for (int c = 0; c < V; ++c) acc.v[c] += r.v[c];
        } else if (v == 0) {
          flag_status(FSA_STATUS_BAD_NEIGHBOR);
        }
      }
      if (take > 0) {
        const float denom = static_cast<float>(take);
#pragma unroll
        for (int c = 0; c < V; ++c) acc.v[c] = acc.v[c] / denom;
      }
      store_vec(a.out + b * a.feature_dim + v * V, acc);
    }
    __syncthreads();
  }
}

// ---------------------------------------------------------------------------
// 2-hop forward: fuseop/fused_sample_agg.cu:134-214
// ---------------------------------------------------------------------------

struct Fwd2Args {
  const int32_t* rowptr;
  const int32_t* col;
  const float* x;
  int64_t num_nodes;
  int64_t num_edges;
  int64_t feature_dim;
  const int32_t* frontier;
  int64_t batch_size;
  int64_t batch_offset;
  int fanout1;
  int fanout2;
  uint64_t seed;
  float* out;
  int32_t* samples1;
  int32_t* samples2;
  int dchunk;  // feature tile width (multiple of the vector width)
};

// Shared-memory layout of the 2-hop forward kernel, in bytes.
struct Layout2 {
  int pre, inner, s1, mbeg, mtake, mvalid, s2, misc, total;
};

__host__ __device__ inline int align16(int v) { return (v + 15) & ~15; }

__host__ __device__ inline Layout2 layout_2hop(int k1, int k2, int dchunk) {
  Layout2 l;
  l.pre = 0;                                    // int64 [k1 + 1]
  l.inner = align16(l.pre + 8 * (k1 + 1));      // float [k1][dchunk]
  l.s1 = align16(l.inner + 4 * k1 * dchunk);    // int32 [k1]
  l.mbeg = l.s1 + 4 * k1;                       // int32 [k1]
  l.mtake = l.mbeg + 4 * k1;                    // int32 [k1]
  l.mvalid = l.mtake + 4 * k1;                  // int32 [k1]
  l.s2 = l.mvalid + 4 * k1;                     // int32 [k1 * k2]
  l.misc = align16(l.s2 + 4 * k1 * k2);         // int32 [4]
  l.total = l.misc + 16;
  return l;
}

template <int V>
__global__ void __launch_bounds__(kThreads2Hop)
    fsa_2hop_forward_kernel(const Fwd2Args a) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const int k1 = a.fanout1;
  const int k2 = a.fanout2;
  const Layout2 L = layout_2hop(k1, k2, a.dchunk);
  long long* pre = reinterpret_cast<long long*>(smem_raw + L.pre);
  float* inner = reinterpret_cast<float*>(smem_raw + L.inner);
  int* s1 = reinterpret_cast<int*>(smem_raw + L.s1);
  int* mbeg = reinterpret_cast<int*>(smem_raw + L.mbeg);
  int* mtake = reinterpret_cast<int*>(smem_raw + L.mtake);
  int* mvalid = reinterpret_cast<int*>(smem_raw + L.mvalid);
  int* s2 = reinterpret_cast<int*>(smem_raw + L.s2);
  int* misc = reinterpret_cast<int*>(smem_raw + L.misc);

  const int tid = threadIdx.x;
  const int nthreads = blockDim.x;
  const int k12 = k1 * k2;
  const int64_t D = a.feature_dim;
  const int64_t N = a.num_nodes;

  for (int64_t b = blockIdx.x; b < a.batch_size; b += gridDim.x) {
    // ---- first hop: reservoir over row(root) -------------------------------
    const int32_t root = a.frontier[b];
    int32_t rbegin = 0, rdegree = 0;
    if (root >= 0 && root < N) {
      if (!read_row(a.rowptr, a.num_edges, root, rbegin, rdegree) && tid == 0) {
        flag_status(FSA_STATUS_BAD_ROW);
      }
    } else if (tid == 0) {
      flag_status(FSA_STATUS_BAD_ROOT);
    }
    const int take1 = rdegree < k1 ? rdegree : k1;
    for (int i = tid; i < k1; i += nthreads) s1[i] = -1;
    for (int e = tid; e < k12; e += nthreads) s2[e] = -1;
    if (tid == 0) misc[0] = 0;
    __syncthreads();
    if (rdegree > take1) {
      const uint64_t s0 = fsa::row_state(a.seed, static_cast<uint64_t>(root), 0,
                                         static_cast<uint64_t>(b + a.batch_offset));
      block_draws_one_row(s0, take1, static_cast<long long>(rdegree - take1), s1);
    }
    __syncthreads();

    // ---- resolve first hop; read the middle rows ---------------------------
    for (int i = tid; i < k1; i += nthreads) {
      int32_t m = -1;
      if (i < take1) {
        const int w = s1[i];
        m = a.col[static_cast<int64_t>(rbegin) + (w >= 0 ? w : i)];
      }
      s1[i] = m;
      if (a.samples1 != nullptr) a.samples1[b * k1 + i] = m;
      int32_t mb = 0, md = 0;
      if (m >= 0) {
        if (m < N) {
          if (!read_row(a.rowptr, a.num_edges, m, mb, md)) flag_status(FSA_STATUS_BAD_ROW);
        } else {
          flag_status(FSA_STATUS_BAD_NEIGHBOR);
        }
      }
      const int mt = md < k2 ? md : k2;
      mbeg[i] = mb;
      mtake[i] = mt;
      pre[i + 1] = static_cast<long long>(md - mt);
    }
    __syncthreads();

    // ---- inclusive scan of per-row draw counts (warp 0) --------------------
    if (tid < 32) {
      const int seg = (k1 + 31) / 32;
      const int i0 = min(tid * seg, k1);
      const int i1 = min(i0 + seg, k1);
      long long local = 0;
      for (int i = i0; i < i1; ++i) local += pre[i + 1];
      long long incl = local;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const long long y = __shfl_up_sync(0xffffffffU, incl, o);
        if (tid >= o) incl += y;
      }
      long long run = incl - local;
      for (int i = i0; i < i1; ++i) {
        run += pre[i + 1];
        pre[i + 1] = run;
      }
      if (tid == 0) pre[0] = 0;
    }
    __syncthreads();

    // ---- second hop: the CTA splits the concatenated draws of all rows -----
    const long long total = pre[k1];
    if (total > 0) {
      const long long per = (total + nthreads - 1) / nthreads;
      const long long chunk = per > kMinChunk ? per : kMinChunk;
      long long g = static_cast<long long>(tid) * chunk;
      if (g < total) {
        const long long gend = g + chunk < total ? g + chunk : total;
        // Largest r with pre[r] <= g (rows with zero draws are skipped).
        int lo = 0, hi = k1 - 1;
        while (lo < hi) {
          const int mid = (lo + hi + 1) >> 1;
          if (pre[mid] <= g) lo = mid; else hi = mid - 1;
        }
        int r = lo;
        while (g < gend) {
          while (pre[r + 1] <= g) ++r;
          const long long row_end = pre[r + 1];
          const long long seg_end = row_end < gend ? row_end : gend;
          const uint64_t s0 = fsa::row_state(a.seed, static_cast<uint64_t>(root), 1,
                                             static_cast<uint64_t>(r));
          run_draws(s0, static_cast<uint32_t>(g - pre[r]),
                    static_cast<uint32_t>(seg_end - pre[r]), mtake[r], s2 + r * k2);
          g = seg_end;
        }
      }
    }
    __syncthreads();

    // ---- resolve second hop -------------------------------------------------
    for (int e = tid; e < k12; e += nthreads) {
      const int i = e / k2;
      const int j = e - i * k2;
      int32_t id = -1;
      if (j < mtake[i]) {
        const int w = s2[e];
        id = a.col[static_cast<int64_t>(mbeg[i]) + (w >= 0 ? w : j)];
      }
      s2[e] = id;
      if (a.samples2 != nullptr) a.samples2[b * k12 + e] = id;
    }
    __syncthreads();
    for (int i = tid; i < k1; i += nthreads) {
      int valid = 0;
      for (int j = 0; j < k2; ++j) {
        const int32_t leaf = s2[i * k2 + j];
        if (leaf >= 0) {
          if (leaf < N) ++valid; else flag_status(FSA_STATUS_BAD_NEIGHBOR);
        }
      }
      mvalid[i] = valid;
      if (valid > 0) atomicAdd(&misc[0], 1);
    }
    __syncthreads();

    // ---- nested mean, one feature tile at a time ----------------------------
    const int nonempty = misc[0];
    for (int64_t f0 = 0; f0 < D; f0 += a.dchunk) {
      const int fc = static_cast<int>(D - f0 < a.dchunk ? D - f0 : a.dchunk);
      const int nv = fc / V;
      const int items = k1 * nv;
      for (int it = tid; it < items; it += nthreads) {
        const int i = it / nv;
        const int v = it - i * nv;
        const int valid = mvalid[i];
        if (valid == 0) continue;
        const int32_t* leaves = s2 + i * k2;
        const float* base = a.x + f0 + v * V;
        VecF<V> acc;
        vzero(acc);
#pragma unroll 4
        for (int j = 0; j < k2; ++j) {
          const int32_t leaf = leaves[j];
          if (leaf >= 0 && leaf < N) {
            const VecF<V> r = load_stream<V>(base + static_cast<int64_t>(leaf) * D);
#pragma unroll
            for (int c = 0; c < V; ++c) acc.v[c] += r.v[c];
          }
        }
        const float denom = static_cast<float>(valid);
#pragma unroll
        for (int c = 0; c < V; ++c) acc.v[c] = acc.v[c] / denom;
        store_vec(inner + i * a.dchunk + v * V, acc);
      }
      __syncthreads();
      for (int v = tid; v < nv; v += nthreads) {
        VecF<V> outer;
        vzero(outer);
        for (int i = 0; i < k1; ++i) {
          if (mvalid[i] > 0) {
            const VecF<V> m = load_vec<V>(inner + i * a.dchunk + v * V);
#pragma unroll
            for (int c = 0; c < V; ++c) outer.v[c] += m.v[c];
          }
        }
        if (nonempty > 0) {
          const float denom = static_cast<float>(nonempty);
#pragma unroll
          for (int c = 0; c < V; ++c) outer.v[c] = outer.v[c] / denom;
        } else {
          vzero(outer);
        }
        store_vec(a.out + b * D + f0 + v * V, outer);
      }
      __syncthreads();
    }
    __syncthreads();
  }
}

// ---------------------------------------------------------------------------
// Backward (saved-index replay): fuseop/fused_sample_agg.cu:106-132, :216-271
// ---------------------------------------------------------------------------

struct Bwd1Args {
  const int32_t* samples;
  const int32_t* takes;
  const float* grad_out;
  int64_t batch_size;
  int64_t feature_dim;
  int fanout;
  float* grad_x;
  int64_t num_nodes;
};

// One warp per root; lanes stride feature vectors.
template <int V>
__global__ void __launch_bounds__(kThreadsBwd)
    fsa_1hop_backward_kernel(const Bwd1Args a) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  const int64_t dvec = a.feature_dim / V;
  for (int64_t b = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
       b < a.batch_size; b += warps) {
    const int take = a.takes[b];
    if (take <= 0) continue;
    const float denom = static_cast<float>(take);
    const int32_t* row = a.samples + b * a.fanout;
    const int lim = take < a.fanout ? take : a.fanout;
    for (int64_t v = lane; v < dvec; v += 32) {
      VecF<V> g = load_vec<V>(a.grad_out + b * a.feature_dim + v * V);
#pragma unroll
      for (int c = 0; c < V; ++c) g.v[c] = g.v[c] / denom;
      for (int i = 0; i < lim; ++i) {
        const int32_t nbr = row[i];
        if (nbr >= 0 && nbr < a.num_nodes) {
          red_add<V>(a.grad_x + static_cast<int64_t>(nbr) * a.feature_dim + v * V, g);
        } else if (v == lane) {
          flag_status(FSA_STATUS_BAD_NEIGHBOR);
        }
      }
    }
  }
}

struct Bwd2Args {
  const float* grad_out;
  const int32_t* samples1;
  const int32_t* samples2;
  int64_t batch_size;
  int64_t feature_dim;
  int fanout1;
  int fanout2;
  float* grad_x;
  int64_t num_nodes;
};

// One CTA per root; items are (first-hop slot, feature vector) pairs.
template <int V>
__global__ void __launch_bounds__(kThreadsBwd)
    fsa_2hop_backward_kernel(const Bwd2Args a) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const int k1 = a.fanout1;
  const int k2 = a.fanout2;
  const int k12 = k1 * k2;
  int* valid = reinterpret_cast<int*>(smem_raw);  // [k1]
  int* s2 = valid + k1;                            // [k1 * k2]
  int* misc = s2 + k12;                            // [1]
  const int tid = threadIdx.x;
  const int nthreads = blockDim.x;
  const int64_t dvec = a.feature_dim / V;

  for (int64_t b = blockIdx.x; b < a.batch_size; b += gridDim.x) {
    if (tid == 0) misc[0] = 0;
    for (int e = tid; e < k12; e += nthreads) s2[e] = a.samples2[b * k12 + e];
    __syncthreads();
    for (int i = tid; i < k1; i += nthreads) {
      int cnt = 0;
      for (int j = 0; j < k2; ++j) cnt += s2[i * k2 + j] >= 0 ? 1 : 0;
      valid[i] = cnt;
      // fused_sample_agg.cu:229-240: a slot is non-empty when its first-hop id
      // is valid and it has at least one valid second-hop id.
      if (cnt > 0 && a.samples1[b * k1 + i] >= 0) atomicAdd(&misc[0], 1);
    }
    __syncthreads();
    const int nonempty = misc[0];
    if (nonempty > 0) {
      const float ne = static_cast<float>(nonempty);
      const int64_t items = static_cast<int64_t>(k1) * dvec;
      for (int64_t it = tid; it < items; it += nthreads) {
        const int i = static_cast<int>(it / dvec);
        const int64_t v = it - static_cast<int64_t>(i) * dvec;
        const int cnt = valid[i];
        if (cnt == 0) continue;
        VecF<V> g = load_vec<V>(a.grad_out + b * a.feature_dim + v * V);
        const float vc = static_cast<float>(cnt);
#pragma unroll
        for (int c = 0; c < V; ++c) g.v[c] = (g.v[c] / ne) / vc;
        const int32_t* leaves = s2 + i * k2;
        for (int j = 0; j < k2; ++j) {
          const int32_t leaf = leaves[j];
          if (leaf < 0) continue;
          if (leaf < a.num_nodes) {
            red_add<V>(a.grad_x + static_cast<int64_t>(leaf) * a.feature_dim + v * V, g);
          } else if (v == 0) {
            flag_status(FSA_STATUS_BAD_NEIGHBOR);
          }
        }
      }
    }
    __syncthreads();
  }
}

// ---------------------------------------------------------------------------
// Dense zero fill of the gradient (replaces at::zeros, fuseop/binding.cpp:137)
// ---------------------------------------------------------------------------

__global__ void __launch_bounds__(kThreadsFill)
    fsa_fill_zero_kernel(float* __restrict__ dst, int64_t count) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  const int64_t t0 = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t n4 = count >> 2;
  float4* d4 = reinterpret_cast<float4*>(dst);
  for (int64_t i = t0; i < n4; i += stride) {
    asm volatile("st.global.cs.v4.f32 [%0], {%1,%1,%1,%1};" ::"l"(d4 + i), "f"(0.0F)
                 : "memory");
  }
  for (int64_t i = (n4 << 2) + t0; i < count; i += stride) dst[i] = 0.0F;
}

__global__ void __launch_bounds__(kThreadsFill)
    fsa_fill_zero_scalar_kernel(float* __restrict__ dst, int64_t count) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
       i < count; i += stride) {
    dst[i] = 0.0F;
  }
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------

int cuda_fail(cudaError_t err) {
  t_last_cuda_error = static_cast<int>(err);
  return FSA_ERR_CUDA;
}

int check_launch() {
  const cudaError_t err = cudaGetLastError();
  if (err != cudaSuccess) return cuda_fail(err);
  g_launches.fetch_add(1, std::memory_order_relaxed);
  return FSA_OK;
}

bool aligned(const void* p, uintptr_t bytes) {
  return (reinterpret_cast<uintptr_t>(p) % bytes) == 0;
}

// Widest vector (4, 2 or 1 floats) that divides D and keeps every listed
// pointer aligned.
int pick_vec(int64_t D, const void* p0, const void* p1) {
  if (D % 4 == 0 && aligned(p0, 16) && aligned(p1, 16)) return 4;
  if (D % 2 == 0 && aligned(p0, 8) && aligned(p1, 8)) return 2;
  return 1;
}

int grid_for(int64_t units) {
  return static_cast<int>(units < kMaxGrid ? units : kMaxGrid);
}

template <class Kernel, class Args>
int launch(Kernel kernel, int grid, int block, int smem, cudaStream_t stream,
           const Args& args) {
  if (smem > 48 * 1024) {
    const cudaError_t err =
        cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (err != cudaSuccess) return cuda_fail(err);
  }
  kernel<<<grid, block, smem, stream>>>(args);
  return check_launch();
}

// Tile width and vector width of the 2-hop forward that fit shared memory.
bool plan_2hop(int k1, int k2, int64_t D, int vec, int* dchunk_out, int* smem_out) {
  int dchunk = 0;
  if (D > 0) {
    const int64_t fit = kInnerBudgetBytes / (4 * static_cast<int64_t>(k1));
    int64_t c = fit < D ? fit : D;
    c -= c % vec;
    if (c < vec) c = vec;
    dchunk = static_cast<int>(c);
  }
  const Layout2 l = layout_2hop(k1, k2, dchunk);
  *dchunk_out = dchunk;
  *smem_out = l.total;
  return l.total <= kMaxSmemBytes;
}

}  // namespace

// ---------------------------------------------------------------------------
// C ABI
// ---------------------------------------------------------------------------

extern "C" {

int fsa_sample_agg_forward(const int32_t* rowptr, const int32_t* col,
                           int64_t num_nodes, int64_t num_edges, const float* x,
                           int64_t feature_dim, const int32_t* frontier,
                           int64_t batch_size, int64_t batch_offset, int32_t fanout,
                           uint64_t seed, float* out, int32_t* samples,
                           int32_t* takes, void* stream) {
  if (fanout < 0 || fanout > FSA_MAX_FANOUT_1HOP || batch_size < 0 ||
      feature_dim < 0 || num_nodes < 0 || num_edges < 0 || batch_offset < 0) {
    return FSA_ERR_INVALID_ARGUMENT;
  }
  if (batch_size == 0 || fanout == 0) return FSA_OK;
  if (rowptr == nullptr || frontier == nullptr || (num_edges > 0 && col == nullptr) ||
      (feature_dim > 0 && (out == nullptr || (num_nodes > 0 && x == nullptr)))) {
    return FSA_ERR_INVALID_ARGUMENT;
  }
  Fwd1Args a{rowptr, col, x, num_nodes, num_edges, feature_dim, frontier,
             batch_size, batch_offset, fanout, seed, out, samples, takes};
  const int vec = pick_vec(feature_dim, x, out);
  const int smem = 4 * fanout;
  const int grid = grid_for(batch_size);
  auto s = static_cast<cudaStream_t>(stream);
  switch (vec) {
    case 4: return launch(fsa_1hop_forward_kernel<4>, grid, kThreads1Hop, smem, s, a);
    case 2: return launch(fsa_1hop_forward_kernel<2>, grid, kThreads1Hop, smem, s, a);
    default: return launch(fsa_1hop_forward_kernel<1>, grid, kThreads1Hop, smem, s, a);
  }
}

int fsa_sample_agg_backward(const int32_t* samples, const int32_t* takes,
                            const float* grad_out, int64_t batch_size,
                            int64_t feature_dim, int32_t fanout, float* grad_x,
                            int64_t num_nodes, void* stream) {
  if (fanout < 0 || batch_size < 0 || feature_dim < 0 || num_nodes < 0) {
    return FSA_ERR_INVALID_ARGUMENT;
  }
  if (batch_size == 0 || fanout == 0 || feature_dim == 0) return FSA_OK;
  if (samples == nullptr || takes == nullptr || grad_out == nullptr ||
      (num_nodes > 0 && grad_x == nullptr)) {
    return FSA_ERR_INVALID_ARGUMENT;
  }
  Bwd1Args a{samples, takes, grad_out, batch_size, feature_dim, fanout, grad_x, num_nodes};
  const int vec = pick_vec(feature_dim, grad_out, grad_x);
  const int64_t blocks = (batch_size + (kThreadsBwd / 32) - 1) / (kThreadsBwd / 32);
  const int grid = grid_for(blocks);
  auto s = static_cast<cudaStream_t>(stream);
  switch (vec) {
    case 4: return launch(fsa_1hop_backward_kernel<4>, grid, kThreadsBwd, 0, s, a);
    case 2: return launch(fsa_1hop_backward_kernel<2>, grid, kThreadsBwd, 0, s, a);
    default: return launch(fsa_1hop_backward_kernel<1>, grid, kThreadsBwd, 0, s, a);
  }
}

int fsa_sample_agg_2hop_forward(const int32_t* rowptr, const int32_t* col,
                                int64_t num_nodes, int64_t num_edges,
                                const float* x, int64_t feature_dim,
                                const int32_t* frontier, int64_t batch_size,
                                int64_t batch_offset, int32_t fanout1,
                                int32_t fanout2, uint64_t seed, float* out,
                                int32_t* samples1, int32_t* samples2,
                                void* stream) {
  if (fanout1 < 0 || fanout2 < 0 || batch_size < 0 || feature_dim < 0 ||
      num_nodes < 0 || num_edges < 0 || batch_offset < 0) {
    return FSA_ERR_INVALID_ARGUMENT;
  }
  if (static_cast<int64_t>(fanout1) + static_cast<int64_t>(fanout1) * fanout2 >
      FSA_MAX_2HOP_ENTRIES) {
    return FSA_ERR_INVALID_ARGUMENT;
  }
  if (batch_size == 0 || fanout1 == 0 || fanout2 == 0) return FSA_OK;
  if (rowptr == nullptr || frontier == nullptr || (num_edges > 0 && col == nullptr) ||
      (feature_dim > 0 && (out == nullptr || (num_nodes > 0 && x == nullptr)))) {
    return FSA_ERR_INVALID_ARGUMENT;
  }
  int vec = pick_vec(feature_dim, x, out);
  int dchunk = 0, smem = 0;
  while (!plan_2hop(fanout1, fanout2, feature_dim, vec, &dchunk, &smem)) {
    if (vec == 1) return FSA_ERR_INVALID_ARGUMENT;
    vec >>= 1;
  }
  Fwd2Args a{rowptr, col, x, num_nodes, num_edges, feature_dim, frontier,
             batch_size, batch_offset, fanout1, fanout2, seed, out, samples1,
             samples2, dchunk};
  const int grid = grid_for(batch_size);
  auto s = static_cast<cudaStream_t>(stream);
  switch (vec) {
    case 4: return launch(fsa_2hop_forward_kernel<4>, grid, kThreads2Hop, smem, s, a);
    case 2: return launch(fsa_2hop_forward_kernel<2>, grid, kThreads2Hop, smem, s, a);
    default: return launch(fsa_2hop_forward_kernel<1>, grid, kThreads2Hop, smem, s, a);
  }
}

int fsa_sample_agg_2hop_backward(const float* grad_out, const int32_t* samples1,
                                 const int32_t* samples2, int64_t batch_size,
                                 int64_t feature_dim, int32_t fanout1,
                                 int32_t fanout2, float* grad_x,
                                 int64_t num_nodes, void* stream) {
  if (fanout1 < 0 || fanout2 < 0 || batch_size < 0 || feature_dim < 0 ||
      num_nodes < 0) {
    return FSA_ERR_INVALID_ARGUMENT;
  }
  if (static_cast<int64_t>(fanout1) + static_cast<int64_t>(fanout1) * fanout2 >
      FSA_MAX_2HOP_ENTRIES) {
    return FSA_ERR_INVALID_ARGUMENT;
  }
  if (batch_size == 0 || fanout1 == 0 || fanout2 == 0 || feature_dim == 0) return FSA_OK;
  if (grad_out == nullptr || samples1 == nullptr || samples2 == nullptr ||
      (num_nodes > 0 && grad_x == nullptr)) {
    return FSA_ERR_INVALID_ARGUMENT;
  }
  Bwd2Args a{grad_out, samples1, samples2, batch_size, feature_dim,
             fanout1, fanout2, grad_x, num_nodes};
  const int vec = pick_vec(feature_dim, grad_out, grad_x);
  const int smem = 4 * (fanout1 + fanout1 * fanout2 + 1);
  const int grid = grid_for(batch_size);
  auto s = static_cast<cudaStream_t>(stream);
  switch (vec) {
    case 4: return launch(fsa_2hop_backward_kernel<4>, grid, kThreadsBwd, smem, s, a);
    case 2: return launch(fsa_2hop_backward_kernel<2>, grid, kThreadsBwd, smem, s, a);
    default: return launch(fsa_2hop_backward_kernel<1>, grid, kThreadsBwd, smem, s, a);
  }
}

int fsa_fill_zero_f32(float* dst, int64_t count, void* stream) {
  if (count < 0 || (count > 0 && dst == nullptr)) return FSA_ERR_INVALID_ARGUMENT;
  if (count == 0) return FSA_OK;
  int device = 0, sms = 0;
  cudaError_t err = cudaGetDevice(&device);
  if (err == cudaSuccess) err = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
  if (err != cudaSuccess) return cuda_fail(err);
  // Enough CTAs for every SM to keep stores in flight; each thread loops.
  const int64_t want = (count / 4 + kThreadsFill - 1) / kThreadsFill;
  const int64_t cap = static_cast<int64_t>(sms) * 8;
  const int grid = static_cast<int>(want < cap ? (want > 0 ? want : 1) : cap);
  auto s = static_cast<cudaStream_t>(stream);
  if (aligned(dst, 16)) {
    fsa_fill_zero_kernel<<<grid, kThreadsFill, 0, s>>>(dst, count);
  } else {
    fsa_fill_zero_scalar_kernel<<<grid, kThreadsFill, 0, s>>>(dst, count);
  }
  return check_launch();
}

const char* fsa_status_string(int status) {
  switch (status) {
    case FSA_OK: return "ok";
    case FSA_ERR_INVALID_ARGUMENT: return "invalid argument";
    case FSA_ERR_CUDA: return "CUDA runtime error";
    default: return "unknown status";
  }
}

int fsa_last_cuda_error(void) { return t_last_cuda_error; }

uint64_t fsa_launch_count(void) { return g_launches.load(std::memory_order_relaxed); }

int fsa_device_status(int device, uint32_t* flags, int reset) {
  if (flags == nullptr) return FSA_ERR_INVALID_ARGUMENT;
  int prev = 0;
  cudaError_t err = cudaGetDevice(&prev);
  if (err != cudaSuccess) return cuda_fail(err);
  err = cudaSetDevice(device);
  if (err != cudaSuccess) return cuda_fail(err);
  err = cudaDeviceSynchronize();
  unsigned int v = 0;
  if (err == cudaSuccess) err = cudaMemcpyFromSymbol(&v, g_status, sizeof(v));
  if (err == cudaSuccess && reset) {
    const unsigned int zero = 0;
    err = cudaMemcpyToSymbol(g_status, &zero, sizeof(zero));
  }
  const cudaError_t err2 = cudaSetDevice(prev);
  if (err != cudaSuccess) return cuda_fail(err);
  if (err2 != cudaSuccess) return cuda_fail(err2);
  *flags = v;
  return FSA_OK;
}

}  // extern "C"
