// Fused reservoir-sample + mean-aggregate kernels for B200 (sm_100a) and the
// C ABI declared in include/fsa_sm100.h.
//
// Reference kernels: fuseop/fused_sample_agg.cu:58-271.  The reference runs
// Algorithm R on one thread per row (fused_sample_agg.cu:40-56): for
// power-law graphs that is tens of thousands of dependent xorshift steps per
// root while the rest of the CTA idles.  Here:
//
//   * Parallel, bit-exact Algorithm R.  A row's draws are cut into chunks of
//     kChunk positions aligned to the row start.  A thread reaches a chunk's
//     first state with GF(2) table products (fsa_rng.cuh), runs its draws and
//     records, per reservoir slot, the largest position that selected it
//     (atomicMax).  The slot then holds col[winner], or col[slot] if never
//     replaced -- exactly what the serial loop leaves behind.
//   * 2-hop forward = three launches (four from 2048 roots up): plan (CTA
//     per root: first hop, table of second-hop rows), [scan (one CTA: chunk
//     prefix over the roots; smaller batches scan it in each draw CTA)], draws
//     (persistent grid; the chunks of all rows are numbered consecutively
//     and a warp draws 32 consecutive chunks at a time, one per lane, so hub
//     rows and light rows balance across the GPU; optionally the same kernel
//     zeroes the backward's dense gradient with spare memory bandwidth) and
//     gather (CTA per root: winners to ids, then the two-level mean).
//   * Gather order = the reference's: per feature, leaves in j order from
//     0.0f, / valid; slot means in i order, / non-empty (IEEE division), so
//     forward outputs are bit-identical.  Rows are read with
//     ld.global.nc.L1::no_allocate.v{4,2,1}.f32 by feature width.
//   * Backward: red.global.add.v{4,2}.f32 of (grad/nonempty)/valid; a
//     sort-by-destination variant (one store per touched row) is kept as a
//     measured alternative.
//   * Draw, gather and backward are programmatic dependent launches: they
//     may start while the kernel before them finishes, and wait for it
//     (griddepcontrol.wait) before reading its results -- so the gradient
//     fill, which needs nothing from the plan kernel, starts early.
//   * No kernel allocates, synchronises with the host or spins on another
//     thread block.  Out-of-range ids are never dereferenced: they are
//     skipped and reported in a per-device status word.
#include <cuda_runtime.h>

#include <array>
#include <atomic>
#include <climits>
#include <cstdint>
#include <cstring>
#include <mutex>
#include <vector>

#include "fsa_rng.cuh"
#include "fsa_sm100.h"

namespace {

using fsa::JumpTables;

__device__ constexpr JumpTables g_jump = fsa::make_jump_tables();
__device__ unsigned int g_status;

constexpr int kThreads1Hop = 128;
// Leaf rows a 1-hop forward thread has in flight (then summed in slot order).
constexpr int kBatch1Hop = 4;
constexpr int kThreadsBwd = 256;
constexpr int kThreadsFill = 256;
// Float4 stores per thread of the zero fill.  A flat grid of short CTAs that
// each write one contiguous 16 KB block sustained ~7.4 TB/s on B200, ~18 %
// more than grid-stride loops over the same buffer.
constexpr int kFillVecsPerThread = 4;
constexpr int64_t kMaxGrid = int64_t{1} << 20;

std::atomic<uint64_t> g_launches{0};
thread_local int t_last_cuda_error = 0;

// ---------------------------------------------------------------------------
// Device helpers
// ---------------------------------------------------------------------------

__device__ __forceinline__ void flag_status(unsigned int bits) {
  atomicOr(&g_status, bits);
}

__device__ constexpr fsa::LaneTables g_lanes1 = fsa::make_lane_tables(fsa::kChunkLog2);
__device__ constexpr fsa::LaneTables g_lanes2 = fsa::make_lane_tables(fsa::kChunkLog2 + 5);
__device__ constexpr fsa::LaneTablesT g_lanes1_t =
    fsa::transpose_lane_tables(fsa::make_lane_tables(fsa::kChunkLog2));

constexpr uint32_t kChunk = 1u << fsa::kChunkLog2;
constexpr uint32_t kStarMulLo = static_cast<uint32_t>(fsa::kStarMul);
constexpr uint32_t kStarMulHi = static_cast<uint32_t>(fsa::kStarMul >> 32);

__device__ __forceinline__ uint64_t apply_table(const uint64_t* tab, uint64_t s) {
  uint64_t acc = 0;
#pragma unroll
  for (int p = 0; p < 16; ++p) {
    acc ^= __ldg(tab + p * 16 + static_cast<int>((s >> (4 * p)) & 15));
  }
  return acc;
}

// State before the first draw of chunk j of a row whose initial state is s0,
// i.e. T^(j * kChunk) s0 (see LaneTables in fsa_rng.cuh).
__device__ __forceinline__ uint64_t chunk_start(uint64_t s0, uint32_t j) {
  uint64_t s = apply_table(&g_lanes1.v[j & 31][0][0], s0);
  if ((j >> 5) & 31) s = apply_table(&g_lanes2.v[(j >> 5) & 31][0][0], s);
  uint32_t hi = j >> 10;
#pragma unroll 1
  while (hi != 0) {
    const int b = __ffs(hi) - 1;
    hi &= hi - 1;
    s = apply_table(&g_jump.v[fsa::kChunkLog2 + 10 + b][0][0], s);
  }
  return s;
}

// Resolves one candidate draw exactly and records a hit.
__device__ __forceinline__ void draw_hit(uint32_t lo, uint32_t r_hi, uint32_t bound,
                                         uint32_t take, int* win) {
  const uint64_t r = (static_cast<uint64_t>(r_hi) << 32) | (lo * kStarMulLo);
  const uint32_t slot = fsa::bounded_draw(r, bound);
  if (slot < take) atomicMax(&win[slot], static_cast<int>(bound - 1u));
}

// A draw with bound >= b_min can only hit (slot < take) if the high word of
// r is below floor(take * 2^32 / b_min) + 1; the double quotient is exact to
// within one unit, so +2 keeps the threshold conservative.
__device__ __forceinline__ uint32_t hit_threshold(uint32_t take, uint32_t b_min) {
  const double q = static_cast<double>(take) * 4294967296.0 / static_cast<double>(b_min);
  return q >= 4294967293.0 ? 0xffffffffU : static_cast<uint32_t>(q) + 2u;
}

constexpr int kDrawGroup = 4;

// `count` consecutive draws of one row starting at row position `pos`
// (>= take) from state s: draw at position p steps the state, forms
// r = state * M and selects slot floor(r * (p+1) / 2^64) if it is < take;
// a hit records p in win[slot] (the largest hit position wins, which is the
// last write of the reference's serial loop, fused_sample_agg.cu:47-52).
// Only r's high word is formed per draw; groups of draws share one branch on
// their smallest high word against the chunk's hit threshold.
__device__ __forceinline__ void chunk_draws(uint64_t s, uint32_t pos, uint32_t count,
                                            uint32_t take, int* win) {
  uint32_t bound = pos + 1u;
  const uint32_t thr = hit_threshold(take, bound);
  uint32_t k = 0;
  for (; k + kDrawGroup <= count; k += kDrawGroup, bound += kDrawGroup) {
    uint32_t l[kDrawGroup], rh[kDrawGroup];
    uint32_t rmin = 0xffffffffU;
#pragma unroll
    for (int u = 0; u < kDrawGroup; ++u) {
      s = fsa::xorshift_step(s);
      l[u] = static_cast<uint32_t>(s);
      rh[u] = __umulhi(l[u], kStarMulLo) + l[u] * kStarMulHi +
              static_cast<uint32_t>(s >> 32) * kStarMulLo;
      rmin = min(rmin, rh[u]);
    }
    if (rmin < thr) {
#pragma unroll
      for (int u = 0; u < kDrawGroup; ++u) draw_hit(l[u], rh[u], bound + u, take, win);
    }
  }
  for (; k < count; ++k, ++bound) {
    s = fsa::xorshift_step(s);
    const uint32_t lo = static_cast<uint32_t>(s);
    const uint32_t rh = __umulhi(lo, kStarMulLo) + lo * kStarMulHi +
                        static_cast<uint32_t>(s >> 32) * kStarMulLo;
    if (rh < thr) draw_hit(lo, rh, bound, take, win);
  }
}

// Chunk j of a row with `take` slots and `ndraws` draws.
__device__ __forceinline__ void row_chunk(uint64_t s0, uint32_t take, uint32_t ndraws,
                                          uint32_t j, int* win) {
  const uint32_t off = j * kChunk;
  const uint32_t count = ndraws - off < kChunk ? ndraws - off : kChunk;
  chunk_draws(chunk_start(s0, j), take + off, count, take, win);
}

// All draws of a single row, chunks spread over the CTA's threads.
__device__ __forceinline__ void block_row_draws(uint64_t s0, int take, int ndraws, int* win) {
  const uint32_t chunks = (static_cast<uint32_t>(ndraws) + kChunk - 1) / kChunk;
  for (uint32_t j = threadIdx.x; j < chunks; j += blockDim.x) {
    row_chunk(s0, static_cast<uint32_t>(take), static_cast<uint32_t>(ndraws), j, win);
  }
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
__global__ void __launch_bounds__(kThreads1Hop, 8)
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
      block_row_draws(s0, take, degree - take, slots);
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
      // kBatch1Hop rows in flight per thread, then summed in slot order.
      for (int i0 = 0; i0 < take; i0 += kBatch1Hop) {
        VecF<V> rows[kBatch1Hop];
        bool ok[kBatch1Hop];
#pragma unroll
        for (int u = 0; u < kBatch1Hop; ++u) {
          const int32_t leaf = i0 + u < take ? slots[i0 + u] : -1;
          ok[u] = leaf >= 0 && leaf < a.num_nodes;
          if (ok[u]) {
            rows[u] = load_stream<V>(a.x + static_cast<int64_t>(leaf) * a.feature_dim + v * V);
          } else if (i0 + u < take && v == 0) {
            flag_status(FSA_STATUS_BAD_NEIGHBOR);
          }
        }
#pragma unroll
        for (int u = 0; u < kBatch1Hop; ++u) {
          if (ok[u]) {
#pragma unroll
            for (int c = 0; c < V; ++c) acc.v[c] += rows[u].v[c];
          }
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
//
// The reference gives each root one CTA whose thread 0 runs the first-hop
// reservoir and then all fanout1 second-hop reservoirs serially
// (fused_sample_agg.cu:151-187).  Second-hop rows are size-biased (hubs), so
// the work per root varies by orders of magnitude.  Here the forward is four
// launches on the caller's stream:
//
//   plan   CTA per root: first-hop reservoir (draws split over the CTA),
//          first-hop ids, and the table of second-hop rows (begin, take,
//          draw count); second-hop winner slots set to -1.
//   scan   one CTA: exclusive prefix of the draw counts of all B*fanout1
//          second-hop rows -- the global draw space.
//   draws  persistent grid: every thread takes an equal contiguous chunk of
//          the global draw space, whichever rows and roots it spans, jumps
//          to its first state and records winners with atomicMax.
//   gather CTA per root: winners -> ids (col lookups), nested mean.
// ---------------------------------------------------------------------------

// Programmatic dependent launch (sm_90+).  The plan (or scan) kernel lets
// the draw kernel launch while its own CTAs are still running; a thread of
// the draw kernel that reads their results first waits for their grid to
// complete and its memory to be visible.  Both are no-ops for a kernel
// launched without the attribute.
__device__ __forceinline__ void launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void wait_prerequisites() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}

constexpr int kThreadsPlan = 128;
constexpr int kThreadsScan = 1024;
constexpr int kThreadsDraw = 768;
// Gather CTA sizes: roots whose (slot, feature-vector) items fit
// kGatherSmallItems run on kThreadsGatherSmall threads (8 CTAs per SM at 64
// registers: 1,184 roots resident at once, so a 1,024-root batch runs in one
// wave); wider rows, tiled in shared memory, on kThreadsGatherWide.
// Measured gather times (us; fraction of measured HBM copy bandwidth):
// 1,024 roots, 15 x 10, D = 100: 256 threads 24.7 (0.33), 128 threads 20.6
// (0.40), 96 22.2, 64 26.2; 4,096 roots, D = 128: 72.3 -> 67.4; 65,536
// roots, D = 128: 944 -> 824 (0.81); D = 602 (rows tiled): 256 threads
// 139.6, 128 threads 159.9.  With no more roots than the wide CTAs hold at
// once the small CTA only adds item rounds (512 roots, 8 x 4, D = 200:
// 128 threads 14.7, 256 threads 12.6), so it is used only above that.
constexpr int kThreadsGatherSmall = 128;
constexpr int kThreadsGatherWide = 256;
constexpr int kGatherSmallItems = 512;
constexpr int kGatherWidePerSm = 1024 / kThreadsGatherWide;  // resident wide CTAs per SM

// Draws of a second-hop row are split into chunks of kChunk positions; the
// chunks of all rows are numbered consecutively (roots in batch order, their
// rows in slot order, each row's chunks in position order) and a warp takes
// 32 consecutive chunks at a time, one per lane, whichever rows they are in.

struct Plan2Args {
  const int32_t* rowptr;
  const int32_t* col;
  int64_t num_nodes;
  int64_t num_edges;
  const int32_t* frontier;
  int64_t batch_size;
  int64_t batch_offset;
  int fanout1;
  int fanout2;
  uint64_t seed;
  int32_t* s1;               // [B][k1] first-hop ids
  int32_t* win2;             // [B][k1][k2] second-hop winners, -1 = slot kept
  int32_t* mbeg;             // [R = B*k1] begin of each second-hop row
  int32_t* mtake;            // [R] reservoir size of each second-hop row
  int32_t* mdraws;           // [R] draws of each second-hop row
  unsigned long long* state; // [R] initial xorshift state of each second-hop row
  long long* lpre;           // [R] chunk prefix of the row within its root
  long long* rgroups;        // [B] chunks of all second-hop rows of a root
  unsigned long long* next;  // draw-kernel fill-block counter, reset here
};

__global__ void __launch_bounds__(kThreadsPlan)
    fsa_2hop_plan_kernel(const Plan2Args a) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  int* s1 = reinterpret_cast<int*>(smem_raw);  // [k1] winners, then ids
  long long* groups = reinterpret_cast<long long*>(smem_raw + ((4 * a.fanout1 + 15) & ~15));
  const int k1 = a.fanout1;
  const int k2 = a.fanout2;
  const int tid = threadIdx.x;
  const int nthreads = blockDim.x;
  const int64_t N = a.num_nodes;
  if (blockIdx.x == 0 && tid == 0) *a.next = 0;  // fill-block counter of the draw kernel
  // The draw kernel may launch now: its fill needs nothing from this kernel,
  // and its readers of this kernel's results wait for this grid first.
  launch_dependents();

  for (int64_t b = blockIdx.x; b < a.batch_size; b += gridDim.x) {
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
    __syncthreads();
    if (rdegree > take1) {
      const uint64_t s0 = fsa::row_state(a.seed, static_cast<uint64_t>(root), 0,
                                         static_cast<uint64_t>(b + a.batch_offset));
      block_row_draws(s0, take1, rdegree - take1, s1);
    }
    __syncthreads();
    for (int i = tid; i < k1; i += nthreads) {
      int32_t m = -1;
      if (i < take1) {
        const int w = s1[i];
        m = a.col[static_cast<int64_t>(rbegin) + (w >= 0 ? w : i)];
      }
      a.s1[b * k1 + i] = m;
      int32_t mb = 0, md = 0;
      if (m >= 0) {
        if (m < N) {
          if (!read_row(a.rowptr, a.num_edges, m, mb, md)) flag_status(FSA_STATUS_BAD_ROW);
        } else {
          flag_status(FSA_STATUS_BAD_NEIGHBOR);
        }
      }
      const int mt = md < k2 ? md : k2;
      const int64_t r = b * k1 + i;
      a.mbeg[r] = mb;
      a.mtake[r] = mt;
      a.mdraws[r] = md - mt;
      a.state[r] = fsa::row_state(a.seed, static_cast<uint64_t>(root), 1, static_cast<uint64_t>(i));
      groups[i] = (static_cast<long long>(md - mt) + kChunk - 1) / kChunk;
    }
    // Every second-hop slot starts as "kept" (no winner).
    for (int64_t e = tid; e < static_cast<int64_t>(k1) * k2; e += nthreads) {
      a.win2[b * k1 * k2 + e] = -1;
    }
    __syncthreads();
    if (tid == 0) {
      long long run = 0;
      for (int i = 0; i < k1; ++i) {
        a.lpre[b * k1 + i] = run;
        run += groups[i];
      }
      a.rgroups[b] = run;
    }
    __syncthreads();
  }
}

struct Scan2Args {
  const long long* counts;  // [n]
  long long* pre;           // [n + 1] exclusive prefix, pre[n] = total
  int64_t n;
};

constexpr int kScanItems = 4;

// Barrier `id` among `nthreads` threads (whole warps) of the CTA; id 0 with
// every thread of the CTA is __syncthreads.
__device__ __forceinline__ void group_sync(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// Exclusive prefix of counts[0, n) into pre[0, n], pre[n] = total, by a
// group of `nthreads` threads (whole warps, at most 1024; `tid` = index in
// the group) meeting at barrier `bar`: tiles of nthreads * kScanItems
// entries; each thread scans its contiguous items, warp shuffles and the
// warp totals give the tile prefix, a running carry joins the tiles.
// `warp_sums` ([32]) and `carry` are shared scratch; pre may be global or
// shared memory.  Every thread of the group must call it.
__device__ __forceinline__ void group_exclusive_scan(const long long* counts, long long* pre,
                                                     int64_t n, long long* warp_sums,
                                                     long long* carry, int tid, int nthreads,
                                                     int bar) {
  const int lane = tid & 31;
  const int warp = tid >> 5;
  const int nw = nthreads >> 5;
  if (tid == 0) *carry = 0;
  group_sync(bar, nthreads);
  const int64_t tile = static_cast<int64_t>(nthreads) * kScanItems;
  for (int64_t t0 = 0; t0 < n; t0 += tile) {
    const int64_t i0 = t0 + static_cast<int64_t>(tid) * kScanItems;
    long long v[kScanItems];
    long long local = 0;
#pragma unroll
    for (int u = 0; u < kScanItems; ++u) {
      v[u] = i0 + u < n ? counts[i0 + u] : 0;
      local += v[u];
    }
    long long incl = local;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const long long y = __shfl_up_sync(0xffffffffU, incl, o);
      if (lane >= o) incl += y;
    }
    if (lane == 31) warp_sums[warp] = incl;
    group_sync(bar, nthreads);
    if (warp == 0) {
      long long w = lane < nw ? warp_sums[lane] : 0;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const long long y = __shfl_up_sync(0xffffffffU, w, o);
        if (lane >= o) w += y;
      }
      if (lane < nw) warp_sums[lane] = w;
    }
    group_sync(bar, nthreads);
    long long run = *carry + (warp > 0 ? warp_sums[warp - 1] : 0) + incl - local;
#pragma unroll
    for (int u = 0; u < kScanItems; ++u) {
      if (i0 + u < n) pre[i0 + u] = run;
      run += v[u];
    }
    group_sync(bar, nthreads);
    if (tid == 0) *carry += warp_sums[nw - 1];
    group_sync(bar, nthreads);
  }
  if (tid == 0) pre[n] = *carry;
  group_sync(bar, nthreads);
}

// The same scan by every thread of the CTA.
__device__ __forceinline__ void block_exclusive_scan(const long long* counts, long long* pre,
                                                     int64_t n, long long* warp_sums,
                                                     long long* carry) {
  group_exclusive_scan(counts, pre, n, warp_sums, carry, static_cast<int>(threadIdx.x),
                       static_cast<int>(blockDim.x), 0);
}

// Chunk prefix over the roots when it does not fit the draw kernel's shared
// memory (batches of kSmemRoots roots or more; smaller batches are scanned
// by every draw CTA itself).
__global__ void __launch_bounds__(kThreadsScan) fsa_2hop_scan_kernel(const Scan2Args a) {
  __shared__ long long warp_sums[32];
  __shared__ long long carry;
  launch_dependents();  // the draw kernel's fill may start (see the plan kernel)
  block_exclusive_scan(a.counts, a.pre, a.n, warp_sums, &carry);
}

struct Draw2Args {
  const long long* rgroups;          // [B] chunks per root
  const long long* rpre;             // [B + 1] chunk prefix over roots (B >= smem_roots)
  const long long* lpre;             // [R] chunk prefix of each row within its root
  const unsigned long long* state;   // [R]
  const int32_t* mtake;              // [R]
  const int32_t* mdraws;             // [R]
  int64_t batch_size;
  int fanout1;
  int fanout2;
  int32_t* win2;                     // [R][k2] winners
  unsigned long long* next;          // fill-block counter
  float4* fill;                      // optional buffer to zero (16-byte aligned)
  int64_t fill_vec4;                 // float4 elements of `fill`
  int smem_roots;                    // rpre staged in shared memory when B < this
  // optional rows to zero instead (fill_vec4 == 0): rows zrows[k] of ztable,
  // zdim4 (<= 32) float4 each, ids outside [0, znum_rows) skipped
  float4* ztable;
  const int32_t* zrows;
  int64_t zrows_count;
  int zdim4;
  uint32_t znum_rows;
};

// Fill work item: 32 KB (kFillItemVec4 float4 stores per lane of a warp).
// Two fillers per CTA share the items: one thread driving the bulk-copy
// (TMA) engine from a zeroed shared block, and one warp of streaming
// stores.  Measured on the 2-hop power-law workload, this pair overlapped
// the draws better than more store warps, than the bulk-copy engine alone,
// or than draw warps that joined the fill after their draws.
constexpr int kFillItemVec4 = 64;
constexpr int kFillWarps = 2;
constexpr int kZeroBytes = 16384;   // zeroed shared source of the bulk copies
constexpr int kFillInFlight = 8;    // bulk-copy groups in flight
constexpr int kSmemRoots = 2048;
constexpr int kDrawTableBytes = static_cast<int>(sizeof(fsa::LaneTablesT));  // 64 KB
constexpr int kRprePad = (8 * (kSmemRoots + 1) + 15) & ~15;  // staged root prefix

// Zeroes fill block `idx` (32 KB) with streaming stores.  A full block is
// 64 stores per lane at immediate offsets from one address: the draws share
// the integer pipe with this loop, so it does no per-store arithmetic.
__device__ __forceinline__ void fill_block(float4* fill, int64_t fill_vec4, long long idx,
                                           int lane) {
  const long long v0 = idx * 32LL * kFillItemVec4;
  const float4 z = make_float4(0.0F, 0.0F, 0.0F, 0.0F);
  float4* p = fill + v0 + lane;
  if (v0 + 32LL * kFillItemVec4 <= fill_vec4) {
#pragma unroll
    for (int k = 0; k < kFillItemVec4; ++k) __stcs(p + 32 * k, z);
  } else {
    for (long long v = v0 + lane; v < fill_vec4; v += 32) __stcs(fill + v, z);
  }
}

// Zeroes fill items base + k for k = 0, 1, ... claimed from *counter
// (shared or global memory) while base + k < end, by bulk copies
// (evict-first in L2) from the zeroed shared block at shared-window address
// `zero`.  One thread; returns after its copies have completed.
__device__ __forceinline__ void fill_items_bulk(unsigned long long* counter, long long base,
                                                long long end, float4* fill,
                                                int64_t fill_vec4, uint32_t zero) {
  constexpr int64_t kItem = 32LL * kFillItemVec4;
  constexpr int64_t kPiece = kZeroBytes / 16;
  uint64_t policy = 0;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(policy));
  bool issued = false;
  for (long long item = base + static_cast<long long>(atomicAdd(counter, 1ULL)); item < end;
       item = base + static_cast<long long>(atomicAdd(counter, 1ULL))) {
    const int64_t v0 = item * kItem;
    const int64_t v1 = fill_vec4 - v0 < kItem ? fill_vec4 : v0 + kItem;
    for (int64_t v = v0; v < v1; v += kPiece) {
      const uint32_t bytes = static_cast<uint32_t>((v1 - v < kPiece ? v1 - v : kPiece) * 16);
      asm volatile(
          "cp.async.bulk.global.shared::cta.bulk_group.L2::cache_hint [%0], [%1], %2, %3;"
          :: "l"(fill + v), "r"(zero), "r"(bytes), "l"(policy) : "memory");
    }
    asm volatile("cp.async.bulk.commit_group;" ::: "memory");
    asm volatile("cp.async.bulk.wait_group.read %0;" :: "n"(kFillInFlight) : "memory");
    issued = true;
  }
  if (issued) asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}

// Zeroes the rows named by list entries [32 item, 32 item + 32): one
// coalesced id load, then one float4 store per lane and row (rows of at most
// 32 float4).  All 32 lanes must call it.
__device__ __forceinline__ void zero_row_tile(const Draw2Args& a, long long item, int lane) {
  const long long e = item * 32 + lane;
  const int32_t mine = e < a.zrows_count ? __ldg(a.zrows + e) : -1;
  const float4 z = make_float4(0.0F, 0.0F, 0.0F, 0.0F);
  float4* base = a.ztable + lane;
  const bool on = lane < a.zdim4;
#pragma unroll
  for (int u = 0; u < 32; ++u) {
    const int32_t r = __shfl_sync(0xffffffffU, mine, u);
    if (static_cast<uint32_t>(r) < a.znum_rows && on) {
      base[static_cast<int64_t>(r) * a.zdim4] = z;
    }
  }
}

// Claims the next work item of counter `c` for the warp (lane 0 adds, the
// value is broadcast).  All 32 lanes must call it.
__device__ __forceinline__ long long claim(unsigned long long* c, int lane) {
  unsigned long long v = 0;
  if (lane == 0) v = atomicAdd(c, 1ULL);
  return static_cast<long long>(__shfl_sync(0xffffffffU, v, 0));
}

// Largest idx in [0, n) with arr[idx] <= key, given arr[0] <= key and arr
// non-decreasing (one thread).
__device__ __forceinline__ int64_t upper_index(const long long* arr, int64_t n, long long key) {
  int64_t lo = 0, hi = n - 1;
  while (hi > lo) {
    const int64_t mid = (lo + hi + 1) >> 1;
    if (arr[mid] <= key) {
      lo = mid;
    } else {
      hi = mid - 1;
    }
  }
  return lo;
}

// Draws of global chunk c (one thread): the root and the row are found in
// the two prefix levels, the chunk's start state is two table products of
// the row's initial state (plus one per set bit of j / 1024 for very long
// rows).
__device__ __forceinline__ void draw_chunk(const Draw2Args& a, const long long* rpre,
                                           const uint64_t* k1, long long c) {
  const int f1 = a.fanout1;
  const int64_t b = upper_index(rpre, a.batch_size, c);
  const long long local = c - rpre[b];
  const int i = static_cast<int>(upper_index(a.lpre + b * f1, f1, local));
  const int64_t r = b * f1 + i;
  const uint32_t j = static_cast<uint32_t>(local - __ldg(a.lpre + r));
  const uint32_t take = static_cast<uint32_t>(__ldg(a.mtake + r));
  const uint32_t nd = static_cast<uint32_t>(__ldg(a.mdraws + r));
  const uint64_t s0 = __ldg(a.state + r);
  const uint32_t off = j * kChunk;
  // T^(j * kChunk) s0: the (j mod 32)-chunk part from the shared copy of the
  // one-chunk lane tables, the rest from global tables that the lanes of a
  // warp mostly share.
  uint64_t st = 0;
  {
    const uint64_t* tab = k1 + (j & 31);
#pragma unroll
    for (int p = 0; p < 16; ++p) st ^= tab[(p * 16 + static_cast<int>((s0 >> (4 * p)) & 15)) * 32];
  }
  if ((j >> 5) & 31) st = apply_table(&g_lanes2.v[(j >> 5) & 31][0][0], st);
  uint32_t hi = j >> 10;
#pragma unroll 1
  while (hi != 0) {
    const int bit = __ffs(hi) - 1;
    hi &= hi - 1;
    st = apply_table(&g_jump.v[fsa::kChunkLog2 + 10 + bit][0][0], st);
  }
  chunk_draws(st, take + off, nd - off < kChunk ? nd - off : kChunk, take,
              a.win2 + r * a.fanout2);
}

// Fill items zeroed from a CTA's own share before the plan kernel has
// finished: kFillStaticNum / kFillStaticDen of all items, split evenly over
// the CTAs; the rest are claimed from the global counter afterwards, which
// balances CTAs that started late.
constexpr int kFillStaticNum = 1;
constexpr int kFillStaticDen = 2;

// Persistent grid, two CTAs of 24 warps per SM.  Each CTA keeps a shared
// copy of the one-chunk lane tables (64 KB, lane index innermost) and of
// the root prefix.  Lane l of group G draws global chunk 32 G + l: two
// binary searches find its root and row, and its start state is one
// shared-table product plus one global-table product that the warp's lanes
// mostly share.
//
// Optionally the kernel also zeroes a buffer (the backward's dense
// gradient) in 32 KB items.  The draw loop is bound by integer issue, the
// fill by HBM writes, so they run side by side: warp 0 of each CTA drives
// the bulk-copy engine (lane 0), warp 1 stores, the other warps draw.
// (Warps that alternated between the two would tie each one's progress to
// the other's.)  The kernel is launched as a programmatic dependent of the
// plan (or scan) kernel: the fill needs nothing from it, so the two fill
// warps start on the CTA's static share of the items at once, and only
// then wait for the plan's grid before claiming the remaining items from
// the counter *next (reset by the plan kernel); the draw warps wait before
// reading the plan's row table.
__global__ void __launch_bounds__(kThreadsDraw, 2) fsa_2hop_draw_kernel(const Draw2Args a) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  uint64_t* s_k1 = reinterpret_cast<uint64_t*>(smem_raw);  // one-chunk lane tables, [p][nib][l]
  long long* s_rpre = reinterpret_cast<long long*>(smem_raw + kDrawTableBytes);  // [B + 1]
  float4* s_zero = reinterpret_cast<float4*>(smem_raw + kDrawTableBytes + kRprePad);
  __shared__ unsigned long long s_fill_next;  // claims within the CTA's static share
  launch_dependents();  // the gather kernel may launch; it waits for this grid
  const int lane = threadIdx.x & 31;
  const int64_t B = a.batch_size;
  const bool staged = B < a.smem_roots;
  {
    const uint4* src = reinterpret_cast<const uint4*>(&g_lanes1_t.v[0][0][0]);
    uint4* dst = reinterpret_cast<uint4*>(s_k1);
    for (int t = threadIdx.x; t < kDrawTableBytes / 16; t += blockDim.x) dst[t] = __ldg(src + t);
  }
  if (threadIdx.x == 0) s_fill_next = 0;
  if (a.fill_vec4 > 0) {
    for (int t = threadIdx.x; t < kZeroBytes / 16; t += blockDim.x) {
      s_zero[t] = make_float4(0.0F, 0.0F, 0.0F, 0.0F);
    }
    // The zeros are read by the bulk-copy (async) proxy.
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  __syncthreads();
  const int warps = static_cast<int>(blockDim.x >> 5);
  const int warp = static_cast<int>(threadIdx.x >> 5);
  // Row mode: zero listed rows (the rows a persistent gradient buffer's
  // previous backwards touched) instead of a whole buffer.  Both filler
  // warps store; the items are tiles of 32 list entries.
  const bool rows_mode = a.fill_vec4 == 0 && a.zrows_count > 0;
  const int fillers = (a.fill_vec4 > 0 || rows_mode) ? kFillWarps : 0;
  if (warp < fillers && rows_mode) {
    const long long nitems = (a.zrows_count + 31) / 32;
    const long long share = nitems * kFillStaticNum / kFillStaticDen / gridDim.x;
    const long long share0 = static_cast<long long>(blockIdx.x) * share;
    const long long dyn0 = static_cast<long long>(gridDim.x) * share;
    for (long long item = share0 + claim(&s_fill_next, lane); item < share0 + share;
         item = share0 + claim(&s_fill_next, lane)) {
      zero_row_tile(a, item, lane);
    }
    wait_prerequisites();
    for (long long item = dyn0 + claim(a.next, lane); item < nitems;
         item = dyn0 + claim(a.next, lane)) {
      zero_row_tile(a, item, lane);
    }
    return;
  }
  if (warp < fillers) {
    const long long nfill = (a.fill_vec4 + 32LL * kFillItemVec4 - 1) / (32LL * kFillItemVec4);
    const long long share = nfill * kFillStaticNum / kFillStaticDen / gridDim.x;
    const long long share0 = static_cast<long long>(blockIdx.x) * share;
    const long long dyn0 = static_cast<long long>(gridDim.x) * share;
    if (warp == 0) {
      if (lane == 0) {
        const uint32_t zero = static_cast<uint32_t>(__cvta_generic_to_shared(s_zero));
        fill_items_bulk(&s_fill_next, share0, share0 + share, a.fill, a.fill_vec4, zero);
        wait_prerequisites();
        fill_items_bulk(a.next, dyn0, nfill, a.fill, a.fill_vec4, zero);
      }
      return;
    }
    for (long long item = share0 + claim(&s_fill_next, lane); item < share0 + share;
         item = share0 + claim(&s_fill_next, lane)) {
      fill_block(a.fill, a.fill_vec4, item, lane);
    }
    wait_prerequisites();
    for (long long item = dyn0 + claim(a.next, lane); item < nfill;
         item = dyn0 + claim(a.next, lane)) {
      fill_block(a.fill, a.fill_vec4, item, lane);
    }
    return;
  }
  wait_prerequisites();
  if (staged) {
    // the chunk prefix over the roots, scanned by this CTA's drawing warps
    // (no scan kernel)
    __shared__ long long s_scan[33];
    group_exclusive_scan(a.rgroups, s_rpre, B, s_scan, s_scan + 32,
                         static_cast<int>(threadIdx.x) - 32 * fillers, 32 * (warps - fillers),
                         1);
  }
  const long long* rpre = staged ? s_rpre : a.rpre;
  const long long total = rpre[B];
  // Groups of 32 chunks cost about the same, so drawing warps take them
  // round robin.
  const long long ngroups = (total + 31) / 32;
  const long long stride = static_cast<long long>(gridDim.x) * (warps - fillers);
  for (long long G = static_cast<long long>(blockIdx.x) * (warps - fillers) + (warp - fillers);
       G < ngroups; G += stride) {
    const long long c = G * 32 + lane;
    if (c < total) draw_chunk(a, rpre, s_k1, c);
  }
}

// Feature (or gradient) rows block-partitioned over up to FSA_MAX_SHARDS
// devices: global row r lives in shard r / rows at local row r % rows.  The
// bases are device pointers valid in this process -- the local shard and
// peers' shards mapped over NVLink (CUDA IPC).  Passed by value.
struct RowShards {
  float* base[FSA_MAX_SHARDS];
  int64_t rows;
  int n;
};

// Row `id` (0 <= id < n * rows) of a table with row stride d.
__device__ __forceinline__ float* shard_row(const RowShards& t, int32_t id, int64_t d) {
  const uint32_t s = static_cast<uint32_t>(id) / static_cast<uint32_t>(t.rows);
  return t.base[s] + (static_cast<int64_t>(id) - static_cast<int64_t>(s) * t.rows) * d;
}

struct Gather2Args {
  const int32_t* col;
  const float* x;
  int64_t num_nodes;
  int64_t feature_dim;
  int64_t batch_size;
  int fanout1;
  int fanout2;
  const int32_t* mbeg;   // [B*k1]
  const int32_t* mtake;  // [B*k1]
  const int32_t* win2;   // [B][k1][k2] winners (position of the last hit, -1 = kept)
  int32_t* samples2;     // optional id output; may alias win2
  float* out;
  int dchunk;            // feature tile width (multiple of the vector width)
  RowShards xs;          // sharded feature rows (kSharded kernels only)
};

// Shared-memory layout of the gather kernel, in bytes.
struct LayoutG {
  int inner, s2, mvalid, total;
};

__host__ __device__ inline int align16(int v) { return (v + 15) & ~15; }

__host__ __device__ inline LayoutG layout_gather(int k1, int k2, int dchunk) {
  LayoutG l;
  l.inner = 0;                              // float [k1][dchunk]
  l.s2 = align16(4 * k1 * dchunk);          // int32 [k1 * k2]
  l.mvalid = align16(l.s2 + 4 * k1 * k2);   // int32 [k1]
  l.total = align16(l.mvalid + 4 * k1);
  return l;
}

// Rows gathered per batch of independent loads (per thread): a whole
// second-hop row of fanout 10 in one round trip.  Measured against 4, 6
// and 8 (with more CTAs per SM): 10 at 4 CTAs per SM was fastest on the
// 2-hop power-law and 1M-node microbenchmark workloads.
constexpr int kGatherBatch = 10;

// CTA per root.  Items are (first-hop slot, feature vector) pairs: an item
// sums its slot's valid leaf rows in j order from 0.0f (loads batched so
// that kGatherBatch rows are in flight per thread) and divides by the valid
// count; then the slot means are summed in slot order and divided by the
// non-empty count (fused_sample_agg.cu:189-213).
template <int V, bool kSharded, int kThreads>
__global__ void __launch_bounds__(kThreads, 1024 / kThreads)
    fsa_2hop_gather_kernel(const Gather2Args a) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const int k1 = a.fanout1;
  const int k2 = a.fanout2;
  const LayoutG L = layout_gather(k1, k2, a.dchunk);
  float* inner = reinterpret_cast<float*>(smem_raw + L.inner);
  int* s2 = reinterpret_cast<int*>(smem_raw + L.s2);
  int* mvalid = reinterpret_cast<int*>(smem_raw + L.mvalid);
  const int tid = threadIdx.x;
  const int nthreads = blockDim.x;
  const int k12 = k1 * k2;
  const int64_t D = a.feature_dim;
  const int64_t N = a.num_nodes;
  // Launched as a programmatic dependent of the draw kernel: everything
  // below reads its results.  The backward may launch behind this kernel.
  wait_prerequisites();
  launch_dependents();

  for (int64_t b = blockIdx.x; b < a.batch_size; b += gridDim.x) {
    // Winners -> second-hop ids: slot j of a row holds col[winner], or
    // col[j] if no draw replaced it -- the serial loop's final reservoir.
    for (int e = tid; e < k12; e += nthreads) {
      const int i = e / k2;
      const int j = e - i * k2;
      const int64_t r = b * k1 + i;
      int32_t id = -1;
      if (j < __ldg(a.mtake + r)) {
        const int w = a.win2[b * k12 + e];
        id = __ldg(a.col + static_cast<int64_t>(__ldg(a.mbeg + r)) + (w >= 0 ? w : j));
      }
      s2[e] = id;
      if (a.samples2 != nullptr) a.samples2[b * k12 + e] = id;
    }
    __syncthreads();
    for (int64_t f0 = 0; f0 < D; f0 += a.dchunk) {
      const int fc = static_cast<int>(D - f0 < a.dchunk ? D - f0 : a.dchunk);
      const int nv = fc / V;
      const int items = k1 * nv;
      for (int it = tid; it < items; it += nthreads) {
        const int i = it / nv;
        const int v = it - i * nv;
        const int32_t* leaves = s2 + i * k2;
        const float* base = a.x + f0 + v * V;
        VecF<V> acc;
        vzero(acc);
        int valid = 0;
        for (int j0 = 0; j0 < k2; j0 += kGatherBatch) {
          VecF<V> rows[kGatherBatch];
          bool ok[kGatherBatch];
#pragma unroll
          for (int u = 0; u < kGatherBatch; ++u) {
            const int32_t leaf = j0 + u < k2 ? leaves[j0 + u] : -1;
            ok[u] = leaf >= 0 && leaf < N;
            if (ok[u]) {
              rows[u] = load_stream<V>(kSharded ? shard_row(a.xs, leaf, D) + f0 + v * V
                                                : base + static_cast<int64_t>(leaf) * D);
            }
            if (leaf >= N && v == 0 && f0 == 0) flag_status(FSA_STATUS_BAD_NEIGHBOR);
          }
#pragma unroll
          for (int u = 0; u < kGatherBatch; ++u) {
            if (ok[u]) {
              ++valid;
#pragma unroll
              for (int c = 0; c < V; ++c) acc.v[c] += rows[u].v[c];
            }
          }
        }
        if (v == 0) mvalid[i] = valid;
        if (valid > 0) {
          const float denom = static_cast<float>(valid);
#pragma unroll
          for (int c = 0; c < V; ++c) acc.v[c] = acc.v[c] / denom;
        }
        store_vec(inner + i * a.dchunk + v * V, acc);
      }
      __syncthreads();
      for (int v = tid; v < nv; v += nthreads) {
        VecF<V> outer;
        vzero(outer);
        int nonempty = 0;
        for (int i = 0; i < k1; ++i) {
          if (mvalid[i] > 0) {
            ++nonempty;
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
  RowShards gs;          // sharded gradient rows (kSharded kernels only)
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

// Slot stride of the backward's shared leaf ids: k2 rounded up to 4, so a
// slot's ids start 16-byte aligned and an item reads them four at a time.
__host__ __device__ inline int bwd_slot_stride(int k2) { return (k2 + 3) & ~3; }

// One CTA per root; items are (first-hop slot, feature vector) pairs.  One
// pass puts the root's leaf ids in shared memory (padded with -1 to the slot
// stride) and counts each slot's valid ids with shared-memory atomics as they
// arrive; a first-hop id of -1 marks its slot empty (fused_sample_agg.cu:
// 229-240: a slot is non-empty when its first-hop id is valid and it has a
// valid second-hop id).  After one barrier every warp counts the non-empty
// slots with ballots.  The counts alternate between two arrays by root, so
// the next root's counting needs no extra barrier to clear them.
template <int V, bool kSharded>
__global__ void __launch_bounds__(kThreadsBwd, 8)
    fsa_2hop_backward_kernel(const Bwd2Args a) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const int k1 = a.fanout1;
  const int k2 = a.fanout2;
  const int k12 = k1 * k2;
  const int k2p = bwd_slot_stride(k2);
  int* s2 = reinterpret_cast<int*>(smem_raw);  // [k1][k2p] leaf ids, -1 padded
  int* valid2 = s2 + k1 * k2p;                 // [2][k1] valid counts, by root parity
  int* mid_ok = valid2 + 2 * k1;               // [k1] first-hop id present
  const int tid = threadIdx.x;
  const int nthreads = blockDim.x;
  const int lane = tid & 31;
  const int64_t dvec = a.feature_dim / V;
  for (int i = tid; i < 2 * k1; i += nthreads) valid2[i] = 0;
  // May be launched as a programmatic dependent of the kernel before it:
  // wait for that grid before reading anything.
  wait_prerequisites();
  __syncthreads();

  int parity = 0;
  for (int64_t b = blockIdx.x; b < a.batch_size; b += gridDim.x, parity ^= 1) {
    int* valid = valid2 + parity * k1;
    int* other = valid2 + (parity ^ 1) * k1;
    for (int i = tid; i < k1; i += nthreads) other[i] = 0;  // the next root's counts
    for (int e = tid; e < k12; e += nthreads) {
      const int i = e / k2;
      const int j = e - i * k2;
      const int32_t leaf = a.samples2[b * k12 + e];
      s2[i * k2p + j] = leaf;
      if (leaf >= 0) atomicAdd(&valid[i], 1);
      if (j == 0) mid_ok[i] = a.samples1[b * k1 + i] >= 0 ? 1 : 0;
    }
    for (int e = tid; e < k1 * (k2p - k2); e += nthreads) {
      const int i = e / (k2p - k2);
      s2[i * k2p + k2 + (e - i * (k2p - k2))] = -1;
    }
    __syncthreads();
    int nonempty = 0;
    for (int i0 = 0; i0 < k1; i0 += 32) {
      const int i = i0 + lane;
      nonempty += __popc(__ballot_sync(0xffffffffU, i < k1 && valid[i] > 0 && mid_ok[i] != 0));
    }
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
        const int4* leaves = reinterpret_cast<const int4*>(s2 + i * k2p);
#pragma unroll 1
        for (int j4 = 0; j4 < k2p / 4; ++j4) {
          const int4 q = leaves[j4];
          const int32_t lv[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const int32_t leaf = lv[u];
            if (leaf < 0) continue;
            if (leaf < a.num_nodes) {
              red_add<V>(kSharded ? shard_row(a.gs, leaf, a.feature_dim) + v * V
                                  : a.grad_x + static_cast<int64_t>(leaf) * a.feature_dim +
                                        v * V,
                         g);
            } else if (v == 0) {
              flag_status(FSA_STATUS_BAD_NEIGHBOR);
            }
          }
        }
      }
    }
    __syncthreads();
  }
}

// ---------------------------------------------------------------------------
// Sort-by-destination 2-hop backward (the alternative to red.global.add):
// contributions are grouped by destination row with a counting sort, then
// one warp per destination row sums them and writes the row once -- no
// atomics on the gradient, one write per touched row.
// ---------------------------------------------------------------------------

struct SortBwdArgs {
  const float* grad_out;
  const int32_t* samples1;
  const int32_t* samples2;
  int64_t batch_size;
  int64_t feature_dim;
  int fanout1;
  int fanout2;
  float* grad_x;
  int64_t num_nodes;
  int32_t* counts;      // [N + 1] entries per destination row, then the valid-entry
                        // total; zero on entry, zero again after the scatter
  int32_t* offsets;     // [N] exclusive prefix of counts
  long long* bsum;      // [ceil(N / kSortTile) + 1] tile totals, then their prefix
  int32_t* skey;        // [E] destination row of each sorted entry
  int32_t* sval;        // [E] (root, slot) = b * k1 + i of each sorted entry
  int32_t* slot_valid;  // [B * k1] valid second-hop ids of each slot
  int32_t* nonempty;    // [B] non-empty slots of each root
  int32_t* nentries;    // = counts + N: valid entries (the sorted length)
};

constexpr int kThreadsSort = 1024;
constexpr int kSortItems = 4;
constexpr int kSortTile = kThreadsSort * kSortItems;
static_assert(kSortItems == kScanItems, "one scan tile per CTA");

// Per root: valid count of every slot, the non-empty count (a slot counts
// when its first-hop id is valid and it has a valid second-hop id,
// fused_sample_agg.cu:229-240), and the histogram of destination rows.
__global__ void __launch_bounds__(256) fsa_2hop_sortbwd_count_kernel(const SortBwdArgs a) {
  __shared__ int ne;
  const int k1 = a.fanout1;
  const int k2 = a.fanout2;
  for (int64_t b = blockIdx.x; b < a.batch_size; b += gridDim.x) {
    if (threadIdx.x == 0) ne = 0;
    __syncthreads();
    for (int i = threadIdx.x; i < k1; i += blockDim.x) {
      int cnt = 0;
      for (int j = 0; j < k2; ++j) {
        const int32_t leaf = a.samples2[(b * k1 + i) * k2 + j];
        if (leaf >= 0) {
          ++cnt;
          if (leaf < a.num_nodes) {
            atomicAdd(a.counts + leaf, 1);
            atomicAdd(a.nentries, 1);
          } else {
            flag_status(FSA_STATUS_BAD_NEIGHBOR);
          }
        }
      }
      a.slot_valid[b * k1 + i] = cnt;
      if (cnt > 0 && a.samples1[b * k1 + i] >= 0) atomicAdd(&ne, 1);
    }
    __syncthreads();
    if (threadIdx.x == 0) a.nonempty[b] = ne;
    __syncthreads();
  }
}

// Tile-local exclusive prefix of counts into offsets; tile totals to bsum.
__global__ void __launch_bounds__(kThreadsSort) fsa_sortbwd_scan_tiles_kernel(const SortBwdArgs a) {
  __shared__ long long warp_sums[32];
  __shared__ long long carry;
  const int64_t t0 = static_cast<int64_t>(blockIdx.x) * kSortTile;
  const int64_t n = a.num_nodes - t0 < kSortTile ? a.num_nodes - t0 : kSortTile;
  // block_exclusive_scan works on long long; scan this tile through a
  // shared copy.
  __shared__ long long vals[kSortTile + 1];
  for (int64_t t = threadIdx.x; t < n; t += blockDim.x) vals[t] = a.counts[t0 + t];
  __syncthreads();
  block_exclusive_scan(vals, vals, n, warp_sums, &carry);
  for (int64_t t = threadIdx.x; t < n; t += blockDim.x) {
    a.offsets[t0 + t] = static_cast<int32_t>(vals[t]);
  }
  if (threadIdx.x == 0) a.bsum[blockIdx.x] = vals[n];
}

// Exclusive prefix of the tile totals (one CTA), in place in global memory
// (every tile's reads precede its writes in block_exclusive_scan).
__global__ void __launch_bounds__(kThreadsSort) fsa_sortbwd_scan_totals_kernel(
    const SortBwdArgs a, int64_t tiles) {
  __shared__ long long warp_sums[32];
  __shared__ long long carry;
  block_exclusive_scan(a.bsum, a.bsum, tiles, warp_sums, &carry);
}

// Every valid entry to its place: destination row's start + a slot claimed
// by decrementing its count (the counts end at zero).
__global__ void __launch_bounds__(256) fsa_2hop_sortbwd_scatter_kernel(const SortBwdArgs a) {
  const int k1 = a.fanout1;
  const int k2 = a.fanout2;
  const int64_t total = a.batch_size * k1 * k2;
  for (int64_t e = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; e < total;
       e += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int32_t leaf = a.samples2[e];
    if (leaf < 0 || leaf >= a.num_nodes) continue;
    const int32_t start = a.offsets[leaf] + static_cast<int32_t>(a.bsum[leaf / kSortTile]);
    const int32_t pos = start + atomicSub(a.counts + leaf, 1) - 1;
    a.skey[pos] = leaf;
    a.sval[pos] = static_cast<int32_t>(e / k2);
  }
}

// One warp per run of equal destinations in the sorted order: lanes over
// feature vectors add ((g / nonempty) / valid) of the run's entries (the
// reference's per-entry arithmetic, fused_sample_agg.cu:247-260) to the
// row's current value and store it once (no atomics).
template <int V>
__global__ void __launch_bounds__(256) fsa_2hop_sortbwd_reduce_kernel(const SortBwdArgs a) {
  const int lane = threadIdx.x & 31;
  const int k1 = a.fanout1;
  const int64_t D = a.feature_dim;
  const int64_t dvec = D / V;
  const int64_t E = *a.nentries;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  for (int64_t w0 = ((static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5) * 32;
       w0 < E; w0 += warps * 32) {
    const int64_t p = w0 + lane;
    const bool head = p < E && (p == 0 || a.skey[p] != a.skey[p - 1]);
    unsigned heads = __ballot_sync(0xffffffffU, head);
    while (heads != 0) {
      const int h = __ffs(heads) - 1;
      heads &= heads - 1;
      const int64_t s0 = w0 + h;
      const int32_t leaf = a.skey[s0];
      float* row = a.grad_x + static_cast<int64_t>(leaf) * D;
      for (int64_t v = lane; v < dvec; v += 32) {
        VecF<V> acc = load_vec<V>(row + v * V);
        for (int64_t q = s0; q < E && a.skey[q] == leaf; ++q) {
          const int32_t bi = a.sval[q];
          const int64_t b = bi / k1;
          const int nonempty = a.nonempty[b];
          if (nonempty == 0) continue;  // the atomic variant skips such roots too
          const float ne = static_cast<float>(nonempty);
          const float vc = static_cast<float>(a.slot_valid[bi]);
          const VecF<V> g = load_vec<V>(a.grad_out + b * D + v * V);
#pragma unroll
          for (int c = 0; c < V; ++c) acc.v[c] += (g.v[c] / ne) / vc;
        }
        store_vec(row + v * V, acc);
      }
    }
  }
}

// ---------------------------------------------------------------------------
// Dense zero fill of the gradient (replaces at::zeros, fuseop/binding.cpp:137)
// ---------------------------------------------------------------------------

__global__ void __launch_bounds__(kThreadsFill)
    fsa_fill_zero_kernel(float* __restrict__ dst, int64_t count) {
  const int64_t n4 = count >> 2;
  const int64_t base =
      static_cast<int64_t>(blockIdx.x) * blockDim.x * kFillVecsPerThread + threadIdx.x;
  float4* d4 = reinterpret_cast<float4*>(dst);
#pragma unroll
  for (int k = 0; k < kFillVecsPerThread; ++k) {
    const int64_t i = base + static_cast<int64_t>(k) * blockDim.x;
    if (i < n4) {
      asm volatile("st.global.cs.v4.f32 [%0], {%1,%1,%1,%1};" ::"l"(d4 + i), "f"(0.0F)
                   : "memory");
    }
  }
  // The count % 4 tail, by the first threads of the last CTA.
  if (blockIdx.x == gridDim.x - 1 && threadIdx.x < (count & 3)) {
    dst[(n4 << 2) + threadIdx.x] = 0.0F;
  }
}

// Zeroes table rows rows[k] (0 <= rows[k] < num_rows; others, such as the -1
// padding of saved ids, are skipped).  A warp takes 32 consecutive list
// entries with one coalesced load, then stores each listed row in turn
// (V-float stores by its lanes), so the stores of 32 rows issue back to back
// behind a single id load.  kOneStore: rows of at most 32 vectors, one
// predicated store per lane and row (about six instructions a row; the
// general loop cost about forty and bound the kernel by instruction issue).
// Plain (L2-allocating) stores: the rows are about to receive the
// backward's red.add, which then hits L2.  A row listed twice is written
// twice with the same zeros.
template <int V, bool kOneStore>
__global__ void __launch_bounds__(kThreadsFill)
    fsa_zero_rows_kernel(float* __restrict__ table, int64_t num_rows, int64_t dim,
                         const int32_t* __restrict__ rows, int64_t count) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  const int64_t dvec = dim / V;
  // ids are int32, so the range check is one unsigned compare
  const uint32_t nrows = num_rows < 0x7fffffffLL ? static_cast<uint32_t>(num_rows) : 0x7fffffffU;
  VecF<V> z;
  vzero(z);
  float* lane_base = table + static_cast<int64_t>(lane) * V;
  const bool lane_on = lane < dvec;
  for (int64_t t0 = (static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5)) * 32;
       t0 < count; t0 += warps * 32) {
    const int32_t mine = t0 + lane < count ? __ldg(rows + t0 + lane) : -1;
    if (kOneStore) {
#pragma unroll
      for (int u = 0; u < 32; ++u) {
        const int32_t r = __shfl_sync(0xffffffffU, mine, u);
        if (static_cast<uint32_t>(r) < nrows && lane_on) {
          store_vec(lane_base + static_cast<int64_t>(r) * dim, z);
        }
      }
    } else {
      for (int u = 0; u < 32; ++u) {
        const int32_t r = __shfl_sync(0xffffffffU, mine, u);
        if (static_cast<uint32_t>(r) >= nrows) continue;  // the same for every lane
        float* p = table + static_cast<int64_t>(r) * dim;
        for (int64_t v = lane; v < dvec; v += 32) store_vec(p + v * V, z);
      }
    }
  }
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

// The same launch as a programmatic dependent of the kernel before it in
// the stream (cudaLaunchAttributeProgrammaticStreamSerialization): it may
// start once every CTA of that kernel has run griddepcontrol.launch_dependents,
// and must itself wait (griddepcontrol.wait) before reading that kernel's
// results.
template <class Kernel, class Args>
int launch_dependent(Kernel kernel, int grid, int block, int smem, cudaStream_t stream,
                     const Args& args) {
  if (smem > 48 * 1024) {
    const cudaError_t err =
        cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (err != cudaSuccess) return cuda_fail(err);
  }
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(static_cast<unsigned int>(grid));
  cfg.blockDim = dim3(static_cast<unsigned int>(block));
  cfg.dynamicSmemBytes = static_cast<size_t>(smem);
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t err = cudaLaunchKernelEx(&cfg, kernel, args);
  if (err != cudaSuccess) return cuda_fail(err);
  return check_launch();
}

size_t align256(size_t v) { return (v + 255) & ~static_cast<size_t>(255); }

// Optional per-kernel timing of the 2-hop forward (fsa_phase_timing): five
// events per call, around plan, scan, draw and gather.  Off by default; the
// forward then records nothing.
constexpr int kPhases = 4;
std::atomic<bool> g_timing{false};
std::mutex g_timing_mu;
std::vector<std::array<cudaEvent_t, kPhases + 1>> g_timing_calls;

struct PhaseEvents {
  std::array<cudaEvent_t, kPhases + 1> ev{};
  bool on = false;
  int mark(int k, cudaStream_t s) {
    if (!on) return FSA_OK;
    const cudaError_t err = cudaEventRecord(ev[k], s);
    return err == cudaSuccess ? FSA_OK : cuda_fail(err);
  }
};

int phase_events_begin(PhaseEvents* pe) {
  pe->on = g_timing.load(std::memory_order_relaxed);
  if (!pe->on) return FSA_OK;
  for (auto& e : pe->ev) {
    const cudaError_t err = cudaEventCreate(&e);
    if (err != cudaSuccess) return cuda_fail(err);
  }
  std::lock_guard<std::mutex> lock(g_timing_mu);
  g_timing_calls.push_back(pe->ev);
  return FSA_OK;
}

// Workspace of the 2-hop forward, in bytes from a 256-byte aligned base.
struct Ws2 {
  size_t rpre, rgroups, lpre, state, mbeg, mtake, mdraws, next, s1, win2, total;
};

Ws2 ws2_layout(int64_t B, int k1, int k2, bool need_s1, bool need_win2) {
  Ws2 l{};
  const size_t rows = static_cast<size_t>(B) * static_cast<size_t>(k1);
  size_t off = 0;
  l.rpre = off;
  off = align256(off + 8 * (static_cast<size_t>(B) + 1));
  l.rgroups = off;
  off = align256(off + 8 * static_cast<size_t>(B));
  l.lpre = off;
  off = align256(off + 8 * rows);
  l.state = off;
  off = align256(off + 8 * rows);
  l.mbeg = off;
  off = align256(off + 4 * rows);
  l.mtake = off;
  off = align256(off + 4 * rows);
  l.mdraws = off;
  off = align256(off + 4 * rows);
  l.next = off;
  off = align256(off + 16);
  l.s1 = off;
  if (need_s1) off = align256(off + 4 * rows);
  l.win2 = off;
  if (need_win2) off = align256(off + 4 * rows * static_cast<size_t>(k2));
  l.total = off;
  return l;
}

// Feature tile width of the gather: the per-slot means of one tile live in
// shared memory.
constexpr int kInnerBudgetBytes = 24 * 1024;
constexpr int kMaxSmemBytes = 227 * 1024;

bool plan_gather(int k1, int k2, int64_t D, int vec, int* dchunk_out, int* smem_out) {
  int dchunk = 0;
  if (D > 0) {
    const int64_t fit = kInnerBudgetBytes / (4 * static_cast<int64_t>(k1));
    int64_t c = fit < D ? fit : D;
    c -= c % vec;
    if (c < vec) c = vec;
    dchunk = static_cast<int>(c);
  }
  const LayoutG l = layout_gather(k1, k2, dchunk);
  *dchunk_out = dchunk;
  *smem_out = l.total;
  return l.total <= kMaxSmemBytes;
}

// The gather kernel for vector width V: the small- or wide-CTA instance, on
// a shard table (plain launch) or as a programmatic dependent of the kernel
// before it.
template <int V>
int launch_gather(bool sharded, bool small, int grid, int threads, int smem, cudaStream_t s,
                  const Gather2Args& ga) {
  if (sharded) {
    return small ? launch(fsa_2hop_gather_kernel<V, true, kThreadsGatherSmall>, grid, threads,
                          smem, s, ga)
                 : launch(fsa_2hop_gather_kernel<V, true, kThreadsGatherWide>, grid, threads,
                          smem, s, ga);
  }
  return small ? launch_dependent(fsa_2hop_gather_kernel<V, false, kThreadsGatherSmall>, grid,
                                  threads, smem, s, ga)
               : launch_dependent(fsa_2hop_gather_kernel<V, false, kThreadsGatherWide>, grid,
                                  threads, smem, s, ga);
}

// Number of SMs of the current device (cached per device).
int sm_count(int* out) {
  static int cached[64] = {0};
  int dev = 0;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return cuda_fail(err);
  if (dev >= 0 && dev < 64 && cached[dev] > 0) {
    *out = cached[dev];
    return FSA_OK;
  }
  int sms = 0;
  err = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (err != cudaSuccess) return cuda_fail(err);
  if (dev >= 0 && dev < 64) cached[dev] = sms;
  *out = sms;
  return FSA_OK;
}

// Persistent grid of the draw kernel.
int draw_grid(int* grid_out) {
  static int cached[64] = {0};
  int dev = 0;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return cuda_fail(err);
  if (dev >= 0 && dev < 64 && cached[dev] > 0) {
    *grid_out = cached[dev];
    return FSA_OK;
  }
  int sms = 0, per_sm = 0;
  err = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (err == cudaSuccess) {
    const int smem = kDrawTableBytes + kRprePad + kZeroBytes;
    err = cudaFuncSetAttribute(fsa_2hop_draw_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               smem);
    if (err == cudaSuccess) {
      err = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fsa_2hop_draw_kernel,
                                                          kThreadsDraw, smem);
    }
  }
  if (err != cudaSuccess) return cuda_fail(err);
  const int grid = sms * (per_sm > 0 ? per_sm : 1);
  if (dev >= 0 && dev < 64) cached[dev] = grid;
  *grid_out = grid;
  return FSA_OK;
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

size_t fsa_sample_agg_2hop_workspace_size(int64_t batch_size, int32_t fanout1,
                                          int32_t fanout2, int has_samples1,
                                          int has_samples2) {
  if (batch_size <= 0 || fanout1 <= 0 || fanout2 <= 0) return 0;
  return ws2_layout(batch_size, fanout1, fanout2, has_samples1 == 0, has_samples2 == 0).total;
}

// Argument checks of the 2-hop forward that need no CUDA call (everything
// but the workspace).
static int check_forward_2hop_args(const int32_t* rowptr, const int32_t* col, int64_t num_nodes,
                                   int64_t num_edges, const float* x, int64_t feature_dim,
                                   const int32_t* frontier, int64_t batch_size,
                                   int64_t batch_offset, int32_t fanout1, int32_t fanout2,
                                   const float* out, const float* zero_fill,
                                   int64_t zero_count) {
  if (fanout1 < 0 || fanout2 < 0 || batch_size < 0 || feature_dim < 0 ||
      num_nodes < 0 || num_edges < 0 || batch_offset < 0 || zero_count < 0 ||
      (zero_count > 0 && zero_fill == nullptr)) {
    return FSA_ERR_INVALID_ARGUMENT;
  }
  if (static_cast<int64_t>(fanout1) + static_cast<int64_t>(fanout1) * fanout2 >
      FSA_MAX_2HOP_ENTRIES) {
    return FSA_ERR_INVALID_ARGUMENT;
  }
  const bool work = batch_size > 0 && fanout1 > 0 && fanout2 > 0;
  if (work && (rowptr == nullptr || frontier == nullptr || (num_edges > 0 && col == nullptr) ||
               (feature_dim > 0 && (out == nullptr || (num_nodes > 0 && x == nullptr))))) {
    return FSA_ERR_INVALID_ARGUMENT;
  }
  return FSA_OK;
}

// The 2-hop forward; `xs` (optional) reads the feature rows from a shard
// table instead of x.
static int forward_2hop(const int32_t* rowptr, const int32_t* col, int64_t num_nodes,
                        int64_t num_edges, const float* x, int64_t feature_dim,
                        const int32_t* frontier, int64_t batch_size, int64_t batch_offset,
                        int32_t fanout1, int32_t fanout2, uint64_t seed, float* out,
                        int32_t* samples1, int32_t* samples2, void* workspace,
                        size_t workspace_bytes, float* zero_fill, int64_t zero_count,
                        void* stream, const RowShards* xs, float* zero_table = nullptr,
                        const int32_t* zero_rows = nullptr, int64_t zero_rows_count = 0,
                        int64_t zero_table_rows = -1) {
  const int arg_status =
      check_forward_2hop_args(rowptr, col, num_nodes, num_edges, x, feature_dim, frontier,
                              batch_size, batch_offset, fanout1, fanout2, out, zero_fill,
                              zero_count);
  if (arg_status != FSA_OK) return arg_status;
  const bool work = batch_size > 0 && fanout1 > 0 && fanout2 > 0;
  const Ws2 wl = ws2_layout(batch_size, fanout1, fanout2, samples1 == nullptr,
                            samples2 == nullptr);
  if (work && (workspace == nullptr || workspace_bytes < wl.total || !aligned(workspace, 256))) {
    return FSA_ERR_INVALID_ARGUMENT;
  }
  // Listed rows of a [num_nodes][feature_dim] table to zero (the row-sparse
  // counterpart of zero_fill): in the draw kernel when the rows are whole
  // float4 vectors (at most 32 of them) and no dense fill rides along, else
  // with the stand-alone row kernel before the forward.
  float4* ztable4 = nullptr;
  const int64_t ztable_rows = zero_table_rows >= 0 ? zero_table_rows : num_nodes;
  if (zero_rows_count > 0) {
    const bool fuse = work && zero_count == 0 && feature_dim % 4 == 0 &&
                      feature_dim / 4 <= 32 && aligned(zero_table, 16) &&
                      ztable_rows <= 0x7fffffffLL;
    if (fuse) {
      ztable4 = reinterpret_cast<float4*>(zero_table);
    } else {
      const int st0 = fsa_zero_rows_f32(zero_table, ztable_rows, feature_dim, zero_rows,
                                        zero_rows_count, stream);
      if (st0 != FSA_OK) return st0;
    }
  }
  // The zero fill rides along in the draw kernel (float4 stores); a buffer
  // that is not 16-byte aligned or has a count % 4 tail, or a call with no
  // sampling work, gets the plain fill.
  float4* fill4 = nullptr;
  int64_t fill_vec4 = 0;
  if (zero_count > 0) {
    if (work && aligned(zero_fill, 16) && (zero_count & 3) == 0) {
      fill4 = reinterpret_cast<float4*>(zero_fill);
      fill_vec4 = zero_count >> 2;
    } else {
      const int st0 = fsa_fill_zero_f32(zero_fill, zero_count, stream);
      if (st0 != FSA_OK) return st0;
    }
  }
  if (!work) return FSA_OK;
  int vec = pick_vec(feature_dim, x, out);
  int dchunk = 0, gsmem = 0;
  while (!plan_gather(fanout1, fanout2, feature_dim, vec, &dchunk, &gsmem)) {
    if (vec == 1) return FSA_ERR_INVALID_ARGUMENT;
    vec >>= 1;
  }
  char* ws = static_cast<char*>(workspace);
  int32_t* s1 = samples1 != nullptr ? samples1 : reinterpret_cast<int32_t*>(ws + wl.s1);
  int32_t* win2 = samples2 != nullptr ? samples2 : reinterpret_cast<int32_t*>(ws + wl.win2);
  auto* rpre = reinterpret_cast<long long*>(ws + wl.rpre);
  auto* rgroups = reinterpret_cast<long long*>(ws + wl.rgroups);
  auto* lpre = reinterpret_cast<long long*>(ws + wl.lpre);
  auto* state = reinterpret_cast<unsigned long long*>(ws + wl.state);
  auto* mbeg = reinterpret_cast<int32_t*>(ws + wl.mbeg);
  auto* mtake = reinterpret_cast<int32_t*>(ws + wl.mtake);
  auto* mdraws = reinterpret_cast<int32_t*>(ws + wl.mdraws);
  auto* next = reinterpret_cast<unsigned long long*>(ws + wl.next);
  auto s = static_cast<cudaStream_t>(stream);

  const Plan2Args pa{rowptr, col, num_nodes, num_edges, frontier, batch_size, batch_offset,
                     fanout1, fanout2, seed, s1, win2, mbeg, mtake, mdraws, state, lpre,
                     rgroups, next};
  PhaseEvents pe;
  int st = phase_events_begin(&pe);
  if (st == FSA_OK) st = pe.mark(0, s);
  if (st != FSA_OK) return st;
  const int psmem = ((4 * fanout1 + 15) & ~15) + 8 * fanout1;
  st = launch(fsa_2hop_plan_kernel, grid_for(batch_size), kThreadsPlan, psmem, s, pa);
  if (st == FSA_OK) st = pe.mark(1, s);
  if (st != FSA_OK) return st;
  // Batches below kSmemRoots roots are scanned inside the draw kernel.
  if (batch_size >= kSmemRoots) {
    const Scan2Args sa{rgroups, rpre, batch_size};
    st = launch(fsa_2hop_scan_kernel, 1, kThreadsScan, 0, s, sa);
  }
  if (st == FSA_OK) st = pe.mark(2, s);
  if (st != FSA_OK) return st;
  int dgrid = 0;
  st = draw_grid(&dgrid);
  if (st != FSA_OK) return st;
  const Draw2Args da{rgroups, rpre, lpre, state, mtake, mdraws, batch_size, fanout1, fanout2,
                     win2, next, fill4, fill_vec4, kSmemRoots, ztable4,
                     ztable4 != nullptr ? zero_rows : nullptr,
                     ztable4 != nullptr ? zero_rows_count : 0,
                     static_cast<int>(feature_dim / 4), static_cast<uint32_t>(ztable_rows)};
  const int dsmem = kDrawTableBytes + kRprePad + (fill_vec4 > 0 ? kZeroBytes : 0);
  st = launch_dependent(fsa_2hop_draw_kernel, dgrid, kThreadsDraw, dsmem, s, da);
  if (st == FSA_OK) st = pe.mark(3, s);
  if (st != FSA_OK) return st;
  Gather2Args ga{col, x, num_nodes, feature_dim, batch_size, fanout1, fanout2, mbeg,
                 mtake, win2, samples2, out, dchunk, RowShards{}};
  if (xs != nullptr) ga.xs = *xs;
  const int ggrid = grid_for(batch_size);
  // The small CTA only pays when the wide one would not hold every root at
  // once (4 wide CTAs per SM); with fewer roots it only adds item rounds.
  int sms = 0;
  st = sm_count(&sms);
  if (st != FSA_OK) return st;
  const bool small = static_cast<int64_t>(fanout1) * (dchunk / vec) <= kGatherSmallItems &&
                     batch_size > static_cast<int64_t>(sms) * kGatherWidePerSm;
  const int threads = small ? kThreadsGatherSmall : kThreadsGatherWide;
  const bool sh = xs != nullptr;
  switch (vec) {
    case 4: st = launch_gather<4>(sh, small, ggrid, threads, gsmem, s, ga); break;
    case 2: st = launch_gather<2>(sh, small, ggrid, threads, gsmem, s, ga); break;
    default: st = launch_gather<1>(sh, small, ggrid, threads, gsmem, s, ga); break;
  }
  if (st == FSA_OK) st = pe.mark(4, s);
  return st;
}

int fsa_sample_agg_2hop_forward(const int32_t* rowptr, const int32_t* col,
                                int64_t num_nodes, int64_t num_edges,
                                const float* x, int64_t feature_dim,
                                const int32_t* frontier, int64_t batch_size,
                                int64_t batch_offset, int32_t fanout1,
                                int32_t fanout2, uint64_t seed, float* out,
                                int32_t* samples1, int32_t* samples2,
                                void* workspace, size_t workspace_bytes,
                                float* zero_fill, int64_t zero_count,
                                void* stream) {
  return forward_2hop(rowptr, col, num_nodes, num_edges, x, feature_dim, frontier, batch_size,
                      batch_offset, fanout1, fanout2, seed, out, samples1, samples2, workspace,
                      workspace_bytes, zero_fill, zero_count, stream, nullptr);
}

int fsa_sample_agg_2hop_forward_zero_rows(const int32_t* rowptr, const int32_t* col,
                                          int64_t num_nodes, int64_t num_edges,
                                          const float* x, int64_t feature_dim,
                                          const int32_t* frontier, int64_t batch_size,
                                          int64_t batch_offset, int32_t fanout1,
                                          int32_t fanout2, uint64_t seed, float* out,
                                          int32_t* samples1, int32_t* samples2,
                                          void* workspace, size_t workspace_bytes,
                                          float* zero_table, const int32_t* zero_rows,
                                          int64_t zero_rows_count, void* stream) {
  if (zero_rows_count < 0 || (zero_rows_count > 0 && zero_rows == nullptr) ||
      (zero_rows_count > 0 && num_nodes > 0 && feature_dim > 0 && zero_table == nullptr)) {
    return FSA_ERR_INVALID_ARGUMENT;
  }
  return forward_2hop(rowptr, col, num_nodes, num_edges, x, feature_dim, frontier, batch_size,
                      batch_offset, fanout1, fanout2, seed, out, samples1, samples2, workspace,
                      workspace_bytes, nullptr, 0, stream, nullptr, zero_table, zero_rows,
                      zero_rows_count);
}

// Shard table from a host array of device pointers; checks the count, the
// partition covers num_nodes, every base is non-null and aligned to 16
// bytes when the rows are float4 vectors (else to the vector width).
static int make_shards(float* const* bases, int64_t shard_rows, int32_t num_shards,
                       int64_t num_nodes, int64_t feature_dim, RowShards* t) {
  if (bases == nullptr || num_shards < 1 || num_shards > FSA_MAX_SHARDS || shard_rows < 1 ||
      shard_rows > 0x7fffffffLL || num_nodes > shard_rows * num_shards) {
    return FSA_ERR_INVALID_ARGUMENT;
  }
  *t = RowShards{};
  t->rows = shard_rows;
  t->n = num_shards;
  const int vec = feature_dim % 4 == 0 ? 4 : (feature_dim % 2 == 0 ? 2 : 1);
  for (int k = 0; k < num_shards; ++k) {
    if (bases[k] == nullptr || !aligned(bases[k], 4 * vec)) return FSA_ERR_INVALID_ARGUMENT;
    t->base[k] = bases[k];
  }
  return FSA_OK;
}

int fsa_sample_agg_2hop_forward_sharded(const int32_t* rowptr, const int32_t* col,
                                        int64_t num_nodes, int64_t num_edges,
                                        const float* const* x_shards, int64_t shard_rows,
                                        int32_t num_shards, int64_t feature_dim,
                                        const int32_t* frontier, int64_t batch_size,
                                        int64_t batch_offset, int32_t fanout1,
                                        int32_t fanout2, uint64_t seed, float* out,
                                        int32_t* samples1, int32_t* samples2,
                                        void* workspace, size_t workspace_bytes,
                                        float* zero_fill, int64_t zero_count,
                                        void* stream) {
  RowShards t;
  if (num_nodes < 0 || feature_dim < 0) return FSA_ERR_INVALID_ARGUMENT;
  const int st = make_shards(const_cast<float* const*>(x_shards), shard_rows, num_shards,
                             num_nodes, feature_dim, &t);
  if (st != FSA_OK) return st;
  return forward_2hop(rowptr, col, num_nodes, num_edges, t.base[0], feature_dim, frontier,
                      batch_size, batch_offset, fanout1, fanout2, seed, out, samples1, samples2,
                      workspace, workspace_bytes, zero_fill, zero_count, stream, &t);
}

int fsa_sample_agg_2hop_forward_sharded_zero_rows(
    const int32_t* rowptr, const int32_t* col, int64_t num_nodes, int64_t num_edges,
    const float* const* x_shards, int64_t shard_rows, int32_t num_shards, int64_t feature_dim,
    const int32_t* frontier, int64_t batch_size, int64_t batch_offset, int32_t fanout1,
    int32_t fanout2, uint64_t seed, float* out, int32_t* samples1, int32_t* samples2,
    void* workspace, size_t workspace_bytes, float* zero_table, int64_t zero_table_rows,
    const int32_t* zero_rows, int64_t zero_rows_count, void* stream) {
  RowShards t;
  if (num_nodes < 0 || feature_dim < 0 || zero_table_rows < 0 || zero_rows_count < 0 ||
      (zero_rows_count > 0 && zero_rows == nullptr) ||
      (zero_rows_count > 0 && zero_table_rows > 0 && feature_dim > 0 && zero_table == nullptr)) {
    return FSA_ERR_INVALID_ARGUMENT;
  }
  const int st = make_shards(const_cast<float* const*>(x_shards), shard_rows, num_shards,
                             num_nodes, feature_dim, &t);
  if (st != FSA_OK) return st;
  return forward_2hop(rowptr, col, num_nodes, num_edges, t.base[0], feature_dim, frontier,
                      batch_size, batch_offset, fanout1, fanout2, seed, out, samples1, samples2,
                      workspace, workspace_bytes, nullptr, 0, stream, &t, zero_table, zero_rows,
                      zero_rows_count, zero_table_rows);
}

static int backward_2hop(const float* grad_out, const int32_t* samples1,
                         const int32_t* samples2, int64_t batch_size, int64_t feature_dim,
                         int32_t fanout1, int32_t fanout2, float* grad_x, int64_t num_nodes,
                         void* stream, const RowShards* gs) {
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
  Bwd2Args a{RowShards{}, grad_out, samples1, samples2, batch_size, feature_dim,
             fanout1, fanout2, grad_x, num_nodes};
  const int vec = pick_vec(feature_dim, grad_out, grad_x);
  const int smem = 4 * (fanout1 * bwd_slot_stride(fanout2) + 3 * fanout1);
  const int grid = grid_for(batch_size);
  auto s = static_cast<cudaStream_t>(stream);
  if (gs != nullptr) {
    a.gs = *gs;
    switch (vec) {
      case 4: return launch(fsa_2hop_backward_kernel<4, true>, grid, kThreadsBwd, smem, s, a);
      case 2: return launch(fsa_2hop_backward_kernel<2, true>, grid, kThreadsBwd, smem, s, a);
      default: return launch(fsa_2hop_backward_kernel<1, true>, grid, kThreadsBwd, smem, s, a);
    }
  }
  switch (vec) {
    case 4: return launch_dependent(fsa_2hop_backward_kernel<4, false>, grid, kThreadsBwd, smem, s, a);
    case 2: return launch_dependent(fsa_2hop_backward_kernel<2, false>, grid, kThreadsBwd, smem, s, a);
    default: return launch_dependent(fsa_2hop_backward_kernel<1, false>, grid, kThreadsBwd, smem, s, a);
  }
}

int fsa_sample_agg_2hop_backward(const float* grad_out, const int32_t* samples1,
                                 const int32_t* samples2, int64_t batch_size,
                                 int64_t feature_dim, int32_t fanout1,
                                 int32_t fanout2, float* grad_x,
                                 int64_t num_nodes, void* stream) {
  return backward_2hop(grad_out, samples1, samples2, batch_size, feature_dim, fanout1, fanout2,
                       grad_x, num_nodes, stream, nullptr);
}

int fsa_sample_agg_2hop_backward_sharded(const float* grad_out, const int32_t* samples1,
                                         const int32_t* samples2, int64_t batch_size,
                                         int64_t feature_dim, int32_t fanout1,
                                         int32_t fanout2, float* const* grad_shards,
                                         int64_t shard_rows, int32_t num_shards,
                                         int64_t num_nodes, void* stream) {
  RowShards t;
  if (num_nodes < 0 || feature_dim < 0) return FSA_ERR_INVALID_ARGUMENT;
  const int st = make_shards(grad_shards, shard_rows, num_shards, num_nodes, feature_dim, &t);
  if (st != FSA_OK) return st;
  return backward_2hop(grad_out, samples1, samples2, batch_size, feature_dim, fanout1, fanout2,
                       t.base[0], num_nodes, stream, &t);
}

// Workspace of the sort-by-destination backward, in bytes from a 256-byte
// aligned base.
struct WsSort {
  size_t counts, offsets, bsum, skey, sval, slot_valid, nonempty, total;
};

static WsSort ws_sort_layout(int64_t N, int64_t B, int k1, int k2) {
  WsSort l{};
  const size_t E = static_cast<size_t>(B) * k1 * k2;
  const size_t tiles = static_cast<size_t>((N + kSortTile - 1) / kSortTile);
  size_t off = 0;
  l.counts = off;     off = align256(off + 4 * (static_cast<size_t>(N) + 1));
  l.offsets = off;    off = align256(off + 4 * static_cast<size_t>(N));
  l.bsum = off;       off = align256(off + 8 * (tiles + 1));
  l.skey = off;       off = align256(off + 4 * E);
  l.sval = off;       off = align256(off + 4 * E);
  l.slot_valid = off; off = align256(off + 4 * static_cast<size_t>(B) * k1);
  l.nonempty = off;   off = align256(off + 4 * static_cast<size_t>(B));
  l.total = off;
  return l;
}

size_t fsa_sample_agg_2hop_backward_sorted_workspace_size(int64_t num_nodes, int64_t batch_size,
                                                          int32_t fanout1, int32_t fanout2) {
  if (num_nodes < 0 || batch_size <= 0 || fanout1 <= 0 || fanout2 <= 0) return 0;
  return ws_sort_layout(num_nodes, batch_size, fanout1, fanout2).total;
}

int fsa_sample_agg_2hop_backward_sorted(const float* grad_out, const int32_t* samples1,
                                        const int32_t* samples2, int64_t batch_size,
                                        int64_t feature_dim, int32_t fanout1, int32_t fanout2,
                                        float* grad_x, int64_t num_nodes, void* workspace,
                                        size_t workspace_bytes, void* stream) {
  if (fanout1 < 0 || fanout2 < 0 || batch_size < 0 || feature_dim < 0 || num_nodes < 0) {
    return FSA_ERR_INVALID_ARGUMENT;
  }
  if (static_cast<int64_t>(fanout1) + static_cast<int64_t>(fanout1) * fanout2 >
      FSA_MAX_2HOP_ENTRIES) {
    return FSA_ERR_INVALID_ARGUMENT;
  }
  if (batch_size == 0 || fanout1 == 0 || fanout2 == 0 || feature_dim == 0 || num_nodes == 0) {
    return FSA_OK;
  }
  const int64_t E = batch_size * fanout1 * fanout2;
  const WsSort wl = ws_sort_layout(num_nodes, batch_size, fanout1, fanout2);
  if (grad_out == nullptr || samples1 == nullptr || samples2 == nullptr || grad_x == nullptr ||
      workspace == nullptr || workspace_bytes < wl.total || !aligned(workspace, 256) ||
      E > 0x7fffffffLL || num_nodes > 0x7fffffffLL) {
    return FSA_ERR_INVALID_ARGUMENT;
  }
  char* ws = static_cast<char*>(workspace);
  SortBwdArgs a{grad_out, samples1, samples2, batch_size, feature_dim, fanout1, fanout2, grad_x,
                num_nodes,
                reinterpret_cast<int32_t*>(ws + wl.counts),
                reinterpret_cast<int32_t*>(ws + wl.offsets),
                reinterpret_cast<long long*>(ws + wl.bsum),
                reinterpret_cast<int32_t*>(ws + wl.skey),
                reinterpret_cast<int32_t*>(ws + wl.sval),
                reinterpret_cast<int32_t*>(ws + wl.slot_valid),
                reinterpret_cast<int32_t*>(ws + wl.nonempty),
                reinterpret_cast<int32_t*>(ws + wl.counts) + num_nodes};
  auto s = static_cast<cudaStream_t>(stream);
  // counts and the entry total start at zero (int32 zero = float zero bits)
  int st = fsa_fill_zero_f32(reinterpret_cast<float*>(a.counts), num_nodes + 1, stream);
  if (st != FSA_OK) return st;
  st = launch(fsa_2hop_sortbwd_count_kernel, grid_for(batch_size), 256, 0, s, a);
  if (st != FSA_OK) return st;
  const int64_t tiles = (num_nodes + kSortTile - 1) / kSortTile;
  st = launch(fsa_sortbwd_scan_tiles_kernel, static_cast<int>(tiles), kThreadsSort, 0, s, a);
  if (st != FSA_OK) return st;
  fsa_sortbwd_scan_totals_kernel<<<1, kThreadsSort, 0, s>>>(a, tiles);
  st = check_launch();
  if (st != FSA_OK) return st;
  st = launch(fsa_2hop_sortbwd_scatter_kernel, grid_for((E + 255) / 256), 256, 0, s, a);
  if (st != FSA_OK) return st;
  const int vec = pick_vec(feature_dim, grad_out, grad_x);
  const int rgrid = grid_for((E + 255) / 256);
  switch (vec) {
    case 4: return launch(fsa_2hop_sortbwd_reduce_kernel<4>, rgrid, 256, 0, s, a);
    case 2: return launch(fsa_2hop_sortbwd_reduce_kernel<2>, rgrid, 256, 0, s, a);
    default: return launch(fsa_2hop_sortbwd_reduce_kernel<1>, rgrid, 256, 0, s, a);
  }
}

int fsa_fill_zero_f32(float* dst, int64_t count, void* stream) {
  if (count < 0 || (count > 0 && dst == nullptr)) return FSA_ERR_INVALID_ARGUMENT;
  if (count == 0) return FSA_OK;
  auto s = static_cast<cudaStream_t>(stream);
  if (aligned(dst, 16)) {
    const int64_t per_cta = static_cast<int64_t>(kThreadsFill) * kFillVecsPerThread;
    const int64_t grid = ((count >> 2) + per_cta - 1) / per_cta;
    if (grid > 0x7fffffff) return FSA_ERR_INVALID_ARGUMENT;
    fsa_fill_zero_kernel<<<static_cast<unsigned int>(grid > 0 ? grid : 1), kThreadsFill, 0, s>>>(
        dst, count);
  } else {
    int device = 0, sms = 0;
    cudaError_t err = cudaGetDevice(&device);
    if (err == cudaSuccess) {
      err = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
    }
    if (err != cudaSuccess) return cuda_fail(err);
    fsa_fill_zero_scalar_kernel<<<sms * 8, kThreadsFill, 0, s>>>(dst, count);
  }
  return check_launch();
}

int fsa_zero_rows_f32(float* table, int64_t num_rows, int64_t dim, const int32_t* rows,
                      int64_t count, void* stream) {
  if (num_rows < 0 || dim < 0 || count < 0 || (count > 0 && rows == nullptr) ||
      (num_rows > 0 && dim > 0 && count > 0 && table == nullptr)) {
    return FSA_ERR_INVALID_ARGUMENT;
  }
  if (count == 0 || num_rows == 0 || dim == 0) return FSA_OK;
  auto s = static_cast<cudaStream_t>(stream);
  const int vec = pick_vec(dim, table, table);
  const int64_t per_cta = kThreadsFill;  // 32 list entries per warp
  const int grid = grid_for((count + per_cta - 1) / per_cta);
  const bool one = dim / vec <= 32;
  switch (vec * 2 + (one ? 1 : 0)) {
    case 9: fsa_zero_rows_kernel<4, true><<<grid, kThreadsFill, 0, s>>>(table, num_rows, dim, rows, count); break;
    case 8: fsa_zero_rows_kernel<4, false><<<grid, kThreadsFill, 0, s>>>(table, num_rows, dim, rows, count); break;
    case 5: fsa_zero_rows_kernel<2, true><<<grid, kThreadsFill, 0, s>>>(table, num_rows, dim, rows, count); break;
    case 4: fsa_zero_rows_kernel<2, false><<<grid, kThreadsFill, 0, s>>>(table, num_rows, dim, rows, count); break;
    case 3: fsa_zero_rows_kernel<1, true><<<grid, kThreadsFill, 0, s>>>(table, num_rows, dim, rows, count); break;
    default: fsa_zero_rows_kernel<1, false><<<grid, kThreadsFill, 0, s>>>(table, num_rows, dim, rows, count); break;
  }
  return check_launch();
}

int fsa_phase_timing(int enable) {
  std::lock_guard<std::mutex> lock(g_timing_mu);
  if (enable) {
    for (auto& call : g_timing_calls) {
      for (auto e : call) cudaEventDestroy(e);
    }
    g_timing_calls.clear();
  }
  g_timing.store(enable != 0, std::memory_order_relaxed);
  return FSA_OK;
}

int fsa_phase_times(double* ms, int64_t* calls) {
  if (ms == nullptr || calls == nullptr) return FSA_ERR_INVALID_ARGUMENT;
  std::lock_guard<std::mutex> lock(g_timing_mu);
  for (int k = 0; k < kPhases; ++k) ms[k] = 0.0;
  int status = FSA_OK;
  for (auto& call : g_timing_calls) {
    for (int k = 0; k < kPhases && status == FSA_OK; ++k) {
      float t = 0.0F;
      cudaError_t err = cudaEventSynchronize(call[k + 1]);
      if (err == cudaSuccess) err = cudaEventElapsedTime(&t, call[k], call[k + 1]);
      if (err != cudaSuccess) status = cuda_fail(err);
      ms[k] += t;
    }
    for (auto e : call) cudaEventDestroy(e);
  }
  *calls = static_cast<int64_t>(g_timing_calls.size());
  g_timing_calls.clear();
  return status;
}

int fsa_ipc_export(const void* ptr, void* handle, uint64_t* offset) {
  if (ptr == nullptr || handle == nullptr || offset == nullptr) return FSA_ERR_INVALID_ARGUMENT;
  // Base of the allocation that holds ptr (an IPC handle names a whole
  // allocation), through the driver's cuMemGetAddressRange.
  using AddressRange = int (*)(unsigned long long*, size_t*, unsigned long long);
  static AddressRange range = nullptr;
  if (range == nullptr) {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q{};
    const cudaError_t err = cudaGetDriverEntryPoint("cuMemGetAddressRange", &fn,
                                                    cudaEnableDefault, &q);
    if (err != cudaSuccess) return cuda_fail(err);
    if (q != cudaDriverEntryPointSuccess || fn == nullptr) return FSA_ERR_CUDA;
    range = reinterpret_cast<AddressRange>(fn);
  }
  unsigned long long base = 0;
  size_t size = 0;
  if (range(&base, &size, reinterpret_cast<unsigned long long>(ptr)) != 0 || base == 0) {
    return FSA_ERR_CUDA;
  }
  cudaIpcMemHandle_t h;
  const cudaError_t err = cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base));
  if (err != cudaSuccess) return cuda_fail(err);
  static_assert(sizeof(cudaIpcMemHandle_t) == FSA_IPC_HANDLE_BYTES, "IPC handle size");
  memcpy(handle, &h, sizeof(h));
  *offset = reinterpret_cast<unsigned long long>(ptr) - base;
  return FSA_OK;
}

int fsa_ipc_open(const void* handle, int device, void** base) {
  if (handle == nullptr || base == nullptr) return FSA_ERR_INVALID_ARGUMENT;
  int prev = 0;
  cudaError_t err = cudaGetDevice(&prev);
  if (err != cudaSuccess) return cuda_fail(err);
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  err = cudaSetDevice(device);
  // Opened in the accessing device's context: the mapping belongs to that
  // device's address space and peer access to the owner is enabled with it.
  if (err == cudaSuccess) err = cudaIpcOpenMemHandle(base, h, cudaIpcMemLazyEnablePeerAccess);
  const cudaError_t err2 = cudaSetDevice(prev);
  if (err != cudaSuccess) return cuda_fail(err);
  if (err2 != cudaSuccess) return cuda_fail(err2);
  return FSA_OK;
}

int fsa_ipc_close(void* base, int device) {
  if (base == nullptr) return FSA_ERR_INVALID_ARGUMENT;
  int prev = 0;
  cudaError_t err = cudaGetDevice(&prev);
  if (err != cudaSuccess) return cuda_fail(err);
  err = cudaSetDevice(device);
  if (err == cudaSuccess) err = cudaIpcCloseMemHandle(base);
  const cudaError_t err2 = cudaSetDevice(prev);
  if (err != cudaSuccess) return cuda_fail(err);
  if (err2 != cudaSuccess) return cuda_fail(err2);
  return FSA_OK;
}

int fsa_enable_peer_access(int device, int peer) {
  if (device == peer) return FSA_OK;
  int prev = 0;
  cudaError_t err = cudaGetDevice(&prev);
  if (err != cudaSuccess) return cuda_fail(err);
  int can = 0;
  err = cudaDeviceCanAccessPeer(&can, device, peer);
  if (err != cudaSuccess) return cuda_fail(err);
  if (!can) return FSA_ERR_INVALID_ARGUMENT;
  err = cudaSetDevice(device);
  if (err == cudaSuccess) {
    err = cudaDeviceEnablePeerAccess(peer, 0);
    if (err == cudaErrorPeerAccessAlreadyEnabled) {
      cudaGetLastError();  // reset the last-error state this call set
      err = cudaSuccess;
    }
  }
  const cudaError_t err2 = cudaSetDevice(prev);
  if (err != cudaSuccess) return cuda_fail(err);
  if (err2 != cudaSuccess) return cuda_fail(err2);
  return FSA_OK;
}

const char* fsa_status_string(int status) {
  switch (status) {
    case FSA_OK: return "ok";
    case FSA_ERR_INVALID_ARGUMENT: return "invalid argument";
    case FSA_ERR_CUDA: return "CUDA runtime error";
    case FSA_ERR_SCRATCH_LIMIT:
      return "batch needs more than the library's static scratch "
             "(FSA_NOALLOC_SCRATCH_BYTES); use the workspace entry point";
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

// ---------------------------------------------------------------------------
// 2-hop forward on library-owned scratch (no counterpart in the reference)
// ---------------------------------------------------------------------------

// Module-scope scratch for fsa_sample_agg_2hop_forward_noalloc: one copy per
// device, reserved when the module is loaded on that device, never freed.
static __device__ __align__(256) unsigned char g_ws2_scratch[FSA_NOALLOC_SCRATCH_BYTES];

namespace {

constexpr int kScratchDevices = 256;
std::atomic<void*> g_scratch_addr[kScratchDevices];

// Device address of g_ws2_scratch on the current device.  The first call
// per device runs cudaGetSymbolAddress (which also loads the module there);
// later calls read the cached pointer.  The cache is per device ordinal and
// is never refreshed: a device reset (cudaDeviceReset, or anything else that
// destroys the primary context) may reload the module at another address,
// so the entry point is not for use across such a reset.
int scratch_address(void** out) {
  int dev = 0;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return cuda_fail(err);
  const bool cached = dev >= 0 && dev < kScratchDevices;
  if (cached) {
    void* p = g_scratch_addr[dev].load(std::memory_order_acquire);
    if (p != nullptr) {
      *out = p;
      return FSA_OK;
    }
  }
  void* p = nullptr;
  err = cudaGetSymbolAddress(&p, g_ws2_scratch);
  if (err != cudaSuccess) return cuda_fail(err);
  if (p == nullptr) return FSA_ERR_CUDA;
  if (cached) g_scratch_addr[dev].store(p, std::memory_order_release);
  *out = p;
  return FSA_OK;
}

}  // namespace

extern "C" {

int fsa_sample_agg_2hop_forward_noalloc(const int32_t* rowptr, const int32_t* col,
                                        int64_t num_nodes, int64_t num_edges,
                                        const float* x, int64_t feature_dim,
                                        const int32_t* frontier, int64_t batch_size,
                                        int64_t batch_offset, int32_t fanout1,
                                        int32_t fanout2, uint64_t seed, float* out,
                                        int32_t* samples1, int32_t* samples2,
                                        float* zero_fill, int64_t zero_count,
                                        void* stream) {
  // The workspace entry point's argument checks first (host only), so that
  // a call with bad arguments is told so whatever its size.
  const int arg_status =
      check_forward_2hop_args(rowptr, col, num_nodes, num_edges, x, feature_dim, frontier,
                              batch_size, batch_offset, fanout1, fanout2, out, zero_fill,
                              zero_count);
  if (arg_status != FSA_OK) return arg_status;
  const bool work = batch_size > 0 && fanout1 > 0 && fanout2 > 0;
  if (!work) {
    // Nothing to sample: no scratch is used.
    return fsa_sample_agg_2hop_forward(rowptr, col, num_nodes, num_edges, x, feature_dim,
                                       frontier, batch_size, batch_offset, fanout1, fanout2,
                                       seed, out, samples1, samples2, nullptr, 0, zero_fill,
                                       zero_count, stream);
  }
  // Then the size limit, before any CUDA call.  A batch with more roots than
  // scratch bytes cannot fit (8 bytes per root alone); checking that first
  // keeps the layout arithmetic far from overflow.
  if (batch_size > static_cast<int64_t>(FSA_NOALLOC_SCRATCH_BYTES) ||
      ws2_layout(batch_size, fanout1, fanout2, samples1 == nullptr, samples2 == nullptr).total >
          static_cast<size_t>(FSA_NOALLOC_SCRATCH_BYTES)) {
    return FSA_ERR_SCRATCH_LIMIT;
  }
  void* scratch = nullptr;
  const int st = scratch_address(&scratch);
  if (st != FSA_OK) return st;
  return fsa_sample_agg_2hop_forward(rowptr, col, num_nodes, num_edges, x, feature_dim,
                                     frontier, batch_size, batch_offset, fanout1, fanout2, seed,
                                     out, samples1, samples2, scratch,
                                     static_cast<size_t>(FSA_NOALLOC_SCRATCH_BYTES), zero_fill,
                                     zero_count, stream);
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Row-sharded 2-hop backward where the owner computes (no counterpart in the
// reference)
// ---------------------------------------------------------------------------
//
// Every rank publishes its step's saved ids and upstream gradient into its
// exchange region (mapped into every peer over CUDA IPC); after a
// cross-device barrier each rank reads every region and adds the
// contributions to its own rows into its own gradient shard.  Per root a
// rank reads 4 (f1 + f1 f2) + 4 D bytes from each peer instead of sending
// 4 D bytes of red.add per remote contribution.

namespace {

constexpr int64_t kExchangeHeader = 256;
constexpr int kThreadsPublish = 256;
constexpr int kThreadsPull = 128;
constexpr int kPullCtasPerSm = 12;

// Bytes of one root's record: samples1 and samples2 (int32), padded to 16
// bytes, then the upstream gradient row (float), padded to 16 bytes.
__host__ __device__ inline int64_t exchange_ids_bytes(int k1, int k2) {
  return (4 * (static_cast<int64_t>(k1) + static_cast<int64_t>(k1) * k2) + 15) & ~int64_t{15};
}

__host__ __device__ inline int64_t exchange_root_bytes(int k1, int k2, int64_t D) {
  return exchange_ids_bytes(k1, k2) + ((4 * D + 15) & ~int64_t{15});
}

struct PublishArgs {
  unsigned char* region;
  const float* grad_out;
  const int32_t* samples1;
  const int32_t* samples2;
  int64_t batch_size;  // roots published (0 when the call has no contributions)
  int64_t feature_dim;
  int fanout1;
  int fanout2;
  int64_t stride;
  int64_t ids_bytes;
};

// CTA per root (grid-stride): the root's record; block 0 writes the header
// (the number of roots).
template <int V>
__global__ void __launch_bounds__(kThreadsPublish) fsa_exchange_publish_kernel(const PublishArgs a) {
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    *reinterpret_cast<long long*>(a.region) = static_cast<long long>(a.batch_size);
  }
  const int k1 = a.fanout1;
  const int k12 = k1 * a.fanout2;
  const int64_t dvec = a.feature_dim / V;
  for (int64_t b = blockIdx.x; b < a.batch_size; b += gridDim.x) {
    unsigned char* rec = a.region + kExchangeHeader + b * a.stride;
    int32_t* ids = reinterpret_cast<int32_t*>(rec);
    for (int e = threadIdx.x; e < k1; e += blockDim.x) ids[e] = a.samples1[b * k1 + e];
    for (int e = threadIdx.x; e < k12; e += blockDim.x) ids[k1 + e] = a.samples2[b * k12 + e];
    float* g = reinterpret_cast<float*>(rec + a.ids_bytes);
    for (int64_t v = threadIdx.x; v < dvec; v += blockDim.x) {
      store_vec(g + v * V, load_vec<V>(a.grad_out + b * a.feature_dim + v * V));
    }
  }
}

struct PullArgs {
  const unsigned char* regions[FSA_MAX_SHARDS];
  int64_t cap_roots;  // records that fit one region
  int num_shards;
  int shard;          // this device's shard
  float* grad;        // this device's gradient shard
  int64_t shard_rows;
  int64_t num_nodes;
  int64_t feature_dim;
  int fanout1;
  int fanout2;
  int64_t stride;
  int64_t ids_bytes;
  int64_t staged_bytes;  // bytes of each record copied to shared memory (ids, or the whole record)
  int32_t* touched;      // optional [cap_roots * num_shards][k1 * k2]: per unit, the local row
                         // of every owned id, -1 elsewhere
};

// Records up to this size are copied to shared memory whole (ids and
// upstream gradient row in one round of 16-byte loads); longer ones keep
// the gradient row in the region.
constexpr int64_t kPullStageBytes = 16 * 1024;

// Units are (region, root) pairs, regions interleaved so that concurrent
// CTAs read from every peer.  A CTA copies the root's record into shared
// memory, counts each slot's valid ids and the ids this shard owns, counts
// the non-empty slots (fused_sample_agg.cu:229-240) with ballots, then adds
// (grad_out / nonempty) / valid of every owned id's slot into its row with
// red.global.add (fused_sample_agg.cu:241-271).
template <int V>
__global__ void __launch_bounds__(kThreadsPull, kPullCtasPerSm)
    fsa_2hop_backward_pull_kernel(const PullArgs a) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  __shared__ long long s_roots[FSA_MAX_SHARDS];
  const int k1 = a.fanout1;
  const int k2 = a.fanout2;
  int* ids = reinterpret_cast<int*>(smem_raw);  // the record: samples1, samples2 (, gradient)
  int* valid = reinterpret_cast<int*>(smem_raw + a.staged_bytes);  // [k1]
  int* mine = valid + k1;                                          // [k1] owned ids per slot
  int* owned = mine + k1;  // [k1][k2] local rows of the owned ids, slot by slot
  const bool staged_grad = a.staged_bytes == a.stride;
  const int tid = threadIdx.x;
  const int nthreads = blockDim.x;
  const int lane = tid & 31;
  for (int s = tid; s < a.num_shards; s += nthreads) {
    const long long n = *reinterpret_cast<const long long*>(a.regions[s]);
    s_roots[s] = n < 0 ? 0 : (n > a.cap_roots ? a.cap_roots : n);
  }
  __syncthreads();
  const int64_t D = a.feature_dim;
  const int64_t dvec = D / V;
  const int64_t N = a.num_nodes;
  const uint64_t rows = static_cast<uint64_t>(a.shard_rows);
  const int64_t lo = static_cast<int64_t>(a.shard) * a.shard_rows;  // this shard: [lo, lo + rows)
  // unit u = b * num_shards + s, walked with a stride of gridDim.x units:
  // (b, s) advance with a carry instead of a 64-bit division per unit
  const int W = a.num_shards;
  const int64_t step = gridDim.x;
  const int64_t db = step / W;
  const int ds = static_cast<int>(step - db * W);
  int64_t b = blockIdx.x / W;
  int s = static_cast<int>(blockIdx.x - b * W);
  const int k12 = k1 * k2;
  for (; b < a.cap_roots; b += db, s += ds) {
    if (s >= W) {
      s -= W;
      ++b;
      if (b >= a.cap_roots) break;
    }
    int32_t* tl = a.touched != nullptr ? a.touched + (b * W + s) * k12 : nullptr;
    if (b >= s_roots[s]) {  // the same for the whole CTA
      if (tl != nullptr) {
        for (int e = tid; e < k12; e += nthreads) tl[e] = -1;
      }
      continue;
    }
    const unsigned char* rec = a.regions[s] + kExchangeHeader + b * a.stride;
    {
      const int4* src = reinterpret_cast<const int4*>(rec);
      int4* dst = reinterpret_cast<int4*>(smem_raw);
      for (int64_t q = tid; q < a.staged_bytes / 16; q += nthreads) dst[q] = src[q];
    }
    __syncthreads();
    for (int i = tid; i < k1; i += nthreads) {
      int cnt = 0;
      int own = 0;
      for (int j = 0; j < k2; ++j) {
        const int32_t leaf = ids[k1 + i * k2 + j];
        int32_t row = -1;
        if (leaf >= 0) {
          ++cnt;
          if (leaf >= N) {
            flag_status(FSA_STATUS_BAD_NEIGHBOR);
          } else if (static_cast<uint64_t>(leaf - lo) < rows) {
            row = static_cast<int32_t>(leaf - lo);
            owned[i * k2 + own++] = row;
          }
        }
        if (tl != nullptr) tl[i * k2 + j] = row;
      }
      valid[i] = cnt;
      mine[i] = own;
    }
    __syncthreads();
    int nonempty = 0;
    for (int i0 = 0; i0 < k1; i0 += 32) {
      const int i = i0 + lane;
      nonempty += __popc(__ballot_sync(0xffffffffU, i < k1 && ids[i] >= 0 && valid[i] > 0));
    }
    if (nonempty > 0) {
      const float ne = static_cast<float>(nonempty);
      const float* go = reinterpret_cast<const float*>(
          (staged_grad ? static_cast<const unsigned char*>(smem_raw) : rec) + a.ids_bytes);
      if (staged_grad) {
        // grad_out / nonempty once per element in the staged copy (the
        // same rounding as in (g / nonempty) / valid below)
        float* gs = reinterpret_cast<float*>(smem_raw + a.ids_bytes);
        for (int64_t f = tid; f < D; f += nthreads) gs[f] = gs[f] / ne;
        __syncthreads();
      }
      const float pre = staged_grad ? 1.0F : ne;
      const int dv = static_cast<int>(dvec);  // k1 * dvec < 2^31 (checked on the host)
      for (int it = tid; it < k1 * dv; it += nthreads) {
        const int i = it / dv;
        if (mine[i] == 0) continue;
        const int v = it - i * dv;
        VecF<V> g = load_vec<V>(go + v * V);
        const float vc = static_cast<float>(valid[i]);
#pragma unroll
        for (int c = 0; c < V; ++c) g.v[c] = (staged_grad ? g.v[c] : g.v[c] / pre) / vc;
        const int* rows_i = owned + i * k2;
        for (int m = 0; m < mine[i]; ++m) {
          red_add<V>(a.grad + static_cast<int64_t>(rows_i[m]) * D + v * V, g);
        }
      }
    }
    __syncthreads();
  }
}

// Per-warp shared memory up to which a warp takes a unit alone
// (fsa_2hop_backward_pull_warp_kernel): no CTA barriers between a unit's
// record load, counts and additions, and every resident warp has a record
// in flight.
constexpr int64_t kPullWarpSliceBytes = 4096;

// A warp's shared memory in fsa_2hop_backward_pull_warp_kernel: the staged
// record, then valid / owned counts and the owned slots ([3][k1] int) and
// the owned ids' local rows ([k1][k2] int), padded to 16 bytes.
__host__ __device__ inline int64_t pull_warp_slice(int64_t staged, int k1, int k2) {
  return staged + 16 * ((4 * (3 * static_cast<int64_t>(k1) + static_cast<int64_t>(k1) * k2) + 15) / 16);
}

// The same additions as fsa_2hop_backward_pull_kernel with one warp per
// (region, root) unit: the warp copies the whole record into its own slice
// of shared memory, lane i counts slot i, the warp counts the non-empty
// slots with ballots and its lanes add the items of the owned ids.
template <int V>
__global__ void __launch_bounds__(kThreadsPull, kPullCtasPerSm)
    fsa_2hop_backward_pull_warp_kernel(const PullArgs a) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  __shared__ long long s_roots[FSA_MAX_SHARDS];
  const int k1 = a.fanout1;
  const int k2 = a.fanout2;
  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int warp = tid >> 5;
  const int nwarps = static_cast<int>(blockDim.x >> 5);
  for (int s = tid; s < a.num_shards; s += blockDim.x) {
    const long long n = *reinterpret_cast<const long long*>(a.regions[s]);
    s_roots[s] = n < 0 ? 0 : (n > a.cap_roots ? a.cap_roots : n);
  }
  __syncthreads();
  const int64_t slice = pull_warp_slice(a.staged_bytes, k1, k2);
  unsigned char* mem = smem_raw + warp * slice;
  const int* ids = reinterpret_cast<const int*>(mem);  // samples1, samples2, gradient row
  int* valid = reinterpret_cast<int*>(mem + a.staged_bytes);  // [k1]
  int* mine = valid + k1;                                     // [k1] owned ids per slot
  int* oslot = mine + k1;                                     // [k1] slots with owned ids
  int* owned = oslot + k1;  // [k1][k2] local rows of the owned ids, slot by slot
  float* go = reinterpret_cast<float*>(mem + a.ids_bytes);  // the staged gradient row
  const int dvec = static_cast<int>(a.feature_dim / V);
  const int64_t D = a.feature_dim;
  const int64_t N = a.num_nodes;
  const uint64_t rows = static_cast<uint64_t>(a.shard_rows);
  const int64_t lo = static_cast<int64_t>(a.shard) * a.shard_rows;  // this shard: [lo, lo + rows)
  // unit u = b * num_shards + s, walked with a stride of gridDim.x * nwarps
  // units: (b, s) advance with a carry instead of a 64-bit division per unit
  const int W = a.num_shards;
  const int64_t step = static_cast<int64_t>(gridDim.x) * nwarps;
  const int64_t db = step / W;
  const int ds = static_cast<int>(step - db * W);
  const int64_t u0 = static_cast<int64_t>(blockIdx.x) * nwarps + warp;
  int64_t b = u0 / W;
  int s = static_cast<int>(u0 - b * W);
  const int k12 = k1 * k2;
  for (; b < a.cap_roots; b += db, s += ds) {
    if (s >= W) {
      s -= W;
      ++b;
      if (b >= a.cap_roots) break;
    }
    int32_t* tl = a.touched != nullptr ? a.touched + (b * W + s) * k12 : nullptr;
    if (b >= s_roots[s]) {  // the same for the whole warp
      if (tl != nullptr) {
        for (int e = lane; e < k12; e += 32) tl[e] = -1;
      }
      continue;
    }
    {
      const int4* src =
          reinterpret_cast<const int4*>(a.regions[s] + kExchangeHeader + b * a.stride);
      int4* dst = reinterpret_cast<int4*>(mem);
      for (int q = lane; q < static_cast<int>(a.staged_bytes / 16); q += 32) dst[q] = src[q];
    }
    for (int i = lane; i < k1; i += 32) {
      valid[i] = 0;
      mine[i] = 0;
    }
    __syncwarp();
    // every lane takes entries lane, lane + 32, ...: (slot, position)
    // advance by (32 / k2, 32 % k2) with a carry; counts and owned rows by
    // shared-memory atomics (the order of a slot's owned rows is free)
    {
      const int di = 32 / k2;
      const int dj = 32 - di * k2;
      int i = lane / k2;
      int j = lane - i * k2;
      for (int e = lane; e < k12; e += 32) {
        const int32_t leaf = ids[k1 + e];
        int32_t row = -1;
        if (leaf >= 0) {
          atomicAdd(&valid[i], 1);
          if (leaf >= N) {
            flag_status(FSA_STATUS_BAD_NEIGHBOR);
          } else if (static_cast<uint64_t>(leaf - lo) < rows) {
            row = static_cast<int32_t>(leaf - lo);
            owned[i * k2 + atomicAdd(&mine[i], 1)] = row;
          }
        }
        if (tl != nullptr) tl[e] = row;
        i += di;
        j += dj;
        if (j >= k2) {
          j -= k2;
          ++i;
        }
      }
    }
    __syncwarp();
    int nonempty = 0;
    int nowned = 0;  // slots with owned ids, listed in oslot
    for (int i0 = 0; i0 < k1; i0 += 32) {
      const int i = i0 + lane;
      const int cnt = i < k1 ? valid[i] : 0;
      const int own = i < k1 ? mine[i] : 0;
      nonempty += __popc(__ballot_sync(0xffffffffU, i < k1 && ids[i] >= 0 && cnt > 0));
      const unsigned has = __ballot_sync(0xffffffffU, own > 0);
      if (own > 0) oslot[nowned + __popc(has & ((1U << lane) - 1U))] = i;
      nowned += __popc(has);
    }
    __syncwarp();
    if (nonempty > 0 && nowned > 0) {
      // grad_out / nonempty once per element (the staged row is this warp's
      // copy), then / valid per owned slot: the same two roundings as
      // (g / nonempty) / valid.
      const float ne = static_cast<float>(nonempty);
      for (int f = lane; f < static_cast<int>(D); f += 32) go[f] = go[f] / ne;
      __syncwarp();
      for (int t = 0; t < nowned; ++t) {
        const int i = oslot[t];
        const float vc = static_cast<float>(valid[i]);
        const int own = mine[i];
        const int* rows_i = owned + i * k2;
        for (int v = lane; v < dvec; v += 32) {
          VecF<V> g = load_vec<V>(go + v * V);
#pragma unroll
          for (int c = 0; c < V; ++c) g.v[c] = g.v[c] / vc;
          for (int m = 0; m < own; ++m) {
            red_add<V>(a.grad + static_cast<int64_t>(rows_i[m]) * D + v * V, g);
          }
        }
      }
    }
    __syncwarp();
  }
}

bool exchange_args_ok(int64_t batch_size, int32_t fanout1, int32_t fanout2, int64_t feature_dim) {
  return batch_size >= 0 && fanout1 >= 0 && fanout2 >= 0 && feature_dim >= 0 &&
         static_cast<int64_t>(fanout1) + static_cast<int64_t>(fanout1) * fanout2 <=
             FSA_MAX_2HOP_ENTRIES &&
         feature_dim <= (int64_t{1} << 40) && batch_size <= (int64_t{1} << 40);
}

}  // namespace

extern "C" {

size_t fsa_exchange_bytes(int64_t batch_size, int32_t fanout1, int32_t fanout2,
                          int64_t feature_dim) {
  if (!exchange_args_ok(batch_size, fanout1, fanout2, feature_dim)) return 0;
  return static_cast<size_t>(kExchangeHeader +
                             batch_size * exchange_root_bytes(fanout1, fanout2, feature_dim));
}

int fsa_sharded_publish_2hop(void* exchange, size_t exchange_bytes, const float* grad_out,
                             const int32_t* samples1, const int32_t* samples2,
                             int64_t batch_size, int64_t feature_dim, int32_t fanout1,
                             int32_t fanout2, void* stream) {
  if (!exchange_args_ok(batch_size, fanout1, fanout2, feature_dim)) {
    return FSA_ERR_INVALID_ARGUMENT;
  }
  if (exchange == nullptr || !aligned(exchange, 256) ||
      exchange_bytes < fsa_exchange_bytes(batch_size, fanout1, fanout2, feature_dim)) {
    return FSA_ERR_INVALID_ARGUMENT;
  }
  const bool work = batch_size > 0 && fanout1 > 0 && fanout2 > 0 && feature_dim > 0;
  if (work && (grad_out == nullptr || samples1 == nullptr || samples2 == nullptr)) {
    return FSA_ERR_INVALID_ARGUMENT;
  }
  const int64_t stride = exchange_root_bytes(fanout1, fanout2, feature_dim);
  const PublishArgs pa{static_cast<unsigned char*>(exchange), grad_out, samples1, samples2,
                       work ? batch_size : 0, feature_dim, fanout1, fanout2, stride,
                       exchange_ids_bytes(fanout1, fanout2)};
  const int grid = grid_for(work ? batch_size : 1);
  auto s = static_cast<cudaStream_t>(stream);
  if (feature_dim % 4 == 0 && aligned(grad_out, 16)) {
    return launch(fsa_exchange_publish_kernel<4>, grid, kThreadsPublish, 0, s, pa);
  }
  return launch(fsa_exchange_publish_kernel<1>, grid, kThreadsPublish, 0, s, pa);
}

int fsa_sample_agg_2hop_backward_sharded_pull(const void* const* exchanges,
                                              size_t exchange_bytes, int32_t num_shards,
                                              int32_t shard, float* grad_shard,
                                              int64_t shard_rows, int64_t num_nodes,
                                              int64_t feature_dim, int32_t fanout1,
                                              int32_t fanout2, int32_t* touched_rows,
                                              int64_t touched_capacity, void* stream) {
  if (!exchange_args_ok(0, fanout1, fanout2, feature_dim) || exchanges == nullptr ||
      num_shards < 1 || num_shards > FSA_MAX_SHARDS || shard < 0 || shard >= num_shards ||
      shard_rows < 1 || shard_rows > 0x7fffffffLL || num_nodes < 0 ||
      num_nodes > shard_rows * num_shards || exchange_bytes < static_cast<size_t>(kExchangeHeader)) {
    return FSA_ERR_INVALID_ARGUMENT;
  }
  PullArgs pa{};
  for (int k = 0; k < num_shards; ++k) {
    if (exchanges[k] == nullptr || !aligned(exchanges[k], 256)) return FSA_ERR_INVALID_ARGUMENT;
    pa.regions[k] = static_cast<const unsigned char*>(exchanges[k]);
  }
  if (fanout1 == 0 || fanout2 == 0 || feature_dim == 0) return FSA_OK;
  if (grad_shard == nullptr || !aligned(grad_shard, 4)) return FSA_ERR_INVALID_ARGUMENT;
  // the kernels index a root's (slot, element) items in 32 bits
  if (static_cast<int64_t>(fanout1) * feature_dim >= 0x7fffffffLL) return FSA_ERR_INVALID_ARGUMENT;
  const int64_t stride = exchange_root_bytes(fanout1, fanout2, feature_dim);
  pa.cap_roots = (static_cast<int64_t>(exchange_bytes) - kExchangeHeader) / stride;
  if (pa.cap_roots == 0) return FSA_OK;
  if (touched_rows != nullptr &&
      touched_capacity < pa.cap_roots * num_shards * fanout1 * static_cast<int64_t>(fanout2)) {
    return FSA_ERR_INVALID_ARGUMENT;
  }
  pa.touched = touched_rows;
  pa.num_shards = num_shards;
  pa.shard = shard;
  pa.grad = grad_shard;
  pa.shard_rows = shard_rows;
  pa.num_nodes = num_nodes;
  pa.feature_dim = feature_dim;
  pa.fanout1 = fanout1;
  pa.fanout2 = fanout2;
  pa.stride = stride;
  pa.ids_bytes = exchange_ids_bytes(fanout1, fanout2);
  pa.staged_bytes = stride <= kPullStageBytes ? stride : pa.ids_bytes;
  int sms = 0;
  const int st = sm_count(&sms);
  if (st != FSA_OK) return st;
  const int64_t units = pa.cap_roots * num_shards;
  const int64_t resident = static_cast<int64_t>(sms) * kPullCtasPerSm;
  const int grid = grid_for(units < resident ? units : resident);
  auto s = static_cast<cudaStream_t>(stream);
  // The records' gradient rows are 16-byte aligned; the shard's rows are
  // when feature_dim % 4 == 0 and its base is.
  const int vec = feature_dim % 4 == 0 && aligned(grad_shard, 16)  ? 4
                  : feature_dim % 2 == 0 && aligned(grad_shard, 8) ? 2
                                                                    : 1;
  const int64_t slice = pull_warp_slice(stride, fanout1, fanout2);
  const int nwarps_sm = kPullCtasPerSm * (kThreadsPull / 32);
  if (stride <= kPullStageBytes && slice <= kPullWarpSliceBytes &&
      units >= static_cast<int64_t>(sms) * nwarps_sm) {
    // a warp per unit, when the units fill every resident warp
    pa.staged_bytes = stride;
    const int nwarps = kThreadsPull / 32;
    const int64_t wunits = (units + nwarps - 1) / nwarps;
    const int wgrid = grid_for(wunits < resident ? wunits : resident);
    const int wsmem = static_cast<int>(nwarps * slice);
    switch (vec) {
      case 4: return launch(fsa_2hop_backward_pull_warp_kernel<4>, wgrid, kThreadsPull, wsmem, s, pa);
      case 2: return launch(fsa_2hop_backward_pull_warp_kernel<2>, wgrid, kThreadsPull, wsmem, s, pa);
      default: return launch(fsa_2hop_backward_pull_warp_kernel<1>, wgrid, kThreadsPull, wsmem, s, pa);
    }
  }
  const int smem =
      static_cast<int>(pa.staged_bytes) + 4 * (2 * fanout1 + fanout1 * fanout2);
  switch (vec) {
    case 4: return launch(fsa_2hop_backward_pull_kernel<4>, grid, kThreadsPull, smem, s, pa);
    case 2: return launch(fsa_2hop_backward_pull_kernel<2>, grid, kThreadsPull, smem, s, pa);
    default: return launch(fsa_2hop_backward_pull_kernel<1>, grid, kThreadsPull, smem, s, pa);
  }
}

}  // extern "C"
