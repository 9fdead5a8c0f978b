/*
 * fsa_sm100.h - C ABI of the B200 (sm_100a) fused reservoir-sample + mean
 * aggregate operator (libfsa_sm100.so).
 *
 * Each compute entry point replaces one host launcher of the reference
 * (declared at fuseop/binding.cpp:57-72, defined at
 * fuseop/fused_sample_agg.cu:275-326).  Differences from those launchers:
 *   - plain C types only; the stream is passed as `void*` (a cudaStream_t);
 *   - an int status is returned instead of throwing (0 = FSA_OK);
 *   - `num_nodes` / `num_edges` are passed so every root, row and neighbour
 *     id is bounds-checked on the device (bad ids are skipped and flagged in
 *     the per-device status word instead of being dereferenced);
 *   - `batch_offset` is added to the batch index that seeds first-hop rows,
 *     so a slice [offset, offset+B) of a larger batch draws exactly the
 *     samples the whole batch would (multi-GPU root partitioning).
 *
 * Layouts: rowptr int32[num_nodes+1], col int32[num_edges] (CSR, neighbour
 * order within a row is significant), x float32[num_nodes][feature_dim]
 * row-major, frontier int32[batch_size].  All pointers are device pointers.
 * Calls are asynchronous and stream-ordered; nothing is allocated (scratch
 * comes from a caller-provided workspace where a call needs one) and the
 * host is never synchronised (except fsa_device_status).  The 2-hop draw,
 * gather and backward kernels are launched as programmatic dependents
 * (cudaLaunchAttributeProgrammaticStreamSerialization) of the kernel before
 * them in the stream: they may be scheduled while it finishes, and every
 * read of earlier work waits for it (griddepcontrol.wait), so the stream
 * order a caller sees is unchanged.
 */
#ifndef FSA_SM100_H_
#define FSA_SM100_H_

#include <stddef.h>
#include <stdint.h>

#if defined(FSA_BUILD_SHARED)
#define FSA_API __attribute__((visibility("default")))
#else
#define FSA_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes. */
#define FSA_OK 0
#define FSA_ERR_INVALID_ARGUMENT 1 /* a size / fanout / pointer check failed */
#define FSA_ERR_CUDA 2             /* a CUDA runtime call failed; see fsa_last_cuda_error */
#define FSA_ERR_SCRATCH_LIMIT 3    /* call too large for FSA_NOALLOC_SCRATCH_BYTES */

/* Limits, same values as the reference (fuseop/binding.cpp:13-14). */
#define FSA_MAX_FANOUT_1HOP 1024
#define FSA_MAX_2HOP_ENTRIES 12000 /* fanout1 + fanout1 * fanout2 */
#define FSA_NOALLOC_SCRATCH_BYTES 4194304 /* scratch of the _noalloc entry point */
#define FSA_MAX_SHARDS 64 /* feature / gradient row shards of the _sharded entry points */
#define FSA_IPC_HANDLE_BYTES 64

/* Bits of the per-device status word (fsa_device_status). */
#define FSA_STATUS_BAD_ROOT 0x1u     /* frontier id outside [0, num_nodes) */
#define FSA_STATUS_BAD_ROW 0x2u      /* rowptr[r] .. rowptr[r+1] not within [0, num_edges] */
#define FSA_STATUS_BAD_NEIGHBOR 0x4u /* sampled id outside [0, num_nodes) */

/*
 * 1-hop forward.  Replaces fused_sample_agg_cuda_forward
 * (fuseop/fused_sample_agg.cu:275-289; kernel :58-104).
 * out[b,:] = mean of x over the reservoir sample of row(frontier[b]).
 * samples int32[batch_size][fanout] (-1 padded) and takes int32[batch_size]
 * are optional (NULL = not written).  batch_size == 0 or fanout == 0 is a
 * no-op (the caller owns zero-initialisation of outputs in that case).
 */
FSA_API int fsa_sample_agg_forward(const int32_t* rowptr, const int32_t* col,
                           int64_t num_nodes, int64_t num_edges,
                           const float* x, int64_t feature_dim,
                           const int32_t* frontier, int64_t batch_size,
                           int64_t batch_offset, int32_t fanout, uint64_t seed,
                           float* out, int32_t* samples, int32_t* takes,
                           void* stream);

/*
 * 1-hop backward (saved-index replay).  Replaces
 * fused_sample_agg_cuda_backward (fuseop/fused_sample_agg.cu:291-301;
 * kernel :106-132).  grad_x[samples[b,i],:] += grad_out[b,:] / takes[b] for
 * i < takes[b].  grad_x float32[num_nodes][feature_dim] must be zeroed (or
 * hold a gradient to accumulate into) by the caller, e.g. with
 * fsa_fill_zero_f32.
 */
FSA_API int fsa_sample_agg_backward(const int32_t* samples, const int32_t* takes,
                            const float* grad_out, int64_t batch_size,
                            int64_t feature_dim, int32_t fanout, float* grad_x,
                            int64_t num_nodes, void* stream);

/*
 * 2-hop forward.  Replaces fused_sample_agg_2hop_cuda_forward
 * (fuseop/fused_sample_agg.cu:303-315; kernel :134-214).
 * out[b,:] = mean over non-empty first-hop slots i of (mean over valid
 * second-hop slots j of x[samples2[b,i,j],:]).  samples1
 * int32[batch_size][fanout1] and samples2 int32[batch_size][fanout1][fanout2]
 * are optional (NULL = not written).
 *
 * Unlike the reference launcher this one needs a device workspace (the
 * second-hop row table, per-row initial states and draw-group prefixes,
 * plus the id buffers that are not requested as outputs): at least
 * fsa_sample_agg_2hop_workspace_size(...) bytes, 256-byte aligned, owned by
 * the caller and not used by anything else until the call's work on `stream`
 * has finished.  Its contents need no initialisation.
 *
 * zero_fill / zero_count (optional, NULL / 0 = none): a float buffer to set
 * to zero as part of the call -- typically the dense feature gradient the
 * backward will scatter into (what the reference allocates with at::zeros,
 * fuseop/binding.cpp:220).  The sampling kernel is bound by integer issue
 * and the fill by HBM writes, so the fill is interleaved into it and costs
 * little extra time.  The buffer is zero when the call's work on `stream`
 * has finished.
 */
FSA_API size_t fsa_sample_agg_2hop_workspace_size(int64_t batch_size, int32_t fanout1,
                                                  int32_t fanout2, int has_samples1,
                                                  int has_samples2);

FSA_API int fsa_sample_agg_2hop_forward(const int32_t* rowptr, const int32_t* col,
                                        int64_t num_nodes, int64_t num_edges,
                                        const float* x, int64_t feature_dim,
                                        const int32_t* frontier, int64_t batch_size,
                                        int64_t batch_offset, int32_t fanout1,
                                        int32_t fanout2, uint64_t seed, float* out,
                                        int32_t* samples1, int32_t* samples2,
                                        void* workspace, size_t workspace_bytes,
                                        float* zero_fill, int64_t zero_count,
                                        void* stream);

/*
 * The 2-hop forward that also zeroes listed rows of a table -- the
 * row-sparse counterpart of zero_fill above, for a feature gradient kept
 * across steps (no counterpart in the reference, whose backward zero-fills a
 * fresh N x D gradient every call, fuseop/binding.cpp:137, :220).  Same
 * arguments and results as fsa_sample_agg_2hop_forward, with zero_fill /
 * zero_count replaced by zero_table float32[num_nodes][feature_dim] and the
 * row list zero_rows int32[zero_rows_count] (typically the samples2 of the
 * previous steps; entries outside [0, num_nodes) such as -1 padding are
 * skipped).  The rows are zero when the call's work on `stream` has
 * finished.  When feature_dim is a multiple of 4 (at most 128) and
 * zero_table is 16-byte aligned, the rows are zeroed inside the sampling
 * kernel, whose draws leave the memory system idle; otherwise
 * fsa_zero_rows_f32 runs first.  zero_table must not be read by this call's
 * forward (it is the gradient, not x).
 */
FSA_API int fsa_sample_agg_2hop_forward_zero_rows(const int32_t* rowptr, const int32_t* col,
                                                  int64_t num_nodes, int64_t num_edges,
                                                  const float* x, int64_t feature_dim,
                                                  const int32_t* frontier, int64_t batch_size,
                                                  int64_t batch_offset, int32_t fanout1,
                                                  int32_t fanout2, uint64_t seed, float* out,
                                                  int32_t* samples1, int32_t* samples2,
                                                  void* workspace, size_t workspace_bytes,
                                                  float* zero_table, const int32_t* zero_rows,
                                                  int64_t zero_rows_count, void* stream);

/*
 * 2-hop forward on library-owned scratch.  No counterpart in the reference:
 * the reference launcher (fuseop/fused_sample_agg.cu:303-315) needs no
 * scratch, and the workspace entry point above takes it from the caller.
 *
 * Same arguments and results as fsa_sample_agg_2hop_forward, without
 * workspace / workspace_bytes.  For callers that cannot allocate device
 * memory at call time: a C / cgo / JNI host that holds only raw device
 * pointers handed over by another runtime and no allocator of its own, or a
 * serving loop that must not call cudaMalloc / cudaFree (both synchronise
 * the whole device) nor route through a framework allocator.  The call
 * allocates nothing; its scratch is a static device array of
 * FSA_NOALLOC_SCRATCH_BYTES (4 MiB) per device, reserved when the library's
 * device code is loaded on that device.
 *
 * Limit: fsa_sample_agg_2hop_workspace_size(batch_size, fanout1, fanout2,
 * samples1 != NULL, samples2 != NULL) must not exceed
 * FSA_NOALLOC_SCRATCH_BYTES, else the call returns FSA_ERR_SCRATCH_LIMIT
 * before any CUDA call.  That covers 1,024 roots at fanouts 15 x 10 (about
 * 1.1 MB without caller id buffers) and up to about 9,500 roots at 15 x 10
 * when samples1 and samples2 are given.
 *
 * The first call on a device does set-up: cudaGetSymbolAddress of the
 * scratch (which loads the module on that device if needed), checked and
 * then cached per device.  Make that first call before any stream capture.
 * The cached address is not refreshed after a device reset (cudaDeviceReset
 * or another end of the primary context), which is unsupported here.
 *
 * Arguments are checked as by the workspace entry point first
 * (FSA_ERR_INVALID_ARGUMENT), then the size limit.
 * Nothing in the scratch needs to start at zero: the call's first kernel
 * writes every word the later kernels read.
 *
 * All calls on one device share the one scratch array, so calls whose work
 * overlaps on the device race and give wrong results: issue them on one
 * stream, or order them with events.
 */
FSA_API int fsa_sample_agg_2hop_forward_noalloc(const int32_t* rowptr, const int32_t* col,
                                                int64_t num_nodes, int64_t num_edges,
                                                const float* x, int64_t feature_dim,
                                                const int32_t* frontier, int64_t batch_size,
                                                int64_t batch_offset, int32_t fanout1,
                                                int32_t fanout2, uint64_t seed, float* out,
                                                int32_t* samples1, int32_t* samples2,
                                                float* zero_fill, int64_t zero_count,
                                                void* stream);

/*
 * 2-hop forward and backward on row-sharded features: the multi-GPU mode
 * for feature tables larger than one device's memory.  No
 * counterpart in the reference, whose binding requires the whole table on
 * one device (fuseop/binding.cpp:35).
 *
 * Feature row r (0 <= r < num_nodes) lives in shard r / shard_rows at local
 * row r % shard_rows; x_shards / grad_shards are HOST arrays of num_shards
 * (<= FSA_MAX_SHARDS) device pointers valid in the calling process -- the
 * local shard and the other devices' shards mapped over NVLink (CUDA IPC).
 * Each shard holds shard_rows rows of feature_dim floats (the last may be
 * shorter as long as num_nodes <= shard_rows * num_shards); bases aligned
 * to 16 bytes when feature_dim % 4 == 0 (8 when % 2 == 0).  The graph
 * (rowptr, col) is whole on every device.  Everything else is as in
 * fsa_sample_agg_2hop_forward / _backward: the same ids and outputs as the
 * unsharded call on the concatenated table; the backward adds into the
 * owning shard's gradient (atomics over NVLink for remote rows).
 *
 * Ordering across devices is the caller's: the shards must not change
 * during the forward, and every gradient shard must be zeroed (e.g. by its
 * own forward's zero_fill) before any device's backward starts.
 */
FSA_API int fsa_sample_agg_2hop_forward_sharded(const int32_t* rowptr, const int32_t* col,
                                                int64_t num_nodes, int64_t num_edges,
                                                const float* const* x_shards, int64_t shard_rows,
                                                int32_t num_shards, int64_t feature_dim,
                                                const int32_t* frontier, int64_t batch_size,
                                                int64_t batch_offset, int32_t fanout1,
                                                int32_t fanout2, uint64_t seed, float* out,
                                                int32_t* samples1, int32_t* samples2,
                                                void* workspace, size_t workspace_bytes,
                                                float* zero_fill, int64_t zero_count,
                                                void* stream);

FSA_API int fsa_sample_agg_2hop_backward_sharded(const float* grad_out, const int32_t* samples1,
                                                 const int32_t* samples2, int64_t batch_size,
                                                 int64_t feature_dim, int32_t fanout1,
                                                 int32_t fanout2, float* const* grad_shards,
                                                 int64_t shard_rows, int32_t num_shards,
                                                 int64_t num_nodes, void* stream);

/*
 * Row-sharded 2-hop backward where each device computes its own rows'
 * gradient ("owner computes"; no counterpart in the reference).  The
 * alternative to fsa_sample_agg_2hop_backward_sharded, which sends one
 * red.add per remote contribution over NVLink: here every device first
 * publishes its saved ids and upstream gradient into its EXCHANGE REGION
 * (fsa_sharded_publish_2hop), the caller orders the devices (every region
 * written before any device reads one), and then every device reads all
 * regions -- its own and its peers', mapped over CUDA IPC -- and adds the
 * contributions to the rows it owns into its own gradient shard
 * (fsa_sample_agg_2hop_backward_sharded_pull).  Per root a device reads
 * 4 (fanout1 + fanout1 fanout2) + 4 feature_dim bytes from each peer.
 *
 * Region layout (exchange_bytes each, the same size on every device, base
 * aligned to 256 bytes): an int64 root count at offset 0, then from byte
 * 256 one record per root of fsa_exchange_bytes(1, ...) - 256 bytes:
 * samples1[fanout1] and samples2[fanout1][fanout2] (int32), padded to 16
 * bytes, then grad_out[feature_dim] (float), padded to 16 bytes.
 * fsa_exchange_bytes(batch_size, ...) is the region size a batch needs (0
 * for invalid arguments).  The pull call adds into grad_shard (rows
 * [shard * shard_rows, ...), pre-zeroed or accumulating), the same result
 * as the push entry point up to the order of the additions.  The caller
 * orders the devices again before any region is rewritten.
 */
FSA_API size_t fsa_exchange_bytes(int64_t batch_size, int32_t fanout1, int32_t fanout2,
                                  int64_t feature_dim);
FSA_API int fsa_sharded_publish_2hop(void* exchange, size_t exchange_bytes, const float* grad_out,
                                     const int32_t* samples1, const int32_t* samples2,
                                     int64_t batch_size, int64_t feature_dim, int32_t fanout1,
                                     int32_t fanout2, void* stream);
FSA_API int fsa_sample_agg_2hop_backward_sharded_pull(const void* const* exchanges,
                                                      size_t exchange_bytes, int32_t num_shards,
                                                      int32_t shard, float* grad_shard,
                                                      int64_t shard_rows, int64_t num_nodes,
                                                      int64_t feature_dim, int32_t fanout1,
                                                      int32_t fanout2, int32_t* touched_rows,
                                                      int64_t touched_capacity, void* stream);

/*
 * Persistent gradient shards for the owner-computed backward.  With
 * touched_rows non-NULL (touched_capacity >= records per region *
 * num_shards * fanout1 * fanout2 int32, records per region =
 * (exchange_bytes - 256) / (fsa_exchange_bytes(1, ...) - 256)), the pull
 * call also writes, for every (region, root) unit, the local row of each id
 * it added (-1 for the others): the rows of grad_shard this step touched.
 * fsa_sample_agg_2hop_forward_sharded_zero_rows is the sharded forward
 * that, instead of zero-filling the whole gradient shard, zeroes the rows
 * listed in zero_rows (entries outside [0, zero_table_rows) skipped) --
 * inside its sampling kernel when the rows are whole float4 vectors of at
 * most 32 -- so that a shard kept across steps holds only the current
 * step's gradient after its backward.
 */
FSA_API int fsa_sample_agg_2hop_forward_sharded_zero_rows(
    const int32_t* rowptr, const int32_t* col, int64_t num_nodes, int64_t num_edges,
    const float* const* x_shards, int64_t shard_rows, int32_t num_shards, int64_t feature_dim,
    const int32_t* frontier, int64_t batch_size, int64_t batch_offset, int32_t fanout1,
    int32_t fanout2, uint64_t seed, float* out, int32_t* samples1, int32_t* samples2,
    void* workspace, size_t workspace_bytes, float* zero_table, int64_t zero_table_rows,
    const int32_t* zero_rows, int64_t zero_rows_count, void* stream);

/*
 * Sharing shards between processes (one process per GPU), no counterpart in
 * the reference.  fsa_ipc_export writes the CUDA IPC handle
 * (FSA_IPC_HANDLE_BYTES bytes) of the allocation holding `ptr` and ptr's
 * byte offset in it.  fsa_ipc_open maps a handle from another process into
 * `device`'s address space (the device whose kernels will access it; peer
 * access to the owner is enabled with the mapping) and returns the
 * allocation's base there: the shard is base + offset.  fsa_ipc_close
 * unmaps it.  The exporting process must keep the allocation alive until
 * every importer has closed it.
 */
FSA_API int fsa_ipc_export(const void* ptr, void* handle, uint64_t* offset);
FSA_API int fsa_ipc_open(const void* handle, int device, void** base);
FSA_API int fsa_ipc_close(void* base, int device);

/*
 * Lets kernels on `device` read and write `peer`'s memory in this process
 * (cudaDeviceEnablePeerAccess; already-enabled is not an error).  Needed
 * before the _sharded entry points touch shards that live on other devices:
 * a peer's shard mapped through CUDA IPC is addressable, but a kernel on
 * another device may only access it once peer access is enabled.  Returns
 * FSA_ERR_INVALID_ARGUMENT when the two devices cannot access each other.
 */
FSA_API int fsa_enable_peer_access(int device, int peer);

/*
 * 2-hop backward (saved-index replay).  Replaces
 * fused_sample_agg_2hop_cuda_backward (fuseop/fused_sample_agg.cu:317-326;
 * kernel :216-271).  grad_x[samples2[b,i,j],:] +=
 * (grad_out[b,:] / nonempty_b) / valid_{b,i}.  grad_x must be pre-zeroed (or
 * accumulate into an existing gradient).
 */
FSA_API int fsa_sample_agg_2hop_backward(const float* grad_out, const int32_t* samples1,
                                 const int32_t* samples2, int64_t batch_size,
                                 int64_t feature_dim, int32_t fanout1,
                                 int32_t fanout2, float* grad_x,
                                 int64_t num_nodes, void* stream);

/*
 * The same 2-hop backward as a sort-by-destination segmented reduction
 * (replaces fused_sample_agg_2hop_cuda_backward, fuseop/fused_sample_agg.cu:
 * 317-326, like fsa_sample_agg_2hop_backward; the reference has only the
 * atomic form).  The (root, slot, leaf) contributions are grouped by
 * destination row with a counting sort over the node ids, then one warp per
 * destination
 * row adds the row's contributions, in the sorted order, to its current
 * value and stores it once — no atomics on grad_x.  Same result as
 * fsa_sample_agg_2hop_backward within fp32 reassociation.  Needs a
 * workspace of fsa_sample_agg_2hop_backward_sorted_workspace_size(...)
 * bytes (256-byte aligned, contents need no initialisation): about
 * 8 bytes per node plus 8 per (root, slot, leaf) entry.  Slower than the
 * atomic variant on power-law graphs (an N-sized sort, hub rows summed by
 * one warp each): measured 109 us vs 29 us for 1024 roots x 15 x 10 on a
 * 2.45M-node graph with D = 100.
 */
FSA_API size_t fsa_sample_agg_2hop_backward_sorted_workspace_size(int64_t num_nodes,
                                                                  int64_t batch_size,
                                                                  int32_t fanout1,
                                                                  int32_t fanout2);
FSA_API int fsa_sample_agg_2hop_backward_sorted(const float* grad_out, const int32_t* samples1,
                                                const int32_t* samples2, int64_t batch_size,
                                                int64_t feature_dim, int32_t fanout1,
                                                int32_t fanout2, float* grad_x,
                                                int64_t num_nodes, void* workspace,
                                                size_t workspace_bytes, void* stream);

/*
 * Zero count floats at dst.  Replaces the dense gradient allocation fill
 * at::zeros({N, D}) of the reference backward (fuseop/binding.cpp:137, :220).
 */
FSA_API int fsa_fill_zero_f32(float* dst, int64_t count, void* stream);

/*
 * Zero the rows rows[0..count) of table float32[num_rows][dim]; entries
 * outside [0, num_rows) -- the -1 padding of saved ids -- are skipped.  The
 * row-sparse counterpart of the fill above: a gradient buffer kept across
 * steps is cleared by zeroing the rows the previous steps' saved ids touched
 * (pass samples2 or samples as the row list), 4 * dim bytes per listed row
 * instead of 4 * num_rows * dim.  No counterpart in the reference, whose
 * backward zero-fills a fresh N x D gradient every call
 * (fuseop/binding.cpp:137, :220).
 */
FSA_API int fsa_zero_rows_f32(float* table, int64_t num_rows, int64_t dim, const int32_t* rows,
                              int64_t count, void* stream);

/*
 * Per-kernel timing of fsa_sample_agg_2hop_forward, for benchmarks (no
 * counterpart in the reference).  fsa_phase_timing(1) discards earlier
 * records and makes every later 2-hop forward record CUDA events around its
 * plan, scan, draw and gather kernels on the call's stream;
 * fsa_phase_timing(0) stops recording.  fsa_phase_times waits for the
 * recorded events, writes the summed milliseconds of the four kernels to
 * ms[0..3] and the number of recorded calls to *calls, and releases the
 * records.  Off by default: the forward then creates and records nothing.
 */
FSA_API int fsa_phase_timing(int enable);
FSA_API int fsa_phase_times(double* ms, int64_t* calls);

/* Human-readable text for a status code (static storage). */
FSA_API const char* fsa_status_string(int status);

/* The cudaError_t of the most recent FSA_ERR_CUDA on this thread (0 if none). */
FSA_API int fsa_last_cuda_error(void);

/* Number of kernels this library has launched in the process (all threads). */
FSA_API uint64_t fsa_launch_count(void);

/*
 * Read (and optionally clear) the status word of `device`: an OR of
 * FSA_STATUS_* bits set by kernels that met out-of-range ids.  Synchronises
 * the device; meant for tests and debugging, not the hot path.
 */
FSA_API int fsa_device_status(int device, uint32_t* flags, int reset);

#ifdef __cplusplus
}
#endif

#endif /* FSA_SM100_H_ */
