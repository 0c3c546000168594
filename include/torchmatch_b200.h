/*
 * torchmatch_b200 -- C ABI of the B200 (sm_100a) batched Jonker-Volgenant
 * solver.
 *
 * These entry points replace the CUDA side of the reference's
 * torch.ops.assignment.jonker_dense_batch (tue-p8n/torchmatch 1.0.3,
 * sources/torchmatch/assignment/) and widen it:
 *
 *   tm_jv_stats_f32         replaces k_scan_sentinel_stats + the scan half of
 *                           compute_inf_sentinel  (cuda/cuda_common.cuh:186-243)
 *   tm_jv_sentinel          replaces the check + formula half of
 *                           compute_inf_sentinel  (cuda/cuda_common.cuh:245-254,
 *                           cpu/ops.cpp:86-92)
 *   tm_jv_solve_f32         replaces rewrite_inf_to_sentinel + the batched
 *                           kernel launch          (cuda/cuda_common.cuh:270-284,
 *                           cuda/jonker_tiled.cuh:203-218,
 *                           cuda/dispatch.cu:156-176); the result follows the
 *                           CPU solver (cpu/ops.cpp:176-289 +
 *                           cpu/jonker_dense_flat.h:124-274) bit for bit
 *   tm_jv_solve_checked_f32 the solve with the statistics pass fused in
 *   tm_jonker_dense_batch_f32  the whole op body of jonker_dense_batch_cuda
 *                           (cuda/dispatch.cu:137-177) for callers without
 *                           torch: one check-mode solve, host check, and a
 *                           sentinel solve only for batches holding +inf
 *   tm_jonker_dense_batch_unpacked_f32, tm_jonker_compact_batch_f32,
 *   tm_jonker_compact_batch_unpacked_f32  the reference's CPU-only unpacked
 *                           and compact ops (cpu/ops.cpp:297-417,
 *                           cpu/jonker_compact_core.h) on the GPU
 *   tm_jonker_dense_batch_async_f32  no host synchronisation (capturable)
 *   tm_jonker_dense_batch_f32_noalloc  no allocation by the caller
 *   tm_jonker_sqeuclidean_batch_f32, tm_jv_points_solve_f32
 *                           squared-Euclidean costs built from two
 *                           point sets inside the solve kernel (no (B, N, M)
 *                           cost tensor in memory)
 *
 * Conventions: plain device pointers and sizes, no torch types, no C++
 * exceptions.  Every function returns a tm_status code; CUDA errors are
 * reported as TM_ERR_CUDA and the cudaError_t is kept for tm_last_cuda_error().
 * Problems that hit a loop bound are reported through TM_WS_UNSOLVED in the
 * workspace status (their rows are -1, like the reference's rc != 0 rows,
 * cpu/ops.cpp:274-278), not through the return code.  A tile copy whose
 * wait runs out (TM_WS_TIMEOUT) leaves its problems as rows of -1 too; the
 * synchronous entry points read the status back in their one
 * synchronisation and return TM_ERR_TIMEOUT for it.  All
 * work is enqueued on the given stream; only the whole-op entry points
 * (tm_jonker_*_f32 except the async one) synchronise it, to read the
 * NaN / -inf verdict as the reference does.
 */
#ifndef TORCHMATCH_B200_H
#define TORCHMATCH_B200_H

#include <stdint.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st *tm_stream_t; /* == cudaStream_t */

typedef enum tm_status {
    TM_OK = 0,
    TM_ERR_NAN = 1,        /* a cell is NaN ("cost matrix contains NaN")      */
    TM_ERR_NEG_INF = 2,    /* a cell is -inf ("cost matrix contains -inf")    */
    TM_ERR_ARG = 3,        /* bad shape / null pointer / unsupported size     */
    TM_ERR_CUDA = 4,       /* a CUDA call failed; see tm_last_cuda_error()    */
    TM_ERR_TOO_LARGE = 5,  /* max(N, M) above tm_jv_max_k()                    */
    TM_ERR_UNSOLVED = 6,   /* a problem hit a loop bound (see TM_WS_UNSOLVED)  */
    TM_ERR_TIMEOUT = 7     /* a cost tile copy did not land within the wait
                              limit (TM_WS_TIMEOUT); its rows are -1          */
} tm_status;

/* Batch statistics, device-resident.  Written by tm_jv_stats_f32. */
typedef struct tm_jv_stats {
    uint32_t flags;     /* TM_STAT_* bits                                    */
    uint32_t max_key;   /* order-preserving key of the largest finite cell   */
} tm_jv_stats;

/* Device scratch of one solve (tm_jv_workspace_bytes() bytes).  `ticket`
 * hands out problems to warps; the solves zero it and `status` on the
 * stream before each launch.  `status` collects TM_WS_* bits (bit OR):
 * a problem that hit a loop bound (its row is all -1), a wait that timed
 * out, and -- in the asynchronous entry point -- NaN / -inf in the batch. */
#define TM_WS_NAN       1
#define TM_WS_NEG_INF   2
#define TM_WS_UNSOLVED  4
#define TM_WS_TIMEOUT   8
typedef struct tm_jv_workspace {
    tm_jv_stats stats;
    unsigned long long ticket;
    int32_t status;
    int32_t reserved[11];
} tm_jv_workspace;

#define TM_STAT_NAN      1u
#define TM_STAT_NEG_INF  2u
#define TM_STAT_FINITE   4u
#define TM_STAT_POS_INF  8u

/* Largest max(N, M) the solver accepts. */
int tm_jv_max_k(void);

/* Scans `count` fp32 cells once and writes the batch statistics to
 * `stats_dev` (zeroed by this call first).  Replaces
 * cuda/cuda_common.cuh:186-243 (k_scan_sentinel_stats). */
int tm_jv_stats_f32(const float *costs, int64_t count, tm_jv_stats *stats_dev,
                    tm_stream_t stream);

/* Host side: checks a copied-back tm_jv_stats and returns the +inf
 * sentinel (max_finite + 1) * (K + 1), or 1 when no cell is finite.
 * Returns TM_ERR_NAN / TM_ERR_NEG_INF like cuda/cuda_common.cuh:245-249.
 * `has_pos_inf` (may be NULL) tells whether any +inf cell exists. */
int tm_jv_sentinel(const tm_jv_stats *stats_host, int K, float *sentinel,
                   int *has_pos_inf);

/* Solves B problems of shape (N, M), costs contiguous fp32 (B, N, M),
 * into out (B, N) int64 (row -> column, -1 = unmatched).  `sentinel`
 * replaces +inf cells (only read when has_pos_inf != 0).  `workspace` is
 * device memory of tm_jv_workspace_bytes() (a tm_jv_workspace) that this
 * call re-initialises on the stream; concurrent solves need their own.
 * Replaces cuda/cuda_common.cuh:270-284 + cuda/jonker_tiled.cuh:203-218. */
int tm_jv_solve_f32(const float *costs, int64_t B, int N, int M, float sentinel,
                    int has_pos_inf, int64_t *out, void *workspace,
                    tm_stream_t stream);

/* One pass that solves every problem whose cells are all finite and, in the
 * same read, accumulates the batch statistics into workspace->stats (zeroed
 * first).  Problems holding NaN, -inf or +inf are left as rows of -1: after
 * reading the statistics back, the caller raises on NaN / -inf or, if the
 * batch holds +inf, calls tm_jv_solve_f32 with the sentinel.  Together this
 * replaces the separate statistics pass of the reference
 * (cuda/cuda_common.cuh:215-255) for batches without +inf. */
int tm_jv_solve_checked_f32(const float *costs, int64_t B, int N, int M, int64_t *out,
                            void *workspace, tm_stream_t stream);

/* Bytes of device scratch (a tm_jv_workspace) for tm_jv_solve_f32 and
 * tm_jonker_dense_batch_f32. */
size_t tm_jv_workspace_bytes(void);

/* The whole jonker_dense_batch op for a caller without torch: statistics,
 * one stream synchronisation for the NaN / -inf verdict, solve.  `workspace`
 * is device memory of tm_jv_workspace_bytes().  Replaces
 * cuda/dispatch.cu:137-177 (jonker_dense_batch_cuda). */
int tm_jonker_dense_batch_f32(const float *costs, int64_t B, int N, int M,
                              int64_t *out, void *workspace, tm_stream_t stream);

/* Same as tm_jonker_dense_batch_f32, for callers that may not allocate
 * device memory themselves (no cudaMalloc and no caching allocator in their
 * process, e.g. an embedding runtime that owns all GPU memory or a hook that
 * runs where allocation is forbidden).  No counterpart in the reference.
 * Its scratch is a fixed 64-byte array in this library's device memory, one
 * per GPU, kept until the process exits, so the only size limit is the
 * solver's own max(N, M) <= tm_jv_max_k() (TM_ERR_TOO_LARGE beyond it).
 * The first call on a device looks up that array's device address and
 * keeps it for the life of the process (a cudaDeviceReset does not refresh
 * it); make that first call before any stream capture.  Every call
 * synchronises its stream, as tm_jonker_dense_batch_f32 does.  All calls on
 * one device share the array: calls that overlap on the GPU (other streams,
 * other host threads) race and must be serialised by the caller.  Because
 * the caller cannot read the shared status word, problems left as rows of
 * -1 by a loop bound are reported as TM_ERR_UNSOLVED, and a timed-out tile
 * copy as TM_ERR_TIMEOUT.  Nothing is allocated or freed. */
int tm_jonker_dense_batch_f32_noalloc(const float *costs, int64_t B, int N, int M,
                                      int64_t *out, tm_stream_t stream);

/* Device outputs of jonker_dense_batch_unpacked (cpu/ops.cpp:290-295):
 * matches (B, N, 2) matched (row, column) pairs in row order, valid in
 * [0, n_matched[b]); unmatched_rows (B, N), valid in [0, N - n_matched[b]);
 * unmatched_cols (B, M) in column order, valid in [0, M - n_matched[b]);
 * n_matched (B,).  Every entry past its count is -1. */
typedef struct tm_jv_unpacked {
    int64_t *matches;
    int64_t *unmatched_rows;
    int64_t *unmatched_cols;
    int64_t *n_matched;
} tm_jv_unpacked;

/* jonker_dense_batch_unpacked for N, M >= 1: the same solve as
 * tm_jonker_dense_batch_f32 with the compaction written by the solve kernel
 * itself.  Replaces cpu/ops.cpp:297-417 (the reference has it on CPU only). */
int tm_jonker_dense_batch_unpacked_f32(const float *costs, int64_t B, int N, int M,
                                       const tm_jv_unpacked *u, void *workspace,
                                       tm_stream_t stream);

/* jonker_dense_batch without any host synchronisation, for CUDA graph
 * capture: the check-mode solve, then a second launch that reads the batch
 * statistics on the device and, only if the batch holds +inf, computes the
 * sentinel there and solves again.  Nothing is read back: NaN / -inf are
 * reported as TM_WS_NAN / TM_WS_NEG_INF in workspace->status (their
 * problems' rows are -1), not as a return code.  The reference's op is not
 * capturable (cuda/dispatch.cu:97-106); its docs describe this as the
 * graph-safe mode (docs/site/content/2.algorithms/1.assignment/
 * 1.quickstart.md:262-263). */
int tm_jonker_dense_batch_async_f32(const float *costs, int64_t B, int N, int M,
                                    int64_t *out, void *workspace, tm_stream_t stream);

/* jonker_compact_batch and jonker_compact_batch_unpacked: the same batch
 * driver over the reference's "compact" solver variant
 * (cpu/jonker_compact_core.h:51-252; CPU-only in the reference), which
 * differs from the dense one in its column-reduction seed, its FLT_MAX
 * initial values, the missing visit bound of the row reduction, the first
 * (not last) free column of a tie group and the rounding of its price
 * update.  Same arguments as the dense entry points. */
int tm_jonker_compact_batch_f32(const float *costs, int64_t B, int N, int M, int64_t *out,
                                void *workspace, tm_stream_t stream);
int tm_jonker_compact_batch_unpacked_f32(const float *costs, int64_t B, int N, int M,
                                         const tm_jv_unpacked *u, void *workspace,
                                         tm_stream_t stream);

/* Fused cost construction: solves jonker_dense_batch on the squared-
 * Euclidean costs of two point sets, x (B, N, D) and y (B, M, D), both
 * contiguous fp32 on the device, without writing the (B, N, M) cost batch.
 * Cell (i, j) of problem b is the fp32 sum over d = 0 .. D-1, in that order,
 * of (x[b][i][d] - y[b][j][d])^2, each subtraction, product and sum rounded
 * separately (no fused multiply-add), starting from 0: the result equals
 * tm_jonker_dense_batch_f32 on the matrix that such a sequential producer
 * writes (the order of the reference's lazy sqeuclidean costs,
 * transport/matrix/cpu/exact/network_simplex_simple.h:453-457, in fp32).
 * NaN / -inf / +inf cells (from non-finite coordinates) behave as in the
 * dense op.  `workspace` is 256-byte aligned device memory of
 * `workspace_bytes` >= tm_jv_points_workspace_bytes(B, N, M) bytes
 * (query on the device that will run the call): shapes whose problems fit
 * in shared memory need only the 256-byte header; larger ones also take
 * one N * M slab per resident warp (a smaller workspace runs fewer warps;
 * TM_ERR_ARG below one slab).  No counterpart op in the reference, whose
 * callers build the cost tensor first (tests/_costgen.py) and pass it. */
size_t tm_jv_points_workspace_bytes(int64_t B, int N, int M);
/* One launch of the fused solve, for callers that combine statistics
 * themselves (e.g. across GPUs): with check != 0 it is the fused form of
 * tm_jv_solve_checked_f32 (statistics zeroed and gathered into
 * workspace->stats, problems with non-finite cells left as rows of -1);
 * with check == 0 the fused form of tm_jv_solve_f32 (`sentinel` replaces
 * +inf cells when has_pos_inf != 0).  Other arguments as for
 * tm_jonker_sqeuclidean_batch_f32. */
int tm_jv_points_solve_f32(const float *x, const float *y, int64_t B, int N, int M, int D,
                           float sentinel, int has_pos_inf, int check, int64_t *out,
                           void *workspace, size_t workspace_bytes, tm_stream_t stream);
int tm_jonker_sqeuclidean_batch_f32(const float *x, const float *y, int64_t B, int N, int M,
                                    int D, int64_t *out, void *workspace,
                                    size_t workspace_bytes, tm_stream_t stream);

/* Test hook: caps every loop of the solver at `bound` iterations (0 restores
 * the real bounds), so tests can drive the loop-bound failure path -- rows
 * of -1 and TM_WS_UNSOLVED in the workspace status -- without a GPU fault.
 * Process-wide; not for production use.  No counterpart in the reference
 * (its CPU solver maps rc != 0 to a row of -1, cpu/ops.cpp:274-278). */
void tm_jv_debug_set_loop_bound(int bound);

/* Test hook: polls of a cost tile copy's mbarrier before the wait counts as
 * timed out (0: the first wait gives up at once; a negative value restores
 * the production limit), so tests can drive the timeout path -- rows of -1,
 * TM_WS_TIMEOUT in the status, TM_ERR_TIMEOUT from the synchronous entry
 * points -- without a GPU fault.  The copy in flight is still waited for
 * (with the production limit) before its tile is reused.  Process-wide; not
 * for production use.  No counterpart in the reference, whose kernel loads
 * its tile with plain loads (cuda/jonker_tiled.cuh:64-71). */
void tm_jv_debug_set_wait_limit(int limit);

/* The cudaError_t of the last TM_ERR_CUDA on this thread. */
int tm_last_cuda_error(void);

/* Human-readable text for a tm_status code. */
const char *tm_status_string(int status);

#ifdef __cplusplus
}
#endif

#endif /* TORCHMATCH_B200_H */
