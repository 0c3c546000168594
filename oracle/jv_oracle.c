/*
 * TEST INFRASTRUCTURE ONLY -- the CPU oracle for the batched Jonker-Volgenant
 * path.  Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg
 * may load this library, and only as the checker or the timed CPU baseline.
 * The product path (torchmatch_b200) never calls into it.
 *
 * What it restates (tue-p8n/torchmatch 1.0.3, paths relative to
 * sources/torchmatch/assignment/):
 *   - cpu/ops.cpp:67-93     batch-global +inf sentinel, NaN / -inf rejection
 *   - cpu/ops.cpp:176-289   solve_batch: pad each problem to K x K (pad cells
 *                           0, non-finite cells -> sentinel), solve, map
 *                           columns >= M to -1
 *   - cpu/jonker_compact_core.h:51-252  the "compact" variant of the same
 *                           phases (jonker_compact_batch), selected by
 *                           jv_work.compact: column minima seeded from row 0,
 *                           FLT_MAX instead of LARGE, no visit bound in the
 *                           row reduction, the FIRST free column of a tie
 *                           group, and the price update (v + d) - min
 *   - cpu/jonker_dense_flat.h:124-274  the four LAPJV phases in fp32:
 *       column reduction + reduction transfer  (ccrrt_dense  :124-176)
 *       augmenting row reduction, run twice    (carr_dense   :178-235)
 *       shortest augmenting path (Dijkstra)     (find_dense :27-43,
 *                                                scan_dense :45-73,
 *                                                find_path_dense :75-122)
 *       path augmentation                       (ca_dense    :237-258)
 *
 * Every floating-point expression keeps the reference's operand order
 * ((c - v) - h, v[j1] - (v2 - v1), v += d - mind) and every comparison keeps
 * its strictness, because the mapping on tied inputs depends on them.  The
 * column permutation used by the Dijkstra phase ("todo" / "ready" regions)
 * is reproduced exactly, including the swap pattern of the minimum search.
 *
 * Pinning: tests/test_oracle.py checks this file against golden vectors
 * produced by the reference's own torch.ops.assignment.jonker_dense_batch
 * (tests/golden/make_golden.py) and, when oracle/_ref is built, against the
 * reference's compiled solver core on the same inputs.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include <float.h>

#ifdef _OPENMP
#include <omp.h>
#endif

#define TMO_BIG 1e18f /* jonker_dense_flat.h:22-23 (LARGE_V<float>) */

typedef struct {
    int has_nan;
    int has_neg_inf;
    int any_finite;
    float max_finite;
} tmo_stats;

/* Per-problem working arrays, one set per thread. */
typedef struct {
    int n;
    int compact;          /* jonker_compact_core.h semantics */
    int32_t *row_of_col;  /* y */
    int32_t *col_of_row;  /* x */
    int32_t *queue;       /* free rows */
    int32_t *pred;
    int32_t *order;       /* column permutation of the Dijkstra phase */
    float *price;         /* v */
    float *dist;          /* d */
    char *single;         /* row owns exactly one column after reduction */
} jv_work;

static int work_init(jv_work *w, int n) {
    w->n = n;
    w->row_of_col = (int32_t *)malloc(sizeof(int32_t) * (size_t)n);
    w->col_of_row = (int32_t *)malloc(sizeof(int32_t) * (size_t)n);
    w->queue = (int32_t *)malloc(sizeof(int32_t) * (size_t)n);
    w->pred = (int32_t *)malloc(sizeof(int32_t) * (size_t)n);
    w->order = (int32_t *)malloc(sizeof(int32_t) * (size_t)n);
    w->price = (float *)malloc(sizeof(float) * (size_t)n);
    w->dist = (float *)malloc(sizeof(float) * (size_t)n);
    w->single = (char *)malloc((size_t)n);
    return w->row_of_col && w->col_of_row && w->queue && w->pred && w->order &&
           w->price && w->dist && w->single;
}

static void work_free(jv_work *w) {
    free(w->row_of_col); free(w->col_of_row); free(w->queue); free(w->pred);
    free(w->order); free(w->price); free(w->dist); free(w->single);
}

/* Phase 1: column reduction and reduction transfer
 * (jonker_dense_flat.h:124-176).  Returns the number of free rows, which are
 * left in w->queue in increasing row order. */
static int phase_reduce(const float *c, jv_work *w) {
    const int n = w->n;
    int32_t *y = w->row_of_col, *x = w->col_of_row;
    float *v = w->price;
    for (int k = 0; k < n; ++k) {
        x[k] = -1;
        v[k] = w->compact ? c[k] : TMO_BIG;  /* compact_core.h:79-80 */
        y[k] = 0;
        w->single[k] = 1;
    }
    /* cheapest row of every column; the first such row wins (strict <) */
    for (int i = w->compact ? 1 : 0; i < n; ++i) {
        const float *ci = c + (size_t)i * n;
        for (int j = 0; j < n; ++j)
            if (ci[j] < v[j]) {
                v[j] = ci[j];
                y[j] = i;
            }
    }
    /* highest column index claims its row; later claimants are dropped */
    for (int j = n - 1; j >= 0; --j) {
        const int i = y[j];
        if (x[i] < 0) {
            x[i] = j;
        } else {
            w->single[i] = 0;
            y[j] = -1;
        }
    }
    /* reduction transfer, in row order (later rows see earlier updates) */
    int nfree = 0;
    for (int i = 0; i < n; ++i) {
        if (x[i] < 0) {
            w->queue[nfree++] = i;
            continue;
        }
        if (!w->single[i])
            continue;
        const float *ci = c + (size_t)i * n;
        const int own = x[i];
        float best = w->compact ? FLT_MAX : TMO_BIG;  /* compact_core.h:104 */
        for (int j = 0; j < n; ++j) {
            if (j == own)
                continue;
            const float r = ci[j] - v[j];
            if (r < best)
                best = r;
        }
        v[own] -= best;
    }
    return nfree;
}

/* Phase 2: augmenting row reduction over the free-row queue
 * (jonker_dense_flat.h:178-235).  Returns the new number of free rows. */
static int phase_arr(const float *c, jv_work *w, int nfree) {
    const int n = w->n;
    int32_t *y = w->row_of_col, *x = w->col_of_row, *q = w->queue;
    float *v = w->price;
    unsigned head = 0, visits = 0;
    int kept = 0;
    while (head < (unsigned)nfree) {
        ++visits;
        const int row = q[head++];
        const float *ci = c + (size_t)row * n;
        /* two smallest reduced costs, first index wins ties */
        int a = 0, b = -1;
        float va = ci[0] - v[0], vb = w->compact ? FLT_MAX : TMO_BIG;
        for (int j = 1; j < n; ++j) {
            const float r = ci[j] - v[j];
            if (r < vb) {
                if (r >= va) {
                    vb = r;
                    b = j;
                } else {
                    vb = va;
                    b = a;
                    va = r;
                    a = j;
                }
            }
        }
        int owner = y[a];
        const float lowered = v[a] - (vb - va);
        const int lowers = lowered < v[a];
        /* the compact variant has no visit bound (compact_core.h:145-169) */
        if (w->compact || visits < head * (unsigned)n) {
            if (lowers) {
                v[a] = lowered;
            } else if (owner >= 0 && (b >= 0 || w->compact)) {
                a = b;
                owner = y[b];
            }
            if (owner >= 0) {
                if (lowers)
                    q[--head] = owner;      /* retry the displaced row next */
                else
                    q[kept++] = owner;      /* defer it to the next pass */
            }
        } else if (owner >= 0) {
            q[kept++] = owner;
        }
        x[row] = a;
        y[a] = row;
    }
    return kept;
}

/* Minimum search over order[lo..n): moves every column that attains the
 * minimum distance to the front of the range, with the reference's swap
 * pattern (jonker_dense_flat.h:27-43).  Returns the end of the tie group. */
static int take_minimum(int n, int lo, const float *d, int32_t *order) {
    int hi = lo + 1;
    float best = d[order[lo]];
    for (int k = hi; k < n; ++k) {
        const int j = order[k];
        if (d[j] <= best) {
            if (d[j] < best) {
                hi = lo;
                best = d[j];
            }
            order[k] = order[hi];
            order[hi++] = j;
        }
    }
    return hi;
}

/* Relaxes the rows of the tie group [*plo,*phi) against the unscanned
 * columns (jonker_dense_flat.h:45-73).  Returns a free column reached at the
 * current minimum distance, or -1 after the group is exhausted. */
static int relax_group(int n, const float *c, int *plo, int *phi, jv_work *w) {
    float *d = w->dist;
    const float *v = w->price;
    int32_t *order = w->order, *pred = w->pred;
    const int32_t *y = w->row_of_col;
    int lo = *plo, hi = *phi;
    while (lo != hi) {
        int j = order[lo++];
        const int i = y[j];
        const float best = d[j];
        const float *ci = c + (size_t)i * n;
        const float h = ci[j] - v[j] - best;
        for (int k = hi; k < n; ++k) {
            j = order[k];
            const float r = ci[j] - v[j] - h;
            if (r < d[j]) {
                d[j] = r;
                pred[j] = i;
                if (r == best) {
                    if (y[j] < 0)
                        return j;
                    order[k] = order[hi];
                    order[hi++] = j;
                }
            }
        }
    }
    *plo = lo;
    *phi = hi;
    return -1;
}

/* Dijkstra search from a free row (jonker_dense_flat.h:75-122); updates the
 * prices of the settled columns and returns the free column reached. */
static int shortest_path(int n, const float *c, int start, jv_work *w) {
    float *d = w->dist, *v = w->price;
    int32_t *order = w->order;
    const int32_t *y = w->row_of_col;
    const float *cs = c + (size_t)start * n;
    int lo = 0, hi = 0, settled = 0, sink = -1;
    for (int k = 0; k < n; ++k) {
        order[k] = k;
        d[k] = cs[k] - v[k];
        w->pred[k] = start;
    }
    while (sink == -1) {
        if (lo == hi) {
            settled = lo;
            hi = take_minimum(n, lo, d, order);
            for (int k = lo; k < hi; ++k)
                if (y[order[k]] < 0) {
                    sink = order[k];   /* last free column of the group */
                    if (w->compact)
                        break;         /* compact: the first (:195-201) */
                }
        }
        if (sink == -1)
            sink = relax_group(n, c, &lo, &hi, w);
    }
    const float best = d[order[lo]];
    for (int k = 0; k < settled; ++k) {
        if (w->compact)
            v[order[k]] = v[order[k]] + d[order[k]] - best;  /* :232-235 */
        else
            v[order[k]] += d[order[k]] - best;
    }
    return sink;
}

/* Phase 3: augmentation of every remaining free row
 * (jonker_dense_flat.h:237-258), including the n-step guard. */
static void phase_augment(const float *c, jv_work *w, int nfree) {
    const int n = w->n;
    int32_t *y = w->row_of_col, *x = w->col_of_row;
    for (int f = 0; f < nfree; ++f) {
        const int start = w->queue[f];
        int j = shortest_path(n, c, start, w);
        int i, steps = 0;
        do {
            i = w->pred[j];
            y[j] = i;
            const int prev = x[i];
            x[i] = j;
            j = prev;
            if (++steps >= n && !w->compact)
                break;
        } while (i != start);
    }
}

/* Full square solve (jonker_dense_flat.h:260-274). */
static void jv_square(const float *c, jv_work *w) {
    int nfree = phase_reduce(c, w);
    for (int pass = 0; pass < 2 && nfree > 0; ++pass)
        nfree = phase_arr(c, w, nfree);
    if (nfree > 0)
        phase_augment(c, w, nfree);
}

/* ------------------------------------------------------------------------ */
/* Exported C ABI of the oracle.                                             */
/* ------------------------------------------------------------------------ */

/* Batch statistics in the reference's classification order
 * (cpu/ops.cpp:67-93): NaN first, then -inf, then finite. */
void tmo_stats_f32(const float *data, int64_t count, tmo_stats *out) {
    tmo_stats s = {0, 0, 0, -FLT_MAX};
    for (int64_t k = 0; k < count; ++k) {
        const float val = data[k];
        if (isnan(val)) {
            s.has_nan = 1;
        } else if (val == -INFINITY) {
            s.has_neg_inf = 1;
        } else if (isfinite(val)) {
            if (val > s.max_finite)
                s.max_finite = val;
            s.any_finite = 1;
        }
    }
    *out = s;
}

/* (max_finite + 1) * (K + 1) in fp32, or 1 when no cell is finite
 * (cpu/ops.cpp:91-92). */
float tmo_sentinel_f32(const tmo_stats *s, int K) {
    return s->any_finite ? (s->max_finite + 1.0f) * (float)(K + 1) : 1.0f;
}

/* The batched solve of cpu/ops.cpp:176-289 (float32 branch).
 * costs: (B, N, M) contiguous fp32; out: (B, N) int64.
 * Returns 0, 1 if the batch holds a NaN, 2 if it holds -inf, 3 on an
 * allocation failure.  nthreads <= 0 uses the OpenMP default. */
static int batch_driver(const float *costs, int64_t B, int N, int M, int64_t *out,
                        int nthreads, int compact) {
    if (B <= 0 || N <= 0 || M <= 0) {
        for (int64_t k = 0; k < (B > 0 ? B : 0) * (N > 0 ? N : 0); ++k)
            out[k] = -1;
        return 0;
    }
    const int K = N > M ? N : M;
    tmo_stats s;
    tmo_stats_f32(costs, B * (int64_t)N * M, &s);
    if (s.has_nan)
        return 1;
    if (s.has_neg_inf)
        return 2;
    const float sentinel = tmo_sentinel_f32(&s, K);
    int failed = 0;
#ifdef _OPENMP
    if (nthreads <= 0)
        nthreads = omp_get_max_threads();
#pragma omp parallel num_threads(nthreads) reduction(| : failed)
#endif
    {
        jv_work w;
        float *pad = (float *)malloc(sizeof(float) * (size_t)K * K);
        const int ok = work_init(&w, K);
        w.compact = compact;
        if (!ok || !pad) {
            failed = 1;
        } else {
#ifdef _OPENMP
#pragma omp for schedule(dynamic, 1)
#endif
            for (int64_t b = 0; b < B; ++b) {
                const float *src = costs + b * (int64_t)N * M;
                for (int i = 0; i < K; ++i)
                    for (int j = 0; j < K; ++j) {
                        float val = 0.0f;
                        if (i < N && j < M) {
                            val = src[(size_t)i * M + j];
                            if (!isfinite(val))
                                val = sentinel;
                        }
                        pad[(size_t)i * K + j] = val;
                    }
                jv_square(pad, &w);
                int64_t *ob = out + b * (int64_t)N;
                for (int i = 0; i < N; ++i) {
                    const int j = w.col_of_row[i];
                    ob[i] = (j >= 0 && j < M) ? j : -1;
                }
            }
        }
        work_free(&w);
        free(pad);
    }
    return failed ? 3 : 0;
}

/* jonker_dense_batch (cpu/ops.cpp:176-289 with jonker_dense_flat.h). */
int tmo_jonker_dense_batch_f32(const float *costs, int64_t B, int N, int M,
                               int64_t *out, int nthreads) {
    return batch_driver(costs, B, N, M, out, nthreads, 0);
}

/* jonker_compact_batch (the same driver with jonker_compact_core.h). */
int tmo_jonker_compact_batch_f32(const float *costs, int64_t B, int N, int M,
                                 int64_t *out, int nthreads) {
    return batch_driver(costs, B, N, M, out, nthreads, 1);
}

/* Squared-Euclidean costs of two point sets, the producer restated by the
 * fused entry point: costs[b][i][j] = sum over d = 0 .. D-1, in that order,
 * of (x[b][i][d] - y[b][j][d])^2 in fp32, each operation rounded on its own
 * (this file builds with -ffp-contract=off), starting from 0.  The order is
 * that of the reference's lazy sqeuclidean costs
 * (transport/matrix/cpu/exact/network_simplex_simple.h:453-457), in fp32. */
void tmo_sqeuclidean_costs_f32(const float *x, const float *y, int64_t B, int N, int M, int D,
                               float *costs) {
    for (int64_t b = 0; b < B; ++b) {
        const float *xb = x + b * (int64_t)N * D;
        const float *yb = y + b * (int64_t)M * D;
        float *cb = costs + b * (int64_t)N * M;
        for (int i = 0; i < N; ++i)
            for (int j = 0; j < M; ++j) {
                float acc = 0.0f;
                for (int d = 0; d < D; ++d) {
                    const float df = xb[(int64_t)i * D + d] - yb[(int64_t)j * D + d];
                    const float sq = df * df;
                    acc = acc + sq;
                }
                cb[(int64_t)i * M + j] = acc;
            }
    }
}
