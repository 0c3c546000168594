// TEST INFRASTRUCTURE ONLY.  Links the reference's own compiled solver core
// (sources/torchmatch/assignment/cpu/jonker_dense_core.cpp, built from the
// reference tree by oracle/Makefile into oracle/_ref/) behind a plain C ABI,
// so the tests can pin oracle/jv_oracle.c against the reference itself and
// bench.py can time the reference's CPU solver as its baseline arm.
//
// The batch driver below restates cpu/ops.cpp:176-289 (float32 branch), used
// for both jonker_dense_batch and jonker_compact_batch:
// batch-global sentinel, pad to K x K, one square solve per problem,
// columns >= M mapped to -1.  The square solve is the reference's
// jonker_dense_solve_square_f32 (jonker_dense_core.cpp:57-60).
#include <cmath>
#include <cstdint>
#include <cfloat>
#include <vector>
#include <omp.h>

#include "jonker_compact_core.h"  // header-only, from the reference tree

namespace match_jonker::detail {
int jonker_dense_solve_square_f32(const float *cost_flat, int n, int64_t *row_to_col,
                                  int64_t *col_to_row);
}

using SquareFn = int (*)(const float *, int, int64_t *, int64_t *);

static int batch(const float *costs, int64_t B, int N, int M, int64_t *out, int nthreads,
                 SquareFn solve) {
    if (B <= 0 || N <= 0 || M <= 0) {
        for (int64_t k = 0; k < (B > 0 ? B : 0) * (N > 0 ? N : 0); ++k) out[k] = -1;
        return 0;
    }
    const int K = N > M ? N : M;
    float top = -FLT_MAX;
    bool any = false, nan = false, ninf = false;
    const int64_t count = B * (int64_t)N * M;
    for (int64_t k = 0; k < count; ++k) {
        const float val = costs[k];
        if (std::isnan(val)) nan = true;
        else if (val == -INFINITY) ninf = true;
        else if (std::isfinite(val)) { if (val > top) top = val; any = true; }
    }
    if (nan) return 1;
    if (ninf) return 2;
    const float sentinel = any ? (top + 1.0f) * (float)(K + 1) : 1.0f;
    if (nthreads <= 0) nthreads = omp_get_max_threads();
    int failed = 0;
#pragma omp parallel num_threads(nthreads) reduction(| : failed)
    {
        std::vector<float> pad((size_t)K * K);
        std::vector<int64_t> r2c(K), c2r(K);
#pragma omp for schedule(dynamic, 1)
        for (int64_t b = 0; b < B; ++b) {
            const float *src = costs + b * (int64_t)N * M;
            for (int i = 0; i < K; ++i)
                for (int j = 0; j < K; ++j) {
                    float val = 0.0f;
                    if (i < N && j < M) {
                        val = src[(size_t)i * M + j];
                        if (!std::isfinite(val)) val = sentinel;
                    }
                    pad[(size_t)i * K + j] = val;
                }
            const int rc = solve(pad.data(), K, r2c.data(), c2r.data());
            int64_t *ob = out + b * (int64_t)N;
            for (int i = 0; i < N; ++i) {
                const int64_t j = r2c[i];
                ob[i] = (rc == 0 && j >= 0 && j < M) ? j : -1;
            }
            if (rc != 0) failed = 1;
        }
    }
    return failed ? 3 : 0;
}

extern "C" int tmref_jonker_dense_batch_f32(const float *costs, int64_t B, int N, int M,
                                            int64_t *out, int nthreads) {
    return batch(costs, B, N, M, out, nthreads,
                 &match_jonker::detail::jonker_dense_solve_square_f32);
}

// jonker_compact_batch: the same driver over the reference's compact solver
// (jonker_compact_core.h:276-300).
extern "C" int tmref_jonker_compact_batch_f32(const float *costs, int64_t B, int N, int M,
                                              int64_t *out, int nthreads) {
    return batch(costs, B, N, M, out, nthreads,
                 &match_jonker::detail::jonker_compact_solve_square_f32);
}
