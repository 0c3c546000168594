// TEST INFRASTRUCTURE ONLY: a C entry point around the reference's own
// batched CUDA kernel (tue-p8n/torchmatch 1.0.3,
// sources/torchmatch/assignment/cuda/jonker_tiled.cuh, included from the
// reference tree at build time by oracle/Makefile, never copied here), built
// for sm_100a into oracle/_ref/libtmref_cuda.so.  It is what the reference's
// jonker_dense_batch_cuda (cuda/dispatch.cu:137-177) launches after its
// statistics scan and +inf rewrite; bench.py's reference arm times it beside
// the CPU solver, and a GPU test compares its mappings.  The reference
// kernel takes square K <= 64 only (jonker_tiled.cuh:186-194).
#include <cstdint>

#include <cuda_runtime.h>

#include "jonker_tiled.cuh"

extern "C" int tmref_cuda_jonker_dense_batch(const float *d_costs, int B, int K,
                                             int64_t *d_out, void *stream) {
    const int tile = match_batch::select_tile(K);
    if (tile < 0 || B < 0 || K <= 0) return 5;
    match_batch::launch(tile, B, K, d_costs, d_out, static_cast<cudaStream_t>(stream));
    return cudaGetLastError() == cudaSuccess ? 0 : 4;
}
