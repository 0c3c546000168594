// Batched Jonker-Volgenant (LAPJV) for B200 / sm_100a.
//
// One warp owns one problem at a time.  Lane `l` owns the columns
// col(s, l) = (s / VEC) * 32 * VEC + l * VEC + s % VEC for slots s < S, so a
// row of the cost matrix is one (or S / VEC vectorised) conflict-free load
// per lane and every reduction over a row is a single warp reduction
// (redux.sync on fp32, new with sm_100a).  Column prices v and Dijkstra
// distances d live in registers of the owning lane (the prices are mirrored
// in shared memory during the augmenting row reduction); the row of each
// column (y), the row-indexed arrays (x, free-row queue) and the column
// permutation of the Dijkstra phase live in a small per-warp shared-memory
// block.
//
// Two storage modes for the cost matrix:
//   TILE = true   the (N, M) block of the problem is staged into shared
//                 memory by one TMA bulk copy (cp.async.bulk + mbarrier)
//                 and rows are read from there; the next problem is
//                 prefetched into L2 while the current one is solved.
//   TILE = false  for matrices that do not fit next to enough warps, rows
//                 are streamed from L2/HBM: each claimed problem is
//                 prefetched into L2, wide square rows (K > 192) pass the
//                 column reduction through a TMA ring in shared memory, and
//                 the single rows of the later phases are read with
//                 read-only vector loads (the wide rows' row reduction keeps
//                 a per-row cache of its best columns).
// With PTS (fused cost construction) the kernel builds each problem's
// squared-Euclidean costs from two point sets itself -- into the tile, or
// into a per-warp slab of the workspace that then stands in for the input.
//
// Algorithm: the reference's CPU solver, reproduced step for step so the
// mapping is identical on every input, ties included
// (sources/torchmatch/assignment/cpu/jonker_dense_flat.h, tue-p8n/torchmatch
// 1.0.3):
//   column reduction + reduction transfer      :124-176
//   augmenting row reduction (two passes)       :178-235, :265-269
//   shortest augmenting path + augmentation     :27-122, :237-258
// and the batch driver of cpu/ops.cpp:176-289 (virtual zero padding to
// K = max(N, M), +inf -> batch-global sentinel, column >= M -> -1).
#include <cuda_runtime.h>
#include <stdint.h>
#include <math.h>
#include <float.h>
#include <stdlib.h>
#include <string.h>

#include <mutex>

#include "torchmatch_b200.h"

namespace tmjv {
// blocks per SM of the statistics scan (several waves of 8 resident blocks
// measured faster than one: 5.3 against 4.6 TB/s on 1 GiB)
constexpr int kStatsBlocksPerSm = 32;

constexpr float kBig = 1e18f;  // LARGE_V<float>, jonker_dense_flat.h:22-23
constexpr unsigned kFull = 0xffffffffu;
constexpr int kMaxSlots = 8;   // K <= 256
constexpr uint32_t kWaitLimit = 1u << 26;  // bounded mbarrier wait

// Optional per-phase cycle counters (build with -DTMJV_PHASE_CLOCKS; the
// kernel then adds clock64() deltas into tmjv_phase_cycles[]).
#ifdef TMJV_PHASE_CLOCKS
__device__ unsigned long long tmjv_phase_cycles[24];
#define TMJV_T(name) const long long name = clock64()
#define TMJV_ACC(idx, t0)                                                            \
    do {                                                                             \
        if ((threadIdx.x & 31) == 0)                                                 \
            atomicAdd(&tmjv_phase_cycles[idx], (unsigned long long)(clock64() - (t0))); \
    } while (0)
#else
#define TMJV_T(name)
#define TMJV_ACC(idx, t0)
#endif

struct Params {
    const float *costs;
    int64_t B;
    int N, M, K;
    float sentinel;
    int sanitize;        // batch holds +inf cells
    int64_t *out;
    int32_t *status;
    unsigned long long *ticket;  // next unclaimed problem (zeroed per launch)
    tm_jv_stats *stats;          // check mode: batch statistics accumulate here
    // optional compacted outputs of jonker_dense_batch_unpacked (cpu/ops.cpp:290-417)
    int64_t *um;                 // (B, N, 2) matched (row, column) pairs
    int64_t *uur;                // (B, N) unmatched rows
    int64_t *uuc;                // (B, M) unmatched columns
    int64_t *unm;                // (B,) number of matches
    int check;                   // check mode: classify cells, bail on non-finite
    int compact;                 // jonker_compact_batch semantics (compact_core.h)
    int l2_prefetch;             // streaming mode: prefetch each claimed problem into L2
    int loop_bound;              // test hook: lower bound on the loop caps (0 = none)
    int gated;                   // run only if *stats shows +inf and no NaN / -inf;
                                 // the sentinel is then computed on the device
    // fused squared-Euclidean costs: x (B, N, D) and y (B, M, D) replace
    // `costs`; streaming shapes give each resident warp a slab of N * M
    // floats at slab + (global warp index) * slab_floats
    int points;          // costs come from x / y (px, py may be null when D == 0)
    const float *px;
    const float *py;
    int D;
    float *slab;
    int64_t slab_floats;
    int64_t slab_warps;  // slabs available in the workspace (host side)
    int warp_bytes;      // shared-memory bytes per warp
    int tile_floats;     // floats reserved for the staged tile (TILE mode)
    int bulk_ok;         // tile base and size are 16-byte multiples
    uint32_t wait_limit; // polls of a tile copy's mbarrier before it counts as timed out
};

// ------------------------------------------------------------- statistics
__device__ __forceinline__ uint32_t order_key(float f) {
    const uint32_t u = __float_as_uint(f);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__host__ __device__ inline float key_to_float(uint32_t k) {
    const uint32_t u = (k & 0x80000000u) ? (k & 0x7fffffffu) : ~k;
#ifdef __CUDA_ARCH__
    return __uint_as_float(u);
#else
    float f;
    memcpy(&f, &u, 4);
    return f;
#endif
}

// Cell classes and the largest finite cell, by integer selects (no branch:
// the classes differ between lanes).
__device__ __forceinline__ void classify(float x, uint32_t &fl, uint32_t &mk) {
    const uint32_t u = __float_as_uint(x);
    const uint32_t a = u & 0x7fffffffu;
    const bool finite = a < 0x7f800000u;
    const uint32_t nonfin = a > 0x7f800000u ? TM_STAT_NAN
                                           : ((u >> 31) ? TM_STAT_NEG_INF : TM_STAT_POS_INF);
    fl |= finite ? TM_STAT_FINITE : nonfin;
    mk = finite ? max(mk, order_key(x)) : mk;
}

// ---------------------------------------------------------------- warp ops
__device__ __forceinline__ float warp_min_f(float x) {
    float r;
    asm volatile("redux.sync.min.f32 %0, %1, %2;" : "=f"(r) : "f"(x), "r"(kFull));
    return r;
}
__device__ __forceinline__ unsigned warp_min_u(unsigned x) {
    return __reduce_min_sync(kFull, x);
}
__device__ __forceinline__ int warp_max_i(int x) { return __reduce_max_sync(kFull, x); }

// Ordered forms for the augmenting row reduction's step.  The step is one
// dependent chain through shared-memory loads and warp reductions, which go
// through one in-order pipe; written as volatile asm they keep the order
// given here, so every load on the chain is issued as soon as its address is
// known and no reduction whose result is needed later sits in front of it.
// They carry no memory clobber: around them, plain C++ accesses to the same
// arrays are fenced by __syncwarp(), which is a compiler barrier.
__device__ __forceinline__ unsigned warp_min_u_ord(unsigned x) {
    unsigned r;
    asm volatile("redux.sync.min.u32 %0, %1, %2;" : "=r"(r) : "r"(x), "r"(kFull));
    return r;
}
__device__ __forceinline__ int lds_s16(const int16_t *p) {
    int r;
    asm volatile("ld.shared.s16 %0, [%1];" : "=r"(r) : "r"((uint32_t)__cvta_generic_to_shared(p)));
    return r;
}
// `old`, or the 16-bit word at p when `pred` holds: one predicated load.
__device__ __forceinline__ int lds_s16_if(bool pred, const int16_t *p, int old) {
    int r;
    asm volatile(
        "{ .reg .pred q; setp.ne.b32 q, %2, 0; mov.b32 %0, %3; @q ld.shared.s16 %0, [%1]; }"
        : "=r"(r)
        : "r"((uint32_t)__cvta_generic_to_shared(p)), "r"((int)pred), "r"(old));
    return r;
}
__device__ __forceinline__ int lds_u8(const uint8_t *p) {
    int r;
    asm volatile("ld.shared.u8 %0, [%1];" : "=r"(r) : "r"((uint32_t)__cvta_generic_to_shared(p)));
    return r;
}
__device__ __forceinline__ float lds_f32(const float *p) {
    float r;
    asm volatile("ld.shared.f32 %0, [%1];" : "=f"(r) : "r"((uint32_t)__cvta_generic_to_shared(p)));
    return r;
}
__device__ __forceinline__ float2 lds_f32x2(const float2 *p) {
    float2 r;
    asm volatile("ld.shared.v2.f32 {%0, %1}, [%2];"
                 : "=f"(r.x), "=f"(r.y)
                 : "r"((uint32_t)__cvta_generic_to_shared(p)));
    return r;
}
__device__ __forceinline__ void sts_s16(int16_t *p, int x) {
    asm volatile("st.shared.u16 [%0], %1;" ::"r"((uint32_t)__cvta_generic_to_shared(p)),
                 "h"((unsigned short)x)
                 );
}
__device__ __forceinline__ void sts_s32(int32_t *p, int x) {
    asm volatile("st.shared.u32 [%0], %1;" ::"r"((uint32_t)__cvta_generic_to_shared(p)), "r"(x)
                 );
}
__device__ __forceinline__ void sts_f32(float *p, float x) {
    asm volatile("st.shared.f32 [%0], %1;" ::"r"((uint32_t)__cvta_generic_to_shared(p)), "f"(x)
                 );
}
// Row i of a square tile whose K is a multiple of 32 * VEC (no padding),
// VEC consecutive columns per lane and group, in issue order.
template <int S, int VEC>
__device__ __forceinline__ void lds_row_full(const float *tile, int i, int lane, float (&c)[S]) {
    const uint32_t base =
        (uint32_t)__cvta_generic_to_shared(tile + i * (32 * S) + lane * VEC);
#pragma unroll
    for (int g = 0; g < S / VEC; ++g) {
        const uint32_t a = base + g * 32 * VEC * 4;
        if constexpr (VEC == 4) {
            asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];"
                         : "=f"(c[g * 4]), "=f"(c[g * 4 + 1]), "=f"(c[g * 4 + 2]), "=f"(c[g * 4 + 3])
                         : "r"(a));
        } else if constexpr (VEC == 2) {
            asm volatile("ld.shared.v2.f32 {%0, %1}, [%2];"
                         : "=f"(c[g * 2]), "=f"(c[g * 2 + 1])
                         : "r"(a));
        } else {
            asm volatile("ld.shared.f32 %0, [%1];" : "=f"(c[g]) : "r"(a));
        }
    }
}

template <int S, int VEC>
struct Layout {
    static_assert(S % VEC == 0, "slots must be a multiple of the vector width");
    __device__ static __forceinline__ int col(int s, int lane) {
        return (s / VEC) * (32 * VEC) + lane * VEC + (s % VEC);
    }
    // columns are never negative here: unsigned math keeps these to shifts
    __device__ static __forceinline__ int lane_of(int j) {
        return (int)(((unsigned)j % (32u * VEC)) / VEC);
    }
    __device__ static __forceinline__ int slot_of(int j) {
        return (int)(((unsigned)j / (32u * VEC)) * VEC + ((unsigned)j % VEC));
    }
};

// Select a[s] for a warp-uniform runtime slot without local-memory indexing.
template <int S>
__device__ __forceinline__ float sel(const float (&a)[S], int s) {
    float r = a[0];
#pragma unroll
    for (int t = 1; t < S; ++t)
        if (s == t) r = a[t];
    return r;
}

template <int S>
__device__ __forceinline__ int seli(const int (&a)[S], int s) {
    int r = a[0];
#pragma unroll
    for (int t = 1; t < S; ++t)
        if (s == t) r = a[t];
    return r;
}
template <int S>
__device__ __forceinline__ void setf(float (&a)[S], int s, float x) {
#pragma unroll
    for (int t = 0; t < S; ++t)
        if (s == t) a[t] = x;
}
template <int S>
__device__ __forceinline__ void seti(int (&a)[S], int s, int x) {
#pragma unroll
    for (int t = 0; t < S; ++t)
        if (s == t) a[t] = x;
}

// --------------------------------------------------------- TMA primitives
__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ void bar_init(uint64_t *bar) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_u32(bar)));
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void bulk_load(void *dst, const void *src, uint32_t bytes,
                                          uint64_t *bar) {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
            "r"(smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}
__device__ __forceinline__ bool bar_wait(uint64_t *bar, uint32_t phase, uint32_t limit) {
    for (uint32_t it = 0; it < limit; ++it) {
        uint32_t done;
        asm volatile(
            "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; "
            "selp.u32 %0, 1, 0, p; }"
            : "=r"(done)
            : "r"(smem_u32(bar)), "r"(phase)
            : "memory");
        if (done) return true;
    }
    return false;
}
__device__ __forceinline__ void prefetch_l2(const void *src, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

// --------------------------------------------------------------- smem view
struct WarpShared {
    float *tile;       // staged (N, M) cost block (TILE mode)
    float *dist;       // d, mirrored for position-ordered access
    int32_t *xrow;     // x: column of each row
    int16_t *ycol;     // y: row of each column
    int16_t *pred;     // predecessor row of each column
    int16_t *queue;    // free-row queue
    int16_t *order;    // column permutation of the Dijkstra phase
    uint8_t *flag;     // per-row "single" bit / per-column event bits
    int32_t *evbuf;    // compacted events of one minimum search
    uint64_t *bar;     // mbarrier of the tile copy
    // row cache of the augmenting row reduction (streaming mode only)
    float *cval;       // [row][kCache]: cost value of each cached column
    uint8_t *ccol;     // [row][kCache]: the cached columns (K <= 256)
    float *cbound;     // [row]: lower bound of every uncached reduced cost
    float *vsh;        // mirror of the prices v (cached mode: the event buffer)
    // streamed rows: the column reduction's ring of kSlots slots of kChunk
    // rows, filled by TMA bulk copies (it shares the row-cache area, unused
    // until the augmenting row reduction), one mbarrier per slot, the parity
    // each slot waits for next, and whether a copy ever failed to land (then
    // the warp reads rows directly from then on)
    float *ring;
    uint64_t *rbar;
    uint32_t rphase;
    bool rdead;
};

constexpr int kCache = 6;  // cached columns per row
constexpr int kSlots = 3;  // slots of the column reduction's TMA ring
constexpr int kChunk = 2;  // rows per slot (one bulk copy)

__host__ __device__ inline int slots_for(int K) { return (K + 31) / 32; }

// Per-warp shared bytes: bookkeeping arrays for KP = 32 * S entries.  With
// the row cache (wide streamed rows), arrays whose phases never overlap share
// space, so 16 warps of K = 256 fit one SM: the price mirror of the row
// reduction lives in the event buffer of the Dijkstra phase, and the per-row
// / per-column flags (claim phase, Dijkstra phase) in the cache bounds of the
// row reduction.
__host__ __device__ inline int book_bytes(int KP, bool cache) {
    int b = KP * 4 /*dist*/ + KP * 4 /*xrow*/ + KP * 2 * 4 /*ycol,pred,queue,order*/ +
            KP * 4 /*evbuf*/ + 48 /*bar + alignment*/;
    if (cache) b += KP * kCache * 5 /*cval, ccol*/ + KP * 4 /*cbound*/ + 8 * kSlots + 8;
    else b += KP /*flag*/;
    return b;
}

__device__ inline WarpShared carve(unsigned char *base, int tile_floats, int KP, bool cache) {
    WarpShared w;
    unsigned char *p = base;
    w.tile = reinterpret_cast<float *>(p);
    p += (size_t)tile_floats * 4;
    w.dist = reinterpret_cast<float *>(p); p += KP * 4;
    w.xrow = reinterpret_cast<int32_t *>(p); p += KP * 4;
    w.ycol = reinterpret_cast<int16_t *>(p); p += KP * 2;
    w.pred = reinterpret_cast<int16_t *>(p); p += KP * 2;
    w.queue = reinterpret_cast<int16_t *>(p); p += KP * 2;
    w.order = reinterpret_cast<int16_t *>(p); p += KP * 2;
    if (!cache) { w.flag = p; p += KP; }
    p = reinterpret_cast<unsigned char *>((reinterpret_cast<uintptr_t>(p) + 15) & ~uintptr_t(15));
    w.evbuf = reinterpret_cast<int32_t *>(p); p += KP * 4;
    w.bar = reinterpret_cast<uint64_t *>(p);
    p += 16;
    w.cval = nullptr; w.ccol = nullptr; w.cbound = nullptr; w.vsh = nullptr;
    if (cache) {
        w.cval = reinterpret_cast<float *>(p); p += (size_t)KP * kCache * 4;
        w.ccol = p; p += (size_t)KP * kCache;
        w.cbound = reinterpret_cast<float *>(p); p += KP * 4;
        w.vsh = reinterpret_cast<float *>(w.evbuf);
        w.flag = reinterpret_cast<uint8_t *>(w.cbound);
        w.rbar = reinterpret_cast<uint64_t *>(p);
        // kSlots * kChunk rows of KP floats fit in the row-cache entries
        static_assert(kSlots * kChunk * 4 <= kCache * 5, "the ring must fit the row-cache area");
        w.ring = w.cval;
    } else {
        w.ring = nullptr;
        w.rbar = nullptr;
    }
    w.rphase = 0;
    w.rdead = false;
    return w;
}

// ------------------------------------------------------------ row access
// Reads row i of the virtual K x K matrix: real cells from `src` (row
// stride M), zeros in the padding (cpu/ops.cpp:262-270).  In streaming mode
// +inf cells become the sentinel here; in TILE mode the tile was already
// sanitised.
// Read-only loads of the input batch go through the non-coherent path.  Rows
// of a points slab (PTS) were written earlier in the same launch, which that
// path does not allow, so they are read with L2-only loads instead.
template <bool PTS, class T>
__device__ __forceinline__ T gload(const T *p) {
    if constexpr (PTS) return __ldcg(p);
    else return __ldg(p);
}

template <int S, int VEC, bool TILE, bool FULL, bool PTS = false>
__device__ __forceinline__ void load_row(const float *__restrict__ src, int i, int N, int M,
                                         int lane, bool sanitize, float sentinel,
                                         float (&c)[S]) {
    using L = Layout<S, VEC>;
    if constexpr (FULL) {
        // square, no padding, K a multiple of 32 * VEC: one aligned vector
        // load per group and no bounds checks
        const float *row = src + i * (32 * S) + lane * VEC;
#pragma unroll
        for (int g = 0; g < S / VEC; ++g) {
            const float *q = row + g * 32 * VEC;
            if constexpr (VEC == 4) {
                const float4 t = TILE ? *reinterpret_cast<const float4 *>(q)
                                      : gload<PTS>(reinterpret_cast<const float4 *>(q));
                c[g * 4 + 0] = t.x; c[g * 4 + 1] = t.y; c[g * 4 + 2] = t.z; c[g * 4 + 3] = t.w;
            } else if constexpr (VEC == 2) {
                const float2 t = TILE ? *reinterpret_cast<const float2 *>(q)
                                      : gload<PTS>(reinterpret_cast<const float2 *>(q));
                c[g * 2 + 0] = t.x; c[g * 2 + 1] = t.y;
            } else {
                c[g] = TILE ? *q : gload<PTS>(q);
            }
        }
        if constexpr (!TILE) {
            if (sanitize) {
#pragma unroll
                for (int s = 0; s < S; ++s)
                    if (isinf(c[s])) c[s] = sentinel;
            }
        }
        return;
    }
    if (i >= N) {
#pragma unroll
        for (int s = 0; s < S; ++s) c[s] = 0.0f;
        return;
    }
    const float *row = src + (size_t)i * M;
#pragma unroll
    for (int g = 0; g < S / VEC; ++g) {
        const int j0 = L::col(g * VEC, lane);
        if (j0 + VEC <= M) {
            if constexpr (VEC == 4) {
                float4 t;
                if constexpr (TILE) t = *reinterpret_cast<const float4 *>(row + j0);
                else t = gload<PTS>(reinterpret_cast<const float4 *>(row + j0));
                c[g * 4 + 0] = t.x; c[g * 4 + 1] = t.y; c[g * 4 + 2] = t.z; c[g * 4 + 3] = t.w;
            } else if constexpr (VEC == 2) {
                float2 t;
                if constexpr (TILE) t = *reinterpret_cast<const float2 *>(row + j0);
                else t = gload<PTS>(reinterpret_cast<const float2 *>(row + j0));
                c[g * 2 + 0] = t.x; c[g * 2 + 1] = t.y;
            } else {
                if constexpr (TILE) c[g] = row[j0];
                else c[g] = gload<PTS>(row + j0);
            }
        } else {
#pragma unroll
            for (int e = 0; e < VEC; ++e) {
                const int j = j0 + e;
                float val = 0.0f;
                if (j < M) {
                    if constexpr (TILE) val = row[j];
                    else val = gload<PTS>(row + j);
                }
                c[g * VEC + e] = val;
            }
        }
    }
    if constexpr (!TILE) {
        if (sanitize) {
#pragma unroll
            for (int s = 0; s < S; ++s)
                if (isinf(c[s])) c[s] = sentinel;
        }
    }
}

// Fused cost construction: cell (i, j) of one problem is
//   sum over d = 0 .. D-1, in that order, of (x[i][d] - y[j][d])^2
// in fp32, every subtraction, product and sum rounded on its own (no fused
// multiply-add), starting from 0.  That is the squared-Euclidean producer of
// the reference's lazy costs (transport/matrix/cpu/exact/
// network_simplex_simple.h:453-457) in single precision, so the solve sees
// exactly the matrix that a sequential fp32 producer would have written.
// Each lane owns kCols columns (lane + 32 t) per pass and accumulates their
// cells of one row in registers over all of D, then stores each cell once;
// the rows stream past with one broadcast load per coordinate of x.  With
// D <= 16 the lane's y points stay in registers for the whole pass;
// otherwise each 16-coordinate chunk is reloaded per row (L1-resident).
// +inf cells become the sentinel when the batch needs it (sanitize).  `dst`
// has row stride M.
template <int kCols>
__device__ void fill_points(float *dst, const float *__restrict__ x,
                            const float *__restrict__ y, int N, int M, int D, int lane,
                            bool sanitize, float sentinel) {
    constexpr int kDims = 16;
    const bool resident = D <= kDims;
    for (int j0 = 0; j0 < M; j0 += 32 * kCols) {
        float yv[kCols][kDims];
        auto load_y = [&](int d0, int dn) {
#pragma unroll
            for (int t = 0; t < kCols; ++t) {
                const int j = j0 + t * 32 + lane;
#pragma unroll
                for (int e = 0; e < kDims; ++e)
                    yv[t][e] = (j < M && e < dn) ? __ldg(y + (int64_t)j * D + d0 + e) : 0.0f;
            }
        };
        if (resident) load_y(0, D);
        for (int i = 0; i < N; ++i) {
            float acc[kCols];
#pragma unroll
            for (int t = 0; t < kCols; ++t) acc[t] = 0.0f;
            for (int d0 = 0; d0 < D; d0 += kDims) {
                const int dn = D - d0 < kDims ? D - d0 : kDims;
                if (!resident) load_y(d0, dn);
                const float *xr = x + (int64_t)i * D + d0;
#pragma unroll
                for (int e = 0; e < kDims; ++e)
                    if (e < dn) {
                        const float xe = __ldg(xr + e);
#pragma unroll
                        for (int t = 0; t < kCols; ++t) {
                            const float df = __fsub_rn(xe, yv[t][e]);
                            acc[t] = __fadd_rn(acc[t], __fmul_rn(df, df));
                        }
                    }
            }
            float *row = dst + (int64_t)i * M;
#pragma unroll
            for (int t = 0; t < kCols; ++t) {
                const int j = j0 + t * 32 + lane;
                if (j < M) row[j] = (sanitize && isinf(acc[t])) ? sentinel : acc[t];
            }
        }
    }
}

// The same cells for D a multiple of 16, latency-hidden: rows go in blocks
// of 8, and one block's x coordinates (one 16-coordinate chunk) arrive with
// 4 independent coalesced loads per lane -- lane l of load k holds
// coordinate l % 16 of row 2k + l / 16 -- and reach every lane by shuffles,
// instead of one dependent L2 round trip per row.  An 8-row x kCols block of
// sums stays in registers over all chunks, in coordinate order, so each cell
// is still the sequential fp32 sum and is stored once.
template <int kCols>
__device__ void fill_points16(float *dst, const float *__restrict__ x,
                              const float *__restrict__ y, int N, int M, int D, int lane,
                              bool sanitize, float sentinel) {
    constexpr int kRows = 8, kDims = 16;
    for (int j0 = 0; j0 < M; j0 += 32 * kCols) {
        float yv[kCols][kDims];
        for (int i0 = 0; i0 < N; i0 += kRows) {
            float acc[kRows][kCols];
#pragma unroll
            for (int r = 0; r < kRows; ++r)
#pragma unroll
                for (int t = 0; t < kCols; ++t) acc[r][t] = 0.0f;
            for (int d0 = 0; d0 < D; d0 += kDims) {
                if (d0 > 0 || i0 == 0 || D > kDims) {
#pragma unroll
                    for (int t = 0; t < kCols; ++t) {
                        const int j = j0 + t * 32 + lane;
#pragma unroll
                        for (int e = 0; e < kDims; ++e)
                            yv[t][e] = j < M ? __ldg(y + (int64_t)j * D + d0 + e) : 0.0f;
                    }
                }
                float xs[kRows / 2];
#pragma unroll
                for (int k = 0; k < kRows / 2; ++k) {
                    const int r = i0 + 2 * k + (lane >> 4);
                    xs[k] = r < N ? __ldg(x + (int64_t)r * D + d0 + (lane & 15)) : 0.0f;
                }
#pragma unroll
                for (int k = 0; k < kRows / 2; ++k)
#pragma unroll
                    for (int h = 0; h < 2; ++h)
#pragma unroll
                        for (int e = 0; e < kDims; ++e) {
                            const float xe = __shfl_sync(kFull, xs[k], h * 16 + e);
#pragma unroll
                            for (int t = 0; t < kCols; ++t) {
                                const float df = __fsub_rn(xe, yv[t][e]);
                                acc[2 * k + h][t] = __fadd_rn(acc[2 * k + h][t], __fmul_rn(df, df));
                            }
                        }
            }
#pragma unroll
            for (int r = 0; r < kRows; ++r) {
                if (i0 + r < N) {
                    float *row = dst + (int64_t)(i0 + r) * M;
#pragma unroll
                    for (int t = 0; t < kCols; ++t) {
                        const int j = j0 + t * 32 + lane;
                        if (j < M)
                            row[j] = (sanitize && isinf(acc[r][t])) ? sentinel : acc[r][t];
                    }
                }
            }
        }
    }
}

// Producer dispatch: the blocked form for D a positive multiple of 16.
template <int kCols>
__device__ __forceinline__ void fill_cells(float *dst, const float *__restrict__ x,
                                           const float *__restrict__ y, int N, int M, int D,
                                           int lane, bool sanitize, float sentinel) {
    if (D > 0 && D % 16 == 0)
        fill_points16<kCols>(dst, x, y, N, M, D, lane, sanitize, sentinel);
    else
        fill_points<kCols>(dst, x, y, N, M, D, lane, sanitize, sentinel);
}

// Writes one problem's result: the packed row -> column mapping (column >= M
// or unsolved -> -1, cpu/ops.cpp:274-283) and, when requested, the compacted
// form of jonker_dense_batch_unpacked (cpu/ops.cpp:378-414): matched pairs in
// row order, unmatched rows, unmatched columns in column order, the count,
// and -1 in every position past the counts.
__device__ void emit_result(const Params &P, WarpShared &w, int lane, int64_t b, int N, int M,
                            bool valid) {
    int64_t *ob = P.out ? P.out + b * (int64_t)N : nullptr;
    if (!P.um) {
        for (int r = lane; r < N; r += 32) {
            const int x = valid ? w.xrow[r] : -1;
            ob[r] = (x >= 0 && x < M) ? (int64_t)x : (int64_t)-1;
        }
        __syncwarp();
        return;
    }
    const unsigned lt = (1u << lane) - 1;
    for (int j = lane; j < M; j += 32) w.flag[j] = 0;
    __syncwarp();
    int64_t *mb = P.um + b * (int64_t)N * 2;
    int64_t *urb = P.uur + b * (int64_t)N;
    int64_t *ucb = P.uuc + b * (int64_t)M;
    int nm = 0, nu = 0;
    for (int r0 = 0; r0 < N; r0 += 32) {
        const int r = r0 + lane;
        int x = -1;
        if (r < N) {
            x = valid ? w.xrow[r] : -1;
            if (!(x >= 0 && x < M)) x = -1;
            if (ob) ob[r] = x;
        }
        const bool hit = r < N && x >= 0, miss = r < N && x < 0;
        const unsigned bh = __ballot_sync(kFull, hit), bm = __ballot_sync(kFull, miss);
        if (hit) {
            const int k = nm + __popc(bh & lt);
            mb[2 * k] = r;
            mb[2 * k + 1] = x;
            w.flag[x] = 1;
        }
        if (miss) urb[nu + __popc(bm & lt)] = r;
        nm += __popc(bh);
        nu += __popc(bm);
    }
    __syncwarp();
    int nc = 0;
    for (int j0 = 0; j0 < M; j0 += 32) {
        const int j = j0 + lane;
        const bool free_col = j < M && !w.flag[j];
        const unsigned bf = __ballot_sync(kFull, free_col);
        if (free_col) ucb[nc + __popc(bf & lt)] = j;
        nc += __popc(bf);
    }
    for (int k = nm + lane; k < N; k += 32) { mb[2 * k] = -1; mb[2 * k + 1] = -1; }
    for (int k = nu + lane; k < N; k += 32) urb[k] = -1;
    for (int k = nc + lane; k < M; k += 32) ucb[k] = -1;
    if (lane == 0) P.unm[b] = nm;
    __syncwarp();
}

// ------------------------------------------- augmenting row reduction
// The two passes of the augmenting row reduction (jonker_dense_flat.h:178-235,
// called twice at :265-269) for rows read directly (shared-memory tile, or
// streamed rows without the row cache).  Step semantics are those of the
// reference's scalar loop; the layout only shortens the dependent chain of
// one step, which bounds the phase:
//   * the prices v stay in the lanes' registers for the row scans and are
//     mirrored in shared memory (the event buffer of the Dijkstra phase is
//     free during this phase), as is the row of each column (ycol), so the
//     owner lookups of the chosen column are single broadcast loads;
//   * the second minimum waits for the first index instead of a tie ballot:
//     the lane holding column j1 offers its own second value, every other
//     lane its best one, so a second lane at v1 makes v2 = v1;
//   * the successor row of a lowering step (the previous owner of j1) is
//     loaded as soon as its index is known, ahead of the step's decisions,
//     and in TILE mode the next queued row is loaded ahead as well, so the
//     next step starts from registers whichever way the step decides;
//   * shared-memory accesses and reductions are volatile asm issued in the
//     order written, so no load on the chain waits behind a later one;
//   * a step commits through selects, not branches: the common step has no
//     branch but the loop's own.  The two rare cases -- a second value at or
//     above the initial LARGE, and a tie that switches the row to j2 --
//     leave the step uncommitted and end the fast loop; that step is then
//     run by the general code below it.
// Returns true when a pass hit its loop bound.
template <int S, int VEC, bool TILE, bool FULL, bool PTS>
__device__ __forceinline__ bool arr_direct(const float *__restrict__ src, const Params &P,
                                           WarpShared &w, int lane, int N, int M, int K,
                                           bool sanitize, float sentinel, const int (&jj)[S],
                                           unsigned valid, float (&v)[S], int &nfree) {
    // rows of a padding-free tile come through the ordered loads
    auto row_of = [&](int i, float (&c)[S]) {
        if constexpr (TILE && FULL) lds_row_full<S, VEC>(src, i, lane, c);
        else load_row<S, VEC, TILE, FULL, PTS>(src, i, N, M, lane, sanitize, sentinel, c);
    };
    // K a power of two: the speculative successor of a step whose column was
    // free (i0 = -1) is read from row K - 1 by a mask instead of a select
    constexpr bool kMask = TILE && FULL && (S & (S - 1)) == 0;
    float *vsh = reinterpret_cast<float *>(w.evbuf);
#pragma unroll
    for (int s = 0; s < S; ++s)
        if (valid >> s & 1) vsh[jj[s]] = v[s];
    __syncwarp();
    const bool compact = P.compact != 0;
    const float big2 = compact ? FLT_MAX : kBig;
    const float inf = __int_as_float(0x7f800000);
    bool failed = false;
    for (int pass = 0; pass < 2 && nfree > 0 && !failed; ++pass) {
        unsigned head = 0, visits = 0;
        int kept = 0;
        unsigned cap = compact ? 64u * (unsigned)K * (unsigned)K + 4096u
                               : (unsigned)K * (unsigned)K + 2u * K + 8u;
        if (P.loop_bound && (unsigned)P.loop_bound < cap) cap = (unsigned)P.loop_bound;
        const unsigned nf = (unsigned)nfree;
        int row = w.queue[0];
        // the queued row of the coming step (push-backs only write consumed
        // slots, so this slot is stable until it is consumed)
        int qnext = w.queue[1 < nf ? 1 : 0];
        float c[S];
        row_of(row, c);
        __syncwarp();
        while (head < nf && visits < cap) {
            // ---- fast steps.  A step commits only while the pass is live
            // (head < nf, visits below the cap) and the step before it was
            // not rare; the loop branch tests that flag, which is known at
            // the top of the step, so it never waits for the step's own
            // decisions.  A rare step commits nothing, so the step after it
            // repeats the same state without committing and the loop ends.
            bool rare = false, live;
            do {
                live = head < nf && visits < cap && !rare;
                const unsigned h1 = head + 1, vis1 = visits + 1;
                const int queued = qnext;
                // lane-local lexicographic (value, column) top-2; the slots
                // of a lane ascend in column.  Selects, not branches: the
                // comparisons differ between lanes.
                float a1 = c[0] - v[0], a2 = inf;
                int c1 = jj[0];
#pragma unroll
                for (int t = 1; t < S; ++t) {
                    const float x = c[t] - v[t];
                    const bool lt1 = x < a1;
                    a2 = lt1 ? a1 : fminf(a2, x);
                    a1 = lt1 ? x : a1;
                    c1 = lt1 ? jj[t] : c1;
                }
                const float v1 = warp_min_f(a1);
                const int j1 = (int)warp_min_u_ord(a1 == v1 ? (unsigned)c1 : 0xffffffffu);
                const int i0 = lds_s16(w.ycol + j1);
                const float vj1 = lds_f32(vsh + j1);
                const float v2 = warp_min_f(c1 == j1 ? a2 : a1);
                float cn[S], cq[S];
                if constexpr (kMask) row_of(i0 & (K - 1), cn);
                else row_of(i0 >= 0 ? i0 : row, cn);
                row_of(queued, cq);
                // rr_cnt < current * n (absent from the compact variant)
                const bool early = compact || vis1 < h1 * (unsigned)K;
                const float lowered = vj1 - (v2 - v1);
                const bool lowers = lowered < vj1;
                rare = !(v2 < big2) || (early && !lowers && i0 >= 0);
                const bool commit = live && !rare;
                const bool lower_now = early && lowers && commit;
                const bool push_front = i0 >= 0 && lower_now;
                const bool push_back = i0 >= 0 && !push_front && commit;
                // every lane stores the same words; a step that does not
                // commit stores the old values back (vsh, ycol) or a slot
                // past the kept entries (queue).  x is not kept here: it is
                // rebuilt from y when the phase ends.
                sts_f32(vsh + j1, lower_now ? lowered : vj1);
#pragma unroll
                for (int t = 0; t < S; ++t) v[t] = (lower_now && jj[t] == j1) ? lowered : v[t];
                sts_s16(w.ycol + j1, commit ? row : i0);
                sts_s16(w.queue + kept, i0);
                kept += push_back;
                head = commit ? h1 - push_front : head;
                visits = commit ? vis1 : visits;
                // the queued row moves on only after a step that consumed it
                qnext = lds_s16_if(commit && !push_front,
                                   w.queue + (h1 + 1 < nf ? h1 + 1 : 0), qnext);
#pragma unroll
                for (int t = 0; t < S; ++t) c[t] = commit ? (push_front ? cn[t] : cq[t]) : c[t];
                row = commit ? (push_front ? i0 : queued) : row;
            } while (live);
            // the loop ended at the pass end, or on a rare step (which then
            // runs below)
            if (!(head < nf && visits < cap)) break;
            // ---- one general step on `row` (uncommitted by the fast loop)
            __syncwarp();
            ++visits;
            ++head;
            const int queued = w.queue[head < nf ? head : 0];
            float a1 = c[0] - v[0], a2 = inf;
            int c1 = jj[0], c2 = 0x7fffffff;
#pragma unroll
            for (int t = 1; t < S; ++t) {
                const float x = c[t] - v[t];
                const bool lt1 = x < a1, lt2 = x < a2;
                a2 = lt1 ? a1 : (lt2 ? x : a2);
                c2 = lt1 ? c1 : (lt2 ? jj[t] : c2);
                a1 = lt1 ? x : a1;
                c1 = lt1 ? jj[t] : c1;
            }
            float v1 = warp_min_f(a1);
            int j1 = (int)warp_min_u(a1 == v1 ? (unsigned)c1 : 0xffffffffu);
            const bool mine = c1 == j1;
            const float bv = mine ? a2 : a1;
            const int bc = mine ? c2 : c1;
            float v2 = warp_min_f(bv);
            int j2 = -2;  // -2: not computed yet
            if (!(v2 < big2)) {
                // a reduced cost at or above LARGE: replay the scalar scan
                // of :193-210 exactly (not the plain top-2 then)
#pragma unroll
                for (int t = 0; t < S; ++t)
                    if (valid >> t & 1) w.dist[jj[t]] = c[t] - v[t];
                __syncwarp();
                int ja = 0, jb = -1;
                float va = 0.0f, vb = big2;
                if (lane == 0) {
                    va = w.dist[0];
                    for (int j = 1; j < K; ++j) {
                        const float t = w.dist[j];
                        if (t < vb) {
                            if (t >= va) { vb = t; jb = j; }
                            else { vb = va; jb = ja; va = t; ja = j; }
                        }
                    }
                }
                j1 = __shfl_sync(kFull, ja, 0);
                j2 = __shfl_sync(kFull, jb, 0);
                v1 = __shfl_sync(kFull, va, 0);
                v2 = __shfl_sync(kFull, vb, 0);
                __syncwarp();
            }
            int i0 = w.ycol[j1];
            const float vj1 = vsh[j1];
            const bool early = compact || visits < head * (unsigned)K;
            const float lowered = vj1 - (v2 - v1);
            const bool lowers = lowered < vj1;
            int jsel = j1;
            if (early && !lowers && i0 >= 0) {
                if (j2 == -2) j2 = (int)warp_min_u(bv == v2 ? (unsigned)bc : 0xffffffffu);
                if (j2 >= 0) {
                    jsel = j2;
                    i0 = w.ycol[j2];
                }
            }
            const bool lower_now = early && lowers;
            const bool push_front = i0 >= 0 && lower_now;
            const bool push_back = i0 >= 0 && !push_front;
            __syncwarp();
            if (lower_now) {
                vsh[j1] = lowered;
#pragma unroll
                for (int t = 0; t < S; ++t) v[t] = jj[t] == j1 ? lowered : v[t];
            }
            w.ycol[jsel] = (int16_t)row;
            if (push_back) w.queue[kept] = (int16_t)i0;
            kept += push_back;
            head -= push_front;
            row = push_front ? i0 : queued;
            __syncwarp();
            qnext = w.queue[head + 1 < nf ? head + 1 : 0];
            row_of(row, c);
            __syncwarp();
        }
#ifdef TMJV_PHASE_CLOCKS
        if (lane == 0) atomicAdd(&tmjv_phase_cycles[5], (unsigned long long)visits);
#endif
        if (head < nf) failed = true;  // loop bound reached
        nfree = kept;
        __syncwarp();
    }
    // x of every assigned row from y (x[i] = j exactly when y[j] = i).  Rows
    // left free keep a stale x, as in the reference: the augmentation reads
    // x only for rows that own a column (the free start row's x is read and
    // discarded, jonker_dense_flat.h:244-255).
#pragma unroll
    for (int s = 0; s < S; ++s)
        if (valid >> s & 1) {
            const int r = w.ycol[jj[s]];
            if (r >= 0) w.xrow[r] = jj[s];
        }
    __syncwarp();
    return failed;
}

// ------------------------------------------------------------- one solve
template <int S, int VEC, bool TILE, bool FULL, bool PTS>
__device__ void solve_problem(const float *__restrict__ src, const Params &P, WarpShared &w,
                              int lane, int64_t b) {
    using L = Layout<S, VEC>;
    // FULL: N == M == K == 32 * S, known at compile time
    const int K = FULL ? 32 * S : P.K;
    const int N = FULL ? 32 * S : P.N;
    const int M = FULL ? 32 * S : P.M;
    const bool sanitize = P.sanitize != 0;
    const float sentinel = P.sentinel;
    constexpr int KP = 32 * S;
    (void)KP;

    int jj[S];
    unsigned valid = 0;
#pragma unroll
    for (int s = 0; s < S; ++s) {
        jj[s] = L::col(s, lane);
        if (jj[s] < K) valid |= 1u << s;
    }
    if constexpr (FULL) valid = (1u << S) - 1;

    float v[S], d[S], c[S];
    bool failed = false;
    TMJV_T(t_col);

    // ---- column reduction (jonker_dense_flat.h:129-144) -------------------
    int ymin[S];
    uint32_t chk_fl = 0, chk_mk = 0;  // check mode: cell classes, max finite key
    // compact variant (jonker_compact_core.h:78-86) seeds each column with
    // row 0; a +inf seed with the same strict < gives exactly that
    const float seed = P.compact ? __int_as_float(0x7f800000) : kBig;
#pragma unroll
    for (int s = 0; s < S; ++s) { v[s] = seed; ymin[s] = 0; }
    bool ring_used = false;
    if constexpr (!TILE && !PTS && FULL && S >= 7) {
        // Streamed square rows: the rows arrive through a ring of kSlots
        // slots of kChunk rows in shared memory, each slot filled by one TMA
        // bulk copy (cp.async.bulk + mbarrier), so the next chunk is in flight
        // while the column minima of the current one are taken.  Chunk q (rows
        // q*kChunk ..) goes to slot q % kSlots.  K is a multiple of 32, so
        // every chunk is whole.
        if (P.bulk_ok && !w.rdead) {
            ring_used = true;
            constexpr int KP = 32 * S;
            constexpr int nchunk = KP / kChunk;
            constexpr uint32_t cb = (uint32_t)(kChunk * KP * 4);
            const bool check = P.check != 0;
            __syncwarp();  // the previous problem's reads of this area are done
            if (lane == 0) {
                for (int q = 0; q < kSlots && q < nchunk; ++q)
                    bulk_load(w.ring + q * (kChunk * KP), src + (int64_t)q * (kChunk * KP), cb,
                              w.rbar + q);
            }
            bool ok = true;
            int q = 0;
            for (; q < nchunk; ++q) {
                const int slot = q % kSlots;
                ok = __all_sync(kFull, bar_wait(w.rbar + slot, (w.rphase >> slot) & 1u,
                                                P.wait_limit));
                if (!ok) break;
                w.rphase ^= 1u << slot;
                const float *chunk = w.ring + slot * (kChunk * KP);
#pragma unroll
                for (int r = 0; r < kChunk; ++r) {
                    const int i = q * kChunk + r;
                    load_row<S, VEC, true, FULL, false>(chunk, r, N, M, lane, false, sentinel, c);
                    if (sanitize) {
#pragma unroll
                        for (int s = 0; s < S; ++s)
                            if (isinf(c[s])) c[s] = sentinel;
                    }
#pragma unroll
                    for (int s = 0; s < S; ++s) {
                        const bool lt = c[s] < v[s];
                        v[s] = lt ? c[s] : v[s];
                        ymin[s] = lt ? i : ymin[s];
                    }
                    if (check) {
#pragma unroll
                        for (int s = 0; s < S; ++s) classify(c[s], chk_fl, chk_mk);
                    }
                }
                __syncwarp();  // every lane has read the slot before it is refilled
                if (lane == 0 && q + kSlots < nchunk)
                    bulk_load(w.ring + slot * (kChunk * KP),
                              src + (int64_t)(q + kSlots) * (kChunk * KP), cb, w.rbar + slot);
            }
            if (!ok) {
                // A copy did not land in time: report it, let every copy in
                // flight (chunks q .. q + kSlots - 1) land before the area is
                // reused, and leave the problem as a row of -1.  If one never
                // lands, this warp stops using the ring.
                if (lane == 0 && P.status) atomicOr(P.status, (int32_t)TM_WS_TIMEOUT);
                for (int r = q; r < q + kSlots && r < nchunk; ++r) {
                    const int slot = r % kSlots;
                    if (__all_sync(kFull, bar_wait(w.rbar + slot, (w.rphase >> slot) & 1u,
                                                   kWaitLimit)))
                        w.rphase ^= 1u << slot;
                    else
                        w.rdead = true;
                }
                __syncwarp();
                emit_result(P, w, lane, b, N, M, false);
                return;
            }
        }
    }
    if (!ring_used) {
        const int nreal = N < K ? N : K;
        int i = 0;
        const bool check = P.check != 0;
        for (; i + 2 <= nreal; i += 2) {
            float c0[S], c1[S];
            load_row<S, VEC, TILE, FULL, PTS>(src, i, N, M, lane, sanitize, sentinel, c0);
            load_row<S, VEC, TILE, FULL, PTS>(src, i + 1, N, M, lane, sanitize, sentinel, c1);
#pragma unroll
            for (int s = 0; s < S; ++s) {
                if (c0[s] < v[s]) { v[s] = c0[s]; ymin[s] = i; }
                if (c1[s] < v[s]) { v[s] = c1[s]; ymin[s] = i + 1; }
            }
            if (check) {
#pragma unroll
                for (int s = 0; s < S; ++s)
                    if (FULL || jj[s] < M) {
                        classify(c0[s], chk_fl, chk_mk);
                        classify(c1[s], chk_fl, chk_mk);
                    }
            }
        }
        for (; i < nreal; ++i) {
            load_row<S, VEC, TILE, FULL, PTS>(src, i, N, M, lane, sanitize, sentinel, c);
#pragma unroll
            for (int s = 0; s < S; ++s)
                if (c[s] < v[s]) { v[s] = c[s]; ymin[s] = i; }
            if (check) {
#pragma unroll
                for (int s = 0; s < S; ++s)
                    if (FULL || jj[s] < M) classify(c[s], chk_fl, chk_mk);
            }
        }
        if (N < K) {  // first all-zero padding row; later ones never win (<)
#pragma unroll
            for (int s = 0; s < S; ++s)
                if (0.0f < v[s]) { v[s] = 0.0f; ymin[s] = N; }
        }
    }
    if (P.check) {
        // Check mode (no sentinel known yet): the column reduction above read
        // every real cell once and classified it.  A problem holding a NaN,
        // -inf or +inf cell stops here: its mapping needs the sentinel (and
        // NaN / -inf are rejected anyway), so the host re-runs the batch with
        // the sentinel or raises.
        const uint32_t fl = __reduce_or_sync(kFull, chk_fl);
        const uint32_t mk = __reduce_max_sync(kFull, chk_mk);
        if (lane == 0) {
            if (fl) atomicOr(&P.stats->flags, fl);
            if (mk) atomicMax(&P.stats->max_key, mk);
        }
        if (fl & (TM_STAT_NAN | TM_STAT_NEG_INF | TM_STAT_POS_INF)) {
            emit_result(P, w, lane, b, N, M, false);
            return;
        }
    }

    TMJV_ACC(1, t_col);
    TMJV_T(t_claim);
    // ---- claim: highest column wins its row (:145-155) -------------------
#pragma unroll
    for (int s = 0; s < S; ++s) {
        const int r = s * 32 + lane;
        if (r < K) { w.xrow[r] = -1; w.flag[r] = 1; }
    }
    __syncwarp();
#pragma unroll
    for (int s = 0; s < S; ++s)
        if (valid >> s & 1) atomicMax(&w.xrow[ymin[s]], jj[s]);
    __syncwarp();
#pragma unroll
    for (int s = 0; s < S; ++s) {
        if (valid >> s & 1) {
            const int r = ymin[s];
            int yv = r;
            if (w.xrow[r] != jj[s]) { w.flag[r] = 0; yv = -1; }
            w.ycol[jj[s]] = (int16_t)yv;
        }
    }
    __syncwarp();

    // Row of each column in registers of its owner lane; prices of the
    // padding lanes (column >= K) become -inf so their reduced costs are +inf.
    int yc[S];
#pragma unroll
    for (int s = 0; s < S; ++s) {
        yc[s] = (valid >> s & 1) ? (int)w.ycol[jj[s]] : -1;
        if (!(valid >> s & 1)) v[s] = -__int_as_float(0x7f800000);
    }

    // ---- free-row list and reduction transfer (:157-174) ------------------
    int nfree = 0;
    unsigned single_mask[S];
#pragma unroll
    for (int s = 0; s < S; ++s) {
        const int r = s * 32 + lane;
        const int xr = r < K ? w.xrow[r] : 0;
        const bool isfree = r < K && xr < 0;
        const bool single = r < K && xr >= 0 && w.flag[r];
        const unsigned bf = __ballot_sync(kFull, isfree);
        single_mask[s] = __ballot_sync(kFull, single);
        if (isfree) w.queue[nfree + __popc(bf & ((1u << lane) - 1))] = (int16_t)r;
        nfree += __popc(bf);
    }
#pragma unroll
    for (int s = 0; s < S; ++s) {
        unsigned m = single_mask[s];
        while (m) {
            const int i = s * 32 + __ffs(m) - 1;
            m &= m - 1;
            const int own = w.xrow[i];
            load_row<S, VEC, TILE, FULL, PTS>(src, i, N, M, lane, sanitize, sentinel, c);
            float loc = P.compact ? FLT_MAX : kBig;  // compact_core.h:104
#pragma unroll
            for (int t = 0; t < S; ++t)
                if (jj[t] != own) loc = fminf(loc, c[t] - v[t]);
            const float mn = warp_min_f(loc);
            if (lane == L::lane_of(own)) setf(v, L::slot_of(own), sel(v, L::slot_of(own)) - mn);
        }
    }
    // flags now serve as per-column event bits; they start cleared
#pragma unroll
    for (int s = 0; s < S; ++s) {
        const int r = s * 32 + lane;
        if (r < K) w.flag[r] = 0;
    }
    TMJV_ACC(2, t_claim);
    TMJV_T(t_arr);

    // ---- augmenting row reduction, at most two passes (:178-235) ----------
    // In streaming mode every visited row keeps a cache of its kCache best
    // columns and a lower bound on all the others.  Prices only fall during
    // this phase, so reduced costs only rise; while the second-best cached
    // value stays below the bound, the cached columns hold the exact
    // lexicographic top-2 of the row and the row need not be read again.
    constexpr bool kCached = !TILE;
    // only wide rows pay for the cache: with K < 192 a miss (row scan + top-5
    // extraction) costs more than the reads it saves (low hit rates on tied
    // or masked costs)
    // Cached mode: streaming rows with K > 192.  Prices and the row of each
    // column then live in shared memory only during this phase (lookups are
    // broadcast loads, updates single stores); the lane registers are
    // refreshed on misses and at the end of the phase.
    constexpr bool use_cache = kCached && S >= 7;
    // TILE rows: the ordered, branch-free step (arr_direct).  Streamed rows
    // keep the loop below, whose step waits on a global load anyway (the
    // ordered step measured slower there).
    if constexpr (TILE) {
        failed = arr_direct<S, VEC, TILE, FULL, PTS>(src, P, w, lane, N, M, K, sanitize,
                                                     sentinel, jj, valid, v, nfree);
    } else {
    if (use_cache) {
#pragma unroll
        for (int s = 0; s < S; ++s) {
            const int r = s * 32 + lane;
            if (r < K) {
                // no cache yet: a bound of -inf makes every lookup miss, and
                // column 0 keeps the (then unused) candidate loads in bounds
                w.cbound[r] = -__int_as_float(0x7f800000);
#pragma unroll
                for (int k = 0; k < kCache; ++k) {
                    w.cval[r * kCache + k] = 0.0f;
                    w.ccol[r * kCache + k] = 0;
                }
            }
            if (valid >> s & 1) w.vsh[jj[s]] = v[s];
        }
    }
    __syncwarp();
    // the two-min scan's initial second value: LARGE (jonker_dense_flat.h:196)
    // or FLT_MAX (compact_core.h:26); below it the scan is the plain top-2
    const float big2 = P.compact ? FLT_MAX : kBig;
    for (int pass = 0; pass < 2 && nfree > 0 && !failed; ++pass) {
        unsigned head = 0, visits = 0;
        int kept = 0;
        // the dense rule `rr_cnt < current * n` bounds the visits by K*K + K;
        // the compact variant has no such rule, so its bound is a safety net
        unsigned cap = P.compact ? 64u * (unsigned)K * (unsigned)K + 4096u
                                 : (unsigned)K * (unsigned)K + 2u * K + 8u;
        if (P.loop_bound && (unsigned)P.loop_bound < cap) cap = (unsigned)P.loop_bound;
        int row = w.queue[0];
        const unsigned nf = (unsigned)nfree;
        // cached mode: the queued row of the coming step, read ahead
        int qnext = w.queue[1 < nf ? 1 : 0];
        (void)qnext;
        while (head < (unsigned)nfree && visits < cap) {
            if constexpr (use_cache) {
                // ---- fast steps: a cache hit that needs neither the LARGE
                // replay nor the j2 switch, in the ordered, branch-free form
                // of arr_direct (prices and y are in shared memory here).
                // A step that is not such a hit commits nothing and ends the
                // fast loop; the general step below then runs it.
                const float inf = __int_as_float(0x7f800000);
                bool ok = true;
                do {
                    const unsigned h1 = head + 1, vis1 = visits + 1;
                    const int queued = qnext;
                    // every lane loads a candidate (lanes >= kCache repeat
                    // the first); only lanes < kCache offer theirs
                    const int ce = row * kCache + (lane < kCache ? lane : 0);
                    const float ex = lds_f32(w.cval + ce);
                    const int cj = lds_u8(w.ccol + ce);
                    const float cb = lds_f32(w.cbound + row);
                    const float vc = lds_f32(w.vsh + cj);
                    const float cv = lane < kCache ? ex - vc : inf;
                    const float v1 = warp_min_f(cv);
                    const int j1 = (int)warp_min_u_ord(cv == v1 ? (unsigned)cj : 0xffffffffu);
                    const int i0 = lds_s16(w.ycol + j1);
                    const float vj1 = lds_f32(w.vsh + j1);
                    const float v2 = warp_min_f(cj == j1 ? inf : cv);
                    const bool early = P.compact || vis1 < h1 * (unsigned)K;
                    const float lowered = vj1 - (v2 - v1);
                    const bool lowers = lowered < vj1;
                    ok = v2 < cb && v2 < big2 && !(early && !lowers && i0 >= 0);
                    const bool lower_now = early && lowers && ok;
                    const bool push_front = i0 >= 0 && lower_now;
                    const bool push_back = i0 >= 0 && !push_front && ok;
                    // the same words from every lane; a step that is not
                    // committed stores the old values back (vsh, ycol), a
                    // free slot (queue) or a word its general step rewrites
                    sts_f32(w.vsh + j1, lower_now ? lowered : vj1);
                    sts_s16(w.ycol + j1, ok ? row : i0);
                    sts_s32(w.xrow + row, j1);
                    sts_s16(w.queue + kept, i0);
                    kept += push_back;
                    head = ok ? h1 - push_front : head;
                    visits = ok ? vis1 : visits;
                    row = ok ? (push_front ? i0 : queued) : row;
                    qnext = lds_s16(w.queue + (head + 1 < nf ? head + 1 : 0));
                } while (ok && head < nf && visits < cap);
                __syncwarp();
                if (ok) break;  // the pass ended inside the fast loop
            }
#ifdef TMJV_PHASE_CLOCKS
            const long long t_gen = clock64();
#endif
            ++visits;
            ++head;
            // the next queued row; push-backs only write consumed slots
            const int queued = w.queue[head < (unsigned)nfree ? head : 0];
            float v1, v2, bv;
            int j1, bc;
            bool hit = false;
            if (use_cache) {
                float cv = __int_as_float(0x7f800000);
                int cj = 0x7fffffff;
                if (lane < kCache) {
                    cj = w.ccol[row * kCache + lane];
                    cv = w.cval[row * kCache + lane] - w.vsh[cj];
                }
                v1 = warp_min_f(cv);
                const bool at1 = cv == v1;
                const unsigned ties = __ballot_sync(kFull, at1);
                j1 = (int)warp_min_u(at1 ? (unsigned)cj : 0xffffffffu);
                // one candidate per lane: with two candidates at v1 the second
                // best is v1 itself, otherwise the best of the other lanes
                const float v2b = warp_min_f(at1 ? __int_as_float(0x7f800000) : cv);
                v2 = __popc(ties) > 1 ? v1 : v2b;
                bv = cj == j1 ? __int_as_float(0x7f800000) : cv;
                bc = cj;
                hit = v2 < w.cbound[row] && v2 < big2;
            }
            if (!hit) {
                load_row<S, VEC, TILE, FULL, PTS>(src, row, N, M, lane, sanitize, sentinel, c);
                if constexpr (use_cache) {
                    if constexpr (FULL && VEC == 4) {
                        // a lane's slots 4g .. 4g+3 are consecutive columns:
                        // one conflict-free 16-byte load per group
#pragma unroll
                        for (int g = 0; g < S / 4; ++g) {
                            const float4 q = *reinterpret_cast<const float4 *>(w.vsh + jj[4 * g]);
                            v[4 * g] = q.x; v[4 * g + 1] = q.y; v[4 * g + 2] = q.z; v[4 * g + 3] = q.w;
                        }
                    } else {
#pragma unroll
                        for (int t = 0; t < S; ++t)
                            if (valid >> t & 1) v[t] = w.vsh[jj[t]];
                    }
                    // lexicographic top-(kCache+1) by repeated extraction:
                    // ranks 0-1 answer this step, ranks 0..kCache-1 are
                    // cached, rank kCache bounds every uncached column
                    // reduced costs once; taken (and padding) slots turn +inf
                    // (a real reduced cost is finite), and each lane offers
                    // its first smallest slot by selects
                    float x[S];
#pragma unroll
                    for (int t = 0; t < S; ++t)
                        x[t] = (valid >> t & 1) ? c[t] - v[t] : __int_as_float(0x7f800000);
                    float rk[kCache + 1];
                    int jk[kCache + 1];
#pragma unroll
                    for (int k = 0; k <= kCache; ++k) {
                        float a = x[0];
                        int sa = 0;
#pragma unroll
                        for (int t = 1; t < S; ++t) {
                            const bool lt = x[t] < a;
                            a = lt ? x[t] : a;
                            sa = lt ? t : sa;
                        }
                        const bool any = a < __int_as_float(0x7f800000);
                        const int ja = any ? L::col(sa, lane) : 0x7fffffff;
                        const float m = warp_min_f(a);
                        const int jm = (int)warp_min_u(any && a == m ? (unsigned)ja : 0xffffffffu);
                        const bool won = ja == jm;
                        if (k < kCache && won) {
                            w.cval[row * kCache + k] = sel(c, sa);
                            w.ccol[row * kCache + k] = (uint8_t)jm;
                        }
#pragma unroll
                        for (int t = 0; t < S; ++t)
                            x[t] = (won && t == sa) ? __int_as_float(0x7f800000) : x[t];
                        rk[k] = m;
                        jk[k] = jm;
                    }
                    if (lane == 0) w.cbound[row] = rk[kCache];
                    v1 = rk[0];
                    j1 = jk[0];
                    v2 = rk[1];
                    bv = v2;  // the lazy j2 lookup below then yields rank 1
                    bc = jk[1];
                } else {
                    // lane-local lexicographic (value, column) top-2; the
                    // slots of a lane ascend in column
                    float a1 = c[0] - v[0], a2 = __int_as_float(0x7f800000);
                    int c1 = jj[0], c2 = 0x7fffffff;
#pragma unroll
                    for (int t = 1; t < S; ++t) {
                        // selects, not branches: the comparisons differ
                        // between lanes
                        const float x = c[t] - v[t];
                        const bool lt1 = x < a1, lt2 = x < a2;
                        a2 = lt1 ? a1 : (lt2 ? x : a2);
                        c2 = lt1 ? c1 : (lt2 ? jj[t] : c2);
                        a1 = lt1 ? x : a1;
                        c1 = lt1 ? jj[t] : c1;
                    }
                    v1 = warp_min_f(a1);
                    const bool at1 = a1 == v1;
                    const unsigned ties = __ballot_sync(kFull, at1);
                    j1 = (int)warp_min_u(at1 ? (unsigned)c1 : 0xffffffffu);
                    // the second best does not wait for j1: with two lanes at
                    // v1 it is v1 itself, else the lane at v1 offers its own
                    // second value
                    const float v2b = warp_min_f(at1 ? a2 : a1);
                    v2 = __popc(ties) > 1 ? v1 : v2b;
                    const bool mine = c1 == j1;
                    bv = mine ? a2 : a1;  // only read by the rare j2 lookup
                    bc = mine ? c2 : c1;
                }
            }
            int j2 = -2;  // -2: not computed yet
            // the owner lane's price and row of j1 are fetched before the rare
            // LARGE check, which would otherwise sit on the critical path
            int l1 = L::lane_of(j1), s1 = L::slot_of(j1);
            float vj1;
            int i0;
            if constexpr (use_cache) {
                vj1 = w.vsh[j1];
                i0 = w.ycol[j1];
            } else {
                vj1 = __shfl_sync(kFull, sel(v, s1), l1);
                i0 = __shfl_sync(kFull, seli(yc, s1), l1);
            }
            if (__builtin_expect(!(v2 < big2), 0)) {
                // a reduced cost at or above LARGE: replay the scalar scan
                // of :193-210 exactly (its result is not the plain top-2 then)
#pragma unroll
                for (int t = 0; t < S; ++t)
                    if (valid >> t & 1) w.dist[jj[t]] = c[t] - v[t];
                __syncwarp();
                int ja = 0, jb = -1;
                float va = 0.0f, vb = big2;
                if (lane == 0) {
                    va = w.dist[0];
                    for (int j = 1; j < K; ++j) {
                        const float t = w.dist[j];
                        if (t < vb) {
                            if (t >= va) { vb = t; jb = j; }
                            else { vb = va; jb = ja; va = t; ja = j; }
                        }
                    }
                }
                j1 = __shfl_sync(kFull, ja, 0);
                j2 = __shfl_sync(kFull, jb, 0);
                v1 = __shfl_sync(kFull, va, 0);
                v2 = __shfl_sync(kFull, vb, 0);
                __syncwarp();
                l1 = L::lane_of(j1);
                s1 = L::slot_of(j1);
                if constexpr (use_cache) {
                    vj1 = w.vsh[j1];
                    i0 = w.ycol[j1];
                } else {
                    vj1 = __shfl_sync(kFull, sel(v, s1), l1);
                    i0 = __shfl_sync(kFull, seli(yc, s1), l1);
                }
            }
            const float lowered = vj1 - (v2 - v1);
            const bool lowers = lowered < vj1;
            int jsel = j1;
            // rr_cnt < current * n (absent from the compact variant)
            const bool early = P.compact || visits < head * (unsigned)K;
            bool push_front = false, push_back = false;
            if (early && !lowers && i0 >= 0) {
                if (j2 == -2) j2 = (int)warp_min_u(bv == v2 ? (unsigned)bc : 0xffffffffu);
                if (j2 >= 0) {
                    jsel = j2;
                    if constexpr (use_cache) i0 = w.ycol[j2];
                    else i0 = __shfl_sync(kFull, seli(yc, L::slot_of(j2)), L::lane_of(j2));
                }
            }
            if (i0 >= 0) {
                push_front = early && lowers;
                push_back = !push_front;
            }
            // branch-free register updates of the owner lanes
            const bool own1 = early && lowers && lane == l1;
            const int ls = L::lane_of(jsel), ss = L::slot_of(jsel);
            if constexpr (use_cache) {
                if (early && lowers) w.vsh[j1] = lowered;  // same word from every lane
                w.ycol[jsel] = (int16_t)row;
            } else {
#pragma unroll
                for (int t = 0; t < S; ++t) {
                    v[t] = (own1 && t == s1) ? lowered : v[t];
                    yc[t] = (lane == ls && t == ss) ? row : yc[t];
                }
            }
            // every lane stores the same word: no divergent branch
            w.xrow[row] = jsel;
            if (push_back) w.queue[kept] = (int16_t)i0;
            kept += push_back;
            head -= push_front;
            row = push_front ? i0 : queued;
            // a hit only stores words that every lane writes itself; a miss
            // wrote per-lane cache entries that other lanes read later
            if (use_cache && !hit) __syncwarp();
            if constexpr (use_cache) {
                __syncwarp();
                qnext = w.queue[head + 1 < nf ? head + 1 : 0];
            }
#ifdef TMJV_PHASE_CLOCKS
            if (lane == 0) {
                atomicAdd(&tmjv_phase_cycles[17], 1ull);
                atomicAdd(&tmjv_phase_cycles[18], (unsigned long long)(clock64() - t_gen));
                atomicAdd(&tmjv_phase_cycles[19], hit ? 0ull : 1ull);
            }
#endif
        }
#ifdef TMJV_PHASE_CLOCKS
        if (lane == 0) atomicAdd(&tmjv_phase_cycles[5], (unsigned long long)visits);
#endif
        if (head < (unsigned)nfree) failed = true;  // loop bound reached
        nfree = kept;
        __syncwarp();
    }
    // the Dijkstra phase reads y through shared memory (and, in cached mode,
    // finds the prices there)
    if constexpr (use_cache) {
#pragma unroll
        for (int s = 0; s < S; ++s) {
            if (valid >> s & 1) v[s] = w.vsh[jj[s]];
            // the flags share the cache bounds' space: clear them again for
            // the Dijkstra phase's event bits
            const int r = s * 32 + lane;
            if (r < K) w.flag[r] = 0;
        }
    } else {
#pragma unroll
        for (int s = 0; s < S; ++s)
            if (valid >> s & 1) w.ycol[jj[s]] = (int16_t)yc[s];
    }
    }  // streamed rows
    __syncwarp();

    TMJV_ACC(3, t_arr);
    TMJV_T(t_sp);
    // ---- shortest augmenting paths (:75-122, :237-258) -------------------
    for (int f = 0; f < nfree && !failed; ++f) {
        const int start = w.queue[f];
        load_row<S, VEC, TILE, FULL, PTS>(src, start, N, M, lane, sanitize, sentinel, c);
        unsigned todo = valid, ready = 0, grp = 0;
#pragma unroll
        for (int s = 0; s < S; ++s) {
            d[s] = c[s] - v[s];
            if (valid >> s & 1) {
                w.dist[jj[s]] = d[s];
                w.pred[jj[s]] = (int16_t)start;
            }
            const int p = s * 32 + lane;
            if (p < K) w.order[p] = (int16_t)p;
        }
        __syncwarp();
        int lo = 0, hi = 0, sink = -1, iter = 0;
        float mind = 0.0f;
        const int icap = (P.loop_bound && P.loop_bound < 4 * K + 8) ? P.loop_bound : 4 * K + 8;
        while (sink < 0) {
            if (++iter > icap) { failed = true; break; }
            if (lo == hi) {
                // -- minimum search with the reference's swap pattern (:27-43)
                TMJV_T(t_find);
                __syncwarp();
                if (lo >= K) { failed = true; break; }
                ready |= grp;
                grp = 0;
                // Positions are scanned lane-major here (lane l holds
                // positions l*S .. l*S+S-1), so the running minimum inside a
                // lane is sequential and one warp scan of the lane minima
                // (plus one of the event counts) replaces S interleaved scans.
                const float inf = __int_as_float(0x7f800000);
                float dv[S];
#pragma unroll
                for (int s = 0; s < S; ++s) {
                    const int p = lane * S + s;
                    dv[s] = (p >= lo && p < K) ? w.dist[w.order[p < K ? p : 0]] : inf;
                }
                float lmin[S];
                lmin[0] = dv[0];
#pragma unroll
                for (int s = 1; s < S; ++s) lmin[s] = fminf(lmin[s - 1], dv[s]);
                float incl = lmin[S - 1];
#pragma unroll
                for (int off = 1; off < 32; off <<= 1) {
                    const float t = __shfl_up_sync(kFull, incl, off);
                    incl = lane >= off ? fminf(incl, t) : incl;
                }
                float before = __shfl_up_sync(kFull, incl, 1);
                before = lane == 0 ? inf : before;
                mind = __shfl_sync(kFull, incl, 31);
                // events: positions after lo whose d is at or below the
                // running minimum of the positions before them (:31-41)
                unsigned evb = 0, rsb = 0;
#pragma unroll
                for (int s = 0; s < S; ++s) {
                    const int p = lane * S + s;
                    const float excl = s == 0 ? before : fminf(before, lmin[s - 1]);
                    const bool live = p > lo && p < K;
                    evb |= (live && dv[s] <= excl) ? 1u << s : 0u;
                    rsb |= (live && dv[s] < excl) ? 1u << s : 0u;
                }
                int cnt = __popc(evb), off0 = cnt;
#pragma unroll
                for (int off = 1; off < 32; off <<= 1) {
                    const int t = __shfl_up_sync(kFull, off0, off);
                    off0 += lane >= off ? t : 0;
                }
                const int base = __shfl_sync(kFull, off0, 31);
                off0 -= cnt;
                {
                    // compact the events (position, original column, reset?)
                    // in position order; columns at event positions are
                    // untouched until their own event, so they are read here
#pragma unroll
                    for (int s = 0; s < S; ++s) {
                        if (evb >> s & 1) {
                            const int k = lane * S + s;
                            w.evbuf[off0] = k | ((int)w.order[k] << 9) | ((int)(rsb >> s & 1) << 18);
                            ++off0;
                        }
                    }
                    __syncwarp();
#ifdef TMJV_PHASE_CLOCKS
                    if (lane == 0) {
                        unsigned nr = 0;
                        nr = 0;
                        atomicAdd(&tmjv_phase_cycles[8], (unsigned long long)base);
                        atomicAdd(&tmjv_phase_cycles[9], (unsigned long long)nr);
                        atomicAdd(&tmjv_phase_cycles[10], 1ull);
                    }
#endif
                    int nh = lo + 1;
                    if (lane == 0 && base > 0) {
                        // replay :31-41 over the events only
                        int ev = w.evbuf[0];
                        for (int q = 0; q < base; ++q) {
                            const int evn = q + 1 < base ? w.evbuf[q + 1] : 0;
                            const int k = ev & 511;
                            const int16_t e = (int16_t)((ev >> 9) & 511);
                            // a reset restarts the group at lo
                            const int tgt = (ev >> 18) ? lo : nh;
                            w.order[k] = w.order[tgt];
                            w.order[tgt] = e;
                            nh = tgt + 1;
                            ev = evn;
                        }
                    }
                    nh = __shfl_sync(kFull, nh, 0);
                    hi = nh;
                }

                __syncwarp();
#pragma unroll
                for (int s = 0; s < S; ++s)
                    if ((todo >> s & 1) && d[s] == mind) grp |= 1u << s;
                todo &= ~grp;
                // last free column of the group, in group order (:107-111);
                // the compact variant takes the first (compact_core.h:195-201)
                int cand = -1, candf = 0x7fffffff;
#pragma unroll
                for (int s = 0; s < S; ++s) {
                    const int p = s * 32 + lane;
                    if (p >= lo && p < hi && w.ycol[w.order[p]] < 0) {
                        cand = p;
                        candf = min(candf, p);
                    }
                }
                int pbest;
                if (P.compact) {
                    pbest = (int)warp_min_u((unsigned)candf);
                    if (pbest == 0x7fffffff) pbest = -1;
                } else {
                    pbest = warp_max_i(cand);
                }
                TMJV_ACC(6, t_find);
                if (pbest >= 0) {
                    sink = w.order[pbest];
                    break;
                }
            }
            // -- relax the rows of the group, in group order (:45-73)
            TMJV_T(t_relax);
            while (lo != hi) {
                const int j = w.order[lo];
                ++lo;
                const int i = w.ycol[j];
                const float dj = w.dist[j];
                const int lj = L::lane_of(j), sj = L::slot_of(j);
                const float vj = __shfl_sync(kFull, sel(v, sj), lj);
                load_row<S, VEC, TILE, FULL, PTS>(src, i, N, M, lane, sanitize, sentinel, c);
                const float cij = __shfl_sync(kFull, sel(c, sj), lj);
                const float h = cij - vj - dj;
                unsigned ev = 0;
#pragma unroll
                for (int s = 0; s < S; ++s) {
                    // selects and predicated stores: the updates differ
                    // between lanes
                    const float rr = c[s] - v[s] - h;
                    const bool upd = (todo >> s & 1) && rr < d[s];
                    d[s] = upd ? rr : d[s];
                    if constexpr (!(FULL && VEC == 4)) {
                        if (upd) w.dist[jj[s]] = rr;
                    }
                    if (upd) w.pred[jj[s]] = (int16_t)i;
                    ev |= (upd && rr == dj) ? 1u << s : 0u;
                }
                if constexpr (FULL && VEC == 4) {
                    // a lane's four consecutive columns per group: one
                    // conflict-free 16-byte store of the mirror (unchanged
                    // entries are stored as they are)
#pragma unroll
                    for (int g = 0; g < S / 4; ++g)
                        *reinterpret_cast<float4 *>(w.dist + jj[4 * g]) =
                            make_float4(d[4 * g], d[4 * g + 1], d[4 * g + 2], d[4 * g + 3]);
                }
                if (!__any_sync(kFull, ev != 0)) continue;
                // tie events: order them by position
#pragma unroll
                for (int s = 0; s < S; ++s)
                    if (ev >> s & 1)
                        w.flag[jj[s]] = (uint8_t)(1 | (w.ycol[jj[s]] < 0 ? 2 : 0));
                __syncwarp();
                unsigned em[S], fm[S];
                int nev = 0;
#pragma unroll
                for (int s = 0; s < S; ++s) {
                    const int p = s * 32 + lane;
                    uint8_t fl = 0;
                    if (p >= hi && p < K) fl = w.flag[w.order[p]];
                    em[s] = __ballot_sync(kFull, fl & 1);
                    fm[s] = __ballot_sync(kFull, fl & 2);
                    nev += __popc(em[s]);
                }
                int first_free = -1;
#pragma unroll
                for (int s = 0; s < S; ++s)
                    if (first_free < 0 && fm[s]) first_free = s * 32 + __ffs(fm[s]) - 1;
                __syncwarp();
#pragma unroll
                for (int s = 0; s < S; ++s)
                    if (ev >> s & 1) w.flag[jj[s]] = 0;
                if (first_free >= 0) {
                    sink = w.order[first_free];
                    __syncwarp();
                    break;
                }
                {
                    int base = 0;
#pragma unroll
                    for (int s = 0; s < S; ++s) {
                        if (em[s] >> lane & 1) {
                            const int k = s * 32 + lane;
                            w.evbuf[base + __popc(em[s] & ((1u << lane) - 1))] =
                                k | ((int)w.order[k] << 9);
                        }
                        base += __popc(em[s]);
                    }
                    __syncwarp();
                    if (lane == 0) {
                        // replay :64-65 (move to the end of the ready group)
                        int nh = hi;
                        int cur = w.evbuf[0];
                        for (int q = 0; q < base; ++q) {
                            const int nxt = q + 1 < base ? w.evbuf[q + 1] : 0;
                            const int k = cur & 511;
                            w.order[k] = w.order[nh];
                            w.order[nh] = (int16_t)((cur >> 9) & 511);
                            ++nh;
                            cur = nxt;
                        }
                    }
                }
                hi += nev;
                grp |= ev;
                todo &= ~ev;
                __syncwarp();
            }
            TMJV_ACC(7, t_relax);
        }
        if (failed) break;
        // price update of the settled columns (:117-119)
#pragma unroll
        for (int s = 0; s < S; ++s)
            if (ready >> s & 1) v[s] = P.compact ? (v[s] + d[s]) - mind : v[s] + (d[s] - mind);
        // augmentation along the predecessor chain (:244-255)
        if (lane == 0) {
            int j = sink, steps = 0, i;
            do {
                i = w.pred[j];
                w.ycol[j] = (int16_t)i;
                const int prev = w.xrow[i];
                w.xrow[i] = j;
                j = prev;
                if (++steps >= K) break;
            } while (i != start);
        }
        __syncwarp();
    }

    TMJV_ACC(4, t_sp);
    // ---- output (cpu/ops.cpp:274-283) ------------------------------------
    __syncwarp();
    emit_result(P, w, lane, b, N, M, !failed);
    if (failed && lane == 0 && P.status) atomicOr(P.status, (int32_t)TM_WS_UNSOLVED);
}

// ------------------------------------------------------------------ kernel
template <int S, int VEC, bool TILE, bool FULL, bool PTS>
__global__ void __launch_bounds__((TILE || S > 4 || PTS) ? 512 : 384, (TILE || S > 4 || PTS) ? 1 : 3) jv_batch_kernel(const Params P0) {
    extern __shared__ __align__(128) unsigned char smem_raw[];
    const int lane = threadIdx.x & 31;
    Params P = P0;
    if (P.gated) {
        // second launch of the asynchronous path: the statistics of the
        // check-mode pass decide on the device whether a sentinel solve is
        // needed (cuda_common.cuh:245-254 without the host round trip)
        const uint32_t fl = *reinterpret_cast<volatile const uint32_t *>(&P.stats->flags);
        const uint32_t mk = *reinterpret_cast<volatile const uint32_t *>(&P.stats->max_key);
        if (blockIdx.x == 0 && threadIdx.x == 0) {
            int st = 0;
            if (fl & TM_STAT_NAN) st |= TM_WS_NAN;
            if (fl & TM_STAT_NEG_INF) st |= TM_WS_NEG_INF;
            if (st) atomicOr(P.status, st);
        }
        if (!(fl & TM_STAT_POS_INF) || (fl & (TM_STAT_NAN | TM_STAT_NEG_INF))) return;
        P.sentinel = (fl & TM_STAT_FINITE)
                         ? __fmul_rn(__fadd_rn(key_to_float(mk), 1.0f), (float)(P.K + 1))
                         : 1.0f;
        P.sanitize = 1;
    }
    const int warp = threadIdx.x >> 5;
    // the row-cache area (which also holds the column reduction's TMA ring)
    // exists for the wide streamed rows only
    WarpShared w = carve(smem_raw + (size_t)warp * P.warp_bytes, TILE ? P.tile_floats : 0, 32 * S,
                         !TILE && S >= 7);
    const int64_t per = (int64_t)P.N * P.M;
    const uint32_t tile_bytes = (uint32_t)(per * 4);
    uint32_t phase = 0;
    if constexpr (TILE) {
        if (lane == 0) bar_init(w.bar);
        __syncwarp();
    } else if constexpr (!PTS && FULL && S >= 7) {
        if (lane == 0)
            for (int r = 0; r < kSlots; ++r) bar_init(w.rbar + r);
        __syncwarp();
    }
    // Problems are claimed one at a time from a global ticket: the work per
    // problem is heavy-tailed, so a static split would leave warps idle
    // behind the unlucky ones.  The next ticket is taken before solving the
    // current problem so its tile can be prefetched into L2 meanwhile.
    auto claim = [&]() -> int64_t {
        unsigned long long t = 0;
        if (lane == 0) t = atomicAdd(P.ticket, 1ull);
        return (int64_t)__shfl_sync(kFull, t, 0);
    };
    // columns per lane in the cost producer: one above S = 6, where the
    // solver itself takes nearly all of the 128 registers a thread may use
    constexpr int kFillCols = S > 6 ? 1 : 2;
    int64_t b = claim();
    while (b < P.B) {
        const int64_t nb = claim();
        const float *g = P.costs + b * per;
        const float *src = g;
        TMJV_T(t_load);
        if constexpr (PTS && TILE) {
            // fused costs, TILE shape: build the problem in the tile itself
            fill_cells<kFillCols>(w.tile, P.px + b * (int64_t)P.N * P.D,
                                  P.py + b * (int64_t)P.M * P.D, P.N, P.M, P.D, lane,
                                  P.sanitize != 0, P.sentinel);
            __syncwarp();
            src = w.tile;
        } else if constexpr (PTS) {
            // fused costs, streaming shape: build the problem in this warp's slab
            float *slab =
                P.slab + ((int64_t)blockIdx.x * (blockDim.x >> 5) + warp) * P.slab_floats;
            fill_cells<kFillCols>(slab, P.px + b * (int64_t)P.N * P.D,
                                  P.py + b * (int64_t)P.M * P.D, P.N, P.M, P.D, lane,
                                  P.sanitize != 0, P.sentinel);
            __syncwarp();  // orders the lanes' slab stores before the row reads
            src = slab;
        } else if constexpr (TILE) {
            bool ok = true;
            if (P.bulk_ok) {
                if (lane == 0) bulk_load(w.tile, g, tile_bytes, w.bar);
                ok = bar_wait(w.bar, phase, P.wait_limit);
                if (!__all_sync(kFull, ok)) {
                    // The copy did not land in time: report it and leave the
                    // problem as a row of -1 rather than unwritten.  The copy
                    // in flight gets a second bounded wait before the tile
                    // may be reused; if it never lands, this warp issues no
                    // further copies and writes every problem it still
                    // claims as a row of -1.
                    if (lane == 0 && P.status) atomicOr(P.status, (int32_t)TM_WS_TIMEOUT);
                    const bool landed = __all_sync(kFull, bar_wait(w.bar, phase, kWaitLimit));
                    phase ^= 1u;
                    emit_result(P, w, lane, b, P.N, P.M, false);
                    if (!landed) {
                        for (int64_t q = nb; q < P.B; q = claim())
                            emit_result(P, w, lane, q, P.N, P.M, false);
                        return;
                    }
                    b = nb;
                    continue;
                }
                phase ^= 1u;
            } else {
                for (int64_t k = lane; k < per; k += 32) w.tile[k] = __ldg(g + k);
            }
            if (P.sanitize) {
                for (int64_t k = lane; k < per; k += 32)
                    if (isinf(w.tile[k])) w.tile[k] = P.sentinel;
            }
            __syncwarp();
            src = w.tile;
            if (P.bulk_ok && lane == 0 && nb < P.B) prefetch_l2(P.costs + nb * per, tile_bytes);
        } else {
            // streaming mode: pull the claimed problem's block into L2 up front
            // (when it is small enough for the resident set to stay there)
            if (P.l2_prefetch && P.bulk_ok && lane == 0) prefetch_l2(g, tile_bytes);
        }
        TMJV_ACC(0, t_load);
        solve_problem<S, VEC, TILE, FULL, PTS>(src, P, w, lane, b);
        b = nb;
    }
}

__global__ void __launch_bounds__(256) jv_stats_kernel(const float *__restrict__ x, int64_t n,
                                                       tm_jv_stats *out) {
    uint32_t fl = 0, mk = 0;
    const int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int64_t nth = (int64_t)gridDim.x * blockDim.x;
    const bool vec = (reinterpret_cast<uintptr_t>(x) & 15) == 0;
    int64_t done = 0;
    if (vec) {
        const int64_t n4 = n / 4;
        const float4 *x4 = reinterpret_cast<const float4 *>(x);
        // four independent 16-byte loads in flight per thread
        int64_t k = tid;
        for (; k + 3 * nth < n4; k += 4 * nth) {
            float4 t[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) t[u] = __ldg(x4 + k + u * nth);
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                classify(t[u].x, fl, mk); classify(t[u].y, fl, mk);
                classify(t[u].z, fl, mk); classify(t[u].w, fl, mk);
            }
        }
        for (; k < n4; k += nth) {
            const float4 t = __ldg(x4 + k);
            classify(t.x, fl, mk); classify(t.y, fl, mk);
            classify(t.z, fl, mk); classify(t.w, fl, mk);
        }
        done = n4 * 4;
    }
    for (int64_t k = done + tid; k < n; k += nth) classify(__ldg(x + k), fl, mk);
    fl = __reduce_or_sync(kFull, fl);
    mk = __reduce_max_sync(kFull, mk);
    if ((threadIdx.x & 31) == 0) {
        if (fl) atomicOr(&out->flags, fl);
        if (mk) atomicMax(&out->max_key, mk);
    }
}

// ------------------------------------------------------------ host launch
static thread_local int g_last_cuda = 0;
// test hook (tm_jv_debug_set_loop_bound): caps every solver loop
static int g_loop_bound = 0;
// test hook (tm_jv_debug_set_wait_limit): polls of a tile copy's mbarrier
// before the wait counts as timed out (-1: the production limit)
static long long g_wait_limit = -1;

static int cuda_fail(cudaError_t e) {
    g_last_cuda = (int)e;
    return TM_ERR_CUDA;
}

// Makes the device that owns `stream` current for the scope of a call, so the
// C ABI works whatever this runtime instance believes the current device is
// (the library links its own static CUDA runtime).
struct StreamDevice {
    int prev = -1;
    int dev = 0;
    cudaError_t err = cudaSuccess;
    explicit StreamDevice(cudaStream_t s) {
        cudaGetDevice(&prev);
        dev = prev;
        if (s != nullptr) {
            // cudaStreamGetDevice is refused while the stream is capturing;
            // a capturing stream belongs to the current device anyway
            cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
            if (cudaStreamIsCapturing(s, &cs) == cudaSuccess && cs != cudaStreamCaptureStatusNone)
                return;
            err = cudaStreamGetDevice(s, &dev);
            if (err == cudaSuccess && dev != prev) err = cudaSetDevice(dev);
        }
    }
    ~StreamDevice() {
        if (prev >= 0 && dev != prev) cudaSetDevice(prev);
    }
};

static int num_sms() {
    static int sms[64] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) dev = 0;
    if (!sms[dev]) {
        int v = 0;
        cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
        sms[dev] = v > 0 ? v : 148;
    }
    return sms[dev];
}

constexpr int kSmemLimit = 227 * 1024;

// Minimum number of resident warps per SM for the shared-memory tile mode
// (TM_JV_TILE_MIN_WARPS overrides the default of 4; 0 disables the mode).
// Prefetch of each claimed problem into L2 in streaming mode
// (TM_JV_L2_PREFETCH=0 disables it).
static int l2_prefetch_enabled() {
    static int v = -1;
    if (v < 0) {
        const char *e = getenv("TM_JV_L2_PREFETCH");
        v = (e && e[0] == '0') ? 0 : 1;
    }
    return v;
}

static int tile_min_warps() {
    static int v = -1;
    if (v < 0) {
        const char *e = getenv("TM_JV_TILE_MIN_WARPS");
        v = e ? atoi(e) : 4;
        if (v < 0) v = 4;
    }
    return v == 0 ? (1 << 20) : v;
}
constexpr int kMaxWarpsPerBlock = 16;

template <int S, int VEC, bool TILE, bool FULL, bool PTS = false>
static int launch_t(const Params &P0, cudaStream_t stream) {
    Params P = P0;
    const int KP = 32 * S;
    int tile_floats = 0;
    if (TILE) tile_floats = (int)(((int64_t)P.N * P.M + 31) / 32 * 32);
    int warp_bytes = tile_floats * 4 + book_bytes(KP, !TILE && S >= 7);
    warp_bytes = (warp_bytes + 127) & ~127;
    P.warp_bytes = warp_bytes;
    P.tile_floats = tile_floats;
    int wpb = kSmemLimit / warp_bytes;
    const int wcap = (TILE || S > 4 || PTS) ? kMaxWarpsPerBlock : 12;
    if (wpb > wcap) wpb = wcap;
    if (wpb < 1) return TM_ERR_TOO_LARGE;
    const int64_t need_warps = P.B;
    if ((int64_t)wpb > need_warps) wpb = (int)need_warps;
    if (PTS && !TILE && (int64_t)wpb > P.slab_warps) wpb = (int)P.slab_warps;  // one slab per warp
    if (wpb < 1) return TM_ERR_ARG;
    auto kern = jv_batch_kernel<S, VEC, TILE, FULL, PTS>;
    // The shared-memory opt-in and the occupancy queries run once per device
    // and launch shape, so a steady-state launch is just the kernel (nothing
    // that a CUDA graph capture would reject).  Streamed dense shapes pick
    // the block size that keeps the most warps resident: with 96 registers a
    // thread, 16 warps fill one 512-thread block while two blocks of 10 warps
    // fit (20 warps).
    struct Cached { int smem = -1, wpb_max = -1, wpb = 0, per_sm = 0; };
    static Cached cache[64];
    static std::mutex mu;
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) dev = 0;
    int per_sm = 0;
    {
        std::lock_guard<std::mutex> lock(mu);
        Cached &c = cache[dev];
        const int smem_max = wpb * warp_bytes;
        if (c.smem != smem_max || c.wpb_max != wpb) {
            cudaError_t e =
                cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_max);
            if (e != cudaSuccess) return cuda_fail(e);
            int best = wpb, best_per = 0;
            e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&best_per, kern, wpb * 32, smem_max);
            if (e != cudaSuccess) return cuda_fail(e);
            if (!TILE && !PTS) {
                for (int cand = wpb - 1; cand >= (wpb + 1) / 2; --cand) {
                    int per = 0;
                    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per, kern, cand * 32,
                                                                      cand * warp_bytes);
                    if (e != cudaSuccess) return cuda_fail(e);
                    if (cand * per > best * best_per) { best = cand; best_per = per; }
                }
            }
            c.smem = smem_max;
            c.wpb_max = wpb;
            c.wpb = best;
            c.per_sm = best_per;
        }
        wpb = c.wpb;
        per_sm = c.per_sm;
    }
    const int smem = wpb * warp_bytes;
    cudaError_t e;
    if (per_sm < 1) per_sm = 1;
    int64_t blocks = (P.B + wpb - 1) / wpb;
    const int64_t resident = (int64_t)num_sms() * per_sm;
    if (blocks > resident) blocks = resident;
    // one slab per resident warp: fewer slabs, fewer blocks
    if (PTS && !TILE && blocks * wpb > P.slab_warps) blocks = P.slab_warps / wpb;
    kern<<<(unsigned)blocks, wpb * 32, smem, stream>>>(P);
    e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e);
    return TM_OK;
}

// Picks the slot count, vector width and storage mode for a problem shape.
static int launch(Params P, cudaStream_t stream) {
    const int S = slots_for(P.K);
    const uintptr_t base = reinterpret_cast<uintptr_t>(P.costs);
    const int64_t per = (int64_t)P.N * P.M;
    P.bulk_ok = ((base & 15) == 0) && ((per * 4) % 16 == 0);
    // TILE mode while at least tile_min_warps() warps fit on one SM with
    // their tiles; larger matrices stream their rows from L2/HBM.
    const int64_t tile_bytes = ((per + 31) / 32 * 32) * 4 + book_bytes(32 * S, false);
    const bool tile = tile_bytes * tile_min_warps() <= kSmemLimit;
    const bool v4 = (P.M % 4 == 0) && (base % 16 == 0);
    const bool v2 = (P.M % 2 == 0) && (base % 8 == 0);
    // square problems with K a multiple of 32 take the padding-free path
    const bool full = P.N == P.M && P.M == 32 * S;
#define TM_L(SS, VV)                                                                     \
    return tile ? launch_t<SS, VV, true, false>(P, stream)                               \
                : launch_t<SS, VV, false, false>(P, stream)
#define TM_F(SS, VV)                                                                     \
    return tile ? launch_t<SS, VV, true, true>(P, stream)                                \
                : launch_t<SS, VV, false, true>(P, stream)
    if (P.points && tile) {
        // fused costs, TILE shape: rows come from the tile the kernel fills
#define TM_P(SS, VV, FF) return launch_t<SS, VV, true, FF, true>(P, stream)
        switch (S) {
        case 1: if (full) { TM_P(1, 1, true); } TM_P(1, 1, false);
        case 2: if (full) { TM_P(2, 2, true); } TM_P(2, 1, false);
        case 3: TM_P(3, 1, false);
        case 4: if (full) { TM_P(4, 4, true); } TM_P(4, 1, false);
        case 5: TM_P(5, 1, false);
        case 6: TM_P(6, 1, false);
        case 7: TM_P(7, 1, false);
        case 8: TM_P(8, 1, false);  // a square K = 256 tile never fits
        default: return TM_ERR_TOO_LARGE;
        }
#undef TM_P
    }
    if (P.points) {
        // fused costs, streaming shape: rows come from the warp slabs, which
        // are 256-byte aligned with row stride M
        const bool s4 = P.M % 4 == 0;
#define TM_P(SS, VV, FF) return launch_t<SS, VV, false, FF, true>(P, stream)
        switch (S) {
        case 4: if (full && s4) { TM_P(4, 4, true); } if (s4) { TM_P(4, 4, false); } TM_P(4, 1, false);
        case 5: TM_P(5, 1, false);
        case 6: TM_P(6, 1, false);
        case 7: TM_P(7, 1, false);
        case 8: if (full && s4) { TM_P(8, 4, true); } if (s4) { TM_P(8, 4, false); } TM_P(8, 1, false);
        default: return TM_ERR_ARG;  // K <= 96 always fits the tile
        }
#undef TM_P
    }
    switch (S) {
    case 1: if (full) { TM_F(1, 1); } TM_L(1, 1);
    case 2: if (full && v2) { TM_F(2, 2); } if (v2) { TM_L(2, 2); } TM_L(2, 1);
    case 3: TM_L(3, 1);
    case 4: if (full && v4) { TM_F(4, 4); } if (v4) { TM_L(4, 4); } TM_L(4, 1);
    case 5: TM_L(5, 1);
    case 6: if (v2) { TM_L(6, 2); } TM_L(6, 1);
    case 7: TM_L(7, 1);
    case 8: if (full && v4) { TM_F(8, 4); } if (v4) { TM_L(8, 4); } TM_L(8, 1);
    default: return TM_ERR_TOO_LARGE;
    }
#undef TM_L
#undef TM_F
}

// Fused squared-Euclidean inputs of one call (host side).
struct Points {
    const float *x;
    const float *y;
    int D;
    float *slab;
    int64_t slab_floats;
    int64_t slab_warps;
};

constexpr size_t kPointsHeader = 256;  // tm_jv_workspace, padded to the slab alignment

// Floats of one warp slab (a multiple of 64, so every slab is 256-byte aligned).
static int64_t points_slab_floats(int N, int M) {
    return ((int64_t)N * M + 63) / 64 * 64;
}

// Slabs a fused call of this shape uses on the current device: none for
// shapes solved in the shared-memory tile, else one per resident warp (an
// upper bound of the launch's residency: shared memory, the block size and
// the blocks per SM of the launch bounds).
static int64_t points_slabs(int64_t B, int N, int M) {
    const int K = N > M ? N : M;
    const int S = slots_for(K);
    const int64_t per = (int64_t)N * M;
    const int64_t tile_bytes = ((per + 31) / 32 * 32) * 4 + book_bytes(32 * S, false);
    if (tile_bytes * tile_min_warps() <= kSmemLimit || B <= 0) return 0;
    const int warp_bytes = (book_bytes(32 * S, S >= 7) + 127) & ~127;
    int wpb = kSmemLimit / warp_bytes;
    // the slab kernels launch like the wide ones: up to 16 warps, one block per SM
    if (wpb > kMaxWarpsPerBlock) wpb = kMaxWarpsPerBlock;
    if ((int64_t)wpb > B) wpb = (int)B;
    int per_sm = 1;
    const int fit = (228 * 1024) / (wpb * warp_bytes);
    if (fit < per_sm) per_sm = fit > 0 ? fit : 1;
    int64_t blocks = (B + wpb - 1) / wpb;
    const int64_t resident = (int64_t)num_sms() * per_sm;
    if (blocks > resident) blocks = resident;
    return blocks * wpb;
}

}  // namespace tmjv

// ====================================================================== C ABI
extern "C" {

int tm_jv_max_k(void) { return 32 * tmjv::kMaxSlots; }

void tm_jv_debug_set_loop_bound(int bound) { tmjv::g_loop_bound = bound > 0 ? bound : 0; }

void tm_jv_debug_set_wait_limit(int limit) { tmjv::g_wait_limit = limit < 0 ? -1 : limit; }

int tm_last_cuda_error(void) { return tmjv::g_last_cuda; }

const char *tm_status_string(int status) {
    switch (status) {
    case TM_OK: return "ok";
    case TM_ERR_NAN:
        return "cost matrix contains NaN; use +inf for forbidden pairs, NaN signals an upstream bug";
    case TM_ERR_NEG_INF: return "cost matrix contains -inf; -inf has no forbidden-edge meaning";
    case TM_ERR_ARG: return "invalid argument";
    case TM_ERR_CUDA: return "batched JV kernel launch failed (CUDA error)";
    case TM_ERR_TOO_LARGE: return "batched JV (CUDA) supports max(N, M) <= 256";
    case TM_ERR_UNSOLVED: return "a problem exceeded the solver's loop bound";
    case TM_ERR_TIMEOUT:
        return "batched JV kernel: a wait for a cost tile copy timed out (rows of -1 written)";
    default: return "unknown status";
    }
}

int tm_jv_stats_f32(const float *costs, int64_t count, tm_jv_stats *stats_dev,
                    tm_stream_t stream_) {
    cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);
    if (!stats_dev || count < 0 || (count > 0 && !costs)) return TM_ERR_ARG;
    tmjv::StreamDevice scope(stream);
    if (scope.err != cudaSuccess) return tmjv::cuda_fail(scope.err);
    cudaError_t e = cudaMemsetAsync(stats_dev, 0, sizeof(tm_jv_stats), stream);
    if (e != cudaSuccess) return tmjv::cuda_fail(e);
    if (count == 0) return TM_OK;
    const int threads = 256;
    int64_t blocks = (count / 4 + threads - 1) / threads;
    const int64_t cap = (int64_t)tmjv::num_sms() * tmjv::kStatsBlocksPerSm;
    if (blocks > cap) blocks = cap;
    if (blocks < 1) blocks = 1;
    tmjv::jv_stats_kernel<<<(unsigned)blocks, threads, 0, stream>>>(costs, count, stats_dev);
    e = cudaGetLastError();
    if (e != cudaSuccess) return tmjv::cuda_fail(e);
    return TM_OK;
}

int tm_jv_sentinel(const tm_jv_stats *st, int K, float *sentinel, int *has_pos_inf) {
    if (!st || !sentinel) return TM_ERR_ARG;
    if (st->flags & TM_STAT_NAN) return TM_ERR_NAN;
    if (st->flags & TM_STAT_NEG_INF) return TM_ERR_NEG_INF;
    if (has_pos_inf) *has_pos_inf = (st->flags & TM_STAT_POS_INF) ? 1 : 0;
    if (!(st->flags & TM_STAT_FINITE)) {
        *sentinel = 1.0f;
    } else {
        const float mx = tmjv::key_to_float(st->max_key);
        volatile float k1 = (float)(K + 1);  // fp32 product, no contraction
        *sentinel = (mx + 1.0f) * k1;
    }
    return TM_OK;
}

static int solve_impl(const float *costs, int64_t B, int N, int M, float sentinel,
                      int has_pos_inf, int check, int64_t *out, void *workspace,
                      tm_stream_t stream_, const tm_jv_unpacked *u = nullptr,
                      int gated = 0, int compact = 0, const tmjv::Points *pts = nullptr) {
    cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);
    if (B < 0 || N < 0 || M < 0) return TM_ERR_ARG;
    if (B == 0 || N == 0) return TM_OK;
    if ((!out && !u) || !workspace || (M > 0 && !costs && !pts)) return TM_ERR_ARG;
    if (u && (!u->matches || !u->unmatched_rows || !u->unmatched_cols || !u->n_matched))
        return TM_ERR_ARG;
    const int K = N > M ? N : M;
    if (K > 32 * tmjv::kMaxSlots) return TM_ERR_TOO_LARGE;
    tmjv::StreamDevice scope(stream);
    if (scope.err != cudaSuccess) return tmjv::cuda_fail(scope.err);
    tm_jv_workspace *ws = reinterpret_cast<tm_jv_workspace *>(workspace);
    // check mode starts the statistics from zero; a plain solve keeps them
    // check mode starts the statistics and status from zero; the gated
    // second launch keeps both and only resets the ticket
    void *zero_from = check ? static_cast<void *>(&ws->stats) : static_cast<void *>(&ws->ticket);
    const size_t zero_bytes = check ? sizeof(ws->stats) + sizeof(ws->ticket) + sizeof(ws->status)
                              : gated ? sizeof(ws->ticket)
                                      : sizeof(ws->ticket) + sizeof(ws->status);
    cudaError_t e = cudaMemsetAsync(zero_from, 0, zero_bytes, stream);
    if (e != cudaSuccess) return tmjv::cuda_fail(e);
    if (M == 0) {
        if (out) {
            e = cudaMemsetAsync(out, 0xff, sizeof(int64_t) * (size_t)B * N, stream);
            if (e != cudaSuccess) return tmjv::cuda_fail(e);
        }
        if (u) return TM_ERR_ARG;  // the unpacked op handles empty shapes itself
        return TM_OK;
    }
    tmjv::Params P{};
    P.costs = costs;
    P.B = B;
    P.N = N;
    P.M = M;
    P.K = K;
    P.sentinel = sentinel;
    P.sanitize = (has_pos_inf && !check) ? 1 : 0;
    P.check = check;
    P.compact = compact;
    P.gated = gated;
    P.l2_prefetch = tmjv::l2_prefetch_enabled();
    P.loop_bound = tmjv::g_loop_bound;
    P.wait_limit = tmjv::g_wait_limit < 0 ? tmjv::kWaitLimit : (uint32_t)tmjv::g_wait_limit;
    P.stats = &ws->stats;
    P.out = out;
    if (u) {
        P.um = u->matches;
        P.uur = u->unmatched_rows;
        P.uuc = u->unmatched_cols;
        P.unm = u->n_matched;
    }
    P.status = &ws->status;
    P.ticket = &ws->ticket;
    if (pts) {
        P.points = 1;
        P.px = pts->x;
        P.py = pts->y;
        P.D = pts->D;
        P.slab = pts->slab;
        P.slab_floats = pts->slab_floats;
        P.slab_warps = pts->slab_warps;
    }
    return tmjv::launch(P, stream);
}

int tm_jv_solve_f32(const float *costs, int64_t B, int N, int M, float sentinel,
                    int has_pos_inf, int64_t *out, void *workspace, tm_stream_t stream_) {
    return solve_impl(costs, B, N, M, sentinel, has_pos_inf, 0, out, workspace, stream_);
}

int tm_jv_solve_checked_f32(const float *costs, int64_t B, int N, int M, int64_t *out,
                            void *workspace, tm_stream_t stream_) {
    return solve_impl(costs, B, N, M, 0.0f, 0, 1, out, workspace, stream_);
}

size_t tm_jv_workspace_bytes(void) { return sizeof(tm_jv_workspace); }

// Copies the workspace header (statistics and status) back to the host in
// one transfer and waits for the stream: the single synchronisation of the
// synchronous entry points.
static int read_workspace(void *workspace, cudaStream_t stream, tm_jv_workspace *h) {
    cudaError_t e = cudaMemcpyAsync(h, workspace, sizeof(*h), cudaMemcpyDeviceToHost, stream);
    if (e != cudaSuccess) return tmjv::cuda_fail(e);
    e = cudaStreamSynchronize(stream);
    if (e != cudaSuccess) return tmjv::cuda_fail(e);
    return TM_OK;
}

// Return code of a finished synchronous call from its device status.  A tile
// copy that timed out is an error (its rows were written as -1).  Rows that a
// loop bound left as -1 are not: the reference's CPU solver maps a failed
// problem to a row of -1 the same way (cpu/ops.cpp:274-278); the status word
// still carries TM_WS_UNSOLVED for callers that read it.
static int status_code(int32_t status) {
    return (status & TM_WS_TIMEOUT) ? TM_ERR_TIMEOUT : TM_OK;
}

// Check-mode solve, one read-back of the verdict, and a sentinel re-solve
// only for a batch holding +inf (then read back again for its status).
// `status_out` (may be null) receives the final TM_WS_* bits.
static int full_op(const float *costs, int64_t B, int N, int M, int64_t *out,
                   void *workspace, tm_stream_t stream_, int compact,
                   int32_t *status_out = nullptr) {
    cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);
    if (B < 0 || N < 0 || M < 0) return TM_ERR_ARG;
    if (B == 0 || N == 0) return TM_OK;
    if (!out || !workspace) return TM_ERR_ARG;
    const int K = N > M ? N : M;
    if (K > tm_jv_max_k()) return TM_ERR_TOO_LARGE;
    if (M == 0) return solve_impl(costs, B, N, M, 0.0f, 0, 0, out, workspace, stream_);
    tmjv::StreamDevice scope(stream);
    if (scope.err != cudaSuccess) return tmjv::cuda_fail(scope.err);
    // one pass solves every all-finite problem and gathers the statistics
    int rc = solve_impl(costs, B, N, M, 0.0f, 0, 1, out, workspace, stream_, nullptr, 0, compact);
    if (rc) return rc;
    tm_jv_workspace h{};
    rc = read_workspace(workspace, stream, &h);
    if (rc) return rc;
    float sentinel = 1.0f;
    int pinf = 0;
    rc = tm_jv_sentinel(&h.stats, K, &sentinel, &pinf);
    if (rc) return rc;
    // +inf cells need the batch-global sentinel: solve again with it
    if (pinf) {
        rc = solve_impl(costs, B, N, M, sentinel, 1, 0, out, workspace, stream_, nullptr, 0,
                        compact);
        if (rc) return rc;
        rc = read_workspace(workspace, stream, &h);
        if (rc) return rc;
    }
    if (status_out) *status_out = h.status;
    return status_code(h.status);
}

int tm_jonker_dense_batch_f32(const float *costs, int64_t B, int N, int M, int64_t *out,
                              void *workspace, tm_stream_t stream_) {
    return full_op(costs, B, N, M, out, workspace, stream_, 0);
}

int tm_jonker_compact_batch_f32(const float *costs, int64_t B, int N, int M, int64_t *out,
                                void *workspace, tm_stream_t stream_) {
    return full_op(costs, B, N, M, out, workspace, stream_, 1);
}

int tm_jonker_dense_batch_async_f32(const float *costs, int64_t B, int N, int M,
                                    int64_t *out, void *workspace, tm_stream_t stream_) {
    if (B < 0 || N < 0 || M < 0) return TM_ERR_ARG;
    if (B == 0 || N == 0) return TM_OK;
    if (!out || !workspace) return TM_ERR_ARG;
    const int K = N > M ? N : M;
    if (K > tm_jv_max_k()) return TM_ERR_TOO_LARGE;
    int rc = solve_impl(costs, B, N, M, 0.0f, 0, 1, out, workspace, stream_);
    if (rc || M == 0) return rc;
    return solve_impl(costs, B, N, M, 0.0f, 0, 0, out, workspace, stream_, nullptr, 1);
}

static int full_unpacked(const float *costs, int64_t B, int N, int M,
                         const tm_jv_unpacked *u, void *workspace, tm_stream_t stream_,
                         int compact) {
    cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);
    if (B < 0 || N <= 0 || M <= 0) return B == 0 ? TM_OK : TM_ERR_ARG;
    if (B == 0) return TM_OK;
    if (!u || !workspace) return TM_ERR_ARG;
    const int K = N > M ? N : M;
    if (K > tm_jv_max_k()) return TM_ERR_TOO_LARGE;
    tmjv::StreamDevice scope(stream);
    if (scope.err != cudaSuccess) return tmjv::cuda_fail(scope.err);
    int rc = solve_impl(costs, B, N, M, 0.0f, 0, 1, nullptr, workspace, stream_, u, 0, compact);
    if (rc) return rc;
    tm_jv_workspace h{};
    rc = read_workspace(workspace, stream, &h);
    if (rc) return rc;
    float sentinel = 1.0f;
    int pinf = 0;
    rc = tm_jv_sentinel(&h.stats, K, &sentinel, &pinf);
    if (rc) return rc;
    if (pinf) {
        rc = solve_impl(costs, B, N, M, sentinel, 1, 0, nullptr, workspace, stream_, u, 0,
                        compact);
        if (rc) return rc;
        rc = read_workspace(workspace, stream, &h);
        if (rc) return rc;
    }
    return status_code(h.status);
}

int tm_jonker_dense_batch_unpacked_f32(const float *costs, int64_t B, int N, int M,
                                       const tm_jv_unpacked *u, void *workspace,
                                       tm_stream_t stream_) {
    return full_unpacked(costs, B, N, M, u, workspace, stream_, 0);
}

int tm_jonker_compact_batch_unpacked_f32(const float *costs, int64_t B, int N, int M,
                                         const tm_jv_unpacked *u, void *workspace,
                                         tm_stream_t stream_) {
    return full_unpacked(costs, B, N, M, u, workspace, stream_, 1);
}

size_t tm_jv_points_workspace_bytes(int64_t B, int N, int M) {
    if (B <= 0 || N <= 0 || M <= 0 || (N > M ? N : M) > tm_jv_max_k())
        return tmjv::kPointsHeader;
    return tmjv::kPointsHeader +
           (size_t)tmjv::points_slabs(B, N, M) * (size_t)tmjv::points_slab_floats(N, M) * 4;
}

int tm_jv_points_solve_f32(const float *x, const float *y, int64_t B, int N, int M, int D,
                           float sentinel, int has_pos_inf, int check, int64_t *out,
                           void *workspace, size_t workspace_bytes, tm_stream_t stream_) {
    cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);
    if (B < 0 || N < 0 || M < 0 || D < 0) return TM_ERR_ARG;
    if (B == 0 || N == 0) return TM_OK;
    if (!out || !workspace || workspace_bytes < tmjv::kPointsHeader) return TM_ERR_ARG;
    if ((reinterpret_cast<uintptr_t>(workspace) & 255) != 0) return TM_ERR_ARG;
    const int K = N > M ? N : M;
    if (K > tm_jv_max_k()) return TM_ERR_TOO_LARGE;
    if (M == 0)
        return solve_impl(nullptr, B, N, M, 0.0f, 0, check ? 1 : 0, out, workspace, stream_);
    if (D > 0 && (!x || !y)) return TM_ERR_ARG;
    tmjv::StreamDevice scope(stream);
    if (scope.err != cudaSuccess) return tmjv::cuda_fail(scope.err);
    tmjv::Points pts{x, y, D, nullptr, tmjv::points_slab_floats(N, M), 0};
    if (tmjv::points_slabs(B, N, M) > 0) {
        pts.slab = reinterpret_cast<float *>(static_cast<unsigned char *>(workspace) +
                                             tmjv::kPointsHeader);
        pts.slab_warps = (int64_t)((workspace_bytes - tmjv::kPointsHeader) / 4) / pts.slab_floats;
        if (pts.slab_warps < 1) return TM_ERR_ARG;
    }
    return check ? solve_impl(nullptr, B, N, M, 0.0f, 0, 1, out, workspace, stream_, nullptr, 0,
                              0, &pts)
                 : solve_impl(nullptr, B, N, M, sentinel, has_pos_inf, 0, out, workspace,
                              stream_, nullptr, 0, 0, &pts);
}

int tm_jonker_sqeuclidean_batch_f32(const float *x, const float *y, int64_t B, int N, int M,
                                    int D, int64_t *out, void *workspace,
                                    size_t workspace_bytes, tm_stream_t stream_) {
    cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);
    if (B < 0 || N < 0 || M < 0 || D < 0) return TM_ERR_ARG;
    if (B == 0 || N == 0 || M == 0)
        return tm_jv_points_solve_f32(x, y, B, N, M, D, 0.0f, 0, 0, out, workspace,
                                      workspace_bytes, stream_);
    const int K = N > M ? N : M;
    tmjv::StreamDevice scope(stream);
    if (scope.err != cudaSuccess) return tmjv::cuda_fail(scope.err);
    // check mode: every all-finite problem is solved and the statistics of
    // the computed cells are gathered in the same pass
    int rc = tm_jv_points_solve_f32(x, y, B, N, M, D, 0.0f, 0, 1, out, workspace,
                                    workspace_bytes, stream_);
    if (rc) return rc;
    tm_jv_workspace h{};
    rc = read_workspace(workspace, stream, &h);
    if (rc) return rc;
    float sentinel = 1.0f;
    int pinf = 0;
    rc = tm_jv_sentinel(&h.stats, K, &sentinel, &pinf);
    if (rc) return rc;
    // +inf cells (coordinates at +-inf) need the batch-global sentinel
    if (pinf) {
        rc = tm_jv_points_solve_f32(x, y, B, N, M, D, sentinel, 1, 0, out, workspace,
                                    workspace_bytes, stream_);
        if (rc) return rc;
        rc = read_workspace(workspace, stream, &h);
        if (rc) return rc;
    }
    return status_code(h.status);
}

}  // extern "C"

#ifdef TMJV_PHASE_CLOCKS
// Reads and clears the per-phase cycle counters (debug builds only).
extern "C" int tm_phase_read(unsigned long long *host8) {
    cudaDeviceSynchronize();
    cudaMemcpyFromSymbol(host8, tmjv::tmjv_phase_cycles, sizeof(unsigned long long) * 24);
    unsigned long long z[24] = {0};
    cudaMemcpyToSymbol(tmjv::tmjv_phase_cycles, z, sizeof(z));
    return 0;
}
#endif

// ============================================= allocation-free entry point
// Scratch of tm_jonker_dense_batch_f32_noalloc: one tm_jv_workspace (64
// bytes) per GPU that loads this library, held until the process exits.
// Host code must not pass `g_noalloc_workspace` itself to a kernel (on the
// host it names a stand-in, not device memory); it asks the runtime for the
// device address once per device.
static __device__ __align__(256) tm_jv_workspace g_noalloc_workspace;


namespace {
std::mutex g_noalloc_mu;
void *g_noalloc_ptr[64] = {nullptr};
}  // namespace

extern "C" int tm_jonker_dense_batch_f32_noalloc(const float *costs, int64_t B, int N, int M,
                                                 int64_t *out, tm_stream_t stream_) {
    cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);
    if (B < 0 || N < 0 || M < 0) return TM_ERR_ARG;
    if (B == 0 || N == 0) return TM_OK;
    if (!out || (M > 0 && !costs)) return TM_ERR_ARG;
    if ((N > M ? N : M) > tm_jv_max_k()) return TM_ERR_TOO_LARGE;
    tmjv::StreamDevice scope(stream);  // the stream's device is current from here on
    if (scope.err != cudaSuccess) return tmjv::cuda_fail(scope.err);
    if (scope.dev < 0 || scope.dev >= 64) return TM_ERR_ARG;
    void *ws = nullptr;
    {
        std::lock_guard<std::mutex> lock(g_noalloc_mu);
        if (!g_noalloc_ptr[scope.dev]) {
            void *p = nullptr;
            const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_workspace);
            if (e != cudaSuccess) return tmjv::cuda_fail(e);
            g_noalloc_ptr[scope.dev] = p;
        }
        ws = g_noalloc_ptr[scope.dev];
    }
    // the regular op body zeroes the statistics, ticket and status, and
    // hands back the final status word: this caller has no other way to
    // read it, so rows left -1 by a loop bound come back as TM_ERR_UNSOLVED
    int32_t status = 0;
    const int rc = full_op(costs, B, N, M, out, ws, stream_, 0, &status);
    if (rc) return rc;
    return (status & TM_WS_UNSOLVED) ? TM_ERR_UNSOLVED : TM_OK;
}
