// FS-B shared device helpers: forest arena indexing and the fixed-order ("halving") reductions every FS-B kernel uses.
#pragma once
#include "common.cuh"

#define FSB_CLUSTER_K 9        // chunks of 2^9 cells and more are built by a thread-block cluster
#define FSB_SMALL_K 5          // chunks of up to 2^5 cells are built in shared memory by the small-chunk kernel
#define FSB_MAX_MCAP 16384     // largest supported cell capacity per row (room for 262 144 tokens plus decode growth)
#define FSB_MAX_CHUNK 8192     // largest chunk the build kernel takes (a chunk of 16 384 cells needs 524 288 admitted tokens)
#define FSB_AUX 4              // floats per node in node_aux
#define FSB_ROOT_PAD 4         // floats after the D mean words of a root32 row (radius + 3 pad)

__host__ __device__ __forceinline__ int fsb_log2(int x) {
    int l = 0;
    while ((1 << l) < x) ++l;
    return l;
}
// Two arenas. Full (compact = 0): every aligned even-j chunk has its own place, so a prefill can name the forest of any
// earlier prefix. Compact (compact = 1): one place per chunk HEIGHT (the reference's decode arena, fsb_tree.py:1496-1522): a
// new chunk of height k is completed exactly when bit k of the admitted count turns on, i.e. when no chunk of that height is
// alive, so the place is free; only the current prefix can be named, which is all a decode step asks.
#define FSB_COMPACT_ROOTS 32   // rows of root32 per forest row in the compact arena (one per height)
// first node id of the chunks of height k inside a row's arena
__host__ __device__ __forceinline__ int64_t fsb_nbase(int k, int m_cap) {
    return (int64_t)k * m_cap - m_cap + (m_cap >> k);
}
__host__ __device__ __forceinline__ int64_t fsb_root_node(int k, int j, int m_cap, int compact = 0) {
    if (compact) return (int64_t)(2 << k) - 2 - k;                        // sum of the sizes 2^{k'+1} - 1 of the lower heights
    return fsb_nbase(k, m_cap) + (int64_t)(j >> 1) * ((2 << k) - 1);
}
__host__ __device__ __forceinline__ int fsb_chunk_id(int k, int j, int m_cap, int compact = 0) {
    return compact ? k : m_cap - (m_cap >> k) + (j >> 1);
}
// nodes per row: full arena (k_cap + 1) m_cap; compact = 1: 4 m_cap (room for every height a row of m_cap cells can have);
// compact > 1: a compact arena of exactly `compact` nodes per row, sized by the caller for the admitted counts it can reach
__host__ __device__ __forceinline__ int64_t fsb_nodes_per_row(int m_cap, int compact = 0) {
    return compact > 1 ? (int64_t)compact : compact ? 4 * (int64_t)m_cap : (int64_t)(fsb_log2(m_cap) + 1) * m_cap;
}
// nodes a compact arena needs for chunks up to height kt: the places of heights 0..kt, sum of 2^{k+1} - 1
__host__ __device__ __forceinline__ int64_t fsb_compact_nodes(int kt) { return ((int64_t)4 << kt) - 3 - kt; }
// most cells a row may admit: m_cap, and in a sized compact arena no count that would need a height without a place
__host__ __device__ __forceinline__ int fsb_admit_limit(int m_cap, int compact) {
    if (compact <= 1) return m_cap;
    int kt = 0;
    while (kt < 30 && fsb_compact_nodes(kt + 1) <= (int64_t)compact) ++kt;
    const int64_t lim = ((int64_t)2 << kt) - 1;                          // all heights 0..kt alive
    return lim < m_cap ? (int)lim : m_cap;
}
__host__ __device__ __forceinline__ int64_t fsb_root_rows(int m_cap, int compact = 0) { return compact ? FSB_COMPACT_ROOTS : m_cap; }

// ---- halving-order sum over the head dimension, one warp per vector ------------------------------------------------
// Lane L holds the values of dims L, L+32, L+64, L+96 (zero beyond D). The order is that of repeated halving over the
// dimension padded to a power of two: x[i] + x[i + n/2], n = DP, DP/2, ..., 2. Every lane returns the same bits.
template <int D>
struct FsbDim {
    static constexpr int DP = (D <= 64) ? 64 : 128;
    static constexpr int NPL = DP / 32;
};

template <int D>
__device__ __forceinline__ float fsb_warp_det_sum(const float (&v)[FsbDim<D>::NPL]) {
    float a;
    if constexpr (FsbDim<D>::NPL == 2) {
        a = f_add(v[0], v[1]);
    } else {
        a = f_add(f_add(v[0], v[2]), f_add(v[1], v[3]));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) a = f_add(a, __shfl_xor_sync(FS_FULL, a, o));
    return a;
}

template <int D>
__device__ __forceinline__ void fsb_load_row(const float* row, int lane, float (&v)[FsbDim<D>::NPL]) {
#pragma unroll
    for (int i = 0; i < FsbDim<D>::NPL; ++i) {
        const int d = lane + 32 * i;
        v[i] = (d < D) ? row[d] : 0.0f;
    }
}
template <int D>
__device__ __forceinline__ void fsb_store_row(float* row, int lane, const float (&v)[FsbDim<D>::NPL]) {
#pragma unroll
    for (int i = 0; i < FsbDim<D>::NPL; ++i) {
        const int d = lane + 32 * i;
        if (d < D) row[d] = v[i];
    }
}

// ---- halving-order sum of D values held by ONE thread (beam / re-rank dot products) -------------------------------------
template <int D>
__device__ __forceinline__ float fsb_thread_det_sum(float (&p)[FsbDim<D>::DP]) {
#pragma unroll
    for (int h = FsbDim<D>::DP / 2; h > 0; h >>= 1) {
#pragma unroll
        for (int i = 0; i < h; ++i) p[i] = f_add(p[i], p[i + h]);
    }
    return p[0];
}
