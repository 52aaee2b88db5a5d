// Dense FS selection of one decode token: the query of every (b,h) scores all cells completed before its query block
// (4096 at 131k tokens: 1 MB of fp32 mean keys per head, HBM/L2-bound) and keeps the kk best by (score desc, cell asc).
// `splits` CTAs per (b,h) form a cluster and take contiguous ranges of cells; 8 lanes share a cell's mean key (16-byte
// loads), every group leader keeps a sorted top-4 of its own cells, and the lists meet in three merges: per CTA in shared
// memory, then in rank 0's shared memory through distributed shared memory. Its output feeds the decode-step kernel's
// ext_sel, exactly as the FS-B selection does.
#include <cooperative_groups.h>

#include "common.cuh"

namespace cg = cooperative_groups;

namespace {

constexpr int DD_WARPS = 8;

// (score, cell) order: score descending, then cell ascending; empty entries (cell -1, score -inf) last
__device__ __forceinline__ bool dd_before(float sa, int ca, float sb, int cb) {
    return sa > sb || (sa == sb && ca >= 0 && (cb < 0 || ca < cb));
}

struct DTop4 {
    float s[4];
    int c[4];
    __device__ __forceinline__ void init() {
#pragma unroll
        for (int i = 0; i < 4; i++) { s[i] = -INFINITY; c[i] = -1; }
    }
    __device__ __forceinline__ void insert(float sv, int cv) {
        if (!dd_before(sv, cv, s[3], c[3])) return;
        s[3] = sv; c[3] = cv;
#pragma unroll
        for (int i = 3; i > 0; i--) {
            if (dd_before(s[i], c[i], s[i - 1], c[i - 1])) {
                const float ts = s[i]; s[i] = s[i - 1]; s[i - 1] = ts;
                const int tc = c[i]; c[i] = c[i - 1]; c[i - 1] = tc;
            }
        }
    }
};

// the best 4 of the warp's 32 x 4 entries, returned in every lane (one warp)
__device__ __forceinline__ void dd_warp_top4(DTop4& mine, float* out_s, int* out_c) {
    int head = 0;                                   // my list is sorted: my best remaining entry is mine.s[head]
#pragma unroll
    for (int k = 0; k < 4; k++) {
        float bs = -INFINITY; int bc = -1;
#pragma unroll
        for (int i = 0; i < 4; i++) if (i == head) { bs = mine.s[i]; bc = mine.c[i]; }
        // order-preserving map float -> uint, then the best score and, among its holders, the lowest cell
        const uint32_t bits = __float_as_uint(bs);
        const uint32_t key = (bits & 0x80000000u) ? ~bits : (bits | 0x80000000u);
        const uint32_t kmax = __reduce_max_sync(FS_FULL, key);
        const uint32_t cmin = __reduce_min_sync(FS_FULL, (key == kmax && bc >= 0) ? (uint32_t)bc : 0x7fffffffu);
        const bool any = kmax > 0x007fffffu && cmin != 0x7fffffffu;     // -inf maps to 0x007fffff
        out_s[k] = any ? bs : -INFINITY;
        // every lane needs the winning score: the winner broadcasts it
        const unsigned who = __ballot_sync(FS_FULL, any && key == kmax && (uint32_t)bc == cmin);
        const int src = who ? __ffs(who) - 1 : 0;
        out_s[k] = any ? __shfl_sync(FS_FULL, bs, src) : -INFINITY;
        out_c[k] = any ? (int)cmin : -1;
        if (any && key == kmax && (uint32_t)bc == cmin) head++;
    }
}

template <int D>
__global__ void __launch_bounds__(DD_WARPS * 32) fs_dense_decode_select_kernel(const fsattn_fs_dense_decode_select_t a) {
    constexpr int F = D / 8;                       // floats per lane when 8 lanes share a mean key
    cg::cluster_group cluster = cg::this_cluster();
    const int S = (int)gridDim.x, rank = (int)blockIdx.x, bh = blockIdx.y;
    const int b = bh / a.H, h = bh - b * a.H;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, s8 = lane & 7, ci = lane >> 3;
    __shared__ float ws[DD_WARPS * 4][4];
    __shared__ int wc[DD_WARPS * 4][4];
    __shared__ float cs[8][4];                     // rank 0: the CTAs' lists
    __shared__ int cc[8][4];

    if (S > 1) cluster.barrier_arrive();           // "every CTA of the cluster has started"
    const int64_t pos = *a.pos;
    const int blk_start = (int)((pos / a.Bq) * a.Bq);
    int m_vis = blk_start / FSATTN_CELL;
    if (m_vis > a.ncell_cap) m_vis = a.ncell_cap;
    if (m_vis < 0) m_vis = 0;
    int chunk = (m_vis + S - 1) / S;
    chunk = (chunk + 3) & ~3;
    const int c_lo = rank * chunk, c_hi = min(m_vis, c_lo + chunk);
    const float lam = a.lam[h];
    const float two_sigma = f_mul(2.0f, a.sigma[h]);
    const float* kbar = a.kbar + b * a.kbar_sb + h * a.kbar_sh;
    const float* ceil = a.ceil + b * a.ceil_sb + h * a.ceil_sh;

    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    const bf16* q = (const bf16*)a.q + b * a.q_sb + h * a.q_sh;
    float qv[F];
#pragma unroll
    for (int j = 0; j < F; j++) qv[j] = __bfloat162float(q[s8 * F + j]);
    const float qpos = (float)pos;

    DTop4 T;
    T.init();
    // Four groups of cells per trip, every load issued before the first use: the hardware issues in order, so a loop body
    // "load a mean key, score it" would pay one memory round trip per group, one after the other.
    constexpr int DU = 4;
    for (int c0 = c_lo + warp * 4; c0 < c_hi; c0 += DD_WARPS * 4 * DU) {
        float4 kv[DU][F / 4];
        float ce[DU];
#pragma unroll
        for (int u = 0; u < DU; u++) {
            const int cell = c0 + u * DD_WARPS * 4 + ci;
            const bool ok = cell < c_hi;
            const float4* kr = reinterpret_cast<const float4*>(kbar + (int64_t)(ok ? cell : c_lo) * D + s8 * F);
#pragma unroll
            for (int j = 0; j < F / 4; j++) kv[u][j] = kr[j];
            ce[u] = ceil[ok ? cell : c_lo];
        }
#pragma unroll
        for (int u = 0; u < DU; u++) {
            const int cell = c0 + u * DD_WARPS * 4 + ci;
            const bool ok = cell < c_hi;
            float dot = 0.0f;
#pragma unroll
            for (int j = 0; j < F / 4; j++) {
                dot = fmaf(qv[4 * j + 0], kv[u][j].x, dot); dot = fmaf(qv[4 * j + 1], kv[u][j].y, dot);
                dot = fmaf(qv[4 * j + 2], kv[u][j].z, dot); dot = fmaf(qv[4 * j + 3], kv[u][j].w, dot);
            }
            dot += __shfl_xor_sync(FS_FULL, dot, 1);
            dot += __shfl_xor_sync(FS_FULL, dot, 2);
            dot += __shfl_xor_sync(FS_FULL, dot, 4);
            if (ok && s8 == 0) {
                const float prior = fs_prior(lam, ce[u], qpos, cell, (float)FSATTN_CELL, two_sigma);
                T.insert(f_add(f_mul(dot, a.scale), prior), cell);
            }
        }
    }
    if (s8 == 0) {
#pragma unroll
        for (int i = 0; i < 4; i++) { ws[warp * 4 + ci][i] = T.s[i]; wc[warp * 4 + ci][i] = T.c[i]; }
    }
    __syncthreads();
    float rs[4]; int rc[4];
    if (warp == 0) {                               // the CTA's list: lane l owns the l-th leader's sorted four
        DTop4 M;
#pragma unroll
        for (int i = 0; i < 4; i++) { M.s[i] = ws[lane][i]; M.c[i] = wc[lane][i]; }
        dd_warp_top4(M, rs, rc);
    }
    if (S > 1) {
        cluster.barrier_wait();                    // rank 0 is running: its shared memory may be written
        if (warp == 0 && lane < 4) {
            float* ds = cluster.map_shared_rank(&cs[rank][0], 0);
            int* dc = cluster.map_shared_rank(&cc[rank][0], 0);
            ds[lane] = rs[lane]; dc[lane] = rc[lane];
        }
        cluster.sync();
        if (rank == 0 && warp == 0) {
            DTop4 M;
            M.init();
            if (lane < S) {
#pragma unroll
                for (int i = 0; i < 4; i++) { M.s[i] = cs[lane][i]; M.c[i] = cc[lane][i]; }
            }
            dd_warp_top4(M, rs, rc);
        }
    }
    if (rank == 0 && warp == 0 && lane < a.kk) a.sel[(int64_t)bh * a.kk + lane] = lane < 4 ? rc[lane] : -1;
}

template <int D>
int launch_dd(const fsattn_fs_dense_decode_select_t* a, cudaStream_t st) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(a->splits, a->B * a->H, 1);
    cfg.blockDim = dim3(DD_WARPS * 32, 1, 1);
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = a->splits; attr[0].val.clusterDim.y = 1; attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = a->pdl ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, fs_dense_decode_select_kernel<D>, *a);
    if (e != cudaSuccess) {
        (void)cudaGetLastError();
        fs_set_error("fs_dense_decode_select: launch failed: %s", cudaGetErrorString(e));
        return FSATTN_ELAUNCH;
    }
    return FSATTN_OK;
}

}  // namespace

extern "C" int fsattn_fs_dense_decode_select(const fsattn_fs_dense_decode_select_t* a, fsattn_stream_t stream) {
    FS_REQUIRE(a != nullptr && a->q && a->kbar && a->ceil && a->lam && a->sigma && a->pos && a->sel, "fs_dense_decode_select: null pointer");
    FS_REQUIRE(a->B > 0 && a->H > 0 && a->Bq > 0 && a->Bq % FSATTN_CELL == 0 && a->ncell_cap >= 0, "fs_dense_decode_select: bad sizes");
    FS_UNSUPPORTED(a->D != 64 && a->D != 96 && a->D != 128, "fs_dense_decode_select: head_dim %d not in {64,96,128}", a->D);
    FS_REQUIRE(a->kk >= 1 && a->kk <= 4, "fs_dense_decode_select: kk = %d (1..4)", a->kk);
    FS_REQUIRE(a->splits == 1 || a->splits == 2 || a->splits == 4 || a->splits == 8, "fs_dense_decode_select: splits %d not in {1,2,4,8}", a->splits);
    FS_REQUIRE(((uintptr_t)a->kbar & 15) == 0 && a->kbar_sb % 4 == 0 && a->kbar_sh % 4 == 0, "fs_dense_decode_select: kbar must be 16-byte aligned");
    cudaStream_t st = (cudaStream_t)stream;
    switch (a->D) {
        case 64: return launch_dd<64>(a, st);
        case 96: return launch_dd<96>(a, st);
        default: return launch_dd<128>(a, st);
    }
}
