// Dense FS selection of a prefill (the variant without a candidate pool): every query scores EVERY completed cell that ends
// at or before its 128-query block, score = (q . Kbar_c) * scale + lam * ceil_c * erf(|p - (c + 0.5) s| / (2 sigma)), and
// keeps the kk best by (score desc, cell asc). At 131k tokens a block sees up to 4096 cells, so the dot products are a real
// contraction: 128 queries x 64 cells x 64 dims per tile on the 5th-generation tensor cores.
//
//   pass 0 (dense_prep_kernel): Kbar fp32 (bf16-exact values) -> bf16 rows, and lam * ceil per cell, into the workspace
//   pass 1 (fs_dense_select_kernel), one CTA per (query block, batch*head), heaviest blocks first:
//        S = Q Kbar^T   tcgen05.mma 128x64x64 (4 k-steps) into one of two TMEM accumulators, operands staged by TMA
//        warps 0-3: one query per thread reads its 64 scores (tcgen05.ld), adds the prior and keeps a sorted top-4 in
//        registers. The prior needs erf only for cells within 8 sigma of the query (erf is 1 in fp32 beyond 4 = x / (2 sigma));
//        for every other cell it is the per-cell constant lam * ceil, read from shared memory.
// Warp 4 is the TMA producer, warp 5 issues the MMAs. Every mbarrier wait is bounded; a timeout is counted in *status.
#include "tc_common.cuh"

namespace {

constexpr int DS_BN = 64;            // cells per tile
constexpr int DS_D = 64;
constexpr int DS_THREADS = 192;
constexpr int DS_SEL_THREADS = 128;
constexpr int DS_STAGES = 4;
constexpr int DS_TMEM_COLS = 128;    // S0 | S1
constexpr int DS_TILE_BYTES = DS_BN * DS_D * 2;
constexpr int DS_LC_BYTES = DS_BN * 4;

constexpr int DSM_Q = 0;
constexpr int DSM_K = 16384;
constexpr int DSM_LC = DSM_K + DS_STAGES * DS_TILE_BYTES;
constexpr int DSM_BAR = DSM_LC + DS_STAGES * DS_LC_BYTES;
constexpr int DSM_TOTAL = DSM_BAR + 128;

enum { DB_Q = 0, DB_FULL = 1, DB_EMPTY = DB_FULL + DS_STAGES, DB_S_FULL = DB_EMPTY + DS_STAGES, DB_S_FREE = DB_S_FULL + 2,
       DB_COUNT = DB_S_FREE + 2 };
static_assert(DB_COUNT * 8 <= 128, "mbarrier area");

__device__ __forceinline__ void bulk_1d(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                 ::"r"(s_u32(dst)), "l"(src), "r"(bytes), "r"(s_u32(bar)) : "memory");
}

// ---- pass 0 -------------------------------------------------------------------------------------------------------------
__global__ void __launch_bounds__(256) dense_prep_kernel(const fsattn_fs_dense_select_t a, bf16* kb16, float* lc, int ncell_pad) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;           // one thread per 8 dims of a cell
    const int64_t total = (int64_t)a.B * a.H * a.ncell * (DS_D / 8);
    if (i >= total) return;
    const int e = (int)(i % (DS_D / 8));
    const int64_t row = i / (DS_D / 8);
    const int c = (int)(row % a.ncell);
    const int64_t bh = row / a.ncell;
    const int b = (int)(bh / a.H), h = (int)(bh - (int64_t)b * a.H);
    const float* src = a.kbar + b * a.kbar_sb + h * a.kbar_sh + (int64_t)c * DS_D + e * 8;
    const float4 x0 = reinterpret_cast<const float4*>(src)[0], x1 = reinterpret_cast<const float4*>(src)[1];
    uint4 o;
    o.x = pack_bf2(x0.x, x0.y); o.y = pack_bf2(x0.z, x0.w); o.z = pack_bf2(x1.x, x1.y); o.w = pack_bf2(x1.z, x1.w);
    reinterpret_cast<uint4*>(kb16 + row * DS_D)[e] = o;
    if (e == 0) lc[bh * ncell_pad + c] = f_mul(a.lam[h], a.ceil[b * a.ceil_sb + h * a.ceil_sh + c]);
}

struct DsParams {
    int N, H, ncell, ncell_pad, nb, Bq, kk;
    float scale;
    const float* sigma;
    const float* lc;
    int32_t* sel;
    int32_t* status;
};

// sorted top-4 of one query: scores descending; among equal scores the smaller cell first (cells arrive in ascending order)
struct Top4 {
    float s0, s1, s2, s3;
    int c0, c1, c2, c3;
    __device__ __forceinline__ void init() { s0 = s1 = s2 = s3 = -INFINITY; c0 = c1 = c2 = c3 = -1; }
    __device__ __forceinline__ void insert(float s, int c) {
        if (!(s > s3)) return;
        if (s > s0) { s3 = s2; c3 = c2; s2 = s1; c2 = c1; s1 = s0; c1 = c0; s0 = s; c0 = c; }
        else if (s > s1) { s3 = s2; c3 = c2; s2 = s1; c2 = c1; s1 = s; c1 = c; }
        else if (s > s2) { s3 = s2; c3 = c2; s2 = s; c2 = c; }
        else { s3 = s; c3 = c; }
    }
};

// ---- pass 1 -------------------------------------------------------------------------------------------------------------
__global__ void __launch_bounds__(DS_THREADS, 4)
fs_dense_select_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k, const DsParams p) {
    extern __shared__ unsigned char ds_smem_raw[];
    __shared__ uint32_t tmem_base_s;
    __shared__ int abort_s;
    unsigned char* base = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(ds_smem_raw) + 1023) & ~(uintptr_t)1023);
    uint64_t* bars = reinterpret_cast<uint64_t*>(base + DSM_BAR);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int n = p.nb - 1 - (int)blockIdx.x;             // the blocks that see the most cells start first
    const int bh = blockIdx.y;
    const int b = bh / p.H, h = bh - b * p.H;
    const int q0 = n * p.Bq;
    int nvis = (q0 / FSATTN_CELL);                        // cells that end at or before the block start
    if (nvis > p.ncell) nvis = p.ncell;
    const int nt = (nvis + DS_BN - 1) / DS_BN;
    int32_t* sel_rows = p.sel + ((int64_t)bh * p.nb * p.Bq + q0) * p.kk;
    if (nt == 0) {                                        // nothing visible: every selection is empty (CTA-uniform exit)
        for (int i = tid; i < p.Bq * p.kk; i += DS_THREADS) sel_rows[i] = -1;
        return;
    }
    if (tid == 0) {
        bar_init(&bars[DB_Q], 1);
        for (int s = 0; s < DS_STAGES; s++) {
            bar_init(&bars[DB_FULL + s], 1);
            bar_init(&bars[DB_EMPTY + s], 1 + DS_SEL_THREADS);      // the MMA's commit + every selecting thread (it reads lc)
        }
        for (int s = 0; s < 2; s++) {
            bar_init(&bars[DB_S_FULL + s], 1);
            bar_init(&bars[DB_S_FREE + s], DS_SEL_THREADS);
        }
        abort_s = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 4) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(s_u32(&tmem_base_s)), "r"(DS_TMEM_COLS) : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_base_s;
    volatile int* abortp = &abort_s;

    if (warp == 4) {
        // ================= TMA producer ====================================================================================
        if (lane == 0) {
            bar_expect_tx(&bars[DB_Q], 16384);
            tma_load_4d(base + DSM_Q, &tm_q, 0, q0, h, b, &bars[DB_Q]);
            for (int i = 0; i < nt && !*abortp; i++) {
                const int s = i % DS_STAGES;
                if (i >= DS_STAGES && !bar_wait<true>(&bars[DB_EMPTY + s], ((i / DS_STAGES) - 1) & 1, abortp)) { *abortp = 1; break; }
                bar_expect_tx(&bars[DB_FULL + s], DS_TILE_BYTES + DS_LC_BYTES);
                tma_load_3d(base + DSM_K + s * DS_TILE_BYTES, &tm_k, 0, i * DS_BN, bh, &bars[DB_FULL + s]);
                bulk_1d(base + DSM_LC + s * DS_LC_BYTES, p.lc + (int64_t)bh * p.ncell_pad + i * DS_BN, DS_LC_BYTES, &bars[DB_FULL + s]);
            }
        }
    } else if (warp == 5) {
        // ================= MMA issuer ======================================================================================
        if (lane == 0) {
            const uint32_t idesc = instr_desc(DS_BN, 0, 1);
            bool ok = bar_wait<true>(&bars[DB_Q], 0, abortp);
            for (int i = 0; i < nt && ok && !*abortp; i++) {
                const int s = i & 1, ks = i % DS_STAGES;
                ok = bar_wait<true>(&bars[DB_FULL + ks], (i / DS_STAGES) & 1, abortp);
                if (ok && i >= 2) ok = bar_wait<true>(&bars[DB_S_FREE + s], ((i >> 1) - 1) & 1, abortp);
                if (!ok) break;
                tc_fence_after();
                const uint32_t aq = s_u32(base + DSM_Q), bk = s_u32(base + DSM_K + ks * DS_TILE_BYTES);
#pragma unroll
                for (int k = 0; k < DS_D / 16; k++)
                    umma(tmem + s * DS_BN, smem_desc(aq + k * 32), smem_desc(bk + k * 32), idesc, k > 0);
                umma_commit(&bars[DB_S_FULL + s]);
                umma_commit(&bars[DB_EMPTY + ks]);
            }
            if (!ok) *abortp = 1;
        }
    } else {
        // ================= selection: one query per thread ==================================================================
        const int r = warp * 32 + lane;
        const float qpos = (float)(q0 + r);
        const uint32_t lane_base = tmem + ((uint32_t)(warp * 32) << 16);
        const float two_sigma = f_mul(2.0f, p.sigma[h]);
        const float inv_two_sigma = 1.0f / two_sigma;      // for the "is erf exactly 1" decision only (taken with a margin)
        Top4 T;
        T.init();
        bool ok = true;
        for (int i = 0; i < nt; i++) {
            const int bb = i & 1, ks = i % DS_STAGES;
            ok = ok && bar_wait<true>(&bars[DB_S_FULL + bb], (i >> 1) & 1, abortp) && !*abortp;
            if (!__all_sync(FS_FULL, ok)) { ok = false; break; }
            tc_fence_after();
            const float* lcs = reinterpret_cast<const float*>(base + DSM_LC + ks * DS_LC_BYTES);
            // eight columns at a time straight from TMEM: one small loop body for the whole tile keeps the kernel's code far
            // below the instruction cache (a fully unrolled 64-column body with its inlined inserts and erf calls is not)
#pragma unroll 1
            for (int j0 = 0; j0 < DS_BN; j0 += 8) {
                const int cell0 = i * DS_BN + j0;
                const int cv = nvis - cell0;                          // valid columns of this group: j < cv
                if (cv <= 0) break;
                float v[8];
                tmem_ld8(lane_base + bb * DS_BN + j0, v);
                const float4 la = reinterpret_cast<const float4*>(lcs + j0)[0];
                const float4 lb = reinterpret_cast<const float4*>(lcs + j0)[1];
                const float lc8[8] = {la.x, la.y, la.z, la.w, lb.x, lb.y, lb.z, lb.w};
                // the nearest cell of the group is its last valid one; beyond x = 4 erf is exactly 1 in fp32
                const int clast = cell0 + (cv < 8 ? cv : 8) - 1;
                const float xmin = fabsf(qpos - ((float)clast + 0.5f) * (float)FSATTN_CELL) * inv_two_sigma;
                float s[8];
                if (xmin >= 4.01f) {                                  // the exact quotient is then >= 4: erf is 1
#pragma unroll
                    for (int j = 0; j < 8; j++) s[j] = f_add(f_mul(v[j], p.scale), lc8[j]);
                } else {
#pragma unroll
                    for (int j = 0; j < 8; j++) {
                        const float x = f_div(fabsf(qpos - f_mul((float)(cell0 + j) + 0.5f, (float)FSATTN_CELL)), two_sigma);
                        s[j] = f_add(f_mul(v[j], p.scale), f_mul(lc8[j], erff(x)));
                    }
                }
                if (cv < 8) {
#pragma unroll
                    for (int j = 0; j < 8; j++) if (j >= cv) s[j] = -INFINITY;
                }
                const float m8 = fmaxf(fmaxf(fmaxf(s[0], s[1]), fmaxf(s[2], s[3])), fmaxf(fmaxf(s[4], s[5]), fmaxf(s[6], s[7])));
                if (m8 > T.s3) {
#pragma unroll
                    for (int j = 0; j < 8; j++) T.insert(s[j], cell0 + j);
                }
            }
            tc_fence_before();
            bar_arrive(&bars[DB_S_FREE + bb]);
            bar_arrive(&bars[DB_EMPTY + ks]);
        }
        if (!ok) *abortp = 1;
        if (ok) {
            int32_t* o = sel_rows + (int64_t)r * p.kk;
            const int cs[4] = {T.c0, T.c1, T.c2, T.c3};
            for (int k = 0; k < p.kk; k++) o[k] = k < 4 ? cs[k] : -1;
        }
    }
    tc_fence_before();
    __syncthreads();
    if (tid == 0 && abort_s && p.status != nullptr) atomicAdd(p.status, 1);
    if (warp == 4) {
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(DS_TMEM_COLS) : "memory");
    }
}

}  // namespace

extern "C" int64_t fsattn_fs_dense_workspace_bytes(int32_t B, int32_t H, int32_t ncell, int32_t D) {
    const int64_t pad = ((int64_t)ncell + DS_BN - 1) / DS_BN * DS_BN + DS_BN;
    return (int64_t)B * H * ((int64_t)ncell * D * 2 + pad * 4) + 256;
}

extern "C" int fsattn_fs_dense_select(const fsattn_fs_dense_select_t* a, fsattn_stream_t stream) {
    FS_REQUIRE(a != nullptr && a->q.ptr && a->kbar && a->ceil && a->lam && a->sigma && a->sel, "fs_dense_select: null pointer");
    FS_REQUIRE(a->B > 0 && a->H > 0 && a->N > 0 && a->ncell >= 0 && a->nb > 0, "fs_dense_select: bad sizes");
    FS_UNSUPPORTED(a->D != DS_D, "fs_dense_select: head_dim %d (the tensor-core kernel is built for 64)", a->D);
    FS_UNSUPPORTED(a->Bq != TC_BM, "fs_dense_select: query blocks of %d (128)", a->Bq);
    FS_REQUIRE(a->kk >= 1 && a->kk <= 4, "fs_dense_select: kk = %d (1..4)", a->kk);
    FS_REQUIRE(a->nb * a->Bq >= a->N, "fs_dense_select: nb * Bq < N");
    FS_REQUIRE(((uintptr_t)a->q.ptr & 15) == 0 && a->q.sn % 8 == 0 && a->q.sh % 8 == 0 && a->q.sb % 8 == 0,
               "fs_dense_select: Q rows must be 16-byte aligned");
    FS_REQUIRE(((uintptr_t)a->kbar & 15) == 0 && a->kbar_sb % 4 == 0 && a->kbar_sh % 4 == 0, "fs_dense_select: kbar must be 16-byte aligned");
    cudaStream_t st = (cudaStream_t)stream;
    if (a->ncell == 0) {
        FS_REQUIRE(cudaMemsetAsync(a->sel, 0xff, (size_t)a->B * a->H * a->nb * a->Bq * a->kk * 4, st) == cudaSuccess,
                   "fs_dense_select: memset failed");
        return FSATTN_OK;
    }
    FS_REQUIRE(a->workspace != nullptr && ((uintptr_t)a->workspace & 15) == 0 &&
               a->workspace_bytes >= fsattn_fs_dense_workspace_bytes(a->B, a->H, a->ncell, a->D),
               "fs_dense_select: workspace of %lld bytes needed (16-byte aligned)",
               (long long)fsattn_fs_dense_workspace_bytes(a->B, a->H, a->ncell, a->D));
    FS_REQUIRE(encode_fn() != nullptr, "fs_dense_select: the driver does not export cuTensorMapEncodeTiled");
    const int64_t BH = (int64_t)a->B * a->H;
    const int ncell_pad = (a->ncell + DS_BN - 1) / DS_BN * DS_BN + DS_BN;
    bf16* kb16 = (bf16*)a->workspace;
    float* lc = (float*)((unsigned char*)a->workspace + (((size_t)BH * a->ncell * DS_D * 2 + 15) & ~(size_t)15));
    {
        const int64_t total = BH * a->ncell * (DS_D / 8);
        const int64_t blocks = (total + 255) / 256;
        FS_REQUIRE(blocks < (1ll << 31), "fs_dense_select: too many cells");
        dense_prep_kernel<<<(unsigned)blocks, 256, 0, st>>>(*a, kb16, lc, ncell_pad);
        const int rc = fs_check_launch("dense_prep");
        if (rc != FSATTN_OK) return rc;
    }
    CUtensorMap tq, tk;
    {
        const cuuint64_t dims[4] = {DS_D, (cuuint64_t)a->N, (cuuint64_t)a->H, (cuuint64_t)a->B};
        const cuuint64_t strides[3] = {(cuuint64_t)a->q.sn * 2, (cuuint64_t)a->q.sh * 2, (cuuint64_t)(a->B > 1 ? a->q.sb : a->q.sn * a->N) * 2};
        const cuuint32_t box[4] = {DS_D, TC_BM, 1, 1};
        FS_REQUIRE(make_map(&tq, const_cast<void*>(a->q.ptr), 4, dims, strides, box), "fs_dense_select: cuTensorMapEncodeTiled failed for Q");
    }
    {
        const cuuint64_t dims[3] = {DS_D, (cuuint64_t)a->ncell, (cuuint64_t)BH};
        const cuuint64_t strides[2] = {DS_D * 2, (cuuint64_t)a->ncell * DS_D * 2};
        const cuuint32_t box[3] = {DS_D, DS_BN, 1};
        FS_REQUIRE(make_map(&tk, kb16, 3, dims, strides, box), "fs_dense_select: cuTensorMapEncodeTiled failed for the mean keys");
    }
    static bool opted[64] = {false};
    int dev = 0;
    cudaGetDevice(&dev);
    const int smem = DSM_TOTAL + 1024;
    if (dev >= 0 && dev < 64 && !opted[dev]) {
        if (cudaFuncSetAttribute(fs_dense_select_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess) {
            (void)cudaGetLastError();
            fs_set_error("fs_dense_select: cannot opt in to %d bytes of shared memory", smem);
            return FSATTN_ELAUNCH;
        }
        opted[dev] = true;
    }
    DsParams p;
    p.N = a->N; p.H = a->H; p.ncell = a->ncell; p.ncell_pad = ncell_pad; p.nb = a->nb; p.Bq = a->Bq; p.kk = a->kk;
    p.scale = a->scale; p.sigma = a->sigma; p.lc = lc; p.sel = a->sel; p.status = a->status;
    dim3 grid(a->nb, (unsigned)BH);
    fs_dense_select_kernel<<<grid, DS_THREADS, smem, st>>>(tq, tk, p);
    return fs_check_launch("fs_dense_select");
}
