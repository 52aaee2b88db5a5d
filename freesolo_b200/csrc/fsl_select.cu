// FS-L prefill selection: per-block prefix top-P of the cell ceilings, candidate slots, chunk-mean-key scoring and the
// per-query top-kk.
#include "common.cuh"
#include "pool_list.cuh"

// ---- prefix top-P --------------------------------------------------------------------------------------------------
// One warp per (b,h) walks the cells in index order and keeps the sorted top-P list in shared memory; after the cells
// visible to block n are in, the list is written out as that block's row. Ceilings are fetched 32 at a time.
__global__ void __launch_bounds__(32) fsl_prefix_topp_kernel(const fsattn_fsl_topp_t a) {
    __shared__ float lc[FSATTN_MAX_POOL];
    __shared__ int li[FSATTN_MAX_POOL];
    const int bh = blockIdx.x;
    const int b = bh / a.H, h = bh - b * a.H;
    const int lane = threadIdx.x;
    const float* ceil = a.ceil + b * a.ceil_sb + h * a.ceil_sh;
    int32_t* out = a.topp + (int64_t)bh * a.nb * a.P;
    int n = 0;      // entries in the list
    int done = 0;   // cells [0, done) are in
    float cbuf = 0.0f;
    int cbase = -32;
    for (int blk = 0; blk < a.nb; blk++) {
        int vis = (int)(((int64_t)blk * a.Bq) / FSATTN_CELL);
        if (vis > a.ncell) vis = a.ncell;
        while (done < vis) {
            if (done >= cbase + 32) {
                cbase = done & ~31;
                cbuf = (cbase + lane < a.ncell) ? ceil[cbase + lane] : 0.0f;
            }
            // the new cells of this 32-cell segment, tested against the list's last entry all at once: most of them rank
            // after it once the list is full, and the entry only ever tightens, so a cell rejected here stays rejected
            const int seg_end = min(vis, cbase + 32);
            const bool mine = lane >= done - cbase && lane < seg_end - cbase;
            const bool full = (n == a.P);
            const float thr_c = full ? lc[a.P - 1] : 0.0f;
            const int thr_i = full ? li[a.P - 1] : 0;
            unsigned pend = __ballot_sync(FS_FULL, mine && (!full || pool_before(cbuf, cbase + lane, thr_c, thr_i)));
            while (pend) {
                const int l = __ffs(pend) - 1;
                pend &= pend - 1;
                const float cv = __shfl_sync(FS_FULL, cbuf, l);
                pool_list_insert(lc, li, n, a.P, cv, cbase + l, lane);
            }
            done = seg_end;
        }
        for (int p = lane; p < a.P; p += 32) out[(int64_t)blk * a.P + p] = (p < n) ? li[p] : -1;
    }
}

extern "C" int fsattn_fsl_prefix_topp(const fsattn_fsl_topp_t* a, fsattn_stream_t stream) {
    FS_REQUIRE(a != nullptr && a->ceil != nullptr && a->topp != nullptr, "prefix_topp: null pointer");
    FS_REQUIRE(a->B > 0 && a->H > 0 && a->ncell >= 0 && a->nb > 0 && a->Bq > 0, "prefix_topp: bad sizes");
    FS_REQUIRE(a->P >= 1 && a->P <= FSATTN_MAX_POOL, "prefix_topp: pool size %d not in [1,%d]", a->P, FSATTN_MAX_POOL);
    fsl_prefix_topp_kernel<<<a->B * a->H, 32, 0, (cudaStream_t)stream>>>(*a);
    return fs_check_launch("fsl_prefix_topp");
}

// ---- candidate scoring + top-kk -------------------------------------------------------------------------------------
// One CTA per (block, b*h): the block's candidate mean keys are staged once in shared memory (fp32), each thread owns
// one query: q in registers, fp32 dot per candidate (shared-memory broadcast reads), prior, running top-(kk+1).
template <int D, int KMAX>
__global__ void __launch_bounds__(128) fsl_select_kernel(const fsattn_fsl_select_t a) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    const int C = a.P + a.Wc;
    float* kb = reinterpret_cast<float*>(smem_raw);            // C * D
    float* cceil = kb + (size_t)C * D;                         // C
    int* ccell = reinterpret_cast<int*>(cceil + C);            // C
    int* cok = ccell + C;                                      // C

    const int blk = blockIdx.x;
    const int bh = blockIdx.y;
    const int b = bh / a.H, h = bh - b * a.H;
    const int tid = threadIdx.x;
    const int blk_start = blk * a.Bq;
    const float* kbar = a.kbar + b * a.kbar_sb + h * a.kbar_sh;
    const float* ceil = a.ceil + b * a.ceil_sb + h * a.ceil_sh;
    const int32_t* topp = a.topp + ((int64_t)bh * (a.topp_nb > 0 ? a.topp_nb : a.nb) + blk) * a.P;

    // candidate slots
    for (int t = tid; t < C; t += blockDim.x) {
        const int cand = (t < a.P) ? topp[t] : (blk_start / FSATTN_CELL - 1) - (t - a.P);
        const int cc = cand < 0 ? 0 : cand;
        ccell[t] = cc;
        cok[t] = (cand >= 0) && ((int64_t)(cc + 1) * FSATTN_CELL <= blk_start) && (cc < a.ncell);
    }
    __syncthreads();
    // a slot repeats an earlier one when an earlier slot holds the same (clamped) cell id, whatever that slot's flags
    for (int t = tid; t < C; t += blockDim.x) {
        int ok = cok[t];
        const int cc = ccell[t];
        for (int j = 0; j < t && ok; j++) ok = (ccell[j] != cc);
        cok[t] = ok;
        cceil[t] = ok ? ceil[cc] : 0.0f;
    }
    __syncthreads();
    // stage the mean keys of the ok slots (zeros elsewhere), 16-byte loads
    constexpr int V4 = D / 4;
    for (int i = tid; i < C * V4; i += blockDim.x) {
        const int t = i / V4, e = i - t * V4;
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if (cok[t]) v = reinterpret_cast<const float4*>(kbar + (int64_t)ccell[t] * D)[e];
        reinterpret_cast<float4*>(kb + (size_t)t * D)[e] = v;
    }
    __syncthreads();
    if (tid >= a.Bq) return;

    const int qi = blk_start + tid;
    float q[D];
    if (qi < a.N) {
        const bf16* qp = (const bf16*)a.q.ptr + b * a.q.sb + h * a.q.sh + (int64_t)qi * a.q.sn;
#pragma unroll
        for (int e = 0; e < D / 8; e++) {
            const uint4 w = reinterpret_cast<const uint4*>(qp)[e];
            q[8 * e + 0] = bf_lo(w.x); q[8 * e + 1] = bf_hi(w.x); q[8 * e + 2] = bf_lo(w.y); q[8 * e + 3] = bf_hi(w.y);
            q[8 * e + 4] = bf_lo(w.z); q[8 * e + 5] = bf_hi(w.z); q[8 * e + 6] = bf_lo(w.w); q[8 * e + 7] = bf_hi(w.w);
        }
    } else {
#pragma unroll
        for (int e = 0; e < D; e++) q[e] = 0.0f;
    }
    const float lam = a.lam[h];
    const float two_sigma = f_mul(2.0f, a.sigma[h]);
    const float qpos = (float)qi;

    // KMAX - 1 >= kk entries are kept (+1 for the margin): 5 for the serve configuration's top-4, so the sorted insert is
    // five compare-and-swap steps per candidate instead of nine
    float ts[KMAX];
    int tslot[KMAX];
#pragma unroll
    for (int j = 0; j < KMAX; j++) { ts[j] = -INFINITY; tslot[j] = -1; }
    const int keep = a.kk + 1;
    for (int t = 0; t < C; t++) {
        float sc = FS_NEG_SCORE;
        if (cok[t]) {
            const float4* kr = reinterpret_cast<const float4*>(kb + (size_t)t * D);
            float d0 = 0.f, d1 = 0.f, d2 = 0.f, d3 = 0.f;
#pragma unroll
            for (int e = 0; e < V4; e++) {
                const float4 kv = kr[e];
                d0 = fmaf(q[4 * e + 0], kv.x, d0);
                d1 = fmaf(q[4 * e + 1], kv.y, d1);
                d2 = fmaf(q[4 * e + 2], kv.z, d2);
                d3 = fmaf(q[4 * e + 3], kv.w, d3);
            }
            const float content = f_mul(f_add(f_add(d0, d2), f_add(d1, d3)), a.scale);
            sc = f_add(content, fs_prior(lam, cceil[t], qpos, ccell[t], (float)FSATTN_CELL, two_sigma));
        }
        // sorted insert; slots arrive in ascending order, so a new entry goes after equal scores (lower slot first).
        // Once an entry is displaced every later position shifts down by one.
        {
            float cs = sc;
            int cslot = t;
            bool shifting = false;
#pragma unroll
            for (int j = 0; j < KMAX; j++) {
                if (j < keep) {
                    const bool take = shifting || (tslot[j] < 0) || (cs > ts[j]);
                    if (take) {
                        const float os = ts[j]; const int oslot = tslot[j];
                        ts[j] = cs; tslot[j] = cslot;
                        cs = os; cslot = oslot;
                        shifting = true;
                    }
                }
            }
        }
    }
    int32_t* so = a.sel + ((int64_t)bh * a.nb * a.Bq + qi) * a.kk;
#pragma unroll
    for (int j = 0; j < KMAX - 1; j++)
        if (j < a.kk) so[j] = (tslot[j] >= 0 && cok[tslot[j]]) ? ccell[tslot[j]] : -1;
    if (a.margin != nullptr) {
        float mg = INFINITY;
#pragma unroll
        for (int j = 0; j < KMAX - 1; j++) {
            if (j < a.kk && tslot[j] >= 0 && tslot[j + 1] >= 0 && ts[j] > FS_NEG_SCORE * 0.5f)
                mg = fminf(mg, ts[j] - ts[j + 1]);
        }
        a.margin[(int64_t)bh * a.nb * a.Bq + qi] = mg;
    }
}

static size_t select_smem(int C, int D) { return (size_t)C * D * 4 + (size_t)C * 12; }

template <int D, int KMAX>
static int launch_select_k(const fsattn_fsl_select_t* a, cudaStream_t st) {
    const size_t smem = select_smem(a->P + a->Wc, D);
    static size_t opted[16] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 16 && opted[dev] < smem) {
        if (cudaFuncSetAttribute(fsl_select_kernel<D, KMAX>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess) {
            fs_set_error("fsl_select: cannot opt in to %zu bytes of shared memory", smem);
            return FSATTN_ELAUNCH;
        }
        opted[dev] = smem;
    }
    dim3 grid(a->nb, a->B * a->H);
    fsl_select_kernel<D, KMAX><<<grid, 128, smem, st>>>(*a);
    return fs_check_launch("fsl_select");
}

template <int D>
static int launch_select(const fsattn_fsl_select_t* a, cudaStream_t st) {
    return a->kk <= 4 ? launch_select_k<D, 5>(a, st) : launch_select_k<D, FSATTN_MAX_KK + 1>(a, st);
}

extern "C" int fsattn_fsl_select(const fsattn_fsl_select_t* a, fsattn_stream_t stream) {
    FS_REQUIRE(a != nullptr && a->q.ptr && a->kbar && a->ceil && a->topp && a->lam && a->sigma && a->sel,
               "fsl_select: null pointer");
    FS_REQUIRE(a->B > 0 && a->H > 0 && a->N > 0 && a->nb > 0 && a->ncell >= 0 && (a->topp_nb == 0 || a->topp_nb >= a->nb), "fsl_select: bad sizes");
    FS_REQUIRE(a->Bq >= 1 && a->Bq <= 128, "fsl_select: query block %d not in [1,128]", a->Bq);
    FS_REQUIRE(a->P >= 1 && a->Wc >= 0 && a->P + a->Wc <= FSATTN_MAX_POOL + 8, "fsl_select: pool %d + %d too large", a->P, a->Wc);
    FS_REQUIRE(a->kk >= 1 && a->kk <= FSATTN_MAX_KK, "fsl_select: kk %d not in [1,%d]", a->kk, FSATTN_MAX_KK);
    FS_UNSUPPORTED(a->D != 64 && a->D != 96 && a->D != 128, "fsl_select: head_dim %d not in {64,96,128}", a->D);
    FS_REQUIRE(((uintptr_t)a->q.ptr & 15) == 0 && a->q.sn % 8 == 0 && a->q.sh % 8 == 0 && a->q.sb % 8 == 0,
               "fsl_select: Q rows must be 16-byte aligned");
    FS_REQUIRE(((uintptr_t)a->kbar & 15) == 0 && a->kbar_sb % 4 == 0 && a->kbar_sh % 4 == 0, "fsl_select: kbar must be 16-byte aligned");
    cudaStream_t st = (cudaStream_t)stream;
    switch (a->D) {
        case 64: return launch_select<64>(a, st);
        case 96: return launch_select<96>(a, st);
        default: return launch_select<128>(a, st);
    }
}
