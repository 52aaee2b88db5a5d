// FS-L prefill selection: per-block prefix top-P of the cell ceilings, candidate slots, chunk-mean-key scoring and the
// per-query top-kk.
#include "common.cuh"

// ---- prefix top-P --------------------------------------------------------------------------------------------------
// A warp keeps the sorted top-P list (ceiling descending, cell index ascending) in registers: list position p lives in
// lane p & 31, register p >> 5. Cells join in index order; the new cells of a block are tested 32 at a time against the
// list's last entry and only the few that pass are inserted (two ballots give the rank, shuffles shift the tail by one).
// After the cells visible to block n are in, the list is written out as that block's row.
constexpr int TOPP_E = FSATTN_MAX_POOL / 32;      // list entries per lane

struct ToppList {
    float c[TOPP_E];
    int i[TOPP_E];
};

// entry at list position P-1 (valid when the list is full), the same in every lane
__device__ __forceinline__ void topp_last(const ToppList& L, int P, float& tc, int& ti) {
    const int jl = (P - 1) >> 5;
    float c = L.c[0];
    int i = L.i[0];
#pragma unroll
    for (int j = 1; j < TOPP_E; j++)
        if (j == jl) { c = L.c[j]; i = L.i[j]; }
    tc = __shfl_sync(FS_FULL, c, (P - 1) & 31);
    ti = __shfl_sync(FS_FULL, i, (P - 1) & 31);
}

__device__ __forceinline__ void topp_insert(ToppList& L, int& n, int P, float cv, int ci, int lane) {
    const int JP = (P + 31) >> 5;
    int ins = 0;                                        // entries that rank before the new cell
#pragma unroll
    for (int j = 0; j < TOPP_E; j++)
        if (j < JP) ins += __popc(__ballot_sync(FS_FULL, (lane + 32 * j) < n && pool_before(L.c[j], L.i[j], cv, ci)));
    if (ins >= P) return;
    const int nn = (n + 1 < P) ? n + 1 : P;
    // position p > ins takes the old entry p-1: the lane below's register j, or lane 31's register j-1 for lane 0
    float pc[TOPP_E];
    int pi[TOPP_E];
#pragma unroll
    for (int j = 0; j < TOPP_E; j++) {
        if (j < JP) {
            pc[j] = __shfl_up_sync(FS_FULL, L.c[j], 1);
            pi[j] = __shfl_up_sync(FS_FULL, L.i[j], 1);
        }
    }
#pragma unroll
    for (int j = TOPP_E - 1; j > 0; j--) {
        if (j < JP) {
            const float wc = __shfl_sync(FS_FULL, L.c[j - 1], 31);
            const int wi = __shfl_sync(FS_FULL, L.i[j - 1], 31);
            if (lane == 0) { pc[j] = wc; pi[j] = wi; }
        }
    }
#pragma unroll
    for (int j = 0; j < TOPP_E; j++) {
        if (j < JP) {
            const int p = lane + 32 * j;
            if (p == ins) { L.c[j] = cv; L.i[j] = ci; }
            else if (p > ins && p < nn) { L.c[j] = pc[j]; L.i[j] = pi[j]; }
        }
    }
    n = nn;
}

__global__ void __launch_bounds__(32) fsl_prefix_topp_kernel(const fsattn_fsl_topp_t a) {
    const int bh = blockIdx.x;
    const int b = bh / a.H, h = bh - b * a.H;
    const int lane = threadIdx.x;
    const float* ceil = a.ceil + b * a.ceil_sb + h * a.ceil_sh;
    int32_t* out = a.topp + (int64_t)bh * a.nb * a.P;
    ToppList L;
#pragma unroll
    for (int j = 0; j < TOPP_E; j++) { L.c[j] = 0.0f; L.i[j] = -1; }
    int n = 0;      // entries in the list
    int done = 0;   // cells [0, done) are in
    float cbuf = 0.0f, cnext = 0.0f;
    int cbase = -32;
    // The blocks of a head are split over gridDim.y warps: a warp first brings its list up to its first block by scanning
    // all earlier cells (a scan costs little more than its ~P ln(n/P) inserts), then walks its own blocks. The rescans are
    // redundant work, but the serial chain per warp shrinks from nb blocks to nb / gridDim.y blocks plus one scan.
    const int per = (a.nb + gridDim.y - 1) / gridDim.y;
    const int b0 = blockIdx.y * per, b1 = min(a.nb, b0 + per);
    const int JP = (a.P + 31) >> 5;
    for (int blk = b0; blk < b1; blk++) {
        int vis = (int)(((int64_t)blk * a.Bq) / FSATTN_CELL);
        if (vis > a.ncell) vis = a.ncell;
        while (done < vis) {
            if (done >= cbase + 32) {                       // next 32 ceilings; the 32 after them are requested one step ahead
                const int nbase = done & ~31;
                cbuf = (nbase == cbase + 32 && cbase >= 0) ? cnext : ((nbase + lane < a.ncell) ? ceil[nbase + lane] : 0.0f);
                cbase = nbase;
                cnext = (cbase + 32 + lane < a.ncell) ? ceil[cbase + 32 + lane] : 0.0f;
            }
            // most new cells rank after the full list's last entry, and that entry only ever tightens, so a cell rejected
            // against it stays rejected
            const int seg_end = min(vis, cbase + 32);
            const bool mine = lane >= done - cbase && lane < seg_end - cbase;
            const bool full = (n == a.P);
            float thr_c = 0.0f;
            int thr_i = 0;
            if (full) topp_last(L, a.P, thr_c, thr_i);
            unsigned pend = __ballot_sync(FS_FULL, mine && (!full || pool_before(cbuf, cbase + lane, thr_c, thr_i)));
            while (pend) {
                const int l = __ffs(pend) - 1;
                pend &= pend - 1;
                const float cv = __shfl_sync(FS_FULL, cbuf, l);
                topp_insert(L, n, a.P, cv, cbase + l, lane);
            }
            done = seg_end;
        }
#pragma unroll
        for (int j = 0; j < TOPP_E; j++) {
            const int p = lane + 32 * j;
            if (j < JP && p < a.P) out[(int64_t)blk * a.P + p] = (p < n) ? L.i[j] : -1;
        }
    }
}

extern "C" int fsattn_fsl_prefix_topp(const fsattn_fsl_topp_t* a, fsattn_stream_t stream) {
    FS_REQUIRE(a != nullptr && a->ceil != nullptr && a->topp != nullptr, "prefix_topp: null pointer");
    FS_REQUIRE(a->B > 0 && a->H > 0 && a->ncell >= 0 && a->nb > 0 && a->Bq > 0, "prefix_topp: bad sizes");
    FS_REQUIRE(a->P >= 1 && a->P <= FSATTN_MAX_POOL, "prefix_topp: pool size %d not in [1,%d]", a->P, FSATTN_MAX_POOL);
    const int nseg = a->nb >= 512 ? 64 : (a->nb >= 128 ? 16 : (a->nb >= 32 ? 4 : 1));
    fsl_prefix_topp_kernel<<<dim3(a->B * a->H, nseg), 32, 0, (cudaStream_t)stream>>>(*a);
    return fs_check_launch("fsl_prefix_topp");
}

// ---- pieces shared by the two selection kernels --------------------------------------------------------------------------
// Sorted list of the best KMAX (score, slot) pairs, scores descending; slots arrive in ascending order and a new entry goes
// after equal scores, so ties keep the lower slot first. Empty entries hold -inf (every real score is >= -1e9): the new
// pair replaces the last entry if it beats it and then bubbles up with strict compare-and-swap steps.
// The candidates arrive roughly best first (the top-P list is sorted by ceiling, and the prior usually outweighs the
// content term), so after the first few a candidate often enters no list of the warp: one vote skips the insert then.
template <int KMAX>
__device__ __forceinline__ void sel_insert(float (&ts)[KMAX], int (&tslot)[KMAX], float cs, int t) {
    if (!__any_sync(__activemask(), cs > ts[KMAX - 1])) return;
    if (cs > ts[KMAX - 1]) { ts[KMAX - 1] = cs; tslot[KMAX - 1] = t; }
#pragma unroll
    for (int j = KMAX - 1; j > 0; j--) {
        const bool up = ts[j] > ts[j - 1];
        const float a = ts[j], b = ts[j - 1];
        const int ia = tslot[j], ib = tslot[j - 1];
        ts[j - 1] = up ? a : b; ts[j] = up ? b : a;
        tslot[j - 1] = up ? ia : ib; tslot[j] = up ? ib : ia;
    }
}
// the prior lam*ceil * erf(|p - centre| / (2 sigma)) from per-slot lam*ceil and centre; the quotient is taken as a product
// with 1/(2 sigma) (one rounding away from the reference's division: far inside the 1e-4 selection margin)
// erf(x) rounds to 1 in fp32 for x >= 4 (1 - erf(4) = 1.5e-8, a quarter of an ulp); with sigma of a few tokens that is every
// cell further than a cell or two from the query, so the warp skips the erf evaluation when all its lanes are there.
__device__ __forceinline__ float sel_prior(float lam_ceil, float centre, float qpos, float inv_two_sigma) {
    const float x = f_mul(fabsf(qpos - centre), inv_two_sigma);
    float e = 1.0f;
    if (__any_sync(__activemask(), x < 4.0f)) e = (x < 4.0f) ? erff(x) : 1.0f;
    return f_mul(lam_ceil, e);
}

// ---- candidate scoring + top-kk -------------------------------------------------------------------------------------
// One CTA per (block, b*h): the block's candidate mean keys are staged once in shared memory (fp32), each thread owns
// one query: q in registers, fp32 dot per candidate (shared-memory broadcast reads), prior, running top-(kk+1).
template <int D, int KMAX>
__global__ void __launch_bounds__(128) fsl_select_kernel(const fsattn_fsl_select_t a) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    const int C = a.P + a.Wc;
    float* kb = reinterpret_cast<float*>(smem_raw);            // C * D
    float* cceil = kb + (size_t)C * D;                         // C: lam * ceiling of the slot's cell
    int* ccell = reinterpret_cast<int*>(cceil + C);            // C
    int* cok = ccell + C;                                      // C
    float* ccen = reinterpret_cast<float*>(cok + C);           // C: centre position of the slot's cell

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
        cceil[t] = ok ? f_mul(a.lam[h], ceil[cc]) : 0.0f;
        ccen[t] = f_mul((float)cc + 0.5f, (float)FSATTN_CELL);
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
    const float inv_two_sigma = f_div(1.0f, f_mul(2.0f, a.sigma[h]));
    const float qpos = (float)qi;

    // KMAX - 1 >= kk entries are kept (+1 for the margin): 5 for the serve configuration's top-4
    float ts[KMAX];
    int tslot[KMAX];
#pragma unroll
    for (int j = 0; j < KMAX; j++) { ts[j] = -INFINITY; tslot[j] = -1; }
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
            sc = f_add(content, sel_prior(cceil[t], ccen[t], qpos, inv_two_sigma));
        }
        sel_insert<KMAX>(ts, tslot, sc, t);
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

// ---- the same selection with the 128 x C x 64 dot products on tensor-core tiles (head_dim 64, whole 128-query blocks) ----------
// The chunk-mean keys are bf16 values (held as fp32), and so is Q: the products are exact in bf16 MMAs with fp32
// accumulation. One CTA per (block, b*h), four warps of 32 queries (two 16-row tiles): the candidates' keys (bf16) and the
// Q tile are staged swizzled in shared memory; per 8-candidate tile two ldmatrix.x4 bring the B fragments of all four
// k-steps and eight mma.sync.m16n8k16 give the 32 x 8 dot products, which go to a per-warp score array in shared memory.
// Then each thread is one query again and walks its row of scores in slot order: prior, sorted insert - the scalar kernel's
// epilogue, so ties resolve identically (lower slot first).
constexpr int SM_MAXC = 80;                // candidate slots rounded up to whole 8-column tiles
constexpr int SM_NTH = SM_MAXC / 16;       // the candidates are scored in two halves of at most 5 tiles: the score array of a
constexpr int SM_SCLD = SM_NTH * 8 + 1;    // half (row pitch in floats, odd: conflict-free column walks) lets 4 CTAs share an SM

struct SelMmaSmem {
    static constexpr size_t KB_OFF = 0;                                        // [80][64] bf16, 16-byte chunks XOR-swizzled by row
    static constexpr size_t Q_OFF = KB_OFF + (size_t)SM_MAXC * 128;            // [128][64] bf16, swizzled
    static constexpr size_t SC_OFF = Q_OFF;     // [128][41] fp32 dot products of one half of the candidates: over the Q tile, which
                                                // is dead once every warp holds its A fragments
    static constexpr size_t META_OFF = SC_OFF + (size_t)128 * SM_SCLD * 4;     // ceil, cell, ok per slot
    static constexpr size_t TOTAL = META_OFF + (size_t)SM_MAXC * 16;           // lam*ceil, cell, ok, centre per slot
};

__device__ __forceinline__ uint32_t sel_sw(int row, int chunk) { return (uint32_t)(row * 128 + ((chunk ^ (row & 7)) << 4)); }

template <int KMAX>
__global__ void __launch_bounds__(128) fsl_select_mma_kernel(const fsattn_fsl_select_t a) {
    constexpr int D = 64;
    extern __shared__ __align__(16) unsigned char smem_raw[];
    unsigned char* kb = smem_raw + SelMmaSmem::KB_OFF;
    unsigned char* qs = smem_raw + SelMmaSmem::Q_OFF;
    float* sc = reinterpret_cast<float*>(smem_raw + SelMmaSmem::SC_OFF);
    float* cceil = reinterpret_cast<float*>(smem_raw + SelMmaSmem::META_OFF);
    int* ccell = reinterpret_cast<int*>(cceil + SM_MAXC);
    int* cok = ccell + SM_MAXC;
    float* ccen = reinterpret_cast<float*>(cok + SM_MAXC);

    const int C = a.P + a.Wc;
    const int NT = (C + 7) / 8;
    const int blk = blockIdx.x, bh = blockIdx.y;
    const int b = bh / a.H, h = bh - b * a.H;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int blk_start = blk * a.Bq;
    const float* kbar = a.kbar + b * a.kbar_sb + h * a.kbar_sh;
    const float* ceil = a.ceil + b * a.ceil_sb + h * a.ceil_sh;
    const int32_t* topp = a.topp + ((int64_t)bh * (a.topp_nb > 0 ? a.topp_nb : a.nb) + blk) * a.P;

    // candidate slots (the scalar kernel's rules)
    for (int t = tid; t < NT * 8; t += 128) {
        int cc = 0, ok = 0;
        if (t < C) {
            const int cand = (t < a.P) ? topp[t] : (blk_start / FSATTN_CELL - 1) - (t - a.P);
            cc = cand < 0 ? 0 : cand;
            ok = (cand >= 0) && ((int64_t)(cc + 1) * FSATTN_CELL <= blk_start) && (cc < a.ncell);
        }
        ccell[t] = cc;
        cok[t] = ok;
    }
    // the Q tile, 16-byte chunks, rows past N zero
    for (int i = tid; i < 128 * 8; i += 128) {
        const int r = i >> 3, e = i & 7;
        uint4 w = make_uint4(0u, 0u, 0u, 0u);
        if (blk_start + r < a.N && r < a.Bq)
            w = reinterpret_cast<const uint4*>((const bf16*)a.q.ptr + b * a.q.sb + h * a.q.sh + (int64_t)(blk_start + r) * a.q.sn)[e];
        *reinterpret_cast<uint4*>(qs + sel_sw(r, e)) = w;
    }
    __syncthreads();
    for (int t = tid; t < C; t += 128) {
        int ok = cok[t];
        const int cc = ccell[t];
        for (int j = 0; j < t && ok; j++) ok = (ccell[j] != cc);
        cok[t] = ok;
        cceil[t] = ok ? f_mul(a.lam[h], ceil[cc]) : 0.0f;
        ccen[t] = f_mul((float)cc + 0.5f, (float)FSATTN_CELL);
    }
    __syncthreads();
    // the candidates' mean keys as bf16 (exact: they are bf16 values), zeros for the slots that are not ok
    for (int i = tid; i < NT * 8 * 8; i += 128) {
        const int t = i >> 3, e = i & 7;
        uint4 w = make_uint4(0u, 0u, 0u, 0u);
        if (cok[t]) {
            const float4 lo = reinterpret_cast<const float4*>(kbar + (int64_t)ccell[t] * D)[2 * e];
            const float4 hi = reinterpret_cast<const float4*>(kbar + (int64_t)ccell[t] * D)[2 * e + 1];
            w.x = pack_bf2(lo.x, lo.y); w.y = pack_bf2(lo.z, lo.w); w.z = pack_bf2(hi.x, hi.y); w.w = pack_bf2(hi.z, hi.w);
        }
        *reinterpret_cast<uint4*>(kb + sel_sw(t, e)) = w;
    }
    __syncthreads();

    // ---- dot products: this warp's 32 queries x all candidate tiles ----
    uint32_t qf[2][4][4];
#pragma unroll
    for (int mt = 0; mt < 2; mt++)
#pragma unroll
        for (int kk = 0; kk < 4; kk++) {
            // matrices: (rows 0-7, chunk 2kk), (rows 8-15, chunk 2kk), (rows 0-7, chunk 2kk+1), (rows 8-15, chunk 2kk+1)
            const int row = warp * 32 + mt * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
            const uint32_t addr = (uint32_t)__cvta_generic_to_shared(qs + sel_sw(row, 2 * kk + (lane >> 4)));
            asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                         : "=r"(qf[mt][kk][0]), "=r"(qf[mt][kk][1]), "=r"(qf[mt][kk][2]), "=r"(qf[mt][kk][3]) : "r"(addr));
        }
    __syncthreads();                            // the score array reuses the Q tile from here on
    const int g = lane >> 2, tg = lane & 3;
    uint32_t k_ld[2];
#pragma unroll
    for (int kp = 0; kp < 2; kp++) k_ld[kp] = (uint32_t)__cvta_generic_to_shared(kb + sel_sw(lane & 7, kp * 4 + (lane >> 3)));
    float* scw = sc + (size_t)warp * 32 * SM_SCLD;
    // ---- one query per thread for the walk over the scores: prior, sorted insert (slots in ascending order) ----
    const int qi = blk_start + tid;
    const float inv_two_sigma = f_div(1.0f, f_mul(2.0f, a.sigma[h]));
    const float qpos = (float)qi;
    const float* myrow = sc + (size_t)tid * SM_SCLD;
    float ts[KMAX];
    int tslot[KMAX];
#pragma unroll
    for (int j = 0; j < KMAX; j++) { ts[j] = -INFINITY; tslot[j] = -1; }
    for (int nt0 = 0; nt0 < NT; nt0 += SM_NTH) {
        const int nt1 = min(NT, nt0 + SM_NTH);
        for (int nt = nt0; nt < nt1; nt++) {
            float c[2][4];
#pragma unroll
            for (int mt = 0; mt < 2; mt++) c[mt][0] = c[mt][1] = c[mt][2] = c[mt][3] = 0.f;
#pragma unroll
            for (int kp = 0; kp < 2; kp++) {
                uint32_t b0, b1, b2, b3;
                asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                             : "=r"(b0), "=r"(b1), "=r"(b2), "=r"(b3) : "r"(k_ld[kp] + nt * 8 * 128));
#pragma unroll
                for (int mt = 0; mt < 2; mt++) {
                    asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
                                 : "+f"(c[mt][0]), "+f"(c[mt][1]), "+f"(c[mt][2]), "+f"(c[mt][3])
                                 : "r"(qf[mt][2 * kp][0]), "r"(qf[mt][2 * kp][1]), "r"(qf[mt][2 * kp][2]), "r"(qf[mt][2 * kp][3]), "r"(b0), "r"(b1));
                    asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
                                 : "+f"(c[mt][0]), "+f"(c[mt][1]), "+f"(c[mt][2]), "+f"(c[mt][3])
                                 : "r"(qf[mt][2 * kp + 1][0]), "r"(qf[mt][2 * kp + 1][1]), "r"(qf[mt][2 * kp + 1][2]), "r"(qf[mt][2 * kp + 1][3]), "r"(b2), "r"(b3));
                }
            }
#pragma unroll
            for (int mt = 0; mt < 2; mt++) {
                const int col = (nt - nt0) * 8 + tg * 2;
                scw[(mt * 16 + g) * SM_SCLD + col] = c[mt][0];
                scw[(mt * 16 + g) * SM_SCLD + col + 1] = c[mt][1];
                scw[(mt * 16 + g + 8) * SM_SCLD + col] = c[mt][2];
                scw[(mt * 16 + g + 8) * SM_SCLD + col + 1] = c[mt][3];
            }
        }
        __syncwarp();
        const int t1 = min(C, nt1 * 8);
        for (int t = nt0 * 8; t < t1; t++) {
            float score = FS_NEG_SCORE;
            if (cok[t]) score = f_add(f_mul(myrow[t - nt0 * 8], a.scale), sel_prior(cceil[t], ccen[t], qpos, inv_two_sigma));
            sel_insert<KMAX>(ts, tslot, score, t);
        }
        __syncwarp();                   // the warp's rows are rewritten by the next half
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

template <int KMAX>
static int launch_select_mma(const fsattn_fsl_select_t* a, cudaStream_t st) {
    static bool opted[16] = {false};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 16 && !opted[dev]) {
        if (cudaFuncSetAttribute(fsl_select_mma_kernel<KMAX>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)SelMmaSmem::TOTAL) != cudaSuccess) {
            (void)cudaGetLastError();
            fs_set_error("fsl_select: cannot opt in to %zu bytes of shared memory", (size_t)SelMmaSmem::TOTAL);
            return FSATTN_ELAUNCH;
        }
        opted[dev] = true;
    }
    dim3 grid(a->nb, a->B * a->H);
    fsl_select_mma_kernel<KMAX><<<grid, 128, SelMmaSmem::TOTAL, st>>>(*a);
    return fs_check_launch("fsl_select_mma");
}

static size_t select_smem(int C, int D) { return (size_t)C * D * 4 + (size_t)C * 16; }

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
    if (a->impl != 1 && a->D == 64 && a->Bq == 128 && a->P + a->Wc <= SM_MAXC)
        return a->kk <= 4 ? launch_select_mma<5>(a, st) : launch_select_mma<FSATTN_MAX_KK + 1>(a, st);
    switch (a->D) {
        case 64: return launch_select<64>(a, st);
        case 96: return launch_select<96>(a, st);
        default: return launch_select<128>(a, st);
    }
}
