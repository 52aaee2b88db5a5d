// Fused readout + combine for whole 128-query blocks, head_dim 64, on tensor-core tiles.
//
// One CTA (8 warps) per (b, h, 128-query block); a warp owns 16 queries for the whole kernel and keeps their softmax
// state (running max, sum, 16 x 64 fp32 output tile) in registers, flash-attention style. The block's distinct selected
// cells are found once (bitmap + ranks); every warp then stages, one after the other, the cells that at least one of its
// queries selected (K and V rows, 16-byte chunks XOR-swizzled by the row, cp.async into private 4 KB buffers, one tile
// ahead of the MMAs - no block-wide barrier in the loop) and processes each: S = Q K^T (16 x 32, bf16
// mma.sync m16n8k16, fp32 accumulate), rows that did not select the cell masked out, online softmax, O += P V with P
// split into a bf16 high and low part (two MMAs) so that the probabilities keep ~16 bits. Cells are visited in ascending
// order, so the result is deterministic. ~110 KB of shared memory: two CTAs per SM.
#include "common.cuh"

namespace {

constexpr int RM_Q = 128;
constexpr int RM_THREADS = 256;
constexpr int RM_WARPS = 8;
constexpr int RM_GC = 8;             // cells staged per round
constexpr int RM_D = 64;
constexpr int RM_ROWB = RM_D * 2;    // 128-byte rows
constexpr int RM_MAXU = RM_Q * FSATTN_MAX_KK;
constexpr int RM_WL = 16 * FSATTN_MAX_KK;   // most distinct cells the 16 queries of one warp can select

struct RmSmem {
    static constexpr size_t Q_OFF = 0;
    static constexpr size_t K_OFF = Q_OFF + (size_t)RM_Q * RM_ROWB;
    static constexpr size_t V_OFF = K_OFF + (size_t)RM_GC * 32 * RM_ROWB;
    static constexpr size_t SELU_OFF = V_OFF + (size_t)RM_GC * 32 * RM_ROWB;          // int16 [128][MAX_KK]
    static constexpr size_t UC_OFF = SELU_OFF + (size_t)RM_Q * FSATTN_MAX_KK * 2;     // int [MAXU] distinct cells ascending
    static constexpr size_t RMASK_OFF = UC_OFF + (size_t)RM_MAXU * 4;                  // uint16 [8 warps][MAXU], as 32-bit words
    static constexpr size_t BM_OFF = RMASK_OFF + (size_t)RM_WARPS * RM_MAXU * 2;       // bitmap 1024 words + ranks 1024 + 8
    static constexpr size_t TOTAL = BM_OFF + (2 * 1024 + 16) * 4;
    static constexpr size_t WL_OFF = BM_OFF;     // per warp: (cell, row mask) of its tiles; reuses the bitmap once it is dead
};
static_assert((size_t)RM_WARPS * RM_WL * 8 <= (2 * 1024 + 16) * 4, "tile lists must fit in the bitmap area");

__device__ __forceinline__ uint32_t rm_sw(int row, int byte_in_row) {
    return (uint32_t)(row * RM_ROWB + ((((byte_in_row >> 4) ^ (row & 7)) << 4) | (byte_in_row & 15)));
}

__device__ __forceinline__ float rm_ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}
__device__ __forceinline__ uint32_t rm_pack(float lo, float hi) {          // cvt.rn.bf16x2.f32: lo in bits 0..15
    const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<const uint32_t*>(&v);
}

__device__ __forceinline__ void rm_mma(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
                 : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
                 : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__global__ void __launch_bounds__(RM_THREADS, 2) readout_mma_kernel(const fsattn_readout_combine_t a) {
    using S = RmSmem;
    extern __shared__ __align__(16) unsigned char rm_smem[];
    unsigned char* qs = rm_smem + S::Q_OFF;
    unsigned char* ks = rm_smem + S::K_OFF;
    unsigned char* vs = rm_smem + S::V_OFF;
    int16_t* selu = reinterpret_cast<int16_t*>(rm_smem + S::SELU_OFF);
    int* ucell = reinterpret_cast<int*>(rm_smem + S::UC_OFF);
    unsigned* rmask = reinterpret_cast<unsigned*>(rm_smem + S::RMASK_OFF);
    unsigned* bitmap = reinterpret_cast<unsigned*>(rm_smem + S::BM_OFF);
    int* wscan = reinterpret_cast<int*>(bitmap + 1024);
    __shared__ int n_distinct_s;
    constexpr int D = RM_D;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int g = lane >> 2, tg = lane & 3;
    const int blk = blockIdx.x, bh = blockIdx.y;
    const int b = bh / a.H, h = bh - b * a.H;
    const int q0 = blk * RM_Q;
    const int bs = ((a.q_pos0 + q0) / a.Bq) * a.Bq;
    const int n_cells = (a.n_kv + FSATTN_CELL - 1) / FSATTN_CELL;
    const int vis_cells = min(n_cells, bs / FSATTN_CELL);
    const int nwords = (vis_cells + 31) / 32;

    // ---- stage q (swizzled), clear the bitmap and the row masks ----
    for (int i = tid; i < RM_Q * (D / 8); i += RM_THREADS) {
        const int r = i / (D / 8), e = i - r * (D / 8);
        uint4 w = make_uint4(0u, 0u, 0u, 0u);
        if (q0 + r < a.N)
            w = reinterpret_cast<const uint4*>((const bf16*)a.q.ptr + b * a.q.sb + h * a.q.sh + (int64_t)(q0 + r) * a.q.sn)[e];
        *reinterpret_cast<uint4*>(qs + rm_sw(r, e * 16)) = w;
    }
    for (int i = tid; i < nwords; i += RM_THREADS) bitmap[i] = 0u;
    for (int i = tid; i < RM_WARPS * RM_MAXU / 2; i += RM_THREADS) rmask[i] = 0u;
    __syncthreads();
    // ---- validated selections -> bitmap of distinct cells ----
    const int32_t* selg = a.sel + b * a.sel_sb + h * a.sel_sh;
    for (int i = tid; i < RM_Q; i += RM_THREADS) {
        int cells[FSATTN_MAX_KK];
#pragma unroll
        for (int j = 0; j < FSATTN_MAX_KK; j++) {
            int c = (j < a.kk && q0 + i < a.N) ? selg[(int64_t)(q0 + i) * a.kk + j] : -1;
            bool ok = (c >= 0) && (c < vis_cells);
#pragma unroll
            for (int jj = 0; jj < FSATTN_MAX_KK; jj++)
                if (jj < j && cells[jj] == c) ok = false;
            cells[j] = ok ? c : -1;
            if (ok) atomicOr(&bitmap[c >> 5], 1u << (c & 31));
            selu[i * FSATTN_MAX_KK + j] = (int16_t)(ok ? 0 : -1);
        }
    }
    __syncthreads();
    {   // rank of every set bit, compact ascending list of the distinct cells
        int mine = 0;
        for (int w = tid * 4; w < tid * 4 + 4; w++) mine += (w < nwords) ? __popc(bitmap[w]) : 0;
        int incl = mine;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) { const int v = __shfl_up_sync(FS_FULL, incl, o); if (lane >= o) incl += v; }
        if (lane == 31) wscan[warp] = incl;
        __syncthreads();
        int base = 0;
        for (int w = 0; w < warp; w++) base += wscan[w];
        int run = base + incl - mine;
        for (int w = tid * 4; w < tid * 4 + 4 && w < nwords; w++) {
            unsigned bits = bitmap[w];
            wscan[8 + w] = run;
            while (bits) {
                const int bit = __ffs(bits) - 1;
                bits &= bits - 1;
                if (run < RM_MAXU) ucell[run] = w * 32 + bit;
                run++;
            }
        }
        if (tid == RM_THREADS - 1) n_distinct_s = base + incl;
    }
    __syncthreads();
    for (int i = tid; i < RM_Q; i += RM_THREADS) {
#pragma unroll
        for (int j = 0; j < FSATTN_MAX_KK; j++) {
            if (j < a.kk && selu[i * FSATTN_MAX_KK + j] == 0) {
                const int c = selg[(int64_t)(q0 + i) * a.kk + j];
                const unsigned below = bitmap[c >> 5] & ((1u << (c & 31)) - 1u);
                const int u = wscan[8 + (c >> 5)] + __popc(below);
                selu[i * FSATTN_MAX_KK + j] = (int16_t)u;
                const int idx = (i >> 4) * RM_MAXU + u;                       // (warp that owns query i, distinct cell u)
                atomicOr(&rmask[idx >> 1], (1u << (i & 15)) << ((idx & 1) * 16));
            }
        }
    }
    __syncthreads();
    const int n_distinct = min(n_distinct_s, RM_MAXU);

    // ---- this warp's queries: A fragments of Q for the four k-steps, softmax state ----
    const int r_lo = warp * 16 + g, r_hi = r_lo + 8;
    uint32_t qf[4][4];
#pragma unroll
    for (int kk = 0; kk < 4; kk++) {
        qf[kk][0] = *reinterpret_cast<const uint32_t*>(qs + rm_sw(r_lo, kk * 32 + tg * 4));
        qf[kk][1] = *reinterpret_cast<const uint32_t*>(qs + rm_sw(r_hi, kk * 32 + tg * 4));
        qf[kk][2] = *reinterpret_cast<const uint32_t*>(qs + rm_sw(r_lo, kk * 32 + 16 + tg * 4));
        qf[kk][3] = *reinterpret_cast<const uint32_t*>(qs + rm_sw(r_hi, kk * 32 + 16 + tg * 4));
    }
    float O[8][4];
#pragma unroll
    for (int nt = 0; nt < 8; nt++)
#pragma unroll
        for (int e = 0; e < 4; e++) O[nt][e] = 0.f;
    float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.f, 0.f};

    const bf16* kbase = (const bf16*)a.k.ptr + b * a.k.sb + h * a.k.sh;
    const bf16* vbase = (const bf16*)a.v.ptr + b * a.v.sb + h * a.v.sh;
    constexpr int CH = D / 8;
    // Every warp walks the distinct cells its own 16 queries selected, in ascending order, and stages each one (K and V
    // rows, 4 KB each) into its private buffers with asynchronous 16-byte copies: no block-wide barrier in the loop. The
    // copies run one tile ahead: K of the next cell is requested as soon as the scores of this one are out of the K buffer,
    // V of the next cell as soon as this cell's P V is done, so a load overlaps the softmax and the other operand's MMAs.
    unsigned char* kw = ks + (size_t)warp * 32 * RM_ROWB;
    unsigned char* vw = vs + (size_t)warp * 32 * RM_ROWB;
    int2* wl = reinterpret_cast<int2*>(rm_smem + S::WL_OFF) + warp * RM_WL;
    int n_tiles = 0;
    for (int u0 = 0; u0 < n_distinct; u0 += 32) {
        const int ul = u0 + lane;
        unsigned mask_l = 0;
        if (ul < n_distinct) {
            const int idx = warp * RM_MAXU + ul;
            mask_l = (rmask[idx >> 1] >> ((idx & 1) * 16)) & 0xffffu;
        }
        const unsigned need = __ballot_sync(FS_FULL, mask_l != 0);
        if (mask_l != 0) wl[n_tiles + __popc(need & ((1u << lane) - 1u))] = make_int2(ucell[ul], (int)mask_l);
        n_tiles += __popc(need);
    }
    __syncwarp();
    // staging: lane -> (row group lane >> 3, 16-byte chunk lane & 7); iteration it adds four rows. The swizzled chunk only
    // depends on the parity of it, so the destination is one of two per-lane bases plus a constant
    const int st_r = lane >> 3, st_e = lane & 7;
    const uint32_t st_d0 = (uint32_t)(st_r * RM_ROWB + ((st_e ^ st_r) << 4));
    const uint32_t st_d1 = (uint32_t)(st_r * RM_ROWB + ((st_e ^ (4 + st_r)) << 4));
    auto stage = [&](unsigned char* dst, const bf16* base, int64_t sn, int cell) {
        const uint32_t d = (uint32_t)__cvta_generic_to_shared(dst);
        const int lim = min(FSATTN_CELL, a.n_kv - cell * FSATTN_CELL);          // rows of the cell that exist (32 but for a ragged tail)
        const bf16* src = base + ((int64_t)cell * FSATTN_CELL + st_r) * sn + st_e * 8;
#pragma unroll
        for (int it = 0; it < CH; it++) {
            const int row = it * 4 + st_r;
            const int nbytes = row < lim ? 16 : 0;
            asm volatile("cp.async.ca.shared.global [%0], [%1], 16, %2;" ::"r"(d + it * 4 * RM_ROWB + ((it & 1) ? st_d1 : st_d0)),
                         "l"(row < lim ? src + (int64_t)it * 4 * sn : base), "r"(nbytes));
        }
    };
    // fragment-load addresses do not change from tile to tile (the warp's buffers are fixed): K by (k-step pair), V by
    // (pair of 8-dim column tiles); the tile row / token half is a constant offset
    uint32_t k_ld[2], v_ld[4];
#pragma unroll
    for (int kp = 0; kp < 2; kp++)
        k_ld[kp] = (uint32_t)__cvta_generic_to_shared(kw + rm_sw(lane & 7, (kp * 4 + (lane >> 3)) * 16));
#pragma unroll
    for (int np = 0; np < 4; np++)
        v_ld[np] = (uint32_t)__cvta_generic_to_shared(vw + rm_sw((lane & 7) + ((lane >> 3) & 1) * 8, (np * 2 + (lane >> 4)) * 16));
    const float sl2 = a.scale * 1.4426950408889634f;
    if (n_tiles > 0) {
        const int c0 = wl[0].x;
        stage(kw, kbase, a.k.sn, c0);
        asm volatile("cp.async.commit_group;" ::: "memory");
        stage(vw, vbase, a.v.sn, c0);
        asm volatile("cp.async.commit_group;" ::: "memory");
    }
    {
        for (int t = 0; t < n_tiles; t++) {
            const int2 ent = wl[t];
            const int cell = ent.x;
            const unsigned mask = (unsigned)ent.y;
            const int next_cell = (t + 1 < n_tiles) ? wl[t + 1].x : -1;
            asm volatile("cp.async.wait_group 1;" ::: "memory");      // K of this cell has landed (V may still be in flight)
            __syncwarp();
            // ---- S = Q K^T over the cell's 32 tokens: per 8-token tile two ldmatrix.x4 bring the B fragments of all four
            // k-steps (matrix j of a load = 16-byte chunk kp*4 + j of the tile's eight rows) ----
            float s[4][4];
#pragma unroll
            for (int nt = 0; nt < 4; nt++) {
#pragma unroll
                for (int e = 0; e < 4; e++) s[nt][e] = 0.f;
#pragma unroll
                for (int kp = 0; kp < 2; kp++) {
                    uint32_t b0, b1, b2, b3;
                    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                                 : "=r"(b0), "=r"(b1), "=r"(b2), "=r"(b3) : "r"(k_ld[kp] + nt * 8 * RM_ROWB));
                    rm_mma(s[nt], qf[2 * kp], b0, b1);
                    rm_mma(s[nt], qf[2 * kp + 1], b2, b3);
                }
            }
            __syncwarp();                                             // every lane has read its K fragments
            if (next_cell >= 0) stage(kw, kbase, a.k.sn, next_cell);
            asm volatile("cp.async.commit_group;" ::: "memory");      // (an empty group after the last tile keeps the count)
            // ---- mask, online softmax in the log2 domain (rows g: s[.][0..1]; rows g+8: s[.][2..3]) ----
            // A selected cell lies wholly before the query block, so every token is causal; only a ragged last cell needs a
            // per-token mask. A row that did not select the cell contributes nothing.
            const int lim = a.n_kv - cell * FSATTN_CELL;
            if (lim < FSATTN_CELL) {
#pragma unroll
                for (int nt = 0; nt < 4; nt++)
#pragma unroll
                    for (int e = 0; e < 4; e++)
                        if (nt * 8 + tg * 2 + (e & 1) >= lim) s[nt][e] = -INFINITY;
            }
            uint32_t p_hi[4][2], p_lo[4][2];           // per n-tile: packed probabilities of row g and row g+8
            float alpha[2];
#pragma unroll
            for (int half = 0; half < 2; half++) {
                if (((mask >> (8 * half)) & 0xffu) == 0u) {            // none of these eight rows selected the cell (warp-uniform)
#pragma unroll
                    for (int nt = 0; nt < 4; nt++) p_hi[nt][half] = p_lo[nt][half] = 0u;
                    alpha[half] = 1.0f;
                    continue;
                }
                const bool rsel = (mask >> (g + 8 * half)) & 1u;
                float mt = fmaxf(fmaxf(fmaxf(s[0][2 * half], s[0][2 * half + 1]), fmaxf(s[1][2 * half], s[1][2 * half + 1])),
                                 fmaxf(fmaxf(s[2][2 * half], s[2][2 * half + 1]), fmaxf(s[3][2 * half], s[3][2 * half + 1])));
                mt = rsel ? mt * sl2 : -INFINITY;
                mt = fmaxf(mt, __shfl_xor_sync(FS_FULL, mt, 1));
                mt = fmaxf(mt, __shfl_xor_sync(FS_FULL, mt, 2));
                const float m_new = fmaxf(m_run[half], mt);
                const float m_safe = (m_new == -INFINITY) ? 0.0f : m_new;      // a row with nothing yet: exp2(-inf - 0) = 0
                const float al = rm_ex2(m_run[half] - m_safe);
                float psum = 0.f;
#pragma unroll
                for (int nt = 0; nt < 4; nt++) {
                    const float p0 = rsel ? rm_ex2(fmaf(s[nt][2 * half], sl2, -m_safe)) : 0.0f;
                    const float p1 = rsel ? rm_ex2(fmaf(s[nt][2 * half + 1], sl2, -m_safe)) : 0.0f;
                    psum += p0 + p1;
                    const uint32_t hi = rm_pack(p0, p1);                       // one packed convert for the pair
                    p_hi[nt][half] = hi;
                    p_lo[nt][half] = rm_pack(p0 - bf_lo(hi), p1 - bf_hi(hi));
                }
                psum += __shfl_xor_sync(FS_FULL, psum, 1);
                psum += __shfl_xor_sync(FS_FULL, psum, 2);
                l_run[half] = l_run[half] * al + psum;
                m_run[half] = m_new;
                alpha[half] = al;
            }
#pragma unroll
            for (int nt = 0; nt < 8; nt++) {
                O[nt][0] *= alpha[0]; O[nt][1] *= alpha[0];
                O[nt][2] *= alpha[1]; O[nt][3] *= alpha[1];
            }
            asm volatile("cp.async.wait_group 1;" ::: "memory");      // V of this cell has landed (the next K may be in flight)
            __syncwarp();
            // ---- O += P V: two k-steps of 16 tokens, eight 8-dim column tiles; V fragments by ldmatrix.trans ----
#pragma unroll
            for (int k2 = 0; k2 < 2; k2++) {
                const uint32_t ah[4] = {p_hi[2 * k2][0], p_hi[2 * k2][1], p_hi[2 * k2 + 1][0], p_hi[2 * k2 + 1][1]};
                const uint32_t alo[4] = {p_lo[2 * k2][0], p_lo[2 * k2][1], p_lo[2 * k2 + 1][0], p_lo[2 * k2 + 1][1]};
#pragma unroll
                for (int np = 0; np < 4; np++) {                       // two column tiles per ldmatrix.x4
                    uint32_t v0, v1, v2, v3;
                    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                                 : "=r"(v0), "=r"(v1), "=r"(v2), "=r"(v3) : "r"(v_ld[np] + k2 * 16 * RM_ROWB));
                    rm_mma(O[np * 2], ah, v0, v1);
                    rm_mma(O[np * 2], alo, v0, v1);
                    rm_mma(O[np * 2 + 1], ah, v2, v3);
                    rm_mma(O[np * 2 + 1], alo, v2, v3);
                }
            }
            __syncwarp();                                             // every lane has read its V fragments
            if (next_cell >= 0) stage(vw, vbase, a.v.sn, next_cell);
            asm volatile("cp.async.commit_group;" ::: "memory");
        }
    }
    asm volatile("cp.async.wait_group 0;" ::: "memory");

    // ---- o -> bf16, lr_norm, combine with the window output ----
    const float glrs = a.lrs[h];
#pragma unroll
    for (int half = 0; half < 2; half++) {
        const int r = half ? r_hi : r_lo;
        const float l = l_run[half];
        float o[16], ss = 0.f;
#pragma unroll
        for (int nt = 0; nt < 8; nt++)
#pragma unroll
            for (int e = 0; e < 2; e++) {
                const float v = (l > 0.f) ? bf_round(O[nt][2 * half + e] / l) : 0.f;
                o[nt * 2 + e] = v;
                ss = fmaf(v, v, ss);
            }
        ss += __shfl_xor_sync(FS_FULL, ss, 1);
        ss += __shfl_xor_sync(FS_FULL, ss, 2);
        if (q0 + r >= a.N) continue;
        const float rn = f_div(1.0f, f_sqrt(f_add(ss * (1.0f / D), a.eps)));
        const int64_t row = ((int64_t)b * a.N + q0 + r) * ((int64_t)a.H * D) + (int64_t)h * D;
        const bf16* srp = (const bf16*)a.sr + row;
        bf16* yp = (bf16*)a.y + row;
#pragma unroll
        for (int nt = 0; nt < 8; nt++) {
            const int d = nt * 8 + tg * 2;
            float y[2];
#pragma unroll
            for (int e = 0; e < 2; e++) {
                const float lr = f_mul(f_mul(o[nt * 2 + e], rn), a.norm_w[d + e]);
                const float sr = (a.sr != nullptr) ? __bfloat162float(srp[d + e]) : 0.0f;
                y[e] = f_add(sr, f_mul(glrs, lr));
            }
            *reinterpret_cast<uint32_t*>(yp + d) = pack_bf2(y[0], y[1]);
        }
    }
}

}  // namespace

int fs_readout_mma(const fsattn_readout_combine_t* a, cudaStream_t st) {
    const size_t smem = RmSmem::TOTAL;
    static bool opted[16] = {false};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 16 && !opted[dev]) {
        if (cudaFuncSetAttribute(readout_mma_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess) {
            (void)cudaGetLastError();
            fs_set_error("readout_combine: cannot opt in to %zu bytes of shared memory", smem);
            return FSATTN_ELAUNCH;
        }
        opted[dev] = true;
    }
    dim3 grid((a->N + RM_Q - 1) / RM_Q, a->B * a->H);
    readout_mma_kernel<<<grid, RM_THREADS, smem, st>>>(*a);
    return fs_check_launch("readout_mma");
}
