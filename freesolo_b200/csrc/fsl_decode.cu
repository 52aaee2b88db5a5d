// One FS-L decode token of one layer in one launch: window branch (RoPE, int8/bf16 KV gather, softmax, PV), long-range
// branch (score the block's candidate pool against the chunk-mean keys, top-kk, readout of kk*32 un-rotated tokens,
// lr_norm), the combine, and the KV bookkeeping (append the new row, close a cell every 32 tokens: statistics + int8
// quantisation [+ slot allocation], refresh the block's top-P list every Bq tokens [+ free unreadable slots]).
//
// Work decomposition: `splits` CTAs per (b,h) form a thread-block cluster. Rank 0 owns the long-range branch, the
// bookkeeping and the final combine; ranks >= 1 split the window rows (with splits == 1 the one CTA does both in turn).
// Window partials (running max, sum, accumulator) travel to rank 0 through distributed shared memory.
//
// HBM traffic per (b,h): (W+1) rows of K and V (int8: D bytes each), P+Wc mean keys (D*4 bytes) + ceilings, kk*32 rows of
// K and V, the new row. Rows are fetched 8 per warp instruction, 4 lanes per row, each lane the same dims of both rotary
// halves so that RoPE needs no shuffles.
#include <cooperative_groups.h>

#include "common.cuh"
#include "cell_warp.cuh"
#include "pool_list.cuh"

namespace cg = cooperative_groups;

namespace {

constexpr int NWARP = 8;
constexpr int MAXC = FSATTN_MAX_POOL + 8;

template <int D>
struct RowL {
    static constexpr int HALF = D / 2;
    static constexpr int DPL = HALF / 4;  // dims per lane and half: 8, 12, 16
    static constexpr int NW = DPL / 4;    // 4-value words per lane and half
};

// raw words of one row for this lane: [0, NW) first half, [NW, 2NW) second half
template <int D, bool I8>
struct RawRow {
    uint2 w[2 * RowL<D>::NW];  // int8 rows use only .x
};

template <int D, bool I8>
__device__ __forceinline__ void raw_load(RawRow<D, I8>& r, const void* row, int sub, bool valid) {
    using L = RowL<D>;
#pragma unroll
    for (int i = 0; i < 2 * L::NW; i++) r.w[i] = make_uint2(0u, 0u);
    if (!valid) return;
    if (I8) {
        const uint32_t* p0 = reinterpret_cast<const uint32_t*>((const int8_t*)row + sub * L::DPL);
        const uint32_t* p1 = reinterpret_cast<const uint32_t*>((const int8_t*)row + L::HALF + sub * L::DPL);
#pragma unroll
        for (int i = 0; i < L::NW; i++) { r.w[i].x = p0[i]; r.w[L::NW + i].x = p1[i]; }
    } else {
        const uint2* p0 = reinterpret_cast<const uint2*>((const bf16*)row + sub * L::DPL);
        const uint2* p1 = reinterpret_cast<const uint2*>((const bf16*)row + L::HALF + sub * L::DPL);
#pragma unroll
        for (int i = 0; i < L::NW; i++) { r.w[i] = p0[i]; r.w[L::NW + i] = p1[i]; }
    }
}

// the lane's values of a row as fp32; int8 rows are read as bf16(f32(code) * f32(scale)) like the reference's int8 read
template <int D, bool I8>
__device__ __forceinline__ void raw_floats(const RawRow<D, I8>& r, float sc, float* lo, float* hi) {
    using L = RowL<D>;
#pragma unroll
    for (int i = 0; i < L::NW; i++) {
        if (I8) {
            unpack4_i8(r.w[i].x, lo + 4 * i);
            unpack4_i8(r.w[L::NW + i].x, hi + 4 * i);
#pragma unroll
            for (int j = 0; j < 4; j++) {
                lo[4 * i + j] = bf_round(f_mul(lo[4 * i + j], sc));
                hi[4 * i + j] = bf_round(f_mul(hi[4 * i + j], sc));
            }
        } else {
            unpack4_bf(r.w[i], lo + 4 * i);
            unpack4_bf(r.w[L::NW + i], hi + 4 * i);
        }
    }
}

// One softmax partial per 4-lane group: all four lanes hold the same m and l and their own dims of acc.
template <int D>
struct Part {
    float m, l;
    float lo[RowL<D>::DPL], hi[RowL<D>::DPL];
    __device__ __forceinline__ void init() {
        m = -INFINITY; l = 0.0f;
#pragma unroll
        for (int j = 0; j < RowL<D>::DPL; j++) { lo[j] = 0.0f; hi[j] = 0.0f; }
    }
};

// score one row (4 lanes), fold it into the group's partial
template <int D, bool I8, bool ROPE>
__device__ __forceinline__ void attend_row(Part<D>& P, const void* krow, const void* vrow, float ksc, float vsc, bool valid,
                                           const bf16* cosr, const bf16* sinr, const float* qlo, const float* qhi,
                                           float scale, int sub) {
    using L = RowL<D>;
    RawRow<D, I8> rk, rv;
    raw_load<D, I8>(rk, krow, sub, valid);
    raw_load<D, I8>(rv, vrow, sub, valid);
    float klo[L::DPL], khi[L::DPL];
    raw_floats<D, I8>(rk, ksc, klo, khi);
    float dot = 0.0f;
    if (ROPE) {
        float c[L::DPL], s[L::DPL];
        if (valid) {
            const uint2* cp = reinterpret_cast<const uint2*>(cosr + sub * L::DPL);
            const uint2* sp = reinterpret_cast<const uint2*>(sinr + sub * L::DPL);
#pragma unroll
            for (int i = 0; i < L::NW; i++) { unpack4_bf(cp[i], c + 4 * i); unpack4_bf(sp[i], s + 4 * i); }
        } else {
#pragma unroll
            for (int j = 0; j < L::DPL; j++) { c[j] = 0.0f; s[j] = 0.0f; }
        }
#pragma unroll
        for (int j = 0; j < L::DPL; j++) {
            const float r1 = bf_round(klo[j] * c[j] - khi[j] * s[j]);
            const float r2 = bf_round(khi[j] * c[j] + klo[j] * s[j]);
            dot = fmaf(qlo[j], r1, dot);
            dot = fmaf(qhi[j], r2, dot);
        }
    } else {
#pragma unroll
        for (int j = 0; j < L::DPL; j++) {
            dot = fmaf(qlo[j], klo[j], dot);
            dot = fmaf(qhi[j], khi[j], dot);
        }
    }
    dot += __shfl_xor_sync(FS_FULL, dot, 1);
    dot += __shfl_xor_sync(FS_FULL, dot, 2);
    if (!valid) return;   // uniform within the 4-lane group; no shuffles below
    const float sc = dot * scale;
    float vlo[L::DPL], vhi[L::DPL];
    raw_floats<D, I8>(rv, vsc, vlo, vhi);
    const float m_new = fmaxf(P.m, sc);
    const float alpha = (P.m == -INFINITY) ? 0.0f : __expf(P.m - m_new);
    const float p = __expf(sc - m_new);
    P.l = P.l * alpha + p;
#pragma unroll
    for (int j = 0; j < L::DPL; j++) {
        P.lo[j] = fmaf(p, vlo[j], P.lo[j] * alpha);
        P.hi[j] = fmaf(p, vhi[j], P.hi[j] * alpha);
    }
    P.m = m_new;
}

// merge the 8 group partials of a warp (xor 4, 8, 16); afterwards every group holds the warp's partial
template <int D>
__device__ __forceinline__ void part_merge_warp(Part<D>& P) {
    using L = RowL<D>;
#pragma unroll
    for (int o = 4; o < 32; o <<= 1) {
        const float m_o = __shfl_xor_sync(FS_FULL, P.m, o);
        const float l_o = __shfl_xor_sync(FS_FULL, P.l, o);
        float m, fa, fb;
        softmax_merge_scalars(P.m, m_o, m, fa, fb);
        P.l = P.l * fa + l_o * fb;
#pragma unroll
        for (int j = 0; j < L::DPL; j++) {
            const float a_o = __shfl_xor_sync(FS_FULL, P.lo[j], o);
            const float b_o = __shfl_xor_sync(FS_FULL, P.hi[j], o);
            P.lo[j] = P.lo[j] * fa + a_o * fb;
            P.hi[j] = P.hi[j] * fa + b_o * fb;
        }
        P.m = m;
    }
}

// shared-memory record of a partial: [0] = m, [1] = l, [2 .. 2+D) = acc in natural dim order
template <int D>
__device__ __forceinline__ void part_store(const Part<D>& P, float* rec, int lane) {
    using L = RowL<D>;
    if (lane < 4) {
        if (lane == 0) { rec[0] = P.m; rec[1] = P.l; }
#pragma unroll
        for (int j = 0; j < L::DPL; j++) {
            rec[2 + lane * L::DPL + j] = P.lo[j];
            rec[2 + L::HALF + lane * L::DPL + j] = P.hi[j];
        }
    }
}

// merge n records (stride rs floats) into (m, l, acc[d]) for this lane's dims d = lane + 32 j; one warp
template <int D>
__device__ __forceinline__ void rec_merge(const float* recs, int n, int rs, int lane, float& l_out, float* acc) {
    float m = -INFINITY;
    for (int i = 0; i < n; i++) m = fmaxf(m, recs[i * rs]);
    float l = 0.0f;
#pragma unroll
    for (int j = 0; j < D / 32; j++) acc[j] = 0.0f;
    for (int i = 0; i < n; i++) {
        const float mi = recs[i * rs];
        if (mi == -INFINITY) continue;
        const float f = __expf(mi - m);
        l = fmaf(recs[i * rs + 1], f, l);
#pragma unroll
        for (int j = 0; j < D / 32; j++) acc[j] = fmaf(recs[i * rs + 2 + lane + 32 * j], f, acc[j]);
    }
    l_out = l;
}

struct RowSrc {
    const void* k; const void* v; float ksc, vsc; bool i8;
};

template <int D>
struct Smem {
    float q_raw[D];
    float q_rot[D];
    float lc[FSATTN_MAX_POOL];
    int li[FSATTN_MAX_POOL];
    int ccell[MAXC];
    int cok[MAXC];
    int cslot[MAXC];
    float cceil[MAXC];
    float score[MAXC];
    int selcell[FSATTN_MAX_KK];
    int selslot[FSATTN_MAX_KK];
    int n_list;
    float wrec[NWARP][D + 2];   // per-warp partials (window, then long-range)
    float win_rec[D + 2];       // this CTA's window partial (read by rank 0 through distributed shared memory)
    float lr_rec[D + 2];
};

template <int D>
__global__ void __launch_bounds__(NWARP * 32) fsl_decode_kernel(const fsattn_fsl_decode_t a) {
    using L = RowL<D>;
    __shared__ Smem<D> sm;
    cg::cluster_group cluster = cg::this_cluster();
    const int S = (int)gridDim.x;              // CTAs per (b,h) = cluster size
    const int rank = (int)blockIdx.x;
    const int bh = blockIdx.y;
    const fsattn_fsl_state_t& st = a.st;
    const int b = bh / st.H, h = bh - b * st.H;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int sub = lane & 3, grp = lane >> 2;
    const int mode = st.store_mode;

    const int64_t pos = *a.pos;
    const int64_t nq = (pos / FSATTN_CELL) * FSATTN_CELL;      // rows below nq are completed cells
    const int blk_start = (int)((pos / st.Bq) * st.Bq);
    const bool pos_ok = pos >= 0 && pos < st.cap_rows;

    const bf16* q_in = (const bf16*)a.q + b * a.in_sb + h * a.in_sh;
    const bf16* k_in = (const bf16*)a.k + b * a.in_sb + h * a.in_sh;
    const bf16* v_in = (const bf16*)a.v + b * a.in_sb + h * a.in_sh;
    const bf16* cosT = (const bf16*)a.cos;
    const bf16* sinT = (const bf16*)a.sin;

    // ---- q: raw and rotated (rounded to bf16 like the reference's rotated query), into shared memory -----------------
    for (int d = tid; d < L::HALF; d += blockDim.x) {
        const float x1 = __bfloat162float(q_in[d]), x2 = __bfloat162float(q_in[d + L::HALF]);
        const float c = __bfloat162float(cosT[pos * D + d]), s = __bfloat162float(sinT[pos * D + d]);
        sm.q_raw[d] = x1; sm.q_raw[d + L::HALF] = x2;
        sm.q_rot[d] = bf_round(x1 * c - x2 * s);
        sm.q_rot[d + L::HALF] = bf_round(x2 * c + x1 * s);
    }
    if (tid == 0 && !pos_ok) atomicAdd(st.status + FSATTN_ST_BAD_INDEX, 1);
    __syncthreads();

    const int8_t* kq = st.kq ? st.kq + b * st.q_sb + h * st.q_sh : nullptr;
    const int8_t* vq = st.vq ? st.vq + b * st.q_sb + h * st.q_sh : nullptr;
    const bf16* ks = st.ks ? (const bf16*)st.ks + b * st.sc_sb + h * st.sc_sh : nullptr;
    const bf16* vs = st.vs ? (const bf16*)st.vs + b * st.sc_sb + h * st.sc_sh : nullptr;
    bf16* khot = st.khot ? (bf16*)st.khot + b * st.hot_sb + h * st.hot_sh : nullptr;
    bf16* vhot = st.vhot ? (bf16*)st.vhot + b * st.hot_sb + h * st.hot_sh : nullptr;
    bf16* kbuf = st.kbuf ? (bf16*)st.kbuf + b * st.buf_sb + h * st.buf_sh : nullptr;
    bf16* vbuf = st.vbuf ? (bf16*)st.vbuf + b * st.buf_sb + h * st.buf_sh : nullptr;
    int32_t* slot_of = st.slot_of ? st.slot_of + b * st.so_sb + h * st.so_sh : nullptr;
    int32_t* cell_in = st.cell_in ? st.cell_in + b * st.ci_sb + h * st.ci_sh : nullptr;
    float* kbar = st.kbar + b * st.kbar_sb + h * st.kbar_sh;
    float* ceil = st.ceil + b * st.ceil_sb + h * st.ceil_sh;

    // ================= window branch =====================================================================================
    const bool do_window = (S == 1) || (rank > 0);
    if (do_window) {
        float qlo[L::DPL], qhi[L::DPL];
#pragma unroll
        for (int j = 0; j < L::DPL; j++) { qlo[j] = sm.q_rot[sub * L::DPL + j]; qhi[j] = sm.q_rot[L::HALF + sub * L::DPL + j]; }
        Part<D> P;
        P.init();
        const int64_t lo_row = (pos - st.W > 0) ? pos - st.W : 0;
        const int nw = (S == 1) ? NWARP : (S - 1) * NWARP;
        const int gw = (S == 1) ? warp : (rank - 1) * NWARP + warp;
        const int64_t g_lo = lo_row >> 3, g_hi = pos >> 3;
        for (int64_t g = g_lo + gw; g <= g_hi; g += nw) {
            const int64_t r = (g << 3) + grp;
            const bool valid = pos_ok && r >= lo_row && r <= pos;
            const void* kp = nullptr; const void* vp = nullptr;
            float ksc = 1.0f, vsc = 1.0f;
            bool i8 = false;
            if (r == pos) { kp = k_in; vp = v_in; }
            else if (mode == 0) { kp = kbuf + r * D; vp = vbuf + r * D; }
            else if (r >= nq) { kp = khot + (r - nq) * D; vp = vhot + (r - nq) * D; }
            else {
                i8 = true;
                int64_t cell = r / FSATTN_CELL;
                int64_t prow = r;
                bool have = true;
                if (mode == 2) {
                    const int slot = valid ? slot_of[cell] : -1;
                    have = slot >= 0;
                    prow = (int64_t)slot * FSATTN_CELL + (r - cell * FSATTN_CELL);
                    cell = slot;
                }
                if (valid && have) {
                    kp = kq + prow * D; vp = vq + prow * D;
                    ksc = __bfloat162float(ks[cell]); vsc = __bfloat162float(vs[cell]);
                }
            }
            const bool ok = valid && kp != nullptr;
            if (valid && !ok && sub == 0) atomicAdd(st.status + FSATTN_ST_POOL_NO_SLOT, 1);
            // all rows of an aligned 8-row group come from the same kind of storage, except the new token's row
            const bool any_i8 = __any_sync(FS_FULL, i8 && ok);
            const bf16* cr = cosT + r * D; const bf16* sr_ = sinT + r * D;
            if (any_i8) {
                attend_row<D, true, true>(P, kp, vp, ksc, vsc, ok && i8, cr, sr_, qlo, qhi, a.scale, sub);
                if (__any_sync(FS_FULL, ok && !i8))
                    attend_row<D, false, true>(P, kp, vp, 1.0f, 1.0f, ok && !i8, cr, sr_, qlo, qhi, a.scale, sub);
            } else {
                attend_row<D, false, true>(P, kp, vp, 1.0f, 1.0f, ok, cr, sr_, qlo, qhi, a.scale, sub);
            }
        }
        part_merge_warp<D>(P);
        part_store<D>(P, sm.wrec[warp], lane);
        __syncthreads();
        if (warp == 0) {
            float l, acc[D / 32];
            rec_merge<D>(&sm.wrec[0][0], NWARP, D + 2, lane, l, acc);
            float m = -INFINITY;
            for (int i = 0; i < NWARP; i++) m = fmaxf(m, sm.wrec[i][0]);
            if (lane == 0) { sm.win_rec[0] = m; sm.win_rec[1] = l; }
#pragma unroll
            for (int j = 0; j < D / 32; j++) sm.win_rec[2 + lane + 32 * j] = acc[j];
        }
        __syncthreads();
    }

    // ================= long-range branch + bookkeeping (rank 0) ==============================================================
    float lr_l = 0.0f;
    if (rank == 0) {
        // ---- append the new row; close the cell when this token completes it (last warp) --------------------------------
        if (warp == NWARP - 1 && pos_ok) {
            const int hr = (int)(pos - nq);
            if (mode == 0) {
                for (int d = lane; d < D; d += 32) { kbuf[pos * D + d] = k_in[d]; vbuf[pos * D + d] = v_in[d]; }
            } else {
                for (int d = lane; d < D; d += 32) { khot[hr * D + d] = k_in[d]; vhot[hr * D + d] = v_in[d]; }
            }
            if (hr == FSATTN_CELL - 1) {
                const int cell = (int)(pos / FSATTN_CELL);
                const bool in_table = cell < st.cap_cells;
                int dst = cell;          // where the quantised rows and the mean key go (cell or slot index)
                bool store_ok = in_table;
                if (mode == 2) {
                    int slot = -1;
                    for (int s0 = 0; s0 < st.n_slots && slot < 0; s0 += 32) {
                        const int si = s0 + lane;
                        const bool free_ = si < st.n_slots && cell_in[si] < 0;
                        const unsigned bal = __ballot_sync(FS_FULL, free_);
                        if (bal) slot = s0 + __ffs(bal) - 1;
                    }
                    store_ok = in_table && slot >= 0;
                    dst = slot;
                    if (!store_ok && lane == 0) atomicAdd(st.status + FSATTN_ST_SLOT_OVERFLOW, 1);
                    if (store_ok && lane == 0) { slot_of[cell] = slot; cell_in[slot] = cell; }
                }
                const bf16* kcell = (mode == 0) ? kbuf + nq * D : khot;
                const bf16* vcell = (mode == 0) ? vbuf + nq * D : vhot;
                CellRegs<D> cr;
                cell_load_rows<D>(cr, kcell, D, lane, k_in);
                float cl_tmp = 0.0f;
                (void)cl_tmp;
                if (mode == 2) {
                    // the ceiling table is indexed by cell, the mean keys by slot
                    cell_stats_warp<D>(cr, lane, store_ok ? kbar + (int64_t)dst * D : nullptr, in_table ? ceil + cell : nullptr);
                } else {
                    cell_stats_warp<D>(cr, lane, in_table ? kbar + (int64_t)cell * D : nullptr, in_table ? ceil + cell : nullptr);
                }
                if (mode != 0 && store_ok) {
                    cell_quant_warp<D>(cr, lane, const_cast<int8_t*>(kq) + (int64_t)dst * FSATTN_CELL * D, const_cast<bf16*>(ks) + dst);
                    cell_load_rows<D>(cr, vcell, D, lane, v_in);
                    cell_quant_warp<D>(cr, lane, const_cast<int8_t*>(vq) + (int64_t)dst * FSATTN_CELL * D, const_cast<bf16*>(vs) + dst);
                }
            }
        }

        // ---- the block's top-P list (refreshed when the block changed) ------------------------------------------------------
        const int M_vis = blk_start / FSATTN_CELL;
        int32_t* top_idx = st.top_idx + (int64_t)bh * st.P;
        if (warp == 0) {
            int n = 0;
            for (int p = lane; p < st.P; p += 32) {
                const int ci = top_idx[p];
                sm.li[p] = ci;
                sm.lc[p] = (ci >= 0) ? ceil[ci] : 0.0f;
                n += (ci >= 0);
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) n += __shfl_xor_sync(FS_FULL, n, o);
            __syncwarp();
            const int have_blk = st.top_blk[bh];
            if (have_blk != blk_start) {
                int c0 = have_blk / FSATTN_CELL; if (c0 < 0) c0 = 0;
                for (int c = c0; c < M_vis; c++) pool_list_insert(sm.lc, sm.li, n, st.P, ceil[c], c, lane);
                for (int p = lane; p < st.P; p += 32) top_idx[p] = (p < n) ? sm.li[p] : -1;
                if (lane == 0) st.top_blk[bh] = blk_start;
                if (mode == 2) {
                    // free the slots of cells no later step reads: below c_lo and outside the top-P
                    int c_lo = (blk_start - st.W) / FSATTN_CELL;
                    if ((blk_start - st.W) < 0) c_lo = -1;      // floor division of a negative number
                    if (M_vis - st.Wc < c_lo) c_lo = M_vis - st.Wc;
                    if (c_lo < 0) c_lo = 0;
                    for (int s0 = 0; s0 < st.n_slots; s0 += 32) {
                        const int si = s0 + lane;
                        if (si < st.n_slots) {
                            const int occ = cell_in[si];
                            if (occ >= 0 && occ < c_lo) {
                                bool in_top = false;
                                for (int p = 0; p < n; p++) in_top |= (sm.li[p] == occ);
                                if (!in_top) { cell_in[si] = -1; slot_of[occ] = -1; }
                            }
                        }
                    }
                }
            }
            if (lane == 0) sm.n_list = n;
        }
        __syncthreads();

        // ---- candidate slots ---------------------------------------------------------------------------------------------------
        const int C = st.P + st.Wc;
        const int n_list = sm.n_list;
        for (int t = tid; t < C; t += blockDim.x) {
            const int cand = (t < st.P) ? ((t < n_list) ? sm.li[t] : -1) : (M_vis - 1) - (t - st.P);
            const int cc = cand < 0 ? 0 : cand;
            sm.ccell[t] = cc;
            sm.cok[t] = (cand >= 0) && (cc < M_vis);
        }
        __syncthreads();
        for (int t = tid; t < C; t += blockDim.x) {
            int ok = sm.cok[t];
            const int cc = sm.ccell[t];
            for (int j = 0; j < t && ok; j++) ok = (sm.ccell[j] != cc);
            int slot = cc;
            if (ok && mode == 2) {
                slot = slot_of[cc];
                if (slot < 0) { atomicAdd(st.status + FSATTN_ST_POOL_NO_SLOT, 1); ok = 0; slot = 0; }
            }
            sm.cok[t] = ok;
            sm.cslot[t] = slot;
            sm.cceil[t] = ok ? ceil[cc] : 0.0f;
        }
        __syncthreads();

        // ---- scores: 8 lanes per candidate ---------------------------------------------------------------------------------------
        {
            constexpr int F = D / 8;             // floats per lane
            const int s8 = lane & 7;
            float qv[F];
#pragma unroll
            for (int j = 0; j < F; j++) qv[j] = sm.q_raw[s8 * F + j];
            const float lam = a.lam[h];
            const float two_sigma = f_mul(2.0f, a.sigma[h]);
            const float qpos = (float)pos;
            for (int t0 = warp * 4; t0 < C; t0 += NWARP * 4) {
                const int t = t0 + (lane >> 3);
                const bool ok = t < C && sm.cok[t];
                float dot = 0.0f;
                if (ok) {
                    const float4* kr = reinterpret_cast<const float4*>(kbar + (int64_t)sm.cslot[t] * D + s8 * F);
#pragma unroll
                    for (int j = 0; j < F / 4; j++) {
                        const float4 kv = kr[j];
                        dot = fmaf(qv[4 * j + 0], kv.x, dot); dot = fmaf(qv[4 * j + 1], kv.y, dot);
                        dot = fmaf(qv[4 * j + 2], kv.z, dot); dot = fmaf(qv[4 * j + 3], kv.w, dot);
                    }
                }
                dot += __shfl_xor_sync(FS_FULL, dot, 1);
                dot += __shfl_xor_sync(FS_FULL, dot, 2);
                dot += __shfl_xor_sync(FS_FULL, dot, 4);
                if (t < C && s8 == 0) {
                    float sc = FS_NEG_SCORE;
                    if (ok) sc = f_add(f_mul(dot, a.scale), fs_prior(lam, sm.cceil[t], qpos, sm.ccell[t], (float)FSATTN_CELL, two_sigma));
                    sm.score[t] = sc;
                }
            }
        }
        __syncthreads();

        // ---- top-kk by (score desc, slot asc): warp 0 ---------------------------------------------------------------------------------
        if (warp == 0) {
            constexpr int PER = (MAXC + 31) / 32;
            float sv[PER];
#pragma unroll
            for (int j = 0; j < PER; j++) { const int t = lane + 32 * j; sv[j] = (t < C) ? sm.score[t] : -INFINITY; }
            for (int k = 0; k < st.kk; k++) {
                float best = -INFINITY; int bslot = 0x7fffffff;
#pragma unroll
                for (int j = 0; j < PER; j++) {
                    const int t = lane + 32 * j;
                    if (sv[j] > best) { best = sv[j]; bslot = t; }     // ascending t: ties keep the lower slot
                }
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) {
                    const float ob = __shfl_xor_sync(FS_FULL, best, o);
                    const int os = __shfl_xor_sync(FS_FULL, bslot, o);
                    if (ob > best || (ob == best && os < bslot)) { best = ob; bslot = os; }
                }
                int cell = -1, slot = -1;
                if (best > -INFINITY && bslot < C) {
                    if (sm.cok[bslot]) { cell = sm.ccell[bslot]; slot = sm.cslot[bslot]; }
#pragma unroll
                    for (int j = 0; j < PER; j++) if (lane + 32 * j == bslot) sv[j] = -INFINITY;
                }
                if (lane == 0) {
                    sm.selcell[k] = cell; sm.selslot[k] = slot;
                    if (a.sel_out != nullptr) a.sel_out[(int64_t)bh * st.kk + k] = cell;
                }
            }
        }
        __syncthreads();

        // ---- readout of the selected cells: 4 groups of 8 rows per cell, spread over the warps ----------------------------------------
        {
            float qlo[L::DPL], qhi[L::DPL];
#pragma unroll
            for (int j = 0; j < L::DPL; j++) { qlo[j] = sm.q_raw[sub * L::DPL + j]; qhi[j] = sm.q_raw[L::HALF + sub * L::DPL + j]; }
            Part<D> P;
            P.init();
            const int ngroups = st.kk * 4;
            for (int gi = warp; gi < ngroups; gi += NWARP) {
                const int k = gi >> 2;
                const int cell = sm.selcell[k];
                if (cell < 0) continue;                       // warp-uniform
                const int rr = ((gi & 3) << 3) + grp;
                const int64_t tok = (int64_t)cell * FSATTN_CELL + rr;
                const bool valid = pos_ok && tok < pos;
                if (mode == 0) {
                    attend_row<D, false, false>(P, kbuf + tok * D, vbuf + tok * D, 1.0f, 1.0f, valid, nullptr, nullptr, qlo, qhi, a.scale, sub);
                } else {
                    const int64_t base = (mode == 2) ? (int64_t)sm.selslot[k] : (int64_t)cell;
                    const int64_t prow = base * FSATTN_CELL + rr;
                    attend_row<D, true, false>(P, kq + prow * D, vq + prow * D, __bfloat162float(ks[base]), __bfloat162float(vs[base]),
                                               valid, nullptr, nullptr, qlo, qhi, a.scale, sub);
                }
            }
            part_merge_warp<D>(P);
            part_store<D>(P, sm.wrec[warp], lane);
        }
        __syncthreads();
        if (warp == 0) {
            float acc[D / 32];
            rec_merge<D>(&sm.wrec[0][0], NWARP, D + 2, lane, lr_l, acc);
            if (lane == 0) sm.lr_rec[1] = lr_l;
#pragma unroll
            for (int j = 0; j < D / 32; j++) sm.lr_rec[2 + lane + 32 * j] = acc[j];
        }
    }

    // ================= exchange + combine ============================================================================================
    if (S > 1) cluster.sync();
    if (rank == 0 && warp == 0) {
        // window: merge the partials of the window CTAs
        float wm = -INFINITY;
        const int first = (S == 1) ? 0 : 1;
        for (int r = first; r < S; r++) {
            const float* rec = (S == 1) ? sm.win_rec : cluster.map_shared_rank(sm.win_rec, r);
            wm = fmaxf(wm, rec[0]);
        }
        float wl = 0.0f, wacc[D / 32];
#pragma unroll
        for (int j = 0; j < D / 32; j++) wacc[j] = 0.0f;
        for (int r = first; r < S; r++) {
            const float* rec = (S == 1) ? sm.win_rec : cluster.map_shared_rank(sm.win_rec, r);
            const float mi = rec[0];
            if (mi == -INFINITY) continue;
            const float f = __expf(mi - wm);
            wl = fmaf(rec[1], f, wl);
#pragma unroll
            for (int j = 0; j < D / 32; j++) wacc[j] = fmaf(rec[2 + lane + 32 * j], f, wacc[j]);
        }
        const float winv = (wl > 0.0f) ? 1.0f / wl : 0.0f;
        const float linv = (lr_l > 0.0f) ? 1.0f / lr_l : 0.0f;
        float o[D / 32], ss = 0.0f;
#pragma unroll
        for (int j = 0; j < D / 32; j++) {
            o[j] = bf_round(sm.lr_rec[2 + lane + 32 * j] * linv);
            ss = fmaf(o[j], o[j], ss);
        }
        ss = warp_sum(ss);
        const float rn = f_div(1.0f, f_sqrt(f_add(ss * (1.0f / D), a.eps)));
        const float g = a.lrs[h];
        bf16* yp = (bf16*)a.y + (int64_t)b * st.H * D + (int64_t)h * D;
#pragma unroll
        for (int j = 0; j < D / 32; j++) {
            const int d = lane + 32 * j;
            const float sr = bf_round(wacc[j] * winv);
            const float lr = f_mul(f_mul(o[j], rn), a.norm_w[d]);
            yp[d] = __float2bfloat16_rn(f_add(sr, f_mul(g, lr)));
        }
    }
    if (S > 1) cluster.sync();   // remote shared memory stays valid until rank 0 has read it
}

template <int D>
int launch_decode(const fsattn_fsl_decode_t* a, cudaStream_t stream) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(a->splits, a->st.B * a->st.H, 1);
    cfg.blockDim = dim3(NWARP * 32, 1, 1);
    cfg.dynamicSmemBytes = 0;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = a->splits;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t e = cudaLaunchKernelEx(&cfg, fsl_decode_kernel<D>, *a);
    if (e != cudaSuccess) {
        fs_set_error("fsl_decode_step: launch failed: %s", cudaGetErrorString(e));
        return FSATTN_ELAUNCH;
    }
    return FSATTN_OK;
}

}  // namespace

extern "C" int fsattn_fsl_decode_step(const fsattn_fsl_decode_t* a, fsattn_stream_t stream) {
    FS_REQUIRE(a != nullptr, "fsl_decode_step: null args");
    const fsattn_fsl_state_t& st = a->st;
    FS_REQUIRE(a->q && a->k && a->v && a->pos && a->cos && a->sin && a->lam && a->sigma && a->lrs && a->norm_w && a->y,
               "fsl_decode_step: null pointer");
    FS_REQUIRE(st.B > 0 && st.H > 0 && st.cap_rows > 0 && st.cap_cells > 0, "fsl_decode_step: bad sizes");
    FS_UNSUPPORTED(st.D != 64 && st.D != 96 && st.D != 128, "fsl_decode_step: head_dim %d not in {64,96,128}", st.D);
    FS_REQUIRE(st.store_mode >= 0 && st.store_mode <= 2, "fsl_decode_step: store_mode %d", st.store_mode);
    FS_REQUIRE(st.P >= 1 && st.P <= FSATTN_MAX_POOL && st.Wc >= 0 && st.Wc <= 8, "fsl_decode_step: pool %d + %d unsupported", st.P, st.Wc);
    FS_REQUIRE(st.kk >= 1 && st.kk <= FSATTN_MAX_KK, "fsl_decode_step: kk %d", st.kk);
    FS_REQUIRE(st.Bq > 0 && st.Bq % FSATTN_CELL == 0, "fsl_decode_step: query block %d must be a multiple of the cell size", st.Bq);
    FS_REQUIRE(st.W >= 0, "fsl_decode_step: window %d", st.W);
    FS_REQUIRE(a->splits == 1 || a->splits == 2 || a->splits == 4 || a->splits == 8, "fsl_decode_step: splits %d not in {1,2,4,8}", a->splits);
    FS_REQUIRE(st.kbar && st.ceil && st.top_idx && st.top_blk && st.status, "fsl_decode_step: null state pointer");
    if (st.store_mode == 0) {
        FS_REQUIRE(st.kbuf && st.vbuf, "fsl_decode_step: bf16 store without buffers");
        FS_REQUIRE(((uintptr_t)st.kbuf & 15) == 0 && ((uintptr_t)st.vbuf & 15) == 0 && st.buf_sb % 8 == 0 && st.buf_sh % 8 == 0,
                   "fsl_decode_step: bf16 store must be 16-byte aligned");
    } else {
        FS_REQUIRE(st.kq && st.vq && st.ks && st.vs && st.khot && st.vhot, "fsl_decode_step: int8 store without buffers");
        FS_REQUIRE(((uintptr_t)st.kq & 15) == 0 && ((uintptr_t)st.vq & 15) == 0 && st.q_sb % 16 == 0 && st.q_sh % 16 == 0,
                   "fsl_decode_step: int8 store must be 16-byte aligned");
        FS_REQUIRE(((uintptr_t)st.khot & 15) == 0 && ((uintptr_t)st.vhot & 15) == 0 && st.hot_sb % 8 == 0 && st.hot_sh % 8 == 0,
                   "fsl_decode_step: hot rows must be 16-byte aligned");
    }
    if (st.store_mode == 2)
        FS_REQUIRE(st.slot_of && st.cell_in && st.n_slots > 0, "fsl_decode_step: bounded store without slot tables");
    FS_REQUIRE(((uintptr_t)a->q & 15) == 0 && ((uintptr_t)a->k & 15) == 0 && ((uintptr_t)a->v & 15) == 0 && a->in_sb % 8 == 0 && a->in_sh % 8 == 0,
               "fsl_decode_step: q/k/v must be 16-byte aligned");
    FS_REQUIRE(((uintptr_t)st.kbar & 15) == 0 && st.kbar_sb % 4 == 0 && st.kbar_sh % 4 == 0, "fsl_decode_step: kbar must be 16-byte aligned");
    FS_REQUIRE(((uintptr_t)a->cos & 15) == 0 && ((uintptr_t)a->sin & 15) == 0, "fsl_decode_step: rope tables must be 16-byte aligned");
    cudaStream_t s = (cudaStream_t)stream;
    switch (st.D) {
        case 64: return launch_decode<64>(a, s);
        case 96: return launch_decode<96>(a, s);
        default: return launch_decode<128>(a, s);
    }
}
