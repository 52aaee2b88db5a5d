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
template <int D>
struct RawRow {
    uint2 w[2 * RowL<D>::NW];  // int8 rows use only .x
};

template <int D, bool I8>
__device__ __forceinline__ void raw_load(RawRow<D>& r, const void* row, int sub, bool valid) {
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
__device__ __forceinline__ void raw_floats(const RawRow<D>& r, float sc, float* lo, float* hi) {
    using L = RowL<D>;
#pragma unroll
    for (int i = 0; i < L::NW; i++) {
        if (I8) {
            unpack4_i8(r.w[i].x, lo + 4 * i);
            unpack4_i8(r.w[L::NW + i].x, hi + 4 * i);
#pragma unroll
            for (int j = 0; j < 4; j += 2) {              // two values per bf16 rounding instruction
                const uint32_t a = pack_bf2(f_mul(lo[4 * i + j], sc), f_mul(lo[4 * i + j + 1], sc));
                const uint32_t b = pack_bf2(f_mul(hi[4 * i + j], sc), f_mul(hi[4 * i + j + 1], sc));
                lo[4 * i + j] = bf_lo(a); lo[4 * i + j + 1] = bf_hi(a);
                hi[4 * i + j] = bf_lo(b); hi[4 * i + j + 1] = bf_hi(b);
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

// A row in flight: its K and V words (and the rotary table words for window rows) are loaded first, consumed later, so a
// warp can keep several rows' loads outstanding.
template <int D>
struct RowFlight {
    RawRow<D> k, v;
    uint2 c[RowL<D>::NW], s[RowL<D>::NW];
    unsigned short ksc, vsc;        // the cell's scales as bf16 bits: converted where they are used, not where they are loaded (a
    bool valid, i8;                 // dependent instruction right after the load would hold up every later load: in-order issue)
};

template <int D, bool ROPE>
__device__ __forceinline__ void row_issue(RowFlight<D>& f, const void* krow, const void* vrow, const bf16* ksc_p, const bf16* vsc_p,
                                          bool valid, bool i8, const bf16* cosr, const bf16* sinr, int sub) {
    using L = RowL<D>;
    f.valid = valid; f.i8 = i8;
    f.ksc = 0x3f80; f.vsc = 0x3f80;             // 1.0 in bf16
    if (valid && i8) {
        f.ksc = *reinterpret_cast<const unsigned short*>(ksc_p);
        f.vsc = *reinterpret_cast<const unsigned short*>(vsc_p);
    }
    if (i8) { raw_load<D, true>(f.k, krow, sub, valid); raw_load<D, true>(f.v, vrow, sub, valid); }
    else { raw_load<D, false>(f.k, krow, sub, valid); raw_load<D, false>(f.v, vrow, sub, valid); }
    if (ROPE) {
#pragma unroll
        for (int i = 0; i < L::NW; i++) {
            f.c[i] = valid ? reinterpret_cast<const uint2*>(cosr + sub * L::DPL)[i] : make_uint2(0u, 0u);
            f.s[i] = valid ? reinterpret_cast<const uint2*>(sinr + sub * L::DPL)[i] : make_uint2(0u, 0u);
        }
    }
}

// score the row (4 lanes cooperate) and fold it into the group's partial; every lane of the warp must call it
template <int D, bool ROPE>
__device__ __forceinline__ void row_consume(Part<D>& P, const RowFlight<D>& f, const float* qlo, const float* qhi, float scale) {
    using L = RowL<D>;
    float klo[L::DPL], khi[L::DPL];
    if (f.i8) raw_floats<D, true>(f.k, __uint_as_float((uint32_t)f.ksc << 16), klo, khi); else raw_floats<D, false>(f.k, 1.0f, klo, khi);
    float dot = 0.0f;
    if (ROPE) {
        float c[L::DPL], s[L::DPL];
#pragma unroll
        for (int i = 0; i < L::NW; i++) { unpack4_bf(f.c[i], c + 4 * i); unpack4_bf(f.s[i], s + 4 * i); }
#pragma unroll
        for (int j = 0; j < L::DPL; j++) {
            const uint32_t rr = pack_bf2(klo[j] * c[j] - khi[j] * s[j], khi[j] * c[j] + klo[j] * s[j]);   // one rounding instruction
            dot = fmaf(qlo[j], bf_lo(rr), dot);
            dot = fmaf(qhi[j], bf_hi(rr), dot);
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
    if (!f.valid) return;   // uniform within the 4-lane group; no shuffles below
    const float sc = dot * scale;
    float vlo[L::DPL], vhi[L::DPL];
    if (f.i8) raw_floats<D, true>(f.v, __uint_as_float((uint32_t)f.vsc << 16), vlo, vhi); else raw_floats<D, false>(f.v, 1.0f, vlo, vhi);
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


#ifdef FSATTN_DEC_TIMING
// debug build only: clock64 phase stamps of CTA (rank 0 / rank 1) of head 0, read back with fsattn_debug_dec_timing
__device__ long long g_dec_stamps[2][16];
#define STAMP(r, i) do { if (bh == 0 && tid == 0 && rank == (r)) g_dec_stamps[(r)][(i)] = clock64(); } while (0)
#else
#define STAMP(r, i) do { } while (0)
#endif

constexpr int WIN_NF = 3;                      // 8-row groups of window rows a warp keeps in flight
constexpr int WIN_STAGES = 2;                  // staged window: tiles of WIN_TILE rows in flight per CTA
constexpr int WIN_TILE = 64;                   // rows per tile = one 8-row group for each of the 8 warps
constexpr int WIN_CELLS = 40;                  // cells a window may touch: W / 32 + 2 (W <= 1216)
constexpr int SC_ITERS = (MAXC + 31) / 32;     // scoring rounds: 32 candidates per round over the 8 warps
static_assert(MAXC <= 224, "the candidates are ranked by the first seven warps, one thread each");

template <int D>
struct Smem {
    float q_raw[D];
    float q_rot[D];
    float lc[FSATTN_MAX_POOL];
    int li[FSATTN_MAX_POOL];
    int ccell[MAXC];
    int cok[MAXC];
    int crow[MAXC];
    float score[MAXC];
    float prior[MAXC];
    int selcell[FSATTN_MAX_KK];
    int selrow[FSATTN_MAX_KK];
    int n_list;
    float wrec[NWARP][D + 2];   // per-warp partials (window, then long-range)
    float win_recs[8][D + 2];   // rank 0: window partials pushed by the window CTAs through distributed shared memory
    float lr_rec[D + 2];
    unsigned long long pool_bar;   // mbarrier of the pool's bulk copy
    int pool_timeout;
    // staged window (many sequences per step): per-cell scales and row bases of the window's cells, stage barriers
    unsigned short win_ks[WIN_CELLS], win_vs[WIN_CELLS];      // bf16 bits
    int win_base[WIN_CELLS];
    unsigned long long stage_bar[WIN_STAGES];
};

// ---- mbarrier + bulk (TMA) copy helpers; every wait is bounded ----------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }
__device__ __forceinline__ void mbar_init(unsigned long long* bar, int count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_expect_tx(unsigned long long* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, unsigned long long* bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                 ::"r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar)) : "memory");
}
// returns false when the phase did not complete within the iteration budget
__device__ __forceinline__ bool mbar_wait_bounded(unsigned long long* bar, uint32_t parity, int max_iters) {
    const uint32_t addr = smem_u32(bar);
    for (int i = 0; i < max_iters; i++) {
        uint32_t done;
        asm volatile("{\n.reg .pred p;\nmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\nselp.u32 %0, 1, 0, p;\n}"
                     : "=r"(done) : "r"(addr), "r"(parity) : "memory");
        if (done) return true;
    }
    return false;
}

// Pointers of one (b,h) into the layer state.
struct HeadPtrs {
    const int8_t* kq; const int8_t* vq; const bf16* ks; const bf16* vs;
    bf16* khot; bf16* vhot; bf16* kbuf; bf16* vbuf;
    int32_t* slot_of; int32_t* cell_in;
    float* kbar; float* ceil;
};

__device__ __forceinline__ HeadPtrs head_ptrs(const fsattn_fsl_state_t& st, int b, int h) {
    HeadPtrs p;
    p.kq = st.kq ? st.kq + b * st.q_sb + h * st.q_sh : nullptr;
    p.vq = st.vq ? st.vq + b * st.q_sb + h * st.q_sh : nullptr;
    p.ks = st.ks ? (const bf16*)st.ks + b * st.sc_sb + h * st.sc_sh : nullptr;
    p.vs = st.vs ? (const bf16*)st.vs + b * st.sc_sb + h * st.sc_sh : nullptr;
    p.khot = st.khot ? (bf16*)st.khot + b * st.hot_sb + h * st.hot_sh : nullptr;
    p.vhot = st.vhot ? (bf16*)st.vhot + b * st.hot_sb + h * st.hot_sh : nullptr;
    p.kbuf = st.kbuf ? (bf16*)st.kbuf + b * st.buf_sb + h * st.buf_sh : nullptr;
    p.vbuf = st.vbuf ? (bf16*)st.vbuf + b * st.buf_sb + h * st.buf_sh : nullptr;
    p.slot_of = st.slot_of ? st.slot_of + b * st.so_sb + h * st.so_sh : nullptr;
    p.cell_in = st.cell_in ? st.cell_in + b * st.ci_sb + h * st.ci_sh : nullptr;
    p.kbar = st.kbar + b * st.kbar_sb + h * st.kbar_sh;
    p.ceil = st.ceil + b * st.ceil_sb + h * st.ceil_sh;
    return p;
}

// ---- window branch: rows [max(0,pos-W), pos) from the store + the new token's row -------------------------------------
// The stored rows depend only on the position and this layer's own state, so a warp issues the loads of its first two
// 8-row groups BEFORE the producer kernel (the QKV projection) has finished; only the arithmetic needs q.
template <int D>
struct WinCtx {
    int64_t pos, nq, lo_row, g_lo, g_hi;
    int nw, gw, mode;
    bool pos_ok;
};

template <int D>
__device__ __forceinline__ void window_issue2(RowFlight<D>* f, const WinCtx<D>& w, const fsattn_fsl_decode_t& a, const HeadPtrs& hp,
                                              int64_t g0, int lane) {
    const int sub = lane & 3, grp = lane >> 2;
    const fsattn_fsl_state_t& st = a.st;
    const bf16* cosT = (const bf16*)a.cos;
    const bf16* sinT = (const bf16*)a.sin;
    int64_t r[WIN_NF]; bool valid[WIN_NF], i8[WIN_NF]; int slot[WIN_NF];
#pragma unroll
    for (int u = 0; u < WIN_NF; u++) {
        const int64_t g = g0 + (int64_t)u * w.nw;
        r[u] = (g << 3) + grp;
        // the new token's row (r == pos) is handled separately: its key and value come from the producer kernel
        valid[u] = w.pos_ok && g <= w.g_hi && r[u] >= w.lo_row && r[u] < w.pos;
        i8[u] = valid[u] && w.mode != 0 && r[u] < w.nq;
        slot[u] = 0;
        if (i8[u] && w.mode == 2) slot[u] = hp.slot_of[r[u] / FSATTN_CELL];
    }
#pragma unroll
    for (int u = 0; u < WIN_NF; u++) {
        const void* kp = nullptr; const void* vp = nullptr;
        const bf16* ksp = nullptr; const bf16* vsp = nullptr;
        bool ok = valid[u];
        if (valid[u]) {
            if (w.mode == 0) { kp = hp.kbuf + r[u] * D; vp = hp.vbuf + r[u] * D; }
            else if (!i8[u]) { kp = hp.khot + (r[u] - w.nq) * D; vp = hp.vhot + (r[u] - w.nq) * D; }
            else {
                int64_t cell = r[u] / FSATTN_CELL;
                int64_t prow = r[u];
                if (w.mode == 2) {
                    if (slot[u] < 0) { ok = false; if (sub == 0) atomicAdd(st.status + FSATTN_ST_POOL_NO_SLOT, 1); }
                    prow = (int64_t)slot[u] * FSATTN_CELL + (r[u] - cell * FSATTN_CELL);
                    cell = slot[u];
                }
                if (ok) { kp = hp.kq + prow * D; vp = hp.vq + prow * D; ksp = hp.ks + cell; vsp = hp.vs + cell; }
            }
        }
        row_issue<D, true>(f[u], kp, vp, ksp, vsp, ok, i8[u] && ok, cosT + r[u] * D, sinT + r[u] * D, sub);
    }
}

// consumes the pre-issued groups, walks the remaining groups of this warp, adds the new token's row (warp gw == 0), and
// leaves the CTA's merged partial in `out_rec` (m, l, acc[D])
template <int D>
__device__ __forceinline__ void window_finish(Smem<D>& sm, RowFlight<D>* f, const WinCtx<D>& w, const fsattn_fsl_decode_t& a,
                                              const HeadPtrs& hp, const bf16* k_in, const bf16* v_in, float* out_rec, int warp, int lane) {
    using L = RowL<D>;
    const int sub = lane & 3, grp = lane >> 2;
    const bf16* cosT = (const bf16*)a.cos;
    const bf16* sinT = (const bf16*)a.sin;
    float qlo[L::DPL], qhi[L::DPL];
#pragma unroll
    for (int j = 0; j < L::DPL; j++) { qlo[j] = sm.q_rot[sub * L::DPL + j]; qhi[j] = sm.q_rot[L::HALF + sub * L::DPL + j]; }
    Part<D> P;
    P.init();
    int64_t g0 = w.g_lo + w.gw;
    for (;;) {
#pragma unroll
        for (int u = 0; u < WIN_NF; u++) row_consume<D, true>(P, f[u], qlo, qhi, a.scale);
        g0 += WIN_NF * (int64_t)w.nw;
        if (g0 > w.g_hi) break;                 // warp-uniform
        window_issue2<D>(f, w, a, hp, g0, lane);
    }
    if (w.gw == 0) {                            // the new token itself: always inside its own window
        RowFlight<D> c;
        const bool mine = w.pos_ok && grp == 0;
        row_issue<D, true>(c, k_in, v_in, nullptr, nullptr, mine, false, cosT + w.pos * D, sinT + w.pos * D, sub);
        row_consume<D, true>(P, c, qlo, qhi, a.scale);
    }
    part_merge_warp<D>(P);
    part_store<D>(P, sm.wrec[warp], lane);
    __syncthreads();
    if (warp == 0) {
        float l, acc[D / 32];
        rec_merge<D>(&sm.wrec[0][0], NWARP, D + 2, lane, l, acc);
        float m = -INFINITY;
        for (int i = 0; i < NWARP; i++) m = fmaxf(m, sm.wrec[i][0]);
        if (lane == 0) { out_rec[0] = m; out_rec[1] = l; }
#pragma unroll
        for (int j = 0; j < D / 32; j++) out_rec[2 + lane + 32 * j] = acc[j];
    }
}

// ---- window branch with the K/V rows staged through shared memory by bulk copies (one CTA per (b,h), int8 stores) ----------
// With many sequences per step the kernel is bandwidth-bound and per-lane 4-byte loads cannot keep enough bytes in flight.
// Here thread 0 streams the window in tiles of 64 rows: the int8 rows of K and V (contiguous in the full store, one piece per
// cell in the slot store) and the rows of the rotary tables, by cp.async.bulk onto an mbarrier, two tiles in flight; the
// warps consume a tile from shared memory with the same per-row arithmetic, the same row-to-warp assignment and the same
// merge order as the direct path, so the result is bit-identical to it. Rows of the open cell (bf16, at most 31) and the
// new token's row are read directly. Stage s holds: K rows [0, 64 D), V rows, cos rows (bf16), sin rows (bf16).
template <int D>
struct WinStage {
    static constexpr int K_OFF = 0, V_OFF = WIN_TILE * D, C_OFF = 2 * WIN_TILE * D, S_OFF = C_OFF + WIN_TILE * D * 2;
    static constexpr int BYTES = S_OFF + WIN_TILE * D * 2;
};

// issue the copies of tile i (rows r0 .. r0+63) into stage buffer `buf`; thread 0 only
template <int D>
__device__ __forceinline__ void stage_issue(Smem<D>& sm, unsigned char* buf, unsigned long long* bar, const WinCtx<D>& w,
                                            const fsattn_fsl_decode_t& a, const HeadPtrs& hp, int64_t r0, int c0) {
    using WS = WinStage<D>;
    int64_t q_end = r0 + WIN_TILE;                       // int8 rows of this tile: [r0, q_end)
    if (q_end > w.nq) q_end = w.nq;
    int64_t t_end = r0 + WIN_TILE;                       // table rows: up to the new token's own position
    if (t_end > w.pos + 1) t_end = w.pos + 1;
    uint32_t bytes = 0;
    if (q_end > r0) bytes += (uint32_t)(q_end - r0) * D * 2;
    if (t_end > r0) bytes += (uint32_t)(t_end - r0) * D * 4;
    mbar_expect_tx(bar, bytes);
    for (int64_t r = r0; r < q_end;) {                   // one piece per cell: rows [r, e)
        const int64_t cell = r / FSATTN_CELL;
        int64_t e = (cell + 1) * FSATTN_CELL;
        if (e > q_end) e = q_end;
        const int bs = sm.win_base[cell - c0];            // a cell without a slot: any valid rows, masked when consumed
        const int64_t src_row = (int64_t)(bs < 0 ? 0 : bs) * FSATTN_CELL + (r - cell * FSATTN_CELL);
        const uint32_t nb = (uint32_t)(e - r) * D;
        bulk_g2s(buf + WS::K_OFF + (r - r0) * D, hp.kq + src_row * D, nb, bar);
        bulk_g2s(buf + WS::V_OFF + (r - r0) * D, hp.vq + src_row * D, nb, bar);
        r = e;
    }
    if (t_end > r0) {
        const uint32_t nb = (uint32_t)(t_end - r0) * D * 2;
        bulk_g2s(buf + WS::C_OFF, (const bf16*)a.cos + r0 * D, nb, bar);
        bulk_g2s(buf + WS::S_OFF, (const bf16*)a.sin + r0 * D, nb, bar);
    }
}

// before the dependency wait: the window's per-cell scales and row bases into shared memory, barriers, first tiles in flight
template <int D>
__device__ __forceinline__ void staged_prologue(Smem<D>& sm, unsigned char* stages, const WinCtx<D>& w, const fsattn_fsl_decode_t& a,
                                                const HeadPtrs& hp, int tid) {
    const fsattn_fsl_state_t& st = a.st;
    const int c0 = (int)(w.lo_row / FSATTN_CELL);
    const int ncq = (int)(w.nq / FSATTN_CELL);          // completed cells: [0, ncq)
    if (tid < WIN_CELLS) {
        const int cell = c0 + tid;
        unsigned short ks = 0x3f80, vs = 0x3f80;         // 1.0 in bf16
        int base = 0;
        if (w.pos_ok && cell < ncq) {
            base = cell;
            if (w.mode == 2) {
                base = hp.slot_of[cell];
                if (base < 0) { atomicAdd(st.status + FSATTN_ST_POOL_NO_SLOT, 1); base = -1; }
            }
            if (base >= 0) {
                ks = *reinterpret_cast<const unsigned short*>(hp.ks + base);
                vs = *reinterpret_cast<const unsigned short*>(hp.vs + base);
            }
        }
        sm.win_ks[tid] = ks; sm.win_vs[tid] = vs; sm.win_base[tid] = base;
    }
    if (tid == 0) {
        for (int s = 0; s < WIN_STAGES; s++) mbar_init(&sm.stage_bar[s], 1);
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    __syncthreads();
    if (tid == 0 && w.pos_ok) {
        const int64_t R0 = w.g_lo << 3;
        const int ntiles = (int)((w.g_hi - w.g_lo) / NWARP) + 1;
        for (int i = 0; i < WIN_STAGES && i < ntiles; i++) {
            // a cell without a slot (counted above) leaves its rows out: they are masked when consumed
            stage_issue<D>(sm, stages + (size_t)i * WinStage<D>::BYTES, &sm.stage_bar[i], w, a, hp, R0 + (int64_t)i * WIN_TILE, c0);
        }
    }
}

template <int D>
__device__ __forceinline__ void window_finish_staged(Smem<D>& sm, unsigned char* stages, const WinCtx<D>& w, const fsattn_fsl_decode_t& a,
                                                     const HeadPtrs& hp, const bf16* k_in, const bf16* v_in, float* out_rec, int warp,
                                                     int lane, int tid) {
    using L = RowL<D>;
    using WS = WinStage<D>;
    const fsattn_fsl_state_t& st = a.st;
    const int sub = lane & 3, grp = lane >> 2;
    const bf16* cosT = (const bf16*)a.cos;
    const bf16* sinT = (const bf16*)a.sin;
    float qlo[L::DPL], qhi[L::DPL];
#pragma unroll
    for (int j = 0; j < L::DPL; j++) { qlo[j] = sm.q_rot[sub * L::DPL + j]; qhi[j] = sm.q_rot[L::HALF + sub * L::DPL + j]; }
    Part<D> P;
    P.init();
    const int c0 = (int)(w.lo_row / FSATTN_CELL);
    const int64_t R0 = w.g_lo << 3;
    const int ntiles = w.pos_ok ? (int)((w.g_hi - w.g_lo) / NWARP) + 1 : 0;
    for (int i = 0; i < ntiles; i++) {
        const int s = i % WIN_STAGES;
        unsigned char* buf = stages + (size_t)s * WS::BYTES;
        bool arrived = mbar_wait_bounded(&sm.stage_bar[s], (uint32_t)(i / WIN_STAGES) & 1u, 1 << 22);
        if (!arrived && lane == 0) atomicAdd(st.status + FSATTN_ST_BAD_INDEX, 1);
        const int64_t r0 = R0 + (int64_t)i * WIN_TILE;
        const int64_t g = w.g_lo + (int64_t)i * NWARP + warp;
        const int64_t r = (g << 3) + grp;
        bool valid = arrived && g <= w.g_hi && r >= w.lo_row && r < w.pos;
        const bool q8 = r < w.nq;                          // warp-uniform: a group never straddles the open cell's start
        RowFlight<D> f;
        if (q8) {
            const int ci = (int)(r / FSATTN_CELL) - c0;
            const int cidx = (ci >= 0 && ci < WIN_CELLS) ? ci : 0;
            valid = valid && ci >= 0 && ci < WIN_CELLS && sm.win_base[cidx] >= 0;
            f.valid = valid; f.i8 = valid;
            f.ksc = sm.win_ks[cidx]; f.vsc = sm.win_vs[cidx];
            raw_load<D, true>(f.k, buf + WS::K_OFF + (r - r0) * D, sub, valid);
            raw_load<D, true>(f.v, buf + WS::V_OFF + (r - r0) * D, sub, valid);
        } else {
            const void* kp = valid ? (const void*)(hp.khot + (r - w.nq) * D) : nullptr;
            const void* vp = valid ? (const void*)(hp.vhot + (r - w.nq) * D) : nullptr;
            f.valid = valid; f.i8 = false; f.ksc = 0x3f80; f.vsc = 0x3f80;
            raw_load<D, false>(f.k, kp, sub, valid);
            raw_load<D, false>(f.v, vp, sub, valid);
        }
        {
            const bf16* cr = reinterpret_cast<const bf16*>(buf + WS::C_OFF) + (r - r0) * D;
            const bf16* sr = reinterpret_cast<const bf16*>(buf + WS::S_OFF) + (r - r0) * D;
#pragma unroll
            for (int u = 0; u < L::NW; u++) {
                f.c[u] = valid ? reinterpret_cast<const uint2*>(cr + sub * L::DPL)[u] : make_uint2(0u, 0u);
                f.s[u] = valid ? reinterpret_cast<const uint2*>(sr + sub * L::DPL)[u] : make_uint2(0u, 0u);
            }
        }
        row_consume<D, true>(P, f, qlo, qhi, a.scale);
        __syncthreads();                                   // every warp is done with this stage's buffer
        if (tid == 0 && i + WIN_STAGES < ntiles)
            stage_issue<D>(sm, buf, &sm.stage_bar[s], w, a, hp, R0 + (int64_t)(i + WIN_STAGES) * WIN_TILE, c0);
    }
    if (w.gw == 0) {                            // the new token itself: always inside its own window
        RowFlight<D> c;
        const bool mine = w.pos_ok && grp == 0;
        row_issue<D, true>(c, k_in, v_in, nullptr, nullptr, mine, false, cosT + w.pos * D, sinT + w.pos * D, sub);
        row_consume<D, true>(P, c, qlo, qhi, a.scale);
    }
    part_merge_warp<D>(P);
    part_store<D>(P, sm.wrec[warp], lane);
    __syncthreads();
    if (warp == 0) {
        float l, acc[D / 32];
        rec_merge<D>(&sm.wrec[0][0], NWARP, D + 2, lane, l, acc);
        float m = -INFINITY;
        for (int i = 0; i < NWARP; i++) m = fmaxf(m, sm.wrec[i][0]);
        if (lane == 0) { out_rec[0] = m; out_rec[1] = l; }
#pragma unroll
        for (int j = 0; j < D / 32; j++) out_rec[2 + lane + 32 * j] = acc[j];
    }
}

// ---- append the new row; close the cell when this token completes it (one warp) ---------------------------------------
template <int D>
__device__ __forceinline__ void append_and_close(const fsattn_fsl_state_t& st, const HeadPtrs& hp, int64_t pos,
                                                 const bf16* k_in, const bf16* v_in, int lane) {
    const int mode = st.store_mode;
    const int64_t nq = (pos / FSATTN_CELL) * FSATTN_CELL;
    const int hr = (int)(pos - nq);
    if (mode == 0) {
        for (int d = lane; d < D; d += 32) { hp.kbuf[pos * D + d] = k_in[d]; hp.vbuf[pos * D + d] = v_in[d]; }
    } else {
        for (int d = lane; d < D; d += 32) { hp.khot[hr * D + d] = k_in[d]; hp.vhot[hr * D + d] = v_in[d]; }
    }
    if (hr != FSATTN_CELL - 1) return;
    const int cell = (int)(pos / FSATTN_CELL);
    const bool in_table = cell < st.cap_cells;
    int dst = cell;          // where the quantised rows and the mean key go (cell or slot index)
    bool store_ok = in_table;
    if (mode == 2) {
        int slot = -1;
        for (int s0 = 0; s0 < st.n_slots && slot < 0; s0 += 32) {
            const int si = s0 + lane;
            const bool free_ = si < st.n_slots && hp.cell_in[si] < 0;
            const unsigned bal = __ballot_sync(FS_FULL, free_);
            if (bal) slot = s0 + __ffs(bal) - 1;
        }
        store_ok = in_table && slot >= 0;
        dst = slot;
        if (!store_ok && lane == 0) atomicAdd(st.status + FSATTN_ST_SLOT_OVERFLOW, 1);
        if (store_ok && lane == 0) { hp.slot_of[cell] = slot; hp.cell_in[slot] = cell; }
    }
    const bf16* kcell = (mode == 0) ? hp.kbuf + nq * D : hp.khot;
    const bf16* vcell = (mode == 0) ? hp.vbuf + nq * D : hp.vhot;
    CellRegs<D> cr;
    cell_load_rows<D>(cr, kcell, D, lane, k_in);
    // the ceiling table is indexed by cell; the mean keys by cell (full stores) or slot (bounded store)
    cell_stats_warp<D>(cr, lane, store_ok ? hp.kbar + (int64_t)dst * D : nullptr, in_table ? hp.ceil + cell : nullptr);
    if (mode != 0 && store_ok) {
        cell_quant_warp<D>(cr, lane, const_cast<int8_t*>(hp.kq) + (int64_t)dst * FSATTN_CELL * D, const_cast<bf16*>(hp.ks) + dst);
        cell_load_rows<D>(cr, vcell, D, lane, v_in);
        cell_quant_warp<D>(cr, lane, const_cast<int8_t*>(hp.vq) + (int64_t)dst * FSATTN_CELL * D, const_cast<bf16*>(hp.vs) + dst);
    }
}

// ---- block change: refresh the top-P list, free unreadable slots, gather the block's candidate pool (whole CTA) -----------
template <int D>
__device__ __forceinline__ void refresh_pool(Smem<D>& sm, const fsattn_fsl_state_t& st, const HeadPtrs& hp, int bh, int blk_start,
                                             int tid, float* pool_s, int4* meta_s) {
    const int warp = tid >> 5, lane = tid & 31;
    const int mode = st.store_mode;
    const int M_vis = blk_start / FSATTN_CELL;
    const int C = st.P + st.Wc;
    int32_t* top_idx = st.top_idx + (int64_t)bh * st.P;
    if (warp == 0) {
        int n = 0;
        for (int p = lane; p < st.P; p += 32) {
            const int ci = top_idx[p];
            sm.li[p] = ci;
            sm.lc[p] = (ci >= 0) ? hp.ceil[ci] : 0.0f;
            n += (ci >= 0);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) n += __shfl_xor_sync(FS_FULL, n, o);
        __syncwarp();
        const int have_blk = st.top_blk[bh];
        if (have_blk != blk_start) {
            int c0 = have_blk / FSATTN_CELL; if (c0 < 0) c0 = 0;
            for (int c = c0; c < M_vis; c++) pool_list_insert(sm.lc, sm.li, n, st.P, hp.ceil[c], c, lane);
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
                        const int occ = hp.cell_in[si];
                        if (occ >= 0 && occ < c_lo) {
                            bool in_top = false;
                            for (int p = 0; p < n; p++) in_top |= (sm.li[p] == occ);
                            if (!in_top) { hp.cell_in[si] = -1; hp.slot_of[occ] = -1; }
                        }
                    }
                }
            }
        }
        if (lane == 0) sm.n_list = n;
    }
    __syncthreads();
    // candidate slots: the top-P list, then the Wc newest visible cells
    const int n_list = sm.n_list;
    for (int t = tid; t < C; t += blockDim.x) {
        const int cand = (t < st.P) ? ((t < n_list) ? sm.li[t] : -1) : (M_vis - 1) - (t - st.P);
        const int cc = cand < 0 ? 0 : cand;
        sm.ccell[t] = cc;
        sm.cok[t] = (cand >= 0) && (cc < M_vis);
    }
    __syncthreads();
    int32_t* meta = st.pool_meta + (int64_t)bh * C * 4;
    for (int t = tid; t < C; t += blockDim.x) {
        int ok = sm.cok[t];
        const int cc = sm.ccell[t];
        for (int j = 0; j < t && ok; j++) ok = (sm.ccell[j] != cc);     // a slot that repeats an earlier slot's cell is out
        int row = cc;
        if (ok && mode == 2) {
            row = hp.slot_of[cc];
            if (row < 0) { atomicAdd(st.status + FSATTN_ST_POOL_NO_SLOT, 1); ok = 0; row = 0; }
        }
        sm.crow[t] = ok ? row : -1;
        const float ce = ok ? hp.ceil[cc] : 0.0f;
        const int4 mv = make_int4(ok ? cc : -1, row, __float_as_int(ce), 0);
        reinterpret_cast<int4*>(meta)[t] = mv;
        meta_s[t] = mv;                          // this step scores from the shared-memory copy
    }
    __syncthreads();
    float* pk = st.pool_kbar + (int64_t)bh * C * D;
    constexpr int V4 = D / 4;
    for (int i = tid; i < C * V4; i += blockDim.x) {
        const int t = i / V4, e = i - t * V4;
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if (sm.crow[t] >= 0) v = reinterpret_cast<const float4*>(hp.kbar + (int64_t)sm.crow[t] * D)[e];
        reinterpret_cast<float4*>(pk + (size_t)t * D)[e] = v;
        reinterpret_cast<float4*>(pool_s + (size_t)t * D)[e] = v;
    }
    if (tid == 0) st.pool_blk[bh] = blk_start;
    __threadfence();
    __syncthreads();
}

// MINB: CTAs the compiler must fit per SM. 1 = all the registers it wants (the batch-1 shape: fewer CTAs than SMs, latency
// is everything); 2 = at most 128 registers, so that two CTAs overlap each other's memory round trips once the grid is
// larger than the machine (many sequences per step: the kernel is then bandwidth-bound and needs the occupancy).
// STAGED: the window rows go through shared memory by bulk copies (one CTA per (b,h), int8 stores; see window_finish_staged).
template <int D, int MINB, bool STAGED>
__global__ void __launch_bounds__(NWARP * 32, MINB) fsl_decode_kernel(const fsattn_fsl_decode_t a) {
    using L = RowL<D>;
    constexpr int F = D / 8;                  // floats per lane when 8 lanes share a mean key
    __shared__ Smem<D> sm;
    extern __shared__ __align__(128) unsigned char dyn_smem[];     // rank 0: the block's candidate pool (mean keys, meta)
    cg::cluster_group cluster = cg::this_cluster();
    const int S = (int)gridDim.x;             // CTAs per (b,h) = cluster size
    const int rank = (int)blockIdx.x;
    const int bh = blockIdx.y;
    const fsattn_fsl_state_t& st = a.st;
    const int b = bh / st.H, h = bh - b * st.H;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int sub = lane & 3, grp = lane >> 2, s8 = lane & 7;
    const int mode = st.store_mode;
    const int C = st.P + st.Wc;
    float* pool_s = reinterpret_cast<float*>(dyn_smem);
    int4* meta_s = reinterpret_cast<int4*>(dyn_smem + (size_t)C * D * 4);
    unsigned char* stages = dyn_smem + (((size_t)C * ((size_t)D * 4 + 16) + 127) & ~(size_t)127);   // STAGED only
    STAMP(0, 0); STAMP(1, 0);

    // "every CTA of the cluster has started": arrive now, wait right before the first distributed-shared-memory access
    if (S > 1) cluster.barrier_arrive();

    const bf16* q_in = (const bf16*)a.q + b * a.in_sb + h * a.in_sh;
    const bf16* k_in = (const bf16*)a.k + b * a.in_sb + h * a.in_sh;
    const bf16* v_in = (const bf16*)a.v + b * a.in_sb + h * a.in_sh;
    const bf16* cosT = (const bf16*)a.cos;
    const bf16* sinT = (const bf16*)a.sin;
    const HeadPtrs hp = head_ptrs(st, b, h);

    // =========== before the producer kernel has finished: everything that depends only on the position and on this
    // layer's own state (last written by this layer's kernel of the previous step, long complete) =====================
    const int64_t pos = *a.pos;
    const bool pos_ok = pos >= 0 && pos < st.cap_rows;
    const int blk_start = (int)((pos / st.Bq) * st.Bq);
    int pool_blk = 0;
    const bool ext = a.ext_sel != nullptr;      // selections come from another kernel (FS-B): no pool, no scoring here
    if (rank == 0 && !ext) {
        if (tid == 0) {
            sm.pool_timeout = 0;
            mbar_init(&sm.pool_bar, 1);
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            const uint32_t kb_bytes = (uint32_t)C * D * 4, mt_bytes = (uint32_t)C * 16;
            mbar_expect_tx(&sm.pool_bar, kb_bytes + mt_bytes);
            bulk_g2s(pool_s, st.pool_kbar + (int64_t)bh * C * D, kb_bytes, &sm.pool_bar);
            bulk_g2s(meta_s, st.pool_meta + (int64_t)bh * C * 4, mt_bytes, &sm.pool_bar);
        }
        pool_blk = st.pool_blk[bh];
        __syncthreads();          // the barrier is initialised before any thread polls it (rank is CTA-uniform)
    }
    // per-head parameters (warp 0 of rank 0 also needs the norm weights of its output dims)
    const float lam = a.lam[h];
    const float two_sigma = f_mul(2.0f, a.sigma[h]);
    const float g_lrs = a.lrs[h];
    float nw_reg[D / 32];
#pragma unroll
    for (int j = 0; j < D / 32; j++) nw_reg[j] = a.norm_w[lane + 32 * j];
    float rc = 0.f, rs = 0.f;
    if (tid < L::HALF && pos_ok) { rc = __bfloat162float(cosT[pos * D + tid]); rs = __bfloat162float(sinT[pos * D + tid]); }
    WinCtx<D> w;
    w.pos = pos; w.pos_ok = pos_ok; w.mode = mode;
    w.nq = (pos / FSATTN_CELL) * FSATTN_CELL;
    w.lo_row = (pos - st.W > 0) ? pos - st.W : 0;
    w.g_lo = w.lo_row >> 3; w.g_hi = pos >> 3;
    w.nw = (S == 1) ? NWARP : (S - 1) * NWARP;
    w.gw = (S == 1) ? warp : (rank - 1) * NWARP + warp;
    const bool do_window = (S == 1) || (rank > 0);
    RowFlight<D> wf[WIN_NF];
    if (STAGED) staged_prologue<D>(sm, stages, w, a, hp, tid);
    else if (do_window) window_issue2<D>(wf, w, a, hp, w.g_lo + w.gw, lane);
    if (rank == 0 && !ext) {
        // the pool's bulk copy; the wait is bounded. The position priors of the candidates need no query: compute them now.
        if (!mbar_wait_bounded(&sm.pool_bar, 0, 1 << 22)) {
            if (lane == 0) { atomicAdd(st.status + FSATTN_ST_BAD_INDEX, 1); sm.pool_timeout = 1; }
        }
        if (pool_blk == blk_start) {
            for (int t = tid; t < C; t += blockDim.x) {
                const int4 mt = meta_s[t];
                sm.prior[t] = (mt.x >= 0) ? fs_prior(lam, __int_as_float(mt.z), (float)pos, mt.x, (float)FSATTN_CELL, two_sigma) : 0.0f;
            }
        }
    }

    // =========== the producer (QKV projection) is complete from here on =====================================================
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    STAMP(0, 1); STAMP(1, 1);

    // q: raw and rotated (rounded to bf16 like the reference's rotated query), into shared memory
    if (tid < L::HALF) {
        const float x1 = __bfloat162float(q_in[tid]), x2 = __bfloat162float(q_in[tid + L::HALF]);
        sm.q_raw[tid] = x1; sm.q_raw[tid + L::HALF] = x2;
        sm.q_rot[tid] = bf_round(x1 * rc - x2 * rs);
        sm.q_rot[tid + L::HALF] = bf_round(x2 * rc + x1 * rs);
    }
    if (tid == 0 && !pos_ok) atomicAdd(st.status + FSATTN_ST_BAD_INDEX, 1);
    __syncthreads();
    STAMP(0, 2); STAMP(1, 2);

    // ================= window branch =====================================================================================
    if (do_window) {
        float* out_rec = sm.win_recs[0];
        if (S > 1) {
            cluster.barrier_wait();                                   // rank 0 is running: its shared memory may be written
            out_rec = cluster.map_shared_rank(&sm.win_recs[rank][0], 0);
        }
        if (STAGED) window_finish_staged<D>(sm, stages, w, a, hp, k_in, v_in, out_rec, warp, lane, tid);
        else window_finish<D>(sm, wf, w, a, hp, k_in, v_in, out_rec, warp, lane);
    }
    STAMP(1, 3);

    // ================= long-range branch + bookkeeping (rank 0) ==============================================================
    float lr_l = 0.0f;
    if (rank == 0) {
        if (!ext && pool_blk != blk_start) {       // CTA-uniform, once per Bq tokens
            refresh_pool<D>(sm, st, hp, bh, blk_start, tid, pool_s, meta_s);
            for (int t = tid; t < C; t += blockDim.x) {
                const int4 mt = meta_s[t];
                sm.prior[t] = (mt.x >= 0) ? fs_prior(lam, __int_as_float(mt.z), (float)pos, mt.x, (float)FSATTN_CELL, two_sigma) : 0.0f;
            }
            __syncthreads();
        }
        STAMP(0, 3);
        if (ext) {
            // the selected cells were chosen by the FS-B selection kernel that ran before this one; full stores only
            if (tid < st.kk) {
                const int cell = a.ext_sel[(int64_t)bh * st.kk + tid];
                const bool okc = cell >= 0 && (int64_t)(cell + 1) * FSATTN_CELL <= pos;
                sm.selcell[tid] = okc ? cell : -1;
                sm.selrow[tid] = okc ? cell : -1;
                if (a.sel_out != nullptr) a.sel_out[(int64_t)bh * st.kk + tid] = okc ? cell : -1;
            }
        } else
        // ---- scores: 8 lanes per candidate, mean keys from shared memory ---------------------------------------------------
        {
            if (tid < FSATTN_MAX_KK) {             // slots no candidate ranks into stay empty
                sm.selcell[tid] = -1; sm.selrow[tid] = -1;
                if (a.sel_out != nullptr && tid < st.kk) a.sel_out[(int64_t)bh * st.kk + tid] = -1;
            }
            float qv[F];
#pragma unroll
            for (int j = 0; j < F; j++) qv[j] = sm.q_raw[s8 * F + j];
            // (the last warp appends the new row instead, below)
            for (int t0 = warp * 4; t0 < C && warp < NWARP - 1; t0 += (NWARP - 1) * 4) {
                const int t = t0 + (lane >> 3);
                int4 mt = make_int4(-1, 0, 0, 0);
                if (t < C) mt = meta_s[t];
                const bool ok = mt.x >= 0;
                float dot = 0.0f;
                if (ok) {
                    const float4* kr = reinterpret_cast<const float4*>(pool_s + (size_t)t * D + s8 * F);
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
                    if (ok) sc = f_add(f_mul(dot, a.scale), sm.prior[t]);
                    sm.score[t] = sc;
                    sm.ccell[t] = mt.x;
                    sm.crow[t] = mt.y;
                }
            }
        }
        // ---- the new row joins the store (and closes its cell) in the last warp, which takes no part in scoring and ranking and
        // skips their barrier: nothing in this step reads the row, so it stays off the path from the query to the output -------------
        if (warp == NWARP - 1) {
            if (pos_ok) append_and_close<D>(st, hp, pos, k_in, v_in, lane);
        } else {
            asm volatile("bar.sync 1, %0;" ::"n"((NWARP - 1) * 32) : "memory");        // the scores of warps 0 .. NWARP-2 are complete
        }
        STAMP(0, 4);

        // ---- top-kk by (score desc, slot asc): every candidate counts the candidates ahead of it (the scores are broadcast
        // reads of shared memory); the kk with the fewest are the selection, in rank order -------------------------------------------
        if (!ext && tid < C) {
            const float sc = sm.score[tid];
            int ahead = 0;
#pragma unroll 8
            for (int u = 0; u < C; u++) {
                const float su = sm.score[u];
                ahead += (su > sc || (su == sc && u < tid)) ? 1 : 0;
            }
            if (ahead < st.kk) {
                const int cell = sm.ccell[tid];
                sm.selcell[ahead] = cell;
                sm.selrow[ahead] = (cell >= 0) ? sm.crow[tid] : -1;
                if (a.sel_out != nullptr) a.sel_out[(int64_t)bh * st.kk + ahead] = cell;
            }
        }
        __syncthreads();
        STAMP(0, 5);

        // ---- readout of the selected cells: 4 groups of 8 rows per cell, spread over the warps, all loads in flight at once -----------
        {
            float qlo[L::DPL], qhi[L::DPL];
#pragma unroll
            for (int j = 0; j < L::DPL; j++) { qlo[j] = sm.q_raw[sub * L::DPL + j]; qhi[j] = sm.q_raw[L::HALF + sub * L::DPL + j]; }
            Part<D> P;
            P.init();
            const int ngroups = st.kk * 4;
            for (int g0 = warp; g0 < ngroups; g0 += 2 * NWARP) {       // warp-uniform; kk = 4: one pass, two groups per warp
                RowFlight<D> f[2];
#pragma unroll
                for (int u = 0; u < 2; u++) {
                    const int gi = g0 + u * NWARP;
                    const int k = (gi >> 2) & (FSATTN_MAX_KK - 1);
                    const int cell = (gi < ngroups) ? sm.selcell[k] : -1;
                    const int rr = ((gi & 3) << 3) + grp;
                    const int64_t tok = (int64_t)cell * FSATTN_CELL + rr;
                    const bool valid = pos_ok && cell >= 0 && tok < pos;
                    const void* kp = nullptr; const void* vp = nullptr; const bf16* ksp = nullptr; const bf16* vsp = nullptr;
                    if (valid) {
                        if (mode == 0) { kp = hp.kbuf + tok * D; vp = hp.vbuf + tok * D; }
                        else {
                            const int64_t base = sm.selrow[k];
                            kp = hp.kq + (base * FSATTN_CELL + rr) * D; vp = hp.vq + (base * FSATTN_CELL + rr) * D;
                            ksp = hp.ks + base; vsp = hp.vs + base;
                        }
                    }
                    row_issue<D, false>(f[u], kp, vp, ksp, vsp, valid, valid && mode != 0, nullptr, nullptr, sub);
                }
#pragma unroll
                for (int u = 0; u < 2; u++) row_consume<D, false>(P, f[u], qlo, qhi, a.scale);
            }
            STAMP(0, 10);
            part_merge_warp<D>(P);
            part_store<D>(P, sm.wrec[warp], lane);
        }
        __syncthreads();
        STAMP(0, 11);
        if (warp == 0) {
            float acc[D / 32];
            rec_merge<D>(&sm.wrec[0][0], NWARP, D + 2, lane, lr_l, acc);
#pragma unroll
            for (int j = 0; j < D / 32; j++) sm.lr_rec[2 + lane + 32 * j] = acc[j];
        }
        if (S > 1) cluster.barrier_wait();        // completes the "everyone started" phase before the final barrier
    }

    // ================= exchange + combine ============================================================================================
    STAMP(0, 6);
    if (S > 1) cluster.sync(); else __syncthreads();     // the window partials are in rank 0's shared memory
    STAMP(0, 7); STAMP(1, 4);
    if (rank == 0 && warp == 0) {
        const int first = (S == 1) ? 0 : 1;
        float wl, wacc[D / 32];
        rec_merge<D>(&sm.win_recs[first][0], (S == 1) ? 1 : S - 1, D + 2, lane, wl, wacc);
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
        bf16* yp = (bf16*)a.y + (int64_t)b * st.H * D + (int64_t)h * D;
#pragma unroll
        for (int j = 0; j < D / 32; j++) {
            const int d = lane + 32 * j;
            const float sr = bf_round(wacc[j] * winv);
            const float lr = f_mul(f_mul(o[j], rn), nw_reg[j]);
            yp[d] = __float2bfloat16_rn(f_add(sr, f_mul(g_lrs, lr)));
        }
    }
    STAMP(0, 8);
}

template <int D, int MINB, bool STAGED>
int launch_decode_v(const fsattn_fsl_decode_t* a, cudaStream_t stream) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(a->splits, a->st.B * a->st.H, 1);
    cfg.blockDim = dim3(NWARP * 32, 1, 1);
    size_t dyn = (size_t)(a->st.P + a->st.Wc) * ((size_t)D * 4 + 16);
    if (STAGED) dyn = ((dyn + 127) & ~(size_t)127) + (size_t)WIN_STAGES * WinStage<D>::BYTES;
    static size_t opted[16] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dyn > 24 * 1024 && dev >= 0 && dev < 16 && opted[dev] < dyn) {
        if (cudaFuncSetAttribute(fsl_decode_kernel<D, MINB, STAGED>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)dyn) != cudaSuccess) {
            (void)cudaGetLastError();
            fs_set_error("fsl_decode_step: cannot opt in to %zu bytes of shared memory", dyn);
            return FSATTN_ELAUNCH;
        }
        opted[dev] = dyn;
    }
    cfg.dynamicSmemBytes = dyn;
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = a->splits;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = a->pdl ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    cudaError_t e = cudaLaunchKernelEx(&cfg, fsl_decode_kernel<D, MINB, STAGED>, *a);
    if (e != cudaSuccess) {
        (void)cudaGetLastError();       // the error is reported through the return code; do not leave it pending
        fs_set_error("fsl_decode_step: launch failed: %s", cudaGetErrorString(e));
        return FSATTN_ELAUNCH;
    }
    return FSATTN_OK;
}

template <int D>
int launch_decode(const fsattn_fsl_decode_t* a, cudaStream_t stream) {
    static int sms = 0;
    if (sms == 0) {
        int dev = 0;
        cudaGetDevice(&dev);
        if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms <= 0) sms = 148;
    }
    const long ctas = (long)a->splits * a->st.B * a->st.H;
    // Many sequences per step: one CTA per (b,h) with the window rows staged through shared memory (int8 stores).
    const bool can_stage = a->splits == 1 && a->st.store_mode != 0 && a->st.W / FSATTN_CELL + 2 <= WIN_CELLS;
    const bool stage = a->window_path == 2 || (a->window_path == 0 && can_stage && ctas > sms);
    if (stage) return launch_decode_v<D, 2, true>(a, stream);
    return ctas > sms ? launch_decode_v<D, 2, false>(a, stream) : launch_decode_v<D, 1, false>(a, stream);
}

}  // namespace

#ifdef FSATTN_DEC_TIMING
extern "C" __attribute__((visibility("default"))) int fsattn_debug_dec_timing(long long* out32) {
    return cudaMemcpyFromSymbol(out32, g_dec_stamps, sizeof(long long) * 32) == cudaSuccess ? 0 : -1;
}
#endif

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
    FS_REQUIRE(st.kbar && st.ceil && st.top_idx && st.top_blk && st.status && st.pool_kbar && st.pool_meta && st.pool_blk, "fsl_decode_step: null state pointer");
    FS_REQUIRE(((uintptr_t)st.pool_kbar & 15) == 0 && ((uintptr_t)st.pool_meta & 15) == 0, "fsl_decode_step: pool buffers must be 16-byte aligned");
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
    FS_REQUIRE(a->window_path >= 0 && a->window_path <= 2, "fsl_decode_step: window_path %d not in {0,1,2}", a->window_path);
    FS_UNSUPPORTED(a->window_path == 2 && (a->splits != 1 || st.store_mode == 0 || st.W / FSATTN_CELL + 2 > WIN_CELLS),
                   "fsl_decode_step: the staged window needs splits = 1, an int8 store and a window of at most %d tokens",
                   (WIN_CELLS - 2) * FSATTN_CELL);
    FS_UNSUPPORTED(a->ext_sel != nullptr && st.store_mode == 2,
                   "fsl_decode_step: external (FS-B) selections need a full KV store, not the bounded slot store");
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
