// FS-B selection: spines, the two beams, union of candidates, token-level re-rank, top-K.
//
// One warp per query. A beam keeps its frontier (<= 16 node refs) in lanes 0..15; each level the 32 lanes score the
// 32 possible children (lane c = child c&1 of frontier slot c>>1), rank them with shuffles and rebuild the frontier:
// carried nodes first in slot order, then children by (score desc, position asc). Node tables are read straight from
// the L2-resident arena (one 2D-byte mean row + one 16-byte aux word per child); the spine nodes of the block live in
// shared memory. The re-rank reads the candidate cells' raw token keys, one token per lane.
#include "fsb.cuh"

namespace {

#ifdef FSATTN_FSB_TIMING
// debug build only: clock64 stamps of the decode selection of row 0 (warp 0 lane 0), read back with fsattn_debug_fsb_timing
__device__ long long g_fsb_stamps[64];
#define FSTAMP(i) do { if (blockIdx.x == 0 && threadIdx.x == 0) g_fsb_stamps[(i)] = clock64(); } while (0)
#else
#define FSTAMP(i) do { } while (0)
#endif

constexpr int SPW = FSATTN_FSB_SPINE_MAX;      // spine slots per forest
constexpr int WMAX = 16;                       // frontier slots

// Node refs: -1 none; <= -2 the spine node of height -(ref+2); >= 0 a chunk node: arena node id in bits 0..19 and the
// height k of its chunk in bits 20..23 (the chunk a descendant belongs to never changes on the way down).
#define REF_ID(r) ((r) & 0xfffff)
#define REF_K(r) ((r) >> 20)

template <int D>
struct SpineSm {
    float node[SPW][D + 8];     // [mu | rad amax pmin cnt chl chr pad pad]
    int root, height, m_b, pad;
    // shallow levels staged in shared memory (prefill): for the chunk of height k, its first stg_cnt[k] nodes (level
    // order, so a prefix of its node array) sit at rows stg_base[k] .. of the staging area
    int stg_base[16], stg_cnt[16];
    int stg_rows;
};

// ---- spine of the first m_b admitted cells of row t (one warp) ------------------------------------------------------
template <int D>
__device__ void build_spine(const fsattn_fsb_forest_t& F, int t, int m_b, SpineSm<D>& S, int lane) {
    constexpr int NPL = FsbDim<D>::NPL;
    const int m_cap = F.m_cap;
    const float4* aux = (const float4*)F.node_aux + (int64_t)t * fsb_nodes_per_row(m_cap, F.compact);
    const float* root32 = F.root32 + (int64_t)t * fsb_root_rows(m_cap, F.compact) * (D + FSB_ROOT_PAD);
    float rmu[NPL];
    float r_rad = 0.f, r_am = 0.f, r_cnt = 0.f;
    int r_pm = 0x7fffffff, r_ref = -1, npres = 0;
#pragma unroll
    for (int i = 0; i < NPL; ++i) rmu[i] = 0.f;
    for (int k = 0; (m_b >> k) != 0; ++k) {
        if (!((m_b >> k) & 1)) continue;
        ++npres;
        const int j = (m_b >> (k + 1)) << 1;
        const int cid = (int)fsb_root_node(k, j, m_cap, F.compact);
        const int cref = cid | (k << 20);
        const float* cr = root32 + (int64_t)fsb_chunk_id(k, j, m_cap, F.compact) * (D + FSB_ROOT_PAD);
        float cmu[NPL];
        fsb_load_row<D>(cr, lane, cmu);
        const float c_rad = cr[D];
        const float4 ca = aux[cid];
        const float c_am = ca.y, c_cnt = (float)(1 << k);
        const int c_pm = __float_as_int(ca.z);
        if (r_ref == -1) {
#pragma unroll
            for (int i = 0; i < NPL; ++i) rmu[i] = cmu[i];
            r_rad = c_rad; r_am = c_am; r_cnt = c_cnt; r_pm = c_pm; r_ref = cref;
            continue;
        }
        const float tot = f_add(c_cnt, r_cnt);
        float nmu[NPL], dc[NPL], dr[NPL];
#pragma unroll
        for (int i = 0; i < NPL; ++i) {
            nmu[i] = f_div(f_add(f_mul(c_cnt, cmu[i]), f_mul(r_cnt, rmu[i])), tot);
            const float a = f_add(cmu[i], -nmu[i]), b = f_add(rmu[i], -nmu[i]);
            dc[i] = f_mul(a, a);
            dr[i] = f_mul(b, b);
        }
        const float nc = f_sqrt(fsb_warp_det_sum<D>(dc)), nr = f_sqrt(fsb_warp_det_sum<D>(dr));
        const float n_rad = fmaxf(f_add(c_rad, nc), f_add(r_rad, nr));
        const float n_am = fmaxf(c_am, r_am);
        const int n_pm = min(c_pm, r_pm);
        fsb_store_row<D>(S.node[k], lane, nmu);
        if (lane == 0) {
            float* x = S.node[k] + D;
            x[0] = n_rad; x[1] = n_am; x[2] = __int_as_float(n_pm); x[3] = tot;
            x[4] = __int_as_float(cref); x[5] = __int_as_float(r_ref);
        }
#pragma unroll
        for (int i = 0; i < NPL; ++i) rmu[i] = nmu[i];
        r_rad = n_rad; r_am = n_am; r_cnt = tot; r_pm = n_pm; r_ref = -(k + 2);
    }
    if (lane == 0) {
        S.root = (m_b > 0) ? r_ref : -1;
        S.height = (m_b > 1) ? (31 - __clz(m_b)) + (npres >= 2 ? 1 : 0) : 0;
        S.m_b = m_b;
    }
}

// Which chunk nodes lie at tree depth <= DS: the chunks hang off the spine chain, the i-th present bit from the top has
// its root at depth i+1 (the lowest one shares the depth of the one above it; a single chunk is the root itself), and a
// chunk whose root is at depth d contributes its levels 0 .. DS-d, i.e. its first 2^(DS-d+1)-1 nodes. At most 2^(DS+1)-1
// rows in total. One thread.
template <int D>
__host__ __device__ constexpr int STG_SW() { return D == 96 ? 3 : 7; }      // 16-byte-chunk XOR mask of a staged row
template <int D>
__host__ __device__ constexpr int STG_DS() { return 7; }                    // deepest staged tree level
template <int D>
__host__ __device__ constexpr int STG_ROWS() { return (2 << STG_DS<D>()); }

template <int D>
__device__ void stage_plan(SpineSm<D>& S, int m_b, int DS) {
    for (int k = 0; k < 16; ++k) { S.stg_base[k] = 0; S.stg_cnt[k] = 0; }
    const int p = __popc(m_b);
    int i = 0, base = 0;
    for (int k = 31 - __clz(m_b | 1); k >= 0 && m_b > 0; --k) {
        if (!((m_b >> k) & 1)) continue;
        const int dep = (p == 1) ? 0 : ((i < p - 1) ? i + 1 : p - 1);
        int cnt = (dep <= DS) ? ((1 << (DS - dep + 1)) - 1) : 0;
        cnt = min(cnt, (2 << k) - 1);
        S.stg_base[k] = base;
        S.stg_cnt[k] = cnt;
        base += cnt;
        ++i;
    }
    S.stg_rows = base;
}

__device__ __forceinline__ int count_below(const int* adm, int m_tot, int E) {
    int lo = 0, hi = m_tot;                       // first index with adm[i] >= E
    while (lo < hi) {
        const int mid = (lo + hi) >> 1;
        if (adm[mid] < E) lo = mid + 1; else hi = mid;
    }
    return lo;
}

// ---- the query-independent head of a beam ------------------------------------------------------------------------------------
// While a round's children all fit in the frontier (carried + 2 x expanding <= W) every child is kept whatever its score, so
// the SET of frontier nodes after those rounds is the same for every query of the block: 1, 2, 4, 8, 16 nodes down the spine
// and the top of the chunks. One warp walks those rounds once per (row, block) without scoring anything and records the
// nodes with the round that created each; a query's beam then starts there, scoring the recorded nodes once to put them
// in the order the skipped rounds would have left them in (older rounds first, a round's nodes by score), instead of
// running three or four full rounds.
struct BeamPre {
    int ref[WMAX], meta[WMAX], nc[WMAX], rnd[WMAX];
    int n, nvis, rounds, pad;
};

template <int D>
__device__ void beam_prefix(const fsattn_fsb_forest_t& F, int t, const SpineSm<D>& S, int width, int lane, BeamPre& P) {
    const float4* aux = (const float4*)F.node_aux + (int64_t)t * fsb_nodes_per_row(F.m_cap, F.compact);
    const int root = S.root;
    int ref = -1, meta = 0, nc = 0, rnd = 0;
    int n = 0, nvis = 0, rounds = 0;
    if (root != -1) {
        const int d0 = S.height;
        const int W = min(width, (d0 >= 5) ? 32 : (1 << d0));
        if (lane == 0) {
            ref = root;
            meta = (root >= 0) ? __float_as_int(aux[REF_ID(root)].w) : 0;
        }
        n = 1;
        for (int it = 0; it < 6; ++it) {
            const bool active = lane < WMAX && ref != -1;
            const bool expand = active && (ref < -1 || meta < 0);
            const unsigned emask = __ballot_sync(FS_FULL, expand);
            const unsigned cmask = __ballot_sync(FS_FULL, active && !expand);
            const int nexp = __popc(emask), ncar = __popc(cmask);
            if (nexp == 0 || ncar + 2 * nexp > W) break;
            const int ps = lane >> 1, side = lane & 1;
            const int pref = __shfl_sync(FS_FULL, ref, ps), pmeta = __shfl_sync(FS_FULL, meta, ps);
            const bool valid = (emask >> ps) & 1;
            int cref = -1, cmeta = 0, cnc = 0;
            if (valid) {
                if (pref >= 0) {
                    const int np = (~pmeta) >> 4;
                    cnc = 2 * np + 1 + side;
                    cref = pref + np + 1 + side;
                } else {
                    const float* x = S.node[-pref - 2] + D;
                    cref = __float_as_int(x[4 + side]);
                }
                if (cref >= 0) cmeta = __float_as_int(aux[REF_ID(cref)].w);
            }
            const unsigned vmask = __ballot_sync(FS_FULL, valid);
            const unsigned lt = (1u << lane) - 1u;
            __syncwarp();
            if (active && !expand) {
                const int pos = __popc(cmask & lt);
                P.ref[pos] = ref; P.meta[pos] = meta; P.nc[pos] = nc; P.rnd[pos] = rnd;
            }
            if (valid) {
                const int pos = ncar + __popc(vmask & lt);
                P.ref[pos] = cref; P.meta[pos] = cmeta; P.nc[pos] = cnc; P.rnd[pos] = rounds + 1;
            }
            __syncwarp();
            n = ncar + __popc(vmask);
            nvis += __popc(vmask);
            ++rounds;
            ref = -1; meta = 0; nc = 0; rnd = 0;
            if (lane < n) { ref = P.ref[lane]; meta = P.meta[lane]; nc = P.nc[lane]; rnd = P.rnd[lane]; }
        }
    }
    __syncwarp();
    if (lane < WMAX) { P.ref[lane] = ref; P.meta[lane] = meta; P.nc[lane] = nc; P.rnd[lane] = rnd; }
    if (lane == 0) { P.n = n; P.nvis = nvis; P.rounds = rounds; }
    __syncwarp();
}

// ---- one beam (one warp). Returns the frontier's cell in lanes 0..15 (-1 none); adds the scored children to nvis ----
template <int D, bool PREFETCH = false, bool STAGED = false>
__device__ int beam(const fsattn_fsb_forest_t& F, int t, const SpineSm<D>& S, const BeamPre& P, const uint32_t (&qp)[D / 2], float qn,
                    float qpos, float lam, float sig, float scale, int width, int lane, int* fr, int& nvis,
                    const unsigned char* stg_mu = nullptr, const float4* stg_aux = nullptr, const float* qf = nullptr) {
    constexpr int DP = FsbDim<D>::DP;
    const int m_cap = F.m_cap;
    const int64_t nrow = (int64_t)t * fsb_nodes_per_row(m_cap, F.compact);
    const bf16* node_mu = (const bf16*)F.node_mu + nrow * D;
    const float4* aux = (const float4*)F.node_aux + nrow;
    if (S.root == -1) return -1;
    const float inv_two_sig = f_div(1.0f, f_mul(2.0f, sig));
    const int d0 = S.height;                                  // delta = 0: stop depth = height, budget 1
    const int W = min(width, (d0 >= 5) ? 32 : (1 << d0));

    // score of one node for this query: a chunk node (ref >= 0; nc = its index inside its chunk) or a spine node
    auto node_score = [&](int cref, int nc, int& cmeta) -> float {
        float rad, am;
        int pm;
        // q . mu with four running sums (plain FMAs: the beam's cut-offs are compared under a score margin, and a
        // different summation order moves a score by ~1e-6)
        float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
        if (cref >= 0) {
            uint4 w[D / 8];
            float4 ax;
            const int ck = REF_K(cref);
            if (STAGED && nc < S.stg_cnt[ck]) {
                const int row = S.stg_base[ck] + nc;
                const unsigned char* mr = stg_mu + (size_t)row * (D * 2);
#pragma unroll
                for (int v = 0; v < D / 8; ++v) w[v] = *(const uint4*)(mr + (((v & ~STG_SW<D>()) | ((v ^ row) & STG_SW<D>())) << 4));
                ax = stg_aux[row];
            } else {
                const uint4* mr = (const uint4*)(node_mu + (int64_t)REF_ID(cref) * D);
#pragma unroll
                for (int v = 0; v < D / 8; ++v) w[v] = mr[v];
                ax = aux[REF_ID(cref)];
            }
            if constexpr (STAGED) {
                // prefill: the query as fp32 from shared memory (two broadcast 16-byte reads per eight dims), which keeps 32
                // registers free and lets a third CTA share the SM; same products, same four running sums
#pragma unroll
                for (int v = 0; v < D / 8; ++v) {
                    const float4 qa = reinterpret_cast<const float4*>(qf)[2 * v], qb = reinterpret_cast<const float4*>(qf)[2 * v + 1];
                    s0 = fmaf(qa.x, bf_lo(w[v].x), s0); s1 = fmaf(qa.y, bf_hi(w[v].x), s1);
                    s2 = fmaf(qa.z, bf_lo(w[v].y), s2); s3 = fmaf(qa.w, bf_hi(w[v].y), s3);
                    s0 = fmaf(qb.x, bf_lo(w[v].z), s0); s1 = fmaf(qb.y, bf_hi(w[v].z), s1);
                    s2 = fmaf(qb.z, bf_lo(w[v].w), s2); s3 = fmaf(qb.w, bf_hi(w[v].w), s3);
                }
            } else {
                // decode (latency-bound): the query sits in registers as bf16 pairs, no shared-memory traffic for it
#pragma unroll
                for (int v = 0; v < D / 8; ++v) {
                    s0 = fmaf(bf_lo(qp[v * 4 + 0]), bf_lo(w[v].x), s0); s1 = fmaf(bf_hi(qp[v * 4 + 0]), bf_hi(w[v].x), s1);
                    s2 = fmaf(bf_lo(qp[v * 4 + 1]), bf_lo(w[v].y), s2); s3 = fmaf(bf_hi(qp[v * 4 + 1]), bf_hi(w[v].y), s3);
                    s0 = fmaf(bf_lo(qp[v * 4 + 2]), bf_lo(w[v].z), s0); s1 = fmaf(bf_hi(qp[v * 4 + 2]), bf_hi(w[v].z), s1);
                    s2 = fmaf(bf_lo(qp[v * 4 + 3]), bf_lo(w[v].w), s2); s3 = fmaf(bf_hi(qp[v * 4 + 3]), bf_hi(w[v].w), s3);
                }
            }
            rad = ax.x; am = ax.y; pm = __float_as_int(ax.z); cmeta = __float_as_int(ax.w);
        } else {
            const float* x = S.node[-cref - 2];
            if constexpr (STAGED) {
#pragma unroll
                for (int d = 0; d < D; d += 4) {
                    s0 = fmaf(qf[d], x[d], s0); s1 = fmaf(qf[d + 1], x[d + 1], s1);
                    s2 = fmaf(qf[d + 2], x[d + 2], s2); s3 = fmaf(qf[d + 3], x[d + 3], s3);
                }
            } else {
#pragma unroll
                for (int d = 0; d < D; d += 4) {
                    s0 = fmaf(bf_lo(qp[d / 2]), x[d], s0); s1 = fmaf(bf_hi(qp[d / 2]), x[d + 1], s1);
                    s2 = fmaf(bf_lo(qp[d / 2 + 1]), x[d + 2], s2); s3 = fmaf(bf_hi(qp[d / 2 + 1]), x[d + 3], s3);
                }
            }
            rad = x[D]; am = x[D + 1]; pm = __float_as_int(x[D + 2]);
            cmeta = 0;
        }
        float content = f_mul((s0 + s1) + (s2 + s3), scale);
        content = f_add(content, f_mul(f_mul(qn, rad), scale));
        const float ppos = f_mul(f_add((float)pm, 0.5f), 32.0f);
        // erf(x) is 1 in fp32 from x = 4 on, which with a sigma of a few tokens is every node further than a cell or two
        // from the query: the evaluation is skipped there (by the whole warp when all its children are that far); the
        // quotient is a product with 1/(2 sigma), one rounding from the reference's division, far inside the margin
        const float x = f_mul(fabsf(f_add(qpos, -ppos)), inv_two_sig);
        const float e = (x < 4.0f) ? erff(x) : 1.0f;
        return f_add(content, f_mul(f_mul(lam, am), e));
    };

    // ---- start from the block's query-independent head, put into this query's order ----
    int ref = -1, meta = 0;
    if (lane < P.n) { ref = P.ref[lane]; meta = P.meta[lane]; }
    if (P.rounds > 0) {
        float sc = FS_NEG_SCORE;
        int rn = 1 << 20;
        if (lane < P.n) {
            int cm;
            rn = P.rnd[lane];
            sc = node_score(ref, P.nc[lane], cm);
        }
        int rank = 0;
#pragma unroll
        for (int o = 0; o < WMAX; ++o) {
            const float so = __shfl_sync(FS_FULL, sc, o);
            const int ro = __shfl_sync(FS_FULL, rn, o);
            rank += (ro < rn || (ro == rn && (so > sc || (so == sc && o < lane)))) ? 1 : 0;
        }
        int* fm = fr + WMAX;
        __syncwarp();
        if (lane < P.n) { fr[rank] = ref; fm[rank] = meta; }
        __syncwarp();
        if (lane < P.n) { ref = fr[lane]; meta = fm[lane]; }
        __syncwarp();
        nvis += P.nvis;
    }
    for (int it = 0; it < 40; ++it) {
        if constexpr (!STAGED) { if (it < 20) FSTAMP(16 + it); }
        const bool active = lane < WMAX && ref != -1;
        const bool expand = active && (ref < -1 || meta < 0);
        const unsigned emask = __ballot_sync(FS_FULL, expand);
        if (emask == 0) break;
        const unsigned cmask = __ballot_sync(FS_FULL, active && !expand);
        // ---- children ----
        const int ps = lane >> 1, side = lane & 1;
        const int pref = __shfl_sync(FS_FULL, ref, ps), pmeta = __shfl_sync(FS_FULL, meta, ps);
        const bool valid = (emask >> ps) & 1;
        int cref = -1, cmeta = 0;
        float score = FS_NEG_SCORE;
        if (valid) {
            int nc = 0;                                     // index of the child inside its chunk
            if (pref >= 0) {
                const int np = (~pmeta) >> 4;
                nc = 2 * np + 1 + side;
                cref = pref + np + 1 + side;                // same chunk: the height bits carry over
                if (PREFETCH && ((~pmeta) & 15) >= 2) {
                    // the two children of this child sit side by side: ask L2 for them now, one level ahead of their use
                    const int gc = REF_ID(cref) + nc + 1;
                    const char* g = (const char*)(node_mu + (int64_t)gc * D);
#pragma unroll
                    for (int o = 0; o < 2 * D * 2; o += 128) asm volatile("prefetch.global.L2 [%0];" ::"l"(g + o));
                    asm volatile("prefetch.global.L2 [%0];" ::"l"(aux + gc));
                }
            } else {
                const float* x = S.node[-pref - 2] + D;
                cref = __float_as_int(x[4 + side]);         // a chunk root (index 0 of its chunk) or a spine node
            }
            score = node_score(cref, nc, cmeta);
        }
        nvis += __popc(__ballot_sync(FS_FULL, valid));
        if constexpr (!STAGED) { if (it < 4 && __float_as_int(score) != 0x7fc00001) FSTAMP(36 + 2 * it); }
        // ---- rank the children: (score desc, position asc) ----
        // (32 independent shuffles pipeline well; a warp-wide max per kept child is a chain of dependent reductions and
        // measured slower in the latency-bound decode kernel and no faster in prefill)
        int rank = 0;
        if constexpr (STAGED) {
            // prefill (issue-bound): strictly better children, then the equal ones in lower lanes - one match instead of a
            // tie test per step
            rank = __popc(__match_any_sync(FS_FULL, __float_as_uint(score + 0.0f)) & ((1u << lane) - 1u));
#pragma unroll 8
            for (int o = 0; o < 32; ++o) rank += (__shfl_sync(FS_FULL, score, o) > score) ? 1 : 0;
        } else {
            // decode (latency-bound): the match sits on the critical path and measured 3 % slower there
#pragma unroll 8
            for (int o = 0; o < 32; ++o) {
                const float so = __shfl_sync(FS_FULL, score, o);
                rank += (so > score || (so == score && o < lane)) ? 1 : 0;
            }
        }
        if constexpr (!STAGED) { if (it < 4 && rank >= 0) FSTAMP(37 + 2 * it); }
        const int ncar = __popc(cmask & 0xffffu);
        int* fm = fr + WMAX;                   // fr: WMAX refs then WMAX metas
        if (lane < WMAX) fr[lane] = -1;
        __syncwarp();
        if (active && !expand) {
            const int pos = __popc(cmask & ((1u << lane) - 1));
            fr[pos] = ref; fm[pos] = meta;
        }
        if (valid && score > 0.5f * FS_NEG_SCORE && ncar + rank < W) {
            fr[ncar + rank] = cref; fm[ncar + rank] = cmeta;
        }
        __syncwarp();
        if (lane < WMAX) { ref = fr[lane]; meta = fm[lane]; }
        __syncwarp();
    }
    return (lane < WMAX && ref >= 0 && meta >= 0) ? meta : -1;
}

// ---- re-rank score of one candidate cell (one warp, lane = token of the cell) -----------------------------------------
// The token keys of one candidate cell as a lane holds them (lane = token), fetched apart from the arithmetic so that a warp
// with several cells to score can have all their rows in flight at once.
template <int D>
struct RrRow {
    uint4 w[D / 8];          // bf16 store: the row; int8 store: its codes in w[0 .. D/16)
    float sc, ceil_c;
};

template <int D>
__device__ __forceinline__ void rr_load(RrRow<D>& r, const fsattn_fsb_select_t& a, int b, int hd, int t, int cell, int lane) {
    const int64_t tok = (int64_t)cell * 32 + lane;
    if (a.k.ptr) {
        const uint4* kr = (const uint4*)((const bf16*)a.k.ptr + b * a.k.sb + hd * a.k.sh + tok * a.k.sn);
#pragma unroll
        for (int v = 0; v < D / 8; ++v) r.w[v] = kr[v];
        r.sc = 1.0f;
    } else {
        const uint4* kr = (const uint4*)(a.kq + b * a.kq_sb + hd * a.kq_sh + tok * D);      // the row's codes, 16 bytes per load
#pragma unroll
        for (int v4 = 0; v4 < D / 16; ++v4) r.w[v4] = kr[v4];
        r.sc = __bfloat162float(((const bf16*)a.ks)[b * a.ks_sb + hd * a.ks_sh + cell]);
    }
    r.ceil_c = a.main.ceil[(int64_t)t * a.main.ceil_st + cell];
}

template <int D>
__device__ __forceinline__ float rr_score(const RrRow<D>& r, const fsattn_fsb_select_t& a, int cell, const float* qs, float qpos,
                                          float lam, float sig) {
    constexpr int DP = FsbDim<D>::DP;
    float p[DP];
    if (a.k.ptr) {
#pragma unroll
        for (int v = 0; v < D / 8; ++v) {
            const uint4 w = r.w[v];
            const float4 qa = *(const float4*)(qs + v * 8), qb = *(const float4*)(qs + v * 8 + 4);
            p[v * 8 + 0] = f_mul(bf_lo(w.x), qa.x); p[v * 8 + 1] = f_mul(bf_hi(w.x), qa.y);
            p[v * 8 + 2] = f_mul(bf_lo(w.y), qa.z); p[v * 8 + 3] = f_mul(bf_hi(w.y), qa.w);
            p[v * 8 + 4] = f_mul(bf_lo(w.z), qb.x); p[v * 8 + 5] = f_mul(bf_hi(w.z), qb.y);
            p[v * 8 + 6] = f_mul(bf_lo(w.w), qb.z); p[v * 8 + 7] = f_mul(bf_hi(w.w), qb.w);
        }
    } else {
        const float sc = r.sc;
#pragma unroll
        for (int v4 = 0; v4 < D / 16; ++v4) {
            const uint4 w4 = r.w[v4];
            const uint32_t ws[4] = {w4.x, w4.y, w4.z, w4.w};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int v = v4 * 4 + j;
                float o[4];
                unpack4_i8(ws[j], o);
#pragma unroll
                for (int e = 0; e < 4; ++e) p[v * 4 + e] = f_mul(bf_round(f_mul(o[e], sc)), qs[v * 4 + e]);
            }
        }
    }
#pragma unroll
    for (int d = D; d < DP; ++d) p[d] = 0.f;
    const float sc = f_mul(fsb_thread_det_sum<D>(p), a.scale);
    const float m = warp_max(sc);
    float e = expf(f_add(sc, -m));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) e = f_add(e, __shfl_xor_sync(FS_FULL, e, o));
    const float lse = f_add(m, logf(e));
    const float cpos = f_mul(f_add((float)cell, 0.5f), 32.0f);
    const float er = erff(f_div(fabsf(f_add(qpos, -cpos)), f_mul(2.0f, sig)));
    return f_add(lse, f_mul(f_mul(lam, r.ceil_c), er));
}

template <int D>
__device__ __forceinline__ float rerank_cell(const fsattn_fsb_select_t& a, int b, int hd, int t, int cell, const float* qs,
                                             float qpos, float lam, float sig, int lane) {
    RrRow<D> r;
    rr_load<D>(r, a, b, hd, t, cell, lane);
    return rr_score<D>(r, a, cell, qs, qpos, lam, sig);
}

struct SelArgs {
    fsattn_fsb_select_t a;
    int H, ncell_k;
};

#include "fsb_beam_block.cuh"

// ---- prefill: one CTA per (128-query block, row) ---------------------------------------------------------------------------
// Per forest: build the block's spine, copy every chunk node of tree depth <= DS into shared memory (<= 2^(DS+1)-1 rows:
// the levels all 128 queries walk through), then one warp per query runs the beam, reading the shallow levels from
// shared memory and only the deep ones from L2. The candidates of both beams meet in shared memory for the union.
#ifndef FSB_SEL_NW
#define FSB_SEL_NW 8
#endif
constexpr int SEL_NW = FSB_SEL_NW;          // warps per prefill selection CTA

template <int D>
struct SelSmem {
    static constexpr size_t MU_OFF = 0;
    static constexpr size_t AUX_OFF = MU_OFF + (size_t)STG_ROWS<D>() * D * 2;
    static constexpr size_t TOTAL = AUX_OFF + (size_t)STG_ROWS<D>() * 16;
};

template <int D, int NWARP>
__global__ void __launch_bounds__(NWARP * 32, (D == 64) ? 3 : 2) fsb_select_kernel(SelArgs A) {
    constexpr int DP = FsbDim<D>::DP;
    constexpr int CH = D / 8;
    const fsattn_fsb_select_t& a = A.a;
    const int blk = blockIdx.x, t = blockIdx.y;
    const int b = t / A.H, hd = t % A.H;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    extern __shared__ __align__(16) unsigned char dsm[];
    unsigned char* stg_mu = dsm + SelSmem<D>::MU_OFF;
    float4* stg_aux = (float4*)(dsm + SelSmem<D>::AUX_OFF);
    __shared__ SpineSm<D> sp;
    __shared__ BeamPre pre;
    __shared__ __align__(16) float qsm[NWARP][DP];
    __shared__ int frs[NWARP][WMAX * 2];
    __shared__ int cand_sm[128][2 * WMAX];
    __shared__ int nv_sm[128];

    const float lam = a.lam[hd], sig = a.sigma[hd];
    const int Wc = a.width + a.width2;
    const int nq = min(a.Bq, a.N - blk * a.Bq);
    const int E = (a.q_pos0 + blk * a.Bq) / 32;
    for (int i = tid; i < 128 * 2 * WMAX; i += NWARP * 32) (&cand_sm[0][0])[i] = -1;
    for (int i = tid; i < 128; i += NWARP * 32) nv_sm[i] = 0;
    const int nbeam = a.width2 > 0 ? 2 : 1;
    for (int f = 0; f < nbeam; ++f) {
        const fsattn_fsb_forest_t& F = f == 0 ? a.main : a.second;
        __syncthreads();
        if (warp == 0) {
            const int m_b = count_below(F.adm + (int64_t)t * F.m_cap, F.m_tot[t], E);
            build_spine<D>(F, t, m_b, sp, lane);
            if (lane == 0) stage_plan<D>(sp, m_b, STG_DS<D>());
            __syncwarp();
            beam_prefix<D>(F, t, sp, f == 0 ? a.width : a.width2, lane, pre);
        }
        __syncthreads();
        {   // stage the shallow levels: rows of chunk k come from its node array's first stg_cnt[k] rows
            const int64_t nrow = (int64_t)t * fsb_nodes_per_row(F.m_cap, F.compact);
            const bf16* node_mu = (const bf16*)F.node_mu + nrow * D;
            const float4* aux = (const float4*)F.node_aux + nrow;
            const int m_b = sp.m_b;
            for (int k = 0; (m_b >> k) != 0; ++k) {
                const int cnt = sp.stg_cnt[k];
                if (!((m_b >> k) & 1) || cnt == 0) continue;
                const int base = sp.stg_base[k];
                const int64_t n0 = fsb_root_node(k, (m_b >> (k + 1)) << 1, F.m_cap, F.compact);
                for (int i = tid; i < cnt * CH; i += NWARP * 32) {
                    const int r = i / CH, v = i % CH, row = base + r;
                    const uint4 w = *(const uint4*)(node_mu + (n0 + r) * D + v * 8);
                    *(uint4*)(stg_mu + (size_t)row * (D * 2) + (((v & ~STG_SW<D>()) | ((v ^ row) & STG_SW<D>())) << 4)) = w;
                }
                for (int i = tid; i < cnt; i += NWARP * 32) stg_aux[base + i] = aux[n0 + i];
            }
        }
        __syncthreads();
        const int width = f == 0 ? a.width : a.width2;
        for (int qi = warp; qi < nq; qi += NWARP) {
            const int qidx = blk * a.Bq + qi;
            const float qpos = (float)(a.q_pos0 + qidx);
            const bf16* qp = (const bf16*)a.q.ptr + b * a.q.sb + hd * a.q.sh + (int64_t)qidx * a.q.sn;
            float* qs = qsm[warp];
            __syncwarp();
            for (int d = lane; d < DP; d += 32) qs[d] = (d < D) ? __bfloat162float(qp[d]) : 0.f;
            __syncwarp();
            float qq[FsbDim<D>::NPL];
#pragma unroll
            for (int i = 0; i < FsbDim<D>::NPL; ++i) { const float v = qs[lane + 32 * i]; qq[i] = f_mul(v, v); }
            const float qn = f_mul(f_sqrt(fsb_warp_det_sum<D>(qq)), a.radius_coef);
            uint32_t qreg[D / 2];
#pragma unroll
            for (int i = 0; i < D / 8; ++i) {
                const uint4 w4 = *(const uint4*)(qp + i * 8);
                qreg[i * 4 + 0] = w4.x; qreg[i * 4 + 1] = w4.y; qreg[i * 4 + 2] = w4.z; qreg[i * 4 + 3] = w4.w;
            }
            int nv = 0;
            const int c = beam<D, false, true>(F, t, sp, pre, qreg, qn, qpos, lam, sig, a.scale, width, lane, frs[warp], nv,
                                               stg_mu, stg_aux, qs);
            if (lane < width) cand_sm[qi][f * WMAX + lane] = c;
            if (lane == 0) nv_sm[qi] += nv;
        }
    }
    __syncthreads();
    // ---- union (second beam's repeats of a main cell blanked), outputs, and the per-query re-rank when asked ----
    for (int qi = warp; qi < a.Bq; qi += NWARP) {
        const int64_t row = ((int64_t)t * gridDim.x + blk) * a.Bq + qi;         // (B,H,Npad) flattened
        if (qi >= nq) {
            if (lane < a.read_top && a.sel) a.sel[row * a.read_top + lane] = -1;
            if (a.cand && lane < Wc) a.cand[row * Wc + lane] = -1;
            if (a.nvis && lane == 0) a.nvis[row] = 0;
            continue;
        }
        int cand = cand_sm[qi][lane];
        {
            bool dup = false;
            for (int o = 0; o < WMAX; ++o) {
                const int mc = __shfl_sync(FS_FULL, cand, o);
                dup |= (lane >= WMAX && mc == cand);
            }
            if (dup) cand = -1;
        }
        if (a.cand) {
            if (lane < a.width) a.cand[row * Wc + lane] = cand;
            if (lane >= WMAX && lane - WMAX < a.width2) a.cand[row * Wc + a.width + lane - WMAX] = cand;
        }
        if (a.nvis && lane == 0) a.nvis[row] = nv_sm[qi];
        if (a.read_top == 0) continue;          // beams only: the block-cooperative re-rank kernel follows
        const int qidx = blk * a.Bq + qi;
        const float qpos = (float)(a.q_pos0 + qidx);
        const bf16* qp = (const bf16*)a.q.ptr + b * a.q.sb + hd * a.q.sh + (int64_t)qidx * a.q.sn;
        float* qs = qsm[warp];
        __syncwarp();
        for (int d = lane; d < DP; d += 32) qs[d] = (d < D) ? __bfloat162float(qp[d]) : 0.f;
        __syncwarp();
        // ---- re-rank: u = LSE_t((q.k_t) scale) + lam ceil erf(|p - (c+.5) 32| / (2 sig)) ----
        float u = -INFINITY;
        for (int i = 0; i < 32; ++i) {
            const int cell = __shfl_sync(FS_FULL, cand, i);
            if (cell < 0) continue;
            const float ui = rerank_cell<D>(a, b, hd, t, cell, qs, qpos, lam, sig, lane);
            if (lane == i) u = ui;
        }
        int rank = 0;
#pragma unroll 8
        for (int o = 0; o < 32; ++o) {
            const float uo = __shfl_sync(FS_FULL, u, o);
            rank += (uo > u || (uo == u && o < lane)) ? 1 : 0;
        }
        if (rank < a.read_top) a.sel[row * a.read_top + rank] = (u == -INFINITY) ? -1 : cand;
    }
}

// ---- decode: one query per row, one CTA per row --------------------------------------------------------------------------
// Warp 0 runs the main beam and warp 1 the second beam at the same time (each a chain of dependent table reads, so the
// chain length, not the bandwidth, sets the time; the grandchildren of every scored node are prefetched into L2 one
// level ahead). All eight warps then share the re-rank of the <= 32 candidates, and warp 0 ranks the scores.
// Everything that does not depend on the new token (spines, parameters) is read before the dependency wait, so under
// programmatic dependent launch it overlaps the tail of the QKV projection.
template <int D>
__global__ void __launch_bounds__(256) fsb_decode_select_kernel(SelArgs A) {
    constexpr int DP = FsbDim<D>::DP;
    constexpr int NW = 8;
    const fsattn_fsb_select_t& a = A.a;
    const int t = blockIdx.x;
    const int b = t / A.H, hd = t % A.H;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    __shared__ SpineSm<D> sp[2];
    __shared__ BeamPre pre[2];
    __shared__ __align__(16) float qs[DP];
    __shared__ int frs[2][WMAX * 2];
    __shared__ int cand_s[32];
    __shared__ float u_s[32];
    __shared__ int nv_s[2];

    FSTAMP(0);
    const int nsp = a.width2 > 0 ? 2 : 1;
    {
        // every load of both spines is issued before the first store to shared memory: a load-then-store loop would wait for
        // each memory round trip in turn (in-order issue), a dozen of them back to back
        constexpr int NSPF = SPW * (D + 8), NIT = (NSPF + 255) / 256;
        float tmp[2][NIT];
#pragma unroll
        for (int w = 0; w < 2; ++w) {
            const float* src = a.spine[w < nsp ? w : 0] + (int64_t)t * NSPF;
#pragma unroll
            for (int j = 0; j < NIT; ++j) tmp[w][j] = (w < nsp && tid + 256 * j < NSPF) ? src[tid + 256 * j] : 0.f;
        }
#pragma unroll
        for (int w = 0; w < 2; ++w) {
            float* dst = &sp[w].node[0][0];
#pragma unroll
            for (int j = 0; j < NIT; ++j)
                if (w < nsp && tid + 256 * j < NSPF) dst[tid + 256 * j] = tmp[w][j];
        }
    }
    const float lam = a.lam[hd], sig = a.sigma[hd];
    const float qpos = (float)(*a.pos);
    if (tid == 0) {
        const int4 h0 = *reinterpret_cast<const int4*>(a.hdr[0] + t * 4);
        const int4 h1 = *reinterpret_cast<const int4*>(a.hdr[nsp > 1 ? 1 : 0] + t * 4);
        sp[0].root = h0.x; sp[0].height = h0.y; sp[0].m_b = h0.z;
        sp[0].pad = h0.w;                         // beam width the stored beam head was computed for (0 = none)
        if (nsp > 1) { sp[1].root = h1.x; sp[1].height = h1.y; sp[1].m_b = h1.z; sp[1].pad = h1.w; }
    }
    if (tid < 32) { cand_s[tid] = -1; u_s[tid] = -INFINITY; }
    __syncthreads();
    // the query-independent head of each beam (a few dependent table reads) also runs before the dependency wait
    FSTAMP(1);
    if (warp < nsp) {
        // the query-independent head of the beam: stored beside the spine at the block change, else walked here
        const int wd = warp == 0 ? a.width : a.width2;
        if (sp[warp].pad == wd) {
            const int* src = reinterpret_cast<const int*>(&sp[warp].node[SPW - 1][0]);
            int* dst = reinterpret_cast<int*>(&pre[warp]);
            for (int i = lane; i < (int)(sizeof(BeamPre) / 4); i += 32) dst[i] = src[i];
            __syncwarp();
        } else {
            beam_prefix<D>(warp == 0 ? a.main : a.second, t, sp[warp], wd, lane, pre[warp]);
        }
    }
    FSTAMP(2);
    asm volatile("griddepcontrol.wait;" ::: "memory");
    FSTAMP(3);
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    const bf16* qp = (const bf16*)a.q.ptr + b * a.q.sb + hd * a.q.sh;
    for (int d = tid; d < DP; d += 256) qs[d] = (d < D) ? __bfloat162float(qp[d]) : 0.f;
    __syncthreads();
    if (warp < nsp) {
        float qq[FsbDim<D>::NPL];
#pragma unroll
        for (int i = 0; i < FsbDim<D>::NPL; ++i) { const float v = qs[lane + 32 * i]; qq[i] = f_mul(v, v); }
        const float qn = f_mul(f_sqrt(fsb_warp_det_sum<D>(qq)), a.radius_coef);
        uint32_t qreg[D / 2];
#pragma unroll
        for (int i = 0; i < D / 8; ++i) {
            const uint4 w4 = *(const uint4*)(qp + i * 8);
            qreg[i * 4 + 0] = w4.x; qreg[i * 4 + 1] = w4.y; qreg[i * 4 + 2] = w4.z; qreg[i * 4 + 3] = w4.w;
        }
        int nv = 0;
        FSTAMP(4);
        const int c = beam<D, true>(warp == 0 ? a.main : a.second, t, sp[warp], pre[warp], qreg, qn, qpos, lam, sig, a.scale,
                                    warp == 0 ? a.width : a.width2, lane, frs[warp], nv);
        if (lane < WMAX) cand_s[warp * WMAX + lane] = (lane < (warp == 0 ? a.width : a.width2)) ? c : -1;
        if (lane == 0) nv_s[warp] = nv;
    }
    FSTAMP(5);
    __syncthreads();
    FSTAMP(6);
    if (warp == 0) {                      // union: blank the second beam's repeats of a main cell
        const int mine = cand_s[lane];
        bool dup = false;
        for (int o = 0; o < WMAX; ++o) dup |= (lane >= WMAX && cand_s[o] == mine);
        __syncwarp();
        if (dup) cand_s[lane] = -1;
        if (a.nvis && lane == 0) a.nvis[t] = nv_s[0] + (nsp > 1 ? nv_s[1] : 0);
    }
    __syncthreads();
    const int Wc = a.width + a.width2;
    if (a.cand && tid < 32) {
        if (tid < a.width) a.cand[(int64_t)t * Wc + tid] = cand_s[tid];
        if (tid >= WMAX && tid - WMAX < a.width2) a.cand[(int64_t)t * Wc + a.width + tid - WMAX] = cand_s[tid];
    }
    // every candidate's token keys are asked for now, so that a warp's second to fourth cell wait in L2, not in HBM
    for (int i = warp; i < 32; i += NW) {
        const int cell = cand_s[i];
        if (cell < 0) continue;
        const char* rows = a.k.ptr ? (const char*)((const bf16*)a.k.ptr + b * a.k.sb + hd * a.k.sh + (int64_t)cell * 32 * a.k.sn)
                                   : (const char*)(a.kq + b * a.kq_sb + hd * a.kq_sh + (int64_t)cell * 32 * D);
        const int nbytes = a.k.ptr ? (int)(32 * a.k.sn * 2) : 32 * D;
        for (int o = lane * 128; o < nbytes; o += 32 * 128) asm volatile("prefetch.global.L2 [%0];" ::"l"(rows + o));
    }
    FSTAMP(7);
    {   // a warp's cells in groups: all rows of a group are requested before the first is scored
        constexpr int RG = (D <= 64) ? 4 : 1;     // wider heads keep one row at a time: two already spill
        for (int i0 = warp; i0 < 32; i0 += NW * RG) {
            RrRow<D> rows[RG];
            int cells[RG];
#pragma unroll
            for (int j = 0; j < RG; ++j) {
                const int i = i0 + j * NW;
                cells[j] = (i < 32) ? cand_s[i] : -1;
                if (cells[j] >= 0) rr_load<D>(rows[j], a, b, hd, t, cells[j], lane);
            }
#pragma unroll
            for (int j = 0; j < RG; ++j) {
                if (cells[j] < 0) continue;
                const float ui = rr_score<D>(rows[j], a, cells[j], qs, qpos, lam, sig);
                if (lane == 0) u_s[i0 + j * NW] = ui;
            }
        }
    }
    FSTAMP(8);
    __syncthreads();
    FSTAMP(9);
    if (warp == 0) {
        const float u = u_s[lane];
        const int cand = cand_s[lane];
        int rank = 0;
#pragma unroll 8
        for (int o = 0; o < 32; ++o) {
            const float uo = __shfl_sync(FS_FULL, u, o);
            rank += (uo > u || (uo == u && o < lane)) ? 1 : 0;
        }
        if (rank < a.read_top) a.sel[(int64_t)t * a.read_top + rank] = (u == -INFINITY) ? -1 : cand;
    }
    FSTAMP(10);
}

// The last spine slot is never a spine node (heights stay below 15): it carries the beam's query-independent head
// (beam_prefix) for the beam width the caller names, so that a decode step only copies it (hdr[3] = that width, 0 = none).
static_assert(sizeof(BeamPre) <= (64 + 8) * sizeof(float), "the beam head must fit one spine slot");

template <int D>
__global__ void fsb_spine_kernel(fsattn_fsb_forest_t F, int n_visible, int width, float* spine, int* hdr) {
    const int t = blockIdx.x, lane = threadIdx.x;
    __shared__ SpineSm<D> S;
    __shared__ BeamPre P;
    for (int i = lane; i < SPW * (D + 8); i += 32) (&S.node[0][0])[i] = 0.f;
    __syncwarp();
    const int m_b = count_below(F.adm + (int64_t)t * F.m_cap, F.m_tot[t], n_visible);
    build_spine<D>(F, t, m_b, S, lane);
    __syncwarp();
    if (width > 0) {
        beam_prefix<D>(F, t, S, width, lane, P);
        int* slot = reinterpret_cast<int*>(&S.node[SPW - 1][0]);
        for (int i = lane; i < (int)(sizeof(BeamPre) / 4); i += 32) slot[i] = reinterpret_cast<const int*>(&P)[i];
        __syncwarp();
    }
    float* dst = spine + (int64_t)t * SPW * (D + 8);
    for (int i = lane; i < SPW * (D + 8); i += 32) dst[i] = (&S.node[0][0])[i];
    if (lane == 0) {
        hdr[t * 4 + 0] = S.root; hdr[t * 4 + 1] = S.height; hdr[t * 4 + 2] = S.m_b; hdr[t * 4 + 3] = width > 0 ? width : 0;
    }
}

}  // namespace

int fs_fsb_check_forest(const fsattn_fsb_forest_t& f, const char* what);
int fs_fsb_rerank_block(const fsattn_fsb_select_t* a, cudaStream_t st);

#ifdef FSATTN_FSB_TIMING
extern "C" __attribute__((visibility("default"))) int fsattn_debug_fsb_timing(long long* out64) {
    return cudaMemcpyFromSymbol(out64, g_fsb_stamps, sizeof(long long) * 64) == cudaSuccess ? 0 : -1;
}
#endif

extern "C" int fsattn_fsb_spines(const fsattn_fsb_forest_t* forests, int32_t n_forests, int32_t n_visible,
                                 float* const* spine, int32_t* const* hdr, const int32_t* widths, fsattn_stream_t stream) {
    FS_REQUIRE(forests && spine && hdr && n_forests >= 1, "fsb_spines: null argument");
    for (int i = 0; i < n_forests; ++i) {
        const fsattn_fsb_forest_t& F = forests[i];
        int rc = fs_fsb_check_forest(F, "fsb_spines");
        if (rc != FSATTN_OK) return rc;
        FS_REQUIRE(spine[i] && hdr[i] && n_visible >= 0, "fsb_spines: null output");
        cudaStream_t st = (cudaStream_t)stream;
        const int width = widths ? widths[i] : 0;
        FS_REQUIRE(width >= 0 && width <= WMAX, "fsb_spines: beam width %d (0 = no beam head, at most %d)", width, WMAX);
        switch (F.D) {
            case 64: fsb_spine_kernel<64><<<F.T, 32, 0, st>>>(F, n_visible, width, spine[i], hdr[i]); break;
            case 96: fsb_spine_kernel<96><<<F.T, 32, 0, st>>>(F, n_visible, width, spine[i], hdr[i]); break;
            default: fsb_spine_kernel<128><<<F.T, 32, 0, st>>>(F, n_visible, width, spine[i], hdr[i]); break;
        }
        rc = fs_check_launch("fsb_spine_kernel");
        if (rc != FSATTN_OK) return rc;
    }
    return FSATTN_OK;
}

extern "C" int fsattn_fsb_select(const fsattn_fsb_select_t* a, fsattn_stream_t stream) {
    FS_REQUIRE(a, "fsb_select: null argument");
    int rc = fs_fsb_check_forest(a->main, "fsb_select(main)");
    if (rc != FSATTN_OK) return rc;
    rc = fs_fsb_check_forest(a->second, "fsb_select(second)");
    if (rc != FSATTN_OK) return rc;
    FS_REQUIRE(a->main.T == a->second.T && a->main.D == a->second.D, "fsb_select: the two forests share T and D");
    FS_REQUIRE(a->B > 0 && a->main.T % a->B == 0, "fsb_select: B = %d does not divide T = %d", a->B, a->main.T);
    FS_REQUIRE(a->q.ptr && a->sel && a->lam && a->sigma, "fsb_select: null q / sel / lam / sigma");
    FS_REQUIRE(a->k.ptr || (a->kq && a->ks), "fsb_select: token keys missing (bf16 k, or int8 kq + scales ks)");
    FS_REQUIRE(a->k.ptr || (((uintptr_t)a->kq & 15) == 0 && a->kq_sb % 16 == 0 && a->kq_sh % 16 == 0),
               "fsb_select: int8 key rows must be 16-byte aligned");
    FS_UNSUPPORTED(a->width < 1 || a->width > WMAX || a->width2 < 0 || a->width2 > WMAX,
                   "fsb_select: beam widths %d / %d (1..16 and 0..16)", a->width, a->width2);
    FS_REQUIRE(a->read_top >= 1 && a->read_top <= 32, "fsb_select: read_top = %d", a->read_top);
    FS_REQUIRE(a->Bq >= 1 && a->N >= 1, "fsb_select: N = %d, Bq = %d", a->N, a->Bq);
    FS_REQUIRE(a->beam_impl >= 0 && a->beam_impl <= 1, "fsb_select: beam_impl = %d (0 or 1)", a->beam_impl);
    if (a->use_spines) {
        FS_REQUIRE(a->spine[0] && a->hdr[0] && a->pos && (a->width2 == 0 || (a->spine[1] && a->hdr[1])),
                   "fsb_select: decode needs the spines, their headers and pos");
        FS_REQUIRE(a->N == 1 && a->Bq == 1, "fsb_select: decode takes one query per row (N = Bq = 1)");
    } else {
        FS_REQUIRE(a->main.compact == 0 && a->second.compact == 0,
                   "fsb_select: a prefill names the forests of earlier prefixes, which only the full arena (compact = 0) keeps");
        FS_REQUIRE((a->q_pos0 % 32) == 0 && ((a->Bq % 32) == 0 || a->N <= a->Bq),
                   "fsb_select: q_pos0 and Bq must be multiples of the cell (Bq may be ragged for a single block)");
    }
    SelArgs A;
    A.a = *a;
    A.H = a->main.T / a->B;
    A.ncell_k = 0;
    // prefill with full 128-query blocks and a candidate buffer: beams per query, then the block-cooperative re-rank
    const bool two_pass = !a->use_spines && a->Bq == 128 && a->cand != nullptr;
    if (two_pass) A.a.read_top = 0;
    const int nb = (a->N + a->Bq - 1) / a->Bq;
    cudaStream_t st = (cudaStream_t)stream;
    dim3 grid(nb, a->main.T);
    if (a->use_spines) {
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(a->main.T, 1, 1);
        cfg.blockDim = dim3(256, 1, 1);
        cfg.stream = st;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = a->pdl ? 1 : 0;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        cudaError_t e;
        switch (a->main.D) {
            case 64: e = cudaLaunchKernelEx(&cfg, fsb_decode_select_kernel<64>, A); break;
            case 96: e = cudaLaunchKernelEx(&cfg, fsb_decode_select_kernel<96>, A); break;
            default: e = cudaLaunchKernelEx(&cfg, fsb_decode_select_kernel<128>, A); break;
        }
        if (e != cudaSuccess) {
            fs_set_error("fsb_select: launch failed: %s", cudaGetErrorString(e));
            return FSATTN_ELAUNCH;
        }
        return FSATTN_OK;
    } else {
        FS_UNSUPPORTED(a->Bq > 128, "fsb_select: query blocks of %d (at most 128)", a->Bq);
        cudaError_t e = cudaSuccess;
        if (two_pass && a->beam_impl != 1) {
            // whole 128-query blocks: one thread per query, the block's distinct nodes scored on tensor-core tiles
            switch (a->main.D) {
                case 64: e = launch_beam_block<64>(A, grid, st); break;
                case 96: e = launch_beam_block<96>(A, grid, st); break;
                default: e = launch_beam_block<128>(A, grid, st); break;
            }
            if (e != cudaSuccess) {
                cudaGetLastError();
                fs_set_error("fsb_select: shared-memory opt-in failed: %s", cudaGetErrorString(e));
                return FSATTN_ELAUNCH;
            }
            rc = fs_check_launch("fsb_beam_block_kernel");
            if (rc != FSATTN_OK) return rc;
            return fs_fsb_rerank_block(a, st);
        }
        switch (a->main.D) {
            case 64:
                e = cudaFuncSetAttribute(fsb_select_kernel<64, SEL_NW>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)SelSmem<64>::TOTAL);
                if (e == cudaSuccess) fsb_select_kernel<64, SEL_NW><<<grid, SEL_NW * 32, SelSmem<64>::TOTAL, st>>>(A);
                break;
            case 96:
                e = cudaFuncSetAttribute(fsb_select_kernel<96, SEL_NW>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)SelSmem<96>::TOTAL);
                if (e == cudaSuccess) fsb_select_kernel<96, SEL_NW><<<grid, SEL_NW * 32, SelSmem<96>::TOTAL, st>>>(A);
                break;
            default:
                e = cudaFuncSetAttribute(fsb_select_kernel<128, SEL_NW>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)SelSmem<128>::TOTAL);
                if (e == cudaSuccess) fsb_select_kernel<128, SEL_NW><<<grid, SEL_NW * 32, SelSmem<128>::TOTAL, st>>>(A);
                break;
        }
        if (e != cudaSuccess) {
            cudaGetLastError();
            fs_set_error("fsb_select: shared-memory opt-in failed: %s", cudaGetErrorString(e));
            return FSATTN_ELAUNCH;
        }
    }
    rc = fs_check_launch("fsb_select_kernel");
    if (rc != FSATTN_OK || !two_pass) return rc;
    return fs_fsb_rerank_block(a, st);
}
