// FS-B forest: admission of cells and construction of the chunk trees (one chunk per newly admitted position).
//
// A chunk tree over n = 2^k cells is built level by level by one CTA. All nodes of a level hold m = n >> l cells in
// consecutive slots of an order array, so every pass below is a flat parallel loop over slots, slot pairs or
// (slot, dim) elements. Reductions keep the halving association order of the reference's det_sum and use explicit
// IEEE intrinsics, so the trees match a CPU build bit for bit:
//   mean     : Y[q] = x[i] + x[i + m/2] then in-place halving steps            (sum over a node's cells)
//   |x-mu|^2 : one warp per cell, lanes hold dims L, L+32, ...                    (sum over the head dimension)
//   split    : farthest member -> two power iterations -> projection -> stable rank sort; lower half goes left.
// Chunks of up to 32 cells live entirely in shared memory; larger ones use an L2-resident scratch area.
#include "fsb.cuh"

namespace {

struct BuildArgs {
    fsattn_fsb_forest_t f[4];
    int nf;
    int k_cap;
    int mode;              // 0: every position of the arena in big-first order; 1: positions m_prev + blockIdx.x
    int x0;                // mode 0: first item index of this launch
    float* scratch;        // big chunks: per forest, per row
    int64_t scratch_per_forest, scratch_per_row;
};

__device__ __forceinline__ int64_t scratch_cells_before(int k, int jj, int k_cap, int m_cap) {
    // cells of scratch in front of chunk (k, jj) inside one row's area; heights below 6 never use it
    return (int64_t)(k - (FSB_SMALL_K + 1)) * (m_cap >> 1) + ((k < k_cap) ? ((int64_t)jj << k) : 0);
}

// ------------------------------------------------------------------------------------------------------------------
// admission: cells [cb, ce) with ceil >= tau[h] are appended to adm in ascending order
// ------------------------------------------------------------------------------------------------------------------
__global__ void __launch_bounds__(256) fsb_admit_kernel(BuildArgs a, int cb, int ce) {
    const fsattn_fsb_forest_t& F = a.f[blockIdx.y];
    const int t = blockIdx.x;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    __shared__ int wsum[8];
    __shared__ int base;
    const float tau = F.tau[t % F.H];
    const float* ceil = F.ceil + (int64_t)t * F.ceil_st;
    int* adm = F.adm + (int64_t)t * F.m_cap;
    const int lim = fsb_admit_limit(F.m_cap, F.compact);      // a sized compact arena admits no more than it has places for
    if (tid == 0) {
        base = F.m_tot[t];
        F.m_prev[t] = base;
    }
    __syncthreads();
    for (int c0 = cb; c0 < ce; c0 += 256) {
        const int c = c0 + tid;
        const bool ok = c < ce && ceil[c] >= tau;
        const unsigned bal = __ballot_sync(FS_FULL, ok);
        if (lane == 0) wsum[warp] = __popc(bal);
        __syncthreads();
        int off = base;
        for (int w = 0; w < warp; ++w) off += wsum[w];
        off += __popc(bal & ((1u << lane) - 1));
        if (ok && off < lim) adm[off] = c;
        __syncthreads();
        if (tid == 0) {
            int tot = 0;
            for (int w = 0; w < 8; ++w) tot += wsum[w];
            base = min(base + tot, lim);
        }
        __syncthreads();
    }
    if (tid == 0) F.m_tot[t] = base;
}

// ------------------------------------------------------------------------------------------------------------------
// chunk build
// ------------------------------------------------------------------------------------------------------------------
// CS > 1: the chunk is built by a thread-block cluster of CS CTAs. Every pass strides over the cluster's threads (or warps)
// instead of the CTA's, and the barriers between passes are cluster barriers (hardware, release / acquire at cluster scope:
// the working arrays live in the L2-resident scratch, so the other CTAs' writes are visible after them). Which thread
// computes an element changes nothing in its arithmetic, so the trees stay bit-identical. Every barrier sits at a point all
// CTAs of the cluster reach the same number of times (the early returns depend on the chunk only, never on the CTA).
template <int CS>
__device__ __forceinline__ void fsb_build_sync() {
    if constexpr (CS == 1) {
        __syncthreads();
    } else {
        asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
    }
}

// The halving steps of a node sum: on entry Y[(g h + i) D + d], i < h, hold the first-level sums of node g; after the
// caller's barrier Y[g h D + d] is the node's sum. Steps over 16 and more pairs per node are flat passes separated by
// barriers; the last four (at most 16 values per node and dimension) are done by one thread in registers, in the same
// association order (v[i] + v[i + s] for s = 8, 4, 2, 1), which saves four barriers per sum.
constexpr int FSB_HALVE_TAIL = 16;
template <int D, int CS>
__device__ __forceinline__ void fsb_halve(float* Y, int nodes, int h, int part, int parts, int T0, int TS, bool own) {
    for (int h2 = h >> 1; h2 >= FSB_HALVE_TAIL; h2 >>= 1) {
        if (own) __syncthreads(); else fsb_build_sync<CS>();
        const int lh2 = 31 - __clz(h2);
        const int tot = nodes * h2 * D;
        const int e_lo = part * (tot / parts), e_hi = e_lo + tot / parts;
        for (int e0 = e_lo + T0; e0 < e_hi; e0 += TS * 4) {
            float ya[4], yb[4];
            int64_t rr[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const int e = (e0 + u * TS < e_hi) ? e0 + u * TS : e_lo;        // the range's first element stands in past the end
                const int d = e % D, q = e / D;
                const int g = q >> lh2, i = q & (h2 - 1);
                rr[u] = ((int64_t)g * h + i) * D + d;
                ya[u] = Y[rr[u]];
                yb[u] = Y[rr[u] + (int64_t)h2 * D];
            }
#pragma unroll
            for (int u = 0; u < 4; ++u)
                if (e0 + u * TS < e_hi) Y[rr[u]] = f_add(ya[u], yb[u]);
        }
    }
    const int w = min(h, FSB_HALVE_TAIL);             // values left per (node, dimension); a power of two
    if (w < 2) return;
    if (own) __syncthreads(); else fsb_build_sync<CS>();
    const int tot = nodes * D;
    const int e_lo = part * (tot / parts), e_hi = e_lo + tot / parts;
    for (int e = e_lo + T0; e < e_hi; e += TS) {
        const int g = e / D, d = e % D;
        float* base = Y + (int64_t)g * h * D + d;
        float v[FSB_HALVE_TAIL];
#pragma unroll
        for (int i = 0; i < FSB_HALVE_TAIL; ++i) v[i] = i < w ? base[(int64_t)i * D] : 0.0f;
#pragma unroll
        for (int sft = FSB_HALVE_TAIL / 2; sft >= 1; sft >>= 1) {
            if (sft < w) {
#pragma unroll
                for (int i = 0; i < sft; ++i) v[i] = f_add(v[i], v[i + sft]);
            }
        }
        base[0] = v[0];
    }
}

template <int D, int THREADS, bool SMALL, int CS>
__global__ void __launch_bounds__(THREADS) fsb_build_kernel(BuildArgs a) {
    static_assert(!SMALL || CS == 1, "small chunks live in one CTA's shared memory");
    constexpr int NPL = FsbDim<D>::NPL;
    constexpr int NW = THREADS / 32 * CS;                 // warps of the cluster
    constexpr int SN = SMALL ? 32 : 1;                    // shared-memory capacity in cells (small kernel)
    const fsattn_fsb_forest_t& F = a.f[blockIdx.z];
    const int t = blockIdx.y;
    const int m_cap = F.m_cap, k_cap = a.k_cap;
    const int ltid = threadIdx.x, lane = ltid & 31;
    int crank = 0;
    if constexpr (CS > 1) asm("mov.u32 %0, %%cluster_ctarank;" : "=r"(crank));
    const int tid = crank * THREADS + ltid, warp = tid >> 5;       // identity inside the cluster
    constexpr int CT = THREADS * CS;
    // The flat passes are chains of dependent reads of L2-resident arrays, and the hardware issues in order: a loop body
    // "load, load, use, store" pays its memory round trips one iteration after the other. They take U elements per trip and
    // issue all their loads before the first use; elements past the end read element 0 and store nothing.
    constexpr int U = 4;

    // ---- which admitted position does this CTA complete a chunk for? ----
    int p;
    if (a.mode == 0) {
        const int x = a.x0 + blockIdx.x / CS;
        if (x == 0) {
            p = m_cap - 1;
        } else {
            const int fl = 31 - __clz(x);
            const int k_ = k_cap - 1 - fl;
            p = ((2 * (x - (1 << fl)) + 1) << k_) - 1;
        }
    } else {
        p = F.m_prev[t] + blockIdx.x / CS;
    }
    if (p < F.m_prev[t] || p >= F.m_tot[t]) return;
    const int k = __ffs(p + 1) - 1;
    if constexpr (SMALL) {
        if (k > FSB_SMALL_K) return;
    } else if constexpr (CS > 1) {
        if (k < FSB_CLUSTER_K) return;
    } else {
        if (k <= FSB_SMALL_K || k >= FSB_CLUSTER_K) return;
    }
    const int n = 1 << k;
    if (n > FSB_MAX_CHUNK) return;             // cannot happen below 524 288 admitted tokens per row
    const int j = ((p + 1) >> k) - 1, jj = j >> 1;
    const int pos0 = p + 1 - n;
    if (F.compact) {
        // one place per height: of the chunks this ingest completes only the one still named by the new admitted count is
        // built (an earlier one of the same height has already been merged into a higher chunk, and would race for the place)
        const int m = F.m_tot[t];
        if (!((m >> k) & 1) || j != ((m >> (k + 1)) << 1)) return;
    }

    const int* adm = F.adm + (int64_t)t * m_cap + pos0;
    const float* kbar = F.kbar + (int64_t)t * F.kbar_st;
    const float* ceil = F.ceil + (int64_t)t * F.ceil_st;
    const int64_t node0 = (int64_t)t * fsb_nodes_per_row(m_cap, F.compact) + fsb_root_node(k, j, m_cap, F.compact);
    bf16* node_mu = (bf16*)F.node_mu + node0 * D;
    float4* node_aux = (float4*)F.node_aux + node0;
    float* root32 = F.root32 + ((int64_t)t * fsb_root_rows(m_cap, F.compact) + fsb_chunk_id(k, j, m_cap, F.compact)) * (D + FSB_ROOT_PAD);

    // ---- working arrays ----
    __shared__ float sm_f[SMALL ? (SN * D * 2 + SN) : 1];
    __shared__ int sm_i[SMALL ? (SN * 2 + SN / 2) : 1];
    __shared__ float sm_proj[SMALL ? 1 : FSB_MAX_CHUNK];
    float *XC, *Y, *VV, *S1;
    int *ordA, *ordB, *FAR;
    if constexpr (SMALL) {
        XC = sm_f; Y = XC + SN * D; VV = Y + (SN / 2) * D; S1 = VV + (SN / 2) * D;
        ordA = sm_i; ordB = ordA + SN; FAR = ordB + SN;
    } else {
        float* base = a.scratch + blockIdx.z * a.scratch_per_forest + t * a.scratch_per_row +
                      scratch_cells_before(k, jj, k_cap, m_cap) * (2 * D + 4);
        XC = base; Y = XC + (int64_t)n * D; VV = Y + (int64_t)(n / 2) * D; S1 = VV + (int64_t)(n / 2) * D;
        ordA = (int*)(S1 + n); ordB = ordA + n; FAR = ordB + n;
    }
    for (int i = tid; i < n; i += CT) ordA[i] = i;
    fsb_build_sync<CS>();

    for (int l = 0; l <= k; ++l) {
        const int lm = k - l, m = 1 << lm, h = m >> 1, nodes = 1 << l;
        // Once a level has at least CS nodes, every CTA of the cluster owns whole subtrees: it walks its own 1/CS of the nodes,
        // members and elements, and its passes are separated by CTA barriers only (no CTA executes a cluster barrier from then
        // on); above that the cluster works together. With CS = 1 this is the plain one-CTA build.
        const bool own = CS > 1 && nodes >= CS;
        const int part = own ? crank : 0, parts = own ? CS : 1;
        const int T0 = own ? ltid : tid, TS = own ? THREADS : CT;                    // flat passes: offset and stride
        const int W0 = own ? (ltid >> 5) : warp, WS = own ? THREADS / 32 : NW;       // per-row passes
        auto lo = [&](int total) { return part * (total / parts); };
        auto hi = [&](int total) { return (part + 1) * (total / parts); };
        auto sync = [&]() { if (own) __syncthreads(); else fsb_build_sync<CS>(); };
        // ---- P1: mean = halving sum of the members / m ----
        if (m >= 2) {
            const int e_lo = lo((n / 2) * D), e_hi = hi((n / 2) * D);
            for (int e0 = e_lo + T0; e0 < e_hi; e0 += TS * U) {
                int o0[U], o1[U];
#pragma unroll
                for (int u = 0; u < U; ++u) {
                    const int e = (e0 + u * TS < e_hi) ? e0 + u * TS : e_lo;       // past the end: the range's first element
                    const int q = e / D;
                    const int g = q >> (lm - 1), i = q & (h - 1);
                    o0[u] = ordA[(g << lm) + i];
                    o1[u] = ordA[(g << lm) + i + h];
                }
#pragma unroll
                for (int u = 0; u < U; ++u) { o0[u] = adm[o0[u]]; o1[u] = adm[o1[u]]; }
                float x0[U], x1[U];
#pragma unroll
                for (int u = 0; u < U; ++u) {
                    const int e = (e0 + u * TS < e_hi) ? e0 + u * TS : e_lo;
                    const int d = e % D;
                    x0[u] = kbar[(int64_t)o0[u] * D + d];
                    x1[u] = kbar[(int64_t)o1[u] * D + d];
                }
#pragma unroll
                for (int u = 0; u < U; ++u) {
                    const int e = e0 + u * TS;
                    if (e < e_hi) Y[e] = f_add(x0[u], x1[u]);
                }
            }
            fsb_halve<D, CS>(Y, nodes, h, part, parts, T0, TS, own);
            sync();
        }
        // ---- P2: centre the members, squared distance ----
        for (int c0 = lo(n) + W0; c0 < hi(n); c0 += WS * 2) {      // two members per trip: both rows are in flight before either is used
            const int c1 = c0 + WS;
            const bool two = c1 < hi(n);
            const int cb = two ? c1 : c0;
            const int o0 = ordA[c0], o1 = ordA[cb];
            const int id0 = adm[o0], id1 = adm[o1];
            float x[2][NPL], mu[2][NPL];
            fsb_load_row<D>(kbar + (int64_t)id0 * D, lane, x[0]);
            fsb_load_row<D>(kbar + (int64_t)id1 * D, lane, x[1]);
            if (m >= 2) {
                fsb_load_row<D>(Y + (int64_t)(c0 >> lm) * h * D, lane, mu[0]);
                fsb_load_row<D>(Y + (int64_t)(cb >> lm) * h * D, lane, mu[1]);
            }
#pragma unroll
            for (int r = 0; r < 2; ++r) {
                if (r == 1 && !two) break;
                float xc[NPL], sq[NPL];
#pragma unroll
                for (int i = 0; i < NPL; ++i) {
                    const float mm = (m >= 2) ? f_div(mu[r][i], (float)m) : x[r][i];
                    xc[i] = f_add(x[r][i], -mm);
                    sq[i] = f_mul(xc[i], xc[i]);
                }
                const int c = r == 0 ? c0 : c1;
                fsb_store_row<D>(XC + (int64_t)c * D, lane, xc);
                const float d2 = fsb_warp_det_sum<D>(sq);
                if (lane == 0) S1[c] = d2;
            }
        }
        sync();
        // ---- P3: node statistics, node tables, farthest member ----
        for (int g = lo(nodes) + W0; g < hi(nodes); g += WS) {
            float best = -1.0f, am = -INFINITY;
            int bi = 0x7fffffff, pm = 0x7fffffff;
            for (int c = (g << lm) + lane; c < ((g + 1) << lm); c += 32) {
                const float v = S1[c];
                if (v > best) { best = v; bi = c; }
                const int id = adm[ordA[c]];
                am = fmaxf(am, ceil[id]);
                pm = min(pm, id);
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                const float ov = __shfl_xor_sync(FS_FULL, best, o);
                const int oi = __shfl_xor_sync(FS_FULL, bi, o);
                if (ov > best || (ov == best && oi < bi)) { best = ov; bi = oi; }
                am = fmaxf(am, __shfl_xor_sync(FS_FULL, am, o));
                pm = min(pm, __shfl_xor_sync(FS_FULL, pm, o));
            }
            if (lane == 0 && l < k) FAR[g] = bi;      // leaves are not split: FAR holds one entry per INNER node (n/2)
            float mu[NPL], er[NPL];
            if (m >= 2) {
                fsb_load_row<D>(Y + (int64_t)g * h * D, lane, mu);
#pragma unroll
                for (int i = 0; i < NPL; ++i) mu[i] = f_div(mu[i], (float)m);
            } else {
                fsb_load_row<D>(kbar + (int64_t)adm[ordA[g]] * D, lane, mu);
            }
            const int nidx = nodes - 1 + g;
#pragma unroll
            for (int i = 0; i < NPL; ++i) {
                const int d = lane + 32 * i;
                const bf16 b = __float2bfloat16_rn(mu[i]);
                if (d < D) node_mu[(int64_t)nidx * D + d] = b;
                const float e = (d < D) ? f_add(mu[i], -__bfloat162float(b)) : 0.0f;
                er[i] = f_mul(e, e);
            }
            const float eps = f_sqrt(fsb_warp_det_sum<D>(er));
            const float rad = f_sqrt(best);
            if (lane == 0) {
                const int meta = (l == k) ? adm[ordA[g]] : ~((nidx << 4) | lm);
                node_aux[nidx] = make_float4(f_add(rad, eps), fmaxf(am, 0.0f), __int_as_float(pm), __int_as_float(meta));
            }
            if (l == 0) {
                fsb_store_row<D>(root32, lane, mu);
                if (lane == 0) root32[D] = rad;
            }
        }
        if (l == k) break;
        sync();
        // ---- P4: start direction = farthest member, normalised ----
        const int v_lo = lo(nodes * D), v_hi = hi(nodes * D);
        for (int e0 = v_lo + T0; e0 < v_hi; e0 += TS * U) {
            int fc[U];
#pragma unroll
            for (int u = 0; u < U; ++u) { const int e = (e0 + u * TS < v_hi) ? e0 + u * TS : v_lo; fc[u] = FAR[e / D]; }
            float xv[U], sv[U];
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const int e = (e0 + u * TS < v_hi) ? e0 + u * TS : v_lo;
                xv[u] = XC[(int64_t)fc[u] * D + e % D];
                sv[u] = S1[fc[u]];
            }
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const int e = e0 + u * TS;
                if (e < v_hi) VV[e] = f_div(xv[u], fmaxf(f_sqrt(sv[u]), 1e-6f));
            }
        }
        sync();
        // ---- P5: two power iterations v <- normalise(sum_c xc_c (xc_c . v)) ; P6: projections ----
        for (int it = 0; it < 3; ++it) {
            for (int c0 = lo(n) + W0; c0 < hi(n); c0 += WS * 2) {
                const int c1 = c0 + WS;
                const bool two = c1 < hi(n);
                const int cb = two ? c1 : c0;
                float xc[2][NPL], v[2][NPL];
                fsb_load_row<D>(XC + (int64_t)c0 * D, lane, xc[0]);
                fsb_load_row<D>(XC + (int64_t)cb * D, lane, xc[1]);
                fsb_load_row<D>(VV + (int64_t)(c0 >> lm) * D, lane, v[0]);
                fsb_load_row<D>(VV + (int64_t)(cb >> lm) * D, lane, v[1]);
#pragma unroll
                for (int r = 0; r < 2; ++r) {
                    if (r == 1 && !two) break;
                    float pr[NPL];
#pragma unroll
                    for (int i = 0; i < NPL; ++i) pr[i] = f_mul(xc[r][i], v[r][i]);
                    const float pv = fsb_warp_det_sum<D>(pr);
                    if (lane == 0) S1[r == 0 ? c0 : c1] = pv;
                }
            }
            sync();
            if (it == 2) break;
            const int e_lo = lo((n / 2) * D), e_hi = hi((n / 2) * D);
            for (int e0 = e_lo + T0; e0 < e_hi; e0 += TS * U) {
                float xa[U], xb[U], sa[U], sb[U];
#pragma unroll
                for (int u = 0; u < U; ++u) {
                    const int e = (e0 + u * TS < e_hi) ? e0 + u * TS : e_lo;
                    const int d = e % D, q = e / D;
                    const int g = q >> (lm - 1), i = q & (h - 1);
                    const int c0 = (g << lm) + i, c1 = c0 + h;
                    xa[u] = XC[(int64_t)c0 * D + d]; xb[u] = XC[(int64_t)c1 * D + d];
                    sa[u] = S1[c0]; sb[u] = S1[c1];
                }
#pragma unroll
                for (int u = 0; u < U; ++u) {
                    const int e = e0 + u * TS;
                    if (e < e_hi) Y[e] = f_add(f_mul(xa[u], sa[u]), f_mul(xb[u], sb[u]));
                }
            }
            fsb_halve<D, CS>(Y, nodes, h, part, parts, T0, TS, own);
            sync();
            for (int g = lo(nodes) + W0; g < hi(nodes); g += WS) {
                float vn[NPL], sq[NPL];
                fsb_load_row<D>(Y + (int64_t)g * h * D, lane, vn);
#pragma unroll
                for (int i = 0; i < NPL; ++i) sq[i] = f_mul(vn[i], vn[i]);
                const float nrm = fmaxf(f_sqrt(fsb_warp_det_sum<D>(sq)), 1e-6f);
#pragma unroll
                for (int i = 0; i < NPL; ++i) vn[i] = f_div(vn[i], nrm);
                fsb_store_row<D>(VV + (int64_t)g * D, lane, vn);
            }
            sync();
        }
        // ---- P7: stable ascending rank of the projections inside each node; the lower half becomes the left child ----
        const float* PJ = S1;
        if constexpr (!SMALL) {
            for (int i = lo(n) + ltid; i < hi(n); i += THREADS) sm_proj[i] = S1[i];      // every CTA keeps its own copy (of its own part)
            __syncthreads();
            PJ = sm_proj;
        }
        for (int c = lo(n) + T0; c < hi(n); c += TS) {
            const int b0 = (c >> lm) << lm;
            const float pc = PJ[c];
            int r = 0;
            for (int o = 0; o < m; ++o) {
                const float po = PJ[b0 + o];
                r += (po < pc || (po == pc && b0 + o < c)) ? 1 : 0;
            }
            ordB[b0 + r] = ordA[c];
        }
        sync();
        int* tmp = ordA; ordA = ordB; ordB = tmp;
    }
}

// chunks of 2^FSB_CLUSTER_K cells and more are built by a cluster of FSB_BUILD_CS CTAs: they are the critical path of an
// ingest (one CTA walks 2048 cells x 11 levels in about 5 ms), and only a few of them exist per row
constexpr int FSB_BUILD_CS = 4;

template <int D>
cudaError_t launch_build_cluster(const BuildArgs& a, int items, int T, cudaStream_t st) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(items * FSB_BUILD_CS, T, a.nf);
    cfg.blockDim = dim3(512);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = FSB_BUILD_CS;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, fsb_build_kernel<D, 512, false, FSB_BUILD_CS>, a);
}

template <int D>
int launch_build(const BuildArgs& a0, int T, int new_cells, cudaStream_t st) {
    BuildArgs a = a0;
    const int m_cap = a.f[0].m_cap;
    cudaError_t ce = cudaSuccess;
    if (a.mode == 0) {
        // item x of the big-first order is a chunk of height k_cap - 1 - floor(log2 x) (x = 0: k_cap): the first m_cap >> K
        // items are the chunks of height K and more
        const int cl_items = (a.k_cap >= FSB_CLUSTER_K) ? (m_cap >> FSB_CLUSTER_K) : 0;
        const int big_items = (a.k_cap > FSB_SMALL_K) ? (m_cap >> (FSB_SMALL_K + 1)) : 0;
        a.x0 = 0;
        if (cl_items > 0) ce = launch_build_cluster<D>(a, cl_items, T, st);
        if (big_items > 0) fsb_build_kernel<D, 512, false, 1><<<dim3(big_items, T, a.nf), 512, 0, st>>>(a);
        a.x0 = big_items;
        if (m_cap - big_items > 0)
            fsb_build_kernel<D, 128, true, 1><<<dim3(m_cap - big_items, T, a.nf), 128, 0, st>>>(a);
    } else {
        if (a.k_cap >= FSB_CLUSTER_K) ce = launch_build_cluster<D>(a, new_cells, T, st);
        if (a.k_cap > FSB_SMALL_K) fsb_build_kernel<D, 512, false, 1><<<dim3(new_cells, T, a.nf), 512, 0, st>>>(a);
        fsb_build_kernel<D, 128, true, 1><<<dim3(new_cells, T, a.nf), 128, 0, st>>>(a);
    }
    if (ce != cudaSuccess) {
        (void)cudaGetLastError();
        fs_set_error("fsb_build_kernel (cluster): launch failed: %s", cudaGetErrorString(ce));
        return FSATTN_ELAUNCH;
    }
    return fs_check_launch("fsb_build_kernel");
}

}  // namespace

int64_t fs_fsb_scratch_cells(int m_cap) {
    const int k_cap = fsb_log2(m_cap);
    if (k_cap <= FSB_SMALL_K) return 0;
    return (int64_t)(k_cap - (FSB_SMALL_K + 1)) * (m_cap >> 1) + m_cap;
}

extern "C" int64_t fsattn_fsb_scratch_floats(int32_t m_cap, int32_t D, int32_t T) {
    if (m_cap <= 0 || D <= 0 || T <= 0) return 0;
    return fs_fsb_scratch_cells(m_cap) * (2 * (int64_t)D + 4) * T;
}

int fs_fsb_check_forest(const fsattn_fsb_forest_t& f, const char* what) {
    FS_REQUIRE(f.T > 0 && f.H > 0 && f.T % f.H == 0, "%s: T = %d must be a positive multiple of H = %d", what, f.T, f.H);
    FS_UNSUPPORTED(f.D != 64 && f.D != 96 && f.D != 128, "%s: head dim %d (64, 96 or 128)", what, f.D);
    FS_REQUIRE(f.m_cap >= 1 && (f.m_cap & (f.m_cap - 1)) == 0, "%s: m_cap = %d must be a power of two", what, f.m_cap);
    FS_UNSUPPORTED(f.m_cap > FSB_MAX_MCAP, "%s: m_cap = %d cells (at most %d)", what, f.m_cap, FSB_MAX_MCAP);
    FS_REQUIRE(f.kbar && f.ceil && f.tau && f.adm && f.m_tot && f.m_prev && f.node_mu && f.node_aux && f.root32,
               "%s: null forest buffer", what);
    FS_REQUIRE(f.compact == 0 || f.compact == 1 || f.compact >= fsb_compact_nodes(0),
               "%s: compact = %d (0: full arena, 1: compact with 4 m_cap nodes per row, n > 1: compact with n nodes per row)", what, f.compact);
    return FSATTN_OK;
}

namespace {
// one CTA per (row, height): the chunk of that height named by the row's admitted count, full arena -> compact arena
template <int D>
__global__ void fsb_compact_kernel(fsattn_fsb_forest_t S, fsattn_fsb_forest_t C) {
    const int t = blockIdx.x, k = blockIdx.y;
    const int m = S.m_tot[t];
    if (!((m >> k) & 1)) return;
    const int j = (m >> (k + 1)) << 1;
    const int n = (2 << k) - 1;
    const int64_t s0 = (int64_t)t * fsb_nodes_per_row(S.m_cap, 0) + fsb_root_node(k, j, S.m_cap, 0);
    if (m > fsb_admit_limit(C.m_cap, C.compact)) return;          // (refused on the host side; never copy past the arena)
    const int64_t d0 = (int64_t)t * fsb_nodes_per_row(C.m_cap, C.compact) + fsb_root_node(k, j, S.m_cap, 1);
    const uint4* smu = (const uint4*)((const bf16*)S.node_mu + s0 * D);
    uint4* dmu = (uint4*)((bf16*)C.node_mu + d0 * D);
    for (int64_t i = threadIdx.x; i < (int64_t)n * (D / 8); i += blockDim.x) dmu[i] = smu[i];
    const float4* sa = (const float4*)S.node_aux + s0;
    float4* da = (float4*)C.node_aux + d0;
    for (int i = threadIdx.x; i < n; i += blockDim.x) da[i] = sa[i];
    const float* sr = S.root32 + ((int64_t)t * fsb_root_rows(S.m_cap, 0) + fsb_chunk_id(k, j, S.m_cap, 0)) * (D + FSB_ROOT_PAD);
    float* dr = C.root32 + ((int64_t)t * fsb_root_rows(S.m_cap, 1) + fsb_chunk_id(k, j, S.m_cap, 1)) * (D + FSB_ROOT_PAD);
    for (int i = threadIdx.x; i < D + FSB_ROOT_PAD; i += blockDim.x) dr[i] = sr[i];
}
}  // namespace

extern "C" int fsattn_fsb_compact(const fsattn_fsb_forest_t* src, const fsattn_fsb_forest_t* dst, fsattn_stream_t stream) {
    FS_REQUIRE(src && dst, "fsb_compact: null argument");
    int rc = fs_fsb_check_forest(*src, "fsb_compact(src)");
    if (rc != FSATTN_OK) return rc;
    rc = fs_fsb_check_forest(*dst, "fsb_compact(dst)");
    if (rc != FSATTN_OK) return rc;
    FS_REQUIRE(src->compact == 0 && dst->compact >= 1, "fsb_compact: from the full arena (compact = 0) to a compact one (>= 1)");
    FS_REQUIRE(src->T == dst->T && src->D == dst->D && src->m_cap == dst->m_cap && src->m_tot == dst->m_tot,
               "fsb_compact: both arenas describe the same forest (T, D, m_cap, m_tot)");
    FS_REQUIRE(src->node_mu != dst->node_mu && src->node_aux != dst->node_aux && src->root32 != dst->root32,
               "fsb_compact: the compact arena needs buffers of its own");
    cudaStream_t st = (cudaStream_t)stream;
    const dim3 grid(src->T, fsb_log2(src->m_cap) + 1);
    switch (src->D) {
        case 64: fsb_compact_kernel<64><<<grid, 256, 0, st>>>(*src, *dst); break;
        case 96: fsb_compact_kernel<96><<<grid, 256, 0, st>>>(*src, *dst); break;
        default: fsb_compact_kernel<128><<<grid, 256, 0, st>>>(*src, *dst); break;
    }
    return fs_check_launch("fsb_compact_kernel");
}

extern "C" int fsattn_fsb_ingest(const fsattn_fsb_forest_t* forests, int32_t n_forests, int32_t cell_begin,
                                 int32_t cell_end, float* scratch, int64_t scratch_floats, fsattn_stream_t stream) {
    FS_REQUIRE(forests && n_forests >= 1 && n_forests <= 4, "fsb_ingest: 1 to 4 forests per call (got %d)", n_forests);
    BuildArgs a{};
    a.nf = n_forests;
    for (int i = 0; i < n_forests; ++i) {
        int rc = fs_fsb_check_forest(forests[i], "fsb_ingest");
        if (rc != FSATTN_OK) return rc;
        FS_REQUIRE(forests[i].T == forests[0].T && forests[i].D == forests[0].D && forests[i].m_cap == forests[0].m_cap,
                   "fsb_ingest: the forests of one call share T, D and m_cap");
        a.f[i] = forests[i];
    }
    const fsattn_fsb_forest_t& f0 = forests[0];
    FS_REQUIRE(cell_begin >= 0 && cell_end >= cell_begin && cell_end <= f0.m_cap,
               "fsb_ingest: cells [%d, %d) outside the capacity %d", cell_begin, cell_end, f0.m_cap);
    if (cell_end == cell_begin) return FSATTN_OK;
    a.k_cap = fsb_log2(f0.m_cap);
    const int64_t per_row = fs_fsb_scratch_cells(f0.m_cap) * (2 * (int64_t)f0.D + 4);
    a.scratch = scratch;
    a.scratch_per_row = per_row;
    a.scratch_per_forest = per_row * f0.T;
    FS_REQUIRE(per_row == 0 || (scratch && scratch_floats >= a.scratch_per_forest * n_forests),
               "fsb_ingest: scratch of %lld floats needed (got %lld)", (long long)(a.scratch_per_forest * n_forests),
               (long long)scratch_floats);
    cudaStream_t st = (cudaStream_t)stream;
    fsb_admit_kernel<<<dim3(f0.T, n_forests), 256, 0, st>>>(a, cell_begin, cell_end);
    int rc = fs_check_launch("fsb_admit_kernel");
    if (rc != FSATTN_OK) return rc;
    const int new_cells = cell_end - cell_begin;
    a.mode = (new_cells > 64) ? 0 : 1;
    switch (f0.D) {
        case 64: return launch_build<64>(a, f0.T, new_cells, st);
        case 96: return launch_build<96>(a, f0.T, new_cells, st);
        default: return launch_build<128>(a, f0.T, new_cells, st);
    }
}
