// FS-B prefill re-rank, block-cooperative: the <= 32 candidate cells of each of the 128 queries of a block are scored
// by the log-sum-exp of their token keys. Queries of one block share most of their candidates, so the block first
// builds the list of DISTINCT candidate cells (bitmap + counting sort of the (query, slot) pairs by cell), then stages
// each distinct cell's 32 token keys in shared memory exactly once and scores all pairs that reference it with
// mma.sync m16n8k16 bf16 tiles (16 queries x 32 tokens per tile; fp32 accumulation). Traffic per block drops from
// pairs x 4 KB to distinct cells x 4 KB; the scores differ from a sequential fp32 sum only in the summation order.
#include "fsb.cuh"

namespace {

constexpr int RB_Q = 128;        // queries per block
constexpr int RB_C = 32;         // candidate slots per query
constexpr int RB_THREADS = 512;
constexpr int RB_WARPS = RB_THREADS / 32;
constexpr int RB_PAIRS = RB_Q * RB_C;

struct RrArgs {
    fsattn_fsb_select_t a;
    int H, C;
};

template <int D>
struct RrSmem {
    static constexpr int ROWB = D * 2;                       // bytes per key / query row
    static constexpr int G = (D > 64) ? 4 : 8;                // cells staged per round (two CTAs share an SM: 32 / 24 / 32 KB of keys)
    static constexpr int SW = (D == 96) ? 3 : 7;             // 16-byte-chunk XOR mask (keeps D = 96 inside its 4-chunk groups)
    static constexpr size_t Q_OFF = 0;
    static constexpr size_t K_OFF = Q_OFF + (size_t)RB_Q * ROWB;
    static constexpr size_t CAND_OFF = K_OFF + (size_t)G * 32 * ROWB;
    static constexpr size_t U_OFF = CAND_OFF + RB_PAIRS * 4;
    static constexpr size_t CUR_OFF = U_OFF + RB_PAIRS * 4;          // int[RB_PAIRS + 1]
    static constexpr size_t PIDX_OFF = K_OFF;                        // u16[RB_PAIRS]: only during the sort, over the key area
    static constexpr size_t SORT_OFF = CUR_OFF + (RB_PAIRS + 4) * 4; // u16[RB_PAIRS]
    static constexpr size_t BM_OFF = SORT_OFF + RB_PAIRS * 2;        // u32[512] bitmap (16 384 cells), int[512] word base
    static constexpr size_t TOTAL = BM_OFF + 512 * 4 * 2 + 64;
};

__device__ __forceinline__ uint32_t sw_off(int row, int byte_in_row, int rowb, int swmask) {
    const int chunk = byte_in_row >> 4;
    return (uint32_t)(row * rowb + (((chunk ^ (row & swmask)) << 4) | (byte_in_row & 15)));
}

__device__ __forceinline__ void mma_bf16(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
                 : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
                 : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

template <int D>
__global__ void __launch_bounds__(RB_THREADS, 2) fsb_rerank_block_kernel(RrArgs A) {
    using SM = RrSmem<D>;
    const fsattn_fsb_select_t& a = A.a;
    extern __shared__ __align__(16) unsigned char smem[];
    unsigned char* Qs = smem + SM::Q_OFF;
    unsigned char* Ks = smem + SM::K_OFF;
    int* cand_s = (int*)(smem + SM::CAND_OFF);
    float* u_s = (float*)(smem + SM::U_OFF);
    int* cur = (int*)(smem + SM::CUR_OFF);
    unsigned short* pidx = (unsigned short*)(smem + SM::PIDX_OFF);
    unsigned short* sorted = (unsigned short*)(smem + SM::SORT_OFF);
    uint32_t* bm = (uint32_t*)(smem + SM::BM_OFF);
    int* wbase = (int*)(bm + 512);
    __shared__ int U_s;

    const int blk = blockIdx.x, t = blockIdx.y;
    const int b = t / A.H, hd = t % A.H;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int C = A.C;
    const int nq = min(RB_Q, a.N - blk * RB_Q);
    const int64_t row0 = ((int64_t)t * gridDim.x + blk) * RB_Q;           // first row of this block in (B,H,Npad)

    // ---- load the block's queries (swizzled rows) and candidate lists ----
    {
        const bf16* qbase = (const bf16*)a.q.ptr + b * a.q.sb + hd * a.q.sh;
        constexpr int CH = D / 8;                                          // 16-byte chunks per row
        for (int i = tid; i < RB_Q * CH; i += RB_THREADS) {
            const int r = i / CH, c = i % CH;
            uint4 v = make_uint4(0, 0, 0, 0);
            if (r < nq) v = *(const uint4*)(qbase + (int64_t)(blk * RB_Q + r) * a.q.sn + c * 8);
            *(uint4*)(Qs + sw_off(r, c * 16, SM::ROWB, SM::SW)) = v;
        }
        for (int i = tid; i < RB_PAIRS; i += RB_THREADS) {
            const int r = i >> 5, s = i & 31;
            cand_s[i] = (r < nq && s < C) ? a.cand[(row0 + r) * C + s] : -1;
            u_s[i] = -INFINITY;
        }
        for (int i = tid; i < 512; i += RB_THREADS) bm[i] = 0;
    }
    __syncthreads();
    // ---- distinct cells: bitmap, rank of each cell, counting sort of the pairs by cell ----
    for (int i = tid; i < RB_PAIRS; i += RB_THREADS) {
        const int c = cand_s[i];
        if (c >= 0) atomicOr(&bm[c >> 5], 1u << (c & 31));
    }
    __syncthreads();
    if (warp == 0) {
        int run = 0;
        for (int w0 = 0; w0 < 512; w0 += 32) {
            const int n = __popc(bm[w0 + lane]);
            int inc = n;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int v = __shfl_up_sync(FS_FULL, inc, o);
                if (lane >= o) inc += v;
            }
            wbase[w0 + lane] = run + inc - n;
            run += __shfl_sync(FS_FULL, inc, 31);
        }
        if (lane == 0) U_s = run;
    }
    __syncthreads();
    const int U = U_s;
    for (int i = tid; i <= U; i += RB_THREADS) cur[i] = 0;
    __syncthreads();
    for (int i = tid; i < RB_PAIRS; i += RB_THREADS) {
        const int c = cand_s[i];
        unsigned short ix = 0xffff;
        if (c >= 0) {
            ix = (unsigned short)(wbase[c >> 5] + __popc(bm[c >> 5] & ((1u << (c & 31)) - 1)));
            atomicAdd(&cur[ix], 1);
        }
        pidx[i] = ix;
    }
    __syncthreads();
    if (warp == 0) {                        // exclusive scan of the per-cell counts (U <= 4096)
        int run = 0;
        for (int i0 = 0; i0 < U; i0 += 32) {
            const int n = (i0 + lane < U) ? cur[i0 + lane] : 0;
            int inc = n;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int v = __shfl_up_sync(FS_FULL, inc, o);
                if (lane >= o) inc += v;
            }
            if (i0 + lane < U) cur[i0 + lane] = run + inc - n;
            run += __shfl_sync(FS_FULL, inc, 31);
        }
    }
    __syncthreads();
    for (int i = tid; i < RB_PAIRS; i += RB_THREADS) {
        const unsigned short ix = pidx[i];
        if (ix != 0xffff) sorted[atomicAdd(&cur[ix], 1)] = (unsigned short)i;       // cur[ix] ends at the cell's list end
    }
    __syncthreads();

    // ---- rounds of G distinct cells: stage their keys, score every pair that references them ----
    const float lam = a.lam[hd], two_sig = f_mul(2.0f, a.sigma[hd]);
    const float* ceil = a.main.ceil + (int64_t)t * a.main.ceil_st;
    const int g = lane >> 2, tg = lane & 3;
    constexpr int CH = D / 8;
    for (int c0 = 0; c0 < U; c0 += SM::G) {
        const int ncell = min(SM::G, U - c0);
        // stage: cell slot j holds distinct cell c0 + j; its id comes from the first pair of its list
        for (int i = tid; i < ncell * 32 * CH; i += RB_THREADS) {
            const int j = i / (32 * CH), rem = i % (32 * CH);
            const int r = rem / CH, c = rem % CH;
            const int ix = c0 + j;
            const int start = ix == 0 ? 0 : cur[ix - 1];
            const int cell = cand_s[sorted[start]];
            const int64_t tok = (int64_t)cell * 32 + r;
            uint4 v;
            if (a.k.ptr) {
                v = *(const uint4*)((const bf16*)a.k.ptr + b * a.k.sb + hd * a.k.sh + tok * a.k.sn + c * 8);
            } else {
                const uint2 w = *(const uint2*)(a.kq + b * a.kq_sb + hd * a.kq_sh + tok * D + c * 8);
                const float sc = __bfloat162float(((const bf16*)a.ks)[b * a.ks_sb + hd * a.ks_sh + cell]);
                float o[8];
                unpack4_i8(w.x, o);
                unpack4_i8(w.y, o + 4);
                v.x = pack_bf2(f_mul(o[0], sc), f_mul(o[1], sc)); v.y = pack_bf2(f_mul(o[2], sc), f_mul(o[3], sc));
                v.z = pack_bf2(f_mul(o[4], sc), f_mul(o[5], sc)); v.w = pack_bf2(f_mul(o[6], sc), f_mul(o[7], sc));
            }
            *(uint4*)(Ks + (size_t)j * 32 * SM::ROWB + sw_off(r, c * 16, SM::ROWB, SM::SW)) = v;
        }
        __syncthreads();
        constexpr int WPC = RB_WARPS / SM::G;                     // warps that share a cell's groups of 16 pairs
        const int cj = warp % SM::G;
        if (cj < ncell) {
            const int ix = c0 + cj;
            const int start = ix == 0 ? 0 : cur[ix - 1], end = cur[ix];
            const int cell = cand_s[sorted[start]];
            const unsigned char* Kc = Ks + (size_t)cj * 32 * SM::ROWB;
            const float pcoef = f_mul(lam, ceil[cell]);
            const float cpos = f_mul(f_add((float)cell, 0.5f), 32.0f);
            for (int p0 = start + 16 * (warp / SM::G); p0 < end; p0 += 16 * WPC) {
                const int pa = p0 + g, pb = p0 + g + 8;
                const int ida = pa < end ? sorted[pa] : -1, idb = pb < end ? sorted[pb] : -1;
                const int qa = ida >= 0 ? (ida >> 5) : 0, qb = idb >= 0 ? (idb >> 5) : 0;
                float acc[4][4];
#pragma unroll
                for (int nt = 0; nt < 4; ++nt)
#pragma unroll
                    for (int e = 0; e < 4; ++e) acc[nt][e] = 0.f;
#pragma unroll
                for (int kp = 0; kp < D / 32; ++kp) {               // two k-steps per round: one ldmatrix.x4 per 8-token tile
                    uint32_t af[2][4];
#pragma unroll
                    for (int h2 = 0; h2 < 2; ++h2) {
                        const int kk = 2 * kp + h2;
                        af[h2][0] = *(const uint32_t*)(Qs + sw_off(qa, kk * 32 + tg * 4, SM::ROWB, SM::SW));
                        af[h2][1] = *(const uint32_t*)(Qs + sw_off(qb, kk * 32 + tg * 4, SM::ROWB, SM::SW));
                        af[h2][2] = *(const uint32_t*)(Qs + sw_off(qa, kk * 32 + 16 + tg * 4, SM::ROWB, SM::SW));
                        af[h2][3] = *(const uint32_t*)(Qs + sw_off(qb, kk * 32 + 16 + tg * 4, SM::ROWB, SM::SW));
                    }
#pragma unroll
                    for (int nt = 0; nt < 4; ++nt) {
                        // matrix j of the load = 16-byte chunk kp*4 + j of the tile's eight key rows
                        const uint32_t addr = (uint32_t)__cvta_generic_to_shared(
                            Kc + sw_off(nt * 8 + (lane & 7), (kp * 4 + (lane >> 3)) * 16, SM::ROWB, SM::SW));
                        uint32_t b0, b1, b2, b3;
                        asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                                     : "=r"(b0), "=r"(b1), "=r"(b2), "=r"(b3) : "r"(addr));
                        mma_bf16(acc[nt], af[0], b0, b1);
                        mma_bf16(acc[nt], af[1], b2, b3);
                    }
                }
                // rows g (acc[.][0..1]) and g+8 (acc[.][2..3]): log-sum-exp over the 32 tokens, spread over the quad
                float mh[2], sh[2];
#pragma unroll
                for (int half = 0; half < 2; ++half) {
                    float m = -INFINITY;
#pragma unroll
                    for (int nt = 0; nt < 4; ++nt) {
                        acc[nt][2 * half] = f_mul(acc[nt][2 * half], a.scale);
                        acc[nt][2 * half + 1] = f_mul(acc[nt][2 * half + 1], a.scale);
                        m = fmaxf(m, fmaxf(acc[nt][2 * half], acc[nt][2 * half + 1]));
                    }
                    m = fmaxf(m, __shfl_xor_sync(FS_FULL, m, 1));
                    m = fmaxf(m, __shfl_xor_sync(FS_FULL, m, 2));
                    float s = 0.f;
#pragma unroll
                    for (int nt = 0; nt < 4; ++nt) s += __expf(acc[nt][2 * half] - m) + __expf(acc[nt][2 * half + 1] - m);
                    s += __shfl_xor_sync(FS_FULL, s, 1);
                    s += __shfl_xor_sync(FS_FULL, s, 2);
                    mh[half] = m; sh[half] = s;
                }
                // the quad's lane 0 finishes row g, lane 1 row g + 8 (one logarithm and one erf per lane, both rows at once);
                // erf is 1 in fp32 from 4 on, which is every cell further than a few sigma from the query
                const int id = tg == 0 ? ida : (tg == 1 ? idb : -1);
                if (id >= 0) {
                    const float qpos = (float)(a.q_pos0 + blk * RB_Q + (id >> 5));
                    const float x = f_div(fabsf(f_add(qpos, -cpos)), two_sig);
                    const float er = x < 4.0f ? erff(x) : 1.0f;
                    u_s[id] = f_add(f_add(tg == 0 ? mh[0] : mh[1], logf(tg == 0 ? sh[0] : sh[1])), f_mul(pcoef, er));
                }
            }
        }
        __syncthreads();
    }

    // ---- per query: stable descending rank of the slots' scores, first read_top ----
    for (int r = warp; r < RB_Q; r += RB_WARPS) {
        const int64_t row = row0 + r;
        if (r >= nq) {
            if (lane < a.read_top) a.sel[row * a.read_top + lane] = -1;
            continue;
        }
        const int cd = cand_s[r * 32 + lane];
        const float u = cd >= 0 ? u_s[r * 32 + lane] : -INFINITY;
        int rank = 0;
#pragma unroll 8
        for (int o = 0; o < 32; ++o) {
            const float uo = __shfl_sync(FS_FULL, u, o);
            rank += (uo > u || (uo == u && o < lane)) ? 1 : 0;
        }
        if (rank < a.read_top) a.sel[row * a.read_top + rank] = (u == -INFINITY) ? -1 : cd;
    }
}

template <int D>
int launch_rr(const RrArgs& A, int nb, int T, cudaStream_t st) {
    static bool attr_done[16] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    const size_t smem = RrSmem<D>::TOTAL;
    if (dev >= 0 && dev < 16 && !attr_done[dev]) {
        if (cudaFuncSetAttribute(fsb_rerank_block_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess) {
            cudaGetLastError();
            fs_set_error("fsb_rerank: %zu bytes of shared memory refused", smem);
            return FSATTN_ELAUNCH;
        }
        attr_done[dev] = true;
    }
    fsb_rerank_block_kernel<D><<<dim3(nb, T), RB_THREADS, smem, st>>>(A);
    return fs_check_launch("fsb_rerank_block_kernel");
}

}  // namespace

// Re-rank of precomputed candidates (a->cand, (B,H,Npad,width+width2) int32) -> a->sel. Internal to fsattn_fsb_select.
int fs_fsb_rerank_block(const fsattn_fsb_select_t* a, cudaStream_t st) {
    RrArgs A;
    A.a = *a;
    A.H = a->main.T / a->B;
    A.C = a->width + a->width2;
    const int nb = (a->N + RB_Q - 1) / RB_Q;
    switch (a->main.D) {
        case 64: return launch_rr<64>(A, nb, a->main.T, st);
        case 96: return launch_rr<96>(A, nb, a->main.T, st);
        default: return launch_rr<128>(A, nb, a->main.T, st);
    }
}
