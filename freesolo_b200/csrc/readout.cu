// Prefill long-range readout with lr_norm and the window combine fused in.
//
// One warp per (query, head): lane t scores token t of each selected cell (fp32 dot over D with q in registers), the
// softmax runs online across the <= kk cells, the value accumulation has every lane own D/32 output dims.
// Reads per query: kk * 32 key rows + kk * 32 value rows (mostly L2 hits: neighbouring queries select the same cells).
#include "common.cuh"

template <int D>
__global__ void __launch_bounds__(256) readout_combine_kernel(const fsattn_readout_combine_t a) {
    constexpr int DPL = D / 32;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int qi = blockIdx.x * 8 + warp;
    if (qi >= a.N) return;
    const int bh = blockIdx.y;
    const int b = bh / a.H, h = bh - b * a.H;
    const int qpos = a.q_pos0 + qi;
    const int bs = (qpos / a.Bq) * a.Bq;
    const int n_cells = (a.n_kv + FSATTN_CELL - 1) / FSATTN_CELL;

    float q[D];
    {
        const uint4* qp = reinterpret_cast<const uint4*>((const bf16*)a.q.ptr + b * a.q.sb + h * a.q.sh + (int64_t)qi * a.q.sn);
#pragma unroll
        for (int e = 0; e < D / 8; e++) {
            const uint4 w = qp[e];
            q[8 * e + 0] = bf_lo(w.x); q[8 * e + 1] = bf_hi(w.x); q[8 * e + 2] = bf_lo(w.y); q[8 * e + 3] = bf_hi(w.y);
            q[8 * e + 4] = bf_lo(w.z); q[8 * e + 5] = bf_hi(w.z); q[8 * e + 6] = bf_lo(w.w); q[8 * e + 7] = bf_hi(w.w);
        }
    }
    const int32_t* sel = a.sel + b * a.sel_sb + h * a.sel_sh + (int64_t)qi * a.kk;
    int cells[FSATTN_MAX_KK];
#pragma unroll
    for (int j = 0; j < FSATTN_MAX_KK; j++) {
        int c = (j < a.kk) ? sel[j] : -1;
        bool ok = (c >= 0) && (c < n_cells) && ((int64_t)(c + 1) * FSATTN_CELL <= bs);
#pragma unroll
        for (int i = 0; i < FSATTN_MAX_KK; i++)
            if (i < j && cells[i] == c) ok = false;
        cells[j] = ok ? c : -1;
    }
    const bf16* kbase = (const bf16*)a.k.ptr + b * a.k.sb + h * a.k.sh;
    const bf16* vbase = (const bf16*)a.v.ptr + b * a.v.sb + h * a.v.sh;
    float m = -INFINITY, l = 0.0f;
    float acc[DPL];
#pragma unroll
    for (int j = 0; j < DPL; j++) acc[j] = 0.0f;
#pragma unroll
    for (int j = 0; j < FSATTN_MAX_KK; j++) {
        const int c = cells[j];
        if (c < 0) continue;                         // warp-uniform
        const int tok = c * FSATTN_CELL + lane;
        const bool tok_ok = (tok < a.n_kv) && (tok < qpos);
        float sc = -INFINITY;
        if (tok_ok) {
            const uint4* kp = reinterpret_cast<const uint4*>(kbase + (int64_t)tok * a.k.sn);
            float d0 = 0.f, d1 = 0.f;
#pragma unroll
            for (int e = 0; e < D / 8; e++) {
                const uint4 w = kp[e];
                d0 = fmaf(q[8 * e + 0], bf_lo(w.x), d0); d1 = fmaf(q[8 * e + 1], bf_hi(w.x), d1);
                d0 = fmaf(q[8 * e + 2], bf_lo(w.y), d0); d1 = fmaf(q[8 * e + 3], bf_hi(w.y), d1);
                d0 = fmaf(q[8 * e + 4], bf_lo(w.z), d0); d1 = fmaf(q[8 * e + 5], bf_hi(w.z), d1);
                d0 = fmaf(q[8 * e + 6], bf_lo(w.w), d0); d1 = fmaf(q[8 * e + 7], bf_hi(w.w), d1);
            }
            sc = (d0 + d1) * a.scale;
        }
        const float tile_m = warp_max(sc);
        if (tile_m == -INFINITY) continue;           // no token of this cell counts (warp-uniform)
        const float m_new = fmaxf(m, tile_m);
        const float alpha = (m == -INFINITY) ? 0.0f : __expf(m - m_new);
        const float p = tok_ok ? __expf(sc - m_new) : 0.0f;
        l = l * alpha + warp_sum(p);
#pragma unroll
        for (int jj = 0; jj < DPL; jj++) acc[jj] *= alpha;
        const bf16* vp = vbase + (int64_t)c * FSATTN_CELL * a.v.sn;
#pragma unroll 8
        for (int t = 0; t < FSATTN_CELL; t++) {
            const float pt = __shfl_sync(FS_FULL, p, t);
            if (pt != 0.0f) {                          // warp-uniform
#pragma unroll
                for (int jj = 0; jj < DPL; jj++)
                    acc[jj] = fmaf(pt, __bfloat162float(vp[(int64_t)t * a.v.sn + lane + 32 * jj]), acc[jj]);
            }
        }
        m = m_new;
    }
    // o -> bf16, lr_norm, combine
    float o[DPL];
    float ss = 0.0f;
#pragma unroll
    for (int jj = 0; jj < DPL; jj++) {
        o[jj] = (l > 0.0f) ? bf_round(acc[jj] / l) : 0.0f;
        ss = fmaf(o[jj], o[jj], ss);
    }
    ss = warp_sum(ss);
    const float r = f_div(1.0f, f_sqrt(f_add(ss * (1.0f / D), a.eps)));
    const float g = a.lrs[h];
    const int64_t row = ((int64_t)b * a.N + qi) * ((int64_t)a.H * D) + (int64_t)h * D;
    const bf16* srp = (const bf16*)a.sr + row;
    bf16* yp = (bf16*)a.y + row;
#pragma unroll
    for (int jj = 0; jj < DPL; jj++) {
        const int d = lane + 32 * jj;
        const float lr = f_mul(f_mul(o[jj], r), a.norm_w[d]);
        const float sr = (a.sr != nullptr) ? __bfloat162float(srp[d]) : 0.0f;
        yp[d] = __float2bfloat16_rn(f_add(sr, f_mul(g, lr)));
    }
}

int fs_readout_block(const fsattn_readout_combine_t* a, cudaStream_t st);
int fs_readout_mma(const fsattn_readout_combine_t* a, cudaStream_t st);

extern "C" int fsattn_readout_combine(const fsattn_readout_combine_t* a, fsattn_stream_t stream) {
    FS_REQUIRE(a != nullptr && a->q.ptr && a->k.ptr && a->v.ptr && a->sel && a->y && a->norm_w && a->lrs,
               "readout_combine: null pointer");
    FS_REQUIRE(a->B > 0 && a->H > 0 && a->N > 0 && a->n_kv > 0 && a->Bq > 0, "readout_combine: bad sizes");
    FS_REQUIRE(a->kk >= 1 && a->kk <= FSATTN_MAX_KK, "readout_combine: kk %d not in [1,%d]", a->kk, FSATTN_MAX_KK);
    FS_UNSUPPORTED(a->D != 64 && a->D != 96 && a->D != 128, "readout_combine: head_dim %d not in {64,96,128}", a->D);
    FS_REQUIRE(((uintptr_t)a->q.ptr & 15) == 0 && a->q.sn % 8 == 0 && a->q.sh % 8 == 0 && a->q.sb % 8 == 0 &&
               ((uintptr_t)a->k.ptr & 15) == 0 && a->k.sn % 8 == 0 && a->k.sh % 8 == 0 && a->k.sb % 8 == 0,
               "readout_combine: Q and K rows must be 16-byte aligned");
    cudaStream_t st = (cudaStream_t)stream;
    // whole query blocks of 128 whose cells fit the block kernel's bitmap: the block-cooperative kernel
    const bool blocks = a->Bq == 128 && a->q_pos0 % 128 == 0 && a->n_kv <= 32768 * FSATTN_CELL && a->N >= 128;
    FS_REQUIRE(a->impl >= 0 && a->impl <= 2, "readout_combine: impl %d", a->impl);
    FS_UNSUPPORTED(a->impl == 2 && !(blocks && a->D == 64), "readout_combine: the tensor-core kernel takes whole 128-query "
                   "blocks at head_dim 64");
    if (blocks && a->D == 64 && a->impl != 1) return fs_readout_mma(a, st);
    if (blocks) return fs_readout_block(a, st);
    dim3 grid((a->N + 7) / 8, a->B * a->H);
    switch (a->D) {
        case 64: readout_combine_kernel<64><<<grid, 256, 0, st>>>(*a); break;
        case 96: readout_combine_kernel<96><<<grid, 256, 0, st>>>(*a); break;
        default: readout_combine_kernel<128><<<grid, 256, 0, st>>>(*a); break;
    }
    return fs_check_launch("readout_combine");
}

// ---- block-cooperative readout (query blocks of 128) -----------------------------------------------------------------------
// One CTA per (b, h, 128-query block). All queries of a block select among the same candidate pool, so the block's
// distinct selected cells (<= 512, typically a few dozen) are staged in shared memory once, eight cells at a time, and every
// (query, selected cell) pair is served from there: global/L2 traffic drops from kk*32 rows of K and V per QUERY to one copy of
// each distinct cell per BLOCK. A warp owns 16 queries; lane t scores token t of a cell; the per-query softmax state
// (max, sum, 64 accumulators) lives in shared memory between cells.
namespace {

constexpr int RB_Q = 128;          // queries per CTA
constexpr int RB_THREADS = 256;

template <int D>
struct RbSmem {
    static constexpr int GC = (D <= 96) ? 8 : 4;                 // cells staged per round
    static constexpr int ROWB = D * 2 + 16;                      // padded row: 16-byte reads of 32 different rows hit distinct banks
    static constexpr size_t K_OFF = 0;
    static constexpr size_t V_OFF = K_OFF + (size_t)GC * 32 * ROWB;
    static constexpr size_t Q_OFF = V_OFF + (size_t)GC * 32 * ROWB;          // 128 x D bf16
    static constexpr size_t ACC_OFF = Q_OFF + (size_t)RB_Q * D * 2;             // 128 x D fp32
    static constexpr size_t ML_OFF = ACC_OFF + (size_t)RB_Q * D * 4;            // 128 x (m, l)
    static constexpr size_t SEL_OFF = ML_OFF + (size_t)RB_Q * 8;                // 128 x kk int16 distinct-cell indices
    static constexpr size_t UC_OFF = SEL_OFF + (size_t)RB_Q * FSATTN_MAX_KK * 2; // distinct cells, ascending
    static constexpr size_t BM_OFF = UC_OFF + (size_t)RB_Q * FSATTN_MAX_KK * 4;  // bitmap words + scan
    static constexpr size_t TOTAL = BM_OFF + (2 * 1024 + 16) * 4;      // bitmap, per-word ranks (offset 8: the first 8 hold the warp totals)
};

template <int D>
__global__ void __launch_bounds__(RB_THREADS) readout_block_kernel(const fsattn_readout_combine_t a) {
    using S = RbSmem<D>;
    extern __shared__ __align__(16) unsigned char rb_smem[];
    unsigned char* ks = rb_smem + S::K_OFF;
    unsigned char* vs = rb_smem + S::V_OFF;
    bf16* qs = reinterpret_cast<bf16*>(rb_smem + S::Q_OFF);
    float* accs = reinterpret_cast<float*>(rb_smem + S::ACC_OFF);
    float2* mls = reinterpret_cast<float2*>(rb_smem + S::ML_OFF);
    int16_t* selu = reinterpret_cast<int16_t*>(rb_smem + S::SEL_OFF);
    int* ucell = reinterpret_cast<int*>(rb_smem + S::UC_OFF);
    unsigned* bitmap = reinterpret_cast<unsigned*>(rb_smem + S::BM_OFF);          // 1024 words = 32768 cells
    int* wscan = reinterpret_cast<int*>(bitmap + 1024);
    __shared__ int n_distinct_s;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int blk = blockIdx.x;
    const int bh = blockIdx.y;
    const int b = bh / a.H, h = bh - b * a.H;
    const int q0 = blk * RB_Q;                       // first query of the block (relative); absolute position q_pos0 + q0
    const int bs = ((a.q_pos0 + q0) / a.Bq) * a.Bq;  // block start shared by the whole CTA (Bq == 128, q_pos0 % 128 == 0)
    const int n_cells = (a.n_kv + FSATTN_CELL - 1) / FSATTN_CELL;
    const int vis_cells = min(n_cells, bs / FSATTN_CELL);           // only cells [0, vis_cells) can be selected
    const int nwords = (vis_cells + 31) / 32;

    // ---- stage q, clear state and bitmap -----------------------------------------------------------------------------------
    for (int i = tid; i < RB_Q * (D / 8); i += RB_THREADS) {
        const int r = i / (D / 8), e = i - r * (D / 8);
        uint4 w = make_uint4(0u, 0u, 0u, 0u);
        if (q0 + r < a.N)
            w = reinterpret_cast<const uint4*>((const bf16*)a.q.ptr + b * a.q.sb + h * a.q.sh + (int64_t)(q0 + r) * a.q.sn)[e];
        reinterpret_cast<uint4*>(qs + r * D)[e] = w;
    }
    for (int i = tid; i < RB_Q * D; i += RB_THREADS) accs[i] = 0.0f;
    for (int i = tid; i < RB_Q; i += RB_THREADS) mls[i] = make_float2(-INFINITY, 0.0f);
    for (int i = tid; i < nwords; i += RB_THREADS) bitmap[i] = 0u;
    __syncthreads();
    // ---- validated selections -> bitmap of distinct cells ---------------------------------------------------------------------
    const int32_t* selg = a.sel + b * a.sel_sb + h * a.sel_sh;
    for (int i = tid; i < RB_Q; i += RB_THREADS) {
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
            selu[i * FSATTN_MAX_KK + j] = (int16_t)(ok ? 0 : -1);        // rank filled in below
        }
    }
    __syncthreads();
    // ---- rank of every set bit (exclusive scan over the words), compact list of distinct cells ------------------------------------
    {
        // each thread owns words tid, tid + 256, ...; first the per-thread totals, then a block scan
        int mine = 0;
        for (int w = tid * 4; w < tid * 4 + 4; w++) mine += (w < nwords) ? __popc(bitmap[w]) : 0;       // 4 consecutive words per thread
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
            wscan[8 + w] = run;                                   // exclusive rank of the word's first bit
            while (bits) {
                const int bit = __ffs(bits) - 1;
                bits &= bits - 1;
                if (run < RB_Q * FSATTN_MAX_KK) ucell[run] = w * 32 + bit;
                run++;
            }
        }
        if (tid == RB_THREADS - 1) n_distinct_s = base + incl;
    }
    __syncthreads();
    for (int i = tid; i < RB_Q; i += RB_THREADS) {
#pragma unroll
        for (int j = 0; j < FSATTN_MAX_KK; j++) {
            if (j < a.kk && selu[i * FSATTN_MAX_KK + j] == 0) {
                const int c = selg[(int64_t)(q0 + i) * a.kk + j];
                const unsigned below = bitmap[c >> 5] & ((1u << (c & 31)) - 1u);
                selu[i * FSATTN_MAX_KK + j] = (int16_t)(wscan[8 + (c >> 5)] + __popc(below));
            }
        }
    }
    __syncthreads();
    const int n_distinct = n_distinct_s;

    // ---- rounds of GC cells --------------------------------------------------------------------------------------------------
    const bf16* kbase = (const bf16*)a.k.ptr + b * a.k.sb + h * a.k.sh;
    const bf16* vbase = (const bf16*)a.v.ptr + b * a.v.sb + h * a.v.sh;
    constexpr int CH = D / 8;
    constexpr int DPL = D / 32;
    for (int g0 = 0; g0 < n_distinct; g0 += S::GC) {
        const int gc = min(S::GC, n_distinct - g0);
        for (int i = tid; i < gc * 32 * CH; i += RB_THREADS) {
            const int row = i / CH, e = i - row * CH;             // row = local cell * 32 + token
            const int64_t tok = (int64_t)ucell[g0 + (row >> 5)] * FSATTN_CELL + (row & 31);
            uint4 kw = make_uint4(0u, 0u, 0u, 0u), vw = kw;
            if (tok < a.n_kv) {
                kw = reinterpret_cast<const uint4*>(kbase + tok * a.k.sn)[e];
                vw = reinterpret_cast<const uint4*>(vbase + tok * a.v.sn)[e];
            }
            *reinterpret_cast<uint4*>(ks + (size_t)row * S::ROWB + e * 16) = kw;
            *reinterpret_cast<uint4*>(vs + (size_t)row * S::ROWB + e * 16) = vw;
        }
        __syncthreads();
        // each warp: its 16 queries, every selection that falls into this round
        for (int qi = warp * 16; qi < warp * 16 + 16; qi++) {
            const int qpos = a.q_pos0 + q0 + qi;
#pragma unroll
            for (int j = 0; j < FSATTN_MAX_KK; j++) {
                if (j >= a.kk) break;
                const int u = selu[qi * FSATTN_MAX_KK + j];
                if (u < g0 || u >= g0 + gc) continue;           // warp-uniform
                const int lc = u - g0;
                const int tok = ucell[u] * FSATTN_CELL + lane;
                const bool tok_ok = (tok < a.n_kv) && (tok < qpos);
                const unsigned char* krow = ks + (size_t)(lc * 32 + lane) * S::ROWB;
                float d0 = 0.f, d1 = 0.f;
#pragma unroll
                for (int e = 0; e < CH; e++) {
                    const uint4 kw = *reinterpret_cast<const uint4*>(krow + e * 16);
                    const uint4 qw = reinterpret_cast<const uint4*>(qs + qi * D)[e];
                    d0 = fmaf(bf_lo(qw.x), bf_lo(kw.x), d0); d1 = fmaf(bf_hi(qw.x), bf_hi(kw.x), d1);
                    d0 = fmaf(bf_lo(qw.y), bf_lo(kw.y), d0); d1 = fmaf(bf_hi(qw.y), bf_hi(kw.y), d1);
                    d0 = fmaf(bf_lo(qw.z), bf_lo(kw.z), d0); d1 = fmaf(bf_hi(qw.z), bf_hi(kw.z), d1);
                    d0 = fmaf(bf_lo(qw.w), bf_lo(kw.w), d0); d1 = fmaf(bf_hi(qw.w), bf_hi(kw.w), d1);
                }
                const float sc = tok_ok ? (d0 + d1) * a.scale : -INFINITY;
                const float tile_m = warp_max(sc);
                if (tile_m == -INFINITY) continue;              // warp-uniform
                const float2 ml = mls[qi];
                const float m_new = fmaxf(ml.x, tile_m);
                const float alpha = (ml.x == -INFINITY) ? 0.0f : __expf(ml.x - m_new);
                const float p = tok_ok ? __expf(sc - m_new) : 0.0f;
                const float l_new = ml.y * alpha + warp_sum(p);
                float acc[DPL];
#pragma unroll
                for (int jj = 0; jj < DPL; jj++) acc[jj] = accs[qi * D + lane + 32 * jj] * alpha;
                const unsigned char* vcell = vs + (size_t)(lc * 32) * S::ROWB;
#pragma unroll 8
                for (int t = 0; t < FSATTN_CELL; t++) {
                    const float pt = __shfl_sync(FS_FULL, p, t);
                    const bf16* vr = reinterpret_cast<const bf16*>(vcell + (size_t)t * S::ROWB);
#pragma unroll
                    for (int jj = 0; jj < DPL; jj++) acc[jj] = fmaf(pt, __bfloat162float(vr[lane + 32 * jj]), acc[jj]);
                }
#pragma unroll
                for (int jj = 0; jj < DPL; jj++) accs[qi * D + lane + 32 * jj] = acc[jj];
                if (lane == 0) mls[qi] = make_float2(m_new, l_new);
                __syncwarp();
            }
        }
        __syncthreads();
    }
    // ---- o -> bf16, lr_norm, combine -------------------------------------------------------------------------------------------------
    const float g = a.lrs[h];
    for (int qi = warp * 16; qi < warp * 16 + 16; qi++) {
        if (q0 + qi >= a.N) break;
        const float l = mls[qi].y;
        float o[DPL], ss = 0.0f;
#pragma unroll
        for (int jj = 0; jj < DPL; jj++) {
            o[jj] = (l > 0.0f) ? bf_round(accs[qi * D + lane + 32 * jj] / l) : 0.0f;
            ss = fmaf(o[jj], o[jj], ss);
        }
        ss = warp_sum(ss);
        const float r = f_div(1.0f, f_sqrt(f_add(ss * (1.0f / D), a.eps)));
        const int64_t row = ((int64_t)b * a.N + q0 + qi) * ((int64_t)a.H * D) + (int64_t)h * D;
        const bf16* srp = (const bf16*)a.sr + row;
        bf16* yp = (bf16*)a.y + row;
#pragma unroll
        for (int jj = 0; jj < DPL; jj++) {
            const int d = lane + 32 * jj;
            const float lr = f_mul(f_mul(o[jj], r), a.norm_w[d]);
            const float sr = (a.sr != nullptr) ? __bfloat162float(srp[d]) : 0.0f;
            yp[d] = __float2bfloat16_rn(f_add(sr, f_mul(g, lr)));
        }
    }
}

template <int D>
int launch_readout_block(const fsattn_readout_combine_t* a, cudaStream_t st) {
    const size_t smem = RbSmem<D>::TOTAL;
    static bool opted[16] = {false};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 16 && !opted[dev]) {
        if (cudaFuncSetAttribute(readout_block_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess) {
            (void)cudaGetLastError();
            fs_set_error("readout_combine: cannot opt in to %zu bytes of shared memory", smem);
            return FSATTN_ELAUNCH;
        }
        opted[dev] = true;
    }
    dim3 grid((a->N + RB_Q - 1) / RB_Q, a->B * a->H);
    readout_block_kernel<D><<<grid, RB_THREADS, smem, st>>>(*a);
    return fs_check_launch("readout_block");
}

}  // namespace

int fs_readout_block(const fsattn_readout_combine_t* a, cudaStream_t st) {
    switch (a->D) {
        case 64: return launch_readout_block<64>(a, st);
        case 96: return launch_readout_block<96>(a, st);
        default: return launch_readout_block<128>(a, st);
    }
}
