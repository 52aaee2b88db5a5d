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

extern "C" int fsattn_readout_combine(const fsattn_readout_combine_t* a, fsattn_stream_t stream) {
    FS_REQUIRE(a != nullptr && a->q.ptr && a->k.ptr && a->v.ptr && a->sel && a->y && a->norm_w && a->lrs,
               "readout_combine: null pointer");
    FS_REQUIRE(a->B > 0 && a->H > 0 && a->N > 0 && a->n_kv > 0 && a->Bq > 0, "readout_combine: bad sizes");
    FS_REQUIRE(a->kk >= 1 && a->kk <= FSATTN_MAX_KK, "readout_combine: kk %d not in [1,%d]", a->kk, FSATTN_MAX_KK);
    FS_UNSUPPORTED(a->D != 64 && a->D != 96 && a->D != 128, "readout_combine: head_dim %d not in {64,96,128}", a->D);
    FS_REQUIRE(((uintptr_t)a->q.ptr & 15) == 0 && a->q.sn % 8 == 0 && a->q.sh % 8 == 0 && a->q.sb % 8 == 0 &&
               ((uintptr_t)a->k.ptr & 15) == 0 && a->k.sn % 8 == 0 && a->k.sh % 8 == 0 && a->k.sb % 8 == 0,
               "readout_combine: Q and K rows must be 16-byte aligned");
    dim3 grid((a->N + 7) / 8, a->B * a->H);
    cudaStream_t st = (cudaStream_t)stream;
    switch (a->D) {
        case 64: readout_combine_kernel<64><<<grid, 256, 0, st>>>(*a); break;
        case 96: readout_combine_kernel<96><<<grid, 256, 0, st>>>(*a); break;
        default: readout_combine_kernel<128><<<grid, 256, 0, st>>>(*a); break;
    }
    return fs_check_launch("readout_combine");
}
