// Warp-level routines over one cell (32 tokens x D bf16): load, statistics, int8 quantisation.
// Shared by the prefill ingest kernel and the decode step's cell close.
//
// Register layout: LPR lanes per token row (8 for D = 64, 16 otherwise), each lane one 16-byte chunk of 8 dims;
// a warp instruction covers RPI = 32 / LPR rows and NIT = 32 / RPI iterations cover the cell:
//     row(i, lane) = i * RPI + lane / LPR,   dims(lane) = 8 * (lane % LPR) .. + 8
#pragma once
#include "common.cuh"

template <int D>
struct CellRegs {
    static constexpr int LPR = (D == 64) ? 8 : 16;
    static constexpr int RPI = 32 / LPR;
    static constexpr int NIT = 32 / RPI;
    static constexpr int CH = D / 8;
    uint4 w[NIT];
};

// rows of the cell at base + row * sn; when row31 != nullptr it replaces the last row (the token being appended)
template <int D>
__device__ __forceinline__ void cell_load_rows(CellRegs<D>& r, const bf16* base, int64_t sn, int lane,
                                               const bf16* row31 = nullptr) {
    using R = CellRegs<D>;
    const int chunk = lane % R::LPR;
    const int r0 = lane / R::LPR;
#pragma unroll
    for (int i = 0; i < R::NIT; i++) {
        const int row = i * R::RPI + r0;
        uint4 v = make_uint4(0u, 0u, 0u, 0u);
        if (chunk < R::CH) {
            const bf16* p = (row31 != nullptr && row == 31) ? row31 : base + (int64_t)row * sn;
            v = *reinterpret_cast<const uint4*>(p + chunk * 8);
        }
        r.w[i] = v;
    }
}

__device__ __forceinline__ void chunk_floats(const uint4& w, float* x) {
    x[0] = bf_lo(w.x); x[1] = bf_hi(w.x); x[2] = bf_lo(w.y); x[3] = bf_hi(w.y);
    x[4] = bf_lo(w.z); x[5] = bf_hi(w.z); x[6] = bf_lo(w.w); x[7] = bf_hi(w.w);
}

// Chunk-mean key and ceiling. The arithmetic order is fixed (no FMA contraction):
//   norm of a token: squares, dims l and l + D/2 ... summed by an adjacent pairwise tree, sqrt.rn; ceiling = max;
//   mean: token t goes to accumulator t % 4 in token order, ((a0 + a1) + a2) + a3, times 1/32, rounded to bf16.
// For D = 64 this is the order of torch's CUDA reductions, which the reference's own statistics kernel replays.
template <int D>
__device__ __forceinline__ void cell_stats_warp(const CellRegs<D>& r, int lane, float* kbar_out, float* ceil_out) {
    using R = CellRegs<D>;
    const int chunk = lane % R::LPR;
    const int r0 = lane / R::LPR;
    float acc_e[8], acc_o[8];
#pragma unroll
    for (int j = 0; j < 8; j++) { acc_e[j] = 0.0f; acc_o[j] = 0.0f; }
    float mx = 0.0f;
#pragma unroll
    for (int i = 0; i < R::NIT; i++) {
        float x[8];
        chunk_floats(r.w[i], x);
        float v[8];
#pragma unroll
        for (int j = 0; j < 8; j++) v[j] = f_mul(x[j], x[j]);
        if (D == 64) {
#pragma unroll
            for (int j = 0; j < 8; j++) v[j] = f_add(v[j], __shfl_xor_sync(FS_FULL, v[j], 4));
        }
        float t = f_add(f_add(f_add(v[0], v[1]), f_add(v[2], v[3])), f_add(f_add(v[4], v[5]), f_add(v[6], v[7])));
        if (D == 64) {
            t = f_add(t, __shfl_xor_sync(FS_FULL, t, 1));
            t = f_add(t, __shfl_xor_sync(FS_FULL, t, 2));
        } else {
            t = f_add(t, __shfl_xor_sync(FS_FULL, t, 1));
            t = f_add(t, __shfl_xor_sync(FS_FULL, t, 2));
            t = f_add(t, __shfl_xor_sync(FS_FULL, t, 4));
            t = f_add(t, __shfl_xor_sync(FS_FULL, t, 8));
        }
        mx = fmaxf(mx, f_sqrt(t));
        if (R::RPI == 4 || (i & 1) == 0) {
#pragma unroll
            for (int j = 0; j < 8; j++) acc_e[j] = f_add(acc_e[j], x[j]);
        } else {
#pragma unroll
            for (int j = 0; j < 8; j++) acc_o[j] = f_add(acc_o[j], x[j]);
        }
    }
    // ceiling: max over the row groups of the warp
#pragma unroll
    for (int o = R::LPR; o < 32; o <<= 1) mx = fmaxf(mx, __shfl_xor_sync(FS_FULL, mx, o));
    if (ceil_out != nullptr && lane == 0) *ceil_out = mx;
    // mean
    float m[8];
#pragma unroll
    for (int j = 0; j < 8; j++) {
        float s;
        if (R::RPI == 4) {
            const float a1 = __shfl_down_sync(FS_FULL, acc_e[j], 8);
            const float a2 = __shfl_down_sync(FS_FULL, acc_e[j], 16);
            const float a3 = __shfl_down_sync(FS_FULL, acc_e[j], 24);
            s = f_add(f_add(f_add(acc_e[j], a1), a2), a3);
        } else {
            const float a1 = __shfl_down_sync(FS_FULL, acc_e[j], 16);
            const float a3 = __shfl_down_sync(FS_FULL, acc_o[j], 16);
            s = f_add(f_add(f_add(acc_e[j], a1), acc_o[j]), a3);
        }
        m[j] = bf_round(f_mul(s, 0.03125f));
    }
    if (kbar_out != nullptr && r0 == 0 && chunk < R::CH) {
        float4* o = reinterpret_cast<float4*>(kbar_out + chunk * 8);
        o[0] = make_float4(m[0], m[1], m[2], m[3]);
        o[1] = make_float4(m[4], m[5], m[6], m[7]);
    }
}

// scale = bf16(max|x| / 127) (1.0 for an all-zero cell); q = rint(x / scale), both divisions IEEE.
// q_out: 32 rows of D codes, contiguous; sc_out: one bf16.
template <int D>
__device__ __forceinline__ void cell_quant_warp(const CellRegs<D>& r, int lane, int8_t* q_out, bf16* sc_out) {
    using R = CellRegs<D>;
    const int chunk = lane % R::LPR;
    const int r0 = lane / R::LPR;
    float amax = 0.0f;
#pragma unroll
    for (int i = 0; i < R::NIT; i++) {
        float x[8];
        chunk_floats(r.w[i], x);
#pragma unroll
        for (int j = 0; j < 8; j++) amax = fmaxf(amax, fabsf(x[j]));
    }
    amax = warp_max(amax);
    const float sc = (amax > 0.0f) ? bf_round(f_div(amax, 127.0f)) : 1.0f;
    if (lane == 0) *sc_out = __float2bfloat16_rn(sc);
#pragma unroll
    for (int i = 0; i < R::NIT; i++) {
        float x[8];
        chunk_floats(r.w[i], x);
        uint32_t b[8];
#pragma unroll
        for (int j = 0; j < 8; j++) b[j] = (uint32_t)(__float2int_rn(f_div(x[j], sc)) & 0xff);
        uint2 o;
        o.x = b[0] | (b[1] << 8) | (b[2] << 16) | (b[3] << 24);
        o.y = b[4] | (b[5] << 8) | (b[6] << 16) | (b[7] << 24);
        if (chunk < R::CH) {
            const int row = i * R::RPI + r0;
            *reinterpret_cast<uint2*>(q_out + (int64_t)row * D + chunk * 8) = o;
        }
    }
}
