// Row-streaming pieces shared by the decode-step projection kernels: a warp holds one weight row in registers (16-byte
// chunks, lane-interleaved), dots it with <= 8 activation rows staged in shared memory, and reduces with shuffles.
#pragma once
#include "common.cuh"

namespace {

#ifndef FS_GEMV_THREADS
#define FS_GEMV_THREADS 256
#endif
constexpr int GEMV_THREADS = FS_GEMV_THREADS;
constexpr int GEMV_WARPS = GEMV_THREADS / 32;

__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

template <int KC>
struct RowRegs {
    uint4 w[KC];
};

template <int KC>
__device__ __forceinline__ void load_row(RowRegs<KC>& r, const bf16* row, int lane, int kchunks) {
#pragma unroll
    for (int j = 0; j < KC; j++) {
        const int c = lane + 32 * j;
        r.w[j] = (row != nullptr && c < kchunks) ? __ldg(reinterpret_cast<const uint4*>(row) + c) : make_uint4(0u, 0u, 0u, 0u);
    }
}

template <int KC, int M>
__device__ __forceinline__ void dot_row(const RowRegs<KC>& r, const uint4* xs, int kchunks, int lane, float* acc) {
#pragma unroll
    for (int m = 0; m < M; m++) acc[m] = 0.0f;
#pragma unroll
    for (int j = 0; j < KC; j++) {
        const int c = lane + 32 * j;
        if (c < kchunks) {
            const uint4 w = r.w[j];
            const float w0 = bf_lo(w.x), w1 = bf_hi(w.x), w2 = bf_lo(w.y), w3 = bf_hi(w.y);
            const float w4 = bf_lo(w.z), w5 = bf_hi(w.z), w6 = bf_lo(w.w), w7 = bf_hi(w.w);
#pragma unroll
            for (int m = 0; m < M; m++) {
                const uint4 x = xs[m * kchunks + c];
                float a = acc[m];
                a = fmaf(w0, bf_lo(x.x), a); a = fmaf(w1, bf_hi(x.x), a);
                a = fmaf(w2, bf_lo(x.y), a); a = fmaf(w3, bf_hi(x.y), a);
                a = fmaf(w4, bf_lo(x.z), a); a = fmaf(w5, bf_hi(x.z), a);
                a = fmaf(w6, bf_lo(x.w), a); a = fmaf(w7, bf_hi(x.w), a);
                acc[m] = a;
            }
        }
    }
#pragma unroll
    for (int m = 0; m < M; m++) acc[m] = warp_sum(acc[m]);
}

}  // namespace
