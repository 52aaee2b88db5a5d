// RMSNorm over the rows of a (M, d) bf16 matrix: out = x * rsqrt(mean(x^2) + eps) * w, computed in fp32 and rounded once,
// as the framework's fused kernel does. One warp per row; the row is read once (16-byte loads, up to 8 chunks per lane
// held in registers, i.e. d <= 2048; longer rows are re-read for the second pass) and written once: 4 d bytes per row.
#include "common.cuh"

namespace {

constexpr int RN_WARPS = 8;
constexpr int RN_KC = 8;

__global__ void __launch_bounds__(RN_WARPS * 32) rms_norm_kernel(const bf16* __restrict__ x, int64_t x_stride,
                                                                 const bf16* __restrict__ w, float eps, bf16* __restrict__ out,
                                                                 int64_t out_stride, int64_t M, int d) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int kchunks = d / 8;
    for (int64_t m = (int64_t)blockIdx.x * RN_WARPS + warp; m < M; m += (int64_t)gridDim.x * RN_WARPS) {
        const uint4* xr = reinterpret_cast<const uint4*>(x + m * x_stride);
        uint4* orow = reinterpret_cast<uint4*>(out + m * out_stride);
        uint4 v[RN_KC];
        float ss = 0.f;
#pragma unroll
        for (int j = 0; j < RN_KC; j++) {
            const int c = lane + 32 * j;
            v[j] = (c < kchunks) ? __ldcs(xr + c) : make_uint4(0u, 0u, 0u, 0u);
        }
#pragma unroll
        for (int j = 0; j < RN_KC; j++) {
            const uint32_t ws[4] = {v[j].x, v[j].y, v[j].z, v[j].w};
#pragma unroll
            for (int k = 0; k < 4; k++) {
                const float a = bf_lo(ws[k]), b = bf_hi(ws[k]);
                ss = fmaf(a, a, ss);
                ss = fmaf(b, b, ss);
            }
        }
        for (int c = lane + 32 * RN_KC; c < kchunks; c += 32) {          // rows longer than the register window
            const uint4 t = xr[c];
            const uint32_t ws[4] = {t.x, t.y, t.z, t.w};
#pragma unroll
            for (int k = 0; k < 4; k++) {
                const float a = bf_lo(ws[k]), b = bf_hi(ws[k]);
                ss = fmaf(a, a, ss);
                ss = fmaf(b, b, ss);
            }
        }
        ss = warp_sum(ss);
        const float rinv = rsqrtf(ss / (float)d + eps);
        auto scale8 = [&](const uint4& t, int c) {
            const uint4 g = *reinterpret_cast<const uint4*>(w + c * 8);
            const uint32_t ws[4] = {t.x, t.y, t.z, t.w}, gs[4] = {g.x, g.y, g.z, g.w};
            uint32_t o[4];
#pragma unroll
            for (int k = 0; k < 4; k++)
                o[k] = pack_bf2(bf_lo(ws[k]) * rinv * bf_lo(gs[k]), bf_hi(ws[k]) * rinv * bf_hi(gs[k]));
            return make_uint4(o[0], o[1], o[2], o[3]);
        };
#pragma unroll
        for (int j = 0; j < RN_KC; j++) {
            const int c = lane + 32 * j;
            if (c < kchunks) orow[c] = scale8(v[j], c);
        }
        for (int c = lane + 32 * RN_KC; c < kchunks; c += 32) orow[c] = scale8(xr[c], c);
    }
}

}  // namespace

extern "C" int fsattn_rms_norm(const void* x, int64_t x_stride, const void* w, float eps, void* out, int64_t out_stride, int64_t M,
                               int32_t d, fsattn_stream_t stream) {
    FS_REQUIRE(x != nullptr && w != nullptr && out != nullptr && M >= 0 && d >= 8, "rms_norm: null pointer or bad sizes");
    FS_REQUIRE(d % 8 == 0 && x_stride % 8 == 0 && out_stride % 8 == 0 && ((uintptr_t)x & 15) == 0 && ((uintptr_t)out & 15) == 0 &&
                   ((uintptr_t)w & 15) == 0,
               "rms_norm: rows and the weight must be 16-byte aligned and d a multiple of 8");
    if (M == 0) return FSATTN_OK;
    const int64_t blocks = (M + RN_WARPS - 1) / RN_WARPS;
    const int grid = (int)(blocks < 148 * 8 ? blocks : 148 * 8);
    rms_norm_kernel<<<grid, RN_WARPS * 32, 0, (cudaStream_t)stream>>>((const bf16*)x, x_stride, (const bf16*)w, eps, (bf16*)out,
                                                                      out_stride, M, d);
    return fs_check_launch("rms_norm_kernel");
}
