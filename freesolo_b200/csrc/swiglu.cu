// Elementwise SwiGLU gate of the prefill trunk: out[m, j] = silu(gu[m, j]) * gu[m, f + j] for the fused gate/up projection
// gu (M, 2f) bf16. One pass over the data (read 2f, write f per row) instead of the two elementwise kernels and the
// intermediate a framework runs; roundings are the same as theirs: silu in fp32 rounded to bf16, then the product rounded.
#include "common.cuh"

namespace {

__device__ __forceinline__ uint4 swiglu8(const uint4& g, const uint4& u) {
    const uint32_t gw[4] = {g.x, g.y, g.z, g.w}, uw[4] = {u.x, u.y, u.z, u.w};
    uint32_t ow[4];
#pragma unroll
    for (int k = 0; k < 4; k++) {
        const float g0 = bf_lo(gw[k]), g1 = bf_hi(gw[k]);
        const float s0 = bf_round(g0 / (1.0f + __expf(-g0))), s1 = bf_round(g1 / (1.0f + __expf(-g1)));
        ow[k] = pack_bf2(s0 * bf_lo(uw[k]), s1 * bf_hi(uw[k]));
    }
    return make_uint4(ow[0], ow[1], ow[2], ow[3]);
}

// two 16-byte chunks per thread and iteration, so that four loads are in flight before the first use
__global__ void __launch_bounds__(256) swiglu_kernel(const uint4* __restrict__ gu, uint4* __restrict__ out, int64_t M, int f8,
                                                     int64_t gu_stride8, int64_t out_stride8) {
    const int64_t total = M * f8;
    const int64_t step = (int64_t)gridDim.x * blockDim.x;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += 2 * step) {
        const int64_t i2 = i + step;
        const bool two = i2 < total;
        const int64_t m = i / f8, m2 = two ? i2 / f8 : m;
        const int j = (int)(i - m * f8), j2 = two ? (int)(i2 - m2 * f8) : j;
        const uint4 g = __ldcs(gu + m * gu_stride8 + j);
        const uint4 u = __ldcs(gu + m * gu_stride8 + f8 + j);
        const uint4 g2 = __ldcs(gu + m2 * gu_stride8 + j2);
        const uint4 u2 = __ldcs(gu + m2 * gu_stride8 + f8 + j2);
        out[m * out_stride8 + j] = swiglu8(g, u);
        if (two) out[m2 * out_stride8 + j2] = swiglu8(g2, u2);
    }
}

}  // namespace

extern "C" int fsattn_swiglu(const void* gu, int64_t gu_stride, void* out, int64_t out_stride, int64_t M, int32_t f,
                             fsattn_stream_t stream) {
    FS_REQUIRE(gu != nullptr && out != nullptr && M >= 0 && f > 0, "swiglu: null pointer or bad sizes");
    FS_REQUIRE(f % 8 == 0 && gu_stride % 8 == 0 && out_stride % 8 == 0 && ((uintptr_t)gu & 15) == 0 && ((uintptr_t)out & 15) == 0,
               "swiglu: rows must be 16-byte aligned and f a multiple of 8");
    if (M == 0) return FSATTN_OK;
    const int64_t total = M * (f / 8);
    const int grid = (int)min((int64_t)148 * 16, (total + 255) / 256);
    swiglu_kernel<<<grid, 256, 0, (cudaStream_t)stream>>>((const uint4*)gu, (uint4*)out, M, f / 8, gu_stride / 8, out_stride / 8);
    return fs_check_launch("swiglu_kernel");
}
