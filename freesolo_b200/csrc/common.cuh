// Shared device helpers for the FreeSolo sparse-attention kernels (sm_100a).
#pragma once
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>
#include <math.h>

#include "../../include/fsattn_b200.h"

#define FS_FULL 0xffffffffu
#define FS_NEG_SCORE (-1e9f)

typedef __nv_bfloat16 bf16;

// host-side error reporting (abi.cu)
void fs_set_error(const char* fmt, ...);
int fs_check_launch(const char* what);

#define FS_REQUIRE(cond, ...)                                   \
    do {                                                        \
        if (!(cond)) {                                          \
            fs_set_error(__VA_ARGS__);                          \
            return FSATTN_EINVAL;                               \
        }                                                       \
    } while (0)

#define FS_UNSUPPORTED(cond, ...)                               \
    do {                                                        \
        if (cond) {                                             \
            fs_set_error(__VA_ARGS__);                          \
            return FSATTN_EUNSUPPORTED;                         \
        }                                                       \
    } while (0)

// ---- IEEE arithmetic that the compiler must not contract into FMAs --------------------------------------------
__device__ __forceinline__ float f_add(float a, float b) { return __fadd_rn(a, b); }
__device__ __forceinline__ float f_mul(float a, float b) { return __fmul_rn(a, b); }
__device__ __forceinline__ float f_div(float a, float b) { return __fdiv_rn(a, b); }
__device__ __forceinline__ float f_sqrt(float a) { return __fsqrt_rn(a); }

// ---- bf16 <-> fp32 ---------------------------------------------------------------------------------------------
__device__ __forceinline__ float bf_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf_hi(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }
__device__ __forceinline__ uint32_t f2bf_bits(float f) {
    return (uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(f));
}
__device__ __forceinline__ float bf_round(float f) { return __bfloat162float(__float2bfloat16_rn(f)); }
__device__ __forceinline__ uint32_t pack_bf2(float lo, float hi) {        // one cvt.rn.bf16x2.f32; lo in bits 0..15
    const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<const uint32_t*>(&v);
}

// four consecutive values starting at element e of a row: from int8 codes (one 32-bit word) or bf16 (one 64-bit word)
// Exact int8 -> fp32 without the conversion unit: byte c + 128 placed in the mantissa of 2^23 (one byte permute), minus
// 2^23 + 128 (one exact add) - the integer-to-float instruction runs at a quarter of the rate of these.
__device__ __forceinline__ void unpack4_i8(uint32_t w, float* o) {
    const uint32_t u = w ^ 0x80808080u;
    o[0] = __fadd_rn(__uint_as_float(__byte_perm(u, 0x4B000000u, 0x7440)), -8388736.0f);
    o[1] = __fadd_rn(__uint_as_float(__byte_perm(u, 0x4B000000u, 0x7441)), -8388736.0f);
    o[2] = __fadd_rn(__uint_as_float(__byte_perm(u, 0x4B000000u, 0x7442)), -8388736.0f);
    o[3] = __fadd_rn(__uint_as_float(__byte_perm(u, 0x4B000000u, 0x7443)), -8388736.0f);
}
__device__ __forceinline__ void unpack4_bf(uint2 w, float* o) {
    o[0] = bf_lo(w.x); o[1] = bf_hi(w.x); o[2] = bf_lo(w.y); o[3] = bf_hi(w.y);
}

// ---- warp reductions -------------------------------------------------------------------------------------------
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(FS_FULL, v, o));
    return v;
}
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(FS_FULL, v, o);
    return v;
}

// ---- (max, sum, acc) softmax partial merge -----------------------------------------------------------------------
// A partial is the running max m, the sum l of exp(score - m) and acc = sum exp(score - m) * v. m = -inf means empty.
__device__ __forceinline__ void softmax_merge_scalars(float m_a, float m_b, float& m, float& fa, float& fb) {
    m = fmaxf(m_a, m_b);
    fa = (m_a == -INFINITY) ? 0.0f : __expf(m_a - m);
    fb = (m_b == -INFINITY) ? 0.0f : __expf(m_b - m);
}

// the selection prior lam * ceil * erf(|p - (c + 0.5) s| / (2 sigma)) with the reference's operation order
__device__ __forceinline__ float fs_prior(float lam, float ceil_c, float qpos, int cell, float s, float two_sigma) {
    const float cen = f_mul((float)cell + 0.5f, s);
    const float dist = fabsf(qpos - cen);
    return f_mul(f_mul(lam, ceil_c), erff(f_div(dist, two_sigma)));
}

// order of the top-P pool: ceiling descending, then cell index ascending
__device__ __forceinline__ bool pool_before(float ca, int ia, float cb, int ib) {
    return ca > cb || (ca == cb && ia < ib);
}
