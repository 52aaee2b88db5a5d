// The two ends of a greedy decode step as one small kernel each, so that a step is nothing but this library's launches:
//   embed_rows_kernel      x[b, :] = table[tok[b], :]                       (torch: embedding gather + copy)
//   argmax_advance_kernel  tok[b] = argmax_v logits[b, v] (lowest index on ties, as torch.argmax), *pos += 1
//                          (torch: argmax, copy, add)
// Both wait for their producer themselves (programmatic dependent launch), like every other kernel of the step.
#include "common.cuh"

namespace {

__global__ void __launch_bounds__(128) embed_rows_kernel(const int64_t* __restrict__ tok, const uint4* __restrict__ table, uint4* __restrict__ x,
                                                         int d8, int64_t vocab) {
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    int64_t t = tok[blockIdx.x];
    if (t < 0 || t >= vocab) t = 0;                      // an id outside the table reads row 0 instead of faulting
    for (int i = threadIdx.x; i < d8; i += blockDim.x) x[(int64_t)blockIdx.x * d8 + i] = table[t * d8 + i];
}

__global__ void __launch_bounds__(1024) argmax_advance_kernel(const bf16* __restrict__ logits, int64_t stride, int V, int64_t* __restrict__ tok,
                                                              int64_t* pos) {
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    const bf16* row = logits + (int64_t)blockIdx.x * stride;
    float best = -INFINITY;
    int bi = 0x7fffffff;
    // 16-byte chunks, two in flight per thread (rows that are not 16-byte aligned are read element by element)
    const int nv = (stride % 8 == 0 && (reinterpret_cast<uintptr_t>(logits) & 15) == 0) ? V / 8 : 0;
    const uint4* r4 = reinterpret_cast<const uint4*>(row);
    for (int c = threadIdx.x; c < nv; c += 2 * blockDim.x) {
        const int c2 = c + blockDim.x;
        const uint4 a = r4[c];
        const uint4 b = c2 < nv ? r4[c2] : make_uint4(0xff80ff80u, 0xff80ff80u, 0xff80ff80u, 0xff80ff80u);      // -inf pairs
        const uint32_t wa[4] = {a.x, a.y, a.z, a.w}, wb[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
        for (int k = 0; k < 4; k++) {
            const float v0 = bf_lo(wa[k]), v1 = bf_hi(wa[k]);
            if (v0 > best) { best = v0; bi = c * 8 + 2 * k; }
            if (v1 > best) { best = v1; bi = c * 8 + 2 * k + 1; }
        }
#pragma unroll
        for (int k = 0; k < 4; k++) {
            const float v0 = bf_lo(wb[k]), v1 = bf_hi(wb[k]);
            if (v0 > best) { best = v0; bi = c2 * 8 + 2 * k; }
            if (v1 > best) { best = v1; bi = c2 * 8 + 2 * k + 1; }
        }
    }
    for (int v = nv * 8 + threadIdx.x; v < V; v += blockDim.x) {
        const float x = __bfloat162float(row[v]);
        if (x > best || (x == best && v < bi)) { best = x; bi = v; }
    }
    // (value desc, index asc) over the block
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ob = __shfl_xor_sync(FS_FULL, best, o);
        const int oi = __shfl_xor_sync(FS_FULL, bi, o);
        if (ob > best || (ob == best && oi < bi)) { best = ob; bi = oi; }
    }
    __shared__ float sb[32];
    __shared__ int si[32];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    if (lane == 0) { sb[warp] = best; si[warp] = bi; }
    __syncthreads();
    if (warp == 0) {
        best = lane < nw ? sb[lane] : -INFINITY;
        bi = lane < nw ? si[lane] : 0x7fffffff;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ob = __shfl_xor_sync(FS_FULL, best, o);
            const int oi = __shfl_xor_sync(FS_FULL, bi, o);
            if (ob > best || (ob == best && oi < bi)) { best = ob; bi = oi; }
        }
        if (lane == 0) {
            tok[blockIdx.x] = bi == 0x7fffffff ? 0 : bi;
            if (pos != nullptr && blockIdx.x == 0) *pos += 1;
        }
    }
}

template <typename... Args>
cudaError_t launch_pdl(void (*kernel)(Args...), dim3 grid, dim3 block, cudaStream_t st, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, args...);
}

}  // namespace

extern "C" int fsattn_embed_rows(const int64_t* tok, const void* table, void* x, int32_t B, int32_t d, int64_t vocab, fsattn_stream_t stream) {
    FS_REQUIRE(tok && table && x && B > 0 && d > 0 && vocab > 0, "embed_rows: null pointer or bad sizes");
    FS_REQUIRE(d % 8 == 0 && ((uintptr_t)table & 15) == 0 && ((uintptr_t)x & 15) == 0, "embed_rows: rows must be 16-byte aligned");
    const cudaError_t e = launch_pdl(embed_rows_kernel, dim3(B), dim3(128), (cudaStream_t)stream, tok, (const uint4*)table, (uint4*)x, d / 8, vocab);
    if (e != cudaSuccess) {
        (void)cudaGetLastError();
        fs_set_error("embed_rows: launch failed: %s", cudaGetErrorString(e));
        return FSATTN_ELAUNCH;
    }
    return FSATTN_OK;
}

extern "C" int fsattn_argmax_advance(const void* logits, int64_t stride, int32_t B, int32_t V, int64_t* tok, int64_t* pos,
                                     fsattn_stream_t stream) {
    FS_REQUIRE(logits && tok && B > 0 && V > 0 && stride >= V, "argmax_advance: null pointer or bad sizes");
    const cudaError_t e = launch_pdl(argmax_advance_kernel, dim3(B), dim3(1024), (cudaStream_t)stream, (const bf16*)logits, stride, (int)V, tok, pos);
    if (e != cudaSuccess) {
        (void)cudaGetLastError();
        fs_set_error("argmax_advance: launch failed: %s", cudaGetErrorString(e));
        return FSATTN_ELAUNCH;
    }
    return FSATTN_OK;
}
