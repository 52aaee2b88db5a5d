// Decode step, everything of a layer after its attention in ONE launch: x += W_o y; act = SwiGLU(W_gu rmsnorm(x));
// x += W_down act; next = W_next rmsnorm'(x) (the next layer's QKV projection, or the LM head after the last layer).
//
// At batch <= 8 each of these projections streams 2-11 MB of weights, one or two microseconds of HBM time, so a chain of
// separate launches is bound by the launch-to-launch dependency latency, not by bandwidth. Here one CTA per SM stays
// resident through the four phases; a phase is the row-streaming GEMV of trunk_gemv.cu (one warp per output row, the
// weight row in registers), and the phases are separated by a grid-wide barrier (an arrival counter in global memory).
// Every warp fetches the first weight row of the NEXT phase before it arrives at the barrier, so weight streaming
// continues while the barrier settles. The kernel is launched cooperatively (all CTAs co-resident, which the barrier
// needs) and every wait is bounded: a barrier that does not complete sets *status and the kernel runs on to its end.
//
// Measured on a B200 (341M model, batch 1): 0.79 ms per step against 0.63 ms for the five-launch chain, i.e. a barrier
// (arrive, poll, fence) plus re-reading the activations through L2 is no cheaper than a dependent launch whose prologue
// already overlaps its producer; the callers therefore keep the separate launches by default and this kernel is opt-in.
//
// Arithmetic and rounding are those of the separate kernels (same per-row reduction order), so the fused step is
// bit-identical to the five-launch step.
#include "trunk_rows.cuh"

namespace {

constexpr int TL_SPIN_LIMIT = 1 << 21;      // ~1 s of polling before a barrier gives up

__device__ __forceinline__ int tl_ld_acquire(const int* p) {
    int v;
    asm volatile("ld.acquire.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void tl_grid_barrier(int* cnt, int nblocks, int* status) {
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        atomicAdd(cnt, 1);
        int spins = 0;
        while (tl_ld_acquire(cnt) < nblocks) {
            if (++spins > TL_SPIN_LIMIT) {
                atomicExch(status, 1);
                break;
            }
        }
        __threadfence();
    }
    __syncthreads();
}

__device__ __forceinline__ uint4 tl_ldcg(const bf16* p) { return __ldcg(reinterpret_cast<const uint4*>(p)); }

// rows of X (written by other SMs earlier in this launch: read through L2) -> shared memory, RMS-normalised when NW != nullptr
template <int M>
__device__ void tl_stage(uint4* xs, const bf16* X, int64_t x_stride, int rows, int K, const bf16* NW, float eps,
                         float (*red)[M]) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int kchunks = K / 8;
    const uint4 zero = make_uint4(0u, 0u, 0u, 0u);
    if (NW != nullptr) {
        float ss[M];
#pragma unroll
        for (int m = 0; m < M; m++) ss[m] = 0.0f;
        for (int c = tid; c < kchunks; c += GEMV_THREADS) {
#pragma unroll
            for (int m = 0; m < M; m++) {
                const uint4 x = (m < rows) ? tl_ldcg(X + (int64_t)m * x_stride + c * 8) : zero;
                float v[8] = {bf_lo(x.x), bf_hi(x.x), bf_lo(x.y), bf_hi(x.y), bf_lo(x.z), bf_hi(x.z), bf_lo(x.w), bf_hi(x.w)};
#pragma unroll
                for (int j = 0; j < 8; j++) ss[m] = fmaf(v[j], v[j], ss[m]);
            }
        }
#pragma unroll
        for (int m = 0; m < M; m++) {
            const float s = warp_sum(ss[m]);
            if (lane == 0) red[warp][m] = s;
        }
        __syncthreads();
        float rinv[M];
#pragma unroll
        for (int m = 0; m < M; m++) {
            float s = 0.0f;
#pragma unroll
            for (int w = 0; w < GEMV_WARPS; w++) s += red[w][m];
            rinv[m] = rsqrtf(s / (float)K + eps);
        }
        for (int c = tid; c < kchunks; c += GEMV_THREADS) {
            const uint4 nw = *reinterpret_cast<const uint4*>(NW + c * 8);
            const float g[8] = {bf_lo(nw.x), bf_hi(nw.x), bf_lo(nw.y), bf_hi(nw.y), bf_lo(nw.z), bf_hi(nw.z), bf_lo(nw.w), bf_hi(nw.w)};
#pragma unroll
            for (int m = 0; m < M; m++) {
                const uint4 x = (m < rows) ? tl_ldcg(X + (int64_t)m * x_stride + c * 8) : zero;
                const float v[8] = {bf_lo(x.x), bf_hi(x.x), bf_lo(x.y), bf_hi(x.y), bf_lo(x.z), bf_hi(x.z), bf_lo(x.w), bf_hi(x.w)};
                uint4 o;
                o.x = pack_bf2(v[0] * rinv[m] * g[0], v[1] * rinv[m] * g[1]);
                o.y = pack_bf2(v[2] * rinv[m] * g[2], v[3] * rinv[m] * g[3]);
                o.z = pack_bf2(v[4] * rinv[m] * g[4], v[5] * rinv[m] * g[5]);
                o.w = pack_bf2(v[6] * rinv[m] * g[6], v[7] * rinv[m] * g[7]);
                xs[m * kchunks + c] = o;
            }
        }
    } else {
        for (int c = tid; c < kchunks; c += GEMV_THREADS) {
#pragma unroll
            for (int m = 0; m < M; m++) xs[m * kchunks + c] = (m < rows) ? tl_ldcg(X + (int64_t)m * x_stride + c * 8) : zero;
        }
    }
    __syncthreads();
}

// first unit of a phase into registers, the next three into L2
template <int KC, bool SW>
__device__ __forceinline__ void tl_preload(RowRegs<KC>& r0, RowRegs<KC>& r1, const bf16* W, int K, int nunits, int u, int nwarps,
                                           int lane) {
    const int kchunks = K / 8;
    load_row<KC>(r0, u < nunits ? W + (int64_t)u * K : nullptr, lane, kchunks);
    if (SW) load_row<KC>(r1, u < nunits ? W + (int64_t)(u + nunits) * K : nullptr, lane, kchunks);
    const int row_bytes = K * 2;
    int pu = u + nwarps;
    for (int n = 0; n < 3 && pu < nunits; n++, pu += nwarps) {
        const char* p0 = reinterpret_cast<const char*>(W + (int64_t)pu * K);
        for (int off = lane * 128; off < row_bytes; off += 32 * 128) {
            asm volatile("prefetch.global.L2 [%0];" ::"l"(p0 + off));
            if (SW) asm volatile("prefetch.global.L2 [%0];" ::"l"(p0 + (int64_t)nunits * row_bytes + off));
        }
    }
}

enum { TL_STORE = 0, TL_RESIDUAL = 1, TL_SWIGLU = 2 };

// the rows of one phase; r0 (and r1) hold unit u's weights on entry
template <int KC, int M, int EPI>
__device__ __forceinline__ void tl_phase(RowRegs<KC>& r0, RowRegs<KC>& r1, const bf16* W, int K, int nunits, int u, int nwarps,
                                         const uint4* xs, int lane, bf16* OUT, int64_t out_stride, int rows) {
    constexpr bool SW = EPI == TL_SWIGLU;
    const int kchunks = K / 8;
    for (; u < nunits; u += nwarps) {
        const int un = u + nwarps;
        RowRegs<KC> n0, n1;
        load_row<KC>(n0, un < nunits ? W + (int64_t)un * K : nullptr, lane, kchunks);
        if (SW) load_row<KC>(n1, un < nunits ? W + (int64_t)(un + nunits) * K : nullptr, lane, kchunks);
        float acc[M], acc2[M];
        dot_row<KC, M>(r0, xs, kchunks, lane, acc);
        if (SW) dot_row<KC, M>(r1, xs, kchunks, lane, acc2);
        if (lane == 0) {
#pragma unroll
            for (int m = 0; m < M; m++) {
                if (m >= rows) continue;
                bf16* o = OUT + (int64_t)m * out_stride + u;
                float v;
                if (EPI == TL_SWIGLU) {
                    const float g = bf_round(acc[m]), up = bf_round(acc2[m]);
                    const float s = bf_round(g / (1.0f + __expf(-g)));
                    v = s * up;
                } else if (EPI == TL_RESIDUAL) {
                    v = __bfloat162float(__ldcg(o)) + bf_round(acc[m]);
                } else {
                    v = acc[m];
                }
                *o = __float2bfloat16_rn(v);
            }
        }
        r0 = n0;
        if (SW) r1 = n1;
    }
}

template <int KCD, int KCF, int M>
__global__ void __launch_bounds__(GEMV_THREADS) trunk_layer_kernel(const fsattn_trunk_layer_t a) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    uint4* xs = reinterpret_cast<uint4*>(smem_raw);                  // M rows of max(d, f) bf16
    __shared__ float red[GEMV_WARPS][M];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int nwarps = gridDim.x * GEMV_WARPS;
    const int gw = blockIdx.x * GEMV_WARPS + warp;
    const int d = a.d, f = a.f, rows = a.M;
    bf16* X = (bf16*)a.x;

    RowRegs<KCD> p0, p1;
    RowRegs<KCF> q0, q1;
    // ---- x += W_o y ----
    tl_preload<KCD, false>(p0, p1, (const bf16*)a.w_o, d, d, gw, nwarps, lane);
    pdl_wait();
    pdl_launch_dependents();
    tl_stage<M>(xs, (const bf16*)a.y, a.y_stride, rows, d, nullptr, 0.f, red);
    tl_phase<KCD, M, TL_RESIDUAL>(p0, p1, (const bf16*)a.w_o, d, d, gw, nwarps, xs, lane, X, a.x_stride, rows);
    // ---- act = silu(gate) * up of W_gu rmsnorm(x) ----
    tl_preload<KCD, true>(p0, p1, (const bf16*)a.w_gu, d, f, gw, nwarps, lane);
    tl_grid_barrier(a.bar + 0, gridDim.x, a.status);
    tl_stage<M>(xs, X, a.x_stride, rows, d, (const bf16*)a.norm2_w, a.eps2, red);
    tl_phase<KCD, M, TL_SWIGLU>(p0, p1, (const bf16*)a.w_gu, d, f, gw, nwarps, xs, lane, (bf16*)a.act, a.act_stride, rows);
    // ---- x += W_down act ----
    tl_preload<KCF, false>(q0, q1, (const bf16*)a.w_down, f, d, gw, nwarps, lane);
    tl_grid_barrier(a.bar + 1, gridDim.x, a.status);
    tl_stage<M>(xs, (const bf16*)a.act, a.act_stride, rows, f, nullptr, 0.f, red);
    tl_phase<KCF, M, TL_RESIDUAL>(q0, q1, (const bf16*)a.w_down, f, d, gw, nwarps, xs, lane, X, a.x_stride, rows);
    // ---- next = W_next rmsnorm'(x) ----
    if (a.w_next != nullptr) {
        tl_preload<KCD, false>(p0, p1, (const bf16*)a.w_next, d, a.n_next, gw, nwarps, lane);
        tl_grid_barrier(a.bar + 2, gridDim.x, a.status);
        tl_stage<M>(xs, X, a.x_stride, rows, d, (const bf16*)a.norm_next_w, a.eps_next, red);
        tl_phase<KCD, M, TL_STORE>(p0, p1, (const bf16*)a.w_next, d, a.n_next, gw, nwarps, xs, lane, (bf16*)a.out_next,
                                   a.out_next_stride, rows);
    }
}

template <int KCD, int KCF, int M>
int launch_layer(const fsattn_trunk_layer_t& a, cudaStream_t st) {
    const size_t smem = (size_t)M * (a.d > a.f ? a.d : a.f) * 2;
    static size_t opted[16] = {0};
    static int sm_count[16] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 16) dev = 0;
    if (sm_count[dev] == 0) cudaDeviceGetAttribute(&sm_count[dev], cudaDevAttrMultiProcessorCount, dev);
    if (smem > 48 * 1024 && opted[dev] < smem) {
        if (cudaFuncSetAttribute(trunk_layer_kernel<KCD, KCF, M>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess) {
            (void)cudaGetLastError();
            fs_set_error("trunk_layer: cannot opt in to %zu bytes of shared memory", smem);
            return FSATTN_ELAUNCH;
        }
        opted[dev] = smem;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(sm_count[dev], 1, 1);          // one CTA per SM: all co-resident (checked by the cooperative launch)
    cfg.blockDim = dim3(GEMV_THREADS, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = a.pdl ? 2 : 1;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, trunk_layer_kernel<KCD, KCF, M>, a);
    if (e != cudaSuccess) {
        (void)cudaGetLastError();
        fs_set_error("trunk_layer: launch failed: %s", cudaGetErrorString(e));
        return FSATTN_ELAUNCH;
    }
    return FSATTN_OK;
}

template <int KCD, int KCF>
int launch_layer_m(const fsattn_trunk_layer_t& a, cudaStream_t st) {
    if (a.M <= 1) return launch_layer<KCD, KCF, 1>(a, st);
    if (a.M <= 2) return launch_layer<KCD, KCF, 2>(a, st);
    if (a.M <= 4) return launch_layer<KCD, KCF, 4>(a, st);
    return launch_layer<KCD, KCF, 8>(a, st);
}

}  // namespace

extern "C" int fsattn_trunk_layer(const fsattn_trunk_layer_t* a, fsattn_stream_t stream) {
    FS_REQUIRE(a != nullptr && a->x && a->y && a->w_o && a->norm2_w && a->w_gu && a->act && a->w_down && a->bar && a->status,
               "trunk_layer: null pointer");
    FS_REQUIRE(a->M >= 1 && a->M <= 8, "trunk_layer: M = %d rows (1..8)", a->M);
    FS_REQUIRE(a->d >= 8 && a->d % 8 == 0 && a->f >= 8 && a->f % 8 == 0, "trunk_layer: d = %d, f = %d must be multiples of 8", a->d, a->f);
    FS_REQUIRE(a->x_stride % 8 == 0 && a->y_stride % 8 == 0 && a->act_stride % 8 == 0, "trunk_layer: row strides must be multiples of 8");
    FS_REQUIRE(a->w_next == nullptr || (a->norm_next_w && a->out_next && a->n_next >= 1), "trunk_layer: next projection incomplete");
    const void* ptrs[] = {a->x, a->y, a->w_o, a->norm2_w, a->w_gu, a->act, a->w_down, a->norm_next_w, a->w_next};
    for (const void* p : ptrs) FS_REQUIRE(((uintptr_t)p & 15) == 0, "trunk_layer: pointers must be 16-byte aligned");
    const int kcd = (a->d + 255) / 256, kcf = (a->f + 255) / 256;
    cudaStream_t st = (cudaStream_t)stream;
    if (kcd <= 4 && kcf <= 11) return launch_layer_m<4, 11>(*a, st);
    if (kcd <= 6 && kcf <= 17) return launch_layer_m<6, 17>(*a, st);
    FS_UNSUPPORTED(true, "trunk_layer: d = %d, f = %d above 1536 / 4352", a->d, a->f);
    return FSATTN_EUNSUPPORTED;
}
