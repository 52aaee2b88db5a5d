// Small-batch trunk projections for the decode step: out = epilogue( [rmsnorm](x) @ W^T ), M <= 8 rows of activations
// per pass, W (Nout, K) bf16 streamed exactly once with 16-byte loads (HBM-bound: 2*Nout*K bytes per call).
//
// One warp per output row (or per gate/up row pair for the SwiGLU epilogue). Every kernel is launched with programmatic
// dependent launch: it fetches its first weight rows into registers BEFORE waiting for the producer kernel, so weight
// streaming continues across kernel boundaries and the post-dependency critical path is "read x, FMA, reduce, store".
#include "trunk_rows.cuh"

namespace {

// KC = ceil(K / 256) 16-byte chunks per lane; M rows of activations; EPI as in the header
template <int KC, int M>
__global__ void __launch_bounds__(GEMV_THREADS) trunk_gemv_kernel(const fsattn_trunk_gemv_t a) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    uint4* xs = reinterpret_cast<uint4*>(smem_raw);                  // M * K bf16 (normalised when norm_w != nullptr)
    __shared__ float red[GEMV_WARPS][M];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int kchunks = a.K / 8;
    const int nwarps = gridDim.x * GEMV_WARPS;
    const int gw = blockIdx.x * GEMV_WARPS + warp;
    const bool swiglu = a.epilogue == FSATTN_EPI_SWIGLU;
    const int nunits = swiglu ? a.n_out / 2 : a.n_out;                // a unit = one output row, or a (gate, up) pair
    const bf16* W = (const bf16*)a.w;

    // ---- weights do not depend on the producer kernel: the first unit goes to registers, the next ones to L2 ---------
    RowRegs<KC> r0, r1;
    int u = gw;
    load_row<KC>(r0, u < nunits ? W + (int64_t)u * a.K : nullptr, lane, kchunks);
    if (swiglu) load_row<KC>(r1, u < nunits ? W + (int64_t)(u + nunits) * a.K : nullptr, lane, kchunks);
    {
        const int row_bytes = a.K * 2;
        int pu = u + nwarps;
        for (int n = 0; n < 3 && pu < nunits; n++, pu += nwarps) {
            const char* p0 = reinterpret_cast<const char*>(W + (int64_t)pu * a.K);
            for (int off = lane * 128; off < row_bytes; off += 32 * 128) {
                asm volatile("prefetch.global.L2 [%0];" ::"l"(p0 + off));
                if (swiglu) asm volatile("prefetch.global.L2 [%0];" ::"l"(p0 + (int64_t)nunits * row_bytes + off));
            }
        }
    }
    // the norm weights do not depend on the producer either: this thread's chunks go to registers now
    constexpr int NIT = (KC + 7) / 8;                                 // activation chunks per thread (256 threads, 8 per lane-row)
    constexpr bool XREG = NIT * M <= 8;                               // small enough to keep the activations in registers
    uint4 nwr[NIT];
    if (a.norm_w != nullptr) {
#pragma unroll
        for (int i = 0; i < NIT; i++) {
            const int c = tid + i * GEMV_THREADS;
            nwr[i] = c < kchunks ? *reinterpret_cast<const uint4*>((const bf16*)a.norm_w + c * 8) : make_uint4(0u, 0u, 0u, 0u);
        }
    }
    // Wait for the producer, THEN release the consumer: at most two kernels of the chain overlap, so a consumer's
    // prologue only ever runs beside its direct producer's main phase.
    pdl_wait();
    pdl_launch_dependents();

    // ---- activations -> shared memory (optionally RMS-normalised, rounded to bf16 like the eager norm's output) ----
    const bf16* X = (const bf16*)a.x + (int64_t)a.m0 * a.x_stride;
    if constexpr (XREG) {
        // every activation chunk of this thread is loaded before anything uses it: a load-use-load loop would pay the memory
        // round trips one after the other (in-order issue), and the normalised pass would read x a second time
        uint4 xr[M][NIT];
#pragma unroll
        for (int i = 0; i < NIT; i++) {
            const int c = tid + i * GEMV_THREADS;
#pragma unroll
            for (int m = 0; m < M; m++)
                xr[m][i] = c < kchunks ? *reinterpret_cast<const uint4*>(X + (int64_t)m * a.x_stride + c * 8) : make_uint4(0u, 0u, 0u, 0u);
        }
        if (a.norm_w != nullptr) {
            float ss[M];
#pragma unroll
            for (int m = 0; m < M; m++) {
                ss[m] = 0.0f;
                // chunk by chunk in the order of the loop version (the sum of squares is rounding-sensitive)
#pragma unroll
                for (int i = 0; i < NIT; i++) {
                    const uint4 x = xr[m][i];
                    const float v[8] = {bf_lo(x.x), bf_hi(x.x), bf_lo(x.y), bf_hi(x.y), bf_lo(x.z), bf_hi(x.z), bf_lo(x.w), bf_hi(x.w)};
#pragma unroll
                    for (int j = 0; j < 8; j++) ss[m] = fmaf(v[j], v[j], ss[m]);
                }
                const float sw = warp_sum(ss[m]);
                if (lane == 0) red[warp][m] = sw;
            }
            __syncthreads();
            float rinv[M];
#pragma unroll
            for (int m = 0; m < M; m++) {
                float sr = 0.0f;
#pragma unroll
                for (int w = 0; w < GEMV_WARPS; w++) sr += red[w][m];
                rinv[m] = rsqrtf(sr / (float)a.K + a.eps);
            }
#pragma unroll
            for (int i = 0; i < NIT; i++) {
                const int c = tid + i * GEMV_THREADS;
                if (c >= kchunks) continue;
                const uint4 nw = nwr[i];
                const float g[8] = {bf_lo(nw.x), bf_hi(nw.x), bf_lo(nw.y), bf_hi(nw.y), bf_lo(nw.z), bf_hi(nw.z), bf_lo(nw.w), bf_hi(nw.w)};
#pragma unroll
                for (int m = 0; m < M; m++) {
                    const uint4 x = xr[m][i];
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
#pragma unroll
            for (int i = 0; i < NIT; i++) {
                const int c = tid + i * GEMV_THREADS;
                if (c >= kchunks) continue;
#pragma unroll
                for (int m = 0; m < M; m++) xs[m * kchunks + c] = xr[m][i];
            }
        }
    } else
    if (a.norm_w != nullptr) {
        float ss[M];
#pragma unroll
        for (int m = 0; m < M; m++) ss[m] = 0.0f;
        for (int c = tid; c < kchunks; c += GEMV_THREADS) {
#pragma unroll
            for (int m = 0; m < M; m++) {
                const uint4 x = *reinterpret_cast<const uint4*>(X + (int64_t)m * a.x_stride + c * 8);
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
            rinv[m] = rsqrtf(s / (float)a.K + a.eps);
        }
        const bf16* NW = (const bf16*)a.norm_w;
        for (int c = tid; c < kchunks; c += GEMV_THREADS) {
            const uint4 nw = *reinterpret_cast<const uint4*>(NW + c * 8);
            const float g[8] = {bf_lo(nw.x), bf_hi(nw.x), bf_lo(nw.y), bf_hi(nw.y), bf_lo(nw.z), bf_hi(nw.z), bf_lo(nw.w), bf_hi(nw.w)};
#pragma unroll
            for (int m = 0; m < M; m++) {
                const uint4 x = *reinterpret_cast<const uint4*>(X + (int64_t)m * a.x_stride + c * 8);
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
            for (int m = 0; m < M; m++) xs[m * kchunks + c] = *reinterpret_cast<const uint4*>(X + (int64_t)m * a.x_stride + c * 8);
        }
    }
    __syncthreads();

    // ---- rows ------------------------------------------------------------------------------------------------------
    bf16* OUT = (bf16*)a.out + (int64_t)a.m0 * a.out_stride;
    const bf16* RES = a.res ? (const bf16*)a.res + (int64_t)a.m0 * a.res_stride : nullptr;
    for (; u < nunits; u += nwarps) {
        const int un = u + nwarps;
        RowRegs<KC> n0, n1;
        // next unit's weights go in flight before this unit's arithmetic
        load_row<KC>(n0, un < nunits ? W + (int64_t)un * a.K : nullptr, lane, kchunks);
        if (swiglu) load_row<KC>(n1, un < nunits ? W + (int64_t)(un + nunits) * a.K : nullptr, lane, kchunks);
        float acc[M], acc2[M];
        dot_row<KC, M>(r0, xs, kchunks, lane, acc);
        if (swiglu) dot_row<KC, M>(r1, xs, kchunks, lane, acc2);
        if (lane == 0) {
#pragma unroll
            for (int m = 0; m < M; m++) {
                float v;
                if (swiglu) {
                    const float g = bf_round(acc[m]), up = bf_round(acc2[m]);
                    const float s = bf_round(g / (1.0f + __expf(-g)));
                    v = s * up;
                } else if (RES != nullptr) {
                    v = __bfloat162float(RES[(int64_t)m * a.res_stride + u]) + bf_round(acc[m]);
                } else {
                    v = acc[m];
                }
                OUT[(int64_t)m * a.out_stride + u] = __float2bfloat16_rn(v);
            }
        }
        r0 = n0;
        if (swiglu) r1 = n1;
    }
}

template <int KC, int M>
int launch_gemv(const fsattn_trunk_gemv_t& a, cudaStream_t st, int sm_count) {
    const size_t smem = (size_t)M * a.K * 2;
    static size_t opted[16] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    if (smem > 48 * 1024 && dev >= 0 && dev < 16 && opted[dev] < smem) {
        if (cudaFuncSetAttribute(trunk_gemv_kernel<KC, M>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess) {
            fs_set_error("trunk_gemv: cannot opt in to %zu bytes of shared memory", smem);
            return FSATTN_ELAUNCH;
        }
        opted[dev] = smem;
    }
    const int nunits = (a.epilogue == FSATTN_EPI_SWIGLU) ? a.n_out / 2 : a.n_out;
    int blocks = (nunits + GEMV_WARPS - 1) / GEMV_WARPS;
    // two resident CTAs per SM, the warps loop over the remaining rows: with one, a warp of the wide projections holds three or
    // four rows of which only the first is in registers when the producer finishes; with three, the next kernel's CTAs no
    // longer fit beside this one's and its prologue (weight prefetch) starts late. Measured on the 341M decode step:
    // 0.640 / 0.596 / 0.657 ms for 1 / 2 / 3.
    if (blocks > 2 * sm_count) blocks = 2 * sm_count;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(blocks, 1, 1);
    cfg.blockDim = dim3(GEMV_THREADS, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = a.pdl ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, trunk_gemv_kernel<KC, M>, a);
    if (e != cudaSuccess) {
        fs_set_error("trunk_gemv: launch failed: %s", cudaGetErrorString(e));
        return FSATTN_ELAUNCH;
    }
    return FSATTN_OK;
}

template <int KC>
int launch_gemv_m(const fsattn_trunk_gemv_t& a, cudaStream_t st, int sm_count, int m) {
    switch (m) {
        case 1: return launch_gemv<KC, 1>(a, st, sm_count);
        case 2: return launch_gemv<KC, 2>(a, st, sm_count);
        case 4: return launch_gemv<KC, 4>(a, st, sm_count);
        default: return launch_gemv<KC, 8>(a, st, sm_count);
    }
}

}  // namespace

extern "C" int fsattn_trunk_gemv(const fsattn_trunk_gemv_t* a, fsattn_stream_t stream) {
    FS_REQUIRE(a != nullptr && a->w && a->x && a->out, "trunk_gemv: null pointer");
    FS_REQUIRE(a->M >= 1 && a->K >= 8 && a->K % 8 == 0 && a->n_out >= 1, "trunk_gemv: bad sizes M=%d K=%d N=%d", a->M, a->K, a->n_out);
    FS_UNSUPPORTED(a->K > 17 * 256, "trunk_gemv: K=%d above %d", a->K, 17 * 256);
    FS_REQUIRE(a->epilogue >= FSATTN_EPI_STORE && a->epilogue <= FSATTN_EPI_SWIGLU, "trunk_gemv: epilogue %d", a->epilogue);
    FS_REQUIRE(a->epilogue != FSATTN_EPI_SWIGLU || a->n_out % 2 == 0, "trunk_gemv: SwiGLU needs gate and up rows");
    FS_REQUIRE(a->epilogue != FSATTN_EPI_RESIDUAL || a->res != nullptr, "trunk_gemv: residual epilogue without a residual");
    FS_REQUIRE(((uintptr_t)a->w & 15) == 0 && ((uintptr_t)a->x & 15) == 0 && a->x_stride % 8 == 0, "trunk_gemv: W and x rows must be 16-byte aligned");
    FS_REQUIRE(a->norm_w == nullptr || ((uintptr_t)a->norm_w & 15) == 0, "trunk_gemv: norm weight must be 16-byte aligned");
    static int sm_count[16] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 16) dev = 0;
    if (sm_count[dev] == 0) cudaDeviceGetAttribute(&sm_count[dev], cudaDevAttrMultiProcessorCount, dev);
    const int kc = (a->K + 255) / 256;
    cudaStream_t st = (cudaStream_t)stream;
    fsattn_trunk_gemv_t t = *a;
    if (t.epilogue != FSATTN_EPI_RESIDUAL) t.res = nullptr;
    // batches above 8 rows run as consecutive passes of <= 8 rows (the weights are re-read per pass)
    for (int m0 = 0; m0 < a->M; m0 += 8) {
        int m = a->M - m0;
        if (m > 8) m = 8;
        const int mt = m >= 8 ? 8 : (m >= 4 ? 4 : (m >= 2 ? 2 : 1));
        // cover m rows with tiles of size mt (e.g. 7 = 4 + 2 + 1)
        int done = 0;
        while (done < m) {
            int tile = mt;
            while (tile > m - done) tile >>= 1;
            t.m0 = m0 + done;
            int rc;
            if (kc <= 4) rc = launch_gemv_m<4>(t, st, sm_count[dev], tile);
            else if (kc <= 6) rc = launch_gemv_m<6>(t, st, sm_count[dev], tile);
            else if (kc <= 11) rc = launch_gemv_m<11>(t, st, sm_count[dev], tile);
            else rc = launch_gemv_m<17>(t, st, sm_count[dev], tile);
            if (rc != FSATTN_OK) return rc;
            done += tile;
        }
    }
    return FSATTN_OK;
}
