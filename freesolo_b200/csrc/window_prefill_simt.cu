// Window branch of a prefill on CUDA cores: the checked, shape-agnostic implementation (any N, W, head dim 64/96/128,
// any position offset). The tensor-core kernel in window_prefill_tc.cu covers the serving shapes; this one serves the
// remaining shapes and is the on-device cross-check for it at sizes the CPU oracle cannot reach.
//
// One CTA = 128 consecutive queries of one (b,h), one thread per query (rotated q, running max/sum and the output row
// in registers). Keys/values arrive in 64-row tiles staged in shared memory as fp32, keys rotated on the way in and
// rounded to bf16 like the stored rotated keys of the reference; all threads read the same key row (broadcast).
#include "common.cuh"

__device__ __forceinline__ void rope8(const uint4& lo, const uint4& hi, const uint4& c, const uint4& s, float* o_lo,
                                      float* o_hi) {
    float a[8], b[8], cc[8], ss[8];
    a[0] = bf_lo(lo.x); a[1] = bf_hi(lo.x); a[2] = bf_lo(lo.y); a[3] = bf_hi(lo.y);
    a[4] = bf_lo(lo.z); a[5] = bf_hi(lo.z); a[6] = bf_lo(lo.w); a[7] = bf_hi(lo.w);
    b[0] = bf_lo(hi.x); b[1] = bf_hi(hi.x); b[2] = bf_lo(hi.y); b[3] = bf_hi(hi.y);
    b[4] = bf_lo(hi.z); b[5] = bf_hi(hi.z); b[6] = bf_lo(hi.w); b[7] = bf_hi(hi.w);
    cc[0] = bf_lo(c.x); cc[1] = bf_hi(c.x); cc[2] = bf_lo(c.y); cc[3] = bf_hi(c.y);
    cc[4] = bf_lo(c.z); cc[5] = bf_hi(c.z); cc[6] = bf_lo(c.w); cc[7] = bf_hi(c.w);
    ss[0] = bf_lo(s.x); ss[1] = bf_hi(s.x); ss[2] = bf_lo(s.y); ss[3] = bf_hi(s.y);
    ss[4] = bf_lo(s.z); ss[5] = bf_hi(s.z); ss[6] = bf_lo(s.w); ss[7] = bf_hi(s.w);
#pragma unroll
    for (int j = 0; j < 8; j++) {
        o_lo[j] = bf_round(a[j] * cc[j] - b[j] * ss[j]);
        o_hi[j] = bf_round(b[j] * cc[j] + a[j] * ss[j]);
    }
}

template <int D>
__global__ void __launch_bounds__(128) window_prefill_simt_kernel(const fsattn_window_prefill_t a) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    float* ks = reinterpret_cast<float*>(smem_raw);     // 64 * D
    float* vs = ks + 64 * D;                            // 64 * D
    constexpr int HALF = D / 2;
    constexpr int CH = HALF / 8;                        // 16-byte chunks per half row
    const int tid = threadIdx.x;
    const int q0 = blockIdx.x * 128;
    const int bh = blockIdx.y;
    const int b = bh / a.H, h = bh - b * a.H;
    const int qi = q0 + tid;
    const bool q_ok = qi < a.N;
    const bf16* cosT = (const bf16*)a.cos;
    const bf16* sinT = (const bf16*)a.sin;

    float q[D];
    if (q_ok) {
        const bf16* qp = (const bf16*)a.q.ptr + b * a.q.sb + h * a.q.sh + (int64_t)qi * a.q.sn;
        const int64_t tp = (int64_t)(a.pos0 + qi) * D;
#pragma unroll
        for (int e = 0; e < CH; e++) {
            const uint4 lo = reinterpret_cast<const uint4*>(qp)[e];
            const uint4 hi = reinterpret_cast<const uint4*>(qp + HALF)[e];
            const uint4 c = reinterpret_cast<const uint4*>(cosT + tp)[e];
            const uint4 s = reinterpret_cast<const uint4*>(sinT + tp)[e];
            rope8(lo, hi, c, s, &q[8 * e], &q[HALF + 8 * e]);
        }
    } else {
#pragma unroll
        for (int e = 0; e < D; e++) q[e] = 0.0f;
    }
    float acc[D];
#pragma unroll
    for (int e = 0; e < D; e++) acc[e] = 0.0f;
    float m = -INFINITY, l = 0.0f;

    int k_lo = q0 - a.W; if (k_lo < 0) k_lo = 0;
    k_lo &= ~63;
    int k_hi = q0 + 128; if (k_hi > a.N) k_hi = a.N;
    const bf16* kbase = (const bf16*)a.k.ptr + b * a.k.sb + h * a.k.sh;
    const bf16* vbase = (const bf16*)a.v.ptr + b * a.v.sb + h * a.v.sh;
    for (int k0 = k_lo; k0 < k_hi; k0 += 64) {
        __syncthreads();
        for (int i = tid; i < 64 * CH; i += 128) {
            const int r = i / CH, e = i - r * CH;
            const int kj = k0 + r;
            float lo_o[8], hi_o[8], v_lo[8], v_hi[8];
            if (kj < a.N) {
                const bf16* kp = kbase + (int64_t)kj * a.k.sn;
                const bf16* vp = vbase + (int64_t)kj * a.v.sn;
                const int64_t tp = (int64_t)(a.pos0 + kj) * D;
                rope8(reinterpret_cast<const uint4*>(kp)[e], reinterpret_cast<const uint4*>(kp + HALF)[e],
                      reinterpret_cast<const uint4*>(cosT + tp)[e], reinterpret_cast<const uint4*>(sinT + tp)[e], lo_o, hi_o);
                const uint4 w0 = reinterpret_cast<const uint4*>(vp)[e];
                const uint4 w1 = reinterpret_cast<const uint4*>(vp + HALF)[e];
                v_lo[0] = bf_lo(w0.x); v_lo[1] = bf_hi(w0.x); v_lo[2] = bf_lo(w0.y); v_lo[3] = bf_hi(w0.y);
                v_lo[4] = bf_lo(w0.z); v_lo[5] = bf_hi(w0.z); v_lo[6] = bf_lo(w0.w); v_lo[7] = bf_hi(w0.w);
                v_hi[0] = bf_lo(w1.x); v_hi[1] = bf_hi(w1.x); v_hi[2] = bf_lo(w1.y); v_hi[3] = bf_hi(w1.y);
                v_hi[4] = bf_lo(w1.z); v_hi[5] = bf_hi(w1.z); v_hi[6] = bf_lo(w1.w); v_hi[7] = bf_hi(w1.w);
            } else {
#pragma unroll
                for (int j = 0; j < 8; j++) { lo_o[j] = hi_o[j] = v_lo[j] = v_hi[j] = 0.0f; }
            }
#pragma unroll
            for (int j = 0; j < 8; j++) {
                ks[r * D + 8 * e + j] = lo_o[j];
                ks[r * D + HALF + 8 * e + j] = hi_o[j];
                vs[r * D + 8 * e + j] = v_lo[j];
                vs[r * D + HALF + 8 * e + j] = v_hi[j];
            }
        }
        __syncthreads();
        if (!q_ok) continue;
        int j0 = qi - a.W - k0; if (j0 < 0) j0 = 0;
        int j1 = qi - k0 + 1; if (j1 > 64) j1 = 64;
        if (k0 + j1 > a.N) j1 = a.N - k0;
        for (int j = j0; j < j1; j++) {
            const float4* kr = reinterpret_cast<const float4*>(ks + j * D);
            float d0 = 0.f, d1 = 0.f, d2 = 0.f, d3 = 0.f;
#pragma unroll
            for (int e = 0; e < D / 4; e++) {
                const float4 kv = kr[e];
                d0 = fmaf(q[4 * e + 0], kv.x, d0); d1 = fmaf(q[4 * e + 1], kv.y, d1);
                d2 = fmaf(q[4 * e + 2], kv.z, d2); d3 = fmaf(q[4 * e + 3], kv.w, d3);
            }
            const float sc = ((d0 + d1) + (d2 + d3)) * a.scale;
            if (sc > m) {
                const float alpha = (m == -INFINITY) ? 0.0f : __expf(m - sc);
                l *= alpha;
#pragma unroll
                for (int e = 0; e < D; e++) acc[e] *= alpha;
                m = sc;
            }
            const float p = __expf(sc - m);
            l += p;
            const float4* vr = reinterpret_cast<const float4*>(vs + j * D);
#pragma unroll
            for (int e = 0; e < D / 4; e++) {
                const float4 vv = vr[e];
                acc[4 * e + 0] = fmaf(p, vv.x, acc[4 * e + 0]); acc[4 * e + 1] = fmaf(p, vv.y, acc[4 * e + 1]);
                acc[4 * e + 2] = fmaf(p, vv.z, acc[4 * e + 2]); acc[4 * e + 3] = fmaf(p, vv.w, acc[4 * e + 3]);
            }
        }
    }
    if (!q_ok) return;
    const float inv = (l > 0.0f) ? 1.0f / l : 0.0f;
    bf16* op = (bf16*)a.out + ((int64_t)b * a.N + qi) * ((int64_t)a.H * D) + (int64_t)h * D;
#pragma unroll
    for (int e = 0; e < D / 8; e++) {
        uint4 w;
        w.x = pack_bf2(acc[8 * e + 0] * inv, acc[8 * e + 1] * inv);
        w.y = pack_bf2(acc[8 * e + 2] * inv, acc[8 * e + 3] * inv);
        w.z = pack_bf2(acc[8 * e + 4] * inv, acc[8 * e + 5] * inv);
        w.w = pack_bf2(acc[8 * e + 6] * inv, acc[8 * e + 7] * inv);
        reinterpret_cast<uint4*>(op)[e] = w;
    }
}

template <int D>
static int launch_simt(const fsattn_window_prefill_t* a, cudaStream_t st) {
    const size_t smem = (size_t)2 * 64 * D * 4;
    static bool opted[16] = {false};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 16 && !opted[dev]) {
        if (cudaFuncSetAttribute(window_prefill_simt_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess) {
            fs_set_error("window_prefill: cannot opt in to %zu bytes of shared memory", smem);
            return FSATTN_ELAUNCH;
        }
        opted[dev] = true;
    }
    dim3 grid((a->N + 127) / 128, a->B * a->H);
    window_prefill_simt_kernel<D><<<grid, 128, smem, st>>>(*a);
    return fs_check_launch("window_prefill_simt");
}

int fs_window_prefill_simt(const fsattn_window_prefill_t* a, cudaStream_t st) {
    switch (a->D) {
        case 64: return launch_simt<64>(a, st);
        case 96: return launch_simt<96>(a, st);
        default: return launch_simt<128>(a, st);
    }
}
