// Window branch of a prefill on the 5th-generation tensor cores: tcgen05.mma with TMEM accumulators, operands staged by
// TMA (cp.async.bulk.tensor, 128-byte swizzle), one CTA per 128 queries of one (batch, head).
//
//   pass 0 (rope_qk_kernel): rotate Q and K once into a (B*H, N, D) bf16 workspace (HBM-bound: 2 reads + 2 writes of N*D)
//   pass 1 (window_tc_kernel): for the W/64 + 2 key tiles (64 keys each) of the band
//        S  = Qr Kr^T        tcgen05.mma 128x64x64 (4 k-steps), accumulator in TMEM
//        P  = exp2(S*c - m)  4 softmax warps, one query row per thread (tcgen05.ld), band mask on the edge tiles. P never
//                            leaves tensor memory: it is split into a bf16 high part and a bf16 low part (p - high), so
//                            that the product keeps about 16 bits of every probability, and both are written with
//                            tcgen05.st over the columns S occupied (64 fp32 columns = 32 packed columns high + 32 low)
//        PV = P V            tcgen05.mma 128x64x64 with A read from tensor memory (4 k-steps for the high part, 4 for the low
//                            part) into a second TMEM accumulator; the running output lives in registers: O = O*alpha + PV
// Warp roles: warps 0-3 softmax/epilogue (TMEM lane quarter = warp id), warp 4 TMA producer, warp 5 MMA issuer. A CTA takes
// 256 TMEM columns (S0, S1, PV0, PV1 of 64 each) and about 100 KB of shared memory, so two CTAs share an SM and one CTA's
// softmax runs while the other's MMAs are in flight.
// Every mbarrier wait is bounded; on a timeout the CTA records it in *status, stops issuing work and still frees its TMEM.
//
// FLOPs per CTA: (W/64+2) tiles * (2*128*64*64 + 2*2*128*64*64); algorithmic FLOPs per query 4*D*min(i+1, W+1).
#include "tc_common.cuh"

namespace {

constexpr int TC_BN = 64;           // keys per tile
constexpr int TC_D = 64;
constexpr int TC_THREADS = 192;     // 4 softmax warps (one per TMEM lane quarter), TMA producer, MMA issuer
constexpr int TC_SOFTMAX_THREADS = 128;
constexpr int TC_TMEM_COLS = 256;   // S0 | S1 | PV0 | PV1, 64 columns each
constexpr int TC_TILE_BYTES = TC_BN * TC_D * 2;      // one K or V tile: 64 rows of 128 bytes

// shared memory map (bytes, from a 1024-byte aligned base)
constexpr int SM_Q = 0;                         // 128 x 64 bf16
constexpr int TC_KV_STAGES = 5;                 // key/value tiles in flight (320 keys): tile loads stay off the critical path
constexpr int SM_K = SM_Q + 16384;              // TC_KV_STAGES stages
constexpr int SM_V = SM_K + TC_KV_STAGES * TC_TILE_BYTES;
constexpr int SM_BAR = SM_V + TC_KV_STAGES * TC_TILE_BYTES;        // mbarriers
constexpr int SM_TOTAL = SM_BAR + 256;

enum { BAR_Q = 0, BAR_KV_FULL = 1, BAR_KV_EMPTY = BAR_KV_FULL + TC_KV_STAGES, BAR_S_FULL = BAR_KV_EMPTY + TC_KV_STAGES,
       BAR_P_FULL = BAR_S_FULL + 2, BAR_PV_FULL = BAR_P_FULL + 2, BAR_PV_FREE = BAR_PV_FULL + 2, BAR_COUNT = BAR_PV_FREE + 2 };
static_assert(BAR_COUNT * 8 <= 256, "mbarrier area");

// ---- pass 0: rotate Q and K into the workspace ----------------------------------------------------------------------
__global__ void __launch_bounds__(256) rope_qk_kernel(const fsattn_window_prefill_t a, bf16* qr, bf16* kr) {
    constexpr int HALF = TC_D / 2, CH = HALF / 8;
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int64_t total = (int64_t)a.B * a.H * a.N * CH;
    if (i >= total) return;
    const int e = (int)(i % CH);
    const int64_t row = i / CH;                         // (b*H + h)*N + n
    const int n = (int)(row % a.N);
    const int64_t bh = row / a.N;
    const int b = (int)(bh / a.H), h = (int)(bh - (int64_t)b * a.H);
    const int64_t tp = (int64_t)(a.pos0 + n) * TC_D;
    const uint4 c = reinterpret_cast<const uint4*>((const bf16*)a.cos + tp)[e];
    const uint4 s = reinterpret_cast<const uint4*>((const bf16*)a.sin + tp)[e];
    const float cc[8] = {bf_lo(c.x), bf_hi(c.x), bf_lo(c.y), bf_hi(c.y), bf_lo(c.z), bf_hi(c.z), bf_lo(c.w), bf_hi(c.w)};
    const float ss[8] = {bf_lo(s.x), bf_hi(s.x), bf_lo(s.y), bf_hi(s.y), bf_lo(s.z), bf_hi(s.z), bf_lo(s.w), bf_hi(s.w)};
#pragma unroll
    for (int t = 0; t < 2; t++) {
        const fsattn_bhnd_t& src = t == 0 ? a.q : a.k;
        const bf16* p = (const bf16*)src.ptr + b * src.sb + h * src.sh + (int64_t)n * src.sn;
        const uint4 lo = reinterpret_cast<const uint4*>(p)[e];
        const uint4 hi = reinterpret_cast<const uint4*>(p + HALF)[e];
        const float x1[8] = {bf_lo(lo.x), bf_hi(lo.x), bf_lo(lo.y), bf_hi(lo.y), bf_lo(lo.z), bf_hi(lo.z), bf_lo(lo.w), bf_hi(lo.w)};
        const float x2[8] = {bf_lo(hi.x), bf_hi(hi.x), bf_lo(hi.y), bf_hi(hi.y), bf_lo(hi.z), bf_hi(hi.z), bf_lo(hi.w), bf_hi(hi.w)};
        uint4 o1, o2;
        o1.x = pack_bf2(x1[0] * cc[0] - x2[0] * ss[0], x1[1] * cc[1] - x2[1] * ss[1]);
        o1.y = pack_bf2(x1[2] * cc[2] - x2[2] * ss[2], x1[3] * cc[3] - x2[3] * ss[3]);
        o1.z = pack_bf2(x1[4] * cc[4] - x2[4] * ss[4], x1[5] * cc[5] - x2[5] * ss[5]);
        o1.w = pack_bf2(x1[6] * cc[6] - x2[6] * ss[6], x1[7] * cc[7] - x2[7] * ss[7]);
        o2.x = pack_bf2(x2[0] * cc[0] + x1[0] * ss[0], x2[1] * cc[1] + x1[1] * ss[1]);
        o2.y = pack_bf2(x2[2] * cc[2] + x1[2] * ss[2], x2[3] * cc[3] + x1[3] * ss[3]);
        o2.z = pack_bf2(x2[4] * cc[4] + x1[4] * ss[4], x2[5] * cc[5] + x1[5] * ss[5]);
        o2.w = pack_bf2(x2[6] * cc[6] + x1[6] * ss[6], x2[7] * cc[7] + x1[7] * ss[7]);
        bf16* dst = (t == 0 ? qr : kr) + row * TC_D;
        reinterpret_cast<uint4*>(dst)[e] = o1;
        reinterpret_cast<uint4*>(dst + HALF)[e] = o2;
    }
}

struct TcParams {
    int N, W, H;
    float c2;              // scale * log2(e)
    bf16* out;             // (B, N, H*D)
    int32_t* status;       // optional: timeouts are counted in status[0]
};

// ---- pass 1 -------------------------------------------------------------------------------------------------------------
__global__ void __launch_bounds__(TC_THREADS, 2)
window_tc_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                 const __grid_constant__ CUtensorMap tm_v, const TcParams p) {
    extern __shared__ unsigned char tc_smem_raw[];
    __shared__ uint32_t tmem_base_s;
    __shared__ int abort_s;
    unsigned char* base = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(tc_smem_raw) + 1023) & ~(uintptr_t)1023);
    uint64_t* bars = reinterpret_cast<uint64_t*>(base + SM_BAR);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int q0 = blockIdx.x * TC_BM;
    const int bh = blockIdx.y;
    const int b = bh / p.H, h = bh - b * p.H;
    // tile t covers the keys q0 - W + 64 t .. + 63; the band of the CTA's 128 queries ends at key q0 + 127
    const int ntile_total = (p.W + TC_BM) / TC_BN;
    int t_first = (p.W - q0) / TC_BN;                 // tiles that lie entirely before the sequence start are skipped
    if (t_first < 0) t_first = 0;
    const int nt = ntile_total - t_first;

    if (tid == 0) {
        bar_init(&bars[BAR_Q], 1);
        for (int s = 0; s < TC_KV_STAGES; s++) {
            bar_init(&bars[BAR_KV_FULL + s], 1);
            bar_init(&bars[BAR_KV_EMPTY + s], 1);
        }
        for (int s = 0; s < 2; s++) {
            bar_init(&bars[BAR_S_FULL + s], 1);
            bar_init(&bars[BAR_P_FULL + s], TC_SOFTMAX_THREADS);
            bar_init(&bars[BAR_PV_FULL + s], 1);
            bar_init(&bars[BAR_PV_FREE + s], TC_SOFTMAX_THREADS);
        }
        abort_s = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 4) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(s_u32(&tmem_base_s)), "r"(TC_TMEM_COLS) : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_base_s;
    const uint32_t tmem_pv = tmem + 2 * TC_BN;          // PV0 | PV1 behind S0 | S1
    volatile int* abortp = &abort_s;

    if (warp == 4) {
        // ================= TMA producer ====================================================================================
        if (lane == 0) {
            bar_expect_tx(&bars[BAR_Q], 16384);
            tma_load_3d(base + SM_Q, &tm_q, 0, q0, bh, &bars[BAR_Q]);
            for (int i = 0; i < nt && !*abortp; i++) {
                const int s = i % TC_KV_STAGES;
                const int kt0 = q0 - p.W + (t_first + i) * TC_BN;
                if (i >= TC_KV_STAGES && !bar_wait(&bars[BAR_KV_EMPTY + s], ((i / TC_KV_STAGES) - 1) & 1, abortp)) { *abortp = 1; break; }
                bar_expect_tx(&bars[BAR_KV_FULL + s], 2 * TC_TILE_BYTES);
                tma_load_3d(base + SM_K + s * TC_TILE_BYTES, &tm_k, 0, kt0, bh, &bars[BAR_KV_FULL + s]);
                tma_load_4d(base + SM_V + s * TC_TILE_BYTES, &tm_v, 0, kt0, h, b, &bars[BAR_KV_FULL + s]);
            }
        }
    } else if (warp == 5) {
        // ================= MMA issuer ======================================================================================
        // Issue order QK(0), QK(1), PV(0), QK(2), PV(1), ...: the tensor pipe runs one thread's MMAs in issue order, so
        // QK(i+2), which overwrites the columns that held P(i), starts after PV(i) has read them - no barrier is needed
        // for the S buffers beyond "P(i) is complete".
        if (lane == 0) {
            const uint32_t idesc_s = instr_desc(TC_BN, 0, 1);
            const uint32_t idesc_pv = instr_desc(TC_D, 1, 1);      // A (P, from TMEM) and B (V) share the bf16 format
            bool ok = bar_wait(&bars[BAR_Q], 0, abortp);
            for (int i = 0; i <= nt && ok && !*abortp; i++) {
                if (i < nt) {
                    const int s = i & 1, ks = i % TC_KV_STAGES;
                    ok = bar_wait(&bars[BAR_KV_FULL + ks], (i / TC_KV_STAGES) & 1, abortp);
                    if (!ok) break;
                    tc_fence_after();
                    const uint32_t aq = s_u32(base + SM_Q), bk = s_u32(base + SM_K + ks * TC_TILE_BYTES);
#pragma unroll
                    for (int k = 0; k < TC_D / 16; k++)
                        umma(tmem + s * TC_BN, smem_desc(aq + k * 32), smem_desc(bk + k * 32), idesc_s, k > 0);
                    umma_commit(&bars[BAR_S_FULL + s]);
                }
                if (i >= 1) {
                    const int j = i - 1, bb = j & 1;
                    ok = bar_wait(&bars[BAR_P_FULL + bb], (j >> 1) & 1, abortp);
                    if (ok && j >= 2) ok = bar_wait(&bars[BAR_PV_FREE + bb], ((j >> 1) - 1) & 1, abortp);
                    if (!ok) break;
                    tc_fence_after();
                    const int vs = j % TC_KV_STAGES;
                    const uint32_t ap = tmem + bb * TC_BN, bv = s_u32(base + SM_V + vs * TC_TILE_BYTES);
                    // 16 keys per step: 8 packed columns of P, 16 rows (2048 bytes) of V; high parts, then low parts
#pragma unroll
                    for (int k = 0; k < TC_BN / 16; k++)
                        umma_ts(tmem_pv + bb * TC_D, ap + k * 8, smem_desc(bv + k * 2048), idesc_pv, k > 0);
#pragma unroll
                    for (int k = 0; k < TC_BN / 16; k++)
                        umma_ts(tmem_pv + bb * TC_D, ap + TC_BN / 2 + k * 8, smem_desc(bv + k * 2048), idesc_pv, 1);
                    umma_commit(&bars[BAR_PV_FULL + bb]);
                    umma_commit(&bars[BAR_KV_EMPTY + vs]);
                }
            }
            if (!ok) *abortp = 1;
        }
    } else {
        // ================= softmax + epilogue: one thread per query row ======================================================
        // Warp w reaches the TMEM lanes 32 w .. 32 w + 31; a thread owns row r: the tile's 64 scores, its running maximum and
        // sum, and the 64 output dims, so the rows never exchange anything.
        const int r = warp * 32 + lane;
        const int qi = q0 + r;
        const uint32_t lane_base = tmem + ((uint32_t)(warp * 32) << 16);
        const uint32_t lane_pv = tmem_pv + ((uint32_t)(warp * 32) << 16);
        const int t_upper = p.W / TC_BN;             // tiles from here on reach past some row's own position
        float m = -INFINITY, l = 0.0f, a_pend = 0.0f;
        float O[TC_D];
#pragma unroll
        for (int d = 0; d < TC_D; d++) O[d] = 0.0f;
        bool ok = true;
        for (int i = 0; i < nt; i++) {
            const int bb = i & 1;
            const int t = t_first + i;
            ok = ok && bar_wait(&bars[BAR_S_FULL + bb], (i >> 1) & 1, abortp) && !*abortp;
            if (!__all_sync(FS_FULL, ok)) { ok = false; break; }
            tc_fence_after();
            const uint32_t s_addr = lane_base + bb * TC_BN;
            // the row's 64 scores, read from TMEM once and kept in registers for both passes
            float v[TC_BN];
            tmem_ld32(s_addr, v);
            tmem_ld32(s_addr + 32, v + 32);
            if (t < 2 || t >= t_upper) {            // edge tile: keys outside [q - W, q] become -inf
                const int c_lo = r - TC_BN * t, c_hi = r + p.W - TC_BN * t;
#pragma unroll
                for (int c = 0; c < TC_BN; c++) v[c] = (c >= c_lo && c <= c_hi) ? v[c] : -INFINITY;
            }
            float mx = -INFINITY;
#pragma unroll
            for (int c = 0; c < TC_BN; c++) mx = fmaxf(mx, v[c]);
            const float m_new = fmaxf(m, mx);
            const float alpha = (m == -INFINITY) ? 0.0f : exp2f((m - m_new) * p.c2);
            const float mc = (m_new == -INFINITY) ? 0.0f : m_new * p.c2;
            // probabilities (ex2.approx of a masked score is exactly 0). Each is split into bf16 high + bf16 low so the
            // tensor core multiplies about 16 bits of it; both parts go back into the columns the scores came from.
            float rowsum = 0.0f;
#pragma unroll
            for (int c0 = 0; c0 < TC_BN; c0 += 16) {
                uint32_t ph[8], pl[8];
#pragma unroll
                for (int c = 0; c < 16; c += 2) {
                    float p0, p1;
                    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(p0) : "f"(fmaf(v[c0 + c], p.c2, -mc)));
                    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(p1) : "f"(fmaf(v[c0 + c + 1], p.c2, -mc)));
                    rowsum += p0 + p1;
                    const __nv_bfloat162 h2 = __floats2bfloat162_rn(p0, p1);
                    const uint32_t hb = *reinterpret_cast<const uint32_t*>(&h2);
                    const __nv_bfloat162 l2 = __floats2bfloat162_rn(p0 - bf_lo(hb), p1 - bf_hi(hb));
                    ph[c >> 1] = hb;
                    pl[c >> 1] = *reinterpret_cast<const uint32_t*>(&l2);
                }
                tmem_st8(s_addr + (c0 >> 1), ph);
                tmem_st8(s_addr + TC_BN / 2 + (c0 >> 1), pl);
            }
            tmem_st_wait();
            tc_fence_before();
            bar_arrive(&bars[BAR_P_FULL + bb]);
            l = l * alpha + rowsum;
            m = m_new;
            // fold the previous tile's P V into the running output
            if (i >= 1) {
                const int j = i - 1, jb = j & 1;
                ok = bar_wait(&bars[BAR_PV_FULL + jb], (j >> 1) & 1, abortp) && !*abortp;
                if (!__all_sync(FS_FULL, ok)) { ok = false; break; }
                tc_fence_after();
#pragma unroll
                for (int hh = 0; hh < 2; hh++) {
                    float pv[32];
                    tmem_ld32(lane_pv + jb * TC_D + hh * 32, pv);
#pragma unroll
                    for (int c = 0; c < 32; c++) O[hh * 32 + c] = fmaf(O[hh * 32 + c], a_pend, pv[c]);
                }
                tc_fence_before();
                bar_arrive(&bars[BAR_PV_FREE + jb]);
            }
            a_pend = alpha;
        }
        if (ok && nt > 0) {
            const int j = nt - 1, jb = j & 1;
            ok = bar_wait(&bars[BAR_PV_FULL + jb], (j >> 1) & 1, abortp) && !*abortp;
            if (__all_sync(FS_FULL, ok)) {
                tc_fence_after();
#pragma unroll
                for (int hh = 0; hh < 2; hh++) {
                    float pv[32];
                    tmem_ld32(lane_pv + jb * TC_D + hh * 32, pv);
#pragma unroll
                    for (int c = 0; c < 32; c++) O[hh * 32 + c] = fmaf(O[hh * 32 + c], a_pend, pv[c]);
                }
                tc_fence_before();
            } else {
                ok = false;
            }
        }
        if (!ok) *abortp = 1;
        if (ok && qi < p.N) {
            const float inv = (l > 0.0f) ? 1.0f / l : 0.0f;
            bf16* op = p.out + ((int64_t)b * p.N + qi) * ((int64_t)p.H * TC_D) + (int64_t)h * TC_D;
#pragma unroll
            for (int e = 0; e < TC_D / 8; e++) {
                uint4 w;
                w.x = pack_bf2(O[8 * e + 0] * inv, O[8 * e + 1] * inv);
                w.y = pack_bf2(O[8 * e + 2] * inv, O[8 * e + 3] * inv);
                w.z = pack_bf2(O[8 * e + 4] * inv, O[8 * e + 5] * inv);
                w.w = pack_bf2(O[8 * e + 6] * inv, O[8 * e + 7] * inv);
                reinterpret_cast<uint4*>(op)[e] = w;
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (tid == 0 && abort_s && p.status != nullptr) atomicAdd(p.status, 1);
    if (warp == 4) {
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TC_TMEM_COLS) : "memory");
    }
}

}  // namespace

// ---- host side -------------------------------------------------------------------------------------------------------------
size_t fs_window_prefill_tc_workspace(const fsattn_window_prefill_t* a) {
    return (size_t)2 * a->B * a->H * a->N * TC_D * sizeof(bf16);
}

bool fs_window_prefill_tc_ok(const fsattn_window_prefill_t* a) {
    return a->D == TC_D && a->W >= TC_BN && a->W % TC_BN == 0 && a->workspace != nullptr &&
           a->workspace_bytes >= (int64_t)fs_window_prefill_tc_workspace(a) && ((uintptr_t)a->workspace & 15) == 0 &&
           (a->v.sn * 2) % 16 == 0 && (a->v.sh * 2) % 16 == 0 && (a->v.sb * 2) % 16 == 0 && encode_fn() != nullptr;
}

int fs_window_prefill_tc(const fsattn_window_prefill_t* a, cudaStream_t st) {
    bf16* qr = (bf16*)a->workspace;
    bf16* kr = qr + (size_t)a->B * a->H * a->N * TC_D;
    {
        const int64_t total = (int64_t)a->B * a->H * a->N * (TC_D / 16);
        const int64_t blocks = (total + 255) / 256;
        FS_REQUIRE(blocks < (1ll << 31), "window_prefill: too many rows");
        rope_qk_kernel<<<(unsigned)blocks, 256, 0, st>>>(*a, qr, kr);
        const int rc = fs_check_launch("rope_qk");
        if (rc != FSATTN_OK) return rc;
    }
    CUtensorMap tq, tk, tv;
    const cuuint64_t BH = (cuuint64_t)a->B * a->H;
    {
        const cuuint64_t dims[3] = {TC_D, (cuuint64_t)a->N, BH};
        const cuuint64_t strides[2] = {TC_D * 2, (cuuint64_t)a->N * TC_D * 2};
        const cuuint32_t box[3] = {TC_D, TC_BM, 1}, boxk[3] = {TC_D, TC_BN, 1};
        FS_REQUIRE(make_map(&tq, qr, 3, dims, strides, box) && make_map(&tk, kr, 3, dims, strides, boxk),
                   "window_prefill: cuTensorMapEncodeTiled failed for the rotated Q/K workspace");
    }
    {
        const cuuint64_t dims[4] = {TC_D, (cuuint64_t)a->N, (cuuint64_t)a->H, (cuuint64_t)a->B};
        const cuuint64_t strides[3] = {(cuuint64_t)a->v.sn * 2, (cuuint64_t)a->v.sh * 2, (cuuint64_t)(a->B > 1 ? a->v.sb : a->v.sn * a->N) * 2};
        const cuuint32_t box[4] = {TC_D, TC_BN, 1, 1};
        FS_REQUIRE(make_map(&tv, const_cast<void*>(a->v.ptr), 4, dims, strides, box), "window_prefill: cuTensorMapEncodeTiled failed for V");
    }
    static bool opted[16] = {false};
    int dev = 0;
    cudaGetDevice(&dev);
    const int smem = SM_TOTAL + 1024;
    if (dev >= 0 && dev < 16 && !opted[dev]) {
        if (cudaFuncSetAttribute(window_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess) {
            (void)cudaGetLastError();
            fs_set_error("window_prefill: cannot opt in to %d bytes of shared memory", smem);
            return FSATTN_ELAUNCH;
        }
        opted[dev] = true;
    }
    TcParams p;
    p.N = a->N; p.W = a->W; p.H = a->H;
    p.c2 = a->scale * 1.4426950408889634f;
    p.out = (bf16*)a->out;
    p.status = a->status;
    dim3 grid((a->N + TC_BM - 1) / TC_BM, a->B * a->H);
    window_tc_kernel<<<grid, TC_THREADS, smem, st>>>(tq, tk, tv, p);
    return fs_check_launch("window_prefill_tc");
}

// ---- allocation-free variant ------------------------------------------------------------------------------------------------
// Some hosts of this library may not create device memory at the moment they need a prefill: a serving process whose
// memory plan was fixed at start-up and hands out no further blocks, a plugin that runs inside another framework's step and
// is not allowed to call that framework's (or CUDA's) allocator from there, a caller on a latency path where cudaMalloc's
// implicit device synchronisation is unacceptable. For them the tensor-core window kernel is offered with its scratch (the
// rotated Q and K) in a fixed array that is part of the library image: every GPU that loads the library holds these
// FSATTN_WINDOW_STATIC_BYTES until the process exits, whether or not the entry point is ever called.
//
// The array's name below is only a host-side handle. The device address is looked up once per device (with that device
// current) by cudaGetSymbolAddress at the first call on that device, so that first call should happen before any stream capture.
// Every call uses the same array and leaves its last contents there; nothing in it has to start at zero (pass 0 rewrites
// every row pass 1 reads), but two calls that overlap on the GPU (different streams, or a graph replayed concurrently) would
// race on it.
static __device__ __align__(256) unsigned char g_window_static_scratch[FSATTN_WINDOW_STATIC_BYTES];

extern "C" int fsattn_window_prefill_static(const fsattn_window_prefill_t* a, fsattn_stream_t stream) {
    FS_REQUIRE(a != nullptr && a->q.ptr && a->k.ptr && a->v.ptr && a->cos && a->sin && a->out, "window_prefill_static: null pointer");
    FS_REQUIRE(a->B > 0 && a->H > 0 && a->N > 0 && a->pos0 >= 0, "window_prefill_static: bad sizes");
    FS_UNSUPPORTED(a->D != TC_D || a->W < TC_BN || a->W % TC_BN != 0,
                   "window_prefill_static: only head_dim 64 and windows that are multiples of 64 (got D=%d, W=%d)", a->D, a->W);
    const fsattn_bhnd_t* t[3] = {&a->q, &a->k, &a->v};
    for (int i = 0; i < 3; i++)
        FS_REQUIRE(((uintptr_t)t[i]->ptr & 15) == 0 && t[i]->sn % 8 == 0 && t[i]->sh % 8 == 0 && t[i]->sb % 8 == 0,
                   "window_prefill_static: Q, K and V rows must be 16-byte aligned");
    FS_REQUIRE(((uintptr_t)a->cos & 15) == 0 && ((uintptr_t)a->sin & 15) == 0 && ((uintptr_t)a->out & 15) == 0,
               "window_prefill_static: tables and output must be 16-byte aligned");
    const size_t need = fs_window_prefill_tc_workspace(a);
    if (need > (size_t)FSATTN_WINDOW_STATIC_BYTES) {
        fs_set_error("window_prefill_static: B*H*N = %lld rows need %zu bytes of scratch, the built-in array holds %d (B*H*N <= %d); "
                     "use fsattn_window_prefill with a caller-owned workspace", (long long)a->B * a->H * a->N, need,
                     FSATTN_WINDOW_STATIC_BYTES, FSATTN_WINDOW_STATIC_BYTES / (2 * TC_D * 2));
        return FSATTN_EINVAL;
    }
    FS_REQUIRE(encode_fn() != nullptr, "window_prefill_static: the driver does not export cuTensorMapEncodeTiled");
    // one-time set-up per device: the array's device address on the current device
    static void* dev_ptr[64] = {nullptr};
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
        (void)cudaGetLastError();
        fs_set_error("window_prefill_static: no current CUDA device");
        return FSATTN_ELAUNCH;
    }
    if (dev_ptr[dev] == nullptr) {
        void* p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_window_static_scratch);
        if (e != cudaSuccess || p == nullptr) {
            (void)cudaGetLastError();
            fs_set_error("window_prefill_static: cudaGetSymbolAddress failed: %s", cudaGetErrorString(e));
            return FSATTN_ELAUNCH;
        }
        dev_ptr[dev] = p;
    }
    fsattn_window_prefill_t b = *a;
    b.workspace = dev_ptr[dev];
    b.workspace_bytes = FSATTN_WINDOW_STATIC_BYTES;
    return fs_window_prefill_tc(&b, (cudaStream_t)stream);
}
