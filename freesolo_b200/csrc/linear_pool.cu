// The streaming FS-L cache (ref: src/fsattn/linear_cache.py) keeps a pool of C = P + Wc cell slots per (b,h): [0, P) the
// cells with the highest ceilings seen so far, [P, C) a ring of the newest cells. Two kernels, one CTA per (b,h) each:
//
//   linear_merge_kernel   at a 128-token block change: the newly completed cells (at most 32) against the top list - the P
//                         best of (list, new) by (ceiling desc, cell id asc) stay; an entering cell is written into the
//                         slot of a leaving one (ids, ceiling, mean key, its 32 K and V rows), nothing else moves; the
//                         newest Wc cells go into the ring at slot P + id mod Wc; the slots' validity (a ring cell that
//                         is also in the list counts once) is written for the selection.
//   linear_select_kernel  one query per thread against the <= 72 pool slots: score = (q . mean) scale + lam ceil
//                         erf(|p - centre| / (2 sigma)), the best kk by (score desc, cell id asc), returned as pool slots.
//
// The reference does both with gathers / concatenations / sorts over the whole pool per block (linear_cache.py:86-118,
// 154-170); here a block change touches the few kilobytes that change.
#include "common.cuh"

namespace {

constexpr int LP_MAXC = 160;      // most pool slots (P + Wc)
constexpr int LP_MAXNEW = 32;     // most new cells per merge
constexpr int LP_THREADS = 256;

__global__ void __launch_bounds__(LP_THREADS) linear_merge_kernel(const fsattn_linear_merge_t a) {
    const int b = blockIdx.x / a.H, h = blockIdx.x % a.H;
    const int tid = threadIdx.x;
    const int P = a.P, Wc = a.Wc, C = P + Wc, cnt = a.count, D = a.D, s = FSATTN_CELL;
    int* ids = a.ids + (int64_t)blockIdx.x * (C + 1);
    float* prio = a.prio + (int64_t)blockIdx.x * (C + 1);
    float* mean = a.mean + (int64_t)blockIdx.x * (C + 1) * D;
    bf16* pk = (bf16*)a.k + (int64_t)blockIdx.x * (C + 1) * s * D;
    bf16* pv = (bf16*)a.v + (int64_t)blockIdx.x * (C + 1) * s * D;
    unsigned char* valid = a.valid + (int64_t)blockIdx.x * C;
    const float* nprio = a.new_prio + (int64_t)blockIdx.x * cnt;
    const float* nmean = a.new_mean + (int64_t)blockIdx.x * cnt * D;
    const bf16* nk = (const bf16*)a.new_k + b * a.nk_sb + h * a.nk_sh;        // rows contiguous: cnt * 32 rows of D
    const bf16* nv = (const bf16*)a.new_v + b * a.nk_sb + h * a.nk_sh;

    __shared__ float c_prio[LP_MAXC + LP_MAXNEW];
    __shared__ int c_id[LP_MAXC + LP_MAXNEW];
    __shared__ unsigned char keep[LP_MAXC + LP_MAXNEW];
    __shared__ int target[LP_MAXNEW];             // pool slot an entering new cell takes, -1 = does not enter

    const int ncand = P + cnt;
    for (int i = tid; i < ncand; i += LP_THREADS) {
        c_prio[i] = i < P ? prio[i] : nprio[i - P];
        c_id[i] = i < P ? ids[i] : a.first_id + (i - P);
    }
    __syncthreads();
    // rank of every candidate by (ceiling desc, id asc); an empty slot (id -1) loses to everything
    for (int i = tid; i < ncand; i += LP_THREADS) {
        const int idi = c_id[i];
        const float pi = c_prio[i];
        int rank = 0;
        for (int j = 0; j < ncand; ++j) {
            const int idj = c_id[j];
            bool before;
            if (idj < 0) before = false;
            else if (idi < 0) before = true;
            else before = pool_before(c_prio[j], idj, pi, idi);
            rank += before ? 1 : 0;
        }
        if (idi < 0) {                            // empty slots among themselves: by slot index, after every real cell
            int real = 0;
            for (int j = 0; j < ncand; ++j) real += c_id[j] >= 0 ? 1 : 0;
            rank = real + i;
        }
        keep[i] = rank < P;
    }
    __syncthreads();
    if (tid == 0) {
        // the r-th entering new cell takes the r-th top slot that is empty or loses its cell (there are at least as many)
        int slot = 0;
        for (int j = 0; j < cnt; ++j) {
            target[j] = -1;
            if (!keep[P + j]) continue;
            while (slot < P && keep[slot] && c_id[slot] >= 0) ++slot;
            target[j] = slot < P ? slot : -1;
            ++slot;
        }
    }
    __syncthreads();
    // an empty slot is "kept" by the rank rule only if fewer than P real cells exist; it still receives an entering cell
    for (int j = 0; j < cnt; ++j) {
        const int tslot = target[j];
        const int ring = (Wc > 0 && j >= cnt - Wc) ? P + (a.first_id + j) % Wc : -1;
        for (int pass = 0; pass < 2; ++pass) {
            const int sl = pass == 0 ? tslot : ring;
            if (sl < 0) continue;
            if (tid == 0) { ids[sl] = a.first_id + j; prio[sl] = nprio[j]; }
            for (int d = tid; d < D; d += LP_THREADS) mean[(int64_t)sl * D + d] = nmean[(int64_t)j * D + d];
            const uint4* sk = (const uint4*)(nk + (int64_t)j * s * D);
            const uint4* sv = (const uint4*)(nv + (int64_t)j * s * D);
            uint4* dk = (uint4*)(pk + (int64_t)sl * s * D);
            uint4* dv = (uint4*)(pv + (int64_t)sl * s * D);
            for (int i = tid; i < s * D / 8; i += LP_THREADS) { dk[i] = sk[i]; dv[i] = sv[i]; }
        }
    }
    __syncthreads();
    // validity for the selection: a slot holds a cell, and a ring cell that is also in the top list counts once
    for (int i = tid; i < C; i += LP_THREADS) {
        const int id = ids[i];
        bool ok = id >= 0;
        if (ok && i >= P)
            for (int j = 0; j < P; ++j) ok &= ids[j] != id;
        valid[i] = ok ? 1 : 0;
    }
}

template <int D>
__global__ void __launch_bounds__(128) linear_select_kernel(const fsattn_linear_select_t a) {
    const int b = blockIdx.x / a.H, h = blockIdx.x % a.H;
    const int tid = threadIdx.x;
    const int C = a.C;
    const int* ids = a.ids + (int64_t)blockIdx.x * (C + 1);
    const float* prio = a.prio + (int64_t)blockIdx.x * (C + 1);
    const float* mean = a.mean + (int64_t)blockIdx.x * (C + 1) * D;
    const unsigned char* valid = a.valid + (int64_t)blockIdx.x * C;
    extern __shared__ __align__(16) float sm[];
    float* s_mean = sm;                           // C x D
    float* s_pc = s_mean + (size_t)C * D;         // lam * ceiling per slot
    float* s_cen = s_pc + C;                      // centre position per slot
    int* s_id = (int*)(s_cen + C);                // cell id, -1 = not a candidate
    const float lam = a.lam[h], two_sigma = f_mul(2.0f, a.sigma[h]);
    for (int i = tid; i < C * D; i += 128) s_mean[i] = mean[i];
    for (int i = tid; i < C; i += 128) {
        const int id = ids[i];
        s_id[i] = valid[i] ? id : -1;
        s_pc[i] = f_mul(lam, prio[i]);
        s_cen[i] = f_mul((float)id + 0.5f, (float)FSATTN_CELL);
    }
    __syncthreads();
    if (tid >= a.n) return;
    const bf16* q = (const bf16*)a.q.ptr + b * a.q.sb + h * a.q.sh + (int64_t)tid * a.q.sn;
    float qv[D];
#pragma unroll
    for (int v = 0; v < D / 8; ++v) {
        const uint4 w = *(const uint4*)(q + v * 8);
        qv[v * 8 + 0] = bf_lo(w.x); qv[v * 8 + 1] = bf_hi(w.x); qv[v * 8 + 2] = bf_lo(w.y); qv[v * 8 + 3] = bf_hi(w.y);
        qv[v * 8 + 4] = bf_lo(w.z); qv[v * 8 + 5] = bf_hi(w.z); qv[v * 8 + 6] = bf_lo(w.w); qv[v * 8 + 7] = bf_hi(w.w);
    }
    const float qpos = (float)(a.pos0 + tid);
    float bs[4];
    int bi[4], bslot[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) { bs[i] = -INFINITY; bi[i] = 0x7fffffff; bslot[i] = -1; }
    for (int c = 0; c < C; ++c) {
        const int id = s_id[c];
        if (id < 0) continue;
        const float* m = s_mean + (size_t)c * D;
        float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
#pragma unroll
        for (int d = 0; d < D; d += 4) {
            s0 = fmaf(qv[d], m[d], s0); s1 = fmaf(qv[d + 1], m[d + 1], s1);
            s2 = fmaf(qv[d + 2], m[d + 2], s2); s3 = fmaf(qv[d + 3], m[d + 3], s3);
        }
        float score = f_mul((s0 + s1) + (s2 + s3), a.scale);
        if (!a.content_only) score = f_add(score, f_mul(s_pc[c], erff(f_div(fabsf(qpos - s_cen[c]), two_sigma))));
        // sorted insert: (score desc, cell id asc)
        if (score > bs[3] || (score == bs[3] && id < bi[3])) {
            bs[3] = score; bi[3] = id; bslot[3] = c;
#pragma unroll
            for (int i = 3; i > 0; --i) {
                if (bs[i] > bs[i - 1] || (bs[i] == bs[i - 1] && bi[i] < bi[i - 1])) {
                    const float ts = bs[i]; bs[i] = bs[i - 1]; bs[i - 1] = ts;
                    const int ti = bi[i]; bi[i] = bi[i - 1]; bi[i - 1] = ti;
                    const int tc = bslot[i]; bslot[i] = bslot[i - 1]; bslot[i - 1] = tc;
                }
            }
        }
    }
    int* out = a.sel + ((int64_t)blockIdx.x * a.n_pad + tid) * a.kk_out;
    int* oid = a.sel_ids ? a.sel_ids + ((int64_t)blockIdx.x * a.n_pad + tid) * a.kk_out : nullptr;
    for (int i = 0; i < a.kk_out; ++i) {
        const bool ok = i < a.kk && i < 4 && bslot[i < 4 ? i : 3] >= 0;
        out[i] = ok ? bslot[i] : -1;
        if (oid) oid[i] = ok ? bi[i] : -1;
    }
}

}  // namespace

extern "C" int fsattn_linear_merge(const fsattn_linear_merge_t* a, fsattn_stream_t stream) {
    FS_REQUIRE(a && a->ids && a->prio && a->mean && a->k && a->v && a->valid, "linear_merge: null pool buffer");
    FS_REQUIRE(a->B > 0 && a->H > 0 && a->P >= 1 && a->Wc >= 0 && a->P + a->Wc <= LP_MAXC, "linear_merge: pool of %d + %d slots (at most %d)",
               a->P, a->Wc, LP_MAXC);
    FS_REQUIRE(a->count >= 0 && a->count <= LP_MAXNEW && a->first_id >= 0, "linear_merge: %d new cells (at most %d)", a->count, LP_MAXNEW);
    FS_UNSUPPORTED(a->D != 64 && a->D != 96 && a->D != 128, "linear_merge: head_dim %d not in {64,96,128}", a->D);
    FS_REQUIRE(a->count == 0 || (a->new_prio && a->new_mean && a->new_k && a->new_v), "linear_merge: null new-cell buffer");
    FS_REQUIRE(((uintptr_t)a->k & 15) == 0 && ((uintptr_t)a->v & 15) == 0 && ((uintptr_t)a->new_k & 15) == 0 && ((uintptr_t)a->new_v & 15) == 0 &&
               a->nk_sb % 8 == 0 && a->nk_sh % 8 == 0, "linear_merge: K/V rows must be 16-byte aligned");
    linear_merge_kernel<<<a->B * a->H, LP_THREADS, 0, (cudaStream_t)stream>>>(*a);
    return fs_check_launch("linear_merge_kernel");
}

extern "C" int fsattn_linear_select(const fsattn_linear_select_t* a, fsattn_stream_t stream) {
    FS_REQUIRE(a && a->ids && a->prio && a->mean && a->valid && a->q.ptr && a->lam && a->sigma && a->sel, "linear_select: null pointer");
    FS_REQUIRE(a->B > 0 && a->H > 0 && a->C >= 1 && a->C <= LP_MAXC, "linear_select: %d pool slots (1..%d)", a->C, LP_MAXC);
    FS_REQUIRE(a->n >= 1 && a->n <= 128 && a->n_pad >= a->n, "linear_select: %d queries per call (1..128)", a->n);
    FS_REQUIRE(a->kk >= 0 && a->kk <= 4 && a->kk_out >= a->kk && a->kk_out >= 1, "linear_select: kk = %d (0..4)", a->kk);
    FS_UNSUPPORTED(a->D != 64 && a->D != 96 && a->D != 128, "linear_select: head_dim %d not in {64,96,128}", a->D);
    FS_REQUIRE(((uintptr_t)a->q.ptr & 15) == 0 && a->q.sn % 8 == 0, "linear_select: query rows must be 16-byte aligned");
    const size_t smem = (size_t)a->C * a->D * 4 + (size_t)a->C * 12;
    cudaStream_t st = (cudaStream_t)stream;
    cudaError_t e = cudaSuccess;
    switch (a->D) {
        case 64: linear_select_kernel<64><<<a->B * a->H, 128, smem, st>>>(*a); break;
        case 96:
            e = cudaFuncSetAttribute(linear_select_kernel<96>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
            if (e == cudaSuccess) linear_select_kernel<96><<<a->B * a->H, 128, smem, st>>>(*a);
            break;
        default:
            e = cudaFuncSetAttribute(linear_select_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
            if (e == cudaSuccess) linear_select_kernel<128><<<a->B * a->H, 128, smem, st>>>(*a);
            break;
    }
    if (e != cudaSuccess) {
        cudaGetLastError();
        fs_set_error("linear_select: shared-memory opt-in failed: %s", cudaGetErrorString(e));
        return FSATTN_ELAUNCH;
    }
    return fs_check_launch("linear_select_kernel");
}
