// FS-L bounded retention pool: fill of the slot store after a prefill. (Cell close, slot allocation, top-P refresh and
// the freeing of unreadable slots at decode time live in the fused decode step, fsl_decode.cu.)
#include "common.cuh"
#include "cell_warp.cuh"

// Pass 1, one CTA per (b,h): keep[c] = (c >= c_lo) or c in the block's top-P; slots are handed out in cell order.
__global__ void __launch_bounds__(256) slot_assign_kernel(const fsattn_slot_prefill_t a, int ncell, int c_lo) {
    extern __shared__ unsigned int bitmap[];     // one bit per cell: member of the top-P list
    __shared__ int warp_tot[8];
    __shared__ int running;
    const fsattn_fsl_state_t& st = a.st;
    const int bh = blockIdx.x;
    const int b = bh / st.H, h = bh - b * st.H;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    int32_t* slot_of = st.slot_of + b * st.so_sb + h * st.so_sh;
    int32_t* cell_in = st.cell_in + b * st.ci_sb + h * st.ci_sh;
    const int32_t* top_idx = st.top_idx + (int64_t)bh * st.P;
    const int nwords = (ncell + 31) / 32;
    for (int i = tid; i < nwords; i += 256) bitmap[i] = 0u;
    for (int64_t i = tid; i < st.cap_cells; i += 256) slot_of[i] = -1;
    for (int i = tid; i < st.n_slots; i += 256) cell_in[i] = -1;
    if (tid == 0) running = 0;
    __syncthreads();
    for (int p = tid; p < st.P; p += 256) {
        const int c = top_idx[p];
        if (c >= 0 && c < ncell) atomicOr(&bitmap[c >> 5], 1u << (c & 31));
    }
    __syncthreads();
    for (int c0 = 0; c0 < ncell; c0 += 256) {
        const int c = c0 + tid;
        const bool keep = c < ncell && (c >= c_lo || ((bitmap[c >> 5] >> (c & 31)) & 1u));
        const unsigned bal = __ballot_sync(FS_FULL, keep);
        if (lane == 0) warp_tot[warp] = __popc(bal);
        __syncthreads();
        int base = running;
        for (int w = 0; w < warp; w++) base += warp_tot[w];
        const int slot = base + __popc(bal & ((1u << lane) - 1u));
        if (keep) {
            if (slot < st.n_slots) { slot_of[c] = slot; cell_in[slot] = c; }
            else atomicAdd(st.status + FSATTN_ST_SLOT_OVERFLOW, 1);
        }
        __syncthreads();
        if (tid == 0) { int t = 0; for (int w = 0; w < 8; w++) t += warp_tot[w]; running += t; }
        __syncthreads();
    }
}

// Pass 2, one warp per (b,h,cell): kept cells are quantised into their slot and their mean key copied.
template <int D>
__global__ void __launch_bounds__(128) slot_fill_kernel(const fsattn_slot_prefill_t a, int ncell) {
    const fsattn_fsl_state_t& st = a.st;
    const int64_t w = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (w >= (int64_t)st.B * st.H * ncell) return;
    const int64_t bh = w / ncell;
    const int c = (int)(w - bh * ncell);
    const int b = (int)(bh / st.H), h = (int)(bh - (int64_t)b * st.H);
    const int slot = st.slot_of[b * st.so_sb + h * st.so_sh + c];
    if (slot < 0) return;
    int8_t* kq = st.kq + b * st.q_sb + h * st.q_sh + (int64_t)slot * FSATTN_CELL * D;
    int8_t* vq = st.vq + b * st.q_sb + h * st.q_sh + (int64_t)slot * FSATTN_CELL * D;
    bf16* ks = (bf16*)st.ks + b * st.sc_sb + h * st.sc_sh + slot;
    bf16* vs = (bf16*)st.vs + b * st.sc_sb + h * st.sc_sh + slot;
    CellRegs<D> r;
    cell_load_rows<D>(r, (const bf16*)a.k.ptr + b * a.k.sb + h * a.k.sh + (int64_t)c * FSATTN_CELL * a.k.sn, a.k.sn, lane);
    cell_quant_warp<D>(r, lane, kq, ks);
    cell_load_rows<D>(r, (const bf16*)a.v.ptr + b * a.v.sb + h * a.v.sh + (int64_t)c * FSATTN_CELL * a.v.sn, a.v.sn, lane);
    cell_quant_warp<D>(r, lane, vq, vs);
    const float* src = a.kbar_cells + b * a.kc_sb + h * a.kc_sh + (int64_t)c * D;
    float* dst = st.kbar + b * st.kbar_sb + h * st.kbar_sh + (int64_t)slot * D;
    for (int d = lane; d < D; d += 32) dst[d] = src[d];
}

extern "C" int fsattn_slot_prefill(const fsattn_slot_prefill_t* a, fsattn_stream_t stream) {
    FS_REQUIRE(a != nullptr, "slot_prefill: null args");
    const fsattn_fsl_state_t& st = a->st;
    FS_REQUIRE(st.store_mode == 2 && st.slot_of && st.cell_in && st.kq && st.vq && st.ks && st.vs && st.kbar && st.top_idx && st.status,
               "slot_prefill: needs a bounded store state");
    FS_REQUIRE(a->k.ptr && a->v.ptr && a->kbar_cells && a->N >= 0, "slot_prefill: null input");
    FS_UNSUPPORTED(st.D != 64 && st.D != 96 && st.D != 128, "slot_prefill: head_dim %d not in {64,96,128}", st.D);
    FS_REQUIRE(((uintptr_t)a->k.ptr & 15) == 0 && a->k.sn % 8 == 0 && a->k.sh % 8 == 0 && a->k.sb % 8 == 0 &&
               ((uintptr_t)a->v.ptr & 15) == 0 && a->v.sn % 8 == 0 && a->v.sh % 8 == 0 && a->v.sb % 8 == 0,
               "slot_prefill: K and V rows must be 16-byte aligned");
    const int ncell = a->N / FSATTN_CELL;
    FS_REQUIRE(ncell <= st.cap_cells, "slot_prefill: store sized for %lld cells, prompt has %d", (long long)st.cap_cells, ncell);
    const int blk = (a->N / st.Bq) * st.Bq;
    int m_vis = blk / FSATTN_CELL; if (m_vis > ncell) m_vis = ncell;
    int c_lo = 0;
    if (m_vis > 0) {
        const int d = blk - st.W;
        int fl = d >= 0 ? d / FSATTN_CELL : -((-d + FSATTN_CELL - 1) / FSATTN_CELL);
        c_lo = fl < m_vis - st.Wc ? fl : m_vis - st.Wc;
        if (c_lo < 0) c_lo = 0;
    }
    cudaStream_t s = (cudaStream_t)stream;
    const size_t smem = (size_t)((ncell + 31) / 32 + 1) * 4;
    FS_REQUIRE(smem <= 48 * 1024, "slot_prefill: %d cells exceed the membership bitmap", ncell);
    slot_assign_kernel<<<st.B * st.H, 256, smem, s>>>(*a, ncell, c_lo);
    int rc = fs_check_launch("slot_assign");
    if (rc != FSATTN_OK || ncell == 0) return rc;
    const int64_t warps = (int64_t)st.B * st.H * ncell;
    const unsigned blocks = (unsigned)((warps + 3) / 4);
    switch (st.D) {
        case 64: slot_fill_kernel<64><<<blocks, 128, 0, s>>>(*a, ncell); break;
        case 96: slot_fill_kernel<96><<<blocks, 128, 0, s>>>(*a, ncell); break;
        default: slot_fill_kernel<128><<<blocks, 128, 0, s>>>(*a, ncell); break;
    }
    return fs_check_launch("slot_fill");
}
