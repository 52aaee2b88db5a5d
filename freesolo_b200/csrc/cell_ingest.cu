// Chunk statistics (chunk-mean key, ceiling) and the per-cell int8 KV codec in one streaming pass.
//
// HBM-bound: every cell (32 tokens x D bf16) is read exactly once with 16-byte loads, one warp per (b,h,cell).
// Algorithmic bytes per cell: 32*D*2 read per tensor; written: D*4 + 4 (statistics), 32*D + 2 per quantised tensor.
#include "common.cuh"
#include "cell_warp.cuh"

template <int D>
__global__ void __launch_bounds__(128) cell_ingest_kernel(const fsattn_cell_ingest_t a) {
    const int64_t w = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    const int64_t total = (int64_t)a.B * a.H * a.ncell;
    if (w >= total) return;
    const int64_t bh = w / a.ncell;
    const int c = (int)(w - bh * a.ncell);
    const int b = (int)(bh / a.H), h = (int)(bh - (int64_t)b * a.H);
    const int co = a.cell0 + c;

    {
        const bf16* kp = (const bf16*)a.k.ptr + b * a.k.sb + h * a.k.sh + (int64_t)c * FSATTN_CELL * a.k.sn;
        CellRegs<D> r;
        cell_load_rows<D>(r, kp, a.k.sn, lane);
        if (a.kbar != nullptr || a.ceil != nullptr) {
            float* kb = a.kbar ? a.kbar + b * a.kbar_sb + h * a.kbar_sh + (int64_t)co * D : nullptr;
            float* cl = a.ceil ? a.ceil + b * a.ceil_sb + h * a.ceil_sh + co : nullptr;
            cell_stats_warp<D>(r, lane, kb, cl);
        }
        if (a.kq != nullptr) {
            int8_t* q = a.kq + b * a.q_sb + h * a.q_sh + (int64_t)co * FSATTN_CELL * D;
            bf16* sc = (bf16*)a.ks + b * a.sc_sb + h * a.sc_sh + co;
            cell_quant_warp<D>(r, lane, q, sc);
        }
    }
    if (a.v.ptr != nullptr && a.vq != nullptr) {
        const bf16* vp = (const bf16*)a.v.ptr + b * a.v.sb + h * a.v.sh + (int64_t)c * FSATTN_CELL * a.v.sn;
        CellRegs<D> r;
        cell_load_rows<D>(r, vp, a.v.sn, lane);
        int8_t* q = a.vq + b * a.q_sb + h * a.q_sh + (int64_t)co * FSATTN_CELL * D;
        bf16* sc = (bf16*)a.vs + b * a.sc_sb + h * a.sc_sh + co;
        cell_quant_warp<D>(r, lane, q, sc);
    }
}

extern "C" int fsattn_cell_ingest(const fsattn_cell_ingest_t* a, fsattn_stream_t stream) {
    FS_REQUIRE(a != nullptr && a->k.ptr != nullptr, "cell_ingest: null K");
    FS_REQUIRE(a->B > 0 && a->H > 0 && a->ncell >= 0 && a->cell0 >= 0, "cell_ingest: bad sizes");
    FS_UNSUPPORTED(a->D != 64 && a->D != 96 && a->D != 128, "cell_ingest: head_dim %d not in {64,96,128}", a->D);
    FS_REQUIRE(((uintptr_t)a->k.ptr & 15) == 0 && a->k.sn % 8 == 0 && a->k.sh % 8 == 0 && a->k.sb % 8 == 0,
               "cell_ingest: K rows must be 16-byte aligned");
    if (a->v.ptr != nullptr)
        FS_REQUIRE(((uintptr_t)a->v.ptr & 15) == 0 && a->v.sn % 8 == 0 && a->v.sh % 8 == 0 && a->v.sb % 8 == 0,
                   "cell_ingest: V rows must be 16-byte aligned");
    if (a->kq != nullptr) {
        FS_REQUIRE(a->ks != nullptr, "cell_ingest: kq without ks");
        FS_REQUIRE(((uintptr_t)a->kq & 7) == 0 && a->q_sb % 8 == 0 && a->q_sh % 8 == 0, "cell_ingest: int8 rows must be 8-byte aligned");
    }
    if (a->vq != nullptr) {
        FS_REQUIRE(a->vs != nullptr && a->v.ptr != nullptr, "cell_ingest: vq needs vs and V");
        FS_REQUIRE(((uintptr_t)a->vq & 7) == 0, "cell_ingest: int8 rows must be 8-byte aligned");
    }
    if (a->kbar != nullptr)
        FS_REQUIRE(((uintptr_t)a->kbar & 15) == 0 && a->kbar_sb % 4 == 0 && a->kbar_sh % 4 == 0, "cell_ingest: kbar must be 16-byte aligned");
    if (a->ncell == 0) return FSATTN_OK;
    const int64_t warps = (int64_t)a->B * a->H * a->ncell;
    const int64_t blocks = (warps + 3) / 4;
    FS_REQUIRE(blocks < (1ll << 31), "cell_ingest: too many cells");
    cudaStream_t st = (cudaStream_t)stream;
    switch (a->D) {
        case 64: cell_ingest_kernel<64><<<(unsigned)blocks, 128, 0, st>>>(*a); break;
        case 96: cell_ingest_kernel<96><<<(unsigned)blocks, 128, 0, st>>>(*a); break;
        default: cell_ingest_kernel<128><<<(unsigned)blocks, 128, 0, st>>>(*a); break;
    }
    return fs_check_launch("cell_ingest");
}

// ---- dequantise ----------------------------------------------------------------------------------------------------
__global__ void __launch_bounds__(256) dequant_kernel(const fsattn_dequant_t a) {
    // one thread per 16 codes; rows of one (b,h) are contiguous
    const int per_row = a.D / 16;
    const int64_t per_bh = a.nrows * per_row;
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= per_bh * a.B * a.H) return;
    const int64_t bh = i / per_bh;
    const int64_t r = i - bh * per_bh;
    const int64_t row = r / per_row;
    const int e = (int)(r - row * per_row) * 16;
    const int b = (int)(bh / a.H), h = (int)(bh - (int64_t)b * a.H);
    const uint4 w = *reinterpret_cast<const uint4*>(a.q + b * a.q_sb + h * a.q_sh + row * a.D + e);
    const float sc = __bfloat162float(((const bf16*)a.sc)[b * a.sc_sb + h * a.sc_sh + row / FSATTN_CELL]);
    float x[16];
    unpack4_i8(w.x, x); unpack4_i8(w.y, x + 4); unpack4_i8(w.z, x + 8); unpack4_i8(w.w, x + 12);
    uint4 o0, o1;
    o0.x = pack_bf2(f_mul(x[0], sc), f_mul(x[1], sc));   o0.y = pack_bf2(f_mul(x[2], sc), f_mul(x[3], sc));
    o0.z = pack_bf2(f_mul(x[4], sc), f_mul(x[5], sc));   o0.w = pack_bf2(f_mul(x[6], sc), f_mul(x[7], sc));
    o1.x = pack_bf2(f_mul(x[8], sc), f_mul(x[9], sc));   o1.y = pack_bf2(f_mul(x[10], sc), f_mul(x[11], sc));
    o1.z = pack_bf2(f_mul(x[12], sc), f_mul(x[13], sc)); o1.w = pack_bf2(f_mul(x[14], sc), f_mul(x[15], sc));
    uint4* op = reinterpret_cast<uint4*>((bf16*)a.out + b * a.o_sb + h * a.o_sh + row * a.D + e);
    op[0] = o0;
    op[1] = o1;
}

extern "C" int fsattn_dequant_cells(const fsattn_dequant_t* a, fsattn_stream_t stream) {
    FS_REQUIRE(a != nullptr && a->q != nullptr && a->sc != nullptr && a->out != nullptr, "dequant: null pointer");
    FS_REQUIRE(a->B > 0 && a->H > 0 && a->nrows >= 0 && a->D % 16 == 0, "dequant: bad sizes");
    FS_REQUIRE(((uintptr_t)a->q & 15) == 0 && a->q_sb % 16 == 0 && a->q_sh % 16 == 0, "dequant: codes must be 16-byte aligned");
    FS_REQUIRE(((uintptr_t)a->out & 15) == 0 && a->o_sb % 8 == 0 && a->o_sh % 8 == 0, "dequant: output must be 16-byte aligned");
    if (a->nrows == 0) return FSATTN_OK;
    const int64_t n = a->nrows * (a->D / 16) * a->B * a->H;
    const int64_t blocks = (n + 255) / 256;
    FS_REQUIRE(blocks < (1ll << 31), "dequant: too many rows");
    dequant_kernel<<<(unsigned)blocks, 256, 0, (cudaStream_t)stream>>>(*a);
    return fs_check_launch("dequant_cells");
}
