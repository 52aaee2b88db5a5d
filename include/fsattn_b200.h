/* C ABI of libfsattn_b200: hand-written sm_100a kernels for the FreeSolo sparse-attention inference hot path.
 *
 * The reference project (zekun-shi/freesolo) has no C ABI of its own: its native kernels are CUDA sources compiled at
 * run time and launched from Python with raw device pointers (src/fsattn/fsl_select_cuda.py:132-142,
 * src/fsattn/fsb_beam_cuda.py:224-237) or Triton kernels. Each entry point below names the reference function or
 * kernel launch it replaces. The conventions mirror how the reference launches its kernels:
 *
 *  - every pointer is a DEVICE pointer owned by the caller; the library never allocates or frees device memory
 *    (outputs are pre-allocated by the caller, as the reference does with torch.empty before each launch);
 *  - every call is asynchronous on the CUDA stream passed in (a cudaStream_t cast to void*; NULL = legacy default
 *    stream), does not synchronise, and reads positions from device scalars, so it may be captured in a CUDA graph;
 *  - strides are in ELEMENTS of the tensor's dtype; the innermost (head-dim) stride is always 1;
 *  - return value 0 = launched; negative = rejected on the host before any launch (fsattn_last_error() has the text).
 *    Conditions detected on the device (slot overflow, pool cell without a slot) are counted in a caller-provided
 *    int32 status buffer, read by the caller where the reference reads its own fault counters
 *    (src/fsattn/kv_bounded.py:104,225-228).
 *
 * Tensor vocabulary: B batch, H heads, D head dim (64, 96 or 128), N tokens, s = 32 tokens per cell ("chunk"),
 * Bq = 128 queries per block, kk cells read per query, P pool size, Wc newest-cell slots, W window.
 */
#ifndef FSATTN_B200_H
#define FSATTN_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define FSATTN_API __attribute__((visibility("default")))
#else
#define FSATTN_API
#endif

#define FSATTN_OK 0
#define FSATTN_EINVAL (-1)        /* bad argument (shape, alignment, null pointer) */
#define FSATTN_EUNSUPPORTED (-2)  /* a configuration the kernels do not cover (no fallback exists) */
#define FSATTN_ELAUNCH (-3)       /* the CUDA runtime refused the launch */

#define FSATTN_CELL 32            /* tokens per cell the kernels are specialised for */
#define FSATTN_MAX_POOL 128       /* P + Wc upper bound */
#define FSATTN_MAX_KK 8

/* status words written by device code (int32 each) */
#define FSATTN_ST_SLOT_OVERFLOW 0 /* completed cell found no free slot (bounded store) */
#define FSATTN_ST_POOL_NO_SLOT 1  /* readable pool cell without a slot (bounded store) */
#define FSATTN_ST_BAD_INDEX 2     /* an index failed a bounds check and its access was skipped */
#define FSATTN_ST_WORDS 4

typedef void* fsattn_stream_t;

FSATTN_API int fsattn_version(void);
FSATTN_API const char* fsattn_last_error(void);
/* Per-device one-time setup (dynamic shared-memory opt-in of the kernels). Call once per device before other calls. */
FSATTN_API int fsattn_init(int device);

/* ---- a (B,H,N,D) view with unit inner stride, bf16 ------------------------------------------------------------- */
typedef struct {
    const void* ptr;
    int64_t sb, sh, sn; /* element strides of batch, head, token */
} fsattn_bhnd_t;

/* ---- chunk statistics + int8 codec ------------------------------------------------------------------------------
 * Replaces: FSKVCache._cell_stats_of / fsl_select_cuda.cache_cell_stats (experiments/scaling/kv_cache.py:274-285,
 * src/fsattn/fsl_select.cu:79-125), kv_int8.quantize_cells_fast / dequant_cells (src/fsattn/kv_int8.py:82-118).
 * One pass over ncell completed cells of K (and V): any of the outputs may be NULL to skip it.
 *   kbar  (B,H,*,D) fp32: chunk-mean key, mean taken in bf16 like the reference (bf16-rounded value stored as fp32)
 *   ceil  (B,H,*)   fp32: largest token-key L2 norm of the cell
 *   kq,vq (B,H,*,D) int8 codes; ks,vs (B,H,*) bf16 scales: scale = bf16(max|x|/127) (1.0 if 0), q = rint(x/scale)
 * Cells [0, ncell) of the inputs are written at cell index cell0 + c of the outputs. */
typedef struct {
    fsattn_bhnd_t k, v; /* v.ptr may be NULL */
    int32_t B, H, D, ncell, cell0;
    float* kbar; int64_t kbar_sb, kbar_sh;   /* cell stride = D */
    float* ceil; int64_t ceil_sb, ceil_sh;   /* cell stride = 1 */
    int8_t* kq; int8_t* vq; int64_t q_sb, q_sh; /* row stride = D */
    void* ks; void* vs; int64_t sc_sb, sc_sh;   /* bf16, cell stride = 1 */
} fsattn_cell_ingest_t;
FSATTN_API int fsattn_cell_ingest(const fsattn_cell_ingest_t* a, fsattn_stream_t stream);

/* x = bf16(f32(q) * f32(scale[row / 32])) for rows [0, nrows) of every (b,h). Replaces kv_int8.dequant_cells
 * (src/fsattn/kv_int8.py:63-71). */
typedef struct {
    const int8_t* q; int64_t q_sb, q_sh;
    const void* sc; int64_t sc_sb, sc_sh;
    void* out; int64_t o_sb, o_sh; /* bf16 (B,H,*,D), row stride D */
    int32_t B, H, D; int64_t nrows;
} fsattn_dequant_t;
FSATTN_API int fsattn_dequant_cells(const fsattn_dequant_t* a, fsattn_stream_t stream);

/* ---- FS-L prefix top-P ---------------------------------------------------------------------------------------------
 * Replaces attention.py:766-778 (topk of the masked ceilings per block) / fsl_topp, fsl_topp_par
 * (src/fsattn/fsl_select.cu:247-391). For every query block n in [0, nb): the min(P, vis_n) best cells among the
 * vis_n = min(ncell, n*Bq/32) visible ones under (ceiling desc, cell index asc), in that order; unused slots -1.
 * topp (B*H, nb, P) int32. */
typedef struct {
    const float* ceil; int64_t ceil_sb, ceil_sh;
    int32_t B, H, ncell, Bq, nb, P;
    int32_t* topp;
} fsattn_fsl_topp_t;
FSATTN_API int fsattn_fsl_prefix_topp(const fsattn_fsl_topp_t* a, fsattn_stream_t stream);

/* ---- FS-L prefill selection -----------------------------------------------------------------------------------------
 * Replaces attention.py:779-821 / fsl_prep + fsl_select + fsl_fused (src/fsattn/fsl_select.cu:396-769): candidate
 * slots = top-P list of the block, then the Wc newest visible cells; score = (q.kbar)*scale + lam*ceil*erf(|p-cen|/
 * (2 sigma)) in fp32, -1e9 for slots that are invalid, invisible or repeat an earlier slot's cell; per query the kk
 * best by (score desc, slot asc); sel holds the cell id or -1. sel (B,H,nb*Bq,kk) int32; queries >= N are padding
 * and are scored as zero vectors like the reference. margin (optional, same leading shape, fp32): smallest gap
 * between consecutive entries of the best kk+1 scores. */
typedef struct {
    fsattn_bhnd_t q;
    const float* kbar; int64_t kbar_sb, kbar_sh;
    const float* ceil; int64_t ceil_sb, ceil_sh;
    const int32_t* topp; /* (B*H, nb, P) */
    const float* lam; const float* sigma; /* (H) */
    int32_t B, H, D, N, ncell, Bq, nb, P, Wc, kk;
    float scale;
    int32_t* sel; float* margin;
    int32_t topp_nb; /* blocks per head in the topp buffer when it holds more than nb (0: nb) */
    int32_t impl;    /* 0: tensor-core dot products where the shape allows (head_dim 64, Bq 128, P+Wc <= 80); 1: CUDA-core kernel */
} fsattn_fsl_select_t;
FSATTN_API int fsattn_fsl_select(const fsattn_fsl_select_t* a, fsattn_stream_t stream);

/* ---- dense FS variant (no candidate pool): selection over every visible cell ---------------------------------------------
 * Prefill: replaces the dense branch of FSAttn._lr_cell_topk (src/fsattn/attention.py:362-423 with
 * _cell_select_blk_logits, 472-517) and its native kernel fsl_dense_fused (src/fsattn/fsl_select.cu:772-1018): for every
 * query the kk best of ALL cells that end at or before its query block, score = (q . Kbar_c) * scale + lam * ceil_c *
 * erf(|p - (c + 0.5) 32| / (2 sigma)), order (score desc, cell asc), -1 where fewer than kk cells are visible.
 * q (B,H,N,D) bf16 view; kbar (B,H,>=ncell,D) fp32 holding bf16-exact values (row stride D); ceil (B,H,>=ncell) fp32;
 * sel (B,H,nb*Bq,kk) int32. Tensor-core kernel (tcgen05 + TMEM + TMA): head_dim 64, Bq = 128, kk <= 4; anything else is
 * refused. workspace: caller-owned scratch of fsattn_fs_dense_workspace_bytes() bytes, 16-byte aligned (bf16 copy of the
 * mean keys and lam * ceil per cell). status (optional int32) counts bounded waits that ran out. */
typedef struct {
    fsattn_bhnd_t q;
    const float* kbar; int64_t kbar_sb, kbar_sh;
    const float* ceil; int64_t ceil_sb, ceil_sh;
    const float* lam; const float* sigma;  /* (H) fp32 */
    int32_t B, H, D, N, ncell, Bq, nb, kk;
    float scale;
    int32_t* sel;
    void* workspace; int64_t workspace_bytes;
    int32_t* status;
} fsattn_fs_dense_select_t;
FSATTN_API int64_t fsattn_fs_dense_workspace_bytes(int32_t B, int32_t H, int32_t ncell, int32_t D);
FSATTN_API int fsattn_fs_dense_select(const fsattn_fs_dense_select_t* a, fsattn_stream_t stream);

/* Decode: replaces FSAttn._lr_decode_step_dense (src/fsattn/attention.py:1159-1185) and fsl_dense_decode_topk
 * (src/fsattn/fsl_select.cu:1026-1164): one query per (b,h) at position *pos scores the cells [0, min(blk_start / 32,
 * ncell_cap)) with blk_start = (*pos / Bq) * Bq and keeps the kk best. The cells are split over `splits` CTAs (1, 2, 4 or
 * 8: a thread-block cluster whose partial lists meet in rank 0's shared memory). sel (B,H,kk) int32 feeds
 * fsattn_fsl_decode_step through ext_sel. kbar (B,H,>=cells,D) fp32, ceil (B,H,>=cells) fp32; q (B,H,D) bf16 (strides sb, sh). */
typedef struct {
    const void* q; int64_t q_sb, q_sh;
    const float* kbar; int64_t kbar_sb, kbar_sh;
    const float* ceil; int64_t ceil_sb, ceil_sh;
    const float* lam; const float* sigma;
    const int64_t* pos;
    int32_t B, H, D, Bq, kk, ncell_cap, splits, pdl;
    float scale;
    int32_t* sel;
} fsattn_fs_dense_decode_select_t;
FSATTN_API int fsattn_fs_dense_decode_select(const fsattn_fs_dense_decode_select_t* a, fsattn_stream_t stream);

/* ---- window branch, prefill -----------------------------------------------------------------------------------------
 * Replaces FSAttn._short_range / _chunked_rope_window (src/fsattn/attention.py:225-259) and
 * local_attention._batched_sliding_window_rope (src/utils/local_attention.py:191-235): causal band softmax attention
 * max(0,p-W) <= j <= p with rotate-half RoPE applied to Q and K at absolute positions pos0 + i. cos/sin (L,D) bf16
 * tables (row stride D). out (B,N,H,D) bf16 = W_o's input layout. */
typedef struct {
    fsattn_bhnd_t q, k, v;
    const void* cos; const void* sin;
    int32_t B, H, D, N, W, pos0;
    float scale;
    void* out; /* (B,N,H*D) bf16 contiguous */
    int32_t impl; /* 0 = default (tensor-core kernel when the shape allows), 1 = force the CUDA-core kernel */
    /* scratch for the tensor-core kernel: the rotated Q and K, 2*B*H*N*D*2 bytes, 16-byte aligned (caller-owned; the
     * kernel is used when head_dim = 64, W is a multiple of 64 and this is large enough, else the CUDA-core kernel runs) */
    void* workspace; int64_t workspace_bytes;
    int32_t* status; /* optional int32: incremented when a bounded wait inside the tensor-core kernel ran out */
} fsattn_window_prefill_t;
FSATTN_API int fsattn_window_prefill(const fsattn_window_prefill_t* a, fsattn_stream_t stream);

/* The same tensor-core window attention for callers that cannot obtain device memory at call time (a process with a frozen
 * memory plan, a plugin that must not touch its host framework's allocator, a latency path that cannot afford cudaMalloc's
 * device synchronisation). It has no counterpart in the reference, which allocates through PyTorch wherever it likes.
 * The scratch for the rotated Q and K is a fixed array inside the library (FSATTN_WINDOW_STATIC_BYTES on every GPU that loads
 * it, until the process exits); a->workspace and a->workspace_bytes are ignored and nothing is allocated or freed.
 * Limits: head_dim 64, W a multiple of 64, and 2*B*H*N*64*2 bytes <= FSATTN_WINDOW_STATIC_BYTES, i.e. B*H*N <= 131072 rows;
 * anything else is rejected with FSATTN_EINVAL / FSATTN_EUNSUPPORTED and a message. The first call on a device looks up the
 * array's device address: make that call before capturing a stream. All calls share the array, so calls that overlap on
 * the GPU race on it; consecutive calls on one stream are safe and need no clearing in between. */
#define FSATTN_WINDOW_STATIC_BYTES (32 * 1024 * 1024)
FSATTN_API int fsattn_window_prefill_static(const fsattn_window_prefill_t* a, fsattn_stream_t stream);

/* ---- fused readout + combine, prefill ---------------------------------------------------------------------------------
 * Replaces FSAttn._cell_fused_lr / readout_triton.readout_combine (src/fsattn/attention.py:344-361,
 * src/fsattn/readout_triton.py:34-159) and indexed_cell_attention (src/fsattn/cell_select_triton.py:97-282):
 * per query softmax attention over the tokens (tok < query position) of its valid distinct selected cells,
 * o rounded to bf16, lr = (o * rsqrt(mean(o^2)+eps)) * norm_w, y = bf16(sr + lrs[h] * lr).
 * sr and y are (B,N,H*D) bf16; y may alias sr (in place, as the reference does). */
typedef struct {
    fsattn_bhnd_t q, k, v;
    const int32_t* sel; int64_t sel_sb, sel_sh; /* (B,H,*,kk), row stride kk */
    const void* sr; void* y;
    const float* norm_w; const float* lrs;
    int32_t B, H, D, N, n_kv, Bq, kk, q_pos0;
    float scale, eps;
    int32_t impl; /* 0 = choose; 1 = CUDA-core kernels; 2 = tensor-core tiles (whole 128-query blocks, head_dim 64) */
} fsattn_readout_combine_t;
FSATTN_API int fsattn_readout_combine(const fsattn_readout_combine_t* a, fsattn_stream_t stream);

/* ---- FS-L decode state + fused decode step -----------------------------------------------------------------------------
 * One layer's decode-time KV state. store_mode: 0 = bf16 full store, 1 = int8 full store (kv_int8), 2 = int8 bounded
 * slot store (kv_bounded.SlotStore: rows of cell c live at slot_of[c]*32 + t%32). Layout per (b,h):
 *   kbuf,vbuf (cap,D) bf16 [mode 0]; kq,vq (rows,D) int8 + ks,vs (cells|slots) bf16 [modes 1,2];
 *   khot,vhot (32,D) bf16 open cell [modes 1,2]; kbar (cells|slots, D) fp32; ceil (cells) fp32;
 *   slot_of (cells) int32, cell_in (slots) int32 [mode 2]; top_idx (P) int32 = the block's top-P cells in pool order,
 *   top_blk (1) int32 = block start that list is valid for; pool_* = the gathered candidate pool (see below).
 * Rows below (pos/32)*32 are completed cells; later rows are the open cell. */
typedef struct {
    int32_t store_mode, B, H, D, P, Wc, W, Bq, kk, n_slots;
    int64_t cap_rows, cap_cells;
    void* kbuf; void* vbuf; int64_t buf_sb, buf_sh;
    int8_t* kq; int8_t* vq; int64_t q_sb, q_sh;
    void* ks; void* vs; int64_t sc_sb, sc_sh;
    void* khot; void* vhot; int64_t hot_sb, hot_sh;
    float* kbar; int64_t kbar_sb, kbar_sh;
    float* ceil; int64_t ceil_sb, ceil_sh;
    int32_t* slot_of; int64_t so_sb, so_sh;
    int32_t* cell_in; int64_t ci_sb, ci_sh;
    int32_t* top_idx; int32_t* top_blk; /* (B,H,P), (B,H) contiguous */
    /* the current block's candidate pool, gathered once per block by the decode step so that the other Bq-1 steps read
     * it without any index indirection: pool_kbar (B,H,P+Wc,D) fp32 mean keys, pool_meta (B,H,P+Wc,4) int32 =
     * {cell id or -1 when the slot is not selectable, row base (cell or slot index), ceiling bits, 0}, pool_blk (B,H)
     * int32 = block start the pool is valid for (-1: rebuild at the next step). All contiguous. */
    float* pool_kbar; int32_t* pool_meta; int32_t* pool_blk;
    int32_t* status;                    /* FSATTN_ST_WORDS int32 */
} fsattn_fsl_state_t;

/* One decode token of one FS-L layer in ONE launch. Replaces the chain of FSAttn.graph_decode_layer
 * (src/fsattn/attention.py:1493-1559): _sr_kv_rope(_int8)_kernel + 2 einsums + _sr_softmax_cast_kernel (window,
 * src/utils/trunk_triton.py:194-480,1086-1211), _lrc_comb_int8_kernel / _fsl_lr_decode_combine_kernel (score the
 * pool, top-kk, readout, lr_norm, combine; trunk_triton.py:536-704,1688-1872), and the host-side bookkeeping between
 * graph replays: the block's pool refresh every Bq tokens (attention.py:1313-1369, kv_bounded.py:175-221) and the
 * cell close every 32 tokens (kv_cache.py:326-382, kv_bounded.py:155-173), both decided on the device from *pos.
 * q,k,v: the new token's projections (B,H,D) bf16 (strides sb, sh). y (B, H*D) bf16 = W_o's input.
 * sel_out (optional) (B,H,kk) int32: the cells read. splits = CTAs per (b,h) (1, 2, 4 or 8; a thread-block cluster). */
typedef struct {
    fsattn_fsl_state_t st;
    const void* q; const void* k; const void* v; int64_t in_sb, in_sh;
    const int64_t* pos;                  /* device scalar: index of the new token */
    const void* cos; const void* sin;    /* (L,D) bf16 */
    const float* lam; const float* sigma; const float* lrs; const float* norm_w;
    float scale, eps;
    void* y; int32_t* sel_out;
    int32_t splits;
    int32_t pdl; /* 1 = launch with programmatic stream serialization (overlaps the launch with the producer's tail) */
    const int32_t* ext_sel; /* optional (B,H,kk) int32: cells chosen by fsattn_fsb_select for this token (FS-B layers); the
                             * kernel then skips its own pool and scoring. Full stores (bf16, int8) only. NULL for FS-L. */
    int32_t window_path; /* how the window rows reach the SMs: 0 = chosen by the library (staged once B*H*splits exceeds the SM
                          * count), 1 = per-lane loads, 2 = staged through shared memory by bulk copies (needs splits = 1
                          * and an int8 store). Both give the same bits. */
} fsattn_fsl_decode_t;
FSATTN_API int fsattn_fsl_decode_step(const fsattn_fsl_decode_t* a, fsattn_stream_t stream);

/* Bounded store after a prefill of N tokens. Replaces SlotStore.prefill (src/fsattn/kv_bounded.py:115-152): keeps the
 * top-P cells visible to the first decode block (top_idx, already filled for block (N/Bq)*Bq) and every cell from
 * c_lo = max(0, min((blk-W)/32, m_vis-Wc)) on; slots in cell order; writes slot_of, cell_in, quantises the kept cells
 * of k/v into their slots and copies their kbar rows (kbar_cells (B,H,ncell,D) fp32 -> st.kbar per slot). */
typedef struct {
    fsattn_fsl_state_t st;
    fsattn_bhnd_t k, v;
    const float* kbar_cells; int64_t kc_sb, kc_sh;
    int32_t N;
} fsattn_slot_prefill_t;
FSATTN_API int fsattn_slot_prefill(const fsattn_slot_prefill_t* a, fsattn_stream_t stream);

/* ---- decode-step trunk projection (small batch) -------------------------------------------------------------------------
 * The glue around the attention kernel in a decode step: out = epilogue([rmsnorm](x) @ W^T) for M rows of activations.
 * Replaces, for B*N == 1.. rows, trunk_triton.rms_norm_cast + the fused QKV / gate-up GEMVs + silu_mul + the residual adds
 * of experiments/scaling/model.py:111-145,211-237 and src/fsattn/attention.py:1396-1420 (cuBLAS + Triton launches there).
 * W (n_out, K) bf16 row-major; x (M, K) bf16 rows x_stride apart; norm_w (K) bf16 or NULL (no norm);
 * epilogue: STORE out[m,n] = acc; RESIDUAL out[m,n] = res[m,n] + acc (out may alias res);
 * SWIGLU: W holds n_out/2 gate rows then n_out/2 up rows, out (M, n_out/2) = silu(gate) * up.
 * m0 is used internally (first row of a pass); pass 0. */
#define FSATTN_EPI_STORE 0
#define FSATTN_EPI_RESIDUAL 1
#define FSATTN_EPI_SWIGLU 2
typedef struct {
    const void* w; const void* x; int64_t x_stride;
    const void* norm_w; float eps;
    void* out; int64_t out_stride;
    const void* res; int64_t res_stride;
    int32_t M, K, n_out, epilogue, m0, pdl;
} fsattn_trunk_gemv_t;
FSATTN_API int fsattn_trunk_gemv(const fsattn_trunk_gemv_t* a, fsattn_stream_t stream);

/* Everything of a layer after its attention, for a decode step of M <= 8 rows, in one cooperative launch:
 *   x += W_o y;  act = silu(gate) * up of W_gu rmsnorm(x; norm2_w);  x += W_down act;
 *   out_next = W_next rmsnorm(x; norm_next_w)   (the next layer's QKV projection or the LM head; skipped when w_next is NULL).
 * Same arithmetic and roundings as four fsattn_trunk_gemv calls (experiments/scaling/model.py:111-145,211-237 and
 * src/fsattn/attention.py:1396-1420 in the reference), without the three launch boundaries: the phases are separated by
 * grid-wide barriers on bar[0..2], which the caller zeroes before every launch (e.g. one memset per step for all layers).
 * A barrier that does not complete within its bound sets *status to 1 and the kernel runs to its end; the caller reads
 * status where it reads its other device flags. x (M, d) is updated in place; act (M, f) is scratch.
 * W_o (d, d), W_gu (2f, d) gate rows then up rows, W_down (d, f), W_next (n_next, d): bf16 row-major, 16-byte aligned. */
typedef struct {
    void* x; int64_t x_stride;
    const void* y; int64_t y_stride;
    const void* w_o;
    const void* norm2_w; float eps2;
    const void* w_gu;
    void* act; int64_t act_stride;
    const void* w_down;
    const void* norm_next_w; float eps_next;
    const void* w_next; void* out_next; int64_t out_next_stride; int32_t n_next;
    int32_t* bar; int32_t* status;
    int32_t M, d, f, pdl;
} fsattn_trunk_layer_t;
FSATTN_API int fsattn_trunk_layer(const fsattn_trunk_layer_t* a, fsattn_stream_t stream);

/* RMSNorm of the prefill trunk: out (M, d) = x * rsqrt(mean(x^2) + eps) * w in fp32, rounded once to bf16 (row strides in
 * elements). Replaces F.rms_norm / trunk_triton.rms_norm_cast of experiments/scaling/model.py:82-108 on the prefill path. */
FSATTN_API int fsattn_rms_norm(const void* x, int64_t x_stride, const void* w, float eps, void* out, int64_t out_stride, int64_t M,
                               int32_t d, fsattn_stream_t stream);

/* The two ends of a greedy decode step (replace torch's embedding gather + copy and argmax + copy + add):
 * x (B,d) bf16 = table[tok[b]] (table (vocab,d) bf16, tok int64; an id outside the table reads row 0), and
 * tok[b] = argmax of logits (B,V) bf16 with row stride `stride` (lowest index on ties), *pos += 1 when pos is given.
 * Both wait for their producer themselves (programmatic dependent launch). */
FSATTN_API int fsattn_embed_rows(const int64_t* tok, const void* table, void* x, int32_t B, int32_t d, int64_t vocab, fsattn_stream_t stream);
FSATTN_API int fsattn_argmax_advance(const void* logits, int64_t stride, int32_t B, int32_t V, int64_t* tok, int64_t* pos,
                                     fsattn_stream_t stream);

/* ---- head-sharded decode: the per-layer exchange of head outputs over peer memory -------------------------------------
 * The reference has no multi-GPU path; its per-head data layout (src/fsattn/attention.py:1450-1491: one decode call per
 * layer over (B, H) rows) is what lets the heads be split over the GPUs of a box, with ONE exchange per layer in front of
 * W_o. This entry point is that exchange as a single small kernel per rank instead of a library all-gather.
 *
 * Every rank owns a slab (fsattn_peer_alloc: cudaMalloc, zeroed), exports it once (fsattn_peer_export: a 64-byte CUDA IPC
 * handle, sent to the peers by any host channel) and opens the peers' slabs (fsattn_peer_open: addresses valid on the
 * calling device). ll_dst[p] is rank p's receive area of fsattn_peer_ll_bytes(B, dl, world, n_slots) bytes, 8-byte words
 * {4 bytes of data, 4 bytes of flag} laid out [slot][call parity][source rank][B dl / 2]. A call takes its call count e =
 * epoch[slot] + 1 (epoch: n_slots int32, local, zero at start), stores its rows y_local (B, dl) bf16 with the flag e into
 * ll_dst[p][slot][e & 1][rank] of every peer p and into the columns [rank dl, (rank+1) dl) of its own y_out (B, world dl)
 * bf16, then polls ll_dst[rank][slot][e & 1][p] for every peer p until every word carries the flag e and writes the data
 * into p's columns of y_out. The polls are bounded by timeout_ns of the global timer: when one runs out bit p of *status
 * is set and the kernel returns (y_out is then incomplete). Stores go to peer memory; no load does, and nothing is
 * multicast. Every rank must make the same sequence of calls (slot, B, dl). */
#define FSATTN_PEER_MAX 8
#define FSATTN_PEER_HANDLE_BYTES 64
typedef struct {
    const void* y_local;
    void* y_out;
    void* ll_dst[FSATTN_PEER_MAX];
    int32_t* epoch;
    int32_t* status;
    int32_t B, dl, rank, world, slot;
    int32_t pdl;                 /* 1: launched as a programmatic dependent launch (the kernel waits for its producer itself) */
    int64_t timeout_ns;          /* (0, 2e9] */
} fsattn_peer_gather_t;
FSATTN_API int fsattn_peer_gather(const fsattn_peer_gather_t* g, fsattn_stream_t stream);
FSATTN_API int64_t fsattn_peer_ll_bytes(int32_t B, int32_t dl, int32_t world, int32_t n_slots);
FSATTN_API int fsattn_peer_alloc(int64_t bytes, void** ptr);
FSATTN_API int fsattn_peer_free(void* ptr);
FSATTN_API int fsattn_peer_export(void* ptr, uint8_t* handle /* FSATTN_PEER_HANDLE_BYTES */);
FSATTN_API int fsattn_peer_open(const uint8_t* handle, void** ptr);
FSATTN_API int fsattn_peer_close(void* ptr);

/* Elementwise SwiGLU gate of the prefill trunk: out (M, f) = silu(gu[:, :f]) * gu[:, f:] for the fused gate/up projection
 * gu (M, 2f) bf16 (row strides in elements). Replaces F.silu + the elementwise product of SwiGLU.forward
 * (experiments/scaling/model.py:111-145; trunk_triton.silu_mul on the reference's fused path), with the same two bf16
 * roundings. */
FSATTN_API int fsattn_swiglu(const void* gu, int64_t gu_stride, void* out, int64_t out_stride, int64_t M, int32_t f,
                             fsattn_stream_t stream);

/* ---- FS-B: two forests over the admitted cells, beam search, candidate re-rank ------------------------------------------
 * One fsattn_fsb_forest_t describes ONE forest (admission threshold tau) of one layer for all T = B*H rows.
 *
 * Layout (own; the reference's packed arena is fsb_tree.py:1008-1046 and its one-chunk-per-height decode arena
 * fsb_tree.py:1496-1522). The forest is the binary counter over the admitted-cell sequence (fsb_tree.py:897-911):
 * chunk (k, j) holds the admitted positions [j 2^k, (j+1) 2^k). Only chunks with EVEN j are ever the root named by a bit
 * of a prefix length (fsb_tree.py:1092-1098), so only those are stored, each at a fixed place: admitted position p
 * completes exactly one of them, (k = ctz(p+1), j = ((p+1) >> k) - 1). A chunk is therefore built once, when its last
 * cell is admitted, and never rebuilt; prefill and the decode-time ingest are the same operation on different ranges.
 *   node id of node n (level order, children 2n+1 / 2n+2) of chunk (k, j):  nbase(k) + (j/2) (2^{k+1}-1) + n,
 *   nbase(k) = k m_cap - m_cap + (m_cap >> k);  nodes per row = (k_cap+1) m_cap;  chunk id = m_cap - (m_cap >> k) + j/2.
 *   node_mu  (T, nodes, D) bf16: the mean the beam scores with;
 *   node_aux (T, nodes, 4) fp32: radius (inflated by the bf16 rounding error of the mean, fsb_tree.py:1049-1066),
 *            max ceiling (>= 0), min cell id (int bits), meta (int bits): >= 0 a leaf's cell id, < 0 ~((n << 4) | log2 cnt);
 *   root32   (T, m_cap, D+4) fp32: each chunk root's exact mean, un-inflated radius (the spines merge these,
 *            fsb_tree.py:1088-1124), 3 pad words.
 * adm (T, m_cap) int32 admitted cell ids ascending, m_tot (T), m_prev (T) (m_tot before the last ingest).
 * kbar (T rows kbar_st floats apart, D per cell) / ceil (T rows ceil_st apart): the cells' statistics (fp32). */
typedef struct {
    int32_t T, H, D, m_cap;
    const float* kbar; int64_t kbar_st;
    const float* ceil; int64_t ceil_st;
    const float* tau;                  /* (H) admission threshold per head */
    int32_t* adm; int32_t* m_tot; int32_t* m_prev;
    void* node_mu; float* node_aux; float* root32;
    int32_t compact;                   /* 0: the arena above (every aligned chunk kept: a prefill can name any earlier prefix).
                                        * 1: one place per chunk height - node id of node n of the chunk of height k:
                                        * 2^{k+1} - 2 - k + n, 4 m_cap nodes per row, chunk id k, root32 (T, 32, D+4) - which
                                        * holds the CURRENT prefix only (decode; the reference's decode arena,
                                        * fsb_tree.py:1496-1522). fsattn_fsb_compact converts 0 -> 1 after a prefill.
                                        * n > 1: the same with n nodes per row instead of 4 m_cap, for a caller that knows
                                        * how far the admitted counts can grow: heights 0..kt need 2^{kt+2} - 3 - kt nodes,
                                        * and a row then admits at most 2^{kt+1} - 1 cells (the admission stops there). */
} fsattn_fsb_forest_t;

/* Admit the cells [cell_begin, cell_end) of every row (ceil >= tau[h], fsb_tree.py:936-941, 1465-1494) into each of
 * the n_forests (<= 4) forests and build every chunk the newly admitted positions complete. Replaces build_forest
 * (fsb_tree.py:932-951, build_trees 616-678, GPU fsb_build.cu) and ForestCache.ingest's carry-chain rebuild
 * (fsb_tree.py:2033-2049). Chunk trees are bit-identical to the reference's CPU trees: every sum runs in the halving
 * order of det_reduce.det_sum and no multiply-add is contracted. scratch: fsattn_fsb_scratch_floats(m_cap, D, T) floats
 * per forest, used only during the call. */
FSATTN_API int64_t fsattn_fsb_scratch_floats(int32_t m_cap, int32_t D, int32_t T);
/* ---- streaming FS-L cache (replaces the pool bookkeeping and selection of src/fsattn/linear_cache.py) -----------------------
 * Pool of one (b,h): C = P + Wc cell slots plus one spare - slots [0, P) the cells with the highest ceilings seen so far (in no
 * particular order), [P, C) a ring of the newest cells (cell c in slot P + c mod Wc); id -1 = empty.
 *   ids (B,H,C+1) int32, prio (B,H,C+1) fp32 ceilings, mean (B,H,C+1,D) fp32 chunk-mean keys, k / v (B,H,(C+1)*32,D) bf16 token
 *   rows of the slots, valid (B,H,C) uint8. All contiguous. */

/* Block change (linear_cache.py:86-118): `count` newly completed cells with ids first_id .. first_id+count-1, their
 * statistics new_prio (B,H,count), new_mean (B,H,count,D) (from fsattn_cell_ingest) and token rows new_k / new_v (B,H,count*32,D)
 * bf16 (batch / head strides nk_sb / nk_sh, rows contiguous). The P best of (top list, new cells) by (ceiling desc, id asc)
 * stay: an entering cell is written into the slot of a leaving one, nothing else moves; the newest Wc cells also go into the
 * ring; valid is rewritten (a ring cell that is in the top list too counts once). count = 0 only rewrites valid. */
typedef struct {
    int32_t* ids; float* prio; float* mean; void* k; void* v; unsigned char* valid;
    const float* new_prio; const float* new_mean; const void* new_k; const void* new_v; int64_t nk_sb, nk_sh;
    int32_t B, H, D, P, Wc, count, first_id;
} fsattn_linear_merge_t;
FSATTN_API int fsattn_linear_merge(const fsattn_linear_merge_t* a, fsattn_stream_t stream);

/* Selection of n <= 128 queries of one block (linear_cache.py:154-170): q (B,H,n,D) bf16 at positions pos0 .. pos0+n-1;
 * score = (q . mean) scale + lam_h ceil erf(|p - (id + 0.5) 32| / (2 sigma_h)) over the valid slots (content_only = 1 drops
 * the second term); the best kk <= 4 by (score desc, cell id asc) as POOL SLOTS in sel (B,H,n_pad,kk_out) int32, -1 for none
 * (and beyond kk); sel_ids (optional, same shape): the cell ids. The slots index the pool's k / v as 32-row cells, which is
 * what fsattn_readout_combine then reads. */
typedef struct {
    const int32_t* ids; const float* prio; const float* mean; const unsigned char* valid;
    fsattn_bhnd_t q; const float* lam; const float* sigma; float scale;
    int32_t B, H, D, C, n, n_pad, kk, kk_out, pos0, content_only;
    int32_t* sel; int32_t* sel_ids;
} fsattn_linear_select_t;
FSATTN_API int fsattn_linear_select(const fsattn_linear_select_t* a, fsattn_stream_t stream);

/* Copies the chunks of the current prefix (one per set bit of m_tot, per row) from a full arena into a compact one.
 * src and dst share T, H, D, m_cap, adm, m_tot, m_prev; dst->compact = 1 (or the nodes per row n) with its own node_mu
 * (T, 4 m_cap or n, D), node_aux (T, 4 m_cap or n, 4) and root32 (T, 32, D+4). After it the decode-time ingest, spines and selection run on dst; the full arena
 * can be released (at 131 072 tokens: 300 MB -> 19 MB per forest and layer at head_dim 64). */
FSATTN_API int fsattn_fsb_compact(const fsattn_fsb_forest_t* src, const fsattn_fsb_forest_t* dst, fsattn_stream_t stream);

FSATTN_API int fsattn_fsb_ingest(const fsattn_fsb_forest_t* forests, int32_t n_forests, int32_t cell_begin,
                                 int32_t cell_end, float* scratch, int64_t scratch_floats, fsattn_stream_t stream);

/* Spines (fsb_tree.py:1070-1132): per forest and row, the nodes that merge the chunk roots named by the bits of
 * m_b = #admitted cells with id < n_visible. spine (T, FSATTN_FSB_SPINE_MAX, D+8) fp32 per forest:
 * [mu (D) | rad, amax, pmin(int), cnt(int), child_l(int), child_r(int), pad, pad]; hdr (T, 4) int32: root ref, height,
 * m_b, w. Node refs: >= 0 a node id of the row's arena, -(k+2) the spine node of height k, -1 none.
 * widths (host array, one beam width per forest, or NULL): with a width w > 0 the last spine slot (never a spine node) also
 * receives the beam's query-independent head for that width - the rounds whose children all fit in the frontier, walked
 * once here instead of in every decode step - and hdr[3] = w; the decode selection uses it when its beam width equals w. */
#define FSATTN_FSB_SPINE_MAX 20
FSATTN_API int fsattn_fsb_spines(const fsattn_fsb_forest_t* forests, int32_t n_forests, int32_t n_visible,
                                 float* const* spine, int32_t* const* hdr, const int32_t* widths, fsattn_stream_t stream);

/* Selection for queries. Replaces traverse_forest in the serve configuration (fsb_tree.py:1183-1317: fixed policy,
 * delta 0, 'bound' node score, second beam, token-LSE re-rank 'lse_pos' with the raw query, read_top): both beams
 * (_forest_beam 1321-1400; fsb_beam.cu / fsb_fast_step.py kernels), union_candidates (711-713), rerank_top (820-869,
 * fsb_rerank.py:83-125). main / second: the two forests (second may equal main).
 * Prefill (n_q > 1): q (B,H,N,D) bf16, queries q_pos0 .. q_pos0+N-1 in blocks of Bq; block b sees the cells
 * [0, (q_pos0 + b Bq) / 32); spines are built on the fly. Decode (use_spines = 1): one query per row at *pos with the
 * spines of fsattn_fsb_spines. k: raw token keys (B,H,>=cells*32,D) bf16, or int8 codes + scales (kq/ks) when k.ptr is NULL.
 * sel (B,H,Npad,K) int32 (-1 pad). cand (B,H,Npad,W_main+W_second) int32: the beams' candidates after the union; in
 * prefill with Bq = 128 it doubles as the hand-off to the block-cooperative re-rank (each distinct candidate cell of a
 * block staged once, scored with bf16 tensor-core tiles) - without it the slower one-warp-per-query re-rank runs.
 * nvis (B,H,Npad) optional visit counts. */
typedef struct {
    fsattn_fsb_forest_t main, second;
    fsattn_bhnd_t q, k;
    const int8_t* kq; const void* ks; int64_t kq_sb, kq_sh, ks_sb, ks_sh;
    const float* lam; const float* sigma;
    float scale, radius_coef;
    int32_t B, N, q_pos0, Bq, width, width2, read_top;
    int32_t use_spines; const float* spine[2]; const int32_t* hdr[2]; const int64_t* pos;
    int32_t* sel; int32_t* cand; int32_t* nvis;
    int32_t pdl;  /* decode: 1 = launch with programmatic stream serialization (the kernel waits for its producer itself) */
    int32_t beam_impl;  /* prefill with Bq = 128 and cand: 0 = one thread per query, the block's distinct nodes scored on
                         * tensor-core tiles; 1 = one warp per query (the kernel ragged blocks always use) */
} fsattn_fsb_select_t;
FSATTN_API int fsattn_fsb_select(const fsattn_fsb_select_t* a, fsattn_stream_t stream);

#ifdef __cplusplus
}
#endif
#endif /* FSATTN_B200_H */
