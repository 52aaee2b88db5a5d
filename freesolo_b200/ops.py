"""Torch-tensor front end of the C ABI: fills the argument structs of include/fsattn_b200.h from tensors and launches on
the current CUDA stream. PyTorch owns every buffer; these functions only allocate outputs the caller did not pass.

Every function raises when its tensors are not CUDA tensors: there is no CPU path.
"""
from __future__ import annotations

import math
import os

import torch

from . import lib as L

CELL = L.CELL


def _need_cuda(*ts):
    for t in ts:
        if t is not None and not t.is_cuda:
            raise RuntimeError("freesolo_b200 kernels need CUDA tensors: there is no CPU fallback")


def _stream(t: torch.Tensor) -> int:
    """The current stream of the tensor's device. The library launches on the CUDA context's current device (kernel
    attributes, SM counts and the static scratch address are per device), so that device must be the tensor's."""
    cur = torch.cuda.current_device()
    idx = t.device.index if t.device.index is not None else cur
    if idx != cur:
        raise RuntimeError(f"freesolo_b200: tensors live on cuda:{idx} but the current device is cuda:{cur}; "
                           f"call under torch.cuda.device({idx})")
    L.init(idx)
    return torch.cuda.current_stream(t.device).cuda_stream


def _bhnd(t: torch.Tensor, name: str) -> L.BHND:
    if t.dim() != 4 or t.stride(-1) != 1 or t.dtype != torch.bfloat16:
        raise ValueError(f"{name}: expected a bf16 (B,H,N,D) view with unit inner stride, got {tuple(t.shape)} {t.dtype} "
                         f"strides {t.stride()}")
    return L.BHND(t.data_ptr(), t.stride(0), t.stride(1), t.stride(2))


def _null() -> L.BHND:
    return L.BHND(None, 0, 0, 0)


def _p(t):
    return None if t is None else t.data_ptr()


def _f32(t: torch.Tensor) -> torch.Tensor:
    return t.detach().to(torch.float32).contiguous()


# ---------------------------------------------------------------------------------------------------------------------
def cell_ingest(K, V=None, *, ncell: int, cell0: int = 0, kbar=None, ceil=None, kq=None, ks=None, vq=None, vs=None):
    """One pass over ncell completed cells of K (and V): chunk-mean keys, ceilings and/or int8 codes + scales, written
    at cell index cell0 + c of the outputs. kbar (B,H,*,D) fp32, ceil (B,H,*) fp32, kq/vq (B,H,*,D) int8 with row stride
    D, ks/vs (B,H,*) bf16."""
    _need_cuda(K, V)
    B, H, _, D = K.shape
    a = L.CellIngest()
    a.k = _bhnd(K, "K")
    a.v = _bhnd(V, "V") if V is not None else _null()
    a.B, a.H, a.D, a.ncell, a.cell0 = B, H, D, int(ncell), int(cell0)
    if kbar is not None:
        assert kbar.dtype == torch.float32 and kbar.stride(-1) == 1 and kbar.stride(2) == D
        a.kbar, a.kbar_sb, a.kbar_sh = kbar.data_ptr(), kbar.stride(0), kbar.stride(1)
    if ceil is not None:
        assert ceil.dtype == torch.float32 and ceil.stride(-1) == 1
        a.ceil, a.ceil_sb, a.ceil_sh = ceil.data_ptr(), ceil.stride(0), ceil.stride(1)
    qs = [t for t in (kq, vq) if t is not None]
    if qs:
        q0 = qs[0]
        for t in qs:
            assert t.dtype == torch.int8 and t.stride(-1) == 1 and t.stride(2) == D and t.stride()[:2] == q0.stride()[:2]
        a.kq, a.vq, a.q_sb, a.q_sh = _p(kq), _p(vq), q0.stride(0), q0.stride(1)
        ss = [t for t in (ks, vs) if t is not None]
        for t in ss:
            assert t.dtype == torch.bfloat16 and t.stride(-1) == 1 and t.stride()[:2] == ss[0].stride()[:2]
        a.ks, a.vs, a.sc_sb, a.sc_sh = _p(ks), _p(vs), ss[0].stride(0), ss[0].stride(1)
    L.call("fsattn_cell_ingest", a, _stream(K))


def cell_stats(K, ncell: int):
    """(kbar (B,H,ncell,D) fp32, ceil (B,H,ncell) fp32) of the first ncell cells of K."""
    B, H, _, D = K.shape
    kbar = torch.empty(B, H, ncell, D, dtype=torch.float32, device=K.device)
    ceil = torch.empty(B, H, ncell, dtype=torch.float32, device=K.device)
    if ncell > 0:
        cell_ingest(K, ncell=ncell, kbar=kbar, ceil=ceil)
    return kbar, ceil


def quantize_cells(x, s: int = CELL, q=None, sc=None):
    """int8 codes and bf16 scales of the whole cells of x (B,H,N,D) bf16; q/sc may be preallocated slices."""
    if s != CELL:
        raise RuntimeError(f"cell size {s} unsupported (kernels are specialised for {CELL})")
    B, H, N, D = x.shape
    nc = N // s
    if q is None:
        q = torch.empty(B, H, nc * s, D, dtype=torch.int8, device=x.device)
    if sc is None:
        sc = torch.empty(B, H, nc, dtype=torch.bfloat16, device=x.device)
    if nc > 0:
        cell_ingest(x, ncell=nc, kq=q, ks=sc)
    return q, sc


def dequant_cells(q, sc, s: int = CELL, dtype=torch.bfloat16, out=None):
    """bf16(f32(q) * f32(scale)) over the quantised rows; out (B,H,>=N,D) optional."""
    _need_cuda(q, sc)
    if s != CELL or dtype != torch.bfloat16:
        raise RuntimeError("dequant_cells: only cell size 32 and bf16 output are supported")
    B, H, N, D = q.shape
    nrows = (N // s) * s
    ret = out
    if out is None:
        out = torch.empty(B, H, nrows, D, dtype=torch.bfloat16, device=q.device)
        ret = out
    assert q.stride(-1) == 1 and q.stride(2) == D and out.stride(-1) == 1 and out.stride(2) == D and sc.stride(-1) == 1
    a = L.Dequant()
    a.q, a.q_sb, a.q_sh = q.data_ptr(), q.stride(0), q.stride(1)
    a.sc, a.sc_sb, a.sc_sh = sc.data_ptr(), sc.stride(0), sc.stride(1)
    a.out, a.o_sb, a.o_sh = out.data_ptr(), out.stride(0), out.stride(1)
    a.B, a.H, a.D, a.nrows = B, H, D, nrows
    L.call("fsattn_dequant_cells", a, _stream(q))
    return ret


# ---------------------------------------------------------------------------------------------------------------------
def fsl_prefix_topp(ceil, ncell: int, Bq: int, nb: int, P: int):
    """(B*H, nb, P) int32: per query block the top-P visible cells in pool order, -1 fill."""
    _need_cuda(ceil)
    B, H = ceil.shape[:2]
    assert ceil.dtype == torch.float32 and ceil.stride(-1) == 1
    if ncell <= 0:
        return torch.full((B * H, nb, P), -1, dtype=torch.int32, device=ceil.device)
    topp = torch.empty(B * H, nb, P, dtype=torch.int32, device=ceil.device)
    a = L.FslTopp()
    a.ceil, a.ceil_sb, a.ceil_sh = ceil.data_ptr(), ceil.stride(0), ceil.stride(1)
    a.B, a.H, a.ncell, a.Bq, a.nb, a.P = B, H, int(ncell), int(Bq), int(nb), int(P)
    a.topp = topp.data_ptr()
    L.call("fsattn_fsl_prefix_topp", a, _stream(ceil))
    return topp


def fsl_select(Q, kbar, ceil, topp, lam, sigma, *, N: int, ncell: int, Bq: int, nb: int, P: int, Wc: int, kk: int,
               scale: float, want_margin: bool = False, impl: int = 0):
    """sel (B,H,nb*Bq,kk) int32 (and the fp32 margins when asked). impl 1 forces the CUDA-core kernel."""
    _need_cuda(Q, kbar, ceil, topp)
    B, H, _, D = Q.shape
    if ncell <= 0:      # nothing completed: no cell can be selected
        sel = torch.full((B, H, nb * Bq, kk), -1, dtype=torch.int32, device=Q.device)
        margin = torch.full((B, H, nb * Bq), float("inf"), dtype=torch.float32, device=Q.device)
        return (sel, margin) if want_margin else sel
    sel = torch.empty(B, H, nb * Bq, kk, dtype=torch.int32, device=Q.device)
    margin = torch.empty(B, H, nb * Bq, dtype=torch.float32, device=Q.device) if want_margin else None
    lam, sigma = _f32(lam), _f32(sigma)
    a = L.FslSelect()
    a.q = _bhnd(Q, "Q")
    assert kbar.dtype == torch.float32 and kbar.stride(-1) == 1 and kbar.stride(2) == D
    a.kbar, a.kbar_sb, a.kbar_sh = kbar.data_ptr(), kbar.stride(0), kbar.stride(1)
    a.ceil, a.ceil_sb, a.ceil_sh = ceil.data_ptr(), ceil.stride(0), ceil.stride(1)
    a.topp, a.lam, a.sigma = topp.data_ptr(), lam.data_ptr(), sigma.data_ptr()
    a.B, a.H, a.D, a.N, a.ncell, a.Bq, a.nb, a.P, a.Wc, a.kk = B, H, D, N, ncell, Bq, nb, P, Wc, kk
    a.scale = float(scale)
    a.sel, a.margin = sel.data_ptr(), _p(margin)
    assert topp.is_contiguous() and topp.shape[0] == B * H and topp.shape[1] >= nb and topp.shape[2] == P
    a.topp_nb = topp.shape[1]
    a.impl = int(impl)
    L.call("fsattn_fsl_select", a, _stream(Q))
    return (sel, margin) if want_margin else sel


def fs_dense_select(Q, kbar, ceil, lam, sigma, *, N: int, ncell: int, Bq: int, nb: int, kk: int, scale: float, status=None):
    """Dense FS prefill selection: sel (B,H,nb*Bq,kk) int32, for every query the kk best of ALL cells completed before its
    query block (tensor-core kernel: head_dim 64, Bq = 128, kk <= 4)."""
    _need_cuda(Q, kbar, ceil)
    B, H, _, D = Q.shape
    sel = torch.empty(B, H, nb * Bq, kk, dtype=torch.int32, device=Q.device)
    lam, sigma = _f32(lam).to(Q.device), _f32(sigma).to(Q.device)
    a = L.FsDenseSelect()
    a.q = _bhnd(Q, "Q")
    assert kbar.dtype == torch.float32 and kbar.stride(-1) == 1 and kbar.stride(2) == D and ceil.dtype == torch.float32 and ceil.stride(-1) == 1
    a.kbar, a.kbar_sb, a.kbar_sh = kbar.data_ptr(), kbar.stride(0), kbar.stride(1)
    a.ceil, a.ceil_sb, a.ceil_sh = ceil.data_ptr(), ceil.stride(0), ceil.stride(1)
    a.lam, a.sigma = lam.data_ptr(), sigma.data_ptr()
    a.B, a.H, a.D, a.N, a.ncell, a.Bq, a.nb, a.kk = B, H, D, int(N), int(ncell), int(Bq), int(nb), int(kk)
    a.scale = float(scale)
    a.sel = sel.data_ptr()
    nbytes = int(L.load().fsattn_fs_dense_workspace_bytes(B, H, int(ncell), D))
    ws = torch.empty(max(nbytes, 16), dtype=torch.uint8, device=Q.device)
    a.workspace, a.workspace_bytes = ws.data_ptr(), nbytes
    a.status = _p(status)
    L.call("fsattn_fs_dense_select", a, _stream(Q))
    ws.record_stream(torch.cuda.current_stream(Q.device))
    return sel


def fs_dense_decode_select(q, kbar, ceil, lam, sigma, pos_t, *, Bq: int, kk: int, scale: float, ncell_cap: int, splits: int = 8,
                           pdl: bool = False, sel=None):
    """Dense FS decode selection: q (B,H,D) bf16 view at device position pos_t -> sel (B,H,kk) int32, the kk best of the
    cells [0, min((pos // Bq) * Bq // 32, ncell_cap)). lam/sigma (H) fp32 device tensors."""
    _need_cuda(q, kbar, ceil, lam, sigma, pos_t)
    B, H, D = q.shape
    if sel is None:
        sel = torch.empty(B, H, kk, dtype=torch.int32, device=q.device)
    assert q.dtype == torch.bfloat16 and q.stride(-1) == 1 and kbar.dtype == torch.float32 and kbar.stride(-1) == 1 and kbar.stride(2) == D
    assert lam.dtype == torch.float32 and sigma.dtype == torch.float32 and pos_t.dtype == torch.int64 and sel.is_contiguous()
    a = L.FsDenseDecodeSelect()
    a.q, a.q_sb, a.q_sh = q.data_ptr(), q.stride(0), q.stride(1)
    a.kbar, a.kbar_sb, a.kbar_sh = kbar.data_ptr(), kbar.stride(0), kbar.stride(1)
    a.ceil, a.ceil_sb, a.ceil_sh = ceil.data_ptr(), ceil.stride(0), ceil.stride(1)
    a.lam, a.sigma, a.pos = lam.data_ptr(), sigma.data_ptr(), pos_t.data_ptr()
    a.B, a.H, a.D, a.Bq, a.kk, a.ncell_cap, a.splits, a.pdl = B, H, D, int(Bq), int(kk), int(ncell_cap), int(splits), 1 if pdl else 0
    a.scale = float(scale)
    a.sel = sel.data_ptr()
    L.call("fsattn_fs_dense_decode_select", a, _stream(q))
    return sel


def window_prefill(Q, K, V, cos, sin, W: int, scale: float, pos0: int = 0, impl: int = 0, out=None, status=None):
    """Causal band attention with RoPE on Q and K. Returns (B,N,H*D) bf16 (W_o's input layout)."""
    _need_cuda(Q, K, V, cos, sin)
    B, H, N, D = Q.shape
    if out is None:
        out = torch.empty(B, N, H * D, dtype=torch.bfloat16, device=Q.device)
    assert cos.dtype == torch.bfloat16 and sin.dtype == torch.bfloat16 and cos.is_contiguous() and sin.is_contiguous()
    assert cos.shape[1] == D and cos.shape[0] >= pos0 + N, "rope table too short"
    assert out.is_contiguous()
    tc = impl == 0 and D == 64 and W >= 64 and W % 64 == 0
    if tc and B == 1 and N > 2 * WINDOW_CHUNK:
        # A long single sequence goes through the tensor-core kernel in chunks of WINDOW_CHUNK queries, LAST chunk first, so
        # that its scratch (rotated Q and K) is chunk-sized: 69 MB instead of 537 MB at 131 072 tokens. A chunk starts one
        # window (rounded up to whole 128-query blocks) early; those rows lack their own left context, their outputs are
        # wrong, and the next call - the chunk before, which ends where this one's own rows begin - overwrites them. Tiles
        # stay aligned to absolute positions, so every query sees the same tiles in the same order as in a single call.
        halo = (int(W) + 127) // 128 * 128
        for c0 in reversed(range(0, N, WINDOW_CHUNK)):
            c1, h0 = min(N, c0 + WINDOW_CHUNK), max(0, c0 - halo)
            _window_prefill_call(Q[:, :, h0:c1], K[:, :, h0:c1], V[:, :, h0:c1], cos, sin, W, scale, pos0 + h0, impl,
                                 out[:, h0:c1], status, tc)
        return out
    _window_prefill_call(Q, K, V, cos, sin, W, scale, pos0, impl, out, status, tc)
    return out


WINDOW_CHUNK = 16384


def _window_prefill_call(Q, K, V, cos, sin, W, scale, pos0, impl, out, status, tc):
    B, H, N, D = Q.shape
    a = L.WindowPrefill()
    a.q, a.k, a.v = _bhnd(Q, "Q"), _bhnd(K, "K"), _bhnd(V, "V")
    a.cos, a.sin = cos.data_ptr(), sin.data_ptr()
    a.B, a.H, a.D, a.N, a.W, a.pos0 = B, H, D, N, int(W), int(pos0)
    a.scale = float(scale)
    a.out = out.data_ptr()
    a.impl = int(impl)
    ws = None
    if tc:
        # scratch of the tensor-core kernel (rotated Q and K); TMA wants a 16-byte aligned base, which torch's allocator
        # (512-byte aligned blocks) always gives
        nbytes = 2 * B * H * N * D * 2
        ws = torch.empty(nbytes, dtype=torch.uint8, device=Q.device)
        a.workspace, a.workspace_bytes = ws.data_ptr(), nbytes
    a.status = _p(status)
    L.call("fsattn_window_prefill", a, _stream(Q))
    if ws is not None:
        ws.record_stream(torch.cuda.current_stream(Q.device))


def window_prefill_static(Q, K, V, cos, sin, W: int, scale: float, pos0: int = 0, out=None, status=None):
    """window_prefill through the allocation-free entry point: the kernel's scratch is a fixed array inside the library, so
    nothing is allocated for it here. For callers that may not create device memory at call time. Only head_dim 64, W a
    multiple of 64 and B*H*N <= 131072; larger or other shapes raise. `out` must be passed by such callers (when it is
    None this convenience wrapper allocates the output, which is not scratch). Calls that overlap on the GPU race on the
    shared array; the first call on a device must come before any stream capture."""
    _need_cuda(Q, K, V, cos, sin)
    B, H, N, D = Q.shape
    if out is None:
        out = torch.empty(B, N, H * D, dtype=torch.bfloat16, device=Q.device)
    assert cos.dtype == torch.bfloat16 and sin.dtype == torch.bfloat16 and cos.is_contiguous() and sin.is_contiguous()
    assert cos.shape[1] == D and cos.shape[0] >= pos0 + N, "rope table too short"
    assert out.is_contiguous()
    a = L.WindowPrefill()
    a.q, a.k, a.v = _bhnd(Q, "Q"), _bhnd(K, "K"), _bhnd(V, "V")
    a.cos, a.sin = cos.data_ptr(), sin.data_ptr()
    a.B, a.H, a.D, a.N, a.W, a.pos0 = B, H, D, N, int(W), int(pos0)
    a.scale = float(scale)
    a.out = out.data_ptr()
    a.status = _p(status)
    L.call("fsattn_window_prefill_static", a, _stream(Q))
    return out


def readout_combine(Q, K, V, sel, sr, norm_w, lrs, eps: float, *, scale: float, Bq: int, n_kv: int | None = None,
                    q_pos0: int = 0, out=None, impl: int | None = None):
    """y (B,N,H*D) bf16 = bf16(sr + lrs[h] * lr_norm(bf16(readout of the selected cells))). sr (B,N,H*D) bf16 or None
    (treated as zero); out may be sr itself (in place)."""
    _need_cuda(Q, K, V, sel)
    B, H, N, D = Q.shape
    kk = sel.shape[-1]
    if out is None:
        out = torch.empty(B, N, H * D, dtype=torch.bfloat16, device=Q.device)
    assert sel.dtype == torch.int32 and sel.stride(-1) == 1 and sel.stride(2) == kk and sel.shape[2] >= N
    assert out.is_contiguous() and (sr is None or (sr.is_contiguous() and sr.dtype == torch.bfloat16))
    norm_w, lrs = _f32(norm_w), _f32(lrs).reshape(-1)
    a = L.ReadoutCombine()
    a.q, a.k, a.v = _bhnd(Q, "Q"), _bhnd(K, "K"), _bhnd(V, "V")
    a.sel, a.sel_sb, a.sel_sh = sel.data_ptr(), sel.stride(0), sel.stride(1)
    a.sr, a.y = _p(sr), out.data_ptr()
    a.norm_w, a.lrs = norm_w.data_ptr(), lrs.data_ptr()
    a.B, a.H, a.D, a.N, a.n_kv, a.Bq, a.kk, a.q_pos0 = B, H, D, N, int(K.shape[2] if n_kv is None else n_kv), Bq, kk, q_pos0
    a.scale, a.eps = float(scale), float(eps)
    a.impl = int(os.environ.get("FSATTN_READOUT_IMPL", "0")) if impl is None else int(impl)
    L.call("fsattn_readout_combine", a, _stream(Q))
    return out


# ---------------------------------------------------------------------------------------------------------------------
class FslDecodeState:
    """Device buffers of one FS-L layer's decode-time KV state (see fsattn_fsl_state_t in include/fsattn_b200.h).

    mode: "bf16" (full bf16 store), "int8" (full int8 store) or "bounded" (int8 slot store that keeps only readable
    cells). cap_rows bounds the absolute token position; the bounded store holds n_slots * 32 rows whatever the length."""

    MODES = {"bf16": 0, "int8": 1, "bounded": 2}

    def __init__(self, B, H, D, cap_rows, device, *, mode="int8", P=64, Wc=8, W=512, Bq=128, kk=4):
        self.B, self.H, self.D = B, H, D
        self.mode = mode
        self.P, self.Wc, self.W, self.Bq, self.kk = P, Wc, W, Bq, kk
        self.cap_rows = int(cap_rows)
        self.cap_cells = max(1, (self.cap_rows + CELL - 1) // CELL)
        dev = torch.device(device)
        z = dict(device=dev)
        self.n_slots = P + max(-(-W // CELL), Wc) + -(-Bq // CELL) + 1
        self.kbuf = self.vbuf = self.kq = self.vq = self.ks = self.vs = self.khot = self.vhot = None
        self.slot_of = self.cell_in = None
        if mode == "bf16":
            self.kbuf = torch.zeros(B, H, self.cap_rows, D, dtype=torch.bfloat16, **z)
            self.vbuf = torch.zeros(B, H, self.cap_rows, D, dtype=torch.bfloat16, **z)
            stat_cells = self.cap_cells
        elif mode == "int8":
            rows = self.cap_cells * CELL
            self.kq = torch.zeros(B, H, rows, D, dtype=torch.int8, **z)
            self.vq = torch.zeros(B, H, rows, D, dtype=torch.int8, **z)
            self.ks = torch.ones(B, H, self.cap_cells, dtype=torch.bfloat16, **z)
            self.vs = torch.ones(B, H, self.cap_cells, dtype=torch.bfloat16, **z)
            stat_cells = self.cap_cells
        elif mode == "bounded":
            rows = self.n_slots * CELL
            self.kq = torch.zeros(B, H, rows, D, dtype=torch.int8, **z)
            self.vq = torch.zeros(B, H, rows, D, dtype=torch.int8, **z)
            self.ks = torch.ones(B, H, self.n_slots, dtype=torch.bfloat16, **z)
            self.vs = torch.ones(B, H, self.n_slots, dtype=torch.bfloat16, **z)
            self.slot_of = torch.full((B, H, self.cap_cells), -1, dtype=torch.int32, **z)
            self.cell_in = torch.full((B, H, self.n_slots), -1, dtype=torch.int32, **z)
            stat_cells = self.n_slots
        else:
            raise ValueError(f"unknown store mode {mode!r}")
        if mode != "bf16":
            self.khot = torch.zeros(B, H, CELL, D, dtype=torch.bfloat16, **z)
            self.vhot = torch.zeros(B, H, CELL, D, dtype=torch.bfloat16, **z)
        self.kbar = torch.zeros(B, H, stat_cells, D, dtype=torch.float32, **z)
        self.ceil = torch.zeros(B, H, self.cap_cells, dtype=torch.float32, **z)
        self.top_idx = torch.full((B, H, P), -1, dtype=torch.int32, **z)
        self.top_blk = torch.zeros(B, H, dtype=torch.int32, **z)
        self.pool_kbar = torch.zeros(B, H, P + Wc, D, dtype=torch.float32, **z)
        self.pool_meta = torch.full((B, H, P + Wc, 4), -1, dtype=torch.int32, **z)
        self.pool_blk = torch.full((B, H), -1, dtype=torch.int32, **z)
        self.status = torch.zeros(L.ST_WORDS, dtype=torch.int32, **z)
        self.prefill_topp = None

    def nbytes(self) -> int:
        ts = (self.kbuf, self.vbuf, self.kq, self.vq, self.ks, self.vs, self.khot, self.vhot, self.slot_of, self.cell_in,
              self.kbar, self.ceil, self.top_idx, self.top_blk, self.pool_kbar, self.pool_meta, self.pool_blk, self.status)
        return sum(t.numel() * t.element_size() for t in ts if t is not None)

    def struct(self) -> L.FslState:
        s = L.FslState()
        s.store_mode = self.MODES[self.mode]
        s.B, s.H, s.D, s.P, s.Wc, s.W, s.Bq, s.kk, s.n_slots = (self.B, self.H, self.D, self.P, self.Wc, self.W, self.Bq,
                                                              self.kk, self.n_slots)
        s.cap_rows, s.cap_cells = self.cap_rows, self.cap_cells
        if self.kbuf is not None:
            s.kbuf, s.vbuf, s.buf_sb, s.buf_sh = self.kbuf.data_ptr(), self.vbuf.data_ptr(), self.kbuf.stride(0), self.kbuf.stride(1)
        if self.kq is not None:
            s.kq, s.vq, s.q_sb, s.q_sh = self.kq.data_ptr(), self.vq.data_ptr(), self.kq.stride(0), self.kq.stride(1)
            s.ks, s.vs, s.sc_sb, s.sc_sh = self.ks.data_ptr(), self.vs.data_ptr(), self.ks.stride(0), self.ks.stride(1)
            s.khot, s.vhot, s.hot_sb, s.hot_sh = self.khot.data_ptr(), self.vhot.data_ptr(), self.khot.stride(0), self.khot.stride(1)
        s.kbar, s.kbar_sb, s.kbar_sh = self.kbar.data_ptr(), self.kbar.stride(0), self.kbar.stride(1)
        s.ceil, s.ceil_sb, s.ceil_sh = self.ceil.data_ptr(), self.ceil.stride(0), self.ceil.stride(1)
        if self.slot_of is not None:
            s.slot_of, s.so_sb, s.so_sh = self.slot_of.data_ptr(), self.slot_of.stride(0), self.slot_of.stride(1)
            s.cell_in, s.ci_sb, s.ci_sh = self.cell_in.data_ptr(), self.cell_in.stride(0), self.cell_in.stride(1)
        s.top_idx, s.top_blk, s.status = self.top_idx.data_ptr(), self.top_blk.data_ptr(), self.status.data_ptr()
        s.pool_kbar, s.pool_meta, s.pool_blk = self.pool_kbar.data_ptr(), self.pool_meta.data_ptr(), self.pool_blk.data_ptr()
        return s

    @torch.no_grad()
    def prefill(self, K, V, N: int, kbar=None, ceil=None):
        """Load the store from the un-rotated K, V (B,H,N,D) of a prompt: cell statistics (recomputed unless handed
        over), the first decode block's top-P list, the completed cells (quantised / copied / the kept slots) and the
        open cell's rows."""
        ncell = N // CELL
        if ncell > self.cap_cells or N > self.cap_rows:
            raise ValueError(f"KV store sized for {self.cap_rows} rows, prompt has {N}")
        if kbar is None or ceil is None:
            kbar, ceil = cell_stats(K, ncell)
        self.status.zero_()
        self.pool_blk.fill_(-1)             # the first decode step gathers the block's candidate pool
        self.top_idx.fill_(-1)
        blk = (N // self.Bq) * self.Bq
        self.top_blk.fill_(blk)
        if ncell > 0:
            self.ceil[:, :, :ncell].copy_(ceil)
            nb = blk // self.Bq + 1
            topp = fsl_prefix_topp(ceil, ncell, self.Bq, nb, self.P)
            self.top_idx.copy_(topp[:, nb - 1].view(self.B, self.H, self.P))
            self.prefill_topp = topp        # per-block lists of the prompt: the layer's own selection reuses them
        if self.mode == "bf16":
            self.kbuf[:, :, :N].copy_(K[:, :, :N])
            self.vbuf[:, :, :N].copy_(V[:, :, :N])
            if ncell > 0:
                self.kbar[:, :, :ncell].copy_(kbar)
        elif self.mode == "int8":
            if ncell > 0:
                cell_ingest(K, V, ncell=ncell, kq=self.kq, ks=self.ks, vq=self.vq, vs=self.vs)
                self.kbar[:, :, :ncell].copy_(kbar)
        else:
            slot_prefill(self, K, V, kbar if ncell > 0 else self.kbar, N)
        r = N - ncell * CELL
        if r > 0 and self.mode != "bf16":
            self.khot[:, :, :r].copy_(K[:, :, ncell * CELL:N])
            self.vhot[:, :, :r].copy_(V[:, :, ncell * CELL:N])

    def faults(self):
        """(slot overflows, readable cells without a slot, rejected indices): a host sync."""
        f = self.status.tolist()
        return int(f[L.ST_SLOT_OVERFLOW]), int(f[L.ST_POOL_NO_SLOT]), int(f[L.ST_BAD_INDEX])


def slot_prefill(state: FslDecodeState, K, V, kbar_cells, N: int):
    _need_cuda(K, V, kbar_cells)
    a = L.SlotPrefill()
    a.st = state.struct()
    a.k, a.v = _bhnd(K, "K"), _bhnd(V, "V")
    assert kbar_cells.dtype == torch.float32 and kbar_cells.stride(-1) == 1 and kbar_cells.stride(2) == state.D
    a.kbar_cells, a.kc_sb, a.kc_sh = kbar_cells.data_ptr(), kbar_cells.stride(0), kbar_cells.stride(1)
    a.N = int(N)
    L.call("fsattn_slot_prefill", a, _stream(K))


def fsl_decode_step(state: FslDecodeState, q, k, v, pos_t, cos, sin, lam, sigma, lrs, norm_w, *, scale: float, eps: float,
                    y=None, sel_out=None, splits: int = 8, pdl: bool = False, ext_sel=None, window_path: int = 0):
    """One decode token of one FS-L layer. q,k,v: (B,H,D) bf16 views with equal strides and unit inner stride (e.g. slices
    of a fused QKV projection); pos_t: int64 device scalar; lam/sigma/lrs (H) fp32, norm_w (D) fp32 (all device tensors
    that stay alive until the launch has run). Returns y (B, H*D) bf16."""
    _need_cuda(q, k, v, pos_t, cos, sin, lam, sigma, lrs, norm_w)
    B, H, D = state.B, state.H, state.D
    for t in (q, k, v):
        assert t.dtype == torch.bfloat16 and tuple(t.shape) == (B, H, D) and t.stride(-1) == 1 and t.stride() == q.stride()
    for t in (lam, sigma, lrs, norm_w):
        assert t.dtype == torch.float32 and t.is_contiguous()
    assert pos_t.dtype == torch.int64 and cos.dtype == torch.bfloat16 and cos.is_contiguous() and cos.shape[1] == D
    if y is None:
        y = torch.empty(B, H * D, dtype=torch.bfloat16, device=q.device)
    a = L.FslDecode()
    a.st = state.struct()
    a.q, a.k, a.v, a.in_sb, a.in_sh = q.data_ptr(), k.data_ptr(), v.data_ptr(), q.stride(0), q.stride(1)
    a.pos = pos_t.data_ptr()
    a.cos, a.sin = cos.data_ptr(), sin.data_ptr()
    a.lam, a.sigma, a.lrs, a.norm_w = lam.data_ptr(), sigma.data_ptr(), lrs.data_ptr(), norm_w.data_ptr()
    a.scale, a.eps = float(scale), float(eps)
    a.y, a.sel_out = y.data_ptr(), _p(sel_out)
    a.splits = int(splits)
    a.window_path = int(window_path)
    a.pdl = 1 if pdl else 0
    if ext_sel is not None:         # FS-B: the cells chosen by fsb_select for this token
        assert ext_sel.is_cuda and ext_sel.dtype == torch.int32 and ext_sel.is_contiguous() and ext_sel.numel() == B * H * state.kk
        a.ext_sel = ext_sel.data_ptr()
    L.call("fsattn_fsl_decode_step", a, _stream(q))
    return y


def trunk_gemv(x, w, *, norm_w=None, eps: float = 1e-6, res=None, swiglu: bool = False, out=None, pdl: bool = True):
    """Decode-step trunk projection for a few rows: out = epilogue([rmsnorm](x) @ w^T).
    x (M,K) bf16 (row stride free), w (n_out,K) bf16 contiguous, norm_w (K) bf16 or None. res (M,n_out) adds a residual
    (out may be res itself); swiglu treats w as [gate rows; up rows] and returns silu(gate)*up (M, n_out/2)."""
    _need_cuda(x, w, norm_w, res)
    M, K = x.shape
    n_out = w.shape[0]
    assert x.dtype == torch.bfloat16 and w.dtype == torch.bfloat16 and w.is_contiguous() and w.shape[1] == K and x.stride(1) == 1
    n_cols = n_out // 2 if swiglu else n_out
    if out is None:
        out = torch.empty(M, n_cols, dtype=torch.bfloat16, device=x.device)
    assert out.dtype == torch.bfloat16 and out.stride(1) == 1 and tuple(out.shape) == (M, n_cols)
    a = L.TrunkGemv()
    a.w, a.x, a.x_stride = w.data_ptr(), x.data_ptr(), x.stride(0)
    if norm_w is not None:
        assert norm_w.dtype == torch.bfloat16 and norm_w.is_contiguous() and norm_w.numel() == K
        a.norm_w = norm_w.data_ptr()
    a.eps = float(eps)
    a.out, a.out_stride = out.data_ptr(), out.stride(0)
    a.epilogue = L.EPI_SWIGLU if swiglu else (L.EPI_RESIDUAL if res is not None else L.EPI_STORE)
    if res is not None:
        assert not swiglu and res.dtype == torch.bfloat16 and res.stride(1) == 1 and tuple(res.shape) == (M, n_out)
        a.res, a.res_stride = res.data_ptr(), res.stride(0)
    a.M, a.K, a.n_out, a.m0, a.pdl = M, K, n_out, 0, 1 if pdl else 0
    L.call("fsattn_trunk_gemv", a, _stream(x))
    return out


def trunk_layer(x, y, w_o, norm2_w, eps2, w_gu, act, w_down, bar, status, *, norm_next_w=None, eps_next: float = 1e-6,
                w_next=None, out_next=None, pdl: bool = True):
    """Everything of a layer after its attention for a decode step of M <= 8 rows, one cooperative launch:
    x += y @ w_o^T; act = SwiGLU(rmsnorm(x) @ w_gu^T); x += act @ w_down^T; out_next = rmsnorm'(x) @ w_next^T.
    x (M,d) is updated in place; bar (>= 3 int32, zeroed by the caller before the launch) carries the grid barriers;
    status (int32[1]) is set to 1 if a barrier ran out of its bound."""
    _need_cuda(x, y, w_o, norm2_w, w_gu, act, w_down, bar, status, norm_next_w, w_next, out_next)
    M, d = x.shape
    f = w_down.shape[1]
    bf = torch.bfloat16
    assert all(t.dtype == bf for t in (x, y, w_o, norm2_w, w_gu, act, w_down)) and x.stride(1) == 1 and y.stride(1) == 1
    assert tuple(y.shape) == (M, d) and tuple(w_o.shape) == (d, d) and tuple(w_gu.shape) == (2 * f, d) and tuple(w_down.shape) == (d, f)
    assert tuple(act.shape) == (M, f) and act.stride(1) == 1 and w_o.is_contiguous() and w_gu.is_contiguous() and w_down.is_contiguous()
    assert bar.dtype == torch.int32 and bar.numel() >= 3 and bar.is_contiguous() and status.dtype == torch.int32
    a = L.TrunkLayer()
    a.x, a.x_stride, a.y, a.y_stride = x.data_ptr(), x.stride(0), y.data_ptr(), y.stride(0)
    a.w_o, a.norm2_w, a.eps2, a.w_gu = w_o.data_ptr(), norm2_w.data_ptr(), float(eps2), w_gu.data_ptr()
    a.act, a.act_stride, a.w_down = act.data_ptr(), act.stride(0), w_down.data_ptr()
    if w_next is not None:
        assert norm_next_w is not None and out_next is not None and w_next.dtype == bf and w_next.is_contiguous()
        assert w_next.shape[1] == d and tuple(out_next.shape) == (M, w_next.shape[0]) and out_next.stride(1) == 1
        assert norm_next_w.dtype == bf and norm_next_w.numel() == d and out_next.dtype == bf
        a.norm_next_w, a.eps_next, a.w_next = norm_next_w.data_ptr(), float(eps_next), w_next.data_ptr()
        a.out_next, a.out_next_stride, a.n_next = out_next.data_ptr(), out_next.stride(0), w_next.shape[0]
    a.bar, a.status = bar.data_ptr(), status.data_ptr()
    a.M, a.d, a.f, a.pdl = M, d, f, 1 if pdl else 0
    L.call("fsattn_trunk_layer", a, _stream(x))
    return x


def default_scale(D: int) -> float:
    return 1.0 / math.sqrt(D)


# ---------------------------------------------------------------------------------------------------------------------
# FS-B: forests, spines, beam + re-rank selection
# ---------------------------------------------------------------------------------------------------------------------
_FSB_SCRATCH = {}


def _fsb_scratch(device, floats: int) -> torch.Tensor:
    """Build scratch shared by every layer of a device (layers run one after another on one stream)."""
    key = (device.type, device.index)
    buf = _FSB_SCRATCH.get(key)
    if buf is None or buf.numel() < floats:
        buf = torch.empty(max(floats, 1), dtype=torch.float32, device=device)
        _FSB_SCRATCH[key] = buf
    return buf


class FsbForests:
    """Device buffers of one layer's FS-B forests (fsattn_fsb_forest_t in include/fsattn_b200.h): the main forest
    (admission tau) and, when tau_u is given, the second beam's forest (tau_u). kbar (B,H,>=cells,D) fp32 and ceil
    (B,H,>=cells) fp32 are the layer's cell statistics; the forests read them in place. cap_cells bounds the number
    of cells ever ingested (rounded up to a power of two)."""

    def __init__(self, kbar, ceil, tau, tau_u=None, *, cap_cells: int):
        _need_cuda(kbar, ceil)
        B, H, _, D = kbar.shape
        assert kbar.dtype == torch.float32 and kbar.is_contiguous() and ceil.dtype == torch.float32 and ceil.is_contiguous()
        self.B, self.H, self.D, self.T = B, H, D, B * H
        m_cap = 1
        while m_cap < max(1, int(cap_cells)):
            m_cap *= 2
        if m_cap > L.FSB_MAX_MCAP:
            raise RuntimeError(f"FS-B: {cap_cells} cells per row exceed the supported {L.FSB_MAX_MCAP}")
        self.m_cap = m_cap
        self.cap_cells = max(1, int(cap_cells))
        self.k_cap = m_cap.bit_length() - 1
        self.kbar, self.ceil = kbar, ceil
        dev = kbar.device
        self.taus = [_f32(tau).to(dev)] + ([_f32(tau_u).to(dev)] if tau_u is not None else [])
        self.nf = len(self.taus)
        T = self.T
        self.adm = [torch.full((T, m_cap), -1, dtype=torch.int32, device=dev) for _ in range(self.nf)]
        self.m_tot = [torch.zeros(T, dtype=torch.int32, device=dev) for _ in range(self.nf)]
        self.m_prev = [torch.zeros(T, dtype=torch.int32, device=dev) for _ in range(self.nf)]
        self.compact = 0
        self._alloc_arena(0)
        self.spine = [torch.zeros(T, L.FSB_SPINE_MAX, D + 8, dtype=torch.float32, device=dev) for _ in range(self.nf)]
        self.hdr = [torch.full((T, 4), -1, dtype=torch.int32, device=dev) for _ in range(self.nf)]
        self.n_seen = 0

    def _arena(self, compact: int, nodes=None):
        """(node_mu, node_aux, root32) lists of a full (every aligned chunk) or compact (one chunk per height) arena;
        nodes: per forest, the nodes per row of a compact arena (default 4 m_cap, room for every height)."""
        T, D, dev = self.T, self.D, self.kbar.device
        if nodes is None:
            nodes = [4 * self.m_cap if compact else (self.k_cap + 1) * self.m_cap] * self.nf
        roots = 32 if compact else self.m_cap
        return ([torch.zeros(T, n, D, dtype=torch.bfloat16, device=dev) for n in nodes],
                [torch.zeros(T, n, 4, dtype=torch.float32, device=dev) for n in nodes],
                [torch.zeros(T, roots, D + 4, dtype=torch.float32, device=dev) for _ in range(self.nf)])

    def _alloc_arena(self, compact: int, nodes=None) -> None:
        self.node_mu, self.node_aux, self.root32 = self._arena(compact, nodes)
        self.compact = compact
        # what the C struct carries: 0 full, 1 compact with 4 m_cap nodes per row, n > 1 compact with n nodes per row
        self.compact_arg = [0] * self.nf if not compact else [1] * self.nf if nodes is None else [int(n) for n in nodes]

    TIGHT_ARENA_FROM = 3000      # cells of capacity above which the decode arena is sized from the admitted counts (one host sync per layer)

    @staticmethod
    def compact_nodes_for(max_admitted: int) -> int:
        """Nodes per row of a compact arena whose rows never admit more than max_admitted cells: the places of the heights
        0 .. floor(log2(max_admitted)), i.e. sum of 2^(k+1) - 1 (csrc/fsb.cuh: fsb_compact_nodes)."""
        kt = max(int(max_admitted), 1).bit_length() - 1
        return max((4 << kt) - 3 - kt, 2)

    def compact_arena(self, n_visible: int | None = None) -> None:
        """After a prefill: keep only the chunks of the current prefix, one place per chunk height, and release the arena
        that held every aligned chunk (which only a prefill, naming earlier prefixes, needs). Decode-time ingest, spines
        and selection continue on the small arena; a later prefill needs reset() first.

        n_visible: the cells the NEXT query can see (the start of its 128-token block, in cells), at most the cells ingested.
        The forest is first taken back to that prefix - the admitted counts drop to the cells below n_visible; the up to
        three later cells are admitted again at the next block change - because the small arena can only name the prefix
        it was compacted at."""
        if self.compact:
            return
        if n_visible is not None and n_visible < self.n_seen:
            for i in range(self.nf):
                below = ((self.adm[i] >= 0) & (self.adm[i] < int(n_visible))).sum(-1).to(torch.int32)
                self.m_tot[i].copy_(torch.minimum(below, self.m_tot[i]))
                self.m_prev[i].copy_(self.m_tot[i])
            self.n_seen = int(n_visible)
        src = [self.struct(i) for i in range(self.nf)]
        old = (self.node_mu, self.node_aux, self.root32)
        # Size of the small arena: a row can still admit the cells that are not ingested yet, so no row's count can pass
        # (its count now) + (capacity - cells seen); the admission kernel holds a sized arena to what it has places for. Reading
        # the counts is one host synchronisation per layer; inside a stream capture the bound is the capacity itself.
        room = max(0, self.cap_cells - self.n_seen)
        if self.cap_cells <= self.TIGHT_ARENA_FROM or torch.cuda.is_current_stream_capturing():
            # short prompts (the arena is a few MB anyway, and their prefill is bound by the host's launch rate, which a
            # synchronisation per layer would stall) and captures: no read-back
            bound = [min(self.m_cap, self.cap_cells)] * self.nf
        else:
            bound = [min(self.m_cap, int(self.m_tot[i].max().item()) + room) for i in range(self.nf)]
        self._alloc_arena(1, [self.compact_nodes_for(b) for b in bound])
        lib = L.load()
        for i in range(self.nf):
            dst = self.struct(i)
            L.check(lib.fsattn_fsb_compact(L.C.byref(src[i]), L.C.byref(dst), _stream(self.kbar)), "fsattn_fsb_compact")
        del old                              # freed in stream order: the copies above were launched on this stream

    def reset(self) -> None:
        """Forget every admitted cell (a new prompt over the same statistics buffers). Chunk nodes need no clearing: a
        chunk is only ever read after the admission count says it is complete, and it is rebuilt before that. A compacted
        forest gets its full arena back."""
        if self.compact:
            self._alloc_arena(0)
        for i in range(self.nf):
            self.adm[i].fill_(-1)
            self.m_tot[i].zero_()
            self.m_prev[i].zero_()
            self.hdr[i].fill_(-1)
        self.n_seen = 0

    def nbytes(self) -> int:
        ts = self.adm + self.m_tot + self.m_prev + self.node_mu + self.node_aux + self.root32 + self.spine + self.hdr
        return sum(t.numel() * t.element_size() for t in ts)

    def struct(self, i: int) -> L.FsbForest:
        f = L.FsbForest()
        f.T, f.H, f.D, f.m_cap = self.T, self.H, self.D, self.m_cap
        f.kbar, f.kbar_st = self.kbar.data_ptr(), self.kbar.stride(1)
        f.ceil, f.ceil_st = self.ceil.data_ptr(), self.ceil.stride(1)
        f.tau = self.taus[i].data_ptr()
        f.adm, f.m_tot, f.m_prev = self.adm[i].data_ptr(), self.m_tot[i].data_ptr(), self.m_prev[i].data_ptr()
        f.node_mu, f.node_aux, f.root32 = self.node_mu[i].data_ptr(), self.node_aux[i].data_ptr(), self.root32[i].data_ptr()
        f.compact = self.compact_arg[i]
        return f

    def ingest(self, cell_end: int) -> None:
        """Admit the cells [n_seen, cell_end) and build the chunks they complete (both forests, one set of launches)."""
        cell_end = int(cell_end)
        if cell_end <= self.n_seen:
            return
        if cell_end > self.m_cap:
            raise RuntimeError(f"FS-B: cell {cell_end} beyond the forest capacity {self.m_cap}")
        lib = L.load()
        floats = lib.fsattn_fsb_scratch_floats(self.m_cap, self.D, self.T) * self.nf
        scratch = _fsb_scratch(self.kbar.device, floats)
        arr = (L.FsbForest * self.nf)(*[self.struct(i) for i in range(self.nf)])
        L.check(lib.fsattn_fsb_ingest(arr, self.nf, self.n_seen, cell_end, scratch.data_ptr(), scratch.numel(),
                                      _stream(self.kbar)), "fsattn_fsb_ingest")
        self.n_seen = cell_end

    def build_spines(self, n_visible: int, widths=None) -> None:
        """Spines of the prefix of cells [0, n_visible) for decode queries (kept until the next call). widths: the beam width
        per forest; with it the beams' query-independent heads are stored beside the spines, and a decode step copies them
        instead of walking them."""
        lib = L.load()
        arr = (L.FsbForest * self.nf)(*[self.struct(i) for i in range(self.nf)])
        sp = (L.vp * self.nf)(*[t.data_ptr() for t in self.spine])
        hd = (L.vp * self.nf)(*[t.data_ptr() for t in self.hdr])
        wd = None if widths is None else (L.i32 * self.nf)(*[int(w) for w in list(widths)[:self.nf]])
        L.check(lib.fsattn_fsb_spines(arr, self.nf, int(n_visible), sp, hd, wd, _stream(self.kbar)), "fsattn_fsb_spines")


def fsb_select(forests: FsbForests, Q, K, lam, sigma, *, scale: float, N: int = None, q_pos0: int = 0, Bq: int = 128,
               width: int = 16, width2: int = 16, read_top: int = 4, radius_coef: float = 8.0, pos=None,
               kq=None, ks=None, debug: bool = False, pdl: bool = False, beam_impl: int = 0):
    """FS-B selection. Prefill (pos None): Q (B,H,N,D) bf16 at positions q_pos0.., blocks of Bq -> sel (B,H,nb*Bq,K)
    int32. Decode (pos = device int64 scalar): Q (B,H,1,D), the spines of forests.build_spines -> sel (B,H,1,K).
    K: raw bf16 token keys (B,H,>=cells*32,D), or None with the int8 codes kq (B,H,rows,D) and scales ks (B,H,cells).
    debug=True also returns the candidates (B,H,Npad,width+width2) and the visit counts. beam_impl (prefill, whole
    128-query blocks): 0 = one thread per query with the block's distinct nodes scored on tensor-core tiles, 1 = one warp
    per query."""
    _need_cuda(Q, K, kq, ks)
    B, H, Nq, D = Q.shape
    decode = pos is not None
    N = Nq if N is None else int(N)
    if decode:
        N, Bq = 1, 1
    Bq = min(Bq, N) if not decode else 1
    nb = (N + Bq - 1) // Bq
    dev = Q.device
    sel = torch.empty(B, H, nb * Bq, read_top, dtype=torch.int32, device=dev)
    # full blocks hand their candidates to the block-cooperative re-rank through this buffer
    need_cand = debug or (not decode and Bq == 128)
    cand = torch.empty(B, H, nb * Bq, width + width2, dtype=torch.int32, device=dev) if need_cand else None
    nvis = torch.empty(B, H, nb * Bq, dtype=torch.int32, device=dev) if debug else None
    lam, sigma = _f32(lam).to(dev), _f32(sigma).to(dev)
    a = L.FsbSelect()
    a.main = forests.struct(0)
    a.second = forests.struct(1 if forests.nf > 1 else 0)
    a.q = _bhnd(Q, "Q")
    if K is not None:
        a.k = _bhnd(K, "K")
    else:
        a.k = _null()
        assert kq.dtype == torch.int8 and kq.stride(2) == D and ks.dtype == torch.bfloat16
        a.kq, a.ks = kq.data_ptr(), ks.data_ptr()
        a.kq_sb, a.kq_sh, a.ks_sb, a.ks_sh = kq.stride(0), kq.stride(1), ks.stride(0), ks.stride(1)
    a.lam, a.sigma = lam.data_ptr(), sigma.data_ptr()
    a.scale, a.radius_coef = float(scale), float(radius_coef)
    a.B, a.N, a.q_pos0, a.Bq = B, N, int(q_pos0), Bq
    a.width, a.width2, a.read_top = int(width), int(width2), int(read_top)
    if decode:
        a.use_spines = 1
        j = 1 if forests.nf > 1 else 0
        a.spine[0], a.spine[1] = forests.spine[0].data_ptr(), forests.spine[j].data_ptr()
        a.hdr[0], a.hdr[1] = forests.hdr[0].data_ptr(), forests.hdr[j].data_ptr()
        assert pos.dtype == torch.int64 and pos.is_cuda
        a.pos = pos.data_ptr()
        a.pdl = 1 if pdl else 0
    a.beam_impl = int(os.environ.get("FSATTN_FSB_BEAM_IMPL", beam_impl))      # A/B switch for measurements
    a.sel, a.cand, a.nvis = sel.data_ptr(), _p(cand), _p(nvis)
    L.call("fsattn_fsb_select", a, _stream(Q))
    return (sel, cand, nvis) if debug else sel



def linear_merge(ids, prio, mean, k, v, valid, *, P: int, Wc: int, first_id: int = 0, new_prio=None, new_mean=None,
                 new_k=None, new_v=None) -> None:
    """Block change of the streaming cache's pool (see fsattn_linear_merge_t): the new cells (statistics new_prio (B,H,n),
    new_mean (B,H,n,D); rows new_k / new_v (B,H,n*32,D) bf16, dense rows, any batch / head strides) enter the top list / the ring in place and `valid`
    is rewritten. Without new cells only `valid` is rewritten."""
    _need_cuda(ids, prio, mean, k, v, valid)
    B, H, C1 = ids.shape
    D = mean.shape[-1]
    assert C1 == P + Wc + 1 and ids.dtype == torch.int32 and prio.dtype == torch.float32 and mean.dtype == torch.float32
    assert k.dtype == torch.bfloat16 and v.dtype == torch.bfloat16 and valid.dtype == torch.uint8
    assert all(t.is_contiguous() for t in (ids, prio, mean, k, v, valid)) and k.shape[2] == C1 * CELL and valid.shape[-1] == C1 - 1
    a = L.LinearMerge()
    a.ids, a.prio, a.mean, a.k, a.v, a.valid = (t.data_ptr() for t in (ids, prio, mean, k, v, valid))
    a.B, a.H, a.D, a.P, a.Wc, a.first_id = B, H, D, int(P), int(Wc), int(first_id)
    a.count = 0
    if new_prio is not None:
        n = new_prio.shape[-1]
        assert new_prio.is_contiguous() and new_mean.is_contiguous()
        # the rows may be a token range of a longer buffer: dense rows, any batch / head strides, the same for k and v
        assert new_k.stride(-1) == 1 and new_k.stride(2) == D and new_v.stride() == new_k.stride()
        assert new_k.shape == (B, H, n * CELL, D) and new_k.dtype == torch.bfloat16 and new_v.shape == new_k.shape and new_v.dtype == new_k.dtype
        a.count = n
        a.new_prio, a.new_mean, a.new_k, a.new_v = new_prio.data_ptr(), new_mean.data_ptr(), new_k.data_ptr(), new_v.data_ptr()
        a.nk_sb, a.nk_sh = new_k.stride(0), new_k.stride(1)
    L.call("fsattn_linear_merge", a, _stream(ids))


def linear_select(q, ids, prio, mean, valid, lam, sigma, *, pos0: int, kk: int, kk_out: int, scale: float,
                  content_only: bool = False, want_ids: bool = False):
    """The streaming cache's selection (see fsattn_linear_select_t): q (B,H,n<=128,D) bf16 -> pool slots (B,H,n,kk_out)
    int32 (-1 none), and the cell ids when asked."""
    _need_cuda(q, ids, prio, mean, valid)
    B, H, n, D = q.shape
    C = valid.shape[-1]
    sel = torch.empty(B, H, n, kk_out, dtype=torch.int32, device=q.device)
    sid = torch.empty(B, H, n, kk_out, dtype=torch.int32, device=q.device) if want_ids else None
    lam, sigma = _f32(lam).to(q.device), _f32(sigma).to(q.device)
    a = L.LinearSelect()
    a.ids, a.prio, a.mean, a.valid = ids.data_ptr(), prio.data_ptr(), mean.data_ptr(), valid.data_ptr()
    a.q = _bhnd(q, "q")
    a.lam, a.sigma, a.scale = lam.data_ptr(), sigma.data_ptr(), float(scale)
    a.B, a.H, a.D, a.C, a.n, a.n_pad, a.kk, a.kk_out, a.pos0 = B, H, D, C, n, n, int(kk), int(kk_out), int(pos0)
    a.content_only = 1 if content_only else 0
    a.sel, a.sel_ids = sel.data_ptr(), _p(sid)
    L.call("fsattn_linear_select", a, _stream(q))
    return (sel, sid) if want_ids else sel


def embed_rows(tok: torch.Tensor, table: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
    """out (B,d) bf16 = table[tok[b]] for tok (B,) or (B,1) int64: the decode step's embedding lookup as one launch."""
    _need_cuda(tok, table, out)
    B = tok.numel()
    assert tok.dtype == torch.int64 and tok.is_contiguous() and table.dtype == torch.bfloat16 and table.is_contiguous()
    assert out.dtype == torch.bfloat16 and out.is_contiguous() and out.numel() == B * table.shape[1]
    L.check(L.load().fsattn_embed_rows(tok.data_ptr(), table.data_ptr(), out.data_ptr(), B, table.shape[1], table.shape[0],
                                       _stream(out)), "fsattn_embed_rows")
    return out


def argmax_advance(logits: torch.Tensor, tok: torch.Tensor, pos: torch.Tensor | None = None) -> torch.Tensor:
    """tok (B,) or (B,1) int64 = argmax over the last dim of logits (B,V) bf16 (lowest index on ties); pos (0-d int64 device
    tensor) is incremented when given: the decode step's sampling tail as one launch."""
    _need_cuda(logits, tok)
    assert logits.dim() == 2 and logits.dtype == torch.bfloat16 and logits.stride(1) == 1 and tok.dtype == torch.int64
    assert tok.is_contiguous() and tok.numel() == logits.shape[0] and (pos is None or (pos.dtype == torch.int64 and pos.is_cuda))
    L.check(L.load().fsattn_argmax_advance(logits.data_ptr(), logits.stride(0), logits.shape[0], logits.shape[1], tok.data_ptr(),
                                           _p(pos), _stream(logits)), "fsattn_argmax_advance")
    return tok


def swiglu(gu: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """out (..., f) = silu(gu[..., :f]) * gu[..., f:] for a fused gate/up projection gu (..., 2f) bf16, one pass."""
    _need_cuda(gu)
    assert gu.dtype == torch.bfloat16 and gu.stride(-1) == 1 and gu.shape[-1] % 16 == 0
    f = gu.shape[-1] // 2
    g2 = gu.reshape(-1, 2 * f)
    if out is None:
        out = torch.empty(*gu.shape[:-1], f, dtype=torch.bfloat16, device=gu.device)
    o2 = out.view(-1, f)
    L.check(L.load().fsattn_swiglu(g2.data_ptr(), g2.stride(0), o2.data_ptr(), o2.stride(0), g2.shape[0], f, _stream(gu)),
            "fsattn_swiglu")
    return out


def rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float, out: torch.Tensor | None = None) -> torch.Tensor:
    """out (..., d) = x * rsqrt(mean(x^2) + eps) * w for bf16 rows, fp32 arithmetic, one rounding; one read and one write."""
    _need_cuda(x, w)
    d = x.shape[-1]
    assert x.dtype == torch.bfloat16 and w.dtype == torch.bfloat16 and x.stride(-1) == 1 and w.is_contiguous() and w.numel() == d
    x2 = x.reshape(-1, d)
    if out is None:
        out = torch.empty(x.shape, dtype=torch.bfloat16, device=x.device)
    o2 = out.view(-1, d)
    L.check(L.load().fsattn_rms_norm(x2.data_ptr(), x2.stride(0), w.data_ptr(), float(eps), o2.data_ptr(), o2.stride(0),
                                     x2.shape[0], d, _stream(x)), "fsattn_rms_norm")
    return out
