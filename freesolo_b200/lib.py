"""ctypes binding of libfsattn_b200.so (the C ABI declared in include/fsattn_b200.h).

The library is built in-tree by ``freesolo_b200/csrc/build.sh`` (``__graft_entry__.build()``). There is no fallback:
if the shared object is missing or a call is rejected, a RuntimeError is raised.
"""
from __future__ import annotations

import ctypes as C
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libfsattn_b200.so")

OK, EINVAL, EUNSUPPORTED, ELAUNCH = 0, -1, -2, -3
CELL = 32
MAX_POOL = 128
MAX_KK = 8
WINDOW_STATIC_BYTES = 32 * 1024 * 1024
ST_SLOT_OVERFLOW, ST_POOL_NO_SLOT, ST_BAD_INDEX, ST_WORDS = 0, 1, 2, 4

i32, i64, f32, vp = C.c_int32, C.c_int64, C.c_float, C.c_void_p


class BHND(C.Structure):
    _fields_ = [("ptr", vp), ("sb", i64), ("sh", i64), ("sn", i64)]


class CellIngest(C.Structure):
    _fields_ = [("k", BHND), ("v", BHND),
                ("B", i32), ("H", i32), ("D", i32), ("ncell", i32), ("cell0", i32),
                ("kbar", vp), ("kbar_sb", i64), ("kbar_sh", i64),
                ("ceil", vp), ("ceil_sb", i64), ("ceil_sh", i64),
                ("kq", vp), ("vq", vp), ("q_sb", i64), ("q_sh", i64),
                ("ks", vp), ("vs", vp), ("sc_sb", i64), ("sc_sh", i64)]


class Dequant(C.Structure):
    _fields_ = [("q", vp), ("q_sb", i64), ("q_sh", i64),
                ("sc", vp), ("sc_sb", i64), ("sc_sh", i64),
                ("out", vp), ("o_sb", i64), ("o_sh", i64),
                ("B", i32), ("H", i32), ("D", i32), ("nrows", i64)]


class FslTopp(C.Structure):
    _fields_ = [("ceil", vp), ("ceil_sb", i64), ("ceil_sh", i64),
                ("B", i32), ("H", i32), ("ncell", i32), ("Bq", i32), ("nb", i32), ("P", i32),
                ("topp", vp)]


class FslSelect(C.Structure):
    _fields_ = [("q", BHND),
                ("kbar", vp), ("kbar_sb", i64), ("kbar_sh", i64),
                ("ceil", vp), ("ceil_sb", i64), ("ceil_sh", i64),
                ("topp", vp), ("lam", vp), ("sigma", vp),
                ("B", i32), ("H", i32), ("D", i32), ("N", i32), ("ncell", i32), ("Bq", i32), ("nb", i32),
                ("P", i32), ("Wc", i32), ("kk", i32),
                ("scale", f32),
                ("sel", vp), ("margin", vp),
                ("topp_nb", i32), ("impl", i32)]


class FsDenseSelect(C.Structure):
    _fields_ = [("q", BHND),
                ("kbar", vp), ("kbar_sb", i64), ("kbar_sh", i64),
                ("ceil", vp), ("ceil_sb", i64), ("ceil_sh", i64),
                ("lam", vp), ("sigma", vp),
                ("B", i32), ("H", i32), ("D", i32), ("N", i32), ("ncell", i32), ("Bq", i32), ("nb", i32), ("kk", i32),
                ("scale", f32),
                ("sel", vp),
                ("workspace", vp), ("workspace_bytes", i64),
                ("status", vp)]


class FsDenseDecodeSelect(C.Structure):
    _fields_ = [("q", vp), ("q_sb", i64), ("q_sh", i64),
                ("kbar", vp), ("kbar_sb", i64), ("kbar_sh", i64),
                ("ceil", vp), ("ceil_sb", i64), ("ceil_sh", i64),
                ("lam", vp), ("sigma", vp),
                ("pos", vp),
                ("B", i32), ("H", i32), ("D", i32), ("Bq", i32), ("kk", i32), ("ncell_cap", i32), ("splits", i32), ("pdl", i32),
                ("scale", f32),
                ("sel", vp)]


class WindowPrefill(C.Structure):
    _fields_ = [("q", BHND), ("k", BHND), ("v", BHND),
                ("cos", vp), ("sin", vp),
                ("B", i32), ("H", i32), ("D", i32), ("N", i32), ("W", i32), ("pos0", i32),
                ("scale", f32),
                ("out", vp),
                ("impl", i32),
                ("workspace", vp), ("workspace_bytes", i64),
                ("status", vp)]


class ReadoutCombine(C.Structure):
    _fields_ = [("q", BHND), ("k", BHND), ("v", BHND),
                ("sel", vp), ("sel_sb", i64), ("sel_sh", i64),
                ("sr", vp), ("y", vp),
                ("norm_w", vp), ("lrs", vp),
                ("B", i32), ("H", i32), ("D", i32), ("N", i32), ("n_kv", i32), ("Bq", i32), ("kk", i32),
                ("q_pos0", i32),
                ("scale", f32), ("eps", f32), ("impl", i32)]


class FslState(C.Structure):
    _fields_ = [("store_mode", i32), ("B", i32), ("H", i32), ("D", i32), ("P", i32), ("Wc", i32), ("W", i32),
                ("Bq", i32), ("kk", i32), ("n_slots", i32),
                ("cap_rows", i64), ("cap_cells", i64),
                ("kbuf", vp), ("vbuf", vp), ("buf_sb", i64), ("buf_sh", i64),
                ("kq", vp), ("vq", vp), ("q_sb", i64), ("q_sh", i64),
                ("ks", vp), ("vs", vp), ("sc_sb", i64), ("sc_sh", i64),
                ("khot", vp), ("vhot", vp), ("hot_sb", i64), ("hot_sh", i64),
                ("kbar", vp), ("kbar_sb", i64), ("kbar_sh", i64),
                ("ceil", vp), ("ceil_sb", i64), ("ceil_sh", i64),
                ("slot_of", vp), ("so_sb", i64), ("so_sh", i64),
                ("cell_in", vp), ("ci_sb", i64), ("ci_sh", i64),
                ("top_idx", vp), ("top_blk", vp),
                ("pool_kbar", vp), ("pool_meta", vp), ("pool_blk", vp),
                ("status", vp)]


class FslDecode(C.Structure):
    _fields_ = [("st", FslState),
                ("q", vp), ("k", vp), ("v", vp), ("in_sb", i64), ("in_sh", i64),
                ("pos", vp),
                ("cos", vp), ("sin", vp),
                ("lam", vp), ("sigma", vp), ("lrs", vp), ("norm_w", vp),
                ("scale", f32), ("eps", f32),
                ("y", vp), ("sel_out", vp),
                ("splits", i32), ("pdl", i32), ("ext_sel", vp), ("window_path", i32)]


class SlotPrefill(C.Structure):
    _fields_ = [("st", FslState), ("k", BHND), ("v", BHND),
                ("kbar_cells", vp), ("kc_sb", i64), ("kc_sh", i64),
                ("N", i32)]


class TrunkGemv(C.Structure):
    _fields_ = [("w", vp), ("x", vp), ("x_stride", i64),
                ("norm_w", vp), ("eps", f32),
                ("out", vp), ("out_stride", i64),
                ("res", vp), ("res_stride", i64),
                ("M", i32), ("K", i32), ("n_out", i32), ("epilogue", i32), ("m0", i32), ("pdl", i32)]


EPI_STORE, EPI_RESIDUAL, EPI_SWIGLU = 0, 1, 2


class TrunkLayer(C.Structure):
    _fields_ = [("x", vp), ("x_stride", i64),
                ("y", vp), ("y_stride", i64),
                ("w_o", vp),
                ("norm2_w", vp), ("eps2", f32),
                ("w_gu", vp),
                ("act", vp), ("act_stride", i64),
                ("w_down", vp),
                ("norm_next_w", vp), ("eps_next", f32),
                ("w_next", vp), ("out_next", vp), ("out_next_stride", i64), ("n_next", i32),
                ("bar", vp), ("status", vp),
                ("M", i32), ("d", i32), ("f", i32), ("pdl", i32)]


class FsbForest(C.Structure):
    _fields_ = [("T", i32), ("H", i32), ("D", i32), ("m_cap", i32),
                ("kbar", vp), ("kbar_st", i64), ("ceil", vp), ("ceil_st", i64), ("tau", vp),
                ("adm", vp), ("m_tot", vp), ("m_prev", vp),
                ("node_mu", vp), ("node_aux", vp), ("root32", vp), ("compact", i32)]


class LinearMerge(C.Structure):
    _fields_ = [("ids", vp), ("prio", vp), ("mean", vp), ("k", vp), ("v", vp), ("valid", vp),
                ("new_prio", vp), ("new_mean", vp), ("new_k", vp), ("new_v", vp), ("nk_sb", i64), ("nk_sh", i64),
                ("B", i32), ("H", i32), ("D", i32), ("P", i32), ("Wc", i32), ("count", i32), ("first_id", i32)]


class LinearSelect(C.Structure):
    _fields_ = [("ids", vp), ("prio", vp), ("mean", vp), ("valid", vp),
                ("q", BHND), ("lam", vp), ("sigma", vp), ("scale", f32),
                ("B", i32), ("H", i32), ("D", i32), ("C", i32), ("n", i32), ("n_pad", i32), ("kk", i32), ("kk_out", i32),
                ("pos0", i32), ("content_only", i32), ("sel", vp), ("sel_ids", vp)]


class FsbSelect(C.Structure):
    _fields_ = [("main", FsbForest), ("second", FsbForest), ("q", BHND), ("k", BHND),
                ("kq", vp), ("ks", vp), ("kq_sb", i64), ("kq_sh", i64), ("ks_sb", i64), ("ks_sh", i64),
                ("lam", vp), ("sigma", vp), ("scale", f32), ("radius_coef", f32),
                ("B", i32), ("N", i32), ("q_pos0", i32), ("Bq", i32), ("width", i32), ("width2", i32), ("read_top", i32),
                ("use_spines", i32), ("spine", vp * 2), ("hdr", vp * 2), ("pos", vp),
                ("sel", vp), ("cand", vp), ("nvis", vp), ("pdl", i32), ("beam_impl", i32)]


FSB_SPINE_MAX = 20
FSB_MAX_MCAP = 16384
PEER_MAX = 8
PEER_HANDLE_BYTES = 64


class PeerGather(C.Structure):
    _fields_ = [("y_local", vp), ("y_out", vp), ("ll_dst", vp * PEER_MAX), ("epoch", vp), ("status", vp),
                ("B", i32), ("dl", i32), ("rank", i32), ("world", i32), ("slot", i32), ("pdl", i32), ("timeout_ns", i64)]


EXTRA_STRUCTS = {"fsattn_fs_dense_select_t": FsDenseSelect, "fsattn_fs_dense_decode_select_t": FsDenseDecodeSelect,
                 "fsattn_trunk_gemv_t": TrunkGemv, "fsattn_trunk_layer_t": TrunkLayer, "fsattn_fsb_forest_t": FsbForest, "fsattn_fsb_select_t": FsbSelect,
                 "fsattn_linear_merge_t": LinearMerge, "fsattn_linear_select_t": LinearSelect,
                 "fsattn_peer_gather_t": PeerGather}

# every exported symbol of include/fsattn_b200.h with its argument struct (None = no struct argument)
ENTRY_POINTS = {
    "fsattn_version": None,
    "fsattn_last_error": None,
    "fsattn_init": None,
    "fsattn_cell_ingest": CellIngest,
    "fsattn_dequant_cells": Dequant,
    "fsattn_fsl_prefix_topp": FslTopp,
    "fsattn_fsl_select": FslSelect,
    "fsattn_fs_dense_workspace_bytes": ([i32, i32, i32, i32], i64),
    "fsattn_fs_dense_select": FsDenseSelect,
    "fsattn_fs_dense_decode_select": FsDenseDecodeSelect,
    "fsattn_window_prefill": WindowPrefill,
    "fsattn_window_prefill_static": WindowPrefill,
    "fsattn_readout_combine": ReadoutCombine,
    "fsattn_fsl_decode_step": FslDecode,
    "fsattn_slot_prefill": SlotPrefill,
    "fsattn_trunk_gemv": TrunkGemv,
    "fsattn_trunk_layer": TrunkLayer,
    "fsattn_swiglu": ([vp, i64, vp, i64, i64, i32, vp], C.c_int),
    "fsattn_embed_rows": ([vp, vp, vp, i32, i32, i64, vp], C.c_int),
    "fsattn_argmax_advance": ([vp, i64, i32, i32, vp, vp, vp], C.c_int),
    "fsattn_rms_norm": ([vp, i64, vp, f32, vp, i64, i64, i32, vp], C.c_int),
    "fsattn_fsb_scratch_floats": ([i32, i32, i32], i64),
    "fsattn_fsb_ingest": ([C.POINTER(FsbForest), i32, i32, i32, vp, i64, vp], C.c_int),
    "fsattn_fsb_compact": ([C.POINTER(FsbForest), C.POINTER(FsbForest), vp], C.c_int),
    "fsattn_linear_merge": LinearMerge,
    "fsattn_linear_select": LinearSelect,
    "fsattn_fsb_spines": ([C.POINTER(FsbForest), i32, i32, C.POINTER(vp), C.POINTER(vp), C.POINTER(i32), vp], C.c_int),
    "fsattn_fsb_select": FsbSelect,
    "fsattn_peer_gather": PeerGather,
    "fsattn_peer_ll_bytes": ([i32, i32, i32, i32], i64),
    "fsattn_peer_alloc": ([i64, C.POINTER(vp)], C.c_int),
    "fsattn_peer_free": ([vp], C.c_int),
    "fsattn_peer_export": ([vp, C.c_char_p], C.c_int),
    "fsattn_peer_open": ([C.c_char_p, C.POINTER(vp)], C.c_int),
    "fsattn_peer_close": ([vp], C.c_int),
}

_lib = None
_inited = set()


def load() -> C.CDLL:
    """The loaded library; raises if the extension has not been built."""
    global _lib
    if _lib is None:
        if not os.path.isfile(LIB_PATH):
            raise RuntimeError(f"{LIB_PATH} is missing: build it with freesolo_b200/csrc/build.sh "
                               "(__graft_entry__.build()); there is no fallback path")
        lib = C.CDLL(LIB_PATH)
        lib.fsattn_version.restype = C.c_int
        lib.fsattn_last_error.restype = C.c_char_p
        lib.fsattn_init.argtypes = [C.c_int]
        lib.fsattn_init.restype = C.c_int
        for name, st in ENTRY_POINTS.items():
            fn = getattr(lib, name)         # AttributeError here = header and library disagree
            if isinstance(st, tuple):       # (argtypes, restype): entry points that do not take one struct
                fn.argtypes, fn.restype = st
            elif st is not None:
                fn.argtypes = [C.POINTER(st), vp]
                fn.restype = C.c_int
        _lib = lib
    return _lib


def last_error() -> str:
    return load().fsattn_last_error().decode("utf-8", "replace")


def check(rc: int, what: str) -> None:
    if rc != OK:
        kind = {EINVAL: "invalid argument", EUNSUPPORTED: "unsupported configuration", ELAUNCH: "launch failure"}.get(rc, rc)
        raise RuntimeError(f"{what}: {kind}: {last_error()}")


def init(device_index: int) -> None:
    if device_index not in _inited:
        check(load().fsattn_init(int(device_index)), "fsattn_init")
        _inited.add(device_index)


def call(name: str, args: C.Structure, stream_ptr: int) -> None:
    check(getattr(load(), name)(C.byref(args), vp(stream_ptr)), name)
