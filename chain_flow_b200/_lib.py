"""ctypes binding of libcfb.so (include/cfb.h).

The product path is CUDA only: importing the binding never falls back to anything. If the
shared library is missing it is built in-tree with nvcc (chain_flow_b200/build.py); if that is
impossible, or no CUDA device is visible when a kernel is requested, the call raises.
"""
from __future__ import annotations

import ctypes as C
import threading
from pathlib import Path

_PKG = Path(__file__).resolve().parent
LIB_PATH = _PKG / "libcfb.so"

CFB_OK = 0
STATUS_NAMES = {
    0: "CFB_OK", 1: "CFB_ERR_INVALID_ARG", 2: "CFB_ERR_UNSUPPORTED", 3: "CFB_ERR_WORKSPACE",
    4: "CFB_ERR_CUDA", 5: "CFB_ERR_COOP_LAUNCH", 6: "CFB_ERR_DEVICE_TIMEOUT",
}
MODE_FLOW, MODE_CHAIN, MODE_TREE, MODE_BEAM_CHAIN, MODE_BEAM_TREE = range(5)
INIT_GIVEN, INIT_REPEAT_LAST, INIT_DELTA = range(3)
INIT_MODES = {"noise": INIT_GIVEN, "repeat_last": INIT_REPEAT_LAST, "delta": INIT_DELTA}

# every extern "C" symbol declared in include/cfb.h
EXPORTED = [
    "cfb_abi_version", "cfb_last_cuda_error", "cfb_packed_bytes", "cfb_pack_linear",
    "cfb_fold_bias", "cfb_time_embed", "cfb_plan_workspace", "cfb_plan_build", "cfb_plan_run",
    "cfb_plan_error", "cfb_plan_info", "cfb_plan_buffer", "cfb_tree_gdn", "cfb_tree_gdn_noalloc",
    "cfb_plan_segments", "cfb_plan_run_segment", "cfb_wide_gemm", "cfb_wide_packed_bytes", "cfb_wide_pack", "cfb_wide_workspace",
    "cfb_wide_create", "cfb_wide_run", "cfb_wide_error", "cfb_wide_info", "cfb_wide_destroy",
    "cfb_ring_write", "cfb_ring_gather", "cfb_tree_gdn_verify", "cfb_vae_workspace", "cfb_vae_create",
    "cfb_vae_plan_workspace", "cfb_vae_plan_build", "cfb_tree_attn_merge", "cfb_tree_verify_workspace",
    "cfb_tree_verify_greedy", "cfb_tree_gdn_factor",
]
ABI_VERSION = 5
XROWS, XFLOATS = 64, 18          # CFB_XROWS, CFB_XFLOATS: the merged-list exchange rows
BUF_PATH_H16, BUF_PATH_MID, BUF_HEAD_IN, BUF_LASTP, BUF_CUM, BUF_QKV0, BUF_X32_0, BUF_KVC0, BUF_PROF, BUF_PHASES, \
    BUF_TP_CAND, BUF_TP_CHEAD = range(12)
PK_PREP, PK_GEMM, PK_ATTN, PK_BEAM, PK_RMERGE, PK_GATHER, PK_TPXA, PK_TPSEL, PK_TPGATH = range(9)  # CFB_BUF_PHASES [0]
PO_NONE, PO_BEAM_CHAIN, PO_BEAM_TREE, PO_PUBLISH = range(4)        # CFB_BUF_PHASES [6]
RUN_PROFILE = 1
# device error word codes (cfb_plan_error / cfb_wide_error)
DEV_ERRORS = {1: "grid barrier wait expired", 2: "loaded-stage wait expired", 3: "free-stage wait expired",
              4: "slot or descriptor wait expired", 5: "bad phase", 6: "split-tile wait expired",
              7: "token or row id outside its table"}
EPI_F32, EPI_F16, EPI_GELU16, EPI_PART = 0, 1, 2, 3      # cfb_wide_gemm epilogues


class CfbError(RuntimeError):
    pass


class Linear(C.Structure):
    _fields_ = [("w", C.c_void_p), ("bias", C.c_void_p), ("colsum", C.c_void_p),
                ("nout", C.c_int), ("k", C.c_int)]


class Block(C.Structure):
    _fields_ = [("qkv", Linear), ("self_out", Linear), ("cross_q", Linear), ("cross_kv", Linear),
                ("cross_out", Linear), ("ffn_up", Linear), ("ffn_down", Linear)]


class Expert(C.Structure):
    _fields_ = [("pos_emb", C.c_void_p), ("temb", C.c_void_p), ("out_proj", Linear),
                ("blocks", C.POINTER(Block))]


class Drafter(C.Structure):
    _fields_ = [("hidden", C.c_int), ("heads", C.c_int), ("layers", C.c_int), ("steps", C.c_int),
                ("draft_len", C.c_int), ("chunk", C.c_int), ("ctx_rows", C.c_int),
                ("n_experts", C.c_int), ("experts", C.POINTER(Expert)),
                ("path_order", C.c_int), ("markov_rank", C.c_int), ("vocab", C.c_int),
                ("shortlist_rows", C.c_int), ("embed", C.c_void_p), ("path_offsets", Linear),
                ("path_offset_bias", C.c_void_p), ("path_up", Linear), ("path_down", Linear),
                ("markov_w1", C.c_void_p), ("head", Linear), ("shortlist", C.c_void_p),
                ("head_row0", C.c_int)]


class Run(C.Structure):
    _fields_ = [("mode", C.c_int), ("init_mode", C.c_int), ("batch", C.c_int), ("width", C.c_int), ("depth", C.c_int),
                ("tree_keep", C.c_int), ("tree_topb", C.c_int), ("grid", C.c_int), ("flags", C.c_int),
                ("ctx", C.c_void_p), ("z0", C.c_void_p), ("known0", C.c_void_p),
                ("pred", C.c_void_p), ("tokens", C.c_void_p),
                ("ranks", C.c_int), ("rank", C.c_int), ("xloc", C.c_void_p), ("xall", C.c_void_p),
                ("twopass_m", C.c_int), ("wait_budget_ns", C.c_uint64)]


class VaeLayer(C.Structure):
    _fields_ = [("qkv", Linear), ("attn_out", Linear), ("ffn_up", Linear), ("ffn_down", Linear)]


class VaeSide(C.Structure):
    _fields_ = [("in_dim", C.c_int), ("width", C.c_int), ("out_dim", C.c_int), ("layers", C.c_int),
                ("heads", C.c_int), ("max_len", C.c_int), ("in_proj", Linear), ("pos", C.c_void_p),
                ("layer", C.POINTER(VaeLayer)), ("out_proj", Linear)]


_lock = threading.Lock()
_lib = None


def _declare(lib):
    vp, i32, i64, sz = C.c_void_p, C.c_int, C.c_int64, C.c_size_t
    lib.cfb_abi_version.restype = i32
    lib.cfb_last_cuda_error.restype = C.c_char_p
    lib.cfb_packed_bytes.argtypes = [i32, i32]
    lib.cfb_packed_bytes.restype = sz
    lib.cfb_pack_linear.argtypes = [vp, i64, vp, i32, i32, vp, vp, i32, i32, vp]
    lib.cfb_fold_bias.argtypes = [vp, i64, i32, i32, vp, vp, vp, vp, vp, vp]
    lib.cfb_time_embed.argtypes = [vp, vp, vp, vp, i32, i32, vp, vp]
    lib.cfb_plan_workspace.argtypes = [C.POINTER(Drafter), C.POINTER(Run), C.POINTER(sz)]
    lib.cfb_plan_build.argtypes = [C.POINTER(Drafter), C.POINTER(Run), vp, sz]
    lib.cfb_plan_run.argtypes = [vp, vp]
    lib.cfb_plan_segments.argtypes = [vp, C.POINTER(i32)]
    lib.cfb_plan_run_segment.argtypes = [vp, i32, vp]
    lib.cfb_plan_error.argtypes = [vp, C.POINTER(i32)]
    lib.cfb_plan_info.argtypes = [vp, C.POINTER(i32), C.POINTER(i32), C.POINTER(i32), C.POINTER(i32)]
    lib.cfb_plan_buffer.argtypes = [vp, i32, C.POINTER(vp), C.POINTER(sz)]
    lib.cfb_tree_gdn.argtypes = [vp, vp, vp, vp, vp, vp, vp, vp, vp, i32, i32, i32, i32, i32, i32, vp]
    lib.cfb_tree_gdn_noalloc.argtypes = [vp, vp, vp, vp, vp, vp, vp, vp, i32, i32, i32, i32, i32, i32, vp]
    lib.cfb_wide_gemm.argtypes = [vp, i64, vp, i64, vp, vp, i64, i32, i32, i32, i32, i32, vp, vp]
    lib.cfb_wide_packed_bytes.argtypes = [i32, i32]
    lib.cfb_wide_packed_bytes.restype = sz
    lib.cfb_wide_pack.argtypes = [vp, i64, i32, i32, vp, vp]
    lib.cfb_wide_workspace.argtypes = [C.POINTER(Drafter), C.POINTER(Run), C.POINTER(sz)]
    lib.cfb_wide_create.argtypes = [C.POINTER(Drafter), C.POINTER(Run), vp, sz, C.POINTER(vp)]
    lib.cfb_wide_run.argtypes = [vp, vp]
    lib.cfb_wide_error.argtypes = [vp, C.POINTER(i32)]
    lib.cfb_wide_info.argtypes = [vp, C.POINTER(i32)]
    lib.cfb_wide_destroy.argtypes = [vp]
    lib.cfb_wide_destroy.restype = None
    lib.cfb_ring_write.argtypes = [vp, vp, vp, i32, i32, i32, vp, i64, vp, vp, vp, vp, vp, i64, i32, i32, vp]
    lib.cfb_ring_gather.argtypes = [vp, vp, vp, i32, i32, i32, vp, i32, vp, vp]
    lib.cfb_tree_gdn_verify.argtypes = [vp, i32, vp, i32, vp, i32, vp, i32, vp, vp, vp, vp, i32, vp, i64, vp, i32,
                                        vp, vp, vp, vp, C.c_float, i32, i32, i32, i32, i32, i32, i32, vp]
    lib.cfb_vae_workspace.argtypes = [C.POINTER(VaeSide), i32, i32, i32, C.POINTER(sz)]
    lib.cfb_vae_create.argtypes = [C.POINTER(VaeSide), i32, i32, i32, vp, vp, vp, sz, C.POINTER(vp)]
    lib.cfb_vae_plan_workspace.argtypes = [C.POINTER(VaeSide), i32, i32, i32, C.POINTER(sz)]
    lib.cfb_vae_plan_build.argtypes = [C.POINTER(VaeSide), i32, i32, i32, vp, vp, vp, sz]
    lib.cfb_tree_attn_merge.argtypes = [vp, i64, i64, vp, i64, i64, vp, i64, i64, vp, i64, i64, vp, i64, i64,
                                        vp, vp, vp, C.c_float, i32, i32, i32, i32, i32, i32, vp]
    lib.cfb_tree_gdn_factor.argtypes = [vp, i32, vp, i32, vp, i32, vp, i32, vp, vp, vp, vp, i32, vp, i64, vp, i32,
                                        vp, vp, vp, vp, i32, i32, C.c_float, i32, i32, i32, i32, vp]
    lib.cfb_tree_verify_workspace.argtypes = [i32, i32]
    lib.cfb_tree_verify_workspace.restype = sz
    lib.cfb_tree_verify_greedy.argtypes = [vp, i64, i32, i32, i32, vp, vp, vp, vp, i32, i32, vp, vp, vp, vp, vp,
                                           sz, vp, vp]
    return lib


def load(build_if_missing: bool = True):
    """The loaded libcfb.so (built in-tree with nvcc on first use if it is missing)."""
    global _lib
    with _lock:
        if _lib is None:
            if build_if_missing and not LIB_PATH.exists():
                from . import build as _build
                _build.build()
            if not LIB_PATH.exists():
                raise CfbError(f"{LIB_PATH} is missing; build it with `python -m chain_flow_b200.build`")
            _lib = _declare(C.CDLL(str(LIB_PATH)))
            if _lib.cfb_abi_version() != ABI_VERSION:
                raise CfbError("libcfb.so ABI version mismatch; rebuild it")
    return _lib


def check(status: int, what: str) -> None:
    if status != CFB_OK:
        lib = load(False)
        detail = lib.cfb_last_cuda_error().decode(errors="replace") if status == 4 else ""
        raise CfbError(f"{what}: {STATUS_NAMES.get(status, status)} {detail}".strip())


def stream_ptr(stream=None) -> int:
    import torch
    s = stream if stream is not None else torch.cuda.current_stream()
    return s.cuda_stream


def require_cuda(t, name: str) -> None:
    if not t.is_cuda:
        raise CfbError(f"{name} must be a CUDA tensor: the chain_flow_b200 engine has no CPU path")
