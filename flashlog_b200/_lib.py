"""ctypes binding of libflashlog_b200.so (the C ABI in include/flashlog_b200.h).

The library is required: importing an op without it raises, there is no CPU
or library fallback.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libflashlog_b200.so")
CSRC = os.path.join(HERE, "csrc")
SOURCES = ["api.cu", "scan.cu", "topc.cu", "hop.cu", "rules.cu", "csr.cu", "readout.cu", "masks.cu"]
NVCC_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-lineinfo", "-std=c++17",
              "-fmad=false", "-Xcompiler", "-fPIC", "-shared"]

FL_SKIP_NONPOS_W = 1
FL_DROP_MASKED = 2
FL_WOT_I = 8
FL_SAMPLED = 16
FL_EDGE_SCORE = 32
FL_EDGE_WEIGHT = 64
FL_NO_ORI = 256
FL_NO_INV = 512
FL_EDGE_POS = 1024
FL_NO_NORMALIZE = 1 << 20
FL_MAX_BITS = 1
FL_MAX_VALUE_ONLY = 2
FL_MASK_U8 = 0
FL_MASK_F32 = 1
FL_ENTRY_INFO_INTS = 5  # int32 values per entry in fl_hop_params.entry_info
NO_BUDGET = 1 << 62
FL_STATUS_SLOT_OVERFLOW = 1


def build(force: bool = False, verbose: bool = False) -> str:
    """Compile the CUDA sources for sm_100a into flashlog_b200/libflashlog_b200.so."""
    srcs = [os.path.join(CSRC, s) for s in SOURCES]
    deps = srcs + [os.path.join(CSRC, h) for h in os.listdir(CSRC) if h.endswith(".cuh")]
    deps.append(os.path.join(os.path.dirname(HERE), "include", "flashlog_b200.h"))
    if not force and os.path.exists(LIB_PATH):
        t = os.path.getmtime(LIB_PATH)
        if all(os.path.getmtime(d) <= t for d in deps):
            return LIB_PATH
    nvcc = os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "bin", "nvcc")
    tmp = LIB_PATH + f".tmp{os.getpid()}"
    cmd = [nvcc, *NVCC_FLAGS, "-o", tmp, *srcs]
    if verbose:
        print(" ".join(cmd))
    subprocess.run(cmd, check=True, cwd=CSRC)
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


class fl_csr_side(ctypes.Structure):
    _fields_ = [("row_ptr", ctypes.c_void_p), ("col", ctypes.c_void_p), ("order", ctypes.c_void_p),
                ("group_ptr", ctypes.c_void_p), ("group_start", ctypes.c_void_p),
                ("group_count", ctypes.c_void_p), ("group_rel", ctypes.c_void_p)]


class fl_hop_params(ctypes.Structure):
    _fields_ = [("rows", ctypes.c_int64), ("L", ctypes.c_int64), ("n", ctypes.c_int64),
                ("r_size", ctypes.c_int64), ("E", ctypes.c_int64), ("topk_edges", ctypes.c_int64),
                ("flags", ctypes.c_int64), ("sampling_seed", ctypes.c_int64), ("eps", ctypes.c_float),
                ("slot_capacity", ctypes.c_int64), ("status", ctypes.c_void_p), ("entry_info", ctypes.c_void_p),
                ("vis_ori", ctypes.c_void_p), ("vis_inv", ctypes.c_void_p), ("work", ctypes.c_void_p),
                ("rel_rank", ctypes.c_void_p), ("rank_row", ctypes.c_void_p),
                ("row_order", ctypes.c_void_p), ("fact_edge", ctypes.c_void_p)]


_P = ctypes.c_void_p
_I64 = ctypes.c_int64
_SZ = ctypes.c_size_t
_SIDE = fl_csr_side
_PARAMS = ctypes.POINTER(fl_hop_params)


class fl_dropout(ctypes.Structure):
    """Mirror of fl_dropout (include/flashlog_b200.h): a fused dropout of hop values."""
    _fields_ = [("p", ctypes.c_double), ("seed", ctypes.c_uint64), ("counter", ctypes.c_void_p),
                ("subseq", ctypes.c_uint64)]


_DROP = ctypes.POINTER(fl_dropout)

# name -> (restype, argtypes)
SIGNATURES = {
    "fl_last_error": (ctypes.c_char_p, []),
    "fl_version": (ctypes.c_int, []),
    "fl_device_sm_count": (ctypes.c_int, []),
    "fl_launch_count": (ctypes.c_ulonglong, []),
    "fl_csr_build_workspace": (_SZ, [_I64, _I64]),
    "fl_csr_build_side": (ctypes.c_int, [_P, _P, _P, _I64, _I64, _I64, _P, _P, _P, _P, _P, _P, _P, _P,
                                         ctypes.POINTER(ctypes.c_int64), _P, _SZ, _P]),
    "fl_coo_to_rows": (ctypes.c_int, [_P, _P, _P, _I64, _I64, _I64, _I64, _P, _P, _P, _P]),
    "fl_rows_to_coo": (ctypes.c_int, [_P, _P, _I64, _I64, _I64, _P, _P]),
    "fl_topc_workspace": (_SZ, [_I64, _I64]),
    "fl_topc_select": (ctypes.c_int, [_P, _P, _P, _I64, _I64, _I64, _P, _P, _P, _P, _P, _I64, _P, _P, _SZ, _P]),
    "fl_topc_candidates": (ctypes.c_int, [_P, _P, _I64, _I64, _I64, ctypes.POINTER(ctypes.c_int64), _P, _SZ, _P]),
    "fl_hop_workspace": (_SZ, [_I64, _I64]),
    "fl_hop_plan": (ctypes.c_int, [_PARAMS, _P, _P, _I64, _SIDE, _SIDE, _P, ctypes.POINTER(ctypes.c_int64), _P,
                                   _SZ, _P]),
    "fl_csr_visibility": (ctypes.c_int, [_P, _I64, _P, _P, _P]),
    "fl_row_order": (ctypes.c_int, [_P, _P, _I64, _P, _P]),
    "fl_csr_mask": (ctypes.c_int, [_P, ctypes.c_int, _P, _I64, _P, _P, _P]),
    "fl_align_rows": (ctypes.c_int, [_P, _P, _P, _I64, _I64, _I64, _P, _P, _P, _P, _P]),
    "fl_relation_rank": (ctypes.c_int, [_P, _I64, _I64, _P, _P, _P]),
    "fl_hop_expand": (ctypes.c_int, [_PARAMS, _P, _P, _P, _I64, _P, _SIDE, _SIDE, _P, _P, _P, _P, _P, _P, _P, _P,
                                     _P, _P, _P]),
    "fl_reduce_workspace": (_SZ, [_I64, _I64]),
    "fl_row_reduce_max": (ctypes.c_int, [_P, _I64, _I64, _I64, _P, _P, _P, _P, _P, _I64, _P, _P, _P, _P,
                                         ctypes.c_int, _P, _P, _SZ, _P]),
    "fl_row_reduce": (ctypes.c_int, [_P, _I64, _I64, _P, _P, _P, _P, _I64, _P, ctypes.c_float, _P, _P, _P, _P, _P,
                                     _P, _P, _P, _SZ, _DROP, _P]),
    "fl_hop_backward_workspace": (_SZ, [_I64, _I64]),
    "fl_hop_backward": (ctypes.c_int, [_PARAMS, _P, _P, _I64, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P,
                                       _SZ, _P]),
    "fl_normalize_forward": (ctypes.c_int, [_P, _P, _I64, ctypes.c_float, _P, _P, _P]),
    "fl_normalize_backward": (ctypes.c_int, [_P, _P, _P, _P, _I64, ctypes.c_float, _P, _P]),
    "fl_hop_stats": (ctypes.c_int, [_P, _I64, _P, _I64, _SIDE, _SIDE, _P, _P, ctypes.c_int, _P, _P]),
    "fl_rule_max_reduce": (ctypes.c_int, [_P, _I64, _P, _P, _I64, _P, _I64, _I64, _I64, _P, _P]),
    "fl_scatter_grad": (ctypes.c_int, [_P, _P, _I64, _P, _P, _I64, _P, _DROP, _P]),
    "fl_edge_weight_grad": (ctypes.c_int, [_PARAMS, _P, _P, _I64, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P,
                                           _P]),
    "fl_readout": (ctypes.c_int, [_P, _P, _P, _I64, _P, _I64, _P, _P]),
    "fl_readout_backward": (ctypes.c_int, [_P, _P, _I64, _P, _I64, _P, _P, _I64, _P, _DROP, _P]),
    "fl_value_dropout": (ctypes.c_int, [_P, _P, _I64, _P, ctypes.c_double, ctypes.c_uint64, _P, ctypes.c_uint64,
                                        _P]),
    "fl_fixed_relation_workspace": (_SZ, [_I64]),
    "fl_fixed_relation_plan": (ctypes.c_int, [_P, _P, _P, _I64, _P, _I64, _I64, _SIDE, _SIDE, _P,
                                              ctypes.POINTER(ctypes.c_int64), _P, _SZ, _P]),
    "fl_fixed_relation_fill": (ctypes.c_int, [_P, _P, _P, _P, _I64, _P, _I64, _I64, _SIDE, _SIDE, _P, _P, _P, _P,
                                              _P]),
    "fl_rule_rank_facts": (ctypes.c_int, [_P, _P, _P, _I64, _I64, _P, _I64, _P, _P, _P, _P, _P, _P, _P]),
    "fl_rule_instance_facts": (ctypes.c_int, [_P, _P, _P, _I64, _P, _I64, _P, _P, _P, _P]),
    "fl_fixed_relation_bitmap": (ctypes.c_int, [_P, _I64, _P, _P, _P, _P, _I64, _SIDE, _SIDE, _P, _I64,
                                                _P]),
    "fl_rule_instance_max": (ctypes.c_int, [_P, _P, _P, _I64, _P, _I64, _I64, _P, _P]),
    "fl_bitmap_rows_workspace": (_SZ, [_I64, _I64]),
    "fl_rows_copy": (ctypes.c_int, [_P, _P, _I64, _P, _P, _P]),
    "fl_bitmap_rows_count": (ctypes.c_int, [_P, _I64, _I64, _P, _P, _P, _SZ, _P]),
    "fl_bitmap_rows_emit": (ctypes.c_int, [_P, _I64, _I64, _P, _P, _P]),
    "fl_filtered_ranks_workspace": (_SZ, [_I64]),
    "fl_filtered_ranks": (ctypes.c_int, [_P, _P, _P, _I64, _P, _P, _I64, _I64, _I64, ctypes.c_int, _P, _P, _SZ,
                                         _P]),
    "fl_filtered_ranks_noalloc": (ctypes.c_int, [_P, _P, _P, _I64, _P, _P, _I64, _I64, _I64, ctypes.c_int, _P, _P]),
}

_lib = None


def lib():
    """Load the library (raises if it was not built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"{LIB_PATH} is missing: build it with flashlog_b200._lib.build() "
                               "(there is no CPU fallback)")
        handle = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(handle, name)
            fn.restype = res
            fn.argtypes = args
        _lib = handle
    return _lib


class FlashLogError(RuntimeError):
    pass


def check(rc: int, what: str = ""):
    if rc != 0:
        msg = lib().fl_last_error().decode(errors="replace")
        if rc == 1:
            raise ValueError(f"{what}: {msg}")
        raise FlashLogError(f"{what}: {msg} (status {rc})")
