"""ctypes binding of libssd_b200.so, the sm_100a kernel library.

There is no fallback: if the library is missing or fails to load, every
operation that needs it raises. The library is built in-tree by
``csrc/build.py`` (``__graft_entry__.build()`` runs it).
"""

from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libssd_b200.so"

P = C.c_void_p
I64 = C.c_int64
I32 = C.c_int
F32 = C.c_float

SSD_OK, SSD_ERR_INVALID, SSD_ERR_UNSUPPORTED, SSD_ERR_CUDA, SSD_ERR_OVERFLOW, SSD_ERR_WORKSPACE = range(6)
SSD_F32, SSD_BF16 = 0, 1
ACT = {"none": 0, "silu": 1, "gelu": 2, "relu": 3}
SEG_CONCAT, SEG_PAIRS = 0, 1
EPI_STORE, EPI_RESIDUAL, EPI_SWIGLU, EPI_STORE_F32 = 0, 1, 2, 3

class SsdNormOut(C.Structure):
    """include/ssd_b200.h SsdNormOut: next RMSNorm input written by a residual epilogue."""
    _fields_ = [("weight", P), ("out", P), ("ldo", I64), ("ssq", P), ("ld_ssq", I64)]


class SsdRowNorm(C.Structure):
    """include/ssd_b200.h SsdRowNorm: per-row RMSNorm scale applied in a GEMM epilogue."""
    _fields_ = [("ssq", P), ("ld", I64), ("parts", I64), ("d", I64), ("eps", F32)]


class SsdLinearArgs(C.Structure):
    """include/ssd_b200.h SsdLinearArgs: one GEMM of ssd_linear_chain."""
    _fields_ = [("x", P), ("ldx", I64), ("K", I64), ("n_seg", C.c_int32), ("seg_layout", C.c_int32),
                ("w", P * 3), ("rows", I64 * 3), ("bias", P * 3), ("epilogue", C.c_int32), ("act", C.c_int32),
                ("out", P), ("ldo", I64), ("resid", P), ("ldr", I64), ("in_norm", SsdRowNorm),
                ("norm_out", SsdNormOut), ("n_heads", I64), ("n_kv_heads", I64), ("head_dim", I64),
                ("rope_cos", P), ("rope_sin", P), ("max_pos", I64), ("positions", P), ("slots", P),
                ("k_cache", P), ("v_cache", P), ("cache_head_stride", I64), ("max_slots", I64)]


EPI_QKV = 16
CHAIN_MAX = 6

TP_MAX_RANKS = 8


class SsdTpGroup(C.Structure):
    """include/ssd_b200.h SsdTpGroup: a tensor-parallel group's exchange regions."""
    _fields_ = [("rank", C.c_int32), ("world", C.c_int32), ("max_rows", I64), ("d", I64),
                ("peer_region", P * TP_MAX_RANKS)]


# name -> (restype, argtypes); mirrors include/ssd_b200.h
SIGNATURES: dict[str, tuple] = {
    "ssd_version": (I32, []),
    "ssd_launch_count": (I64, []),
    "ssd_last_error": (C.c_char_p, []),
    "ssd_device_sm_count": (I32, [I32]),
    "ssd_workspace_bytes": (I64, [I64, I64, I64]),
    "ssd_embed": (I32, [P, I64, P, I64, I64, I32, P, P, P, P]),
    "ssd_rmsnorm": (I32, [P, I64, I64, I64, P, F32, P, I64, I32, P]),
    "ssd_linear": (I32, [P, I64, I64, I64, I32, P, P, P, I32, I32, I32, P, I64, P, I64, I32, P, I64, P, P, P, P]),
    "ssd_linear_noalloc": (I32, [P, I64, I64, I64, I32, P, P, P, I32, I32, I32, P, I64, P, I64, I32, P, P]),
    "ssd_qkv_rope": (I32, [P, I64, I64, I64, P, P, P, I64, I64, I64, P, P, I64, P, P, P, P, I64, I64, P, I64, I32,
                           P, I64, P, P, P]),
    "ssd_tree_attention": (I32, [P, I64, I64, I64, I64, I64, P, P, I64, I64, P, P, P, P, I64, I64, P, I64, I32, P,
                                 I64, P, P]),
    "ssd_linear_chain": (I32, [C.c_int32, P, I64, I32, P, I64, P, P]),
    "ssd_head_argmax": (I32, [P, I64, I64, I64, P, I64, P, P, P, I32, P, I64, P, P, P]),
    "ssd_head_topk": (I32, [P, I64, I64, I64, P, I64, P, I64, P, P, I32, P, I64, P, P, P]),
    "ssd_level_prune": (I32, [P, P, I64, I64, I64, I64, P, P, P, P, P, P, P, P, P, I64, P, I32, I64, P, P, P, P, P,
                              P, I64, P, P]),
    "ssd_tree_prune": (I32, [P, I64, P, P, P, P, P, P, I64, P]),
    "ssd_verify_prep": (I32, [P, I64, P, P, P, P, P, P, P, P, P, P, P, I64, P, P]),
    "ssd_tree_walk_greedy": (I32, [P, I64, P, P, P, P, P, P, P, P, P, P, P]),
    "ssd_kv_compact": (I32, [P, I64, I64, I64, I64, I64, I64, P, P, P, I64, I32, P, P]),
    "ssd_round_commit": (I32, [P, P, P, P, P, P, P, P, I64, P, P, P]),
    "ssd_causal_prep": (I32, [P, I64, P, P, P, P, P, P]),
    "ssd_warp_params": (I32, [P, I64, I64, I64, F32, F32, P, P]),
    "ssd_warp_probs": (I32, [P, I64, I64, I64, P, P, I64, P]),
    "ssd_gumbel_topk": (I32, [P, I64, I64, I64, P, I64, P, P, P, I64, P, P, P]),
    "ssd_warp_sample_topk": (I32, [P, I64, I64, I64, F32, F32, I64, I64, P, P, P, I64, P, P, P, P]),
    "ssd_sample_token": (I32, [P, I64, F32, F32, P, P, I64, I64, P, P, P]),
    "ssd_tree_walk_sample": (I32, [P, I64, P, P, P, P, P, P, I64, P, I64, P, I64, P, I64, I64, P, P, P, P, P, P, P,
                                   P, P, P, P, P]),
    "ssd_tp_region_bytes": (I64, [I64, I64]),
    "ssd_tp_partial_offset": (I64, [I64, I64, I32]),
    "ssd_tp_set_spin_limit": (C.c_uint32, [C.c_uint32]),
    "ssd_tp_allreduce_residual": (I32, [P, I32, I64, P, I64, P, I32, P, P]),
    "ssd_tp_head_argmax": (I32, [P, P, I64, I64, I64, P, I64, I64, P, P, P, I32, P, I64, P, P, P]),
    "ssd_tp_head_topk": (I32, [P, P, I64, I64, I64, P, I64, I64, P, I64, P, P, I32, P, I64, P, P, P]),
    "ssd_fill_normal": (I32, [P, I64, I64, I64, I64, I64, I64, C.c_uint64, C.c_uint64, F32, F32, I32, P]),
}

_lib = None


class SSDError(RuntimeError):
    pass


def load() -> C.CDLL:
    """Load the kernel library (once). Raises if it is missing: no fallback."""
    global _lib
    if _lib is not None:
        return _lib
    path = Path(os.environ.get("SSD_B200_LIB", LIB_PATH))
    if not path.exists():
        raise SSDError(
            f"{path} not found: build it with `python subnetwork-speculative-decoding_b200/csrc/build.py` "
            "(the SSD B200 path has no CPU fallback)"
        )
    lib = C.CDLL(str(path))
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def exported_symbols() -> list[str]:
    return list(SIGNATURES)


def check(rc: int, what: str) -> None:
    """Map a status code to the Python exception the reference raises."""
    if rc == SSD_OK:
        return
    msg = load().ssd_last_error().decode(errors="replace")
    text = f"{what}: {msg} (status {rc})"
    if rc == SSD_ERR_INVALID:
        raise ValueError(text)
    if rc == SSD_ERR_OVERFLOW:
        raise RuntimeError(text)
    raise SSDError(text)


def launch_count() -> int:
    """Kernels the library launched (or captured into a graph) so far, counted
    by the library itself at every launch."""
    return int(load().ssd_launch_count())


def call(name: str, *args) -> None:
    check(getattr(load(), name)(*args), name)
