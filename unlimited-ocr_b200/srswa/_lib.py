"""ctypes binding of libsrswa.so (the C ABI declared in include/srswa.h).

The library is required: importing a compute entry point without it, or
calling one on a machine without a CUDA device, raises -- there is no CPU
fallback anywhere in this package.
"""

from __future__ import annotations

import ctypes as C
import os

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.environ.get("SRSWA_LIB", os.path.join(_HERE, "libsrswa.so"))

F32, BF16, F16, F8E4M3, F8E5M2 = 0, 1, 2, 3, 4
# fp8 only where an entry point accepts it (the attends' K/V caches)
_DTYPES = {torch.float32: F32, torch.bfloat16: BF16, torch.float16: F16, torch.float8_e4m3fn: F8E4M3,
           torch.float8_e5m2: F8E5M2}

EINVAL, EUNSUPPORTED, EALIGN, EWORKSPACE, ETOOLARGE = -1, -2, -3, -4, -5

i64 = C.c_int64
vp = C.c_void_p


class RouteParams(C.Structure):
    _fields_ = [("block_size", i64), ("local_blocks", i64), ("topk", i64), ("topm", i64),
                ("idx_scale", C.c_float), ("prior_floor", C.c_float), ("sigma", C.c_float)]


class GatherDesc(C.Structure):
    _fields_ = [("B", i64), ("T", i64), ("HQ", i64), ("Hkv", i64), ("HI", i64), ("D", i64), ("S", i64),
                ("block_size", i64), ("local_window", i64), ("scale", C.c_float), ("dtype", C.c_int),
                ("sqb", i64), ("sqt", i64), ("sqh", i64), ("skb", i64), ("skt", i64), ("skh", i64),
                ("svb", i64), ("svt", i64), ("svh", i64)]


class DecodeDesc(C.Structure):
    _fields_ = [("N", i64), ("H", i64), ("Hkv", i64), ("D", i64), ("K", i64),
                ("block_size", i64), ("local_blocks", i64), ("sm_scale", C.c_float),
                ("q_dtype", C.c_int), ("kv_dtype", C.c_int), ("out_dtype", C.c_int),
                ("s_qn", i64), ("s_qh", i64), ("s_page", i64), ("s_pos", i64), ("s_head", i64),
                ("s_on", i64), ("s_oh", i64), ("R", i64), ("W", i64), ("s_req", i64),
                ("rows_per_req", i64), ("idx_is64", C.c_int), ("s_ti_h", i64), ("s_ti_n", i64),
                ("s_b_h", i64), ("s_b_n", i64), ("nsplit", C.c_int), ("skip_local", C.c_int),
                ("overlap", C.c_int)]


class KlDesc(C.Structure):
    _fields_ = [(n, i64) for n in ("B", "C", "Sk", "H", "Hkv", "D", "d", "S", "block_size", "local_window")] + \
               [("scaling", C.c_float), ("logits_bf16", C.c_int), ("iq_dtype", C.c_int), ("ik_dtype", C.c_int),
                ("qm_dtype", C.c_int), ("km_dtype", C.c_int)] + \
               [(n, i64) for n in ("s_iq_b", "s_iq_c", "s_ik_b", "s_ik_s", "s_qm_b", "s_qm_c", "s_qm_h", "s_km_b",
                                   "s_km_s", "s_km_h")]


class Peer(C.Structure):
    """srswa_peer: one peer-memory exchange region (device pointers)."""
    _fields_ = [("regions", vp), ("own_region", vp), ("slot_bytes", i64), ("rank", i64), ("world", i64),
                ("counter", vp), ("tickets", vp), ("status", vp), ("ll", i64)]


_SIGS = {
    "srswa_version": (C.c_int, []),
    "srswa_status_string": (C.c_char_p, [C.c_int]),
    "srswa_kbar_contig": (C.c_int, [vp, C.c_int, i64, i64, i64, i64, i64, i64, vp, vp, vp, vp]),
    "srswa_kbar_paged": (C.c_int, [vp, C.c_int, i64, i64, i64, i64, vp, i64, i64, vp, i64, i64, vp, vp,
                                   i64, vp]),
    "srswa_kbar_pages": (C.c_int, [vp, C.c_int, i64, i64, i64, i64, vp, vp, i64, vp, vp, i64, vp]),
    "srswa_route_workspace_size": (C.c_size_t, [i64, i64, i64, RouteParams, C.c_int]),
    "srswa_route": (C.c_int, [vp, C.c_int, i64, i64, i64, vp, i64, i64, i64, vp, i64, vp, i64, vp, vp, vp, i64,
                              RouteParams, vp, vp, vp, vp, vp, vp, C.c_size_t, vp]),
    "srswa_route_select": (C.c_int, [vp, i64, i64, i64, vp, i64, RouteParams, vp, vp, vp, vp, vp]),
    "srswa_route_shard_workspace_size": (C.c_size_t, [i64, i64, RouteParams]),
    "srswa_route_shard_keys": (C.c_int, [vp, C.c_int, i64, i64, i64, vp, i64, i64, i64, i64, i64, vp, i64, vp,
                                         i64, vp, RouteParams, vp, vp, C.c_size_t, vp, vp]),
    "srswa_route_merge_keys": (C.c_int, [vp, i64, i64, i64, i64, i64, RouteParams, vp, vp, vp, vp, i64, i64,
                                         vp, vp, vp]),
    "srswa_route_shard_select": (C.c_int, [vp, C.c_int, i64, i64, i64, vp, i64, i64, i64, i64, i64, vp, i64, vp,
                                           i64, vp, RouteParams, vp, vp, vp, vp, i64, i64, vp, vp, C.c_size_t,
                                           vp, vp]),
    "srswa_block_max_score": (C.c_int, [vp, C.c_int, i64, i64, vp, C.c_int, i64, i64, vp, vp, i64, i64,
                                        i64, i64, i64, i64, i64, C.c_int, vp, vp]),
    "srswa_pack_selection": (C.c_int, [vp, C.c_int, i64, i64, i64, vp, vp]),
    "srswa_gather_fwd_workspace_size": (C.c_size_t, [C.POINTER(GatherDesc)]),
    "srswa_gather_fwd": (C.c_int, [C.POINTER(GatherDesc), vp, vp, vp, vp, vp, vp, vp, C.c_int, i64, i64,
                                   i64, vp, vp, C.c_size_t, vp]),
    "srswa_gather_fwd_paged_workspace_size": (C.c_size_t, [C.POINTER(GatherDesc), i64]),
    "srswa_gather_fwd_paged": (C.c_int, [C.POINTER(GatherDesc), vp, vp, vp, i64, vp, i64, vp, vp, vp, i64, i64,
                                         i64, vp, vp, C.c_size_t, vp]),
    "srswa_gather_bwd_workspace_size": (C.c_size_t, [C.POINTER(GatherDesc)]),
    "srswa_gather_bwd": (C.c_int, [C.POINTER(GatherDesc), vp, vp, vp, vp, i64, i64, i64, vp, vp, vp, vp,
                                   vp, vp, vp, vp, vp, vp, C.c_size_t, vp]),
    "srswa_gather_bwd_noalloc_max_scratch": (C.c_size_t, []),
    "srswa_gather_bwd_noalloc": (C.c_int, [C.POINTER(GatherDesc), vp, vp, vp, vp, i64, i64, i64, vp, vp, vp,
                                           vp, vp, vp, vp, vp, vp, vp]),
    "srswa_decode_attend": (C.c_int, [C.POINTER(DecodeDesc), vp, vp, vp, vp, vp, vp, vp, vp, vp, vp, vp,
                                      vp]),
    "srswa_decode_attend_push": (C.c_int, [C.POINTER(DecodeDesc), vp, vp, vp, vp, vp, vp, vp, vp, vp, vp, vp,
                                           vp, vp]),
    "srswa_decode_attend_exchange": (C.c_int, [C.POINTER(DecodeDesc), vp, vp, vp, vp, vp, vp, vp, vp, vp, vp,
                                               vp, vp, vp, C.c_int, vp, vp]),
    "srswa_prefill_attend": (C.c_int, [C.POINTER(DecodeDesc), vp, vp, vp, vp, vp, vp, vp, vp, vp, vp, vp]),
    "srswa_workspace_status": (C.c_int, [vp, C.POINTER(C.c_int), vp]),
    "srswa_gather_bwd_noalloc_status": (C.c_int, [C.POINTER(C.c_int), vp]),
    "srswa_lse_merge": (C.c_int, [vp, vp, i64, i64, i64, i64, i64, i64, vp, C.c_int, vp, vp, vp]),
    "srswa_page_scan_workspace_size": (C.c_size_t, [i64, i64]),
    "srswa_page_ids": (C.c_int, [vp, i64, i64, i64, i64, i64, i64, i64, C.c_int, vp, vp, vp, vp, vp,
                                 C.c_size_t, vp]),
    "srswa_page_block_desc": (C.c_int, [vp, vp, i64, i64, i64, i64, i64, vp, vp]),
    "srswa_page_cand_mask": (C.c_int, [vp, vp, i64, i64, i64, i64, i64, vp, i64, i64, vp, i64, i64, C.c_int,
                                       C.c_int, vp, vp]),
    "srswa_decode_allow_state": (C.c_int, [vp, i64, i64, i64, i64, i64, i64, i64, vp, vp, vp, vp, vp,
                                           C.c_size_t, vp]),
    "srswa_decode_allow": (C.c_int, [vp, i64, i64, i64, vp, vp, i64, i64, vp, vp, i64, vp, vp]),
    "srswa_win_bounds_decode": (C.c_int, [vp, i64, i64, vp, i64, i64, i64, i64, i64, i64, vp, vp, vp, vp]),
    "srswa_gather_kl_fwd": (C.c_int, [C.POINTER(KlDesc), vp, vp, vp, vp, vp, vp, vp, vp, vp, vp]),
    "srswa_gather_kl_fwd_save": (C.c_int, [C.POINTER(KlDesc), vp, vp, vp, vp, vp, vp, vp, vp, vp, vp, vp]),
    "srswa_gather_kl_bwd_saved": (C.c_int, [C.POINTER(KlDesc), vp, vp, vp, vp, vp, vp, vp, vp, vp, vp,
                                            C.c_size_t, vp]),
    "srswa_gather_kl_bwd_workspace_size": (C.c_size_t, [C.POINTER(KlDesc)]),
    "srswa_gather_kl_bwd": (C.c_int, [C.POINTER(KlDesc), vp, vp, vp, vp, vp, vp, vp, vp, vp, vp, vp, C.c_size_t,
                                      vp]),
    "srswa_peer_region_size": (C.c_int, [i64, i64, C.POINTER(C.c_size_t)]),
    "srswa_peer_region_alloc": (C.c_int, [C.c_size_t, C.POINTER(vp)]),
    "srswa_peer_region_free": (C.c_int, [vp]),
    "srswa_peer_ipc_handle": (C.c_int, [vp, vp]),
    "srswa_peer_ipc_open": (C.c_int, [vp, C.POINTER(vp)]),
    "srswa_peer_ipc_close": (C.c_int, [vp]),
    "srswa_peer_push": (C.c_int, [vp, i64, vp, vp]),
    "srswa_peer_allgather": (C.c_int, [vp, i64, vp, vp]),
    "srswa_rope2d_pos_workspace_size": (C.c_size_t, [i64, i64]),
    "srswa_rope2d_pos": (C.c_int, [vp, i64, i64, i64, i64, i64, i64, i64, vp, vp, vp, i64, vp, vp, C.c_size_t,
                                   vp]),
    "srswa_rope2d_table": (C.c_int, [vp, vp, i64, i64, i64, vp, i64, vp, i64, i64, vp, vp, C.c_int, vp]),
    "srswa_rope2d_apply": (C.c_int, [vp, C.c_int, i64, i64, i64, i64, i64, i64, i64, vp, vp, i64, vp, i64, vp,
                                     i64, i64, C.c_int, vp]),
    "srswa_rope2d_decode": (C.c_int, [vp, i64, i64, i64, vp, vp, vp, i64, i64, vp]),
}

_lib = None


class SrswaError(RuntimeError):
    pass


def lib():
    """Load (once) and return the ctypes handle; raises if the .so is absent."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise SrswaError(
                f"libsrswa.so not found at {LIB_PATH}; build it with "
                f"`python unlimited-ocr_b200/csrc/build.py` (no CPU fallback exists)")
        h = C.CDLL(LIB_PATH)
        for name, (res, args) in _SIGS.items():
            fn = getattr(h, name)
            fn.restype = res
            fn.argtypes = args
        _lib = h
    return _lib


def exported_symbols():
    return list(_SIGS)


def status_text(rc: int) -> str:
    return lib().srswa_status_string(rc).decode()


def check(rc: int, what: str):
    """Map a library status to Python: <0 -> ValueError/NotImplementedError,
    >0 (CUDA error) -> SrswaError."""
    if rc == 0:
        return
    msg = f"{what}: {status_text(rc)} (status {rc})"
    if rc == EUNSUPPORTED or rc == ETOOLARGE:
        raise NotImplementedError(msg)
    if rc < 0:
        raise ValueError(msg)
    raise SrswaError(msg)


def dtype_code(t: torch.Tensor) -> int:
    try:
        return _DTYPES[t.dtype]
    except KeyError:
        raise NotImplementedError(f"dtype {t.dtype} not supported") from None


def ptr(t):
    return None if t is None else t.data_ptr()


# the current stream's raw handle without building a torch Stream object
# (torch.cuda.current_stream costs ~10 us of host time per call)
_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def stream_of(t: torch.Tensor):
    if not t.is_cuda:
        raise SrswaError("srswa kernels need CUDA tensors (no CPU fallback)")
    if _raw_stream is not None:
        return _raw_stream(t.device.index)
    return torch.cuda.current_stream(t.device).cuda_stream
