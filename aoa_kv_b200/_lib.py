"""ctypes binding of libaoakv.so (the C ABI declared in include/aoakv.h).

The library is built in-tree (``python -m aoa_kv_b200.build``) and loaded from
``aoa_kv_b200/libaoakv.so``. There is no fallback: if the library is missing
or fails to load, every operator raises.
"""
from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libaoakv.so"

OK = 0
ERR_NAMES = {1: "INVALID_ARG", 2: "UNSUPPORTED", 3: "CUDA", 4: "WORKSPACE"}
DEV_ERR_NAMES = {0: "OK", 1: "BAD_PAGE", 2: "TIMEOUT", 3: "NO_PAGES"}
DTYPE_F16, DTYPE_F32 = 0, 1
LAYOUT_NHD, LAYOUT_HND = 0, 1
SCORE_QUEST, SCORE_AOAKV = 0, 1

_c_i32, _c_i64, _c_p, _c_f = ctypes.c_int32, ctypes.c_int64, ctypes.c_void_p, ctypes.c_float
_c_size = ctypes.c_size_t
_c_ip = ctypes.POINTER(ctypes.c_int32)
_c_sizep = ctypes.POINTER(ctypes.c_size_t)
_c_pp = ctypes.POINTER(ctypes.c_void_p)
PLAN_CHAIN = 1
PLAN_SHARD = 2

# name -> argtypes (restype is int unless listed in _RESTYPE)
SIGNATURES = {
    "aoakv_last_error": [],
    "aoakv_version": [],
    "aoakv_get_device_error": [_c_ip, _c_i32],
    "aoakv_debug_wait_flag": [_c_p, _c_i32, _c_i32, _c_p],
    "aoakv_apply_rope_in_place": [_c_p, _c_p, _c_i32, _c_i32, _c_i32, _c_i32, _c_f, _c_f, _c_p],
    "aoakv_rms_norm": [_c_p, _c_p, _c_p, _c_i32, _c_i32, _c_f, _c_p],
    "aoakv_append_kv_cache_decode": [_c_p, _c_p, _c_p, _c_p, _c_i32, _c_i32, _c_i32, _c_p, _c_p,
                                     _c_i32, _c_i32, _c_i32, _c_p, _c_i32, _c_i32, _c_i32, _c_i32, _c_p],
    "aoakv_append_kv_cache_prefill": [_c_p, _c_p, _c_i32, _c_p, _c_p, _c_i32, _c_i32, _c_i32, _c_p,
                                      _c_p, _c_i32, _c_i32, _c_i32, _c_p, _c_i32, _c_i32, _c_i32,
                                      _c_i32, _c_p],
    "aoakv_estimate_attn_score": [_c_p, _c_p, _c_i32, _c_i64, _c_p, _c_p, _c_i32, _c_i32, _c_i32,
                                  _c_p, _c_i32, _c_p, _c_i32, _c_i32, _c_i32, _c_i32, _c_i32, _c_p],
    "aoakv_topk_filtering": [_c_p, _c_i32, _c_i64, _c_p, _c_i64, _c_i32, _c_i32, _c_i32, _c_p,
                             _c_i64, _c_p, _c_i64, _c_i32, _c_p],
    "aoakv_decode_workspace_size": [_c_i32, _c_i32, _c_i32, _c_sizep],
    "aoakv_sparse_decode": [_c_p, _c_p, _c_p, _c_i32, _c_p, _c_i64, _c_i32, _c_i32, _c_i32, _c_i32,
                            _c_i32, _c_i32, _c_i32, _c_f, _c_p, _c_size, _c_p],
    "aoakv_sparse_decode_noalloc": [_c_p, _c_p, _c_p, _c_i32, _c_p, _c_i64, _c_i32, _c_i32, _c_i32,
                                    _c_i32, _c_i32, _c_i32, _c_i32, _c_f, _c_p],
    "aoakv_sparse_decode_partial": [_c_p, _c_p, _c_p, _c_p, _c_i32, _c_p, _c_i64, _c_i32, _c_i32,
                                    _c_i32, _c_i32, _c_i32, _c_i32, _c_i32, _c_f, _c_p, _c_size,
                                    _c_p],
    "aoakv_merge_states": [_c_p, _c_p, _c_i32, _c_i32, _c_i32, _c_p, _c_p, _c_p],
    "aoakv_map_pages": [_c_p, _c_i64, _c_i32, _c_i32, _c_p, _c_p, _c_p],
    "aoakv_step_workspace_size": [_c_i32, _c_i32, _c_i32, _c_i32, _c_sizep],
    "aoakv_step_launches": [_c_i32, _c_i32, _c_i32, _c_i32, _c_i32, _c_i32, _c_i32, _c_ip],
    "aoakv_decode_step": [_c_p, _c_p, _c_p, _c_p, _c_p, _c_p, _c_i32, _c_i32, _c_i32, _c_p, _c_p,
                          _c_i32, _c_p, _c_i32, _c_i32, _c_i32, _c_i32, _c_i32, _c_i32, _c_p, _c_p,
                          _c_size, _c_p],
    "aoakv_step_plan_create": [_c_pp, _c_p, _c_i32, _c_p, _c_i32, _c_p, _c_i32, _c_i32, _c_i32,
                               _c_i32, _c_i32, _c_i32, _c_i32, _c_i32, _c_i32],
    "aoakv_step_plan_run": [_c_p, _c_p, _c_p, _c_p, _c_p, _c_p, _c_i32, _c_i32, _c_p, _c_p, _c_p,
                            _c_size, _c_p],
    "aoakv_step_plan_info": [_c_p, _c_i32, _c_i32, _c_ip, _c_ip],
    "aoakv_step_plan_destroy": [_c_p],
    "aoakv_step_plan_set_rope": [_c_p, _c_f, _c_f],
    "aoakv_decode_step_batched": [_c_p, _c_p, _c_p, _c_p, _c_p, _c_i32, _c_p, _c_p, _c_p, _c_p,
                                  _c_i32, _c_p, _c_p, _c_p, _c_i32, _c_i32, _c_i32, _c_i32, _c_i32,
                                  _c_i32, _c_i32, _c_i32, _c_p, _c_p],
    "aoakv_page_table_bytes": [_c_i32, _c_i32, _c_i32, _c_i32, _c_i32, _c_sizep],
    "aoakv_page_table_create": [_c_pp, _c_i32, _c_i32, _c_i32, _c_i32, _c_i32, _c_p, _c_size,
                                _c_p],
    "aoakv_page_table_destroy": [_c_p],
    "aoakv_page_table_append": [_c_p, _c_i32, _c_i32, _c_p],
    "aoakv_page_table_release": [_c_p, _c_i32, _c_p],
    "aoakv_page_table_layout": [_c_p, ctypes.POINTER(ctypes.c_int64)],
    "aoakv_decode_step_table": [_c_p, _c_p, _c_p, _c_p, _c_p, _c_p, _c_i32, _c_p, _c_i32, _c_p,
                                _c_i32, _c_i32, _c_i32, _c_i32, _c_i32, _c_p, _c_f, _c_f, _c_p],
    "aoakv_shard_propose": [_c_p, _c_p, _c_p, _c_i32, _c_i32, _c_i32, _c_p, _c_p, _c_p],
    "aoakv_shard_finish": [_c_p, _c_p, _c_p, _c_p, _c_p, _c_i32, _c_i32, _c_i32, _c_i32, _c_p,
                           _c_p, _c_i32, _c_i32, _c_p, _c_p, _c_p],
    "aoakv_merge_packed_states": [_c_p, _c_i32, _c_i32, _c_i32, _c_p, _c_p],
    "aoakv_shard_mailbox_create": [_c_pp, _c_i32, _c_i32, _c_i32, _c_i32, _c_i32, _c_p],
    "aoakv_shard_mailbox_connect": [_c_p, _c_p],
    "aoakv_shard_mailbox_destroy": [_c_p],
    "aoakv_shard_propose_p2p": [_c_p, _c_p, _c_p, _c_p, _c_i32, _c_i32, _c_i32, _c_p, _c_p],
    "aoakv_shard_finish_p2p": [_c_p, _c_p, _c_p, _c_p, _c_p, _c_p, _c_i32, _c_i32, _c_i32,
                               _c_i32, _c_p, _c_p, _c_p],
    "aoakv_shard_merge_p2p": [_c_p, _c_i32, _c_p, _c_p],
    "aoakv_prefill_paged": [_c_p, _c_p, _c_p, _c_p, _c_i32, _c_p, _c_i32, _c_i32, _c_i32, _c_i32,
                            _c_i32, _c_i32, _c_i32, _c_i32, _c_i32, _c_f, _c_p],
    "aoakv_decode_step_gqa": [_c_p, _c_p, _c_p, _c_p, _c_p, _c_p, _c_i32, _c_i32, _c_i32, _c_p,
                              _c_p, _c_i32, _c_p, _c_i32, _c_i32, _c_i32, _c_i32, _c_i32,
                              _c_i32, _c_i32, _c_p, _c_p, _c_size, _c_p],
    "aoakv_decode_step_grid": [_c_p, _c_p, _c_p, _c_p, _c_p, _c_p, _c_i32, _c_i32, _c_i32, _c_p,
                               _c_p, _c_i32, _c_p, _c_i32, _c_i32, _c_i32, _c_i32, _c_i32,
                               _c_i32, _c_p, _c_p, _c_size, _c_i32, _c_p],
}
_RESTYPE = {"aoakv_last_error": ctypes.c_char_p}

_lock = threading.Lock()
_lib = None


class AoaKvError(RuntimeError):
    """A libaoakv entry point returned a non-OK status."""


def load() -> ctypes.CDLL:
    """Loads libaoakv.so once and declares every ABI signature."""
    global _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise AoaKvError(
                    f"{LIB_PATH} is missing; build it with `python -m aoa_kv_b200.build` "
                    "(there is no CPU fallback)")
            lib = ctypes.CDLL(str(LIB_PATH), mode=os.RTLD_NOW | os.RTLD_LOCAL)
            for name, argtypes in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.argtypes = argtypes
                fn.restype = _RESTYPE.get(name, ctypes.c_int)
            _lib = lib
    return _lib


def call(name: str, *args) -> None:
    """Calls entry point `name`; raises AoaKvError with the library's message."""
    lib = load()
    rc = getattr(lib, name)(*args)
    if rc != OK:
        msg = lib.aoakv_last_error().decode(errors="replace")
        raise AoaKvError(f"{name} failed ({ERR_NAMES.get(rc, rc)}): {msg}")


def size_query(name: str, *args) -> int:
    out = ctypes.c_size_t(0)
    call(name, *args, ctypes.byref(out))
    return int(out.value)


def device_error(clear: bool = True) -> int:
    """Device-side error word of the current device (synchronises it)."""
    code = ctypes.c_int32(0)
    call("aoakv_get_device_error", ctypes.byref(code), 1 if clear else 0)
    return int(code.value)


def check_device(clear: bool = True) -> None:
    code = device_error(clear)
    if code:
        raise AoaKvError(f"device-side error {DEV_ERR_NAMES.get(code, code)}")
