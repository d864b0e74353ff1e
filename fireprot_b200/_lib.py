"""ctypes binding of ``libfireprot_b200.so`` (the only compute path).

Loading never compiles and never falls back: a missing or stale library raises
``ImportError``-style ``RuntimeError`` at first use, and every non-zero status
returned by an entry point raises ``RuntimeError`` (the reference's launch
policy, ``python/fireprot/backends/amd/lt_bmm.py:76-82``).
"""
from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path

_LOCK = threading.Lock()
_LIB = None
LIB_PATH = Path(os.environ.get("FIREPROT_B200_LIBRARY",
                               Path(__file__).resolve().parent / "libfireprot_b200.so"))

c_int, c_size_t, c_void_p, c_float = ctypes.c_int, ctypes.c_size_t, ctypes.c_void_p, ctypes.c_float
c_char_p = ctypes.c_char_p

# capability callback of the registry core: (signature_json, user, reason, cap) -> int
CAPABILITY_FN = ctypes.CFUNCTYPE(c_int, c_char_p, c_void_p, c_void_p, c_size_t)

# name -> (restype, argtypes); must match include/fireprot_b200.h
SIGNATURES = {
    "fpb_abi_version": (c_int, []),
    "fpb_status_string": (ctypes.c_char_p, [c_int]),
    "fpb_device_supported": (c_int, [c_int]),
    "fpb_workspace_status": (c_int, [c_void_p, c_void_p, ctypes.POINTER(c_int)]),
    "fpb_packed_bmm_workspace_size": (c_size_t, [c_int, c_int, c_int]),
    "fpb_packed_bmm": (c_int, [c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int,
                               c_void_p, c_size_t, c_void_p]),
    "fpb_trimul_workspace_size": (c_size_t, [c_int, c_int, c_int]),
    "fpb_trimul": (c_int, [c_void_p, c_void_p, c_int, c_int] + [c_void_p] * 10
                   + [c_float, c_int, c_int, c_int, c_void_p, c_size_t, c_void_p]),
    "fpb_triattn_workspace_size": (c_size_t, [c_int] * 6),
    "fpb_triattn": (c_int, [c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int]
                    + [c_void_p] * 10
                    + [c_float, c_int, c_int, c_void_p, c_size_t, c_void_p]),
    "fpb_transition_workspace_size": (c_size_t, [c_int, c_int, c_int]),
    "fpb_transition": (c_int, [c_void_p, c_void_p, ctypes.c_longlong, c_int, c_int]
                       + [c_void_p] * 5
                       + [c_float, c_int, c_void_p, c_size_t, c_void_p]),
    "fpb_transition_noalloc": (c_int, [c_void_p, c_void_p, ctypes.c_longlong, c_int, c_int]
                               + [c_void_p] * 5
                               + [c_float, c_int, ctypes.POINTER(c_int), c_void_p]),
    "fpb_pair_block_workspace_size": (c_size_t, [c_int, c_int, c_int]),
    "fpb_pair_block": (c_int, [c_void_p, c_void_p, c_int, c_void_p, c_float, c_int, c_void_p,
                               c_size_t, c_void_p]),
    "fpb_single_block_workspace_size": (c_size_t, [c_int, c_int, c_int]),
    "fpb_single_block": (c_int, [c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int,
                                 c_void_p, c_float, c_int, c_void_p, c_size_t, c_void_p]),
    "fpb_triangle_contract_workspace_size": (c_size_t, [c_int, c_int, c_int]),
    "fpb_triangle_contract": (c_int, [c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int,
                                      c_void_p, c_size_t, c_void_p]),
    "fpb_timing_enable": (c_int, [c_int]),
    "fpb_timing_collect": (c_int, [ctypes.c_char_p, c_size_t]),
    "fpb_attention_core_workspace_size": (c_size_t, [c_int] * 6),
    "fpb_attention_core": (c_int, [c_void_p, c_void_p] * 3 + [c_int] * 4
                           + [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_void_p,
                              c_size_t, c_void_p]),
    "fpb_attention_core_ex": (c_int, [c_void_p, c_void_p] * 3 + [c_int] * 4
                              + [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int,
                                 c_void_p, c_size_t, c_void_p]),
    "fpb_trimul_shard_workspace_size": (c_size_t, [c_int]),
    "fpb_trimul_plane_ld": (c_size_t, [c_int, c_int]),
    "fpb_trimul_shard_proj": (c_int, [c_void_p, c_void_p, c_int, c_int, c_int, c_int]
                              + [c_void_p] * 6 + [c_float] + [c_void_p] * 4
                              + [c_int, c_int, c_int, c_void_p, c_size_t, c_void_p]),
    "fpb_trimul_shard_proj_scatter": (c_int, [c_void_p, c_void_p, c_int, c_int, c_int, c_int]
                                      + [c_void_p] * 6 + [c_float] + [c_void_p] * 2
                                      + [c_int, c_int, c_int, c_int, c_int, c_void_p, c_size_t,
                                         c_void_p]),
    "fpb_split_tf32": (c_int, [c_void_p, c_void_p, c_void_p, c_size_t, c_void_p]),
    "fpb_trimul_shard_contract": (c_int, [c_void_p, c_void_p, c_int, c_int, c_void_p, c_void_p,
                                          c_int, c_int, c_int, c_size_t, c_int, c_int, c_void_p,
                                          c_int, c_void_p, c_size_t, c_void_p]),
    "fpb_trimul_group_contract": (c_int, [c_void_p, c_void_p, c_int, c_int, c_void_p, c_void_p,
                                          c_int, c_int, c_int, c_size_t, c_int, c_int, c_int,
                                          c_void_p, c_int, c_void_p, c_size_t, c_void_p]),
    "fpb_trimul_group_contract_scatter": (c_int, [c_void_p, c_void_p, c_int, c_int, c_void_p,
                                                  c_void_p, c_int, c_int, c_int, c_size_t, c_int,
                                                  c_int, c_int, c_void_p, c_int, c_int, c_int,
                                                  c_int, c_void_p, c_size_t, c_void_p]),
    "fpb_trimul_group_gather": (c_int, [c_void_p, c_int, c_int, c_int, c_int, c_int, c_int,
                                        c_void_p, c_void_p, c_int, c_int, c_void_p]),
    "fpb_trimul_shard_finish": (c_int, [c_void_p, c_int, c_int, c_void_p] + [c_void_p] * 6
                                + [c_float, c_int, c_int, c_void_p, c_size_t, c_void_p]),
    "fpb_triattn_bias_ld": (c_size_t, [c_int]),
    "fpb_triattn_shard_workspace_size": (c_size_t, [c_int, c_int, c_int, c_int]),
    "fpb_triattn_shard_proj": (c_int, [c_void_p, c_void_p, c_int, c_int, c_int] + [c_void_p] * 8
                               + [c_float, c_void_p, c_int, c_void_p, c_size_t, c_void_p]),
    "fpb_triattn_shard_finish": (c_int, [c_void_p, c_void_p, c_int, c_int, c_int, c_void_p]
                                 + [c_void_p] * 2 + [c_int, c_void_p, c_size_t, c_void_p]),
    "fpb_ipc_handle_bytes": (c_size_t, []),
    "fpb_ipc_export": (c_int, [c_void_p, c_void_p, ctypes.POINTER(c_size_t)]),
    "fpb_ipc_import": (c_int, [c_void_p, c_size_t, ctypes.POINTER(c_void_p),
                               ctypes.POINTER(c_void_p)]),
    "fpb_ipc_close": (c_int, [c_void_p]),
    "fpb_copy_async": (c_int, [c_void_p, c_void_p, c_size_t, c_void_p]),
    "fpb_peer_scatter": (c_int, [c_void_p, c_void_p, c_void_p, c_int, c_void_p]),
    "fpb_peer_transpose_rows": (c_int, [c_void_p, c_int, c_int, c_int, c_int, c_int, c_void_p,
                                        c_void_p]),
    "fpb_registry_new": (c_void_p, []),
    "fpb_registry_free": (None, [c_void_p]),
    "fpb_registry_register": (c_int, [c_void_p, c_char_p, CAPABILITY_FN, c_void_p]),
    "fpb_registry_unregister": (c_int, [c_void_p, c_char_p, c_char_p]),
    "fpb_registry_resolve": (c_int, [c_void_p, c_char_p, c_char_p, c_size_t]),
    "fpb_registry_manifest": (c_int, [c_void_p, c_char_p, c_size_t]),
    "fpb_registry_clear_runtime_state": (c_int, [c_void_p]),
}

ABI_VERSION = 1


def load():
    """Return the loaded library, binding every declared entry point."""
    global _LIB
    with _LOCK:
        if _LIB is not None:
            return _LIB
        if not LIB_PATH.is_file():
            raise RuntimeError(
                f"fireprot_b200 CUDA library is missing: {LIB_PATH}. "
                "Build it with `python -m fireprot_b200.build`.")
        lib = ctypes.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        if lib.fpb_abi_version() != ABI_VERSION:
            raise RuntimeError(f"unsupported fireprot_b200 ABI {lib.fpb_abi_version()}")
        _LIB = lib
        return lib


def check(status: int, what: str) -> None:
    if status != 0:
        msg = load().fpb_status_string(status).decode()
        raise RuntimeError(f"{what} failed with status {status} ({msg})")
