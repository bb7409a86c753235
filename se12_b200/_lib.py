"""ctypes binding of libse12_b200.so (the C ABI declared in include/se12.h).

The shared object is built ahead of time into this package directory
(``se12_b200._build``). Loading fails loudly when it is missing: there is
no CPU fallback anywhere in the product path.
"""

from __future__ import annotations

import ctypes
import pathlib

LIBRARY_PATH = pathlib.Path(__file__).resolve().parent / "libse12_b200.so"

SE12_OK = 0
STATUS_NAMES = {
    0: "SE12_OK",
    1: "SE12_ERR_INVALID_ARGUMENT",
    2: "SE12_ERR_UNSUPPORTED_FORMAT",
    3: "SE12_ERR_MISALIGNED",
    4: "SE12_ERR_WORKSPACE_TOO_SMALL",
    5: "SE12_ERR_CUDA",
    6: "SE12_ERR_UNSUPPORTED_DEVICE",
    7: "SE12_ERR_DEVICE_FAULT",
}

c_int, c_size_t, c_void_p, c_uint, c_char_p = ctypes.c_int, ctypes.c_size_t, ctypes.c_void_p, ctypes.c_uint, ctypes.c_char_p


class Se12StreamsStruct(ctypes.Structure):
    """Mirror of ``se12_streams`` in include/se12.h."""

    _fields_ = [
        ("rows", ctypes.c_int32),
        ("cols", ctypes.c_int32),
        ("tile_rows", ctypes.c_int32),
        ("tile_cols", ctypes.c_int32),
        ("escape_budget", ctypes.c_int32),
        ("format_version", ctypes.c_int32),
        ("codebook", ctypes.c_uint8 * 15),
        ("sm", c_void_p),
        ("ec", c_void_p),
        ("esc", c_void_p),
        ("fallback_bitmap", c_void_p),
        ("fallback_raw", c_void_p),
        ("escape_pos", c_void_p),
        ("fallback_index", c_void_p),
    ]


class Se12LaunchConfigStruct(ctypes.Structure):
    """Mirror of ``se12_launch_config`` in include/se12.h."""

    _fields_ = [(name, ctypes.c_int32) for name in
                ("grid", "threads", "smem_bytes", "ctas_per_sm", "stage_tiles", "stages", "x_resident", "row_mode", "wide")]


class Se12PeerGroupStruct(ctypes.Structure):
    """Mirror of ``se12_peer_group`` in include/se12.h (SE12_MAX_PEERS = 8)."""

    _fields_ = [("world", ctypes.c_int32), ("rank", ctypes.c_int32), ("rows_cap", ctypes.c_int32),
                ("recv", c_void_p * 8), ("epoch", c_void_p)]


# name -> (restype, argtypes)
SIGNATURES = {
    "se12_escape_pos_bytes": (c_size_t, [c_int, c_int]),
    "se12_fallback_index_bytes": (c_size_t, [c_int, c_int]),
    "se12_matrix_create": (c_int, [ctypes.POINTER(Se12StreamsStruct), ctypes.POINTER(c_void_p)]),
    "se12_matrix_create_segmented": (c_int, [ctypes.POINTER(Se12StreamsStruct), c_int, ctypes.POINTER(ctypes.c_int32),
                                             ctypes.POINTER(ctypes.c_uint8), ctypes.POINTER(c_void_p)]),
    "se12_matrix_prepare": (c_int, [c_void_p, c_void_p]),
    "se12_matrix_destroy": (None, [c_void_p]),
    "se12_gemv_workspace_bytes": (c_size_t, [c_void_p, c_int]),
    "se12_workspace_clear": (c_int, [c_void_p, c_size_t, c_void_p]),
    "se12_gemv_launch_config": (c_int, [c_void_p, c_int, ctypes.POINTER(Se12LaunchConfigStruct)]),
    "se12_gemv_plan": (c_int, [c_int, c_int, c_int, c_int, ctypes.POINTER(Se12LaunchConfigStruct)]),
    "se12_gemv": (c_int, [c_void_p, c_void_p, c_int, c_int, c_void_p, c_int, c_void_p, c_size_t, c_void_p]),
    "se12_gemv_noalloc": (c_int, [c_void_p, c_void_p, c_int, c_int, c_void_p, c_int, c_void_p]),
    "se12_ipc_handle": (c_int, [c_void_p, ctypes.POINTER(ctypes.c_uint8), ctypes.POINTER(ctypes.c_uint64)]),
    "se12_ipc_open": (c_int, [ctypes.POINTER(ctypes.c_uint8), ctypes.c_uint64, ctypes.POINTER(c_void_p), ctypes.POINTER(c_void_p)]),
    "se12_ipc_close": (c_int, [c_void_p]),
    "se12_peer_recv_bytes": (c_size_t, [c_int, c_int]),
    "se12_gemv_allreduce": (c_int, [c_void_p, c_void_p, c_int, c_int, c_void_p, c_int, c_void_p, c_size_t,
                                    ctypes.POINTER(Se12PeerGroupStruct), c_void_p]),
    "se12_gemv_allgather": (c_int, [c_void_p, c_void_p, c_int, c_int, c_void_p, c_int, c_int, c_int, c_void_p, c_size_t,
                                    ctypes.POINTER(Se12PeerGroupStruct), c_void_p]),
    "se12_decode": (c_int, [c_void_p, c_void_p, c_int, c_void_p]),
    "se12_decode_rows": (c_int, [c_void_p, c_void_p, c_int, c_void_p, c_int, c_void_p]),
    "bf16_gemv_workspace_bytes": (c_size_t, [c_int, c_int, c_int]),
    "bf16_gemv": (c_int, [c_void_p, c_int, c_int, c_int, c_void_p, c_int, c_int, c_void_p, c_int, c_void_p, c_size_t, c_void_p]),
    "se12_encode_histogram": (c_int, [c_void_p, c_int, c_int, c_int, c_void_p, c_void_p]),
    "se12_codebook_from_counts": (c_int, [c_void_p, c_void_p]),
    "se12_encode_tiles": (c_int, [c_void_p, c_int, c_int, c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p]),
    "se12_encode_bitmap": (c_int, [c_void_p, c_int, c_void_p, c_void_p, c_void_p, c_void_p]),
    "se12_encode_raw": (c_int, [c_void_p, c_int, c_int, c_int, c_void_p, c_void_p, c_void_p]),
    "se12_tile_records_bytes": (c_size_t, [c_int, c_int]),
    "se12_matrix_prepare_records": (c_int, [c_void_p, c_void_p, c_void_p]),
    "se12_chain_create": (c_int, [c_int, c_int, ctypes.POINTER(c_void_p)]),
    "se12_chain_add_gemv": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_void_p, c_int]),
    "se12_chain_add_gemv_allreduce": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_void_p, c_int,
                                              ctypes.POINTER(Se12PeerGroupStruct)]),
    "se12_chain_add_dense": (c_int, [c_void_p, c_void_p, c_int, c_int, c_int, c_void_p, c_int, c_void_p, c_int]),
    "se12_chain_ops": (c_int, [c_void_p]),
    "se12_chain_descriptor_bytes": (c_size_t, [c_void_p]),
    "se12_chain_workspace_bytes": (c_size_t, [c_void_p]),
    "se12_chain_upload": (c_int, [c_void_p, c_void_p, c_void_p, c_size_t, c_void_p]),
    "se12_chain_run": (c_int, [c_void_p, c_void_p]),
    "se12_chain_reset": (c_int, [c_void_p, c_void_p]),
    "se12_chain_info": (c_int, [c_void_p, ctypes.POINTER(c_int), ctypes.POINTER(c_int), ctypes.POINTER(c_int),
                                ctypes.POINTER(c_int)]),
    "se12_chain_destroy": (None, [c_void_p]),
    "bf16_gemv_plan": (c_int, [c_int, c_int, c_int, c_int, ctypes.POINTER(Se12LaunchConfigStruct)]),
    "se12_gemv_order_matched": (c_int, [c_void_p, c_void_p, c_int, c_int, c_void_p, c_int, c_void_p, c_size_t, c_void_p]),
    "se12_device_status": (c_int, [ctypes.POINTER(c_uint), c_int]),
    "se12_set_wait_limit_ns": (c_int, [ctypes.c_ulonglong]),
    "se12_wait_limit_ns": (c_int, [ctypes.POINTER(ctypes.c_ulonglong)]),
    "se12_status_string": (c_char_p, [c_int]),
    "se12_last_error": (c_char_p, []),
    "se12_abi_version": (c_int, []),
}


class Se12Error(RuntimeError):
    """A libse12_b200 call returned a non-zero status."""

    def __init__(self, status: int, function: str, detail: str):
        self.status = status
        self.function = function
        super().__init__(f"{function}: {STATUS_NAMES.get(status, status)}: {detail}")


_LIB = None


def load() -> ctypes.CDLL:
    """The loaded library. Raises if the AOT build is missing."""
    global _LIB
    if _LIB is not None:
        return _LIB
    if not LIBRARY_PATH.exists():
        raise RuntimeError(
            f"{LIBRARY_PATH} is missing: build it with `python -m se12_b200._build` "
            "(nvcc, sm_100a). The SE12 path has no CPU fallback."
        )
    lib = ctypes.CDLL(str(LIBRARY_PATH))
    for name, (restype, argtypes) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = restype
        fn.argtypes = argtypes
    _LIB = lib
    return lib


def is_loaded() -> bool:
    """Whether this process has loaded the library already."""
    return _LIB is not None


def check(status: int, function: str) -> None:
    if status != SE12_OK:
        detail = load().se12_last_error().decode(errors="replace")
        raise Se12Error(status, function, detail)


def call(name: str, *args):
    """Calls an int-returning entry point and raises Se12Error on failure."""
    status = getattr(load(), name)(*args)
    check(status, name)
    return status
