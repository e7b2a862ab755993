"""ctypes binding of libfastdecode_b200.so (the C ABI in include/fastdecode_b200.h).

Nothing here needs a GPU to import: loading the library and reading its
symbols works on a CPU-only host; the first kernel launch needs a device.
The library must have been built (python -m vllm_fastdecoder_b200.build); a
missing library raises instead of falling back to anything else.
"""

from __future__ import annotations

import ctypes
import threading
from ctypes import POINTER, c_char_p, c_float, c_int32, c_int64, c_size_t, c_void_p
from pathlib import Path

from vllm_fastdecoder_b200.build import library_path

FD_DTYPE_F16 = 0
FD_DTYPE_BF16 = 1
FD_DTYPE_F32 = 2

FD_OK = 0
FD_ERR_WORKSPACE = 4
NOALLOC_SCRATCH_BYTES = 32 << 20  # FD_NOALLOC_SCRATCH_BYTES
STATUS_NAMES = {
    1: "FD_ERR_INVALID", 2: "FD_ERR_UNSUPPORTED", 3: "FD_ERR_ALIGN",
    4: "FD_ERR_WORKSPACE", 5: "FD_ERR_CUDA", 6: "FD_ERR_RANGE",
}


class FdKvTier(ctypes.Structure):
    _fields_ = [
        ("k", c_void_p), ("v", c_void_p),
        ("blk_stride", c_int64), ("head_stride", c_int64), ("tok_stride", c_int64),
        ("num_blocks", c_int64), ("host_mapped", c_int32), ("_pad", c_int32),
    ]


class FdDecodeArgs(ctypes.Structure):
    _fields_ = [
        ("q", c_void_p), ("q_stride_n", c_int64), ("q_stride_h", c_int64), ("q_rows", c_void_p),
        ("tier", FdKvTier * 2), ("tier_split", c_int64),
        ("block_table", c_void_p), ("bt_stride", c_int64), ("bt_width", c_int32),
        ("lens", c_void_p),
        ("n", c_int32), ("num_heads", c_int32), ("num_kv_heads", c_int32),
        ("head_size", c_int32), ("block_size", c_int32), ("scale", c_float), ("dtype", c_int32),
        ("out", c_void_p), ("out_dtype", c_int32), ("_pad0", c_int32),
        ("out_stride_n", c_int64), ("out_stride_h", c_int64), ("out_rows", c_void_p),
        ("lse", c_void_p), ("lse_stride_h", c_int64), ("lse_stride_n", c_int64),
        ("max_len", c_int32), ("tiles_per_split", c_int32),
        ("workspace", c_void_p), ("workspace_bytes", c_size_t), ("error", c_void_p),
        ("bt_rows", c_void_p), ("flags", c_int32), ("_pad1", c_int32),
    ]


FD_DECODE_PDL = 1  # fd_decode_args.flags: programmatic dependent launch


# fd_plan_header slots and fd_plan_flags bits
PLAN_HEADER_LEN = 32
PLAN_FIELDS = {
    "flags": 0, "n_tok": 1, "n_cpu_w": 2, "n_p": 3, "n_p_tok": 4, "p_max_q": 5, "p_max_k": 6, "n_s": 7,
    "s_gpu_width": 8, "s_max_gpu_len": 9, "s_cpu_width": 10, "n_f": 11, "n_f_tok": 12, "f_max": 13,
    "s_max_len": 14, "n_pd": 15, "pd_max_len": 16, "n_pp": 17, "n_pp_tok": 18, "pp_max_q": 19,
    "pp_max_k": 20, "n_decode": 21, "decode_max_len": 22,
}
PLAN_TOUCHES_HOST, PLAN_BAD_BLOCK_ID, PLAN_HOST_EXTEND, PLAN_BAD_OFFSETS = 1, 2, 4, 8


class FdPlanArgs(ctypes.Structure):
    _fields_ = [
        ("query_start_loc", c_void_p), ("seq_lens", c_void_p), ("block_table", c_void_p),
        ("bt_stride", c_int64), ("bt_width", c_int32), ("num_reqs", c_int32),
        ("slot_mapping", c_void_p), ("max_tokens", c_int32), ("block_size", c_int32),
        ("num_gpu_blocks", c_int64), ("num_cpu_blocks", c_int64),
        ("header", c_void_p),
        ("gpu_slot_mapping", c_void_p), ("cpu_w_tok", c_void_p), ("cpu_w_slot", c_void_p),
        ("p_tok", c_void_p), ("p_cu", c_void_p), ("p_seqlens", c_void_p), ("p_req", c_void_p),
        ("s_tok", c_void_p), ("s_gpu_bt", c_void_p), ("s_gpu_bt_stride", c_int64), ("s_gpu_lens", c_void_p),
        ("s_cpu_bt", c_void_p), ("s_cpu_bt_stride", c_int64), ("s_cpu_lens", c_void_p),
        ("f_tok", c_void_p), ("f_cu", c_void_p),
        ("s_req", c_void_p), ("s_seq_lens", c_void_p),
        ("pd_req", c_void_p), ("pd_tok", c_void_p), ("pd_seq_lens", c_void_p),
        ("pp_req", c_void_p), ("pp_tok", c_void_p), ("pp_cu", c_void_p), ("pp_seqlens", c_void_p),
        ("d_tok", c_void_p), ("d_row", c_void_p), ("d_lens", c_void_p),
        ("error", c_void_p),
    ]


MAX_PEERS = 8  # FD_MAX_PEERS
IPC_HANDLE_BYTES = 64  # FD_IPC_HANDLE_BYTES
PEER_RECV_OFFSET = 8192  # FD_PEER_RECV_OFFSET
PEER_MAX_CTAS = 64  # exchange CTAs per launch, at most


class FdPrefillArgs(ctypes.Structure):
    _fields_ = [
        ("q", c_void_p), ("q_stride_t", c_int64), ("q_stride_h", c_int64),
        ("out", c_void_p), ("out_stride_t", c_int64), ("out_stride_h", c_int64),
        ("kv", FdKvTier), ("block_table", c_void_p), ("bt_stride", c_int64), ("bt_width", c_int32),
        ("num_tokens", c_int32), ("q_start", c_void_p), ("q_len", c_void_p), ("k_len", c_void_p),
        ("bt_row", c_void_p), ("n", c_int32), ("num_heads", c_int32), ("num_kv_heads", c_int32),
        ("head_size", c_int32), ("block_size", c_int32), ("scale", c_float), ("dtype", c_int32),
        ("total_q", c_int32), ("error", c_void_p),
    ]


class FdPeerExchange(ctypes.Structure):
    _fields_ = [("base", c_void_p * MAX_PEERS), ("rank", c_int32), ("world", c_int32), ("slot_floats", c_int64)]


# name -> (restype, argtypes); mirrors include/fastdecode_b200.h
SIGNATURES = {
    "fd_decode_workspace_size": (c_size_t, [POINTER(FdDecodeArgs)]),
    "fd_decode_attn": (c_int32, [POINTER(FdDecodeArgs), c_void_p]),
    "fd_decode_attn_partials": (c_int32, [POINTER(FdDecodeArgs), c_void_p]),
    "fd_decode_attn_combine": (c_int32, [POINTER(FdDecodeArgs), c_void_p]),
    "fd_decode_attn_noalloc": (c_int32, [POINTER(FdDecodeArgs), c_void_p]),
    "fd_decode_attn_paged": (c_int32, [
        c_void_p, c_void_p, c_void_p, c_int32, c_void_p, c_void_p, c_int32, c_int32, c_int32,
        c_int32, c_int32, c_int64, c_int32, c_float, c_int32, c_void_p, c_void_p, c_void_p,
        c_size_t, c_void_p, c_void_p]),
    "fd_decode_attn_paged_workspace_size": (c_size_t, [
        c_int32, c_int32, c_int32, c_int32, c_int32, c_int32, c_int32]),
    "fd_merge_attn_states": (c_int32, [
        c_void_p, c_int32, c_int64, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
        c_int32, c_int32, c_int32, c_int32, c_void_p]),
    "fd_merge_partials": (c_int32, [
        c_void_p, c_void_p, c_int64, c_int32, c_int32, c_int32, c_int32, c_void_p, c_int32,
        c_void_p, c_void_p]),
    "fd_store_kv": (c_int32, [
        c_void_p, c_int64, c_int64, c_void_p, c_int64, c_int64, c_void_p, c_int32, c_int32,
        c_int32, c_int32, c_int32, POINTER(FdKvTier), c_int64, c_void_p, c_void_p]),
    "fd_last_error_message": (c_char_p, []),
    "fd_device_error_string": (c_char_p, [c_int32]),
    "fd_read_error": (c_int32, [c_void_p, POINTER(c_int32), c_int32, c_void_p]),
    "fd_host_device_pointer": (c_int32, [c_void_p, POINTER(c_void_p)]),
    "fd_host_register": (c_int32, [c_void_p, c_size_t]),
    "fd_host_unregister": (c_int32, [c_void_p]),
    "fd_plan_step": (c_int32, [POINTER(FdPlanArgs), c_void_p]),
    "fd_peer_buffer_bytes": (c_size_t, [c_int32, c_int64]),
    "fd_peer_alloc": (c_int32, [c_size_t, POINTER(c_void_p), c_void_p]),
    "fd_peer_open": (c_int32, [c_void_p, POINTER(c_void_p)]),
    "fd_peer_close": (c_int32, [c_void_p]),
    "fd_peer_free": (c_int32, [c_void_p]),
    "fd_exchange_merge": (c_int32, [
        POINTER(FdPeerExchange), c_void_p, c_int32, c_int32, c_int32, c_void_p, c_int32, c_void_p, c_int32,
        c_int64, c_void_p, c_void_p]),
    "fd_decode_exchange_merge": (c_int32, [
        POINTER(FdDecodeArgs), POINTER(FdPeerExchange), c_void_p, c_int32, c_void_p, c_int32, c_int64, c_void_p]),
    "fd_exchange_merge_decoded": (c_int32, [
        POINTER(FdDecodeArgs), POINTER(FdPeerExchange), c_void_p, c_int32, c_void_p, c_int32, c_int64, c_void_p]),
    "fd_plan_args_bytes": (c_size_t, []),
    "fd_prefill_attn": (c_int32, [POINTER(FdPrefillArgs), c_void_p]),
    "fd_prefill_args_bytes": (c_size_t, []),
    "fd_version": (c_int32, []),
    "fd_abi_sizes": (c_int32, [POINTER(c_size_t), POINTER(c_size_t)]),
}

_LIB = None
_LOCK = threading.Lock()


def lib_path() -> Path:
    """The library to load: FASTDECODE_B200_LIB if set (e.g. a build with
    other compile-time options), else the in-tree build."""
    import os

    env = os.environ.get("FASTDECODE_B200_LIB")
    return Path(env) if env else library_path()


def load() -> ctypes.CDLL:
    """Load the native library (once) and attach the C signatures."""
    global _LIB
    if _LIB is not None:
        return _LIB
    with _LOCK:
        if _LIB is not None:
            return _LIB
        path = lib_path()
        if not path.exists():
            raise RuntimeError(
                f"fastdecode_b200: native library {path} is missing; build it with "
                "`python -m vllm_fastdecoder_b200.build` (there is no fallback path)"
            )
        lib = ctypes.CDLL(str(path))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _LIB = lib
        return lib


def check(status: int, what: str) -> None:
    """Raise RuntimeError for a nonzero fd_status, with the library's message."""
    if status != FD_OK:
        msg = load().fd_last_error_message()
        text = msg.decode() if msg else ""
        raise RuntimeError(f"{what}: {STATUS_NAMES.get(status, status)}: {text}")


def device_error_string(code: int) -> str:
    return load().fd_device_error_string(int(code)).decode()
