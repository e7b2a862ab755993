"""The C-ABI library loads on a CPU-only host and exports exactly the entry
points include/*.h declares, with the struct sizes the ctypes mirrors assume.
No kernel is launched here."""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest

from vllm_fastdecoder_b200 import _native as nat

ROOT = Path(__file__).resolve().parents[1]


def declared_symbols() -> set[str]:
    names: set[str] = set()
    for h in (ROOT / "include").glob("*.h"):
        text = h.read_text()
        names |= set(re.findall(r"^FD_API\s+[\w\s\*]+?\b(fd_\w+)\s*\(", text, flags=re.M))
    return names


def test_header_declares_entry_points():
    names = declared_symbols()
    for must in ("fd_decode_attn", "fd_decode_attn_paged", "fd_merge_attn_states", "fd_merge_partials",
                 "fd_store_kv", "fd_decode_workspace_size"):
        assert must in names


def test_library_exports_every_declared_symbol():
    lib = nat.load()
    for name in declared_symbols():
        assert hasattr(lib, name), name
    assert set(nat.SIGNATURES) == declared_symbols()


def test_struct_mirrors_match_the_library():
    lib = nat.load()
    a, b = ctypes.c_size_t(), ctypes.c_size_t()
    assert lib.fd_abi_sizes(ctypes.byref(a), ctypes.byref(b)) == 0
    assert a.value == ctypes.sizeof(nat.FdDecodeArgs)
    assert b.value == ctypes.sizeof(nat.FdKvTier)
    assert lib.fd_plan_args_bytes() == ctypes.sizeof(nat.FdPlanArgs)
    assert lib.fd_prefill_args_bytes() == ctypes.sizeof(nat.FdPrefillArgs)


def test_plan_step_host_checks_need_no_gpu():
    """fd_plan_step rejects bad sizes and missing buffers before any launch."""
    lib = nat.load()
    a = nat.FdPlanArgs()
    a.num_reqs, a.bt_width, a.block_size, a.bt_stride = 4, 8, 16, 4  # stride < width
    assert lib.fd_plan_step(ctypes.byref(a), None) == 1
    assert b"bt_stride" in lib.fd_last_error_message()
    a.bt_stride, a.s_gpu_bt_stride, a.s_cpu_bt_stride = 8, 16, 8
    assert lib.fd_plan_step(ctypes.byref(a), None) == 1  # buffers missing
    assert b"null" in lib.fd_last_error_message()


def test_host_side_argument_checks_need_no_gpu():
    """Argument validation runs before any CUDA call."""
    lib = nat.load()
    args = nat.FdDecodeArgs()
    args.n = 0
    assert lib.fd_decode_attn(ctypes.byref(args), None) == 0  # empty batch: nothing to do
    args.n = 4
    args.dtype = 7
    assert lib.fd_decode_attn(ctypes.byref(args), None) == 2  # FD_ERR_UNSUPPORTED
    assert b"dtype" in lib.fd_last_error_message()
    assert lib.fd_merge_attn_states(None, 0, 0, None, None, None, None, None, None, 0, -1, 4, 64, None) == 1
    assert lib.fd_device_error_string(1).startswith(b"block id")
    assert lib.fd_version() >= 100


def test_workspace_size_arithmetic():
    lib = nat.load()
    # persistent schedule (<= 1024 rows): partial slots + row prefix, always
    ws = lib.fd_decode_attn_paged_workspace_size(16, 32, 32, 128, 16, 128, 0)
    assert ws > 0 and ws % 256 == 0
    # the split grid (explicit tiles_per_split): none when every row fits one split
    a = nat.FdDecodeArgs()
    a.n, a.num_heads, a.num_kv_heads, a.head_size, a.block_size = 4, 8, 8, 64, 16
    a.bt_width, a.dtype, a.tiles_per_split = 1, 0, 8
    assert lib.fd_decode_workspace_size(ctypes.byref(a)) == 0
    a.bt_width = 64  # 64 tiles per row, 8 per split -> 8 splits of partials
    assert lib.fd_decode_workspace_size(ctypes.byref(a)) >= 4 * 8 * 8 * 64 * 4


def _valid_args():
    """Arguments that pass every host-side check (fp16, D 128, 8/8 heads,
    block size 16); the pointers are placeholders, never dereferenced by the
    checks these tests reach."""
    a = nat.FdDecodeArgs()
    a.q, a.out, a.block_table, a.lens = 4096, 8192, 12288, 16384
    a.q_stride_n, a.q_stride_h = 8 * 128, 128
    a.n, a.num_heads, a.num_kv_heads, a.head_size, a.block_size = 4, 8, 8, 128, 16
    a.bt_width, a.bt_stride, a.dtype, a.out_dtype = 8, 8, 0, 0
    a.scale = 0.088
    return a


@pytest.mark.parametrize("field,value,code,msg", [
    ("n", -1, 1, b"n must be"),
    ("out_dtype", 1, 2, b"out_dtype"),
    ("q", None, 1, b"required"),
    ("bt_width", 0, 1, b"bt_width"),
    ("n", 70000, 2, b"65535"),
    ("block_size", 24, 2, b"block_size"),
    ("num_heads", 6, 1, b"multiple"),
    ("head_size", 60, 2, b"head_size"),
    ("q", 4104, 3, b"q pointer"),
    ("q_stride_h", 132, 3, b"q pointer"),
])
def test_decode_rejects_bad_arguments_before_any_launch(field, value, code, msg):
    """Each bad argument is reported with its status code and message before
    the library touches the GPU (the checks of fd_decode_attn)."""
    lib = nat.load()
    a = _valid_args()
    setattr(a, field, value)
    assert lib.fd_decode_attn(ctypes.byref(a), None) == code
    assert msg in lib.fd_last_error_message()
