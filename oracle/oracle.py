"""TEST INFRASTRUCTURE ONLY -- the CPU checker for the decode path.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline/reference legs
import this module.  The product (vllm_fastdecoder_b200) never does.

Contents
  decode_attn / decode_attn_tiered   the C restatement (fd_oracle.c) of the
                                     reference decode_attn
                                     (fastdecode/csrc/cpu_attn.cpp:298-411)
  store_kv                           cpu_attn.cpp:413-431,506-510
  merge2 / merge_parts               fastdecode/cpu_ops.py:93-113
  ref_decode_attn_f64                float64 restatement of
                                     fastdecode/cpu_ops.py:54-81
  load_reference_ext()               the reference's own AVX2 kernel compiled
                                     from its source into oracle/_ref/ (see
                                     Makefile), or None when not built
Tensors are torch CPU tensors (the C code reads their storage directly).
"""

from __future__ import annotations

import ctypes
import importlib
import math
import sys
from ctypes import POINTER, c_float, c_int32, c_int64, c_uint16, c_void_p
from pathlib import Path

import torch

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "libfd_oracle.so"
REF_DIR = HERE / "_ref"

F16, BF16, F32 = 0, 1, 2
_CODE = {torch.float16: F16, torch.bfloat16: BF16, torch.float32: F32}


class _Tier(ctypes.Structure):
    _fields_ = [("k", c_void_p), ("v", c_void_p), ("blk_stride", c_int64), ("head_stride", c_int64),
                ("tok_stride", c_int64), ("num_blocks", c_int64)]


_LIB = None


def lib() -> ctypes.CDLL:
    global _LIB
    if _LIB is None:
        if not LIB_PATH.exists():
            raise RuntimeError(f"oracle library {LIB_PATH} missing: run `make -C oracle oracle`")
        L = ctypes.CDLL(str(LIB_PATH))
        L.fdo_decode_attn.restype = c_int32
        L.fdo_decode_attn.argtypes = [
            c_void_p, c_int64, c_int64, POINTER(_Tier), POINTER(_Tier), c_int64, c_void_p, c_int64,
            c_int32, c_void_p, c_int32, c_int32, c_int32, c_int32, c_int32, c_float, c_int32,
            c_void_p, c_int32, c_int64, c_int64, c_void_p, c_int64, c_int64]
        L.fdo_decode_attn_paged.restype = c_int32
        L.fdo_decode_attn_paged.argtypes = [
            c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int32, c_int32, c_int32, c_int32,
            c_int32, c_int64, c_int32, c_float, c_int32, c_void_p, c_void_p]
        L.fdo_store_kv.restype = c_int32
        L.fdo_store_kv.argtypes = [c_void_p, c_void_p, c_void_p, c_int32, c_int32, c_int32, c_int32,
                                   c_int64, c_int32, c_void_p, c_void_p]
        L.fdo_merge2.restype = None
        L.fdo_merge2.argtypes = [c_void_p, c_void_p, c_void_p, c_void_p, c_int32, c_int32, c_int32,
                                 c_int32, c_void_p, c_void_p]
        L.fdo_merge_parts.restype = None
        L.fdo_merge_parts.argtypes = [c_void_p, c_void_p, c_int64, c_int32, c_int32, c_int32, c_int32,
                                      c_void_p, c_void_p]
        L.fdo_float_to_half.restype = c_uint16
        L.fdo_float_to_half.argtypes = [c_float]
        L.fdo_float_to_bf16.restype = c_uint16
        L.fdo_float_to_bf16.argtypes = [c_float]
        L.fdo_half_to_float.restype = c_float
        L.fdo_half_to_float.argtypes = [c_uint16]
        _LIB = L
    return _LIB


def _cpu(t: torch.Tensor) -> torch.Tensor:
    assert t.device.type == "cpu", "oracle works on CPU tensors"
    return t


def decode_attn(q, k_cache, v_cache, block_table, lens, scale, out, lse) -> None:
    """Reference signature (cpu_attn.cpp:456): contiguous CPU tensors, caches
    [C,KVH,BS,D], cache-relative block ids."""
    for t in (q, k_cache, v_cache, block_table, lens, out, lse):
        _cpu(t)
        assert t.is_contiguous()
    n, H, D = q.shape
    C, KVH, BS, _ = k_cache.shape
    rc = lib().fdo_decode_attn_paged(q.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(),
                                     block_table.data_ptr(), lens.data_ptr(), n, H, KVH, D, BS, C,
                                     block_table.shape[1], float(scale), _CODE[q.dtype],
                                     out.data_ptr(), lse.data_ptr())
    if rc != 0:
        raise RuntimeError(f"oracle decode_attn: error {rc}")


def _tier(k: torch.Tensor | None, v: torch.Tensor | None):
    if k is None:
        return None
    t = _Tier()
    t.k, t.v = k.data_ptr(), v.data_ptr()
    s = k.stride()
    t.blk_stride, t.head_stride, t.tok_stride = s[0], s[1], s[2]
    t.num_blocks = k.shape[0]
    return t


def decode_attn_tiered(q, tier0, tier1, split, block_table, lens, scale, out, lse=None, threads: int = 1) -> None:
    """Two-tier version: tier0/tier1 are (k, v) views [B, KVH, BS, D] (any
    strides, contiguous last dim) or None; ids < split -> tier0, else tier1
    at id - split.  out [n,H,D] of q's dtype or fp32; lse [H,n] or None.
    threads > 1 splits the rows over host threads (each row is computed by
    one call of the same C code, so the result does not depend on it)."""
    n, H, D = q.shape
    t0 = _tier(*tier0) if tier0 is not None else None
    t1 = _tier(*tier1) if tier1 is not None else None
    ref = tier0 if tier0 is not None else tier1
    KVH, BS = ref[0].shape[1], ref[0].shape[2]
    assert block_table.stride(1) == 1 and lens.is_contiguous()
    qe, oe = q.element_size(), out.element_size()

    def run(i0: int, i1: int) -> int:
        return lib().fdo_decode_attn(
            q.data_ptr() + i0 * q.stride(0) * qe, q.stride(0), q.stride(1), ctypes.byref(t0) if t0 else None,
            ctypes.byref(t1) if t1 else None, int(split), block_table.data_ptr() + i0 * block_table.stride(0) * 4,
            block_table.stride(0), block_table.shape[1], lens.data_ptr() + i0 * 4, i1 - i0, H, KVH, D, BS,
            float(scale), _CODE[q.dtype], out.data_ptr() + i0 * out.stride(0) * oe, _CODE[out.dtype], out.stride(0),
            out.stride(1), lse.data_ptr() + i0 * lse.stride(1) * 4 if lse is not None else None,
            lse.stride(0) if lse is not None else 0, lse.stride(1) if lse is not None else 0)

    if threads <= 1 or n <= 1:
        rcs = [run(0, n)]
    else:
        from concurrent.futures import ThreadPoolExecutor

        with ThreadPoolExecutor(max_workers=min(threads, n)) as ex:  # ctypes calls release the GIL
            rcs = list(ex.map(lambda i: run(i, i + 1), range(n)))
    bad = [rc for rc in rcs if rc != 0]
    if bad:
        raise RuntimeError(f"oracle decode_attn_tiered: error {bad[0]}")


def host_threads() -> int:
    """Threads the tests give the oracle (all of this host's cores)."""
    import os

    return os.cpu_count() or 1


def store_kv(k, v, slots, k_cache, v_cache) -> None:
    C, KVH, BS, D = k_cache.shape
    rc = lib().fdo_store_kv(k.data_ptr(), v.data_ptr(), slots.data_ptr(), k.shape[0], KVH, D, BS, C,
                            _CODE[k.dtype], k_cache.data_ptr(), v_cache.data_ptr())
    if rc != 0:
        raise RuntimeError("CPU slot out of range")


def merge2(o_a, lse_a, o_b, lse_b, out_lse: torch.Tensor | None = None) -> torch.Tensor:
    """merge_partials_torch (cpu_ops.py:93-113); returns fp32 [n,H,D]."""
    n, H, D = o_a.shape
    out = torch.empty(n, H, D, dtype=torch.float32)
    assert o_a.dtype == o_b.dtype
    lib().fdo_merge2(o_a.contiguous().data_ptr(), lse_a.contiguous().data_ptr(), o_b.contiguous().data_ptr(),
                     lse_b.contiguous().data_ptr(), _CODE[o_a.dtype], n, H, D, out.data_ptr(),
                     out_lse.data_ptr() if out_lse is not None else None)
    return out


def merge_parts(parts: torch.Tensor, P: int, n: int, H: int, D: int, out_lse=None) -> torch.Tensor:
    """P-way merge of packed fp32 parts [P, n*H*D + H*n]."""
    parts = parts.contiguous()
    stride = n * H * D + H * n
    out = torch.empty(n, H, D, dtype=torch.float32)
    base = parts.data_ptr()
    lib().fdo_merge_parts(base, base + 4 * n * H * D, stride, P, n, H, D, out.data_ptr(),
                          out_lse.data_ptr() if out_lse is not None else None)
    return out


def ref_decode_attn_f64(q, k_cache, v_cache, block_table, lens, scale):
    """float64 restatement of ref_decode_attn (fastdecode/cpu_ops.py:54-81)."""
    n, H, D = q.shape
    _, KVH, BS, _ = k_cache.shape
    G = H // KVH
    out = torch.zeros(n, H, D, dtype=torch.float64)
    lse = torch.full((H, n), float("-inf"), dtype=torch.float64)
    for i in range(n):
        L = int(lens[i])
        if L == 0:
            continue
        nb = (L + BS - 1) // BS
        blks = block_table[i, :nb].long()
        k = k_cache[blks].permute(1, 0, 2, 3).reshape(KVH, nb * BS, D)[:, :L].double()
        v = v_cache[blks].permute(1, 0, 2, 3).reshape(KVH, nb * BS, D)[:, :L].double()
        k = k.repeat_interleave(G, dim=0)
        v = v.repeat_interleave(G, dim=0)
        s = torch.einsum("hd,hld->hl", q[i].double(), k) * scale
        lse[:, i] = torch.logsumexp(s, dim=-1)
        out[i] = torch.einsum("hl,hld->hd", torch.softmax(s, dim=-1), v)
    return out, lse


def _cpu_flags() -> set[str]:
    try:
        for ln in open("/proc/cpuinfo"):
            if ln.startswith("flags"):
                return set(ln.split(":", 1)[1].split())
    except OSError:
        pass
    return set()


def reference_ext_variant() -> str | None:
    """Which compiled reference module load_reference_ext() takes: the
    -march=native build (the reference loader's default, fastdecode/
    cpu_ops.py:32-34) when this host's CPU has every flag of the CPU it was
    built on, else the portable x86-64-v3 build; None when neither exists."""
    native = REF_DIR / "fd_ref_cpu_attn_native.so"
    flags = REF_DIR / "native_flags.txt"
    if native.exists() and flags.exists():
        need = set(flags.read_text().split())
        if need and need <= _cpu_flags():
            return "fd_ref_cpu_attn_native"
    if (REF_DIR / "fd_ref_cpu_attn.so").exists():
        return "fd_ref_cpu_attn"
    return None


def load_reference_ext():
    """The reference's compiled AVX2 module from oracle/_ref, or None."""
    name = reference_ext_variant()
    if name is None:
        return None
    if str(REF_DIR) not in sys.path:
        sys.path.insert(0, str(REF_DIR))
    return importlib.import_module(name)


def rand_case(n, H, KVH, D, BS, C, dtype, max_len, seed):
    """Seeded inputs built the way the reference tests build them
    (tests/test_cpu_kernel.py:14-35): N(0,1) q/K/V, lens ~ U[0,max_len] with
    lens[0] = max_len and lens[1] = 1, distinct random blocks per row."""
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(n, H, D, generator=g).to(dtype)
    k_cache = torch.randn(C, KVH, BS, D, generator=g).to(dtype)
    v_cache = torch.randn(C, KVH, BS, D, generator=g).to(dtype)
    lens = torch.randint(0, max_len + 1, (n,), generator=g, dtype=torch.int32)
    lens[0] = max_len
    if n > 1:
        lens[1] = 1
    W = (max_len + BS - 1) // BS
    perm = torch.randperm(C, generator=g)
    bt = torch.zeros(n, W, dtype=torch.int32)
    pos = 0
    for i in range(n):
        nb = (int(lens[i]) + BS - 1) // BS
        if pos + nb > C:
            perm = torch.randperm(C, generator=g)
            pos = 0
        bt[i, :nb] = perm[pos:pos + nb].to(torch.int32)
        pos += nb
    return q, k_cache, v_cache, bt, lens


def default_scale(D: int) -> float:
    return 1.0 / math.sqrt(D)
