"""Torch-level front end of the sm_100a kernels (the C ABI in include/).

Mirrors the reference operator interface of fastdecode/cpu_ops.py and
fastdecode/csrc/cpu_attn.cpp:
  load_ext()                          -> object with decode_attn / store_kv /
                                         set_num_threads / get_num_threads /
                                         has_avx2, like cpu_ops.load_ext
                                         (cpu_ops.py:21-46)
  decode_attn(q, k_cache, v_cache, block_table, lens, scale, out, lse)
                                      (cpu_attn.cpp:456-489), same argument
                                      meaning and the same RuntimeError
                                      checks (:460-477), on device tensors or
                                      on pinned host caches read over PCIe
  store_kv(k, v, slots, k_cache, v_cache)
                                      (cpu_attn.cpp:492-517), range error ->
                                      RuntimeError (:506-510)
  merge_attn_states(out, o_a, lse_a, o_b, lse_b)
                                      vLLM's op as called at backend.py:54-55
plus the two-tier entry points the backend uses (decode_tiered, store_kv_tiered,
merge_partials).  Every call is asynchronous on the current CUDA stream.
There is no CPU path: without the native library or a CUDA device these raise.
"""

from __future__ import annotations

import ctypes
import math
import os
from dataclasses import dataclass

import torch

from vllm_fastdecoder_b200 import _native as nat

_DTYPE = {torch.float16: nat.FD_DTYPE_F16, torch.bfloat16: nat.FD_DTYPE_BF16, torch.float32: nat.FD_DTYPE_F32}


def dtype_code(dt: torch.dtype) -> int:
    try:
        return _DTYPE[dt]
    except KeyError:
        raise RuntimeError(f"unsupported dtype {dt}") from None


def _check(cond: bool, msg: str) -> None:
    if not cond:
        raise RuntimeError(msg)


def _stream(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


# ------------------------------------------------------------- per-device state

_WS: dict[int, torch.Tensor] = {}
_ERR: dict[int, torch.Tensor] = {}
_HOST_PTR: dict[int, int] = {}


def workspace(device: torch.device, nbytes: int) -> torch.Tensor:
    """Grow-only scratch buffer (256-byte aligned) for split partials."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    buf = _WS.get(idx)
    if buf is None or buf.numel() < nbytes:
        cap = max(nbytes, 1 << 20, 2 * (buf.numel() if buf is not None else 0))
        buf = torch.empty(cap, dtype=torch.uint8, device=torch.device("cuda", idx))
        _WS[idx] = buf
    return buf


def error_word(device: torch.device) -> torch.Tensor:
    """The int32 device error word the kernels on `device` report into."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    w = _ERR.get(idx)
    if w is None:
        w = torch.zeros(1, dtype=torch.int32, device=torch.device("cuda", idx))
        _ERR[idx] = w
    return w


def check_device_errors(device: torch.device | None = None) -> None:
    """Synchronise and raise RuntimeError if a kernel on `device` flagged an
    error since the last check (the word is cleared)."""
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else device
    w = error_word(dev)
    val = ctypes.c_int32(0)
    nat.check(nat.load().fd_read_error(w.data_ptr(), ctypes.byref(val), 1, _stream(dev)), "fd_read_error")
    if val.value != 0:
        raise RuntimeError(f"fastdecode_b200 device error {val.value}: {nat.device_error_string(val.value)}")


def host_device_pointer(t: torch.Tensor) -> int:
    """Device address of t.data_ptr() for a pinned, mapped host tensor (the
    storage base is translated once and cached; views keep their offset)."""
    _check(t.device.type == "cpu", "expected a host tensor")
    _check(t.is_pinned(), "host KV tier must be pinned (pin_memory=True) to be read by the GPU")
    base = t.untyped_storage().data_ptr()
    if base not in _HOST_PTR:
        out = ctypes.c_void_p()
        nat.check(nat.load().fd_host_device_pointer(base, ctypes.byref(out)), "fd_host_device_pointer")
        _HOST_PTR[base] = out.value or 0
    return _HOST_PTR[base] + (t.data_ptr() - base)


def forget_host_pointer(t: torch.Tensor) -> None:
    """Drop the cached device address of t's storage (its memory is about to
    be unregistered)."""
    _HOST_PTR.pop(t.untyped_storage().data_ptr(), None)


# ------------------------------------------------------------- KV tiers


@dataclass
class KVTier:
    """One KV tier viewed as K/V tensors of logical shape [B, KVH, BS, D]
    (any strides with a contiguous last dim).  Device tensors are streamed
    with TMA; pinned host tensors are read over PCIe through their mapped
    device address."""

    k: torch.Tensor
    v: torch.Tensor

    def __post_init__(self) -> None:
        _check(self.k.dim() == 4 and self.v.dim() == 4, "KV tier views must be 4-D [B, KVH, BS, D]")
        _check(self.k.shape == self.v.shape, "K and V views must have the same shape")
        _check(self.k.stride() == self.v.stride(), "K and V views must have the same strides")
        _check(self.k.stride(3) == 1, "head_size must be the contiguous dimension")
        _check(self.k.dtype == self.v.dtype, "K and V dtypes differ")

    @property
    def host(self) -> bool:
        return self.k.device.type == "cpu"

    def to_c(self) -> nat.FdKvTier:
        t = nat.FdKvTier()
        if self.host:
            t.k = host_device_pointer(self.k)
            t.v = host_device_pointer(self.v)
        else:
            t.k = self.k.data_ptr()
            t.v = self.v.data_ptr()
        s = self.k.stride()
        t.blk_stride, t.head_stride, t.tok_stride = s[0], s[1], s[2]
        t.num_blocks = self.k.shape[0]
        t.host_mapped = 1 if self.host else 0
        return t


def _empty_tier() -> nat.FdKvTier:
    return nat.FdKvTier()


def _tier_device(t: KVTier | None) -> torch.device | None:
    if t is None or t.host:
        return None
    return t.k.device


# ------------------------------------------------------------- host-tier staging

_STAGE: dict[int, torch.Tensor] = {}


def stage_host_blocks(tier: KVTier, lo: int, hi: int, device: torch.device) -> KVTier:
    """Copy host-tier blocks [lo, hi) into device memory with the copy engine
    (two cudaMemcpyAsync on the current stream: K, then V) and return the
    device tier over the copy.  The copy engine reads pinned memory faster
    than SM loads over PCIe (B200: 55.6 vs ~51 GB/s), so a step that reads
    most of a compact range of host blocks gains by staging it; decode with
    tier_split + lo as the split so that host id h maps to staged block
    h - lo.  The staging buffer is shared and grow-only (per device): it
    is overwritten by the next staging call on the same device."""
    _check(tier.host, "stage_host_blocks: the tier must be the pinned host tier")
    _check(0 <= lo <= hi <= tier.k.shape[0], f"stage_host_blocks: range [{lo}, {hi}) outside the tier")
    _check(tier.k.is_contiguous() and tier.v.is_contiguous(), "stage_host_blocks: host tier must be contiguous")
    idx = device.index if device.index is not None else torch.cuda.current_device()
    per = tier.k[0].numel()
    need = 2 * max(1, hi - lo) * per
    buf = _STAGE.get(idx)
    if buf is None or buf.numel() < need or buf.dtype != tier.k.dtype:
        buf = torch.empty(need, dtype=tier.k.dtype, device=torch.device("cuda", idx))
        _STAGE[idx] = buf
    shape = (max(1, hi - lo),) + tuple(tier.k.shape[1:])
    k = buf[: need // 2].view(shape)
    v = buf[need // 2: need].view(shape)
    if hi > lo:
        k[: hi - lo].copy_(tier.k[lo:hi], non_blocking=True)
        v[: hi - lo].copy_(tier.v[lo:hi], non_blocking=True)
    return KVTier(k[: max(1, hi - lo)], v[: max(1, hi - lo)])


def host_block_range(block_table: torch.Tensor, lens: torch.Tensor, block_size: int, tier_split: int) -> tuple[int, int]:
    """[lo, hi) of the host-tier blocks (ids >= tier_split, host-relative)
    a step reads, from CPU copies of its block table and lengths."""
    W = block_table.shape[1]
    nb = ((lens.to(torch.int64) + block_size - 1) // block_size).clamp(max=W)
    used = torch.arange(W).unsqueeze(0) < nb.unsqueeze(1)
    ids = block_table.to(torch.int64)[used]
    ids = ids[ids >= tier_split]
    if ids.numel() == 0:
        return 0, 0
    return int(ids.min()) - tier_split, int(ids.max()) - tier_split + 1


@dataclass
class ChunkedStaging:
    """One step's host-tier blocks cut into chunks that are staged into HBM
    one after another on a side stream (plan_chunked_staging).  Part 0 is
    every row's HBM-tier blocks; part j (1..k) is every row's host blocks
    with host-relative ids in chunks[j - 1] = [c_lo, c_hi).  Per part,
    `tables[p]` (int32 [n, W_p], CPU) lists a row's blocks of that part in
    table order, the row's last (partly filled) block moved to the end, with
    ids as the part's decode reads them (HBM ids for part 0, ids relative to
    the staged range [lo, hi) for the others), and `lens[p]` (int32 [n]) is
    the tokens they hold (0: the row has no block in the part)."""

    lo: int
    hi: int
    chunks: list[tuple[int, int]]
    tables: list[torch.Tensor]
    lens: list[torch.Tensor]
    _dev: dict | None = None

    def on(self, device: torch.device) -> list[tuple[torch.Tensor, torch.Tensor]]:
        """(table, lens) of every part on `device`, copied once (one packed
        host-to-device copy) and cached, so that a step captured in a CUDA
        graph copies nothing."""
        key = str(device)
        if self._dev is None:
            self._dev = {}
        if key not in self._dev:
            flat = torch.cat([t.flatten() for t in self.tables] + list(self.lens)).to(device)
            out, o = [], 0
            for t in self.tables:
                out.append(flat[o:o + t.numel()].view(t.shape))
                o += t.numel()
            lens = []
            for ln in self.lens:
                lens.append(flat[o:o + ln.numel()])
                o += ln.numel()
            self._dev[key] = list(zip(out, lens))
        return self._dev[key]


def plan_chunked_staging(block_table: torch.Tensor, lens: torch.Tensor, block_size: int, tier_split: int,
                         chunks: int) -> ChunkedStaging:
    """Cut a step's host-tier range [lo, hi) into `chunks` equal block ranges
    and build the per-part block tables of ChunkedStaging from CPU copies of
    the step's block table and lengths (blocks may lie anywhere in the range:
    each part holds whichever of a row's blocks fall into it)."""
    _check(chunks >= 1, "plan_chunked_staging: chunks must be >= 1")
    n, W = block_table.shape
    BS = block_size
    L = lens.to(torch.int64).clamp(min=0)
    nb = ((L + BS - 1) // BS).clamp(max=W)
    col = torch.arange(W).unsqueeze(0).expand(n, W)
    used = col < nb.unsqueeze(1)
    ids = block_table.to(torch.int64)
    host = used & (ids >= tier_split)
    rel = ids - tier_split
    if bool(host.any()):
        lo, hi = int(rel[host].min()), int(rel[host].max()) + 1
    else:
        lo = hi = 0
    k = max(1, min(chunks, hi - lo)) if hi > lo else 0
    bounds = [lo + ((hi - lo) * j) // k for j in range(k + 1)] if k else []
    spans = [(bounds[j], bounds[j + 1]) for j in range(k)]
    last = col == (nb - 1).unsqueeze(1)  # the row's last block (L - (nb-1)*BS tokens)
    tail = (L - (nb - 1).clamp(min=0) * BS).unsqueeze(1).expand(n, W)
    tok = torch.where(last, tail, torch.full_like(tail, BS))
    masks = [used & (ids < tier_split)] + [host & (rel >= c_lo) & (rel < c_hi) for c_lo, c_hi in spans]
    tables, part_lens = [], []
    for p, m in enumerate(masks):
        key = torch.where(m, torch.where(last, torch.full_like(col, W), col), torch.full_like(col, 2 * W))
        order = key.argsort(dim=1, stable=True)
        cnt = m.sum(dim=1)
        wp = max(1, int(cnt.max()) if n else 1)
        vals = (ids if p == 0 else rel - lo).gather(1, order)[:, :wp]
        keep = torch.arange(wp).unsqueeze(0) < cnt.unsqueeze(1)
        tables.append(torch.where(keep, vals, torch.zeros_like(vals)).to(torch.int32).contiguous())
        part_lens.append(torch.where(m, tok, torch.zeros_like(tok)).sum(dim=1).to(torch.int32))
    return ChunkedStaging(lo, hi, spans, tables, part_lens)


_SIDE: dict[int, torch.cuda.Stream] = {}
_PARTS: dict[int, torch.Tensor] = {}


def _side_stream(device: torch.device) -> torch.cuda.Stream:
    idx = device.index if device.index is not None else torch.cuda.current_device()
    st = _SIDE.get(idx)
    if st is None:
        st = torch.cuda.Stream(torch.device("cuda", idx))
        _SIDE[idx] = st
    return st


def decode_staged_chunks(q: torch.Tensor, tiers: tuple[KVTier | None, KVTier | None],
                         scale: float, out: torch.Tensor, lse: torch.Tensor | None, plan: ChunkedStaging, *,
                         q_rows: torch.Tensor | None = None, out_rows: torch.Tensor | None = None,
                         parts_buf: torch.Tensor | None = None) -> None:
    """Decode over an HBM tier and a pinned host tier whose blocks are
    staged into HBM chunk by chunk, the copies overlapping the decode.

    The copy engine copies chunk j of `plan` into the staging buffer on a
    side stream and records an event; on the current stream the HBM-tier
    blocks are decoded first (while the first chunk copies), then each
    chunk's blocks once its event has fired, every part into fp32 partials
    (o, lse), and one P-way log-sum-exp merge (fd_merge_partials) combines
    the k + 1 partials into `out` (rows out_rows[i] or i) and `lse` [H, n].
    Only the last chunk's decode and the merge follow the last copy.  The
    staging buffer is the one stage_host_blocks uses; the side stream waits
    for earlier work on the current stream before overwriting it.  The
    side stream forks from and joins the current stream, so a step can be
    captured in a CUDA graph (`parts_buf`: fp32 partials owned by the
    caller, e.g. for a captured step)."""
    host = tiers[1]
    _check(host is not None and host.host, "decode_staged_chunks: tiers[1] must be the pinned host tier")
    _check(host.k.is_contiguous() and host.v.is_contiguous(), "decode_staged_chunks: host tier must be contiguous")
    dev = q.device
    idx = dev.index if dev.index is not None else torch.cuda.current_device()
    n = plan.tables[0].shape[0]
    H, D = q.shape[-2], q.shape[-1]
    P = 1 + len(plan.chunks)
    stride = n * H * D + H * n
    if parts_buf is None:
        parts_buf = _PARTS.get(idx)
        if parts_buf is None or parts_buf.numel() < P * stride:
            parts_buf = torch.empty(P * stride, dtype=torch.float32, device=dev)
            _PARTS[idx] = parts_buf
    _check(parts_buf.dtype == torch.float32 and parts_buf.numel() >= P * stride, "parts_buf too small")
    parts = parts_buf[: P * stride].view(P, stride)
    main = torch.cuda.current_stream(dev)
    side = _side_stream(dev)
    lo, hi = plan.lo, plan.hi
    per = host.k[0].numel()
    need = 2 * max(1, hi - lo) * per
    buf = _STAGE.get(idx)
    if buf is None or buf.numel() < need or buf.dtype != host.k.dtype:
        buf = torch.empty(need, dtype=host.k.dtype, device=torch.device("cuda", idx))
        _STAGE[idx] = buf
    shape = (max(1, hi - lo),) + tuple(host.k.shape[1:])
    kb = buf[: need // 2].view(shape)
    vb = buf[need // 2: need].view(shape)
    staged = KVTier(kb, vb)
    dev_parts = plan.on(dev)

    def part(p: int, t: tuple[KVTier | None, KVTier | None], split: int) -> None:
        bt, ln = dev_parts[p]
        o = parts[p, : n * H * D].view(n, H, D)
        ls = parts[p, n * H * D:].view(H, n)
        a = decode_args(q, t, split, bt, ln, scale, o, ls, q_rows=q_rows,
                        max_len=int(plan.lens[p].max()) if n else 0)
        launch_decode(a, dev)

    ready = torch.cuda.Event()
    ready.record(main)  # earlier readers of the staging buffer come first
    side.wait_event(ready)
    evs = []
    with torch.cuda.stream(side):
        for c_lo, c_hi in plan.chunks:
            kb[c_lo - lo: c_hi - lo].copy_(host.k[c_lo:c_hi], non_blocking=True)
            vb[c_lo - lo: c_hi - lo].copy_(host.v[c_lo:c_hi], non_blocking=True)
            ev = torch.cuda.Event()
            ev.record(side)
            evs.append(ev)
    # no record_stream for the side stream: every use of the buffer there is
    # followed, on the current stream, by a wait on its event, so the
    # buffer's lifetime on the current stream covers the side stream's too
    if tiers[0] is not None:
        part(0, (tiers[0], None), 1 << 40)
    else:
        parts[0, : n * H * D].zero_()
        parts[0, n * H * D:].fill_(float("-inf"))
    for j, ev in enumerate(evs):
        main.wait_event(ev)
        part(j + 1, (None, staged), 0)
    if out_rows is None:
        merge_partials(parts, P, n, H, D, out, lse)
    else:
        tmp = torch.empty(n, H, D, dtype=out.dtype, device=dev)
        merge_partials(parts, P, n, H, D, tmp, lse)
        out.index_copy_(0, out_rows.to(torch.int64), tmp)


# ------------------------------------------------------------- decode


def choose_tiles_per_split(total_tokens: int, n_ctas_per_row: int, block_size: int,
                           num_sms: int = 148) -> int:
    """Tiles (min(block_size,16) tokens) per split so that the grid holds about
    eight waves of two CTAs per SM, given the real token count of the batch."""
    tt = block_size if block_size <= 16 else 16
    tiles = max(1, math.ceil(total_tokens / tt)) * max(1, n_ctas_per_row)
    tps = max(8, math.ceil(tiles / (num_sms * 2 * 8)))
    return (tps + 3) // 4 * 4


def decode_kernel_name(dtype: torch.dtype, head_size: int, num_heads: int, num_kv_heads: int, block_size: int,
                       n: int, tiles_per_split: int = 0) -> str:
    """Name of the kernel fd_decode_attn launches for this shape, mirroring
    the library's dispatch (fd_decode.cu geometry(), fd_decode_mma.cu
    mma_eligible()): the tcgen05 kernel for 16-bit KV, head size 128, query
    group 2/4/8, block size a multiple of 16 and the persistent schedule
    (<= 1024 rows, no explicit split), unless FASTDECODE_B200_MMA=0."""
    G = num_heads // max(1, num_kv_heads)
    persistent = tiles_per_split <= 0 and 0 < n <= 1024
    mma = (persistent and dtype in (torch.float16, torch.bfloat16) and head_size == 128 and G in (2, 4, 8)
           and block_size % 16 == 0 and not os.environ.get("FASTDECODE_B200_MMA", "").startswith("0"))
    return "fd_decode_mma_kernel" if mma else "fd_decode_kernel"


def decode_args(q: torch.Tensor, tiers: tuple[KVTier | None, KVTier | None], tier_split: int,
                block_table: torch.Tensor, lens: torch.Tensor, scale: float, out: torch.Tensor,
                lse: torch.Tensor | None = None, *, q_rows: torch.Tensor | None = None,
                out_rows: torch.Tensor | None = None, max_len: int = 0,
                tiles_per_split: int = 0, n: int | None = None,
                bt_rows: torch.Tensor | None = None,
                workspace_buf: torch.Tensor | None = None, pdl: bool = False) -> nat.FdDecodeArgs:
    """Validate and pack the arguments of fd_decode_attn (workspace included).
    The tensors must stay alive, unmoved, while the returned args are used.
    With bt_rows (int32 [n]) work row i reads table row bt_rows[i]; a
    negative out_rows[i] writes nothing for row i (a device-built decode
    list, plan.plan_on_device).  workspace_buf (uint8, on q's device) replaces
    the shared grow-only workspace, e.g. for launches captured in a CUDA graph,
    whose pointers must stay valid for the graph's lifetime.  pdl=True
    launches the decode as a programmatic dependent of the kernel ahead on
    the stream (FD_DECODE_PDL): only when that kernel writes none of lens,
    block_table, the row maps and q (e.g. it is the layer's KV write or the
    previous decode's combine)."""
    lib = nat.load()
    dev = q.device
    _check(dev.type == "cuda", "q must be a CUDA tensor")
    H, D = q.shape[-2], q.shape[-1]
    _check(q.stride(-1) == 1 and out.stride(-1) == 1, "q and out need a contiguous head dim")
    n = (block_table.shape[0] if bt_rows is None else bt_rows.shape[0]) if n is None else n
    if bt_rows is not None:
        _check(bt_rows.dtype == torch.int32 and bt_rows.device == dev and bt_rows.numel() >= n,
               "bt_rows must be int32 on q's device with n entries")
    for nm, rows in (("q_rows", q_rows), ("out_rows", out_rows)):
        if rows is not None:  # the kernels read them as int64 (fd_decode_args)
            _check(rows.dtype == torch.int64 and rows.device == dev and rows.is_contiguous() and rows.numel() >= n,
                   f"{nm} must be a contiguous int64 tensor on q's device with n entries")
    _check(block_table.dtype == torch.int32 and lens.dtype == torch.int32, "block_table and lens must be int32")
    _check(block_table.stride(-1) == 1, "block_table rows must be contiguous")
    _check(block_table.device == dev and lens.device == dev, "block_table and lens must be on q's device")
    t0, t1 = tiers
    ref = t0 if t0 is not None else t1
    _check(ref is not None, "at least one KV tier is required")
    _check(ref.k.dtype == q.dtype, "q and KV cache dtypes differ")
    KVH, BS = ref.k.shape[1], ref.k.shape[2]
    _check(ref.k.shape[3] == D, "head size mismatch")
    for t in tiers:
        if t is not None:
            _check(t.k.shape[1:] == ref.k.shape[1:], "tiers must share [KVH, BS, D]")
            _check(t.host or t.k.device == dev, "device tier must live on q's device")
    a = nat.FdDecodeArgs()
    a.q = q.data_ptr()
    a.q_stride_n = q.stride(0)
    a.q_stride_h = q.stride(1)
    a.q_rows = _ptr(q_rows)
    a.tier[0] = t0.to_c() if t0 is not None else _empty_tier()
    a.tier[1] = t1.to_c() if t1 is not None else _empty_tier()
    a.tier_split = int(tier_split)
    a.block_table = block_table.data_ptr()
    a.bt_stride = block_table.stride(0)
    a.bt_width = block_table.shape[1]
    a.lens = lens.data_ptr()
    a.n = n
    a.num_heads = H
    a.num_kv_heads = KVH
    a.head_size = D
    a.block_size = BS
    a.scale = float(scale)
    a.dtype = dtype_code(q.dtype)
    a.out = out.data_ptr()
    a.out_dtype = dtype_code(out.dtype)
    a.out_stride_n = out.stride(0)
    a.out_stride_h = out.stride(1)
    a.out_rows = _ptr(out_rows)
    if lse is not None:
        _check(lse.dtype == torch.float32 and lse.device == dev, "lse must be fp32 on q's device")
        a.lse = lse.data_ptr()
        a.lse_stride_h = lse.stride(0)
        a.lse_stride_n = lse.stride(1)
    a.bt_rows = _ptr(bt_rows)
    a.flags = nat.FD_DECODE_PDL if pdl else 0
    a.max_len = int(max_len)
    a.tiles_per_split = int(tiles_per_split)
    a.error = error_word(dev).data_ptr()
    need = lib.fd_decode_workspace_size(ctypes.byref(a))
    if need:
        if workspace_buf is not None:
            _check(workspace_buf.device == dev and workspace_buf.dtype == torch.uint8 and workspace_buf.numel() >= need,
                   f"workspace_buf must be uint8 on q's device with >= {need} bytes")
            ws = workspace_buf
        else:
            ws = workspace(dev, need)
        a.workspace = ws.data_ptr()
        a.workspace_bytes = ws.numel()
    return a


def launch_decode(a: nat.FdDecodeArgs, device: torch.device, phase: str = "all") -> None:
    """Launch fd_decode_attn ("all") or one of its two kernels ("partials",
    "combine") on the current stream of `device`."""
    lib = nat.load()
    fn = {"all": lib.fd_decode_attn, "partials": lib.fd_decode_attn_partials,
          "combine": lib.fd_decode_attn_combine}[phase]
    nat.check(fn(ctypes.byref(a), _stream(device)), f"fd_decode_attn[{phase}]")


def decode_tiered(q: torch.Tensor, tiers: tuple[KVTier | None, KVTier | None], tier_split: int,
                  block_table: torch.Tensor, lens: torch.Tensor, scale: float, out: torch.Tensor,
                  lse: torch.Tensor | None = None, **kw) -> None:
    """Paged decode attention over a two-tier block table (fd_decode_attn).

    q [T, H, D] (rows q_rows[i] or i), tiers[0]/tiers[1] the HBM and host
    tiers (ids < tier_split and >= tier_split), block_table [n, W] int32,
    lens [n] int32, out [*, H, D] (rows out_rows[i] or i; q dtype or fp32),
    lse [H, n] fp32 or None.  Keywords: q_rows, out_rows, max_len,
    tiles_per_split, n (see decode_args), and host_range = (lo, hi): stage
    host-tier blocks [lo, hi) (every host block the step reads) into device
    memory with the copy engine first (stage_host_blocks) and decode from
    there."""
    host_range = kw.pop("host_range", None)
    if host_range is not None and tiers[1] is not None and tiers[1].host:
        lo, hi = host_range
        tiers = (tiers[0], stage_host_blocks(tiers[1], lo, hi, q.device))
        tier_split = tier_split + lo
    a = decode_args(q, tiers, tier_split, block_table, lens, scale, out, lse, **kw)
    launch_decode(a, q.device)


def decode_attn(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                block_table: torch.Tensor, lens: torch.Tensor, scale: float,
                out: torch.Tensor, lse: torch.Tensor) -> None:
    """Reference signature (fastdecode/csrc/cpu_attn.cpp:456-489).

    q [n,H,D] on the GPU; k_cache/v_cache [C,KVH,BS,D] contiguous, either on
    the GPU or pinned host memory (the host tier, read over PCIe);
    block_table [n,W] int32 cache-relative ids; lens [n] int32; out [n,H,D]
    (q dtype); lse [H,n] fp32."""
    for t, name in ((q, "q"), (k_cache, "k_cache"), (v_cache, "v_cache"), (block_table, "block_table"),
                    (lens, "lens"), (out, "out"), (lse, "lse")):
        _check(t.is_contiguous(), f"{name} must be contiguous")
    _check(q.dim() == 3 and k_cache.dim() == 4 and v_cache.shape == k_cache.shape,
           "expected q [n,H,D] and caches [C,KVH,BS,D]")
    _check(block_table.dtype == torch.int32 and lens.dtype == torch.int32, "block_table and lens must be int32")
    _check(lse.dtype == torch.float32, "lse must be float32")
    _check(q.dtype == k_cache.dtype and out.dtype == q.dtype, "q, cache and out dtypes must match")
    n, H, D = q.shape
    KVH, BS = k_cache.shape[1], k_cache.shape[2]
    _check(k_cache.shape[3] == D, "head size mismatch")
    _check(H % KVH == 0, "num_heads must be a multiple of num_kv_heads")
    _check(block_table.dim() == 2 and block_table.shape[0] == n and lens.shape[0] == n,
           "block_table [n, W] and lens [n] expected")
    _check(out.shape == q.shape and lse.shape == (H, n), "out [n,H,D] and lse [H,n] expected")
    if n == 0:
        return
    _check(q.is_cuda, "q must be a CUDA tensor")
    dev = q.device
    bt = block_table if block_table.device == dev else block_table.to(dev, non_blocking=True)
    ln = lens if lens.device == dev else lens.to(dev, non_blocking=True)
    decode_tiered(q, (KVTier(k_cache, v_cache), None), 1 << 62, bt, ln, scale, out, lse)


# ------------------------------------------------------------- KV write


def store_kv_tiered(key: torch.Tensor, value: torch.Tensor, slots: torch.Tensor,
                    tiers: tuple[KVTier | None, KVTier | None], tier_split_blocks: int) -> None:
    """Write new K/V rows [m, KVH, D] to slots (int64, -1 = skip) in either tier."""
    lib = nat.load()
    dev = key.device
    _check(dev.type == "cuda", "key must be a CUDA tensor")
    _check(slots.dtype == torch.int64 and slots.device == dev, "slots must be int64 on key's device")
    _check(key.stride(-1) == 1 and value.stride(-1) == 1, "key/value need a contiguous head dim")
    t0, t1 = tiers
    ref = t0 if t0 is not None else t1
    _check(ref is not None and key.dtype == ref.k.dtype and value.dtype == key.dtype, "dtype mismatch")
    m = slots.shape[0]
    KVH, BS, D = ref.k.shape[1], ref.k.shape[2], ref.k.shape[3]
    _check(key.shape[1] == KVH and key.shape[2] == D and value.shape[1:] == key.shape[1:],
           "key/value must be [m, KVH, D]")
    arr = (nat.FdKvTier * 2)()
    arr[0] = t0.to_c() if t0 is not None else _empty_tier()
    arr[1] = t1.to_c() if t1 is not None else _empty_tier()
    nat.check(lib.fd_store_kv(key.data_ptr(), key.stride(0), key.stride(1), value.data_ptr(),
                              value.stride(0), value.stride(1), slots.data_ptr(), m, KVH, D, BS,
                              dtype_code(key.dtype), arr, int(tier_split_blocks),
                              error_word(dev).data_ptr(), _stream(dev)), "fd_store_kv")


def store_kv(k: torch.Tensor, v: torch.Tensor, slots: torch.Tensor, k_cache: torch.Tensor,
             v_cache: torch.Tensor) -> None:
    """Reference signature (fastdecode/csrc/cpu_attn.cpp:492-517): k, v [m,KVH,D]
    on the GPU; slots [m] int64 cache-relative; caches [C,KVH,BS,D] on the GPU
    or pinned host memory.  An out-of-range slot raises RuntimeError and
    nothing is written."""
    for t, name in ((k, "k"), (v, "v"), (slots, "slots"), (k_cache, "k_cache"), (v_cache, "v_cache")):
        _check(t.is_contiguous(), f"{name} must be contiguous")
    _check(slots.dtype == torch.int64, "slots must be int64")
    _check(k.dtype == k_cache.dtype and v.dtype == k.dtype, "dtype mismatch")
    m = k.shape[0]
    if m == 0:
        return
    C, KVH, BS, D = k_cache.shape
    _check(k.shape[1] == KVH and k.shape[2] == D and v.shape == k.shape, "k/v must be [m, KVH, D]")
    cap = C * BS
    if slots.device.type == "cpu":
        bad = (slots < 0) | (slots >= cap)
        if bool(bad.any()):
            raise RuntimeError(f"CPU slot out of range: {int(slots[bad][0])}")
        slots = slots.to(k.device, non_blocking=True)
    dev = k.device
    store_kv_tiered(k, v, slots, (KVTier(k_cache, v_cache), None), 1 << 62)
    if not torch.cuda.is_current_stream_capturing():
        try:
            check_device_errors(dev)
        except RuntimeError as e:
            raise RuntimeError(f"CPU slot out of range ({e})") from None


# ------------------------------------------------------------- merge


def prefill_attn(q: torch.Tensor, out: torch.Tensor, q_start: torch.Tensor, q_len: torch.Tensor,
                 k_len: torch.Tensor, scale: float, *, kv: KVTier | None = None,
                 block_table: torch.Tensor | None = None, bt_row: torch.Tensor | None = None,
                 k: torch.Tensor | None = None, v: torch.Tensor | None = None,
                 total_q: int | None = None) -> None:
    """Causal prefill attention on the tensor cores (fd_prefill_attn), the
    replacement of flash_attn_varlen_func(causal=True) for the P and F
    classes (fastdecode/backend.py:317-340).

    q, out [T, H, 128] fp16/bf16 (batch rows); per request r (int32 device
    tensors [n]): q_start (first query row), q_len, k_len >= q_len; query i
    sees keys 0 .. k_len - q_len + i.  Keys/values either from the paged
    HBM tier (kv [B, KVH, BS, D] views, block_table [R, W] int32, optional
    bt_row [n] int32 table row of each request) or from the batch's own new
    rows (k, v [T, KVH, D]; key j of request r is row q_start[r] + j).
    total_q bounds the grid (sum of q_len; computed with a host sync when
    not given).  Only the requests' rows of out are written."""
    lib = nat.load()
    dev = q.device
    _check(dev.type == "cuda", "q must be a CUDA tensor")
    _check(q.dim() == 3 and out.shape == q.shape and out.dtype == q.dtype, "q and out must be [T, H, D] alike")
    _check(q.stride(-1) == 1 and out.stride(-1) == 1, "q and out need a contiguous head dim")
    for nm, t in (("q_start", q_start), ("q_len", q_len), ("k_len", k_len)) + ((("bt_row", bt_row),) if bt_row is not None else ()):
        _check(t.dtype == torch.int32 and t.device == dev and t.is_contiguous(), f"{nm} must be contiguous int32 on q's device")
    n = q_len.numel()
    _check(q_start.numel() == n and k_len.numel() == n and (bt_row is None or bt_row.numel() == n),
           "per-request arrays must have the same length")
    T, H, D = q.shape
    a = nat.FdPrefillArgs()
    a.q, a.q_stride_t, a.q_stride_h = q.data_ptr(), q.stride(0), q.stride(1)
    a.out, a.out_stride_t, a.out_stride_h = out.data_ptr(), out.stride(0), out.stride(1)
    t = nat.FdKvTier()
    if block_table is not None:
        _check(kv is not None and not kv.host, "paged prefill needs the device KV tier")
        _check(block_table.dtype == torch.int32 and block_table.device == dev and block_table.stride(-1) == 1,
               "block_table must be int32 on q's device with contiguous rows")
        _check(kv.k.dtype == q.dtype and kv.k.shape[3] == D, "KV tier dtype / head size mismatch")
        t = kv.to_c()
        KVH, BS = kv.k.shape[1], kv.k.shape[2]
        a.block_table, a.bt_stride, a.bt_width = block_table.data_ptr(), block_table.stride(0), block_table.shape[1]
        a.block_size = BS
    else:
        _check(k is not None and v is not None, "give either kv + block_table or k and v")
        _check(k.shape == v.shape and k.stride() == v.stride() and k.dim() == 3 and k.stride(-1) == 1,
               "k and v must be [T, KVH, D] alike with a contiguous head dim")
        _check(k.dtype == q.dtype and k.device == dev and k.shape[2] == D, "k / v dtype, device or head size mismatch")
        KVH = k.shape[1]
        t.k, t.v = k.data_ptr(), v.data_ptr()
        t.blk_stride, t.head_stride, t.tok_stride = 0, k.stride(1), k.stride(0)
        t.num_blocks = k.shape[0]
        a.block_size = 0
    a.kv = t
    a.num_tokens = T
    a.q_start, a.q_len, a.k_len = q_start.data_ptr(), q_len.data_ptr(), k_len.data_ptr()
    a.bt_row = _ptr(bt_row)
    a.n, a.num_heads, a.num_kv_heads, a.head_size = n, H, KVH, D
    a.scale = float(scale)
    a.dtype = dtype_code(q.dtype)
    a.total_q = int(q_len.sum().item()) if total_q is None else int(total_q)
    a.error = error_word(dev).data_ptr()
    nat.check(lib.fd_prefill_attn(ctypes.byref(a), _stream(dev)), "fd_prefill_attn")


def merge_attn_states(out: torch.Tensor, o_a: torch.Tensor, lse_a: torch.Tensor, o_b: torch.Tensor,
                      lse_b: torch.Tensor, out_lse: torch.Tensor | None = None,
                      out_rows: torch.Tensor | None = None) -> None:
    """vLLM merge_attn_states(output, prefix_output, prefix_lse, suffix_output,
    suffix_lse) with the reference's rule (fastdecode/cpu_ops.py:93-113).
    o_a/o_b [n,H,D] contiguous, lse [H,n] fp32; out rows out_rows[i] or i."""
    _check(o_a.shape == o_b.shape and o_a.dtype == o_b.dtype, "o_a and o_b must match")
    _check(o_a.is_contiguous() and o_b.is_contiguous(), "partials must be contiguous")
    n, H, D = o_a.shape
    _check(lse_a.shape == (H, n) and lse_b.shape == (H, n), "lse must be [H, n]")
    _check(lse_a.dtype == torch.float32 and lse_b.dtype == torch.float32, "lse must be float32")
    _check(lse_a.is_contiguous() and lse_b.is_contiguous(), "lse must be contiguous")
    _check(out.stride(-1) == 1 and out.stride(1) == D, "out rows must be [H, D] contiguous")
    dev = o_a.device
    if out_rows is not None:  # read as int64 by the kernel
        _check(out_rows.dtype == torch.int64 and out_rows.device == dev and out_rows.is_contiguous()
               and out_rows.numel() >= n, "out_rows must be a contiguous int64 tensor on the device with n entries")
    nat.check(nat.load().fd_merge_attn_states(
        out.data_ptr(), dtype_code(out.dtype), out.stride(0), _ptr(out_rows), _ptr(out_lse),
        o_a.data_ptr(), lse_a.data_ptr(), o_b.data_ptr(), lse_b.data_ptr(), dtype_code(o_a.dtype),
        n, H, D, _stream(dev)), "fd_merge_attn_states")


def merge_partials(parts: torch.Tensor, num_parts: int, n: int, H: int, D: int, out: torch.Tensor,
                   out_lse: torch.Tensor | None = None) -> None:
    """P-way merge of packed fp32 partials: part p occupies parts[p] =
    [o (n*H*D) | lse (H*n)]."""
    _check(parts.dtype == torch.float32 and parts.is_contiguous(), "parts must be contiguous fp32")
    stride = n * H * D + H * n
    _check(parts.numel() >= num_parts * stride, "parts buffer too small")
    _check(out.is_contiguous() and out.shape == (n, H, D), "out must be [n, H, D] contiguous")
    base = parts.data_ptr()
    nat.check(nat.load().fd_merge_partials(
        base, base + 4 * n * H * D, stride, num_parts, n, H, D, out.data_ptr(), dtype_code(out.dtype),
        _ptr(out_lse), _stream(parts.device)), "fd_merge_partials")


# ------------------------------------------------------------- load_ext shim


class _Ext:
    """Object returned by load_ext(), shaped like the reference's pybind
    module (fastdecode/csrc/cpu_attn.cpp:531-537)."""

    decode_attn = staticmethod(decode_attn)
    store_kv = staticmethod(store_kv)
    merge_attn_states = staticmethod(merge_attn_states)

    @staticmethod
    def set_num_threads(n: int) -> None:  # the GPU path has no host thread pool
        del n

    @staticmethod
    def get_num_threads() -> int:
        return 1

    @staticmethod
    def has_avx2() -> bool:  # no host SIMD kernel exists in this engine
        return False


def load_ext(verbose: bool = False) -> _Ext:
    """Load the native library; raises if it is missing (no fallback)."""
    del verbose
    nat.load()
    return _Ext()
