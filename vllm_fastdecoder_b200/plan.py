"""Per-step execution plan: which tokens and requests go to which path.

Same contract as the reference planner (fastdecode/plan.py:1-245): block ids
< G live in the HBM tier, ids >= G in the host tier at id - G, and every
request of the step is in exactly one class

  P  all of its KV blocks are in HBM
  S  a decode (query_len == 1) with at least one host block
  F  a fresh prefill (no prior context) that touches host blocks

A request with query_len > 1, prior context and host blocks (chunked-prefill
continuation, prefix-cache hit) raises NotImplementedError, as in the
reference (plan.py:142-149).  Every HostPlan field the reference defines has
the same name, dtype, shape and value (bit-exact); the fields after them are
this engine's additions for the single-pass two-tier kernel (the S rows'
full block-table rows and lengths, and the P requests that are decodes).

All of build_host_plan runs on CPU tensors, so it is testable without a GPU.
plan_on_device computes the same plan on the GPU from the step's device
tensors (fd_plan_step, one launch, no host copies); device_plan_to_host
reads it back for tests and statistics.
"""

from __future__ import annotations

from dataclasses import dataclass, field

import torch

_I64 = torch.int64
_I32 = torch.int32


@dataclass
class HostPlan:
    n_tok: int
    # KV writes
    gpu_slot_mapping: torch.Tensor  # [n_tok] int64, host-tier slots replaced by -1
    cpu_w_tok: torch.Tensor  # [nw] int64 token rows whose KV goes to the host tier
    cpu_w_slot: torch.Tensor  # [nw] int64 host-tier-relative slots
    # P
    p_tok: torch.Tensor  # [nP_tok] int64
    p_cu: torch.Tensor  # [nP + 1] int32
    p_seqlens: torch.Tensor  # [nP] int32
    p_req: torch.Tensor  # [nP] int64 rows of the block table
    p_max_q: int
    p_max_k: int
    # S
    s_tok: torch.Tensor  # [nS] int64
    s_gpu_bt: torch.Tensor  # [nS, Wg] int32 HBM ids, compacted, width padded to 16
    s_gpu_lens: torch.Tensor  # [nS] int32
    s_max_gpu_len: int
    s_cpu_bt: torch.Tensor  # [nS, Wc] int32 host-relative ids, compacted
    s_cpu_lens: torch.Tensor  # [nS] int32
    # F
    f_tok: torch.Tensor  # [nF_tok] int64
    f_cu: torch.Tensor  # [nF + 1] int32
    f_max: int
    # --- additions of this engine (not in the reference plan)
    s_req: torch.Tensor = field(default_factory=lambda: torch.zeros(0, dtype=_I64))  # [nS] rows
    s_seq_lens: torch.Tensor = field(default_factory=lambda: torch.zeros(0, dtype=_I32))  # [nS]
    s_max_len: int = 0
    pd_req: torch.Tensor = field(default_factory=lambda: torch.zeros(0, dtype=_I64))  # P decodes
    pd_tok: torch.Tensor = field(default_factory=lambda: torch.zeros(0, dtype=_I64))
    pd_seq_lens: torch.Tensor = field(default_factory=lambda: torch.zeros(0, dtype=_I32))
    pd_max_len: int = 0
    pp_req: torch.Tensor = field(default_factory=lambda: torch.zeros(0, dtype=_I64))  # P prefills
    pp_tok: torch.Tensor = field(default_factory=lambda: torch.zeros(0, dtype=_I64))
    pp_cu: torch.Tensor = field(default_factory=lambda: torch.zeros(1, dtype=_I32))
    pp_seqlens: torch.Tensor = field(default_factory=lambda: torch.zeros(0, dtype=_I32))
    pp_max_q: int = 0
    pp_max_k: int = 0
    num_gpu_blocks: int = 0
    block_size: int = 0
    # host-relative range [host_lo, host_hi) of the host blocks the step
    # reads, and how many of them it reads (for staging them in one copy)
    host_lo: int = 0
    host_hi: int = 0
    host_used: int = 0

    @property
    def n_s(self) -> int:
        return int(self.s_tok.numel())

    @property
    def n_p_tok(self) -> int:
        return int(self.p_tok.numel())

    @property
    def n_f_tok(self) -> int:
        return int(self.f_tok.numel())


def spans(starts: torch.Tensor, lengths: torch.Tensor) -> torch.Tensor:
    """Concatenation of arange(s, s + l) over (s, l) pairs, as one int64 tensor."""
    lengths = lengths.to(_I64)
    total = int(lengths.sum()) if lengths.numel() else 0
    if total == 0:
        return torch.zeros(0, dtype=_I64)
    owner = torch.repeat_interleave(torch.arange(lengths.numel(), dtype=_I64), lengths)
    first = torch.cumsum(lengths, 0) - lengths  # output index where each span begins
    return starts.to(_I64)[owner] + (torch.arange(total, dtype=_I64) - first[owner])


def prefix_offsets(lengths: torch.Tensor) -> torch.Tensor:
    """[0, l0, l0+l1, ...] as int32 (cu_seqlens)."""
    out = torch.zeros(lengths.numel() + 1, dtype=_I32)
    if lengths.numel():
        out[1:] = torch.cumsum(lengths.to(_I64), 0).to(_I32)
    return out


def pack_rows(ids: torch.Tensor, keep: torch.Tensor, offset: int, multiple: int = 1) -> torch.Tensor:
    """Per row, move the kept ids (minus `offset`) to the front in their
    original order and zero the rest; width = max kept count (at least 1)
    rounded up to `multiple`.  Returns int32 [rows, width].

    The HBM table is padded to a multiple of 16 like the reference
    (plan.py:82-100), because a FlashAttention-style consumer resolves a whole
    tile of table entries before masking."""
    rows = ids.shape[0]
    if ids.numel() == 0:
        return torch.zeros(rows, multiple, dtype=_I32)
    counts = keep.sum(1)
    width = max(1, int(counts.max()))
    width = -(-width // multiple) * multiple
    dest = torch.cumsum(keep.to(_I64), 1) - 1  # destination column of each kept id
    dest = torch.where(keep, dest, torch.full_like(dest, width))  # dropped -> spill column
    packed = torch.zeros(rows, width + 1, dtype=_I64)
    packed.scatter_(1, dest, torch.where(keep, ids - offset, torch.zeros_like(ids)))
    return packed[:, :width].to(_I32).contiguous()


def build_host_plan(
    query_start_loc: torch.Tensor,  # [R + 1] (cpu)
    seq_lens: torch.Tensor,  # [R] (cpu), tokens including this step's
    block_table: torch.Tensor,  # [R, W] int32 (cpu), W >= ceil(max seq / bs)
    slot_mapping: torch.Tensor,  # [>= n_tok] int64 (cpu)
    num_gpu_blocks: int,
    num_cpu_blocks: int,
    block_size: int,
) -> HostPlan | None:
    """Classify the step's requests and route KV writes (reference
    fastdecode/plan.py:103-199).  Returns None when no request touches the
    host tier and no new token is written there (the plain all-HBM step)."""
    G, bs = int(num_gpu_blocks), int(block_size)
    qsl = query_start_loc.to(_I64)
    seq = seq_lens.to(_I64)
    q_len = qsl[1:] - qsl[:-1]
    prior = seq - q_len
    n_tok = int(qsl[-1]) if qsl.numel() else 0
    slots = slot_mapping[:n_tok].to(_I64)

    blocks_used = (seq + bs - 1) // bs
    W = block_table.shape[1]
    col = torch.arange(W, dtype=_I64).unsqueeze(0)
    in_row = col < blocks_used.unsqueeze(1)
    ids = block_table.to(_I64)
    host_blk = in_row & (ids >= G)
    hbm_blk = in_row & (ids < G)
    touches_host = host_blk.any(1)
    host_slot = slots >= G * bs

    if not bool(touches_host.any()) and not bool(host_slot.any()):
        return None

    host_ids = ids[host_blk]
    if host_ids.numel() and int(host_ids.max()) >= G + num_cpu_blocks:
        raise RuntimeError(
            "FastDecode: block id beyond GPU+CPU capacity; engine and worker "
            "disagree on FASTDECODE_CPU_BLOCKS / FASTDECODE_CPU_KV_GB"
        )

    live = q_len > 0
    cls_s = live & touches_host & (q_len == 1)
    cls_f = live & touches_host & (q_len > 1) & (prior == 0)
    if bool((live & touches_host & (q_len > 1) & (prior > 0)).any()):
        raise NotImplementedError(
            "FastDecode: a request with prior context is being extended by >1 token "
            "while part of its KV is on the CPU (chunked prefill or prefix-cache hit). "
            "Run with enable_prefix_caching=False and "
            "max_num_batched_tokens >= max_model_len."
        )
    cls_p = live & ~touches_host

    gpu_slot_mapping = torch.where(host_slot, torch.full_like(slots, -1), slots)
    cpu_w_tok = host_slot.nonzero().flatten()
    cpu_w_slot = (slots[cpu_w_tok] - G * bs).contiguous()

    p_req = cls_p.nonzero().flatten()
    p_q = q_len[p_req]
    p_seqlens = seq[p_req].to(_I32)

    s_req = cls_s.nonzero().flatten()
    # tokens held by each block of the row: bs, except the row's last block
    per_blk = torch.full_like(ids, bs)
    last = (blocks_used - 1).unsqueeze(1)
    per_blk = torch.where(col == last, (seq - (blocks_used - 1) * bs).unsqueeze(1), per_blk)
    per_blk = per_blk * in_row
    s_ids, s_hbm, s_host, s_per = ids[s_req], hbm_blk[s_req], host_blk[s_req], per_blk[s_req]
    s_gpu_lens = (s_per * s_hbm).sum(1).to(_I32)
    s_cpu_lens = (s_per * s_host).sum(1).to(_I32)

    f_req = cls_f.nonzero().flatten()
    f_q = q_len[f_req]

    pd_req = (cls_p & (q_len == 1)).nonzero().flatten()
    pp_req = (cls_p & (q_len > 1)).nonzero().flatten()
    pp_q = q_len[pp_req]
    pp_seq = seq[pp_req].to(_I32)
    s_seq = seq[s_req].to(_I32)
    pd_seq = seq[pd_req].to(_I32)

    return HostPlan(
        n_tok=n_tok,
        gpu_slot_mapping=gpu_slot_mapping,
        cpu_w_tok=cpu_w_tok,
        cpu_w_slot=cpu_w_slot,
        p_tok=spans(qsl[p_req], p_q),
        p_cu=prefix_offsets(p_q),
        p_seqlens=p_seqlens,
        p_req=p_req,
        p_max_q=int(p_q.max()) if p_q.numel() else 0,
        p_max_k=int(p_seqlens.max()) if p_seqlens.numel() else 0,
        s_tok=qsl[s_req],
        s_gpu_bt=pack_rows(s_ids, s_hbm, 0, multiple=16),
        s_gpu_lens=s_gpu_lens,
        s_max_gpu_len=int(s_gpu_lens.max()) if s_gpu_lens.numel() else 0,
        s_cpu_bt=pack_rows(s_ids, s_host, G),
        s_cpu_lens=s_cpu_lens.contiguous(),
        f_tok=spans(qsl[f_req], f_q),
        f_cu=prefix_offsets(f_q),
        f_max=int(f_q.max()) if f_q.numel() else 0,
        s_req=s_req,
        s_seq_lens=s_seq,
        s_max_len=int(s_seq.max()) if s_seq.numel() else 0,
        pd_req=pd_req,
        pd_tok=qsl[pd_req],
        pd_seq_lens=pd_seq,
        pd_max_len=int(pd_seq.max()) if pd_seq.numel() else 0,
        pp_req=pp_req,
        pp_tok=spans(qsl[pp_req], pp_q),
        pp_cu=prefix_offsets(pp_q),
        pp_seqlens=pp_seq,
        pp_max_q=int(pp_q.max()) if pp_q.numel() else 0,
        pp_max_k=int(pp_seq.max()) if pp_seq.numel() else 0,
        num_gpu_blocks=G,
        block_size=bs,
        host_lo=int(host_ids.min()) - G if host_ids.numel() else 0,
        host_hi=int(host_ids.max()) - G + 1 if host_ids.numel() else 0,
        host_used=int(host_ids.numel()),
    )


@dataclass
class DevicePlan:
    """HostPlan with the tensors the GPU needs on the device (reference
    fastdecode/plan.py:202-221), plus this engine's additions."""

    host: HostPlan
    gpu_slot_mapping: torch.Tensor
    cpu_w_tok: torch.Tensor
    p_tok: torch.Tensor
    p_cu: torch.Tensor
    p_seqlens: torch.Tensor
    p_bt: torch.Tensor  # [nP, W] int32 rows of the batch block table
    s_tok: torch.Tensor
    s_gpu_rows: torch.Tensor  # [nG] int64 S rows with HBM tokens
    s_gpu_cu: torch.Tensor  # arange(nG + 1) int32
    s_gpu_bt: torch.Tensor  # [nG, Wg] int32
    s_gpu_lens: torch.Tensor  # [nG] int32, all > 0
    f_tok: torch.Tensor
    f_cu: torch.Tensor
    # --- additions
    slot_mapping: torch.Tensor | None = None  # [n_tok] int64 unified slots (both tiers)
    s_bt: torch.Tensor | None = None  # [nS, W] int32 full rows (both tiers)
    s_seq_lens: torch.Tensor | None = None  # [nS] int32
    pd_tok: torch.Tensor | None = None
    pd_bt: torch.Tensor | None = None
    pd_seq_lens: torch.Tensor | None = None
    s_cpu_bt: torch.Tensor | None = None  # host-relative compacted table on the device
    s_cpu_lens: torch.Tensor | None = None
    pp_tok: torch.Tensor | None = None
    pp_cu: torch.Tensor | None = None
    pp_seqlens: torch.Tensor | None = None
    pp_bt: torch.Tensor | None = None


def to_device(hp: HostPlan, block_table_dev: torch.Tensor, device) -> DevicePlan:
    """Move the plan to `device` (reference fastdecode/plan.py:224-245).  The
    copies are blocking, like the reference's, so the host tensors can be
    reused right after."""

    def put(t: torch.Tensor) -> torch.Tensor:
        return t.to(device, non_blocking=False)

    with_hbm = (hp.s_gpu_lens > 0).nonzero().flatten()

    def rows(idx: torch.Tensor) -> torch.Tensor:
        if idx.numel():
            return block_table_dev.index_select(0, put(idx))
        return block_table_dev[:0]

    # unified slots for the single tier-aware KV write: HBM slots as they are,
    # host slots restored to their G+C value, skipped (-1) tokens stay -1
    slot_all = hp.gpu_slot_mapping.clone()
    if hp.cpu_w_tok.numel():
        slot_all[hp.cpu_w_tok] = hp.cpu_w_slot + hp.num_gpu_blocks * hp.block_size
    return DevicePlan(
        host=hp,
        gpu_slot_mapping=put(hp.gpu_slot_mapping),
        cpu_w_tok=put(hp.cpu_w_tok),
        p_tok=put(hp.p_tok),
        p_cu=put(hp.p_cu),
        p_seqlens=put(hp.p_seqlens),
        p_bt=rows(hp.p_req),
        s_tok=put(hp.s_tok),
        s_gpu_rows=put(with_hbm),
        s_gpu_cu=torch.arange(with_hbm.numel() + 1, dtype=_I32, device=device),
        s_gpu_bt=put(hp.s_gpu_bt[with_hbm]),
        s_gpu_lens=put(hp.s_gpu_lens[with_hbm]),
        f_tok=put(hp.f_tok),
        f_cu=put(hp.f_cu),
        slot_mapping=put(slot_all),
        s_bt=rows(hp.s_req),
        s_seq_lens=put(hp.s_seq_lens),
        pd_tok=put(hp.pd_tok),
        pd_bt=rows(hp.pd_req),
        pd_seq_lens=put(hp.pd_seq_lens),
        s_cpu_bt=put(hp.s_cpu_bt),
        s_cpu_lens=put(hp.s_cpu_lens),
        pp_tok=put(hp.pp_tok),
        pp_cu=put(hp.pp_cu),
        pp_seqlens=put(hp.pp_seqlens),
        pp_bt=rows(hp.pp_req),
    )


# ------------------------------------------------------------------ on the GPU


class DeviceStepPlan:
    """Device buffers of the plan computed by fd_plan_step (the reference
    planner, fastdecode/plan.py:103-245, run on the GPU): capacities R
    requests, T tokens, table width W; the int32 header (device) says how many
    entries are valid.  Reusable across steps of the same capacities."""

    def __init__(self, R: int, T: int, W: int, device):
        R, T, W = max(1, int(R)), max(1, int(T)), max(1, int(W))
        self.R, self.T, self.W = R, T, W
        self.gw_cap = -(-W // 16) * 16

        def i32(*shape):
            return torch.zeros(shape, dtype=_I32, device=device)

        def i64(*shape):
            return torch.zeros(shape, dtype=_I64, device=device)

        self.header = i32(32)
        self.gpu_slot_mapping, self.cpu_w_tok, self.cpu_w_slot = i64(T), i64(T), i64(T)
        self.p_tok, self.p_cu, self.p_seqlens, self.p_req = i64(T), i32(R + 1), i32(R), i64(R)
        self.s_tok, self.s_gpu_bt, self.s_gpu_lens = i64(R), i32(R, self.gw_cap), i32(R)
        self.s_cpu_bt, self.s_cpu_lens = i32(R, W), i32(R)
        self.f_tok, self.f_cu = i64(T), i32(R + 1)
        self.s_req, self.s_seq_lens = i64(R), i32(R)
        self.pd_req, self.pd_tok, self.pd_seq_lens = i64(R), i64(R), i32(R)
        self.pp_req, self.pp_tok, self.pp_cu, self.pp_seqlens = i64(R), i64(T), i32(R + 1), i32(R)
        self.d_tok, self.d_row, self.d_lens = i64(R), i32(R), i32(R)
        # set by plan_on_device for the step
        self.num_reqs = 0
        self.num_gpu_blocks = 0
        self.block_size = 0
        self.block_table: torch.Tensor | None = None

    def fits(self, R: int, T: int, W: int) -> bool:
        return R <= self.R and T <= self.T and W <= self.W


@dataclass
class DeviceDecodeStep:
    """A decode-only step planned on the GPU, as the backend's attention
    metadata carries it: the device plan and the host-side sizes the
    launches need (all known without reading the device)."""

    plan: DeviceStepPlan
    num_reqs: int
    n_tok: int
    max_seq: int


def plan_on_device(query_start_loc: torch.Tensor, seq_lens: torch.Tensor, block_table: torch.Tensor,
                   slot_mapping: torch.Tensor, num_gpu_blocks: int, num_cpu_blocks: int, block_size: int,
                   out: DeviceStepPlan | None = None, max_tokens: int | None = None) -> DeviceStepPlan:
    """Launch fd_plan_step on the current stream: the step's plan from its
    device tensors (query_start_loc [R+1] int32, seq_lens [R] int32,
    block_table [R, W] int32 with contiguous rows, slot_mapping [>= T] int64),
    no host synchronisation.  `out` is reused when its capacities fit."""
    import ctypes

    from vllm_fastdecoder_b200 import _native as nat
    from vllm_fastdecoder_b200 import gpu_ops

    dev = block_table.device
    R = int(query_start_loc.numel()) - 1
    W = int(block_table.shape[1])
    T = int(slot_mapping.numel()) if max_tokens is None else int(max_tokens)
    if query_start_loc.dtype != _I32 or seq_lens.dtype != _I32 or block_table.dtype != _I32:
        raise RuntimeError("plan_on_device: query_start_loc, seq_lens and block_table must be int32")
    if slot_mapping.dtype != _I64 or int(slot_mapping.numel()) < T:
        raise RuntimeError("plan_on_device: slot_mapping must be int64 with at least max_tokens entries")
    if block_table.stride(1) != 1 or int(block_table.shape[0]) < R or int(seq_lens.numel()) < R:
        raise RuntimeError("plan_on_device: block_table rows must be contiguous and cover every request")
    if out is None or not out.fits(R, T, W):
        out = DeviceStepPlan(R, T, W, dev)
    p = lambda t: t.data_ptr()  # noqa: E731
    a = nat.FdPlanArgs()
    a.query_start_loc, a.seq_lens, a.block_table = p(query_start_loc), p(seq_lens), p(block_table)
    a.bt_stride, a.bt_width, a.num_reqs = block_table.stride(0), W, R
    a.slot_mapping, a.max_tokens, a.block_size = p(slot_mapping), T, int(block_size)
    a.num_gpu_blocks, a.num_cpu_blocks = int(num_gpu_blocks), int(num_cpu_blocks)
    a.header = p(out.header)
    for name in ("gpu_slot_mapping", "cpu_w_tok", "cpu_w_slot", "p_tok", "p_cu", "p_seqlens", "p_req", "s_tok",
                 "s_gpu_bt", "s_gpu_lens", "s_cpu_bt", "s_cpu_lens", "f_tok", "f_cu", "s_req", "s_seq_lens",
                 "pd_req", "pd_tok", "pd_seq_lens", "pp_req", "pp_tok", "pp_cu", "pp_seqlens", "d_tok", "d_row",
                 "d_lens"):
        setattr(a, name, p(getattr(out, name)))
    a.s_gpu_bt_stride, a.s_cpu_bt_stride = out.s_gpu_bt.stride(0), out.s_cpu_bt.stride(0)
    a.error = gpu_ops.error_word(dev).data_ptr()
    lib = nat.load()
    nat.check(lib.fd_plan_step(ctypes.byref(a), gpu_ops._stream(dev)), "fd_plan_step")
    out.num_reqs, out.num_gpu_blocks, out.block_size, out.block_table = R, int(num_gpu_blocks), int(block_size), \
        block_table
    return out


def device_plan_to_host(dp: DeviceStepPlan, num_cpu_blocks: int) -> HostPlan | None:
    """The device plan as a HostPlan (synchronises; for tests and statistics),
    raising exactly where the reference planner raises."""
    from vllm_fastdecoder_b200 import _native as nat

    h = dp.header.cpu().tolist()
    F = nat.PLAN_FIELDS
    flags = h[F["flags"]]
    if flags & nat.PLAN_BAD_OFFSETS:
        raise RuntimeError("FastDecode: query_start_loc is not a 0-based, non-decreasing offset array within "
                           "the token capacity")
    if not flags & nat.PLAN_TOUCHES_HOST:
        return None
    if flags & nat.PLAN_BAD_BLOCK_ID:
        raise RuntimeError("FastDecode: block id beyond GPU+CPU capacity; engine and worker disagree on "
                           "FASTDECODE_CPU_BLOCKS / FASTDECODE_CPU_KV_GB")
    if flags & nat.PLAN_HOST_EXTEND:
        raise NotImplementedError(
            "FastDecode: a request with prior context is being extended by >1 token while part of its KV is on "
            "the CPU (chunked prefill or prefix-cache hit). Run with enable_prefix_caching=False and "
            "max_num_batched_tokens >= max_model_len.")
    n = {k: h[v] for k, v in F.items()}

    def cut(t, k):
        return t[:k].cpu().contiguous()

    nS = n["n_s"]
    return HostPlan(
        n_tok=n["n_tok"],
        gpu_slot_mapping=cut(dp.gpu_slot_mapping, n["n_tok"]),
        cpu_w_tok=cut(dp.cpu_w_tok, n["n_cpu_w"]),
        cpu_w_slot=cut(dp.cpu_w_slot, n["n_cpu_w"]),
        p_tok=cut(dp.p_tok, n["n_p_tok"]),
        p_cu=cut(dp.p_cu, n["n_p"] + 1),
        p_seqlens=cut(dp.p_seqlens, n["n_p"]),
        p_req=cut(dp.p_req, n["n_p"]),
        p_max_q=n["p_max_q"],
        p_max_k=n["p_max_k"],
        s_tok=cut(dp.s_tok, nS),
        s_gpu_bt=dp.s_gpu_bt[:nS, :n["s_gpu_width"]].cpu().contiguous(),
        s_gpu_lens=cut(dp.s_gpu_lens, nS),
        s_max_gpu_len=n["s_max_gpu_len"],
        s_cpu_bt=dp.s_cpu_bt[:nS, :n["s_cpu_width"]].cpu().contiguous(),
        s_cpu_lens=cut(dp.s_cpu_lens, nS),
        f_tok=cut(dp.f_tok, n["n_f_tok"]),
        f_cu=cut(dp.f_cu, n["n_f"] + 1),
        f_max=n["f_max"],
        s_req=cut(dp.s_req, nS),
        s_seq_lens=cut(dp.s_seq_lens, nS),
        s_max_len=n["s_max_len"],
        pd_req=cut(dp.pd_req, n["n_pd"]),
        pd_tok=cut(dp.pd_tok, n["n_pd"]),
        pd_seq_lens=cut(dp.pd_seq_lens, n["n_pd"]),
        pd_max_len=n["pd_max_len"],
        pp_req=cut(dp.pp_req, n["n_pp"]),
        pp_tok=cut(dp.pp_tok, n["n_pp_tok"]),
        pp_cu=cut(dp.pp_cu, n["n_pp"] + 1),
        pp_seqlens=cut(dp.pp_seqlens, n["n_pp"]),
        pp_max_q=n["pp_max_q"],
        pp_max_k=n["pp_max_k"],
        num_gpu_blocks=dp.num_gpu_blocks,
        block_size=dp.block_size,
    )
