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

    if bool(host_blk.any()) and int(ids[host_blk].max()) >= G + num_cpu_blocks:
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
