"""Seeded synthetic batches of the benchmark configurations.

The reference uses no dataset for this path; these generators produce inputs
with the configurations' shapes and value distributions (N(0,1) q/K/V,
1/sqrt(head_size) scale), deterministic in the seed:

  c0  16 rows, 32/32 heads, D 128, fp16, BS 16, lens ~ U[64, 2048], one
      4096-block pool [C, KVH, BS, D], disjoint random blocks per row
      (the reference's CPU-runnable kernel case)
  c1  64 rows, same heads, lens ~ U[256, 4096]; per row a host fraction in
      {0, .25, .5, .75, 1}; blocks are an HBM prefix (ids < G = 2048, vLLM
      NHD layout) and a host suffix (ids >= G, pinned [C, KVH, BS, D]); HBM
      ids are handed out GPU-first, so rows whose prefix no longer fits in
      the 2048 HBM blocks spill the rest of the prefix to the host tier
  c2  256 rows, 32/8 heads, bf16, lens = clip(round(exp(N(ln 1024, 0.75^2))),
      32, 8192) (the spread is not given by the configuration; 0.75 is this
      engine's choice), all HBM (NHD)
  c3  8 rows of 131072 tokens, 32/8 heads, bf16; each row's 8192 blocks are
      cut into P contiguous shards, rank r holding shard r in its HBM
  c4  a continuous-batching decode trace (trace4): 32 layers, 32/32 heads,
      D 128, fp16, BS 16, HBM tier 2048 blocks, host tier up to 32768
      blocks, up to 128 running requests, Poisson arrivals, prompts
      U[128, 1024], outputs U[64, 1024]; blocks are handed out HBM-first and
      reused last-in-first-out after a request finishes

A Batch holds the CPU-side description (lengths, unified block table, tier
sizes); materialize() puts the KV tiers and queries in memory.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch

from vllm_fastdecoder_b200.gpu_ops import KVTier


@dataclass
class Batch:
    name: str
    n: int
    H: int
    KVH: int
    D: int
    BS: int
    dtype: torch.dtype
    lens: torch.Tensor  # [n] int32 (cpu)
    block_table: torch.Tensor  # [n, W] int32 (cpu), unified ids
    G: int  # ids < G: HBM tier
    num_hbm_blocks: int
    num_host_blocks: int
    hbm_layout: str  # "nhd" (vLLM [B, BS, KVH, 2D]) or "hnd" ([B, KVH, BS, D])
    seed: int

    @property
    def scale(self) -> float:
        return 1.0 / math.sqrt(self.D)

    @property
    def elem(self) -> int:
        return torch.empty((), dtype=self.dtype).element_size()

    def tier_tokens(self) -> tuple[int, int]:
        """(tokens read from HBM, tokens read from the host tier) per step."""
        hbm = host = 0
        for i in range(self.n):
            L = int(self.lens[i])
            nb = (L + self.BS - 1) // self.BS
            for j in range(nb):
                t = self.BS if j < nb - 1 else L - (nb - 1) * self.BS
                if int(self.block_table[i, j]) < self.G:
                    hbm += t
                else:
                    host += t
        return hbm, host

    def kv_bytes(self) -> tuple[int, int]:
        """Algorithmic K+V bytes per step from (HBM, host)."""
        hbm, host = self.tier_tokens()
        per_tok = 2 * self.KVH * self.D * self.elem
        return hbm * per_tok, host * per_tok

    def step_bytes(self) -> int:
        """All algorithmic bytes of one step: K/V once, q, o, lse, table rows."""
        hbm, host = self.kv_bytes()
        qo = 2 * self.n * self.H * self.D * self.elem
        lse = 4 * self.n * self.H
        table = 4 * sum((int(x) + self.BS - 1) // self.BS for x in self.lens)
        return hbm + host + qo + lse + table


def _disjoint_table(lens: list[int], BS: int, pool: int, g: torch.Generator, base: int = 0) -> torch.Tensor:
    nbs = [(L + BS - 1) // BS for L in lens]
    W = max(1, max(nbs))
    perm = torch.randperm(pool, generator=g)
    bt = torch.zeros(len(lens), W, dtype=torch.int32)
    pos = 0
    for i, nb in enumerate(nbs):
        assert pos + nb <= pool, "pool too small for disjoint blocks"
        bt[i, :nb] = (perm[pos:pos + nb] + base).to(torch.int32)
        pos += nb
    return bt


def config0(seed: int = 0) -> Batch:
    g = torch.Generator().manual_seed(seed)
    n, H, KVH, D, BS, C = 16, 32, 32, 128, 16, 4096
    lens = torch.randint(64, 2049, (n,), generator=g, dtype=torch.int32)
    bt = _disjoint_table(lens.tolist(), BS, C, g)
    return Batch("c0", n, H, KVH, D, BS, torch.float16, lens, bt, G=C, num_hbm_blocks=C,
                 num_host_blocks=0, hbm_layout="hnd", seed=seed)


def config1(seed: int = 0, G: int = 2048) -> Batch:
    g = torch.Generator().manual_seed(seed)
    n, H, KVH, D, BS = 64, 32, 32, 128, 16
    lens = torch.randint(256, 4097, (n,), generator=g, dtype=torch.int32)
    frac = torch.randint(0, 5, (n,), generator=g).double() / 4.0
    hbm_free = torch.randperm(G, generator=g).tolist()
    rows = []
    for i in range(n):
        nb = (int(lens[i]) + BS - 1) // BS
        want_host = int(math.floor(float(frac[i]) * nb + 0.5))
        want_hbm = nb - want_host
        take = min(want_hbm, len(hbm_free))
        hbm_ids = [hbm_free.pop() for _ in range(take)]
        rows.append((hbm_ids, nb - take))  # prefix in HBM, the rest on the host
    C = sum(k for _, k in rows)
    host_perm = (torch.randperm(max(C, 1), generator=g) + G).tolist()
    W = max(len(h) + k for h, k in rows)
    bt = torch.zeros(n, W, dtype=torch.int32)
    pos = 0
    for i, (hbm_ids, k) in enumerate(rows):
        ids = hbm_ids + host_perm[pos:pos + k]
        pos += k
        bt[i, :len(ids)] = torch.tensor(ids, dtype=torch.int32)
    return Batch("c1", n, H, KVH, D, BS, torch.float16, lens, bt, G=G, num_hbm_blocks=G,
                 num_host_blocks=max(C, 1), hbm_layout="nhd", seed=seed)


def config2(seed: int = 0, sigma: float = 0.75) -> Batch:
    g = torch.Generator().manual_seed(seed)
    n, H, KVH, D, BS = 256, 32, 8, 128, 16
    z = torch.randn(n, generator=g, dtype=torch.float64)
    lens = torch.exp(z * sigma + math.log(1024.0)).round().clamp(32, 8192).to(torch.int32)
    pool = int(sum((int(L) + BS - 1) // BS for L in lens))
    bt = _disjoint_table(lens.tolist(), BS, pool, g)
    return Batch("c2", n, H, KVH, D, BS, torch.bfloat16, lens, bt, G=pool, num_hbm_blocks=pool,
                 num_host_blocks=0, hbm_layout="nhd", seed=seed)


def config3(world: int = 1, rank: int = 0, seed: int = 0, ctx: int = 131072) -> Batch:
    """The shard of rank `rank` out of `world`: every row keeps tokens
    [rank*ctx/world, (rank+1)*ctx/world) in a local pool."""
    n, H, KVH, D, BS = 8, 32, 8, 128, 16
    assert ctx % (BS * world) == 0
    local = ctx // world
    g = torch.Generator().manual_seed(seed * 1000 + rank)
    lens = torch.full((n,), local, dtype=torch.int32)
    pool = n * local // BS
    bt = _disjoint_table(lens.tolist(), BS, pool, g)
    return Batch(f"c3/{world}", n, H, KVH, D, BS, torch.bfloat16, lens, bt, G=pool, num_hbm_blocks=pool,
                 num_host_blocks=0, hbm_layout="nhd", seed=seed)


CONFIGS = {"c0": config0, "c1": config1, "c2": config2, "c3": config3}


@dataclass
class TraceStep:
    """One decode step of the trace: every running request adds one token."""

    block_table: torch.Tensor  # [R, W] int32, unified ids (junk-free past each row's end: zeros)
    lens: torch.Tensor  # [R] int32, context including the new token
    slots: torch.Tensor  # [R] int64, unified slot of the new token (id * BS + offset)

    @property
    def rows(self) -> int:
        return int(self.lens.numel())


@dataclass
class Trace:
    name: str
    layers: int
    H: int
    KVH: int
    D: int
    BS: int
    dtype: torch.dtype
    G: int  # HBM tier blocks (ids < G)
    host_blocks: int  # host-tier blocks the trace touches (ids G .. G + host_blocks - 1)
    steps: list[TraceStep]
    seed: int

    @property
    def scale(self) -> float:
        return 1.0 / math.sqrt(self.D)

    def batch(self, k: int) -> Batch:
        """Step k as a Batch (for byte counts and the reference's CPU leg)."""
        st = self.steps[k]
        return Batch(f"{self.name}[{k}]", st.rows, self.H, self.KVH, self.D, self.BS, self.dtype, st.lens,
                     st.block_table, G=self.G, num_hbm_blocks=self.G, num_host_blocks=self.host_blocks,
                     hbm_layout="nhd", seed=self.seed)


def trace4(seed: int = 0, steps: int = 16, layers: int = 32, max_running: int = 128, G: int = 2048,
           C: int = 32768, prompt: tuple[int, int] = (128, 1024), output: tuple[int, int] = (64, 1024)) -> Trace:
    """Config 4: a continuous-batching decode trace, simulated on the CPU.

    The trace starts in steady state: max_running requests whose prompts
    and output lengths are drawn from the configuration's distributions and
    whose progress through their outputs is uniform.  Each step every running
    request decodes one token (taking a new block at a block boundary);
    requests that reach their output length finish and free their blocks;
    Poisson arrivals at the rate that keeps max_running busy (max_running /
    mean output length) join when there is room.  Blocks are handed out
    HBM-first (ids 1 .. G-1; id 0 is vLLM's null block), then from the host
    tier (ids >= G), and freed blocks of either tier are reused
    last-in-first-out, so the host ids in use stay compact."""
    rng = torch.Generator().manual_seed(seed)
    BS = 16

    def uni(lo, hi):
        return int(torch.randint(lo, hi + 1, (1,), generator=rng))

    free_hbm = list(range(1, G))
    free_host = list(range(G, G + C))

    def alloc():
        if free_hbm:
            return free_hbm.pop(0)
        if free_host:
            return free_host.pop(0)
        raise RuntimeError("trace4: out of KV blocks")

    def release(blocks):
        free_hbm[:0] = [b for b in reversed(blocks) if b < G]
        free_host[:0] = [b for b in reversed(blocks) if b >= G]

    running = []

    def admit(progress: bool):
        P, out = uni(*prompt), uni(*output)
        done = uni(0, out - 1) if progress else 0
        ctx = P + done
        blocks = [alloc() for _ in range((ctx + BS - 1) // BS)]
        running.append({"ctx": ctx, "left": out - done, "blocks": blocks})

    for _ in range(max_running):
        admit(True)
    rate = max_running / ((output[0] + output[1]) / 2)
    queue = 0
    out_steps = []
    max_host = G - 1
    for _ in range(steps):
        queue += int(torch.poisson(torch.tensor([rate]), generator=rng))
        while queue > 0 and len(running) < max_running:
            admit(False)
            queue -= 1
        R = len(running)
        W = max((r["ctx"] + BS) // BS + 1 for r in running)
        bt = torch.zeros(R, W, dtype=torch.int32)
        lens = torch.empty(R, dtype=torch.int32)
        slots = torch.empty(R, dtype=torch.int64)
        for i, r in enumerate(running):
            pos = r["ctx"]  # the new token's position
            if pos % BS == 0:
                r["blocks"].append(alloc())
            bl = r["blocks"]
            bt[i, :len(bl)] = torch.tensor(bl, dtype=torch.int32)
            lens[i] = pos + 1
            slots[i] = bl[pos // BS] * BS + pos % BS
            max_host = max(max_host, max(bl))
        out_steps.append(TraceStep(bt, lens, slots))
        for r in list(running):
            r["ctx"] += 1
            r["left"] -= 1
            if r["left"] == 0:
                running.remove(r)
                release(r["blocks"])
    return Trace("c4", layers, 32, 32, 128, BS, torch.float16, G, max(1, max_host - G + 1), out_steps, seed)


@dataclass
class Resident:
    """A batch placed in memory: queries and tables on the device, the HBM
    tier on the device, the host tier pinned and mapped."""

    batch: Batch
    q: torch.Tensor  # [n, H, D] device
    tiers: tuple[KVTier | None, KVTier | None]
    hbm_storage: torch.Tensor | None  # the physical HBM tensor (NHD or HND)
    block_table: torch.Tensor  # device
    lens: torch.Tensor  # device


def _fill_normal(t: torch.Tensor, gen: torch.Generator) -> None:
    t.normal_(generator=gen)


def materialize(b: Batch, device: torch.device, seed: int | None = None) -> Resident:
    seed = b.seed if seed is None else seed
    gen = torch.Generator(device=device).manual_seed(seed + 1)
    dt, KVH, BS, D = b.dtype, b.KVH, b.BS, b.D
    hbm_tier = None
    phys = None
    if b.num_hbm_blocks > 0:
        if b.hbm_layout == "nhd":
            phys = torch.empty(b.num_hbm_blocks, BS, KVH, 2 * D, dtype=dt, device=device)
            _fill_normal(phys, gen)
            k = phys[..., :D].permute(0, 2, 1, 3)
            v = phys[..., D:].permute(0, 2, 1, 3)
        else:
            phys = torch.empty(2, b.num_hbm_blocks, KVH, BS, D, dtype=dt, device=device)
            _fill_normal(phys, gen)
            k, v = phys[0], phys[1]
        hbm_tier = KVTier(k, v)
    host_tier = None
    if b.num_host_blocks > 0:
        shape = (b.num_host_blocks, KVH, BS, D)
        hk = torch.empty(shape, dtype=dt, pin_memory=True)
        hv = torch.empty(shape, dtype=dt, pin_memory=True)
        chunk = max(1, (256 << 20) // (KVH * BS * D * hk.element_size()))
        tmp = torch.empty((chunk,) + shape[1:], dtype=dt, device=device)
        for dst in (hk, hv):
            for s in range(0, shape[0], chunk):
                e = min(shape[0], s + chunk)
                _fill_normal(tmp[:e - s], gen)
                dst[s:e].copy_(tmp[:e - s])
        del tmp
        host_tier = KVTier(hk, hv)
    q = torch.empty(b.n, b.H, D, dtype=dt, device=device)
    _fill_normal(q, gen)
    if device is not None and torch.device(device).type == "cuda":
        torch.cuda.synchronize(device)
    return Resident(b, q, (hbm_tier, host_tier), phys, b.block_table.to(device), b.lens.to(device))
