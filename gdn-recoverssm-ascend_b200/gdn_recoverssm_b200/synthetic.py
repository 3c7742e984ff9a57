"""Seeded synthetic workloads with the shapes and value distributions of the
benchmark configurations (no dataset is involved anywhere on this path).

Distributions: checkpoint states ~ N(0, 0.1^2); q, k ~ N(0, 1) then
L2-normalised per head; v ~ N(0, 1); g = -softplus(N(0, 1)) (so the decay
exp(g) lies in (0, 1)); beta = sigmoid(N(0, 1)).  Metadata (slots, accepted
lengths, block tables, positions) comes from a CPU generator so that every
rank of a sharded run sees identical metadata.  Every per-head tensor (q, k
per key head; v, g, beta, the state tiles and the raw gate inputs per value
head) comes from a device generator seeded by (seed, config, tensor, global
head index) and drawn in fixed-size pieces, so a rank's shard holds exactly
the values of its heads in the unsharded workload.

Configurations (``CONFIGS``):
  0  B=4,    H=HV=4,      K=V=64,  Q=4, fp32 everything, pool 8, none mode
  1  B=64,   H=16, HV=32, K=V=128, Q=4, bf16 q/k/v, pool 256, none mode
  2  B=512,  H=16, HV=32, K=V=128, Q=4, bf16, align (block 64), pool 4096
  3  B=1024, H=16, HV=32, K=V=128, Q=1, bf16, pool 2048, every token accepted
  4  B=1024, H=32, HV=64, K=V=128, Q=8, bf16, align (block 64), pool 2048,
     accepted ~ geometric(0.35) clipped to [1, 8]; source page = bt[C//64]
     so a crossed boundary aliases the source page
Sharding (``world``/``rank``): a rank owns value heads
[rank*HV/world, (rank+1)*HV/world) and the matching key heads, and a state
pool of its heads only.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch

from .sharding import head_shard

CONFIGS = {
    0: dict(B=4, H=4, HV=4, D=64, Q=4, pool=8, act=torch.float32, align=False, accept="uniform"),
    1: dict(B=64, H=16, HV=32, D=128, Q=4, pool=256, act=torch.bfloat16, align=False, accept="uniform"),
    2: dict(B=512, H=16, HV=32, D=128, Q=4, pool=4096, act=torch.bfloat16, align=True, accept="uniform",
            block=64, max_pos=8192, layout="three_pages"),
    3: dict(B=1024, H=16, HV=32, D=128, Q=1, pool=2048, act=torch.bfloat16, align=False, accept="all"),
    4: dict(B=1024, H=32, HV=64, D=128, Q=8, pool=2048, act=torch.bfloat16, align=True, accept="geometric",
            block=64, max_pos=8192, layout="source_aliases_boundary"),
}


@dataclass
class Workload:
    """One verify + commit step's device tensors (single layer)."""

    cfg: int
    B: int
    H: int
    HV: int
    D: int
    Q: int
    q: torch.Tensor
    k: torch.Tensor
    v: torch.Tensor
    g: torch.Tensor
    beta: torch.Tensor
    state: torch.Tensor
    records: torch.Tensor
    out: torch.Tensor
    qsl: torch.Tensor
    state_indices: torch.Tensor
    accepted: torch.Tensor
    request_indices: torch.Tensor
    block_table: torch.Tensor | None = None
    num_computed: torch.Tensor | None = None
    block_size: int | None = None
    conv: torch.Tensor | None = None
    # raw gate inputs of the fused-gating verify (make(..., gated=True)):
    # a, b [T, HV] in the activation dtype; A_log, dt_bias [HV] fp32
    a: torch.Tensor | None = None
    b: torch.Tensor | None = None
    A_log: torch.Tensor | None = None
    dt_bias: torch.Tensor | None = None
    extra: dict = field(default_factory=dict)

    @property
    def tokens(self) -> int:
        return self.B * self.Q

    @property
    def units(self) -> int:
        return self.B * self.HV


def _unit_norm(x):
    return x / x.norm(dim=-1, keepdim=True).clamp_min(1e-6)


def _accepted(spec, gen):
    B, Q = spec["B"], spec["Q"]
    if spec["accept"] == "all":
        return torch.full((B,), Q, dtype=torch.int32)
    if spec["accept"] == "uniform":
        return torch.randint(1, Q + 1, (B,), generator=gen, dtype=torch.int32)
    # geometric(p) on {1, 2, ...}: number of trials to the first success
    p = 0.35
    u = torch.rand(B, generator=gen, dtype=torch.float64)
    a = torch.floor(torch.log1p(-u) / math.log1p(-p)) + 1
    return a.clamp(1, Q).to(torch.int32)


def spec_of(cfg: int, rows: int | None = None, pool: int | None = None) -> dict:
    """The configuration's shape, optionally with fewer rows / a smaller pool
    (reduced cases for profiling; the benchmark uses the full shapes)."""
    spec = dict(CONFIGS[cfg])
    if rows is not None:
        spec["B"] = int(rows)
    if pool is not None:
        spec["pool"] = int(pool)
    return spec


def metadata(cfg: int, seed: int = 0, rows: int | None = None, pool: int | None = None):
    """Host-side (CPU) metadata of a configuration; identical on every rank."""
    spec = spec_of(cfg, rows, pool)
    gen = torch.Generator().manual_seed(1000 + seed * 17 + cfg)
    B, Q, pool = spec["B"], spec["Q"], spec["pool"]
    accepted = _accepted(spec, gen)
    qsl = torch.arange(B + 1, dtype=torch.int32) * Q
    meta = dict(accepted=accepted, qsl=qsl, request_indices=torch.arange(B, dtype=torch.int64))
    if not spec["align"]:
        ids = torch.randperm(pool - 1, generator=gen)[:B] + 1
        meta["state_indices"] = ids.to(torch.int32)
        return meta
    bs, max_pos = spec["block"], spec["max_pos"]
    W = -(-(max_pos + Q) // bs)
    C = torch.randint(0, max_pos, (B,), generator=gen, dtype=torch.int64)
    bt = torch.zeros(B, W, dtype=torch.int32)
    if spec["layout"] == "three_pages":
        ids = torch.randperm(pool - 1, generator=gen)[: 3 * B] + 1
        ids = ids.view(B, 3)
        src = ids[:, 0]
        cols = C // bs
        bt[torch.arange(B), cols] = ids[:, 1].to(torch.int32)
        nxt = (cols + 1).clamp(max=W - 1)
        bt[torch.arange(B), nxt] = ids[:, 2].to(torch.int32)
    else:
        cols = C // bs
        crossing = (C % bs) >= bs - Q  # only these rows can cross with <= Q tokens
        need = B + int(crossing.sum())
        ids = torch.randperm(pool - 1, generator=gen)[:need] + 1
        src = ids[:B]
        bt[torch.arange(B), cols] = src.to(torch.int32)
        extra = ids[B:]
        rows = crossing.nonzero().flatten()
        nxt = (cols[rows] + 1).clamp(max=W - 1)
        bt[rows, nxt] = extra.to(torch.int32)
    meta.update(
        state_indices=src.to(torch.int32),
        block_table=bt,
        num_computed=C.to(torch.int32),
        block_size=bs,
    )
    return meta


_STATE_PAGES_PER_DRAW = 256  # state pages drawn per generator call (fixed: values do not depend on the pool size)


def _head_generator(dev, seed: int, cfg: int, kind: int, head: int):
    """The generator of one (tensor, global head): independent of world size
    and rank."""
    return torch.Generator(device=dev).manual_seed(
        (seed + 1) * 1_000_003 + cfg * 100_003 + kind * 10_007 + head * 101 + 17)


def make(cfg: int, device, *, seed: int = 0, world: int = 1, rank: int = 0, conv_dim: int = 0,
         rows: int | None = None, pool: int | None = None, gated: bool = False) -> Workload:
    """Allocate and fill one configuration's tensors on ``device`` (this
    rank's head shard: exactly those heads' values of the unsharded
    workload).  ``gated`` adds the raw gate inputs of the fused-gating verify:
    a, b ~ N(0, 1) in the activation dtype, A_log = log(U(1, 16)) and dt_bias
    = softplus^-1(dt) with dt log-uniform in [1e-3, 1e-1] per value head."""
    spec = spec_of(cfg, rows, pool)
    B, H, HV, D, Q, pool = spec["B"], spec["H"], spec["HV"], spec["D"], spec["Q"], spec["pool"]
    shard = head_shard(H, HV, world, rank)
    H, HV = shard.key_heads, shard.value_heads
    act = spec["act"]
    meta = metadata(cfg, seed, rows, pool)
    dev = torch.device(device)
    T = B * Q

    def key_head(kind, j, shape):  # local key head j
        return torch.randn(shape, generator=_head_generator(dev, seed, cfg, kind, shard.key_begin + j), device=dev)

    def value_head(kind, j, shape):  # local value head j
        return torch.randn(shape, generator=_head_generator(dev, seed, cfg, kind, shard.value_begin + j), device=dev)

    q = torch.empty(1, T, H, D, dtype=act, device=dev)
    k = torch.empty(1, T, H, D, dtype=act, device=dev)
    for j in range(H):
        q[0, :, j] = _unit_norm(key_head(0, j, (T, D))).to(act)
        k[0, :, j] = _unit_norm(key_head(1, j, (T, D))).to(act)
    v = torch.empty(1, T, HV, D, dtype=act, device=dev)
    g = torch.empty(T, HV, device=dev)
    beta = torch.empty(T, HV, device=dev)
    state = torch.empty(pool, HV, D, D, device=dev)
    for j in range(HV):
        v[0, :, j] = value_head(2, j, (T, D)).to(act)
        gb = value_head(3, j, (2, T))
        g[:, j] = -torch.nn.functional.softplus(gb[0])
        beta[:, j] = torch.sigmoid(gb[1])
        gen = _head_generator(dev, seed, cfg, 4, shard.value_begin + j)
        for p0 in range(0, pool, _STATE_PAGES_PER_DRAW):
            p1 = min(pool, p0 + _STATE_PAGES_PER_DRAW)
            state[p0:p1, j] = torch.randn((p1 - p0, D, D), generator=gen, device=dev) * 0.1
    records = torch.zeros(B, HV, Q, 2 * D + 1, device=dev)
    out = torch.zeros(1, T, HV, D, dtype=act, device=dev)
    wl = Workload(
        cfg=cfg, B=B, H=H, HV=HV, D=D, Q=Q, q=q, k=k, v=v, g=g, beta=beta, state=state, records=records, out=out,
        qsl=meta["qsl"].to(dev), state_indices=meta["state_indices"].to(dev), accepted=meta["accepted"].to(dev),
        request_indices=meta["request_indices"].to(dev),
    )
    if spec["align"]:
        wl.block_table = meta["block_table"].to(dev)
        wl.num_computed = meta["num_computed"].to(dev)
        wl.block_size = meta["block_size"]
    if conv_dim:  # the conv state of this rank's channels (not a head slice of anything)
        gen = torch.Generator(device=dev).manual_seed(7919 * (seed + 1) + 104729 * rank + cfg)
        wl.conv = torch.randn(pool, conv_dim, 3 + Q - 1, generator=gen, device=dev).to(act)
    if gated:
        wl.a = torch.empty(T, HV, dtype=act, device=dev)
        wl.b = torch.empty(T, HV, dtype=act, device=dev)
        wl.A_log = torch.empty(HV, device=dev)
        wl.dt_bias = torch.empty(HV, device=dev)
        lo, hi = math.log(1e-3), math.log(1e-1)
        for j in range(HV):
            ab = value_head(5, j, (2, T))
            wl.a[:, j] = ab[0].to(act)
            wl.b[:, j] = ab[1].to(act)
            u = torch.rand(2, generator=_head_generator(dev, seed, cfg, 6, shard.value_begin + j), device=dev)
            wl.A_log[j] = torch.log(u[0] * 15.0 + 1.0)
            dt = torch.exp(u[1] * (hi - lo) + lo)
            wl.dt_bias[j] = dt + torch.log(-torch.expm1(-dt))
    wl.extra["meta"] = meta
    wl.extra["shard"] = shard
    return wl


def verify_bytes(wl: Workload, units: int | None = None) -> int:
    """Algorithmic bytes of one verify call (packed records): state read,
    q/k/v/g/beta read (the raw a/b of the fused-gating form instead, when the
    workload has them), output and record write, qsl + index read."""
    sa = wl.q.element_size()
    U = wl.units if units is None else units
    T, H, HV, D = wl.tokens, wl.H, wl.HV, wl.D
    gates = (wl.a.element_size() + wl.b.element_size()) if wl.a is not None else (4 + wl.beta.element_size())
    return (U * D * D * 4 + T * H * D * sa * 2 + T * HV * D * sa + T * HV * gates
            + T * HV * D * sa + T * HV * (2 * D + 1) * 4 + 8 * wl.B)


def conv_bytes(wl: Workload, lengths, boundary_written, history: int) -> int:
    """Algorithmic bytes of one conv compaction: per working row the history
    window read and written (twice where a boundary snapshot is also taken)."""
    n = torch.as_tensor(lengths).long()
    working = int((n > 0).sum())
    per = wl.conv.shape[1] * history * wl.conv.element_size() * 2
    return (working + int(boundary_written)) * per


def conv_floor_bytes(wl: Workload, lengths, source, final, boundary, boundary_written) -> int:
    """Bytes one conv compaction must move in a dim-first pool, whose channel
    windows are adjacent W-element rows: the history positions of every row
    cover every 32-byte sector of a page's channel block, and stores of the
    first ``history`` positions leave the rest of each sector to be preserved.
    Per working row: the source block read, the final block read and written
    (written only, in place), and per boundary snapshot the boundary block
    read and written (written only, when it is the source page)."""
    n = torch.as_tensor(lengths).long()
    src, fin, bnd = (torch.as_tensor(t).long() for t in (source, final, boundary))
    written = torch.as_tensor(boundary_written).bool()
    work = n > 0
    page = wl.conv.shape[1] * wl.conv.shape[2] * wl.conv.element_size()
    blocks = work.sum() + (work & (fin != src)).sum() * 2 + (work & (fin == src)).sum()
    blocks += (work & written & (bnd != src)).sum() * 2 + (work & written & (bnd == src)).sum()
    return int(blocks) * page


def commit_bytes(wl: Workload, lengths, boundary_written) -> int:
    """Algorithmic bytes of one fold call: state read + final write (+ the
    boundary snapshot where one is written) + the accepted records read."""
    HV, D = wl.HV, wl.D
    n = torch.as_tensor(lengths).long()
    working = int((n > 0).sum())
    rec = int(n.sum()) * HV * (2 * D + 1) * 4
    return working * HV * D * D * 4 * 2 + int(boundary_written) * HV * D * D * 4 + rec + 24 * wl.B
