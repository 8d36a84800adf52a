"""Sharded compression across the GPUs of one node (one process per GPU).

Once the keep set is known every (layer, KV head) row block compresses
independently.  Two plans:

* ``heads`` (when the world size divides the KV heads and leaves every rank at
  least ``MIN_HEADS_PER_RANK`` of them): rank r owns KV heads [r*h/N, (r+1)*h/N)
  of every layer -- the same slice it scores -- so every rank moves exactly 1/N of
  the cache, protected layers included.
* ``layers`` (otherwise): ranks own whole layers, balanced by cost
  (longest-processing-time greedy).  A compress tile covers up to 8 heads of one
  token, which share that token's RoPE row; with fewer heads per layer on a rank
  the key tiles read one RoPE row per vector and the kernel slows down (config 4
  at 8 ranks: 0.23 of the HBM peak with one head per rank against 0.33 with all
  eight), which costs more than the whole-layer plan's imbalance (10 against an
  even 9.5 quantized layers per rank at 8 ranks).

The only cross-GPU traffic:

1. Keep set.  Under ``NexusQuantEvict.compress`` semantics layer 0's importance
   decides every layer (nexusquant/pipeline.py:1066-1098).  Each rank scores a
   contiguous block of layer 0's KV heads and the per-head column sums
   ``[b, h_local, T]`` are all-gathered; every rank then reduces all heads in
   head order and selects, so the keep sets are identical without an index
   broadcast.
2. Compressed-cache index.  Each rank's per-layer compressed byte sizes are
   all-gathered, giving every rank the global layer -> (owner, offset) table.

The compressed payload stays on its owner GPU.  Everything here is plain
``torch.distributed`` over whatever backend the group uses (NCCL on the GPUs,
gloo for the CPU tests).
"""
from __future__ import annotations

import math
import time
from dataclasses import dataclass
from typing import Iterable, List, Optional, Sequence, Tuple

import torch
import torch.distributed as dist

# Cost of an fp16-kept (boundary-protected) layer relative to a compressed one, from the
# kernels' measured times on B200: the kept-row gather of K and V of a protected layer takes
# ~53 us against ~95 us for compressing a layer's K and V (config 4, 26240 kept rows).
PROTECTED_LAYER_COST = 0.56


def protected_layers(n_layers: int, protect_boundary: int) -> set:
    """First and last ``protect_boundary`` layers (nexusquant/pipeline.py:1110-1120)."""
    if protect_boundary <= 0:
        return set()
    return set(range(min(protect_boundary, n_layers))) | set(range(max(0, n_layers - protect_boundary), n_layers))


def assign_layers(n_layers: int, protected: Iterable[int], world: int,
                  protected_cost: float = PROTECTED_LAYER_COST) -> List[List[int]]:
    """Cost-balanced layer -> rank assignment (longest-processing-time greedy, ties to the
    lower rank and lower layer index).  Deterministic: every rank computes the same plan."""
    if world < 1:
        raise ValueError("world must be >= 1")
    prot = set(protected)
    cost = {l: (protected_cost if l in prot else 1.0) for l in range(n_layers)}
    order = sorted(range(n_layers), key=lambda l: (-cost[l], l))
    load = [0.0] * world
    owned: List[List[int]] = [[] for _ in range(world)]
    for l in order:
        r = min(range(world), key=lambda i: (load[i], i))
        owned[r].append(l)
        load[r] += cost[l]
    return [sorted(o) for o in owned]


def head_block(heads: int, rank: int, world: int) -> Tuple[int, int, int]:
    """(head_begin, head_end, heads_per_rank): rank r scores heads [r*per, (r+1)*per) clipped to h."""
    per = math.ceil(heads / world)
    return min(heads, rank * per), min(heads, (rank + 1) * per), per


@dataclass(frozen=True)
class ShardPlan:
    rank: int
    world: int
    n_layers: int
    heads: int
    layers: Tuple[int, ...]       # all layers this rank holds rows of
    quantized: Tuple[int, ...]    # those that are compressed
    protected: Tuple[int, ...]    # those kept at fp16
    head_begin: int               # KV heads this rank scores
    head_end: int
    heads_per_rank: int
    mode: str = "layers"          # "heads": [head_begin, head_end) of every layer; "layers": whole layers

    @property
    def scores_heads(self) -> bool:
        return self.head_end > self.head_begin

    @property
    def layer_heads(self) -> Tuple[int, int]:
        """KV heads of each owned layer that this rank compresses."""
        return (self.head_begin, self.head_end) if self.mode == "heads" else (0, self.heads)


# Fewest KV heads per layer a rank keeps under the ``heads`` plan chosen by ``mode="auto"``:
# the compress kernel's tiles group up to 8 heads of a token around one RoPE row.
MIN_HEADS_PER_RANK = 8


def plan_mode(heads: int, world: int, mode: str = "auto") -> str:
    if mode == "auto":
        if world == 1:
            return "heads"
        return "heads" if heads % world == 0 and heads // world >= MIN_HEADS_PER_RANK else "layers"
    if mode not in ("heads", "layers"):
        raise ValueError(f"mode must be 'auto', 'heads' or 'layers', got {mode!r}")
    if mode == "heads" and heads % world:
        raise ValueError(f"mode='heads' needs the world size ({world}) to divide the KV heads ({heads})")
    return mode


def make_plan(n_layers: int, heads: int, protect_boundary: int, rank: int, world: int,
              mode: str = "auto") -> ShardPlan:
    if not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world {world}")
    m = plan_mode(heads, world, mode)
    prot = protected_layers(n_layers, protect_boundary)
    owned = list(range(n_layers)) if m == "heads" else assign_layers(n_layers, prot, world)[rank]
    h0, h1, per = head_block(heads, rank, world)
    return ShardPlan(rank, world, n_layers, heads, tuple(owned), tuple(l for l in owned if l not in prot),
                     tuple(l for l in owned if l in prot), h0, h1, per, m)


def gather_head_scores(per_head: torch.Tensor, plan: ShardPlan, group=None,
                       gathered: Optional[torch.Tensor] = None) -> torch.Tensor:
    """All-gather this rank's per-head column sums ``[b, h_local, T]`` into ``[b, heads, T]``
    in head order (identical on every rank).  ``gathered`` is an optional reusable buffer of
    ``world * b * heads_per_rank * T`` fp32 elements on the group's device."""
    b, hl, T = per_head.shape
    if hl != plan.head_end - plan.head_begin:
        raise ValueError(f"per_head has {hl} heads, plan scores {plan.head_end - plan.head_begin}")
    if plan.world == 1:
        return per_head
    per = plan.heads_per_rank
    buf = per_head
    if hl != per:  # the last rank(s) may own fewer heads: pad to the common block
        buf = torch.zeros((b, per, T), dtype=per_head.dtype, device=per_head.device)
        buf[:, :hl] = per_head
    if gathered is None:
        gathered = torch.empty((plan.world * b * per, T), dtype=per_head.dtype, device=per_head.device)
    dist.all_gather_into_tensor(gathered, buf.contiguous().reshape(b * per, T), group=group)
    return gathered.reshape(plan.world, b, per, T).transpose(0, 1).reshape(b, plan.world * per, T)[:, :plan.heads]


def local_layer_sizes(plan: ShardPlan, compressed_bytes: Sequence[int], protected_bytes: Sequence[int],
                      device=None) -> torch.Tensor:
    """int64 [n_layers]: this rank's byte size of each layer it owns (0 elsewhere)."""
    sizes = [0] * plan.n_layers
    for l, n in zip(plan.quantized, compressed_bytes):
        sizes[l] = int(n)
    for l, n in zip(plan.protected, protected_bytes):
        sizes[l] = int(n)
    return torch.tensor(sizes, dtype=torch.int64, device=device)


def gather_layer_index(sizes: torch.Tensor, plan: ShardPlan, group=None,
                       sizes_all: Optional[torch.Tensor] = None, async_op: bool = False):
    """All-gather per-layer sizes -> int64 [world, n_layers] (row r = rank r's sizes).
    async_op=True returns (table, work): with fixed-capacity outputs the sizes are known before
    the layers are compressed, so the exchange can run while they are; call work.wait()
    (work is None on one rank) before reading the table."""
    if plan.world == 1:
        table = sizes.reshape(1, -1)
        return (table, None) if async_op else table
    if sizes_all is None:
        sizes_all = torch.empty((plan.world * sizes.numel(),), dtype=torch.int64, device=sizes.device)
    work = dist.all_gather_into_tensor(sizes_all.view(-1), sizes.view(-1), group=group, async_op=async_op)
    table = sizes_all.view(plan.world, -1)
    return (table, work) if async_op else table


def layer_owners(assignment: Sequence[Sequence[int]], n_layers: int) -> List[int]:
    """Owner rank of each layer from an ``assign_layers`` result."""
    owner = [-1] * n_layers
    for r, ls in enumerate(assignment):
        for l in ls:
            if owner[l] != -1:
                raise ValueError(f"layer {l} assigned twice")
            owner[l] = r
    if -1 in owner:
        raise ValueError(f"layer {owner.index(-1)} has no owner")
    return owner


def unit_table(sizes_all: torch.Tensor) -> List[Tuple[int, int, int, int]]:
    """Global index for either plan: (layer, rank, byte offset, size) of every non-empty
    (layer, rank) block, in layer-major then rank order -- the concatenation order of the
    compressed cache (a layer's head slices follow each other in head order)."""
    s = sizes_all.cpu()
    world, n_layers = s.shape
    out, off = [], 0
    for l in range(n_layers):
        for r in range(world):
            n = int(s[r, l])
            if n:
                out.append((l, r, off, n))
                off += n
    return out


def layer_table(sizes_all: torch.Tensor, owners: Sequence[int]) -> List[Tuple[int, int, int]]:
    """Global index of the compressed cache: per layer (owner rank, byte offset in the
    concatenation of all layers in layer order, size)."""
    s = sizes_all.cpu()
    table, off = [], 0
    for l, r in enumerate(owners):
        n = int(s[r, l])
        table.append((r, off, n))
        off += n
    return table


# ------------------------------------------------------------------ failure handling
class RankFailure(RuntimeError):
    """A peer rank did not reach a step in time, or sent an invalid message."""


def step_checkpoint(store, rank: int, world: int, step: int, timeout: float = 30.0) -> None:
    """Host heartbeat before a step's collectives.  Every rank posts ``step`` to the store and
    waits (bounded) for all others, so a rank that left between steps is named before any
    collective of the next step is launched -- the survivors raise RankFailure instead of
    blocking in NCCL.  ``store`` is the process group's store (or any c10d Store)."""
    key = "nq/step/{}/{}".format
    deadline = time.monotonic() + timeout
    missing = [r for r in range(world) if r != rank]
    try:
        store.set(key(step, rank), b"1")
        while missing:
            missing = [r for r in missing if not store.check([key(step, r)])]
            if not missing:
                return
            if time.monotonic() > deadline:
                raise RankFailure(f"rank(s) {missing} did not reach step {step} within {timeout:g} s")
            time.sleep(0.005)
    except RankFailure:
        raise
    except RuntimeError as e:
        # the store itself went away: the rank hosting it (rank 0 for a TCPStore) has left,
        # which is a peer failure like any other
        raise RankFailure(f"rank(s) {missing} did not reach step {step}: store unreachable "
                          f"({type(e).__name__})") from e


def validate_index(sizes_all: torch.Tensor, n_layers: int, heads: int, protect_boundary: int,
                   expected=None) -> None:
    """Check a gathered size table before using it: every rank's row must be non-negative and
    non-zero exactly at the layers its plan holds, and equal ``expected(rank, layer)`` where that
    is given (fixed-capacity outputs make the sizes known).  Raises RankFailure naming the rank."""
    s = sizes_all.detach().cpu().reshape(-1, n_layers)
    world = s.shape[0]
    for r in range(world):
        plan = make_plan(n_layers, heads, protect_boundary, r, world)
        held = set(plan.layers)
        for l in range(n_layers):
            n = int(s[r, l])
            if n < 0 or (n > 0) != (l in held):
                raise RankFailure(f"rank {r} reported {n} bytes for layer {l}, which it "
                                  f"{'holds' if l in held else 'does not hold'}")
            if expected is not None and l in held and n != int(expected(r, l)):
                raise RankFailure(f"rank {r} reported {n} bytes for layer {l}, expected {int(expected(r, l))}")

