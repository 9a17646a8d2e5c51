"""Multi-GPU partitioning of the hot path: one process per GPU, no data-path collective.

Every kernel of this package works on independent units -- (batch, kv head)
pairs for prefill/backward (the GQA group-sum never leaves a unit) and whole
sequences for decode -- so scaling out is partitioning, not communication:

* ``unit_slices`` splits the (batch, kv-head) units of a prefill/backward step;
* ``greedy_balance`` assigns decode sequences to ranks by total cached length;
* ``local_paged_problem`` builds a rank's own page pool and remapped block
  table for its sequences (page contents copied byte-for-byte, so each rank's
  paged decode is bit-identical to the single-GPU one for those sequences);
* ``split_batch`` / ``gather_batch`` run the tiny-LLaMA generation data
  parallel over ranks and gather the generated tokens with one all_gather
  (NCCL over NVLink on GPUs; gloo in the CPU tests) -- the only collective.

The reference has no multi-device code (it runs on one TPU core).
"""

from __future__ import annotations

from typing import Callable, List, Sequence, Tuple

import torch
import torch.distributed as dist


def unit_slices(batch: int, num_kv_heads: int, world: int, rank: int) -> List[Tuple[int, int]]:
    """The (batch, kv_head) units of ``rank`` out of ``batch * num_kv_heads``, contiguous and balanced."""
    n = batch * num_kv_heads
    lo = rank * n // world
    hi = (rank + 1) * n // world
    return [(u // num_kv_heads, u % num_kv_heads) for u in range(lo, hi)]


def greedy_balance(weights: Sequence[int], world: int) -> List[List[int]]:
    """Longest-processing-time assignment of items to ``world`` bins (returns item ids per bin).

    Used for decode: a sequence's cost is its cached length, so bins balance the
    bytes each GPU streams.  Deterministic (ties broken by item id, then bin id).
    """
    order = sorted(range(len(weights)), key=lambda i: (-int(weights[i]), i))
    load = [0] * world
    bins: List[List[int]] = [[] for _ in range(world)]
    for i in order:
        r = min(range(world), key=lambda j: (load[j], j))
        bins[r].append(i)
        load[r] += int(weights[i])
    return [sorted(b) for b in bins]


def local_paged_problem(q: torch.Tensor, k_pages: torch.Tensor, v_pages: torch.Tensor,
                        block_tables: torch.Tensor, context_lens: torch.Tensor,
                        seq_ids: Sequence[int]):
    """A self-contained paged-decode problem for the sequences ``seq_ids``.

    Returns ``(q_local, k_pool, v_pool, tables_local, lens_local)``: only the
    pages those sequences use (``ceil(len / page_size)`` leading table entries)
    are copied, renumbered 0..n-1 in first-use order; unused table entries are 0.
    """
    ps = k_pages.shape[2]
    ids = torch.as_tensor(list(seq_ids), dtype=torch.long)
    tables = block_tables.to("cpu", torch.long)[ids]
    lens = context_lens.to("cpu", torch.long)[ids]
    remap: dict = {}
    new_tables = torch.zeros_like(tables)
    for r in range(tables.shape[0]):
        n = (int(lens[r]) + ps - 1) // ps
        for p in range(n):
            phys = int(tables[r, p])
            if phys not in remap:
                remap[phys] = len(remap)
            new_tables[r, p] = remap[phys]
    phys_ids = torch.tensor(sorted(remap, key=remap.get) or [0], dtype=torch.long)
    dev = k_pages.device
    k_pool = k_pages.index_select(0, phys_ids.to(dev))
    v_pool = v_pages.index_select(0, phys_ids.to(dev))
    return (q.index_select(0, ids.to(q.device)), k_pool, v_pool,
            new_tables.to(device=block_tables.device, dtype=torch.int32),
            lens.to(device=context_lens.device, dtype=torch.int32))


def split_batch(n: int, world: int, rank: int) -> slice:
    """Contiguous batch slice of ``rank`` (sizes differ by at most one)."""
    return slice(rank * n // world, (rank + 1) * n // world)


def gather_batch(local: torch.Tensor, n: int, world: int, group=None) -> torch.Tensor:
    """All-gather per-rank batch slices (``split_batch`` layout) into the full ``[n, ...]`` tensor."""
    if world == 1:
        return local
    rows = max((r + 1) * n // world - r * n // world for r in range(world))
    pad = torch.zeros((rows,) + tuple(local.shape[1:]), dtype=local.dtype, device=local.device)
    pad[: local.shape[0]] = local
    parts = [torch.empty_like(pad) for _ in range(world)]
    dist.all_gather(parts, pad, group=group)
    out = [parts[r][: (r + 1) * n // world - r * n // world] for r in range(world)]
    return torch.cat(out, dim=0)


def generate_data_parallel(generate_fn: Callable[[torch.Tensor], torch.Tensor], prompts: torch.Tensor,
                           world: int, rank: int, group=None) -> torch.Tensor:
    """Runs ``generate_fn`` (e.g. ``lambda p: generate_cached(params, p, n, cfg)``) on this
    rank's prompts and gathers every rank's tokens: the multi-GPU model path."""
    sl = split_batch(prompts.shape[0], world, rank)
    local = generate_fn(prompts[sl])
    return gather_batch(local, prompts.shape[0], world, group)
