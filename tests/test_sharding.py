"""Multi-process partitioning logic on CPU ranks (gloo, world_size 2).

The kernels need no exchange; what crosses ranks is the batch split of the
model path and its single all_gather of generated tokens.  These tests run two
gloo processes on 127.0.0.1 and check the gather (uneven batches), the unit
and sequence partitions, and the per-rank paged problems against the oracle's
block-table gather -- with plain tensor ops standing in for the GPU kernels.
"""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from pallas_flash import sharding
from oracle import attention_oracle as orc


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, n, queue):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        prompts = torch.arange(n * 3).reshape(n, 3)
        # stand-in for generate_cached: append (row sum, rank) per prompt
        fn = lambda p: torch.cat([p, p.sum(1, keepdim=True), torch.full((p.shape[0], 1), rank)], 1)  # noqa: E731
        out = sharding.generate_data_parallel(fn, prompts, world, rank)
        queue.put((rank, out.numpy()))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("n", [5, 16])
def test_data_parallel_generation_gather_gloo(n):
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, n, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    prompts = np.arange(n * 3).reshape(n, 3)
    owner = np.array([0] * (n // 2) + [1] * (n - n // 2))
    want = np.concatenate([prompts, prompts.sum(1, keepdims=True), owner[:, None]], 1)
    for r in range(world):
        np.testing.assert_array_equal(results[r], want)


def test_unit_slices_cover_every_unit_once():
    for world in (1, 2, 3, 8):
        units = [u for r in range(world) for u in sharding.unit_slices(4, 8, world, r)]
        assert sorted(units) == [(b, h) for b in range(4) for h in range(8)]
        sizes = [len(sharding.unit_slices(4, 8, world, r)) for r in range(world)]
        assert max(sizes) - min(sizes) <= 1


def test_greedy_balance_is_a_partition_and_balanced():
    rng = np.random.default_rng(0)
    lens = rng.integers(512, 32769, size=256)
    bins = sharding.greedy_balance(lens, 8)
    assert sorted(i for b in bins for i in b) == list(range(256))
    loads = [int(lens[b].sum()) for b in bins]
    assert max(loads) - min(loads) <= lens.max()


def test_local_paged_problem_preserves_every_sequence_bytes():
    rng = np.random.default_rng(1)
    ps, hkv, d, B = 4, 2, 8, 5
    lens = np.array([1, 9, 16, 3, 12])
    pps = 4
    pool = 30
    kp = torch.tensor(rng.standard_normal((pool, hkv, ps, d)), dtype=torch.float32)
    vp = torch.tensor(rng.standard_normal((pool, hkv, ps, d)), dtype=torch.float32)
    tables = np.stack([rng.choice(pool, size=pps, replace=False) for _ in range(B)]).astype(np.int32)
    tables[1, :] = tables[2, :]  # shared prefix pages
    q = torch.randn((B, 4, 1, d))
    for seqs in ([0, 2, 4], [1, 3], [1, 2]):
        ql, kl, vl, tl, ll = sharding.local_paged_problem(q, kp, vp, torch.tensor(tables), torch.tensor(lens), seqs)
        assert torch.equal(ql, q[seqs])
        for j, b in enumerate(seqs):
            L = int(lens[b])
            want_k = orc.gather_contiguous(kp.numpy(), tables[b], pps, L)
            got_k = orc.gather_contiguous(kl.numpy(), tl[j].numpy(), (L + ps - 1) // ps, L)
            np.testing.assert_array_equal(got_k, want_k)
            want_v = orc.gather_contiguous(vp.numpy(), tables[b], pps, L)
            got_v = orc.gather_contiguous(vl.numpy(), tl[j].numpy(), (L + ps - 1) // ps, L)
            np.testing.assert_array_equal(got_v, want_v)
        assert kl.shape[0] <= sum((int(lens[b]) + ps - 1) // ps for b in seqs)
