"""The bench's multi-rank host logic on CPU: two gloo ranks in spawned
processes (the scaling run launches one process per GPU the same way, over
NCCL). Replicas only: no data-path collective, so what needs checking is
- the reductions the bench takes over ranks (max of times, sum of work),
  here on host tensors;
- each rank's share of the config-4 requests: rank, rank + N, ...,
  disjoint, and together all of them;
- the batched box's slot scheduling on each rank's share, against a
  stand-in batch that records its calls: every request is prefilled once
  into a free slot and advanced by exactly its patches, the slots refilling
  as requests end.
"""

import os
import socket
import sys
from pathlib import Path
from types import SimpleNamespace

import pytest

ROOT = Path(__file__).resolve().parent.parent


class RecordingBatch:
    """GeneratorBatch's Prefill/Step interface, recording the schedule."""

    def __init__(self, slots):
        self.slots = slots
        self.owner = [None] * slots
        self.prefills = []      # (slot, prompt rows)
        self.patches = {}       # request -> patches produced
        self.current = [None] * slots
        self.next_request = None

    def Prefill(self, slot, tokens, text_mask, audio_mask, feats):
        assert 0 <= slot < self.slots
        assert self.current[slot] is None or self.patches[self.current[slot]] > 0
        self.prefills.append((slot, len(tokens)))
        request = self.next_request.pop(0)
        self.current[slot] = request
        self.patches[request] = 0

    def Step(self, noise, active, timesteps, cfg):
        assert noise.shape[0] == self.slots and len(active) == self.slots
        assert timesteps == 10 and cfg == 2.0
        for s in range(self.slots):
            if active[s]:
                assert self.current[s] is not None
                self.patches[self.current[s]] += 1


def _rank(rank, world, port, out_dir):
    import numpy as np
    import torch.distributed as dist

    sys.path.insert(0, str(ROOT))
    import bench

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        assert bench.max_over_ranks(world, 1.5 + rank) == 1.5 + world - 1
        assert bench.sum_over_ranks(world, 1.0 + rank) == sum(1.0 + r for r in range(world))
        share = bench.box_share(rank, world)
        assert share == list(range(rank, bench.BOX_REQUESTS, world))
        # Every rank's share, gathered: disjoint, and all the requests.
        gathered = [None] * world
        dist.all_gather_object(gathered, share)
        flat = [r for s in gathered for r in s]
        assert len(flat) == len(set(flat)) == bench.BOX_REQUESTS
        # The batched box's schedule on this rank's share.
        c = SimpleNamespace(vocab=64, patch_size=4, feat_dim=64)
        slots, patches = 4, 3
        batch = RecordingBatch(slots)
        batch.next_request = list(share)
        steps = bench.drive_box(batch, c, share, slots, patches)
        assert sorted(batch.patches) == sorted(share)
        assert all(n == patches for n in batch.patches.values())
        assert len(batch.prefills) == len(share)
        assert steps == patches * -(-len(share) // slots)
        # Prompts are the requests' own seeded prompts (16..128 tokens + 1).
        assert all(17 <= rows <= 129 for _, rows in batch.prefills)
        np.save(Path(out_dir) / f"rank{rank}.npy", np.array(share))
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_two_gloo_ranks(tmp_path):
    import numpy as np
    import torch.multiprocessing as mp

    world = 2
    mp.spawn(_rank, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True)
    shares = [np.load(tmp_path / f"rank{r}.npy").tolist() for r in range(world)]
    assert shares[0][:3] == [0, 2, 4] and shares[1][:3] == [1, 3, 5]


def test_one_rank_needs_no_process_group():
    sys.path.insert(0, str(ROOT))
    import bench

    assert bench.max_over_ranks(1, 3.0) == 3.0 and bench.sum_over_ranks(1, 2.0) == 2.0
    assert bench.box_share(0, 1) == list(range(bench.BOX_REQUESTS))
    assert bench.box_share(7, 8) == list(range(7, bench.BOX_REQUESTS, 8))
