"""Series-group sharding on the GPU (configs[4] shapes).

A global batch is split into shards of whole groups
(sharding.partition_groups); each shard's forecasts must be bit-identical to
the same series' forecasts in the unsharded forward (the forward has no
cross-series coupling outside a group and a fixed reduction order), and
gather_forecasts must put them back in the global order.  The multi-rank
collective itself is covered on CPU ranks (gloo) in test_host_cpu.py; here it
runs as a one-rank NCCL group.
"""

import pytest
import torch
import torch.distributed as dist

from cutechronos_b200.model import CuteChronos2Config, CuteChronos2Model
from cutechronos_b200.sharding import gather_forecasts, partition_groups
from cutechronos_b200.workloads import config4, seeded_init_

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.fixture(scope="module")
def model():
    return seeded_init_(CuteChronos2Model(CuteChronos2Config()), seed=0).to(DEV, torch.bfloat16).eval()


@pytest.mark.parametrize("grouped", [False, True])
@pytest.mark.parametrize("world", [2, 3, 8])
def test_shards_reassemble_bit_identical(model, world, grouped):
    w = config4(B=1024)
    B = w.context.shape[0]
    gid = torch.arange(B) // 8 if grouped else None
    ctx = w.context.to(DEV)
    full = model(ctx, num_output_patches=4, group_ids=gid)
    shards = partition_groups(gid, B, world)
    assert sorted(torch.cat(shards).tolist()) == list(range(B))
    if gid is not None:  # no group split across shards
        owner = {}
        for r, s in enumerate(shards):
            for g in gid[s].tolist():
                assert owner.setdefault(g, r) == r
    out = torch.empty_like(full)
    for s in shards:
        y = model(ctx[s.to(DEV)], num_output_patches=4, group_ids=gid[s] if gid is not None else None)
        out[s.to(DEV)] = y
    assert torch.equal(out, full)


def test_gather_forecasts_one_rank_nccl(model, tmp_path):
    w = config4(B=256)
    ctx = w.context.to(DEV)
    full = model(ctx, num_output_patches=4)
    store = dist.FileStore(str(tmp_path / "store"), 1)
    dist.init_process_group("nccl", store=store, rank=0, world_size=1, device_id=torch.device(DEV, 0))
    try:
        shards = partition_groups(None, 256, 1)
        got = gather_forecasts(model(ctx[shards[0].to(DEV)], num_output_patches=4), shards)
    finally:
        dist.destroy_process_group()
    assert torch.equal(got, full)
