"""CPU, world size 2 over gloo: the KV-head shard plan and the output
all-gather reproduce the unsharded decode (oracle per rank)."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, result):
    import oracle
    from sf37_b200 import synth
    from sf37_b200.shard import ShardPlan, gather_outputs
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    plan = ShardPlan(world, rank)
    layers, cap, pos = 3, 300, 299
    outs = []
    for l in range(layers):
        k = torch.from_numpy(synth.normal(10 + l, (cap, 1024)))
        v = torch.from_numpy(synth.normal(20 + l, (cap, 1024)))
        q = torch.from_numpy(synth.normal(30 + l, (64, 128)))
        g = torch.from_numpy(synth.normal(40 + l, (64,)))
        a, b = plan.q_range
        outs.append(torch.from_numpy(oracle.attention_decode_at(
            plan.slice_q(q).numpy(), plan.slice_rows(k).contiguous().numpy(),
            plan.slice_rows(v).contiguous().numpy(), g[a:b].numpy(), pos, cap, plan.q_local,
            plan.kv_local, 128, sliding=l == 1, window=128)))
    full = gather_outputs(torch.stack(outs), plan)
    if rank == 0:
        result.put(full.numpy())
    dist.barrier()
    dist.destroy_process_group()


def test_plan_slices():
    from sf37_b200.shard import ShardPlan
    p = ShardPlan(4, 2)
    assert p.kv_range == (4, 6) and p.q_range == (32, 48)
    with pytest.raises(ValueError):
        ShardPlan(3, 0)


def test_sharded_decode_equals_unsharded_gloo():
    import oracle
    from sf37_b200 import synth
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    ps = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    got = q.get(timeout=120)
    for p in ps:
        p.join(timeout=60)
        assert p.exitcode == 0
    for l in range(3):
        k = synth.normal(10 + l, (300, 1024))
        v = synth.normal(20 + l, (300, 1024))
        want = oracle.attention_decode_at(synth.normal(30 + l, (64, 128)), k, v, synth.normal(40 + l, (64,)),
                                          299, 300, 64, 8, 128, sliding=l == 1, window=128)
        np.testing.assert_allclose(got[l], want, atol=1e-6, rtol=1e-5)
