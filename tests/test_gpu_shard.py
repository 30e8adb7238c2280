"""GPU, 2 ranks over NCCL (needs >= 2 GPUs): KV-head-sharded decode through
the C ABI plus the output gather (NCCL all-gather, or the decode kernels'
own stores into peer memory) equals the oracle on the full heads."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                                 reason="needs 2 GPUs")]


def _worker(rank, world, port, result, mode="nccl"):
    import torch.distributed as dist
    from sf37_b200 import kv, synth
    from sf37_b200._lib import lib
    from sf37_b200.shard import PeerGather, ShardPlan, gather_outputs
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world)
    plan = ShardPlan(world, rank)
    layers, cap, pos = 4, 5000, 4999
    descs, outs = [], torch.empty(layers, plan.q_local, 128, device="cuda")
    for l in range(layers):
        k = torch.from_numpy(synth.normal(10 + l, (cap, 1024))).cuda()
        v = torch.from_numpy(synth.normal(20 + l, (cap, 1024))).cuda()
        q = torch.from_numpy(synth.normal(30 + l, (64, 128))).cuda()
        a, b = plan.q_range
        descs.append(dict(k_cache=plan.slice_rows(k).half().contiguous(),
                          v_cache=plan.slice_rows(v).half().contiguous(), cap=cap, pos=pos,
                          q=plan.slice_q(q).contiguous(), out=outs[l]))
    if mode == "nccl":
        kv.decode(descs, plan.q_local, plan.kv_local, 128, kv.F16)
        full = gather_outputs(outs, plan)
        got = [full.cpu().numpy()]
    else:
        # three steps at positions 4997..4999 exercise both buffer halves
        pg = PeerGather(plan, layers)
        got = []
        for p in (4997, 4998, 4999):
            for d in descs:
                d["pos"] = p
            pg.step(descs, kv.F16)
            got.append(pg.heads().cpu().numpy())
        assert lib().sf37kv_device_error(1) == 0
        dist.barrier()
        torch.cuda.synchronize()
        pg.close()
    if rank == 0:
        result.put(got)
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("mode", ["nccl", "peer"])
def test_sharded_decode_2gpu(mode):
    import oracle
    from sf37_b200 import synth
    from tests.helpers import assert_close
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    ps = [ctx.Process(target=_worker, args=(r, 2, port, q, mode)) for r in range(2)]
    for p in ps:
        p.start()
    got = q.get(timeout=300)
    for p in ps:
        p.join(timeout=120)
        assert p.exitcode == 0
    positions = [4999] if mode == "nccl" else [4997, 4998, 4999]
    assert len(got) == len(positions)
    for l in range(4):
        k = oracle.f16_bits_to_f32(oracle.f32_to_f16_bits(synth.normal(10 + l, (5000, 1024))))
        v = oracle.f16_bits_to_f32(oracle.f32_to_f16_bits(synth.normal(20 + l, (5000, 1024))))
        for step, pos in enumerate(positions):
            want = oracle.attention_decode_at(synth.normal(30 + l, (64, 128)), k, v, None, pos, 5000, 64, 8, 128)
            assert_close(got[step][l], want)


def _oproj_worker(rank, world, port, result):
    import torch.distributed as dist
    from sf37_b200 import _lib, synth
    from sf37_b200.shard import PeerReduce
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world)
    layers, in_dim, out_dim = 3, 8192, 4096
    local = in_dim // world
    pr = PeerReduce(world, rank, layers, out_dim)
    got = []
    for step in range(3):  # both buffer halves
        ws, xs = [], []
        for l in range(layers):
            w = torch.from_numpy(synth.q8_0_weights(10 * step + l, out_dim, in_dim)).cuda()
            x = torch.from_numpy(synth.normal(100 * step + l, (in_dim,)) * (l + 1)).cuda()
            off, stride = PeerReduce.weight_slice(w, world, rank)
            ws.append((w, off, stride))
            xs.append(x[rank * local:(rank + 1) * local].contiguous())
        arr = (_lib.OprojLayer * layers)(*[_lib.OprojLayer(w.data_ptr() + off, xs[l].data_ptr(), 0)
                                          for l, (w, off, stride) in enumerate(ws)])
        out = torch.empty(layers, out_dim, device="cuda")
        pr.step(arr, local, ws[0][2], out)
        got.append(out.cpu().numpy())
    assert _lib.lib().sf37kv_device_error(1) == 0
    dist.barrier()
    torch.cuda.synchronize()
    pr.close()
    result.put((rank, got))
    dist.barrier()
    dist.destroy_process_group()


def test_row_parallel_oproj_2gpu():
    import oracle
    from sf37_b200 import synth
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    ps = [ctx.Process(target=_oproj_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = dict(q.get(timeout=300) for _ in range(2))
    for p in ps:
        p.join(timeout=120)
        assert p.exitcode == 0
    for step in range(3):
        assert np.array_equal(res[0][step], res[1][step])  # same bits on every rank
        for l in range(3):
            w = synth.q8_0_weights(10 * step + l, 4096, 8192)
            x = synth.normal(100 * step + l, (8192,)) * (l + 1)
            want = oracle.q8_0_matvec(w, x, 4096)
            bound = 4e-6 * oracle.q8_0_abs_terms(w, x, 4096) + 1e-30
            assert np.all(np.abs(res[0][step][l] - want) <= bound)
