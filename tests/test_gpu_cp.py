"""Multi-GPU parity of the context-parallel decode, both exchanges (NVLink
peer stores from the decode kernel + bounded-wait combine; NCCL all-gather +
LSE merge kernel): 2, 4 or 8 ranks, each holding a contiguous position shard of every
sequence, must reproduce the single-GPU decode over the whole cache.
Skipped with fewer GPUs than ranks."""

import os
import queue
import socket
import time

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank(rank, world, port, out_q):
    import torch.distributed as dist
    from datetime import timedelta
    from kessie_b200 import ops
    from kessie_b200.context_parallel import ContextParallelFogDecode, shard_range
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60), device_id=dev)
    B, Hq, Hkv, D, ps = 2, 16, 4, 128, 16
    N = 4096 + 48                                       # ragged: not a multiple of the shard size
    g = torch.Generator().manual_seed(7)
    P = B * ((N + ps - 1) // ps)
    kv_full = torch.randn(P, ps, 2, Hkv, D, generator=g).to(torch.bfloat16)
    bt_full = torch.randperm(P, generator=g).to(torch.int32).view(B, -1)
    q = torch.randn(B, Hq, D, generator=g).to(torch.bfloat16).to(dev)
    a, b = shard_range(N, rank, world, ps)
    pg0, pg1 = a // ps, (b + ps - 1) // ps
    bt_loc = bt_full[:, pg0:pg1].contiguous().to(dev)
    kv = kv_full.to(dev)                                 # all pages resident; the shard only references its own
    lens = torch.full((B,), b - a, dtype=torch.int32, device=dev)
    off = torch.full((B,), a, dtype=torch.int32, device=dev)
    qpos = torch.full((B,), N - 1, dtype=torch.int32, device=dev)
    cs = torch.full((B,), N - 512, dtype=torch.int32, device=dev)
    outs = {}
    for exchange in ("p2p", "nccl"):
        dec = ContextParallelFogDecode(B, Hq, D, torch.bfloat16, dev, num_kv_heads=Hkv, exchange=exchange)
        for _ in range(3):              # several steps: both slots of the exchange buffers
            out = dec(q, kv[:, :, 0], kv[:, :, 1], bt_loc, lens, off, qpos, cs, 0.5, 0, None, (pg1 - pg0) * ps)
        outs[exchange] = out.clone()
        torch.cuda.synchronize()
        dec.close()
    status = ops.read_device_status()
    if rank == 0:
        full = ops.paged_fog_decode(q, kv[:, :, 0], kv[:, :, 1], bt_full.to(dev),
                                    torch.full((B,), N, dtype=torch.int32, device=dev),
                                    clear_start=cs, fog_alpha=0.5)
        torch.cuda.synchronize()
        out_q.put((outs["p2p"].float().cpu().numpy(), outs["nccl"].float().cpu().numpy(),
                   full.float().cpu().numpy(), status))
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4, 8])
def test_context_parallel_gpus_match_single_gpu(world):
    if not torch.cuda.is_available() or torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    ctx = mp.get_context("spawn")
    out_q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, world, port, out_q)) for r in range(world)]
    for p in procs:
        p.start()
    deadline = time.time() + 300
    res = None
    while res is None:
        try:
            res = out_q.get(timeout=2)
        except queue.Empty:
            dead = [p.exitcode for p in procs if p.exitcode not in (None, 0)]
            if dead or time.time() > deadline:
                for p in procs:
                    if p.is_alive():
                        p.kill()
                pytest.fail(f"rank process failed (exit codes {[p.exitcode for p in procs]})")
    got, got_nccl, want, status = res
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert status == 0
    np.testing.assert_allclose(got, want, atol=2e-2, rtol=1e-2)
    np.testing.assert_allclose(got_nccl, want, atol=2e-2, rtol=1e-2)
    assert np.isfinite(got).all()
