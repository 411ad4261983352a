"""CPU (gloo) tests of the context-parallel plumbing: shard coverage, the
shard-partial -> all-gather -> log-sum-exp merge decomposition that
kessie_b200.context_parallel runs on NCCL, and failure handling when a rank
dies before the exchange.  No GPU is used: per-rank partials come from the
oracle, the exchange is a real 2- or 4-rank gloo all-gather."""

import os
import socket
import time

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from kessie_b200.context_parallel import shard_range
from oracle import fog_oracle as O


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def test_shard_ranges_cover_sequence_page_aligned():
    for N in (1, 15, 16, 1000, 1 << 20):
        for G in (1, 2, 3, 4, 8):
            spans = [shard_range(N, r, G, 16) for r in range(G)]
            assert spans[0][0] == 0 and spans[-1][1] == N
            for (a, b), (c, d) in zip(spans, spans[1:]):
                assert b == c and a <= b
            for a, b in spans:
                assert (a % 16 == 0 or a == N) and (b % 16 == 0 or b == N)


def _rank_main(rank, world, port, q, k, v, cs, out_q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    from datetime import timedelta
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=120))
    N = k.shape[1]
    a, b = shard_range(N, rank, world, 16)
    w = O.fog_weights_from_clear_start(N, cs, 0.5)
    _, (m, l, o) = O.fog_attention_rows(q, k[:, a:b], v[:, a:b], np.array([N - 1]), w[a:b],
                                        k_pos=np.arange(a, b), return_partials=True)
    trip = torch.from_numpy(O.partials_from_rows(m[:, 0], l[:, 0], o[:, 0]))          # [Hq, D+2]
    gathered = torch.empty((world * trip.shape[0],) + tuple(trip.shape[1:]), dtype=torch.float32)
    dist.all_gather_into_tensor(gathered, trip)            # concatenated along dim 0, as the CUDA path
    g = gathered.view((world,) + tuple(trip.shape)).numpy().astype(np.float64)
    D = q.shape[-1]
    ms, ls = g[..., D], g[..., D + 1]
    os_ = g[..., :D] * ls[..., None]
    merged = O.lse_combine(ms, ls, os_)
    out_q.put((rank, merged))
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_gloo_merge_equals_unsplit(world):
    """world ranks each attend over their page-aligned shard of 1000 keys
    (uneven at 4 ranks), all-gather the (m, l, o) partials and merge them;
    every rank gets the unsplit attention."""
    rng = np.random.default_rng(0)
    Hq, Hkv, D, N = 8, 2, 64, 1000
    q = rng.standard_normal((Hq, 1, D)); k = rng.standard_normal((Hkv, N, D)); v = rng.standard_normal((Hkv, N, D))
    cs = N - 256
    want = O.fog_attention_rows(q, k, v, np.array([N - 1]), O.fog_weights_from_clear_start(N, cs, 0.5))[:, 0]
    ctx = mp.get_context("spawn")
    out_q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, q, k, v, cs, out_q)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict(out_q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for r in range(world):
        np.testing.assert_allclose(res[r], want, atol=1e-6)


def _dying_rank(rank, world, port, out_q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    from datetime import timedelta
    # Rendezvous gets a long limit (spawned interpreters start slowly on a busy
    # host); the step's collectives run in a group with a short one.
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=120))
    step_group = dist.new_group(timeout=timedelta(seconds=4))
    if rank == 1:
        os._exit(3)                     # dies between steps, before the exchange
    t0 = time.time()
    try:
        x = torch.zeros(4)
        out = torch.empty(8)
        dist.all_gather_into_tensor(out, x, group=step_group)
        out_q.put(("no-error", time.time() - t0))
    except Exception as e:               # the survivor learns of it through the collective
        out_q.put(("error", time.time() - t0, type(e).__name__))


def test_rank_failure_surfaces_as_error_not_hang():
    ctx = mp.get_context("spawn")
    out_q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_dying_rank, args=(r, 2, port, out_q)) for r in range(2)]
    for p in procs:
        p.start()
    msg = out_q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert msg[0] == "error", msg
    assert msg[1] < 60
