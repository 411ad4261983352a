"""GPU tests of the context-parallel exchange on ONE GPU.  World-size-W
ranks are emulated in one process: every "rank" owns an exchange buffer
(kessie_cp_exchange_alloc) on the same device, runs the decode phase over
its position shard, and only after all of them were launched (stream
order) runs its combine phase.  No kernel ever waits for another launch that
has not already completed, so the emulation cannot deadlock; the real
multi-GPU path is tests/test_gpu_cp.py."""

import ctypes

import numpy as np
import pytest
import torch

from oracle import fog_oracle as O
from tests.kessie_testutil import ROUND, TOL, make_paged, rnd, to_dev, to_np

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    yield


class _Buffers:
    def __init__(self, world, B, Hq, Hkv, D):
        from kessie_b200 import _lib
        self.shape = (B, Hq, Hkv, D)
        self.lib = _lib.load()
        n = self.lib.kessie_cp_exchange_bytes(world, B, Hq, Hkv, D)
        assert n > 0
        self.ptrs = []
        for _ in range(world):
            p = ctypes.c_void_p()
            h = (ctypes.c_uint8 * 64)()
            _lib.check(self.lib.kessie_cp_exchange_alloc(n, ctypes.byref(p), h), "alloc")
            self.ptrs.append(p.value)
        self.arr = (ctypes.c_void_p * world)(*self.ptrs)

    def free(self):
        for p in self.ptrs:
            self.lib.kessie_cp_exchange_free(p)


class _View:
    """What ops.paged_fog_decode_cp needs from an exchange (ptrs, rank, world)."""
    def __init__(self, bufs, rank, world):
        self.ptrs, self.rank, self.world, self.shape = bufs.arr, rank, world, bufs.shape


def _shards(N, world, ps):
    from kessie_b200.context_parallel import shard_range
    return [shard_range(N, r, world, ps) for r in range(world)]


@pytest.mark.parametrize("world,window", [(2, 0), (3, 0), (8, 0), (4, 700)])
def test_cp_p2p_emulated_ranks_match_full_decode(world, window):
    from kessie_b200 import ops
    B, Hq, Hkv, D, ps = 3, 16, 4, 128, 16
    N = 6000 + 8 * world                    # ragged shard ends
    pages = (N + ps - 1) // ps
    kvn, kv = make_paged(70 + world, B * pages, ps, Hkv, D, "bf16")
    bt_full = np.random.default_rng(71).permutation(B * pages).astype(np.int32).reshape(B, pages)
    bufs = _Buffers(world, B, Hq, Hkv, D)
    try:
        cs = torch.full((B,), N - 256, dtype=torch.int32, device="cuda")
        qpos = torch.full((B,), N - 1, dtype=torch.int32, device="cuda")
        for epoch in (1, 2, 3):             # both slots of the buffer, then the first again
            q = ROUND["bf16"](rnd(72 + epoch, (B, Hq, D)))
            qd = to_dev(q, "bf16")
            for r, (a, b) in enumerate(_shards(N, world, ps)):
                p0, p1 = a // ps, (b + ps - 1) // ps
                bt = torch.from_numpy(np.ascontiguousarray(bt_full[:, p0:max(p1, p0 + 1)])).cuda()
                ws = torch.zeros(1 << 22, dtype=torch.uint8, device="cuda")
                ops.paged_fog_decode_cp(_View(bufs, r, world), epoch, qd, kv[:, :, 0], kv[:, :, 1], bt,
                                        torch.full((B,), b - a, dtype=torch.int32, device="cuda"), clear_start=cs,
                                        fog_alpha=0.5, window_size=window,
                                        kv_pos_offset=torch.full((B,), a, dtype=torch.int32, device="cuda"),
                                        q_positions=qpos, max_seq_len=bt.shape[1] * ps, phases=1, ws=ws)
            outs = []
            for r in range(world):
                o = torch.empty(B, Hq, D, dtype=torch.bfloat16, device="cuda")
                part = torch.empty(B, Hq, D + 2, dtype=torch.float32, device="cuda")
                ops.cp_combine(_View(bufs, r, world), epoch, B, Hq, Hkv, out=o, out_partial=part)
                outs.append((o, part))
            torch.cuda.synchronize()
            assert ops.read_device_status() == 0
            want = O.paged_fog_decode(q, kvn[:, :, 0], kvn[:, :, 1], bt_full, [N] * B, [N - 256] * B, 0.5, window)
            for o, part in outs:
                np.testing.assert_allclose(to_np(o), want, **TOL["bf16"])
                np.testing.assert_allclose(part[..., :D].cpu().numpy(), want, **TOL["bf16"])
            for o, _ in outs[1:]:
                assert torch.equal(o, outs[0][0])          # every rank holds the same merged result
    finally:
        torch.cuda.synchronize()
        bufs.free()


def test_cp_combine_wait_runs_out_and_reports():
    """A flag that no rank ever raises: the combine's bounded wait gives up
    after its limit, records KESSIE_DEV_WAIT_TIMEOUT, writes zero rows, and
    the context stays usable."""
    from kessie_b200 import ops
    B, Hq, Hkv, D = 2, 8, 2, 128
    bufs = _Buffers(2, B, Hq, Hkv, D)
    try:
        ops.read_device_status()
        o = torch.full((B, Hq, D), 7.0, dtype=torch.bfloat16, device="cuda")
        ops.cp_combine(_View(bufs, 0, 2), 5, B, Hq, Hkv, out=o, wait_timeout_s=0.02)
        st = ops.read_device_status()
        assert st & 0x2
        assert (o.float() == 0).all()
        # the device still works
        x = torch.arange(10, device="cuda").sum().item()
        assert x == 45
    finally:
        torch.cuda.synchronize()
        bufs.free()


def test_cp_steps_back_to_back():
    """Single-rank context-parallel steps (decode + combine) with nothing in
    between and no synchronisation.  The combine lets the next step's decode
    start at once, so that decode may read ahead while this step's decode
    and combine finish: steps with their own q and outputs, then a chain whose
    combined output is the next step's q (those must wait), then a page
    gather right after a combine.  Every result equals the same steps run one
    at a time."""
    from kessie_b200 import ops
    B, Hq, Hkv, D, ps = 2, 16, 4, 128, 16
    N = 5000
    pages = (N + ps - 1) // ps
    _, kv = make_paged(81, B * pages, ps, Hkv, D, "bf16")
    bt = torch.from_numpy(np.random.default_rng(82).permutation(B * pages).astype(np.int32).reshape(B, pages)).cuda()
    sl = torch.full((B,), N, dtype=torch.int32, device="cuda")
    cs = torch.full((B,), N - 256, dtype=torch.int32, device="cuda")
    qs = [to_dev(ROUND["bf16"](rnd(83 + i, (B, Hq, D))), "bf16") for i in range(2)]
    ws = torch.empty(ops.decode_workspace_bytes(B, Hq, Hkv, D, pages * ps, ps), dtype=torch.uint8, device="cuda")
    gid = torch.arange(8, dtype=torch.int32, device="cuda")
    epoch = [0]

    def run(sync):
        bufs = _Buffers(1, B, Hq, Hkv, D)
        try:
            view = _View(bufs, 0, 1)
            outs = [torch.empty(B, Hq, D, dtype=torch.bfloat16, device="cuda") for _ in range(4)]
            chain = [qs[0].clone()] + [torch.empty(B, Hq, D, dtype=torch.bfloat16, device="cuda") for _ in range(3)]
            gk = torch.empty(8 * ps, Hkv, D, dtype=torch.bfloat16, device="cuda")
            gv = torch.empty_like(gk)
            torch.cuda.synchronize()
            steps = [(qs[j % 2], outs[j]) for j in range(4)] + [(chain[j], chain[j + 1]) for j in range(3)]
            for i, (q, o) in enumerate(steps):
                epoch[0] += 1
                ops.paged_fog_decode_cp(view, epoch[0], q, kv[:, :, 0], kv[:, :, 1], bt, sl, clear_start=cs,
                                        out=o, ws=ws, phases=3)
                if i == 3:
                    ops.page_gather(kv, gid, out_keys=gk, out_values=gv)
                if sync:
                    torch.cuda.synchronize()
            torch.cuda.synchronize()
            assert ops.read_device_status() == 0
            return outs + chain[1:] + [gk, gv]
        finally:
            torch.cuda.synchronize()
            bufs.free()

    got, want = run(False), run(True)
    for a, b in zip(got, want):
        assert torch.equal(a, b)
    assert torch.equal(got[0], got[2]) and not torch.equal(got[4], got[5])
