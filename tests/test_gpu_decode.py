"""GPU parity: paged fog decode (split-KV, GQA) and the LSE combine against
the numpy oracle (bf16 / fp16: 2e-2 max-abs, 1e-2 rel)."""

import os

import numpy as np
import pytest
import torch

from oracle import fog_oracle as O
from tests.kessie_testutil import ROUND, TOL, TORCH_DT, make_paged, random_block_table, rnd, to_dev, to_np

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    yield


def run_case(seed, B, Hq, Hkv, D, dt, lens, ps=16, window=0, fog=True, alpha=0.5, fog_window=None,
             kv_off=None, q_pos=None, explicit_weights=False, layout="kessie", spare=3, nan_fill=False,
             scale=None):
    from kessie_b200 import ops
    lens = np.asarray(lens, np.int64)
    need = int(sum((n + ps - 1) // ps for n in lens))
    P = need + spare
    kvn, kv = make_paged(seed, P, ps, Hkv, D, dt, scale=(scale if scale is not None else 1.0))
    if nan_fill:
        # stale slots beyond each sequence hold NaN: they must not leak
        kv_nan = kv.clone()
    bt = random_block_table(seed + 1, lens, ps, P)
    if nan_fill:
        for b, n in enumerate(lens):
            npg = (n + ps - 1) // ps
            if n % ps:
                last = bt[b, npg - 1]
                kv[last, n % ps:] = float("nan")
                kvn[last, n % ps:] = np.nan
    q = ROUND[dt](rnd(seed + 2, (B, Hq, D)))
    off = np.zeros(B, np.int64) if kv_off is None else np.asarray(kv_off)
    cs = None
    if fog:
        fw = fog_window if fog_window is not None else 64
        cs = np.array([off[b] + lens[b] - fw for b in range(B)], np.int32)
    k_cache, v_cache = kv[:, :, 0], kv[:, :, 1]
    fwt = None
    if explicit_weights:
        total = int((off + lens).max())
        fwt = O.fog_weights_from_clear_start(total, int(cs[0]), alpha)
    out = ops.paged_fog_decode(
        to_dev(q, dt), k_cache, v_cache, torch.from_numpy(bt).cuda(), torch.from_numpy(lens.astype(np.int32)).cuda(),
        clear_start=None if cs is None else torch.from_numpy(cs).cuda(), fog_alpha=alpha,
        fog_weights=None if fwt is None else torch.from_numpy(fwt).cuda(), window_size=window,
        kv_pos_offset=None if kv_off is None else torch.from_numpy(off.astype(np.int32)).cuda(),
        q_positions=None if q_pos is None else torch.from_numpy(np.asarray(q_pos, np.int32)).cuda(),
        sm_scale=scale and 1.0 / np.sqrt(D))
    torch.cuda.synchronize()
    kp = kvn[:, :, 0]; vp = kvn[:, :, 1]
    if explicit_weights:
        want = O.paged_fog_decode(q, kp, vp, bt, lens, None, alpha, window, kv_pos_offset=kv_off, q_pos=q_pos,
                                  fog_weights=fwt)
    else:
        want = O.paged_fog_decode(q, kp, vp, bt, lens, cs if fog else np.zeros(B, np.int32), alpha if fog else 0.0,
                                  window, kv_pos_offset=kv_off, q_pos=q_pos)
    got = to_np(out)
    return got, want


@pytest.mark.parametrize("dt", ["bf16", "fp16"])
@pytest.mark.parametrize("Hq,Hkv", [(8, 8), (8, 2), (32, 8), (64, 8), (16, 1), (12, 2), (6, 3)])
def test_decode_gqa_shapes(dt, Hq, Hkv):
    B = 3
    got, want = run_case(Hq * 10 + Hkv, B, Hq, Hkv, 128, dt, [700, 16, 2049])
    np.testing.assert_allclose(got, want, **TOL[dt])


@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("lens", [[1], [15, 17, 33], [4096], [9000, 12345]])
def test_decode_lengths(D, lens):
    got, want = run_case(sum(lens), len(lens), 8, 2, D, "bf16", lens)
    np.testing.assert_allclose(got, want, **TOL["bf16"])


@pytest.mark.parametrize("window", [1, 16, 100, 3000])
def test_decode_reference_literal_window(window):
    """window_size > 0 masks keys with q_pos - j >= W (kessie_hip_kernels.py:585-587)."""
    got, want = run_case(window, 2, 8, 2, 128, "bf16", [2500, 333], window=window)
    np.testing.assert_allclose(got, want, **TOL["bf16"])


@pytest.mark.parametrize("alpha,fogw", [(0.5, 64), (1.5, 300), (0.0, 64), (0.5, 0), (0.5, 5000)])
def test_decode_fog_params(alpha, fogw):
    got, want = run_case(7, 2, 8, 2, 128, "bf16", [1000, 4000], alpha=alpha, fog_window=fogw)
    np.testing.assert_allclose(got, want, **TOL["bf16"])


def test_decode_no_fog_and_explicit_weights():
    got, want = run_case(8, 2, 16, 4, 128, "fp16", [800, 801], fog=False)
    np.testing.assert_allclose(got, want, **TOL["fp16"])
    got, want = run_case(9, 1, 16, 4, 128, "bf16", [1500], explicit_weights=True)
    np.testing.assert_allclose(got, want, **TOL["bf16"])


def test_decode_stale_nan_tail_does_not_leak():
    got, want = run_case(10, 2, 8, 2, 128, "bf16", [37, 100], nan_fill=True)
    assert np.isfinite(got).all()
    np.testing.assert_allclose(got, want, **TOL["bf16"])


def test_decode_page_size_32_and_64():
    for ps in (32, 64):
        got, want = run_case(11 + ps, 2, 8, 2, 128, "bf16", [500, 77], ps=ps)
        np.testing.assert_allclose(got, want, **TOL["bf16"])


def test_decode_context_parallel_shards_merge():
    """Split one sequence across 3 'ranks' by position; merging the shard
    partials with lse_combine equals the unsplit decode."""
    from kessie_b200 import ops
    D, Hq, Hkv, ps = 128, 16, 2, 16
    N = 3 * 1024
    kvn, kv = make_paged(31, N // ps, ps, Hkv, D, "bf16")
    q = ROUND["bf16"](rnd(32, (1, Hq, D)))
    qd = to_dev(q, "bf16")
    cs = torch.tensor([N - 512], dtype=torch.int32, device="cuda")
    parts = torch.empty(3, 1, Hq, D + 2, dtype=torch.float32, device="cuda")
    for r in range(3):
        bt = torch.arange(r * 64, (r + 1) * 64, dtype=torch.int32, device="cuda")[None]
        ops.paged_fog_decode(qd, kv[:, :, 0], kv[:, :, 1], bt, torch.tensor([1024], dtype=torch.int32, device="cuda"),
                             clear_start=cs, fog_alpha=0.5, kv_pos_offset=torch.tensor([r * 1024], dtype=torch.int32,
                                                                                       device="cuda"),
                             q_positions=torch.tensor([N - 1], dtype=torch.int32, device="cuda"),
                             out_partial=parts[r], want_out=False)
    merged = ops.lse_combine(parts.contiguous(), out_dtype=torch.float32)
    torch.cuda.synchronize()
    bt_full = np.arange(N // ps, dtype=np.int32)[None]
    want = O.paged_fog_decode(q, kvn[:, :, 0], kvn[:, :, 1], bt_full, [N], [N - 512], 0.5)
    np.testing.assert_allclose(to_np(merged), want, atol=2e-2, rtol=1e-2)
    # partial triples agree with the oracle's (m, l) in natural-log units
    _, (ms, ls, os_) = O.paged_fog_decode(q, kvn[:, :, 0], kvn[:, :, 1], np.arange(64, dtype=np.int32)[None],
                                          [1024], [N - 512], 0.5, return_partials=True)
    p0 = parts[0].cpu().numpy()
    np.testing.assert_allclose(p0[0, :, D], ms[0], atol=1e-3, rtol=1e-3)
    np.testing.assert_allclose(p0[0, :, D + 1], ls[0], rtol=1e-2)


def test_config1_golden_decode(golden_dir):
    """Benchmark config 1 (fp32 in the reference) through the bf16/fp16 kernel:
    the inputs are rounded to fp16 and compared with the stated fp16 bar; the
    oracle at the same rounded inputs is checked at the tighter 5e-3."""
    from kessie_b200 import ops
    d = np.load(os.path.join(golden_dir, "config1_decode.npz"))
    B, Hq, Hkv, D, N, W, seed = (int(x) for x in d["cfg"])
    q = rnd(seed, (N, Hq, D)); k = rnd(seed + 1, (N, Hkv, D)); v = rnd(seed + 2, (N, Hkv, D))
    pos = np.arange(N); zero = np.zeros(N, np.int64)
    q = O.rope_remap(q, zero, pos, 1e4); k = O.rope_remap(k, zero, pos, 1e4)
    qh = O.round_f16(q[-1])[None]
    kh = O.round_f16(k); vh = O.round_f16(v)
    ps = 16
    kv = np.stack([kh, vh], axis=1).reshape(N // ps, ps, 2, Hkv, D)
    kvd = to_dev(kv, "fp16")
    bt = torch.arange(N // ps, dtype=torch.int32, device="cuda")[None]
    for win, key in ((0, "out_causal_fog"), (W, "out_window_fog")):
        out = ops.paged_fog_decode(to_dev(qh, "fp16"), kvd[:, :, 0], kvd[:, :, 1], bt,
                                   torch.tensor([N], dtype=torch.int32, device="cuda"),
                                   clear_start=torch.tensor([int(d["clear_start"])], dtype=torch.int32, device="cuda"),
                                   fog_alpha=0.5, window_size=win)
        torch.cuda.synchronize()
        got = to_np(out)[0]
        np.testing.assert_allclose(got, d[key], atol=2e-2, rtol=1e-2)
        want = O.paged_fog_decode(qh, kv[:, :, 0], kv[:, :, 1], np.arange(N // ps)[None], [N],
                                  [int(d["clear_start"])], 0.5, win)[0]
        np.testing.assert_allclose(got, want, atol=5e-3, rtol=5e-3)


def test_decode_bad_page_id_flagged_not_faulting():
    from kessie_b200 import ops
    ops.read_device_status()
    kvn, kv = make_paged(41, 8, 16, 2, 128, "bf16")
    bt = torch.tensor([[0, 1, 12345, 3]], dtype=torch.int32, device="cuda")
    q = to_dev(rnd(42, (1, 8, 128)), "bf16")
    out = ops.paged_fog_decode(q, kv[:, :, 0], kv[:, :, 1], bt, torch.tensor([64], dtype=torch.int32, device="cuda"))
    st = ops.read_device_status()
    assert st & 0x1
    assert torch.isfinite(out.float()).all()
    # keys of the bad page are excluded: equals decode over pages 0, 1, 3
    want = O.fog_attention_rows(ROUND["bf16"](rnd(42, (1, 8, 128)))[0][:, None],
                                np.transpose(np.concatenate([kvn[i, :, 0] for i in (0, 1, 3)]), (1, 0, 2)),
                                np.transpose(np.concatenate([kvn[i, :, 1] for i in (0, 1, 3)]), (1, 0, 2)),
                                np.array([10 ** 6]))[:, 0]
    np.testing.assert_allclose(to_np(out)[0], want, **TOL["bf16"])


def test_lse_combine_matches_oracle():
    from kessie_b200 import ops
    rng = np.random.default_rng(3)
    S, R, D = 5, 7, 128
    ms = rng.standard_normal((S, R)) * 3
    ms[1, 2] = -np.inf                       # an empty shard
    ls = rng.random((S, R)) + 0.1
    ls[1, 2] = 0.0
    os_ = rng.standard_normal((S, R, D)) * ls[..., None]
    parts = torch.from_numpy(O.partials_from_rows(ms, ls, os_)).cuda()
    out = ops.lse_combine(parts, out_dtype=torch.float32)
    torch.cuda.synchronize()
    np.testing.assert_allclose(to_np(out), O.lse_combine(ms, ls, os_), atol=1e-5, rtol=1e-5)


def test_decode_empty_and_excluded_sequences():
    """Sequences with no visible key (length 0, or a window that ends before
    the shard) give zero rows and do not disturb their neighbours."""
    got, want = run_case(51, 4, 8, 2, 128, "bf16", [0, 300, 0, 45])
    np.testing.assert_allclose(got, want, **TOL["bf16"])
    assert (got[0] == 0).all() and (got[2] == 0).all()
    got, want = run_case(52, 3, 8, 2, 128, "bf16", [200, 700, 64], window=100, q_pos=[5000, 699, 63],
                         kv_off=[0, 0, 0])
    np.testing.assert_allclose(got, want, **TOL["bf16"])
    assert (got[0] == 0).all()


@pytest.mark.parametrize("B,D", [(100, 128), (70, 64)])
def test_decode_large_batch_many_segments(B, D):
    """More sequences than a warp (multi-round range search) and many short
    groups per CTA (many segments, many group merges)."""
    lens = np.random.default_rng(B).integers(1, 400, size=B)
    got, want = run_case(B + D, B, 8, 2, D, "bf16", lens)
    np.testing.assert_allclose(got, want, **TOL["bf16"])


def test_decode_workspace_reuse_is_deterministic():
    """The per-group arrival counters return to zero after every call: calls
    of different shapes that share the cached workspace, then the first
    shape again, give bit-identical results (the merge order is fixed by
    slot, not by arrival)."""
    from kessie_b200 import ops
    outs = []
    for lens in ([5000, 3000, 17], [40], [5000, 3000, 17]):
        B = len(lens)
        kvn, kv = make_paged(61, 1000, 16, 2, 128, "bf16")
        bt = torch.from_numpy(random_block_table(62, lens, 16, 1000)).cuda()
        q = to_dev(rnd(63, (B, 8, 128)), "bf16")
        o = ops.paged_fog_decode(q, kv[:, :, 0], kv[:, :, 1], bt, torch.tensor(lens, dtype=torch.int32, device="cuda"),
                                 clear_start=torch.tensor([n - 64 for n in lens], dtype=torch.int32, device="cuda"))
        outs.append(o.clone())
    torch.cuda.synchronize()
    assert torch.equal(outs[0], outs[2])
    assert ops.read_device_status() == 0


def test_decode_workspace_garbage_is_ignored():
    """A workspace full of leftover bytes (another shape's partials, random
    data) needs no clearing: stale arrival counters carry another tag."""
    from kessie_b200 import ops, _lib
    lens = [3000, 40, 999, 1]
    B = len(lens)
    kvn, kv = make_paged(81, 400, 16, 2, 128, "bf16")
    bt_np = random_block_table(82, lens, 16, 400)
    bt = torch.from_numpy(bt_np).cuda()
    q = ROUND["bf16"](rnd(83, (B, 8, 128)))
    need = _lib.load().kessie_paged_fog_decode_workspace_size(B, 8, 2, 128, bt.shape[1] * 16, 16)
    g = torch.Generator(device="cuda").manual_seed(84)
    ws = torch.randint(0, 256, (need,), dtype=torch.uint8, device="cuda", generator=g)
    cs = [n - 64 for n in lens]
    out = ops.paged_fog_decode(to_dev(q, "bf16"), kv[:, :, 0], kv[:, :, 1], bt,
                               torch.tensor(lens, dtype=torch.int32, device="cuda"),
                               clear_start=torch.tensor(cs, dtype=torch.int32, device="cuda"), ws=ws)
    torch.cuda.synchronize()
    want = O.paged_fog_decode(q, kvn[:, :, 0], kvn[:, :, 1], bt_np, lens, cs, 0.5)
    np.testing.assert_allclose(to_np(out), want, **TOL["bf16"])


def test_decode_back_to_back():
    """Decodes enqueued with nothing in between and no synchronisation, as
    the steps of a serving loop run them: each may load its pages and q
    before the previous decode has finished when that decode wrote none of
    those bytes.  Independent decodes over three caches in turn (twice), then
    a chain whose output is the next step's q (those must wait); every result
    equals the same launches run one at a time."""
    from kessie_b200 import ops
    B, Hq, Hkv, D, ps = 4, 16, 4, 128, 16
    lens = np.array([3000, 1777, 4096, 2500])
    P = int(sum((n + ps - 1) // ps for n in lens)) + 2
    caches = [make_paged(90 + i, P, ps, Hkv, D, "bf16")[1] for i in range(3)]
    bt = torch.from_numpy(random_block_table(93, lens, ps, P)).cuda()
    sl = torch.from_numpy(lens.astype(np.int32)).cuda()
    cs = torch.from_numpy((lens - 64).astype(np.int32)).cuda()
    qs = [to_dev(ROUND["bf16"](rnd(94 + i, (B, Hq, D))), "bf16") for i in range(3)]
    ws = torch.empty(ops.decode_workspace_bytes(B, Hq, Hkv, D, bt.shape[1] * ps, ps), dtype=torch.uint8,
                     device="cuda")

    def run(sync):
        outs = [torch.empty(B, Hq, D, dtype=torch.bfloat16, device="cuda") for _ in range(6)]
        chain = [qs[0].clone()] + [torch.empty(B, Hq, D, dtype=torch.bfloat16, device="cuda") for _ in range(4)]
        torch.cuda.synchronize()
        for j in range(6):
            c = caches[j % 3]
            ops.paged_fog_decode(qs[j % 3], c[:, :, 0], c[:, :, 1], bt, sl, clear_start=cs, ws=ws, out=outs[j])
            if sync:
                torch.cuda.synchronize()
        for j in range(4):
            c = caches[j % 3]
            ops.paged_fog_decode(chain[j], c[:, :, 0], c[:, :, 1], bt, sl, clear_start=cs, ws=ws, out=chain[j + 1])
            if sync:
                torch.cuda.synchronize()
        torch.cuda.synchronize()
        return outs + chain[1:]

    got, want = run(False), run(True)
    assert ops.read_device_status() == 0
    for a, b in zip(got, want):
        assert torch.equal(a, b)
    assert torch.equal(got[0], got[3]) and not torch.equal(got[6], got[7])
