"""GPU parity: RoPE remap, page evict/compaction, insert(+remap), gather
against the numpy oracle (bit-exact for integer/copy work, north_star
tolerances for rotated values)."""

import ctypes
import os

import numpy as np
import pytest
import torch

from oracle import fog_oracle as O
from tests.kessie_testutil import ROUND, TOL, TORCH_DT, make_paged, rnd, to_dev, to_np

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from kessie_b200 import _lib
    _lib.load()
    yield


def _status():
    from kessie_b200 import ops
    return ops.read_device_status()


# ----------------------------------------------------------------- RoPE remap
@pytest.mark.parametrize("i", range(5))
def test_rope_remap_golden(golden_dir, i):
    from kessie_b200 import ops
    d = np.load(os.path.join(golden_dir, "rope_remap.npz"))
    seed, T, H, D, theta = d[f"case{i}_meta"]
    dt = {"float32": "fp32", "bfloat16": "bf16", "float16": "fp16"}[str(d[f"case{i}_dtype"])]
    kin = d[f"case{i}_kin"]
    k = to_dev(kin, dt)
    ops.rope_remap(k, torch.from_numpy(d[f"case{i}_orig"]).cuda(), torch.from_numpy(d[f"case{i}_tgt"]).cuda(), theta)
    got = to_np(k)
    want = ROUND[dt](O.rope_remap(kin, d[f"case{i}_orig"], d[f"case{i}_tgt"], theta))
    np.testing.assert_allclose(got, want, **TOL[dt])
    if dt != "fp32":
        # reference's own golden output (torch): same bar
        np.testing.assert_allclose(got, d[f"case{i}_kout"], **TOL[dt])


@pytest.mark.parametrize("dt", ["bf16", "fp16", "fp32"])
@pytest.mark.parametrize("T,H,D", [(1, 1, 64), (37, 3, 128), (300, 8, 128), (65, 2, 32), (16, 4, 256)])
def test_rope_remap_shapes(dt, T, H, D):
    from kessie_b200 import ops
    x = ROUND[dt](rnd(T * 7 + H, (T, H, D)))
    rng = np.random.default_rng(T)
    orig = rng.integers(0, 200000, T).astype(np.int32)
    tgt = rng.integers(0, 200000, T).astype(np.int32)
    k = to_dev(x, dt)
    ops.rope_remap(k, orig, tgt, 500000.0)
    np.testing.assert_allclose(to_np(k), ROUND[dt](O.rope_remap(x, orig, tgt, 500000.0)), **TOL[dt])


def test_rope_remap_strided_and_identity_roundtrip():
    from kessie_b200 import ops
    # a strided view: K half of a [T, 2, H, D] buffer
    base = to_dev(rnd(3, (64, 2, 8, 128)), "fp16")
    k = base[:, 0]
    k0 = k.clone()
    v0 = base[:, 1].clone()
    o = torch.arange(100, 164, dtype=torch.int32, device="cuda")
    t = torch.arange(5000, 5064, dtype=torch.int32, device="cuda")
    ops.rope_remap(k, o, t)
    ops.rope_remap(k, t, o)
    assert (k.float() - k0.float()).abs().max().item() < 0.05          # kessie_hip_kernels.py:675
    assert torch.equal(base[:, 1], v0)                                  # V untouched
    k2 = k0.clone()
    ops.rope_remap(k2, o, o)
    assert (k2.float() - k0.float()).abs().max().item() < 1e-5          # identity, kessie_hip_kernels.py:681


def test_legacy_rope_remap_launcher():
    from kessie_b200 import _lib
    lib = _lib.load()
    x = O.round_f16(rnd(9, (48, 4, 128)))
    k = to_dev(x, "fp16")
    rng = np.random.default_rng(1)
    orig = torch.from_numpy(rng.integers(0, 4096, 48).astype(np.int32)).cuda()
    tgt = torch.from_numpy(rng.integers(0, 4096, 48).astype(np.int32)).cuda()
    lib.launch_kessie_rope_remap(k.data_ptr(), orig.data_ptr(), tgt.data_ptr(), ctypes.c_float(1e4), 48, 4, 64, None)
    _lib.check_legacy("launch_kessie_rope_remap")
    torch.cuda.synchronize()
    want = O.round_f16(O.rope_remap(x, orig.cpu().numpy(), tgt.cpu().numpy(), 1e4))
    np.testing.assert_allclose(to_np(k), want, **TOL["fp16"])


# ----------------------------------------------------------------- evict
def test_legacy_evict_kat():
    """kessie_kernels_v2.hip:1008-1023: 256 pages, first 128 valid at i*128,
    threshold 8192 -> 64 evicted."""
    from kessie_b200 import _lib
    lib = _lib.load()
    valid = torch.zeros(256, dtype=torch.int8, device="cuda"); valid[:128] = 1
    pos = torch.zeros(256, dtype=torch.int32, device="cuda"); pos[:128] = torch.arange(128, device="cuda") * 128
    cnt = torch.zeros(1, dtype=torch.int32, device="cuda")
    lib.launch_kessie_page_evict(valid.data_ptr(), pos.data_ptr(), cnt.data_ptr(), 8192, 256, None)
    _lib.check_legacy("launch_kessie_page_evict")
    assert cnt.item() == 64
    assert valid[:64].sum().item() == 0 and valid[64:128].sum().item() == 64


@pytest.mark.parametrize("P", [1, 7, 4096, 4097, 8192, 100003])
@pytest.mark.parametrize("with_alloc", [False, True])
def test_evict_v2_matches_oracle(P, with_alloc):
    from kessie_b200 import ops
    rng = np.random.default_rng(P)
    valid = (rng.random(P) < 0.7).astype(np.int8)
    valid[rng.random(P) < 0.05] = 2                 # non-1 values are not evicted (== 1 test)
    pos = rng.integers(0, 1 << 20, P).astype(np.int32)
    thr = 1 << 19
    alloc = ((valid != 0) | (rng.random(P) < 0.1)).astype(np.int8)
    v_d = torch.from_numpy(valid).cuda(); p_d = torch.from_numpy(pos).cuda()
    a_d = torch.from_numpy(alloc).cuda() if with_alloc else None
    cnt, ids = ops.page_evict(v_d, p_d, thr, a_d)
    nv, n, evicted = O.page_evict(valid, pos, thr)
    assert np.array_equal(v_d.cpu().numpy(), nv)
    if with_alloc:
        freed = np.nonzero((alloc == 1) & (nv == 0))[0].astype(np.int32)
        na = alloc.copy(); na[freed] = 0
        assert np.array_equal(a_d.cpu().numpy(), na)
    else:
        freed = evicted
    c = cnt.item()
    assert c == len(freed)
    assert np.array_equal(ids[:c].cpu().numpy(), freed)


def test_config2_eviction_exactly_quarter():
    """Config 2: P=8192, pos[p] = 16*perm[p], threshold 32768 -> 2048 pages."""
    from kessie_b200 import ops
    perm = np.random.default_rng(2).permutation(8192)
    pos = (16 * perm).astype(np.int32)
    valid = np.ones(8192, np.int8)
    cnt, ids = ops.page_evict(torch.from_numpy(valid).cuda(), torch.from_numpy(pos).cuda(), 32768)
    _, n, want = O.page_evict(valid, pos, 32768)
    assert cnt.item() == n == 2048
    assert np.array_equal(ids[:2048].cpu().numpy(), want)


def test_list_valid_pages():
    from kessie_b200 import ops
    rng = np.random.default_rng(4)
    valid = (rng.random(10000) < 0.3).astype(np.int8)
    cnt, ids = ops.list_valid_pages(torch.from_numpy(valid).cuda())
    want = np.nonzero(valid)[0]
    assert cnt.item() == len(want) and np.array_equal(ids[:len(want)].cpu().numpy(), want)


# ----------------------------------------------------------------- insert / gather
@pytest.mark.parametrize("dt", ["bf16", "fp16", "fp32"])
@pytest.mark.parametrize("T", [1, 16, 45, 160])
def test_page_insert_matches_oracle(dt, T):
    from kessie_b200 import ops
    P, ps, H, D = 40, 16, 4, 128
    cache_np = np.zeros((P, ps, 2, H, D), np.float32)
    kv = to_dev(cache_np, dt)
    keys = ROUND[dt](rnd(T, (T, H, D))); vals = ROUND[dt](rnd(T + 1, (T, H, D)))
    npg = (T + ps - 1) // ps
    ids = np.random.default_rng(T).permutation(P)[:npg].astype(np.int32)
    valid = torch.zeros(P, dtype=torch.int8, device="cuda"); posd = torch.zeros(P, dtype=torch.int32, device="cuda")
    ops.page_insert(kv, to_dev(keys, dt), to_dev(vals, dt), ids, valid, posd, conv_pos=777)
    torch.cuda.synchronize()
    want = cache_np.copy()
    for p_, pid in enumerate(ids):
        s, e = p_ * ps, min((p_ + 1) * ps, T)
        want[pid, :e - s, 0] = keys[s:e]; want[pid, :e - s, 1] = vals[s:e]
    assert np.array_equal(to_np(kv), want)
    vv = np.zeros(P, np.int8); vv[ids] = 1
    pp = np.zeros(P, np.int32); pp[ids] = 777 + np.arange(npg) * ps
    assert np.array_equal(valid.cpu().numpy(), vv) and np.array_equal(posd.cpu().numpy(), pp)


def test_legacy_page_insert_launcher():
    from kessie_b200 import _lib
    lib = _lib.load()
    P, ps, H, D, T = 12, 16, 2, 64, 40
    kv = torch.zeros(P, ps, 2, H, D, dtype=torch.float16, device="cuda")
    keys = to_dev(O.round_f16(rnd(1, (T, H, D))), "fp16"); vals = to_dev(O.round_f16(rnd(2, (T, H, D))), "fp16")
    ids = torch.tensor([5, 99, 2], dtype=torch.int32, device="cuda")          # 99 is out of range -> skipped
    valid = torch.zeros(P, dtype=torch.int8, device="cuda"); pos = torch.zeros(P, dtype=torch.int32, device="cuda")
    lib.launch_kessie_page_insert(kv.data_ptr(), keys.data_ptr(), vals.data_ptr(), ids.data_ptr(), valid.data_ptr(),
                                  pos.data_ptr(), 1000, T, H, D, ps, P, None)
    _lib.check_legacy("launch_kessie_page_insert")
    torch.cuda.synchronize()
    assert torch.equal(kv[5, :, 0], keys[:16]) and torch.equal(kv[2, :8, 1], vals[32:40])
    assert valid.tolist() == [0, 0, 1, 0, 0, 1] + [0] * 6
    assert pos[5].item() == 1000 and pos[2].item() == 1032
    assert _status() & 0x1     # bad page id recorded


@pytest.mark.parametrize("dt", ["bf16", "fp16"])
def test_fused_insert_remap(dt):
    """Recall path: insert K re-rotated from old to new positions (theta 5e5)."""
    from kessie_b200 import ops
    P, ps, H, D, T = 64, 16, 8, 128, 96
    kv = torch.zeros(P, ps, 2, H, D, dtype=TORCH_DT[dt], device="cuda")
    keys = ROUND[dt](rnd(11, (T, H, D))); vals = ROUND[dt](rnd(12, (T, H, D)))
    orig = np.random.default_rng(3).integers(0, 32768, T).astype(np.int32)
    ids = np.random.default_rng(5).permutation(P)[:T // ps].astype(np.int32)
    ops.page_insert(kv, to_dev(keys, dt), to_dev(vals, dt), ids, conv_pos=131072, orig_positions=orig,
                    rope_theta=500000.0)
    torch.cuda.synchronize()
    rot = ROUND[dt](O.rope_remap(keys, orig, 131072 + np.arange(T), 500000.0))
    got = to_np(kv)
    for p_, pid in enumerate(ids):
        np.testing.assert_allclose(got[pid, :, 0], rot[p_ * ps:(p_ + 1) * ps], **TOL[dt])
        assert np.array_equal(got[pid, :, 1], vals[p_ * ps:(p_ + 1) * ps])


@pytest.mark.parametrize("layout", ["kessie", "vllm"])
@pytest.mark.parametrize("dt", ["bf16", "fp32"])
def test_page_gather_matches_oracle(layout, dt):
    from kessie_b200 import ops
    P, ps, H, D = 33, 16, 4, 128
    kvn, kv = make_paged(21, P, ps, H, D, dt)              # [P, ps, 2, H, D]
    if layout == "vllm":
        kv = kv.permute(2, 0, 1, 3, 4).contiguous()         # [2, P, ps, H, D]
    ids = np.array([3, 0, 32, 17, 3], dtype=np.int32)
    K, V = ops.page_gather(kv, ids, layout=layout)
    wk, wv = O.page_gather(kvn, ids)
    assert np.array_equal(to_np(K), wk) and np.array_equal(to_np(V), wv)


def test_page_gather_back_to_back():
    """Gathers enqueued with nothing in between and no synchronisation, as a
    multi-layer recall runs them: each may start loading its pages before the
    previous gather has finished, which is allowed only when that gather
    wrote none of the bytes it reads.  Four caches in turn, three rounds, then
    a gather whose output overwrites part of the next gather's cache (that
    one must wait); all bit-exact."""
    from kessie_b200 import ops
    P, ps, H, D, n = 64, 16, 8, 128, 24
    caches = [make_paged(40 + i, P, ps, H, D, "bf16") for i in range(4)]
    rng = np.random.default_rng(5)
    ids = [rng.permutation(P)[:n].astype(np.int32) for _ in range(4)]
    ids_d = [torch.from_numpy(x).cuda() for x in ids]
    outs = [(torch.empty(n * ps, H, D, dtype=torch.bfloat16, device="cuda"),
             torch.empty(n * ps, H, D, dtype=torch.bfloat16, device="cuda")) for _ in range(4)]
    torch.cuda.synchronize()
    for _ in range(3):
        for i in range(4):
            ops.page_gather(caches[i][1], ids_d[i], out_keys=outs[i][0], out_values=outs[i][1])
    # cache 1's K pages land in the first bytes of cache 0, which the next gather reads
    c0 = caches[0][1]
    k_into_c0 = c0.view(-1)[:n * ps * H * D].view(n * ps, H, D)
    ops.page_gather(caches[1][1], ids_d[1], out_keys=k_into_c0, want_values=False)
    K0, V0 = ops.page_gather(c0, ids_d[0])
    torch.cuda.synchronize()
    for i in range(4):
        wk, wv = O.page_gather(caches[i][0], ids[i])
        assert np.array_equal(to_np(outs[i][0]), wk) and np.array_equal(to_np(outs[i][1]), wv)
    c0n = caches[0][0].copy().reshape(-1)
    c0n[:n * ps * H * D] = O.page_gather(caches[1][0], ids[1])[0].reshape(-1)
    wk, wv = O.page_gather(c0n.reshape(P, ps, 2, H, D), ids[0])
    assert np.array_equal(to_np(K0), wk) and np.array_equal(to_np(V0), wv)
    assert np.array_equal(to_np(c0).reshape(-1), c0n)


def test_remap_and_insert_back_to_back():
    """RoPE remaps and fused inserts enqueued with nothing in between and no
    synchronisation, as a multi-layer recall runs them: a launch may copy its
    rows in before the previous one has finished when that one wrote none of
    them.  Four K buffers remapped in turn twice, a gather followed at once by
    a remap of its output (which must wait for it), and fused inserts into
    three caches in turn."""
    from kessie_b200 import ops
    T, H, D, P, ps, theta = 256, 8, 128, 64, 16, 500000.0
    rng = np.random.default_rng(8)
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    xs = [ROUND["bf16"](rnd(60 + i, (T, H, D))) for i in range(4)]
    ks = [to_dev(x, "bf16") for x in xs]
    # per-token positions (no shared delta) for two buffers, page-aligned shifts for the others
    origs = [rng.integers(0, 100000, T).astype(np.int32) if i < 2 else
             (16 * np.repeat(rng.permutation(1000)[:T // 16], 16) + np.tile(np.arange(16), T // 16)).astype(np.int32)
             for i in range(4)]
    tgts = [(131072 + np.arange(T)).astype(np.int32) for _ in range(4)]
    od, td = [dev(o) for o in origs], [dev(t) for t in tgts]
    kvn, kv = make_paged(70, P, ps, H, D, "bf16")
    gids = rng.permutation(P)[:T // ps].astype(np.int32)
    gids_d = dev(gids)
    caches = [torch.zeros(P, ps, 2, H, D, dtype=torch.bfloat16, device="cuda") for _ in range(3)]
    vals = [ROUND["bf16"](rnd(80 + i, (T, H, D))) for i in range(3)]
    vals_d = [to_dev(v, "bf16") for v in vals]
    ins_ids = [rng.permutation(P)[:T // ps].astype(np.int32) for _ in range(3)]
    ins_d = [dev(x) for x in ins_ids]
    torch.cuda.synchronize()
    for _ in range(2):
        for i in range(4):
            ops.rope_remap(ks[i], od[i], td[i], theta)
    K, _ = ops.page_gather(kv, gids_d)
    ops.rope_remap(K, od[3], td[3], theta)
    for i in range(3):
        ops.page_insert(caches[i], ks[i], vals_d[i], ins_d[i], conv_pos=131072, orig_positions=od[i], rope_theta=theta)
    torch.cuda.synchronize()
    want = []
    for i in range(4):
        w = ROUND["bf16"](O.rope_remap(xs[i], origs[i], tgts[i], theta))
        w = ROUND["bf16"](O.rope_remap(w, origs[i], tgts[i], theta))
        want.append(w)
        np.testing.assert_allclose(to_np(ks[i]), w, **TOL["bf16"])
    wk = O.page_gather(kvn, gids)[0]
    np.testing.assert_allclose(to_np(K), ROUND["bf16"](O.rope_remap(wk, origs[3], tgts[3], theta)), **TOL["bf16"])
    for i in range(3):
        got = to_np(caches[i])
        rot = ROUND["bf16"](O.rope_remap(to_np(ks[i]), origs[i], 131072 + np.arange(T), theta))
        for p_, pid in enumerate(ins_ids[i]):
            np.testing.assert_allclose(got[pid, :, 0], rot[p_ * ps:(p_ + 1) * ps], **TOL["bf16"])
            assert np.array_equal(got[pid, :, 1], vals[i][p_ * ps:(p_ + 1) * ps])


def test_page_gather_bad_id_zero_and_flag():
    from kessie_b200 import ops
    _status()
    kvn, kv = make_paged(1, 8, 16, 2, 64, "bf16")
    K, V = ops.page_gather(kv, np.array([1, 8, -1], np.int32))
    assert np.array_equal(to_np(K)[:16], kvn[1, :, 0].reshape(16, 2, 64))
    assert (to_np(K)[16:] == 0).all() and (to_np(V)[16:] == 0).all()
    assert _status() & 0x1


@pytest.mark.parametrize("dt", ["bf16", "fp32"])
def test_fused_insert_remap_ragged_and_bad_page(dt):
    """Ragged last page (T % ps != 0), explicit target positions, and one
    out-of-range page id: that page is skipped and flagged, the rest match."""
    from kessie_b200 import ops
    _status()
    P, ps, H, D, T = 20, 16, 4, 128, 45
    kv = torch.zeros(P, ps, 2, H, D, dtype=TORCH_DT[dt], device="cuda")
    keys = ROUND[dt](rnd(31, (T, H, D))); vals = ROUND[dt](rnd(32, (T, H, D)))
    orig = np.random.default_rng(7).integers(0, 50000, T).astype(np.int32)
    tgt = np.random.default_rng(8).integers(0, 50000, T).astype(np.int32)
    ids = np.array([4, 999, 11], dtype=np.int32)
    valid = torch.zeros(P, dtype=torch.int8, device="cuda"); posd = torch.zeros(P, dtype=torch.int32, device="cuda")
    ops.page_insert(kv, to_dev(keys, dt), to_dev(vals, dt), ids, valid, posd, conv_pos=100, orig_positions=orig,
                    target_positions=tgt, rope_theta=500000.0)
    assert _status() & 0x1
    got = to_np(kv)
    rot = ROUND[dt](O.rope_remap(keys, orig, tgt, 500000.0))
    np.testing.assert_allclose(got[4, :, 0], rot[0:16], **TOL[dt])
    np.testing.assert_allclose(got[11, :13, 0], rot[32:45], **TOL[dt])
    assert np.array_equal(got[11, :13, 1], vals[32:45]) and (got[11, 13:] == 0).all()
    assert valid.cpu().numpy()[[4, 11]].tolist() == [1, 1] and int(valid.sum()) == 2
    assert posd.cpu().numpy()[[4, 11]].tolist() == [100, 132]
