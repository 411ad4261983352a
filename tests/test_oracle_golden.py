"""Pin the numpy oracle against golden vectors produced by the reference's
own Python functions (tests/golden/make_golden.py)."""

import os

import numpy as np
import pytest

from oracle import fog_oracle as O


def rnd(seed, shape):
    return np.random.default_rng(seed).standard_normal(shape, dtype=np.float32)


def load(golden_dir, name):
    return np.load(os.path.join(golden_dir, name))


def test_fog_weights_match_reference(golden_dir):
    d = load(golden_dir, "fog_weights.npz")
    for i in range(int(d["ncases"])):
        n, a, fs = d[f"case{i}_params"]
        n = int(n)
        cs = O.clear_start_for(n, fs)
        assert cs == int(d[f"case{i}_clear_start"])
        w = O.build_fog_weights(n, a, fs)
        idx = d[f"case{i}_idx"]
        # pow may differ from torch's by one ulp; the ratio t is exact
        np.testing.assert_allclose(w[idx], d[f"case{i}_w"], rtol=2.5e-7, atol=0)
        if a > 0 and cs > 1:
            assert w[0] == 0.0 and w[min(cs, n) - 1] == 1.0


def test_rope_freq_table_bit_exact(golden_dir):
    d = load(golden_dir, "rope_remap.npz")
    for theta in (10000, 500000):
        for half in (32, 64):
            ref = d[f"freqs_{theta}_{half}"]
            assert np.array_equal(O.rope_freqs(half, float(theta)), ref)


@pytest.mark.parametrize("i", range(5))
def test_rope_remap_matches_reference(golden_dir, i):
    d = load(golden_dir, "rope_remap.npz")
    seed, T, H, D, theta = d[f"case{i}_meta"]
    dt = str(d[f"case{i}_dtype"])
    kin = d[f"case{i}_kin"]
    if dt == "float32":
        # the reference's fp32 torch path aliases k1 (see
        # rope_remap_fp32_inplace_reference); pin that behaviour, and check
        # the first half, which both formulas share, with the HIP rotation.
        alias = O.rope_remap_fp32_inplace_reference(kin, d[f"case{i}_orig"], d[f"case{i}_tgt"], theta)
        np.testing.assert_allclose(alias, d[f"case{i}_kout"], atol=1e-5, rtol=0)
        hip = O.rope_remap(kin, d[f"case{i}_orig"], d[f"case{i}_tgt"], theta)
        half = int(D) // 2
        np.testing.assert_allclose(hip[..., :half], d[f"case{i}_kout"][..., :half], atol=1e-5, rtol=0)
        return
    out = O.rope_remap(kin, d[f"case{i}_orig"], d[f"case{i}_tgt"], theta)
    rnd_fn = {"float32": lambda x: x, "bfloat16": O.round_bf16, "float16": O.round_f16}[dt]
    out = rnd_fn(out)
    ref = d[f"case{i}_kout"]
    if dt == "float32":
        np.testing.assert_allclose(out, ref, atol=1e-4, rtol=0)
    else:
        # at most one storage ulp apart (cos/sin of |delta| up to 1.6e5 rad)
        np.testing.assert_allclose(out, ref, atol=2e-2, rtol=1e-2)
        assert np.mean(out == ref) > 0.98


def test_rope_reference_kats(golden_dir):
    d = load(golden_dir, "rope_remap.npz")
    assert float(d["kat_roundtrip_maxdiff"]) < 0.05          # kessie_hip_kernels.py:675
    k = O.round_f16(rnd(16, (64, 8, 128)))
    o = np.arange(100, 164); t = np.arange(5000, 5064)
    back = O.round_f16(O.rope_remap(O.round_f16(O.rope_remap(k, o, t)), t, o))
    assert np.abs(back - k).max() < 0.05
    ident = O.round_f16(O.rope_remap(k, o, o))
    assert np.abs(ident - k).max() < 1e-5                    # kessie_hip_kernels.py:681


def test_windowed_and_fog_attention_match_reference(golden_dir):
    d = load(golden_dir, "attention.npz")
    for i in range(int(d["nwin"])):
        Z, H, N, D, W, causal, seed = (int(x) for x in d[f"win{i}_cfg"])
        q, k, v = (rnd(seed + j, (Z, H, N, D)) for j in range(3))
        out = O.windowed_attention(q, k, v, W, bool(causal))
        np.testing.assert_allclose(out[:, :, d[f"win{i}_rows"]], d[f"win{i}_out"], atol=2e-5, rtol=0)
    for i in range(int(d["nfog"])):
        Z, H, N, D, W, causal, seed = (int(x) for x in d[f"fog{i}_cfg"])
        a, fs = d[f"fog{i}_fog"]
        q, k, v = (rnd(seed + j, (Z, H, N, D)) for j in range(3))
        fog = O.build_fog_weights(N, a, fs)
        out = O.fused_fog_attention(q, k, v, fog, W, bool(causal))
        np.testing.assert_allclose(out[:, :, d[f"fog{i}_rows"]], d[f"fog{i}_out"], atol=2e-5, rtol=0)


def test_decode_restatement_matches_reference_config1(golden_dir):
    """Config 1: the query-offset GQA restatement at position 4095 equals the
    last row of the reference's full square attention (both fog mappings)."""
    d = load(golden_dir, "config1_decode.npz")
    B, Hq, Hkv, D, N, W, seed = (int(x) for x in d["cfg"])
    q = rnd(seed, (N, Hq, D)); k = rnd(seed + 1, (N, Hkv, D)); v = rnd(seed + 2, (N, Hkv, D))
    pos = np.arange(N); zero = np.zeros(N, dtype=np.int64)
    q = O.rope_remap(q, zero, pos, 10000.0)
    k = O.rope_remap(k, zero, pos, 10000.0)
    np.testing.assert_allclose(q[-1], d["q_rot_last"], atol=2e-5)
    np.testing.assert_allclose(k[::257], d["k_rot_sample"], atol=2e-5)
    cs = int(d["clear_start"])
    assert cs == N - W
    w = O.fog_weights_from_clear_start(N, cs, 0.5)
    qh = np.transpose(q[-1:], (1, 0, 2))       # [Hq,1,D]
    kh = np.transpose(k, (1, 0, 2)); vh = np.transpose(v, (1, 0, 2))
    oa = O.fog_attention_rows(qh, kh, vh, np.array([N - 1]), w, 0, True)[:, 0]
    ob = O.fog_attention_rows(qh, kh, vh, np.array([N - 1]), w, W, True)[:, 0]
    np.testing.assert_allclose(oa, d["out_causal_fog"], atol=1e-5)
    np.testing.assert_allclose(ob, d["out_window_fog"], atol=1e-5)


def test_split_lse_combine_equals_unsplit():
    rng = np.random.default_rng(5)
    Hq, Hkv, D, N = 8, 2, 64, 700
    q = rng.standard_normal((Hq, 1, D)); k = rng.standard_normal((Hkv, N, D)); v = rng.standard_normal((Hkv, N, D))
    w = O.fog_weights_from_clear_start(N, 500, 0.5)
    full = O.fog_attention_rows(q, k, v, np.array([N - 1]), w)
    cuts = [0, 100, 333, 334, 700]
    parts = [O.fog_attention_rows(q, k[:, a:b], v[:, a:b], np.array([N - 1]), w[a:b],
                                  k_pos=np.arange(a, b), return_partials=True)[1] for a, b in zip(cuts, cuts[1:])]
    ms = np.stack([p[0] for p in parts]); ls = np.stack([p[1] for p in parts]); os_ = np.stack([p[2] for p in parts])
    np.testing.assert_allclose(O.lse_combine(ms, ls, os_), full, atol=1e-12)


@pytest.mark.parametrize("dt", ["float16", "bfloat16"])
def test_paged_cache_bookkeeping_matches_reference(golden_dir, dt):
    d = load(golden_dir, "paged_cache.npz")
    steps = eval(str(d["steps"]))
    P, ps, L, H, D = 48, 16, 2, 2, 64
    c = O.PagedKVCacheOracle(P, ps, L, H, D, np_dtype=np.float32)
    rounder = O.round_f16 if dt == "float16" else O.round_bf16
    results = []
    for si, st in enumerate(steps):
        if st[0] == "insert":
            _, layer, T, conv = st
            kk = rounder(rnd(500 + si, (T, H, D))); vv = rounder(rnd(600 + si, (T, H, D)))
            results.append(int(c.insert_probe_kv(layer, kk, vv, conv) is not False))
        else:
            results.append(c.evict_before(st[1]))
        assert c.free_pages == list(d[f"{dt}_step{si}_free"]), si
        assert np.array_equal(c.page_valid, d[f"{dt}_step{si}_valid"]), si
        assert np.array_equal(c.page_positions, d[f"{dt}_step{si}_pos"]), si
        if si == 6:
            for layer in range(L):
                K, V = c.get_layer_kv(layer)
                assert np.array_equal(K, d[f"{dt}_mid_layer{layer}_K"])
                assert np.array_equal(V, d[f"{dt}_mid_layer{layer}_V"])
    assert results == list(d[f"{dt}_results"])
    for layer in range(L):
        K, V = c.get_layer_kv(layer)
        assert np.array_equal(K, d[f"{dt}_layer{layer}_K"]) and np.array_equal(V, d[f"{dt}_layer{layer}_V"])
    st = c.get_stats()
    ref = d[f"{dt}_stats"]
    assert [st["total_pages"], st["active_pages"], st["free_pages"], st["active_tokens"]] == list(ref[:4].astype(int))
    assert [st["total_evictions"], st["total_insertions"]] == list(ref[5:].astype(int))


def test_hip_evict_kats():
    """kessie_kernels_v2.hip:1008-1023 (64 of 128) and kessie_hip_build.py smoke (32)."""
    valid = np.zeros(256, np.int8); pos = np.zeros(256, np.int32)
    valid[:128] = 1; pos[:128] = np.arange(128) * 128
    assert O.page_evict(valid, pos, 8192)[1] == 64
    valid2 = np.zeros(64, np.int8); valid2[:] = 1; pos2 = np.arange(64, dtype=np.int32) * 128
    assert O.page_evict(valid2, pos2, 4096)[1] == 32


def test_group_decode_fp32_equals_rows():
    rng = np.random.default_rng(9)
    q = rng.standard_normal((8, 128)).astype(np.float32)
    k = rng.standard_normal((3000, 128)).astype(np.float32); v = rng.standard_normal((3000, 128)).astype(np.float32)
    w = O.fog_weights_from_clear_start(3000, 2000, 0.5)
    a = O.fog_decode_group_fp32(q, k, v, w)
    b = O.fog_attention_rows(q[:, None], k[None], v[None], np.array([2999]), w)[:, 0]
    np.testing.assert_allclose(a, b, atol=1e-5)


def test_fog_bias_values_match_reference_buffers(golden_dir):
    """The additive fog bias (kessie_attention.py:114-139) against the
    reference's torch buffers.  fp32: bit for bit.  bf16 / fp16: the golden
    ran torch's CPU arange, which for reduced types rounds each vector chunk's
    base and adds the offsets in the reduced type (4113 -> 4096 in bf16); the
    reference runs this buffer on the query's device, whose arange rounds every
    element (4113 -> 4128), and that is the definition followed here.  Where
    the two aranges differ the bias differs by at most one ulp of the dtype at
    the bias magnitude; elsewhere it is bit for bit."""
    import ast
    d = np.load(os.path.join(golden_dir, "fog_bias.npz"))
    cases = ast.literal_eval(str(d["cases"]))
    ulp = {"bfloat16": 2.0 ** -8, "float16": 2.0 ** -11}
    for ci, (n, alpha, fs, rec, boost) in enumerate(cases):
        for dn in ("float32", "bfloat16", "float16"):
            with np.errstate(over="ignore", invalid="ignore"):
                got = O.fog_bias_values(n, alpha, fs, rec, boost, dn)
            want = d[f"case{ci}_{dn}"]
            if dn == "float32":
                np.testing.assert_array_equal(got, want, err_msg=f"case {ci} {dn}")
                continue
            same = (got == want) | (np.isinf(got) & np.isinf(want) & (np.sign(got) == np.sign(want)))
            finite = np.isfinite(want) & np.isfinite(got)
            diff = np.abs(got[finite] - want[finite])
            assert diff.max(initial=0.0) <= ulp[dn], f"case {ci} {dn}: {diff.max()}"
            assert (~same).mean() < 0.05, f"case {ci} {dn}: {(~same).mean()}"
            # the two aranges agree below 256 (bf16) / 2048 (fp16): bit for bit there
            k = min(n, 256 if dn == "bfloat16" else 2048)
            np.testing.assert_array_equal(got[:k], want[:k], err_msg=f"case {ci} {dn} head")


def test_index_query_matches_vector_index(golden_dir):
    """Top-k ids and cosine scores of VectorIndex.search (kessie_exp3.py:58-110)
    from the oracle over the VectorIndex-normalised rows."""
    d = np.load(os.path.join(golden_dir, "index_query.npz"))
    n, dim, seed = (int(x) for x in d["cfg"])
    mat = np.random.default_rng(seed).standard_normal((n, dim), dtype=np.float32)
    mat[7] = 0.0
    rows = O.vector_index_rows(mat)
    for qi in range(3):
        q = np.random.default_rng(seed + 1 + qi).standard_normal((dim,), dtype=np.float32)
        _, ids, scores = O.index_query(q, rows, normalize_rows=False, top_k=10)
        np.testing.assert_array_equal(ids, d[f"q{qi}_ids"])
        np.testing.assert_allclose(scores, d[f"q{qi}_scores"], rtol=1e-5, atol=1e-6)
    assert int(d["tiny_query_result_len"]) == 0      # VectorIndex returns nothing for a ~zero query


def test_vector_index_search_fp32_reproduces_reference(golden_dir):
    """The timed CPU baseline of the index query is the reference's own numpy
    search: same ids and scores as the recorded VectorIndex.search results."""
    d = np.load(os.path.join(golden_dir, "index_query.npz"))
    n, dim, seed = (int(v) for v in d["cfg"])
    mat = np.random.default_rng(seed).standard_normal((n, dim), dtype=np.float32)
    mat[7] = 0.0
    rows = O.vector_index_rows(mat)
    for qi in range(3):
        q = np.random.default_rng(seed + 1 + qi).standard_normal((dim,), dtype=np.float32)
        ids, scores = O.vector_index_search_fp32(rows, q, 10)
        np.testing.assert_array_equal(ids, d[f"q{qi}_ids"])
        np.testing.assert_allclose(scores, d[f"q{qi}_scores"], rtol=1e-6)
    assert len(O.vector_index_search_fp32(rows, np.full(dim, 1e-12, np.float32), 10)[0]) == int(d["tiny_query_result_len"])


def test_mirror_rope_remap_ref_equals_the_reference_checker(golden_dir):
    """The mirror module's _rope_remap_ref gives the reference checker's own
    numbers (kessie_hip_kernels.py:596-606), fp32 view behaviour included:
    checked against the golden outputs the reference produced."""
    import torch
    from kessie_b200 import kessie_hip_kernels as K
    d = load(golden_dir, "rope_remap.npz")
    for i in range(5):
        dt = str(d[f"case{i}_dtype"])
        theta = float(d[f"case{i}_meta"][4])
        kin = d[f"case{i}_kin"]
        tdt = {"float32": torch.float32, "float16": torch.float16, "bfloat16": torch.bfloat16}[dt]
        k = torch.from_numpy(np.ascontiguousarray(kin, dtype=np.float32)).to(tdt)
        out = K._rope_remap_ref(k, torch.from_numpy(d[f"case{i}_orig"].astype(np.int32)),
                                torch.from_numpy(d[f"case{i}_tgt"].astype(np.int32)), theta)
        np.testing.assert_array_equal(out.float().numpy(), d[f"case{i}_kout"], err_msg=f"case {i} ({dt})")
