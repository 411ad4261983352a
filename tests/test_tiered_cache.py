"""HF tiered KV cache (KeSSieCache, kessie_exp3.py:342-627).

CPU: the oracle (oracle/tiered_cache_oracle.py) replays the golden schedule
recorded from the reference class and matches its returned fogged V, K and
bookkeeping.  GPU: kessie_b200.kessie_cache.KeSSieCache replays the same
schedule (tiered-update kernel, strided pack / unpack on evict and recall) and
matches the golden values bit for bit where the fog weights take torch's
exact routes (sqrt, fog off) and within 1 fp32 ulp-level tolerance with
pow(); plus relayout, fog-boundary, multi-token and fp16 cases against the
oracle."""

import json
import os

import numpy as np
import pytest
import torch

from oracle import fog_oracle as FO
from oracle.tiered_cache_oracle import TieredCacheModel, tiered_fog_weights

CASES = {"bf16_a05": ("bfloat16", 0.5, 0.5), "f32_a07": ("float32", 0.7, 0.3), "bf16_off": ("bfloat16", 0.0, 0.5)}
LAYERS, WINDOW, (B, H, D) = 3, 48, (1, 2, 32)


def _rnd(seed, shape):
    return np.random.default_rng(seed).standard_normal(shape, dtype=np.float32)


def _golden(golden_dir):
    return np.load(os.path.join(golden_dir, "tiered_cache.npz"))


def _unpack(a, dt):
    return FO.bf16_bits_to_f32(a) if dt == "bfloat16" else np.asarray(a, np.float32)


def _inputs(seed, T, layer, dt):
    k = FO._ROUND[dt](_rnd(seed + layer, (B, H, T, D)))
    v = FO._ROUND[dt](_rnd(seed + 50 + layer, (B, H, T, D)))
    return k, v


def _replay(schedule, dt, update, evict, recall, record):
    rec = 0
    last = None
    for op in schedule:
        if op[0] == "u":
            last = [update(*_inputs(op[2], op[1], l, dt), l) for l in range(LAYERS)]
        elif op[0] == "e":
            evict()
        elif op[0] == "r":
            record(("recall", op[1], recall(op[1])))
        elif op[0] == "rec":
            record(("rec", rec, last))
            rec += 1


def _check_stats(got, want):
    for key in ("kv_seq_len", "kv_window_start", "kv_layers", "kv_gpu_bytes", "kv_cpu_chunks", "kv_cpu_tokens",
                "fog_tokens", "clear_tokens", "total_evictions", "total_recalls", "cpu_kv_bytes", "seen_tokens"):
        assert got[key] == want[key], (key, got[key], want[key])


@pytest.mark.parametrize("tag", list(CASES))
def test_oracle_matches_reference_schedule(golden_dir, tag):
    g = _golden(golden_dir)
    dt, alpha, fstart = CASES[tag]
    schedule = json.loads(str(g["schedule"]))
    want_stats = json.loads(str(g[f"{tag}_stats"]))
    m = TieredCacheModel(WINDOW, alpha, fstart, dt)
    events = []
    _replay(schedule, dt, m.update, m.evict_if_needed, m.recall_from_cpu,
            lambda ev: events.append((ev, m.stats(), [[s, e] for s, e, _ in m.cpu_kv_store])))
    for si, (ev, st, chunks) in enumerate(events):
        want = want_stats[si]
        if ev[0] == "recall":
            assert ev[2] == want["ok"]
            continue
        _, r, last = ev
        np.testing.assert_array_equal(last[0][0], _unpack(g[f"{tag}_r{r}_l0_k"], dt))
        for l in range(LAYERS):
            got_v, want_v = last[l][1], _unpack(g[f"{tag}_r{r}_l{l}_v"], dt)
            if alpha in (0.0, 0.5):
                np.testing.assert_array_equal(got_v, want_v)
            else:
                np.testing.assert_allclose(got_v, want_v, rtol=1e-6, atol=1e-7)
        _check_stats(st, want)
        assert chunks == want["chunks"]


def test_oracle_fog_boundary_uses_double_fog_start():
    # int(S * fog_start) in double: S = 10, fog_start = 0.7 -> cc = 7, fc = 3
    w = tiered_fog_weights(10, 0.5, 0.7)
    assert (w[3:] == 1).all() and w[2] == 1.0 and w[0] == np.float32(0.01)
    assert tiered_fog_weights(1, 0.5, 0.5) is None and tiered_fog_weights(5, 0.0, 0.5) is None


# ----------------------------------------------------------------- GPU
def _to_dev(a, dt):
    return torch.from_numpy(a).to(getattr(torch, dt)).cuda()


def _np(t):
    return t.float().cpu().numpy()


@pytest.mark.gpu
@pytest.mark.parametrize("tag", list(CASES))
def test_gpu_cache_replays_reference_schedule(golden_dir, tag):
    from kessie_b200.kessie_cache import KeSSieCache
    g = _golden(golden_dir)
    dt, alpha, fstart = CASES[tag]
    schedule = json.loads(str(g["schedule"]))
    want_stats = json.loads(str(g[f"{tag}_stats"]))
    c = KeSSieCache(window_size=WINDOW, fog_alpha=alpha, fog_start=fstart)
    m = TieredCacheModel(WINDOW, alpha, fstart, dt)
    events = []

    def record(ev):
        st = c.get_stats() | {"cpu_kv_bytes": c.cpu_kv_bytes, "seen_tokens": c.seen_tokens}
        events.append((ev, st, [[s, e] for s, e, _ in c.cpu_kv_store]))

    def update(k, v, l):
        m.update(k, v, l)
        ko, vo = c.update(_to_dev(k, dt), _to_dev(v, dt), l)
        return _np(ko), _np(vo)

    def recall(pos):
        m.recall_from_cpu(pos)
        return c.recall_from_cpu(pos, "cuda")

    def evict():
        m.evict_if_needed()
        c.evict_if_needed()

    _replay(schedule, dt, update, evict, recall, record)
    torch.cuda.synchronize()
    for si, (ev, st, chunks) in enumerate(events):
        want = want_stats[si]
        if ev[0] == "recall":
            assert ev[2] == want["ok"]
            continue
        _check_stats(st, want)
        assert chunks == want["chunks"]
        _, r, last = ev
        np.testing.assert_array_equal(last[0][0], _unpack(g[f"{tag}_r{r}_l0_k"], dt))
        for l in range(LAYERS):
            got_v, want_v = last[l][1], _unpack(g[f"{tag}_r{r}_l{l}_v"], dt)
            if alpha in (0.0, 0.5):
                np.testing.assert_array_equal(got_v, want_v)
            else:
                np.testing.assert_allclose(got_v, want_v, rtol=2e-6, atol=1e-7)
    st = c.get_stats()
    _check_stats(st | {"cpu_kv_bytes": c.cpu_kv_bytes, "seen_tokens": c.seen_tokens}, m.stats())
    assert [(s, e) for s, e, _ in c.cpu_kv_store] == [(s, e) for s, e, _ in m.cpu_kv_store]
    for l in range(LAYERS):                       # raw windows and the stored chunks
        np.testing.assert_array_equal(_np(c.key_cache[l]), m.key_cache[l])
        np.testing.assert_array_equal(_np(c.value_cache[l]), m.value_cache[l])
        for (_, _, cl), (_, _, ml) in zip(c.cpu_kv_store, m.cpu_kv_store):
            np.testing.assert_array_equal(cl[l][0].float().numpy(), ml[l][0])
            np.testing.assert_array_equal(cl[l][1].float().numpy(), ml[l][1])


@pytest.mark.gpu
@pytest.mark.parametrize("dt,alpha,fstart", [("float16", 0.5, 0.7), ("bfloat16", 1.0, 0.7), ("float32", 2.0, 0.25),
                                             ("bfloat16", 1.3, 0.5)])
def test_gpu_cache_relayout_recall_and_boundaries(dt, alpha, fstart):
    """Prefill longer than twice the window, decode with evictions, recall of
    the older chunk after a newer one (no room in front: relayout), a miss,
    reset, and fog boundaries where int(S * fog_start) depends on double
    precision (fog_start 0.7).  Weights off torch's exact routes (pow) may
    differ by an fp32 ulp, which can move a bf16 / fp16 rounding: those cases
    use the dtype's bar."""
    from kessie_b200.kessie_cache import KeSSieCache
    w, L, Bb, Hh, Dd = 16, 2, 2, 3, 64
    c = KeSSieCache(window_size=w, fog_alpha=alpha, fog_start=fstart)
    m = TieredCacheModel(w, alpha, fstart, dt)
    if alpha in (0.5, 1.0, 2.0):
        tol = dict(rtol=0, atol=0)
    else:
        tol = dict(rtol=2e-6, atol=1e-7) if dt == "float32" else dict(rtol=1e-2, atol=2e-2)
    rng = np.random.default_rng(9)

    def step(T):
        for l in range(L):
            k = FO._ROUND[dt](rng.standard_normal((Bb, Hh, T, Dd), dtype=np.float32))
            v = FO._ROUND[dt](rng.standard_normal((Bb, Hh, T, Dd), dtype=np.float32))
            mk, mv = m.update(k, v, l)
            ck, cv = c.update(_to_dev(k, dt), _to_dev(v, dt), l)
            np.testing.assert_array_equal(_np(ck), mk)
            np.testing.assert_allclose(_np(cv), mv, **tol)

    step(40)                                  # 40 > 2w: evicts 24 at the first check
    c.evict_if_needed(); m.evict_if_needed()
    for _ in range(20):
        step(1)
        c.evict_if_needed(); m.evict_if_needed()
    assert len(c.cpu_kv_store) == len(m.cpu_kv_store) >= 2
    first = c.cpu_kv_store[0][0]
    assert c.recall_from_cpu(first, "cuda") and m.recall_from_cpu(first)   # older chunk first
    step(3)
    assert not c.recall_from_cpu(10 ** 9, "cuda")
    st_c, st_m = c.get_stats(), m.stats()
    assert st_c["kv_seq_len"] == st_m["kv_seq_len"] and c.window_start == m.window_start
    assert c.cpu_kv_bytes == m.cpu_kv_bytes and c.total_recalls == m.total_recalls
    for l in range(L):
        np.testing.assert_array_equal(_np(c.key_cache[l]), m.key_cache[l])
        np.testing.assert_array_equal(_np(c.value_cache[l]), m.value_cache[l])
    c.reset()
    assert c.get_seq_length() == 0 and c.cpu_kv_store == [] and c.cpu_kv_bytes == 0


@pytest.mark.gpu
def test_gpu_cache_kv_dtype_cast_and_strided_input():
    """kv_cache_dtype casts the incoming states; states given as a transposed
    view ([B, T, H, D] -> [B, H, T, D]) are read through their strides."""
    from kessie_b200.kessie_cache import KeSSieCache
    c = KeSSieCache(window_size=32, fog_alpha=0.5, fog_start=0.5, kv_cache_dtype=torch.bfloat16)
    m = TieredCacheModel(32, 0.5, 0.5, "bfloat16")
    rng = np.random.default_rng(4)
    for T in (20, 1, 1, 7):
        k = rng.standard_normal((1, T, 4, 128), dtype=np.float32)
        v = rng.standard_normal((1, T, 4, 128), dtype=np.float32)
        kt = torch.from_numpy(k).cuda().transpose(1, 2)             # fp32 strided view
        vt = torch.from_numpy(v).cuda().transpose(1, 2)
        ck, cv = c.update(kt, vt, 0)
        mk, mv = m.update(FO.round_bf16(k.transpose(0, 2, 1, 3)), FO.round_bf16(v.transpose(0, 2, 1, 3)), 0)
        assert ck.dtype == torch.bfloat16
        np.testing.assert_array_equal(_np(ck), mk)
        np.testing.assert_array_equal(_np(cv), mv)


def test_host_bookkeeping_matches_reference(golden_dir):
    """append_conversation overflow (index positions and turn boundaries shift
    or drop; a turn longer than the cap keeps all its tokens, as the
    reference does), get_turn_for_position, get_token_distance, the seeded
    projection and get_stats of a cache holding no KV (kessie_exp3.py:535-608)
    against the reference class's recorded values."""
    from kessie_b200.kessie_cache import KeSSieCache
    with open(os.path.join(golden_dir, "tiered_bookkeeping.json")) as f:
        g = json.load(f)
    c = KeSSieCache(window_size=64, fog_alpha=0.5, fog_start=0.25, max_conversation_tokens=50)
    plan = [(list(range(0, 20)), "user"), (list(range(20, 45)), "assistant"), (list(range(45, 70)), "user"),
            (list(range(70, 72)), "assistant"), (list(range(72, 140)), "user")]
    for i, ((tids, role), want) in enumerate(zip(plan, g["steps"])):
        if i == 1:
            c.index_embeddings = [np.full(4, k, np.float32) for k in range(3)]
            c.index_positions = [5, 30, 44]
        c.append_conversation(tids, role)
        assert c.conversation_tokens == want["conversation_tokens"]
        assert c.index_positions == want["index_positions"]
        assert [float(e[0]) for e in c.index_embeddings] == want["index_embeddings"]
        assert [list(t) for t in c.turn_boundaries] == want["turn_boundaries"]
        assert {str(p): list(c.get_turn_for_position(p)) for p in (-1, 0, 4, 5, 24, 25, 30, 49, 100)} == want["turns"]
        assert {str(p): c.get_token_distance(p) for p in (0, 10, 49)} == want["distance"]
        assert c.get_stats() == want["stats"]
    np.testing.assert_allclose(c._get_projection(64, 16), np.array(g["projection_64_16"]), rtol=0, atol=1e-7)
    c.full_reset()
    assert c.get_stats() == g["after_full_reset"]


def test_host_guards_without_gpu():
    """The product path refuses CPU tensors instead of computing on the CPU;
    an empty cache behaves as the reference's (length 0, eviction no-op,
    recall miss); the ops wrappers check their buffers before launching."""
    from kessie_b200 import ops
    from kessie_b200.kessie_cache import KeSSieCache
    from kessie_b200.vector_index import VectorIndex
    c = KeSSieCache(window_size=8)
    assert c.get_seq_length() == 0 and len(c) == 0
    c.evict_if_needed()
    assert c.recall_from_cpu(3, "cpu") is False
    k = torch.zeros(1, 2, 4, 32, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError):
        c.update(k, k, 0)
    with pytest.raises(ValueError):
        ops.tiered_update(k, k, 0, 0, k, k, None, 0.5, 0.5)
    with pytest.raises(ValueError):
        ops.index_query(torch.zeros(8), torch.zeros(4, 8))
    vi = VectorIndex(dim=8)
    assert vi.search(np.ones(8, np.float32)) == [] and vi.count == 0
    vi.rebuild([], [])
    if not torch.cuda.is_available():
        with pytest.raises(RuntimeError):
            vi.rebuild([np.ones(8, np.float32)], [1])


@pytest.mark.gpu
@pytest.mark.parametrize("layers,pattern", [(1, "in_order"), (2, "in_order"), (5, "in_order"), (3, "repeat_first")])
def test_gpu_back_to_back_updates(layers, pattern):
    """Decode steps enqueued with no other kernel and no synchronisation in
    between, as a model's update loop runs: each update may start reading its
    V store while the previous update drains, which is allowed only when that
    update wrote another store.  One layer (every update follows one of the
    same layer), two layers (A B A B: the update before the previous one wrote
    this store) and a repeated layer in the order all end bit-exact."""
    from kessie_b200.kessie_cache import KeSSieCache
    Bq, Hh, Dd, S0, steps = 1, 8, 128, 3000, 12
    order = list(range(layers)) if pattern == "in_order" else [0, 0] + list(range(1, layers))
    c = KeSSieCache(window_size=4096, fog_alpha=0.5, fog_start=0.5)
    m = TieredCacheModel(4096, 0.5, 0.5, "bfloat16")
    rng = np.random.default_rng(17)
    rnd = lambda T: FO.round_bf16(rng.standard_normal((Bq, Hh, T, Dd), dtype=np.float32))
    for l in range(layers):
        k, v = rnd(S0), rnd(S0)
        m.update(k, v, l)
        c.update(_to_dev(k, "bfloat16"), _to_dev(v, "bfloat16"), l)
    host = [[(rnd(1), rnd(1)) for _ in order] for _ in range(steps)]
    dev = [[(_to_dev(k, "bfloat16"), _to_dev(v, "bfloat16")) for k, v in row] for row in host]
    torch.cuda.synchronize()
    last = {}
    for row in dev:                                # no host sync and no other kernel in between
        for l, (k, v) in zip(order, row):
            last[l] = c.update(k, v, l)
    want = {}
    for row in host:
        for l, (k, v) in zip(order, row):
            want[l] = m.update(k, v, l)
    torch.cuda.synchronize()
    for l in range(layers):
        np.testing.assert_array_equal(_np(last[l][0]), want[l][0])
        np.testing.assert_array_equal(_np(last[l][1]), want[l][1])
        np.testing.assert_array_equal(_np(c.value_cache[l]), m.value_cache[l])
