"""Generate the golden vectors under tests/golden/ from the REFERENCE itself.

Runs the sentinelXVI/KeSSie Python reference functions (kessie_hip_kernels.py:
kessie_build_fog_weights, kessie_windowed_attention_ref,
kessie_fused_fog_attention_ref, _rope_remap_ref, KeSSiePagedKVCache) on
seeded numpy inputs and stores their outputs.  Inputs are not stored when
they can be regenerated from the recorded seed (numpy PCG64 standard_normal
is stable across numpy versions); the oracle tests regenerate them.

Needs the reference source tree, named by $KESSIE_REF; it is run once where
that tree exists and its outputs are committed.  Nothing on the GPU box runs
this script.

    KESSIE_REF=<reference tree> python tests/golden/make_golden.py
"""

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REF = os.environ.get("KESSIE_REF")
if not REF or not os.path.exists(os.path.join(REF, "kessie_hip_kernels.py")):
    sys.exit("make_golden.py: set KESSIE_REF to the reference source tree (kessie_hip_kernels.py not found)")
sys.dont_write_bytecode = True
sys.path.insert(0, REF)

import torch  # noqa: E402

import kessie_hip_kernels as R  # noqa: E402

R.HAS_TRITON = False   # the Triton branches need a GPU driver; the refs are torch-only
torch.set_num_threads(os.cpu_count() or 1)


def rnd(seed, shape):
    return np.random.default_rng(seed).standard_normal(shape, dtype=np.float32)


def to_bf16_vals(x):
    return torch.from_numpy(x).to(torch.bfloat16).float().numpy()


def save(name, **arrs):
    np.savez_compressed(os.path.join(HERE, name), **arrs)
    print("wrote", name, {k: getattr(v, "shape", v) for k, v in arrs.items()})


def gen_fog():
    cases = [(4096, 0.5, 512 / 4096), (4096, 0.5, 0.5), (1000, 0.7, 0.3), (17, 1.5, 0.9),
             (512, 0.0, 0.5), (64, 0.5, 1.0), (64, 0.5, 0.0),
             (131072, 0.5, 4096 / 131072), (1048576, 0.5, 8192 / 1048576), (262144, 0.5, 4096 / 262144)]
    out = {}
    for i, (n, a, fs) in enumerate(cases):
        w = R.kessie_build_fog_weights(n, a, fs).numpy()
        idx = np.arange(n) if n <= 4096 else np.unique(np.concatenate(
            [np.arange(64), np.arange(n - 64, n), np.random.default_rng(i).integers(0, n, 4096)]))
        out[f"case{i}_params"] = np.array([n, a, fs], dtype=np.float64)
        out[f"case{i}_idx"] = idx.astype(np.int64)
        out[f"case{i}_w"] = w[idx]
        out[f"case{i}_clear_start"] = np.array(int(n * (1.0 - fs)))
    out["ncases"] = np.array(len(cases))
    save("fog_weights.npz", **out)


def gen_rope():
    out = {}
    for theta in (10000.0, 500000.0):
        for half in (32, 64):
            f = 1.0 / (theta ** (torch.arange(half, dtype=torch.float32) / half))
            out[f"freqs_{int(theta)}_{half}"] = f.numpy()
    cases = [
        # seed, T, H, D, dtype, theta, position mode
        (11, 64, 2, 128, "float32", 10000.0, "small"),
        (12, 64, 2, 128, "bfloat16", 500000.0, "recall"),
        (13, 48, 3, 64, "float16", 10000.0, "small"),
        (14, 32, 2, 128, "bfloat16", 10000.0, "neg"),
        (15, 16, 8, 128, "float16", 500000.0, "recall"),
    ]
    for i, (seed, T, H, D, dt, theta, mode) in enumerate(cases):
        rng = np.random.default_rng(seed + 1000)
        if mode == "small":
            orig = rng.integers(0, 4096, T); tgt = rng.integers(0, 4096, T)
        elif mode == "recall":
            orig = rng.integers(0, 32768, T); tgt = 131072 + np.arange(T)
        else:
            orig = rng.integers(100000, 131072, T); tgt = rng.integers(0, 1000, T)
        tdt = getattr(torch, dt)
        k = torch.from_numpy(rnd(seed, (T, H, D))).to(tdt)
        kin = k.float().numpy().copy()
        R._rope_remap_ref(k, torch.from_numpy(orig.astype(np.int32)),
                          torch.from_numpy(tgt.astype(np.int32)), theta)
        out[f"case{i}_meta"] = np.array([seed, T, H, D, theta], dtype=np.float64)
        out[f"case{i}_dtype"] = np.array(dt)
        out[f"case{i}_orig"] = orig.astype(np.int32)
        out[f"case{i}_tgt"] = tgt.astype(np.int32)
        out[f"case{i}_kin"] = kin
        out[f"case{i}_kout"] = k.float().numpy()
    out["ncases"] = np.array(len(cases))
    # reference self-test KATs (kessie_hip_kernels.py:662-683): round trip and identity
    k = torch.from_numpy(rnd(16, (64, 8, 128))).half()
    k0 = k.clone()
    o = torch.arange(100, 164, dtype=torch.int32); t = torch.arange(5000, 5064, dtype=torch.int32)
    R._rope_remap_ref(k, o, t); R._rope_remap_ref(k, t, o)
    out["kat_roundtrip_maxdiff"] = np.array((k0.float() - k.float()).abs().max().item())
    save("rope_remap.npz", **out)


def gen_attention():
    out = {}
    # the reference's own windowed-attention test configs (kessie_hip_kernels.py:623-626)
    cfgs = [(1, 4, 128, 64, 0, True), (1, 4, 128, 64, 64, True), (1, 8, 256, 128, 128, True),
            (2, 8, 512, 128, 256, True), (1, 2, 96, 64, 0, False), (1, 2, 80, 128, 24, False)]
    for i, (Z, H, N, D, W, causal) in enumerate(cfgs):
        seed = 100 + i
        q, k, v = (torch.from_numpy(rnd(seed + j, (Z, H, N, D))) for j in range(3))
        o = R.kessie_windowed_attention_ref(q, k, v, W, causal).numpy()
        rows = np.unique(np.concatenate([np.arange(0, N, 7), [N - 1]]))
        out[f"win{i}_cfg"] = np.array([Z, H, N, D, W, int(causal), seed])
        out[f"win{i}_rows"] = rows
        out[f"win{i}_out"] = o[:, :, rows]
    out["nwin"] = np.array(len(cfgs))
    # fused fog test (kessie_hip_kernels.py:647-652) plus windowed/bidirectional variants
    fcfgs = [(1, 8, 512, 128, 0.5, 0.5, 0, True), (1, 2, 256, 64, 0.7, 0.25, 64, True),
             (1, 2, 128, 128, 0.5, 0.5, 0, False)]
    for i, (Z, H, N, D, a, fs, W, causal) in enumerate(fcfgs):
        seed = 200 + i
        q, k, v = (torch.from_numpy(rnd(seed + j, (Z, H, N, D))) for j in range(3))
        fog = R.kessie_build_fog_weights(N, a, fs)
        o = R.kessie_fused_fog_attention_ref(q, k, v, fog, W, causal).numpy()
        rows = np.unique(np.concatenate([np.arange(0, N, 5), [N - 1]]))
        out[f"fog{i}_cfg"] = np.array([Z, H, N, D, W, int(causal), seed])
        out[f"fog{i}_fog"] = np.array([a, fs])
        out[f"fog{i}_rows"] = rows
        out[f"fog{i}_out"] = o[:, :, rows]
    out["nfog"] = np.array(len(fcfgs))
    save("attention.npz", **out)


def gen_config1():
    """Benchmark config 1: B1 Hq8/Hkv2 D128 N4096 W512 fp32, RoPE theta 1e4 at
    positions 0..4095, decode query = position 4095.  GQA by repeat_interleave.
    Two fog mappings: (a) causal + clear_start = N-W; (b) reference-literal
    window_size=W mask plus the same fog weights."""
    B, Hq, Hkv, D, N, W = 1, 8, 2, 128, 4096, 512
    seed = 301
    q = torch.from_numpy(rnd(seed, (N, Hq, D)))
    k = torch.from_numpy(rnd(seed + 1, (N, Hkv, D)))
    v = torch.from_numpy(rnd(seed + 2, (N, Hkv, D)))
    pos = torch.arange(N, dtype=torch.int32)
    zero = torch.zeros(N, dtype=torch.int32)
    # _rope_remap_ref on an fp32 tensor aliases k1 (``.float()`` returns the
    # same storage, kessie_hip_kernels.py:603-605), so rotate float64 copies:
    # the arithmetic is still fp32, the results are exact in float64.
    q = R._rope_remap_ref(q.double(), zero, pos, 10000.0).float()
    k = R._rope_remap_ref(k.double(), zero, pos, 10000.0).float()
    qf = q.permute(1, 0, 2)[None]                                  # [1,Hq,N,D]
    kf = k.permute(1, 0, 2)[None].repeat_interleave(Hq // Hkv, dim=1)
    vf = v.permute(1, 0, 2)[None].repeat_interleave(Hq // Hkv, dim=1)
    fog = R.kessie_build_fog_weights(N, 0.5, W / N)
    oa = R.kessie_fused_fog_attention_ref(qf, kf, vf, fog, 0, True)[0, :, -1].numpy()
    ob = R.kessie_fused_fog_attention_ref(qf, kf, vf, fog, W, True)[0, :, -1].numpy()
    save("config1_decode.npz", cfg=np.array([B, Hq, Hkv, D, N, W, seed]),
         q_rot_last=q[-1].numpy(), k_rot_sample=k[::257].numpy(),
         out_causal_fog=oa, out_window_fog=ob, clear_start=np.array(int(N * (1.0 - W / N))))


def gen_paged():
    """KeSSiePagedKVCache bookkeeping (kessie_hip_kernels.py:484-570) driven on
    CPU.  evict_before's no-Triton branch never clears page_valid, so the
    device rule of kessie_kernels_v2.hip:403-406 is applied to page_valid
    first; the reference's own Python scan then rebuilds free_pages."""
    out = {}
    for dt_name in ("float16", "bfloat16"):
        dt = getattr(torch, dt_name)
        P, ps, L, H, D = 48, 16, 2, 2, 64
        c = R.KeSSiePagedKVCache(P, ps, L, H, D, torch.device("cpu"), dtype=dt)
        log = []
        steps = [("insert", 0, 40, 0), ("insert", 1, 100, 40), ("insert", 0, 16, 1000),
                 ("evict", 48), ("insert", 1, 33, 2000), ("evict", 1001), ("insert", 0, 200, 3000),
                 ("insert", 0, 700, 5000), ("evict", 100000), ("insert", 1, 5, 7)]
        for si, st in enumerate(steps):
            if st[0] == "insert":
                _, layer, T, conv = st
                kk = torch.from_numpy(rnd(500 + si, (T, H, D))).to(dt)
                vv = torch.from_numpy(rnd(600 + si, (T, H, D))).to(dt)
                ok = c.insert_probe_kv(layer, kk, vv, conv)
                log.append(int(ok))
            else:
                thr = st[1]
                hit = (c.page_valid == 1) & (c.page_positions < thr)
                c.page_valid[hit] = 0
                log.append(c.evict_before(thr))
            out[f"{dt_name}_step{si}_free"] = np.array(c.free_pages, dtype=np.int32)
            out[f"{dt_name}_step{si}_valid"] = c.page_valid.numpy().copy()
            out[f"{dt_name}_step{si}_pos"] = c.page_positions.numpy().copy()
            if si == 6:
                for layer in range(L):
                    K, V = c.get_layer_kv(layer)
                    out[f"{dt_name}_mid_layer{layer}_K"] = K.float().numpy()
                    out[f"{dt_name}_mid_layer{layer}_V"] = V.float().numpy()
        for layer in range(L):
            K, V = c.get_layer_kv(layer)
            out[f"{dt_name}_layer{layer}_K"] = K.float().numpy()
            out[f"{dt_name}_layer{layer}_V"] = V.float().numpy()
        out[f"{dt_name}_results"] = np.array(log)
        st = c.get_stats()
        out[f"{dt_name}_stats"] = np.array([st["total_pages"], st["active_pages"], st["free_pages"],
                                            st["active_tokens"], st["vram_gb"], st["total_evictions"],
                                            st["total_insertions"]], dtype=np.float64)
    out["steps"] = np.array(repr(steps))
    save("paged_cache.npz", **out)


def gen_kv_store():
    """KeSSieCPUKVStore bookkeeping (kessie_kv_connector.py:65-229) on CPU."""
    import json
    import kessie_kv_connector as C
    sys.path.insert(0, HERE)
    from kv_store_script import run_kv_store_script
    log = run_kv_store_script(C.KeSSieCPUKVStore, C, torch)
    with open(os.path.join(HERE, "kv_store.json"), "w") as f:
        json.dump(log, f, indent=0)
    print("wrote kv_store.json", len(log), "steps")


FOG_BIAS_CASES = [  # (kv_len, fog_alpha, fog_start, recall positions, recall_boost)
    (128, 0.5, 0.5, [], 0.1),
    (128, 0.5, 0.5, [10, 50, 100], 0.1),
    (256, 0.8, 0.3, [5], 0.1),
    (4096, 0.5, 0.5, [100, 200, 300], 0.1),
    (131072, 0.5, 0.03125, [1000, 70000, 130000], 0.25),
    (1000, 0.0, 0.5, [3], 0.1),
    (777, 1.3, 0.9, [0, 776, 800], 0.5),
    (50000, 0.5, 0.5, [], 0.1),
]


def gen_fog_bias():
    """_FogCache._compute_into (kessie_attention.py:114-139): the additive fog
    bias of the vLLM path, in buffers of each dtype."""
    import kessie_attention as A
    A._torch = torch
    out = {}
    for ci, (n, alpha, fs, rec, boost) in enumerate(FOG_BIAS_CASES):
        for dn in ("float32", "bfloat16", "float16"):
            buf = torch.zeros(n + 7, dtype=getattr(torch, dn))
            A._FogCache._compute_into(buf, n, alpha, fs, set(rec), boost)
            out[f"case{ci}_{dn}"] = buf[:n].float().numpy()
    out["cases"] = np.array(repr(FOG_BIAS_CASES))
    save("fog_bias.npz", **out)


def gen_index_query():
    """VectorIndex.search (kessie_exp3.py:58-110, numpy path): top-k ids and
    cosine scores over a seeded index (row 7 all zero: the norm guard)."""
    import kessie_exp3 as E
    n, dim, seed = 20000, 256, 77
    mat = rnd(seed, (n, dim))
    mat[7] = 0.0
    vi = E.VectorIndex(dim=dim)
    vi.rebuild([mat[i] for i in range(n)], list(range(n)))
    out = {"cfg": np.array([n, dim, seed])}
    for qi in range(3):
        q = rnd(seed + 1 + qi, (dim,))
        res = vi.search(q, top_k=10)
        out[f"q{qi}_ids"] = np.array([r[0] for r in res], dtype=np.int64)
        out[f"q{qi}_scores"] = np.array([r[1] for r in res], dtype=np.float64)
    out["tiny_query_result_len"] = np.array(len(vi.search(np.full(dim, 1e-12, np.float32), top_k=10)))
    save("index_query.npz", **out)


# Tiered-cache schedule (window 48, 3 layers, [1, 2, T, 32]): prefill 70,
# decode steps with an eviction check after each, recalls (one of a position
# that is not stored), a 5-token append.  ("u", T, seed) = update every layer
# with rnd(seed + layer) K and rnd(seed + 50 + layer) V; "rec" entries record
# the returned fogged V of every layer, layer 0's K and the stats (bf16 arrays
# as uint16 bit patterns).
TIERED_SCHEDULE = ([["u", 70, 100], ["rec"]] +
                   sum([[["u", 1, 200 + i], ["e"]] + ([["rec"]] if i in (0, 26, 29) else []) for i in range(30)], []) +
                   [["r", 10], ["rec"], ["u", 1, 300], ["rec"], ["e"], ["rec"], ["r", 5000], ["u", 5, 400], ["rec"],
                    ["r", 52], ["u", 1, 500], ["rec"]])
TIERED_CASES = [("bf16_a05", "bfloat16", 0.5, 0.5), ("f32_a07", "float32", 0.7, 0.3), ("bf16_off", "bfloat16", 0.0, 0.5)]
TIERED_SHAPE = (1, 2, 32)          # B, H, D
TIERED_LAYERS = 3
TIERED_WINDOW = 48


def gen_tiered_cache():
    """KeSSieCache (kessie_exp3.py:342-627) on CPU torch through TIERED_SCHEDULE."""
    import json
    import kessie_exp3 as E
    B, H, D = TIERED_SHAPE
    out = {"schedule": np.array(json.dumps(TIERED_SCHEDULE))}
    for tag, dt, alpha, fstart in TIERED_CASES:
        tdt = getattr(torch, dt)
        c = E.KeSSieCache(window_size=TIERED_WINDOW, fog_alpha=alpha, fog_start=fstart)
        last = None
        stats, rec = [], 0
        for op in TIERED_SCHEDULE:
            if op[0] == "u":
                _, T, seed = op
                last = []
                for l in range(TIERED_LAYERS):
                    k = torch.from_numpy(rnd(seed + l, (B, H, T, D))).to(tdt)
                    v = torch.from_numpy(rnd(seed + 50 + l, (B, H, T, D))).to(tdt)
                    ko, vo = c.update(k, v, l)
                    last.append((ko.float().numpy().copy(), vo.float().numpy().copy()))
            elif op[0] == "e":
                c.evict_if_needed()
            elif op[0] == "r":
                stats.append({"recall": op[1], "ok": bool(c.recall_from_cpu(op[1], "cpu"))})
            elif op[0] == "rec":
                # fogged V of every layer, K of layer 0 (K is a copy); bf16 as bit patterns
                pack = ((lambda a: torch.from_numpy(a).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16))
                        if dt == "bfloat16" else (lambda a: a))
                out[f"{tag}_r{rec}_l0_k"] = pack(last[0][0])
                for l, (ko, vo) in enumerate(last):
                    out[f"{tag}_r{rec}_l{l}_v"] = pack(vo)
                st = c.get_stats()
                stats.append({k: st[k] for k in ("kv_seq_len", "kv_window_start", "kv_layers", "kv_gpu_bytes",
                                                 "kv_cpu_chunks", "kv_cpu_tokens", "fog_tokens", "clear_tokens",
                                                 "total_evictions", "total_recalls")} |
                             {"cpu_kv_bytes": c.cpu_kv_bytes, "seen_tokens": c.seen_tokens,
                              "chunks": [[s_, e_] for s_, e_, _ in c.cpu_kv_store]})
                rec += 1
        out[f"{tag}_stats"] = np.array(json.dumps(stats))
    save("tiered_cache.npz", **out)


def gen_tiered_bookkeeping():
    """KeSSieCache's host bookkeeping (kessie_exp3.py:535-608): conversation
    overflow with index / turn shifting, turn lookups, token distances, the
    seeded projection and the stats of a cache without KV."""
    import json
    import kessie_exp3 as E
    c = E.KeSSieCache(window_size=64, fog_alpha=0.5, fog_start=0.25, max_conversation_tokens=50)
    out = {"steps": []}
    plan = [(list(range(0, 20)), "user"), (list(range(20, 45)), "assistant"), (list(range(45, 70)), "user"),
            (list(range(70, 72)), "assistant"), (list(range(72, 140)), "user")]
    for i, (tids, role) in enumerate(plan):
        if i == 1:
            c.index_embeddings = [np.full(4, k, np.float32) for k in range(3)]
            c.index_positions = [5, 30, 44]
        c.append_conversation(tids, role)
        out["steps"].append({
            "conversation_tokens": list(c.conversation_tokens),
            "index_positions": list(c.index_positions),
            "index_embeddings": [float(e[0]) for e in c.index_embeddings],
            "turn_boundaries": [list(t) for t in c.turn_boundaries],
            "turns": {str(p): list(c.get_turn_for_position(p)) for p in (-1, 0, 4, 5, 24, 25, 30, 49, 100)},
            "distance": {str(p): c.get_token_distance(p) for p in (0, 10, 49)},
            "stats": c.get_stats()})
    proj = c._get_projection(64, 16)
    out["projection_64_16"] = proj.astype(np.float64).round(7).tolist()
    c.full_reset()
    out["after_full_reset"] = c.get_stats()
    with open(os.path.join(HERE, "tiered_bookkeeping.json"), "w") as f:
        json.dump(out, f)
    print("wrote tiered_bookkeeping.json")


if __name__ == "__main__":
    gen_fog()
    gen_rope()
    gen_attention()
    gen_config1()
    gen_paged()
    gen_kv_store()
    gen_fog_bias()
    gen_index_query()
    gen_tiered_cache()
    gen_tiered_bookkeeping()
