"""Scripted operations on a KV block store (KeSSieCPUKVStore interface,
kessie_kv_connector.py:65-229) and the observations recorded after each one.
make_golden.py runs it against the reference's store to write kv_store.json;
tests/test_kv_connector.py runs it against kessie_b200's store and compares.
No reference import here."""

import numpy as np


class _Tok:
    """Tokenizer stub: ids -> text."""
    @staticmethod
    def decode(ids, skip_special_tokens=True):
        return " ".join(str(i) for i in ids)


def kv_store_embed(text):
    """Deterministic 16-d embedding of a text (shared with the test)."""
    import hashlib
    seed = int(hashlib.md5(text.encode()).hexdigest()[:8], 16)
    return np.random.default_rng(seed).standard_normal(16).astype(np.float32)


def kv_store_script():
    """Operations on a KeSSieCPUKVStore: saves past a byte budget (oldest
    evicted), a replacement of the same (layer, block_id), semantic entries,
    searches with exclusions, position lookups."""
    ops_ = []
    for i in range(12):
        ops_.append(("save", f"layer{i % 3}", 100 + i // 3, 2 + (i % 4), 16 * (i // 3) + (i % 2)))
    ops_.append(("save", "layer1", 101, 5, 16))                 # replaces (layer1, 101)
    for j in range(6):
        ops_.append(("sem", list(range(10 * j, 10 * j + 7)), 16 * j))
    ops_ += [("search", "q-a", 3, []), ("search", "q-b", 5, [16, 48]), ("search", "", 2, [])]
    ops_ += [("get", 16, 32, "layer1"), ("get", 0, 16, "layer0"), ("get", 48, 64, "layer2"), ("range", 0, 64)]
    for i in range(5):
        ops_.append(("save", f"layer{i % 2}", 200 + i, 6, 100 + i))
    ops_ += [("range", 0, 200), ("get", 100, 116, "layer0")]
    return ops_


def run_kv_store_script(store_cls, module, torch_mod):
    """Drive a store through kv_store_script(); returns the observation log.
    time.time in `module` is replaced by a counter so eviction order is fixed."""
    import json
    tick = [0.0]

    class _T:
        @staticmethod
        def time():
            tick[0] += 1.0
            return tick[0]
    real_time = module.time
    module.time = _T
    try:
        store = store_cls(max_cpu_bytes=2600)
        store.set_embedder(kv_store_embed)
        log = []
        for op in kv_store_script():
            if op[0] == "save":
                _, layer, bid, t, pos = op
                data = torch_mod.arange(2 * t * 2 * 4, dtype=torch_mod.float32).reshape(2, t, 2, 4) + bid
                store.save_block(layer, bid, data, list(range(t)), pos)
                res = None
            elif op[0] == "sem":
                store.save_semantic_entry(op[1], op[2], tokenizer=_Tok)
                res = None
            elif op[0] == "search":
                r = store.semantic_search(op[1], top_k=op[2], exclude_positions=set(op[3]))
                res = [[a, b, round(c, 6)] for a, b, c in r]
            elif op[0] == "get":
                b = store.get_blocks_for_positions(op[1], op[2], op[3])
                res = None if b is None else [b.layer_name, b.block_id, b.position_start, b.position_end,
                                              float(b.kv_data.sum())]
            else:
                r = store.get_all_blocks_for_range(op[1], op[2])
                res = {k: [[b.block_id, b.position_start] for b in v] for k, v in sorted(r.items())}
            st = store.stats()
            keys = sorted([list(k) for k in store._blocks.keys()])
            pidx = {str(k): [list(x) for x in v] for k, v in sorted(store._position_index.items())}
            log.append({"op": json.loads(json.dumps(op)), "res": res, "stats": st, "keys": keys, "pidx": pidx})
        return log
    finally:
        module.time = real_time
