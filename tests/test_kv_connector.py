"""KV connector mirror (kessie_kv_connector.py): the CPU block store's
bookkeeping against the reference's own store (golden log), the connector's
host logic, and -- on a GPU -- bit-exact batched save / load against the
reference semantics kv_layer[:, block_id, :tokens]."""

import json
import os
import sys
from types import SimpleNamespace

import pytest
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "golden"))

from kv_store_script import kv_store_embed, run_kv_store_script  # noqa: E402


def _golden():
    with open(os.path.join(HERE, "golden", "kv_store.json")) as f:
        return json.load(f)


def test_store_bookkeeping_matches_reference_log():
    """Budget eviction order, same-key replacement accounting, position index
    (duplicates included), lookups and semantic search equal the log the
    reference's KeSSieCPUKVStore produced."""
    from kessie_b200 import kessie_kv_connector as C
    got = json.loads(json.dumps(run_kv_store_script(C.KeSSieCPUKVStore, C, torch)))
    want = _golden()
    assert len(got) == len(want)
    for i, (g, w) in enumerate(zip(got, want)):
        assert g == w, f"step {i} {w['op']}"


def test_store_singleton_and_recall_state():
    from kessie_b200 import kessie_kv_connector as C
    assert C.get_kessie_store() is C.get_kessie_store(123)
    st = C.RecallState()
    assert st.recalled_positions == [] and st.num_recalled_tokens == 0 and not st.load_pending


def test_connector_host_logic_without_gpu():
    """Recall bookkeeping: matched tokens come from the semantic index
    (similarity >= 0.3), are cached per request, cleared on finish."""
    from kessie_b200 import kessie_kv_connector as C
    conn = C.KeSSieKVConnector()
    store = C.KeSSieCPUKVStore()
    conn.store = store
    # an embedder that maps every query onto entry 2's direction
    target = kv_store_embed("e2")
    store.set_embedder(lambda text: target if text.startswith("tokens:") else kv_store_embed(text))
    tok = SimpleNamespace(decode=lambda ids, skip_special_tokens=True: f"e{ids[0]}")
    for j in range(4):
        store.save_semantic_entry([j, 1, 2], 100 * j, tokenizer=tok)
    req = SimpleNamespace(prompt_token_ids=list(range(40)), request_id="r1")
    n = conn.get_num_new_matched_tokens(req)
    assert n >= 3 and (200, 203) in C._RECALL_STATES["r1"].recalled_positions
    assert conn.get_num_new_matched_tokens(req) == n            # cached
    conn.update_state_after_alloc(req, None, n)
    assert C._RECALL_STATES["r1"].load_pending
    assert conn.request_finished(req, []) == (False, None)
    assert "r1" not in C._RECALL_STATES
    assert conn.build_connector_meta(None) is None
    # no prompt -> nothing to recall
    assert conn.get_num_new_matched_tokens(SimpleNamespace(prompt_token_ids=[], request_id="r2")) == 0


# ----------------------------------------------------------------- GPU: the batched data path
def _vllm_cache(seed, nb, bs, H, D, dtype=torch.bfloat16):
    g = torch.Generator(device="cuda").manual_seed(seed)
    return torch.randn(2, nb, bs, H, D, device="cuda", generator=g).to(dtype)


@pytest.mark.gpu
def test_save_kv_layer_is_bit_exact_per_block():
    """save_kv_layer stores, for every sequence and block, exactly
    kv_layer[:, block_id, :tokens] (kessie_kv_connector.py:453-491), with one
    gather kernel + one device-to-host copy for the whole layer."""
    from kessie_b200 import kessie_kv_connector as C
    nb, bs, H, D = 300, 16, 8, 128
    cache = _vllm_cache(1, nb, bs, H, D)
    conn = C.KeSSieKVConnector()
    conn.store = C.KeSSieCPUKVStore()
    conn.register_kv_caches([cache], ["l0"])
    assert conn._block_size == bs
    seq_lens = torch.tensor([37, 16, 1, 250], dtype=torch.int32)
    perm = torch.randperm(nb, generator=torch.Generator().manual_seed(2))[:64].to(torch.int32)
    bt = torch.full((4, 16), -1, dtype=torch.int32)
    o = 0
    for s, n in enumerate(seq_lens.tolist()):
        k = (n + bs - 1) // bs
        bt[s, :k] = perm[o:o + k]
        o += k
    meta = SimpleNamespace(block_tables=bt.cuda(), seq_lens=seq_lens.cuda())
    conn.save_kv_layer("l0", cache, meta)
    conn.wait_for_save()
    for s, n in enumerate(seq_lens.tolist()):
        for b in range((n + bs - 1) // bs):
            bid = int(bt[s, b])
            blk = conn.store._blocks[("l0", bid)]
            ntok = min(bs, n - b * bs)
            assert blk.position_start == b * bs and blk.kv_data.shape == (2, ntok, H, D)
            assert torch.equal(blk.kv_data, cache[:, bid, :ntok].cpu())
    assert conn.store.total_bytes == sum(2 * min(bs, n - b * bs) * H * D * 2
                                         for n in seq_lens.tolist() for b in range((n + bs - 1) // bs))


@pytest.mark.gpu
def test_start_load_kv_writes_recalled_blocks_into_their_slots():
    """Recalled blocks land in cache[:, block_id, :tokens] bit-exactly; other
    blocks are untouched."""
    from kessie_b200 import kessie_kv_connector as C
    nb, bs, H, D = 64, 16, 4, 128
    src = _vllm_cache(3, nb, bs, H, D)
    conn = C.KeSSieKVConnector()
    conn.store = C.KeSSieCPUKVStore()
    conn.register_kv_caches([src], ["l0"])
    ids = [5, 9, 40]
    for b, bid in enumerate(ids):
        ntok = 16 if b < 2 else 7
        conn.store.save_block("l0", bid, src[:, bid, :ntok], [], 16 * b)
    dst = _vllm_cache(4, nb, bs, H, D)
    before = dst.clone()
    C._RECALL_STATES.clear()
    C._RECALL_STATES["r"] = C.RecallState("r", [(0, 16), (16, 32), (32, 39)], 39, True)
    conn.start_load_kv([dst], ["l0"])
    conn.wait_for_layer_load("l0")
    torch.cuda.synchronize()
    for b, bid in enumerate(ids):
        ntok = 16 if b < 2 else 7
        assert torch.equal(dst[:, bid, :ntok], src[:, bid, :ntok])
    untouched = [i for i in range(nb) if i not in ids]
    assert torch.equal(dst[:, untouched], before[:, untouched])
    assert not C._RECALL_STATES["r"].load_pending
    C._RECALL_STATES.clear()


@pytest.mark.gpu
def test_save_then_load_blocks_round_trip_large():
    """Batched gather -> pinned host -> scatter into other slots of another
    cache reproduces the blocks exactly (2048 blocks of 64 KB)."""
    from kessie_b200 import kessie_kv_connector as C
    nb, bs, H, D = 4096, 16, 8, 128
    a = _vllm_cache(5, nb, bs, H, D)
    ids = torch.randperm(nb, generator=torch.Generator().manual_seed(6))[:2048].to(torch.int32)
    host = C.save_blocks(a, ids.cuda())
    torch.cuda.synchronize()
    assert torch.equal(host, a[:, ids.long()].cpu())
    b = torch.zeros_like(a)
    dst_ids = torch.randperm(nb, generator=torch.Generator().manual_seed(7))[:2048].to(torch.int32)
    C.load_blocks(b, host, dst_ids.cuda())
    torch.cuda.synchronize()
    assert torch.equal(b[:, dst_ids.long()], a[:, ids.long()])
    empty = C.save_blocks(a, torch.empty(0, dtype=torch.int32, device="cuda"))
    assert empty.shape[1] == 0
