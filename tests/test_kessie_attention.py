"""vLLM attention mirror (kessie_attention.py): state / switch / delegation on
CPU; on a GPU the _FogCache API against the oracle and KeSSieAttentionImpl.
forward (decode step and mixed decode + chunked-prefill step over a vLLM
[2, num_blocks, block_size, H, D] cache) against the oracle attention with the
fog bias on the scores."""

from types import SimpleNamespace

import numpy as np
import pytest
import torch

from oracle import fog_oracle as O
from tests.kessie_testutil import ROUND, TOL, rnd, to_dev, to_np


class _FakeInner:
    """Stands in for vLLM's FlashAttentionImpl: records delegated calls."""

    def __init__(self, num_heads=8, num_kv_heads=2, head_size=128, scale=None):
        self.num_heads, self.num_kv_heads, self.head_size = num_heads, num_kv_heads, head_size
        self.scale = scale if scale is not None else head_size ** -0.5
        self.sliding_window = (-1, -1)
        self.alibi_slopes = None
        self.sinks = None
        self.logits_soft_cap = None
        self.calls = 0

    def forward(self, layer, query, key, value, kv_cache, attn_metadata, output=None, output_scale=None,
                output_block_scale=None):
        self.calls += 1
        return "inner"

    def do_kv_cache_update(self, *args):
        return "kv-update"


def _reset_state(**kw):
    from kessie_b200 import kessie_attention as A
    A.KESSIE_STATE.update(**kw)
    A.KESSIE_STATE.enabled = True
    return A


def test_state_api_and_switch():
    from kessie_b200 import kessie_attention as A
    st = A.KeSSieAttentionState()
    g0 = st.get()["generation"]
    st.update(fog_alpha=0.7, recall_positions=[3, 5])
    got = st.get()
    assert got["generation"] == g0 + 1 and got["fog_alpha"] == 0.7 and got["recall_positions"] == {3, 5}
    got["recall_positions"].add(99)
    assert st.get()["recall_positions"] == {3, 5}                 # get() returns a copy
    assert not A._fog_active({"enabled": True, "fog_alpha": 0.5, "prompt_len": 0})
    assert not A._fog_active({"enabled": True, "fog_alpha": 0.0, "prompt_len": 10})
    assert not A._fog_active({"enabled": False, "fog_alpha": 0.5, "prompt_len": 10})
    assert A._fog_active({"enabled": True, "fog_alpha": 0.5, "prompt_len": 10})


def test_impl_delegates_when_fog_is_off_or_uncovered():
    A = _reset_state(fog_alpha=0.5, prompt_len=0)
    inner = _FakeInner()
    impl = A.KeSSieAttentionImpl(_inner_impl=inner)
    q = torch.zeros(4, 8, 128)
    md = SimpleNamespace(num_actual_tokens=4, max_query_len=1)
    assert impl.forward(None, q, q, q, torch.zeros(2, 1, 16, 2, 128), md, torch.zeros(4, 8 * 128)) == "inner"
    A.KESSIE_STATE.update(prompt_len=100)                          # fog on, but CPU tensors: not covered
    assert impl.forward(None, q, q, q, torch.zeros(2, 1, 16, 2, 128), md, torch.zeros(4, 8 * 128)) == "inner"
    assert impl.forward(None, q, q, q, None, None, None) == "inner"   # profiling run
    assert inner.calls == 3
    assert impl.do_kv_cache_update() == "kv-update"               # everything else is the wrapped impl's
    A.KESSIE_STATE.update(prompt_len=0)


# ----------------------------------------------------------------- GPU
@pytest.mark.gpu
def test_fog_cache_api_matches_reference_semantics():
    """Values equal the oracle; same view for the same generation; a new
    generation lands in the other buffer with the same values; zero alpha
    gives an all-zero bias (the reference's self-test, kessie_attention.py:355-436)."""
    from kessie_b200 import kessie_attention as A
    cache = A._FogCache()
    dev = torch.device("cuda")
    st = {"fog_alpha": 0.5, "fog_start": 0.5, "prompt_len": 100, "recall_positions": {10, 50, 100},
          "recall_boost": 0.1, "enabled": True, "generation": 1}
    for dt, name in ((torch.float32, "float32"), (torch.bfloat16, "bfloat16")):
        cache = A._FogCache()
        b1 = cache.get_fog_bias(128, dev, dt, st)
        assert b1.shape == (1, 1, 1, 128)
        np.testing.assert_array_equal(b1.view(-1).float().cpu().numpy(),
                                      O.fog_bias_values(128, 0.5, 0.5, [10, 50, 100], 0.1, name))
        assert cache.get_fog_bias(128, dev, dt, st).data_ptr() == b1.data_ptr()
        st2 = dict(st, generation=2)
        b2 = cache.get_fog_bias(128, dev, dt, st2)
        assert b2.data_ptr() != b1.data_ptr() and torch.equal(b1, b2)
    off = cache.get_fog_bias(128, dev, torch.float32, dict(st, fog_alpha=0.0, recall_positions=set(), generation=9))
    assert off.abs().sum().item() == 0


def _vllm_setup(seed, seq_lens, q_lens, Hq=16, Hkv=4, D=128, bs=16, dt="bf16"):
    nb = int(sum((n + bs - 1) // bs for n in seq_lens)) + 3
    g = np.random.default_rng(seed)
    cache_np = ROUND[dt](rnd(seed, (2, nb, bs, Hkv, D)))
    perm = g.permutation(nb).astype(np.int32)
    maxb = max((n + bs - 1) // bs for n in seq_lens)
    bt = np.zeros((len(seq_lens), maxb), np.int32)
    o = 0
    for b, n in enumerate(seq_lens):
        k = (n + bs - 1) // bs
        bt[b, :k] = perm[o:o + k]
        o += k
    n_tok = int(sum(q_lens))
    q_np = ROUND[dt](rnd(seed + 1, (n_tok, Hq, D)))
    qsl = np.concatenate([[0], np.cumsum(q_lens)]).astype(np.int32)
    md = SimpleNamespace(num_actual_tokens=n_tok, max_query_len=int(max(q_lens)),
                         query_start_loc=torch.from_numpy(qsl).cuda(),
                         seq_lens=torch.from_numpy(np.asarray(seq_lens, np.int32)).cuda(),
                         block_table=torch.from_numpy(bt).cuda(), max_seq_len=int(max(seq_lens)))
    return cache_np, to_dev(cache_np, dt), bt, q_np, to_dev(q_np, dt), qsl, md


def _oracle_rows(cache_np, bt, q_np, qsl, seq_lens, q_lens, spec, D):
    rows = []
    for b, (n, ql) in enumerate(zip(seq_lens, q_lens)):
        qb = q_np[qsl[b]:qsl[b] + ql]                            # [ql, Hq, D]
        want = O.paged_fog_prefill(np.transpose(qb, (1, 0, 2)), cache_np[0], cache_np[1], bt[b], n, n - ql, 0, 0.0,
                                   bias_spec=spec)
        rows.append(np.transpose(want, (1, 0, 2)))
    return np.concatenate(rows)


@pytest.mark.gpu
@pytest.mark.parametrize("seq_lens,q_lens", [([3000, 129, 7000, 1], [1, 1, 1, 1]),
                                             ([900, 4500, 300, 2049, 640], [1, 1, 37, 1, 128])])
def test_impl_forward_applies_the_fog(seq_lens, q_lens):
    A = _reset_state(fog_alpha=1.5, fog_start=0.4, prompt_len=100, recall_positions=[5, 250, 2000, 4400],
                     recall_boost=0.5)
    Hq, Hkv, D = 16, 4, 128
    cache_np, cache, bt, q_np, q, qsl, md = _vllm_setup(sum(seq_lens), seq_lens, q_lens, Hq, Hkv, D)
    inner = _FakeInner(Hq, Hkv, D)
    impl = A.KeSSieAttentionImpl(_inner_impl=inner)
    out = torch.empty(len(q_np), Hq * D, dtype=torch.bfloat16, device="cuda")
    res = impl.forward(None, q, q, q, cache, md, out)
    torch.cuda.synchronize()
    assert res is out and inner.calls == 0
    spec = (1.5, 0.4, [5, 250, 2000, 4400], 0.5, "bfloat16")
    want = _oracle_rows(cache_np, bt, q_np, qsl, seq_lens, q_lens, spec, D)
    np.testing.assert_allclose(to_np(out).reshape(len(q_np), Hq, D), want, **TOL["bf16"])
    A.KESSIE_STATE.update(prompt_len=0)
