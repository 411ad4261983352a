"""GPU parity of the conversation-index query (kessie_hip_kernels.py:343-360,
VectorIndex kessie_exp3.py:58-110): similarities against the oracle (fp32,
1e-5), top-k ids bit-exact (descending, ties to the lower index) and against
the reference VectorIndex's golden results."""

import os

import numpy as np
import pytest
import torch

from oracle import fog_oracle as O

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    yield


def _run(q, x, k, normalize_rows=True):
    from kessie_b200 import ops
    ids, scores, sims = ops.index_query(torch.from_numpy(q).cuda(), torch.from_numpy(x).cuda(), top_k=k,
                                        normalize_rows=normalize_rows, return_sims=True)
    torch.cuda.synchronize()
    return ids.cpu().numpy(), scores.cpu().numpy(), sims.cpu().numpy()


@pytest.mark.parametrize("n,dim,k", [(1, 256, 5), (3, 256, 5), (1000, 256, 1), (78125, 256, 5), (20001, 64, 32),
                                     (5000, 4, 8), (250000, 256, 10)])
def test_index_query_matches_oracle(n, dim, k):
    rng = np.random.default_rng(n + dim)
    x = rng.standard_normal((n, dim), dtype=np.float32)
    x[n // 2] = 0.0                                          # zero row: the +1e-8 guard
    q = rng.standard_normal(dim, dtype=np.float32)
    ids, scores, sims = _run(q, x, k)
    want_sims, want_ids, want_scores = O.index_query(q, x, True, k)
    np.testing.assert_allclose(sims, want_sims, rtol=1e-5, atol=1e-6)
    np.testing.assert_array_equal(ids, want_ids)
    np.testing.assert_allclose(scores, want_scores, rtol=1e-5, atol=1e-6)


def test_index_query_ties_go_to_the_lower_index():
    rng = np.random.default_rng(1)
    base = rng.standard_normal((50, 128), dtype=np.float32)
    x = np.concatenate([base, base, base])                     # every row three times
    q = base[17] + 0.01 * rng.standard_normal(128, dtype=np.float32)
    ids, scores, _ = _run(q, x, 6)
    want_ids = O.index_query(q, x, True, 6)[1]
    np.testing.assert_array_equal(ids, want_ids)
    assert list(ids[:3]) == [17, 67, 117]


def test_index_query_matches_reference_vector_index(golden_dir):
    d = np.load(os.path.join(golden_dir, "index_query.npz"))
    n, dim, seed = (int(v) for v in d["cfg"])
    mat = np.random.default_rng(seed).standard_normal((n, dim), dtype=np.float32)
    mat[7] = 0.0
    rows = O.vector_index_rows(mat)
    for qi in range(3):
        q = np.random.default_rng(seed + 1 + qi).standard_normal((dim,), dtype=np.float32)
        ids, scores, _ = _run(q, rows, 10, normalize_rows=False)
        np.testing.assert_array_equal(ids, d[f"q{qi}_ids"])
        np.testing.assert_allclose(scores, d[f"q{qi}_scores"], rtol=1e-5, atol=1e-6)


def test_index_query_drop_in_function():
    from kessie_b200 import kessie_hip_kernels as K
    rng = np.random.default_rng(5)
    x = torch.from_numpy(rng.standard_normal((4000, 256), dtype=np.float32)).cuda()
    q = torch.from_numpy(rng.standard_normal(256, dtype=np.float32)).cuda()
    sims = K.kessie_index_query(q, x)
    sims2, ids, scores = K.kessie_index_query(q, x, top_k=4)
    torch.cuda.synchronize()
    want = O.index_query(q.cpu().numpy(), x.cpu().numpy(), True, 4)
    np.testing.assert_allclose(sims.cpu().numpy(), want[0], rtol=1e-5, atol=1e-6)
    assert torch.equal(sims, sims2)
    np.testing.assert_array_equal(ids.cpu().numpy(), want[1])


def test_vector_index_mirror_matches_reference(golden_dir):
    """kessie_b200.vector_index.VectorIndex against the reference VectorIndex's
    golden results (ids mapped through the stored id list), the tiny-query
    guard, k = min(top_k, count), and top_k above the device list length."""
    from kessie_b200.vector_index import VectorIndex
    d = np.load(os.path.join(golden_dir, "index_query.npz"))
    n, dim, seed = (int(v) for v in d["cfg"])
    mat = np.random.default_rng(seed).standard_normal((n, dim), dtype=np.float32)
    mat[7] = 0.0
    vi = VectorIndex(dim=dim)
    assert vi.search(mat[0]) == [] and vi.count == 0
    vi.rebuild([mat[i] for i in range(n)], [5000 + i for i in range(n)])
    assert vi.count == n
    for qi in range(3):
        q = np.random.default_rng(seed + 1 + qi).standard_normal((dim,), dtype=np.float32)
        got = vi.search(q, top_k=10)
        assert [g[0] for g in got] == [5000 + int(i) for i in d[f"q{qi}_ids"]]
        np.testing.assert_allclose([g[1] for g in got], d[f"q{qi}_scores"], rtol=1e-5, atol=1e-6)
    assert len(vi.search(np.full(dim, 1e-12, np.float32), top_k=10)) == int(d["tiny_query_result_len"])
    q = np.random.default_rng(3).standard_normal((dim,), dtype=np.float32)
    big = vi.search(q, top_k=100)                                  # beyond 32: similarity output + stable sort
    rows = O.vector_index_rows(mat)
    _, want_ids, want_scores = O.index_query(q / np.linalg.norm(q), rows, False, 100)
    assert [g[0] for g in big] == [5000 + int(i) for i in want_ids]
    np.testing.assert_allclose([g[1] for g in big], want_scores, rtol=1e-5, atol=1e-6)
    small = VectorIndex(dim=4)
    small.rebuild([np.array([1, 0, 0, 0], np.float32), np.array([0, 1, 0, 0], np.float32)], [11, 12])
    got = small.search(np.array([1, 0.5, 0, 0], np.float32), top_k=5)
    assert [g[0] for g in got] == [11, 12]
    small.rebuild([], [])
    assert small.search(np.ones(4, np.float32)) == [] and small.count == 0
