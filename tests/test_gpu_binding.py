"""GPU parity of the torch extension module kessie_hip (the reference's
pybind11 boundary, kessie_hip_binding.cpp:216-239, over this library): each
of its five functions against the oracle, on the current CUDA stream."""

import math

import numpy as np
import pytest
import torch

from oracle import fog_oracle as O
from tests.kessie_testutil import TOL, rnd, to_dev, to_np

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def kh():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from kessie_b200 import _lib
    return _lib.load_binding()


@pytest.mark.parametrize("W,causal", [(0, True), (64, True), (0, False)])
def test_binding_attention(kh, W, causal):
    B, H, N, D = 1, 4, 256, 64
    q, k, v = (O.round_f16(rnd(11 + j, (B, H, N, D))) for j in range(3))
    out = kh.windowed_attention(to_dev(q, "fp16"), to_dev(k, "fp16"), to_dev(v, "fp16"), W, causal)
    torch.cuda.synchronize()
    np.testing.assert_allclose(to_np(out), O.windowed_attention(q, k, v, W, causal), **TOL["fp16"])
    fog = O.build_fog_weights(N, 0.5, 0.5)
    out = kh.fused_fog_attention(to_dev(q, "fp16"), to_dev(k, "fp16"), to_dev(v, "fp16"),
                                 torch.from_numpy(fog).cuda(), W, causal)
    torch.cuda.synchronize()
    np.testing.assert_allclose(to_np(out), O.fused_fog_attention(q, k, v, fog, W, causal), **TOL["fp16"])


def test_binding_checks_raise(kh):
    q = torch.zeros(1, 2, 16, 64, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(RuntimeError, match="FP16"):
        kh.windowed_attention(q, q, q)
    q = torch.zeros(1, 2, 16, 96, dtype=torch.float16, device="cuda")
    with pytest.raises(RuntimeError, match="head_dim"):
        kh.windowed_attention(q, q, q)


def test_binding_rope_and_pages(kh):
    T, H, D = 64, 8, 128
    k = O.round_f16(rnd(21, (T, H, D)))
    orig = np.random.default_rng(22).integers(0, 32768, T).astype(np.int32)
    tgt = (131072 + np.arange(T)).astype(np.int32)
    kd = to_dev(k, "fp16")
    kh.rope_remap(kd, torch.from_numpy(orig).cuda(), torch.from_numpy(tgt).cuda(), 500000.0)
    torch.cuda.synchronize()
    np.testing.assert_allclose(to_np(kd), O.round_f16(O.rope_remap(k, orig, tgt, 500000.0)), **TOL["fp16"])
    # evict: the reference self-test's 64 of 128 (kessie_kernels_v2.hip:1008-1023)
    valid = torch.ones(128, dtype=torch.int8, device="cuda")
    pos = torch.arange(128, dtype=torch.int32, device="cuda") * 64
    cnt = kh.page_evict(valid, pos, 64 * 64)
    torch.cuda.synchronize()
    assert int(cnt.item()) == 64 and int(valid.sum().item()) == 64
    # insert: 40 tokens into pages 5, 2, 9 of a [P, ps, 2, H, D] cache
    P, ps = 12, 16
    cache = torch.zeros(P, ps, 2, H, D, dtype=torch.float16, device="cuda")
    nk, nv = (O.round_f16(rnd(30 + j, (40, H, D))) for j in range(2))
    ids = torch.tensor([5, 2, 9], dtype=torch.int32, device="cuda")
    pv = torch.zeros(P, dtype=torch.int8, device="cuda")
    pp = torch.zeros(P, dtype=torch.int32, device="cuda")
    kh.page_insert(cache, to_dev(nk, "fp16"), to_dev(nv, "fp16"), ids, pv, pp, 1000)
    torch.cuda.synchronize()
    c = to_np(cache)
    for i, pg in enumerate([5, 2, 9]):
        n = min(ps, 40 - i * ps)
        np.testing.assert_array_equal(c[pg, :n, 0], nk[i * ps:i * ps + n])
        np.testing.assert_array_equal(c[pg, :n, 1], nv[i * ps:i * ps + n])
        assert int(pv[pg]) == 1 and int(pp[pg]) == 1000 + i * ps
