"""GPU parity: dense (legacy launchers + v2) and paged chunked-prefill fog
attention against the oracle and the reference's golden outputs."""

import ctypes
import math
import os

import numpy as np
import pytest
import torch

from oracle import fog_oracle as O
from tests.kessie_testutil import ROUND, TOL, make_paged, random_block_table, rnd, to_dev, to_np

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True, params=["tcgen05", "mma"])
def _cuda(request):
    """Every prefill test runs on both implementations: the tcgen05/TMEM
    kernel (default for head_dim 128) and the warp-level mma.sync kernel."""
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    old = os.environ.get("KESSIE_PREFILL_IMPL")
    if request.param == "mma":
        os.environ["KESSIE_PREFILL_IMPL"] = "mma"
    else:
        os.environ.pop("KESSIE_PREFILL_IMPL", None)
    yield request.param
    if old is None:
        os.environ.pop("KESSIE_PREFILL_IMPL", None)
    else:
        os.environ["KESSIE_PREFILL_IMPL"] = old


def _legacy(fn_name, q, k, v, fog, W, causal):
    from kessie_b200 import _lib
    lib = _lib.load()
    B, H, N, D = q.shape
    o = torch.empty_like(q)
    args = [q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr()]
    if fog is not None:
        args.append(fog.data_ptr())
    args += [ctypes.c_float(1.0 / math.sqrt(D)), B, H, N, D, W, 1 if causal else 0, None]
    getattr(lib, fn_name)(*args)
    _lib.check_legacy(fn_name)
    torch.cuda.synchronize()
    return to_np(o)


def test_legacy_windowed_attn_reference_configs(golden_dir):
    """The reference's own windowed-attention test configs
    (kessie_hip_kernels.py:623-626) through launch_kessie_windowed_attn."""
    d = np.load(os.path.join(golden_dir, "attention.npz"))
    for i in range(int(d["nwin"])):
        Z, H, N, D, W, causal, seed = (int(x) for x in d[f"win{i}_cfg"])
        q, k, v = (O.round_f16(rnd(seed + j, (Z, H, N, D))) for j in range(3))
        got = _legacy("launch_kessie_windowed_attn", to_dev(q, "fp16"), to_dev(k, "fp16"), to_dev(v, "fp16"),
                      None, W, causal)
        rows = d[f"win{i}_rows"]
        np.testing.assert_allclose(got[:, :, rows], d[f"win{i}_out"], **TOL["fp16"])
        np.testing.assert_allclose(got, O.windowed_attention(q, k, v, W, bool(causal)), **TOL["fp16"])


def test_legacy_fused_fog_attn_reference_configs(golden_dir):
    d = np.load(os.path.join(golden_dir, "attention.npz"))
    for i in range(int(d["nfog"])):
        Z, H, N, D, W, causal, seed = (int(x) for x in d[f"fog{i}_cfg"])
        a, fs = d[f"fog{i}_fog"]
        q, k, v = (O.round_f16(rnd(seed + j, (Z, H, N, D))) for j in range(3))
        fog = O.build_fog_weights(N, a, fs)
        got = _legacy("launch_kessie_fused_fog_attn", to_dev(q, "fp16"), to_dev(k, "fp16"), to_dev(v, "fp16"),
                      torch.from_numpy(fog).cuda(), W, causal)
        np.testing.assert_allclose(got[:, :, d[f"fog{i}_rows"]], d[f"fog{i}_out"], **TOL["fp16"])
        np.testing.assert_allclose(got, O.fused_fog_attention(q, k, v, fog, W, bool(causal)), **TOL["fp16"])


def test_legacy_unsupported_head_dim_reports_error():
    from kessie_b200 import _lib
    lib = _lib.load()
    x = torch.zeros(1, 1, 16, 96, dtype=torch.float16, device="cuda")
    lib.launch_kessie_windowed_attn(x.data_ptr(), x.data_ptr(), x.data_ptr(), x.data_ptr(), ctypes.c_float(0.1),
                                    1, 1, 16, 96, 0, 1, None)
    st, msg = _lib.last_error()
    assert st == 2 and "head_dim" in msg


@pytest.mark.parametrize("dt", ["bf16", "fp16"])
@pytest.mark.parametrize("B,Hq,Hkv,N,D,W,causal", [(1, 8, 2, 300, 128, 0, True), (2, 4, 4, 77, 64, 0, False),
                                                     (1, 12, 3, 200, 128, 50, True), (1, 16, 2, 1, 128, 0, True),
                                                     (1, 2, 1, 1000, 64, 0, True)])
def test_fog_attention_v2_gqa(dt, B, Hq, Hkv, N, D, W, causal):
    from kessie_b200 import ops
    q = ROUND[dt](rnd(1, (B, Hq, N, D))); k = ROUND[dt](rnd(2, (B, Hkv, N, D))); v = ROUND[dt](rnd(3, (B, Hkv, N, D)))
    fog = O.build_fog_weights(N, 0.5, 0.5)
    out = ops.fog_attention(to_dev(q, dt), to_dev(k, dt), to_dev(v, dt), torch.from_numpy(fog).cuda(), W, causal)
    torch.cuda.synchronize()
    g = Hq // Hkv
    want = O.fused_fog_attention(q, np.repeat(k, g, axis=1), np.repeat(v, g, axis=1), fog, W, causal)
    np.testing.assert_allclose(to_np(out), want, **TOL[dt])


@pytest.mark.parametrize("staged", [True, False])
@pytest.mark.parametrize("ps", [16, 32])
@pytest.mark.parametrize("Hq,Hkv,kv_len,T,W,fogw", [(32, 8, 1000, 100, 0, 256), (8, 2, 333, 333, 0, 64),
                                                    (8, 8, 2048, 64, 300, 100), (16, 4, 500, 1, 0, 0),
                                                    (4, 1, 4111, 257, 0, 4096)])
def test_paged_prefill_matches_oracle(staged, ps, Hq, Hkv, kv_len, T, W, fogw):
    from kessie_b200 import ops
    D, dt = 128, "bf16"
    lens = [kv_len]
    P = (kv_len + ps - 1) // ps + 2
    kvn, kv = make_paged(kv_len + T, P, ps, Hkv, D, dt)
    bt = random_block_table(7, lens, ps, P)
    q = ROUND[dt](rnd(5, (1, T, Hq, D)))
    cs = kv_len - fogw
    out = ops.paged_fog_prefill(to_dev(q, dt), kv[:, :, 0], kv[:, :, 1], torch.from_numpy(bt).cuda(),
                                torch.tensor([kv_len], dtype=torch.int32, device="cuda"),
                                clear_start=torch.tensor([cs], dtype=torch.int32, device="cuda"), fog_alpha=0.5,
                                window_size=W, staged=staged)
    torch.cuda.synchronize()
    want = O.paged_fog_prefill(np.transpose(q[0], (1, 0, 2)), kvn[:, :, 0], kvn[:, :, 1], bt[0], kv_len, kv_len - T,
                               cs, 0.5, W)
    np.testing.assert_allclose(to_np(out)[0], np.transpose(want, (1, 0, 2)), **TOL[dt])


@pytest.mark.parametrize("staged", [True, False])
def test_paged_prefill_batched_with_stale_nan_and_qstart(staged):
    from kessie_b200 import ops
    D, dt, ps, Hq, Hkv = 64, "fp16", 16, 8, 2
    lens = [90, 200]
    T = 40
    P = sum((n + ps - 1) // ps for n in lens) + 1
    kvn, kv = make_paged(3, P, ps, Hkv, D, dt)
    bt = random_block_table(9, lens, ps, P)
    # NaN in the stale tail of sequence 0's last page
    kv[bt[0, 5], 90 % ps:] = float("nan")
    q = ROUND[dt](rnd(8, (2, T, Hq, D)))
    qs = np.array([50, 160], np.int32)
    out = ops.paged_fog_prefill(to_dev(q, dt), kv[:, :, 0], kv[:, :, 1], torch.from_numpy(bt).cuda(),
                                torch.tensor(lens, dtype=torch.int32, device="cuda"),
                                q_start=torch.from_numpy(qs).cuda(), clear_start=None, fog_alpha=0.0, staged=staged)
    torch.cuda.synchronize()
    got = to_np(out)
    assert np.isfinite(got).all()
    for b in range(2):
        want = O.paged_fog_prefill(np.transpose(q[b], (1, 0, 2)), kvn[:, :, 0], kvn[:, :, 1], bt[b], lens[b],
                                   int(qs[b]), 0, 0.0)
        np.testing.assert_allclose(got[b], np.transpose(want, (1, 0, 2)), **TOL[dt])
