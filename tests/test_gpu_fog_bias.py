"""GPU parity of the additive fog bias of the vLLM path
(kessie_attention.py:114-139): the bias builder against the oracle bit for
bit, and paged decode / chunked prefill with the bias applied in-kernel
against the oracle attention with the bias added to the scaled scores
(bf16 / fp16: 2e-2 max-abs, 1e-2 rel)."""

import numpy as np
import pytest
import torch

from oracle import fog_oracle as O
from tests.kessie_testutil import ROUND, TOL, make_paged, random_block_table, rnd, to_dev, to_np

pytestmark = pytest.mark.gpu

CASES = [(128, 0.5, 0.5, [], 0.1), (128, 0.5, 0.5, [10, 50, 100], 0.1), (256, 0.8, 0.3, [5], 0.1),
         (4096, 0.5, 0.5, [100, 200, 300], 0.1), (131072, 0.5, 0.03125, [1000, 70000, 130000], 0.25),
         (777, 1.3, 0.9, [0, 776, 800], 0.5), (50000, 0.5, 0.5, [], 0.1)]
NAMES = {torch.float32: "float32", torch.bfloat16: "bfloat16", torch.float16: "float16"}


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    yield


@pytest.mark.parametrize("dt", [torch.float32, torch.bfloat16, torch.float16])
def test_bias_builder_matches_oracle(dt):
    from kessie_b200 import ops
    for n, alpha, fs, rec, boost in CASES:
        b = ops.FogBias(alpha, fs, rec, boost, dtype=dt)
        got = ops.build_fog_bias(n, b).view(-1).float().cpu().numpy()
        want = O.fog_bias_values(n, alpha, fs, rec, boost, NAMES[dt])
        np.testing.assert_array_equal(got, want, err_msg=f"{(n, alpha, fs)} {dt}")


def _decode_case(seed, lens, Hq, Hkv, D, dt, alpha, fs, rec, boost, window=0):
    from kessie_b200 import ops
    ps = 16
    lens = np.asarray(lens)
    P = int(sum((n + ps - 1) // ps for n in lens)) + 2
    kvn, kv = make_paged(seed, P, ps, Hkv, D, dt)
    bt = random_block_table(seed + 1, lens, ps, P)
    q = ROUND[dt](rnd(seed + 2, (len(lens), Hq, D)))
    tdt = {"bf16": torch.bfloat16, "fp16": torch.float16}[dt]
    bias = ops.FogBias(alpha, fs, rec, boost, dtype=tdt)
    out = ops.paged_fog_decode(to_dev(q, dt), kv[:, :, 0], kv[:, :, 1], torch.from_numpy(bt).cuda(),
                               torch.from_numpy(lens.astype(np.int32)).cuda(), fog_alpha=0.0,
                               window_size=window, bias=bias)
    torch.cuda.synchronize()
    spec = (alpha, fs, rec, boost, NAMES[tdt])
    want = O.paged_fog_decode(q, kvn[:, :, 0], kvn[:, :, 1], bt, lens, np.zeros(len(lens), np.int32), 0.0,
                              window, bias_spec=spec)
    return to_np(out), want


@pytest.mark.parametrize("dt", ["bf16", "fp16"])
@pytest.mark.parametrize("lens,alpha,fs,rec", [([300, 1000], 0.5, 0.5, []),
                                                ([4096, 77, 9000], 2.0, 0.25, [5, 70, 4000, 8000]),
                                                ([20000], 4.0, 0.1, [100, 19999])])
def test_decode_with_bias_matches_oracle(dt, lens, alpha, fs, rec):
    got, want = _decode_case(sum(lens), lens, 16, 4, 128, dt, alpha, fs, rec, 0.75)
    np.testing.assert_allclose(got, want, **TOL[dt])


def test_decode_bias_changes_the_output():
    """The bias is not a no-op: a strong fog moves the output away from the
    unbiased decode, and recall boosts pull it toward the recalled keys."""
    from kessie_b200 import ops
    got_fog, want_fog = _decode_case(5, [2000], 8, 2, 128, "bf16", 8.0, 0.2, [], 0.1)
    got_plain, want_plain = _decode_case(5, [2000], 8, 2, 128, "bf16", 0.0, 0.2, [], 0.1)
    assert np.abs(want_fog - want_plain).max() > 0.05
    np.testing.assert_allclose(got_fog, want_fog, **TOL["bf16"])
    np.testing.assert_allclose(got_plain, want_plain, **TOL["bf16"])


@pytest.mark.parametrize("dt,D,staged", [("bf16", 128, True), ("bf16", 128, False), ("fp16", 64, True)])
def test_prefill_with_bias_matches_oracle(dt, D, staged):
    from kessie_b200 import ops
    ps, Hq, Hkv = 16, 8, 2
    lens = np.array([1200, 700])
    T = 160
    P = int(sum((n + ps - 1) // ps for n in lens)) + 2
    kvn, kv = make_paged(31, P, ps, Hkv, D, dt)
    bt = random_block_table(32, lens, ps, P)
    q = ROUND[dt](rnd(33, (2, T, Hq, D)))
    tdt = {"bf16": torch.bfloat16, "fp16": torch.float16}[dt]
    spec = (1.5, 0.4, [3, 250, 1100], 0.5, NAMES[tdt])
    bias = ops.FogBias(*spec[:4], dtype=tdt)
    out = ops.paged_fog_prefill(to_dev(q, dt), kv[:, :, 0], kv[:, :, 1], torch.from_numpy(bt).cuda(),
                                torch.from_numpy(lens.astype(np.int32)).cuda(), fog_alpha=0.0, staged=staged,
                                bias=bias)
    torch.cuda.synchronize()
    got = to_np(out)
    for b in range(2):
        want = O.paged_fog_prefill(np.transpose(q[b], (1, 0, 2)), kvn[:, :, 0], kvn[:, :, 1], bt[b], lens[b],
                                   lens[b] - T, 0, 0.0, bias_spec=spec)
        np.testing.assert_allclose(got[b], np.transpose(want, (1, 0, 2)), **TOL[dt])


def test_biased_decode_back_to_back():
    """Biased decodes (the vLLM path) enqueued with nothing in between and no
    synchronisation: each may read q, its pages and the recall bitmap before
    the previous decode finishes, when that decode wrote none of them.
    Independent steps, then a chain whose output is the next step's q (those
    must wait); every result equals the same launches run one at a time, and
    the first matches the oracle."""
    from kessie_b200 import ops
    B, Hq, Hkv, D, ps = 3, 16, 4, 128, 16
    lens = np.array([2000, 3333, 1500])
    P = int(sum((n + ps - 1) // ps for n in lens)) + 2
    kvn, kv = make_paged(61, P, ps, Hkv, D, "bf16")
    btn = random_block_table(62, lens, ps, P)
    bt = torch.from_numpy(btn).cuda()
    sl = torch.from_numpy(lens.astype(np.int32)).cuda()
    qn = [ROUND["bf16"](rnd(63 + i, (B, Hq, D))) for i in range(2)]
    qs = [to_dev(x, "bf16") for x in qn]
    spec = (0.5, 0.5, [7, 900, 2500], 0.25)
    bias = ops.FogBias(*spec, dtype=torch.bfloat16)
    ws = torch.empty(ops.decode_workspace_bytes(B, Hq, Hkv, D, bt.shape[1] * ps, ps), dtype=torch.uint8,
                     device="cuda")

    def run(sync):
        outs = [torch.empty(B, Hq, D, dtype=torch.bfloat16, device="cuda") for _ in range(4)]
        chain = [qs[0].clone()] + [torch.empty(B, Hq, D, dtype=torch.bfloat16, device="cuda") for _ in range(3)]
        torch.cuda.synchronize()
        steps = [(qs[j % 2], outs[j]) for j in range(4)] + [(chain[j], chain[j + 1]) for j in range(3)]
        for q, o in steps:
            ops.paged_fog_decode(q, kv[:, :, 0], kv[:, :, 1], bt, sl, fog_alpha=0.0, bias=bias, ws=ws, out=o)
            if sync:
                torch.cuda.synchronize()
        torch.cuda.synchronize()
        return outs + chain[1:]

    got, want = run(False), run(True)
    assert ops.read_device_status() == 0
    for a, b in zip(got, want):
        assert torch.equal(a, b)
    ref = O.paged_fog_decode(qn[0], kvn[:, :, 0], kvn[:, :, 1], btn, lens, np.zeros(B, np.int32), 0.0, 0,
                             bias_spec=spec + ("bfloat16",))
    np.testing.assert_allclose(to_np(got[0]), ref, **TOL["bf16"])
