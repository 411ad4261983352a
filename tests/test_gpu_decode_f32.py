"""GPU parity: the fp32 paged fog decode against the reference's fp32 outputs
(benchmark config 1) and the numpy oracle, at the fp32 bar of 1e-4 max-abs.

The reference's own path is fp32 (kessie_windowed_attention_ref /
kessie_fused_fog_attention_ref, kessie_hip_kernels.py:577-593); these tests
run the library's fp32 kernel on fp32 inputs, not rounded copies."""

import os

import numpy as np
import pytest
import torch

from oracle import fog_oracle as O
from tests.kessie_testutil import TOL, make_paged, random_block_table, rnd, to_dev, to_np
from tests.test_gpu_decode import run_case

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    yield


def test_config1_golden_decode_fp32(golden_dir):
    """Benchmark config 1 at its own precision: B1, Hq8/Hkv2, D128, 4096
    tokens, W512, fp32, RoPE theta 1e4 applied to q and k.  Both fog mappings
    (causal + clear_start = N - W; the reference-literal window W plus fog)
    match the reference's recorded fp32 outputs within 1e-4."""
    from kessie_b200 import ops
    d = np.load(os.path.join(golden_dir, "config1_decode.npz"))
    B, Hq, Hkv, D, N, W, seed = (int(x) for x in d["cfg"])
    q = rnd(seed, (N, Hq, D)); k = rnd(seed + 1, (N, Hkv, D)); v = rnd(seed + 2, (N, Hkv, D))
    pos = np.arange(N); zero = np.zeros(N, np.int64)
    q = O.rope_remap(q, zero, pos, 1e4).astype(np.float32)
    k = O.rope_remap(k, zero, pos, 1e4).astype(np.float32)
    # the rotated inputs are the reference's (recorded rows)
    np.testing.assert_allclose(q[-1], d["q_rot_last"], atol=1e-5)
    np.testing.assert_allclose(k[::257], d["k_rot_sample"], atol=1e-5)
    ps = 16
    kv = np.stack([k, v], axis=1).reshape(N // ps, ps, 2, Hkv, D)
    kvd = to_dev(kv, "fp32")
    bt = torch.arange(N // ps, dtype=torch.int32, device="cuda")[None]
    cs = int(d["clear_start"])
    for win, key in ((0, "out_causal_fog"), (W, "out_window_fog")):
        out = ops.paged_fog_decode(to_dev(q[-1][None], "fp32"), kvd[:, :, 0], kvd[:, :, 1], bt,
                                   torch.tensor([N], dtype=torch.int32, device="cuda"),
                                   clear_start=torch.tensor([cs], dtype=torch.int32, device="cuda"),
                                   fog_alpha=0.5, window_size=win)
        torch.cuda.synchronize()
        assert out.dtype == torch.float32
        got = to_np(out)[0]
        np.testing.assert_allclose(got, d[key], **TOL["fp32"])
        want = O.paged_fog_decode(q[-1][None], kv[:, :, 0], kv[:, :, 1], np.arange(N // ps)[None], [N], [cs], 0.5,
                                  win)[0]
        np.testing.assert_allclose(got, want, **TOL["fp32"])


@pytest.mark.parametrize("Hq,Hkv", [(8, 8), (8, 2), (32, 8), (64, 8), (16, 1), (12, 2), (6, 3)])
def test_decode_fp32_gqa_shapes(Hq, Hkv):
    got, want = run_case(Hq * 10 + Hkv + 7, 3, Hq, Hkv, 128, "fp32", [700, 16, 2049])
    np.testing.assert_allclose(got, want, **TOL["fp32"])


@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("lens", [[1], [15, 17, 33], [4096], [9000, 12345], [70000]])
def test_decode_fp32_lengths(D, lens):
    """From one key to 70,000 keys (many splits per group, each split's
    partial merged by the group's last CTA)."""
    got, want = run_case(sum(lens) + 3, len(lens), 8, 2, D, "fp32", lens)
    np.testing.assert_allclose(got, want, **TOL["fp32"])


@pytest.mark.parametrize("window", [1, 16, 100, 3000])
def test_decode_fp32_reference_literal_window(window):
    got, want = run_case(window + 5, 2, 8, 2, 128, "fp32", [2500, 333], window=window)
    np.testing.assert_allclose(got, want, **TOL["fp32"])


@pytest.mark.parametrize("alpha,fogw", [(0.5, 64), (1.5, 300), (0.0, 64), (0.5, 0), (0.5, 5000), (0.7, 900)])
def test_decode_fp32_fog_params(alpha, fogw):
    got, want = run_case(17, 2, 8, 2, 128, "fp32", [1000, 4000], alpha=alpha, fog_window=fogw)
    np.testing.assert_allclose(got, want, **TOL["fp32"])


def test_decode_fp32_explicit_weights_offsets_and_pages():
    got, want = run_case(19, 1, 16, 4, 128, "fp32", [1500], explicit_weights=True)
    np.testing.assert_allclose(got, want, **TOL["fp32"])
    got, want = run_case(20, 3, 8, 2, 128, "fp32", [200, 700, 64], window=100, q_pos=[5000, 699, 63],
                         kv_off=[0, 0, 0])
    np.testing.assert_allclose(got, want, **TOL["fp32"])
    assert (got[0] == 0).all()
    for ps in (32, 64):
        got, want = run_case(21 + ps, 2, 8, 2, 128, "fp32", [500, 77], ps=ps)
        np.testing.assert_allclose(got, want, **TOL["fp32"])


def test_decode_fp32_empty_sequences_and_stale_nan():
    got, want = run_case(23, 4, 8, 2, 128, "fp32", [0, 300, 0, 45], nan_fill=True)
    assert np.isfinite(got).all()
    np.testing.assert_allclose(got, want, **TOL["fp32"])
    assert (got[0] == 0).all() and (got[2] == 0).all()


@pytest.mark.parametrize("B,D", [(100, 128), (70, 64)])
def test_decode_fp32_large_batch(B, D):
    lens = np.random.default_rng(B + 1).integers(1, 400, size=B)
    got, want = run_case(B + D + 1, B, 8, 2, D, "fp32", lens)
    np.testing.assert_allclose(got, want, **TOL["fp32"])


def test_decode_fp32_partials_for_the_lse_combine():
    """out_partial holds (O/l, m, l) with m in natural-log units; three shard
    decodes merged by the LSE combine equal the unsplit fp32 decode."""
    from kessie_b200 import ops
    D, Hq, Hkv, ps = 128, 16, 2, 16
    N = 3 * 1024
    kvn, kv = make_paged(31, N // ps, ps, Hkv, D, "fp32")
    q = rnd(32, (1, Hq, D))
    qd = to_dev(q, "fp32")
    cs = torch.tensor([N - 512], dtype=torch.int32, device="cuda")
    parts = torch.empty(3, 1, Hq, D + 2, dtype=torch.float32, device="cuda")
    for r in range(3):
        bt = torch.arange(r * 64, (r + 1) * 64, dtype=torch.int32, device="cuda")[None]
        ops.paged_fog_decode(qd, kv[:, :, 0], kv[:, :, 1], bt, torch.tensor([1024], dtype=torch.int32, device="cuda"),
                             clear_start=cs, fog_alpha=0.5,
                             kv_pos_offset=torch.tensor([r * 1024], dtype=torch.int32, device="cuda"),
                             q_positions=torch.tensor([N - 1], dtype=torch.int32, device="cuda"),
                             out_partial=parts[r], want_out=False)
    merged = ops.lse_combine(parts.contiguous(), out_dtype=torch.float32)
    torch.cuda.synchronize()
    want = O.paged_fog_decode(q, kvn[:, :, 0], kvn[:, :, 1], np.arange(N // ps, dtype=np.int32)[None], [N],
                              [N - 512], 0.5)
    np.testing.assert_allclose(to_np(merged), want, **TOL["fp32"])
    _, (ms, ls, _) = O.paged_fog_decode(q, kvn[:, :, 0], kvn[:, :, 1], np.arange(64, dtype=np.int32)[None], [1024],
                                        [N - 512], 0.5, return_partials=True)
    p0 = parts[0].cpu().numpy()
    np.testing.assert_allclose(p0[0, :, D], ms[0], atol=1e-5, rtol=1e-5)
    np.testing.assert_allclose(p0[0, :, D + 1], ls[0], rtol=1e-5)


def test_decode_fp32_bad_page_id_flagged_not_faulting():
    from kessie_b200 import ops
    ops.read_device_status()
    kvn, kv = make_paged(41, 8, 16, 2, 128, "fp32")
    bt = torch.tensor([[0, 1, 12345, 3]], dtype=torch.int32, device="cuda")
    q = rnd(42, (1, 8, 128))
    out = ops.paged_fog_decode(to_dev(q, "fp32"), kv[:, :, 0], kv[:, :, 1], bt,
                               torch.tensor([64], dtype=torch.int32, device="cuda"))
    st = ops.read_device_status()
    assert st & 0x1
    want = O.fog_attention_rows(q[0][:, None],
                                np.transpose(np.concatenate([kvn[i, :, 0] for i in (0, 1, 3)]), (1, 0, 2)),
                                np.transpose(np.concatenate([kvn[i, :, 1] for i in (0, 1, 3)]), (1, 0, 2)),
                                np.array([10 ** 6]))[:, 0]
    np.testing.assert_allclose(to_np(out)[0], want, **TOL["fp32"])


def test_decode_fp32_workspace_garbage_and_reuse():
    """Leftover workspace bytes are ignored, and repeated calls are
    bit-identical (the split merge order is fixed by slot)."""
    from kessie_b200 import ops, _lib
    lens = [3000, 40, 999, 1]
    B = len(lens)
    kvn, kv = make_paged(81, 400, 16, 2, 128, "fp32")
    bt_np = random_block_table(82, lens, 16, 400)
    bt = torch.from_numpy(bt_np).cuda()
    q = rnd(83, (B, 8, 128))
    need = _lib.load().kessie_paged_fog_decode_workspace_size(B, 8, 2, 128, bt.shape[1] * 16, 16)
    g = torch.Generator(device="cuda").manual_seed(84)
    ws = torch.randint(0, 256, (need,), dtype=torch.uint8, device="cuda", generator=g)
    cs = [n - 64 for n in lens]
    args = (to_dev(q, "fp32"), kv[:, :, 0], kv[:, :, 1], bt, torch.tensor(lens, dtype=torch.int32, device="cuda"))
    kw = dict(clear_start=torch.tensor(cs, dtype=torch.int32, device="cuda"), ws=ws)
    a = ops.paged_fog_decode(*args, **kw).clone()
    b = ops.paged_fog_decode(*args, **kw).clone()
    torch.cuda.synchronize()
    want = O.paged_fog_decode(q, kvn[:, :, 0], kvn[:, :, 1], bt_np, lens, cs, 0.5)
    np.testing.assert_allclose(to_np(a), want, **TOL["fp32"])
    assert torch.equal(a, b)
    assert ops.read_device_status() == 0


def test_decode_fp32_rejects_the_additive_bias():
    """The additive-bias decode form (vLLM path) is f16/bf16 only: an fp32
    call is refused with a status and launches nothing."""
    from kessie_b200 import _lib, ops
    kvn, kv = make_paged(91, 4, 16, 2, 128, "fp32")
    bt = torch.arange(4, dtype=torch.int32, device="cuda")[None]
    with pytest.raises(_lib.KessieError):
        ops.paged_fog_decode(to_dev(rnd(92, (1, 8, 128)), "fp32"), kv[:, :, 0], kv[:, :, 1], bt,
                             torch.tensor([64], dtype=torch.int32, device="cuda"),
                             bias=ops.FogBias(0.5, 0.5, dtype=torch.float32))


# ---------------------------------------------------------------- dense fp32 attention
def _dense(q, k, v, fog, W, causal):
    from kessie_b200 import kessie_hip_kernels as K
    qd, kd, vd = (to_dev(x, "fp32") for x in (q, k, v))
    if fog is None:
        out = K.kessie_windowed_attention(qd, kd, vd, W, causal)
    else:
        out = K.kessie_fused_fog_attention(qd, kd, vd, torch.from_numpy(np.asarray(fog, np.float32)).cuda(), W,
                                           causal)
    torch.cuda.synchronize()
    assert out.dtype == torch.float32
    return to_np(out)


def test_dense_fp32_reference_test_configs(golden_dir):
    """The reference's own attention test configurations
    (kessie_hip_kernels.py:623-626, :647-652) in fp32 through the dense entry
    points, against the outputs the reference's fp32 torch path recorded."""
    d = np.load(os.path.join(golden_dir, "attention.npz"))
    for i in range(int(d["nwin"])):
        Z, H, N, D, W, causal, seed = (int(x) for x in d[f"win{i}_cfg"])
        q, k, v = (rnd(seed + j, (Z, H, N, D)) for j in range(3))
        got = _dense(q, k, v, None, W, bool(causal))
        np.testing.assert_allclose(got[:, :, d[f"win{i}_rows"]], d[f"win{i}_out"], **TOL["fp32"],
                                   err_msg=f"windowed config {i}")
    for i in range(int(d["nfog"])):
        Z, H, N, D, W, causal, seed = (int(x) for x in d[f"fog{i}_cfg"])
        a, fs = d[f"fog{i}_fog"]
        q, k, v = (rnd(seed + j, (Z, H, N, D)) for j in range(3))
        got = _dense(q, k, v, O.build_fog_weights(N, a, fs), W, bool(causal))
        np.testing.assert_allclose(got[:, :, d[f"fog{i}_rows"]], d[f"fog{i}_out"], **TOL["fp32"],
                                   err_msg=f"fog config {i}")


def test_dense_fp32_config1_full_square(golden_dir):
    """Config 1 as the reference evaluates it: the whole 4096 x 4096 fp32
    attention (GQA 8/2, RoPE'd q/k, fog), whose last row the reference
    recorded for both fog mappings."""
    d = np.load(os.path.join(golden_dir, "config1_decode.npz"))
    B, Hq, Hkv, D, N, W, seed = (int(x) for x in d["cfg"])
    q = rnd(seed, (N, Hq, D)); k = rnd(seed + 1, (N, Hkv, D)); v = rnd(seed + 2, (N, Hkv, D))
    pos = np.arange(N); zero = np.zeros(N, np.int64)
    q = O.rope_remap(q, zero, pos, 1e4).astype(np.float32)
    k = O.rope_remap(k, zero, pos, 1e4).astype(np.float32)
    qh, kh, vh = (np.ascontiguousarray(np.transpose(x, (1, 0, 2))[None]) for x in (q, k, v))
    fog = O.build_fog_weights(N, 0.5, W / N)
    for win, key in ((0, "out_causal_fog"), (W, "out_window_fog")):
        got = _dense(qh, kh, vh, fog, win, True)
        np.testing.assert_allclose(got[0, :, -1], d[key], **TOL["fp32"])
        rows = np.array([0, 1, 511, 512, 2047, N - 2])
        want = O.fog_attention_rows(qh[0][:, rows], kh[0], vh[0], rows, fog, window_size=win)
        np.testing.assert_allclose(got[0][:, rows], want, **TOL["fp32"])


@pytest.mark.parametrize("W,causal", [(0, True), (0, False), (37, True), (37, False)])
def test_dense_fp32_ragged_gqa(W, causal):
    """N not a multiple of 8 (the last key chunk ends inside the tensor),
    GQA 6/3, head_dim 64, two sequences, every row against the oracle."""
    B, Hq, Hkv, N, D = 2, 6, 3, 1001, 64
    q = rnd(71, (B, Hq, N, D)); k = rnd(72, (B, Hkv, N, D)); v = rnd(73, (B, Hkv, N, D))
    fog = O.fog_weights_from_clear_start(N, N - 300, 0.5)
    got = _dense(q, k, v, fog, W, causal)
    for b in range(B):
        want = O.fog_attention_rows(q[b], k[b], v[b], np.arange(N), fog, window_size=W, causal=causal)
        np.testing.assert_allclose(got[b], want, **TOL["fp32"], err_msg=f"sequence {b}")
