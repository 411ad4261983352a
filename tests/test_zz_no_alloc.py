"""GPU test of the allocation-free decode entry point.

kessie_paged_fog_decode_noalloc_v2 is for callers that cannot allocate device
memory when they decode (their allocator is fixed or owned by another
runtime), so it keeps its split-KV scratch in an array built into the
library.  This file checks, through the C ABI, that two calls in a row give
the same results as kessie_paged_fog_decode_v2 with a caller-provided
workspace and as the oracle, and that a shape too large for the built-in
array is refused.
The file name sorts last so a run that stops at the first failure has
already run every other test; it also passes on its own in a fresh process.
"""

import ctypes
import math

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

TOL = dict(atol=2e-2, rtol=1e-2)     # the bf16 bar used by every decode test


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    yield


def _inputs(seed, lens, Hq=32, Hkv=8, D=128, ps=16):
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    need = [(n + ps - 1) // ps for n in lens]
    P = sum(need) + 2
    kv = torch.randn(P, ps, 2, Hkv, D, generator=g, device="cuda").to(torch.bfloat16)
    perm = torch.randperm(P, generator=g, device="cuda").to(torch.int32)
    bt = torch.zeros(len(lens), max(need), dtype=torch.int32, device="cuda")
    o = 0
    for b, k in enumerate(need):
        bt[b, :k] = perm[o:o + k]
        o += k
    q = torch.randn(len(lens), Hq, D, generator=g, device="cuda").to(torch.bfloat16)
    sl = torch.tensor(lens, dtype=torch.int32, device="cuda")
    cs = (sl - 256).clamp_min(0).to(torch.int32)
    return q, kv, bt, sl, cs, P, ps


def _args(q, kv, bt, sl, cs, P, ps, Hkv, D):
    k, v = kv[:, :, 0], kv[:, :, 1]
    return [q.data_ptr(), q.stride(0), q.stride(1), k.data_ptr(), v.data_ptr(), k.stride(0), k.stride(1),
            k.stride(2), P, ps, bt.data_ptr(), bt.stride(0), sl.data_ptr(), None, None, cs.data_ptr(),
            ctypes.c_float(0.5), None, 0, ctypes.c_float(1.0 / math.sqrt(D)), q.shape[0], q.shape[1], Hkv, D,
            bt.shape[1] * ps, 1]


def test_noalloc_decode_matches_workspace_decode_twice():
    from kessie_b200 import _lib
    lib = _lib.load()
    Hkv, D = 8, 128
    for seed, lens in ((1, [1000, 40, 3000]), (2, [5000, 17])):
        q, kv, bt, sl, cs, P, ps = _inputs(seed, lens)
        args = _args(q, kv, bt, sl, cs, P, ps, Hkv, D)
        ws_n = lib.kessie_paged_fog_decode_workspace_size(q.shape[0], q.shape[1], Hkv, D, bt.shape[1] * ps, ps)
        ws = torch.empty(ws_n, dtype=torch.uint8, device="cuda")
        ref = torch.empty_like(q)
        _lib.check(lib.kessie_paged_fog_decode_v2(*args, ref.data_ptr(), None, ws.data_ptr(), ws_n, None),
                   "workspace decode")
        got = torch.full_like(q, float("nan"))
        _lib.check(lib.kessie_paged_fog_decode_noalloc_v2(*args, got.data_ptr(), None, None), "noalloc decode")
        torch.cuda.synchronize()
        np.testing.assert_allclose(got.float().cpu().numpy(), ref.float().cpu().numpy(), **TOL)
        # and directly against the oracle restatement of the reference's decode
        from oracle import fog_oracle as O
        kvn = kv.float().cpu().numpy()
        want = O.paged_fog_decode(q.float().cpu().numpy(), kvn[:, :, 0], kvn[:, :, 1], bt.cpu().numpy(),
                                  sl.cpu().numpy(), cs.cpu().numpy(), 0.5)
        np.testing.assert_allclose(got.float().cpu().numpy(), want, **TOL)


def test_noalloc_decode_rejects_shapes_beyond_its_scratch():
    from kessie_b200 import _lib
    lib = _lib.load()
    # the scratch holds one fp32 partial per query head for every (CTA, group)
    # segment: 1024 sequences x 128 query heads is far beyond the built-in array
    need = lib.kessie_paged_fog_decode_workspace_size(1024, 128, 8, 128, 4096, 16)
    assert need > 16 * 1024 * 1024
    z = torch.zeros(16, dtype=torch.int32, device="cuda")
    rc = lib.kessie_paged_fog_decode_noalloc_v2(z.data_ptr(), 0, 0, z.data_ptr(), z.data_ptr(), 0, 0, 0, 1, 16,
                                                z.data_ptr(), 0, z.data_ptr(), None, None, None, ctypes.c_float(0.5),
                                                None, 0, ctypes.c_float(0.1), 1024, 128, 8, 128, 4096, 1,
                                                z.data_ptr(), None, None)
    assert rc == 3
    st, msg = _lib.last_error()
    assert st == 3 and "scratch" in msg
