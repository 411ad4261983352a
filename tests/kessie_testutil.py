"""Helpers shared by the GPU parity tests (seeded inputs, paged caches)."""

import numpy as np
import torch

from oracle import fog_oracle as O

TORCH_DT = {"bf16": torch.bfloat16, "fp16": torch.float16, "fp32": torch.float32}
ROUND = {"bf16": O.round_bf16, "fp16": O.round_f16, "fp32": lambda x: np.asarray(x, np.float32)}

# the bf16 / fp16 / fp32 parity bars of the target path (1e-4 fp32; 2e-2 abs / 1e-2 rel bf16, fp16)
TOL = {"bf16": dict(atol=2e-2, rtol=1e-2), "fp16": dict(atol=2e-2, rtol=1e-2), "fp32": dict(atol=1e-4, rtol=0)}


def rnd(seed, shape, scale=1.0):
    return np.random.default_rng(seed).standard_normal(shape, dtype=np.float32) * np.float32(scale)


def to_dev(x, dt, device="cuda"):
    return torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32)).to(device=device, dtype=TORCH_DT[dt])


def to_np(t):
    return t.detach().float().cpu().numpy()


def make_paged(seed, num_pages, ps, Hkv, D, dt, fill_nan=False, scale=1.0):
    """A [P, ps, 2, Hkv, D] cache with random contents (values in `dt`)."""
    kv = rnd(seed, (num_pages, ps, 2, Hkv, D), scale)
    kv = ROUND[dt](kv)
    t = to_dev(kv, dt)
    return kv, t


def random_block_table(seed, seq_lens, ps, num_pages):
    """Non-contiguous random placement: one permutation of the pool."""
    rng = np.random.default_rng(seed)
    need = [(int(n) + ps - 1) // ps for n in seq_lens]
    assert sum(need) <= num_pages
    perm = rng.permutation(num_pages)
    maxp = max(max(need), 1)
    bt = np.full((len(seq_lens), maxp), -1, dtype=np.int32)
    o = 0
    for b, k in enumerate(need):
        bt[b, :k] = perm[o:o + k]
        o += k
    return bt
