"""numpy restatement of the reference's fog-attention hot path (test oracle).

TEST INFRASTRUCTURE ONLY -- imported by tests/, __graft_entry__.smoke() and
bench.py's CPU baseline, never by the product package.

Every function cites the reference file:line whose semantics it restates
(paths are relative to the sentinelXVI/KeSSie source tree).  Attention is
evaluated in float64 on the given (already dtype-rounded) inputs; element
copies (page insert / gather) are done on raw storage so they are bit-exact
for any dtype.
"""

from __future__ import annotations

import math
from typing import List, Optional, Sequence, Tuple

import numpy as np

__all__ = [
    "f32_to_bf16_bits", "bf16_bits_to_f32", "round_bf16", "round_f16",
    "clear_start_for", "build_fog_weights", "fog_weights_from_clear_start",
    "windowed_attention", "fused_fog_attention", "fog_attention_rows",
    "rope_freqs", "rope_remap", "rope_remap_fp32_inplace_reference", "page_evict", "PagedKVCacheOracle",
    "page_gather", "paged_fog_decode", "paged_fog_prefill", "lse_combine",
    "partials_from_rows", "fog_decode_group_fp32",
]


# ---------------------------------------------------------------------------
# dtype helpers (bf16 round-to-nearest-even, as torch's .to(torch.bfloat16))
# ---------------------------------------------------------------------------

def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    r = ((u >> 16) & 1) + np.uint32(0x7FFF)
    out = ((u + r) >> 16).astype(np.uint16)
    out[nan] = 0x7FC0
    return out


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.ascontiguousarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def round_bf16(x: np.ndarray) -> np.ndarray:
    return bf16_bits_to_f32(f32_to_bf16_bits(x))


def round_f16(x: np.ndarray) -> np.ndarray:
    return np.asarray(x, dtype=np.float32).astype(np.float16).astype(np.float32)


# ---------------------------------------------------------------------------
# Additive fog bias of the vLLM path -- kessie_attention.py:114-139
# (_FogCache._compute_into)
# ---------------------------------------------------------------------------

_ROUND = {"float32": lambda x: np.asarray(x, dtype=np.float32), "bfloat16": round_bf16, "float16": round_f16}


def fog_bias_values(kv_len: int, fog_alpha: float, fog_start: float, recall_positions=(),
                    recall_boost: float = 0.1, dtype: str = "float32") -> np.ndarray:
    """The reference's bias buffer of kv_len entries: -fog_alpha * (1 - j/fb)^2
    for j < fb = int(kv_len * (1 - fog_start)), 0 after, recall_boost at the
    recalled positions; every torch op of the reference (arange, divide,
    rsub, square, scale) rounded to `dtype` like its buffer, the arange
    element by element (as on the GPU the reference runs it on).  fp32 values."""
    rnd = _ROUND[dtype]
    out = np.zeros(kv_len, dtype=np.float32)
    fb = int(kv_len * (1.0 - fog_start))
    if fb > 0:
        with np.errstate(over="ignore", invalid="ignore"):     # fp16 positions above 65504 are inf
            pos = rnd(np.arange(fb, dtype=np.float32))
            t = rnd(pos / np.float32(fb))
            d = rnd(np.float32(1.0) - t)
            d = rnd(d * d)
            out[:fb] = rnd(d * np.float32(-fog_alpha))
    boost = np.asarray(rnd(np.array([recall_boost], dtype=np.float32)), dtype=np.float32)[0]
    for p in recall_positions:
        if 0 <= p < kv_len:
            out[p] = boost
    return out


# ---------------------------------------------------------------------------
# Fog weights -- kessie_hip_kernels.py:403-413 (kessie_build_fog_weights)
# ---------------------------------------------------------------------------

def clear_start_for(seq_len: int, fog_start: float) -> int:
    """kessie_hip_kernels.py:409 -- ``int(seq_len * (1.0 - fog_start))`` in
    Python float64; kernels receive this integer, never recompute it."""
    return int(seq_len * (1.0 - fog_start))


def fog_weights_from_clear_start(n: int, clear_start: int, fog_alpha: float) -> np.ndarray:
    """Weights for positions 0..n-1 given the clear-zone start.

    kessie_hip_kernels.py:408-412: ones, then for j < clear_start (when
    alpha > 0 and clear_start > 0) ``(j / max(cs-1, 1)) ** alpha``.  The ratio
    is a float32 division (exact integer operands below 2**24)."""
    w = np.ones(n, dtype=np.float32)
    cs = int(clear_start)
    if fog_alpha > 0 and cs > 0:
        m = min(cs, n)
        t = np.arange(m, dtype=np.float32) / np.float32(max(cs - 1, 1))
        w[:m] = np.power(t.astype(np.float64), float(np.float32(fog_alpha))).astype(np.float32)
    return w


def build_fog_weights(seq_len: int, fog_alpha: float = 0.5, fog_start: float = 0.5) -> np.ndarray:
    """kessie_hip_kernels.py:403-413."""
    return fog_weights_from_clear_start(seq_len, clear_start_for(seq_len, fog_start), fog_alpha)


# ---------------------------------------------------------------------------
# Attention -- kessie_hip_kernels.py:577-593 (the reference's PyTorch oracle)
# ---------------------------------------------------------------------------

def _mask(q_pos: np.ndarray, k_pos: np.ndarray, window_size: int, causal: bool) -> np.ndarray:
    """kessie_hip_kernels.py:582-587: causal keeps j <= i; window W > 0 keeps
    0 <= i - j < W (which implies causal)."""
    dist = q_pos[:, None].astype(np.int64) - k_pos[None, :].astype(np.int64)
    ok = np.ones(dist.shape, dtype=bool)
    if causal:
        ok &= dist >= 0
    if window_size > 0:
        ok &= (dist >= 0) & (dist < window_size)
    return ok


def _softmax_rows_pv(scores: np.ndarray, ok: np.ndarray, vw: np.ndarray) -> np.ndarray:
    s = np.where(ok, scores, -np.inf)
    m = s.max(axis=-1, keepdims=True)
    m = np.where(np.isfinite(m), m, 0.0)
    p = np.exp(s - m)
    l = p.sum(axis=-1, keepdims=True)
    with np.errstate(invalid="ignore", divide="ignore"):
        return (p @ vw) / l


def windowed_attention(q, k, v, window_size: int = 0, causal: bool = True,
                       sm_scale: Optional[float] = None) -> np.ndarray:
    """kessie_hip_kernels.py:577-588: square [Z,H,N,D] attention."""
    Z, H, N, D = q.shape
    if sm_scale is None:
        sm_scale = 1.0 / math.sqrt(D)
    pos = np.arange(N)
    ok = _mask(pos, pos, window_size, causal)
    q64, k64, v64 = (np.asarray(t, dtype=np.float64) for t in (q, k, v))
    out = np.empty((Z, H, N, D), dtype=np.float64)
    for z in range(Z):
        for h in range(H):
            s = (q64[z, h] @ k64[z, h].T) * sm_scale
            out[z, h] = _softmax_rows_pv(s, ok, v64[z, h])
    return out


def fused_fog_attention(q, k, v, fog_weights, window_size: int = 0, causal: bool = True,
                        sm_scale: Optional[float] = None) -> np.ndarray:
    """kessie_hip_kernels.py:591-593: windowed attention on V * fog[j]."""
    vw = np.asarray(v, dtype=np.float64) * np.asarray(fog_weights, dtype=np.float64)[None, None, :, None]
    return windowed_attention(q, k, vw, window_size, causal, sm_scale)


def fog_attention_rows(q, k, v, q_pos, fog_w=None, window_size: int = 0, causal: bool = True,
                       sm_scale: Optional[float] = None, k_pos=None,
                       return_partials: bool = False, dtype=np.float64, score_bias=None):
    """Query-offset, GQA restatement of kessie_hip_kernels.py:577-593.

    q: [Hq, Nq, D] at absolute positions q_pos[Nq]; k, v: [Hkv, N, D] at
    positions k_pos (default 0..N-1); fog_w: [N] weight per key.  Query head
    h reads KV head h // (Hq // Hkv).  Same mask, softmax and ``@ (v*fog)``
    as the square reference; validated against its last rows.
    With return_partials, also returns (m, l, O_unnormalised) in natural-log
    units for the LSE combine.  dtype=np.float32 evaluates in fp32 like the
    reference's torch path (used for the timed CPU baseline).
    A row with no visible key (N == 0, or every key masked) is 0 with
    m = -inf, l = 0: the reference's softmax of an all-masked row is NaN, so
    this build defines the empty row as the neutral element of the merge
    (a context-parallel shard may hold none of a sequence's window).
    score_bias: optional [N] added to the scaled scores (the vLLM path's
    additive fog bias, kessie_attention.py:114-139)."""
    q = np.asarray(q, dtype=dtype)
    k = np.asarray(k, dtype=dtype)
    v = np.asarray(v, dtype=dtype)
    Hq, Nq, D = q.shape
    Hkv, N, _ = k.shape
    g = Hq // Hkv
    if sm_scale is None:
        sm_scale = 1.0 / math.sqrt(D)
    if k_pos is None:
        k_pos = np.arange(N)
    ok = _mask(np.asarray(q_pos), np.asarray(k_pos), window_size, causal)
    w = np.ones(N, dtype=dtype) if fog_w is None else np.asarray(fog_w, dtype=dtype)
    out = np.empty((Hq, Nq, D), dtype=dtype)
    ms = np.empty((Hq, Nq), dtype=dtype); ls = np.empty((Hq, Nq), dtype=dtype); os_ = np.empty((Hq, Nq, D), dtype=dtype)
    for h in range(Hq):
        kh = h // g
        s = (q[h] @ k[kh].T) * dtype(sm_scale)
        if score_bias is not None:
            s = s + np.asarray(score_bias, dtype=dtype)[None, :]
        s = np.where(ok, s, dtype(-np.inf))
        m = s.max(axis=-1, keepdims=True, initial=-np.inf)
        mf = np.where(np.isfinite(m), m, 0.0)
        p = np.exp(s - mf)
        l = p.sum(axis=-1, keepdims=True)
        o = p @ (v[kh] * w[:, None])
        with np.errstate(invalid="ignore", divide="ignore"):
            out[h] = np.where(l > 0, o / np.where(l > 0, l, 1.0), 0.0)
        ms[h] = m[:, 0]; ls[h] = l[:, 0]; os_[h] = o
    if return_partials:
        return out, (ms, ls, os_)
    return out


def fog_decode_group_fp32(q: np.ndarray, k: np.ndarray, v: np.ndarray, w: np.ndarray,
                          sm_scale: Optional[float] = None) -> np.ndarray:
    """Last-row (decode) evaluation of kessie_hip_kernels.py:577-593 for the
    G query heads of one KV head, in fp32 like the reference's torch path:
    q [G, D]; k, v [N, D] (all N keys visible); w [N] fog weights.  Batched
    as two GEMMs (scores [G, N], then P @ (V * w)); used as the timed CPU
    baseline."""
    q = np.asarray(q, np.float32); k = np.asarray(k, np.float32); v = np.asarray(v, np.float32)
    if sm_scale is None:
        sm_scale = 1.0 / math.sqrt(q.shape[-1])
    s = (q @ k.T) * np.float32(sm_scale)
    s -= s.max(axis=1, keepdims=True)
    np.exp(s, out=s)
    l = s.sum(axis=1, keepdims=True)
    vw = v * np.asarray(w, np.float32)[:, None]
    return (s @ vw) / l


def lse_combine(ms: np.ndarray, ls: np.ndarray, os_: np.ndarray) -> np.ndarray:
    """Merge split partials: M = max m_s, L = sum l_s e^(m_s-M),
    O = sum O_s e^(m_s-M) / L.  The per-split rescale is the online-softmax
    step of kessie_hip_kernels.py:142-146,158,162 applied across splits
    (the reference itself has no split-KV path).
    ms, ls: [S, ...]; os_: [S, ..., D] (unnormalised sums)."""
    M = np.max(ms, axis=0)
    Mf = np.where(np.isfinite(M), M, 0.0)
    sc = np.where(np.isfinite(ms), np.exp(ms - Mf[None]), 0.0)
    L = (ls * sc).sum(axis=0)
    O = (os_ * sc[..., None]).sum(axis=0)
    with np.errstate(invalid="ignore", divide="ignore"):
        return np.where(L[..., None] > 0, O / np.where(L > 0, L, 1.0)[..., None], 0.0)


def partials_from_rows(ms, ls, os_):
    """Pack (m, l, O_unnormalised) into the [.., D+2] triple layout used by
    the CUDA library: [O/l (D values), m, l] in float32."""
    D = os_.shape[-1]
    out = np.zeros(ms.shape + (D + 2,), dtype=np.float32)
    with np.errstate(invalid="ignore", divide="ignore"):
        out[..., :D] = np.where(ls[..., None] > 0, os_ / np.where(ls > 0, ls, 1.0)[..., None], 0.0)
    out[..., D] = np.where(np.isfinite(ms), ms, -np.inf)
    out[..., D + 1] = ls
    return out


# ---------------------------------------------------------------------------
# RoPE remap -- kessie_hip_kernels.py:596-606 (_rope_remap_ref),
#               kessie_kernels_v2.hip:670-707 (kessie_rope_remap)
# ---------------------------------------------------------------------------

def rope_freqs(half_dim: int, rope_theta: float) -> np.ndarray:
    """kessie_hip_kernels.py:600: ``1 / theta ** (arange(half)/half)`` in
    float32.  theta**e is evaluated in float64 and rounded to float32 before
    the float32 reciprocal; this reproduces torch's table bit-for-bit at the
    thetas the configs use (1e4, 5e5), pinned by tests/golden/rope_*.npz."""
    e = np.arange(half_dim, dtype=np.float32) / np.float32(half_dim)
    p = np.power(np.float64(np.float32(rope_theta)), e.astype(np.float64)).astype(np.float32)
    return (np.float32(1.0) / p).astype(np.float32)


def rope_remap(k: np.ndarray, orig_positions, target_positions, rope_theta: float = 10000.0,
               freqs: Optional[np.ndarray] = None) -> np.ndarray:
    """kessie_hip_kernels.py:596-606.  k: [T, H, D] float32 values (already
    rounded to the storage dtype).  Returns float32 results before the final
    cast to storage dtype (caller rounds).  Rotate-half pairs (d, d+D/2):
    k1' = k1 cos - k2 sin, k2' = k1 sin + k2 cos with delta = (tgt-orig)*f_d."""
    T, H, D = k.shape
    half = D // 2
    f = rope_freqs(half, rope_theta) if freqs is None else freqs
    dp = (np.asarray(target_positions, dtype=np.int64) - np.asarray(orig_positions, dtype=np.int64)).astype(np.float32)
    delta = dp[:, None] * f[None, :]                       # float32 outer product
    c = np.cos(delta.astype(np.float64)).astype(np.float32)[:, None, :]
    s = np.sin(delta.astype(np.float64)).astype(np.float32)[:, None, :]
    k = np.asarray(k, dtype=np.float32)
    k1, k2 = k[:, :, :half], k[:, :, half:]
    out = np.empty_like(k)
    out[:, :, :half] = k1 * c - k2 * s
    out[:, :, half:] = k1 * s + k2 * c
    return out


def rope_remap_fp32_inplace_reference(k: np.ndarray, orig_positions, target_positions,
                                      rope_theta: float = 10000.0) -> np.ndarray:
    """What kessie_hip_kernels.py:603-605 actually computes for an fp32 K:
    ``k1 = k_tensor[..., :half].float()`` is a VIEW for fp32 storage, so the
    second half is rotated with the already-updated first half
    (k2' = k1' sin + k2 cos).  Kept only to pin that golden vector and
    document the divergence; the CUDA library follows the HIP kernel
    (kessie_kernels_v2.hip:697-706), which rotates from the loaded pair."""
    T, H, D = k.shape
    half = D // 2
    f = rope_freqs(half, rope_theta)
    dp = (np.asarray(target_positions, dtype=np.int64) - np.asarray(orig_positions, dtype=np.int64)).astype(np.float32)
    delta = dp[:, None] * f[None, :]
    c = np.cos(delta.astype(np.float64)).astype(np.float32)[:, None, :]
    s = np.sin(delta.astype(np.float64)).astype(np.float32)[:, None, :]
    k = np.asarray(k, dtype=np.float32)
    out = np.empty_like(k)
    out[:, :, :half] = k[:, :, :half] * c - k[:, :, half:] * s
    out[:, :, half:] = out[:, :, :half] * s + k[:, :, half:] * c
    return out


# ---------------------------------------------------------------------------
# Paged KV cache -- kessie_kernels_v2.hip:393-456, kessie_hip_kernels.py:484-570
# ---------------------------------------------------------------------------

def page_evict(page_valid: np.ndarray, page_positions: np.ndarray, evict_before_pos: int):
    """kessie_kernels_v2.hip:393-407: valid==1 and pos < thr -> valid=0 and
    count += 1.  Returns (new_valid, count, evicted_ids ascending)."""
    v = np.array(page_valid, dtype=np.int8, copy=True)
    hit = (v == 1) & (np.asarray(page_positions, dtype=np.int64) < int(evict_before_pos))
    v[hit] = 0
    ids = np.nonzero(hit)[0].astype(np.int32)
    return v, int(hit.sum()), ids


def page_gather(kv_pages: np.ndarray, page_ids: Sequence[int]):
    """kessie_hip_kernels.py:558-564 (get_layer_kv): pages [P, ps, 2, H, D] ->
    K, V [n*ps, H, D] in the order of page_ids."""
    sel = kv_pages[np.asarray(page_ids, dtype=np.int64)]
    n, ps, _, H, D = sel.shape
    kv = sel.reshape(-1, 2, H, D)
    return kv[:, 0].copy(), kv[:, 1].copy()


class PagedKVCacheOracle:
    """Host bookkeeping of KeSSiePagedKVCache (kessie_hip_kernels.py:484-570)
    with device eviction semantics taken from kessie_kernels_v2.hip:393-407
    (the Triton evict grid of :527-533 examines only ceil(P/256) pages and the
    no-Triton branch never clears page_valid; the HIP kernel is the
    authoritative rule).  Storage is a numpy array of the element dtype so
    copies are bit-exact."""

    def __init__(self, num_pages, page_size, num_layers, num_heads, head_dim, np_dtype=np.uint16):
        self.num_pages, self.page_size = num_pages, page_size
        self.num_layers, self.num_heads, self.head_dim = num_layers, num_heads, head_dim
        self.kv_data = np.zeros((num_layers, num_pages, page_size, 2, num_heads, head_dim), dtype=np_dtype)
        self.page_positions = np.zeros(num_pages, dtype=np.int32)
        self.page_valid = np.zeros(num_pages, dtype=np.int8)
        self.free_pages: List[int] = list(range(num_pages))          # :501
        self.total_evictions = 0
        self.total_insertions = 0

    @property
    def active_pages(self):                                          # :513-514
        return self.num_pages - len(self.free_pages)

    def allocate_pages(self, n):                                     # :520-524 (LIFO pop)
        if len(self.free_pages) < n:
            return None
        return [self.free_pages.pop() for _ in range(n)]

    def evict_before(self, position):                                # :526-540
        hit = (self.page_valid == 1) & (self.page_positions.astype(np.int64) < position)
        self.page_valid[hit] = 0
        free = set(self.free_pages)
        evicted = 0
        for i in range(self.num_pages):                              # ascending scan, :535-538
            if self.page_valid[i] == 0 and i not in free:
                self.free_pages.append(i)
                evicted += 1
        self.total_evictions += evicted
        return evicted

    def insert_probe_kv(self, layer_idx, keys, values, conv_position):   # :542-556
        T = keys.shape[0]
        need = (T + self.page_size - 1) // self.page_size
        ids = self.allocate_pages(need)
        if ids is None:
            return False
        for p, pid in enumerate(ids):
            s, e = p * self.page_size, min((p + 1) * self.page_size, T)
            self.kv_data[layer_idx, pid, : e - s, 0] = keys[s:e]
            self.kv_data[layer_idx, pid, : e - s, 1] = values[s:e]
            self.page_valid[pid] = 1
            self.page_positions[pid] = conv_position + s
        self.total_insertions += T
        return ids

    def get_layer_kv(self, layer_idx):                               # :558-564
        valid = np.nonzero(self.page_valid != 0)[0]
        return page_gather(self.kv_data[layer_idx], valid)

    def get_stats(self):                                             # :566-570
        es = self.kv_data.dtype.itemsize
        return {"total_pages": self.num_pages, "active_pages": self.active_pages,
                "free_pages": len(self.free_pages), "active_tokens": self.active_pages * self.page_size,
                "vram_gb": self.kv_data.size * es / 1e9,
                "total_evictions": self.total_evictions, "total_insertions": self.total_insertions}


# ---------------------------------------------------------------------------
# Paged decode / prefill restatements (new entry points; math of a3 + GQA)
# ---------------------------------------------------------------------------

def _gather_seq(pages: np.ndarray, block_row: np.ndarray, n: int, page_size: int) -> np.ndarray:
    """pages: [P, ps, Hkv, D] float -> [Hkv, n, D] for the first n tokens."""
    npg = (n + page_size - 1) // page_size
    sel = pages[np.asarray(block_row[:npg], dtype=np.int64)]            # [npg, ps, H, D]
    flat = sel.reshape(npg * page_size, *sel.shape[2:])[:n]
    return np.transpose(flat, (1, 0, 2))


def paged_fog_decode(q, k_pages, v_pages, block_table, seq_lens, clear_start, fog_alpha,
                     window_size=0, sm_scale=None, kv_pos_offset=None, q_pos=None,
                     fog_weights=None, return_partials=False, bias_spec=None):
    """Decode restatement over a paged cache.

    q: [B, Hq, D]; k_pages/v_pages: [P, ps, Hkv, D] (values); block_table:
    [B, maxP]; seq_lens[b] local keys; kv_pos_offset[b] global position of
    local key 0 (context-parallel shards, default 0); q_pos[b] query
    position (default offset+len-1); clear_start[b] in global positions.
    Fog weight of key at global position j: kessie_hip_kernels.py:411-412
    with clear_start[b] (or fog_weights[j] when given).  bias_spec =
    (fog_alpha, fog_start, recall_positions, recall_boost, dtype) adds the
    vLLM path's fog bias of a qp+1-key sequence to the scores."""
    B, Hq, D = q.shape
    ps = k_pages.shape[1]
    out = np.zeros((B, Hq, D))
    parts = []
    for b in range(B):
        n = int(seq_lens[b])
        off = 0 if kv_pos_offset is None else int(kv_pos_offset[b])
        qp = off + n - 1 if q_pos is None else int(q_pos[b])
        kpos = off + np.arange(n)
        if fog_weights is not None:
            w = np.asarray(fog_weights, dtype=np.float64)[kpos]
        else:
            cs = int(clear_start[b])
            w = fog_weights_from_clear_start(off + n, cs, fog_alpha)[off:off + n]
        kk = _gather_seq(k_pages, block_table[b], n, ps)
        vv = _gather_seq(v_pages, block_table[b], n, ps)
        sb = None
        if bias_spec is not None:
            sb = fog_bias_values(qp + 1, *bias_spec)[kpos] if n else np.zeros(0, np.float32)
        o, (m, l, ou) = fog_attention_rows(q[b][:, None, :], kk, vv, np.array([qp]), w,
                                           window_size, True, sm_scale, k_pos=kpos,
                                           return_partials=True, score_bias=sb)
        out[b] = o[:, 0]
        parts.append((m[:, 0], l[:, 0], ou[:, 0]))
    if return_partials:
        ms = np.stack([p[0] for p in parts]); ls = np.stack([p[1] for p in parts])
        os_ = np.stack([p[2] for p in parts])
        return out, (ms, ls, os_)
    return out


def paged_fog_prefill(q, k_pages, v_pages, block_table, kv_len, q_start, clear_start, fog_alpha,
                      window_size=0, sm_scale=None, fog_weights=None, bias_spec=None):
    """Chunked-prefill restatement: q [Hq, Nq, D] are the queries at absolute
    positions q_start..q_start+Nq-1 attending causally (plus optional window)
    over kv_len paged keys; one sequence.  bias_spec as in paged_fog_decode
    (the bias of a kv_len-key sequence; no V fog is applied with it)."""
    ps = k_pages.shape[1]
    n = int(kv_len)
    Nq = q.shape[1]
    if fog_weights is not None:
        w = np.asarray(fog_weights, dtype=np.float64)[:n]
    else:
        w = fog_weights_from_clear_start(n, clear_start, fog_alpha)
    kk = _gather_seq(k_pages, block_table, n, ps)
    vv = _gather_seq(v_pages, block_table, n, ps)
    sb = fog_bias_values(n, *bias_spec) if bias_spec is not None else None
    return fog_attention_rows(q, kk, vv, q_start + np.arange(Nq), w, window_size, True, sm_scale, score_bias=sb)


# ---------------------------------------------------------------------------
# Conversation-index query -- kessie_hip_kernels.py:343-360 (the GPU kernel)
# and VectorIndex (kessie_exp3.py:58-110, rows stored normalised)
# ---------------------------------------------------------------------------

def vector_index_rows(index: np.ndarray) -> np.ndarray:
    """Rows normalised as VectorIndex.rebuild stores them (norm < 1e-8 -> 1)."""
    mat = np.asarray(index, dtype=np.float32)
    norms = np.linalg.norm(mat, axis=1, keepdims=True)
    norms[norms < 1e-8] = 1.0
    return mat / norms


def index_query(query: np.ndarray, index: np.ndarray, normalize_rows: bool = True, top_k: int = 0):
    """(sims, top ids, top scores) in float64.  The query is divided by
    sqrt(|q|^2 + 1e-8); with normalize_rows each row by sqrt(|x|^2 + 1e-8)
    (the GPU kernel), else the rows are taken as stored.  Top-k: descending
    score, ties to the lower row index."""
    q = np.asarray(query, dtype=np.float64)
    x = np.asarray(index, dtype=np.float64)
    qn = q / np.sqrt((q * q).sum() + 1e-8)
    if normalize_rows:
        x = x / np.sqrt((x * x).sum(axis=1, keepdims=True) + 1e-8)
    sims = x @ qn
    order = np.lexsort((np.arange(len(sims)), -sims))[:top_k]
    return sims, order, sims[order]


def vector_index_search_fp32(rows: np.ndarray, query: np.ndarray, top_k: int = 5):
    """VectorIndex.search's numpy path (kessie_exp3.py:89-103) in float32, as
    the reference runs it: the query divided by its norm (empty result below
    1e-8), sims = rows @ q over the stored normalised rows, the k = min(top_k,
    rows) largest by a full argsort, best first.  The timed CPU baseline of the
    index query; returns (ids, scores)."""
    q = np.asarray(query, dtype=np.float32).reshape(1, -1)
    qn = np.linalg.norm(q)
    if qn < 1e-8 or len(rows) == 0:
        return np.zeros(0, np.int64), np.zeros(0, np.float32)
    q = q / qn
    sims = (rows @ q.T).ravel()
    k = min(top_k, len(sims))
    idx = np.argsort(sims)[-k:][::-1]
    return idx, sims[idx]
