"""numpy restatement of the HF tiered KV cache (KeSSieCache,
kessie_exp3.py:342-627) for parity tests.

TEST INFRASTRUCTURE ONLY -- imported by tests/ (and the golden-vector
script), never by the product package.

Per layer the model keeps K and V as float32 arrays [B, H, S, D] holding
dtype-representable values; evicted chunks are kept as copies.  update()
returns (K, fogged V) rounded to the dtype as the reference's
(v.float() * fog).to(k.dtype) does.  Paths are relative to the
sentinelXVI/KeSSie source tree.
"""

from __future__ import annotations

from typing import List, Optional, Tuple

import numpy as np

from .fog_oracle import _ROUND

__all__ = ["tiered_fog_weights", "TieredCacheModel"]


def tiered_fog_weights(seq_len: int, fog_alpha: float, fog_start: float) -> Optional[np.ndarray]:
    """KeSSieCache._compute_fog_mask (kessie_exp3.py:415-423) as float32 [S],
    or None where the reference returns None.  (pos / max(fc - 1, 1)) is a
    float32 division; pow with the exponents torch evaluates without pow()
    (0.5 -> sqrt, 1, 2, 3) follows the same route."""
    if fog_alpha <= 0 or seq_len == 0:
        return None
    cc = max(1, int(seq_len * fog_start))
    fc = seq_len - cc
    if fc <= 0:
        return None
    x = np.arange(fc, dtype=np.float32) / np.float32(max(fc - 1, 1))
    if fog_alpha == 0.5:
        fw = np.sqrt(x)
    elif fog_alpha == 1.0:
        fw = x
    elif fog_alpha == 2.0:
        fw = x * x
    elif fog_alpha == 3.0:
        fw = x * x * x
    else:
        fw = np.power(x, np.float32(fog_alpha))
    fw = np.maximum(fw, np.float32(0.01)).astype(np.float32)
    return np.concatenate([fw, np.ones(cc, np.float32)])


class TieredCacheModel:
    """The reference's window / eviction / recall bookkeeping
    (kessie_exp3.py:353-533) over numpy arrays; dtype is "float32",
    "bfloat16" or "float16"."""

    def __init__(self, window_size: int = 4096, fog_alpha: float = 0.5, fog_start: float = 0.5,
                 dtype: str = "bfloat16"):
        self.window_size = window_size
        self.fog_alpha, self.fog_start = fog_alpha, fog_start
        self.round = _ROUND[dtype]
        self.key_cache: List[Optional[np.ndarray]] = []
        self.value_cache: List[Optional[np.ndarray]] = []
        self.cpu_kv_store: List[Tuple[int, int, List[Tuple[np.ndarray, np.ndarray]]]] = []
        self.cpu_kv_bytes = 0
        self.window_start = 0
        self.seen_tokens = 0
        self.total_evictions = 0
        self.total_recalls = 0
        self.elem_bytes = 4 if dtype == "float32" else 2

    def get_seq_length(self, li: int = 0) -> int:
        if li < len(self.key_cache) and self.key_cache[li] is not None and self.key_cache[li].size:
            return self.key_cache[li].shape[-2]
        return 0

    def update(self, k: np.ndarray, v: np.ndarray, layer_idx: int):
        """:425-450 -- append on the sequence axis, fog the whole V."""
        while len(self.key_cache) <= layer_idx:
            self.key_cache.append(None)
            self.value_cache.append(None)
        if self.key_cache[layer_idx] is None:
            self.key_cache[layer_idx] = np.array(k, np.float32)
            self.value_cache[layer_idx] = np.array(v, np.float32)
        else:
            self.key_cache[layer_idx] = np.concatenate([self.key_cache[layer_idx], k], axis=-2)
            self.value_cache[layer_idx] = np.concatenate([self.value_cache[layer_idx], v], axis=-2)
        if layer_idx == 0:
            self.seen_tokens = self.window_start + self.key_cache[0].shape[-2]
        kk, vv = self.key_cache[layer_idx], self.value_cache[layer_idx]
        w = tiered_fog_weights(vv.shape[-2], self.fog_alpha, self.fog_start)
        if w is not None:
            vv = self.round(vv * w.reshape(1, 1, -1, 1))
        return kk, vv

    def evict_if_needed(self):
        """:452-486 -- above twice the window, move all but the last window
        tokens of every layer to the CPU store."""
        if not self.key_cache or self.key_cache[0] is None:
            return
        cl = self.key_cache[0].shape[-2]
        if cl <= self.window_size * 2:
            return
        ev = cl - self.window_size
        layers, nbytes = [], 0
        for i in range(len(self.key_cache)):
            if self.key_cache[i] is not None:
                ke = self.key_cache[i][:, :, :ev, :].copy()
                ve = self.value_cache[i][:, :, :ev, :].copy()
                nbytes += (ke.size + ve.size) * self.elem_bytes
                layers.append((ke, ve))
                self.key_cache[i] = self.key_cache[i][:, :, ev:, :]
                self.value_cache[i] = self.value_cache[i][:, :, ev:, :]
            else:
                layers.append((None, None))
        self.cpu_kv_store.append((self.window_start, self.window_start + ev, layers))
        self.cpu_kv_bytes += nbytes
        self.window_start += ev
        self.total_evictions += ev
        self.seen_tokens = self.window_start + self.key_cache[0].shape[-2]

    def recall_from_cpu(self, position: int) -> bool:
        """:488-533 -- the first stored chunk holding `position` goes back in
        front of every layer; window_start becomes the chunk's start; the byte
        count drops by half the recalled bytes, as the reference's does."""
        hit = None
        for idx, (start, end, layers) in enumerate(self.cpu_kv_store):
            if start <= position < end:
                hit = idx
                break
        if hit is None:
            return False
        start, end, layers = self.cpu_kv_store[hit]
        recalled = 0
        for i in range(len(self.key_cache)):
            if i < len(layers) and layers[i][0] is not None:
                kr, vr = layers[i]
                recalled += kr.size * self.elem_bytes * 2
                if self.key_cache[i] is not None and self.key_cache[i].size:
                    self.key_cache[i] = np.concatenate([kr, self.key_cache[i]], axis=-2)
                    self.value_cache[i] = np.concatenate([vr, self.value_cache[i]], axis=-2)
                else:
                    self.key_cache[i], self.value_cache[i] = kr, vr
        self.window_start = start
        self.seen_tokens = self.window_start + self.key_cache[0].shape[-2]
        self.total_recalls += 1
        del self.cpu_kv_store[hit]
        self.cpu_kv_bytes -= recalled // 2
        return True

    def stats(self) -> dict:
        """The bookkeeping keys of get_stats (kessie_exp3.py:570-608)."""
        kv_seq = self.get_seq_length()
        gpu = sum((k.size + v.size) * self.elem_bytes for k, v in zip(self.key_cache, self.value_cache)
                  if k is not None)
        fog_tokens = int(kv_seq * (1.0 - self.fog_start)) if kv_seq > 0 else 0
        return {"kv_seq_len": kv_seq, "kv_window_start": self.window_start, "kv_layers": len(self.key_cache),
                "kv_gpu_bytes": gpu, "kv_cpu_chunks": len(self.cpu_kv_store),
                "kv_cpu_tokens": sum(e - s for s, e, _ in self.cpu_kv_store), "cpu_kv_bytes": self.cpu_kv_bytes,
                "fog_tokens": fog_tokens, "clear_tokens": kv_seq - fog_tokens,
                "total_evictions": self.total_evictions, "total_recalls": self.total_recalls,
                "seen_tokens": self.seen_tokens}
