"""Drop-in for the HF tiered KV cache ``KeSSieCache`` (kessie_exp3.py:342-627):
the same constructor, attributes (``key_cache``, ``value_cache``,
``cpu_kv_store``, ``window_start``, counters, conversation bookkeeping) and
methods, with the device work on stores that never move on append.

Per layer, K and V each live in one store ``[B, H, cap, D]`` with the live
tokens at ``[lo, hi)``; ``key_cache[l]`` / ``value_cache[l]`` are views of that
range.  So:

* ``update`` (kessie_exp3.py:425-450) is ONE launch
  (``kessie_tiered_update_v2``): the new tokens are written in place at ``hi``
  and, with the fog on, the fogged V of the whole live range is written to a
  per-layer buffer -- one read and one write of V per step, where the
  reference's ``torch.cat`` re-copies K and V and its fog goes through fp32
  temporaries.  The returned V is that buffer (contiguous); it is rewritten by
  the next ``update`` of the same layer.
* ``evict_if_needed`` (:452-486) packs the evicted range of every layer with
  ONE ``kessie_strided_pack_v2`` launch, moves it with ONE device-to-host copy
  into pinned host memory (the CPU chunk's per-layer tensors are views of it) and
  trims by moving ``lo`` -- no ``.contiguous()`` re-copy of the window.
* ``recall_from_cpu`` (:488-533) brings a chunk back with ONE host-to-device
  copy (for chunks this class evicted) and ONE unpack launch into the room in
  front of ``lo``; only when that room is missing is a store re-laid out.

Returned values match the reference: the fog weights are computed in fp32
exactly as ``_compute_fog_mask`` (:415-423) does (true division, sqrt for
alpha 0.5), and ``(float(v) * w).to(dtype)`` rounds once.  The byte
accounting keeps the reference's (``cpu_kv_bytes`` drops by half the recalled
bytes, :530).  Store dtypes: float32, bfloat16, float16; head_dim * element
size a multiple of 16 bytes.
"""

from __future__ import annotations

import logging
from typing import Any, Dict, List, Optional, Tuple

import numpy as np
import torch

from . import ops

logger = logging.getLogger(__name__)

_ALIGN_TOKENS = 64


def _round_up(x: int, a: int) -> int:
    return (x + a - 1) // a * a


class _Store:
    """One layer's K and V stores and its fog buffer."""

    __slots__ = ("k", "v", "cap", "lo", "hi", "vfog")

    def __init__(self, B: int, H: int, D: int, cap: int, dtype, device, lo: int = 0):
        self.k = torch.empty(B, H, cap, D, dtype=dtype, device=device)
        self.v = torch.empty(B, H, cap, D, dtype=dtype, device=device)
        self.cap, self.lo, self.hi = cap, lo, lo
        self.vfog: Optional[torch.Tensor] = None

    @property
    def length(self) -> int:
        return self.hi - self.lo

    def kview(self) -> torch.Tensor:
        return self.k[:, :, self.lo:self.hi]

    def vview(self) -> torch.Tensor:
        return self.v[:, :, self.lo:self.hi]

    def relayout(self, front: int, back: int):
        """New stores with `front` free tokens before the live range and at
        least `back` after it (a rare path: capacity growth, or a recall with
        no room in front)."""
        B, H, _, D = self.k.shape
        live = self.length
        cap = _round_up(front + live + max(back, live // 2, _ALIGN_TOKENS), _ALIGN_TOKENS)
        k = torch.empty(B, H, cap, D, dtype=self.k.dtype, device=self.k.device)
        v = torch.empty_like(k)
        if live:
            k[:, :, front:front + live].copy_(self.kview())
            v[:, :, front:front + live].copy_(self.vview())
        self.k, self.v, self.cap, self.lo, self.hi = k, v, cap, front, front + live


class KeSSieCache:
    """Tiered KV cache: the hot window in HBM, fogged/evicted KV in host
    memory, recalled on a hit (kessie_exp3.py:342-351)."""

    def __init__(self, window_size=4096, index_granularity=128, fog_alpha=0.5, fog_start=0.5,
                 kv_cache_dtype=None, max_conversation_tokens=10_000_000):
        self.window_size = window_size
        self.fog_alpha = fog_alpha
        self.fog_start = fog_start
        self.index_granularity = index_granularity
        self.kv_cache_dtype = kv_cache_dtype
        self.max_conversation_tokens = max_conversation_tokens
        self.conversation_tokens: List[int] = []
        self.index_embeddings: List[np.ndarray] = []
        self.index_positions: List[int] = []
        self.key_cache: List[torch.Tensor] = []
        self.value_cache: List[torch.Tensor] = []
        self.cpu_kv_store: List[Tuple[int, int, List[Tuple[Any, Any]]]] = []
        self.cpu_kv_bytes = 0
        self.window_start = 0
        self.seen_tokens = 0
        self._seen_tokens = 0
        self.total_evictions = 0
        self.total_recalls = 0
        self._proj_matrix = None
        self.has_previous_state = False
        self.ssm_states = {}
        self.conv_states = {}
        self.turn_boundaries: List[Tuple[int, str, int]] = []
        self._turn_counter = 0
        self._stores: List[Optional[_Store]] = []
        self._packed: Dict[int, Tuple[torch.Tensor, List[int], Tuple]] = {}   # id(chunk layers) -> host buffer

    # ----------------------------------------------------------- cache protocol
    def _cast_kv(self, t):
        if self.kv_cache_dtype is not None and t.dtype != self.kv_cache_dtype:
            return t.to(self.kv_cache_dtype)
        return t

    def __len__(self):
        return len(self.key_cache)

    def __getitem__(self, i):
        return (self.key_cache[i], self.value_cache[i])

    def get_seq_length(self, li=0):
        if li < len(self.key_cache) and self._valid(self.key_cache[li]):
            return self.key_cache[li].shape[-2]
        return 0

    def get_max_length(self):
        return self.window_size * 2

    def get_usable_length(self, n, li=0):
        return max(0, self.get_seq_length(li))

    def get_mask_sizes(self, cp, li):
        return self.get_seq_length(li) + cp.shape[0], 0

    @staticmethod
    def _valid(t):
        return t is not None and isinstance(t, torch.Tensor) and t.numel() > 0

    def _sync_views(self, li: int):
        st = self._stores[li]
        self.key_cache[li] = st.kview()
        self.value_cache[li] = st.vview()

    def _compute_fog_mask(self, seq_len, device, dtype):
        """The reference's fog mask as a [1, 1, S, 1] tensor (kessie_exp3.py:415-423);
        update() evaluates the same weights inside its kernel."""
        if self.fog_alpha <= 0 or seq_len == 0:
            return None
        cc = max(1, int(seq_len * self.fog_start))
        fc = seq_len - cc
        if fc <= 0:
            return None
        pos = torch.arange(fc, dtype=dtype, device=device)
        fw = (pos / max(fc - 1, 1)).pow(self.fog_alpha).clamp(min=0.01)
        return torch.cat([fw, torch.ones(cc, dtype=dtype, device=device)]).view(1, 1, seq_len, 1)

    # ----------------------------------------------------------- update
    def update(self, key_states, value_states, layer_idx, cache_kwargs=None):
        """Append this step's K/V of one layer; return (K, fogged V) of the
        whole window (kessie_exp3.py:425-450)."""
        key_states = self._cast_kv(key_states)
        value_states = self._cast_kv(value_states)
        if not key_states.is_cuda:
            raise RuntimeError("KeSSieCache: key/value states must be CUDA tensors (the cache lives in HBM)")
        while len(self.key_cache) <= layer_idx:
            self.key_cache.append(torch.tensor([], device=key_states.device))
            self.value_cache.append(torch.tensor([], device=key_states.device))
            self._stores.append(None)
        B, H, T, D = key_states.shape
        st = self._stores[layer_idx]
        if st is None or not self._valid(self.key_cache[layer_idx]) or st.k.shape[0] != B or st.k.shape[1] != H \
                or st.k.shape[3] != D or st.k.dtype != key_states.dtype:
            cap = _round_up(max(2 * self.window_size + 1, T) + _ALIGN_TOKENS, _ALIGN_TOKENS)
            st = _Store(B, H, D, cap, key_states.dtype, key_states.device)
            self._stores[layer_idx] = st
        if st.hi + T > st.cap:
            st.relayout(0, T)
        S = st.length + T
        need = B * H * S * D
        if st.vfog is None or st.vfog.numel() < need:
            st.vfog = torch.empty(_round_up(need + need // 4, 4096), dtype=st.v.dtype, device=st.v.device)
        fog_on = ops.tiered_update(st.k, st.v, st.lo, st.hi, key_states, value_states, st.vfog, self.fog_alpha,
                                   self.fog_start)
        st.hi += T
        self._sync_views(layer_idx)
        if layer_idx == 0:
            self.seen_tokens = self.window_start + self.key_cache[0].shape[-2]
            self._seen_tokens = self.seen_tokens
        v = st.vfog[:need].view(B, H, S, D) if fog_on else self.value_cache[layer_idx]
        return self.key_cache[layer_idx], v

    # ----------------------------------------------------------- evict / recall
    def _layer_groups(self, layers: List[int]) -> List[List[int]]:
        """Layers with one (B, H, D, dtype, device), packed together."""
        groups: Dict[Tuple, List[int]] = {}
        for li in layers:
            st = self._stores[li]
            B, H, _, D = st.k.shape
            groups.setdefault((B, H, D, st.k.dtype, st.k.device), []).append(li)
        return list(groups.values())

    @staticmethod
    def _bases(stores: List[_Store], token: List[int], device) -> Tuple[torch.Tensor, torch.Tensor]:
        """int64 device arrays: address of each (layer, K/V) store at its token,
        and the bytes between its [b, h] rows."""
        addr, pitch = [], []
        for st, t in zip(stores, token):
            row = st.k.shape[3] * st.k.element_size()
            for buf in (st.k, st.v):
                addr.append(buf.data_ptr() + t * row)
                pitch.append(st.cap * row)
        return (torch.tensor(addr, dtype=torch.int64).to(device, non_blocking=True),
                torch.tensor(pitch, dtype=torch.int64).to(device, non_blocking=True))

    def evict_if_needed(self):
        """Above twice the window, move all but the last window tokens of every
        layer to host memory (kessie_exp3.py:452-486)."""
        if not self.key_cache or not self._valid(self.key_cache[0]):
            return
        cl = self.key_cache[0].shape[-2]
        if cl <= self.window_size * 2:
            return
        ev = cl - self.window_size
        if ev <= 0:
            return
        layers = [i for i in range(len(self.key_cache)) if self._valid(self.key_cache[i])]
        cpu_layers: List[Tuple[Any, Any]] = [(None, None)] * len(self.key_cache)
        chunk_bytes = 0
        stream = torch.cuda.current_stream(self._stores[layers[0]].k.device)
        packed = []
        for grp in self._layer_groups(layers):
            st0 = self._stores[grp[0]]
            B, H, _, D = st0.k.shape
            dev = st0.k.device
            nel = len(grp) * 2 * B * H * ev * D
            staging = torch.empty(nel, dtype=st0.k.dtype, device=dev)
            # pinned, from torch's caching host allocator: a recalled chunk's block
            # returns there and the next eviction of that size reuses it
            host = torch.empty(nel, dtype=st0.k.dtype, pin_memory=True)
            bases, pitch = self._bases([self._stores[i] for i in grp], [self._stores[i].lo for i in grp], dev)
            ops.strided_pack(bases, pitch, B * H, ev, D * st0.k.element_size(), staging, unpack=False)
            host.copy_(staging, non_blocking=True)
            view = host.view(len(grp), 2, B, H, ev, D)
            for j, li in enumerate(grp):
                cpu_layers[li] = (view[j, 0], view[j, 1])
                chunk_bytes += 2 * view[j, 0].numel() * view[j, 0].element_size()
            packed.append((host, grp, (B, H, D)))
        stream.synchronize()                 # host chunk complete; staging free
        for li in layers:
            self._stores[li].lo += ev
            self._sync_views(li)
        start_pos, end_pos = self.window_start, self.window_start + ev
        self.cpu_kv_store.append((start_pos, end_pos, cpu_layers))
        self._packed[id(cpu_layers)] = packed
        self.cpu_kv_bytes += chunk_bytes
        self.window_start += ev
        self.total_evictions += ev
        self.seen_tokens = self.window_start + self.key_cache[0].shape[-2]
        self._seen_tokens = self.seen_tokens
        logger.info("tiered cache: evicted positions %d-%d to host memory (%.1f MB; %d chunks, %.1f MB held)",
                    start_pos, end_pos, chunk_bytes / 1048576, len(self.cpu_kv_store), self.cpu_kv_bytes / 1048576)

    def recall_from_cpu(self, position: int, device) -> bool:
        """Bring the stored chunk holding `position` back in front of the
        window of every layer (kessie_exp3.py:488-533)."""
        hit = None
        for idx, (start, end, _layers) in enumerate(self.cpu_kv_store):
            if start <= position < end:
                hit = idx
                break
        if hit is None:
            return False
        start, end, cpu_layers = self.cpu_kv_store[hit]
        recalled_bytes = 0
        todo = [i for i in range(len(self.key_cache)) if i < len(cpu_layers) and cpu_layers[i][0] is not None]
        packed = self._packed.pop(id(cpu_layers), None)
        fast = {}                  # layer -> (pinned host buffer, its layers): one copy for the group
        if packed is not None:
            for host, grp, shp in packed:
                view = host.view(len(grp), 2, *shp[:2], -1, shp[2])
                if all(li in todo and cpu_layers[li][0].data_ptr() == view[j, 0].data_ptr()
                       and cpu_layers[li][1].data_ptr() == view[j, 1].data_ptr() for j, li in enumerate(grp)):
                    for li in grp:
                        fast[li] = (host, grp)
        for li in todo:
            kr, vr = cpu_layers[li]
            recalled_bytes += kr.numel() * kr.element_size() * 2
        # stores with room in front of the window for every recalled layer
        for li in todo:
            kr = cpu_layers[li][0]
            n = kr.shape[-2]
            st = self._stores[li]
            if st is None or not self._valid(self.key_cache[li]):
                B, H, _, D = kr.shape
                dev = self._stores[li].k.device if st is not None else torch.device(device)
                cap = _round_up(max(2 * self.window_size + 1, n) + _ALIGN_TOKENS, _ALIGN_TOKENS)
                st = _Store(B, H, D, cap, kr.dtype, dev, lo=n)
                self._stores[li] = st
            elif st.lo < n:
                st.relayout(n, _ALIGN_TOKENS)
        done = set()
        for li in todo:
            if li in done:
                continue
            if li in fast:
                src, grp = fast[li]
            else:
                grp = [li]
                kr, vr = cpu_layers[li]
                src = torch.empty(kr.numel() + vr.numel(), dtype=kr.dtype)
                src[:kr.numel()].copy_(kr.reshape(-1))
                src[kr.numel():].copy_(vr.reshape(-1))
            st0 = self._stores[grp[0]]
            B, H, _, D = st0.k.shape
            n = cpu_layers[grp[0]][0].shape[-2]
            staging = src.to(st0.k.device, non_blocking=True)
            stores = [self._stores[g] for g in grp]
            bases, pitch = self._bases(stores, [s.lo - n for s in stores], st0.k.device)
            ops.strided_pack(bases, pitch, B * H, n, D * st0.k.element_size(), staging, unpack=True)
            for g in grp:
                self._stores[g].lo -= n
                self._sync_views(g)
                done.add(g)
        self.window_start = start
        self.seen_tokens = self.window_start + self.key_cache[0].shape[-2]
        self._seen_tokens = self.seen_tokens
        self.total_recalls += 1
        del self.cpu_kv_store[hit]
        self.cpu_kv_bytes -= recalled_bytes // 2
        logger.info("tiered cache: recalled positions %d-%d (%.1f MB), window now %d tokens", start, end,
                    recalled_bytes / 1048576, self.get_seq_length())
        return True

    # ----------------------------------------------------------- resets
    def reset(self):
        self.key_cache.clear()
        self.value_cache.clear()
        self._stores.clear()
        self.cpu_kv_store.clear()
        self._packed.clear()
        self.cpu_kv_bytes = 0
        self.window_start = 0
        self.seen_tokens = 0
        self._seen_tokens = 0
        self.has_previous_state = False
        self.ssm_states.clear()
        self.conv_states.clear()

    def full_reset(self):
        """Clear everything including the conversation store and index."""
        self.reset()
        self.conversation_tokens.clear()
        self.index_embeddings.clear()
        self.index_positions.clear()
        self.turn_boundaries.clear()
        self._turn_counter = 0
        self.total_evictions = 0
        self.total_recalls = 0

    # ----------------------------------------------------------- conversation bookkeeping (host)
    def append_conversation(self, tids, role="assistant"):
        """Append token ids and a turn boundary, dropping the oldest tokens
        (and the index entries / boundaries they carry) beyond
        max_conversation_tokens (kessie_exp3.py:535-559)."""
        overflow = (len(self.conversation_tokens) + len(tids)) - self.max_conversation_tokens
        if overflow > 0:
            self.conversation_tokens = self.conversation_tokens[overflow:]
            kept = [(e, p - overflow) for e, p in zip(self.index_embeddings, self.index_positions) if p - overflow >= 0]
            self.index_embeddings = [e for e, _ in kept]
            self.index_positions = [p for _, p in kept]
            self.turn_boundaries = [(s - overflow, r, n) for s, r, n in self.turn_boundaries if s - overflow >= 0]
        pos = len(self.conversation_tokens)
        self.conversation_tokens.extend(tids)
        self._turn_counter += 1
        self.turn_boundaries.append((pos, role, self._turn_counter))

    def get_turn_for_position(self, token_pos: int):
        """(role, turn number, total turns) of the last turn starting at or
        before token_pos, ("unknown", 0, total) before the first."""
        role, turn = "unknown", 0
        for start_pos, r, n in self.turn_boundaries:
            if start_pos > token_pos:
                break
            role, turn = r, n
        return role, turn, self._turn_counter

    def get_token_distance(self, token_pos: int) -> int:
        return len(self.conversation_tokens) - token_pos

    def _get_projection(self, ed, target=256):
        """Seeded Gaussian projection ed -> target (numpy seed 42, scaled by
        1/sqrt(ed)), as kessie_exp3.py:565-569 builds it."""
        if self._proj_matrix is None or self._proj_matrix.shape[0] != ed:
            np.random.seed(42)
            self._proj_matrix = np.random.randn(ed, target).astype(np.float32) / np.sqrt(ed)
        return self._proj_matrix

    def get_stats(self):
        kv_gpu_bytes, kv_dtype = 0, None
        kv_seq = self.get_seq_length()
        for k, v in zip(self.key_cache, self.value_cache):
            if self._valid(k):
                kv_gpu_bytes += k.numel() * k.element_size() + v.numel() * v.element_size()
                if kv_dtype is None:
                    kv_dtype = str(k.dtype)
        fog_tokens = int(kv_seq * (1.0 - self.fog_start)) if kv_seq > 0 else 0
        return {
            "conversation_tokens": len(self.conversation_tokens),
            "semantic_index_count": len(self.index_embeddings),
            "kv_seq_len": kv_seq,
            "kv_window_start": self.window_start,
            "kv_layers": len(self.key_cache),
            "kv_gpu_bytes": kv_gpu_bytes,
            "kv_gpu_mb": round(kv_gpu_bytes / 1048576, 2),
            "kv_cpu_mb": round(self.cpu_kv_bytes / 1048576, 2),
            "kv_cpu_chunks": len(self.cpu_kv_store),
            "kv_cpu_tokens": sum(e - s for s, e, _ in self.cpu_kv_store),
            "kv_dtype": kv_dtype,
            "fog_tokens": fog_tokens,
            "clear_tokens": kv_seq - fog_tokens,
            "window_capacity": self.window_size,
            "window_fill_pct": round(kv_seq / max(self.window_size, 1) * 100, 1),
            "total_evictions": self.total_evictions,
            "total_recalls": self.total_recalls,
        }
