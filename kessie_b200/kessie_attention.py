"""Drop-in for the reference's ``kessie_attention`` module (KeSSie attention
backend for vLLM V1), with the fog actually applied.

The reference (kessie_attention.py:26-307) computes an additive fog bias
once per step (``_FogCache``) and passes it to vLLM's own attention as
``attn_bias``.  vLLM's FlashAttention implementation takes no such argument,
so the fog never reaches the scores; the reference also sizes the bias from
``key.shape[-2]``, the KV-head count of vLLM's [tokens, heads, dim] keys.
Here ``KeSSieAttentionImpl`` computes the attention itself with the paged
decode / chunked-prefill kernels of this library, the bias applied to the
scaled scores inside the kernels, per request of kv_len = its sequence
length:
    fb = int(kv_len * (1 - fog_start))
    bias(j) = -fog_alpha * (1 - j/fb)^2 for j < fb, 0 after,
    bias(j) = recall_boost at recalled positions
(the values of _FogCache._compute_into, kessie_attention.py:114-139).
Everything else (KV-cache write, metadata, cache layout) stays vLLM's:
the backend subclasses the FlashAttention backend and the impl delegates
to the wrapped FlashAttention impl.

Same names and state API as the reference: ``KeSSieAttentionState``,
``KESSIE_STATE``, ``_FogCache.get_fog_bias`` (the materialised
(1, 1, 1, kv_len) bias, built by a kernel), ``register_kessie_attention``,
``KeSSieAttentionBackend``, ``KeSSieAttentionImpl``.
"""

from __future__ import annotations

import logging
import os
import threading
from typing import Optional, Set

import torch

from . import ops

logger = logging.getLogger("KeSSie.Attention")


class KeSSieAttentionState:
    """Thread-safe global fog parameters (kessie_attention.py:26-60)."""

    def __init__(self):
        self._lock = threading.Lock()
        self.fog_alpha: float = 0.5
        self.fog_start: float = 0.5
        self.prompt_len: int = 0
        self.recall_positions: Set[int] = set()
        self.recall_boost: float = 0.1
        self.enabled: bool = True
        self.generation: int = 0

    def update(self, fog_alpha=None, fog_start=None, prompt_len=None, recall_positions=None, recall_boost=None):
        with self._lock:
            if fog_alpha is not None:
                self.fog_alpha = fog_alpha
            if fog_start is not None:
                self.fog_start = fog_start
            if prompt_len is not None:
                self.prompt_len = prompt_len
            if recall_positions is not None:
                self.recall_positions = set(recall_positions)
            if recall_boost is not None:
                self.recall_boost = recall_boost
            self.generation += 1

    def get(self):
        with self._lock:
            return {"fog_alpha": self.fog_alpha, "fog_start": self.fog_start, "prompt_len": self.prompt_len,
                    "recall_positions": set(self.recall_positions), "recall_boost": self.recall_boost,
                    "enabled": self.enabled, "generation": self.generation}


KESSIE_STATE = KeSSieAttentionState()


class _FogCache:
    """The materialised bias of the reference API (kessie_attention.py:66-185):
    computed once per (generation, kv_len, device, dtype) into one of two
    ping-pong buffers by the library's bias kernel; later calls of the same
    generation return the same view.  The attention path below does not need
    it (the bias is evaluated inside the kernels)."""

    def __init__(self):
        self._gen = -1
        self._kv_len = 0
        self._buf = [None, None]
        self._active = 0
        self._alloc_len = 0
        self._device = None
        self._dtype = None
        self._view = None
        self._compute_lock = threading.Lock()

    def _ensure_alloc(self, kv_len, device, dtype):
        if self._alloc_len >= kv_len and self._device == device and self._dtype == dtype:
            return
        alloc = (max(kv_len, 2048) + 255) & ~255
        self._buf = [torch.zeros(alloc, device=device, dtype=dtype), torch.zeros(alloc, device=device, dtype=dtype)]
        self._alloc_len, self._device, self._dtype = alloc, device, dtype
        self._gen = -1
        self._view = None

    @staticmethod
    def _compute_into(buf, kv_len, fog_alpha, fog_start, recall_pos, recall_boost=0.1):
        """Bias of kv_len keys into buf[:kv_len] (kessie_attention.py:114-139)."""
        bias = ops.FogBias(fog_alpha, fog_start, recall_pos, recall_boost, dtype=buf.dtype, device=buf.device)
        ops.build_fog_bias(kv_len, bias, out=buf[:kv_len])

    def get_fog_bias(self, kv_len, device, dtype, state):
        """(1, 1, 1, kv_len) bias of the state's generation."""
        gen = state["generation"]
        if self._gen == gen and self._kv_len == kv_len and self._view is not None:
            return self._view
        with self._compute_lock:
            if self._gen == gen and self._kv_len == kv_len and self._view is not None:
                return self._view
            self._ensure_alloc(kv_len, device, dtype)
            self._active = 1 - self._active          # a new generation lands in the other buffer
            buf = self._buf[self._active]
            self._compute_into(buf, kv_len, state["fog_alpha"], state["fog_start"],
                               frozenset(state["recall_positions"]), state.get("recall_boost", 0.1))
            self._gen, self._kv_len = gen, kv_len
            self._view = buf[:kv_len].view(1, 1, 1, kv_len)
            return self._view


def _fog_active(state) -> bool:
    """The reference's switch (kessie_attention.py:276-277)."""
    return bool(state["enabled"]) and state["fog_alpha"] > 0 and state["prompt_len"] > 0


class _BiasCache:
    """FogBias (device recall bitmap included) of the current generation."""

    def __init__(self):
        self._lock = threading.Lock()
        self._key = None
        self._bias = None

    def get(self, state, dtype, device) -> "ops.FogBias":
        key = (state["generation"], dtype, device)
        with self._lock:
            if self._key != key:
                self._bias = ops.FogBias(state["fog_alpha"], state["fog_start"], state["recall_positions"],
                                         state.get("recall_boost", 0.1), dtype=dtype, device=device)
                self._key = key
            return self._bias


_BIAS_CACHE = _BiasCache()
_FOG_CACHE = _FogCache()


class KeSSieAttentionImpl:
    """Per-layer attention: with the fog active, decode and chunked prefill run
    in this library's paged kernels with the fog bias applied to the scores;
    otherwise (fog off, profiling run, features the kernels do not cover) the
    wrapped vLLM implementation runs.  Attributes and methods not defined here
    (e.g. the KV-cache write) are the wrapped implementation's."""

    def __init__(self, *args, _inner_impl=None, **kwargs):
        if _inner_impl is None:
            if not HAS_VLLM:
                raise RuntimeError("KeSSieAttentionImpl needs vLLM or an injected implementation")
            _inner_impl = KeSSieAttentionBackend._get_original().get_impl_cls()(*args, **kwargs)
        object.__setattr__(self, "_inner", _inner_impl)
        inner = _inner_impl
        self._num_heads = int(inner.num_heads)
        self._num_kv_heads = int(getattr(inner, "num_kv_heads", inner.num_heads))
        self._head_size = int(inner.head_size)
        self._scale = float(inner.scale)
        sw = getattr(inner, "sliding_window", None)
        if sw is None or (isinstance(sw, (tuple, list)) and sw[0] < 0):
            self._window = 0
        elif isinstance(sw, (tuple, list)):
            self._window = int(sw[0]) + 1                 # vLLM keeps (window - 1, 0)
        else:
            self._window = int(sw)
        self._meta_ref = None
        self._meta_host = None

    def __getattr__(self, name):
        return getattr(object.__getattribute__(self, "_inner"), name)

    # ------------------------------------------------------------------ dispatch
    def _kernels_cover(self, query, kv_cache, output, output_scale) -> bool:
        inner = self._inner
        if output is None or output_scale is not None or kv_cache is None or not query.is_cuda:
            return False
        if query.dtype not in (torch.bfloat16, torch.float16) or kv_cache.dtype != query.dtype:
            return False
        if self._head_size not in (64, 128) or self._num_heads % self._num_kv_heads:
            return False
        if self._num_heads // self._num_kv_heads > 16:
            return False
        if getattr(inner, "alibi_slopes", None) is not None or getattr(inner, "sinks", None) is not None:
            return False
        if getattr(inner, "logits_soft_cap", 0) not in (None, 0, 0.0):
            return False
        return kv_cache.dim() == 5 and kv_cache.shape[0] == 2

    def forward(self, layer, query, key, value, kv_cache, attn_metadata, output=None, output_scale=None,
                output_block_scale=None):
        state = KESSIE_STATE.get()
        if attn_metadata is None or not _fog_active(state) or \
                not self._kernels_cover(query, kv_cache, output, output_scale):
            return self._inner.forward(layer, query, key, value, kv_cache, attn_metadata, output, output_scale,
                                       output_block_scale)
        return self._fog_forward(query, kv_cache, attn_metadata, output, state)

    def _host_meta(self, md):
        """Query offsets and sequence lengths on the host, once per step (the
        same metadata object serves every layer of a step)."""
        if self._meta_ref is not md:
            qsl = md.query_start_loc.detach().cpu().tolist()
            sl = md.seq_lens.detach().cpu().tolist()
            self._meta_ref, self._meta_host = md, (qsl, sl)
        return self._meta_host

    def _fog_forward(self, query, kv_cache, md, output, state):
        n = int(md.num_actual_tokens)
        Hq, D = self._num_heads, self._head_size
        q = query[:n].view(n, Hq, D)
        out = output[:n].view(n, Hq, D)
        key_cache, value_cache = kv_cache.unbind(0)      # [num_blocks, block_size, Hkv, D] each
        bias = _BIAS_CACHE.get(state, query.dtype, query.device)
        bt, sl = md.block_table, md.seq_lens
        kw = dict(window_size=self._window, sm_scale=self._scale, fog_alpha=0.0, bias=bias)
        if int(md.max_query_len) == 1:                 # decode step: one launch for the batch
            ops.paged_fog_decode(q, key_cache, value_cache, bt[:n], sl[:n], out=out, **kw)
            return output
        qsl, slh = self._host_meta(md)
        B = len(slh)
        b = 0
        while b < B:
            ql = qsl[b + 1] - qsl[b]
            if ql <= 0:
                b += 1
                continue
            r0 = qsl[b]
            if ql == 1:                                  # a run of decode requests: one launch
                e = b
                while e < B and qsl[e + 1] - qsl[e] == 1:
                    e += 1
                ops.paged_fog_decode(q[r0:r0 + e - b], key_cache, value_cache, bt[b:e], sl[b:e],
                                     out=out[r0:r0 + e - b], **kw)
                b = e
                continue
            ops.paged_fog_prefill(q[r0:r0 + ql].unsqueeze(0), key_cache, value_cache, bt[b:b + 1], sl[b:b + 1],
                                  causal=True, out=out[r0:r0 + ql].unsqueeze(0), max_kv_len=int(slh[b]), **kw)
            b += 1
        return output


# ----------------------------------------------------------------- vLLM registration
try:
    from vllm.v1.attention.backends.flash_attn import FlashAttentionBackend as _FlashAttentionBackend
    HAS_VLLM = True
except Exception:                                      # pragma: no cover - depends on the vLLM build
    _FlashAttentionBackend = None
    HAS_VLLM = False

if HAS_VLLM:
    class KeSSieAttentionBackend(_FlashAttentionBackend):
        """FlashAttention backend whose implementation applies the fog
        (kessie_attention.py:228-260); metadata, builder and cache layout are
        FlashAttention's."""

        @classmethod
        def _get_original(cls):
            return _FlashAttentionBackend

        @staticmethod
        def get_name() -> str:
            return "KeSSie"

        @staticmethod
        def get_impl_cls():
            return KeSSieAttentionImpl
else:
    class KeSSieAttentionBackend:                      # pragma: no cover
        pass


def register_kessie_attention() -> bool:
    """Register the KeSSie backend in place of FLASH_ATTN; call before the
    engine is created (kessie_attention.py:188-212)."""
    if not HAS_VLLM:
        logger.warning("vLLM V1 attention registry not available")
        return False
    try:
        from vllm.v1.attention.backends.registry import AttentionBackendEnum, register_backend
    except ImportError:
        logger.warning("vLLM V1 attention registry not available")
        return False
    target = AttentionBackendEnum.FLASH_ATTN
    os.environ["_KESSIE_ORIGINAL_ATTN_PATH"] = target.value
    register_backend(target, "kessie_b200.kessie_attention.KeSSieAttentionBackend")
    logger.info("KeSSie attention registered (wrapping %s)", target.value)
    return True
