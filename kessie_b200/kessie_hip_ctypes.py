"""Drop-in replacement for the reference module ``kessie_hip_ctypes``.

``KeSSieKernels`` loads the B200 library through ctypes exactly as the
reference does (kessie_hip_ctypes.py:39-346): same search list
(``build/libkessie_hip.so`` next to this file first), same method names,
arguments, stream handling (``stream=None`` -> launch on the legacy default
stream and synchronise) and asserts.  fp16 tensors go through the five legacy
launchers with the reference's argument lists; bf16 tensors go through the
``_v2`` entry points.  A failed launch raises ``KessieError`` with the
library's message (the reference's void launchers fail silently).
"""

from __future__ import annotations

import ctypes
import math
import os
from typing import Optional

import torch

from . import _lib, ops


class KeSSieKernels:
    """Python interface to the KeSSie B200 kernels via ctypes."""

    def __init__(self, lib_path: str = None):
        if lib_path is None:
            candidates = [
                os.path.join(os.path.dirname(__file__), "build", "libkessie_hip.so"),
                os.path.join(os.path.dirname(__file__), "libkessie_hip.so"),
                "/usr/local/lib/libkessie_hip.so",
            ]
            for p in candidates:
                if os.path.exists(p):
                    lib_path = p
                    break
        if lib_path is None or not os.path.exists(lib_path):
            raise FileNotFoundError(
                "libkessie_hip.so not found. Build with: python -m kessie_b200.build\n"
                f"Searched: {candidates if lib_path is None else [lib_path]}")
        os.environ.setdefault("KESSIE_LIB", lib_path)
        self.lib = ctypes.CDLL(lib_path)
        self._setup_signatures()
        self._streams = {}
        print(f"KeSSie B200 kernels loaded from {lib_path}")

    def _setup_signatures(self):
        for name, (res, args) in _lib.SIGNATURES.items():
            if hasattr(self.lib, name):
                fn = getattr(self.lib, name)
                fn.restype = res
                fn.argtypes = args

    def _check(self, what):
        buf = ctypes.create_string_buffer(512)
        st = self.lib.kessie_get_last_error(buf, 512)
        if st != 0:
            raise _lib.KessieError(st, f"{what}: {buf.value.decode(errors='replace')}")

    # ------------------------------------------------------------- streams
    def create_stream(self, name: str = "probe") -> torch.cuda.Stream:
        s = torch.cuda.Stream()
        self._streams[name] = s
        return s

    def sync_stream(self, name: str = "probe"):
        if name in self._streams:
            self._streams[name].synchronize()

    def _get_stream_ptr(self, stream=None) -> ctypes.c_void_p:
        if stream is None:
            return ctypes.c_void_p(0)
        if isinstance(stream, str):
            stream = self._streams.get(stream)
        if isinstance(stream, torch.cuda.Stream):
            return ctypes.c_void_p(stream.cuda_stream)
        return ctypes.c_void_p(0)

    @staticmethod
    def _ptr(tensor: torch.Tensor) -> ctypes.c_void_p:
        assert tensor.is_cuda, f"Tensor must be on GPU, got {tensor.device}"
        assert tensor.is_contiguous(), "Tensor must be contiguous"
        return ctypes.c_void_p(tensor.data_ptr())

    # ------------------------------------------------------------- attention
    def windowed_attention(self, Q, K, V, window_size: int = 0, causal: bool = True,
                           sm_scale: Optional[float] = None, stream=None) -> torch.Tensor:
        """Q, K, V: [B, H, N, D] fp16 (or bf16) on GPU (kessie_hip_ctypes.py:163-198)."""
        assert Q.dtype in (torch.float16, torch.bfloat16)
        assert Q.shape == K.shape == V.shape
        B, H, N, D = Q.shape
        assert D in (64, 128)
        if sm_scale is None:
            sm_scale = 1.0 / math.sqrt(D)
        O = torch.empty_like(Q)
        Q, K, V = Q.contiguous(), K.contiguous(), V.contiguous()
        if Q.dtype == torch.float16:
            self.lib.launch_kessie_windowed_attn(self._ptr(Q), self._ptr(K), self._ptr(V), self._ptr(O),
                                                 ctypes.c_float(sm_scale), B, H, N, D, window_size,
                                                 1 if causal else 0, self._get_stream_ptr(stream))
            self._check("windowed_attention")
        else:
            ops.fog_attention(Q, K, V, None, window_size, causal, sm_scale, out=O,
                              stream=self._get_stream_ptr(stream).value or 0)
        if stream is None:
            torch.cuda.synchronize()
        return O

    def fused_fog_attention(self, Q, K, V, fog_weights, window_size: int = 0, causal: bool = True,
                            sm_scale: Optional[float] = None, stream=None) -> torch.Tensor:
        """Fog on V fused into attention (kessie_hip_ctypes.py:200-242)."""
        assert Q.dtype in (torch.float16, torch.bfloat16)
        assert fog_weights.dtype == torch.float32
        assert Q.shape == K.shape == V.shape
        B, H, N, D = Q.shape
        assert fog_weights.shape[0] == N
        if sm_scale is None:
            sm_scale = 1.0 / math.sqrt(D)
        O = torch.empty_like(Q)
        Q, K, V = Q.contiguous(), K.contiguous(), V.contiguous()
        fog_weights = fog_weights.contiguous()
        if Q.dtype == torch.float16:
            self.lib.launch_kessie_fused_fog_attn(self._ptr(Q), self._ptr(K), self._ptr(V), self._ptr(O),
                                                  self._ptr(fog_weights), ctypes.c_float(sm_scale), B, H, N, D,
                                                  window_size, 1 if causal else 0, self._get_stream_ptr(stream))
            self._check("fused_fog_attention")
        else:
            ops.fog_attention(Q, K, V, fog_weights, window_size, causal, sm_scale, out=O,
                              stream=self._get_stream_ptr(stream).value or 0)
        if stream is None:
            torch.cuda.synchronize()
        return O

    # ------------------------------------------------------------- RoPE
    def rope_remap(self, k_data, orig_positions, target_positions, rope_theta: float = 10000.0, stream=None):
        """In-place re-rotation of K [T, H, D] (kessie_hip_ctypes.py:248-286)."""
        assert k_data.is_cuda and k_data.is_contiguous()
        num_tokens, num_heads, head_dim = k_data.shape
        assert head_dim % 2 == 0
        half_dim = head_dim // 2
        orig_positions = orig_positions.contiguous().to(torch.int32)
        target_positions = target_positions.contiguous().to(torch.int32)
        if k_data.dtype == torch.float16:
            self.lib.launch_kessie_rope_remap(self._ptr(k_data), self._ptr(orig_positions),
                                              self._ptr(target_positions), ctypes.c_float(rope_theta), num_tokens,
                                              num_heads, half_dim, self._get_stream_ptr(stream))
            self._check("rope_remap")
        else:
            ops.rope_remap(k_data, orig_positions, target_positions, rope_theta,
                           stream=self._get_stream_ptr(stream).value or 0)
        if stream is None:
            torch.cuda.synchronize()

    # ------------------------------------------------------------- pages
    def page_evict(self, page_valid, page_positions, evict_before_pos: int, stream=None) -> int:
        """Evict pages with position below the threshold; returns the count
        (kessie_hip_ctypes.py:292-314)."""
        assert page_valid.dtype == torch.int8
        assert page_positions.dtype == torch.int32
        num_pages = page_valid.shape[0]
        evict_count = torch.zeros(1, dtype=torch.int32, device=page_valid.device)
        self.lib.launch_kessie_page_evict(self._ptr(page_valid), self._ptr(page_positions), self._ptr(evict_count),
                                          evict_before_pos, num_pages, self._get_stream_ptr(stream))
        self._check("page_evict")
        if stream is None:
            torch.cuda.synchronize()
        return evict_count.item()

    def page_insert(self, kv_cache, new_keys, new_values, target_page_ids, page_valid, page_positions,
                    insert_conv_position: int, stream=None):
        """Insert probe KV into allocated pages (kessie_hip_ctypes.py:316-346)."""
        assert kv_cache.dtype in (torch.float16, torch.bfloat16)
        assert new_keys.dtype == kv_cache.dtype
        num_tokens, num_heads, head_dim = new_keys.shape
        page_size = kv_cache.shape[1]
        max_pages = kv_cache.shape[0]
        if kv_cache.dtype == torch.float16:
            self.lib.launch_kessie_page_insert(self._ptr(kv_cache), self._ptr(new_keys), self._ptr(new_values),
                                               self._ptr(target_page_ids), self._ptr(page_valid),
                                               self._ptr(page_positions), insert_conv_position, num_tokens,
                                               num_heads, head_dim, page_size, max_pages,
                                               self._get_stream_ptr(stream))
            self._check("page_insert")
        else:
            ops.page_insert(kv_cache, new_keys, new_values, target_page_ids, page_valid, page_positions,
                            insert_conv_position, stream=self._get_stream_ptr(stream).value or 0)
        if stream is None:
            torch.cuda.synchronize()
