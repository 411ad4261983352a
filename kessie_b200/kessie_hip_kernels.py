"""Drop-in replacement for the reference module ``kessie_hip_kernels``.

Same public names, signatures and defaults as kessie_hip_kernels.py:367-606;
every accelerated entry point runs on libkessie_cuda.so (sm_100a) and there is
no Triton or CPU path behind them -- if the library is missing, the call
raises ``KessieLibraryError``.

    kessie_fused_fog_attention   kessie_hip_kernels.py:367-400
    kessie_windowed_attention    kessie_hip_kernels.py:416-440
    kessie_build_fog_weights     kessie_hip_kernels.py:403-413
    kessie_rope_remap            kessie_hip_kernels.py:443-477
    KeSSiePagedKVCache           kessie_hip_kernels.py:484-570
    *_ref                        kessie_hip_kernels.py:577-606 (reference math, torch)

Differences from the reference, all deliberate:
  * inputs may be fp16 or bf16, with Hq a multiple of Hkv (GQA);
  * ``kessie_rope_remap`` works in place on strided K without copying and
    rotates every element (the reference's Triton grid rotates only the
    first ceil(T*H*half/256) pairs, kessie_hip_kernels.py:313-316,466-467);
  * ``KeSSiePagedKVCache.evict_before`` runs the eviction rule of the HIP
    kernel (kessie_kernels_v2.hip:403-406) with an ordered device compaction,
    reproducing the reference's free-list order with one device->host copy
    instead of one sync per page (kessie_hip_kernels.py:535-538).
"""

from __future__ import annotations

import logging
import math
from typing import List, Optional, Tuple

import torch

from . import ops
from ._lib import KessieLibraryError  # noqa: F401  (re-exported for callers)

logger = logging.getLogger("KeSSie.B200")

HAS_KESSIE_CUDA = True


def _device_of(t: torch.Tensor) -> torch.device:
    if not t.is_cuda:
        raise ValueError(f"KeSSie B200 kernels need CUDA tensors, got {t.device}")
    return t.device


# =============================================================================
# Attention
# =============================================================================

def kessie_fused_fog_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, fog_weights: torch.Tensor,
                               window_size: int = 0, causal: bool = True,
                               sm_scale: Optional[float] = None) -> torch.Tensor:
    """Flash attention with fused fog decay on V (kessie_hip_kernels.py:367-400).

    q: [Z, Hq, N, D]; k, v: [Z, Hkv, N, D] (fp16, bf16 or fp32); fog_weights: [N]
    float32, 1.0 = clear, < 1.0 = fogged."""
    Z, H, N, D = q.shape
    assert fog_weights.shape == (N,)
    _device_of(q)
    return ops.fog_attention(q.contiguous(), k.contiguous(), v.contiguous(), fog_weights.to(q.device),
                             window_size, causal, sm_scale)


def kessie_windowed_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, window_size: int = 0,
                              causal: bool = True, sm_scale: Optional[float] = None) -> torch.Tensor:
    """Windowed flash attention without fog (kessie_hip_kernels.py:416-440)."""
    _device_of(q)
    return ops.fog_attention(q.contiguous(), k.contiguous(), v.contiguous(), None, window_size, causal, sm_scale)


def kessie_build_fog_weights(seq_len: int, fog_alpha: float = 0.5, fog_start: float = 0.5,
                             device: torch.device = None) -> torch.Tensor:
    """Fog decay weights, 1.0 = clear, < 1.0 = fogged (kessie_hip_kernels.py:403-413).

    clear_start = int(seq_len * (1.0 - fog_start)) is evaluated here in Python
    float64, exactly as the reference; the vector is built on the GPU and
    returned on ``device`` (the current CUDA device when None is given, as
    there is no CPU path)."""
    clear_start = int(seq_len * (1.0 - fog_start))
    dev = torch.device(device) if device is not None else None
    build_dev = dev if (dev is not None and dev.type == "cuda") else None
    w = ops.build_fog_weights(seq_len, clear_start, fog_alpha, build_dev)
    if dev is not None and dev.type != "cuda":
        w = w.to(dev)
    return w


def kessie_rope_remap(k_tensor: torch.Tensor, orig_positions: torch.Tensor, target_positions: torch.Tensor,
                      rope_theta: float = 10000.0) -> torch.Tensor:
    """Re-rotate K from original to target RoPE positions, in place
    (kessie_hip_kernels.py:443-477).  k_tensor: [T, H, D] with D contiguous."""
    _device_of(k_tensor)
    return ops.rope_remap(k_tensor, orig_positions.to(k_tensor.device), target_positions.to(k_tensor.device),
                          rope_theta)


# =============================================================================
# KeSSiePagedKVCache
# =============================================================================

class KeSSiePagedKVCache:
    """Paged KV cache with KeSSie fog-of-war semantics (kessie_hip_kernels.py:484-570).

    Same state and methods as the reference: ``kv_data`` [L, P, ps, 2, H, D],
    ``page_positions`` int32 [P], ``page_valid`` int8 [P], the host free list
    ``free_pages`` (source of truth for allocation order: pops from the end),
    ``total_evictions`` / ``total_insertions`` and ``get_stats()``.
    Additionally keeps ``page_allocated`` int8 [P] on the device, the mirror of
    "not in free_pages" that the device eviction needs to reproduce the
    reference's free-list rebuild."""

    def __init__(self, num_pages, page_size, num_layers, num_heads, head_dim, device, dtype=torch.float16):
        self.num_pages = num_pages
        self.page_size = page_size
        self.num_layers = num_layers
        self.num_heads = num_heads
        self.head_dim = head_dim
        self.device = torch.device(device)
        if self.device.type != "cuda":
            raise ValueError("KeSSiePagedKVCache on B200 lives on a CUDA device")
        self.dtype = dtype
        self.kv_data = torch.zeros(num_layers, num_pages, page_size, 2, num_heads, head_dim, device=self.device,
                                   dtype=dtype)
        self.page_positions = torch.zeros(num_pages, dtype=torch.int32, device=self.device)
        self.page_valid = torch.zeros(num_pages, dtype=torch.int8, device=self.device)
        self.page_allocated = torch.zeros(num_pages, dtype=torch.int8, device=self.device)
        self.free_pages: List[int] = list(range(num_pages))
        self.total_evictions = 0
        self.total_insertions = 0
        self._host_buf = torch.empty(num_pages + 1, dtype=torch.int32, pin_memory=True)
        logger.info(f"KeSSiePagedKVCache: {num_pages}p x {page_size}t, {num_layers}L x {num_heads}H x {head_dim}D, "
                    f"VRAM={self.vram_bytes / 1e9:.2f} GB")

    @property
    def vram_bytes(self):
        return self.kv_data.nelement() * self.kv_data.element_size()

    @property
    def active_pages(self):
        return self.num_pages - len(self.free_pages)

    @property
    def active_tokens(self):
        return self.active_pages * self.page_size

    def allocate_pages(self, n):
        """Pop n page ids from the END of free_pages (kessie_hip_kernels.py:520-524)."""
        if len(self.free_pages) < n:
            return None
        ids = [self.free_pages.pop() for _ in range(n)]
        t = torch.tensor(ids, dtype=torch.int32, device=self.device)
        if n:
            self.page_allocated[t.long()] = 1
        return t

    def evict_before(self, position):
        """Evict valid pages whose position < `position`; freed pages are
        appended to free_pages in ascending page order
        (kessie_hip_kernels.py:526-540, rule kessie_kernels_v2.hip:403-406)."""
        cnt, ids = ops.page_evict(self.page_valid, self.page_positions, int(position), self.page_allocated)
        # one device->host copy of [count, ids...]
        self._host_buf[0:1].copy_(cnt, non_blocking=True)
        self._host_buf[1:1 + self.num_pages].copy_(ids[:self.num_pages], non_blocking=True)
        torch.cuda.current_stream(self.device).synchronize()
        n = int(self._host_buf[0])
        if n:
            self.free_pages.extend(self._host_buf[1:1 + n].tolist())
        self.total_evictions += n
        return n

    def insert_probe_kv(self, layer_idx, keys, values, conv_position, orig_positions=None,
                        rope_theta: float = 10000.0):
        """Insert probe KV [T, H, D] into freshly allocated pages
        (kessie_hip_kernels.py:542-556) with one device copy kernel.
        With ``orig_positions`` (int32 [T]) the keys are also re-rotated from
        their original positions to conv_position + t (the recall path,
        fused insert + RoPE remap)."""
        num_tokens = keys.shape[0]
        pages_needed = (num_tokens + self.page_size - 1) // self.page_size
        page_ids = self.allocate_pages(pages_needed)
        if page_ids is None:
            return False
        k = keys.to(device=self.device, dtype=self.dtype)
        v = values.to(device=self.device, dtype=self.dtype)
        if k.stride(-1) != 1 or k.stride() != v.stride():
            k, v = k.contiguous(), v.contiguous()
        ops.page_insert(self.kv_data[layer_idx], k, v, page_ids, self.page_valid, self.page_positions,
                        int(conv_position), orig_positions=orig_positions, rope_theta=rope_theta)
        self.total_insertions += num_tokens
        return True

    def get_layer_kv(self, layer_idx):
        """K, V [n_valid * ps, H, D] of the valid pages in physical-page order
        (kessie_hip_kernels.py:558-564)."""
        cnt, ids = ops.list_valid_pages(self.page_valid)
        n = int(cnt.item())
        if n == 0:
            empty = torch.empty(0, self.num_heads, self.head_dim, device=self.device, dtype=self.dtype)
            return empty, empty.clone()
        return ops.page_gather(self.kv_data[layer_idx], ids[:n])

    def get_stats(self):
        return {"total_pages": self.num_pages, "active_pages": self.active_pages,
                "free_pages": len(self.free_pages), "active_tokens": self.active_tokens,
                "vram_gb": self.vram_bytes / 1e9,
                "total_evictions": self.total_evictions, "total_insertions": self.total_insertions}


# =============================================================================
# Reference implementations (kessie_hip_kernels.py:577-606), torch math.
# Kept for API compatibility with the reference module (its tests compare
# against them); no accelerated entry point above calls them.
# =============================================================================

def kessie_windowed_attention_ref(q, k, v, window_size=0, causal=True, sm_scale=None):
    Z, H, N, D = q.shape
    if sm_scale is None:
        sm_scale = 1.0 / math.sqrt(D)
    scores = torch.matmul(q, k.transpose(-2, -1)) * sm_scale
    pos = torch.arange(N, device=q.device)
    dist = pos[:, None] - pos[None, :]
    keep = torch.ones(N, N, dtype=torch.bool, device=q.device)
    if causal:
        keep &= dist >= 0
    if window_size > 0:
        keep &= (dist >= 0) & (dist < window_size)
    scores = scores.masked_fill(~keep, float("-inf"))
    return torch.matmul(torch.softmax(scores, dim=-1), v)


def kessie_fused_fog_attention_ref(q, k, v, fog_weights, window_size=0, causal=True, sm_scale=None):
    return kessie_windowed_attention_ref(q, k, v * fog_weights[None, None, :, None], window_size, causal, sm_scale)


def _rope_remap_ref(k_tensor, orig_positions, target_positions, rope_theta=10000.0):
    """In-place rotate-half re-rotation by torch ops, computing exactly what
    the reference's checker computes (kessie_hip_kernels.py:596-606), so code
    that uses it as its checker gets the same numbers.  For an fp32 K the
    ``.float()`` of the low half is a view of K itself: the high half is then
    rotated from the already-rotated low half.  The library's kernels follow
    the HIP rule instead (kessie_kernels_v2.hip:697-706: both halves from the
    loaded pair); for fp16 / bf16 K the two agree."""
    num_tokens, num_heads, head_dim = k_tensor.shape
    half_dim = head_dim // 2
    exponents = torch.arange(half_dim, dtype=torch.float32, device=k_tensor.device) / half_dim
    freqs = 1.0 / (rope_theta ** exponents)
    delta = torch.outer((target_positions - orig_positions).float(), freqs)
    cos_d, sin_d = delta.cos()[:, None, :], delta.sin()[:, None, :]
    low = k_tensor[:, :, :half_dim].float()        # a view of k_tensor when K is fp32
    high = k_tensor[:, :, half_dim:].float()
    k_tensor[:, :, :half_dim] = (low * cos_d - high * sin_d).to(k_tensor.dtype)
    k_tensor[:, :, half_dim:] = (low * sin_d + high * cos_d).to(k_tensor.dtype)
    return k_tensor


def kessie_index_query(query_embed: torch.Tensor, index_embeds: torch.Tensor, top_k: int = 0):
    """Cosine similarity between a query and every index embedding -- the
    operation of the reference's _kessie_index_query_kernel
    (kessie_hip_kernels.py:343-360), whose module docstring lists
    kessie_index_query without defining it.  Returns sims [N]; with top_k > 0
    also (top ids, top scores), descending, ties to the lower row index."""
    ids, scores, sims = ops.index_query(query_embed.float(), index_embeds.float(), top_k=max(top_k, 1),
                                        normalize_rows=True, return_sims=True)
    return (sims, ids, scores) if top_k > 0 else sims


# ---------------------------------------------------------------------------
# Self-test suite (kessie_hip_kernels.py:613-747): the same test names,
# configurations and pass thresholds, run on this library's kernels against
# the *_ref functions above.  Without a CUDA device every test logs SKIP and
# passes, as the reference's does without Triton.
# ---------------------------------------------------------------------------
class KeSSieKernelTests:
    WINDOWED_CONFIGS = [(1, 4, 128, 64, 0, True), (1, 4, 128, 64, 64, True),
                        (1, 8, 256, 128, 128, True), (2, 8, 512, 128, 256, True)]

    def __init__(self, device="cuda"):
        self.device = torch.device(device) if torch.cuda.is_available() else torch.device("cpu")
        if self.device.type == "cuda":
            logger.info(f"GPU: {torch.cuda.get_device_name(self.device)}")

    def _gpu(self) -> bool:
        return self.device.type == "cuda"

    def _rand(self, *shape):
        return torch.randn(*shape, device=self.device, dtype=torch.float16)

    def test_windowed_attention_correctness(self) -> bool:
        logger.info("TEST: windowed attention vs kessie_windowed_attention_ref (max-abs < 0.05, fp16)")
        ok = True
        for Z, H, N, D, W, causal in self.WINDOWED_CONFIGS:
            if not self._gpu():
                logger.info(f"  Z={Z} H={H} N={N} D={D} W={W} | SKIP")
                continue
            q, k, v = self._rand(Z, H, N, D), self._rand(Z, H, N, D), self._rand(Z, H, N, D)
            ref = kessie_windowed_attention_ref(q.float(), k.float(), v.float(), W, causal).half()
            md = (ref - kessie_windowed_attention(q, k, v, W, causal)).abs().max().item()
            passed = md < 0.05
            ok &= passed
            logger.info(f"  Z={Z} H={H} N={N} D={D} W={W} | max_diff={md:.6f} [{'PASS' if passed else 'FAIL'}]")
        return ok

    def test_fused_fog_attention(self) -> bool:
        logger.info("TEST: fused fog attention vs kessie_fused_fog_attention_ref (max-abs < 0.1, fp16)")
        if not self._gpu():
            logger.info("  SKIP")
            return True
        Z, H, N, D = 1, 8, 512, 128
        q, k, v = self._rand(Z, H, N, D), self._rand(Z, H, N, D), self._rand(Z, H, N, D)
        fog = kessie_build_fog_weights(N, 0.5, 0.5, self.device)
        ref = kessie_fused_fog_attention_ref(q.float(), k.float(), v.float(), fog).half()
        md = (ref - kessie_fused_fog_attention(q, k, v, fog)).abs().max().item()
        logger.info(f"  N={N} fog_alpha=0.5 | max_diff={md:.6f} [{'PASS' if md < 0.1 else 'FAIL'}]")
        return md < 0.1

    def test_rope_remap(self) -> bool:
        logger.info("TEST: RoPE remap round trip 100 -> 5000 -> 100 (< 0.05) and identity (< 1e-5)")
        if not self._gpu():
            logger.info("  SKIP")
            return True
        L, H, D = 64, 8, 128
        k = self._rand(L, H, D)
        k0 = k.clone()
        orig = torch.arange(100, 100 + L, dtype=torch.int32, device=self.device)
        tgt = torch.arange(5000, 5000 + L, dtype=torch.int32, device=self.device)
        kessie_rope_remap(k, orig, tgt)
        kessie_rope_remap(k, tgt, orig)
        md = (k0.float() - k.float()).abs().max().item()
        k2 = self._rand(L, H, D)
        k2o = k2.clone()
        kessie_rope_remap(k2, orig, orig)
        md2 = (k2o.float() - k2.float()).abs().max().item()
        logger.info(f"  round trip max_diff={md:.6f} [{'PASS' if md < 0.05 else 'FAIL'}]  "
                    f"identity max_diff={md2:.6f} [{'PASS' if md2 < 1e-5 else 'FAIL'}]")
        return md < 0.05 and md2 < 1e-5

    def test_paged_kv_cache(self) -> bool:
        logger.info("TEST: paged KV cache insert 512 at position 0, evict before 5000")
        if not self._gpu():
            logger.info("  SKIP")
            return True
        cache = KeSSiePagedKVCache(64, 128, 2, 8, 64, self.device)
        keys, vals = self._rand(512, 8, 64), self._rand(512, 8, 64)
        ok = cache.insert_probe_kv(0, keys, vals, 0)
        logger.info(f"  insert: {'OK' if ok else 'FAIL'}, active={cache.active_pages}")
        freed = cache.evict_before(5000)
        logger.info(f"  evict <5000: {freed} freed, active={cache.active_pages}")
        return True

    def bench_fused_vs_separate(self, seq_len=4096):
        """Fog folded into V then windowed attention, against the fused kernel
        (CUDA-event timings, 20 runs after 3 warm-ups)."""
        logger.info(f"BENCH: fused vs separate fog (N={seq_len})")
        if not self._gpu():
            logger.info("  SKIP")
            return None
        Z, H, D = 1, 8, 128
        q, k, v = self._rand(Z, H, seq_len, D), self._rand(Z, H, seq_len, D), self._rand(Z, H, seq_len, D)
        fog = kessie_build_fog_weights(seq_len, 0.5, 0.5, self.device)

        def timed(fn):
            for _ in range(3):
                fn()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            for _ in range(20):
                fn()
            b.record()
            torch.cuda.synchronize()
            return a.elapsed_time(b) / 20

        t_sep = timed(lambda: kessie_windowed_attention(q, k, v * fog[None, None, :, None].to(v.dtype)))
        t_fused = timed(lambda: kessie_fused_fog_attention(q, k, v, fog))
        logger.info(f"  separate: {t_sep:.3f} ms | fused: {t_fused:.3f} ms | speedup: {t_sep / t_fused:.2f}x")
        return t_sep, t_fused

    def run_all(self) -> bool:
        logger.info(f"KeSSie B200 kernel test suite (device {self.device})")
        ok = self.test_windowed_attention_correctness()
        ok &= self.test_fused_fog_attention()
        ok &= self.test_rope_remap()
        ok &= self.test_paged_kv_cache()
        if self._gpu():
            self.bench_fused_vs_separate()
        logger.info("done")
        return ok


if __name__ == "__main__":
    import argparse
    logging.basicConfig(level=logging.INFO, format="%(message)s")
    ap = argparse.ArgumentParser(description="KeSSie B200 kernel tests")
    ap.add_argument("--device", default="cuda", choices=["cuda", "cpu"])
    ap.add_argument("--test", default="all",
                    choices=["all", "correctness", "fused-fog", "rope-remap", "bench-fog", "bench-paged"])
    ap.add_argument("--seq-len", type=int, default=4096)
    a = ap.parse_args()
    t = KeSSieKernelTests(device=a.device)
    {"all": t.run_all, "correctness": t.test_windowed_attention_correctness,
     "fused-fog": t.test_fused_fog_attention, "rope-remap": t.test_rope_remap,
     "bench-fog": lambda: t.bench_fused_vs_separate(a.seq_len), "bench-paged": t.test_paged_kv_cache}[a.test]()
