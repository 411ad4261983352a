"""Tensor-level wrappers over the C ABI (PyTorch tensors are buffers only).

Every function here launches CUDA kernels of libkessie_cuda.so on the given
stream (default: torch's current stream) and never computes on the CPU.
Shapes follow the reference: K rows are [tokens, heads, head_dim] with
head_dim contiguous; KV caches are addressed by (page, token, kv, head)
strides so both the KeSSie layout [P, ps, 2, H, D]
(kessie_hip_kernels.py:496-498) and vLLM's [2, P, ps, H, D]
(kessie_kv_connector.py:309,465) work without copies.
"""

from __future__ import annotations

import ctypes
import math
import threading
from typing import Optional, Tuple

import torch

from . import _lib

_DT = {torch.float16: _lib.DTYPE_F16, torch.bfloat16: _lib.DTYPE_BF16, torch.float32: _lib.DTYPE_F32}

_ws_lock = threading.Lock()
_ws_cache: dict = {}


def dtype_code(t: torch.Tensor) -> int:
    try:
        return _DT[t.dtype]
    except KeyError:
        raise TypeError(f"unsupported dtype {t.dtype}") from None


def _p(t: Optional[torch.Tensor]):
    return None if t is None else t.data_ptr()


_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def _stream(stream, device_index: Optional[int] = None) -> int:
    """The cudaStream_t to launch on: `stream`, or torch's current stream of
    `device_index` (the current device when None).  The current stream is
    read as a raw handle, without building a torch.cuda.Stream per call."""
    if stream is None:
        if _raw_stream is not None:
            return _raw_stream(torch.cuda.current_device() if device_index is None else device_index)
        return torch.cuda.current_stream(device_index).cuda_stream
    if isinstance(stream, torch.cuda.Stream):
        return stream.cuda_stream
    return int(stream)


def _need_cuda(*ts):
    for t in ts:
        if t is not None and not t.is_cuda:
            raise ValueError(f"tensor must be on a CUDA device, got {t.device}")


def _i32(t: Optional[torch.Tensor], device) -> Optional[torch.Tensor]:
    if t is None:
        return None
    if not torch.is_tensor(t):
        t = torch.as_tensor(t, dtype=torch.int32, device=device)
    if t.dtype != torch.int32:
        t = t.to(torch.int32)
    return t.contiguous()


def workspace(nbytes: int, device, tag: str = "default") -> torch.Tensor:
    """A cached uint8 scratch buffer of at least nbytes on device (reused by
    later calls with the same tag, so steady-state calls allocate nothing).
    Calls that share a tag must be ordered on one stream."""
    dev = torch.device(device)
    key = (dev.index if dev.index is not None else torch.cuda.current_device(), tag)
    with _ws_lock:
        buf = _ws_cache.get(key)
        if buf is None or buf.numel() < nbytes:
            buf = torch.empty(max(int(nbytes), 256), dtype=torch.uint8, device=dev)
            _ws_cache[key] = buf
        return buf


def read_device_status(stream=None) -> int:
    """Synchronise the stream and return/clear the device status bits."""
    r = _lib.load().kessie_read_device_status(_stream(stream))
    if r < 0:
        _lib.check(r, "read_device_status")
    return r


# --------------------------------------------------------------------- RoPE
def rope_remap(k: torch.Tensor, orig_positions, target_positions, rope_theta: float = 10000.0, stream=None):
    """In-place re-rotation of K [T, H, D] (kessie_hip_kernels.py:596-606)."""
    _need_cuda(k)
    if k.dim() != 3 or k.stride(2) != 1:
        raise ValueError("k must be [tokens, heads, head_dim] with head_dim contiguous")
    T, H, D = k.shape
    o = _i32(orig_positions, k.device)
    t = _i32(target_positions, k.device)
    if o.numel() != T or t.numel() != T:
        raise ValueError("positions must have one entry per token")
    lib = _lib.load()
    _lib.check(lib.kessie_rope_remap_v2(k.data_ptr(), dtype_code(k), T, H, D, k.stride(0), k.stride(1),
                                        o.data_ptr(), t.data_ptr(), float(rope_theta), _stream(stream)),
               "rope_remap")
    return k


# --------------------------------------------------------------------- fog weights
def build_fog_weights(seq_len: int, clear_start: int, fog_alpha: float, device=None, stream=None) -> torch.Tensor:
    """fp32 [seq_len] fog weights on a CUDA device (kessie_hip_kernels.py:403-413)."""
    dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
    if dev.type != "cuda":
        raise ValueError("fog weights are built on a CUDA device")
    w = torch.empty(int(seq_len), dtype=torch.float32, device=dev)
    _lib.check(_lib.load().kessie_build_fog_weights_v2(_p(w) if seq_len else None, int(seq_len), int(clear_start),
                                                       float(fog_alpha), _stream(stream)), "build_fog_weights")
    return w


# --------------------------------------------------------------------- pages
def kv_layout_strides(kv: torch.Tensor, layout: str = "kessie") -> Tuple[int, int, int, int, int, int, int, int]:
    """(page, token, kv, head strides, num_pages, page_size, heads, head_dim)."""
    if layout == "kessie":          # [P, ps, 2, H, D]
        P, ps, two, H, D = kv.shape
        s = kv.stride()
        return s[0], s[1], s[2], s[3], P, ps, H, D
    if layout == "vllm":            # [2, P, ps, H, D]
        two, P, ps, H, D = kv.shape
        s = kv.stride()
        return s[1], s[2], s[0], s[3], P, ps, H, D
    raise ValueError(f"unknown layout {layout}")


def page_evict(page_valid: torch.Tensor, page_positions: torch.Tensor, evict_before_pos: int,
               page_allocated: Optional[torch.Tensor] = None, stream=None) -> Tuple[torch.Tensor, torch.Tensor]:
    """Device eviction + ordered compaction.  Returns (count int32[1],
    ids int32[P]); ids[:count] are the freed page ids in ascending order."""
    _need_cuda(page_valid, page_positions, page_allocated)
    P = page_valid.numel()
    dev = page_valid.device
    count = torch.zeros(1, dtype=torch.int32, device=dev)
    ids = torch.empty(max(P, 1), dtype=torch.int32, device=dev)
    lib = _lib.load()
    ws_n = lib.kessie_page_evict_workspace_size(P)
    ws = workspace(ws_n, dev, "compaction")
    _lib.check(lib.kessie_page_evict_v2(page_valid.data_ptr(), page_positions.data_ptr(), _p(page_allocated), P,
                                        int(evict_before_pos), count.data_ptr(), ids.data_ptr(), ws.data_ptr(),
                                        ws.numel(), _stream(stream)), "page_evict")
    return count, ids


def list_valid_pages(page_valid: torch.Tensor, stream=None) -> Tuple[torch.Tensor, torch.Tensor]:
    """Ascending ids of pages with page_valid != 0: (count int32[1], ids int32[P])."""
    _need_cuda(page_valid)
    P = page_valid.numel()
    dev = page_valid.device
    count = torch.zeros(1, dtype=torch.int32, device=dev)
    ids = torch.empty(max(P, 1), dtype=torch.int32, device=dev)
    lib = _lib.load()
    ws = workspace(lib.kessie_page_evict_workspace_size(P), dev, "compaction")
    _lib.check(lib.kessie_page_list_valid_v2(page_valid.data_ptr(), P, count.data_ptr(), ids.data_ptr(),
                                             ws.data_ptr(), ws.numel(), _stream(stream)), "list_valid_pages")
    return count, ids


def page_insert(kv: torch.Tensor, keys: torch.Tensor, values: torch.Tensor, page_ids, page_valid=None,
                page_positions=None, conv_pos: int = 0, orig_positions=None, target_positions=None,
                rope_theta: float = 10000.0, layout: str = "kessie", stream=None):
    """Copy keys/values [T, H, D] into pages page_ids (token t -> page
    page_ids[t // ps], slot t % ps), optionally re-rotating K from
    orig_positions to target_positions (default conv_pos + t)."""
    _need_cuda(kv, keys, values)
    if keys.dtype != kv.dtype or values.dtype != kv.dtype:
        raise TypeError("keys/values dtype must match the cache")
    if keys.stride(2) != 1 or values.stride(2) != 1 or keys.stride() != values.stride():
        raise ValueError("keys/values must share strides with head_dim contiguous")
    ps_, ts_, kvs_, hs_, P, ps, H, D = kv_layout_strides(kv, layout)
    T = keys.shape[0]
    ids = _i32(page_ids, kv.device)
    o = _i32(orig_positions, kv.device)
    tg = _i32(target_positions, kv.device)
    lib = _lib.load()
    _lib.check(lib.kessie_page_insert_v2(kv.data_ptr(), dtype_code(kv), ps_, ts_, kvs_, hs_, P, ps, keys.data_ptr(),
                                         values.data_ptr(), keys.stride(0), keys.stride(1), T, H, D, ids.data_ptr(),
                                         _p(page_valid), _p(page_positions), int(conv_pos), _p(o), _p(tg),
                                         float(rope_theta), _stream(stream)), "page_insert")


def page_gather(kv: torch.Tensor, page_ids, layout: str = "kessie", out_keys=None, out_values=None,
                want_keys: bool = True, want_values: bool = True, stream=None):
    """Gather pages -> dense K, V [n*ps, H, D] in the order of page_ids."""
    _need_cuda(kv)
    ps_, ts_, kvs_, hs_, P, ps, H, D = kv_layout_strides(kv, layout)
    ids = _i32(page_ids, kv.device)
    n = ids.numel()
    if want_keys and out_keys is None:
        out_keys = torch.empty(n * ps, H, D, dtype=kv.dtype, device=kv.device)
    if want_values and out_values is None:
        out_values = torch.empty(n * ps, H, D, dtype=kv.dtype, device=kv.device)
    lib = _lib.load()
    _lib.check(lib.kessie_page_gather_v2(kv.data_ptr(), dtype_code(kv), ps_, ts_, kvs_, hs_, P, ps, ids.data_ptr(), n,
                                         H, D, _p(out_keys if want_keys else None),
                                         _p(out_values if want_values else None), _stream(stream)), "page_gather")
    return out_keys, out_values


# --------------------------------------------------------------------- additive fog bias
class FogBias:
    """Additive fog bias of the vLLM attention path (kessie_attention.py:114-139),
    applied inside the attention kernels: per sequence of kv_len keys,
    fb = int(kv_len * (1 - fog_start)); bias(j) = -fog_alpha * (1 - j/fb)^2
    for j < fb, 0 after, recall_boost at recalled positions.  ``dtype`` is the
    dtype whose rounding the bias follows (the reference builds it in the
    query dtype).  Holds the device bitmap of the recalled positions."""

    def __init__(self, fog_alpha: float = 0.5, fog_start: float = 0.5, recall_positions=(),
                 recall_boost: float = 0.1, dtype=torch.bfloat16, device=None):
        import numpy as np
        self.fog_alpha, self.fog_start, self.recall_boost = float(fog_alpha), float(fog_start), float(recall_boost)
        self.dtype = dtype
        pos = np.asarray(sorted(int(x) for x in recall_positions if int(x) >= 0), dtype=np.int64)
        self.recall_nbits = int(pos[-1]) + 1 if pos.size else 0
        self.bits = None
        if pos.size:
            words = np.zeros((self.recall_nbits + 31) // 32, dtype=np.uint32)
            np.bitwise_or.at(words, pos >> 5, (np.uint32(1) << (pos & 31).astype(np.uint32)))
            dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
            self.bits = torch.from_numpy(words.view(np.int32)).to(dev)

    def c_struct(self):
        return _lib.KessieFogBias(self.fog_alpha, self.fog_start, self.recall_boost, _p(self.bits),
                                  self.recall_nbits, _DT[self.dtype])


def build_fog_bias(kv_len: int, bias: "FogBias", out: Optional[torch.Tensor] = None, device=None,
                   stream=None) -> torch.Tensor:
    """The reference's bias buffer (1, 1, 1, kv_len) in bias.dtype."""
    dev = torch.device(device) if device is not None else (bias.bits.device if bias.bits is not None
                                                           else torch.device("cuda", torch.cuda.current_device()))
    if out is None:
        out = torch.empty(kv_len, dtype=bias.dtype, device=dev)
    _need_cuda(out)
    cs = bias.c_struct()
    _lib.check(_lib.load().kessie_build_fog_bias_v2(out.data_ptr(), dtype_code(out), int(kv_len), ctypes.byref(cs),
                                                    _stream(stream)), "build_fog_bias")
    return out.view(1, 1, 1, kv_len)


# --------------------------------------------------------------------- decode
def decode_workspace_bytes(batch, num_q_heads, num_kv_heads, head_dim, max_seq_len, page_size=16) -> int:
    return int(_lib.load().kessie_paged_fog_decode_workspace_size(batch, num_q_heads, num_kv_heads, head_dim,
                                                                  max_seq_len, page_size))


def _decode_args(q, k_cache, v_cache, block_table, seq_lens, clear_start, fog_alpha, fog_weights, window_size,
                 sm_scale, kv_pos_offset, q_positions, max_seq_len, ws, tag="decode"):
    """Checks + the argument tuple shared by the decode entry points (all
    arguments up to and including dtype), plus the workspace."""
    _need_cuda(q, k_cache, v_cache, block_table, seq_lens)
    B, Hq, D = q.shape
    P, ps, Hkv, Dk = k_cache.shape
    ks, qs = k_cache.stride(), q.stride()
    if Dk != D or v_cache.shape != k_cache.shape or v_cache.stride() != ks:
        raise ValueError("k_cache/v_cache must be matching [P, ps, Hkv, D] views")
    if k_cache.dtype != q.dtype or v_cache.dtype != q.dtype:
        raise TypeError("q and the cache must share a dtype")
    if qs[2] != 1 or ks[3] != 1:
        raise ValueError("head_dim must be contiguous")
    bt = block_table if block_table.dtype == torch.int32 else block_table.to(torch.int32)
    if bt.stride(1) != 1:
        bt = bt.contiguous()
    sl = _i32(seq_lens, q.device)
    if max_seq_len is None:
        max_seq_len = bt.shape[1] * ps
    if max_seq_len > bt.shape[1] * ps:
        raise ValueError(f"max_seq_len {max_seq_len} exceeds the block table capacity {bt.shape[1] * ps}")
    if sm_scale is None:
        sm_scale = 1.0 / math.sqrt(D)
    cs = _i32(clear_start, q.device)
    off = _i32(kv_pos_offset, q.device)
    qp = _i32(q_positions, q.device)
    fw = None
    if fog_weights is not None:
        fw = fog_weights if fog_weights.dtype == torch.float32 else fog_weights.float()
        fw = fw.contiguous()
    lib = _lib.load()
    need = lib.kessie_paged_fog_decode_workspace_size(B, Hq, Hkv, D, int(max_seq_len), ps)
    if ws is None:
        ws = workspace(need, q.device, tag)
    # keep the converted tensors alive until the launch
    keep = (bt, sl, cs, off, qp, fw)
    args = (q.data_ptr(), qs[0], qs[1], k_cache.data_ptr(), v_cache.data_ptr(), ks[0],
            ks[1], ks[2], P, ps, bt.data_ptr(), bt.stride(0), sl.data_ptr(), _p(off), _p(qp),
            _p(cs), float(fog_alpha), _p(fw), int(window_size), float(sm_scale), B, Hq, Hkv, D, int(max_seq_len),
            dtype_code(q))
    return lib, args, ws, keep


def paged_fog_decode(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, block_table: torch.Tensor,
                     seq_lens: torch.Tensor, clear_start=None, fog_alpha: float = 0.5, fog_weights=None,
                     window_size: int = 0, sm_scale: Optional[float] = None, kv_pos_offset=None,
                     q_positions=None, max_seq_len: Optional[int] = None, out: Optional[torch.Tensor] = None,
                     out_partial: Optional[torch.Tensor] = None, want_out: bool = True, stream=None,
                     ws: Optional[torch.Tensor] = None, phases: int = 3, bias: Optional["FogBias"] = None):
    """Paged fog decode: q [B, Hq, D]; k_cache / v_cache [P, ps, Hkv, D]
    views (any page/token/head strides, D contiguous); block_table [B, maxP]
    int32; seq_lens [B] int32.  Returns out [B, Hq, D] (q.dtype) and, if
    requested, out_partial fp32 [B, Hq, D+2] = (O/l, m, l) for the
    context-parallel combine.  One kernel launch (the split merge is fused)."""
    B, Hq, D = q.shape
    if want_out and out is None:
        out = torch.empty(B, Hq, D, dtype=q.dtype, device=q.device)
    lib, args, ws, keep = _decode_args(q, k_cache, v_cache, block_table, seq_lens, clear_start, fog_alpha,
                                       fog_weights, window_size, sm_scale, kv_pos_offset, q_positions, max_seq_len, ws)
    if bias is not None:
        cs = bias.c_struct()
        _lib.check(lib.kessie_paged_fog_decode_biased_v2(*args, ctypes.byref(cs), _p(out if want_out else None),
                                                         _p(out_partial), ws.data_ptr(), ws.numel(), _stream(stream)),
                   "paged_fog_decode")
        return out
    _lib.check(lib.kessie_paged_fog_decode_ex_v2(*args, _p(out if want_out else None), _p(out_partial), ws.data_ptr(),
                                                 ws.numel(), int(phases), _stream(stream, q.device.index)),
               "paged_fog_decode")
    return out


class CpExchange:
    """This rank's context-parallel exchange buffer plus the mapped buffers
    of the other ranks (CUDA IPC over NVLink).  Created collectively: every
    rank of `group` constructs it with the same shapes."""

    def __init__(self, world: int, rank: int, batch: int, num_q_heads: int, num_kv_heads: int, head_dim: int,
                 device, group=None):
        import ctypes
        import torch.distributed as dist
        lib = _lib.load()
        self.world, self.rank = int(world), int(rank)
        self.shape = (int(batch), int(num_q_heads), int(num_kv_heads), int(head_dim))
        self.nbytes = lib.kessie_cp_exchange_bytes(self.world, batch, num_q_heads, num_kv_heads, head_dim)
        if self.nbytes == 0:
            raise ValueError("cp exchange: unsupported shape / world size")
        dev = torch.device(device)
        with torch.cuda.device(dev):
            own = ctypes.c_void_p()
            handle = (ctypes.c_uint8 * 64)()
            _lib.check(lib.kessie_cp_exchange_alloc(self.nbytes, ctypes.byref(own), handle), "cp_exchange_alloc")
            self._own = own.value
            mine = torch.tensor(list(bytes(handle)), dtype=torch.uint8, device=dev)
            allh = torch.empty(self.world * 64, dtype=torch.uint8, device=dev)
            dist.all_gather_into_tensor(allh, mine, group=group)
            allh = allh.view(self.world, 64).cpu()
            self._opened = []
            ptrs = []
            for r in range(self.world):
                if r == self.rank:
                    ptrs.append(self._own)
                    continue
                hb = (ctypes.c_uint8 * 64)(*allh[r].tolist())
                pp = ctypes.c_void_p()
                _lib.check(lib.kessie_cp_exchange_open(hb, ctypes.byref(pp)), "cp_exchange_open")
                self._opened.append(pp.value)
                ptrs.append(pp.value)
        self.ptrs = (ctypes.c_void_p * self.world)(*ptrs)
        self.device = dev
        self._epoch = 0

    def next_epoch(self) -> int:
        """1, 2, 3, ...; wraps keeping the odd/even alternation."""
        self._epoch = self._epoch % 0x7FFFFFFE + 1
        return self._epoch

    def close(self):
        """Unmap the peers' buffers, then free this rank's.  Call on every
        rank after a barrier that follows the last step."""
        lib = _lib.load()
        with torch.cuda.device(self.device):
            for p in self._opened:
                lib.kessie_cp_exchange_close(p)
            self._opened = []
            if self._own:
                lib.kessie_cp_exchange_free(self._own)
                self._own = None


def paged_fog_decode_cp(exchange: "CpExchange", epoch: int, q: torch.Tensor, k_cache: torch.Tensor,
                        v_cache: torch.Tensor, block_table: torch.Tensor, seq_lens: torch.Tensor, clear_start=None,
                        fog_alpha: float = 0.5, fog_weights=None, window_size: int = 0,
                        sm_scale: Optional[float] = None, kv_pos_offset=None, q_positions=None,
                        max_seq_len: Optional[int] = None, out: Optional[torch.Tensor] = None,
                        out_partial: Optional[torch.Tensor] = None, wait_timeout_s: float = 2.0, phases: int = 3,
                        stream=None, ws: Optional[torch.Tensor] = None):
    """One context-parallel decode step over this rank's shard: the decode
    kernel pushes the shard result of each (seq, kv_head) group into every
    rank's exchange buffer (phases bit 0); the combine kernel waits for all
    ranks and writes out / out_partial (bit 1)."""
    B, Hq, D = q.shape
    if tuple(exchange.shape) != (B, Hq, k_cache.shape[2], D):
        raise ValueError(f"exchange buffers were sized for {tuple(exchange.shape)}, this step is "
                         f"{(B, Hq, k_cache.shape[2], D)} (B, Hq, Hkv, D)")
    if (phases & 2) and out is None and out_partial is None:
        out = torch.empty(B, Hq, D, dtype=q.dtype, device=q.device)
    lib, args, ws, keep = _decode_args(q, k_cache, v_cache, block_table, seq_lens, clear_start, fog_alpha,
                                       fog_weights, window_size, sm_scale, kv_pos_offset, q_positions, max_seq_len, ws)
    _lib.check(lib.kessie_paged_fog_decode_cp_v2(
        *args, exchange.ptrs, exchange.rank, exchange.world, int(epoch), int(wait_timeout_s * 1e9), _p(out),
        _p(out_partial), ws.data_ptr(), ws.numel(), int(phases), _stream(stream, q.device.index)), "paged_fog_decode_cp")
    return out


def cp_combine(exchange: "CpExchange", epoch: int, batch: int, num_q_heads: int, num_kv_heads: int,
               out: Optional[torch.Tensor] = None, out_partial: Optional[torch.Tensor] = None,
               wait_timeout_s: float = 2.0, stream=None):
    """Phase 2 of paged_fog_decode_cp on its own: wait for every rank's
    shard results of `epoch` and merge them into out [B, Hq, D] and/or
    out_partial [B, Hq, D+2]."""
    t = out if out is not None else out_partial
    if t is None:
        raise ValueError("cp_combine needs out or out_partial")
    _need_cuda(t)
    D = out.shape[-1] if out is not None else out_partial.shape[-1] - 2
    if tuple(exchange.shape) != (batch, num_q_heads, num_kv_heads, D):
        raise ValueError(f"exchange buffers were sized for {tuple(exchange.shape)}, not "
                         f"{(batch, num_q_heads, num_kv_heads, D)}")
    for t_ in (out, out_partial):
        if t_ is not None and (not t_.is_contiguous() or t_.shape[:2] != (batch, num_q_heads)):
            raise ValueError("cp_combine outputs must be contiguous [B, Hq, ...]")
    dt = dtype_code(out) if out is not None else 1          # bf16 (unused: no out)
    _lib.check(_lib.load().kessie_cp_combine_v2(exchange.ptrs, exchange.rank, exchange.world, int(epoch),
                                                int(wait_timeout_s * 1e9), batch, num_q_heads, num_kv_heads, D, dt,
                                                _p(out), _p(out_partial), _stream(stream)), "cp_combine")
    return out


def lse_combine(partials: torch.Tensor, out: Optional[torch.Tensor] = None, out_dtype=torch.bfloat16,
                out_partial: Optional[torch.Tensor] = None, stream=None):
    """Merge partial triples [S, rows..., D+2] (fp32) into out [rows..., D]."""
    _need_cuda(partials)
    if partials.dtype != torch.float32 or not partials.is_contiguous():
        raise ValueError("partials must be contiguous fp32 [S, ..., D+2]")
    S = partials.shape[0]
    D = partials.shape[-1] - 2
    rows = partials[0].numel() // (D + 2)
    if out is None:
        out = torch.empty(*partials.shape[1:-1], D, dtype=out_dtype, device=partials.device)
    lib = _lib.load()
    _lib.check(lib.kessie_lse_combine_v2(partials.data_ptr(), S, partials.stride(0), rows, D, _p(out),
                                         dtype_code(out), _p(out_partial), _stream(stream)), "lse_combine")
    return out


# --------------------------------------------------------------------- prefill / dense
def fog_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, fog_weights: Optional[torch.Tensor] = None,
                  window_size: int = 0, causal: bool = True, sm_scale: Optional[float] = None,
                  out: Optional[torch.Tensor] = None, stream=None) -> torch.Tensor:
    """Dense fog attention: q [B, Hq, N, D], k/v [B, Hkv, N, D] (f16/bf16/f32,
    contiguous), fog_weights fp32 [N] or None (kessie_hip_kernels.py:367-440)."""
    _need_cuda(q, k, v, fog_weights)
    if not (q.is_contiguous() and k.is_contiguous() and v.is_contiguous()):
        raise ValueError("q, k, v must be contiguous [B, H, N, D]")
    B, Hq, N, D = q.shape
    Hkv = k.shape[1]
    if k.shape != (B, Hkv, N, D) or v.shape != k.shape:
        raise ValueError("k/v must be [B, Hkv, N, D] matching q")
    if sm_scale is None:
        sm_scale = 1.0 / math.sqrt(D)
    fw = None
    if fog_weights is not None:
        if fog_weights.numel() != N:
            raise ValueError("fog_weights must have N entries")
        fw = fog_weights.float().contiguous()
    if out is None:
        out = torch.empty_like(q)
    lib = _lib.load()
    _lib.check(lib.kessie_fog_attention_v2(q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), dtype_code(q),
                                           _p(fw), float(sm_scale), B, Hq, Hkv, N, D, int(window_size),
                                           1 if causal else 0, _stream(stream)), "fog_attention")
    return out


def paged_fog_prefill(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, block_table: torch.Tensor,
                      kv_lens, q_start=None, clear_start=None, fog_alpha: float = 0.5, fog_weights=None,
                      window_size: int = 0, causal: bool = True, sm_scale: Optional[float] = None,
                      out: Optional[torch.Tensor] = None, stream=None, staged: bool = True,
                      max_kv_len: Optional[int] = None, bias: Optional["FogBias"] = None) -> torch.Tensor:
    """Chunked prefill: q [B, T, Hq, D] (query t of sequence b at position
    q_start[b] + t, default kv_lens[b] - T) over k_cache / v_cache
    [P, ps, Hkv, D] views through block_table [B, maxP].  With staged=True the
    visible K/V are first gathered into a cached head-major workspace so the
    tensor-core kernel reads 128-token tiles (max_kv_len bounds kv_lens;
    default: the block table's capacity)."""
    _need_cuda(q, k_cache, v_cache, block_table)
    B, T, Hq, D = q.shape
    P, ps, Hkv, Dk = k_cache.shape
    if Dk != D or v_cache.shape != k_cache.shape or v_cache.stride() != k_cache.stride():
        raise ValueError("k_cache/v_cache must be matching [P, ps, Hkv, D] views")
    if q.stride(3) != 1 or k_cache.stride(3) != 1:
        raise ValueError("head_dim must be contiguous")
    bt = block_table if block_table.dtype == torch.int32 else block_table.to(torch.int32)
    if bt.stride(1) != 1:
        bt = bt.contiguous()
    kl = _i32(kv_lens, q.device)
    qs = _i32(q_start, q.device)
    cs = _i32(clear_start, q.device)
    fw = None
    fw_sb = 0
    if fog_weights is not None:
        fw = fog_weights.float().contiguous()
        fw_sb = fw.shape[-1] if fw.dim() == 2 else 0
    if sm_scale is None:
        sm_scale = 1.0 / math.sqrt(D)
    if out is None:
        out = torch.empty_like(q)
    lib = _lib.load()
    ws_ptr, ws_n, mkv = None, 0, 0
    if staged:
        mkv = int(max_kv_len) if max_kv_len is not None else bt.shape[1] * ps
        if mkv > bt.shape[1] * ps:
            raise ValueError(f"max_kv_len {mkv} exceeds the block table capacity {bt.shape[1] * ps}")
        ws_n = lib.kessie_paged_fog_prefill_workspace_size(B, Hkv, D, mkv)
        ws = workspace(ws_n, q.device, "prefill_stage")
        ws_ptr, ws_n = ws.data_ptr(), ws.numel()
    if bias is not None:
        cb = bias.c_struct()
        _lib.check(lib.kessie_paged_fog_prefill_biased_v2(
            q.data_ptr(), q.stride(0), q.stride(1), q.stride(2), k_cache.data_ptr(), v_cache.data_ptr(),
            k_cache.stride(0), k_cache.stride(1), k_cache.stride(2), P, ps, bt.data_ptr(), bt.stride(0), kl.data_ptr(),
            _p(qs), int(window_size), 1 if causal else 0, float(sm_scale), B, T, Hq, Hkv, D, dtype_code(q),
            ctypes.byref(cb), out.data_ptr(), out.stride(0), out.stride(1), out.stride(2), mkv, ws_ptr, ws_n,
            _stream(stream)), "paged_fog_prefill")
        return out
    _lib.check(lib.kessie_paged_fog_prefill_ex_v2(
        q.data_ptr(), q.stride(0), q.stride(1), q.stride(2), k_cache.data_ptr(), v_cache.data_ptr(),
        k_cache.stride(0), k_cache.stride(1), k_cache.stride(2), P, ps, bt.data_ptr(), bt.stride(0), kl.data_ptr(),
        _p(qs), _p(cs), float(fog_alpha), _p(fw), fw_sb, int(window_size), 1 if causal else 0, float(sm_scale),
        B, T, Hq, Hkv, D, dtype_code(q), out.data_ptr(), out.stride(0), out.stride(1), out.stride(2), mkv, ws_ptr,
        ws_n, _stream(stream)), "paged_fog_prefill")
    return out


# --------------------------------------------------------------------- conversation index
def index_query(query: torch.Tensor, index: torch.Tensor, top_k: int = 5, normalize_rows: bool = True,
                return_sims: bool = False, stream=None, out_ids: torch.Tensor = None, out_scores: torch.Tensor = None):
    """Cosine similarity of query [dim] against index [N, dim] (fp32, CUDA):
    (top ids int32 [k'], top scores fp32 [k'][, sims [N]]) with k' = min(top_k, N),
    descending, ties to the lower row index (kessie_hip_kernels.py:343-360; with
    normalize_rows=False the rows are taken as already normalised, as
    VectorIndex keeps them, kessie_exp3.py:69-81).  out_ids (int32) /
    out_scores (fp32), contiguous with at least top_k elements, receive the
    results instead of fresh tensors."""
    _need_cuda(query, index)
    if query.dtype != torch.float32 or index.dtype != torch.float32:
        raise TypeError("index_query: fp32 query and index")
    q = query.contiguous().view(-1)
    x = index.contiguous()
    N, dim = x.shape
    if q.numel() != dim:
        raise ValueError("query and index rows differ in length")
    if top_k > 32:
        raise ValueError("index_query: top_k <= 32")
    sims = torch.empty(N, dtype=torch.float32, device=x.device) if return_sims else None
    k = max(int(top_k), 0)
    ids, scores = out_ids, out_scores
    for t, dt, name in ((ids, torch.int32, "out_ids"), (scores, torch.float32, "out_scores")):
        if t is not None and (t.dtype != dt or not t.is_contiguous() or t.numel() < k or t.device != x.device):
            raise ValueError(f"index_query: {name} must be a contiguous {dt} tensor of >= top_k elements on "
                             f"the index's device")
    if ids is None:
        ids = torch.empty(max(k, 1), dtype=torch.int32, device=x.device)
    if scores is None:
        scores = torch.empty(max(k, 1), dtype=torch.float32, device=x.device)
    lib = _lib.load()
    ws = None
    if k > 0:
        ws = workspace(lib.kessie_index_query_workspace_size(N, k), x.device, "index_query")
    _lib.check(lib.kessie_index_query_v2(q.data_ptr(), x.data_ptr(), N, dim, 1 if normalize_rows else 0, _p(sims), k,
                                         ids.data_ptr() if k else None, scores.data_ptr() if k else None, _p(ws),
                                         ws.numel() if ws is not None else 0, _stream(stream)), "index_query")
    kk = min(k, N)
    out = (ids[:kk], scores[:kk])
    return out + (sims,) if return_sims else out


# --------------------------------------------------------------------- tiered cache
def tiered_update(k_store: torch.Tensor, v_store: torch.Tensor, lo: int, hi: int, k_new: torch.Tensor,
                  v_new: torch.Tensor, v_fog: Optional[torch.Tensor], fog_alpha: float, fog_start: float,
                  stream=None) -> bool:
    """KeSSieCache.update's device work (kessie_exp3.py:425-450) on a store
    pair [B, H, cap, D]: appends k_new / v_new [B, H, T, D] at [hi, hi + T)
    and, when the reference's fog mask exists for S = hi + T - lo, writes the
    fogged V of [lo, hi + T) into v_fog (>= B*H*S*D contiguous elements).
    Returns whether the fog was applied."""
    _need_cuda(k_store, v_store, k_new, v_new, v_fog)
    B, H, cap, D = k_store.shape
    T = k_new.shape[2]
    if v_store.shape != k_store.shape or k_new.shape != (B, H, T, D) or v_new.shape != k_new.shape:
        raise ValueError("tiered_update: store / new-token shapes differ")
    for t in (k_store, v_store, k_new, v_new):
        if t.dtype != k_store.dtype:
            raise TypeError("tiered_update: one dtype for stores and new tokens")
    if not (k_store.is_contiguous() and v_store.is_contiguous()):
        raise ValueError("tiered_update: stores must be contiguous [B, H, cap, D]")
    if k_new.stride() != v_new.stride() or k_new.stride(3) != 1:
        k_new, v_new = k_new.contiguous(), v_new.contiguous()
    S = hi + T - lo
    if v_fog is not None and (not v_fog.is_contiguous() or v_fog.numel() < B * H * S * D or v_fog.dtype != k_store.dtype):
        raise ValueError("tiered_update: v_fog must be contiguous with >= B*H*S*D elements of the store dtype")
    cc = max(1, int(S * fog_start))
    fog_on = fog_alpha > 0 and S > 0 and S - cc > 0
    _lib.check(_lib.load().kessie_tiered_update_v2(
        k_store.data_ptr(), v_store.data_ptr(), cap, int(lo), int(hi), k_new.data_ptr(), v_new.data_ptr(),
        k_new.stride(0), k_new.stride(1), k_new.stride(2), B, H, T, D, dtype_code(k_store),
        _p(v_fog) if fog_on else None, float(fog_alpha), float(fog_start), _stream(stream)), "tiered_update")
    return fog_on


def strided_pack(bases: torch.Tensor, pitch_bytes: torch.Tensor, rows_per_store: int, tokens: int, row_bytes: int,
                 staging: torch.Tensor, unpack: bool, stream=None):
    """Copy tokens of len(bases) strided stores to (unpack=False) or from
    (unpack=True) the contiguous staging [stores][rows][tokens][row_bytes]
    (kessie_exp3.py:452-533's per-layer slicing copies, in one launch).
    bases / pitch_bytes: int64 CUDA tensors (device address of each store's
    first copied token, bytes between its rows)."""
    _need_cuda(bases, pitch_bytes, staging)
    if bases.dtype != torch.int64 or pitch_bytes.dtype != torch.int64 or bases.numel() != pitch_bytes.numel():
        raise ValueError("strided_pack: int64 bases / pitch_bytes of one length")
    if staging.numel() * staging.element_size() < bases.numel() * rows_per_store * tokens * row_bytes:
        raise ValueError("strided_pack: staging too small")
    _lib.check(_lib.load().kessie_strided_pack_v2(bases.data_ptr(), pitch_bytes.data_ptr(), bases.numel(),
                                                   int(rows_per_store), int(tokens), int(row_bytes),
                                                   staging.data_ptr(), 1 if unpack else 0, _stream(stream)),
               "strided_pack")
