"""Drop-in for the reference's ``kessie_kv_connector`` module (vLLM V1 KV
connector + CPU KV block store), with the block copies moved onto the
library's kernels.

Same names, signatures and bookkeeping as kessie_kv_connector.py:
``KVBlock``, ``KeSSieCPUKVStore``, ``get_kessie_store``, ``RecallState`` and
``KeSSieKVConnector`` with ``register_kv_caches``,
``get_num_new_matched_tokens``, ``update_state_after_alloc``,
``start_load_kv``, ``wait_for_layer_load``, ``save_kv_layer``,
``wait_for_save``, ``request_finished``, ``build_connector_meta``
(kessie_kv_connector.py:51-508).

What changes is the data path (kessie_kv_connector.py:388-491):

* save: the reference walks every (sequence, block) with a device sync
  per ``.item()`` and one ``.cpu().clone()`` per block.  Here the block
  tables and lengths come to the host once, ONE gather kernel packs every
  saved block of the layer into a device staging buffer
  [2][n][block_size][H][D], and ONE asynchronous copy moves it to pinned
  host memory; each stored ``KVBlock.kv_data`` is a [2, tokens, H, D] view
  of that host buffer (the same tensor the reference stores).
* load: the recalled blocks of a layer are packed into one pinned host
  buffer, copied with ONE asynchronous host-to-device copy and written into
  their block slots by ONE scatter kernel, on a side stream that
  ``wait_for_layer_load`` synchronises.  The reference's
  ``gpu_cache[block.block_id].copy_(...)`` (kessie_kv_connector.py:441)
  indexes the K/V dimension of vLLM's [2, num_blocks, block_size, H, D]
  cache; the load here writes ``cache[:, block_id, :tokens]``, the slot the
  block was saved from, as the surrounding comments intend.

The semantic index (cosine top-k over stored embeddings) keeps the
reference's per-entry evaluation; it is host-side bookkeeping, not part of
the GPU path.
"""

from __future__ import annotations

import hashlib
import logging
import threading
import time
from collections import defaultdict
from dataclasses import dataclass, field
from typing import Any, Dict, List, Optional, Set, Tuple

import numpy as np
import torch

from . import ops

logger = logging.getLogger("KeSSie.KVConnector")


# ----------------------------------------------------------------- CPU block store
@dataclass
class KVBlock:
    """A single KV cache block stored in CPU RAM (kessie_kv_connector.py:51-62)."""
    layer_name: str
    block_id: int
    token_ids: List[int]
    kv_data: Any
    position_start: int
    position_end: int
    timestamp: float = 0.0
    embedding: Optional[np.ndarray] = None


def _nbytes(t) -> int:
    return t.nelement() * t.element_size() if hasattr(t, "nelement") else 0


class KeSSieCPUKVStore:
    """CPU-side KV block store with a position index, a byte budget (oldest
    block evicted first) and a semantic index (kessie_kv_connector.py:65-229)."""

    def __init__(self, max_cpu_bytes: int = 0, embed_dim: int = 256):
        self._lock = threading.Lock()
        self._blocks: Dict[Tuple[str, int], KVBlock] = {}
        self._position_index: Dict[int, List[Tuple[str, int]]] = defaultdict(list)
        self._semantic_index: List[Tuple[np.ndarray, int, int, List[int]]] = []
        self.embed_dim = embed_dim
        self.max_cpu_bytes = max_cpu_bytes
        self.total_bytes = 0
        self._embedder = None
        self.conversation_tokens: List[int] = []

    def set_embedder(self, fn):
        self._embedder = fn

    def save_block(self, layer_name: str, block_id: int, kv_data, token_ids: List[int], position_start: int):
        """Store one block; a tensor argument is copied to the host
        (kessie_kv_connector.py:93-132)."""
        cpu_data = kv_data.detach().cpu().clone() if hasattr(kv_data, "cpu") else kv_data
        self._put(layer_name, block_id, cpu_data, token_ids, position_start)

    def _put(self, layer_name, block_id, cpu_data, token_ids, position_start, timestamp=None):
        """Insert an already host-resident block (no copy).  Same accounting
        as save_block: evict oldest while over budget, replace a block with
        the same (layer, block_id) key, append to the position index."""
        with self._lock:
            key = (layer_name, block_id)
            block = KVBlock(layer_name=layer_name, block_id=block_id, token_ids=list(token_ids), kv_data=cpu_data,
                            position_start=position_start, position_end=position_start + len(token_ids),
                            timestamp=time.time() if timestamp is None else timestamp)
            block_bytes = _nbytes(cpu_data)
            if self.max_cpu_bytes > 0:
                while self.total_bytes + block_bytes > self.max_cpu_bytes and self._blocks:
                    self._evict_oldest()
            old = self._blocks.get(key)
            if old is not None and hasattr(old.kv_data, "nelement"):
                self.total_bytes -= _nbytes(old.kv_data)
            self._blocks[key] = block
            self._position_index[position_start].append(key)
            self.total_bytes += block_bytes

    def save_semantic_entry(self, token_ids: List[int], position_start: int, tokenizer=None):
        if self._embedder is None or tokenizer is None:
            return
        text = tokenizer.decode(token_ids, skip_special_tokens=True)
        if not text.strip():
            return
        emb = self._embedder(text)
        if emb is not None:
            with self._lock:
                self._semantic_index.append((emb, position_start, position_start + len(token_ids), list(token_ids)))

    def semantic_search(self, query_text: str, top_k: int = 5,
                        exclude_positions: Optional[Set[int]] = None) -> List[Tuple[int, int, float]]:
        """[(position_start, position_end, cosine similarity)] best first
        (kessie_kv_connector.py:148-177; ties keep insertion order)."""
        if self._embedder is None or not self._semantic_index:
            return []
        q = self._embedder(query_text)
        if q is None:
            return []
        exclude = exclude_positions or set()
        results = []
        with self._lock:
            for emb, pos_start, pos_end, _ in self._semantic_index:
                if pos_start in exclude:
                    continue
                sim = np.dot(q, emb) / max(np.linalg.norm(q) * np.linalg.norm(emb), 1e-8)
                results.append((pos_start, pos_end, float(sim)))
        results.sort(key=lambda x: -x[2])
        return results[:top_k]

    def get_blocks_for_positions(self, position_start: int, position_end: int, layer_name: str) -> Optional[KVBlock]:
        with self._lock:
            for key in self._position_index.get(position_start, []):
                if key[0] == layer_name and key in self._blocks:
                    block = self._blocks[key]
                    if block.position_start == position_start:
                        return block
        return None

    def get_all_blocks_for_range(self, position_start: int, position_end: int) -> Dict[str, List[KVBlock]]:
        result: Dict[str, List[KVBlock]] = defaultdict(list)
        with self._lock:
            for pos in range(position_start, position_end):
                for key in self._position_index.get(pos, []):
                    if key in self._blocks:
                        block = self._blocks[key]
                        result[block.layer_name].append(block)
        return dict(result)

    def _evict_oldest(self):
        if not self._blocks:
            return
        oldest_key = min(self._blocks.keys(), key=lambda k: self._blocks[k].timestamp)
        block = self._blocks.pop(oldest_key)
        if hasattr(block.kv_data, "nelement"):
            self.total_bytes -= _nbytes(block.kv_data)
        pos_keys = self._position_index.get(block.position_start, [])
        if oldest_key in pos_keys:
            pos_keys.remove(oldest_key)

    def stats(self) -> Dict[str, Any]:
        with self._lock:
            return {"total_blocks": len(self._blocks), "total_bytes": self.total_bytes,
                    "total_mb": self.total_bytes / 1048576, "semantic_entries": len(self._semantic_index),
                    "conversation_tokens": len(self.conversation_tokens),
                    "position_ranges": len(self._position_index)}


_KESSIE_STORE: Optional[KeSSieCPUKVStore] = None
_KESSIE_STORE_LOCK = threading.Lock()


def get_kessie_store(max_cpu_bytes: int = 0) -> KeSSieCPUKVStore:
    """Process-wide store shared by connector instances (kessie_kv_connector.py:234-242)."""
    global _KESSIE_STORE
    with _KESSIE_STORE_LOCK:
        if _KESSIE_STORE is None:
            _KESSIE_STORE = KeSSieCPUKVStore(max_cpu_bytes=max_cpu_bytes)
        return _KESSIE_STORE


@dataclass
class RecallState:
    """Distant KV ranges to load for a request (kessie_kv_connector.py:246-252)."""
    request_id: str = ""
    recalled_positions: List[Tuple[int, int]] = field(default_factory=list)
    num_recalled_tokens: int = 0
    load_pending: bool = False


_RECALL_STATES: Dict[str, RecallState] = {}
_RECALL_LOCK = threading.Lock()


# ----------------------------------------------------------------- batched block copies
def save_blocks(kv_layer: torch.Tensor, block_ids: torch.Tensor, stream=None,
                out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Gather blocks ``block_ids`` of a vLLM-layout layer cache
    [2, num_blocks, block_size, H, D] into pinned host memory
    [2, n, block_size, H, D]: one gather kernel into a device staging buffer,
    then one asynchronous device-to-host copy, both on ``stream``.  The host
    tensor is valid after the stream is synchronised."""
    two, nb, bs, H, D = kv_layer.shape
    n = int(block_ids.numel())
    dev = kv_layer.device
    if out is None:
        out = torch.empty(2, n, bs, H, D, dtype=kv_layer.dtype, pin_memory=True)
    if n == 0:
        return out
    s = stream or torch.cuda.current_stream(dev)
    with torch.cuda.stream(s):
        # staging allocated on `s`: the caching allocator keeps it for `s`'s work
        st = torch.empty(2, n, bs, H, D, dtype=kv_layer.dtype, device=dev)
        ops.page_gather(kv_layer, block_ids, layout="vllm", out_keys=st[0].view(n * bs, H, D),
                        out_values=st[1].view(n * bs, H, D), stream=s)
        out.copy_(st, non_blocking=True)
    return out


def load_blocks(kv_layer: torch.Tensor, host_kv: torch.Tensor, block_ids: torch.Tensor, stream=None):
    """Write host blocks [2, n, block_size, H, D] (pinned) into block slots
    ``block_ids`` of a vLLM-layout layer cache: one asynchronous
    host-to-device copy into a device staging buffer, then one scatter
    kernel, both on ``stream``."""
    two, n, bs, H, D = host_kv.shape
    if n == 0:
        return
    dev = kv_layer.device
    s = stream or torch.cuda.current_stream(dev)
    with torch.cuda.stream(s):
        st = torch.empty(2, n, bs, H, D, dtype=host_kv.dtype, device=dev)
        st.copy_(host_kv, non_blocking=True)
        ops.page_insert(kv_layer, st[0].view(n * bs, H, D), st[1].view(n * bs, H, D), block_ids, layout="vllm",
                        stream=s)


# ----------------------------------------------------------------- the connector
try:                                                       # vLLM's V1 connector base, when installed
    from vllm.distributed.kv_transfer.kv_connector.v1.base import KVConnectorBase_V1 as _ConnectorBase
    HAS_VLLM_CONNECTOR = True
except Exception:                                          # pragma: no cover - depends on the vLLM build
    try:
        from vllm.distributed.kv_transfer.kv_connector.v1.base import KVConnectorBase_v1 as _ConnectorBase
        HAS_VLLM_CONNECTOR = True
    except Exception:
        _ConnectorBase = object
        HAS_VLLM_CONNECTOR = False


class KeSSieKVConnector(_ConnectorBase):
    """KV connector: saves every computed block to the CPU store and loads
    semantically recalled blocks back into vLLM's paged cache
    (kessie_kv_connector.py:277-508), with batched copies."""

    def __init__(self, *args, **kwargs):
        if _ConnectorBase is not object and (args or kwargs.get("vllm_config") is not None):
            super().__init__(*args, **{k: v for k, v in kwargs.items() if k != "kv_connector_extra_config"})
        extra = kwargs.get("kv_connector_extra_config", {}) or {}
        max_gb = float(extra.get("max_cpu_gb", 64))
        self.store = get_kessie_store(max_cpu_bytes=int(max_gb * 1073741824))
        self._kv_caches = []
        self._layer_names = []
        self._block_size = 16
        self._copy_streams: Dict[int, torch.cuda.Stream] = {}

    def register_kv_caches(self, kv_caches, layer_names=None, **kwargs):
        """References to vLLM's per-layer caches [2, num_blocks, block_size, H, D]."""
        if isinstance(kv_caches, dict):                   # vLLM passes {layer_name: tensor}
            layer_names = list(kv_caches.keys()) if layer_names is None else layer_names
            kv_caches = [kv_caches[n] for n in layer_names]
        self._kv_caches = list(kv_caches)
        self._layer_names = list(layer_names or [])
        if self._kv_caches and hasattr(self._kv_caches[0], "shape"):
            self._block_size = self._kv_caches[0].shape[2] if self._kv_caches[0].dim() >= 4 else 16

    def get_num_new_matched_tokens(self, request, *args, **kwargs) -> int:
        """Tokens the semantic index can supply for this request (kessie_kv_connector.py:314-381)."""
        token_ids = list(request.prompt_token_ids) if hasattr(request, "prompt_token_ids") else []
        if not token_ids:
            return 0
        req_id = str(request.request_id) if hasattr(request, "request_id") else ""
        with _RECALL_LOCK:
            if req_id in _RECALL_STATES:
                return _RECALL_STATES[req_id].num_recalled_tokens
        # the reference hashes bytes(last 128 ids) (kessie_kv_connector.py:337-343), which raises for ids
        # above 255; ids are folded to bytes here so real vocabularies work (same hash when all ids < 256)
        query_text = f"tokens:{hashlib.md5(bytes(t % 256 for t in token_ids[-128:])).hexdigest()}"
        results = self.store.semantic_search(query_text, top_k=3, exclude_positions=set())
        if not results:
            return 0
        recalled, total = [], 0
        for pos_start, pos_end, sim in results:
            if sim < 0.3:
                continue
            recalled.append((pos_start, pos_end))
            total += pos_end - pos_start
        if total > 0:
            with _RECALL_LOCK:
                _RECALL_STATES[req_id] = RecallState(request_id=req_id, recalled_positions=recalled,
                                                     num_recalled_tokens=total, load_pending=True)
        return total

    def update_state_after_alloc(self, request, blocks, num_external_tokens, **kwargs):
        req_id = str(request.request_id) if hasattr(request, "request_id") else ""
        with _RECALL_LOCK:
            state = _RECALL_STATES.get(req_id)
            if state and num_external_tokens > 0:
                state.load_pending = True

    def start_load_kv(self, kv_caches=None, layer_names=None, **kwargs):
        """Load every pending recalled block into its slot: per layer one
        host pack, one host-to-device copy and one scatter kernel on the copy
        stream (kessie_kv_connector.py:388-447)."""
        kv_caches = self._kv_caches if kv_caches is None else kv_caches
        layer_names = self._layer_names if layer_names is None else layer_names
        if isinstance(kv_caches, dict):
            kv_caches = [kv_caches[n] for n in layer_names]
        with _RECALL_LOCK:
            pending = {k: v for k, v in _RECALL_STATES.items() if v.load_pending}
        if not pending:
            return
        for i, layer_name in enumerate(layer_names):
            if i >= len(kv_caches):
                break
            blocks = []
            for state in pending.values():
                for pos_start, pos_end in state.recalled_positions:
                    b = self.store.get_blocks_for_positions(pos_start, pos_end, layer_name)
                    if b is not None and hasattr(b.kv_data, "shape"):
                        blocks.append(b)
            if blocks:
                self._load_layer(kv_caches[i], blocks)
        with _RECALL_LOCK:
            for state in pending.values():
                state.load_pending = False

    def _load_layer(self, cache: torch.Tensor, blocks: List[KVBlock]):
        two, nb, bs, H, D = cache.shape
        host = torch.zeros(2, len(blocks), bs, H, D, dtype=cache.dtype, pin_memory=True)
        for j, b in enumerate(blocks):                     # host-side pack of [2, tokens, H, D] blocks
            t = b.kv_data.shape[1]
            host[:, j, :t].copy_(b.kv_data)
        stream = self._get_copy_stream(cache.device)
        stream.wait_stream(torch.cuda.current_stream(cache.device))
        with torch.cuda.stream(stream):
            ids = torch.tensor([b.block_id for b in blocks], dtype=torch.int32).to(cache.device)
        load_blocks(cache, host, ids, stream=stream)
        # keep the pinned buffer alive until the copy stream has consumed it
        self._inflight = getattr(self, "_inflight", [])
        self._inflight.append(host)

    def wait_for_layer_load(self, layer_name: str, **kwargs):
        for stream in self._copy_streams.values():
            stream.synchronize()
        self._inflight = []

    def save_kv_layer(self, layer_name: str, kv_layer, attn_metadata, **kwargs):
        """Save every block of every sequence in the batch: one gather kernel
        and one device-to-host copy per layer (kessie_kv_connector.py:453-491).
        Blocks are keyed (layer_name, block_id) with position_start = block
        index * block_size, as in the reference."""
        block_tables = getattr(attn_metadata, "block_tables", None)
        if block_tables is None:
            block_tables = getattr(attn_metadata, "block_table", None)
        seq_lens = getattr(attn_metadata, "seq_lens", None)
        if block_tables is None or seq_lens is None or kv_layer is None or not hasattr(block_tables, "shape"):
            return
        bs = self._block_size
        bt = block_tables.detach().cpu() if torch.is_tensor(block_tables) else torch.as_tensor(block_tables)
        sl = (seq_lens.detach().cpu() if torch.is_tensor(seq_lens) else torch.as_tensor(seq_lens)).tolist()
        ids, meta = [], []
        for seq_idx in range(min(len(sl), bt.shape[0])):
            n_blocks = (int(sl[seq_idx]) + bs - 1) // bs
            row = bt[seq_idx, :n_blocks].tolist()
            for b, block_id in enumerate(row):
                pos_start = b * bs
                meta.append((int(block_id), pos_start, min(bs, int(sl[seq_idx]) - pos_start)))
                ids.append(int(block_id))
        if not ids:
            return
        stream = self._get_copy_stream(kv_layer.device)
        stream.wait_stream(torch.cuda.current_stream(kv_layer.device))    # the layer's KV is written
        with torch.cuda.stream(stream):
            id_t = torch.tensor(ids, dtype=torch.int32).to(kv_layer.device)
        host = save_blocks(kv_layer, id_t, stream=stream)
        for j, (block_id, pos_start, ntok) in enumerate(meta):
            self.store._put(layer_name, block_id, host[:, j, :ntok], [], pos_start)

    def wait_for_save(self, **kwargs):
        for stream in self._copy_streams.values():
            stream.synchronize()

    def request_finished(self, request, block_ids, **kwargs):
        req_id = str(request.request_id) if hasattr(request, "request_id") else ""
        with _RECALL_LOCK:
            _RECALL_STATES.pop(req_id, None)
        return (False, None)

    def build_connector_meta(self, scheduler_output, **kwargs):
        return None

    def _get_copy_stream(self, device) -> torch.cuda.Stream:
        idx = device.index if getattr(device, "index", None) is not None else torch.cuda.current_device()
        if idx not in self._copy_streams:
            self._copy_streams[idx] = torch.cuda.Stream(device=device)
        return self._copy_streams[idx]
