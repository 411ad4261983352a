"""GPU-resident drop-in for the conversation index ``VectorIndex``
(kessie_exp3.py:58-110): same constructor, ``rebuild``, ``search`` and
``count``; the normalised index matrix lives in HBM and ``search`` is one
index-query call (cosine similarity + device top-k,
``kessie_index_query_v2``) instead of a CPU matrix-vector product and a
full argsort.

Semantics kept from the reference:
* ``rebuild`` stores each row divided by its L2 norm, a norm below 1e-8
  replaced by 1 (kessie_exp3.py:69-76) -- computed on the host with the same
  numpy expression, so the stored rows are the reference's;
* ``search`` divides the query by its norm and returns [] for a norm below
  1e-8 or an empty index (kessie_exp3.py:89-95); k = min(top_k, count);
  results are ``(id, score)`` best first.
Ties: equal scores come back lower row first (the reference's numpy path
orders ties by argsort's unstable quicksort, so no tie order is defined
there).  ``top_k`` above the kernel's list length (32) takes the kernel's
similarity output and a stable device sort, which keeps the same order.
"""

from __future__ import annotations

import threading
from typing import List, Optional, Tuple

import numpy as np
import torch

from . import ops

_MAX_DEVICE_K = 32


class VectorIndex:
    """CPU-bound cosine similarity in the reference; here the rows sit in HBM."""

    def __init__(self, dim: int = 256, device: Optional[torch.device] = None):
        self.dim = dim
        self._lock = threading.RLock()
        self._vectors: List[np.ndarray] = []
        self._ids: List[int] = []
        self._mat: Optional[torch.Tensor] = None            # [n, dim] fp32, rows normalised
        self._device = torch.device(device) if device is not None else None
        self._bufs = None                                   # pinned / device query and result buffers

    def _dev(self) -> torch.device:
        if self._device is None:
            if not torch.cuda.is_available():
                raise RuntimeError("VectorIndex: the GPU index needs a CUDA device")
            self._device = torch.device("cuda", torch.cuda.current_device())
        return self._device

    def rebuild(self, vectors: List[np.ndarray], ids: List[int]):
        if not vectors:
            with self._lock:
                self._vectors, self._ids, self._mat = [], [], None
            return
        mat = np.stack([v.astype(np.float32) for v in vectors])
        norms = np.linalg.norm(mat, axis=1, keepdims=True)
        norms[norms < 1e-8] = 1.0
        mat_normed = np.ascontiguousarray(mat / norms, dtype=np.float32)
        dev_mat = torch.from_numpy(mat_normed).to(self._dev())
        with self._lock:
            self._vectors = [v.astype(np.float32) for v in vectors]
            self._ids = list(ids)
            self._mat = dev_mat

    def search(self, query: np.ndarray, top_k: int = 5) -> List[Tuple[int, float]]:
        q = np.asarray(query).astype(np.float32).reshape(-1)
        qn = np.linalg.norm(q.reshape(1, -1))
        if qn < 1e-8:
            return []
        q = q / qn
        with self._lock:
            if not self._ids or self._mat is None:
                return []
            k = min(int(top_k), len(self._ids))
            if k <= 0:
                return []
            if k <= _MAX_DEVICE_K:
                idx, scores = self._search_small(q, k)
            else:
                qd = torch.from_numpy(np.ascontiguousarray(q, dtype=np.float32)).to(self._mat.device)
                sims = ops.index_query(qd, self._mat, top_k=0, normalize_rows=False, return_sims=True)[2]
                scores, idx = torch.sort(sims, descending=True, stable=True)
                idx, scores = idx[:k], scores[:k]
                idx = idx.cpu().numpy()
                scores = scores.cpu().numpy()
            return [(self._ids[int(i)], float(s)) for i, s in zip(idx, scores) if 0 <= int(i) < len(self._ids)]

    def _search_small(self, q: np.ndarray, k: int):
        """One query upload from pinned memory, the index-query launches, one
        download of ids and scores packed in a [2, 32] int32 buffer."""
        dev = self._mat.device
        if self._bufs is None or self._bufs[1].device != dev:
            self._bufs = (torch.empty(self.dim, dtype=torch.float32).pin_memory(),
                          torch.empty(self.dim, dtype=torch.float32, device=dev),
                          torch.empty(2, _MAX_DEVICE_K, dtype=torch.int32, device=dev),
                          torch.empty(2, _MAX_DEVICE_K, dtype=torch.int32).pin_memory())
        qh, qd, rd, rh = self._bufs
        qh.numpy()[:] = q
        qd.copy_(qh, non_blocking=True)
        ops.index_query(qd, self._mat, top_k=k, normalize_rows=False, out_ids=rd[0], out_scores=rd[1].view(torch.float32))
        rh.copy_(rd, non_blocking=True)
        torch.cuda.current_stream(dev).synchronize()
        return rh[0, :k].numpy().copy(), rh[1].view(torch.float32)[:k].numpy().copy()

    @property
    def count(self):
        with self._lock:
            return len(self._ids)
