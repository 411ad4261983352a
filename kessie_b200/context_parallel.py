"""Context-parallel fog decode: the KV sequence is sharded across ranks.

Each rank holds a contiguous position range of every sequence's pages
(rank r of G: positions [r*N/G, (r+1)*N/G), page aligned).  A step is:

  1. the decode kernel over the local shard (fog weights at GLOBAL
     positions).  The CTA that completes a (seq, kv_head) group merges the
     group's split partials and stores the shard result -- fp32 (O/l, m, l)
     per query head -- straight into every rank's exchange buffer over
     NVLink (CUDA IPC mappings, plain peer stores).  Each value travels with
     the step's epoch in one 8-byte word, so no fence or flag is needed and
     the decode never waits on the remote stores                [CUDA]
  2. a combine kernel, launched as a programmatic dependent of the decode,
     that polls (bounded) its OWN exchange buffer until every rank's words
     of a row carry the epoch, then log-sum-exp merges the G shard results
     -> O                                                        [CUDA]

So a step is two kernel launches per rank and no collective-library call.
``exchange="nccl"`` keeps the collective form (decode -> NCCL all-gather of
[B, Hq, D+2] -> LSE merge kernel) for process groups without peer access.

The reference has no context parallelism (long context there is fog +
window truncation + CPU offload); this module is new and is the only
multi-GPU path of the library.
"""

from __future__ import annotations

from typing import Optional

import torch
import torch.distributed as dist

from . import ops


def shard_range(seq_len: int, rank: int, world: int, page_size: int = 16):
    """[start, end) positions owned by `rank`; shard boundaries are page-aligned."""
    pages = (seq_len + page_size - 1) // page_size
    per = (pages + world - 1) // world
    start = min(rank * per * page_size, seq_len)
    end = min((rank + 1) * per * page_size, seq_len)
    return start, end


class ContextParallelFogDecode:
    """Decode over a KV cache sharded by position across a process group.

    ``__call__(q, k_cache, v_cache, block_table, local_lens, kv_pos_offset,
    q_positions, clear_start)`` with this rank's shard (local block table /
    lengths, global offsets) returns the merged output on every rank.
    With a world size of 1 it is a plain paged fog decode.  Every rank must
    make the same calls in the same order (like a collective)."""

    def __init__(self, batch: int, num_q_heads: int, head_dim: int, dtype=torch.bfloat16, device=None,
                 group: Optional[dist.ProcessGroup] = None, num_kv_heads: Optional[int] = None,
                 exchange: str = "p2p", wait_timeout_s: float = 2.0):
        self.group = group
        inited = dist.is_available() and dist.is_initialized()
        self.world = dist.get_world_size(group) if inited else 1
        self.rank = dist.get_rank(group) if inited else 0
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        if exchange not in ("p2p", "nccl"):
            raise ValueError("exchange must be 'p2p' or 'nccl'")
        self.exchange_kind = exchange if self.world > 1 else "none"
        self.batch, self.num_q_heads, self.head_dim = batch, num_q_heads, head_dim
        self.num_kv_heads = num_kv_heads
        self.wait_timeout_s = wait_timeout_s
        D = head_dim
        self.out = torch.empty(batch, num_q_heads, D, dtype=dtype, device=self.device)
        self.partial = None
        self.gathered = None
        if self.exchange_kind == "nccl":
            self.partial = torch.empty(batch, num_q_heads, D + 2, dtype=torch.float32, device=self.device)
            self.gathered = torch.empty(self.world, batch, num_q_heads, D + 2, dtype=torch.float32, device=self.device)
        self.xch: Optional[ops.CpExchange] = None
        self._epoch = 0
        self.dtype = dtype

    # ------------------------------------------------------------------ set-up
    def _exchange(self, num_kv_heads: int) -> ops.CpExchange:
        if self.xch is None:
            if self.num_kv_heads is not None and self.num_kv_heads != num_kv_heads:
                raise ValueError("num_kv_heads differs from the constructor's")
            self.num_kv_heads = num_kv_heads
            self.xch = ops.CpExchange(self.world, self.rank, self.batch, self.num_q_heads, num_kv_heads,
                                      self.head_dim, self.device, self.group)
        return self.xch

    def close(self):
        """Release the exchange buffers (collective: every rank calls it after
        its last step; includes a barrier so no rank unmaps memory that a
        slower rank still writes)."""
        if self.xch is not None:
            torch.cuda.synchronize(self.device)
            dist.barrier(group=self.group)
            self.xch.close()
            self.xch = None

    # ------------------------------------------------------------------ step
    def local(self, q, k_cache, v_cache, block_table, local_lens, kv_pos_offset=None, q_positions=None,
              clear_start=None, fog_alpha: float = 0.5, window_size: int = 0, sm_scale=None, max_seq_len=None,
              stream=None):
        """Step 1 (the dominant kernel): decode the local shard and publish
        its result (p2p: into every rank's exchange buffer; nccl: into the
        local triple buffer)."""
        common = dict(clear_start=clear_start, fog_alpha=fog_alpha, window_size=window_size, sm_scale=sm_scale,
                      kv_pos_offset=kv_pos_offset, q_positions=q_positions, max_seq_len=max_seq_len, stream=stream)
        if self.exchange_kind == "none":
            ops.paged_fog_decode(q, k_cache, v_cache, block_table, local_lens, out=self.out, **common)
        elif self.exchange_kind == "nccl":
            ops.paged_fog_decode(q, k_cache, v_cache, block_table, local_lens, out_partial=self.partial,
                                 want_out=False, **common)
        else:
            xch = self._exchange(k_cache.shape[2])
            self._epoch = xch.next_epoch()
            ops.paged_fog_decode_cp(xch, self._epoch, q, k_cache, v_cache, block_table, local_lens,
                                    wait_timeout_s=self.wait_timeout_s, phases=1, **common)

    def merge(self, stream=None):
        """Step 2: combine the shard results of all ranks into self.out."""
        if self.exchange_kind == "none":
            return self.out
        if self.exchange_kind == "nccl":
            flat = self.gathered.view(-1, *self.partial.shape[1:])     # concatenated form (every backend)
            dist.all_gather_into_tensor(flat, self.partial, group=self.group)
            ops.lse_combine(self.gathered, out=self.out, stream=stream)
            return self.out
        self._merge_p2p(stream)
        return self.out

    def _merge_p2p(self, stream):
        B, Hq, _ = self.out.shape
        ops.cp_combine(self.xch, self._epoch, B, Hq, self.num_kv_heads, out=self.out,
                       wait_timeout_s=self.wait_timeout_s, stream=stream)

    def __call__(self, q, k_cache, v_cache, block_table, local_lens, kv_pos_offset=None, q_positions=None,
                 clear_start=None, fog_alpha: float = 0.5, window_size: int = 0, sm_scale=None, max_seq_len=None,
                 stream=None):
        if self.world > 1 and kv_pos_offset is None:
            raise ValueError("context-parallel decode needs kv_pos_offset (global position of each shard)")
        if self.exchange_kind == "p2p":
            xch = self._exchange(k_cache.shape[2])
            self._epoch = xch.next_epoch()
            ops.paged_fog_decode_cp(xch, self._epoch, q, k_cache, v_cache, block_table, local_lens,
                                    clear_start=clear_start, fog_alpha=fog_alpha, window_size=window_size,
                                    sm_scale=sm_scale, kv_pos_offset=kv_pos_offset, q_positions=q_positions,
                                    max_seq_len=max_seq_len, out=self.out, wait_timeout_s=self.wait_timeout_s,
                                    phases=3, stream=stream)
            return self.out
        self.local(q, k_cache, v_cache, block_table, local_lens, kv_pos_offset, q_positions, clear_start, fog_alpha,
                   window_size, sm_scale, max_seq_len, stream)
        return self.merge(stream)
