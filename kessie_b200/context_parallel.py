"""Context-parallel fog decode: the KV sequence is sharded across ranks.

Each rank holds a contiguous position range of every sequence's pages
(rank r of G: positions [r*N/G, (r+1)*N/G)).  A step is:

  1. local split-KV fog decode over the shard (fog weights at GLOBAL
     positions) -> fp32 triple (O/l, m, l) per (seq, q_head)  [CUDA]
  2. all-gather of the [B, Hq, D+2] triples over NCCL (NVLink/NVSwitch;
     133 KB per rank at the 70B shape)
  3. log-sum-exp merge of the G triples -> O                  [CUDA]

Fog scales V only, so the merge is the plain LSE combine.  The reference has
no context parallelism (long context there is fog + window truncation + CPU
offload); this module is new and is the only multi-GPU path of the library.
"""

from __future__ import annotations

from dataclasses import dataclass
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


@dataclass
class CPDecodeState:
    """Per-rank buffers reused by every step (no allocation in steady state)."""
    partial: torch.Tensor        # [B, Hq, D+2] fp32, this rank's triple
    gathered: torch.Tensor       # [G, B, Hq, D+2] fp32
    out: torch.Tensor            # [B, Hq, D]


class ContextParallelFogDecode:
    """Decode over a KV cache sharded by position across a process group.

    ``__call__(q, k_cache, v_cache, block_table, local_lens, kv_pos_offset,
    q_positions, clear_start)`` with this rank's shard (local block table /
    lengths, global offsets) returns the merged output on every rank.
    With a world size of 1 it is a plain paged fog decode."""

    def __init__(self, batch: int, num_q_heads: int, head_dim: int, dtype=torch.bfloat16, device=None,
                 group: Optional[dist.ProcessGroup] = None):
        self.group = group
        self.world = dist.get_world_size(group) if (dist.is_available() and dist.is_initialized()) else 1
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        D = head_dim
        self.state = CPDecodeState(
            partial=torch.empty(batch, num_q_heads, D + 2, dtype=torch.float32, device=self.device),
            gathered=torch.empty(self.world, batch, num_q_heads, D + 2, dtype=torch.float32, device=self.device),
            out=torch.empty(batch, num_q_heads, D, dtype=dtype, device=self.device))
        self.dtype = dtype

    def local(self, q, k_cache, v_cache, block_table, local_lens, kv_pos_offset=None, q_positions=None,
              clear_start=None, fog_alpha: float = 0.5, window_size: int = 0, sm_scale=None, max_seq_len=None,
              phases: int = 3, stream=None):
        """Step 1 only (the dominant kernel); returns the local triple buffer."""
        if self.world == 1:
            ops.paged_fog_decode(q, k_cache, v_cache, block_table, local_lens, clear_start=clear_start,
                                 fog_alpha=fog_alpha, window_size=window_size, sm_scale=sm_scale,
                                 kv_pos_offset=kv_pos_offset, q_positions=q_positions, max_seq_len=max_seq_len,
                                 out=self.state.out, phases=phases, stream=stream)
            return None
        ops.paged_fog_decode(q, k_cache, v_cache, block_table, local_lens, clear_start=clear_start,
                             fog_alpha=fog_alpha, window_size=window_size, sm_scale=sm_scale,
                             kv_pos_offset=kv_pos_offset, q_positions=q_positions, max_seq_len=max_seq_len,
                             out_partial=self.state.partial, want_out=False, phases=phases, stream=stream)
        return self.state.partial

    def merge(self):
        """Steps 2-3: NCCL all-gather of the triples, then the LSE merge."""
        if self.world == 1:
            return self.state.out
        # concatenated-along-dim-0 output form (accepted by every backend)
        flat = self.state.gathered.view(-1, *self.state.partial.shape[1:])
        dist.all_gather_into_tensor(flat, self.state.partial, group=self.group)
        ops.lse_combine(self.state.gathered, out=self.state.out)
        return self.state.out

    def __call__(self, q, k_cache, v_cache, block_table, local_lens, kv_pos_offset=None, q_positions=None,
                 clear_start=None, fog_alpha: float = 0.5, window_size: int = 0, sm_scale=None, max_seq_len=None):
        if self.world > 1 and kv_pos_offset is None:
            raise ValueError("context-parallel decode needs kv_pos_offset (global position of each shard)")
        self.local(q, k_cache, v_cache, block_table, local_lens, kv_pos_offset, q_positions, clear_start, fog_alpha,
                   window_size, sm_scale, max_seq_len)
        return self.merge()

