"""Sequence-parallel state used by the attention path.

Mirrors the names the reference's hot path reads from
``hymm.utils.parallel_states`` (``nccl_info`` at parallel_states.py:149 with
``sp_group`` / ``sp_size`` / ``rank_within_spgroup``,
``get_sequence_parallel_state`` / ``set_sequence_parallel_state``, and the
``sp_seq_ctx`` full-length registry at :323-356), so code written against the
reference can point at this module instead.  Device meshes, FSDP and the rest
of the reference's training topology are outside the attention path.
"""
from __future__ import annotations

from typing import Optional

import torch.distributed as dist


class COMM_INFO:
    def __init__(self):
        self.sp_group = None
        self.sp_size = 1
        self.global_rank = 0
        self.rank_within_spgroup = 0


nccl_info = COMM_INFO()
_SEQUENCE_PARALLEL_STATE = False


def set_sequence_parallel_state(state: bool):
    global _SEQUENCE_PARALLEL_STATE
    _SEQUENCE_PARALLEL_STATE = bool(state)


def get_sequence_parallel_state() -> bool:
    return _SEQUENCE_PARALLEL_STATE


def initialize_sequence_parallel(group: Optional[dist.ProcessGroup] = None):
    """Use `group` (default: the world) as the Ulysses SP group."""
    if group is None:
        group = dist.group.WORLD
    nccl_info.sp_group = group
    nccl_info.sp_size = dist.get_world_size(group)
    nccl_info.global_rank = dist.get_rank()
    nccl_info.rank_within_spgroup = dist.get_group_rank(group, dist.get_rank())
    set_sequence_parallel_state(nccl_info.sp_size > 1)


def reset_sequence_parallel():
    nccl_info.sp_group = None
    nccl_info.sp_size = 1
    nccl_info.global_rank = 0
    nccl_info.rank_within_spgroup = 0
    set_sequence_parallel_state(False)


class SPSequenceContext:
    """Full (pre-shard) sequence length per SP stream (parallel_states.py:323-356)."""

    __slots__ = ("visual", "audio")

    def __init__(self):
        self.visual = None
        self.audio = None

    def set(self, visual=None, audio=None):
        if visual is not None:
            self.visual = int(visual)
        if audio is not None:
            self.audio = int(audio)

    def get(self, stream: str):
        return getattr(self, stream, None)

    def clear(self):
        self.visual = None
        self.audio = None


sp_seq_ctx = SPSequenceContext()
