"""Sequence-parallel state read by the cached attention (mirror of the fields of
``hymm/distributed/parallel_states.py:135-198`` that the hot path uses).

When the drop-in is installed into the reference process (``install.install``), the
attention reads the reference's own ``nccl_info`` / ``get_sequence_parallel_state``
instead; standalone users (tests, ``bench.py``) initialise this module.
"""
from __future__ import annotations

import torch.distributed as dist


class COMM_INFO:
    def __init__(self):
        self.sp_group = None
        self.sp_size = 1
        self.rank_within_spgroup = 0
        self.global_rank = 0


nccl_info = COMM_INFO()
_SEQUENCE_PARALLEL_STATE = False


def set_sequence_parallel_state(state: bool) -> None:
    global _SEQUENCE_PARALLEL_STATE
    _SEQUENCE_PARALLEL_STATE = bool(state)


def get_sequence_parallel_state() -> bool:
    return _SEQUENCE_PARALLEL_STATE


def initialize_sequence_parallel_group(group=None) -> None:
    """Use ``group`` (default: the world) as the Ulysses sequence-parallel group."""
    nccl_info.__init__()
    if not dist.is_initialized():
        set_sequence_parallel_state(False)
        return
    group = group if group is not None else dist.group.WORLD
    nccl_info.sp_group = group
    nccl_info.sp_size = dist.get_world_size(group)
    nccl_info.rank_within_spgroup = dist.get_rank(group)
    nccl_info.global_rank = dist.get_rank()
    set_sequence_parallel_state(nccl_info.sp_size > 1)


def destroy_sequence_parallel_group() -> None:
    nccl_info.__init__()
    set_sequence_parallel_state(False)
