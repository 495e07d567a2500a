"""Explicit communicator set-up for expert parallelism.

The reference writes its NCCL settings from the layer constructor
(``setup_nccl_optimizations``, models/ultimate_moe.py:15-31, called from ``__init__``),
i.e. after the process group exists, when NCCL has already read its environment.
``init_expert_parallel`` applies the same settings first and then creates the group,
one process per GPU (torchrun's RANK / WORLD_SIZE / LOCAL_RANK)."""
from __future__ import annotations

import datetime
import os
from typing import Optional

import torch
import torch.distributed as dist

from .ultimate_moe import setup_nccl_optimizations


def init_expert_parallel(backend: Optional[str] = None, *, timeout_s: float = 120.0, nccl_defaults: bool = True,
                         nvls: Optional[bool] = None, init_method: Optional[str] = None):
    """Create the default process group for expert-parallel layers; returns
    ``(rank, world_size, local_rank)``.

    * ``backend``: ``"nccl"`` when CUDA is available, else ``"gloo"``.
    * ``nccl_defaults``: the reference's NCCL settings (only variables not already set).
    * ``nvls``: ``True`` / ``False`` sets ``NCCL_NVLS_ENABLE`` (NVLink SHARP reductions in
      the switch) unless it is already set; ``None`` leaves NCCL's choice.
    * With NCCL the current device becomes ``cuda:LOCAL_RANK`` and the group is bound to
      it (eager communicator creation).
    * ``timeout_s`` bounds every collective, so ranks waiting for a rank that died end
      with an error instead of hanging.

    If a default group already exists nothing is changed (its settings were read when it
    was created) and its rank and size are returned."""
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if dist.is_initialized():
        return dist.get_rank(), dist.get_world_size(), local
    if backend is None:
        backend = "nccl" if torch.cuda.is_available() else "gloo"
    if nccl_defaults:
        setup_nccl_optimizations()
    if nvls is not None and "NCCL_NVLS_ENABLE" not in os.environ:
        os.environ["NCCL_NVLS_ENABLE"] = "1" if nvls else "0"
    kwargs = dict(timeout=datetime.timedelta(seconds=timeout_s))
    if init_method is not None:
        kwargs["init_method"] = init_method
        kwargs["rank"] = int(os.environ.get("RANK", "0"))
        kwargs["world_size"] = int(os.environ.get("WORLD_SIZE", "1"))
    if backend == "nccl":
        torch.cuda.set_device(local)
        kwargs["device_id"] = torch.device("cuda", local)
    dist.init_process_group(backend, **kwargs)
    return dist.get_rank(), dist.get_world_size(), local
