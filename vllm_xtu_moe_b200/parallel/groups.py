"""Process-group set-up: one process per GPU, torch.distributed over NCCL (or gloo on
a host without GPUs), rendezvous from the usual RANK / WORLD_SIZE / MASTER_* variables."""
from __future__ import annotations

import os
from datetime import timedelta

import torch
import torch.distributed as dist


def rank_info() -> tuple[int, int, int]:
    """(rank, world_size, local_rank) from the launcher's environment (1 process: 0, 1, 0)."""
    return (int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1")),
            int(os.environ.get("LOCAL_RANK", os.environ.get("RANK", "0"))))


def init_distributed(backend: str | None = None, timeout_s: float = 300.0) -> tuple[int, int, torch.device]:
    """Initialise the default group once; returns (rank, world, device)."""
    rank, world, local = rank_info()
    if torch.cuda.is_available():
        dev = torch.device("cuda", local % torch.cuda.device_count())
        torch.cuda.set_device(dev)
    else:
        dev = torch.device("cpu")
    if world > 1 and not dist.is_initialized():
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        os.environ.setdefault("MASTER_PORT", "29500")
        be = backend or ("nccl" if dev.type == "cuda" else "gloo")
        kw = {"device_id": dev} if be == "nccl" else {}
        dist.init_process_group(be, rank=rank, world_size=world, timeout=timedelta(seconds=timeout_s), **kw)
    return rank, world, dev
