"""Process-group bootstrap and the tensor-parallel communicators.

One process per GPU (torchrun sets RANK / LOCAL_RANK / WORLD_SIZE /
MASTER_ADDR / MASTER_PORT). ``NcclComm`` is the library baseline: an NCCL
all-reduce of each row-parallel output. ``make_comm`` returns the fused
in-kernel NVLink communicator when ``comm == "fused"`` and the fused kernels
are available, else the NCCL one.
"""

from __future__ import annotations

import datetime
import os

import torch
import torch.distributed as dist


def rank_world():
    if dist.is_available() and dist.is_initialized():
        return dist.get_rank(), dist.get_world_size()
    return int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1))


def local_rank() -> int:
    return int(os.environ.get("LOCAL_RANK", rank_world()[0]))


def init_distributed(backend: str = None, timeout_s: float = 120.0):
    """Initialise the default process group from torchrun's environment (idempotent)."""
    if dist.is_initialized():
        return dist.group.WORLD
    world = int(os.environ.get("WORLD_SIZE", 1))
    if world == 1:
        return None
    if backend is None:
        backend = "nccl" if torch.cuda.is_available() else "gloo"
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    if backend == "nccl":
        torch.cuda.set_device(local_rank())
    kw = {}
    if backend == "nccl":
        kw["device_id"] = torch.device("cuda", local_rank())
    dist.init_process_group(backend=backend, timeout=datetime.timedelta(seconds=timeout_s), **kw)
    return dist.group.WORLD


class NcclComm:
    """Tensor-parallel reduction through library collectives (NCCL on GPU, gloo on CPU)."""

    kind = "nccl"

    def __init__(self, group=None, device="cuda"):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.device = torch.device(device)

    def reduce_parts(self, t: torch.Tensor, tag: str):
        dist.all_reduce(t, group=self.group)
        return [t]

    def all_gather_small(self, t: torch.Tensor) -> torch.Tensor:
        flat = torch.empty(self.world * t.numel(), dtype=t.dtype, device=t.device)
        dist.all_gather_into_tensor(flat, t.contiguous().view(-1), group=self.group)
        return flat.view((self.world,) + tuple(t.shape))

    def gather_vocab(self, logits: torch.Tensor, vocab_size: int = None) -> torch.Tensor:
        """[B, V_local] shards (equal padded width, last shard may be shorter) -> [B, V]."""
        B, v = logits.shape
        width = torch.tensor([v], device=logits.device, dtype=torch.int64)
        widths = self.all_gather_small(width).view(-1).tolist()
        w = max(widths)
        pad = logits
        if v < w:
            pad = torch.full((B, w), float("-inf"), dtype=logits.dtype, device=logits.device)
            pad[:, :v] = logits
        allv = self.all_gather_small(pad)          # [R, B, w]
        return torch.cat([allv[r, :, :widths[r]] for r in range(self.world)], dim=1)

    def broadcast(self, t: torch.Tensor, src: int = 0):
        dist.broadcast(t, src=src, group=self.group)
        return t

    def barrier(self):
        dist.barrier(group=self.group)


def make_comm(cfgE, device, model_cfg):
    group = init_distributed()
    if cfgE.comm == "fused" and device.type == "cuda":
        from b200serve.parallel.fused_comm import FusedComm, fused_available
        if fused_available():
            return FusedComm(group, device, model_cfg, cfgE)
    return NcclComm(group, device)
