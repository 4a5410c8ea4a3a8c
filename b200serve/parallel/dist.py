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


def tp_mode() -> str:
    """How row-parallel outputs are combined: "ar" (all-reduce: every rank keeps the whole
    residual stream), "rsag" (reduce-scatter to the token owner, norm on the owned rows,
    all-gather of the normalised rows) or "auto" (rsag for prefill-sized steps, ar for decode).
    Set with B200_TP_MODE."""
    m = os.environ.get("B200_TP_MODE", "auto").lower()
    return m if m in ("ar", "rsag", "auto") else "auto"


class RSParts(list):
    """Partials of this rank's token shard after a reduce-scatter (``T`` tokens in the step).
    ``flags_ptr`` (fused path): flags the consumer waits for before reading the partials."""

    def __init__(self, views, T, flags_ptr=None, epoch_ptr=None, err_ptr=None, n_flags=None):
        super().__init__(views)
        self.T = T
        self.flags_ptr, self.epoch_ptr, self.err_ptr = flags_ptr, epoch_ptr, err_ptr
        self.n_flags = len(views) if n_flags is None else n_flags     # flags to wait for (one per rank)


class NcclComm:
    """Tensor-parallel reduction through library collectives (NCCL on GPU, gloo on CPU)."""

    kind = "nccl"

    def __init__(self, group=None, device="cuda"):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.device = torch.device(device)

    # ---- token-sharded residual stream: reduce-scatter + all-gather (library collectives) ----
    def use_rsag(self, T: int) -> bool:
        return tp_mode() == "rsag"

    def shard(self, T: int):
        """Rows per rank, first row and row count of this rank's token shard."""
        Tw = -(-T // self.world)
        row0 = self.rank * Tw
        return Tw, row0, max(0, min(T, row0 + Tw) - row0)

    def rs_linear(self, x, w, tag):
        from b200serve import ops
        y = ops.linear(x, w)
        T, H = y.shape
        Tw, row0, _ = self.shard(T)
        pad = torch.zeros(Tw * self.world, H, dtype=y.dtype, device=y.device)
        pad[:T] = y
        if pad.is_cuda:
            own = torch.empty(Tw, H, dtype=y.dtype, device=y.device)
            dist.reduce_scatter_tensor(own, pad, group=self.group)
        else:                       # gloo has no reduce-scatter: same result through all-reduce
            dist.all_reduce(pad, group=self.group)
            own = pad[row0:row0 + Tw].contiguous()
        return RSParts([own], T)

    def norm_ag(self, parts, weight, eps, residual):
        """RMSNorm of this rank's rows (+ residual, updated in place), then all-gather."""
        from b200serve import ops
        xo = ops.rmsnorm(list(parts), weight, eps, residual=residual, residual_out=residual)
        Tw, H = xo.shape
        full = torch.empty(Tw * self.world * H, dtype=xo.dtype, device=xo.device)
        dist.all_gather_into_tensor(full, xo.contiguous().view(-1), group=self.group)
        return full.view(Tw * self.world, H)[:parts.T], None

    def reduce_parts(self, t: torch.Tensor, tag: str):
        dist.all_reduce(t, group=self.group)
        return [t]

    # ---- expert parallelism on a token-sharded stream: all-to-all dispatch and combine ----
    def ep_moe(self, moe, layer: int, x_own: torch.Tensor, ids: torch.Tensor, wts: torch.Tensor, T: int):
        """Expert FFN of this rank's own rows, experts spread over the ranks (library collectives:
        the reference the fused NVLink path is checked against). Every (token, expert) pair is
        computed by the rank owning the expert; its routing-weighted output comes back to the
        token's owner as pair row (t, j). Returns the k pair rows as parts [k][Tw, H], which the
        owner's norm sums in j order."""
        Tw, H = x_own.shape
        k = ids.shape[1]
        xs = [torch.empty_like(x_own) for _ in range(self.world)]
        idl = [torch.empty_like(ids) for _ in range(self.world)]
        wl = [torch.empty_like(wts) for _ in range(self.world)]
        dist.all_gather(xs, x_own.contiguous(), group=self.group)
        dist.all_gather(idl, ids.contiguous(), group=self.group)
        dist.all_gather(wl, wts.contiguous(), group=self.group)
        x_all, id_all, w_all = torch.cat(xs), torch.cat(idl), torch.cat(wl)
        contrib = moe.pair_outputs(layer, x_all, id_all, w_all)          # [world*Tw, k, H], zeros elsewhere
        dist.all_reduce(contrib, group=self.group)                       # one rank owns each pair
        mine = contrib[self.rank * Tw:(self.rank + 1) * Tw]
        return RSParts([mine[:, j].contiguous() for j in range(k)], T)

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
