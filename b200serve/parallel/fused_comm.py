"""In-kernel tensor-parallel all-reduce over NVLink P2P (decode-sized outputs).

Each rank owns one CUDA IPC region, mapped by every other rank:
  data  [2 slots][world][max_tokens][hidden] bf16   (slot = site parity)
  flags [n_sites][world] int32                      (flag[site][r] = epoch of r's push)
Row-parallel GEMMs (o_proj, down) run ``gemm_tc_push``: the epilogue stores
each bf16 tile into slot [site % 2][my rank] of every rank and the last CTA
raises flag[site][my rank] = epoch on every rank. The next fused add+RMSNorm
kernel waits for all ``world`` flags of the site (bounded wait) and sums the
``world`` local slots, so the reduction costs no extra kernel and no NCCL
call. Outputs with more tokens than ``max_tokens`` (prefill chunks) use NCCL,
which runs them through NVLS at full bandwidth.

The epoch is a device counter bumped by a one-thread kernel at the start of
every forward (inside the CUDA graph as well), so flags never need resetting.
A wait that runs out records a code in a host-mapped error word; ``check()``
raises ``CollectiveTimeout`` on the host.
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from b200serve import ops
from b200serve.parallel.dist import NcclComm


class CollectiveTimeout(RuntimeError):
    """A fused collective's bounded wait expired (a peer rank did not publish)."""


def check_error_word(host_ptr: int, rank: int = 0):
    """Read (and clear) a host-mapped error word written by the kernels' bounded waits;
    raise CollectiveTimeout when one of them gave up. Codes: 100+r / 120+r / 140+r = the
    norm, the all-gather GEMM or the flag-wait kernel stopped waiting for rank r."""
    code = ops.ext().read_host_word(host_ptr, 0, True)
    if code:
        raise CollectiveTimeout(f"fused collective wait expired on rank {rank} (code {code})")


def fused_available() -> bool:
    try:
        return hasattr(ops.ext(), "gemm_tc_push")
    except Exception:
        return False


class FusedParts(list):
    """The local receive slots of one site plus what the consumer must wait for."""

    def __init__(self, views, flags_ptr, epoch_ptr, err_ptr):
        super().__init__(views)
        self.flags_ptr, self.epoch_ptr, self.err_ptr = flags_ptr, epoch_ptr, err_ptr


class LamportParts(list):
    """The local receive slots of one flag-free site (one view per source rank). The consumer
    polls the data itself; ``launch_mark`` is the launch count right after the push GEMM, so the
    norm can tell whether it directly follows that GEMM."""

    lamport = True

    def __init__(self, views, err_ptr, launch_mark):
        super().__init__(views)
        self.err_ptr, self.launch_mark = err_ptr, launch_mark


def _lamport_default() -> bool:
    import os
    return os.environ.get("B200_TP_LAMPORT", "1") != "0"


def _nvls_default() -> bool:
    import os
    return os.environ.get("B200_TP_NVLS", "1") != "0"


def _multicast_slots(nbytes: int, device, group):
    """(tensor, local ptr, multicast ptr) of a symmetric buffer bound to an NVLink multicast object
    (NVLS through the NVSwitch), or None when the box or the driver offers none."""
    try:
        import torch.distributed._symmetric_memory as symm
        if hasattr(symm, "enable_symm_mem_for_group"):
            symm.enable_symm_mem_for_group(group.group_name)
        t = symm.empty(nbytes, dtype=torch.uint8, device=device)
        h = symm.rendezvous(t, group)
        if not getattr(h, "has_multicast_support", False) or not h.multicast_ptr:
            return None
        return t, h, int(t.data_ptr()), int(h.multicast_ptr)
    except Exception:  # no symmetric memory / multicast here: the P2P slots serve
        return None


class FusedComm:
    kind = "fused-p2p"

    def __init__(self, group, device, model_cfg, cfgE, max_tokens: int = None):
        self.nccl = NcclComm(group, device)
        self.group = group
        self.world = self.nccl.world
        self.rank = self.nccl.rank
        self.device = torch.device(device)
        H = model_cfg.hidden_size
        self.H = H
        self.max_tokens = max_tokens or max(cfgE.max_batch, 64)
        # largest step (a prefill chunk plus the decode tokens riding along) for the
        # reduce-scatter / all-gather path
        self.max_step = max(self.max_tokens, int(getattr(cfgE, "prefill_chunk", 0) or 0) + cfgE.max_batch)
        # MoE steps on a token-sharded stream use five sites per layer (RS, AG, counts, dispatch, combine)
        self.n_sites = (6 if model_cfg.is_moe else 4) * model_cfg.num_layers + 8
        self.slot_rows = max(self.max_tokens, -(-self.max_step // self.world))
        self.slot_elems = self.slot_rows * H
        data_bytes = 2 * self.world * self.slot_elems * 2
        self.ag_off = (data_bytes + 4095) // 4096 * 4096
        ag_bytes = 2 * self.max_step * H * 2                  # gathered rows, [2 parities][max_step][H]
        self.flag_off = (self.ag_off + ag_bytes + 4095) // 4096 * 4096
        # flag-free all-reduce slots: [3 rotations][world][max_tokens][H] bf16, 0xFFFF while empty
        self.lam_elems = self.max_tokens * H
        self.lam_off = (self.flag_off + self.n_sites * self.world * 4 + 4095) // 4096 * 4096
        self.lam_bytes = 3 * self.world * self.lam_elems * 2
        total = self.lam_off + self.lam_bytes
        # expert-parallel all-to-all (MoE): count matrices of every rank, expert-sorted receive rows
        # and their (home rank, pair, weight) metadata, and the k combine slots of the owned rows
        self.ep = None
        if model_cfg.is_moe and self.world > 1:
            k, per = model_cfg.experts_per_tok, model_cfg.num_experts // self.world
            rcap = self.world * self.slot_rows * k
            lay = {}
            off = (total + 4095) // 4096 * 4096
            for name, nbytes in (("cnt", self.world * self.world * per * 4), ("rows", rcap * H * 2),
                                 ("meta", rcap * 16), ("comb", k * self.slot_rows * H * 2)):
                lay[name] = off
                off = (off + nbytes + 4095) // 4096 * 4096
            self.ep = {"k": k, "per": per, "rcap": rcap, "off": lay}
            total = off
        self.lamport = _lamport_default()
        e = ops.ext()
        self.base = e.ipc_malloc(total)
        handle = e.ipc_handle(self.base)
        handles = [None] * self.world
        dist.all_gather_object(handles, handle.tolist(), group=group)
        self.peer = []
        for r in range(self.world):
            if r == self.rank:
                self.peer.append(self.base)
            else:
                self.peer.append(e.ipc_open(torch.tensor(handles[r], dtype=torch.uint8)))
        self.epoch = torch.zeros(1, dtype=torch.int32, device=self.device)
        self.ep_done = torch.zeros(1, dtype=torch.int32, device=self.device)
        self.tile_done = torch.zeros(1, dtype=torch.int32, device=self.device)
        self.ag_done = torch.zeros(1, dtype=torch.int32, device=self.device)
        self._ag_ptrs = {}
        # NVLS: the flag-free slots in a symmetric buffer with a multicast mapping, so one
        # multimem store per 16 bytes reaches every GPU (same layout as the P2P slots)
        self.mc = _multicast_slots(self.lam_bytes, self.device, group) if (self.world > 1 and _nvls_default()) else None
        self.use_mc = self.mc is not None
        self.kind = "fused-nvls" if self.use_mc else "fused-p2p"
        self.reset_lamport()
        self.err = e.host_error_word()       # [host ptr, device ptr]
        self.err_host, self.err_dev = int(self.err[0]), int(self.err[1])
        self.ws = ops.GemmWorkspace(self.device, max_elems=8 << 20, max_tiles=1 << 14)
        self.site = 0
        self._views = {}
        self._ptrs = {}
        dist.barrier(group=group)

    # ------------------------------------------------------------ helpers
    def _slot_ptr(self, rank_base: int, slot: int, src_rank: int) -> int:
        return rank_base + (slot * self.world + src_rank) * self.slot_elems * 2

    def _flag_ptr(self, rank_base: int, site: int, src_rank: int) -> int:
        return rank_base + self.flag_off + (site * self.world + src_rank) * 4

    def reset_lamport(self):
        """Mark every flag-free slot of this rank empty (at start-up and after a failed step, whose
        consumers may not have emptied the slots they were reading)."""
        region = _tensor_from_ptr(self.base + self.lam_off, self.lam_bytes // 2, self.device)
        region.view(torch.int16).fill_(-1)
        if getattr(self, "mc", None) is not None:
            self.mc[0].fill_(0xFF)
        torch.cuda.synchronize(self.device)

    def _lam_ptr(self, rank_base: int, rot: int, src_rank: int) -> int:
        return rank_base + self.lam_off + (rot * self.world + src_rank) * self.lam_elems * 2

    def _lam_local(self, rot: int, src_rank: int) -> int:
        if self.use_mc:
            return self.mc[2] + (rot * self.world + src_rank) * self.lam_elems * 2
        return self._lam_ptr(self.base, rot, src_rank)

    def _lam_views(self, rot: int, T: int):
        key = ("lam", rot, T, self.use_mc)
        if key not in self._views:
            self._views[key] = [_tensor_from_ptr(self._lam_local(rot, r), T * self.H, self.device)
                                .view(T, self.H) for r in range(self.world)]
        return self._views[key]

    def _local_views(self, slot: int, T: int):
        key = (slot, T)
        if key not in self._views:
            vs = []
            for r in range(self.world):
                storage = _tensor_from_ptr(self._slot_ptr(self.base, slot, r), T * self.H, self.device)
                vs.append(storage.view(T, self.H))
            self._views[key] = vs
        return self._views[key]

    def _push_ptrs(self, site: int):
        if site not in self._ptrs:
            slot = site % 2
            dst = torch.tensor([self._slot_ptr(self.peer[r], slot, self.rank) for r in range(self.world)],
                               dtype=torch.int64)
            flg = torch.tensor([self._flag_ptr(self.peer[r], site, self.rank) for r in range(self.world)],
                               dtype=torch.int64)
            self._ptrs[site] = (dst, flg)
        return self._ptrs[site]

    # ------------------------------------------------------------ comm interface
    def begin_step(self):
        ops._cuda(self.epoch)
        ops.ext().epoch_inc(self.epoch.data_ptr())
        self.site = 0

    def linear_reduce(self, x: torch.Tensor, w: torch.Tensor, tag: str):
        """Row-parallel GEMM + all-reduce. Returns the parts the next RMSNorm sums."""
        T = x.shape[0]
        if (isinstance(w, ops.QuantWeight) and self.lamport and T <= 16 and x.is_cuda
                and w.N == self.H and w.K % 256 == 0):
            # GGUF row-parallel projection: the stream-K GEMV stores each finished bf16 tile straight
            # into every rank's flag-free slot (P2P or one multicast store)
            site = self.site
            self.site += 1
            assert site < self.n_sites, "more fused sites than allocated"
            rot = site % 3
            key = ("lamdst", rot)
            if key not in self._ptrs:
                self._ptrs[key] = torch.tensor([self._lam_ptr(self.peer[r], rot, self.rank)
                                                for r in range(self.world)], dtype=torch.int64)
            mc = self.mc[3] + (rot * self.world + self.rank) * self.lam_elems * 2 if self.use_mc else 0
            dst = self._ptrs[key]
            if self.use_mc:
                dst = torch.tensor([self._lam_local(rot, self.rank)], dtype=torch.int64)   # unused with mc
            ops.gguf_stream(x, [w], 4, None, self.H, dst, mc)
            return LamportParts(self._lam_views(rot, T), self.err_dev, ops.launch_count())
        if T > self.max_tokens or not isinstance(w, (torch.Tensor, ops.PackedWeight)):
            # large chunks (NVLS all-reduce is bandwidth-optimal) and other quantised shapes take NCCL
            y = ops.linear(x, w)
            return self.nccl.reduce_parts(y, tag)
        site = self.site
        self.site += 1
        assert site < self.n_sites, "more fused sites than allocated"
        dst, flg = self._push_ptrs(site)
        ops._cuda(x)
        packed_n = w.N if isinstance(w, ops.PackedWeight) else 0
        if self.lamport:
            rot = site % 3
            key = ("lamdst", rot)
            if key not in self._ptrs:
                self._ptrs[key] = torch.tensor([self._lam_ptr(self.peer[r], rot, self.rank)
                                                for r in range(self.world)], dtype=torch.int64)
            mc = self.mc[3] + (rot * self.world + self.rank) * self.lam_elems * 2 if self.use_mc else 0
            ops.ext().gemm_tc_push(x, w.data if packed_n else w, self._ptrs[key], self.H, flg,
                                   self.epoch.data_ptr(), self.tile_done, None, self.ws.ws, self.ws.counters,
                                   self.err_dev, packed_n, 0, 1, mc)
            return LamportParts(self._lam_views(rot, T), self.err_dev, ops.launch_count())
        ops.ext().gemm_tc_push(x, w.data if packed_n else w, dst, self.H, flg, self.epoch.data_ptr(), self.tile_done,
                               None, self.ws.ws, self.ws.counters, self.err_dev, packed_n, 0, 0)
        return FusedParts(self._local_views(site % 2, T), self._flag_ptr(self.base, site, 0),
                          self.epoch.data_ptr(), self.err_dev)

    # ------------------------------------------------------------ reduce-scatter / all-gather
    def use_rsag(self, T: int) -> bool:
        from b200serve.parallel.dist import tp_mode
        m = tp_mode()
        if T > self.max_step:
            return False
        return m == "rsag" or (m == "auto" and T > self.max_tokens)

    def shard(self, T: int):
        return self.nccl.shard(T)

    def _next_site(self) -> int:
        site = self.site
        self.site += 1
        assert site < self.n_sites, "more fused sites than allocated"
        return site

    def rs_linear(self, x: torch.Tensor, w, tag: str):
        """GEMM -> reduce-scatter: the epilogue pushes token row t only to its owner rank
        (rows T/world per rank), which sums the ``world`` partials in its norm."""
        from b200serve.parallel.dist import RSParts
        T = x.shape[0]
        Tw, _, _ = self.shard(T)
        if not isinstance(w, (torch.Tensor, ops.PackedWeight)):
            return self.nccl.rs_linear(x, w, tag)
        site = self._next_site()
        dst, flg = self._push_ptrs(site)
        ops._cuda(x)
        packed_n = w.N if isinstance(w, ops.PackedWeight) else 0
        ops.ext().gemm_tc_push(x, w.data if packed_n else w, dst, self.H, flg, self.epoch.data_ptr(),
                               self.tile_done, None, self.ws.ws, self.ws.counters, self.err_dev, packed_n, Tw, 0)
        return RSParts(self._local_views(site % 2, Tw), T, self._flag_ptr(self.base, site, 0),
                       self.epoch.data_ptr(), self.err_dev)

    def _ag_base(self, rank_base: int, parity: int) -> int:
        return rank_base + self.ag_off + parity * self.max_step * self.H * 2

    def norm_ag(self, parts, weight, eps, residual):
        """Norm of this rank's token shard fused with the all-gather of its output rows: the
        kernel stores each normalised row into every rank's gathered buffer and raises their
        flags. Returns (gathered rows [T, H] on this rank, AGWait for consumers)."""
        T = parts.T
        Tw, row0, _ = self.shard(T)
        if parts.flags_ptr is None:             # partials came through NCCL
            return self.nccl.norm_ag(parts, weight, eps, residual)
        site = self._next_site()
        par = site % 2
        key = (site, par)
        if key not in self._ag_ptrs:
            dst = torch.tensor([self._ag_base(self.peer[r], par) for r in range(self.world)], dtype=torch.int64)
            flg = torch.tensor([self._flag_ptr(self.peer[r], site, self.rank) for r in range(self.world)],
                               dtype=torch.int64)
            self._ag_ptrs[key] = (dst, flg)
        dst, flg = self._ag_ptrs[key]
        ops._cuda(residual)
        ops.ext().rmsnorm_rs_ag(list(parts), residual, residual, weight, float(eps), parts.flags_ptr,
                                self.epoch.data_ptr(), self.err_dev, dst, flg, row0, T, self.ag_done,
                                getattr(parts, "n_flags", len(parts)))
        full = _tensor_from_ptr(self._ag_base(self.base, par), T * self.H, self.device).view(T, self.H)
        return full, ops.AGWait(self._flag_ptr(self.base, site, 0), self.world, self.epoch.data_ptr(), self.err_dev)

    # ------------------------------------------------------------ expert-parallel all-to-all
    def _ep_ptr(self, rank_base: int, name: str) -> int:
        return rank_base + self.ep["off"][name]

    def ep_moe(self, moe, layer: int, x_own: torch.Tensor, ids: torch.Tensor, wts: torch.Tensor, T: int):
        """Expert FFN of this rank's token rows over NVLink: counts broadcast to every rank (one
        host read of the small count matrix sizes the grouped GEMMs), each (token, expert) pair's
        row pushed into its expert-sorted slot on the expert's owner, the owner's grouped
        SwiGLU GEMM waiting for the rows inside the kernel, and the grouped down GEMM's epilogue
        pushing routing-weighted rows back to the home rank's k combine slots. Returns those slots
        as the parts of the next norm, which waits for one flag per rank."""
        if self.ep is None or not x_own.is_cuda:
            return self.nccl.ep_moe(moe, layer, x_own, ids, wts, T)
        e = ops.ext()
        Tw, H = x_own.shape
        k, per, world, me = ids.shape[1], self.ep["per"], self.world, self.rank
        assert k == self.ep["k"] and Tw <= self.slot_rows
        _, _, valid = self.shard(T)
        ids_c, wts_c = ids.contiguous(), wts.float().contiguous()
        epoch = self.epoch.data_ptr()
        peers = range(world)
        i64 = lambda v: torch.tensor(v, dtype=torch.int64)
        # 1. counts -> every rank
        s1 = self._next_site()
        pos = torch.empty(max(1, Tw * k), dtype=torch.int32, device=self.device)
        e.ep_count(ids_c, valid, per, me, pos, i64([self._ep_ptr(self.peer[r], "cnt") for r in peers]),
                   i64([self._flag_ptr(self.peer[r], s1, me) for r in peers]), epoch)
        e.flag_wait(self._flag_ptr(self.base, s1, 0), world, epoch, self.err_dev)
        cnt_t = _tensor_from_ptr(self._ep_ptr(self.base, "cnt"), world * world * per * 2, self.device)
        cnt = cnt_t.view(torch.int32).view(world, world, per).cpu()           # host read: sizes the GEMMs
        self.check()
        mine = cnt[:, me, :].sum(0)                                           # rows per local expert
        offsets = torch.zeros(per + 1, dtype=torch.int32)
        offsets[1:] = torch.cumsum(mine, 0)
        R, max_rows = int(offsets[-1]), int(mine.max())
        offsets = offsets.to(self.device)
        # 2. dispatch rows to their experts' owners
        s2 = self._next_site()
        e.ep_dispatch(x_own.contiguous(), ids_c, wts_c, pos, valid, per, me, self._ep_ptr(self.base, "cnt"),
                      self._flag_ptr(self.base, s1, 0), i64([self._ep_ptr(self.peer[r], "cnt") for r in peers]),
                      i64([self._ep_ptr(self.peer[r], "rows") for r in peers]),
                      i64([self._ep_ptr(self.peer[r], "meta") for r in peers]),
                      i64([self._flag_ptr(self.peer[r], s2, me) for r in peers]), epoch, self.ep_done, self.err_dev)
        ops._launches[0] += 3
        s3 = self._next_site()
        flg3 = i64([self._flag_ptr(self.peer[r], s3, me) for r in peers])
        comb_rows = self.slot_rows
        if R == 0:
            # nothing routed here: wait for the (empty) dispatch, then release the combine consumers
            e.flag_wait(self._flag_ptr(self.base, s2, 0), world, epoch, self.err_dev)
            e.publish_flags(flg3, epoch)
        else:
            gu, n_gu, dn, n_dn = moe.packed[layer]
            rows = _tensor_from_ptr(self._ep_ptr(self.base, "rows"), R * H, self.device).view(R, H)
            act = torch.empty(R, n_gu // 2, dtype=x_own.dtype, device=self.device)
            empty = torch.empty(0, dtype=torch.int32)
            e.gemm_grouped_ep(rows, gu, n_gu, per, offsets, max_rows, act, self.ws.ws, self.ws.counters,
                              ops.EPI_SWIGLU, self._flag_ptr(self.base, s2, 0), world, epoch, empty, 0, 0,
                              torch.empty(0, dtype=torch.int64), 0, torch.empty(0, dtype=torch.int64),
                              self.tile_done, 0, self.err_dev)
            bn = 16 if max_rows <= 16 else 32 if max_rows <= 32 else 64 if max_rows <= 64 else \
                128 if max_rows <= 128 else 256
            tiles = int(sum((int(c) + bn - 1) // bn for c in mine)) * ((n_dn + 127) // 128)
            meta = _tensor_from_ptr(self._ep_ptr(self.base, "meta"), R * 8, self.device).view(torch.int32)
            e.gemm_grouped_ep(act, dn, n_dn, per, offsets, max_rows, act, self.ws.ws, self.ws.counters,
                              ops.EPI_PUSH, 0, 0, epoch, meta, k, comb_rows,
                              i64([self._ep_ptr(self.peer[r], "comb") for r in peers]), H, flg3, self.tile_done,
                              tiles, self.err_dev)
            ops._launches[0] += 2
        views = [_tensor_from_ptr(self._ep_ptr(self.base, "comb") + j * comb_rows * H * 2, Tw * H, self.device)
                 .view(Tw, H) for j in range(k)]
        from b200serve.parallel.dist import RSParts
        return RSParts(views, T, self._flag_ptr(self.base, s3, 0), epoch, self.err_dev, n_flags=world)

    def moe_combine_reduce(self, y, wts, pos, k, T):
        """Expert-parallel combine fused with the cross-rank sum: the combine kernel pushes each
        token's weighted expert sum into every rank's slot and raises the site's flags; the
        next norm waits for them and sums the ``world`` slots."""
        site = self._next_site()
        dst, flg = self._push_ptrs(site)
        ops._cuda(y)
        ops.ext().moe_combine_push(y, wts, pos, k, T, self.H, dst, flg, self.epoch.data_ptr(), self.ag_done)
        return FusedParts(self._local_views(site % 2, T), self._flag_ptr(self.base, site, 0),
                          self.epoch.data_ptr(), self.err_dev)

    def reduce_parts(self, t: torch.Tensor, tag: str):
        return self.nccl.reduce_parts(t, tag)

    def all_gather_small(self, t):
        return self.nccl.all_gather_small(t)

    def gather_vocab(self, logits):
        return self.nccl.gather_vocab(logits)

    def broadcast(self, t, src=0):
        return self.nccl.broadcast(t, src)

    def barrier(self):
        self.nccl.barrier()

    def check(self):
        try:
            check_error_word(self.err_host, self.rank)
        except CollectiveTimeout:
            self.reset_lamport()
            raise

    def close(self):
        e = ops.ext()
        for r, p in enumerate(self.peer):
            if r != self.rank:
                e.ipc_close(p)
        e.ipc_free(self.base)
        self.peer = []


def _tensor_from_ptr(ptr: int, numel: int, device) -> torch.Tensor:
    """A bf16 view of device memory owned by FusedComm (no copy, no ownership):
    built through the CUDA array interface on int16, then reinterpreted."""
    class _CAI:
        def __init__(self):
            self.__cuda_array_interface__ = {"shape": (numel,), "typestr": "<i2", "data": (ptr, False),
                                             "version": 3, "strides": None}
    return torch.as_tensor(_CAI(), device=device).view(torch.bfloat16)
