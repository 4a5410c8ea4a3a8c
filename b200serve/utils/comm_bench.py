"""Fused tensor-parallel collective micro-benchmark (run under torchrun, one rank per GPU).

One site of the decode step: row-parallel GEMM [T, K/world] x [K/world, H] whose
outputs are summed over ranks, then add+RMSNorm. Compares
  lamport: push-GEMM storing tiles into every rank's flag-free slot (empty = 0xFFFF) +
         a RMSNorm that polls the data itself,
  fused: push-GEMM (epilogue stores tiles into every rank's slot over NVLink) +
         flag-waiting RMSNorm,
  nccl:  GEMM + NCCL all-reduce + RMSNorm,
and reports the fused time against its roofline: the slower of streaming the
weight shard at the measured HBM bandwidth and moving (world-1) x T x H x 2
bytes per rank over NVLink at 770 GB/s (the measured peer-copy rate).
Device-timed with CUDA events, max over ranks.

  torchrun --nproc-per-node 8 --master-addr 127.0.0.1 -m b200serve.utils.comm_bench
"""

from __future__ import annotations

import json
import os

import torch
import torch.distributed as dist

from b200serve import ops
from b200serve.core.config import EngineConfig
from b200serve.models.config import BUILTIN
from b200serve.parallel.dist import init_distributed
from b200serve.parallel.fused_comm import FusedComm
from b200serve.utils.kbench import peaks
from b200serve.utils.timing import max_over_ranks

NVLINK_GBPS = 770.0


def _tensor_from_ptr_i32(ptr: int) -> torch.Tensor:
    class _CAI:
        def __init__(self):
            self.__cuda_array_interface__ = {"shape": (1,), "typestr": "<i4", "data": (ptr, False), "version": 3,
                                             "strides": None}
    return torch.as_tensor(_CAI(), device="cuda")


def main():
    init_distributed("nccl", timeout_s=120)
    rank, world = dist.get_rank(), dist.get_world_size()
    torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", rank)))
    cfg = BUILTIN["qwen3-8b"]
    H = cfg.hidden_size
    comm = FusedComm(dist.group.WORLD, torch.device("cuda"), cfg, EngineConfig(max_batch=64, prefill_chunk=1024))
    hbm, _, src = peaks()
    results = []
    # raw cross-GPU flag round trip between rank 0 and every other rank (P2P st.release /
    # ld.acquire .sys), the floor under any in-kernel collective on this box
    if world > 1:
        e = ops.ext()
        out = torch.zeros(1, dtype=torch.int64, device="cuda")
        rtts = {}
        for mode, peer in [(0, p) for p in range(1, world)] + [(1, 1), (2, 1)]:
            comm.begin_step()
            torch.cuda.synchronize()
            dist.barrier()
            if rank in (0, peer):
                other = peer if rank == 0 else 0
                # flag words of site n_sites-1: mine = (site, src=other) locally, peer's = (site, src=me) there
                site = comm.n_sites - 1
                mine = comm._flag_ptr(comm.base, site, other)
                theirs = comm._flag_ptr(comm.peer[other], site, rank)
                e.flag_pingpong(mine, theirs, 1000, 1 if rank == 0 else 0, mode, out)
                torch.cuda.synchronize()
                if rank == 0:
                    rtts[f"{['acq_rel', 'relaxed', 'volatile'][mode]}:{peer}"] = round(out.item() / 1000.0 / 1000.0, 3)
            dist.barrier()
            # reset the flag words used above for the next pair
            if rank in (0, peer):
                other = peer if rank == 0 else 0
                _tensor_from_ptr_i32(comm._flag_ptr(comm.base, comm.n_sites - 1, other)).zero_()
            torch.cuda.synchronize()
            dist.barrier()
        if rank == 0:
            print(json.dumps({"case": "flag_round_trip_us", "world": world, "per_peer": rtts}), flush=True)
    for name, Kfull in (("o_proj", cfg.q_size), ("down", cfg.intermediate_size)):
        K = Kfull // world
        w = ops.pack_weight((torch.randn(H, K, device="cuda") * 0.02).bfloat16())
        nw = torch.ones(H, device="cuda").bfloat16()
        for T in (1, 32, 1024):
            x = torch.randn(T, K, device="cuda").bfloat16()
            res = torch.randn(T, H, device="cuda").bfloat16()
            out = torch.empty(T, H, device="cuda").bfloat16()

            def lamport_nvls():
                comm.lamport, comm.use_mc = True, comm.mc is not None
                comm.begin_step()
                for _ in range(8):
                    parts = comm.linear_reduce(x, w, "o")
                    ops.rmsnorm(parts, nw, 1e-6, residual=res, out=out)

            def lamport():
                comm.lamport, comm.use_mc = True, False
                comm.begin_step()
                for _ in range(8):
                    parts = comm.linear_reduce(x, w, "o")
                    ops.rmsnorm(parts, nw, 1e-6, residual=res, out=out)

            def fused():
                comm.lamport, comm.use_mc = False, False
                comm.begin_step()
                for _ in range(8):   # 8 sites per replay, as in 4 layers of a decode step
                    parts = comm.linear_reduce(x, w, "o")
                    ops.rmsnorm(parts, nw, 1e-6, residual=res, out=out)

            def nccl():
                for _ in range(8):
                    y = ops.linear(x, w)
                    dist.all_reduce(y)
                    ops.rmsnorm([y], nw, 1e-6, residual=res, out=out)

            Tw, row0, cnt = comm.shard(T)
            res_own = torch.zeros(Tw, H, device="cuda").bfloat16()

            def rsag():
                comm.begin_step()
                for _ in range(8):
                    parts = comm.rs_linear(x, w, "o")
                    _, ag = comm.norm_ag(parts, nw, 1e-6, res_own)
                    ag.wait()

            def local():
                for _ in range(8):
                    y = ops.linear(x, w)
                    ops.rmsnorm([y], nw, 1e-6, residual=res, out=out)

            row = {"site": name, "T": T, "world": world, "K_shard": K}
            variants = [("lamport", lamport), ("fused", fused), ("rsag", rsag), ("nccl", nccl), ("local", local)]
            if comm.mc is not None:
                variants.insert(0, ("lamport_nvls", lamport_nvls))
            for label, fn in variants:
                for _ in range(3):
                    fn()
                torch.cuda.synchronize()
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g):
                    fn()
                for _ in range(3):
                    g.replay()
                dist.barrier()
                torch.cuda.synchronize()
                s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                iters = 20
                s.record()
                for _ in range(iters):
                    g.replay()
                e.record()
                torch.cuda.synchronize()
                ms = max_over_ranks(s.elapsed_time(e) / iters / 8)
                row[label + "_us"] = round(ms * 1e3, 2)
                del g
            wbytes = H * K * 2
            nv_bytes = (world - 1) * T * H * 2
            roof_us = max(wbytes / (hbm * 1e3), nv_bytes / (NVLINK_GBPS * 1e3)) if world > 1 else wbytes / (hbm * 1e3)
            row["roofline_us"] = round(roof_us, 2)
            rs_bytes = 2 * (world - 1) * (-(-T // world)) * H * 2
            row["rsag_roofline_us"] = round(max(wbytes / (hbm * 1e3), rs_bytes / (NVLINK_GBPS * 1e3)), 2)
            row["fused_frac_of_roofline"] = round(roof_us / row["fused_us"], 3)
            row["lamport_frac_of_roofline"] = round(roof_us / row["lamport_us"], 3)
            if "lamport_nvls_us" in row:
                # NVLS: every tile crosses the sender's NVLink once; the switch fans it out
                mc_roof = max(wbytes / (hbm * 1e3), T * H * 2 / (NVLINK_GBPS * 1e3))
                row["nvls_roofline_us"] = round(mc_roof, 2)
                row["lamport_nvls_frac_of_roofline"] = round(mc_roof / row["lamport_nvls_us"], 3)
            row["speedup_vs_nccl"] = round(row["nccl_us"] / row["fused_us"], 3)
            row["peaks"] = src
            results.append(row)
            if rank == 0:
                print(json.dumps(row), flush=True)
    comm.check()
    comm.close()
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
