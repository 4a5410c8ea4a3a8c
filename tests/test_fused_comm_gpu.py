"""Fused tensor-parallel all-reduce over NVLink P2P (needs >= 2 GPUs).

Each rank runs the push-GEMM (epilogue stores tiles into every rank's receive
slot and raises flags) and the flag-waiting add+RMSNorm; the result must equal
an NCCL all-reduce of the same partial GEMM outputs followed by the same norm,
over several steps (epochs and slot alternation)."""

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

needs2 = pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                            reason="needs 2 GPUs")


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _fused_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    import torch.distributed as dist
    from b200serve import ops
    from b200serve.core.config import EngineConfig
    from b200serve.models.config import BUILTIN
    from b200serve.parallel.dist import init_distributed
    from b200serve.parallel.fused_comm import FusedComm
    init_distributed("nccl", timeout_s=60)
    torch.cuda.set_device(rank)
    cfg = BUILTIN["qwen3-8b"]
    comm = FusedComm(dist.group.WORLD, torch.device("cuda", rank), cfg, EngineConfig(max_batch=32))
    g = torch.Generator(device="cuda").manual_seed(100 + rank)     # this rank's shard
    gs = torch.Generator(device="cuda").manual_seed(7)              # replicated tensors
    errs = []
    for step in range(6):
        comm.begin_step()
        for site in range(3):
            T = [32, 7, 1][site]
            x = torch.randn(T, 1536, device="cuda", generator=g).bfloat16()
            w = ops.pack_weight((torch.randn(4096, 1536, device="cuda", generator=g) * 0.03).bfloat16())
            res = torch.randn(T, 4096, device="cuda", generator=gs).bfloat16()
            nw = torch.randn(4096, device="cuda", generator=gs).bfloat16()
            comm.lamport = step % 3 != 2          # flag-free slots on most steps, flags on the rest
            comm.use_mc = comm.mc is not None and step % 2 == 0    # NVLS multicast push when offered
            parts = comm.linear_reduce(x, w, "o")
            if site == 1:                          # another launch between the GEMM and its norm
                y = ops.linear(x, w)
                out = ops.rmsnorm(parts, nw, 1e-6, residual=res)
            else:                                  # the norm directly follows the push GEMM
                out = ops.rmsnorm(parts, nw, 1e-6, residual=res)
                y = ops.linear(x, w)
            dist.all_reduce(y)
            ref = ops.rmsnorm([y], nw, 1e-6, residual=res)
            errs.append(((out.float() - ref.float()).norm() / ref.float().norm()).item())
            # every rank sums the partials in rank order: the outputs agree bit for bit
            outs = [torch.empty_like(out) for _ in range(world)]
            dist.all_gather(outs, out)
            if not all(torch.equal(outs[0], o) for o in outs):
                errs.append(1.0)
    torch.cuda.synchronize()
    comm.check()
    comm.close()
    q.put((rank, max(errs)))
    if rank == 0:
        print("multicast slots:", comm.mc is not None, flush=True)
    dist.barrier()
    dist.destroy_process_group()


@needs2
def test_fused_allreduce_matches_nccl():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    ps = [ctx.Process(target=_fused_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = dict(q.get(timeout=300) for _ in ps)
    for p in ps:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert max(res.values()) < 2e-2, res


def _tp_worker(rank, world, port, comm_kind, q, model="qwen3-8b", env=None):
    os.environ.update(env or {})
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    from b200serve.core.config import EngineConfig
    from b200serve.engine.b200_engine import B200Engine
    from b200serve.engine.sampler import SamplingParams
    from b200serve.parallel.worker import worker_loop
    moe = model != "qwen3-8b"
    graphs = (env or {}).get("B200_TEST_GRAPHS", "1") != "0"
    cfg = EngineConfig(model=model, num_layers_override=2, tp_size=world, ep_size=world if moe else 1,
                       comm=comm_kind, max_batch=8, max_seq=512, kv_blocks=256, cuda_graphs=graphs)
    eng = B200Engine(cfg)
    eng.load()
    if rank == 0:
        g = torch.Generator().manual_seed(0)
        prompts = [torch.randint(0, 150000, (n,), generator=g).tolist() for n in (40, 100, 7)]
        reqs = eng.generate(prompts, SamplingParams(temperature=0.0, max_tokens=12, ignore_eos=True), timeout=300)
        q.put([r.output for r in reqs])
        eng.stop_loop()
    else:
        worker_loop(eng.runner.inner, eng.comm)
    import torch.distributed as dist
    eng.runner.inner.release_graphs()
    dist.barrier()
    dist.destroy_process_group()


def _run_tp(kind, model="qwen3-8b", env=None):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    ps = [ctx.Process(target=_tp_worker, args=(r, 2, port, kind, q, model, env)) for r in range(2)]
    for p in ps:
        p.start()
    out = q.get(timeout=600)
    for p in ps:
        p.join(timeout=120)
        assert p.exitcode == 0
    return out


@needs2
def test_tp2_fused_equals_nccl():
    # the two paths round the cross-rank sum differently (fp32 sum of bf16
    # partials vs NCCL's bf16 result), so only the first greedy tokens are
    # required to agree exactly
    a, b = _run_tp("fused"), _run_tp("nccl")
    assert [x[:4] for x in a] == [x[:4] for x in b]


def _rsag_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    import torch.distributed as dist
    from b200serve import ops
    from b200serve.core.config import EngineConfig
    from b200serve.models.config import BUILTIN
    from b200serve.parallel.dist import init_distributed
    from b200serve.parallel.fused_comm import FusedComm
    init_distributed("nccl", timeout_s=60)
    torch.cuda.set_device(rank)
    cfg = BUILTIN["qwen3-8b"]
    comm = FusedComm(dist.group.WORLD, torch.device("cuda", rank), cfg,
                     EngineConfig(max_batch=32, prefill_chunk=1024))
    g = torch.Generator(device="cuda").manual_seed(200 + rank)
    gs = torch.Generator(device="cuda").manual_seed(7)          # same on every rank
    errs = []
    for step in range(4):
        comm.begin_step()
        for T in (37, 300, 1040):
            x = torch.randn(T, 1536, device="cuda", generator=g).bfloat16()
            w = ops.pack_weight((torch.randn(4096, 1536, device="cuda", generator=gs) * 0.03).bfloat16())
            w2 = ops.pack_weight((torch.randn(1024, 4096, device="cuda", generator=gs) * 0.03).bfloat16())
            res = torch.randn(T, 4096, device="cuda", generator=gs).bfloat16()
            nw = torch.randn(4096, device="cuda", generator=gs).bfloat16()
            Tw, row0, cnt = comm.shard(T)
            res_own = torch.zeros(Tw, 4096, dtype=torch.bfloat16, device="cuda")
            res_own[:cnt] = res[row0:row0 + cnt]
            parts = comm.rs_linear(x, w, "o")
            xf, ag = comm.norm_ag(parts, nw, 1e-6, res_own)
            y2 = ops.linear(xf, w2, ag=ag)
            y = ops.linear(x, w)
            dist.all_reduce(y)
            res_ref = res.clone()
            ref = ops.rmsnorm([y], nw, 1e-6, residual=res, residual_out=res_ref)
            ref2 = ops.linear(ref, w2)
            errs.append(((y2.float() - ref2.float()).norm() / ref2.float().norm()).item())
            errs.append(((res_own[:cnt].float() - res_ref[row0:row0 + cnt].float()).norm()
                         / res_ref[row0:row0 + cnt].float().norm()).item())
    torch.cuda.synchronize()
    comm.check()
    comm.close()
    q.put((rank, max(errs)))
    if rank == 0:
        print("multicast slots:", comm.mc is not None, flush=True)
    dist.barrier()
    dist.destroy_process_group()


@needs2
def test_fused_reduce_scatter_all_gather_matches_nccl():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    ps = [ctx.Process(target=_rsag_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = dict(q.get(timeout=300) for _ in ps)
    for p in ps:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert max(res.values()) < 3e-2, res


@needs2
def test_tp2_rsag_equals_nccl():
    os.environ["B200_TP_MODE"] = "rsag"
    try:
        a = _run_tp("fused")
    finally:
        os.environ.pop("B200_TP_MODE", None)
    b = _run_tp("nccl")
    assert [x[:4] for x in a] == [x[:4] for x in b]


def _moe_combine_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    import torch.distributed as dist
    from b200serve import ops
    from b200serve.core.config import EngineConfig
    from b200serve.models.config import BUILTIN
    from b200serve.parallel.dist import init_distributed
    from b200serve.parallel.fused_comm import FusedComm
    init_distributed("nccl", timeout_s=60)
    torch.cuda.set_device(rank)
    cfg = BUILTIN["qwen3-30b-a3b"]
    comm = FusedComm(dist.group.WORLD, torch.device("cuda", rank), cfg, EngineConfig(max_batch=32))
    g = torch.Generator(device="cuda").manual_seed(300 + rank)
    H, k, errs = cfg.hidden_size, 8, []
    for step in range(4):
        comm.begin_step()
        for T in (1, 13, 32):
            rows = T * k
            y = torch.randn(rows, H, device="cuda", generator=g).bfloat16()
            wts = torch.rand(T, k, device="cuda", generator=g)
            pos = torch.randperm(rows, device="cuda", generator=g).int().view(T, k)
            pos[:, ::3] = -1                                       # slots owned by the other rank
            nw = torch.randn(H, device="cuda", generator=g).bfloat16()
            res = torch.randn(T, H, device="cuda", generator=g).bfloat16()
            parts = comm.moe_combine_reduce(y, wts, pos, k, T)
            out = ops.rmsnorm(parts, nw, 1e-6, residual=res)
            loc = torch.empty(T, H, device="cuda").bfloat16()
            ops.ext().moe_combine(y, wts, pos, k, loc)
            dist.all_reduce(loc)
            ref = ops.rmsnorm([loc], nw, 1e-6, residual=res)
            errs.append(((out.float() - ref.float()).norm() / ref.float().norm()).item())
    torch.cuda.synchronize()
    comm.check()
    comm.close()
    q.put((rank, max(errs)))
    if rank == 0:
        print("multicast slots:", comm.mc is not None, flush=True)
    dist.barrier()
    dist.destroy_process_group()


@needs2
def test_fused_moe_combine_matches_nccl():
    """Expert-parallel combine kernel with the NVLink push + flags vs local combine + NCCL."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    ps = [ctx.Process(target=_moe_combine_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = dict(q.get(timeout=300) for _ in ps)
    for p in ps:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert max(res.values()) < 2e-2, res


@needs2
def test_ep2_moe_fused_combine_engine():
    """Engine with expert parallelism over 2 GPUs: the fused combine and NCCL agree on the
    prefill token and the first decode token (random-init MoE routing amplifies rounding
    differences in later steps)."""
    a, b = _run_tp("fused", "qwen3-30b-a3b"), _run_tp("nccl", "qwen3-30b-a3b")
    assert [x[:2] for x in a] == [x[:2] for x in b]


@needs2
def test_ep2_all_to_all_matches_replicated():
    """Token-sharded expert parallelism over NVLink (count broadcast, rows pushed into the
    owners' expert-sorted buffers, grouped GEMM waiting for them in-kernel, weighted rows pushed
    back by the down GEMM's epilogue) against the replicated-token path, on every step (eager
    steps: the all-to-all reads the exchanged counts on the host, so captured steps stay
    replicated)."""
    a = _run_tp("fused", "qwen3-30b-a3b", {"B200_EP_MODE": "a2a", "B200_TEST_GRAPHS": "0"})
    b = _run_tp("fused", "qwen3-30b-a3b", {"B200_EP_MODE": "replicated", "B200_TEST_GRAPHS": "0"})
    assert [x[:2] for x in a] == [x[:2] for x in b]
