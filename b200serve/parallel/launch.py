"""Tensor-parallel serving launch: run under torchrun with one rank per GPU.

  torchrun --nproc-per-node 8 --master-addr 127.0.0.1 -m b200serve.api.server --tp-size 8

Every rank builds its shard of the model; rank 0 serves HTTP and runs the
scheduler, the other ranks execute the broadcast steps (parallel/worker.py).
"""

from __future__ import annotations

import logging

_log = logging.getLogger(__name__)


def serve_tp(cfg, host, port, create_app):
    from b200serve.engine.b200_engine import B200Engine
    from b200serve.parallel.dist import init_distributed, rank_world
    from b200serve.parallel.worker import worker_loop
    init_distributed()
    rank, world = rank_world()
    eng = B200Engine(cfg)
    eng.load()
    if rank != 0:
        worker_loop(eng.runner.inner, eng.comm)
        return
    import uvicorn
    try:
        uvicorn.run(create_app(engine=eng), host=host, port=port, log_level="info")
    finally:
        eng.unload()
