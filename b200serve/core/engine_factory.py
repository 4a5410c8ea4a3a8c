"""Backend name -> engine instance (reference: core/engine_factory.py:13-54).

The reference dispatches to external runtimes (transformers, llama.cpp,
Ollama, Claude CLI, WebGPU). Here the only in-process backend is ``b200``,
which owns the decoder forward on Blackwell GPUs. The other names are kept
as recognised backend strings so configuration written for Artifex still
parses, and resolve to the b200 engine (there is exactly one local compute
path in this framework).
"""

from b200serve.core.config import get_active_backend, get_engine_config

KNOWN_BACKENDS = ("b200", "transformers", "llama_cpp", "ollama", "claude_cli", "webgpu")


def create_engine(config=None):
    """Create an engine for the active backend.

    ``config`` (an ``EngineConfig``) overrides the process-wide one.
    """
    backend = get_active_backend()
    if backend not in KNOWN_BACKENDS:
        raise RuntimeError(f"unknown backend {backend!r}")
    from b200serve.engine.b200_engine import B200Engine
    return B200Engine(config or get_engine_config())
