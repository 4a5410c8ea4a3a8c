"""b200serve: a Blackwell (sm_100a) local-LLM serving engine.

Layers (top to bottom):
  api/       OpenAI-compatible HTTP server (chat/completions, models, tokenize, health, queue, engine)
  core/      engine contract, factory, config, sampler presets, inference utilities, GGUF metadata,
             TurboQuant codec, request estimation, model queue, resilience, sessions, telemetry
  engine/    B200Engine: tokenizer, continuous-batching scheduler, paged KV manager, sampler, stats
  models/    Qwen2/Qwen3 dense and Qwen3-MoE decoders, weight loaders (safetensors, GGUF), TP/EP sharding
  parallel/  process-group bootstrap, IPC symmetric buffers, fused compute+collective kernels, heartbeat
  ops/       hand-written sm_100a CUDA kernels (tcgen05/TMEM GEMM, paged attention, norms, RoPE, sampling, ...)
  utils/     device timing (CUDA events, max over ranks), clock sampling
"""

__version__ = "0.1.0"
