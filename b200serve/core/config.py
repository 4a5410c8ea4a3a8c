"""Runtime configuration (reference: core/config.py).

Keeps the reference's getter/setter names (``get_active_backend``,
``set_active_backend``, ``get_turboquant_kv``, ``get_context_profile`` ...)
under one lock, and adds one typed ``EngineConfig`` that describes the B200
engine: model, parallelism, KV format and batch limits. ``EngineConfig`` is
settable from environment variables (``B200_*``), a JSON file and the CLI.
"""

from __future__ import annotations

import dataclasses
import json
import logging
import os
import threading
from dataclasses import dataclass, field

_log = logging.getLogger(__name__)

BASE_DIR = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
SESSION_DIR = os.environ.get("B200_SESSION_DIR", os.path.join(BASE_DIR, "sessions"))
MODELS_DIR = os.environ.get("B200_MODELS_DIR", os.path.join(BASE_DIR, "models"))
TRUST_REMOTE_CODE = os.environ.get("ARTIFEX_TRUST_REMOTE_CODE", "").strip() == "1"

_config_lock = threading.Lock()

BACKENDS = ("b200", "transformers", "llama_cpp", "ollama", "claude_cli", "webgpu")
_active_backend = os.environ.get("ARTIFEX_BACKEND", "b200")


def get_active_backend() -> str:
    return _active_backend


def set_active_backend(name: str) -> bool:
    global _active_backend
    with _config_lock:
        if name not in BACKENDS:
            return False
        _active_backend = name
    return True


# ----- inference switches (same names as the reference) -----
_cuda_graphs = True
_turboquant_kv = False


def get_torch_compile() -> bool:
    """The reference's torch.compile switch; here it maps onto CUDA-graph capture."""
    return _cuda_graphs


def set_torch_compile(enabled) -> bool:
    global _cuda_graphs
    with _config_lock:
        _cuda_graphs = bool(enabled)
    return True


def get_turboquant_kv() -> bool:
    return _turboquant_kv


def set_turboquant_kv(enabled) -> bool:
    global _turboquant_kv
    with _config_lock:
        _turboquant_kv = bool(enabled)
    return True


# ----- model registry: directories under MODELS_DIR plus built-in shapes -----
BUILTIN_MODELS = ("tiny-qwen2", "qwen3-8b", "qwen3-30b-a3b")


def scan_models(models_dir: str = None) -> dict:
    """name -> path for every model directory or .gguf file in ``models_dir``."""
    out = {}
    d = models_dir or MODELS_DIR
    if os.path.isdir(d):
        for name in sorted(os.listdir(d)):
            full = os.path.join(d, name)
            if name.startswith("."):
                continue
            if os.path.isdir(full) or name.endswith(".gguf"):
                out[name] = full
    return out


MODELS = scan_models()
_active_model = os.environ.get("B200_MODEL", "qwen3-8b")


def get_active_model_name() -> str:
    return _active_model


def set_active_model(name: str) -> bool:
    global _active_model
    with _config_lock:
        if name not in BUILTIN_MODELS and name not in MODELS and not os.path.exists(name):
            return False
        _active_model = name
    return True


def get_active_model_path():
    """Filesystem path of the active model, or None for a built-in random-init shape."""
    if _active_model in MODELS:
        return MODELS[_active_model]
    if os.path.exists(_active_model):
        return _active_model
    return None


def get_model_names() -> list:
    return list(BUILTIN_MODELS) + [m for m in MODELS if m not in BUILTIN_MODELS]


# ----- GPU tier (reference: core/config.py:606-650) -----
def _detect_gpu_tier() -> str:
    try:
        import torch
        if not torch.cuda.is_available():
            return "TIGHT"
        gb = torch.cuda.get_device_properties(0).total_memory / 1e9
    except Exception:
        return "TIGHT"
    if gb >= 20:
        return "ABUNDANT"
    if gb >= 14:
        return "COMFORTABLE"
    return "TIGHT"


_gpu_tier = None


def get_gpu_tier() -> str:
    global _gpu_tier
    if _gpu_tier is None:
        _gpu_tier = _detect_gpu_tier()
    return _gpu_tier


def get_gpu_count() -> int:
    try:
        import torch
        return torch.cuda.device_count()
    except Exception:
        return 0


_active_device = 0


def get_active_device() -> int:
    return _active_device


def set_active_device(idx: int) -> bool:
    global _active_device
    with _config_lock:
        _active_device = int(idx)
    return True


# ----- modes and context profiles (reference: core/config.py:678-790) -----
@dataclass
class ModeConfig:
    max_tokens: int
    temperature: float
    context_window: int
    enable_thinking: bool = True


_TIER_LIMITS = {"TIGHT": (2048, 6), "COMFORTABLE": (3072, 10), "ABUNDANT": (4096, 15)}


def get_modes() -> dict:
    mt, cw = _TIER_LIMITS[get_gpu_tier()]
    return {
        "ASSISTANT": ModeConfig(max_tokens=mt, temperature=0.7, context_window=cw),
        "CODE": ModeConfig(max_tokens=min(mt * 2, 8192), temperature=0.2, context_window=cw),
    }


@dataclass
class ContextProfile:
    max_total_input_tokens: int
    max_output_tokens: int
    max_history_tokens: int
    knowledge_token_budget: int
    workspace_token_budget: int
    session_map_token_budget: int
    tool_output_limit: int
    read_chunk_size: int


CONTEXT_PROFILES = {
    "STANDARD": ContextProfile(10000, 1536, 6000, 550, 300, 250, 5000, 4000),
    "HIGH": ContextProfile(14000, 2048, 10000, 750, 400, 400, 6000, 6000),
}
_DEFAULT_PROFILES = {"TIGHT": "STANDARD", "COMFORTABLE": "STANDARD", "ABUNDANT": "HIGH"}
_active_profile = None


def get_context_profile_name() -> str:
    if _active_profile is None:
        return _DEFAULT_PROFILES.get(get_gpu_tier(), "STANDARD")
    return _active_profile


def get_context_profile() -> ContextProfile:
    return CONTEXT_PROFILES[get_context_profile_name()]


def set_context_profile(name: str) -> bool:
    global _active_profile
    with _config_lock:
        if name not in CONTEXT_PROFILES:
            return False
        _active_profile = name
    return True


# ----- the B200 engine configuration -----
@dataclass
class EngineConfig:
    """Everything the B200 engine needs to build a model replica.

    model        built-in shape name (tiny-qwen2, qwen3-8b, qwen3-30b-a3b), an HF
                 safetensors directory, or a .gguf file
    weights      "random" (N(0, init_std) from ``seed``), "safetensors" or "gguf"
    tp_size      tensor-parallel ranks (1/2/4/8); ep_size: expert-parallel ranks
    kv_format    "bf16", "int4g128" (4-bit K/V with fp16 scale per 128 values) or
                 "turboquant" (WHT + Lloyd-Max codes, ``kv_key_bits``/``kv_value_bits``;
                 ``kv_boundary_layers`` N keeps the first and last N attention layers in bf16;
                 ``kv_residual_tokens`` R keeps each sequence's newest R..R+15 tokens (whole
                 16-token pages) in bf16 beside their codes; the reference's default is 128)
    kv_block     tokens per KV page
    max_batch    most sequences decoded together (CUDA-graph buckets up to this)
    max_seq      longest sequence (prompt + completion) accepted; 0 = the largest context
                 tier whose KV fits (core/ctx_planner.py)
    kv_blocks    KV pages to allocate (0 = size from ``kv_mem_fraction`` of free memory)
    comm         "fused" (in-kernel NVLink P2P) or "nccl" (library collectives)
    spec_ngram   draft tokens per step for n-gram speculative decoding of greedy
                 requests (0 = off): the longest recent n-gram match in the request's
                 own tokens proposes a continuation, one forward verifies it
    spec_mtp     speculative decoding with the checkpoint's MTP head (models/mtp.py; random
                 weights get a random head): one draft per step, verified like the n-gram
                 drafts; single-rank attention-only models
    shard_cache  directory of pre-sharded per-rank weights (models/shard_cache.py): a
                 valid cache is read instead of the checkpoint, otherwise it is written
    step_timeout_s  watchdog: a forward step running longer fails the requests it holds
                 (their streams end with an error) and marks the engine stalled (0 = off)
    quantize     "" or "q4_k_m": quantise a bf16 checkpoint's projections to 4-bit blocks while
                 loading (GPU only; the counterpart of loading an HF model in 4 bits)
    """

    model: str = "qwen3-8b"
    weights: str = "random"
    seed: int = 0
    init_std: float = 0.02
    dtype: str = "bfloat16"
    tp_size: int = 1
    ep_size: int = 1
    kv_format: str = "bf16"
    kv_key_bits: int = 4
    kv_value_bits: int = 4
    kv_boundary_layers: int = 0
    kv_residual_tokens: int = 0
    kv_block: int = 16
    max_batch: int = 64
    max_seq: int = 4096
    kv_blocks: int = 0
    kv_mem_fraction: float = 0.85
    prefill_chunk: int = 8192
    cuda_graphs: bool = True
    use_kernels: bool = True
    comm: str = "fused"
    device: str = "cuda"
    num_layers_override: int = 0
    spec_ngram: int = 0
    spec_mtp: bool = False
    shard_cache: str = ""
    step_timeout_s: float = 600.0
    quantize: str = ""
    extra: dict = field(default_factory=dict)

    @classmethod
    def from_env(cls, base: "EngineConfig" = None) -> "EngineConfig":
        cfg = dataclasses.replace(base) if base else cls()
        for f in dataclasses.fields(cls):
            key = "B200_" + f.name.upper()
            if key in os.environ and f.name != "extra":
                setattr(cfg, f.name, _coerce(f.type, os.environ[key], getattr(cfg, f.name)))
        return cfg

    @classmethod
    def from_json(cls, path: str) -> "EngineConfig":
        with open(path) as fh:
            data = json.load(fh)
        names = {f.name for f in dataclasses.fields(cls)}
        unknown = set(data) - names
        if unknown:
            raise ValueError(f"unknown EngineConfig keys: {sorted(unknown)}")
        return cls(**data)

    def to_dict(self) -> dict:
        return dataclasses.asdict(self)

    def validate(self) -> "EngineConfig":
        if self.tp_size not in (1, 2, 4, 8):
            raise ValueError("tp_size must be 1, 2, 4 or 8")
        if self.kv_format not in ("bf16", "int4g128", "turboquant"):
            raise ValueError(f"unknown kv_format {self.kv_format!r}")
        if self.kv_block != 16:
            raise ValueError("kv_block must be 16 (the attention kernels are written for 16-token pages)")
        if self.comm not in ("fused", "nccl"):
            raise ValueError("comm must be 'fused' or 'nccl'")
        if not (1 <= self.kv_key_bits <= 4 and 1 <= self.kv_value_bits <= 4):
            raise ValueError("TurboQuant bits must be 1..4")
        return self


def _coerce(typ, text, current):
    kind = type(current)
    if kind is bool:
        return text.strip().lower() in ("1", "true", "yes", "on")
    if kind is int:
        return int(text)
    if kind is float:
        return float(text)
    return text


_engine_config = None


def get_engine_config() -> EngineConfig:
    global _engine_config
    if _engine_config is None:
        _engine_config = EngineConfig.from_env(EngineConfig(model=_active_model))
    return _engine_config


def set_engine_config(cfg: EngineConfig) -> None:
    global _engine_config
    with _config_lock:
        _engine_config = cfg.validate()


def add_engine_cli_args(parser) -> None:
    """Add one ``--<field>`` option per EngineConfig field to an argparse parser."""
    for f in dataclasses.fields(EngineConfig):
        if f.name == "extra":
            continue
        default = f.default
        flag = "--" + f.name.replace("_", "-")
        if isinstance(default, bool):
            parser.add_argument(flag, type=lambda s: s.lower() in ("1", "true", "yes", "on"), default=None)
        else:
            parser.add_argument(flag, type=type(default), default=None)


def engine_config_from_args(args, base: EngineConfig = None) -> EngineConfig:
    cfg = dataclasses.replace(base) if base else EngineConfig.from_env()
    for f in dataclasses.fields(EngineConfig):
        v = getattr(args, f.name, None)
        if v is not None:
            setattr(cfg, f.name, v)
    return cfg.validate()
