"""Decoder models (Qwen2/Qwen3 dense, Qwen3-MoE) and their weight loaders."""

from b200serve.models.config import ModelConfig, get_model_config  # noqa: F401
