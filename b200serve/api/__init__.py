"""OpenAI-compatible HTTP API."""
