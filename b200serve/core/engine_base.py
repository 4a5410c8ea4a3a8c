"""The engine contract every backend implements.

Same method set and keyword names as the reference's ``BaseEngine``
(core/engine_base.py:9-91), so callers written against Artifex (the API
server, the agent loop, pipelines) drive this framework unchanged.
"""

from abc import ABC, abstractmethod


class BaseEngine(ABC):
    """Unified engine interface for model loading and streaming generation.

    ``stream_starts_in_think`` tells the API server's ThinkFilter whether the
    token stream begins inside a ``<think>`` block (chat templates that
    pre-fill ``<think>``) or emits explicit tags inline.
    """

    stream_starts_in_think: bool = True

    @abstractmethod
    def load(self, status_callback=None):
        """Load the model (no-op when already loaded)."""

    @abstractmethod
    def unload(self, status_callback=None):
        """Release the model and its device memory."""

    @abstractmethod
    def is_loaded(self) -> bool:
        """True once the model can serve requests."""

    @abstractmethod
    def needs_reload(self) -> bool:
        """True when the configured model differs from the loaded one."""

    @abstractmethod
    def periodic_cleanup(self):
        """Light housekeeping between generations."""

    def get_context_size(self) -> int:
        """Maximum context in tokens (0 = unknown)."""
        return 0

    @abstractmethod
    def count_tokens(self, text: str) -> int:
        """Number of tokens ``text`` encodes to."""

    @abstractmethod
    def generate_streaming(self, messages, max_tokens, temperature,
                           on_token=None, on_complete=None,
                           enable_thinking=True,
                           grammar=None, response_format=None,
                           web_tools=False,
                           reasoning_effort=None,
                           on_telemetry=None,
                           sampling=None) -> str:
        """Stream a completion for ``messages``.

        ``on_token(str)`` receives each decoded text piece (thinking included),
        ``on_complete(str)`` the cleaned final answer, which is also returned.
        ``sampling`` is a fully explicit sampler dict (see core.sampling); its
        ``temperature`` overrides the positional argument. Options a backend
        does not implement (grammar, web_tools, reasoning_effort) are accepted
        and ignored.
        """
