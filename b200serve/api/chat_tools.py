"""Server-side tool rounds for chat completions (reference: api/server.py:1218-1571
``_stream_with_tools_impl``, api/web_tools.py, api/chat_tools.py).

With ``web_tools: true`` the server itself runs the model's web_search / web_read (and
knowledge_search, when a knowledge base is attached) calls for up to ``max_rounds`` rounds,
feeding the results back, and returns only the final answer. Tool progress is streamed as
``x_tool`` SSE events. Network access goes through the sandbox's egress allowlist
(B200_EGRESS_ALLOW); the search backend is a JSON endpoint in B200_SEARCH_URL
(``GET <url>?q=...&format=json`` -> {"results": [{title, url, content}]}), or a callable a
caller installs with ``set_search_backend``.
"""

import json
import os
import tempfile
import urllib.parse

from b200serve.agent.loop import AgentConfig, AgentRunner
from b200serve.agent.sandbox import Sandbox
from b200serve.agent.tools import ToolBox, _http_get

_search_backend = None
_fetcher = None
_knowledge = None


def set_search_backend(fn):
    """fn(query, max_results) -> [{"title", "url", "snippet"}]"""
    global _search_backend
    _search_backend = fn


def set_fetcher(fn):
    global _fetcher
    _fetcher = fn


def set_knowledge(kb):
    global _knowledge
    _knowledge = kb


def _env_search(query, n):
    base = os.environ.get("B200_SEARCH_URL", "")
    if not base:
        raise RuntimeError("no web search backend configured (B200_SEARCH_URL)")
    url = base + ("&" if "?" in base else "?") + urllib.parse.urlencode({"q": query, "format": "json"})
    data = json.loads((_fetcher or _http_get)(url))
    return [{"title": r.get("title", ""), "url": r.get("url", ""), "snippet": r.get("content", "")}
            for r in data.get("results", [])[:n]]


def web_toolbox(workspace: str = None) -> ToolBox:
    sb = Sandbox(workspace or tempfile.mkdtemp(prefix="b200-chat-tools-"), level="permissive")
    enabled = ["web_search", "web_read"] + (["knowledge_search"] if _knowledge is not None else [])
    return ToolBox(sb, fetch=_fetcher, search=_search_backend or _env_search, knowledge=_knowledge, enabled=enabled)


def run_tool_rounds(engine, messages, max_tokens, temperature, on_tool=None, max_rounds: int = 4):
    """Answer ``messages`` with server-run tool rounds. Returns (answer, stats, n_tool_calls)."""
    def ev(e):
        if on_tool is not None and e.kind in ("tool_call", "tool_result"):
            on_tool(e.to_dict())
    system = next((m.get("content") for m in messages if m.get("role") == "system"), None)
    cfg = AgentConfig(max_rounds=max_rounds, max_tokens=max_tokens, temperature=temperature,
                      system_prompt=(system or "") + "\nYou can search the web and read pages with the tools; "
                                                     "answer directly when you know enough, citing the URLs used.")
    runner = AgentRunner(engine, web_toolbox(), cfg, on_event=ev)
    goal_idx = max((i for i, m in enumerate(messages) if m.get("role") == "user"), default=None)
    history = [m for m in messages if m.get("role") != "system"]
    goal = ""
    if goal_idx is not None:
        goal = messages[goal_idx].get("content") if isinstance(messages[goal_idx].get("content"), str) else ""
        history = [m for i, m in enumerate(messages) if m.get("role") != "system" and i != goal_idx]
    res = runner.run(goal, history)
    stats = dict(getattr(engine, "_last_gen_stats", None) or {})
    stats["tool_rounds"] = res.rounds
    return res.answer, stats, res.tool_calls
