"""Tools an agent (or a server-side chat tool round) can call, with OpenAI function schemas
(reference: tools/agent_tools.py, api/web_tools.py).

``ToolBox`` holds the tools, exposes their schemas for the chat template, and runs a call
through the sandbox: policy decision, then the tool, then the outcome recorded (circuit
breaker, audit log). Tool results are text, truncated to ``max_output`` characters.

Built-in tools: read_file, write_file, edit_file, list_dir, glob, grep (files inside the
workspace jail), python and shell (subprocess in the workspace, time-limited), sysinfo,
web_search and web_read (through an injectable fetcher and search backend, host-checked by
the egress allowlist), knowledge_search (a Knowledge store, when one is attached).
"""

from __future__ import annotations

import fnmatch
import json
import os
import re
import subprocess
import sys
from dataclasses import dataclass
from typing import Callable, Optional

from b200serve.agent.sandbox import Sandbox


@dataclass
class Tool:
    name: str
    description: str
    params: dict                       # JSON-schema properties
    required: tuple
    fn: Callable                       # (toolbox, **args) -> str
    action: Optional[str] = None       # sandbox action name (default: the tool name)
    content_arg: Optional[str] = None  # argument the policy inspects (e.g. the shell command)

    def schema(self) -> dict:
        return {"type": "function", "function": {
            "name": self.name, "description": self.description,
            "parameters": {"type": "object", "properties": self.params, "required": list(self.required)}}}


class ToolError(Exception):
    pass


def _http_get(url: str, timeout: float = 20.0) -> str:
    import urllib.request
    req = urllib.request.Request(url, headers={"User-Agent": "b200serve-agent/1.0"})
    with urllib.request.urlopen(req, timeout=timeout) as r:      # noqa: S310 (host checked by egress)
        raw = r.read(2 << 20)
        return raw.decode(r.headers.get_content_charset() or "utf-8", errors="replace")


def html_to_text(html: str) -> str:
    html = re.sub(r"(?is)<(script|style|noscript)[^>]*>.*?</\1>", " ", html)
    html = re.sub(r"(?i)<br\s*/?>|</p>|</div>|</li>|</h\d>", "\n", html)
    text = re.sub(r"<[^>]+>", " ", html)
    for a, b in (("&nbsp;", " "), ("&amp;", "&"), ("&lt;", "<"), ("&gt;", ">"), ("&quot;", '"'), ("&#39;", "'")):
        text = text.replace(a, b)
    lines = [" ".join(ln.split()) for ln in text.splitlines()]
    return "\n".join(ln for ln in lines if ln)


class ToolBox:
    def __init__(self, sandbox: Sandbox, fetch: Callable = None, search: Callable = None, knowledge=None,
                 max_output: int = 12000, timeout_s: float = 60.0, enabled=None):
        self.sandbox = sandbox
        self.fetch = fetch or _http_get
        self.search = search
        self.knowledge = knowledge
        self.max_output, self.timeout_s = max_output, timeout_s
        self.tools = {t.name: t for t in _builtin_tools()}
        if knowledge is None:
            self.tools.pop("knowledge_search")
        if enabled is not None:
            self.tools = {n: t for n, t in self.tools.items() if n in set(enabled)}

    def schemas(self) -> list:
        return [t.schema() for t in self.tools.values()]

    def register(self, tool: Tool):
        self.tools[tool.name] = tool

    def call(self, name: str, arguments) -> dict:
        """Run one tool call: {"ok", "output", "decision"}. Never raises for tool failures."""
        tool = self.tools.get(name)
        if tool is None:
            return {"ok": False, "output": f"error: unknown tool {name!r}", "decision": "deny"}
        if isinstance(arguments, str):
            try:
                arguments = json.loads(arguments or "{}")
            except json.JSONDecodeError as e:
                return {"ok": False, "output": f"error: arguments are not JSON ({e})", "decision": "deny"}
        missing = [r for r in tool.required if r not in arguments]
        if missing:
            return {"ok": False, "output": f"error: missing argument(s) {missing}", "decision": "deny"}
        action = tool.action or tool.name
        content = str(arguments.get(tool.content_arg, "")) if tool.content_arg else json.dumps(arguments)[:500]
        d = self.sandbox.check(action, content)
        if not d.allowed:
            return {"ok": False, "output": f"denied by policy: {d.reason}", "decision": d.verdict}
        try:
            out = tool.fn(self, **arguments)
            ok = True
        except (ToolError, PermissionError, OSError, ValueError, subprocess.SubprocessError) as e:
            out, ok = f"error: {e}", False
        self.sandbox.record(action, ok, out[:200])
        if len(out) > self.max_output:
            out = out[: self.max_output] + f"\n[... {len(out) - self.max_output} more characters]"
        return {"ok": ok, "output": out, "decision": "allow"}


# ------------------------------------------------------------------ built-in tools
def _read_file(tb, path, offset=0, limit=400):
    p = tb.sandbox.jail.resolve(path)
    with open(p, encoding="utf-8", errors="replace") as fh:
        lines = fh.readlines()
    offset, limit = max(0, int(offset)), max(1, int(limit))
    body = "".join(f"{i + 1:6d}\t{ln}" for i, ln in enumerate(lines[offset:offset + limit], start=offset))
    more = len(lines) - offset - limit
    return body + (f"\n[{more} more lines]" if more > 0 else "")


def _write_file(tb, path, content):
    p = tb.sandbox.jail.resolve(path)
    os.makedirs(os.path.dirname(p), exist_ok=True)
    tmp = p + ".tmp-agent"
    with open(tmp, "w", encoding="utf-8") as fh:
        fh.write(content)
    os.replace(tmp, p)
    return f"wrote {len(content)} characters to {os.path.relpath(p, tb.sandbox.jail.roots[0])}"


def _edit_file(tb, path, old, new, replace_all=False):
    p = tb.sandbox.jail.resolve(path)
    with open(p, encoding="utf-8") as fh:
        text = fh.read()
    n = text.count(old)
    if n == 0:
        raise ToolError("the text to replace was not found")
    if n > 1 and not replace_all:
        raise ToolError(f"the text to replace occurs {n} times; pass more context or replace_all")
    text = text.replace(old, new) if replace_all else text.replace(old, new, 1)
    with open(p, "w", encoding="utf-8") as fh:
        fh.write(text)
    return f"replaced {n if replace_all else 1} occurrence(s)"


def _list_dir(tb, path="."):
    p = tb.sandbox.jail.resolve(path)
    rows = []
    for name in sorted(os.listdir(p)):
        full = os.path.join(p, name)
        rows.append(name + ("/" if os.path.isdir(full) else f"  ({os.path.getsize(full)} B)"))
    return "\n".join(rows) or "(empty)"


def _walk(tb, root):
    base = tb.sandbox.jail.resolve(root)
    for d, dirs, files in os.walk(base):
        dirs[:] = [x for x in dirs if not x.startswith(".") and x not in ("node_modules", "__pycache__")]
        for f in files:
            yield os.path.join(d, f)


def _glob(tb, pattern, path="."):
    ws = tb.sandbox.jail.roots[0]
    hits = [os.path.relpath(f, ws) for f in _walk(tb, path) if fnmatch.fnmatch(os.path.relpath(f, ws), pattern)
            or fnmatch.fnmatch(os.path.basename(f), pattern)]
    return "\n".join(sorted(hits)[:500]) or "(no matches)"


def _grep(tb, pattern, path=".", glob="*"):
    rx = re.compile(pattern)
    ws = tb.sandbox.jail.roots[0]
    out = []
    for f in _walk(tb, path):
        if not fnmatch.fnmatch(os.path.basename(f), glob):
            continue
        try:
            with open(f, encoding="utf-8", errors="strict") as fh:
                for i, ln in enumerate(fh, 1):
                    if rx.search(ln):
                        out.append(f"{os.path.relpath(f, ws)}:{i}: {ln.rstrip()[:300]}")
                        if len(out) >= 300:
                            return "\n".join(out) + "\n[truncated]"
        except (UnicodeDecodeError, OSError):
            continue
    return "\n".join(out) or "(no matches)"


def _limits(cpu_s: int, mem_bytes: int, file_bytes: int):
    """Resource limits applied in the child before exec: CPU seconds, address space, file size."""
    def apply():
        import resource
        resource.setrlimit(resource.RLIMIT_CPU, (cpu_s, cpu_s))
        resource.setrlimit(resource.RLIMIT_AS, (mem_bytes, mem_bytes))
        resource.setrlimit(resource.RLIMIT_FSIZE, (file_bytes, file_bytes))
    return apply


def _run(tb, argv, stdin=None):
    r = subprocess.run(argv, cwd=tb.sandbox.jail.roots[0], input=stdin, capture_output=True, text=True,
                       timeout=tb.timeout_s, env={**os.environ, "PYTHONDONTWRITEBYTECODE": "1"},
                       preexec_fn=_limits(int(tb.timeout_s) + 1, 8 << 30, 256 << 20))
    out = r.stdout + (("\n[stderr]\n" + r.stderr) if r.stderr.strip() else "")
    return out + (f"\n[exit code {r.returncode}]" if r.returncode else "")


def _python(tb, code):
    return _run(tb, [sys.executable, "-I", "-c", code])


def _shell(tb, command):
    return _run(tb, ["/bin/bash", "-c", command])


def _sysinfo(tb):
    import platform
    info = {"python": platform.python_version(), "platform": platform.platform(), "cpus": os.cpu_count()}
    try:
        from b200serve.core.metrics import gpu_memory
        info["gpus"] = gpu_memory()
    except Exception:
        pass
    return json.dumps(info)


def _web_search(tb, query, max_results=5):
    if tb.search is None:
        raise ToolError("no search backend is configured (set ToolBox(search=...))")
    hits = tb.search(query, int(max_results))
    lines = []
    for i, h in enumerate(hits[: int(max_results)], 1):
        tb.sandbox.egress.check(h["url"])
        lines.append(f"[{i}] {h.get('title', '')}\n    {h['url']}\n    {h.get('snippet', '')}")
    return "\n".join(lines) or "(no results)"


def _web_read(tb, url, max_chars=8000):
    tb.sandbox.egress.check(url)
    raw = tb.fetch(url)
    text = html_to_text(raw) if "<" in raw[:2000] else raw
    return text[: int(max_chars)]


def _knowledge_search(tb, query, k=5):
    hits = tb.knowledge.search(query, int(k))
    return "\n\n".join(f"[{h['source']} #{h['chunk']}] (score {h['score']:.3f})\n{h['text']}" for h in hits) \
        or "(nothing relevant)"


def _builtin_tools():
    S, I, B = {"type": "string"}, {"type": "integer"}, {"type": "boolean"}
    return [
        Tool("read_file", "Read a text file of the workspace with line numbers.",
             {"path": S, "offset": I, "limit": I}, ("path",), _read_file),
        Tool("write_file", "Create or overwrite a workspace file with the given content.",
             {"path": S, "content": S}, ("path", "content"), _write_file),
        Tool("edit_file", "Replace an exact piece of text in a workspace file.",
             {"path": S, "old": S, "new": S, "replace_all": B}, ("path", "old", "new"), _edit_file),
        Tool("list_dir", "List a workspace directory.", {"path": S}, (), _list_dir),
        Tool("glob", "Find workspace files whose path matches a glob pattern.", {"pattern": S, "path": S},
             ("pattern",), _glob),
        Tool("grep", "Search workspace files for a regular expression.", {"pattern": S, "path": S, "glob": S},
             ("pattern",), _grep),
        Tool("python", "Run a Python snippet in the workspace and return its output.", {"code": S}, ("code",),
             _python, content_arg="code"),
        Tool("shell", "Run a bash command in the workspace and return its output.", {"command": S},
             ("command",), _shell, content_arg="command"),
        Tool("sysinfo", "Describe this machine (Python, OS, CPUs, GPUs).", {}, (), _sysinfo),
        Tool("web_search", "Search the web; returns titles, URLs and snippets.", {"query": S, "max_results": I},
             ("query",), _web_search, content_arg="query"),
        Tool("web_read", "Fetch a web page and return its text.", {"url": S, "max_chars": I}, ("url",),
             _web_read, content_arg="url"),
        Tool("knowledge_search", "Search the local knowledge base for passages relevant to a query.",
             {"query": S, "k": I}, ("query",), _knowledge_search, content_arg="query"),
    ]
