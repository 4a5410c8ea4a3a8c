"""Execution policy for agent actions (reference: core/sandbox/policy.py and its helpers
fs_sandbox, egress, circuit_breaker, audit, human_gate).

Every tool call an agent makes goes through ``Sandbox.check(action, content)`` before it
runs and ``Sandbox.record(...)`` after. The decision combines:
  * a risk class per action (read-only file tools SAFE ... shell HIGH), raised for shell
    commands that do more than read (analysed segment by segment);
  * the policy level: strict (everything needs a human), moderate (reads run, writes and
    execution ask), permissive (only shell and downloads ask), auto (everything runs);
  * a filesystem jail: paths must resolve, symlinks included, inside the workspace roots;
  * an egress allowlist for network tools (host suffixes);
  * a circuit breaker: after ``max_failures`` consecutive failures of one action the
    action is refused until a cool-down passes;
  * an append-only JSONL audit log of every decision and outcome.
A "confirm" decision is resolved by the human-gate callback when one is installed (the
API's approval route), else treated as a denial. The policy names follow the reference
(ARTIFEX_POLICY / B200_POLICY = strict | moderate | permissive | auto).
"""

from __future__ import annotations

import json
import os
import shlex
import threading
import time
from dataclasses import dataclass, field
from enum import IntEnum
from typing import Callable, Optional
from urllib.parse import urlparse


class Risk(IntEnum):
    SAFE = 0
    LOW = 1
    MEDIUM = 2
    HIGH = 3
    CRITICAL = 4


# default risk of each built-in action
ACTION_RISK = {
    "read_file": Risk.SAFE, "list_dir": Risk.SAFE, "glob": Risk.SAFE, "grep": Risk.SAFE, "sysinfo": Risk.SAFE,
    "web_search": Risk.LOW, "web_read": Risk.LOW, "knowledge_search": Risk.SAFE,
    "write_file": Risk.MEDIUM, "edit_file": Risk.MEDIUM, "python": Risk.MEDIUM,
    "download": Risk.HIGH, "shell": Risk.HIGH,
}

# the highest risk each policy level runs without asking; above it the decision is "confirm"
LEVEL_LIMIT = {"strict": -1, "moderate": Risk.LOW, "permissive": Risk.MEDIUM, "auto": Risk.CRITICAL}

# commands that only read: a shell command made solely of these (no redirection into files,
# no command substitution) counts as LOW instead of HIGH
READ_ONLY_COMMANDS = frozenset({
    "ls", "cat", "head", "tail", "wc", "grep", "rg", "find", "pwd", "echo", "which", "file", "stat", "du",
    "df", "uname", "date", "whoami", "env", "printenv", "sort", "uniq", "cut", "tr", "diff", "tree",
    "nvidia-smi", "git",
})
READ_ONLY_GIT = frozenset({"status", "log", "diff", "show", "branch", "rev-parse", "ls-files", "blame"})
# never run, whatever the level
FORBIDDEN = ("rm -rf /", "mkfs", ":(){", "dd if=", "shutdown", "reboot", "chmod -R 777 /", "> /dev/sd")


def shell_segments(command: str) -> list:
    """Split a command line at ; && || | and newlines, outside quotes."""
    segs, cur, quote, i = [], [], None, 0
    while i < len(command):
        c = command[i]
        if quote:
            cur.append(c)
            if c == quote:
                quote = None
            elif c == "\\" and quote == '"' and i + 1 < len(command):
                cur.append(command[i + 1])
                i += 1
        elif c in "'\"":
            quote = c
            cur.append(c)
        elif c in ";|\n" or command.startswith("&&", i):
            if command.startswith("&&", i) or command.startswith("||", i):
                i += 1
            segs.append("".join(cur).strip())
            cur = []
        else:
            cur.append(c)
        i += 1
    segs.append("".join(cur).strip())
    return [s for s in segs if s]


def _segment_reads_only(seg: str) -> bool:
    if "$(" in seg or "`" in seg or ">" in seg.replace("2>&1", "").replace(">/dev/null", ""):
        return False
    try:
        words = shlex.split(seg)
    except ValueError:
        return False
    while words and "=" in words[0] and not words[0].startswith("="):
        words = words[1:]                       # VAR=value prefixes
    if not words:
        return True
    cmd = os.path.basename(words[0])
    if cmd not in READ_ONLY_COMMANDS:
        return False
    if cmd == "git":
        return len(words) > 1 and words[1] in READ_ONLY_GIT
    if cmd == "find":
        return not any(w in ("-delete", "-exec", "-execdir", "-ok") for w in words)
    return True


def shell_risk(command: str) -> Risk:
    low = command.lower()
    if any(f in low for f in FORBIDDEN):
        return Risk.CRITICAL
    segs = shell_segments(command)
    if segs and all(_segment_reads_only(s) for s in segs):
        return Risk.LOW
    return Risk.HIGH


def classify(action: str, content: str = "") -> Risk:
    if action == "shell":
        return shell_risk(content)
    return ACTION_RISK.get(action, Risk.HIGH)          # unknown actions are treated as dangerous


@dataclass
class Decision:
    verdict: str                 # "allow" | "deny" | "confirm"
    risk: Risk
    reason: str = ""

    @property
    def allowed(self) -> bool:
        return self.verdict == "allow"


def policy_level() -> str:
    lvl = (os.environ.get("B200_POLICY") or os.environ.get("ARTIFEX_POLICY") or "strict").strip().lower()
    if lvl == "auto" and not (os.environ.get("B200_AGENT_KEY") or os.environ.get("ARTIFEX_AGENT_KEY")):
        return "moderate"            # unattended execution must be unlocked explicitly
    return lvl if lvl in LEVEL_LIMIT else "strict"


class PathJail:
    """Resolves paths against workspace roots; a path (after following symlinks) outside
    every root is refused."""

    def __init__(self, roots):
        self.roots = [os.path.realpath(r) for r in roots]

    def resolve(self, path: str) -> str:
        base = self.roots[0]
        full = os.path.realpath(path if os.path.isabs(path) else os.path.join(base, path))
        for r in self.roots:
            if full == r or full.startswith(r.rstrip(os.sep) + os.sep):
                return full
        raise PermissionError(f"{path!r} is outside the workspace")


class Egress:
    """Host allowlist for network tools: a URL passes when its host equals an entry or ends
    with '.' + entry. An empty allowlist refuses every host; '*' allows any."""

    def __init__(self, allowed=None):
        env = os.environ.get("B200_EGRESS_ALLOW", "")
        self.allowed = [h.strip().lower() for h in (allowed if allowed is not None else env.split(",")) if h.strip()]

    def check(self, url: str):
        u = urlparse(url)
        host = (u.hostname or "").lower()
        if u.scheme not in ("http", "https") or not host:
            raise PermissionError(f"only http(s) URLs are fetched, not {url!r}")
        if "*" in self.allowed or any(host == h or host.endswith("." + h) for h in self.allowed):
            return
        raise PermissionError(f"host {host!r} is not on the egress allowlist")


class CircuitBreaker:
    def __init__(self, max_failures: int = 3, cooldown_s: float = 60.0):
        self.max_failures, self.cooldown_s = max_failures, cooldown_s
        self._fails = {}
        self._opened = {}

    def is_open(self, action: str) -> bool:
        t = self._opened.get(action)
        if t is None:
            return False
        if time.monotonic() - t >= self.cooldown_s:
            del self._opened[action]
            self._fails[action] = 0
            return False
        return True

    def record(self, action: str, ok: bool):
        if ok:
            self._fails[action] = 0
            return
        n = self._fails.get(action, 0) + 1
        self._fails[action] = n
        if n >= self.max_failures:
            self._opened[action] = time.monotonic()


class AuditLog:
    def __init__(self, path: str = None):
        self.path = path
        self.entries = []
        self._lock = threading.Lock()

    def write(self, **rec):
        rec.setdefault("t", round(time.time(), 3))
        with self._lock:
            self.entries.append(rec)
            if self.path:
                with open(self.path, "a", encoding="utf-8") as fh:
                    fh.write(json.dumps(rec, ensure_ascii=False, default=str) + "\n")


@dataclass
class Sandbox:
    workspace: str = "."
    level: Optional[str] = None
    extra_roots: list = field(default_factory=list)
    egress_allow: Optional[list] = None
    audit_path: Optional[str] = None
    human_gate: Optional[Callable] = None        # (action, content, risk) -> bool
    max_failures: int = 3

    def __post_init__(self):
        self.level = (self.level or policy_level()).lower()
        if self.level not in LEVEL_LIMIT:
            raise ValueError(f"unknown policy level {self.level!r}")
        os.makedirs(self.workspace, exist_ok=True)
        self.jail = PathJail([self.workspace] + list(self.extra_roots))
        self.egress = Egress(self.egress_allow)
        self.breaker = CircuitBreaker(self.max_failures)
        self.audit = AuditLog(self.audit_path)

    def decide(self, action: str, content: str = "") -> Decision:
        risk = classify(action, content)
        if risk >= Risk.CRITICAL:
            return Decision("deny", risk, "forbidden command")
        if self.breaker.is_open(action):
            return Decision("deny", risk, f"{action} failed repeatedly; paused")
        if risk <= LEVEL_LIMIT[self.level]:
            return Decision("allow", risk)
        return Decision("confirm", risk, f"{action} ({risk.name}) needs approval at policy {self.level}")

    def check(self, action: str, content: str = "") -> Decision:
        """The decision after the human gate (a "confirm" becomes allow or deny)."""
        d = self.decide(action, content)
        if d.verdict == "confirm":
            ok = bool(self.human_gate and self.human_gate(action, content, d.risk))
            d = Decision("allow" if ok else "deny", d.risk, "approved" if ok else (d.reason + "; not approved"))
        self.audit.write(event="decision", action=action, verdict=d.verdict, risk=d.risk.name, reason=d.reason,
                         content=content[:500])
        return d

    def record(self, action: str, ok: bool, detail: str = ""):
        self.breaker.record(action, ok)
        self.audit.write(event="result", action=action, ok=ok, detail=detail[:500])
