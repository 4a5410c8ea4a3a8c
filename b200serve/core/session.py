"""Conversation persistence as JSON files (reference: core/session.py:35-236)."""

from __future__ import annotations

import json
import os
import time

from b200serve.core import config

AUTO_SAVE_KEEP = 5


def _dir(session_dir=None):
    d = session_dir or config.SESSION_DIR
    os.makedirs(d, exist_ok=True)
    return d


def save_session(name, messages, session_map=None, metadata=None, session_dir=None) -> str:
    safe = "".join(c if c.isalnum() or c in "-_." else "_" for c in name) or "session"
    path = os.path.join(_dir(session_dir), safe + ".json")
    data = {"name": name, "saved_at": time.time(), "messages": messages,
            "session_map": session_map, "metadata": metadata or {}}
    tmp = path + ".tmp"
    with open(tmp, "w") as fh:
        json.dump(data, fh, indent=1)
    os.replace(tmp, path)  # a reader never sees a half-written file
    return path


def auto_save(messages, session_map=None, metadata=None, session_dir=None) -> str:
    d = _dir(session_dir)
    path = save_session(time.strftime("autosave_%Y%m%d_%H%M%S") + f"_{int(time.time() * 1e6) % 1000000}",
                        messages, session_map, metadata, d)
    autos = sorted(f for f in os.listdir(d) if f.startswith("autosave_") and f.endswith(".json"))
    for old in autos[:-AUTO_SAVE_KEEP]:
        os.remove(os.path.join(d, old))
    return path


def load_session(path) -> dict:
    with open(path) as fh:
        data = json.load(fh)
    if not isinstance(data.get("messages"), list):
        raise ValueError(f"{path}: not a session file")
    return data


def list_sessions(session_dir=None) -> list:
    d = _dir(session_dir)
    out = []
    for f in sorted(os.listdir(d)):
        if f.endswith(".json"):
            p = os.path.join(d, f)
            try:
                data = load_session(p)
            except (ValueError, json.JSONDecodeError, OSError):
                continue
            out.append({"path": p, "name": data.get("name", f[:-5]),
                        "saved_at": data.get("saved_at", 0), "messages": len(data["messages"])})
    return sorted(out, key=lambda s: -s["saved_at"])


def find_session(name_or_index, session_dir=None):
    sessions = list_sessions(session_dir)
    if isinstance(name_or_index, int) or str(name_or_index).isdigit():
        i = int(name_or_index)
        return sessions[i]["path"] if 0 <= i < len(sessions) else None
    for s in sessions:
        if s["name"] == name_or_index:
            return s["path"]
    return None


def purge_sessions(session_dir=None) -> int:
    d = _dir(session_dir)
    n = 0
    for f in os.listdir(d):
        if f.endswith(".json"):
            os.remove(os.path.join(d, f))
            n += 1
    return n
