"""Conversation sessions over HTTP: list, read, create/replace, delete.

Routes and fields follow the reference (api/session_api.py:144-200): ``GET /v1/sessions``
-> {"sessions": [{id, title, updated, message_count, model}]}, ``GET/PUT/DELETE
/v1/sessions/{id}``; PUT stores the conversation without system messages, keeps the newest
messages up to a cap, derives a title from the first user message when none is given, and
refuses oversized bodies with 413. Storage is one JSON file per session written atomically
(temp file + rename) in the directory ``core/session.py`` uses; the oldest files beyond
``max_sessions`` are pruned after each write.
"""


import json
import os
import re
import threading
import time
from typing import List, Optional

from pydantic import BaseModel

_ID = re.compile(r"^[A-Za-z0-9_-]{1,64}$")


class SessionUpsert(BaseModel):
    messages: List[dict]
    title: Optional[str] = None
    model: Optional[str] = None


def _title_of(messages) -> str:
    for m in messages:
        if m.get("role") == "user":
            c = m.get("content")
            if isinstance(c, list):
                c = " ".join(p.get("text", "") for p in c if isinstance(p, dict))
            text = " ".join(str(c or "").split())
            if text:
                return text if len(text) <= 60 else text[:57] + "..."
    return "New chat"


class SessionStore:
    def __init__(self, root: str = None, max_sessions: int = 200, max_messages: int = 500,
                 max_bytes: int = 4 << 20):
        if root is None:
            from b200serve.core import config
            root = os.path.join(config.SESSION_DIR, "api")
        self.root = root
        os.makedirs(root, exist_ok=True)
        self.max_sessions, self.max_messages, self.max_bytes = max_sessions, max_messages, max_bytes
        self._lock = threading.Lock()

    def path(self, sid: str) -> str:
        if not _ID.match(sid or ""):
            raise ValueError("session id: 1-64 letters, digits, '-' or '_'")
        return os.path.join(self.root, sid + ".json")

    def list(self) -> list:
        out = []
        for name in os.listdir(self.root):
            if not name.endswith(".json"):
                continue
            try:
                with open(os.path.join(self.root, name), encoding="utf-8") as fh:
                    d = json.load(fh)
            except (OSError, json.JSONDecodeError):
                continue
            out.append({"id": d.get("id", name[:-5]), "title": d.get("title", "?"), "updated": d.get("updated", 0),
                        "message_count": len(d.get("messages", [])), "model": d.get("model")})
        out.sort(key=lambda m: m["updated"], reverse=True)
        return out

    def get(self, sid: str) -> dict:
        with open(self.path(sid), encoding="utf-8") as fh:
            return json.load(fh)

    def put(self, sid: str, body: SessionUpsert) -> dict:
        path = self.path(sid)
        msgs = [m for m in body.messages if isinstance(m, dict) and m.get("role") != "system"]
        msgs = msgs[-self.max_messages:]
        rec = {"id": sid, "title": (body.title or "").strip() or _title_of(msgs), "model": body.model,
               "updated": round(time.time(), 3), "messages": msgs}
        raw = json.dumps(rec, ensure_ascii=False)
        if len(raw.encode("utf-8")) > self.max_bytes:
            raise OverflowError("session too large")
        with self._lock:
            tmp = f"{path}.{os.getpid()}.tmp"
            with open(tmp, "w", encoding="utf-8") as fh:
                fh.write(raw)
            os.replace(tmp, path)
            self._prune()
        return {"ok": True, "id": sid, "title": rec["title"], "message_count": len(msgs)}

    def delete(self, sid: str):
        os.remove(self.path(sid))

    def _prune(self):
        files = [os.path.join(self.root, n) for n in os.listdir(self.root) if n.endswith(".json")]
        files.sort(key=os.path.getmtime, reverse=True)
        for stale in files[self.max_sessions:]:
            try:
                os.remove(stale)
            except OSError:
                pass


def register_session_routes(app, auth, store: SessionStore = None):
    from fastapi import HTTPException, Request

    store = store or SessionStore()
    app.state.sessions = store

    def guard(fn, *a):
        try:
            return fn(*a)
        except ValueError as e:
            raise HTTPException(status_code=400, detail=str(e))
        except FileNotFoundError:
            raise HTTPException(status_code=404, detail="No such session")
        except OverflowError:
            raise HTTPException(status_code=413, detail="Session too large")
        except (OSError, json.JSONDecodeError) as e:
            raise HTTPException(status_code=500, detail=f"Session unreadable: {e}")

    @app.get("/v1/sessions")
    async def list_sessions(request: Request):
        auth(request)
        return {"sessions": guard(store.list)}

    @app.get("/v1/sessions/{session_id}")
    async def get_session(session_id: str, request: Request):
        auth(request)
        return guard(store.get, session_id)

    @app.put("/v1/sessions/{session_id}")
    async def put_session(session_id: str, body: SessionUpsert, request: Request):
        auth(request)
        return guard(store.put, session_id, body)

    @app.delete("/v1/sessions/{session_id}")
    async def delete_session(session_id: str, request: Request):
        auth(request)
        guard(store.delete, session_id)
        return {"ok": True, "deleted": session_id}

    return store
