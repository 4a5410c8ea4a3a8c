"""Knowledge-base routes (reference: core/knowledge.py, core/rag.py behind the app's
knowledge panel):

  GET    /v1/knowledge                  sources and passage counts
  POST   /v1/knowledge                  add or replace a document {source, text}
  DELETE /v1/knowledge/{source}         remove a document
  POST   /v1/knowledge/search           {query, k} -> passages with scores

The store embeds with the serving engine's model when it offers ``embed`` (falls back to the
model-free hashing embedder otherwise) and persists under B200_KNOWLEDGE_DIR when set. Chat
completions use it with ``options.rag = k`` (passages put before the last user turn) and
the web-tool rounds get a knowledge_search tool.
"""

import os

from pydantic import BaseModel

from b200serve.agent.knowledge import HashEmbedder, Knowledge, engine_embedder


class DocIn(BaseModel):
    source: str
    text: str


class SearchIn(BaseModel):
    query: str
    k: int = 5


_kb = None


def get_knowledge(engine=None) -> Knowledge:
    global _kb
    if _kb is None:
        emb = engine_embedder(engine) if (engine is not None and hasattr(engine, "embed")
                                          and os.environ.get("B200_KNOWLEDGE_EMBED", "engine") == "engine") \
            else HashEmbedder()
        _kb = Knowledge(emb, path=os.environ.get("B200_KNOWLEDGE_DIR") or None)
        from b200serve.api import chat_tools
        chat_tools.set_knowledge(_kb)
    return _kb


def reset_knowledge():
    global _kb
    _kb = None
    from b200serve.api import chat_tools
    chat_tools.set_knowledge(None)


def register_knowledge_routes(app, auth, get_engine):
    import asyncio
    from fastapi import HTTPException, Request

    def kb():
        return get_knowledge(get_engine())

    def persist(k):
        if k.path:
            k.save()

    @app.get("/v1/knowledge")
    async def kb_list(request: Request):
        auth(request)
        k = await asyncio.to_thread(kb)
        return {"sources": k.sources(), "passages": len(k.passages)}

    @app.post("/v1/knowledge")
    async def kb_add(request: Request, body: DocIn):
        auth(request)
        if not body.source.strip() or not body.text.strip():
            raise HTTPException(status_code=400, detail="source and text are required")
        k = await asyncio.to_thread(kb)
        n = await asyncio.to_thread(k.add, body.source, body.text)
        await asyncio.to_thread(persist, k)
        return {"ok": True, "source": body.source, "passages": n}

    @app.delete("/v1/knowledge/{source}")
    async def kb_delete(source: str, request: Request):
        auth(request)
        k = await asyncio.to_thread(kb)
        n = k.remove(source)
        if not n:
            raise HTTPException(status_code=404, detail="no such source")
        await asyncio.to_thread(persist, k)
        return {"ok": True, "removed": n}

    @app.post("/v1/knowledge/search")
    async def kb_search(request: Request, body: SearchIn):
        auth(request)
        k = await asyncio.to_thread(kb)
        return {"results": await asyncio.to_thread(k.search, body.query, max(1, min(body.k, 50)))}
