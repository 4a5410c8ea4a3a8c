"""Local knowledge base and retrieval-augmented generation (reference: core/knowledge.py,
core/rag.py).

Documents are split into overlapping passages (paragraph-aware, ``chunk_chars`` each), embedded
and kept in one matrix. A query is scored two ways and the scores are mixed:
  * dense: cosine similarity of the query embedding against every passage (one
    matrix-vector product over the normalised vectors);
  * lexical: BM25 over the passages' words.
The embedder is any ``texts -> vectors`` callable: ``engine_embedder(engine)`` uses the
serving engine's own model (mean-pooled final hidden states, the /v1/embeddings path);
``HashEmbedder`` is a model-free fallback (feature-hashed unigrams and bigrams).
``augment(messages, query)`` puts the best passages into a system message, with their
sources, before generation. The store persists to a directory (passages as JSONL, vectors
as .npy, a meta file written last as the completion marker).
"""

from __future__ import annotations

import hashlib
import json
import math
import os
import re
import threading
from collections import Counter

import numpy as np

_WORD = re.compile(r"[A-Za-z0-9_]+")


def words(text: str) -> list:
    return [w.lower() for w in _WORD.findall(text)]


class HashEmbedder:
    """Feature-hashed bag of unigrams and bigrams, L2-normalised (no model needed)."""

    def __init__(self, dim: int = 512):
        self.dim = dim

    def _slot(self, tok: str):
        h = int.from_bytes(hashlib.blake2b(tok.encode(), digest_size=8).digest(), "little")
        return h % self.dim, 1.0 if (h >> 63) & 1 else -1.0

    def __call__(self, texts):
        out = np.zeros((len(texts), self.dim), dtype=np.float32)
        for i, t in enumerate(texts):
            ws = words(t)
            for tok in ws + [a + " " + b for a, b in zip(ws, ws[1:])]:
                j, s = self._slot(tok)
                out[i, j] += s
        n = np.linalg.norm(out, axis=1, keepdims=True)
        return out / np.maximum(n, 1e-9)


def engine_embedder(engine):
    """Embed with the serving engine's model (B200Engine.embed), L2-normalised."""
    def embed(texts):
        vecs, _ = engine.embed(list(texts))
        v = np.asarray(vecs, dtype=np.float32)
        return v / np.maximum(np.linalg.norm(v, axis=1, keepdims=True), 1e-9)
    return embed


def split_passages(text: str, chunk_chars: int = 1200, overlap: int = 200) -> list:
    """Paragraph-aware chunks of at most ``chunk_chars``; consecutive chunks share ``overlap``
    characters so a fact on a boundary is found whole in one of them."""
    paras = [p.strip() for p in re.split(r"\n\s*\n", text) if p.strip()]
    chunks, cur = [], ""
    for p in paras:
        while len(p) > chunk_chars:                         # a paragraph longer than a chunk
            if cur:
                chunks.append(cur)
                cur = ""
            chunks.append(p[:chunk_chars])
            p = p[chunk_chars - overlap:]
        if cur and len(cur) + 2 + len(p) > chunk_chars:
            chunks.append(cur)
            cur = cur[-overlap:] + "\n\n" + p if overlap else p
        else:
            cur = (cur + "\n\n" + p) if cur else p
    if cur:
        chunks.append(cur)
    return chunks


class Knowledge:
    def __init__(self, embedder=None, chunk_chars: int = 1200, overlap: int = 200, alpha: float = 0.7,
                 path: str = None):
        self.embed = embedder or HashEmbedder()
        self.chunk_chars, self.overlap, self.alpha = chunk_chars, overlap, alpha
        self.path = path
        self.passages = []          # {"source", "chunk", "text"}
        self.vectors = None         # [n, d] float32
        self._df = Counter()
        self._tf = []
        self._lock = threading.Lock()
        if path and os.path.exists(os.path.join(path, "meta.json")):
            self.load(path)

    # ------------------------------------------------------------ building
    def add(self, source: str, text: str) -> int:
        """Index ``text`` under ``source`` (replacing an earlier version). Returns passages added."""
        self.remove(source)
        chunks = split_passages(text, self.chunk_chars, self.overlap)
        if not chunks:
            return 0
        vecs = np.asarray(self.embed(chunks), dtype=np.float32)
        with self._lock:
            base = len(self.passages)
            for i, c in enumerate(chunks):
                self.passages.append({"source": source, "chunk": i, "text": c})
                tf = Counter(words(c))
                self._tf.append(tf)
                self._df.update(tf.keys())
            self.vectors = vecs if self.vectors is None else np.concatenate([self.vectors, vecs])
            assert self.vectors.shape[0] == base + len(chunks)
        return len(chunks)

    def add_file(self, path: str, source: str = None) -> int:
        with open(path, encoding="utf-8", errors="replace") as fh:
            return self.add(source or os.path.basename(path), fh.read())

    def remove(self, source: str) -> int:
        with self._lock:
            keep = [i for i, p in enumerate(self.passages) if p["source"] != source]
            gone = len(self.passages) - len(keep)
            if gone:
                for i, p in enumerate(self.passages):
                    if p["source"] == source:
                        self._df.subtract(self._tf[i].keys())
                self.passages = [self.passages[i] for i in keep]
                self._tf = [self._tf[i] for i in keep]
                self.vectors = self.vectors[keep] if keep else None
                self._df = +self._df
            return gone

    def sources(self) -> dict:
        return dict(Counter(p["source"] for p in self.passages))

    # ------------------------------------------------------------ retrieval
    def _bm25(self, query_words, k1: float = 1.5, b: float = 0.75) -> np.ndarray:
        n = len(self.passages)
        lens = np.array([sum(tf.values()) for tf in self._tf], dtype=np.float32)
        avg = float(lens.mean()) if n else 1.0
        s = np.zeros(n, dtype=np.float32)
        for w in set(query_words):
            df = self._df.get(w, 0)
            if not df:
                continue
            idf = math.log(1 + (n - df + 0.5) / (df + 0.5))
            tf = np.array([t.get(w, 0) for t in self._tf], dtype=np.float32)
            s += idf * tf * (k1 + 1) / (tf + k1 * (1 - b + b * lens / max(avg, 1e-9)))
        return s

    def search(self, query: str, k: int = 5) -> list:
        """Top-k passages: alpha * cosine + (1 - alpha) * BM25 scaled to [0, 1]."""
        with self._lock:
            if not self.passages:
                return []
            q = np.asarray(self.embed([query]), dtype=np.float32)[0]
            dense = self.vectors @ q
            lex = self._bm25(words(query))
            if lex.max() > 0:
                lex = lex / lex.max()
            score = self.alpha * dense + (1 - self.alpha) * lex
            top = np.argsort(-score)[:k]
            return [dict(self.passages[i], score=float(score[i])) for i in top if score[i] > 0]

    def augment(self, messages: list, query: str = None, k: int = 4, max_chars: int = 6000) -> list:
        """Messages with a system message of retrieved passages inserted before the last user
        turn (the query defaults to that turn's text)."""
        if query is None:
            query = next((m.get("content", "") for m in reversed(messages)
                          if m.get("role") == "user" and isinstance(m.get("content"), str)), "")
        hits = self.search(query, k) if query else []
        if not hits:
            return list(messages)
        parts, used = [], 0
        for h in hits:
            block = f"[{h['source']} #{h['chunk']}]\n{h['text']}"
            if used + len(block) > max_chars:
                break
            parts.append(block)
            used += len(block)
        ctx = {"role": "system", "content": "Relevant passages from the local knowledge base "
                                            "(cite them by [source #chunk]):\n\n" + "\n\n".join(parts)}
        last_user = max((i for i, m in enumerate(messages) if m.get("role") == "user"), default=len(messages))
        return list(messages[:last_user]) + [ctx] + list(messages[last_user:])

    # ------------------------------------------------------------ persistence
    def save(self, path: str = None):
        path = path or self.path
        os.makedirs(path, exist_ok=True)
        meta = os.path.join(path, "meta.json")
        if os.path.exists(meta):
            os.remove(meta)                          # incomplete until the marker is rewritten
        with self._lock:
            with open(os.path.join(path, "passages.jsonl"), "w", encoding="utf-8") as fh:
                for p in self.passages:
                    fh.write(json.dumps(p, ensure_ascii=False) + "\n")
            np.save(os.path.join(path, "vectors.npy"), self.vectors if self.vectors is not None
                    else np.zeros((0, 1), np.float32))
            with open(meta, "w") as fh:
                json.dump({"passages": len(self.passages), "chunk_chars": self.chunk_chars,
                           "overlap": self.overlap}, fh)

    def load(self, path: str):
        with open(os.path.join(path, "meta.json")) as fh:
            meta = json.load(fh)
        with open(os.path.join(path, "passages.jsonl"), encoding="utf-8") as fh:
            passages = [json.loads(ln) for ln in fh if ln.strip()]
        vecs = np.load(os.path.join(path, "vectors.npy"))
        if len(passages) != meta["passages"] or (passages and vecs.shape[0] != len(passages)):
            raise ValueError(f"{path}: knowledge store is inconsistent")
        with self._lock:
            self.passages = passages
            self.vectors = vecs if passages else None
            self._tf = [Counter(words(p["text"])) for p in passages]
            self._df = Counter()
            for tf in self._tf:
                self._df.update(tf.keys())
