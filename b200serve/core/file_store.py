"""Managed storage for uploaded and generated files (images, audio, video, documents, meshes).

Behaviour follows the reference's file manager (core/services/file_manager.py:64-326) and its
HTTP routes (api/server.py:2477-2572): files get an opaque id, a category from their name
(image / audio / video / document / mesh; anything else is refused), a MIME type, a size and
a creation time, and can be listed (by purpose or category), read back, deleted and aged out.

Design: every file is two entries in one directory, the data ``<id>.bin`` and a sidecar
``<id>.json`` with its metadata, each written to a temporary name and renamed into place, so a
crash leaves either a whole record or none and no shared index file is ever rewritten. The
in-memory table is rebuilt from the sidecars at start-up (orphaned data files are removed).
The category also checks the leading bytes of the data for the common formats, so a file whose
content contradicts its extension (a PE binary named ``x.png``) is refused.
"""

from __future__ import annotations

import json
import mimetypes
import os
import secrets
import threading
import time
from dataclasses import asdict, dataclass, field
from typing import Dict, List, Optional

from b200serve.core.config import BASE_DIR

FILES_DIR = os.environ.get("B200_FILES_DIR", os.path.join(BASE_DIR, "files"))
MAX_FILE_BYTES = int(os.environ.get("B200_MAX_FILE_MB", "512")) << 20

CATEGORIES = {
    "image": (".png", ".jpg", ".jpeg", ".webp", ".bmp", ".gif", ".tiff"),
    "audio": (".wav", ".mp3", ".flac", ".ogg", ".m4a"),
    "video": (".mp4", ".avi", ".webm", ".mov", ".mkv"),
    "document": (".pdf", ".txt", ".md", ".docx", ".csv", ".json"),
    "mesh": (".ply", ".obj", ".stl", ".glb", ".gltf", ".pt"),
}
_CATEGORY_OF = {ext: cat for cat, exts in CATEGORIES.items() for ext in exts}

# leading bytes of formats whose extension we can cross-check: extension -> accepted prefixes
_MAGIC = {
    ".png": (b"\x89PNG\r\n\x1a\n",),
    ".jpg": (b"\xff\xd8\xff",), ".jpeg": (b"\xff\xd8\xff",),
    ".gif": (b"GIF87a", b"GIF89a"),
    ".bmp": (b"BM",),
    ".webp": (b"RIFF",), ".wav": (b"RIFF",), ".avi": (b"RIFF",),
    ".pdf": (b"%PDF",),
    ".flac": (b"fLaC",),
    ".ogg": (b"OggS",),
    ".glb": (b"glTF",),
}
# prefixes of executables and archives that are never accepted under a media or text name
_FORBIDDEN = (b"MZ", b"\x7fELF", b"\xca\xfe\xba\xbe", b"\xcf\xfa\xed\xfe", b"#!")


def category_of(name: str) -> str:
    return _CATEGORY_OF.get(os.path.splitext(name)[1].lower(), "unknown")


def content_matches(name: str, head: bytes) -> bool:
    """False when the data's leading bytes contradict the name's extension or mark an executable."""
    ext = os.path.splitext(name)[1].lower()
    if any(head.startswith(p) for p in _FORBIDDEN):
        return False
    want = _MAGIC.get(ext)
    return want is None or any(head.startswith(p) for p in want)


@dataclass
class FileInfo:
    id: str
    filename: str
    bytes: int
    file_type: str
    content_type: str
    purpose: str
    created_at: float
    metadata: dict = field(default_factory=dict)

    def api(self) -> dict:
        return {"id": self.id, "object": "file", "filename": self.filename, "purpose": self.purpose,
                "bytes": self.bytes, "file_type": self.file_type, "created_at": int(self.created_at)}


class FileStore:
    def __init__(self, root: str = None, max_bytes: int = MAX_FILE_BYTES):
        self.root = root or FILES_DIR
        self.max_bytes = max_bytes
        self._lock = threading.Lock()
        self._files: Dict[str, FileInfo] = {}
        os.makedirs(self.root, exist_ok=True)
        self._scan()

    # ------------------------------------------------------------ storage
    def _path(self, fid: str, kind: str) -> str:
        return os.path.join(self.root, f"{fid}.{kind}")

    def _write(self, path: str, data: bytes):
        tmp = f"{path}.{secrets.token_hex(4)}.tmp"
        with open(tmp, "wb") as fh:
            fh.write(data)
            fh.flush()
            os.fsync(fh.fileno())
        os.replace(tmp, path)

    def _scan(self):
        seen = set()
        for name in os.listdir(self.root):
            if name.endswith(".tmp"):
                os.unlink(os.path.join(self.root, name))
                continue
            if not name.endswith(".json"):
                continue
            try:
                with open(os.path.join(self.root, name), encoding="utf-8") as fh:
                    info = FileInfo(**json.load(fh))
            except (OSError, ValueError, TypeError):
                continue
            if os.path.exists(self._path(info.id, "bin")):
                self._files[info.id] = info
                seen.add(info.id)
        for name in os.listdir(self.root):
            if name.endswith(".bin") and name[:-4] not in seen:
                os.unlink(os.path.join(self.root, name))

    # ------------------------------------------------------------ public API
    def put(self, data: bytes, filename: str, content_type: str = None, purpose: str = "upload",
            metadata: dict = None) -> FileInfo:
        """Store ``data`` under a new id. ValueError for an unsupported name, content that does not
        match it, or a file over the size limit."""
        filename = os.path.basename(filename or "unnamed").strip() or "unnamed"
        cat = category_of(filename)
        if cat == "unknown":
            raise ValueError(f"unsupported file type: {filename} (accepted: "
                             + ", ".join(sorted(CATEGORIES)) + ")")
        if len(data) > self.max_bytes:
            raise ValueError(f"file too large: {len(data)} bytes > {self.max_bytes}")
        if not content_matches(filename, data[:16]):
            raise ValueError(f"content of {filename} does not match its type")
        if not content_type or content_type == "application/octet-stream":
            content_type = mimetypes.guess_type(filename)[0] or "application/octet-stream"
        info = FileInfo(id="file-" + secrets.token_hex(8), filename=filename, bytes=len(data), file_type=cat,
                        content_type=content_type, purpose=purpose, created_at=time.time(),
                        metadata=dict(metadata or {}))
        with self._lock:
            self._write(self._path(info.id, "bin"), data)
            self._write(self._path(info.id, "json"), json.dumps(asdict(info)).encode())
            self._files[info.id] = info
        return info

    def put_path(self, path: str, purpose: str = "upload", metadata: dict = None) -> FileInfo:
        if os.path.islink(path):
            raise ValueError(f"refusing to store a symbolic link: {path}")
        with open(path, "rb") as fh:
            return self.put(fh.read(), os.path.basename(path), purpose=purpose, metadata=metadata)

    def get(self, fid: str) -> Optional[FileInfo]:
        return self._files.get(fid)

    def path(self, fid: str) -> Optional[str]:
        if fid not in self._files:
            return None
        p = self._path(fid, "bin")
        return p if os.path.exists(p) else None

    def read(self, fid: str) -> Optional[bytes]:
        p = self.path(fid)
        if p is None:
            return None
        with open(p, "rb") as fh:
            return fh.read()

    def delete(self, fid: str) -> bool:
        with self._lock:
            info = self._files.pop(fid, None)
            if info is None:
                return False
            for kind in ("json", "bin"):              # metadata first: a crash leaves an orphan, not a ghost
                try:
                    os.unlink(self._path(fid, kind))
                except FileNotFoundError:
                    pass
        return True

    def list(self, purpose: str = None, file_type: str = None) -> List[FileInfo]:
        out = [f for f in self._files.values()
               if (purpose is None or f.purpose == purpose) and (file_type is None or f.file_type == file_type)]
        return sorted(out, key=lambda f: f.created_at, reverse=True)

    def expire(self, max_age_s: float, now: float = None) -> int:
        """Delete files older than ``max_age_s``; returns how many went."""
        now = time.time() if now is None else now
        old = [f.id for f in list(self._files.values()) if now - f.created_at > max_age_s]
        return sum(self.delete(fid) for fid in old)

    def clear(self) -> int:
        return sum(self.delete(fid) for fid in list(self._files))

    def usage(self) -> dict:
        by = {}
        for f in self._files.values():
            c = by.setdefault(f.file_type, {"files": 0, "bytes": 0})
            c["files"] += 1
            c["bytes"] += f.bytes
        return {"files": len(self._files), "bytes": sum(f.bytes for f in self._files.values()), "by_type": by}


_store: Optional[FileStore] = None


def get_file_store() -> FileStore:
    global _store
    if _store is None:
        _store = FileStore()
    return _store
