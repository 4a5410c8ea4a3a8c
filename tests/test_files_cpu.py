"""File storage and /v1/files: upload, list by purpose and type, download (both routes),
metadata, delete; unsupported names, content that contradicts its extension and oversized files
are refused; records survive a restart and orphaned data is cleaned up; age-based expiry."""

import os
import time

import pytest

fastapi = pytest.importorskip("fastapi")
from fastapi import FastAPI  # noqa: E402
from fastapi.testclient import TestClient  # noqa: E402

from b200serve.api.files_api import register_file_routes  # noqa: E402
from b200serve.core.file_store import FileStore  # noqa: E402

PNG = b"\x89PNG\r\n\x1a\n" + b"\x00" * 64


def test_store_round_trip_restart_and_expiry(tmp_path):
    st = FileStore(str(tmp_path), max_bytes=1024)
    a = st.put(PNG, "../../etc/pic.png")
    assert a.filename == "pic.png" and a.file_type == "image" and a.content_type == "image/png"
    b = st.put(b"hello", "notes.txt", purpose="assistants")
    assert st.read(a.id) == PNG and st.get(b.id).bytes == 5
    with pytest.raises(ValueError):
        st.put(b"MZ\x90\x00", "evil.png")              # executable named as an image
    with pytest.raises(ValueError):
        st.put(b"abc", "tool.exe")                     # unsupported category
    with pytest.raises(ValueError):
        st.put(b"x" * 2000, "big.txt")                 # over the size limit
    with pytest.raises(ValueError):
        st.put(b"not a png", "fake.png")               # content contradicts the extension
    assert [f.id for f in st.list(purpose="assistants")] == [b.id]
    assert [f.id for f in st.list(file_type="image")] == [a.id]
    # a restart rebuilds the table from the sidecars and drops data without metadata
    open(os.path.join(str(tmp_path), "file-orphan.bin"), "wb").write(b"zz")
    st2 = FileStore(str(tmp_path), max_bytes=1024)
    assert {f.id for f in st2.list()} == {a.id, b.id}
    assert not os.path.exists(os.path.join(str(tmp_path), "file-orphan.bin"))
    assert st2.usage()["by_type"]["image"] == {"files": 1, "bytes": len(PNG)}
    assert st2.expire(60.0, now=time.time() + 3600) == 2 and st2.list() == []


def test_files_routes(tmp_path):
    app = FastAPI()
    register_file_routes(app, lambda request: None, FileStore(str(tmp_path)))
    with TestClient(app) as c:
        r = c.post("/v1/files", files={"file": ("cat.png", PNG, "image/png")}, data={"purpose": "vision"})
        assert r.status_code == 200, r.text
        meta = r.json()
        assert meta["object"] == "file" and meta["bytes"] == len(PNG) and meta["purpose"] == "vision"
        fid = meta["id"]
        assert c.post("/v1/files", files={"file": ("run.sh", b"#!/bin/sh", "text/plain")}).status_code == 400
        assert c.post("/v1/files", data={"purpose": "x"}).status_code == 400
        lst = c.get("/v1/files", params={"file_type": "image"}).json()
        assert lst["object"] == "list" and [d["id"] for d in lst["data"]] == [fid]
        assert c.get("/v1/files", params={"purpose": "other"}).json()["data"] == []
        for path in (f"/v1/files/{fid}", f"/v1/files/{fid}/content"):
            d = c.get(path)
            assert d.status_code == 200 and d.content == PNG and d.headers["content-type"] == "image/png"
            assert 'filename="cat.png"' in d.headers["content-disposition"]
        assert c.get(f"/v1/files/{fid}/info").json()["filename"] == "cat.png"
        assert c.delete(f"/v1/files/{fid}").json() == {"id": fid, "object": "file", "deleted": True}
        assert c.get(f"/v1/files/{fid}").status_code == 404
        assert c.delete(f"/v1/files/{fid}").status_code == 404
