"""/v1/files: upload (multipart ``file`` + optional ``purpose``), list (``?purpose=``,
``?file_type=``), download (``GET /v1/files/{id}``, as the reference serves it, and the OpenAI
form ``/v1/files/{id}/content``), metadata (``/v1/files/{id}/info``) and delete. Routes and
response fields follow the reference (api/server.py:2477-2572); storage is core/file_store.py.
"""

from b200serve.core.file_store import FileStore, get_file_store


def register_file_routes(app, auth, store: FileStore = None):
    from fastapi import HTTPException, Request
    from fastapi.responses import Response

    app.state.files = store                  # None: the process-wide store, created on first use

    def _store() -> FileStore:
        if app.state.files is None:
            app.state.files = get_file_store()
        return app.state.files

    def _found(fid: str):
        info = _store().get(fid)
        if info is None:
            raise HTTPException(status_code=404, detail="File not found")
        return info

    @app.post("/v1/files")
    async def upload_file(request: Request):
        auth(request)
        try:
            form = await request.form()
        except Exception as e:                                     # malformed multipart body
            raise HTTPException(status_code=400, detail=f"Expected multipart form data: {e}")
        upload = form.get("file")
        if upload is None or not hasattr(upload, "read"):
            raise HTTPException(status_code=400, detail="No file provided. Use multipart form with a 'file' field.")
        data = await upload.read()
        try:
            info = _store().put(data, upload.filename or "unnamed", upload.content_type,
                                purpose=str(form.get("purpose") or "upload"))
        except ValueError as e:
            raise HTTPException(status_code=400, detail=str(e))
        return info.api()

    @app.get("/v1/files")
    async def list_files(request: Request, purpose: str = None, file_type: str = None):
        auth(request)
        return {"object": "list", "data": [f.api() for f in _store().list(purpose, file_type)]}

    def _content(fid: str):
        info = _found(fid)
        data = _store().read(fid)
        if data is None:
            raise HTTPException(status_code=404, detail="File data missing from disk")
        safe = info.filename.replace('"', "")
        return Response(content=data, media_type=info.content_type,
                        headers={"Content-Disposition": f'attachment; filename="{safe}"'})

    @app.get("/v1/files/{file_id}")
    async def download_file(file_id: str, request: Request):
        auth(request)
        return _content(file_id)

    @app.get("/v1/files/{file_id}/content")
    async def file_content(file_id: str, request: Request):
        auth(request)
        return _content(file_id)

    @app.get("/v1/files/{file_id}/info")
    async def file_info(file_id: str, request: Request):
        auth(request)
        return _found(file_id).api()

    @app.delete("/v1/files/{file_id}")
    async def delete_file(file_id: str, request: Request):
        auth(request)
        if not _store().delete(file_id):
            raise HTTPException(status_code=404, detail="File not found")
        return {"id": file_id, "object": "file", "deleted": True}
