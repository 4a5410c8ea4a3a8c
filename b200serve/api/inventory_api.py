"""Model inventory over HTTP (reference: api/inventory_api.py): ``GET /v1/inventory`` lists
every reachable model with its status, ``GET /v1/inventory/proposal?path=`` the entry proposed
for an unconfigured checkpoint, ``POST /v1/inventory/add`` {path | entry, name?} writes an
entry (only when the server allows registry writes). Logic in core/model_inventory.py."""

import os


def register_inventory_routes(app, auth, registry_path: str = None, allow_write: bool = None):
    from fastapi import HTTPException, Request
    from b200serve.core import model_inventory as mi

    if allow_write is None:
        allow_write = os.environ.get("B200_INVENTORY_WRITE", "0") == "1"

    @app.get("/v1/inventory")
    async def inventory(request: Request):
        auth(request)
        return mi.scan(registry_path)

    @app.get("/v1/inventory/proposal")
    async def proposal(path: str, request: Request):
        auth(request)
        try:
            return mi.propose_entry(path, registry_path)
        except ValueError as e:
            raise HTTPException(status_code=400, detail=str(e))

    @app.post("/v1/inventory/add")
    async def add(request: Request):
        auth(request)
        if not allow_write:
            raise HTTPException(status_code=403, detail="registry writes are disabled (B200_INVENTORY_WRITE=1)")
        body = await request.json()
        try:
            if "entry" in body:
                name, entry = body.get("name"), body["entry"]
            else:
                prop = mi.propose_entry(body.get("path", ""), registry_path)
                name, entry = body.get("name") or prop["name"], prop["entry"]
            written = mi.add_entry(name, entry, registry_path, overwrite=bool(body.get("overwrite")))
        except ValueError as e:
            raise HTTPException(status_code=400, detail=str(e))
        return {"name": name, "entry": entry, "registry": written}
