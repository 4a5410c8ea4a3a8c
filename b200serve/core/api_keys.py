"""Hashed API-key store (reference: core/api_keys.py:71 ``KeyStore``).

Keys are stored as salted SHA-256 hashes in a JSON file; ``match`` compares in
constant time. With no keys configured the API is open (local use)."""

from __future__ import annotations

import hashlib
import hmac
import json
import os
import secrets
import threading
import time


class KeyStore:
    def __init__(self, path: str = None):
        self.path = path or os.environ.get("B200_API_KEYS", "")
        self._lock = threading.Lock()
        self._keys = []
        self._load()
        env = os.environ.get("ARTIFEX_API_KEY", "")
        if env:
            self._keys.append(self._entry(env, "env"))

    def _load(self):
        if self.path and os.path.exists(self.path):
            with open(self.path) as fh:
                self._keys = json.load(fh).get("keys", [])

    def _save(self):
        if not self.path:
            return
        tmp = self.path + ".tmp"
        with open(tmp, "w") as fh:
            json.dump({"keys": [k for k in self._keys if k.get("id") != "env"]}, fh, indent=1)
        os.replace(tmp, self.path)

    @staticmethod
    def _hash(key: str, salt: str) -> str:
        return hashlib.sha256((salt + key).encode()).hexdigest()

    def _entry(self, key, name):
        salt = secrets.token_hex(8)
        return {"id": secrets.token_hex(4) if name != "env" else "env", "name": name, "salt": salt,
                "hash": self._hash(key, salt), "created": time.time()}

    def configured(self) -> bool:
        return bool(self._keys)

    def create(self, name: str = "device") -> str:
        key = "ak-" + secrets.token_urlsafe(24)
        with self._lock:
            self._keys.append(self._entry(key, name))
            self._save()
        return key

    def revoke(self, key_id: str) -> bool:
        with self._lock:
            n = len(self._keys)
            self._keys = [k for k in self._keys if k["id"] != key_id]
            self._save()
            return len(self._keys) != n

    def rotate(self, key_id: str) -> str:
        """Replace key ``key_id`` with a fresh one of the same name; the old key stops working.
        Returns the new plaintext key (shown once). KeyError for an unknown id."""
        with self._lock:
            old = next((k for k in self._keys if k["id"] == key_id), None)
            if old is None or key_id == "env":
                raise KeyError(key_id)
            key = "ak-" + secrets.token_urlsafe(24)
            entry = self._entry(key, old.get("name", "device"))
            entry["rotated_from"] = key_id
            self._keys = [k for k in self._keys if k["id"] != key_id] + [entry]
            self._save()
        return key

    def list(self) -> list:
        """Key metadata without salts or hashes."""
        return [{"id": k["id"], "name": k.get("name"), "created": k.get("created")} for k in self._keys]

    def match(self, token: str):
        hit = None
        for k in self._keys:
            if hmac.compare_digest(self._hash(token, k["salt"]), k["hash"]):
                hit = k
        return hit
