"""Local model store.  A root directory holds one folder per model with its weight files
(safetensors / GGUF), `config.json` and an index entry with per-file SHA-256 digests, so a
restart can verify files without re-fetching.  Network fetch is out of scope offline."""
from __future__ import annotations

import hashlib
import json
import os
import shutil


def file_digest(path: str, chunk: int = 8 << 20) -> str:
    h = hashlib.sha256()
    with open(path, "rb") as f:
        while True:
            b = f.read(chunk)
            if not b:
                break
            h.update(b)
    return h.hexdigest()


class ModelStore:
    def __init__(self, root: str):
        self.root = root
        os.makedirs(root, exist_ok=True)
        self.index_path = os.path.join(root, "index.json")
        self.index = json.load(open(self.index_path)) if os.path.exists(self.index_path) else {}

    def _save(self):
        tmp = self.index_path + ".tmp"
        with open(tmp, "w") as f:
            json.dump(self.index, f, indent=1, sort_keys=True)
        os.replace(tmp, self.index_path)

    def add(self, name: str, src_dir: str) -> dict:
        dst = os.path.join(self.root, name)
        if os.path.abspath(src_dir) != os.path.abspath(dst):
            shutil.copytree(src_dir, dst, dirs_exist_ok=True)
        files = {}
        for fn in sorted(os.listdir(dst)):
            p = os.path.join(dst, fn)
            if os.path.isfile(p):
                files[fn] = {"sha256": file_digest(p), "bytes": os.path.getsize(p)}
        entry = {"path": dst, "files": files, "model_id": hashlib.sha256(
            json.dumps(files, sort_keys=True).encode()).hexdigest()[:16]}
        self.index[name] = entry
        self._save()
        return entry

    def list(self) -> list[str]:
        return sorted(self.index)

    def path(self, name: str) -> str:
        return self.index[name]["path"]

    def verify(self, name: str) -> list[str]:
        """Names of files whose digest no longer matches (empty = intact)."""
        bad = []
        e = self.index[name]
        for fn, meta in e["files"].items():
            p = os.path.join(e["path"], fn)
            if not os.path.exists(p) or file_digest(p) != meta["sha256"]:
                bad.append(fn)
        return bad

    def remove(self, name: str):
        e = self.index.pop(name)
        shutil.rmtree(e["path"], ignore_errors=True)
        self._save()
