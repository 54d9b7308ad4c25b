"""Local model registry and downloader (reference ``src/model_hub.rs``).

Registry entries (repo id, file name, alias, local path, SHA-256) live in
``~/.air/registry.json``; files under ``~/.air/models/``. ``pull`` downloads
``https://huggingface.co/<repo>/resolve/main/<file>`` and verifies the digest when one is
known; ``resolve`` maps an alias / repo id / file name to a local path without network.
"""
from __future__ import annotations

import hashlib
import json
import os
import urllib.request
from dataclasses import asdict, dataclass

HF_BASE_URL = "https://huggingface.co"


def _home() -> str:
    return os.environ.get("AIR_HOME", os.path.join(os.path.expanduser("~"), ".air"))


@dataclass
class ModelEntry:
    repo_id: str
    filename: str
    alias: str | None = None
    local_path: str | None = None
    sha256: str | None = None
    size_bytes: int = 0


class ModelRegistry:
    def __init__(self, entries: list[ModelEntry] | None = None):
        self.entries = entries or []

    @staticmethod
    def path() -> str:
        return os.path.join(_home(), "registry.json")

    @classmethod
    def load(cls) -> "ModelRegistry":
        p = cls.path()
        if not os.path.exists(p):
            return cls()
        with open(p) as f:
            data = json.load(f)
        return cls([ModelEntry(**e) for e in data.get("models", [])])

    def save(self):
        os.makedirs(_home(), exist_ok=True)
        with open(self.path(), "w") as f:
            json.dump({"models": [asdict(e) for e in self.entries]}, f, indent=2)

    def find(self, key: str) -> ModelEntry | None:
        for e in self.entries:
            if key in (e.alias, e.repo_id, e.filename, f"{e.repo_id}/{e.filename}"):
                return e
        return None

    def register(self, entry: ModelEntry):
        self.entries = [e for e in self.entries if not (e.repo_id == entry.repo_id and e.filename == entry.filename)]
        self.entries.append(entry)
        self.save()

    def list(self) -> list[ModelEntry]:
        return list(self.entries)


def sha256_file(path: str, chunk: int = 1 << 22) -> str:
    h = hashlib.sha256()
    with open(path, "rb") as f:
        while True:
            b = f.read(chunk)
            if not b:
                break
            h.update(b)
    return h.hexdigest()


def download_url(repo_id: str, filename: str) -> str:
    return f"{HF_BASE_URL}/{repo_id}/resolve/main/{filename}"


def pull(repo_id: str, filename: str, alias: str | None = None, sha256: str | None = None) -> str:
    """Download a GGUF into the model cache and register it (needs network access)."""
    dest_dir = os.path.join(_home(), "models", repo_id.replace("/", "__"))
    os.makedirs(dest_dir, exist_ok=True)
    dest = os.path.join(dest_dir, filename)
    if not os.path.exists(dest):
        tmp = dest + ".part"
        urllib.request.urlretrieve(download_url(repo_id, filename), tmp)
        os.replace(tmp, dest)
    digest = sha256_file(dest)
    if sha256 and digest != sha256:
        os.remove(dest)
        raise ValueError(f"checksum mismatch for {filename}: {digest} != {sha256}")
    reg = ModelRegistry.load()
    reg.register(ModelEntry(repo_id, filename, alias, dest, digest, os.path.getsize(dest)))
    return dest


def resolve(key: str) -> str:
    if os.path.exists(key):
        return key
    e = ModelRegistry.load().find(key)
    if e is None or not e.local_path or not os.path.exists(e.local_path):
        raise FileNotFoundError(f"{key!r} is neither a file nor a registered model (run `air-rs pull`)")
    return e.local_path
