"""Immutable, content-addressed artifact generations with publication locks.

Reference behaviour (``difflet/serving/artifact_manager.py:31-319``): an artifact (a compiled
bundle, a decoded video and its metadata) is published as a new *generation* that is never
modified afterwards: files are staged in a private directory, fsynced, inventoried (path, size,
sha256 per file; the content digest is the sha256 of that inventory), then renamed into place in
one step, under an exclusive lock so that concurrent publishers of the same name serialise.
Readers resolve the newest generation whose inventory still validates, or a pinned digest; a
generation whose files were altered is rejected, and staging directories abandoned by a crashed
publisher are removed on the next publication.

Storage is bounded as in the reference's video storage (``difflet/serving/video_storage.py:133-604``):
a publication larger than ``max_bytes`` (8 GiB by default) is refused before anything is written,
and so is one that would leave less than ``reserve_bytes`` free on the file system.  ``delete``
removes every generation of a name in one rename (readers see all of it or none) and ``sweep``
removes the names a caller no longer knows (what a crash between a job record's deletion and
its files' left behind) together with abandoned staging and trash directories.

Layout::

    <root>/<name>/generations/<generation id>/files...   + inventory.json
    <root>/<name>/.staging/<random>/                       (in-flight publications)
    <root>/<name>/.lock
    <root>/.trash/<random>/                                 (deleted names, removed after the rename)
"""

from __future__ import annotations

import fcntl
import hashlib
import json
import os
import shutil
import time
import uuid
from contextlib import contextmanager
from dataclasses import dataclass
from pathlib import Path

INVENTORY = "inventory.json"


class ArtifactIntegrityError(RuntimeError):
    """A generation's files no longer match its inventory."""


class ArtifactTooLarge(ValueError):
    """A publication above the store's size limit."""


class ArtifactNoSpace(OSError):
    """A publication that would leave less than the reserved free space."""

DEFAULT_MAX_BYTES = 8 << 30
DEFAULT_RESERVE_BYTES = 1 << 30


@dataclass(frozen=True)
class Generation:
    name: str
    id: str
    digest: str
    path: Path
    files: tuple

    def file(self, rel: str) -> Path:
        return self.path / rel


def _sha256_file(p: Path) -> str:
    h = hashlib.sha256()
    with open(p, "rb") as f:
        for chunk in iter(lambda: f.read(1 << 20), b""):
            h.update(chunk)
    return h.hexdigest()


def _fsync_dir(p: Path) -> None:
    fd = os.open(str(p), os.O_RDONLY)
    try:
        os.fsync(fd)
    finally:
        os.close(fd)


class ImmutableArtifacts:
    def __init__(self, root: str | os.PathLike, *, lock_timeout: float = 300.0, max_bytes: int = DEFAULT_MAX_BYTES,
                 reserve_bytes: int = DEFAULT_RESERVE_BYTES):
        self.root = Path(root).resolve()
        self.lock_timeout = lock_timeout
        self.max_bytes = int(max_bytes)
        self.reserve_bytes = int(reserve_bytes)
        self.root.mkdir(parents=True, exist_ok=True)

    def available_bytes(self) -> int:
        st = os.statvfs(self.root)
        return st.f_bavail * st.f_frsize

    def _check_size(self, files: dict) -> int:
        total = 0
        for rel, content in files.items():
            if isinstance(content, (bytes, bytearray)):
                total += len(content)
            else:
                src = Path(content)
                if src.is_symlink() or not src.is_file():
                    raise ValueError(f"artifact source {rel!r} must be a regular file, not {src}")
                total += src.stat().st_size
        if total > self.max_bytes:
            raise ArtifactTooLarge(f"{total} bytes exceed the artifact limit of {self.max_bytes}")
        if self.available_bytes() - total < self.reserve_bytes:
            raise ArtifactNoSpace(f"publishing {total} bytes would leave under {self.reserve_bytes} bytes free")
        return total

    # ---------------------------------------------------------------------- helpers
    def _base(self, name: str) -> Path:
        if not name or "/" in name or name.startswith(".") or len(name) > 200:
            raise ValueError(f"bad artifact name {name!r}")
        base = self.root / name
        if base.is_symlink():
            raise ValueError(f"artifact directory {base} is a symbolic link")
        return base

    @contextmanager
    def _locked(self, name: str):
        base = self._base(name)
        base.mkdir(parents=True, exist_ok=True)
        with open(base / ".lock", "a+") as fh:
            deadline = time.monotonic() + self.lock_timeout
            while True:
                try:
                    fcntl.flock(fh.fileno(), fcntl.LOCK_EX | fcntl.LOCK_NB)
                    break
                except BlockingIOError:
                    if time.monotonic() > deadline:
                        raise TimeoutError(f"artifact {name!r} is locked by another publisher") from None
                    time.sleep(0.05)
            try:
                yield base
            finally:
                fcntl.flock(fh.fileno(), fcntl.LOCK_UN)

    @staticmethod
    def _inventory(root: Path) -> list[dict]:
        out = []
        for p in sorted(root.rglob("*")):
            if p.is_file() and p.name != INVENTORY:
                rel = p.relative_to(root).as_posix()
                out.append({"path": rel, "size": p.stat().st_size, "sha256": _sha256_file(p)})
        return out

    @staticmethod
    def _digest(inventory: list[dict]) -> str:
        blob = json.dumps(inventory, sort_keys=True, separators=(",", ":")).encode()
        return hashlib.sha256(blob).hexdigest()

    # ---------------------------------------------------------------------- publish / resolve
    def publish(self, name: str, files: dict) -> Generation:
        """Publish ``files`` ({relative path: bytes or a source file path}) as a new generation."""
        self._check_size(files)
        with self._locked(name) as base:
            staging_root = base / ".staging"
            if staging_root.exists():  # abandoned by a crashed publisher (we hold the lock)
                shutil.rmtree(staging_root)
            stage = staging_root / uuid.uuid4().hex
            stage.mkdir(parents=True)
            for rel, content in files.items():
                dst = (stage / rel).resolve()
                if not str(dst).startswith(str(stage.resolve()) + os.sep):
                    raise ValueError(f"artifact file escapes its generation: {rel!r}")
                dst.parent.mkdir(parents=True, exist_ok=True)
                if isinstance(content, (bytes, bytearray)):
                    with open(dst, "wb") as f:
                        f.write(content)
                        f.flush()
                        os.fsync(f.fileno())
                else:
                    shutil.copyfile(content, dst)
                    with open(dst, "rb") as f:
                        os.fsync(f.fileno())
            inv = self._inventory(stage)
            digest = self._digest(inv)
            with open(stage / INVENTORY, "w") as f:
                json.dump({"name": name, "digest": digest, "files": inv, "created": time.time()}, f)
                f.flush()
                os.fsync(f.fileno())
            gens = base / "generations"
            gens.mkdir(exist_ok=True)
            gen_id = f"{int(time.time() * 1e3):013d}-{digest[:12]}"
            final = gens / gen_id
            os.rename(stage, final)  # the generation appears complete or not at all
            _fsync_dir(gens)
            shutil.rmtree(staging_root, ignore_errors=True)
            return Generation(name, gen_id, digest, final, tuple(e["path"] for e in inv))

    def _load(self, name: str, gen_dir: Path, verify: bool) -> Generation:
        with open(gen_dir / INVENTORY) as f:
            meta = json.load(f)
        if verify:
            inv = self._inventory(gen_dir)
            if inv != meta["files"] or self._digest(inv) != meta["digest"]:
                raise ArtifactIntegrityError(f"generation {gen_dir.name} of {name!r} no longer matches its inventory")
        return Generation(name, gen_dir.name, meta["digest"], gen_dir, tuple(e["path"] for e in meta["files"]))

    def generations(self, name: str) -> list[str]:
        gens = self._base(name) / "generations"
        return sorted(p.name for p in gens.iterdir() if p.is_dir()) if gens.exists() else []

    def resolve(self, name: str, digest: str | None = None, verify: bool = True) -> Generation | None:
        """The newest generation that validates (or the one with ``digest``); None if there is none."""
        gens = self._base(name) / "generations"
        for gid in reversed(self.generations(name)):
            try:
                g = self._load(name, gens / gid, verify)
            except (ArtifactIntegrityError, OSError, ValueError, KeyError):
                if digest is not None and gid.endswith(digest[:12]):
                    raise
                continue
            if digest is None or g.digest == digest:
                return g
        return None


    # ---------------------------------------------------------------------- retention
    def names(self) -> list[str]:
        return sorted(p.name for p in self.root.iterdir() if p.is_dir() and not p.name.startswith("."))

    def delete(self, name: str) -> bool:
        """Remove every generation of ``name``; False when it had none.  The directory is renamed
        out of the way under the publication lock first, so a reader never sees part of it."""
        base = self._base(name)
        if not base.exists():
            return False
        trash = self.root / ".trash"
        trash.mkdir(exist_ok=True)
        with self._locked(name):
            dst = trash / uuid.uuid4().hex
            try:
                os.rename(base, dst)
            except FileNotFoundError:  # a concurrent delete (the retention sweep) got there first
                return False
            _fsync_dir(self.root)
        shutil.rmtree(dst, ignore_errors=True)
        return True

    def sweep(self, keep) -> list[str]:
        """Delete the names not in ``keep`` and leftover trash; returns the names removed."""
        keep = set(keep)
        gone = [n for n in self.names() if n not in keep]
        for n in gone:
            self.delete(n)
        shutil.rmtree(self.root / ".trash", ignore_errors=True)
        return gone


__all__ = ["ArtifactIntegrityError", "ArtifactNoSpace", "ArtifactTooLarge", "Generation", "ImmutableArtifacts"]
