"""Page-cache control limited to the files a benchmark reads, without root.

A cold end-to-end run must load the weights from storage, a warm one from memory.  Dropping the
whole host's page cache needs root and slows every other job on the machine, so this module
touches only the given files: ``evict`` asks the kernel to drop their pages
(``posix_fadvise(POSIX_FADV_DONTNEED)``), ``warm`` reads them through once, and ``residency``
measures how much of each file is actually cached (``mincore`` over a read-only mapping).  The
kernel drops only clean, unmapped, unlocked pages -- another process that maps the same weights
keeps them resident -- so a run records the measured residency instead of assuming the eviction
worked.  Reference behaviour: ``difflet/bench/pagecache.py``.
"""

from __future__ import annotations

import ctypes
import ctypes.util
import mmap
import os
from pathlib import Path
from typing import Iterable

_PAGE = mmap.PAGESIZE
_libc = None


def _mincore():
    global _libc
    if _libc is None:
        _libc = ctypes.CDLL(ctypes.util.find_library("c") or "libc.so.6", use_errno=True)
        _libc.mincore.argtypes = (ctypes.c_void_p, ctypes.c_size_t, ctypes.POINTER(ctypes.c_ubyte))
        _libc.mincore.restype = ctypes.c_int
    return _libc.mincore


def files_under(paths: Iterable[str | os.PathLike], suffixes=(".safetensors", ".bin", ".pt", ".json")) -> list[Path]:
    """The regular files named, and those under the directories named (weights and configs)."""
    out = []
    for p in map(Path, paths):
        if p.is_file():
            out.append(p)
        elif p.is_dir():
            out += sorted(q for q in p.rglob("*") if q.is_file() and not q.is_symlink() and q.suffix in suffixes)
    return out


def evict(files: Iterable[str | os.PathLike]) -> int:
    """Ask the kernel to drop the files' cached pages; returns the bytes covered."""
    total = 0
    for f in files:
        fd = os.open(f, os.O_RDONLY)
        try:
            if os.access(f, os.W_OK):
                os.fsync(fd)  # only clean pages can be dropped
            os.posix_fadvise(fd, 0, 0, os.POSIX_FADV_DONTNEED)
            total += os.fstat(fd).st_size
        finally:
            os.close(fd)
    return total


def warm(files: Iterable[str | os.PathLike], chunk: int = 8 << 20) -> int:
    """Read the files through once so their pages are cached; returns the bytes read."""
    total = 0
    for f in files:
        with open(f, "rb", buffering=0) as fh:
            while True:
                b = fh.read(chunk)
                if not b:
                    break
                total += len(b)
    return total


def residency(files: Iterable[str | os.PathLike]) -> dict:
    """{"bytes", "resident_bytes", "fraction", "files": {path: fraction}} measured with mincore."""
    mincore = _mincore()
    per, total, resident = {}, 0, 0
    for f in files:
        size = os.path.getsize(f)
        if size == 0:
            per[str(f)] = 1.0
            continue
        with open(f, "rb") as fh, mmap.mmap(fh.fileno(), size, prot=mmap.PROT_READ) as mm:
            pages = (size + _PAGE - 1) // _PAGE
            vec = (ctypes.c_ubyte * pages)()
            if mincore(ctypes.c_void_p(_buffer_address(mm)), size, vec) != 0:
                raise OSError(ctypes.get_errno(), "mincore failed", str(f))
            res_pages = sum(v & 1 for v in vec)
        r = min(size, res_pages * _PAGE)
        per[str(f)] = round(r / size, 4)
        total += size
        resident += r
    return {"bytes": total, "resident_bytes": resident, "fraction": round(resident / total, 4) if total else 1.0,
            "files": per}


class _Py_buffer(ctypes.Structure):
    _fields_ = [("buf", ctypes.c_void_p), ("obj", ctypes.py_object), ("len", ctypes.c_ssize_t),
                ("itemsize", ctypes.c_ssize_t), ("readonly", ctypes.c_int), ("ndim", ctypes.c_int),
                ("format", ctypes.c_char_p), ("shape", ctypes.c_void_p), ("strides", ctypes.c_void_p),
                ("suboffsets", ctypes.c_void_p), ("internal", ctypes.c_void_p)]


def _buffer_address(obj) -> int:
    """Start address of an object's buffer (a read-only mapping: ctypes' ``from_buffer`` wants
    a writable one)."""
    b = _Py_buffer()
    get = ctypes.pythonapi.PyObject_GetBuffer
    get.argtypes = (ctypes.py_object, ctypes.POINTER(_Py_buffer), ctypes.c_int)
    get.restype = ctypes.c_int
    if get(obj, ctypes.byref(b), 0) != 0:
        raise OSError("buffer of the mapping is not available")
    try:
        return int(b.buf)
    finally:
        rel = ctypes.pythonapi.PyBuffer_Release
        rel.argtypes = (ctypes.POINTER(_Py_buffer),)
        rel(ctypes.byref(b))


__all__ = ["evict", "files_under", "residency", "warm"]
