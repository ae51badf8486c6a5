"""Image / video output without external codecs.

Images are PNG (PIL).  Videos are Motion-JPEG in an AVI (RIFF) container written
here in pure Python with PIL encoding each frame -- a standard, widely playable
format (the reference encodes MP4 through PyAV, ``difflet/serving/video_media.py:51-133``,
which this image does not ship).
"""

from __future__ import annotations

import io
import struct
from pathlib import Path

import numpy as np


def save_image(img, path: str) -> str:
    from PIL import Image

    arr = img.cpu().numpy() if hasattr(img, "cpu") else np.asarray(img)
    Image.fromarray(arr.astype(np.uint8)).save(path)
    return path


def encode_png(img) -> bytes:
    from PIL import Image

    arr = img.cpu().numpy() if hasattr(img, "cpu") else np.asarray(img)
    buf = io.BytesIO()
    Image.fromarray(arr.astype(np.uint8)).save(buf, format="PNG")
    return buf.getvalue()


def _chunk(tag: bytes, data: bytes) -> bytes:
    pad = b"\0" if len(data) % 2 else b""
    return tag + struct.pack("<I", len(data)) + data + pad


def _list(tag: bytes, body: bytes) -> bytes:
    return b"LIST" + struct.pack("<I", len(body) + 4) + tag + body


def encode_mjpeg_avi(frames, fps: int = 16, quality: int = 90) -> bytes:
    """frames: [F, H, W, 3] uint8 -> AVI bytes (MJPEG)."""
    from PIL import Image

    arr = frames.cpu().numpy() if hasattr(frames, "cpu") else np.asarray(frames)
    F, H, W, _ = arr.shape
    jpgs = []
    for f in range(F):
        b = io.BytesIO()
        Image.fromarray(arr[f].astype(np.uint8)).save(b, format="JPEG", quality=quality)
        jpgs.append(b.getvalue())
    usec = int(1_000_000 / fps)
    maxbytes = max(len(j) for j in jpgs)
    avih = struct.pack("<IIIIIIIIIIIIII", usec, maxbytes * fps, 0, 0x10, F, 0, 1, maxbytes, W, H, 0, 0, 0, 0)
    strh = struct.pack("<4s4sIHHIIIIIIIIhhhh", b"vids", b"MJPG", 0, 0, 0, 0, 1, fps, 0, F, maxbytes, 0xFFFFFFFF, 0,
                       0, 0, W, H)
    strf = struct.pack("<IiiHH4sIiiII", 40, W, H, 1, 24, b"MJPG", W * H * 3, 0, 0, 0, 0)
    hdrl = _list(b"hdrl", _chunk(b"avih", avih) + _list(b"strl", _chunk(b"strh", strh) + _chunk(b"strf", strf)))
    movi_body = b""
    index = b""
    off = 4
    for j in jpgs:
        c = _chunk(b"00dc", j)
        index += struct.pack("<4sIII", b"00dc", 0x10, off, len(j))
        movi_body += c
        off += len(c)
    movi = _list(b"movi", movi_body)
    body = b"AVI " + hdrl + movi + _chunk(b"idx1", index)
    return b"RIFF" + struct.pack("<I", len(body)) + body


def save_video(frames, path: str, fps: int = 16) -> str:
    p = Path(path)
    if p.suffix.lower() not in (".avi",):
        p = p.with_suffix(".avi")
    p.write_bytes(encode_mjpeg_avi(frames, fps))
    return str(p)
