"""Artifact stores for generated media: a local directory, or any S3-compatible object store
reached through presigned URLs (no cloud SDK: requests are signed here with AWS Signature
Version 4, query-string form, from the published algorithm).

Reference behaviour (``difflet/serving/artifact_store.py:20-256``): ``put_bytes`` stores an
object under ``<prefix>/<key>`` and returns a reference; ``get_url`` returns a time-limited URL
a client can fetch without credentials; configuration from ``DIFFLET_S3_*`` variables
(bucket, endpoint, access key id / secret / session token, region, addressing style, timeout).
"""

from __future__ import annotations

import datetime as _dt
import hashlib
import hmac
import os
import urllib.parse
import urllib.request
from dataclasses import dataclass


@dataclass(frozen=True)
class ArtifactRef:
    key: str
    size: int
    sha256: str
    content_type: str


class LocalArtifactStore:
    """Objects as files under ``root`` (written to a temporary name, fsynced, renamed)."""

    def __init__(self, root: str, base_url: str | None = None):
        self.root = os.path.abspath(root)
        self.base_url = base_url
        os.makedirs(self.root, exist_ok=True)

    def _path(self, key: str) -> str:
        p = os.path.abspath(os.path.join(self.root, key))
        if not p.startswith(self.root + os.sep):
            raise ValueError(f"artifact key escapes the store: {key!r}")
        return p

    def put_bytes(self, key: str, data: bytes, content_type: str = "application/octet-stream") -> ArtifactRef:
        path = self._path(key)
        os.makedirs(os.path.dirname(path), exist_ok=True)
        tmp = path + ".partial"
        with open(tmp, "wb") as f:
            f.write(data)
            f.flush()
            os.fsync(f.fileno())
        os.replace(tmp, path)
        return ArtifactRef(key, len(data), hashlib.sha256(data).hexdigest(), content_type)

    def get_bytes(self, ref: ArtifactRef) -> bytes:
        with open(self._path(ref.key), "rb") as f:
            return f.read()

    def delete(self, key: str) -> bool:
        """Remove an object; False when there was none."""
        try:
            os.unlink(self._path(key))
            return True
        except FileNotFoundError:
            return False

    def get_url(self, ref: ArtifactRef, ttl_seconds: int = 3600) -> str:
        if self.base_url:
            return self.base_url.rstrip("/") + "/" + urllib.parse.quote(ref.key)
        return "file://" + self._path(ref.key)


# ------------------------------------------------------------------------------ SigV4 presign
def _q(s: str, safe: str = "-_.~") -> str:
    """RFC 3986 percent-encoding (unreserved characters kept)."""
    return urllib.parse.quote(s, safe=safe)


def _hmac(key: bytes, msg: str) -> bytes:
    return hmac.new(key, msg.encode(), hashlib.sha256).digest()


def presign_url(method: str, *, host: str, path: str, access_key: str, secret_key: str, region: str,
                expires: int, when: _dt.datetime, scheme: str = "https", session_token: str | None = None,
                service: str = "s3") -> str:
    """A presigned URL (AWS Signature Version 4, query-string authentication, unsigned payload):
    canonical request -> string to sign -> HMAC chain date / region / service / aws4_request."""
    amz_date = when.strftime("%Y%m%dT%H%M%SZ")
    day = when.strftime("%Y%m%d")
    scope = f"{day}/{region}/{service}/aws4_request"
    params = {
        "X-Amz-Algorithm": "AWS4-HMAC-SHA256",
        "X-Amz-Credential": f"{access_key}/{scope}",
        "X-Amz-Date": amz_date,
        "X-Amz-Expires": str(int(expires)),
        "X-Amz-SignedHeaders": "host",
    }
    if session_token:
        params["X-Amz-Security-Token"] = session_token
    query = "&".join(f"{_q(k)}={_q(v)}" for k, v in sorted(params.items()))
    canonical_path = _q(path, safe="/-_.~")
    canonical = "\n".join([method, canonical_path, query, f"host:{host}\n", "host", "UNSIGNED-PAYLOAD"])
    to_sign = "\n".join(["AWS4-HMAC-SHA256", amz_date, scope, hashlib.sha256(canonical.encode()).hexdigest()])
    key = _hmac(("AWS4" + secret_key).encode(), day)
    for part in (region, service, "aws4_request"):
        key = _hmac(key, part)
    signature = hmac.new(key, to_sign.encode(), hashlib.sha256).hexdigest()
    return f"{scheme}://{host}{canonical_path}?{query}&X-Amz-Signature={signature}"


class S3ArtifactStore:
    """A private bucket of an S3-compatible store; objects are written and read through presigned
    URLs (PUT with the body, GET for clients)."""

    def __init__(self, *, bucket: str, endpoint_url: str | None = None, access_key_id: str | None = None,
                 secret_access_key: str | None = None, session_token: str | None = None, prefix: str = "difflet",
                 region: str | None = None, addressing_style: str | None = None, timeout: float = 60.0):
        if not bucket:
            raise ValueError("an S3 artifact store needs a bucket")
        if bool(access_key_id) != bool(secret_access_key):
            raise ValueError("give the S3 access key id and secret access key together")
        if session_token and not access_key_id:
            raise ValueError("an S3 session token needs explicit access keys")
        if addressing_style not in (None, "auto", "virtual", "path"):
            raise ValueError("S3 addressing style is one of auto, virtual, path")
        if not access_key_id:
            raise ValueError("presigned URLs need credentials (DIFFLET_S3_ACCESS_KEY_ID / _SECRET_ACCESS_KEY)")
        self.bucket, self.prefix = bucket, prefix.strip("/")
        self.access_key, self.secret_key, self.session_token = access_key_id, secret_access_key, session_token
        self.region = region or "us-east-1"
        self.timeout = float(timeout)
        if endpoint_url:
            u = urllib.parse.urlsplit(endpoint_url)
            self.scheme, self.endpoint_host = u.scheme or "https", u.netloc
            style = addressing_style if addressing_style in ("virtual", "path") else "path"
        else:
            self.scheme, self.endpoint_host = "https", f"s3.{self.region}.amazonaws.com"
            style = addressing_style if addressing_style in ("virtual", "path") else "virtual"
        self.style = style

    @classmethod
    def from_env(cls) -> "S3ArtifactStore":
        env = os.environ
        missing = [n for n in ("DIFFLET_S3_BUCKET", "DIFFLET_S3_ACCESS_KEY_ID", "DIFFLET_S3_SECRET_ACCESS_KEY")
                   if not env.get(n, "").strip()]
        if missing:
            raise ValueError("S3 artifact store is not configured; missing " + ", ".join(missing))
        return cls(bucket=env["DIFFLET_S3_BUCKET"].strip(), endpoint_url=env.get("DIFFLET_S3_ENDPOINT_URL") or None,
                   access_key_id=env["DIFFLET_S3_ACCESS_KEY_ID"].strip(),
                   secret_access_key=env["DIFFLET_S3_SECRET_ACCESS_KEY"].strip(),
                   session_token=env.get("DIFFLET_S3_SESSION_TOKEN") or None, prefix=env.get("DIFFLET_S3_PREFIX", "difflet"),
                   region=env.get("DIFFLET_S3_REGION") or env.get("AWS_REGION") or env.get("AWS_DEFAULT_REGION"),
                   addressing_style=env.get("DIFFLET_S3_ADDRESSING_STYLE") or None,
                   timeout=float(env.get("DIFFLET_S3_CLIENT_TIMEOUT", "60")))

    @classmethod
    def from_env_if_configured(cls) -> "S3ArtifactStore | None":
        if not any(k.startswith("DIFFLET_S3_") for k in os.environ):
            return None
        return cls.from_env()

    def _object(self, key: str) -> tuple[str, str]:
        full = f"{self.prefix}/{key}" if self.prefix else key
        if self.style == "virtual":
            return f"{self.bucket}.{self.endpoint_host}", "/" + full
        return self.endpoint_host, f"/{self.bucket}/{full}"

    def presign(self, method: str, key: str, ttl_seconds: int, when: _dt.datetime | None = None) -> str:
        host, path = self._object(key)
        when = when or _dt.datetime.now(_dt.timezone.utc)
        return presign_url(method, host=host, path=path, access_key=self.access_key, secret_key=self.secret_key,
                           region=self.region, expires=ttl_seconds, when=when, scheme=self.scheme,
                           session_token=self.session_token)

    def put_bytes(self, key: str, data: bytes, content_type: str = "application/octet-stream") -> ArtifactRef:
        url = self.presign("PUT", key, 900)
        req = urllib.request.Request(url, data=data, method="PUT", headers={"Content-Type": content_type})
        with urllib.request.urlopen(req, timeout=self.timeout) as resp:
            if resp.status // 100 != 2:
                raise OSError(f"S3 PUT of {key!r} failed with HTTP {resp.status}")
        return ArtifactRef(key, len(data), hashlib.sha256(data).hexdigest(), content_type)

    def get_url(self, ref: ArtifactRef, ttl_seconds: int = 3600) -> str:
        return self.presign("GET", ref.key, ttl_seconds)

    def get_bytes(self, ref: ArtifactRef) -> bytes:
        with urllib.request.urlopen(self.get_url(ref, 300), timeout=self.timeout) as resp:
            return resp.read()

    def delete(self, key: str) -> bool:
        """DELETE through a presigned URL; a missing object (404) counts as deleted.  Raises
        OSError on any other failure so the caller can retry later."""
        import urllib.error

        req = urllib.request.Request(self.presign("DELETE", key, 900), method="DELETE")
        try:
            with urllib.request.urlopen(req, timeout=self.timeout) as resp:
                if resp.status // 100 != 2:
                    raise OSError(f"S3 DELETE of {key!r} failed with HTTP {resp.status}")
        except urllib.error.HTTPError as exc:
            if exc.code == 404:
                return False
            raise OSError(f"S3 DELETE of {key!r} failed with HTTP {exc.code}") from exc
        return True


def make_artifact_store(local_dir: str | None = None):
    """S3 when any ``DIFFLET_S3_*`` variable is set, else a local directory."""
    s3 = S3ArtifactStore.from_env_if_configured()
    if s3 is not None:
        return s3
    import tempfile

    return LocalArtifactStore(local_dir or tempfile.mkdtemp(prefix="difflet_artifacts_"))


__all__ = ["ArtifactRef", "LocalArtifactStore", "S3ArtifactStore", "make_artifact_store", "presign_url"]
