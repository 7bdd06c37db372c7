"""Loader for the in-tree native extension ``autodrive_b200._C``.

The extension is built in place by ``python setup.py build_ext --inplace``
(``__graft_entry__.build`` does this). It holds both the sm_100a kernels and
their host twins. There is deliberately no pure-Python fallback for the
simulator: a missing extension is an error on every device.
"""
from __future__ import annotations

import importlib

_EXT = None
_ERR: Exception | None = None


def extension():
    global _EXT, _ERR
    if _EXT is None and _ERR is None:
        try:
            import torch  # noqa: F401 - loads libc10 / libtorch, which _C links against
            _EXT = importlib.import_module("autodrive_b200._C")
        except Exception as exc:  # noqa: BLE001 - surfaced by require_extension
            _ERR = exc
    return _EXT


def require_extension():
    ext = extension()
    if ext is None:
        raise RuntimeError(
            "autodrive_b200._C is not built; run `python setup.py build_ext --inplace` "
            f"({type(_ERR).__name__}: {_ERR})")
    return ext


# ---------------------------------------------------------------------------
# Identity of the loaded native binary (provenance for checkpoints and runs):
# the in-tree file that is actually mapped into this process, its SHA-256,
# and whether it matches the build manifest written next to it by the build
# (binary digest and the digests of every C++/CUDA source it was built from).
# ---------------------------------------------------------------------------
import hashlib as _hashlib
import json as _json
import os as _os
from pathlib import Path as _Path

_CSRC = _Path(__file__).resolve().parent.parent / "csrc"
_MANIFEST_NAME = "_C.manifest.json"


def source_digests() -> dict[str, str]:
    """SHA-256 of every C++ / CUDA source and header of the extension."""
    out = {}
    for p in sorted(_CSRC.iterdir()):
        if p.suffix in (".cu", ".cpp", ".h", ".cuh"):
            out[p.name] = _hashlib.sha256(p.read_bytes()).hexdigest()
    return out


def build_fingerprint(digests: dict[str, str] | None = None) -> str:
    digests = source_digests() if digests is None else digests
    return _hashlib.sha256(_json.dumps(digests, sort_keys=True).encode()).hexdigest()


def _file_identity(path: _Path) -> dict:
    before = path.stat()
    digest = _hashlib.sha256(path.read_bytes()).hexdigest()
    after = path.stat()
    if (before.st_ino, before.st_size, before.st_mtime_ns) != (after.st_ino, after.st_size, after.st_mtime_ns):
        raise RuntimeError(f"{path} changed while its digest was read")
    return {"path": str(path), "sha256": digest, "size": after.st_size, "mtime_ns": after.st_mtime_ns,
            "device": after.st_dev, "inode": after.st_ino}


def write_build_manifest(binary: str | _Path) -> dict:
    """Record the built binary's digest and its sources' digests beside it."""
    binary = _Path(binary).resolve()
    digests = source_digests()
    manifest = {"module": "autodrive_b200._C", "binary_sha256": _file_identity(binary)["sha256"],
                "build_fingerprint": build_fingerprint(digests), "sources": digests,
                "arch": "sm_100a"}
    tmp = binary.with_name(_MANIFEST_NAME + ".tmp")
    tmp.write_text(_json.dumps(manifest, indent=1, sort_keys=True))
    tmp.replace(binary.with_name(_MANIFEST_NAME))
    return manifest


def _mapped(path: _Path) -> bool:
    """The binary at `path` (same device and inode) is mapped into this
    process (Linux /proc/self/maps); None where that file does not exist."""
    maps = _Path("/proc/self/maps")
    if not maps.exists():
        return None
    st = path.stat()
    want = (_os.major(st.st_dev), _os.minor(st.st_dev), st.st_ino)
    for line in maps.read_text().splitlines():
        parts = line.split(None, 5)
        if len(parts) < 6 or not parts[5].endswith(path.name):
            continue
        major, minor = (int(x, 16) for x in parts[3].split(":"))
        if (major, minor, int(parts[4])) == want:
            return True
    return False


def native_extension_identity(strict: bool = False) -> dict:
    """Identity of the loaded extension: its in-tree path, SHA-256, the check
    that this very file is mapped into the process, and whether it matches
    the build manifest (binary digest and current sources). With `strict`, a
    mismatch raises instead of being reported."""
    ext = require_extension()
    path = _Path(ext.__file__).resolve()
    ident = {"module": "autodrive_b200._C", **_file_identity(path), "mapped": _mapped(path)}
    manifest_path = path.with_name(_MANIFEST_NAME)
    if manifest_path.exists():
        manifest = _json.loads(manifest_path.read_text())
        ident["manifest_binary_match"] = manifest.get("binary_sha256") == ident["sha256"]
        ident["sources_match_build"] = manifest.get("build_fingerprint") == build_fingerprint()
        ident["build_fingerprint"] = manifest.get("build_fingerprint")
    else:
        ident["manifest_binary_match"] = ident["sources_match_build"] = None
    if strict:
        if ident["mapped"] is False:
            raise RuntimeError(f"the loaded extension is not the file at {path}")
        if ident["manifest_binary_match"] is False:
            raise RuntimeError("the extension binary differs from its build manifest")
        if ident["sources_match_build"] is False:
            raise RuntimeError("the extension sources changed after the build; rebuild it")
    return ident
