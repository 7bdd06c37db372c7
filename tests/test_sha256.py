"""SHA-256 kernels against hashlib (CPU host twin; GPU kernel)."""
import hashlib

import pytest
import torch

from autodrive_b200.ops import require_extension
from autodrive_b200.utils.provenance import chunk_digests, state_dict_digest, tensor_digest


def _tree(data: bytes, chunk: int) -> str:
    level = [hashlib.sha256(data[i:i + chunk]).digest() for i in range(0, max(len(data), 1), chunk)] or \
        [hashlib.sha256(b"").digest()]
    while len(level) > 1:
        level = [hashlib.sha256(level[i] + level[i + 1]).digest() if i + 1 < len(level) else level[i]
                 for i in range(0, len(level), 2)]
    return level[0].hex()


@pytest.mark.parametrize("n", [0, 1, 55, 56, 63, 64, 65, 119, 1000, 70000])
def test_host_digests_match_hashlib(n):
    g = torch.Generator().manual_seed(n)
    t = torch.randint(0, 256, (n,), dtype=torch.uint8, generator=g)
    data = bytes(t.tolist())
    assert chunk_digests(t, 1 << 20)[0] == hashlib.sha256(data).hexdigest()
    assert tensor_digest(t, 100) == _tree(data, 100)


def test_state_dict_digest_detects_changes():
    sd = {"w": torch.arange(10.), "b": torch.zeros(3)}
    d1 = state_dict_digest(sd)
    sd["w"][3] += 1e-6
    assert state_dict_digest(sd) != d1


@pytest.mark.gpu
def test_gpu_matches_host():
    g = torch.Generator().manual_seed(5)
    t = torch.randint(0, 256, (3 * 4096 + 17,), dtype=torch.uint8, generator=g)
    ext = require_extension()
    assert torch.equal(ext.sha256_chunks(t.cuda(), 4096).cpu(), ext.sha256_chunks(t, 4096))
    assert tensor_digest(t.cuda(), 1000) == tensor_digest(t, 1000) == _tree(bytes(t.tolist()), 1000)
    w = torch.randn(1000, 137)
    assert tensor_digest(w.cuda()) == tensor_digest(w)


def test_native_extension_identity():
    """The loaded extension is the in-tree file mapped into this process, and
    (once built with its manifest) matches the manifest and current sources."""
    from autodrive_b200.ops.ext import build_fingerprint, native_extension_identity, source_digests
    ident = native_extension_identity()
    assert ident["mapped"] in (True, None) and len(ident["sha256"]) == 64
    assert ident["path"].endswith(".so")
    assert "sim.cu" in source_digests() and len(build_fingerprint()) == 64
    if ident["manifest_binary_match"] is not None:
        assert ident["manifest_binary_match"]
