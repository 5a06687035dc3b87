"""The pack cache's host side: keying by checkpoint files and layout version, atomic writes, the
free-space rule, the off switch, and the library's blob validation, which refuses malformed or
foreign blobs before any device call (so it runs here, without a GPU)."""
import os
import struct
import time

import numpy as np
import pytest

from opennpu_b200 import libonpu as L
from opennpu_b200.packcache import PackCache


def _blob(kind=L.BLOB_DENSE, mats=((64, 64, 1, 2, 0),), version=None, extra=0, cut=0, nbytes=None):
    """A blob with zero weights: mats = (N, K, E, fmt, flags) per matrix, payload sized by the
    GPU layout (rows in groups of 64, K in chunks of 64, 576-byte strips; 640 for q4nx)."""
    lib = L.load()
    v = lib.onpu_layout_version() if version is None else version
    out = bytearray(L.BLOB_MAGIC + struct.pack("<IIII", v, kind, len(mats), 0) + bytes(40))
    for N, K, E, fmt, flags in mats:
        pay = ((N + 63) // 64) * ((K + 63) // 64) * 4 * (640 if fmt == 0 else 576) * E
        out += struct.pack("<qqqiIq", N, K, E, fmt, flags, pay if nbytes is None else nbytes) + bytes(24)
        out += bytes((pay + 63) // 64 * 64)
    out += bytes(extra)
    return np.frombuffer(bytes(out[:len(out) - cut]), dtype=np.uint8)


@pytest.fixture
def ckpt(tmp_path):
    d = tmp_path / "ckpt"
    d.mkdir()
    (d / "model.safetensors").write_bytes(b"x" * 100)
    (d / "config.json").write_text("{}")
    return d


def test_entries_follow_checkpoint_files(ckpt, tmp_path):
    """An entry counts only while the checkpoint's *.safetensors / *.json files are unchanged
    (names, sizes, mtimes); other files do not matter; the first store after a change empties the
    directory."""
    root = tmp_path / "cache"
    blob = _blob()
    c = PackCache(ckpt, root=root, keep_free=0)
    assert c.save_blob("w", blob)
    assert np.array_equal(PackCache(ckpt, root=root).load_blob("w"), blob)
    (ckpt / "notes.txt").write_text("ignored")                         # not a checkpoint file
    assert PackCache(ckpt, root=root).load_blob("w") is not None
    manifests = []
    for change in (lambda: (ckpt / "model.safetensors").write_bytes(b"x" * 101),          # size
                   lambda: os.utime(ckpt / "model.safetensors", (time.time() + 100,) * 2),  # mtime
                   lambda: (ckpt / "generation_config.json").write_text("{}")):           # a new file
        change()
        c2 = PackCache(ckpt, root=root, keep_free=0)
        assert c2.root == c.root and not c2.current()
        assert c2.load_blob("w") is None and c2.misses == 1
        assert c2.save_blob("v", blob) and c2.current()
        assert not c2._path("w").exists() and c2._path("v").exists()   # the stale entry was dropped
        assert c2.save_blob("w", blob)
        manifests.append(c2.manifest)
    assert manifests[0] != manifests[1] != manifests[2]
    assert c.root.parent == root / f"gpu-layout-v{L.load().onpu_layout_version()}"
    assert c.root.name.startswith("ckpt-")


def test_checkpoints_with_one_name_do_not_share_entries(tmp_path):
    a, b = tmp_path / "a" / "ckpt", tmp_path / "b" / "ckpt"
    for d in (a, b):
        d.mkdir(parents=True)
        (d / "model.safetensors").write_bytes(b"y")
    assert PackCache(a, root=tmp_path / "cache").root != PackCache(b, root=tmp_path / "cache").root


def test_save_then_load_is_atomic_and_exact(ckpt, tmp_path):
    c = PackCache(ckpt, root=tmp_path / "cache", keep_free=0)
    blob = _blob(mats=((128, 96, 1, 1, 1),))
    assert c.load_blob("layer.0.mlp") is None and c.misses == 1
    assert c.save_blob("layer.0.mlp", blob)
    got = c.load_blob("layer.0.mlp")
    assert np.array_equal(got, blob)
    assert not list(c.root.glob("*.tmp"))
    assert c.load_blob("layer.1.mlp") is None                          # names do not collide
    assert c._path("a/b") != c._path("a_b")
    c2 = PackCache(ckpt, root=tmp_path / "cache", keep_free=0)         # a second load finds it
    assert np.array_equal(c2.load_blob("layer.0.mlp"), blob)


def test_free_space_rule_and_off_switch(ckpt, tmp_path, monkeypatch):
    c = PackCache(ckpt, root=tmp_path / "cache", keep_free=1 << 62)
    assert not c.save_blob("w", _blob())
    assert not c._path("w").exists()
    monkeypatch.setenv("OPENNPU_NPU4_CACHE", "0")
    off = PackCache(ckpt, root=tmp_path / "cache", keep_free=0)
    assert not off.save_blob("w", _blob())
    assert off.load_blob("w") is None and not off._path("w").exists()


def test_blob_of_another_layout_version_is_a_miss(ckpt, tmp_path):
    c = PackCache(ckpt, root=tmp_path / "cache", keep_free=0)
    c.save_blob("w", _blob(version=L.load().onpu_layout_version() + 1))
    assert c.load_blob("w") is None and c.misses == 1
    c._path("v").write_bytes(b"not a blob at all")
    assert c.load_blob("v") is None


def test_blob_headers_parse():
    kind, mats = L.blob_sections(_blob(kind=L.BLOB_FFN, mats=((1536, 2048, 4, 2, 1), (2048, 768, 4, 2, 0))))
    assert kind == L.BLOB_FFN
    assert [(m["N"], m["K"], m["E"], m["flags"]) for m in mats] == [(1536, 2048, 4, 1), (2048, 768, 4, 0)]


@pytest.mark.parametrize("case,blob,fn,msg", [
    ("short", np.zeros(10, np.uint8), "onpu_dense_import", "shorter than its header"),
    ("magic", np.zeros(256, np.uint8), "onpu_dense_import", "bad magic"),
    ("version", _blob(version=999), "onpu_dense_import", "layout version"),
    ("kind", _blob(kind=L.BLOB_BANK), "onpu_dense_import", "expected kind"),
    ("nmats", _blob(kind=L.BLOB_FFN), "onpu_ffn_import", "expected kind"),
    ("truncated", _blob(cut=64), "onpu_dense_import", "truncated"),
    ("trailing", _blob(extra=64), "onpu_dense_import", "after the last matrix"),
    ("bytes", _blob(nbytes=1024), "onpu_dense_import", "payload bytes"),
    ("fmt", _blob(mats=((64, 64, 1, 7, 0),)), "onpu_dense_import", "invalid header"),
    ("flags", _blob(mats=((64, 64, 1, 2, 4),)), "onpu_dense_import", "invalid header"),
    ("k32", _blob(mats=((64, 48, 1, 2, 0),)), "onpu_dense_import", "invalid header"),
    ("n0", _blob(mats=((0, 64, 1, 2, 0),)), "onpu_dense_import", "invalid header"),
    ("experts", _blob(mats=((64, 64, 2, 2, 0),)), "onpu_dense_import", "one matrix"),
    ("both", _blob(mats=((64, 64, 1, 2, 3),)), "onpu_dense_import", "not both"),
    ("bank2pass", _blob(kind=L.BLOB_BANK, mats=((64, 64, 2, 2, 2),)), "onpu_bank_import", "two-pass"),
    ("ffnE", _blob(kind=L.BLOB_FFN, mats=((128, 64, 2, 2, 1), (64, 64, 3, 2, 0))), "onpu_ffn_import",
     "same expert count"),
])
def test_library_refuses_malformed_blobs(case, blob, fn, msg):
    lib = L.load()
    assert getattr(lib, fn)(blob.ctypes.data, blob.size) is None
    assert msg in (L.last_error() or ""), (case, L.last_error())
