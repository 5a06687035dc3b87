"""Packed weights on disk in the GPU layout, so a model's second load skips reading and quantising
the checkpoint and the GPU repack: it reads each matrix's blob and makes one host->device copy.

The reference keeps its NPU upload bytes in a cache of the same purpose (PackCache,
opennpu/native/npu4/model.py:712-759): entries invalidated by a change to the checkpoint's
``*.safetensors`` / ``*.json`` files, written atomically, stored only while enough disk stays free
(20 GiB), switched off by ``OPENNPU_NPU4_CACHE=0``. Those behaviours are kept; the store is this
library's own:

- ``<root>/gpu-layout-v<N>/<checkpoint dir name>-<crc32 of its path>/``: one directory per
  checkpoint and GPU layout version (``onpu_layout_version``), so a layout change never meets an
  old blob (the library would refuse it anyway: it reads as a miss);
- ``manifest.json`` in it records the layout version and the checkpoint's fingerprint (name,
  size, mtime in ns of every ``*.safetensors`` / ``*.json``); entries count only while the
  manifest matches the checkpoint as it is now, and the first store after a change empties the
  directory and writes the new manifest;
- one ``<name>-<crc32>.blob`` per entry, the blob of ``DenseMatrix.export`` / ``ExpertFFN.export``
  (onpu_*_export), written to a temporary file in the same directory and renamed over the entry.
"""
import json
import os
import re
import shutil
import tempfile
import zlib
from pathlib import Path

import numpy as np

from . import libonpu as L


def default_root():
    """$OPENNPU_CACHE_DIR, else ~/.cache/opennpu_b200."""
    env = os.environ.get("OPENNPU_CACHE_DIR")
    return Path(env) if env else Path.home() / ".cache" / "opennpu_b200"


def checkpoint_fingerprint(ckpt_dir):
    """[name, size, mtime_ns] of the checkpoint's weight and config files, sorted by name."""
    d = Path(ckpt_dir)
    files = [f for f in d.iterdir() if f.is_file() and f.suffix in (".safetensors", ".json")]
    return [[f.name, f.stat().st_size, f.stat().st_mtime_ns] for f in sorted(files, key=lambda f: f.name)]


def _crc(text):
    return f"{zlib.crc32(text.encode()):08x}"


def _atomic_write(path, data):
    fd, tmp = tempfile.mkstemp(dir=path.parent, prefix=path.name + ".", suffix=".tmp")
    try:
        with os.fdopen(fd, "wb") as f:
            f.write(data)
        os.replace(tmp, path)
    except BaseException:
        if os.path.exists(tmp):
            os.unlink(tmp)
        raise


class PackCache:
    KEEP_FREE = 20 * 2**30      # bytes of disk that must stay free after a store

    def __init__(self, ckpt_dir, root=None, keep_free=None):
        self.ckpt = Path(ckpt_dir).resolve()
        self.layout = int(L.load().onpu_layout_version())
        base = Path(root) if root is not None else default_root()
        self.root = base / f"gpu-layout-v{self.layout}" / f"{self.ckpt.name}-{_crc(str(self.ckpt))}"
        self.manifest = {"layout": self.layout, "files": checkpoint_fingerprint(self.ckpt)}
        self.keep_free = self.KEEP_FREE if keep_free is None else keep_free
        self.enabled = os.environ.get("OPENNPU_NPU4_CACHE", "1") != "0"
        self.hits = self.misses = 0

    def _path(self, name):
        stem = re.sub(r"[^A-Za-z0-9._-]", "_", name)[:96]
        return self.root / f"{stem}-{_crc(name)}.blob"

    def current(self):
        """True when the stored entries belong to the checkpoint as it is now."""
        try:
            return json.loads((self.root / "manifest.json").read_text()) == self.manifest
        except (OSError, ValueError):
            return False

    def _claim(self):
        """Before a store: a directory of another fingerprint is emptied and re-labelled."""
        if self.current():
            return
        self.root.mkdir(parents=True, exist_ok=True)
        for f in self.root.glob("*.blob"):
            f.unlink()
        _atomic_write(self.root / "manifest.json", json.dumps(self.manifest).encode())

    # ---------------------------------------------------------------- raw blobs
    def load_blob(self, name):
        """The stored blob (uint8 numpy array), or None (off, absent, stale, or not a blob of this
        layout version)."""
        p = self._path(name)
        if not self.enabled or not self.current() or not p.exists():
            self.misses += 1
            return None
        blob = np.fromfile(p, dtype=np.uint8)
        try:
            _, mats = L.blob_sections(blob)
            ok = all(m["version"] == self.layout for m in mats)
        except L.OnpuError:
            ok = False
        if not ok:
            self.misses += 1
            return None
        return blob

    def save_blob(self, name, blob):
        """Store a blob atomically; False when off or when the disk would keep less than keep_free."""
        if not self.enabled:
            return False
        blob = L.as_blob(blob)
        self.root.mkdir(parents=True, exist_ok=True)
        if shutil.disk_usage(self.root).free < blob.size + self.keep_free:
            return False
        self._claim()
        _atomic_write(self._path(name), memoryview(blob))
        return True

    # ---------------------------------------------------------------- handles
    def _get(self, name, build, from_blob):
        blob = self.load_blob(name)
        if blob is not None:
            try:
                obj = from_blob(blob)
            except L.OnpuError:          # a damaged or foreign file: rebuild and overwrite it
                self.misses += 1
            else:
                self.hits += 1
                return obj
        obj = build()
        self.save_blob(name, obj.export())
        return obj

    def dense(self, name, build):
        """The DenseMatrix stored as `name`, or build() (quantise / repack) and store it."""
        from .dense import DenseMatrix
        return self._get(name, build, DenseMatrix.from_blob)

    def experts(self, name, build):
        """The ExpertFFN stored as `name`, or build() and store it."""
        from .moe import ExpertFFN
        return self._get(name, build, ExpertFFN.from_blob)
