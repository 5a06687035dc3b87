"""Packed weights on disk in the GPU layout, so a model's second load skips reading and quantising
the checkpoint and the GPU repack: it reads each matrix's blob and makes one host->device copy.

Mirrors the reference's ``PackCache`` (opennpu/native/npu4/model.py:712-759): one file per
buffer, keyed by the checkpoint (file names, sizes and mtimes of its ``*.safetensors`` and
``*.json``) and the packing version, written atomically (``.part`` then rename) and only while
``KEEP_FREE`` bytes of disk stay free; ``OPENNPU_NPU4_CACHE=0`` turns it off. The version here is
the library's GPU layout version (``onpu_layout_version``): a layout change gives a new cache
directory, and the library refuses a blob of another version, which then reads as a miss.

The files are the blobs of ``DenseMatrix.export`` / ``ExpertFFN.export`` (onpu_*_export).
"""
import hashlib
import os
from pathlib import Path

import numpy as np

from . import libonpu as L


def default_root():
    """$OPENNPU_CACHE_DIR, else ~/.cache/opennpu_b200."""
    env = os.environ.get("OPENNPU_CACHE_DIR")
    return Path(env) if env else Path.home() / ".cache" / "opennpu_b200"


class PackCache:
    VERSION = "b200-gpu-layout"
    KEEP_FREE = 20 * 2**30

    def __init__(self, ckpt_dir, root=None, keep_free=None):
        d = Path(ckpt_dir).resolve()
        sig = [self.VERSION, str(L.load().onpu_layout_version()), str(d)]
        for f in sorted(d.glob("*.safetensors")) + sorted(d.glob("*.json")):
            st = f.stat()
            sig.append(f"{f.name}:{st.st_size}:{int(st.st_mtime)}")
        base = Path(root) if root is not None else default_root()
        self.root = base / "npu4" / (d.name + "-" + hashlib.sha1("|".join(sig).encode()).hexdigest()[:12])
        self.keep_free = self.KEEP_FREE if keep_free is None else keep_free
        self.enabled = os.environ.get("OPENNPU_NPU4_CACHE", "1") != "0"
        self.hits = self.misses = 0

    def _path(self, name):
        return self.root / (hashlib.sha1(name.encode()).hexdigest()[:20] + ".bin")

    # ---------------------------------------------------------------- raw blobs
    def load_blob(self, name):
        """The stored blob (uint8 numpy array), or None (off, absent, or not a blob of this version)."""
        p = self._path(name)
        if not self.enabled or not p.exists():
            self.misses += 1
            return None
        blob = np.fromfile(p, dtype=np.uint8)
        try:
            kind, mats = L.blob_sections(blob)
            ok = all(m["version"] == L.load().onpu_layout_version() for m in mats)
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
        import shutil
        if shutil.disk_usage(self.root).free < blob.size + self.keep_free:
            return False
        p = self._path(name)
        tmp = p.with_suffix(".part")
        with open(tmp, "wb") as f:
            f.write(memoryview(blob))
        tmp.replace(p)
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
