"""On-disk weight bundles: read the exporter's ``manifest.json`` + ``*.bin``
files, verify them, and upload them straight to the GPU.

Follows the reference's bundle contract (``npu/backend.py:104-117`` the
bundle record, ``:285-346`` path resolution and verification, ``:729-752``
canonical sizes, ``:1095-1118`` expert slices; ``export/README.md`` the
manifest keys):

* ``manifest.json`` is a dict with a ``bundles`` list (or a bare list); each
  entry has ``bundle`` (name), ``format`` (``q4nx_gemv``, ``bfp16_gemv``,
  ``q4nx_gemv_bundle``, ``bfp16_gemv_bundle``; ``host_safetensors`` entries are
  host tensors and skipped), ``file`` (relative to the manifest), ``size_bytes``,
  ``original_shape``, ``padded_shape``, ``sha256``, for MoE bundles
  ``expert_count`` / ``expert_bytes``, and optionally ``components``: the
  tensors packed into the bundle, each ``{"name", "row_start", "row_end"}``
  (``npu/backend.py:88-99,893-911``; several projections share one bundle).
* A file must resolve inside the weights directory; its size must equal both
  the manifest's ``size_bytes`` and the canonical size of its format and padded
  shape (q4nx: 5 bits, bfp16ebs8: 9 bits per weight; MoE bundles: experts x
  matrix bytes); its SHA-256 must match (checked once per file version: path,
  size and modification time).
* A ``*_gemv`` bundle is one [M, K] matrix (its padded shape) in the GEMV
  packing that ``rc_upload_q4nx`` / ``rc_upload_bfp16`` take unchanged; a
  ``*_gemv_bundle`` holds ``expert_count`` such matrices back to back.

Errors are the reference's: ``ValueError`` for a bad manifest, size or digest,
``FileNotFoundError`` for a missing file, ``KeyError`` for an unknown bundle.
"""

from __future__ import annotations

import hashlib
import json
import re
from dataclasses import dataclass
from pathlib import Path

GEMV_FORMATS = ("q4nx_gemv", "bfp16_gemv")
MOE_FORMATS = ("q4nx_gemv_bundle", "bfp16_gemv_bundle")


class _DigestMemo:
    """SHA-256 hex digests of files, remembered per file version: a file whose
    device, inode, size and change times are unchanged is not read again."""

    def __init__(self):
        self._by_version: dict[tuple[int, int, int, int, int], str] = {}

    def sha256(self, path: Path, st) -> str:
        version = (st.st_dev, st.st_ino, st.st_size, st.st_mtime_ns, st.st_ctime_ns)
        known = self._by_version.get(version)
        if known is None:
            with path.open("rb") as f:
                known = hashlib.file_digest(f, "sha256").hexdigest()
            self._by_version[version] = known
        return known


_DIGESTS = _DigestMemo()


@dataclass(frozen=True)
class Component:
    """A named tensor inside a bundle: rows [row_start, row_end) of its matrix."""
    name: str
    row_start: int
    row_end: int
    expert_id: int | None = None


@dataclass(frozen=True)
class Bundle:
    name: str
    fmt: str
    file: str
    size_bytes: int
    original_shape: tuple[int, ...]
    padded_shape: tuple[int, ...]
    sha256: str
    layer: int | None = None
    expert_count: int = 0
    expert_bytes: int = 0
    components: tuple[Component, ...] = ()

    @property
    def rows(self) -> int:
        return self.padded_shape[-2]

    @property
    def cols(self) -> int:
        return self.padded_shape[-1]

    @property
    def weight_format(self) -> str:
        return "q4nx" if self.fmt.startswith("q4nx") else "bfp16"


def matrix_bytes(fmt: str, rows: int, cols: int) -> int:
    """Packed bytes of one [rows, cols] matrix (``npu/backend.py:729-752``)."""
    if fmt.startswith("q4nx"):
        if rows % 32 or cols % 256:
            raise ValueError(f"q4nx shape [{rows}, {cols}] is not tile-aligned (32 x 256)")
        return rows * cols * 5 // 8
    if fmt.startswith("bfp16"):
        if cols % 8:
            raise ValueError(f"bfp16 shape [{rows}, {cols}] is not block-aligned (8 columns)")
        return rows * (cols // 8) * 9
    raise ValueError(f"unknown bundle format {fmt!r}")


def _positive_int(v) -> bool:
    return isinstance(v, int) and not isinstance(v, bool) and v >= 0


def read_manifest(weights_dir) -> dict[str, Bundle]:
    """Parse and validate ``weights_dir/manifest.json``; no file is read besides it."""
    root = Path(weights_dir)
    payload = json.loads((root / "manifest.json").read_text())
    if isinstance(payload, dict):
        entries = payload.get("bundles")
        if not isinstance(entries, list):
            raise ValueError("manifest dict missing 'bundles' list")
    elif isinstance(payload, list):
        entries = payload
    else:
        raise ValueError("invalid manifest top-level structure")
    out: dict[str, Bundle] = {}
    seen_components: set[str] = set()
    for item in entries:
        if not isinstance(item, dict):
            raise ValueError(f"invalid manifest bundle entry: {item!r}")
        fmt = item.get("format")
        if fmt == "host_safetensors":
            continue
        name = item.get("bundle")
        if not isinstance(name, str) or not name:
            raise ValueError(f"manifest bundle entry without a name: {item!r}")
        if name in out:
            raise ValueError(f"duplicate bundle in manifest: {name}")
        if fmt not in GEMV_FORMATS + MOE_FORMATS:
            raise ValueError(f"unknown format {fmt!r} for bundle {name}")
        rel = item.get("file")
        if not isinstance(rel, str) or not rel:
            raise ValueError(f"manifest file missing for {name}")
        size = item.get("size_bytes")
        if not _positive_int(size):
            raise ValueError(f"invalid size_bytes for {name}: {size!r}")
        sha = item.get("sha256")
        if not isinstance(sha, str) or not re.fullmatch(r"[0-9a-fA-F]{64}", sha):
            raise ValueError(f"invalid sha256 for {name}: {sha!r}")
        padded, orig = item.get("padded_shape"), item.get("original_shape")
        dims = 3 if fmt in MOE_FORMATS else 2
        for key, shape in (("padded_shape", padded), ("original_shape", orig)):
            if not (isinstance(shape, list) and len(shape) == dims and all(_positive_int(v) and v > 0 for v in shape)):
                raise ValueError(f"invalid {key} for {name}: {shape!r}")
        if any(o > p for o, p in zip(orig[-2:], padded[-2:])):
            raise ValueError(f"original_shape {orig} exceeds padded_shape {padded} for {name}")
        mbytes = matrix_bytes(fmt, padded[-2], padded[-1])
        count = ebytes = 0
        if fmt in MOE_FORMATS:
            count, ebytes = item.get("expert_count"), item.get("expert_bytes")
            if not _positive_int(count) or count != padded[0] or orig[0] != padded[0]:
                raise ValueError(f"expert_count mismatch for {name}: {count!r} vs shape {padded}")
            if ebytes != mbytes:
                raise ValueError(f"expert_bytes mismatch for {name}: {ebytes!r} != {mbytes}")
            canonical = mbytes * count
        else:
            canonical = mbytes
        if size != canonical:
            raise ValueError(f"canonical size_bytes mismatch for {name}: {size} != {canonical}")
        _resolve(root, rel, name)
        comps = _components(item.get("components", []), name, orig[-2], seen_components)
        out[name] = Bundle(name=name, fmt=fmt, file=rel, size_bytes=size, original_shape=tuple(orig),
                           padded_shape=tuple(padded), sha256=sha.lower(), layer=item.get("layer"),
                           expert_count=count, expert_bytes=ebytes, components=comps)
    return out


def _components(raw, bundle: str, rows: int, seen: set[str]) -> tuple[Component, ...]:
    """Validate a bundle's ``components`` list: named entries, unique over the
    manifest, rows inside the bundle's original rows (absent rows = all of them)."""
    if not isinstance(raw, list):
        raise ValueError(f"invalid components for {bundle}: {raw!r}")
    out = []
    for c in raw:
        if not isinstance(c, dict) or not isinstance(c.get("name"), str) or not c["name"]:
            raise ValueError(f"invalid component entry for {bundle}: {c!r}")
        cname = c["name"]
        if cname in seen:
            raise ValueError(f"duplicate component {cname!r} (bundle {bundle})")
        seen.add(cname)
        r0, r1 = c.get("row_start", 0), c.get("row_end", rows)
        if not (_positive_int(r0) and _positive_int(r1) and r0 < r1 <= rows):
            raise ValueError(f"row range of component {cname!r} outside bundle {bundle} of {rows} rows: "
                             f"({r0!r}, {r1!r})")
        eid = c.get("expert_id")
        if eid is not None and not _positive_int(eid):
            raise ValueError(f"invalid expert_id of component {cname!r}: {eid!r}")
        out.append(Component(cname, r0, r1, eid))
    return tuple(out)


def _resolve(root: Path, rel: str, name: str) -> Path:
    """The bundle file, which must lie inside the weights directory (``npu/backend.py:285-291``)."""
    base = root.resolve()
    path = (base / rel).resolve()
    try:
        path.relative_to(base)
    except ValueError as exc:
        raise ValueError(f"manifest file escapes the weights directory for {name}: {rel!r}") from exc
    return path


def verify(weights_dir, b: Bundle) -> Path:
    """The bundle's file after checking it against the manifest: it exists,
    its length is ``size_bytes`` and its SHA-256 is ``sha256`` (the contract of
    ``npu/backend.py:319-346``; the digest is computed once per file version)."""
    path = _resolve(Path(weights_dir), b.file, b.name)
    if not path.is_file():
        raise FileNotFoundError(f"bundle {b.name}: no file at {path}")
    st = path.stat()
    if st.st_size != b.size_bytes:
        raise ValueError(f"bundle {b.name}: {path.name} holds {st.st_size} bytes, size_bytes says {b.size_bytes}")
    if _DIGESTS.sha256(path, st) != b.sha256:
        raise ValueError(f"bundle {b.name}: the sha256 of {path.name} differs from the manifest's")
    return path


def read_matrix(weights_dir, b: Bundle, expert: int | None = None) -> bytes:
    """The packed bytes of a ``*_gemv`` bundle, or of one expert of a
    ``*_gemv_bundle`` (``npu/backend.py:1095-1118``), after verification."""
    path = verify(weights_dir, b)
    if b.fmt in GEMV_FORMATS:
        if expert is not None:
            raise ValueError(f"{b.name} is a single matrix, not an expert bundle")
        return path.read_bytes()
    if expert is None or not (0 <= expert < b.expert_count):
        raise ValueError(f"invalid expert slice request: {b.name} expert={expert}")
    with path.open("rb") as f:
        f.seek(expert * b.expert_bytes)
        chunk = f.read(b.expert_bytes)
    if len(chunk) != b.expert_bytes:
        raise ValueError(f"short read in {path} for expert {expert}: got {len(chunk)}, expected {b.expert_bytes}")
    return chunk


class BundleLoader:
    """Uploads verified bundles of a weights directory to a ``device.Context``."""

    def __init__(self, ctx, weights_dir):
        self.ctx = ctx
        self.dir = Path(weights_dir)
        self.bundles = read_manifest(self.dir)

    def __getitem__(self, name: str) -> Bundle:
        try:
            return self.bundles[name]
        except KeyError:
            raise KeyError(f"unknown bundle {name!r}") from None

    def upload(self, name: str, expert: int | None = None):
        """A ``Q4nxWeight`` / ``Bfp16Weight`` of the bundle's matrix (padded shape)."""
        import numpy as np
        b = self[name]
        data = np.frombuffer(read_matrix(self.dir, b, expert), dtype=np.uint8)
        if b.weight_format == "q4nx":
            return self.ctx.upload_q4nx(data, b.rows, b.cols)
        return self.ctx.upload_bfp16(data, b.rows, b.cols)

    def load_moe_experts(self, layer, gate_up: str, down: str, experts=None) -> None:
        """Feed a ``MoeLayer`` its experts from two expert bundles: q4nx gate/up
        [2I, H] and K-padded down [H, I_pad] in q4nx or bfp16ebs8 (the
        reference's ``moe_b1`` / ``moe_b2``); ``experts`` defaults to all of
        them, the shared one being id E if present."""
        gu, dn = self[gate_up], self[down]
        if gu.fmt != "q4nx_gemv_bundle":
            raise ValueError(f"{gu.name}: the MoE layer takes q4nx gate/up bundles, not {gu.fmt}")
        if dn.fmt not in MOE_FORMATS:
            raise ValueError(f"{dn.name}: not an expert bundle ({dn.fmt})")
        if gu.expert_count != dn.expert_count:
            raise ValueError(f"expert counts differ: {gu.name} {gu.expert_count}, {dn.name} {dn.expert_count}")
        for e in (range(gu.expert_count) if experts is None else experts):
            layer.set_expert(e, read_matrix(self.dir, gu, e), read_matrix(self.dir, dn, e), down_format=dn.weight_format)
