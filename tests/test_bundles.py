"""On-disk bundles (``raon_npu_b200.bundles``): manifest validation, file
verification and expert slices on CPU, following the reference's bundle
contract (``npu/backend.py:104-117,285-346,729-752,1095-1118``); one GPU test
that a bundle-uploaded matrix computes exactly what the direct upload does."""

from __future__ import annotations

import hashlib
import json

import numpy as np
import pytest

from raon_npu_b200 import bundles as bd


def _write(tmp, entries, files):
    """files: rel -> bytes; entries: manifest bundle dicts (sha/size filled in when absent)."""
    for rel, data in files.items():
        p = tmp / rel
        p.parent.mkdir(parents=True, exist_ok=True)
        p.write_bytes(data)
    for e in entries:
        data = files.get(e["file"], b"")
        e.setdefault("size_bytes", len(data))
        e.setdefault("sha256", hashlib.sha256(data).hexdigest())
    (tmp / "manifest.json").write_text(json.dumps({"version": "1.0", "bundles": entries}))


def _entry(name, fmt, rel, shape, **kw):
    e = {"bundle": name, "format": fmt, "file": rel, "original_shape": list(shape), "padded_shape": list(shape)}
    e.update(kw)
    return e


def _rand(n, seed=0):
    return np.random.default_rng(seed).integers(0, 256, n, dtype=np.uint8).tobytes()


@pytest.fixture
def good(tmp_path):
    files = {"L00/proj.bin": _rand(128 * 256 * 5 // 8, 1), "lm_head.bin": _rand(128 * 512 * 9 // 8, 2),
             "L01/moe_b1.bin": _rand(3 * 256 * 256 * 5 // 8, 3)}
    entries = [_entry("L00/proj", "q4nx_gemv", "L00/proj.bin", (128, 256), layer=0),
               _entry("lm_head", "bfp16_gemv", "lm_head.bin", (128, 512)),
               _entry("L01/moe_b1", "q4nx_gemv_bundle", "L01/moe_b1.bin", (3, 256, 256), layer=1,
                      expert_count=3, expert_bytes=256 * 256 * 5 // 8),
               {"bundle": "host_global", "format": "host_safetensors", "file": "host_global.safetensors"}]
    _write(tmp_path, entries, files)
    return tmp_path, files


def test_manifest_reads_and_slices(good):
    root, files = good
    m = bd.read_manifest(root)
    assert set(m) == {"L00/proj", "lm_head", "L01/moe_b1"}          # host tensors are skipped
    assert m["lm_head"].weight_format == "bfp16" and (m["lm_head"].rows, m["lm_head"].cols) == (128, 512)
    assert bd.read_matrix(root, m["L00/proj"]) == files["L00/proj.bin"]
    eb = m["L01/moe_b1"].expert_bytes
    for e in range(3):
        assert bd.read_matrix(root, m["L01/moe_b1"], e) == files["L01/moe_b1.bin"][e * eb:(e + 1) * eb]
    with pytest.raises(ValueError):
        bd.read_matrix(root, m["L01/moe_b1"], 3)
    with pytest.raises(ValueError):
        bd.read_matrix(root, m["L00/proj"], 0)


def test_bare_list_manifest(tmp_path):
    files = {"a.bin": _rand(128 * 256 * 5 // 8)}
    _write(tmp_path, [_entry("a", "q4nx_gemv", "a.bin", (128, 256))], files)
    payload = json.loads((tmp_path / "manifest.json").read_text())["bundles"]
    (tmp_path / "manifest.json").write_text(json.dumps(payload))
    assert list(bd.read_manifest(tmp_path)) == ["a"]


@pytest.mark.parametrize("change, message", [
    (lambda e: e.update(size_bytes=e["size_bytes"] + 1), "size_bytes"),
    (lambda e: e.update(sha256="xyz"), "sha256"),
    (lambda e: e.update(file="../outside.bin"), "escapes"),
    (lambda e: e.update(format="q8_gemv"), "unknown format"),
    (lambda e: e.update(padded_shape=[128, 300], original_shape=[128, 300]), "tile-aligned"),
    (lambda e: e.update(original_shape=[256, 256]), "exceeds"),
])
def test_manifest_rejections(tmp_path, change, message):
    files = {"a.bin": _rand(128 * 256 * 5 // 8)}
    e = _entry("a", "q4nx_gemv", "a.bin", (128, 256))
    _write(tmp_path, [e], files)
    change(e)
    (tmp_path / "manifest.json").write_text(json.dumps({"bundles": [e]}))
    with pytest.raises(ValueError, match=message):
        bd.read_manifest(tmp_path)


def test_duplicate_and_expert_geometry(tmp_path):
    files = {"a.bin": _rand(128 * 256 * 5 // 8), "m.bin": _rand(2 * 128 * 256 * 5 // 8)}
    a = _entry("a", "q4nx_gemv", "a.bin", (128, 256))
    _write(tmp_path, [a, dict(a)], files)
    with pytest.raises(ValueError, match="duplicate"):
        bd.read_manifest(tmp_path)
    m = _entry("m", "q4nx_gemv_bundle", "m.bin", (2, 128, 256), expert_count=2, expert_bytes=999)
    _write(tmp_path, [m], files)
    with pytest.raises(ValueError, match="expert_bytes"):
        bd.read_manifest(tmp_path)


def test_file_tampering_detected(good):
    root, files = good
    m = bd.read_manifest(root)
    data = bytearray(files["L00/proj.bin"])
    data[5] ^= 1
    (root / "L00/proj.bin").write_bytes(bytes(data))
    with pytest.raises(ValueError, match="sha256"):
        bd.read_matrix(root, m["L00/proj"])
    (root / "lm_head.bin").write_bytes(files["lm_head.bin"][:-9])
    with pytest.raises(ValueError, match="size_bytes"):
        bd.read_matrix(root, m["lm_head"])
    (root / "lm_head.bin").unlink()
    with pytest.raises(FileNotFoundError):
        bd.read_matrix(root, m["lm_head"])


def test_components(tmp_path):
    files = {"a.bin": _rand(128 * 512 * 5 // 8), "b.bin": _rand(128 * 256 * 5 // 8)}
    a = _entry("a", "q4nx_gemv", "a.bin", (128, 512), original_shape=[120, 448],
               components=[{"name": "q_proj", "row_start": 0, "row_end": 64},
                           {"name": "kv_proj", "row_start": 64, "row_end": 120}])
    b = _entry("b", "q4nx_gemv", "b.bin", (128, 256))
    _write(tmp_path, [a, b], files)
    m = bd.read_manifest(tmp_path)
    assert m["a"].components == (bd.Component("q_proj", 0, 64), bd.Component("kv_proj", 64, 120))
    assert m["b"].components == ()
    for comps, message in (([{"name": "x", "row_start": 0, "row_end": 129}], "outside"),
                           ([{"name": "x", "row_start": 5, "row_end": 5}], "outside"),
                           ([{"name": "q_proj"}], "duplicate"),
                           ([{"row_start": 0}], "invalid component"),
                           ({"name": "x"}, "invalid components")):
        b2 = dict(b, components=comps)
        _write(tmp_path, [a, b2], files)
        with pytest.raises(ValueError, match=message):
            bd.read_manifest(tmp_path)


def test_load_moe_experts_passes_the_down_format(tmp_path):
    """q4nx gate/up (moe_b1) with a bfp16ebs8 down bundle (moe_b2): every
    expert's slices reach the layer with ``down_format="bfp16"``; a bfp16
    gate/up bundle is refused."""
    E, H, I = 3, 256, 256
    gu_b, dn_b = 2 * I * H * 5 // 8, H * I * 9 // 8
    files = {"b1.bin": _rand(E * gu_b, 4), "b2.bin": _rand(E * dn_b, 5), "b2q.bin": _rand(E * dn_b, 6)}
    _write(tmp_path, [_entry("L1/moe_b1", "q4nx_gemv_bundle", "b1.bin", (E, 2 * I, H), expert_count=E,
                             expert_bytes=gu_b),
                      _entry("L1/moe_b2", "bfp16_gemv_bundle", "b2.bin", (E, H, I), expert_count=E,
                             expert_bytes=dn_b),
                      _entry("L1/bad_b1", "bfp16_gemv_bundle", "b2q.bin", (E, H, I), expert_count=E,
                             expert_bytes=dn_b)], files)

    class Layer:
        def __init__(self):
            self.calls = []

        def set_expert(self, e, gu, dn, down_format="q4nx"):
            self.calls.append((e, gu, dn, down_format))

    loader = bd.BundleLoader(None, tmp_path)
    layer = Layer()
    loader.load_moe_experts(layer, "L1/moe_b1", "L1/moe_b2")
    assert [c[0] for c in layer.calls] == [0, 1, 2]
    for e, gu, dn, fmt in layer.calls:
        assert fmt == "bfp16"
        assert gu == files["b1.bin"][e * gu_b:(e + 1) * gu_b] and dn == files["b2.bin"][e * dn_b:(e + 1) * dn_b]
    with pytest.raises(ValueError, match="gate/up"):
        loader.load_moe_experts(layer, "L1/bad_b1", "L1/moe_b2")


@pytest.mark.gpu
def test_backend_load_bundles_components(tmp_path):
    """CudaBackend.load_bundles: components are row slices of the uploaded
    matrix, and an unpadded activation of original K equals the zero-padded one."""
    from oracle import bfp16 as ob16
    from oracle import q4nx as oq
    from raon_npu_b200.backend import CudaBackend
    rng = np.random.default_rng(5)
    wq = (rng.standard_normal((256, 512)) * 0.02).astype(np.float32)
    wq[:, 448:] = 0.0
    q = oq.pack_gemv(*oq.quantize(wq))
    wb = (rng.standard_normal((128, 256)) * 0.02).astype(np.float32)
    bb = ob16.pack_gemv(wb)
    _write(tmp_path, [_entry("L0/qkv", "q4nx_gemv", "q.bin", (256, 512), original_shape=[200, 448],
                             components=[{"name": "q_proj", "row_start": 0, "row_end": 136},
                                         {"name": "kv_proj", "row_start": 136, "row_end": 200}]),
                      _entry("lm_head", "bfp16_gemv", "b.bin", (128, 256))],
           {"q.bin": q, "b.bin": bb})
    be = CudaBackend(0)
    try:
        be.load_bundles(tmp_path)
        direct = be.ctx.upload_q4nx(np.frombuffer(q, np.uint8), 256, 512)
        x = (rng.standard_normal((3, 448)) * 0.5).astype(np.float32)
        x16 = (x.view(np.uint32) >> 16).astype(np.uint16)
        xp = np.zeros((3, 512), np.uint16)
        xp[:, :448] = x16
        full = direct.gemv_host(xp)
        assert np.array_equal(be.linear("q_proj", x16), full[:, :136])
        assert np.array_equal(be.linear("kv_proj", x16), full[:, 136:200])
        with pytest.raises(KeyError):
            be.linear("L0/qkv", x16)
        xl = np.ascontiguousarray(xp[:, :256])
        yl = be.linear("lm_head", xl)
        e, mnt = ob16.parse_gemv(bb, 256, 128)
        ref = np.stack([ob16.gemv(e, mnt, xl[t]) for t in range(3)])
        diff = np.abs(yl.astype(np.int32) - ref.astype(np.int32))
        assert diff.max() <= 1 and (diff > 0).mean() <= 0.05
        direct.free()
    finally:
        be.close()


@pytest.mark.gpu
def test_bundle_upload_matches_direct_upload(tmp_path):
    import torch
    from oracle import bfp16 as ob16
    from oracle import q4nx as oq
    from raon_npu_b200.build import build
    from raon_npu_b200.device import Context
    build()
    rng = np.random.default_rng(11)
    wq = (rng.standard_normal((256, 512)) * 0.02).astype(np.float32)
    q = oq.pack_gemv(*oq.quantize(wq))
    wb = (rng.standard_normal((384, 512)) * 0.02).astype(np.float32)
    bb = ob16.pack_gemv(wb)
    _write(tmp_path, [_entry("q", "q4nx_gemv", "q.bin", (256, 512)), _entry("b", "bfp16_gemv", "b.bin", (384, 512))],
           {"q.bin": q, "b.bin": bb})
    ctx = Context(0)
    try:
        loader = bd.BundleLoader(ctx, tmp_path)
        x = torch.randn((3, 512), device="cuda").to(torch.bfloat16).view(torch.int16).contiguous()
        for name, direct in (("q", ctx.upload_q4nx(np.frombuffer(q, np.uint8), 256, 512)),
                             ("b", ctx.upload_bfp16(np.frombuffer(bb, np.uint8), 384, 512))):
            w = loader.upload(name)
            y0 = torch.empty((3, w.n), dtype=torch.int16, device="cuda")
            y1 = torch.empty_like(y0)
            w.gemv_into(x, y0, 3)
            direct.gemv_into(x, y1, 3)
            torch.cuda.synchronize()
            assert torch.equal(y0, y1), name
            w.free()
            direct.free()
        ctx.sync()
    finally:
        ctx.close()
