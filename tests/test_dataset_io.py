"""Dataset I/O in the reference's format (CPU only): the Blender transforms JSON +
PNG loader and writer of libnerf_b200 (nerf_b200_blender_*, nerf_b200_png_*).

The PNG decoder is checked against images encoded here with Python's zlib --
dynamic and fixed Huffman blocks, every PNG filter type, every colour type --
so the library's inflate and unfiltering are tested against an independent
encoder.  The camera remap is checked against a float32 restatement of the
reference driver's conversion (benchmark.cpp:148-286).
"""
import ctypes as C
import json
import os
import struct
import zlib

import numpy as np
import pytest

import nerf_b200
from nerf_b200 import abi


def _lib():
    return abi.load()


def _chunk(tag: bytes, data: bytes) -> bytes:
    return struct.pack(">I", len(data)) + tag + data + struct.pack(">I", zlib.crc32(tag + data) & 0xFFFFFFFF)


def _filter_rows(raw: np.ndarray, ch: int, filters) -> bytes:
    """Applies PNG filter types per row (raw: [h][w*ch] uint8)."""
    h, stride = raw.shape
    out = bytearray()
    prev = np.zeros(stride, np.int32)
    for y in range(h):
        cur = raw[y].astype(np.int32)
        f = filters[y % len(filters)]
        a = np.concatenate([np.zeros(ch, np.int32), cur[:-ch]])
        c = np.concatenate([np.zeros(ch, np.int32), prev[:-ch]])
        if f == 0:
            line = cur
        elif f == 1:
            line = cur - a
        elif f == 2:
            line = cur - prev
        elif f == 3:
            line = cur - ((a + prev) >> 1)
        else:
            p = a + prev - c
            pa, pb, pc = np.abs(p - a), np.abs(p - prev), np.abs(p - c)
            pred = np.where((pa <= pb) & (pa <= pc), a, np.where(pb <= pc, prev, c))
            line = cur - pred
        out.append(f)
        out += (line & 0xFF).astype(np.uint8).tobytes()
        prev = cur
    return bytes(out)


def _png(raw: np.ndarray, w: int, h: int, ctype: int, ch: int, filters, level=9, strategy=None, extra=b"") -> bytes:
    data = _filter_rows(raw.reshape(h, w * ch), ch, filters)
    if strategy is None:
        z = zlib.compress(data, level)
    else:
        co = zlib.compressobj(level, zlib.DEFLATED, 15, 9, strategy)
        z = co.compress(data) + co.flush()
    ihdr = struct.pack(">IIBBBBB", w, h, 8, ctype, 0, 0, 0)
    # two IDAT chunks: the decoder must concatenate them
    half = len(z) // 2
    return (b"\x89PNG\r\n\x1a\n" + _chunk(b"IHDR", ihdr) + extra + _chunk(b"IDAT", z[:half]) + _chunk(b"IDAT", z[half:])
            + _chunk(b"IEND", b""))


def _read(path):
    lib = _lib()
    w, h = C.c_uint32(), C.c_uint32()
    abi.check("png size", lib.nerf_b200_png_read(str(path).encode(), None, 0, C.byref(w), C.byref(h)))
    out = np.zeros((h.value, w.value, 4), np.uint8)
    abi.check("png read", lib.nerf_b200_png_read(str(path).encode(), out.ctypes.data, out.nbytes, None, None))
    return out


def _smooth_image(rng, h, w, ch):
    # smooth gradients plus noise: long matches for the compressor, all filter paths exercised
    y, x = np.mgrid[0:h, 0:w]
    base = np.stack([(x * 7 + y * 3 + 40 * k) % 256 for k in range(ch)], -1)
    noise = rng.integers(0, 4, size=(h, w, ch))
    return ((base + noise) % 256).astype(np.uint8)


@pytest.mark.parametrize("strategy", [None, zlib.Z_FIXED, zlib.Z_HUFFMAN_ONLY, zlib.Z_RLE])
@pytest.mark.parametrize("filters", [[0], [1], [2], [3], [4], [0, 1, 2, 3, 4]])
def test_png_decoder_rgba_against_zlib(tmp_path, strategy, filters):
    rng = np.random.default_rng(1)
    h, w = 37, 53
    img = _smooth_image(rng, h, w, 4)
    p = tmp_path / "a.png"
    p.write_bytes(_png(img, w, h, 6, 4, filters, strategy=strategy))
    assert np.array_equal(_read(p), img)


@pytest.mark.parametrize("ctype,ch", [(0, 1), (2, 3), (4, 2), (3, 1)])
def test_png_decoder_colour_types(tmp_path, ctype, ch):
    rng = np.random.default_rng(2)
    h, w = 19, 23
    img = _smooth_image(rng, h, w, ch)
    extra = b""
    if ctype == 3:  # palette of 256 colours, alpha for the first 100 entries
        pal = rng.integers(0, 256, size=(256, 3), dtype=np.uint8)
        trns = rng.integers(0, 256, size=100, dtype=np.uint8)
        extra = _chunk(b"PLTE", pal.tobytes()) + _chunk(b"tRNS", trns.tobytes())
    p = tmp_path / "c.png"
    p.write_bytes(_png(img, w, h, ctype, ch, [0, 1, 2, 3, 4], extra=extra))
    got = _read(p)
    if ctype == 0:
        want = np.concatenate([np.repeat(img, 3, -1), np.full((h, w, 1), 255, np.uint8)], -1)
    elif ctype == 2:
        want = np.concatenate([img, np.full((h, w, 1), 255, np.uint8)], -1)
    elif ctype == 4:
        want = np.concatenate([np.repeat(img[..., :1], 3, -1), img[..., 1:2]], -1)
    else:
        idx = img[..., 0].astype(np.int64)
        a = np.full(256, 255, np.uint8)
        a[:100] = trns
        want = np.concatenate([pal[idx], a[idx][..., None]], -1)
    assert np.array_equal(got, want)


def test_png_writer_roundtrip_and_zlib_compatible(tmp_path):
    rng = np.random.default_rng(3)
    img = rng.integers(0, 256, size=(70, 300, 4), dtype=np.uint8)  # rows of 1201 bytes: several stored blocks
    p = tmp_path / "w.png"
    abi.check("png write", _lib().nerf_b200_png_write(str(p).encode(), img.ctypes.data, 300, 70))
    assert np.array_equal(_read(p), img)
    # the written stream is plain zlib: Python decompresses it to the filtered rows
    b = p.read_bytes()
    assert b[:8] == b"\x89PNG\r\n\x1a\n"
    pos, idat = 8, b""
    while pos < len(b):
        n = struct.unpack(">I", b[pos:pos + 4])[0]
        tag = b[pos + 4:pos + 8]
        if tag == b"IDAT":
            idat += b[pos + 8:pos + 8 + n]
        pos += 12 + n
    rows = np.frombuffer(zlib.decompress(idat), np.uint8).reshape(70, 1 + 300 * 4)
    assert not rows[:, 0].any() and np.array_equal(rows[:, 1:].reshape(70, 300, 4), img)


def test_png_malformed_inputs(tmp_path):
    rng = np.random.default_rng(4)
    img = _smooth_image(rng, 8, 8, 4)
    good = _png(img, 8, 8, 6, 4, [4])
    lib = _lib()
    out = np.zeros((8, 8, 4), np.uint8)
    bad = {
        "signature": b"\x00" + good[1:],
        "crc": good[:40] + bytes([good[40] ^ 1]) + good[41:],
        "truncated": good[:-20],
        "empty": b"",
    }
    for name, data in bad.items():
        p = tmp_path / f"{name}.png"
        p.write_bytes(data)
        assert lib.nerf_b200_png_read(str(p).encode(), out.ctypes.data, out.nbytes, None, None) == abi.NERF_STATUS_IO_ERROR, name
    p = tmp_path / "ok.png"
    p.write_bytes(good)
    small = np.zeros(10, np.uint8)
    assert lib.nerf_b200_png_read(str(p).encode(), small.ctypes.data, small.nbytes, None, None) == abi.NERF_STATUS_INVALID_USAGE
    assert lib.nerf_b200_png_read(str(tmp_path / "missing.png").encode(), out.ctypes.data, out.nbytes, None, None) == \
        abi.NERF_STATUS_IO_ERROR


def _load(path, remap, n, w, h, threads=4):
    lib = _lib()
    imgs = np.zeros((n, h, w, 4), np.uint8)
    cams = np.zeros((n, 4, 4), np.float32)
    intr = np.zeros(4, np.float32)
    abi.check("blender load", lib.nerf_b200_blender_load(str(path).encode(), remap, threads, imgs.ctypes.data, imgs.nbytes,
                                                         cams.ctypes.data, intr.ctypes.data))
    return imgs, cams, intr


def _reference_remap(m: np.ndarray) -> np.ndarray:
    """float32 restatement of the reference driver's conversion (benchmark.cpp:211-286): W = basis of source world
    axes (+x, -z, +y), sums over k in order, translation * 0.33f then + 0.5f."""
    f = np.float32
    W = np.array([[1, 0, 0], [0, 0, 1], [0, -1, 0]], np.float32)
    out = np.zeros((4, 4), np.float32)
    rot, tr = m[:3, :3].astype(np.float32), m[:3, 3].astype(np.float32)
    tmp = np.zeros((3, 3), np.float32)
    for r in range(3):
        for c in range(3):
            s = f(0)
            for k in range(3):
                s = f(s + f(W[r, k] * rot[k, c]))
            tmp[r, c] = s
    for r in range(3):
        t = f(0)
        for k in range(3):
            t = f(t + f(W[r, k] * tr[k]))
        out[r, :3] = tmp[r]  # the camera basis map is the identity
        out[r, 3] = f(f(t * f(0.33)) + f(0.5))
    out[3, 3] = 1.0
    return out


def test_blender_write_probe_load_roundtrip(tmp_path):
    ds = nerf_b200.make_scene(kind=1, seed=3, n_primitives=4, n_views=5, width=40, height=24, fov=0.69, radius=4.0,
                              camera_mode=1)
    lib = _lib()
    imgs = np.ascontiguousarray(ds.images)
    cams = np.ascontiguousarray(ds.cameras)
    angle = 0.69
    abi.check("write", lib.nerf_b200_blender_write(str(tmp_path).encode(), imgs.ctypes.data, cams.ctypes.data, 5, 40, 24,
                                                  angle, 3))
    js = json.loads((tmp_path / "transforms_train.json").read_text())
    assert len(js["frames"]) == 5 and js["frames"][0]["file_path"] == "./train/r_0"
    info = abi.NerfB200BlenderInfo()
    abi.check("probe", lib.nerf_b200_blender_probe(str(tmp_path).encode(), C.byref(info)))  # directory form
    assert (info.image_count, info.width, info.height) == (5, 40, 24)
    assert info.camera_angle_x == np.float32(angle)
    got, gcams, intr = _load(tmp_path / "transforms_train.json", 0, 5, 40, 24)
    assert np.array_equal(got, imgs)
    assert np.array_equal(gcams, cams)  # %.9g round-trips every float32
    fx = np.float32(np.float32(0.5) * np.float32(40)) / np.float32(np.tan(np.float32(angle) * np.float32(0.5)))
    assert abs(intr[0] - fx) <= 2e-6 * fx and intr[1] == intr[0]
    assert intr[2] == np.float32(19.5) and intr[3] == np.float32(11.5)
    _, rcams, _ = _load(tmp_path, 1, 5, 40, 24, threads=1)
    for i in range(5):
        assert np.array_equal(rcams[i], _reference_remap(cams[i])), i


def test_blender_errors(tmp_path):
    lib = _lib()
    info = abi.NerfB200BlenderInfo()
    assert lib.nerf_b200_blender_probe(str(tmp_path / "none.json").encode(), C.byref(info)) == abi.NERF_STATUS_IO_ERROR
    (tmp_path / "bad.json").write_text('{"camera_angle_x": 0.5, "frames": [')
    assert lib.nerf_b200_blender_probe(str(tmp_path / "bad.json").encode(), C.byref(info)) == abi.NERF_STATUS_IO_ERROR
    # images of different sizes in one set
    rng = np.random.default_rng(5)
    a = rng.integers(0, 256, size=(8, 8, 4), dtype=np.uint8)
    b = rng.integers(0, 256, size=(8, 9, 4), dtype=np.uint8)
    for name, im in (("a", a), ("b", b)):
        abi.check("w", lib.nerf_b200_png_write(str(tmp_path / f"{name}.png").encode(), im.ctypes.data, im.shape[1], im.shape[0]))
    eye = np.eye(4).tolist()
    (tmp_path / "mixed.json").write_text(json.dumps({"camera_angle_x": 0.5, "frames": [
        {"file_path": "a", "transform_matrix": eye}, {"file_path": "./b.png", "transform_matrix": eye}]}))
    imgs = np.zeros((2, 8, 8, 4), np.uint8)
    cams = np.zeros((2, 4, 4), np.float32)
    intr = np.zeros(4, np.float32)
    rc = lib.nerf_b200_blender_load(str(tmp_path / "mixed.json").encode(), 0, 2, imgs.ctypes.data, imgs.nbytes,
                                    cams.ctypes.data, intr.ctypes.data)
    assert rc == abi.NERF_STATUS_INVALID_USAGE
    assert lib.nerf_b200_blender_load(str(tmp_path / "mixed.json").encode(), 0, 2, imgs.ctypes.data, 100,
                                      cams.ctypes.data, intr.ctypes.data) == abi.NERF_STATUS_INVALID_USAGE
