"""The map file (``SILICON``) reader and writer, on the CPU.

Restates the reference's map tests: RobustnessTests.swift:20-126 (hand-written maps with 16-byte pages:
a valid one reads; an aberrant header length, a page of zero or less, negative offsets and sizes, and
overflowing shapes are refused as a damaged map; headerLength and elementCount at their bounds; refused
opens leak no descriptor) and QuantizedMapTests.swift:149-216 (a published 8-bit linear forged to the
map: the codes transposed byte for byte, the scales kept in their type at offset 48 after 36 values),
plus the scale and rotation checks of Artifact.swift:378-418.
"""
import json
import os

import numpy as np
import pytest

from siliconed_b200 import artifact, configs
from siliconed_b200.artifact import Artifact, MapError, MapTensor, element_count, header_length

INT_MAX = (1 << 63) - 1


def hand_map(tmp_path, header: dict, data=(1.0, 2.0, 3.0, 4.0), length: int | None = None, data_offset: int = 256,
             raw_data: bytes | None = None) -> str:
    """``SILICON`` v3, the header's length (or ``length``), the JSON, the data at ``data_offset``."""
    text = json.dumps(header).encode()
    body = b"SILICON" + bytes([3]) + (len(text) if length is None else length).to_bytes(8, "little") + text
    assert len(body) <= data_offset, "header longer than the test's layout"
    body += bytes(data_offset - len(body))
    body += raw_data if raw_data is not None else np.asarray(data, np.float32).tobytes()
    path = tmp_path / f"m-{abs(hash((text, length, data_offset, body[-8:])))}.silicon"
    path.write_bytes(body)
    return str(path)


def header(page=16, offset=256, nbytes=16, shape=(4,)) -> dict:
    return {"page": page, "order": ["w"],
            "tensors": {"w": {"offset": offset, "bytes": nbytes, "shape": list(shape), "dtype": "float32"}}}


def assert_corrupt(path: str) -> MapError:
    with pytest.raises(MapError) as e:
        Artifact(path)
    assert e.value.path == path and e.value.kind != "cannot_open"
    return e.value


def test_a_valid_hand_written_map_reads(tmp_path):
    with Artifact(hand_map(tmp_path, header())) as m:
        assert m.order == ["w"] and m.page == 16
        assert m.array("w").tolist() == [1, 2, 3, 4]


def test_an_aberrant_header_length_is_refused(tmp_path):
    for length in (2 ** 64 - 1, INT_MAX, 1 << 40, 100_000):
        path = hand_map(tmp_path, header(), length=length)
        assert_corrupt(path)
        with pytest.raises(MapError):
            Artifact.read_header(path)
    assert header_length(2 ** 64 - 1, 1000) is None
    assert header_length(985, 1000) is None
    assert header_length(984, 1000) == 984


def test_a_page_of_zero_or_less_is_refused(tmp_path):
    assert_corrupt(hand_map(tmp_path, header(page=0)))
    assert_corrupt(hand_map(tmp_path, header(page=-16)))


def test_negative_offsets_and_sizes_are_refused(tmp_path):
    assert_corrupt(hand_map(tmp_path, header(offset=-16)))
    assert_corrupt(hand_map(tmp_path, header(offset=-4096)))
    assert_corrupt(hand_map(tmp_path, header(nbytes=-16)))
    assert_corrupt(hand_map(tmp_path, header(offset=INT_MAX // 16 * 16)))  # beyond the file, no overflow


def test_a_shape_whose_count_overflows_is_refused(tmp_path):
    assert_corrupt(hand_map(tmp_path, header(shape=(INT_MAX, 4))))
    assert_corrupt(hand_map(tmp_path, header(shape=(-1, -4))))
    assert element_count([INT_MAX, 2]) is None
    assert element_count([3, -1]) is None
    assert element_count([]) == 1
    assert element_count([3, 0]) == 0


def test_other_damage_is_named(tmp_path):
    e = assert_corrupt(hand_map(tmp_path, header(offset=264)))
    assert e.kind == "unaligned"
    assert assert_corrupt(hand_map(tmp_path, header(nbytes=12))).kind == "bad_header"  # bytes disagree with shape
    h = header()
    h["order"] = ["w", "x"]
    assert assert_corrupt(hand_map(tmp_path, h)).kind == "bad_header"
    h = header()
    h["tensors"]["w"]["dtype"] = "float64"
    assert assert_corrupt(hand_map(tmp_path, h)).kind == "bad_header"
    p = tmp_path / "short.silicon"
    p.write_bytes(b"SILICON\x03")
    assert assert_corrupt(str(p)).kind == "truncated"
    p = tmp_path / "magic.silicon"
    p.write_bytes(b"SILICON\x01" + bytes(40))
    assert assert_corrupt(str(p)).kind == "bad_magic"
    with pytest.raises(MapError) as e:
        Artifact(str(tmp_path / "absent.silicon"))
    assert e.value.kind == "cannot_open"


def test_a_refused_map_leaks_no_descriptor(tmp_path):
    bad = hand_map(tmp_path, header(page=0))
    before = len(os.listdir("/proc/self/fd"))
    for _ in range(3000):
        with pytest.raises(MapError) as e:
            Artifact(bad)
        assert e.value.kind == "bad_header" and e.value.path == bad
    assert len(os.listdir("/proc/self/fd")) == before
    Artifact(hand_map(tmp_path, header())).close()


def quantized_entry(offset=256, nbytes=60, shape=(6, 6), dtype="int8", scale=None, rotation=None) -> dict:
    e = {"offset": offset, "bytes": nbytes, "shape": list(shape), "dtype": dtype,
         "scale": scale if scale is not None else {"offset": 48, "dtype": "float16", "shape": [shape[1]]}}
    if rotation is not None:
        e["rotation"] = rotation
    return e


def test_scale_entries_are_checked_against_their_tensor(tmp_path):
    def open_with(entry):
        return Artifact(hand_map(tmp_path, {"page": 16, "tensors": {"w": entry}}, raw_data=bytes(entry["bytes"])))

    m = open_with(quantized_entry())  # 36 values, 12 bytes of padding, 6 fp16 scales at 48: 60 bytes
    t = m.tensor("w")
    assert (t.scale.offset, t.scale.dtype, t.scale.shape, t.scale.layout) == (48, "float16", (6,), "columns")
    m.close()
    bad_scales = [
        {"offset": 40, "dtype": "float16", "shape": [6]},            # not a multiple of 16
        {"offset": 32, "dtype": "float16", "shape": [6]},            # inside the values
        {"offset": 48, "dtype": "int8", "shape": [6]},               # not a scale type
        {"offset": 48, "dtype": "float16", "shape": [5]},            # not one per column
        {"offset": 48, "dtype": "float16", "shape": [6], "block": 2},
        {"offset": 48, "dtype": "float16", "shape": [2, 6], "block": 2},   # 2 blocks of 2 rows != 6 rows
        {"offset": 48, "dtype": "float16", "shape": [1, 1, 6]},
    ]
    for s in bad_scales:
        with pytest.raises(MapError) as e:
            open_with(quantized_entry(scale=s))
        assert e.value.kind == "bad_header", s
    m = open_with(quantized_entry(nbytes=84, scale={"offset": 48, "dtype": "float16", "shape": [3, 6], "block": 2}))
    assert m.tensor("w").scale.layout == "blocks"
    m.close()
    t = open_with(quantized_entry(nbytes=52, scale={"offset": 48, "dtype": "float32", "shape": []})).tensor("w")
    assert t.scale.layout == "tensor"
    with pytest.raises(MapError):  # a scale on a 16-bit tensor
        open_with({"offset": 256, "bytes": 8, "shape": [4], "dtype": "bfloat16",
                   "scale": {"offset": 0, "dtype": "float32", "shape": []}})


def test_rotations_are_checked(tmp_path):
    def open_with(entry):
        data = bytes(entry["bytes"])
        return Artifact(hand_map(tmp_path, {"page": 16, "tensors": {"w": entry}}, raw_data=data))

    k, n = 256, 4
    ok = quantized_entry(nbytes=k * n + 16, shape=(k, n), scale={"offset": k * n, "dtype": "float32", "shape": [n]},
                         rotation={"kind": "convrot", "group": 256})
    assert open_with(ok).tensor("w").rotation == artifact.Rotation("convrot", 256)
    for rotation in ({"kind": "hadamard", "group": 256}, {"kind": "convrot", "group": 128},
                     {"kind": "convrot", "group": 1024}, {"kind": "convrot"}):
        with pytest.raises(MapError) as e:
            open_with(dict(ok, rotation=rotation))
        assert e.value.kind == "bad_header"
    with pytest.raises(MapError):  # convrot is int8 only
        open_with(dict(ok, dtype="float8_e4m3"))
    with pytest.raises(MapError):  # K not a multiple of the group
        open_with(quantized_entry(nbytes=320 * n + 16, shape=(320, n),
                                  scale={"offset": 320 * n, "dtype": "float32", "shape": [n]},
                                  rotation={"kind": "convrot", "group": 256}))


def test_a_published_linear_forges_to_the_maps_layout(tmp_path):
    """QuantizedMapTests.swift:149-216: N = K = 6, so 36 values, 12 bytes of padding, then the scales."""
    rng = np.random.default_rng(0)
    n, k = 6, 6
    cases = [("int8", "bfloat16", (n, 1)), ("int8", "float32", (n, 1)), ("float8_e4m3", "float32", ()),
             ("int8", "float16", ())]
    tensors, published = [], {}
    for i, (dtype, st, sshape) in enumerate(cases):
        q = rng.integers(0, 256, (n, k), dtype=np.uint16).astype(np.uint8)
        if st == "bfloat16":
            s = rng.integers(0x3C00, 0x3D00, sshape, dtype=np.uint16)
        else:
            s = (np.abs(rng.standard_normal(sshape)) * 1e-2 + 1e-3).astype(np.float32 if st == "float32" else np.float16)
        name = f"layers.0.l{i}.weight"
        tensors.append(artifact.forge_linear(name, q, s, dtype, st))
        published[name] = (q, s, dtype, st)
    bias = np.arange(n, dtype=np.float32)
    tensors.append(MapTensor("layers.0.l0.bias", "float32", (n,), bias))
    path = str(tmp_path / "forged.silicon")
    size = artifact.write_map(path, tensors, header={"kind": "test"})
    assert size == os.path.getsize(path)
    with Artifact(path) as m:
        assert m.linear_weights_transposed and m.header["kind"] == "test"
        assert m.order == [t.name for t in tensors]
        assert m.quantized_names() == [t.name for t in tensors[:4]]
        data_start = m.header["data_start"]
        assert data_start % artifact.PAGE == 0
        for name, (q, s, dtype, st) in published.items():
            t = m.tensor(name)
            assert t.offset % artifact.PAGE == 0 and t.offset >= data_start
            assert (t.dtype, t.shape) == (dtype, (k, n))
            assert t.scale.offset == 48, "36 values, then 12 bytes of padding, then the scales"
            assert t.scale.dtype == st and t.scale.shape == ((n,) if s.size == n else ())
            assert np.array_equal(m.values(name), q.T), "the published bytes, transposed"
            got_type, got = m.scale_values(name)
            assert got_type == st and got.tobytes() == np.ascontiguousarray(s).tobytes(), "the scales, in their type"
            assert not m.raw(name)[k * n:48].any()
        assert m.array("layers.0.l0.bias").tolist() == bias.tolist()
        assert Artifact.read_header(path) == m.header


def test_sq_and_packed_tensors_are_sized(tmp_path):
    k, n = 256, 3
    sq = MapTensor("sq", "sq4", (k, n), bytes(n * artifact.sq_row_bytes(k, 4)), np.ones(n, np.float32), "float32", (n,),
                   rotation=256)
    q8 = MapTensor("q8", "q4_0", (64, 2), bytes(64 * 2 // 32 * 18))
    path = str(tmp_path / "packed.silicon")
    artifact.write_map(path, [sq, q8])
    with Artifact(path) as m:
        assert m.tensor("sq").bytes == (n * (128 + 16) + 15) // 16 * 16 + 4 * n
        assert m.tensor("q8").bytes == 72
        assert m.quantized_names() == []


def test_a_tensor_larger_than_its_destination_is_refused_before_writing(tmp_path):
    """RobustnessTests.swift:116-131: refused (does_not_fit, a damaged map) and not a value lands."""
    path = hand_map(tmp_path, header())
    with Artifact(path) as m:
        out = np.full(3, -7, np.float32)
        with pytest.raises(MapError) as e:
            m.materialize("w", out)
        assert e.value.kind == "does_not_fit" and e.value.path == path
        assert out.tolist() == [-7, -7, -7], "nothing written"
        out = np.zeros(5, np.float32)
        assert m.materialize("w", out) == 4
        assert out.tolist() == [1, 2, 3, 4, 0]


def test_sixteen_bit_tensors_materialize_exactly(tmp_path):
    bits = np.array([0x3F80, 0xBF81, 0x7F80, 0x0001], np.uint16)   # 1, -1.0078125, +inf, the smallest subnormal
    halves = np.array([1.0, -2.5, 65504.0, 2.0 ** -24], np.float16)
    path = str(tmp_path / "sixteen.silicon")
    artifact.write_map(path, [MapTensor("b", "bfloat16", (4,), bits), MapTensor("h", "float16", (2, 2), halves)])
    with Artifact(path) as m:
        out = np.empty(4, np.float32)
        m.materialize("b", out)
        assert out.view(np.uint32).tolist() == (bits.astype(np.uint32) << 16).tolist()
        m.materialize("h", out)
        assert out.tolist() == halves.astype(np.float32).tolist()
        with pytest.raises(Exception):
            m.materialize("h", np.empty(4, np.float64))   # the destination is fp32


def test_the_forge_refuses_what_the_reference_refuses():
    """QuantizedMapTests.swift:485-503, 620-641: int8 without a scale, a scale neither per tensor nor per
    row, subnormal products (1e-39 for int8; 2^-120 fine for int8 but not for e4m3); an fp8 weight
    without a scale is a plain cast."""
    q = np.arange(8, dtype=np.uint8).reshape(2, 4)
    with pytest.raises(artifact.ForgeRefusal, match="without a scale"):
        artifact.forge_linear("a.weight", q, None, "int8", None)
    with pytest.raises(artifact.ForgeRefusal, match="only one per tensor or one per row"):
        artifact.forge_linear("a.weight", q, np.zeros((2, 2), np.float32), "int8", "float32")
    with pytest.raises(artifact.ForgeRefusal, match="only one per tensor or one per row"):
        artifact.forge_linear("a.weight", np.zeros((4, 4), np.uint8), np.ones((1, 4), np.float32), "int8", "float32")
    with pytest.raises(artifact.ForgeRefusal, match="subnormal"):
        artifact.forge_linear("a.weight", q, np.array(1e-39, np.float32), "int8", "float32")
    small = np.array(2.0 ** -120, np.float32)
    assert artifact.forge_linear("a.weight", q, small, "int8", "float32").scale_shape == ()
    with pytest.raises(artifact.ForgeRefusal, match="subnormal"):
        artifact.forge_linear("a.weight", q, small, "float8_e4m3", "float32")
    # rotated: the smallest product is |s| / sqrt(G)
    q256 = np.zeros((2, 256), np.uint8)
    with pytest.raises(artifact.ForgeRefusal, match="subnormal"):
        artifact.forge_linear("a.weight", q256, np.array(2.0 ** -123, np.float32), "int8", "float32", rotation=256)
    with pytest.raises(artifact.ForgeRefusal, match="rotation"):
        artifact.forge_linear("a.weight", q, np.ones(2, np.float32), "int8", "float32", rotation=256)
    # zero scales are not refused; an fp8 weight without a scale is a plain cast
    assert artifact.forge_linear("a.weight", q, np.zeros(2, np.float32), "int8", "float32").scale_shape == (2,)
    cast = artifact.forge_linear("c.weight", q, None, "float8_e4m3", None)
    assert cast.scale is None and cast.shape == (4, 2) and cast.total_bytes() == 8


def test_a_linear_stored_in_the_arena_layout_round_trips(tmp_path):
    """The re-tiled map (this library's extension, ``"layout": "arena"``): the codes stored as the device
    arena keeps them, [n_pad][k_pad] with int8 biased and the padding the code of zero, computed here
    independently; the reader gives back the published [K, N] codes and the scale as published."""
    rng = np.random.default_rng(5)
    qi = rng.integers(-128, 128, (300, 200), dtype=np.int16).astype(np.int8)         # [N, K]
    si = configs.to_bf16_bits((np.abs(rng.standard_normal((300, 1))) * 1e-3 + 1e-5).astype(np.float32))
    qe = configs.to_e4m3_codes(rng.standard_normal((70, 128), dtype=np.float32) * 8)
    qe[3, 5] = 0x7F                                                                   # a NaN code
    se = np.array([0.5], np.float32)
    ts = [artifact.forge_linear("i.weight", qi, si, "int8", "bfloat16", layout="arena"),
          artifact.forge_linear("e.weight", qe, se, "float8_e4m3", "float32", layout="arena"),
          artifact.forge_linear("r.weight", qi[:, :192], si, "int8", "bfloat16", rotation=64, layout="arena")]
    path = str(tmp_path / "arena.silicon")
    artifact.write_map(path, ts)
    with artifact.Artifact(path) as a:
        t = a.tensor("i.weight")
        assert t.layout == "arena" and t.shape == (200, 300) and not t.nan_codes
        want = np.full((512, 256), 0x80, np.uint8)
        want[:300, :200] = qi.view(np.uint8) ^ 0x80
        assert np.array_equal(a.stored("i.weight"), want)
        assert t.scale.offset == 512 * 256 and t.bytes == 512 * 256 + 600
        assert np.array_equal(a.values("i.weight"), qi.view(np.uint8).T)
        assert np.array_equal(a.scale_values("i.weight")[1].reshape(-1), si.reshape(-1))
        e = a.tensor("e.weight")
        assert e.nan_codes and e.scale.shape == ()
        want = np.zeros((256, 128), np.uint8)
        want[:70] = qe
        assert np.array_equal(a.stored("e.weight"), want)
        assert np.array_equal(a.values("e.weight"), qe.T)
        r = a.tensor("r.weight")
        assert r.rotation.group == 64 and r.layout == "arena"
        assert np.array_equal(a.values("r.weight"), qi[:, :192].view(np.uint8).T)


def test_the_arena_layout_is_checked(tmp_path):
    rng = np.random.default_rng(6)
    q = rng.integers(-128, 128, (40, 64), dtype=np.int16).astype(np.int8)
    t = artifact.forge_linear("w", q, np.full(40, 1e-3, np.float32), "int8", "float32", layout="arena")
    good = str(tmp_path / "good.silicon")
    artifact.write_map(good, [t])
    raw = bytearray(open(good, "rb").read())
    n = int.from_bytes(raw[8:16], "little")
    header = json.loads(raw[16:16 + n])
    for change in ({"layout": "tiled"}, {"dtype": "bfloat16"}, {"bytes": header["tensors"]["w"]["bytes"] - 16},
                   {"nan_codes": 1}):
        h = json.loads(json.dumps(header))
        h["tensors"]["w"].update(change)
        text = json.dumps(h).encode()
        bad = str(tmp_path / "bad.silicon")
        with open(bad, "wb") as f:
            f.write(raw[:8] + len(text).to_bytes(8, "little") + text + bytes(header["data_start"] - 16 - len(text))
                    + raw[header["data_start"]:])
        with pytest.raises(artifact.MapError):
            artifact.Artifact(bad)
    with pytest.raises(artifact.ForgeRefusal):
        artifact.forge_linear("w", q, np.full(40, 1e-3, np.float32), "int8", "float32", layout="tiled")
