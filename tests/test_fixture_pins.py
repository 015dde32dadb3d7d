"""The reference's published checkpoints against this library (CPU).

tests/golden/quant_fixture_pins.json is extracted by make_fixture_pins.py from the reference's own
fixtures (Tests/SiliconedTests/Fixtures/quant/<checkpoint>/header.json and manifest.json): every 8-bit
linear weight of each published checkpoint the reference reads (torchao int8 and fp8, SDNQ int8,
ComfyUI convrot int8, DiT and text encoders), reduced to its layout, and what the reference recorded
about the publishers' dequantization on sampled rows.  The tests check that every one of these layouts is
a weight this library takes as published (shapes, scale types and shapes, convrot groups), that each
layout goes through the forge, the map writer and the map reader with the reference's stored layout
(values [K, N] byte for byte, the scale on the next 16-byte boundary in its published type, the
rotation recorded), and that the oracle's dequantization of it is the value the manifests pin: q * s in
fp32 exactly (torchao / SDNQ: ``vs_q_times_s_fp32.different == 0``), and for convrot the exact value of
(H q) s / sqrt(G) rounded once (the manifests' ``rounded_exact`` form, within 2^-24 of fp64 per value).
"""
import json
import os

import numpy as np
import pytest

import oracle
from siliconed_b200 import artifact, configs

HERE = os.path.dirname(os.path.abspath(__file__))
PINS = json.load(open(os.path.join(HERE, "golden", "quant_fixture_pins.json")))["checkpoints"]
KIND = {"int8": oracle.INT8, "float8_e4m3": oracle.E4M3}
SCALE = {"float32": oracle.SCALE_F32, "bfloat16": oracle.SCALE_BF16, "float16": oracle.SCALE_F16}


def linears():
    for name, ck in PINS.items():
        for kind, n, k, sdt, sshape, group, count in ck.get("linears", []):
            yield name, kind, n, k, sdt, sshape, group, count


def test_the_pins_cover_the_reference_checkpoints():
    formats = {ck["format"] for ck in PINS.values()}
    assert {"torchao", "sdnq", "convrot", "encoder", "gguf"} <= formats, formats
    kinds = {(kind, sdt, group is not None) for _, kind, _, _, sdt, _, group, _ in linears()}
    assert kinds == {("int8", "float32", False), ("float8_e4m3", "float32", False), ("int8", "bfloat16", False),
                     ("int8", "float32", True)}, kinds
    assert sum(c for *_, c in linears()) > 2500


def test_every_published_8bit_linear_is_a_weight_this_library_takes():
    """The checks sc_weight_create and sc_weight_set_rotation make, on every published linear: K a multiple of
    8 (16-byte activation rows), one scale per output row ([N, 1]) or one for the tensor, in fp32 / bf16 /
    fp16, and a convrot group that is a power of 4 up to 256 dividing K, on int8 only."""
    for ck, kind, n, k, sdt, sshape, group, count in linears():
        where = (ck, kind, n, k)
        assert kind in KIND, where
        assert k % 8 == 0 and n > 0, where
        assert sdt in SCALE, where
        assert sshape in ([n, 1], [n], [], [1]), where
        if group is not None:
            assert kind == "int8" and artifact.is_rotation_group(group) and k % group == 0, where


def test_the_manifests_pin_q_times_s():
    """Every sampled torchao / SDNQ tensor: the publisher's own weight equals q * s in fp32, value for value
    (the recorded statement this library's exact dequantization rests on)."""
    seen = 0
    for ck in PINS.values():
        for name, c in ck.get("comparisons", {}).items():
            if "q_times_s_different" in c:
                assert c["q_times_s_different"] == 0, name
                seen += 1
    assert seen >= 10


def layouts():
    out = {}
    for ck, kind, n, k, sdt, sshape, group, count in linears():
        out.setdefault((kind, k, sdt, group), (ck, n))
    return sorted(out.items(), key=str)


def synthetic(kind, n, k, sdt, seed):
    g = np.random.default_rng(seed)
    if kind == "int8":
        q = g.integers(-127, 128, (n, k), dtype=np.int16).astype(np.int8).view(np.uint8)
        s32 = (np.abs(g.standard_normal(n)) * 0.02 / 127 + 1e-4).astype(np.float32)
    else:
        q = configs.to_e4m3_codes(g.standard_normal((n, k), dtype=np.float32) * 8)
        s32 = (np.abs(g.standard_normal(n)) * 0.02 / 448 + 1e-4).astype(np.float32)
    if sdt == "bfloat16":
        s = configs.to_bf16_bits(s32)
        sf = (s.astype(np.uint32) << 16).view(np.float32)
    elif sdt == "float16":
        s = s32.astype(np.float16)
        sf = s.astype(np.float32)
    else:
        s, sf = s32, s32
    return q, s.reshape(n, 1), sf


@pytest.mark.parametrize("layout", [l for l, _ in layouts()], ids=lambda l: f"{l[0]}-K{l[1]}-{l[2]}-G{l[3]}")
def test_published_layout_through_forge_map_and_oracle(layout, tmp_path):
    kind, k, sdt, group = layout
    n = 40  # rows of the published [N, K]: a slice (the real N only scales the same layout)
    q, s, sf = synthetic(kind, n, k, sdt, seed=k + n)
    name = "blocks.0.linear.weight"
    mt = artifact.forge_linear(name, q, s, kind, sdt, rotation=group)
    path = str(tmp_path / "one.silicon")
    artifact.write_map(path, [mt])
    with artifact.Artifact(path) as a:
        t = a.tensor(name)
        assert t.dtype == kind and t.shape == (k, n)
        assert t.scale is not None and t.scale.dtype == sdt and t.scale.shape == (n,)
        assert t.scale.offset == (k * n + 15) // 16 * 16, "the scale on the next 16-byte boundary after the values"
        assert (t.rotation.group if t.rotation else None) == group
        values = np.array(a.values(name))
        assert np.array_equal(values, q.T), "the published bytes, transposed"
        st, sv = a.scale_values(name)
        assert np.array_equal(np.asarray(sv).reshape(-1).view(np.uint8), s.reshape(-1).view(np.uint8))
    if group is None:
        got = oracle.dequantize(values, KIND[kind], s.reshape(-1), SCALE[sdt], oracle.LAYOUT_COLUMNS, n)
        if kind == "int8":
            qf = q.view(np.int8).T.astype(np.float32)
        else:
            qf = oracle.e4m3_table()[q.T.astype(np.int64)]
        want = (qf * sf[None, :]).astype(np.float32)   # one IEEE fp32 multiply per value
        assert np.array_equal(got.view(np.uint32), want.reshape(-1).view(np.uint32))
    else:
        got = oracle.dequantize_rotated(values.view(np.int8), group, sf).astype(np.float64)
        # the regular Hadamard of the convrot format: Kronecker powers of H4 (DequantizeTests.swift:159-172)
        h4 = np.array([[1, 1, 1, -1], [1, 1, -1, 1], [1, -1, 1, 1], [-1, 1, 1, 1]], np.float64)
        h = h4
        while h.shape[0] < group:
            h = np.kron(h, h4)
        qk = values.view(np.int8).astype(np.float64).reshape(k // group, group, n)
        exact = (np.einsum("ij,bjn->bin", h, qk).reshape(k, n)) * (sf.astype(np.float64)[None, :] / np.sqrt(group))
        assert np.all(np.abs(got - exact) <= 2.0 ** -24 * np.abs(exact)), "the exact value, rounded once"
