"""8-bit linears read from a map file (``SILICON`` v3) into the library, on a B200.

A map forged from published weights (int8 with a bf16 scale per row, fp8 with one fp32 scale, fp8
published without a scale, int8 convrot with an fp32 scale per row) is opened with the reader of
Artifact.swift:263-418, and every 8-bit tensor is registered in place.  Bars: the export
(sc_dequantize) bit-exact against the oracle's Widen.dequantize / dequantizeRotated of the published
bytes; the products through WeightProducts.linear bit-identical to the same weight registered from
the arrays directly (the map only supplies the bytes), the bias taken from the map.
"""
import numpy as np
import pytest

import oracle
from siliconed_b200 import abi, artifact, configs

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():  # collected on CPU boxes, skipped there
    pytest.skip("needs a CUDA device", allow_module_level=True)

from siliconed_b200.products import Context, QuantizedWeight, WeightProducts  # noqa: E402


@pytest.fixture(scope="module")
def ctx():
    c = Context(0)
    yield c
    c.close()


def canonical(a: np.ndarray) -> np.ndarray:
    b = a.view(np.uint32).copy()
    b[np.isnan(a)] = 0x7FC00000
    return b


def bf16_dev(bits: np.ndarray):
    return torch.from_numpy(np.ascontiguousarray(bits.astype(np.uint16)).view(np.int16)).cuda().view(torch.bfloat16)


def test_a_forged_map_registers_in_place(ctx, tmp_path):
    rng = np.random.default_rng(11)
    pub = {}
    # int8 [N = 300, K = 512] with a bf16 scale per row, and its bf16 bias
    qa = rng.integers(-128, 128, (300, 512), dtype=np.int16).astype(np.int8)
    sa = configs.to_bf16_bits((np.abs(rng.standard_normal((300, 1))) * 0.02 / 127 + 1e-5).astype(np.float32))
    ba = configs.to_bf16_bits(rng.standard_normal(300, dtype=np.float32) * 0.01)
    pub["a.weight"] = artifact.forge_linear("a.weight", qa, sa, "int8", "bfloat16")
    # e4m3 [N = 200, K = 128] with one fp32 scale
    qb = configs.to_e4m3_codes(rng.standard_normal((200, 128), dtype=np.float32) * 8)
    sb = np.array([0.0125], np.float32)
    pub["b.weight"] = artifact.forge_linear("b.weight", qb, sb, "float8_e4m3", "float32")
    # e4m3 published without a scale: a plain cast, w = f8 (every code, NaN ones included)
    qc = np.arange(256 * 64, dtype=np.uint32).astype(np.uint8).reshape(64, 256)
    pub["c.weight"] = artifact.MapTensor("c.weight", "float8_e4m3", (64, 256), qc)
    # int8 convrot, group 256, [K = 512, N = 264], fp32 scale per column
    qd = rng.integers(-128, 128, (264, 512), dtype=np.int16).astype(np.int8)
    sd = (np.abs(rng.standard_normal(264)) * 0.02 / 127 + 1e-5).astype(np.float32)
    pub["d.weight"] = artifact.forge_linear("d.weight", qd, sd, "int8", "float32", rotation=256)
    tensors = list(pub.values()) + [artifact.MapTensor("a.bias", "bfloat16", (300,), ba)]
    path = str(tmp_path / "forged.silicon")
    artifact.write_map(path, tensors)

    m = artifact.Artifact(path)
    products = WeightProducts(ctx)
    assert products.register_map(m) == ["a.weight", "b.weight", "c.weight", "d.weight"]
    assert "a.weight" in products.biases and "b.weight" not in products.biases

    # the exports, bit-exact against the oracle on the published bytes
    want = {
        "a.weight": oracle.dequantize(qa.T.copy(), oracle.INT8, sa.reshape(-1), oracle.SCALE_BF16,
                                      oracle.LAYOUT_COLUMNS, 300).reshape(512, 300),
        "b.weight": oracle.dequantize(qb.T.copy(), oracle.E4M3, sb, oracle.SCALE_F32, oracle.LAYOUT_TENSOR)
                    .reshape(128, 200),
        "c.weight": oracle.dequantize(qc, oracle.E4M3, None, oracle.SCALE_F32, oracle.LAYOUT_TENSOR).reshape(64, 256),
        "d.weight": oracle.dequantize_rotated(qd.T.copy(), 256, sd),
    }
    for name, ref in want.items():
        got = products.weights[name].dequantize().cpu().numpy()
        assert np.array_equal(canonical(got), canonical(ref)), name
    assert products.weights["d.weight"].rotation == 256
    # materialize: the same bits into a caller's fp32 buffer, host or device
    for name in ("a.weight", "d.weight"):
        out = np.full(want[name].size + 3, -7, np.float32)
        assert m.materialize(name, out, ctx=ctx) == want[name].size
        assert np.array_equal(canonical(out[:-3]), canonical(want[name].reshape(-1))) and (out[-3:] == -7).all()
    out = torch.empty(want["b.weight"].size, dtype=torch.float32, device="cuda")
    m.materialize("b.weight", out, ctx=ctx)
    assert np.array_equal(canonical(out.cpu().numpy()), canonical(want["b.weight"].reshape(-1)))

    # the products: the same bits as the weight registered from the arrays
    direct = {
        "a.weight": QuantizedWeight(ctx, qa.view(np.uint8), abi.WEIGHT_INT8,
                                    torch.from_numpy(sa.reshape(-1).view(np.int16).copy()).view(torch.bfloat16),
                                    published_nk=True),
        "b.weight": QuantizedWeight(ctx, qb, abi.WEIGHT_E4M3, sb, published_nk=True),
        "d.weight": QuantizedWeight(ctx, qd.view(np.uint8), abi.WEIGHT_INT8, sd, published_nk=True, rotation=256),
    }
    for name, w in direct.items():
        k, n = w.k, w.n
        for rows in (3, 40, 700):
            x = bf16_dev(configs.to_bf16_bits(rng.standard_normal((rows, k), dtype=np.float32)))
            c = torch.empty((rows, n), dtype=torch.bfloat16, device="cuda")
            products.linear(name, x, c, rows, k, n)
            need = w.workspace_bytes(rows)  # as WeightProducts.linear: a workspace only when the route needs one
            ws = torch.empty(need, dtype=torch.uint8, device="cuda") if need else None
            ref = w.linear(x, bias=products.biases.get(name), workspace=ws)
            ctx.poll_errors()
            assert torch.equal(c.view(torch.int16), ref.view(torch.int16)), f"{name}, {rows} rows"
        w.close()
    products.close()
    m.close()


def test_a_map_stored_in_the_arena_layout_registers_with_one_copy(ctx, tmp_path):
    """The same published weights forged in the map's [K, N] layout and in the arena layout (the codes
    re-tiled at forge time, registration one copy, no re-tiling kernel): identical exports and identical
    product bits, for int8 with bf16 row scales, e4m3 holding NaN codes, and int8 convrot; a stored
    padding byte that is not the code of zero is refused at registration."""
    rng = np.random.default_rng(21)
    q1 = rng.integers(-128, 128, (600, 1024), dtype=np.int16).astype(np.int8)
    s1 = configs.to_bf16_bits((np.abs(rng.standard_normal((600, 1))) * 0.02 / 127 + 1e-5).astype(np.float32))
    q2 = configs.to_e4m3_codes(rng.standard_normal((300, 512), dtype=np.float32) * 8)
    q2[rng.integers(0, 300, 5), rng.integers(0, 512, 5)] = 0x7F
    s2 = (np.abs(rng.standard_normal(300)) * 0.02 / 448 + 1e-5).astype(np.float32)
    q3 = rng.integers(-128, 128, (264, 512), dtype=np.int16).astype(np.int8)
    s3 = (np.abs(rng.standard_normal(264)) * 0.02 / 127 + 1e-5).astype(np.float32)
    specs = [("a.weight", q1, s1, "int8", "bfloat16", None), ("b.weight", q2, s2, "float8_e4m3", "float32", None),
             ("c.weight", q3, s3, "int8", "float32", 256)]
    maps = {}
    for layout in (None, "arena"):
        ts = [artifact.forge_linear(n, q, s, d, sd, rotation=r, layout=layout) for n, q, s, d, sd, r in specs]
        path = str(tmp_path / f"{layout}.silicon")
        artifact.write_map(path, ts)
        maps[layout] = artifact.Artifact(path)
    for name, q, *_ in specs:
        plain, arena = maps[None].register(ctx, name), maps["arena"].register(ctx, name)
        assert canonical(plain.dequantize().cpu().numpy()).tobytes() == canonical(arena.dequantize().cpu().numpy()).tobytes()
        for m in (3, 200, 1600):
            x = bf16_dev(configs.to_bf16_bits(rng.standard_normal((m, plain.k), dtype=np.float32)))
            a, b = plain.linear(x), arena.linear(x)
            torch.cuda.synchronize()
            assert canonical(a.float().cpu().numpy()).tobytes() == canonical(b.float().cpu().numpy()).tobytes(), (name, m)
        plain.close()
        arena.close()
    for m in maps.values():
        m.close()
    # a K padding byte that is not the code of zero: refused before anything is uploaded
    t = artifact.forge_linear("w", q1[:, :1000], s1, "int8", "bfloat16", layout="arena")
    t.data[0, 1010] = 0x81
    bad = str(tmp_path / "bad.silicon")
    artifact.write_map(bad, [t])
    with artifact.Artifact(bad) as a:
        with pytest.raises(abi.SiliconedError) as e:
            a.register(ctx, "w")
        assert e.value.status == abi.INVALID_ARG
