"""Extracts tests/golden/quant_fixture_pins.json from the reference's published-checkpoint fixtures.

The reference keeps, for every checkpoint it reads (Tests/SiliconedTests/Fixtures/quant/<name>/), the
checkpoint's published safetensors header (header.json) and a manifest of what it verified on 256
sampled rows (manifest.json): for torchao / SDNQ int8 and fp8, whether the publisher's own weight equals
q * s in fp32 (``vs_q_times_s_fp32``); for ComfyUI's convrot int8, the channel errors of the publisher's
fp32 dequantization and of the rounded exact value against fp64.  These are the only reference-held data
on this path (the sampled tensors themselves are not in the tree).  This script keeps, per checkpoint:

* every 8-bit linear weight of the header (I8 / F8_E4M3, two dimensions), reduced to its layout: kind,
  published [N, K], scale type and shape, convrot group (from the manifest's ``comfy_quant`` records),
  with the number of tensors of that layout;
* the manifest's recorded comparisons for the sampled tensors;
* for the GGUF checkpoints only their tensor types (packed blocks, not this library's products).

Run it where the reference tree exists:  python tests/golden/make_fixture_pins.py [FIXTURES_DIR]
"""
from __future__ import annotations

import json
import os
import sys
from collections import Counter

HERE = os.path.dirname(os.path.abspath(__file__))
DEFAULT = "/root/reference/Tests/SiliconedTests/Fixtures/quant"
KINDS = {"I8": "int8", "F8_E4M3": "float8_e4m3"}
SCALES = {"F32": "float32", "BF16": "bfloat16", "F16": "float16"}


def scale_of(header: dict, base: str):
    for cand in (base + "._weight_scale", base + ".weight_scale", base + ".scale"):
        if cand in header:
            return cand, header[cand]
    return None, None


def group_of(manifest: dict, base: str):
    text = (manifest.get("comfy_quant") or {}).get(base + ".comfy_quant")
    if not text:
        return None
    q = json.loads(text)
    return int(q.get("convrot_groupsize", 0)) if q.get("convrot") else None


def checkpoint(folder: str) -> dict | None:
    mpath, hpath = os.path.join(folder, "manifest.json"), os.path.join(folder, "header.json")
    if not (os.path.exists(mpath) and os.path.exists(hpath)):
        return None
    manifest = json.load(open(mpath))
    raw = json.load(open(hpath))
    if manifest.get("format") == "gguf" or "tensors" in raw and "alignment" in raw:
        return {"repo": manifest.get("repo"), "file": manifest.get("file"), "format": "gguf",
                "gguf_types": manifest.get("types")}
    header = {k: v for k, v in raw.items() if k != "__metadata__"}
    fmt = manifest.get("format") or ("torchao" if any(k.endswith("._weight_qdata") for k in header) else "sdnq")
    out = {"repo": manifest.get("repo"), "revision": manifest.get("revision"), "file": manifest.get("file"),
           "format": fmt}
    layouts = Counter()
    for name, t in header.items():
        if t["dtype"] not in KINDS or len(t["shape"]) != 2 or name.endswith("_zero_point"):
            continue  # (torchao's zero points are I8 [N, 1] and all zero; the manifests record it)
        base = name
        for suffix in ("._weight_qdata", ".weight"):
            if name.endswith(suffix):
                base = name[: -len(suffix)]
                break
        sname, s = scale_of(header, base)
        layouts[(KINDS[t["dtype"]], t["shape"][0], t["shape"][1], SCALES.get(s["dtype"]) if s else None,
                 tuple(s["shape"]) if s else None, group_of(manifest, base))] += 1
    out["linears"] = [[k, n, kk, sd, list(ss) if ss is not None else None, g, c]
                      for (k, n, kk, sd, ss, g), c in sorted(layouts.items(), key=lambda e: str(e[0]))]
    comps = {}
    for name, c in (manifest.get("comparisons") or {}).items():
        rec = {"kind": c.get("kind")}
        if "vs_q_times_s_fp32" in c:
            rec["q_times_s_different"] = c["vs_q_times_s_fp32"]["different"]
        if "group" in c:
            rec["group"] = c["group"]
        for key in ("comfy_fp32_vs_exact_fp64", "rounded_exact_vs_exact_fp64"):
            if key in c and "channel_error_worst" in c[key]:
                rec[key + "_worst"] = c[key]["channel_error_worst"]
        comps[name] = rec
    out["comparisons"] = comps
    return out


def main() -> None:
    root = sys.argv[1] if len(sys.argv) > 1 else DEFAULT
    pins = {}
    for name in sorted(os.listdir(root)):
        rec = checkpoint(os.path.join(root, name))
        if rec is not None:
            pins[name] = rec
    with open(os.path.join(HERE, "quant_fixture_pins.json"), "w") as f:
        json.dump({"source": "Tests/SiliconedTests/Fixtures/quant/*/{header,manifest}.json", "checkpoints": pins}, f,
                  indent=0, separators=(",", ":"))
        f.write("\n")


if __name__ == "__main__":
    main()
