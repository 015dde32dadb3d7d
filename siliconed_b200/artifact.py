"""Siliconed's map file (``SILICON`` v2 / v3): the on-disk source of every 8-bit weight, read and written.

The reader restates the checks of the reference's ``Artifact`` (Sources/Siliconed/Artifact.swift:146-396):

- the prologue is ``SILICON``, a version byte in 2...3, then the JSON header's length as a little-endian
  uint64, bounded by the file before anything is read for it (``headerLength``, :246-249);
- the header is a JSON object with a positive ``page``, a ``tensors`` table and an optional ``order``
  (default: the names sorted) naming the same tensors (:295-374);
- every tensor has an int ``offset`` and ``bytes`` (both >= 0, the offset a multiple of the page, the
  region inside the file), a ``shape`` whose element count does not overflow (``elementCount``,
  :252-261) and a known ``dtype``; its ``bytes`` equal what the dtype, shape and scale require;
- an 8-bit tensor's ``scale`` sits inside the tensor's own region, at a multiple of 16 at or after the
  values, in bf16 / fp16 / fp32, shaped ``[]``, ``[N]`` or ``[K/b, N]`` with ``block`` b (``scale``,
  :378-403);
- a ``rotation`` is ComfyUI's ``convrot`` only, on an int8 ``[K, N]`` with a tensor or column scale, its
  group a power of 4 up to 256 dividing K (``rotation``, :405-418).

Every refusal raises ``MapError`` naming the file, as ``Artifact.Failure.inFile`` does.  An opened map
is memory-mapped read-only; ``register`` hands an 8-bit tensor's values and scale, in place, to
``sc_weight_create`` (which copies them once into the device arena).  Block scales (GGUF Q8_0) and the
packed GGUF / SQ types are parsed and checked but not registered: they are not this library's products.

The writer restates ``MapWriter.write`` (Sources/Siliconed/Forge/Map.swift:156-335): a whole number of
16 KiB pages of prologue, each tensor on a page boundary, an 8-bit tensor's scale on the next 16-byte
boundary after its values; and ``forge_linear`` restates the forge's move of a published ``nn.Linear``
weight ``[N, K]`` with its per-row scale ``[N, 1]`` (or one for the tensor) to the map's ``[K, N]`` with
a scale ``[N]`` (QuantizedMapTests.swift:149-216: the published bytes transposed, the scales as
published, in their own type).

This library extends the map with one tensor key, ``"layout": "arena"`` (``forge_linear(...,
layout="arena")``): an 8-bit linear whose codes are stored as the device arena keeps them, rows of K for
each output, ``[n_pad][k_pad]`` with N padded to 256 and K to 64, int8 biased by 128, every padding byte
the code of zero (``"nan_codes": true`` when an e4m3 tensor holds NaN codes); its scale follows at the next
16-byte boundary as published.  Registering such a tensor is one copy into the arena, with no staging
buffer and no re-tiling kernel (SC_WEIGHT_ARENA_LAYOUT); ``values`` still returns the published
``[K, N]`` codes (a decoded copy) and ``stored`` the bytes as they lie.  Maps without the key are read as
the reference writes them.
"""
from __future__ import annotations

import json
import mmap
import os
from dataclasses import dataclass

import numpy as np

from . import abi
from .abi import SiliconedError

SIGNATURE = b"SILICON"
SUPPORTED_VERSIONS = (2, 3)
WRITE_VERSION = 3
PAGE = 16384
INT_MAX = (1 << 63) - 1

# Bytes per value of the types that have one.
VALUE_SIZES = {"bfloat16": 2, "float16": 2, "float32": 4, "int8": 1, "float8_e4m3": 1}
# ggml's blocks: (values, bytes) (Artifact.DType.packedBlock).
PACKED_BLOCKS = {"q4_0": (32, 18), "q4_1": (32, 20), "q5_0": (32, 22), "q5_1": (32, 24),
                 "q4_k": (256, 144), "q5_k": (256, 176), "q6_k": (256, 210)}
# Siliconed's own 4 and 5 bits: groups of 16 and a rotation of 256 (SQ.swift:34-52).
SQ_BITS = {"sq4": 4, "sq5": 5}
SQ_GROUP, SQ_ROTATION = 16, 256
SCALE_TYPES = ("bfloat16", "float16", "float32")
ARENA_N, ARENA_K = 256, 64  # the library's arena tiles: N padded to 256 rows, K to 64 bytes
DTYPES = tuple(VALUE_SIZES) + tuple(PACKED_BLOCKS) + tuple(SQ_BITS)


class MapError(Exception):
    """A refused map.  ``kind``: cannot_open, bad_magic, truncated, bad_header, unaligned or does_not_fit
    (Artifact.Failure); ``path``: the file, once known."""

    def __init__(self, kind: str, why: str, path: str | None = None):
        self.kind, self.why, self.path = kind, why, path
        super().__init__(f"{path}: {why}" if path else why)

    def in_file(self, path: str) -> "MapError":
        return self if self.path is not None else MapError(self.kind, self.why, path)


def header_length(raw: int, file_size: int) -> int | None:
    """The header's length if the file can hold it after the 16-byte prologue, else None
    (Artifact.headerLength, Artifact.swift:246-249)."""
    if file_size < 16 or raw > file_size - 16:
        return None
    return int(raw)


def element_count(shape) -> int | None:
    """The values of a shape; None for a negative dimension or a count past int64 (elementCount :252-261)."""
    count = 1
    for d in shape:
        if d < 0:
            return None
        count *= d
        if count > INT_MAX:
            return None
    return count


def sq_row_bytes(k: int, bits: int) -> int:
    """Bytes of one output row of an SQ tensor: the codes, then one byte per group (SQ.rowBytes)."""
    return k * bits // 8 + k // SQ_GROUP


def is_rotation_group(g: int) -> bool:
    """A power of 4 from 4 to 256 (Widen.isRotationGroup)."""
    p = 4
    while p < g:
        p *= 4
    return p == g and g <= 256


def _is_int(v) -> bool:
    return isinstance(v, int) and not isinstance(v, bool) and -INT_MAX - 1 <= v <= INT_MAX


def _int_list(v) -> list[int] | None:
    if not isinstance(v, list) or not all(_is_int(d) for d in v):
        return None
    return list(v)


@dataclass(frozen=True)
class Scale:
    """An 8-bit tensor's scale, inside the tensor's region (Artifact.Scale, Artifact.swift:31-57)."""
    offset: int            # from the tensor's start, a multiple of 16
    dtype: str             # bfloat16 / float16 / float32, as published
    shape: tuple[int, ...]  # () for the tensor, (N,) per column, (K/b, N) per block of b rows
    block: int | None = None

    @property
    def count(self) -> int:
        return element_count(self.shape) or 0

    @property
    def layout(self) -> str:
        return ("tensor", "columns", "blocks")[min(len(self.shape), 2)]


@dataclass(frozen=True)
class Rotation:
    """A published rotation of the input (Artifact.Rotation): only ComfyUI's convrot."""
    kind: str
    group: int


@dataclass(frozen=True)
class Tensor:
    """One tensor of the map (Artifact.Tensor, Artifact.swift:15-29)."""
    name: str
    offset: int  # absolute, in the file
    bytes: int
    shape: tuple[int, ...]
    dtype: str
    scale: Scale | None = None
    rotation: Rotation | None = None
    layout: str | None = None   # "arena": the codes stored re-tiled, [n_pad][k_pad] (this library's extension)
    nan_codes: bool = False     # an arena-layout e4m3 tensor holding NaN codes (0x7F / 0xFF)

    @property
    def count(self) -> int:
        return element_count(self.shape) or 0

    @property
    def is_quantized(self) -> bool:
        return self.dtype in ("int8", "float8_e4m3")


def arena_dims(k: int, n: int) -> tuple[int, int]:
    """(n_pad, k_pad) of a [K, N] weight in the library's arena: N rounded up to 256, K to 64."""
    return -(-n // ARENA_N) * ARENA_N, -(-k // ARENA_K) * ARENA_K


def arena_codes(values_nk: np.ndarray, dtype: str) -> np.ndarray:
    """The arena's bytes [n_pad][k_pad] of published codes [N, K]: rows of K contiguous, int8 stored biased
    (q + 128), e4m3 as published, every padding byte the code of zero (0x80 for int8, 0x00 for e4m3)."""
    q = np.ascontiguousarray(values_nk).view(np.uint8)
    n, k = q.shape
    n_pad, k_pad = arena_dims(k, n)
    zero = 0x80 if dtype == "int8" else 0x00
    out = np.full((n_pad, k_pad), zero, np.uint8)
    out[:n, :k] = (q ^ 0x80) if dtype == "int8" else q
    return out


def _scale_entry(raw, name: str, shape: list[int], dtype: str) -> Scale:
    """Artifact.scale (Artifact.swift:378-403): a scale checked against its tensor's shape."""
    if not (dtype in ("int8", "float8_e4m3") or dtype in SQ_BITS) or not isinstance(raw, dict):
        raise MapError("bad_header", f"{name}: malformed scale")
    offset, st, sshape = raw.get("offset"), raw.get("dtype"), _int_list(raw.get("shape"))
    if not _is_int(offset) or st not in SCALE_TYPES or sshape is None:
        raise MapError("bad_header", f"{name}: malformed scale")
    block = raw.get("block")
    if block is not None and not _is_int(block):
        raise MapError("bad_header", f"{name}: malformed scale")
    count = element_count(shape)
    if count is None or element_count(sshape) is None:
        raise MapError("bad_header", f"{name}: a scale {sshape} for {shape}")
    if len(sshape) == 0:
        fits = block is None
    elif len(sshape) == 1:
        fits = len(shape) == 2 and sshape[0] == shape[1] and block is None
    elif len(sshape) == 2:
        fits = (len(shape) == 2 and sshape[1] == shape[1] and (block or 0) > 0
                and element_count([sshape[0], block]) == shape[0])
    else:
        fits = False
    if not fits or offset < (count if dtype not in SQ_BITS else 0) or offset % 16 != 0:
        raise MapError("bad_header", f"{name}: a scale {sshape} (block {block if block is not None else '-'}) "
                                     f"at {offset} does not fit {shape}")
    return Scale(offset, st, tuple(sshape), block)


def _rotation_entry(raw, name: str, shape: list[int], dtype: str, scale: Scale | None) -> Rotation:
    """Artifact.rotation (Artifact.swift:405-418): convrot only, checked against the tensor."""
    if not isinstance(raw, dict) or not isinstance(raw.get("kind"), str) or not _is_int(raw.get("group")):
        raise MapError("bad_header", f"{name}: malformed rotation")
    kind, group = raw["kind"], raw["group"]
    if kind != "convrot":
        raise MapError("bad_header", f'{name}: rotation "{kind}" unknown - refused rather than read without it')
    ok = ((dtype == "int8" or (dtype in SQ_BITS and group == SQ_ROTATION)) and len(shape) == 2
          and scale is not None and scale.block is None and len(scale.shape) <= 1
          and is_rotation_group(group) and shape[0] % group == 0)
    if not ok:
        raise MapError("bad_header", f"{name}: rotation convrot of group {group} on {dtype} {shape} - not read")
    return Rotation(kind, group)


def parse(buf, size: int) -> tuple[dict, int, list[str], dict[str, Tensor]]:
    """(header, page, order, tensors) of a map's bytes; every number bounded before it is used
    (Artifact.parse, Artifact.swift:263-374)."""
    if size < 16:
        raise MapError("truncated", "shorter than a prologue")
    head = bytes(buf[:8])
    if head[:7] != SIGNATURE or head[7] not in SUPPORTED_VERSIONS:
        raise MapError("bad_magic", f"not a Siliconed map (signature {list(head)})")
    raw = int.from_bytes(bytes(buf[8:16]), "little")
    length = header_length(raw, size)
    if length is None:
        raise MapError("truncated", f"header length {raw}")
    try:
        header = json.loads(bytes(buf[16:16 + length]))
    except (ValueError, UnicodeDecodeError):
        header = None
    if not isinstance(header, dict):
        raise MapError("bad_header", "not a JSON object")
    page = header.get("page")
    if not _is_int(page):
        raise MapError("bad_header", "no page size")
    if page <= 0:  # `offset % page` below: zero would divide by zero, a negative page accept anything
        raise MapError("bad_header", f"page size {page}")
    table = header.get("tensors")
    if not isinstance(table, dict) or not all(isinstance(e, dict) for e in table.values()):
        raise MapError("bad_header", "no tensor table")
    order = header.get("order")
    if order is None:
        order = sorted(table)
    elif not isinstance(order, list) or not all(isinstance(n, str) for n in order):
        raise MapError("bad_header", "`order` is not a list of names")
    tensors: dict[str, Tensor] = {}
    for name, entry in table.items():
        offset, nbytes, shape, dtype = entry.get("offset"), entry.get("bytes"), _int_list(entry.get("shape")), \
            entry.get("dtype")
        if not _is_int(offset) or not _is_int(nbytes) or shape is None or dtype not in DTYPES:
            raise MapError("bad_header", f"tensor {name} is incomplete")
        if offset < 0 or nbytes < 0:  # signs first: a negative multiple of the page passes the alignment test
            raise MapError("bad_header", f"{name}: offset {offset}, {nbytes} bytes")
        if offset % page != 0:
            raise MapError("unaligned", f"{name} starts at {offset}, not a multiple of {page} - "
                                        "the mapping would straddle two pages")
        if offset > size or nbytes > size - offset:
            raise MapError("truncated", f"{name} runs past the end")
        count = element_count(shape)
        if count is None:
            raise MapError("bad_header", f"{name}: shape {shape}")
        scale = _scale_entry(entry["scale"], name, shape, dtype) if "scale" in entry else None
        layout = entry.get("layout")
        if layout is not None:
            # this library's extension: an 8-bit linear stored as its arena keeps it (values [n_pad][k_pad])
            if layout != "arena" or dtype not in ("int8", "float8_e4m3") or len(shape) != 2 or \
                    (scale is not None and scale.block is not None) or not isinstance(entry.get("nan_codes", False), bool):
                raise MapError("bad_header", f"{name}: layout {layout!r} on {dtype} {shape}")
            n_pad, k_pad = arena_dims(shape[0], shape[1])
            stored = n_pad * k_pad
            if scale is not None and scale.offset < stored:
                raise MapError("bad_header", f"{name}: a scale at {scale.offset} inside the {stored} arena bytes")
            count = stored if scale is None else count
        if dtype in PACKED_BLOCKS:
            values, per = PACKED_BLOCKS[dtype]
            if len(shape) != 2 or shape[0] % values != 0 or "scale" in entry or "rotation" in entry:
                raise MapError("bad_header", f"{name}: {dtype} on {shape} - only a `[K, N]` whose K is a multiple "
                                             f"of {values}, without a scale or a rotation")
            expected = count // values * per
        elif dtype in SQ_BITS:
            bits = SQ_BITS[dtype]
            if (len(shape) != 2 or shape[0] % SQ_ROTATION != 0 or scale is None or scale.dtype != "float32"
                    or scale.shape != (shape[1],) or scale.offset < shape[1] * sq_row_bytes(shape[0], bits)
                    or "rotation" not in entry):
                raise MapError("bad_header", f"{name}: {dtype} on {shape} - only a `[K, N]` whose K is a multiple "
                                             "of 256, with its fp32 scale per column after its rows and a rotation")
            expected = scale.offset + 4 * shape[1]
        elif scale is not None:
            expected = scale.offset + scale.count * VALUE_SIZES[scale.dtype]
        else:
            expected = count * VALUE_SIZES[dtype]
        if expected > INT_MAX or nbytes != expected:
            raise MapError("bad_header", f"{name}: {nbytes} bytes for {shape} of {dtype}")
        rotation = _rotation_entry(entry["rotation"], name, shape, dtype, scale) if "rotation" in entry else None
        tensors[name] = Tensor(name, offset, nbytes, tuple(shape), dtype, scale, rotation, layout,
                               bool(entry.get("nan_codes", False)))
    if set(order) != set(tensors):
        raise MapError("bad_header", "`order` and `tensors` disagree")
    return header, page, list(order), tensors


class Artifact:
    """A map, memory-mapped read-only, its header checked (the reference's Artifact).

    ``tensors`` by name, ``order`` as the file lays them out.  ``values`` / ``scale_values`` / ``array``
    are zero-copy views of the mapped bytes; ``register`` makes an 8-bit tensor a ``QuantizedWeight``.
    """

    def __init__(self, path: str):
        self.path = str(path)
        try:
            fd = os.open(self.path, os.O_RDONLY)
        except OSError as e:
            raise MapError("cannot_open", f"cannot open {self.path}: {e.strerror}", self.path) from None
        self._mm = None
        try:
            size = os.fstat(fd).st_size
            if size <= 16:
                raise MapError("truncated", "shorter than a prologue")
            self._mm = mmap.mmap(fd, size, prot=mmap.PROT_READ)
            # (slices of an mmap are bytes: no view of it outlives the parse, so a refusal can close it)
            self.header, self.page, self.order, self.tensors = parse(self._mm, size)
        except MapError as e:
            if self._mm is not None:
                self._mm.close()
            raise e.in_file(self.path) from None
        finally:
            os.close(fd)  # the mapping keeps the pages; the descriptor is not needed past this point
        self.size = size

    @staticmethod
    def read_header(path: str) -> dict:
        """The header alone, without mapping the tensors (Artifact.header)."""
        path = str(path)
        try:
            with open(path, "rb") as f:
                prologue = f.read(16)
                if len(prologue) < 16:
                    raise MapError("truncated", "less than a prologue")
                if prologue[:7] != SIGNATURE or prologue[7] not in SUPPORTED_VERSIONS:
                    raise MapError("bad_magic", f"not a Siliconed map (signature {list(prologue[:8])})")
                raw = int.from_bytes(prologue[8:16], "little")
                length = header_length(raw, os.fstat(f.fileno()).st_size)
                if length is None:
                    raise MapError("truncated", f"header length {raw}")
                text = f.read(length)
        except OSError as e:
            raise MapError("cannot_open", f"cannot open {path}: {e.strerror}", path) from None
        except MapError as e:
            raise e.in_file(path) from None
        try:
            header = json.loads(text)
        except (ValueError, UnicodeDecodeError):
            header = None
        if len(text) != length or not isinstance(header, dict):
            raise MapError("bad_header", "not a JSON object", path)
        return header

    @property
    def linear_weights_transposed(self) -> bool:
        """Linear weights stored ``[input, output]`` (the header's ``linear_weights_transposed``)."""
        return self.header.get("linear_weights_transposed") is True

    def close(self) -> None:
        if self._mm is not None:
            try:
                self._mm.close()
            except BufferError:  # a view of the map is still alive; the mapping goes with it
                pass
            self._mm = None

    def __enter__(self) -> "Artifact":
        return self

    def __exit__(self, *exc) -> None:
        self.close()

    def tensor(self, name: str) -> Tensor:
        t = self.tensors.get(name)
        if t is None:
            raise KeyError(f"{self.path}: no tensor {name}")
        return t

    def raw(self, name: str) -> np.ndarray:
        """The tensor's whole region (values, padding and scale) as bytes, zero-copy."""
        t = self.tensor(name)
        return np.frombuffer(self._mm, dtype=np.uint8, count=t.bytes, offset=t.offset)

    def values(self, name: str) -> np.ndarray:
        """An 8-bit tensor's codes in the map's layout (``[K, N]`` for a linear), uint8, zero-copy; for a
        tensor stored in the arena layout, a copy decoded back to ``[K, N]`` as published."""
        t = self.tensor(name)
        if not t.is_quantized:
            raise MapError("bad_header", f"{name}: {t.dtype} is not an 8-bit type", self.path)
        if t.layout == "arena":
            a = self.stored(name)[: t.shape[1], : t.shape[0]]
            return np.ascontiguousarray((a ^ 0x80) if t.dtype == "int8" else a).T.copy()
        return np.frombuffer(self._mm, dtype=np.uint8, count=t.count, offset=t.offset).reshape(t.shape)

    def stored(self, name: str) -> np.ndarray:
        """An arena-layout tensor's bytes as stored, ``[n_pad, k_pad]``, zero-copy."""
        t = self.tensor(name)
        if t.layout != "arena":
            raise MapError("bad_header", f"{name}: not stored in the arena layout", self.path)
        n_pad, k_pad = arena_dims(t.shape[0], t.shape[1])
        return np.frombuffer(self._mm, dtype=np.uint8, count=n_pad * k_pad, offset=t.offset).reshape(n_pad, k_pad)

    def scale_values(self, name: str) -> tuple[str, np.ndarray] | None:
        """(dtype, scale) of an 8-bit tensor, zero-copy: float32 / float16 arrays, bf16 as uint16 bits;
        None for an fp8 cast published without a scale."""
        t = self.tensor(name)
        if t.scale is None:
            return None
        np_type = {"float32": np.float32, "float16": np.float16, "bfloat16": np.uint16}[t.scale.dtype]
        a = np.frombuffer(self._mm, dtype=np_type, count=t.scale.count, offset=t.offset + t.scale.offset)
        return t.scale.dtype, a.reshape(t.scale.shape)

    def array(self, name: str) -> np.ndarray:
        """A float32 / float16 tensor as its array, a bfloat16 one as its uint16 bits, zero-copy."""
        t = self.tensor(name)
        np_type = {"float32": np.float32, "float16": np.float16, "bfloat16": np.uint16}.get(t.dtype)
        if np_type is None:
            raise MapError("bad_header", f"{name}: {t.dtype} has no plain array", self.path)
        return np.frombuffer(self._mm, dtype=np_type, count=t.count, offset=t.offset).reshape(t.shape)

    def materialize(self, name: str, out, ctx=None) -> int:
        """The tensor's values as fp32 into ``out`` (a float32 numpy array or torch tensor, at least its
        count long); returns the count (Artifact.materialize, Artifact.swift:670-715).  A tensor larger
        than ``out`` is refused before a value is written (``does_not_fit``).  bf16 / fp16 / fp32 widen
        exactly on the host; an 8-bit linear is dequantized by the library on ``ctx``'s device
        (sc_dequantize: ``float(q) * s``, its convrot applied), so ``ctx`` is required for one."""
        t = self.tensor(name)
        contiguous = out.is_contiguous() if hasattr(out, "is_contiguous") else out.flags.c_contiguous
        if not contiguous or str(out.dtype) not in ("float32", "torch.float32"):
            raise SiliconedError(abi.INVALID_ARG, f"{name}: the destination must be a contiguous float32 buffer")
        capacity = int(np.prod(out.shape)) if len(out.shape) else 1
        if t.count > capacity:
            raise MapError("does_not_fit", f"{name}: {t.count} values for a buffer of {capacity} - "
                                           "not the map this model reads", self.path)
        if t.dtype in ("float32", "float16", "bfloat16"):
            a = self.array(name).reshape(-1)
            vals = (a.astype(np.uint32) << 16).view(np.float32) if t.dtype == "bfloat16" else a.astype(np.float32)
            flat = out.reshape(-1)
            if hasattr(flat, "copy_"):  # a torch tensor
                import torch
                flat[: t.count].copy_(torch.from_numpy(np.ascontiguousarray(vals)))
            else:
                flat[: t.count] = vals
            return t.count
        if not t.is_quantized or len(t.shape) != 2:
            raise SiliconedError(abi.UNSUPPORTED_SHAPE, f"{self.path}: {name}: {t.dtype} is not read here")
        if ctx is None:
            raise SiliconedError(abi.INVALID_ARG, f"{name}: an 8-bit tensor is dequantized on a device: pass ctx")
        w = self.register(ctx, name)
        try:
            dense = w.dequantize()
            flat = out.reshape(-1)
            if hasattr(flat, "copy_"):
                flat[: t.count].copy_(dense.reshape(-1))
            else:
                flat[: t.count] = dense.reshape(-1).cpu().numpy()
        finally:
            w.close()
        return t.count

    def register(self, ctx, name: str, **kw):
        """The 8-bit linear ``name`` as a ``QuantizedWeight`` on ``ctx``: its ``[K, N]`` codes and its scale
        read in place (WeightProducts.inPlaceInt8, WeightProducts.swift:855-861), its convrot group
        applied.  An fp8 tensor published without a scale is a plain cast, w = f8: its scale is 1.0, an
        exact multiply.  Raises SiliconedError(UNSUPPORTED_SHAPE) for block scales (GGUF Q8_0)."""
        from .products import QuantizedWeight

        t = self.tensor(name)
        if not t.is_quantized or len(t.shape) != 2:
            raise SiliconedError(abi.INVALID_ARG, f"{self.path}: {name}: {t.dtype} {list(t.shape)} is not an 8-bit linear")
        kind = abi.WEIGHT_INT8 if t.dtype == "int8" else abi.WEIGHT_E4M3
        sv = self.scale_values(name)
        scale_type = None
        if sv is None:
            scales = np.ones((), np.float32)
        else:
            st, scales = sv
            if t.scale.block is not None:
                raise SiliconedError(abi.UNSUPPORTED_SHAPE,
                                     f"{self.path}: {name}: a scale per block of {t.scale.block} rows is not a weight-only "
                                     "per-output product")
            if st == "bfloat16":
                scale_type = abi.SCALE_BF16
        rotation = t.rotation.group if t.rotation is not None else 0
        if t.layout == "arena":  # one copy into the device arena, no re-tiling
            return QuantizedWeight(ctx, self.stored(name), kind, scales, scale_type=scale_type, rotation=rotation,
                                   arena=t.shape, nan_codes=t.nan_codes, **kw)
        return QuantizedWeight(ctx, self.values(name), kind, scales, scale_type=scale_type, rotation=rotation, **kw)

    def quantized_names(self) -> list[str]:
        """The 8-bit linears of the map, in file order."""
        return [n for n in self.order if self.tensors[n].is_quantized and len(self.tensors[n].shape) == 2]


# ---- the writer (the forge side) --------------------------------------------------------------------


@dataclass
class MapTensor:
    """One tensor to write: ``data`` its values in the map's layout (``[K, N]`` for a linear), and for an
    8-bit tensor its scale (``scale`` bytes or an array; ``scale_dtype``, ``scale_shape``, ``block``) and
    convrot ``rotation`` group (MapWriter.Tensor, Sources/Siliconed/Forge/Map.swift:204-263)."""
    name: str
    dtype: str
    shape: tuple[int, ...]
    data: bytes | np.ndarray
    scale: bytes | np.ndarray | None = None
    scale_dtype: str | None = None
    scale_shape: tuple[int, ...] | None = None
    block: int | None = None
    rotation: int | None = None
    transposed: bool | None = None
    layout: str | None = None      # "arena": data holds the arena bytes [n_pad][k_pad] (arena_codes)
    nan_codes: bool | None = None

    def value_bytes(self) -> int:
        count = element_count(self.shape)
        if self.layout == "arena":
            n_pad, k_pad = arena_dims(self.shape[0], self.shape[1])
            return n_pad * k_pad
        if self.dtype in SQ_BITS:
            return self.shape[1] * sq_row_bytes(self.shape[0], SQ_BITS[self.dtype])
        if self.dtype in PACKED_BLOCKS:
            v, b = PACKED_BLOCKS[self.dtype]
            return count // v * b
        return count * VALUE_SIZES[self.dtype]

    def scale_offset(self) -> int:
        """Where the scale starts, from the tensor's start: the next 16-byte boundary after the values."""
        return (self.value_bytes() + 15) // 16 * 16

    def total_bytes(self) -> int:
        if self.scale is None:
            return self.value_bytes()
        return self.scale_offset() + (element_count(self.scale_shape) or 0) * VALUE_SIZES[self.scale_dtype]


def _as_bytes(a) -> bytes:
    return a.tobytes() if isinstance(a, np.ndarray) else bytes(a)


def write_map(path: str, tensors: list[MapTensor], header: dict | None = None, page: int = PAGE) -> int:
    """Writes a ``SILICON`` v3 map (MapWriter.write, Map.swift:290-335); returns its size in bytes.

    Tensors are laid out in the given order, each on a page boundary; the prologue (signature, length,
    JSON) takes a whole number of pages; ``header`` adds its keys before ``tensors`` and ``data_start``.
    """
    offsets, end = [], 0
    for t in tensors:
        p = end + (page - end % page) % page
        offsets.append(p)
        end = p + t.total_bytes()

    def prologue(begin: int) -> bytes:
        table = {}
        for t, rel in zip(tensors, offsets):
            e = {"offset": rel + begin, "bytes": t.total_bytes(), "shape": list(t.shape), "dtype": t.dtype}
            if t.transposed is not None:
                e["transposed"] = t.transposed
            if t.scale is not None:
                s = {"offset": t.scale_offset(), "dtype": t.scale_dtype, "shape": list(t.scale_shape)}
                if t.block is not None:
                    s["block"] = t.block
                e["scale"] = s
            if t.rotation:
                e["rotation"] = {"kind": "convrot", "group": int(t.rotation)}
            if t.layout is not None:
                e["layout"] = t.layout
                if t.nan_codes:
                    e["nan_codes"] = True
            table[t.name] = e
        h = {"format": 1, "page": page, "linear_weights_transposed": True}
        h.update(header or {})
        h["order"] = [t.name for t in tensors]
        h["tensors"] = table
        h["data_start"] = begin
        text = json.dumps(h, separators=(",", ":")).encode()
        return SIGNATURE + bytes([WRITE_VERSION]) + len(text).to_bytes(8, "little") + text

    begin = (len(prologue(0)) + page - 1) // page * page
    while len(prologue(begin)) > begin:
        begin += page
    head = prologue(begin)
    with open(path, "wb") as f:
        f.write(head + bytes(begin - len(head)))
        for t, rel in zip(tensors, offsets):
            f.seek(begin + rel)
            values = _as_bytes(t.data)
            if len(values) != t.value_bytes():
                raise ValueError(f"{t.name}: {len(values)} value bytes for {t.shape} of {t.dtype}")
            f.write(values)
            if t.scale is not None:
                scale = _as_bytes(t.scale)
                f.write(bytes(t.scale_offset() - len(values)))
                if len(scale) != t.total_bytes() - t.scale_offset():
                    raise ValueError(f"{t.name}: {len(scale)} scale bytes for {t.scale_shape} of {t.scale_dtype}")
                f.write(scale)
        f.truncate(begin + end)
    return begin + end


class ForgeRefusal(ValueError):
    """A published 8-bit weight the forge does not keep, with the reason (the reference's forge refusals,
    QuantizedMapTests.swift:485-503, 620-641)."""


def _scale_as_f32(s: np.ndarray, scale_dtype: str) -> np.ndarray:
    if scale_dtype == "bfloat16":
        return (s.astype(np.uint32) << 16).view(np.float32)
    return s.astype(np.float32)


def forge_linear(name: str, values_nk: np.ndarray, scales: np.ndarray | None, dtype: str, scale_dtype: str | None,
                 rotation: int | None = None, layout: str | None = None) -> MapTensor:
    """A published 8-bit ``nn.Linear`` weight as the map keeps it (the forge's ``kept8bit`` outcome,
    QuantizedMapTests.swift:149-216): the codes ``[N, K]`` transposed to ``[K, N]`` byte for byte, the
    scale (``[N, 1]`` / ``[N]`` per output row, or ``[]`` / ``[1]`` for the tensor) kept in its published
    type and flattened to ``[N]`` or ``[]``.  ``scales`` holds bf16 as uint16 bits.

    Refused (``ForgeRefusal``), as the forge does: an int8 weight without a scale (an fp8 one without a
    scale is a plain cast, w = f8); a scale shaped otherwise than one per tensor or one per row; a nonzero
    scale whose smallest product ``|s| * min|q| / sqrt(G)`` is subnormal in fp32 (min|q| = 1 for int8,
    2^-9 for e4m3; ``QuantizedLayouts.checkSubnormal``, Forge/Quantization.swift:380-402).

    ``layout="arena"`` (this library's extension of the map) stores the codes as the device arena keeps
    them (``arena_codes``: [n_pad][k_pad], int8 biased), so that registering the tensor is one copy with
    no re-tiling kernel; the header records ``"layout": "arena"`` and, for e4m3, whether NaN codes occur."""
    if dtype not in ("int8", "float8_e4m3"):
        raise ForgeRefusal(f"{name}: {dtype} is not an 8-bit weight type")
    q = np.ascontiguousarray(values_nk).view(np.uint8)
    if q.ndim != 2:
        raise ForgeRefusal(f"{name}: a linear weight is [N, K], not {list(q.shape)}")
    n, k = q.shape
    if scales is None:
        if dtype == "int8":
            raise ForgeRefusal(f"{name}: int8 without a scale")
        if rotation:
            raise ForgeRefusal(f"{name}: a rotation needs a scale")
        return MapTensor(name, dtype, (k, n), np.ascontiguousarray(q.T), transposed=True)
    if scale_dtype not in SCALE_TYPES:
        raise ForgeRefusal(f"{name}: a scale of type {scale_dtype}")
    s = np.ascontiguousarray(scales)
    if s.shape in ((), (1,)):
        s_shape: tuple[int, ...] = ()
    elif s.shape in ((n,), (n, 1)):
        s_shape = (n,)
    else:
        raise ForgeRefusal(f"{name}: a scale {list(s.shape)} for [{n}, {k}]: only one per tensor or one per row")
    # in fp32, as the forge computes it (a product rounded to the nearest subnormal can reach 2^-126)
    smallest = np.float32((1.0 if dtype == "int8" else 2.0 ** -9) / np.sqrt(float(rotation or 1)))
    sf = np.abs(_scale_as_f32(s.reshape(-1), scale_dtype))
    with np.errstate(under="ignore"):
        low = (sf != 0) & (sf * smallest < np.float32(2.0 ** -126))
    if np.any(low):
        raise ForgeRefusal(f"{name}: a scale whose products can fall below 2^-126 (subnormal)")
    if rotation and (dtype != "int8" or not is_rotation_group(rotation) or k % rotation != 0):
        raise ForgeRefusal(f"{name}: rotation convrot of group {rotation} on {dtype} [{n}, {k}]")
    if layout == "arena":
        nan = dtype == "float8_e4m3" and bool(np.any((q & 0x7F) == 0x7F))
        return MapTensor(name, dtype, (k, n), arena_codes(q, dtype), s.reshape(s_shape), scale_dtype, s_shape,
                         rotation=rotation, transposed=True, layout="arena", nan_codes=nan)
    if layout is not None:
        raise ForgeRefusal(f"{name}: unknown layout {layout!r}")
    return MapTensor(name, dtype, (k, n), np.ascontiguousarray(q.T), s.reshape(s_shape), scale_dtype, s_shape,
                     rotation=rotation, transposed=True)
