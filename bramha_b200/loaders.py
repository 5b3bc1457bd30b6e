"""On-disk model formats of the reference, read straight into the device registry.

* **Manifest directory** (``src/storage/tensor_db.rs:625-690``, written by
  ``src/bin/quantize_model.rs:284-306``): ``manifest.json`` (serde JSON of
  ``ModelManifest``; ``layers`` maps a layer id to its ``LayerMetadata``) next to
  one shard per layer named after the layer id with ``.`` replaced by ``_``:
  ``<name>_u4.bin`` (``Int4PerChannel``: ``quantize_to_int4`` bytes, u8 [N][K/2]),
  ``<name>_i8.bin`` (``Int8Linear``: i8 [N][K]), ``<name>.bin`` (raw f32), with the
  per-row scales of a quantized layer in ``<name>_scale.bin`` (f32 [N], little
  endian).  Candidate names are tried in the reference's order; a non-empty
  ``checksum`` is the SHA-256 of the chosen shard file and must match.
* **``.spanda``** (``spanda-engine/src/lib.rs:85-139``): the magic ``SPANDA07``
  followed by ``SpandaModel`` {``metadata: ModelMetadata``, ``tensors:
  HashMap<String, SpandaTensor>``} encoded with bincode 2.0.0-rc.3 (pinned in the
  reference's Cargo.toml) and ``bincode::config::standard()``: little endian,
  variable-length integers (value < 251: one byte; else a marker 251 / 252 / 253
  followed by the value as u16 / u32 / u64), ``u8``/``i8`` one raw byte, ``f32``
  four bytes, strings and sequences a varint length then their items, enum
  variants a varint index then the fields, structs their fields in order, maps a
  varint length then key / value pairs.  ``SpandaTensor`` variants: 0 ``Dense
  (Vec<f32>)``, 1 ``BlockSparse2_4 {shape: Vec<usize>, masks: Vec<u16>,
  nonzero_values: Vec<f32>}``, 2 ``Quant4Log {data: Vec<u8>, scales:
  Vec<f32>}``, 3 ``Quant8Linear {data: Vec<i8>, scales: Vec<f32>}``.

This module is host I/O around the C ABI: weights go to the device through
``bramha_cuda_register_weight`` (the reference's row-major packed bytes; the
library repacks them for its kernels).
"""
from __future__ import annotations

import hashlib
import json
import os
import struct
from dataclasses import dataclass
from typing import Dict, Optional, Sequence, Tuple

import numpy as np

from .plane import packed_nbytes

MAGIC = b"SPANDA07"


# ------------------------------------------------------------------ bincode 2
class _Reader:
    def __init__(self, buf: bytes, pos: int = 0):
        self.b, self.p = memoryview(buf), pos

    def take(self, n: int) -> memoryview:
        if self.p + n > len(self.b):
            raise ValueError("truncated .spanda data")
        v = self.b[self.p:self.p + n]
        self.p += n
        return v

    def u8(self) -> int:
        return self.take(1)[0]

    def varint(self) -> int:
        t = self.u8()
        if t < 251:
            return t
        if t == 251:
            return struct.unpack("<H", self.take(2))[0]
        if t == 252:
            return struct.unpack("<I", self.take(4))[0]
        if t == 253:
            return struct.unpack("<Q", self.take(8))[0]
        raise ValueError(f"unsupported varint marker {t}")

    def string(self) -> str:
        return bytes(self.take(self.varint())).decode("utf-8")

    def f32s(self) -> np.ndarray:
        n = self.varint()
        return np.frombuffer(self.take(4 * n), dtype="<f4").astype(np.float32)

    def bytes_(self, dtype) -> np.ndarray:
        n = self.varint()
        return np.frombuffer(self.take(n), dtype=dtype).copy()

    def varints(self) -> np.ndarray:
        return np.array([self.varint() for _ in range(self.varint())], dtype=np.int64)


def _varint(v: int) -> bytes:
    if v < 0:
        raise ValueError("unsigned varint expected")
    if v < 251:
        return bytes([v])
    if v < 1 << 16:
        return b"\xfb" + struct.pack("<H", v)
    if v < 1 << 32:
        return b"\xfc" + struct.pack("<I", v)
    return b"\xfd" + struct.pack("<Q", v)


def _string(s: str) -> bytes:
    e = s.encode("utf-8")
    return _varint(len(e)) + e


def _f32s(a) -> bytes:
    a = np.ascontiguousarray(a, dtype="<f4")
    return _varint(a.size) + a.tobytes()


META_FIELDS = ("name", "architecture", "hidden_size", "num_attention_heads", "num_key_value_heads", "head_dim",
               "num_hidden_layers", "vocab_size")


@dataclass
class SpandaTensor:
    kind: str                               # "dense" | "sparse24" | "log4" | "int8"
    data: np.ndarray                        # f32 values, packed u8 codes or i8 codes
    scales: Optional[np.ndarray] = None     # log4 / int8
    shape: Optional[Tuple[int, ...]] = None  # sparse24
    masks: Optional[np.ndarray] = None      # sparse24 (u16 per 4-group)


def read_spanda(path: str) -> Tuple[dict, Dict[str, SpandaTensor]]:
    """SpandaModel::load_from_file (lib.rs:123-139): (metadata, tensors)."""
    with open(path, "rb") as f:
        buf = f.read()
    if buf[:8] != MAGIC:
        raise ValueError("Invalid file magic: Expected SPANDA07")
    r = _Reader(buf, 8)
    meta = {}
    for k in META_FIELDS:
        meta[k] = r.string() if k in ("name", "architecture") else r.varint()
    tensors = {}
    for _ in range(r.varint()):
        name = r.string()
        v = r.varint()
        if v == 0:
            tensors[name] = SpandaTensor("dense", r.f32s())
        elif v == 1:
            shape = tuple(int(s) for s in r.varints())
            masks = r.varints().astype(np.uint16)
            tensors[name] = SpandaTensor("sparse24", r.f32s(), shape=shape, masks=masks)
        elif v == 2:
            data = r.bytes_(np.uint8)
            tensors[name] = SpandaTensor("log4", data, scales=r.f32s())
        elif v == 3:
            data = r.bytes_(np.int8)
            tensors[name] = SpandaTensor("int8", data, scales=r.f32s())
        else:
            raise ValueError(f"unknown SpandaTensor variant {v}")
    # decode_from_std_read stops after the model: trailing bytes are ignored
    return meta, tensors


def write_spanda(path: str, meta: dict, tensors: Dict[str, SpandaTensor]):
    """SpandaModel::save_to_file (lib.rs:109-121), same encoding."""
    out = [MAGIC]
    for k in META_FIELDS:
        out.append(_string(meta[k]) if k in ("name", "architecture") else _varint(int(meta[k])))
    out.append(_varint(len(tensors)))
    for name, t in tensors.items():
        out.append(_string(name))
        if t.kind == "dense":
            out += [_varint(0), _f32s(t.data)]
        elif t.kind == "sparse24":
            out += [_varint(1), _varint(len(t.shape))] + [_varint(int(s)) for s in t.shape]
            out += [_varint(len(t.masks))] + [_varint(int(m)) for m in t.masks] + [_f32s(t.data)]
        elif t.kind in ("log4", "int8"):
            d = np.ascontiguousarray(t.data, dtype=np.uint8 if t.kind == "log4" else np.int8)
            out += [_varint(2 if t.kind == "log4" else 3), _varint(d.size), d.tobytes(), _f32s(t.scales)]
        else:
            raise ValueError(t.kind)
    with open(path, "wb") as f:
        f.write(b"".join(out))


# ------------------------------------------------------------ manifest dirs
_CANDIDATES = {
    "Int4PerChannel": ("_u4.bin", "_scale.bin", ".bin"),
    "Int8Linear": ("_i8.bin", "_scale.bin", ".bin"),
    "Svd": ("_svd.bin", ".bin"),
    "ColumnarDict": ("_cd.bin", ".bin"),
}


def _fmt_name(cf) -> str:
    return cf if isinstance(cf, str) else next(iter(cf))  # unit variant, or {"Variant": payload}


def read_manifest_dir(path: str) -> Tuple[dict, Dict[str, dict]]:
    """The manifest branch of the reference's model restore (tensor_db.rs:625-720):
    for every layer, the first existing candidate shard in the reference's order,
    its SHA-256 checked against a non-empty ``checksum`` (a mismatch raises, where
    the reference panics), layers without a shard skipped.  Returns (manifest,
    {layer_id: {"format", "shape", "file", "data"}}) with ``data`` as raw bytes
    (u8): the caller reads them by format, as the page dtype does."""
    with open(os.path.join(path, "manifest.json")) as f:
        manifest = json.load(f)
    layers = {}
    for meta in manifest["layers"].values():
        lid = meta["layer_id"]
        safe = lid.replace(".", "_")
        fmt = _fmt_name(meta.get("compression_format", "None"))
        cands = [safe + suf for suf in _CANDIDATES.get(fmt, (".bin",))]
        found = next((c for c in cands if os.path.exists(os.path.join(path, c))), None)
        if found is None:
            continue
        with open(os.path.join(path, found), "rb") as fh:
            raw = fh.read()
        if meta.get("checksum"):
            digest = hashlib.sha256(raw).hexdigest()
            if digest != meta["checksum"]:
                raise ValueError(f"checksum mismatch for tensor shard {found}: expected {meta['checksum']}, "
                                 f"actual {digest}")
        layers[lid] = {"format": fmt, "shape": tuple(int(v) for v in meta["shape"]), "file": found,
                       "data": np.frombuffer(raw, dtype=np.uint8)}
    return manifest, layers


def _scales_for(layers: dict, lid: str) -> np.ndarray:
    """The ``<layer>.scale`` page that the reference pairs with a quantized weight
    (cpu_engine.rs:142-158; quantize_model.rs:298-301 writes it as its own
    layer of shape [out_features])."""
    sp = layers.get(lid + ".scale")
    if sp is None:
        raise ValueError(f"Scale not found for quantized weight: {lid}")
    return sp["data"].view("<f4").astype(np.float32)


def register_manifest_dir(plane, path: str, model_name: Optional[str] = None,
                          f32_weights: Sequence[str] = ()) -> Dict[str, object]:
    """Restores a manifest directory onto the device.  Quantized 2-D weights are
    registered under ``"model:layer"`` (the weight keys of get_or_create_op,
    wgpu_backend.rs:603-722): an ``Int4PerChannel`` layer read from its
    ``_u4.bin`` shard as W4ZP8, an ``Int8Linear`` layer read from its ``_i8.bin``
    shard as W8, each with the scales of its ``.scale`` layer; the f32 layers
    named in ``f32_weights`` (an unquantized lm_head, say) as F32.  Every other
    layer (embedding, norms, biases, scales) is returned as an f32 numpy array of
    its shape.  Returns {layer_id: Weight | np.ndarray}.

    Two shapes of directory that the reference reads silently wrong raise here:
    a quantized layer whose candidate search lands on its ``_scale.bin`` (the
    ``_u4.bin`` / ``_i8.bin`` shard missing), and a shard whose size disagrees
    with its shape.  The reference types ``Int8Linear`` pages as f32
    (tensor_db.rs:681-690); this loader gives them the i8 meaning their
    ``_i8.bin`` name states."""
    manifest, layers = read_manifest_dir(path)
    model = model_name or manifest.get("name", "model")
    out = {}
    for lid, e in layers.items():
        shape, fmt, data, f = e["shape"], e["format"], e["data"], e["file"]
        quant = {"Int4PerChannel": ("_u4.bin", "w4zp8"), "Int8Linear": ("_i8.bin", "w8")}.get(fmt)
        if quant is not None and not f.endswith(quant[0]):
            raise ValueError(f"{lid}: {fmt} layer without its {lid.replace('.', '_')}{quant[0]} shard (found {f})")
        if quant is not None and len(shape) == 2:
            n, k = shape
            want = packed_nbytes(quant[1], n, k)
            if data.size != want:
                raise ValueError(f"{lid}: shard {f} has {data.size} bytes, shape {shape} needs {want}")
            out[lid] = plane.register(f"{model}:{lid}", quant[1], n, k, data, _scales_for(layers, lid))
            continue
        vals = data.view("<f4").astype(np.float32) if data.size % 4 == 0 else None
        if vals is None or (shape and vals.size != int(np.prod(shape))):
            raise ValueError(f"{lid}: shard {f} has {data.size} bytes, f32 shape {shape} needs "
                             f"{4 * int(np.prod(shape))}")
        if lid in f32_weights:
            if len(shape) != 2:
                raise ValueError(f"{lid}: an f32 GEMV weight needs a 2-D shape, got {shape}")
            out[lid] = plane.register(f"{model}:{lid}", "f32", shape[0], shape[1], vals.reshape(shape))
        else:
            out[lid] = vals.reshape(shape) if shape else vals
    return out


_SUFFIX = {"w4zp8": ("_u4.bin", "Int4PerChannel", 4), "w8": ("_i8.bin", "Int8Linear", 8)}


def _layer_meta(lid: str, shape, fmt: str, bits, stored: int, checksum: str) -> dict:
    n = int(np.prod(shape)) if shape else 0
    crit = any(t in lid for t in ("embed", "lm_head", "norm", "attn"))
    return {"layer_id": lid, "shape": [int(v) for v in shape], "num_elements": n, "original_bytes": 4 * n,
            "stored_bytes": stored, "compression_format": fmt, "storage_tier": "Critical" if crit else "Important",
            "reference_tensor": None, "statistics": {"access_count": 0, "last_accessed_timestamp": None},
            "quantization_bits": bits, "reference_layer": None, "checksum": checksum, "svd_rank": None,
            "dict_size": None, "chunks": None}


def write_manifest_dir(path: str, name: str, layers: Dict[str, object], *, architecture: str = "qwen2",
                       hidden_size: int = 0, num_heads: int = 0, num_kv_heads: int = 0, checksums: bool = True):
    """Writes a manifest directory the reference's restore reads: the inverse of
    :func:`read_manifest_dir`, with the layout quantize_model.rs:284-306 produces.
    ``layers`` maps a layer id to an f32 array (written as ``<name>.bin``) or to a
    tuple ``(fmt, out_features, in_features, q, scales)`` with fmt ``"w4zp8"``
    (``<name>_u4.bin``, Int4PerChannel) or ``"w8"`` (``<name>_i8.bin``,
    Int8Linear); a quantized layer also gets its ``<name>.scale`` layer (f32 [N]
    in ``<name>_scale.bin``).  With ``checksums`` each layer records the SHA-256
    of its shard.  manifest.json carries every field of ModelManifest and
    LayerMetadata (storage_manifest.rs:64-127, 201-263) that serde requires."""
    os.makedirs(path, exist_ok=True)
    metas = {}

    def put(lid, fname, raw: bytes, shape, fmt, bits):
        with open(os.path.join(path, fname), "wb") as f:
            f.write(raw)
        metas[lid] = _layer_meta(lid, shape, fmt, bits, len(raw), hashlib.sha256(raw).hexdigest() if checksums else "")

    for lid, v in layers.items():
        safe = lid.replace(".", "_")
        if isinstance(v, tuple):
            fmt, n, k, q, sc = v
            suf, cf, bits = _SUFFIX[fmt]
            qa = np.ascontiguousarray(q, dtype=np.uint8 if fmt == "w4zp8" else np.int8)
            if qa.size != packed_nbytes(fmt, n, k):
                raise ValueError(f"{lid}: {qa.size} code bytes for a {n} x {k} {fmt} weight")
            put(lid, safe + suf, qa.tobytes(), (n, k), cf, bits)
            put(lid + ".scale", safe + "_scale.bin", np.ascontiguousarray(sc, dtype="<f4").tobytes(), (n,), "None",
                None)
        else:
            a = np.ascontiguousarray(v, dtype="<f4")
            put(lid, safe + ".bin", a.tobytes(), a.shape, "None", None)
    orig = sum(m["original_bytes"] for m in metas.values())
    stored = sum(m["stored_bytes"] for m in metas.values())
    tiers = [m["storage_tier"] for m in metas.values()]
    ratio = orig / stored if stored else 1.0
    manifest = {
        "name": name, "variant": "q4" if any(isinstance(v, tuple) for v in layers.values()) else "base",
        "num_layers": len(metas), "architecture": architecture, "hidden_size": hidden_size, "num_heads": num_heads,
        "num_kv_heads": num_kv_heads, "layers": metas, "total_original_size": orig, "total_stored_size": stored,
        "created_at": 0, "last_modified": 0, "manifest_checksum": "", "storage_path": path,
        "avg_compression_ratio": ratio, "max_compression_ratio": ratio, "min_compression_ratio": ratio,
        "quantized_layers": sum(m["quantization_bits"] is not None for m in metas.values()),
        "full_precision_layers": sum(m["quantization_bits"] is None for m in metas.values()),
        "critical_count": tiers.count("Critical"), "important_count": tiers.count("Important"),
        "robust_count": 0, "redundant_count": 0, "num_experts": None, "expert_routing_top_k": None,
    }
    with open(os.path.join(path, "manifest.json"), "w") as f:
        json.dump(manifest, f, indent=2)


def register_spanda(plane, path: str) -> Tuple[dict, Dict[str, object]]:
    """Reads a .spanda file and registers its tensors on the device:
    BlockSparse2_4 with a 2-D shape as a compressed 2:4 weight (rows =
    shape[0], cols = shape[1], as the SPANDA forward loop reads it,
    lib.rs:256-266); Quant4Log -> LOG4 and Quant8Linear -> W8 with one scale
    per output row (N = len(scales), the packed codes give K).  Dense tensors
    (and 2:4 tensors without a 2-D shape) are returned as read."""
    meta, tensors = read_spanda(path)
    model = meta["name"]
    out = {}
    for name, t in tensors.items():
        if t.kind == "sparse24" and len(t.shape) == 2:
            out[name] = plane.register_sparse24_compressed(f"{model}:{name}", t.shape[0], t.shape[1], t.masks, t.data)
        elif t.kind in ("log4", "int8"):
            n = int(t.scales.size)
            if n == 0 or t.data.size % n:
                raise ValueError(f"{name}: {t.data.size} code bytes do not split into {n} rows")
            k = t.data.size // n * (2 if t.kind == "log4" else 1)
            out[name] = plane.register(f"{model}:{name}", "log4" if t.kind == "log4" else "w8", n, k, t.data,
                                       t.scales)
        else:
            out[name] = t
    return meta, out
