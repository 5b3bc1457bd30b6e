"""On-disk formats: the manifest directory (tensor_db.rs:625-720,
quantize_model.rs:284-306) and the ``.spanda`` container (spanda-engine/src/lib.rs:
85-139, bincode 2.0.0-rc.3 standard config).

The reference ships no fixture files for either format, so the bincode reader
is pinned to known-answer byte strings assembled here from bincode's published
encoding rules (varint thresholds 251/252/253, little endian, raw u8/i8, f32 as
4 bytes, enum index then fields), independently of this package's writer.  The
GPU tests check that a loaded weight computes exactly what the same bytes
registered directly compute, and matches the oracle's GEMV.
"""
import hashlib
import json
import os
import struct

import numpy as np
import pytest

import oracle
from bramha_b200 import loaders as L
from tests._util import GEMV_TOL, make_weight, make_x, normwise_err, rng


# ------------------------------------------------------------------ bincode
@pytest.mark.parametrize("value,encoded", [
    (0, b"\x00"), (250, b"\xfa"), (251, b"\xfb\xfb\x00"), (896, b"\xfb\x80\x03"), (65535, b"\xfb\xff\xff"),
    (65536, b"\xfc\x00\x00\x01\x00"), (151936, b"\xfc\x80\x51\x02\x00"), (2**32 - 1, b"\xfc\xff\xff\xff\xff"),
    (2**32, b"\xfd\x00\x00\x00\x00\x01\x00\x00\x00"), (2**64 - 1, b"\xfd" + b"\xff" * 8)])
def test_varint_known_answers(value, encoded):
    assert L._varint(value) == encoded
    r = L._Reader(encoded)
    assert r.varint() == value and r.p == len(encoded)


def test_varint_rejects_u128_marker():
    with pytest.raises(ValueError, match="varint marker 254"):
        L._Reader(b"\xfe" + b"\x00" * 16).varint()


def _kat_bytes():
    """SpandaModel {metadata {name "t", architecture "qwen2", 896, 14, 2, 64, 24,
    151936}, tensors {"a": Quant4Log {data [0x1f, 0xf0], scales [0.5]},
    "b": BlockSparse2_4 {shape [1, 4], masks [5, 300], nonzero_values [1, -2]},
    "c": Quant8Linear {data [-1, 127], scales [0.25]}, "d": Dense([3.0])}}."""
    f = lambda *v: struct.pack("<%df" % len(v), *v)
    return (b"SPANDA07" + b"\x01t" + b"\x05qwen2" + b"\xfb\x80\x03" + b"\x0e" + b"\x02" + b"\x40" + b"\x18"
            + b"\xfc\x80\x51\x02\x00"
            + b"\x04"
            + b"\x01a" + b"\x02" + b"\x02\x1f\xf0" + b"\x01" + f(0.5)
            + b"\x01b" + b"\x01" + b"\x02\x01\x04" + b"\x02\x05\xfb\x2c\x01" + b"\x02" + f(1.0, -2.0)
            + b"\x01c" + b"\x03" + b"\x02\xff\x7f" + b"\x01" + f(0.25)
            + b"\x01d" + b"\x00" + b"\x01" + f(3.0))


def test_spanda_reader_known_answer(tmp_path):
    p = tmp_path / "kat.spanda"
    p.write_bytes(_kat_bytes())
    meta, t = L.read_spanda(str(p))
    assert meta == {"name": "t", "architecture": "qwen2", "hidden_size": 896, "num_attention_heads": 14,
                    "num_key_value_heads": 2, "head_dim": 64, "num_hidden_layers": 24, "vocab_size": 151936}
    assert list(t) == ["a", "b", "c", "d"]
    assert t["a"].kind == "log4" and t["a"].data.tolist() == [0x1F, 0xF0] and t["a"].scales.tolist() == [0.5]
    assert t["b"].kind == "sparse24" and t["b"].shape == (1, 4) and t["b"].masks.tolist() == [5, 300]
    assert t["b"].data.tolist() == [1.0, -2.0]
    assert t["c"].kind == "int8" and t["c"].data.dtype == np.int8 and t["c"].data.tolist() == [-1, 127]
    assert t["d"].kind == "dense" and t["d"].data.tolist() == [3.0]
    # the writer reproduces the same bytes (HashMap order is the file's order)
    q = tmp_path / "w.spanda"
    L.write_spanda(str(q), meta, t)
    assert q.read_bytes() == _kat_bytes()
    # Quant4Log bytes decode as dequantize_log4 does: high nibble first, 2^c - 1
    assert oracle.dequantize_log4(t["a"].data, 0.5).tolist() == [0.5, 16383.5, 16383.5, 0.0]


def test_spanda_errors_and_trailing_bytes(tmp_path):
    p = tmp_path / "x.spanda"
    p.write_bytes(b"SPANDA06" + _kat_bytes()[8:])
    with pytest.raises(ValueError, match="Expected SPANDA07"):
        L.read_spanda(str(p))
    p.write_bytes(_kat_bytes()[:-3])
    with pytest.raises(ValueError, match="truncated"):
        L.read_spanda(str(p))
    bad = bytearray(_kat_bytes())
    bad[bad.index(b"\x01d") + 2] = 7  # variant index 7
    p.write_bytes(bytes(bad))
    with pytest.raises(ValueError, match="variant 7"):
        L.read_spanda(str(p))
    p.write_bytes(_kat_bytes() + b"\x00\x01")  # decode_from_std_read ignores what follows
    assert len(L.read_spanda(str(p))[1]) == 4


def test_spanda_round_trip_large(tmp_path):
    r = rng(3)
    meta = {"name": "qwen2-0.5b", "architecture": "qwen2", "hidden_size": 896, "num_attention_heads": 14,
            "num_key_value_heads": 2, "head_dim": 64, "num_hidden_layers": 24, "vocab_size": 151936}
    _, q4, s4 = make_weight("log4", 300, 512, seed=1)
    _, q8, s8 = make_weight("w8", 70, 896, seed=2)
    dense = r.normal(0, 1, 1000).astype(np.float32)
    masks = r.integers(0, 1 << 16, 600).astype(np.uint16)
    t = {"model.layers.0.mlp.up_proj.weight": L.SpandaTensor("log4", q4, scales=s4),
         "model.layers.0.self_attn.o_proj.weight": L.SpandaTensor("int8", q8.view(np.int8), scales=s8),
         "model.norm.weight": L.SpandaTensor("dense", dense),
         "model.layers.0.mlp.gate_proj.weight": L.SpandaTensor("sparse24", dense[:600], shape=(600, 2),
                                                               masks=masks),
         "ü.名前": L.SpandaTensor("dense", np.zeros(0, np.float32))}
    p = str(tmp_path / "m.spanda")
    L.write_spanda(p, meta, t)
    meta2, t2 = L.read_spanda(p)
    assert meta2 == meta and list(t2) == list(t)
    for k, v in t.items():
        w = t2[k]
        assert w.kind == v.kind and np.array_equal(w.data, v.data) and w.data.dtype == np.asarray(v.data).dtype
        if v.scales is not None:
            assert np.array_equal(w.scales, v.scales)
        if v.kind == "sparse24":
            assert w.shape == v.shape and np.array_equal(w.masks, v.masks)


# ------------------------------------------------------------- manifest dirs
def _model_layers(n=256, k=128, inter=384):
    r = rng(9)
    _, qq, sq = make_weight("w4zp8", n, k, seed=4)
    _, qd, sd = make_weight("w8", k, inter, seed=5)
    return {"model.layers.0.self_attn.q_proj.weight": ("w4zp8", n, k, qq, sq),
            "model.layers.0.mlp.down_proj.weight": ("w8", k, inter, qd, sd),
            "model.norm.weight": r.normal(1, 0.1, k).astype(np.float32),
            "lm_head.weight": r.normal(0, 0.02, (64, k)).astype(np.float32)}


def test_manifest_dir_layout_and_read_back(tmp_path):
    d = str(tmp_path / "m")
    layers = _model_layers()
    L.write_manifest_dir(d, "tiny", layers, hidden_size=128, num_heads=4, num_kv_heads=2)
    names = sorted(os.listdir(d))
    assert names == sorted(["manifest.json", "model_layers_0_self_attn_q_proj_weight_u4.bin",
                            "model_layers_0_self_attn_q_proj_weight_scale.bin",
                            "model_layers_0_mlp_down_proj_weight_i8.bin",
                            "model_layers_0_mlp_down_proj_weight_scale.bin", "model_norm_weight.bin",
                            "lm_head_weight.bin"])
    with open(os.path.join(d, "manifest.json")) as f:
        man = json.load(f)
    ql = man["layers"]["model.layers.0.self_attn.q_proj.weight"]
    assert ql["compression_format"] == "Int4PerChannel" and ql["quantization_bits"] == 4 and ql["shape"] == [256, 128]
    assert man["layers"]["model.layers.0.self_attn.q_proj.weight.scale"]["shape"] == [256]
    raw = open(os.path.join(d, "model_layers_0_self_attn_q_proj_weight_u4.bin"), "rb").read()
    assert ql["checksum"] == hashlib.sha256(raw).hexdigest() and raw == layers[
        "model.layers.0.self_attn.q_proj.weight"][3].tobytes()
    _, got = L.read_manifest_dir(d)
    assert got["model.layers.0.mlp.down_proj.weight"]["file"].endswith("_i8.bin")
    assert got["model.layers.0.self_attn.q_proj.weight.scale"]["file"].endswith("_scale.bin")


class _FakePlane:
    def __init__(self):
        self.calls = []

    def register(self, key, fmt, n, k, q, s=None):
        self.calls.append((key, fmt, n, k, np.array(q), None if s is None else np.array(s)))
        return (key, fmt, n, k)

    def register_sparse24_compressed(self, key, rows, cols, masks, values):
        self.calls.append((key, "sp24_f32", rows, cols, np.array(masks), np.array(values)))
        return (key, "sp24_f32", rows, cols)


def test_register_manifest_dir_mapping(tmp_path):
    d = str(tmp_path / "m")
    layers = _model_layers()
    L.write_manifest_dir(d, "tiny", layers)
    plane = _FakePlane()
    out = L.register_manifest_dir(plane, d, f32_weights=["lm_head.weight"])
    calls = {c[0]: c for c in plane.calls}
    assert set(calls) == {"tiny:model.layers.0.self_attn.q_proj.weight", "tiny:model.layers.0.mlp.down_proj.weight",
                          "tiny:lm_head.weight"}
    key, fmt, n, k, q, s = calls["tiny:model.layers.0.self_attn.q_proj.weight"]
    src = layers["model.layers.0.self_attn.q_proj.weight"]
    assert (fmt, n, k) == ("w4zp8", 256, 128) and np.array_equal(q, src[3]) and np.array_equal(s, src[4])
    key, fmt, n, k, q, s = calls["tiny:model.layers.0.mlp.down_proj.weight"]
    src = layers["model.layers.0.mlp.down_proj.weight"]
    assert (fmt, n, k) == ("w8", 128, 384) and np.array_equal(q.view(np.int8), src[3].view(np.int8))
    assert calls["tiny:lm_head.weight"][1] == "f32"
    assert np.array_equal(out["model.norm.weight"], layers["model.norm.weight"])
    assert out["model.layers.0.self_attn.q_proj.weight.scale"].shape == (256,)


def test_manifest_checksum_mismatch_and_missing_shards(tmp_path):
    d = str(tmp_path / "m")
    L.write_manifest_dir(d, "tiny", _model_layers())
    p = os.path.join(d, "model_norm_weight.bin")
    raw = bytearray(open(p, "rb").read())
    raw[0] ^= 1
    open(p, "wb").write(bytes(raw))
    with pytest.raises(ValueError, match="checksum mismatch for tensor shard model_norm_weight.bin"):
        L.read_manifest_dir(d)
    os.remove(p)  # a layer without a shard is skipped, as in the reference
    _, got = L.read_manifest_dir(d)
    assert "model.norm.weight" not in got and "lm_head.weight" in got
    # a quantized weight without its scale layer: the reference's lookup error
    os.remove(os.path.join(d, "model_layers_0_mlp_down_proj_weight_scale.bin"))
    with pytest.raises(ValueError, match="Scale not found for quantized weight: model.layers.0.mlp.down_proj"):
        L.register_manifest_dir(_FakePlane(), d)
    # an int4 layer whose candidate search lands on _scale.bin is refused
    L.write_manifest_dir(d, "tiny", _model_layers(), checksums=False)
    os.remove(os.path.join(d, "model_layers_0_self_attn_q_proj_weight_u4.bin"))
    with pytest.raises(ValueError, match="without its model_layers_0_self_attn_q_proj_weight_u4.bin shard"):
        L.register_manifest_dir(_FakePlane(), d)


def test_manifest_reads_variant_payloads_and_shape_mismatch(tmp_path):
    d = str(tmp_path / "m")
    L.write_manifest_dir(d, "tiny", {"a.w": np.ones((4, 8), np.float32)}, checksums=False)
    mp = os.path.join(d, "manifest.json")
    man = json.load(open(mp))
    man["layers"]["a.w"]["compression_format"] = {"DeltaFromLayer": "b.w"}  # a serde newtype variant
    json.dump(man, open(mp, "w"))
    _, got = L.read_manifest_dir(d)
    assert got["a.w"]["format"] == "DeltaFromLayer"
    man["layers"]["a.w"]["shape"] = [4, 9]
    json.dump(man, open(mp, "w"))
    with pytest.raises(ValueError, match="f32 shape"):
        L.register_manifest_dir(_FakePlane(), d)


def test_register_spanda_mapping(tmp_path):
    _, q4, s4 = make_weight("log4", 40, 64, seed=1)
    _, q8, s8 = make_weight("w8", 24, 32, seed=2)
    meta = {k: 1 for k in L.META_FIELDS}
    meta.update(name="m", architecture="qwen2")
    p = str(tmp_path / "m.spanda")
    masks, vals = oracle.compress_2_4(rng(3).normal(0, 1, 16 * 32).astype(np.float32))
    L.write_spanda(p, meta, {"x": L.SpandaTensor("log4", q4, scales=s4),
                             "y": L.SpandaTensor("int8", q8.view(np.int8), scales=s8),
                             "z": L.SpandaTensor("dense", np.ones(3, np.float32)),
                             "s": L.SpandaTensor("sparse24", vals, shape=(16, 32), masks=masks),
                             "s1": L.SpandaTensor("sparse24", vals, shape=(512,), masks=masks)})
    plane = _FakePlane()
    _, out = L.register_spanda(plane, p)
    assert [(c[0], c[1], c[2], c[3]) for c in plane.calls] == [("m:x", "log4", 40, 64), ("m:y", "w8", 24, 32),
                                                              ("m:s", "sp24_f32", 16, 32)]
    assert np.array_equal(plane.calls[2][4], masks) and np.array_equal(plane.calls[2][5], vals)
    assert out["z"].kind == "dense" and out["s1"].kind == "sparse24"
    L.write_spanda(p, meta, {"x": L.SpandaTensor("log4", q4[:-1], scales=s4)})
    with pytest.raises(ValueError, match="do not split into 40 rows"):
        L.register_spanda(_FakePlane(), p)


# ---------------------------------------------------------------------- GPU
@pytest.fixture(scope="module")
def plane():
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from bramha_b200 import CudaComputePlane
    p = CudaComputePlane(0)
    yield p
    p.close()


@pytest.mark.gpu
def test_loaded_weights_compute_like_direct_registration(plane, tmp_path):
    """Manifest (W4ZP8, W8) and .spanda (LOG4, W8) weights at Qwen2-0.5B shapes:
    the GEMV of a loaded weight equals, bit for bit, the GEMV of the same bytes
    registered directly, and matches the oracle within the GEMV tolerance."""
    shapes = {"q": (896, 896), "gate": (4864, 896), "down": (896, 4864)}
    ws = {f"model.layers.0.{n}.weight": (fmt, *shapes[n], *make_weight(fmt, *shapes[n], seed=i)[1:])
          for i, (n, fmt) in enumerate([("q", "w4zp8"), ("gate", "w8"), ("down", "w4zp8")])}
    d = str(tmp_path / "m")
    L.write_manifest_dir(d, "ld", ws)
    loaded = L.register_manifest_dir(plane, d)
    sp = str(tmp_path / "m.spanda")
    meta = {k: 1 for k in L.META_FIELDS}
    meta.update(name="sp", architecture="qwen2")
    _, q4, s4 = make_weight("log4", 4864, 896, seed=11)
    _, q8, s8 = make_weight("w8", 896, 4864, seed=12)
    L.write_spanda(sp, meta, {"up": L.SpandaTensor("log4", q4, scales=s4),
                              "down8": L.SpandaTensor("int8", q8.view(np.int8), scales=s8)})
    _, sl = L.register_spanda(plane, sp)
    cases = [(loaded[k], v[0], v[3], v[4]) for k, v in ws.items()]
    cases += [(sl["up"], "log4", q4, s4), (sl["down8"], "w8", q8, s8)]
    for w, fmt, q, s in cases:
        x = make_x(1, w.K, seed=w.N)
        direct = plane.register(f"direct:{w.key}", fmt, w.N, w.K, q, s)
        y = plane.gemv(w, x)
        assert np.array_equal(y, plane.gemv(direct, x)), w.key
        ref = oracle.matvec_mul_into(fmt, x[0], q, s, w.N)
        assert normwise_err(y, ref) <= GEMV_TOL, w.key
        plane.evict(direct.key)
        plane.evict(w.key)
