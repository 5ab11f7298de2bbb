"""The native GGUF reader (cwx_gguf_*) on the CPU: against the plain-Python restatement of candle's
reader (oracle/gguf_file.py) and against ggml's own `gguf` package, on files that package writes
and on hand-assembled corners of the format; truncated and corrupted headers fail the same way on
both sides. No GPU: these calls only read the mapped file."""

from __future__ import annotations

import ctypes
import struct

import numpy as np
import pytest

import oracle as O
from oracle import gguf_file as OG
from tests.gguf_files import handmade, write_layers
from tests.layers import Spec, build_cpu

gguf = pytest.importorskip("gguf")

SPEC = Spec(hidden=512, n_experts=8, top_k=2, inter=256, gate_type=O.IQ2_S, up_type=O.Q4_K, down_type=O.IQ3_S,
            shared_inter=256, sh_types=(O.Q8_0, O.Q6_K, O.MXFP4), seed=3)


@pytest.fixture(scope="module")
def lib():
    from coachwhip_b200 import _lib

    return _lib.lib()


@pytest.fixture(scope="module")
def layer_file(tmp_path_factory):
    L = build_cpu(SPEC)
    L2 = build_cpu(Spec(**{**SPEC.__dict__, "layer": 1}))
    path = str(tmp_path_factory.mktemp("gguf") / "layers.gguf")
    write_layers(path, [L, L2], arch="qwen3next", extra_meta=True)
    return path, [L, L2]


def _open(path):
    from coachwhip_b200.gguf import GgufFile

    return GgufFile(path)


def test_tensor_infos_match_oracle_and_gguf_package(layer_file):
    path, _ = layer_file
    data = open(path, "rb").read()
    ref = OG.read(data)
    pkg = gguf.GGUFReader(path)
    f = _open(path)
    assert (f.version, f.alignment, f.data_offset, f.n_tensors) == (ref["version"], ref["alignment"],
                                                                     ref["data_offset"], len(ref["tensors"]))
    assert f.n_tensors == len(pkg.tensors)
    for t in pkg.tensors:
        ne, gt, off = ref["tensors"][t.name]
        assert list(t.shape) == ne and int(t.tensor_type) == gt
        assert ref["data_offset"] + off == t.data_offset
        assert f.tensor_info(t.name) == (gt, tuple(ne), t.data_offset)


def test_expert_descriptors_point_at_the_tensor_bytes(layer_file):
    path, layers = layer_file
    data = open(path, "rb").read()
    pkg = {t.name: t for t in gguf.GGUFReader(path).tensors}
    f = _open(path)
    for li, L in enumerate(layers):
        E, H, I = L["n_experts"], L["hidden"], L["inter"]
        for m, key, n, k, e in (("gate", "gate_bank", I, H, E), ("up", "up_bank", I, H, E),
                                ("down", "down_bank", H, I, E), ("gate_shexp", "sh_gate", I, H, None)):
            name = f"blk.{li}.ffn_{m}{'' if m.endswith('shexp') else '_exps'}.weight"
            d = f.matrix(name)
            assert (d.n, d.k, d.n_experts) == (n, k, e or 1)
            got = ctypes.string_at(d.host_ptr, d.n_experts * d.bytes_per_expert)
            assert got == np.ascontiguousarray(L[key], dtype=np.uint8).tobytes()
            off = pkg[name].data_offset
            assert got == data[off:off + len(got)]


def test_dense_tensors_and_metadata(layer_file):
    path, layers = layer_file
    f = _open(path)
    assert f.architecture == "qwen3next"
    assert f.meta_int("qwen3next.block_count") == 2
    assert f.meta_int("qwen3next.expert_used_count") == SPEC.top_k
    assert f.meta_int("test.i8") == -5 and f.meta_int("test.u64") == 1 << 40
    assert f.meta_float("test.f32") == 0.25
    assert f.meta_str("test.nul") == "padded"  # trailing NULs dropped, as candle does
    assert f.meta_int("missing.key", 7) == 7
    with pytest.raises(Exception):
        f.meta_int("general.architecture")  # a string, not an integer
    for li, L in enumerate(layers):
        assert np.array_equal(f.dense(f"blk.{li}.ffn_gate_inp.weight"), L["router_w"])
        assert np.array_equal(f.dense(f"blk.{li}.ffn_gate_inp_shexp.weight").reshape(-1), L["sh_gate_inp"])
    ref = OG.read(open(path, "rb").read())["metadata"]
    assert ref["test.strings"][1] == ["a", "bc", ""] and ref["test.nested"][1] == [[1, 2], [3]]


def test_f16_and_bf16_tensors_read_as_f32(tmp_path, lib):
    from gguf.constants import GGMLQuantizationType as G

    rng = np.random.default_rng(0)
    x = rng.standard_normal(96).astype(np.float32)
    x[:4] = [0.0, -0.0, 6e-8, 65504.0]  # zero signs, an f16 subnormal, the f16 maximum
    h = x.astype(np.float16)
    bf = (x.view(np.uint32) >> 16).astype(np.uint16)
    w = gguf.GGUFWriter(str(tmp_path / "d.gguf"), "qwen3moe")
    w.add_tensor("h", h.reshape(4, 24))
    w.add_tensor("b", bf.reshape(4, 24), raw_dtype=G.BF16)
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    f = _open(str(tmp_path / "d.gguf"))
    assert np.array_equal(f.dense("h").view(np.uint32), h.astype(np.float32).view(np.uint32).reshape(4, 24))
    want = (bf.astype(np.uint32) << 16).view(np.float32).reshape(4, 24)
    assert np.array_equal(f.dense("b").view(np.uint32), want.view(np.uint32))
    with pytest.raises(Exception):
        f.matrix("h")  # not an expert format


@pytest.mark.parametrize("version", [1, 2, 3])
def test_handmade_versions_and_alignment_rules(tmp_path, version):
    # alignment 64 as a u32 is taken; as a u64 it is ignored (candle reads 8/16/32-bit keys only)
    for atype, enc, want in ((4, struct.pack("<I", 64), 64), (10, struct.pack("<Q", 64), 32),
                             (5, struct.pack("<i", -64), 32), (2, struct.pack("<H", 16), 16)):
        rb = O.row_bytes(O.Q8_0, 64)
        data = bytes(range(256)) * 2
        b = handmade(version, [("general.alignment", atype, enc), ("general.architecture", 8,
                                                                    struct.pack("<Q" if version > 1 else "<I", 3) + b"foo")],
                     [("blk.0.ffn_up_exps.weight", [64, 2, 2], O.Q8_0, 0)], data[:4 * rb], pad_to=want)
        p = str(tmp_path / f"v{version}_{atype}.gguf")
        open(p, "wb").write(b)
        ref = OG.read(b)
        f = _open(p)
        assert f.alignment == ref["alignment"] == want
        assert f.data_offset == ref["data_offset"] == len(b) - 4 * rb
        assert f.meta_str("general.architecture") == "foo"
        d = f.matrix("blk.0.ffn_up_exps.weight")
        assert (d.n_experts, d.n, d.k, d.bytes_per_expert) == (2, 2, 64, 2 * rb)
        assert ctypes.string_at(d.host_ptr, 4 * rb) == data[:4 * rb]


def test_swapped_magic_is_accepted(tmp_path):
    b = handmade(3, [], [], magic=b"FUGG")
    p = str(tmp_path / "m.gguf")
    open(p, "wb").write(b)
    assert _open(p).n_tensors == 0 and OG.read(b)["tensors"] == {}


def _opens(path) -> bool:
    from coachwhip_b200 import _lib

    h = ctypes.c_void_p()
    rc = _lib.lib().cwx_gguf_open(path.encode(), ctypes.byref(h))
    if rc == _lib.OK:
        _lib.lib().cwx_gguf_close(h)
    return rc == _lib.OK


def _oracle_opens(b: bytes) -> bool:
    try:
        OG.read(b)
        return True
    except (OG.GgufError, struct.error):
        return False


def test_truncated_and_corrupted_headers(tmp_path, layer_file):
    from coachwhip_b200 import _lib

    path, _ = layer_file
    full = open(path, "rb").read()
    head = OG.read(full)["data_offset"]
    p = str(tmp_path / "cut.gguf")
    for cut in sorted(set(list(range(0, 64)) + list(range(64, head + 8, 37)) + [head - 1, head])):
        open(p, "wb").write(full[:cut])
        assert _opens(p) == _oracle_opens(full[:cut]), cut
    # a file cut inside the tensor data opens, but the tensors past the end are refused
    open(p, "wb").write(full[:head + 100])
    f = _open(p)
    with pytest.raises(_lib.CwxError, match="outside the file"):
        f.matrix("blk.1.ffn_down_exps.weight")
    rng = np.random.default_rng(5)
    for i in range(300):  # single-byte corruptions of the header agree with the oracle
        b = bytearray(full[:head + 64])
        at = int(rng.integers(0, head))
        b[at] = int(rng.integers(0, 256))
        open(p, "wb").write(bytes(b))
        assert _opens(p) == _oracle_opens(bytes(b)), (i, at)
    for bad in (b"GGUX" + full[4:], full[:4] + struct.pack("<I", 4) + full[8:], b""):
        open(p, "wb").write(bad)
        with pytest.raises(_lib.CwxError):
            _open(p)


def test_missing_tensor_and_slice_errors(layer_file, lib):
    from coachwhip_b200 import _lib

    path, _ = layer_file
    f = _open(path)
    assert not f.has("blk.9.ffn_up_exps.weight") and f.has("blk.1.ffn_up_exps.weight")
    with pytest.raises(_lib.CwxError, match="no tensor named"):
        f.matrix("blk.9.ffn_up_exps.weight")
    h = ctypes.c_void_p()
    for first, n in ((-1, 2), (7, 2), (0, 0), (8, -1)):
        rc = lib.cwx_bank_from_gguf(0, f.handle, b"blk.0.ffn_up_exps.weight", first, n, ctypes.byref(h))
        assert rc == _lib.EINVAL, (first, n)
