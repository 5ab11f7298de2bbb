"""GGUF test files: synthetic MoE layers (tests/layers.py) written with ggml's own `gguf` package
writer, so the library's reader is checked against an independent implementation, and tiny
hand-assembled files for the format's corners (version 1 u32 lengths, 64-bit alignment keys)."""

from __future__ import annotations

import struct

import numpy as np

import oracle as O


def _gtype(fmt: int):
    from gguf.constants import GGMLQuantizationType as G

    return {O.Q4_K: G.Q4_K, O.Q6_K: G.Q6_K, O.Q8_0: G.Q8_0, O.MXFP4: G.MXFP4, O.IQ2_S: G.IQ2_S,
            O.IQ3_S: G.IQ3_S, O.IQ2_XXS: G.IQ2_XXS, O.IQ3_XXS: G.IQ3_XXS, O.IQ4_XS: G.IQ4_XS}[fmt]


def _quant(w, name: str, data: np.ndarray, fmt: int, e: int | None, n: int, k: int) -> None:
    rb = O.row_bytes(fmt, k)
    shape = (n, rb) if e is None else (e, n, rb)
    w.add_tensor(name, np.ascontiguousarray(data, dtype=np.uint8).reshape(shape), raw_dtype=_gtype(fmt))


def write_layers(path: str, layers: list[dict], arch: str = "qwen3moe", alignment: int | None = None,
                 shared_ffn: int | None = None, extra_meta: bool = False) -> None:
    """One GGUF with block_count = len(layers), each layer's tensors under blk.L (build_cpu dicts
    of one shape). Expert biases and router bias are written for gpt-oss."""
    import gguf

    w = gguf.GGUFWriter(path, arch)
    L0 = layers[0]
    w.add_block_count(len(layers))
    w.add_expert_used_count(L0["top_k"])
    w.add_uint32(f"{arch}.expert_count", L0["n_experts"])
    if shared_ffn is not None:
        w.add_uint32(f"{arch}.expert_shared_feed_forward_length", shared_ffn)
    if alignment is not None:
        w.add_custom_alignment(alignment)
    if extra_meta:  # every value type, nested arrays, a NUL-padded string
        w.add_int8("test.i8", -5)
        w.add_uint64("test.u64", 1 << 40)
        w.add_float32("test.f32", 0.25)
        w.add_bool("test.bool", True)
        w.add_string("test.nul", "padded\0\0")
        w.add_array("test.strings", ["a", "bc", ""])
        w.add_array("test.nested", [[1, 2], [3]])
        w.add_array("test.bools", [True, False, True])
    for li, L in enumerate(layers):
        p = f"blk.{li}"
        E, H, I = L["n_experts"], L["hidden"], L["inter"]
        w.add_tensor(f"{p}.ffn_gate_inp.weight", np.ascontiguousarray(L["router_w"], dtype=np.float32))
        _quant(w, f"{p}.ffn_gate_exps.weight", L["gate_bank"], L["gate_type"], E, I, H)
        _quant(w, f"{p}.ffn_up_exps.weight", L["up_bank"], L["up_type"], E, I, H)
        _quant(w, f"{p}.ffn_down_exps.weight", L["down_bank"], L["down_type"], E, H, I)
        if arch == "gpt-oss":
            w.add_tensor(f"{p}.ffn_gate_inp.bias", np.ascontiguousarray(L["router_b"], dtype=np.float32))
            for m in ("gate", "up", "down"):
                w.add_tensor(f"{p}.ffn_{m}_exps.bias", np.ascontiguousarray(L[f"{m}_b"], dtype=np.float32))
        if L.get("shared_inter"):
            Is = L["shared_inter"]
            w.add_tensor(f"{p}.ffn_gate_inp_shexp.weight", np.ascontiguousarray(L["sh_gate_inp"], dtype=np.float32))
            _quant(w, f"{p}.ffn_gate_shexp.weight", L["sh_gate"], L["sh_gate_type"], None, Is, H)
            _quant(w, f"{p}.ffn_up_shexp.weight", L["sh_up"], L["sh_up_type"], None, Is, H)
            _quant(w, f"{p}.ffn_down_shexp.weight", L["sh_down"], L["sh_down_type"], None, H, Is)
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()


def handmade(version: int, meta: list[tuple[str, int, bytes]], tensors: list[tuple[str, list[int], int, int]],
             data: bytes = b"", magic: bytes = b"GGUF", pad_to: int = 32) -> bytes:
    """GGUF bytes from parts: meta = (key, value type, encoded value), tensors = (name, ne
    innermost first, ggml type, offset); data follows the header padded to pad_to."""
    ln = (lambda n: struct.pack("<I", n)) if version == 1 else (lambda n: struct.pack("<Q", n))
    s = lambda t: ln(len(t)) + t.encode()  # noqa: E731
    b = magic + struct.pack("<I", version) + ln(len(tensors)) + ln(len(meta))
    for k, t, v in meta:
        b += s(k) + struct.pack("<I", t) + v
    for name, ne, t, off in tensors:
        b += s(name) + struct.pack("<I", len(ne))
        b += b"".join(struct.pack("<I" if version == 1 else "<Q", d) for d in ne)
        b += struct.pack("<IQ", t, off)
    b += b"\0" * ((-len(b)) % pad_to)
    return b + data
