"""MoE layers straight from a GGUF model file, through libcwx.so's native reader.

Mirrors the reference's loaders for the hot path's inputs:
  ExpertStore::new (crates/engine/src/experts.rs:697-717): every layer's
      blk.L.ffn_{gate,up,down}_exps.weight, (E, n, k), resident in HBM;
  Qwen3Moe::load (crates/engine/src/model.rs:139-175): router ffn_gate_inp.weight, top_k =
      <arch>.expert_used_count, norm_topk_prob when <arch>.expert_shared_feed_forward_length is
      absent or 0, SiLU experts;
  Qwen3Next::load (crates/engine/src/model_next.rs:1036-1053): the same plus the shared expert
      ffn_{gate,up,down}_shexp.weight gated by ffn_gate_inp_shexp.weight, norm_topk_prob on;
  GptOss::load (crates/engine/src/model_gptoss.rs:115-181): router bias ffn_gate_inp.bias,
      clamped SwiGLU (alpha 1.702, limit 7.0) with the expert biases ffn_{gate,up,down}_exps.bias,
      norm_topk_prob on.
Dense tensors (F32/F16/BF16) are read to f32 on the host and copied to the device once; expert
tensors go from the mapped file to HBM without a host copy. An expert-parallel rank loads its
slice of experts (first, n_experts).
"""

from __future__ import annotations

import ctypes

import numpy as np
import torch

from . import _lib
from ._lib import check
from .moe import Bank, ExpertAct, ExpertStore, SharedExpert, StreamedMoe

SWIGLU_ALPHA, SWIGLU_LIMIT = 1.702, 7.0
ARCHS = ("qwen3moe", "qwen3next", "qwen35moe", "gpt-oss")


class GgufFile:
    """An open GGUF file (cwx_gguf): metadata, tensor infos, dense tensors and expert banks."""

    def __init__(self, path: str):
        h = ctypes.c_void_p()
        check(_lib.lib().cwx_gguf_open(str(path).encode(), ctypes.byref(h)))
        self.handle, self.path = h, str(path)
        v, n, a, d = ctypes.c_int32(), ctypes.c_int64(), ctypes.c_int64(), ctypes.c_int64()
        check(_lib.lib().cwx_gguf_info(h, ctypes.byref(v), ctypes.byref(n), ctypes.byref(a), ctypes.byref(d)))
        self.version, self.n_tensors, self.alignment, self.data_offset = v.value, n.value, a.value, d.value

    def close(self) -> None:
        if self.handle:
            _lib.lib().cwx_gguf_close(self.handle)
            self.handle = None

    def __enter__(self) -> "GgufFile":
        return self

    def __exit__(self, *exc) -> None:
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def has(self, name: str) -> bool:
        return _lib.lib().cwx_gguf_tensor_info(self.handle, name.encode(), None, None, None, None) == _lib.OK

    def tensor_info(self, name: str) -> tuple[int, tuple[int, ...], int]:
        """(ggml type, ne innermost first, file offset of the data)."""
        t, nd, off = ctypes.c_int32(), ctypes.c_int32(), ctypes.c_int64()
        ne = (ctypes.c_int64 * 4)()
        check(_lib.lib().cwx_gguf_tensor_info(self.handle, name.encode(), ctypes.byref(t), ctypes.byref(nd), ne,
                                              ctypes.byref(off)))
        return t.value, tuple(ne[i] for i in range(nd.value)), off.value

    def matrix(self, name: str) -> _lib.MatrixDesc:
        d = _lib.MatrixDesc()
        check(_lib.lib().cwx_gguf_tensor(self.handle, name.encode(), ctypes.byref(d)))
        return d

    def dense(self, name: str) -> np.ndarray:
        """An F32/F16/BF16 tensor as f32, shaped outermost first."""
        _, ne, _ = self.tensor_info(name)
        out = np.empty(int(np.prod(ne)) if ne else 1, dtype=np.float32)
        check(_lib.lib().cwx_gguf_tensor_f32(self.handle, name.encode(), out.ctypes.data, out.size))
        return out.reshape(tuple(reversed(ne)))

    def bank(self, name: str, device: int = 0, first: int = 0, n_experts: int | None = None) -> Bank:
        """Experts [first, first + n_experts) of an expert tensor resident in HBM."""
        d = self.matrix(name)
        ne = d.n_experts - first if n_experts is None else n_experts
        h = ctypes.c_void_p()
        check(_lib.lib().cwx_bank_from_gguf(device, self.handle, name.encode(), first, ne, ctypes.byref(h)))
        return Bank(h, d.ggml_type, d.n, d.k, ne, device)

    def meta_int(self, key: str, default: int | None = None) -> int:
        v = ctypes.c_int64()
        rc = _lib.lib().cwx_gguf_meta_int(self.handle, key.encode(), ctypes.byref(v))
        if rc != _lib.OK and default is not None:
            return default
        check(rc)
        return v.value

    def meta_float(self, key: str, default: float | None = None) -> float:
        v = ctypes.c_double()
        rc = _lib.lib().cwx_gguf_meta_f64(self.handle, key.encode(), ctypes.byref(v))
        if rc != _lib.OK and default is not None:
            return default
        check(rc)
        return v.value

    def meta_str(self, key: str, default: str | None = None) -> str:
        n = ctypes.c_int64()
        rc = _lib.lib().cwx_gguf_meta_str(self.handle, key.encode(), None, 0, ctypes.byref(n))
        if rc != _lib.OK and default is not None:
            return default
        check(rc)
        buf = ctypes.create_string_buffer(n.value + 1)
        check(_lib.lib().cwx_gguf_meta_str(self.handle, key.encode(), buf, n.value + 1, None))
        return buf.raw[:n.value].decode("utf-8", errors="replace")

    @property
    def architecture(self) -> str:
        return self.meta_str("general.architecture")


def expert_store(f: GgufFile, layers: int | None = None, device: int = 0, first: int = 0,
                 n_experts: int | None = None) -> ExpertStore:
    """Every layer's (gate, up, down) expert banks in HBM (ExpertStore::new, all resident);
    layers defaults to <arch>.block_count."""
    if layers is None:
        layers = f.meta_int(f"{f.architecture}.block_count")
    banks = []
    for layer in range(layers):
        banks.append(tuple(f.bank(f"blk.{layer}.ffn_{m}_exps.weight", device, first, n_experts)
                           for m in ("gate", "up", "down")))
    return ExpertStore(banks)


def _dev(a: np.ndarray, device: int) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(f"cuda:{device}")


def layer_weights(f: GgufFile, layer: int, device: int = 0, first: int = 0, n_experts: int | None = None) -> dict:
    """The dense inputs of one MoE layer and its activation, per the file's architecture:
    {arch, top_k, norm_topk_prob, gate, gate_bias, act, shared} (device tensors and banks).
    first / n_experts pick the expert rows of per-expert biases (an expert-parallel rank's)."""
    arch = f.architecture
    if arch not in ARCHS:
        raise ValueError(f"this model's architecture is {arch!r}, which has no MoE loader here "
                         f"(supported: {', '.join(ARCHS)})")
    p = f"blk.{layer}"
    top_k = f.meta_int(f"{arch}.expert_used_count")
    gate = _dev(f.dense(f"{p}.ffn_gate_inp.weight"), device)
    gate_bias, shared, act = None, None, ExpertAct.Silu()
    if arch == "qwen3moe":
        norm = f.meta_int(f"{arch}.expert_shared_feed_forward_length", 0) == 0
    else:
        norm = True
    if arch in ("qwen3next", "qwen35moe"):
        shared = SharedExpert(_dev(f.dense(f"{p}.ffn_gate_inp_shexp.weight").reshape(-1), device),
                              f.bank(f"{p}.ffn_gate_shexp.weight", device),
                              f.bank(f"{p}.ffn_up_shexp.weight", device),
                              f.bank(f"{p}.ffn_down_shexp.weight", device))
    if arch == "gpt-oss":
        gate_bias = _dev(f.dense(f"{p}.ffn_gate_inp.bias").reshape(-1), device)
        e = gate.shape[0]
        sl = slice(first, e if n_experts is None else first + n_experts)
        act = ExpertAct.ClampedSwiglu(SWIGLU_ALPHA, SWIGLU_LIMIT,
                                      *(_dev(f.dense(f"{p}.ffn_{m}_exps.bias").reshape(e, -1)[sl], device)
                                        for m in ("gate", "up", "down")))
    return dict(arch=arch, top_k=top_k, norm_topk_prob=norm, gate=gate, gate_bias=gate_bias, act=act,
                shared=shared)


def load_moe(f: GgufFile, layer: int, store: ExpertStore, device: int = 0,
             act_mode: int = _lib.ACT_MODE_CANDLE) -> StreamedMoe:
    """StreamedMoe of `layer` over `store` (expert_store of the same file) with the file's router,
    activation and shared expert."""
    w = layer_weights(f, layer, device)
    moe = StreamedMoe(layer, w["gate"], w["top_k"], w["norm_topk_prob"], w["act"], store, gate_bias=w["gate_bias"],
                      shared=w["shared"], act_mode=act_mode)
    moe._keep = (w["act"], w["shared"], w["gate_bias"])
    return moe


def load_ep_engine(f: GgufFile, layer: int, world: int, rank: int, device: int = 0,
                   act_mode: int = _lib.ACT_MODE_CANDLE):
    """This rank's expert-parallel engine of `layer`: its slice of the experts and their biases,
    the full router and the shared expert."""
    from .ep import CudaEngine

    e = f.matrix(f"blk.{layer}.ffn_gate_exps.weight").n_experts
    if e % world:
        raise ValueError(f"{e} experts do not split over {world} ranks")
    epr = e // world
    banks = tuple(f.bank(f"blk.{layer}.ffn_{m}_exps.weight", device, rank * epr, epr) for m in ("gate", "up", "down"))
    w = layer_weights(f, layer, device, rank * epr, epr)
    eng = CudaEngine(w["gate"], w["top_k"], w["norm_topk_prob"], w["act"], banks, world, rank,
                     gate_bias=w["gate_bias"], shared=w["shared"], act_mode=act_mode)
    eng._keep = (w["act"], w["shared"], w["gate_bias"])
    return eng


__all__ = ["GgufFile", "expert_store", "layer_weights", "load_moe", "load_ep_engine", "ARCHS"]
