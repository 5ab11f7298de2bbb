"""MoE layers loaded straight from GGUF files (cwx_bank_from_gguf + the architecture loaders in
coachwhip_b200/gguf.py) on the GPU: the banks hold the file's bytes (whole tensors and
expert-parallel slices), and a layer loaded from a file computes exactly what the same layer built
from the same bytes computes, within the oracle's bar (relative L2 1e-3)."""

from __future__ import annotations

import numpy as np
import pytest

import oracle as O
from tests.ep_common import run_emulated
from tests.gguf_files import write_layers
from tests.layers import Spec, build_cpu, build_gpu, make_input, rel_l2

torch = pytest.importorskip("torch")
gguf = pytest.importorskip("gguf")
pytestmark = pytest.mark.gpu

RTOL = 1e-3
CASES = {
    # arch, spec: the three loaders of the reference (qwen3moe, qwen3next with a shared expert,
    # gpt-oss with biases and clamped SwiGLU)
    "qwen3moe": ("qwen3moe", Spec(hidden=512, n_experts=16, top_k=4, inter=256, gate_type=O.IQ2_S,
                                  up_type=O.IQ2_S, down_type=O.IQ3_S, seed=21)),
    "qwen3next": ("qwen3next", Spec(hidden=512, n_experts=32, top_k=8, inter=256, gate_type=O.IQ3_S,
                                    up_type=O.IQ3_S, down_type=O.Q4_K, shared_inter=256, seed=22)),
    # the reference's own file family (Qwen3.6 UD-IQ2_M): qwen35moe, IQ2_XXS gate/up, IQ3_XXS
    # down, IQ4_XS shared expert
    "qwen35moe": ("qwen35moe", Spec(hidden=512, n_experts=32, top_k=8, inter=256, gate_type=O.IQ2_XXS,
                                    up_type=O.IQ2_XXS, down_type=O.IQ3_XXS, shared_inter=256,
                                    sh_types=(O.IQ4_XS, O.IQ4_XS, O.IQ4_XS), seed=24)),
    "gpt-oss": ("gpt-oss", Spec(hidden=576, n_experts=16, top_k=4, inter=576, gate_type=O.MXFP4, up_type=O.MXFP4,
                                down_type=O.MXFP4, act=O.ACT_CLAMPED_SWIGLU, router_bias=True, expert_bias=True,
                                seed=23)),
}


@pytest.fixture(scope="module")
def files(tmp_path_factory):
    out = {}
    d = tmp_path_factory.mktemp("gguf_gpu")
    for name, (arch, s) in CASES.items():
        layers = [build_cpu(Spec(**{**s.__dict__, "layer": li})) for li in range(2)]
        path = str(d / f"{name}.gguf")
        write_layers(path, layers, arch=arch, alignment=64 if name == "qwen3next" else None)
        out[name] = (path, layers)
    return out


def test_banks_hold_the_file_bytes(files):
    from coachwhip_b200.gguf import GgufFile

    path, layers = files["qwen3next"]
    f = GgufFile(path)
    for li, L in enumerate(layers):
        for m, key in (("gate", "gate_bank"), ("up", "up_bank"), ("down", "down_bank")):
            name = f"blk.{li}.ffn_{m}_exps.weight"
            want = np.ascontiguousarray(L[key], dtype=np.uint8)
            b = f.bank(name)
            assert np.array_equal(b.download(), want)
            bpe = b.bytes_per_expert
            s = f.bank(name, first=5, n_experts=3)  # an expert-parallel slice
            assert s.n_experts == 3 and np.array_equal(s.download(), want[5 * bpe:8 * bpe])
        sh = f.bank(f"blk.{li}.ffn_down_shexp.weight")
        assert sh.n_experts == 1 and np.array_equal(sh.download(), np.ascontiguousarray(L["sh_down"], dtype=np.uint8))


@pytest.mark.parametrize("name", list(CASES))
@pytest.mark.parametrize("T", [1, 37, 300])
def test_layer_from_file_matches_layer_from_bytes(files, name, T):
    from coachwhip_b200 import _lib
    from coachwhip_b200.gguf import GgufFile, expert_store, load_moe

    path, layers = files[name]
    f = GgufFile(path)
    store = expert_store(f)
    assert len(store.banks) == 2
    for li, L in enumerate(layers):
        x = make_input(CASES[name][1], T, seed=li + 40)
        xt = torch.from_numpy(x).cuda()[None]
        moe = load_moe(f, li, store)
        got = moe.forward(xt)[0].cpu().numpy()
        want = build_gpu(L).forward(xt)[0].cpu().numpy()
        _lib.status(0)
        assert np.array_equal(got, want)
        err = rel_l2(got, O.moe_forward(L, x, O.MODE_CANDLE)["out"])
        assert err < RTOL, err


def test_qwen3moe_norm_follows_shared_ffn_length(tmp_path):
    # model.rs: norm_topk_prob is on only when expert_shared_feed_forward_length is absent or 0
    from coachwhip_b200.gguf import GgufFile, layer_weights

    _, s = CASES["qwen3moe"]
    L = build_cpu(s)
    for ffn, want in ((None, True), (0, True), (512, False)):
        p = str(tmp_path / f"n{ffn}.gguf")
        write_layers(p, [L], arch="qwen3moe", shared_ffn=ffn)
        assert layer_weights(GgufFile(p), 0)["norm_topk_prob"] is want


def test_unsupported_architecture_is_refused(tmp_path):
    from coachwhip_b200.gguf import GgufFile, layer_weights

    _, s = CASES["qwen3moe"]
    p = str(tmp_path / "llama.gguf")
    write_layers(p, [build_cpu(s)], arch="llama")
    with pytest.raises(ValueError, match="architecture"):
        layer_weights(GgufFile(p), 0)


@pytest.mark.parametrize("name,world", [("qwen3next", 2), ("gpt-oss", 4)])
def test_expert_parallel_ranks_from_file(files, name, world):
    from coachwhip_b200.gguf import GgufFile, load_ep_engine

    path, layers = files[name]
    f = GgufFile(path)
    L = layers[1]
    x = make_input(CASES[name][1], 64, seed=7)
    out = run_emulated([load_ep_engine(f, 1, world, r) for r in range(world)], x)
    err = rel_l2(out, O.moe_forward(L, x, O.MODE_CANDLE)["out"])
    assert err < RTOL, err
