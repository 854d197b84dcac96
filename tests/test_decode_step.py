"""Decode-step integration (PFlashDecoder): a two-layer Llama-style model
(tests/decode_model.py: INT4 group-128 packed linears, GQA 4/2 heads, RoPE,
SwiGLU) against golden logits from the reference's own
PFlashModelForCausalLM (tests/golden/make_decode_golden.py): a 20-token
prefill (tensor-core GEMM for the linears, causal mask) and three cached
single-token steps (streaming GEMV, CUDA-graph replays).

Tolerances: the fp32 restatement reproduces the reference's logits within
1e-5 (normwise); the GPU decoder within 1e-2 (its linears compute with fp16
x', 1e-3 per linear, compounded over two layers)."""
import os

import numpy as np
import pytest
import torch

import decode_model as dm

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "decode_step.npz")


def _rel(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.abs(a - b).max() / np.abs(b).max())


def test_restatement_matches_reference_logits():
    g = np.load(GOLD)
    w = dm.build()
    caches = [{} for _ in range(dm.CFG["num_hidden_layers"])]
    pre = dm.reference_forward(w, g["prompt"].tolist(), caches).numpy()
    assert _rel(pre, g["prefill_logits"]) < 1e-5
    for i, tok in enumerate(g["decode"].tolist()):
        lg = dm.reference_forward(w, [tok], caches)[-1].numpy()
        assert _rel(lg, g["step_logits"][i]) < 1e-5


def _decoder(w, max_seq=32):
    from polarflash_b200.decode import DecoderLayer, PFlashDecoder
    from polarflash_b200.hadamard import column_signs, effective_block
    from polarflash_b200.qweight import QWeight

    dev = torch.device("cuda")
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a, np.float32)).to(dev)  # noqa: E731
    layers = []
    for ly in w["layers"]:
        qw = {}
        for name, M, K in dm.LIN:
            p = ly[name]
            qw[name] = QWeight(1, M, K, torch.from_numpy(p["words"].view(np.uint8).reshape(-1).copy()).to(dev),
                               torch.from_numpy(p["s"].copy()).to(dev), torch.from_numpy(p["m"].copy()).to(dev),
                               effective_block(128, K), column_signs(K, 128, dev))
        layers.append(DecoderLayer(qw["q"], qw["k"], qw["v"], qw["o"], qw["gate"], qw["up"], qw["down"],
                                   t(ly["in_norm"]), t(ly["post_norm"])))
    return PFlashDecoder(dm.CFG, layers, t(w["embed"]), t(w["final_norm"]), t(w["lm_head"]), max_seq)


@pytest.mark.gpu
def test_prefill_and_graph_steps_match_reference():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    g = np.load(GOLD)
    dec = _decoder(dm.build())
    pre = dec.forward(torch.tensor(g["prompt"], device="cuda")).cpu().numpy()
    assert _rel(pre, g["prefill_logits"]) < 1e-2
    dec.capture()
    for i, tok in enumerate(g["decode"].tolist()):
        lg = dec.step(tok)[0].cpu().numpy()
        assert _rel(lg, g["step_logits"][i]) < 1e-2, f"step {i}"
    assert dec.length == len(g["prompt"]) + len(g["decode"])


@pytest.mark.gpu
def test_graph_steps_equal_eager_steps():
    """The captured step (attention over the whole cache under a mask, token
    and position from device tensors) agrees with eager single-token calls."""
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    g = np.load(GOLD)
    w = dm.build()
    a, b = _decoder(w), _decoder(w)
    prompt = torch.tensor(g["prompt"], device="cuda")
    a.forward(prompt)
    b.forward(prompt)
    b.capture()
    for tok in g["decode"].tolist():
        ea = a.forward(torch.tensor([tok], device="cuda"))[0]
        eb = b.step(tok)[0]
        assert _rel(eb.cpu().numpy(), ea.cpu().numpy()) < 1e-5
