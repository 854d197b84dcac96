"""Recursive polar with learned angle codebooks against the reference's own
outputs (tests/golden/polar_codebooks.npz, made by
make_polar_codebook_golden.py from RecursivePolarQuant.fit_codebooks,
encode_packed and decode_packed, polar_quant.py:274-300, 381-575).

CPU: the mirror's Lloyd-Max codebooks and packed bytes equal the reference's
bit for bit (including codebook indices wider than their 1-3 bit fields,
which the reference ORs in unmasked), and the oracle's codebook decode
agrees with decode_packed (1e-6 absolute: libm vs torch cos / sin).  GPU:
decode_packed on the device, and the packed linear at batch 1 (table GEMV,
block 8, 1.75 bpw) and batch 3 (CUDA-core kernel) with learned codebooks,
within the parity suite's 1e-3 of the oracle.
"""
import json
import os

import numpy as np
import pytest
import torch

import oracle

HERE = os.path.dirname(os.path.abspath(__file__))
G = np.load(os.path.join(HERE, "golden", "polar_codebooks.npz"))
with open(os.path.join(HERE, "golden", "polar_codebooks_meta.json")) as f:
    META = json.load(f)
CASES = sorted(META)


def _books(name):
    return [G[f"{name}_cb{lvl}"] for lvl in range(META[name]["levels"])]


def _fitted(name):
    from polarflash_b200.polar import RecursivePolarQuant

    m = META[name]
    rpq = RecursivePolarQuant(block_size=m["block_size"], norm_bits=4, angle_bits=m["angle_bits"])
    rpq.fit_codebooks(torch.from_numpy(G[f"{name}_train"]), iters=m["iters"])
    return rpq


@pytest.mark.parametrize("name", CASES)
def test_codebooks_match_reference(name):
    rpq = _fitted(name)
    assert len(rpq.learned_codebooks) == META[name]["levels"]
    for cb, ref in zip(rpq.learned_codebooks, _books(name)):
        assert cb.numel() == 2 ** META[name]["angle_bits"]
        assert torch.all(cb[1:] >= cb[:-1])
        np.testing.assert_array_equal(cb.numpy(), ref)


@pytest.mark.parametrize("name", CASES)
def test_payload_matches_reference(name):
    rpq = _fitted(name)
    m = META[name]
    packed, meta = rpq.encode_packed(torch.from_numpy(G[f"{name}_test"]), target_bpw=m["bpw"])
    assert packed == G[f"{name}_payload"].tobytes()
    assert meta["has_learned_codebooks"] is True
    for k in ("alloc", "num_blocks", "pad_len", "orig_shape"):
        assert meta[k] == m[k], k
    assert meta["r_scale"] == m["r_scale"]


@pytest.mark.parametrize("name", CASES)
def test_oracle_decode_matches_reference(name):
    m = META[name]
    out = oracle.polar_decode(G[f"{name}_payload"].tobytes(), m["num_blocks"], m["block_size"], m["alloc"],
                              m["r_scale"], _books(name))
    ref = G[f"{name}_recon"].reshape(-1)
    np.testing.assert_allclose(out[:ref.size], ref, rtol=0, atol=1e-6)
    # the same payload decoded without the codebooks differs: the codebooks are in effect
    plain = oracle.polar_decode(G[f"{name}_payload"].tobytes(), m["num_blocks"], m["block_size"], m["alloc"],
                                m["r_scale"])
    assert np.max(np.abs(plain[:ref.size] - ref)) > 1e-3


def test_angle_table_layout():
    from polarflash_b200.encoders import polar_angle_table

    books = [np.linspace(-3, 3, 16, dtype=np.float32), np.linspace(0.1, 1.5, 4, dtype=np.float32)]
    alloc = [3, 2, 2, 2, 2, 1, 1, 1]
    tab = polar_angle_table(8, alloc, books).view(7, 64).numpy()
    for j in range(4):  # level 0 columns: codebook 0
        np.testing.assert_array_equal(tab[j, :4], books[0][:4])
    for j in (4, 5):  # level 1: codebook 1 (2 entries reachable with 1 bit)
        np.testing.assert_array_equal(tab[j, :2], books[1][:2])
    # level 2 has no codebook: the uniform grid (c + 0.5) / 2 * pi / 2
    np.testing.assert_allclose(tab[6, :2], [(0.5 / 2) * np.pi / 2, (1.5 / 2) * np.pi / 2], rtol=1e-6)
    short = polar_angle_table(8, [3, 3, 3, 3, 3, 1, 1, 1], [np.array([0.5, 1.0], np.float32)]).view(7, 64).numpy()
    np.testing.assert_array_equal(short[0, :8], [0.5] + [1.0] * 7)  # clamp to the last entry


@pytest.mark.gpu
@pytest.mark.parametrize("name", CASES)
def test_device_decode_packed(name):
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    rpq = _fitted(name)
    m = META[name]
    meta = {k: m[k] for k in ("alloc", "num_blocks", "pad_len", "orig_shape", "r_scale", "has_learned_codebooks")}
    meta["block_size"] = m["block_size"]
    out = rpq.decode_packed(G[f"{name}_payload"].tobytes(), meta).cpu().numpy()
    np.testing.assert_allclose(out, G[f"{name}_recon"], rtol=0, atol=1e-6)


@pytest.mark.gpu
@pytest.mark.parametrize("N", [1, 3])
def test_linear_with_learned_codebooks(N):
    """512 x 2048 weight (RWHT-128) encoded at 1.75 bpw with the d8_b4
    codebooks: batch 1 runs the table GEMV, batch 3 the CUDA-core kernel."""
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from test_gpu_parity import _w, _x, assert_rel

    from polarflash_b200 import encoders, qlinear
    from polarflash_b200.quantizer import rwht_cpu
    from polarflash_b200.qweight import qweight_from_payload

    M, K = 512, 2048
    Wr = rwht_cpu(_w(M, K, 91), 128)
    payload, meta = encoders.polar_encode(Wr, 8, 1.75, codebooks=_books("d8_b4"))
    meta.update(hadamard_rotation=True, hadamard_block_size=128)
    qw = qweight_from_payload("polar_recursive", meta, payload, M, K, "cuda")
    assert qw.scales is not None
    x = _x(N, K, 92)
    y = qlinear(qw, x.cuda()).cpu().numpy()
    assert_rel(y, oracle.linear("polar_recursive", payload.numpy().tobytes(), M, K, meta, x.float().numpy()))
