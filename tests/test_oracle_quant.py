"""Pin the C restatement of the Q8_0 / Q4_K formats (oracle/quant.c) against golden vectors made
by gguf-py (tests/golden/gen_golden.py), bit for bit."""
import os

import numpy as np

import oracle

GOLD = os.path.join(os.path.dirname(__file__), "golden")


def test_q8_0_quantize_matches_gguf_py_bytes():
    g = np.load(os.path.join(GOLD, "q8_0.npz"))
    raw = oracle.quantize(g["x"], "q8_0")
    assert raw.shape == g["raw"].shape
    assert np.array_equal(raw, g["raw"])


def test_q8_0_dequantize_bit_exact():
    g = np.load(os.path.join(GOLD, "q8_0.npz"))
    out, inn = g["x"].shape
    y = oracle.dequantize(g["raw"], "q8_0", out, inn)
    assert np.array_equal(y.view(np.uint32), g["deq"].view(np.uint32))


def test_q4_k_dequantize_bit_exact_random_blocks():
    g = np.load(os.path.join(GOLD, "q4_k.npz"))
    out = g["raw_rand"].shape[0]
    inn = g["raw_rand"].shape[1] // 144 * 256
    y = oracle.dequantize(g["raw_rand"], "q4_k", out, inn)
    assert np.array_equal(y.view(np.uint32), g["deq_rand"].view(np.uint32))


def test_q4_k_encoder_roundtrip_and_bit_exact_decode():
    g = np.load(os.path.join(GOLD, "q4_k.npz"))
    w = g["w"]
    raw = oracle.quantize(w, "q4_k")
    assert np.array_equal(raw, g["raw_enc"])
    y = oracle.dequantize(raw, "q4_k", *w.shape)
    assert np.array_equal(y.view(np.uint32), g["deq_enc"].view(np.uint32))
    # an encoder is only useful if it is accurate: 4-bit affine codes of N(0, 0.02)
    rel = np.linalg.norm(y - w) / np.linalg.norm(w)
    assert rel < 0.12, rel


def test_q8_0_edge_blocks():
    x = np.zeros((1, 64), np.float32)
    x[0, 32:] = -2.5
    raw = oracle.quantize(x, "q8_0")
    assert raw[0, :2].view(np.float16)[0] == 0        # zero block -> d = 0
    y = oracle.dequantize(raw, "q8_0", 1, 64)
    assert np.all(y[0, :32] == 0) and np.allclose(y[0, 32:], -2.5, rtol=1e-3)


def test_dora_magnitude_known_answer():
    # tests/train_lora_test.cpp:19-22,72: W = 1..32 as ggml [4, 8] (in = 4, out = 8);
    # dora-rows magnitude m[0] = |W[0, :]| = sqrt(1 + 4 + 9 + 16) = 5.477...
    w = np.arange(1, 33, dtype=np.float32).reshape(8, 4)
    nsq, nrm = oracle.row_norms(w)
    assert 5.47 < nrm[0] < 5.48
    assert np.isclose(nsq[0], 30.0 + 4 * 1e-12)


def test_package_encoder_q8_0_matches_gguf_py_bytes():
    import gguf_blocks
    g = np.load(os.path.join(GOLD, "q8_0.npz"))
    assert np.array_equal(gguf_blocks.q8_0(g["x"]), g["raw"])


def test_package_encoder_q4_k_is_a_valid_accurate_encoding():
    import gguf_blocks
    rng = np.random.default_rng(9)
    w = rng.normal(0, 0.02, (16, 1536)).astype(np.float32)
    raw = gguf_blocks.q4_k(w)
    y = oracle.dequantize(raw, "q4_k", *w.shape)
    assert np.linalg.norm(y - w) / np.linalg.norm(w) < 0.12
