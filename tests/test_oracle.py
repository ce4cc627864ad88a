"""The CPU oracle pinned against gguf-py goldens and its own known answers."""
import os

import numpy as np
import pytest

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def test_q8_0_quantize_matches_ggufpy_goldens(oracle):
    g = np.load(os.path.join(GOLD, "q8_0_ggufpy.npz"))
    for key in ("kat", "rnd", "wide"):
        got = oracle.quantize_q8_0(g[f"{key}_x"])
        assert got.shape == g[f"{key}_q"].shape
        assert np.array_equal(got, g[f"{key}_q"]), key


def test_q8_0_known_answers(oracle):
    g = np.load(os.path.join(GOLD, "q8_0_ggufpy.npz"))
    q = oracle.quantize_q8_0(g["kat_x"])
    d = q[:, :2].copy().view(np.float16).astype(np.float32).ravel()
    qs = q[:, 2:].view(np.int8)
    assert d[0] == 1.0 and (qs[0] == 127).all()
    assert d[1] == 0.0 and (qs[1] == 0).all()
    # round half away from zero (roundf), d = 1
    assert list(qs[2, :9]) == [127, 1, -1, 2, -2, 3, -3, 127, -127]
    assert 0 < d[3] < 6.1e-5  # f16 subnormal scale
    assert qs[4].min() == -127


def test_q8_0_against_live_ggufpy(oracle):
    gq = pytest.importorskip("gguf.quants")
    from gguf.constants import GGMLQuantizationType

    x = oracle.normal(7, (33, 320), 0.0, 0.5)
    assert np.array_equal(oracle.quantize_q8_0(x), gq.quantize(x, GGMLQuantizationType.Q8_0))
    deq = gq.dequantize(gq.quantize(x, GGMLQuantizationType.Q8_0), GGMLQuantizationType.Q8_0)
    assert np.array_equal(oracle.dequant_q8_0(oracle.quantize_q8_0(x), 33, 320), deq)


def test_dequant_transpose(oracle):
    x = oracle.normal(8, (40, 96), 0.0, 0.1)
    q = oracle.quantize_q8_0(x)
    assert np.array_equal(oracle.dequant_q8_0_t(q, 40, 96), oracle.dequant_q8_0(q, 40, 96).T)


def test_half_and_bf16_rounding(oracle):
    rng = np.random.default_rng(3)
    v = (rng.standard_normal(20000) * 10.0 ** rng.integers(-9, 6, 20000)).astype(np.float32)
    v = np.concatenate([v, np.array([65519, 65520, 65504, 2 ** -25, 2 ** -24, 2 ** -14, -0.0], np.float32)])
    with np.errstate(over="ignore"):
        ref = v.astype(np.float16).view(np.uint16)
    mine = np.array([oracle.f32_to_f16_bits(float(t)) for t in v], np.uint16)
    assert np.array_equal(mine, ref)
    # bf16 RNE: ties to even
    assert oracle.f32_to_bf16_bits(float(np.uint32(0x3F808000).view(np.float32))) == 0x3F80
    assert oracle.f32_to_bf16_bits(float(np.uint32(0x3F818000).view(np.float32))) == 0x3F82
    assert oracle.f32_to_bf16_bits(float(np.uint32(0x3F808001).view(np.float32))) == 0x3F81


def test_matmul_goldens_reproduce(oracle):
    g = np.load(os.path.join(GOLD, "matmul_small.npz"))
    tags = sorted({k.rsplit("_", 1)[0] for k in g.files})
    assert len(tags) == 6
    for tag in tags:
        x, q = g[f"{tag}_x"], g[f"{tag}_q"]
        n = g[f"{tag}_exact"].shape[1]
        assert np.array_equal(oracle.matmul_fbgemm_bf16(x, q, n), g[f"{tag}_fbgemm"]), tag
        assert np.array_equal(oracle.matmul_qtiled(x, q, n), g[f"{tag}_qtiled"]), tag
        assert np.allclose(oracle.matmul_exact(x, q, n), g[f"{tag}_exact"], rtol=1e-12, atol=1e-12), tag
        # the reference's two semantics agree with the exact product to bf16 / Q8 level
        assert oracle.max_rel_err(g[f"{tag}_fbgemm"], g[f"{tag}_exact"], 1.0) < 1.5e-2
        assert oracle.max_rel_err(g[f"{tag}_qtiled"], g[f"{tag}_exact"], 1.0) < 5e-2


def test_epilogues(oracle):
    y = np.array([[-2.0, 0.0, 1.0, 3.0]], np.float64)
    b = np.array([0.5, 0.0, 0.0, -1.0], np.float32)
    silu = oracle.epilogue(y, b, oracle.EPI_SILU)
    assert np.allclose(silu, (y + b) / (1 + np.exp(-(y + b))))
    glu = oracle.epilogue(y, None, oracle.EPI_GLU_SIGMOID)
    assert glu.shape == (1, 2)
    assert np.allclose(glu, y[:, :2] / (1 + np.exp(-y[:, 2:])))
    glus = oracle.epilogue(y, None, oracle.EPI_GLU_SILU)
    assert np.allclose(glus, y[:, :2] * y[:, 2:] / (1 + np.exp(-y[:, 2:])))
    import math
    gelu = oracle.epilogue(np.array([[1.0]]), None, oracle.EPI_GELU_ERF)
    assert abs(gelu[0, 0] - 0.5 * (1 + math.erf(1 / math.sqrt(2)))) < 1e-12


def test_rng_is_deterministic(oracle):
    a = oracle.normal(5, (1000,))
    b = oracle.normal(5, (1000,))
    assert np.array_equal(a, b)
    assert abs(float(a.mean())) < 0.1 and abs(float(a.std()) - 1) < 0.1
    u = oracle.uniform(6, (1000,), 2.0, 30.0)
    assert u.min() >= 2.0 and u.max() < 30.0
