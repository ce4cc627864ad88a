"""The CPU oracle against third-party implementations of the same arithmetic.

The reference (Rust, candle, fbgemm-rs) cannot be built here, and its tests hold
no numeric goldens.  These tests pin each piece of the oracle that an
independent implementation in this image can check:

* the whole FastConformer encoder (oracle/encoder_oracle.c, restating
  src/parakeet/fast_conformer.rs:69-1104) against transformers 5.5.0's
  ParakeetEncoder, a separate port of the same NeMo model, in float64 on the
  same seeded Q8_0 weights (stored outputs in tests/golden/
  encoder_hf_parakeet.npz, from tests/golden/make_hf_parakeet_golden.py, and a
  live run when transformers is importable);
* the bf16 packing of MatMul::from_tensor (src/fast_matmul.rs:191-208) against
  torch's float32 -> bfloat16 cast, bit for bit;
* the FbgemmBf16Op product (src/fast_matmul.rs:138-167) against torch's CPU
  matmul of the same bf16-rounded weights, which differs from the oracle only
  in summation order;
* the packed CPU-baseline kernels (oracle/fbgemm_cpu.c) against the scalar
  oracle, bit for bit on both instruction sets.
"""
import os
import sys

import numpy as np
import pytest

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
sys.path.insert(0, GOLD)

import make_hf_parakeet_golden as G  # noqa: E402


def _case(name):
    for c in G.CASES:
        if c[0] == name:
            return c
    raise KeyError(name)


@pytest.mark.parametrize("name", [c[0] for c in G.CASES])
def test_encoder_oracle_matches_hf_parakeet(oracle, name):
    from nspeech_b200 import synthetic as S
    _, kw, wseed, frames, mseed = _case(name)
    spec = S.EncoderSpec(**kw)
    g = np.load(os.path.join(GOLD, "encoder_hf_parakeet.npz"))
    ref = g[f"{name}_hf"].astype(np.float64)
    _, blocks = G.dequantized_tensors(spec, wseed)
    mel = oracle.normal(mseed, (frames, spec.feat_in))
    # exact dequantized weights: the same model, summation order aside
    y = oracle.encoder_forward(spec.as_dict(), blocks, mel, weight_mode=1)
    assert y.shape == ref.shape
    err = oracle.max_rel_err(y, ref, 1.0)
    assert err < 2e-5, err
    assert (y.argmax(1) == ref.argmax(1)).all()
    # fast_matmul semantics (bf16-packed weights): the bf16 rounding of the
    # weights is the whole difference
    yb = oracle.encoder_forward(spec.as_dict(), blocks, mel, weight_mode=0)
    err_b = oracle.max_rel_err(yb, ref, 1.0)
    assert 1e-4 < err_b < 5e-2, err_b


def test_hf_parakeet_golden_reproduces(oracle):
    """The stored outputs come from the committed generator (live run)."""
    pytest.importorskip("transformers.models.parakeet.modeling_parakeet")
    from nspeech_b200 import synthetic as S
    name, kw, wseed, frames, mseed = G.CASES[1]
    spec = S.EncoderSpec(**kw)
    y = G.hf_forward(spec, wseed, oracle.normal(mseed, (frames, spec.feat_in)))
    g = np.load(os.path.join(GOLD, "encoder_hf_parakeet.npz"))
    np.testing.assert_allclose(y.astype(np.float32), g[f"{name}_hf"], rtol=1e-6, atol=1e-6)


def test_bf16_packing_matches_torch_cast(oracle):
    torch = pytest.importorskip("torch")
    rng = np.random.default_rng(11)
    v = (rng.standard_normal(50000) * 10.0 ** rng.integers(-40, 38, 50000)).astype(np.float32)
    ties = np.array([0x3F808000, 0x3F818000, 0x3F808001, 0x00008000, 0x7F7FFFFF, 0x00000001, 0x80018000],
                    np.uint32).view(np.float32)
    v = np.concatenate([v, ties, np.array([0.0, -0.0, np.inf, -np.inf], np.float32)])
    ref = torch.from_numpy(v).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    mine = oracle.pack_bf16(v)
    assert np.array_equal(mine, ref)


@pytest.mark.parametrize("m,n,k", [(1, 640, 640), (125, 1024, 1024), (200, 768, 2048), (17, 130, 4096)])
def test_fbgemm_semantics_match_torch_matmul(oracle, m, n, k):
    """f32 x times bf16-rounded dequantized W: the oracle and torch's CPU matmul
    (another summation order) agree to summation-order rounding."""
    torch = pytest.importorskip("torch")
    x = oracle.normal(40 + m, (m, k))
    q = oracle.quantize_q8_0(oracle.normal(41 + n, (n, k), 0.0, 0.02))
    wb = torch.from_numpy(oracle.dequant_q8_0(q, n, k)).to(torch.bfloat16)
    ref64 = (torch.from_numpy(x).double() @ wb.double().T).numpy()
    ref32 = (torch.from_numpy(x) @ wb.float().T).numpy()
    got = oracle.matmul_fbgemm_bf16(x, q, n)
    # k-sequential f32 rounding (the oracle) vs blocked f32 (torch): both within
    # 1e-5 of the f64 product, row-rms normalised
    assert oracle.max_rel_err(got, ref64, 1.0) < 1e-5
    assert oracle.max_rel_err(ref32, ref64, 1.0) < 1e-5


@pytest.mark.parametrize("m,n,k", [(1, 64, 64), (5, 130, 96), (49, 37, 32), (125, 1024, 1024), (7, 1000, 4096)])
def test_packed_cpu_kernels_bit_identical(oracle, m, n, k):
    x = oracle.normal(1 + m, (m, k))
    q = oracle.quantize_q8_0(oracle.normal(2 + n, (n, k), 0.0, 0.02))
    ref = oracle.matmul_fbgemm_bf16(x, q, n)
    isa = oracle.cpu_isa()
    try:
        for forced in (512, 256):
            oracle.force_isa(forced)
            assert np.array_equal(oracle.matmul_fbgemm_packed(x, q, n), ref), forced
    finally:
        oracle.force_isa(isa)
    exact = oracle.matmul_exact(x, q, n)
    assert oracle.max_rel_err(oracle.matmul_fbgemm_packed(x, q, n, bf16=False), exact, 1.0) < 1e-5


@pytest.mark.parametrize("cin,cout,k,stride,pad,dil,leaky", [(128, 128, 3, 1, 1, 1, 1.0), (64, 64, 11, 1, 25, 5, 0.1),
                                                            (128, 22, 7, 1, 3, 1, 0.01), (1, 1, 3, 2, 1, 1, 1.0),
                                                            (512, 64, 1, 1, 0, 1, 1.0)])
def test_conv1d_oracle_matches_torch(oracle, cin, cout, k, stride, pad, dil, leaky):
    """The Kokoro conv1d restatement against torch.nn.functional.conv1d (f64)."""
    torch = pytest.importorskip("torch")
    rng = np.random.default_rng(cin + k)
    x = rng.standard_normal((cin, 97))
    w = rng.standard_normal((cout, cin, k)) * 0.1
    b = rng.standard_normal(cout)
    y = oracle.conv1d_ref(x, w, b, stride, pad, dil, leaky)
    xt = torch.from_numpy(np.where(x >= 0, x, x * leaky))[None]
    ref = torch.nn.functional.conv1d(xt, torch.from_numpy(w), torch.from_numpy(b), stride, pad, dil)[0].numpy()
    assert y.shape == ref.shape
    np.testing.assert_allclose(y, ref, rtol=1e-12, atol=1e-12)


@pytest.mark.parametrize("cin,cout,k,stride,pad,opad", [(512, 256, 20, 10, 5, 0), (256, 128, 12, 6, 3, 0),
                                                         (64, 64, 3, 2, 1, 1)])
def test_conv_transpose1d_oracle_matches_torch(oracle, cin, cout, k, stride, pad, opad):
    torch = pytest.importorskip("torch")
    rng = np.random.default_rng(cin + k)
    x = rng.standard_normal((cin, 23))
    w = rng.standard_normal((cin, cout, k)) * 0.1
    b = rng.standard_normal(cout)
    y = oracle.conv_transpose1d_ref(x, w, b, stride, pad, opad, 0.1)
    xt = torch.from_numpy(np.where(x >= 0, x, x * 0.1))[None]
    ref = torch.nn.functional.conv_transpose1d(xt, torch.from_numpy(w), torch.from_numpy(b), stride, pad, opad)[0]
    np.testing.assert_allclose(y, ref.numpy(), rtol=1e-12, atol=1e-12)
