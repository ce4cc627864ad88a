"""GPU parity of the Q8_0 linear path against the CPU oracle.

Contract (per shape): max |y - y_ref| / max(|y_ref|, rms(y_ref row)) <= 1e-2,
with y_ref the reference's executing semantics (FbgemmBf16Op: f32 activations
times bf16-rounded dequantized weights, f32 accumulation) on identical inputs.
bf16 activations are compared against the same semantics applied to the
bf16 values.  The kernels carry f32 activations as bf16 hi + lo planes, so
the observed error is far below the contract; EXPECT_TOL pins that too.
"""
import os

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
CONTRACT_TOL = 1e-2   # north-star bound (row-rms-normalised max relative error)
EXPECT_TOL = 2e-3     # what the hi/lo f32 path and bf16-exact weights deliver

CFG1_SHAPES = [(1024, 4096), (4096, 1024), (1024, 3072), (1024, 1024), (1024, 2048), (1024, 1024)]
# configs[3] Kokoro linears (K -> N) at M = 200 phonemes: ALBERT Q/K/V/dense
# 768 -> 768, FFN 768 -> 2048 (GELU-erf), FFN output 2048 -> 768
# (src/kokoro/albert.rs:126-149), bert_encoder 768 -> 512 (src/kokoro/model.rs:84-87).
KOKORO_SHAPES = [(768, 768, 0), (768, 2048, 2), (2048, 768, 0), (768, 512, 0)]


@pytest.fixture(scope="module")
def nq():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from nspeech_b200 import lib
    lib.init(0)
    return lib


def _bf16_round(x: np.ndarray) -> np.ndarray:
    return torch.from_numpy(x).to(torch.bfloat16).to(torch.float32).numpy()


def _ref(oracle, x, q, n, bias=None, epi=0):
    y = oracle.matmul_fbgemm_bf16(x, q, n).astype(np.float64)
    return oracle.epilogue(y, bias, epi)


def _run(w, x_np, dtype=torch.float32, bias=None, epi=0, out_dtype=torch.float32):
    x = torch.from_numpy(x_np).cuda().to(dtype)
    b = torch.from_numpy(bias).cuda() if bias is not None else None
    y = w.linear(x, bias=b, epilogue=epi, out_dtype=out_dtype)
    torch.cuda.synchronize()
    return y.float().cpu().numpy()


def _check(oracle, got, ref, tag):
    err = oracle.max_rel_err(got, ref, 1.0)
    assert np.isfinite(got).all(), tag
    assert err <= CONTRACT_TOL, f"{tag}: rel err {err:.3e}"
    return err


def test_golden_fixtures(nq, oracle):
    from nspeech_b200.fast_matmul import QWeight
    g = np.load(os.path.join(GOLD, "matmul_small.npz"))
    tags = sorted({k.rsplit("_", 1)[0] for k in g.files})
    for tag in tags:
        x, q, ref = g[f"{tag}_x"], g[f"{tag}_q"], g[f"{tag}_fbgemm"]
        n, k = ref.shape[1], x.shape[1]
        w = QWeight.from_q8_0(q, n, k)
        got = _run(w, x)
        err = _check(oracle, got, ref.astype(np.float64), tag)
        assert err <= EXPECT_TOL, f"{tag}: {err}"
        assert oracle.max_rel_err(got, g[f"{tag}_exact"], 1.0) <= CONTRACT_TOL


@pytest.mark.parametrize("k,n", CFG1_SHAPES[:5])
@pytest.mark.parametrize("xdt", ["f32", "bf16"])
def test_cfg1_block_shapes(nq, oracle, k, n, xdt):
    from nspeech_b200.fast_matmul import QWeight
    x = oracle.normal(0, (125, k), 0.0, 1.0)
    wf = oracle.normal(1000 + k + n, (n, k), 0.0, 0.02)
    q = oracle.quantize_q8_0(wf)
    bias = oracle.normal(7, (n,), 0.0, 0.01)
    w = QWeight.from_q8_0(q, n, k)
    if xdt == "bf16":
        x = _bf16_round(x)
    got = _run(w, x, torch.float32 if xdt == "f32" else torch.bfloat16, bias=bias)
    err = _check(oracle, got, _ref(oracle, x, q, n, bias), f"cfg1 {k}->{n} {xdt}")
    assert err <= EXPECT_TOL


@pytest.mark.parametrize("k,n,epi", KOKORO_SHAPES)
@pytest.mark.parametrize("xdt", ["f32", "bf16"])
@pytest.mark.parametrize("keep", [False, True])
def test_kokoro_shapes(nq, oracle, k, n, epi, xdt, keep):
    """200 phoneme rows, f32 bias N(0, 0.01), both GEMM paths (the
    fused-dequantize kernel below 128 rows is not reached at M = 200: Q8_0
    tiles dequantized per call, or a kept bf16 copy)."""
    from nspeech_b200.fast_matmul import QWeight
    x = oracle.normal(3, (200, k), 0.0, 1.0)
    q = oracle.quantize_q8_0(oracle.normal(3000 + k + n, (n, k), 0.0, 0.02))
    bias = oracle.normal(8, (n,), 0.0, 0.01)
    w = QWeight.from_q8_0(q, n, k)
    if keep:
        w.keep_bf16()
    if xdt == "bf16":
        x = _bf16_round(x)
    got = _run(w, x, torch.float32 if xdt == "f32" else torch.bfloat16, bias=bias, epi=epi)
    err = _check(oracle, got, _ref(oracle, x, q, n, bias, epi), f"kokoro {k}->{n} {xdt} keep={keep}")
    assert err <= EXPECT_TOL


@pytest.mark.parametrize("m", [1, 2, 3, 4, 8, 9, 16, 17, 33, 64, 125, 128, 129, 256, 300, 1024])
def test_m_sweep(nq, oracle, m):
    from nspeech_b200.fast_matmul import QWeight
    k, n = 1024, 1024
    q = oracle.quantize_q8_0(oracle.normal(5, (n, k), 0.0, 0.02))
    w = QWeight.from_q8_0(q, n, k)
    x = oracle.normal(100 + m, (m, k))
    got = _run(w, x)
    assert _check(oracle, got, _ref(oracle, x, q, n), f"m={m}") <= EXPECT_TOL
    xb = _bf16_round(x)
    got = _run(w, xb, torch.bfloat16, out_dtype=torch.bfloat16)
    # bf16 output adds one bf16 rounding of the result (2^-9 relative).
    assert _check(oracle, got, _ref(oracle, xb, q, n), f"m={m} bf16") <= 5e-3


@pytest.mark.parametrize("m", [1, 5, 16, 40, 200])
@pytest.mark.parametrize("epi", [1, 2, 3, 4])
def test_epilogues(nq, oracle, m, epi):
    from nspeech_b200 import lib
    from nspeech_b200.fast_matmul import QWeight
    k, n = 640, 1024
    q = oracle.quantize_q8_0(oracle.normal(9 + epi, (n, k), 0.0, 0.05))
    bias = oracle.normal(10, (n,), 0.0, 0.1)
    glu = epi in (3, 4)
    w = QWeight.from_q8_0(q, n, k, flags=lib.NQ_PACK_GLU if glu else 0)
    x = oracle.normal(11, (m, k))
    got = _run(w, x, bias=bias, epi=epi)
    assert got.shape == (m, n // 2 if glu else n)
    assert _check(oracle, got, _ref(oracle, x, q, n, bias, epi), f"epi={epi} m={m}") <= EXPECT_TOL


# (1, 4096, 4096), (2, 32768, 512), (16, 8192, 1024): GEMV CTAs that stream more
# k chunks than their shared-memory ring holds, so every stage is refilled.
@pytest.mark.parametrize("m,n,k", [(1, 17, 32), (3, 130, 96), (17, 200, 160), (33, 129, 64), (129, 96, 32),
                                   (16, 640, 640), (300, 1920, 768), (2, 32768, 640), (1, 4096, 4096),
                                   (2, 32768, 512), (16, 8192, 1024), (1, 640, 2560), (9, 1024, 4096)])
def test_ragged_shapes(nq, oracle, m, n, k):
    from nspeech_b200.fast_matmul import QWeight
    q = oracle.quantize_q8_0(oracle.normal(m + n + k, (n, k), 0.0, 0.02))
    w = QWeight.from_q8_0(q, n, k)
    x = oracle.normal(3, (m, k))
    assert _check(oracle, _run(w, x), _ref(oracle, x, q, n), f"{m}x{n}x{k}") <= EXPECT_TOL


def test_glu_odd_half_and_padding(nq, oracle):
    from nspeech_b200 import lib
    from nspeech_b200.fast_matmul import QWeight
    for m in (1, 20):
        n, k = 2 * 100, 96  # half = 100: not a multiple of the 64-row GLU tile half
        q = oracle.quantize_q8_0(oracle.normal(21, (n, k), 0.0, 0.05))
        w = QWeight.from_q8_0(q, n, k, flags=lib.NQ_PACK_GLU)
        x = oracle.normal(22, (m, k))
        got = _run(w, x, epi=lib.NQ_EPI_GLU_SILU)
        assert _check(oracle, got, _ref(oracle, x, q, n, None, 4), "glu") <= EXPECT_TOL


def test_qkv_fused_gemv(nq, oracle):
    from nspeech_b200 import dispatch
    from nspeech_b200.fast_matmul import QWeight
    k = 640
    qs = [oracle.quantize_q8_0(oracle.normal(30 + i, (n, k), 0.0, 0.02)) for i, n in enumerate((640, 640, 512))]
    ws = [QWeight.from_q8_0(q, q.shape[0], k) for q in qs]
    x = oracle.normal(33, (1, k))
    xt = torch.from_numpy(x).cuda()
    outs = [torch.empty(w.n, device="cuda") for w in ws]
    dispatch.enc_gemv_qkv_splitk(xt, ws[0], ws[1], ws[2], *outs)
    torch.cuda.synchronize()
    for q, w, o in zip(qs, ws, outs):
        _check(oracle, o.cpu().numpy()[None], _ref(oracle, x, q, w.n), "qkv")


def test_dispatch_entry_points(nq, oracle):
    from nspeech_b200 import dispatch, lib
    from nspeech_b200.fast_matmul import QWeight
    k, n = 768, 3072
    q = oracle.quantize_q8_0(oracle.normal(40, (n, k), 0.0, 0.02))
    w = QWeight.from_q8_0(q, n, k)
    bias = oracle.normal(41, (n,), 0.0, 0.01)
    b = torch.from_numpy(bias).cuda()
    x = oracle.normal(42, (50, k))
    xt = torch.from_numpy(x).cuda()
    _check(oracle, dispatch.triton_matmul(xt, w).cpu().numpy(), _ref(oracle, x, q, n), "triton_matmul")
    _check(oracle, dispatch.triton_matmul_bias(xt, w, b).cpu().numpy(), _ref(oracle, x, q, n, bias), "bias")
    _check(oracle, dispatch.triton_matmul_bias_gelu(xt, w, b).cpu().numpy(), _ref(oracle, x, q, n, bias, 2), "gelu")
    out = torch.empty((64, n), device="cuda")
    dispatch.enc_matmul_bias(xt, w, b, out, 50)
    _check(oracle, out[:50].cpu().numpy(), _ref(oracle, x, q, n, bias), "enc_matmul_bias")
    o1 = torch.empty(n, device="cuda")
    dispatch.enc_gemv_splitk_bias(xt[0], w, b, o1)
    _check(oracle, o1.cpu().numpy()[None], _ref(oracle, x[:1], q, n, bias), "gemv bias")
    wg = QWeight.from_q8_0(q, n, k, flags=lib.NQ_PACK_GLU)
    o2 = torch.empty(n // 2, device="cuda")
    dispatch.enc_gemv_glu_splitk(xt[0], wg, b, o2)
    _check(oracle, o2.cpu().numpy()[None], _ref(oracle, x[:1], q, n, bias, 4), "gemv glu")


def test_matmul_mirror_api(nq, oracle):
    from nspeech_b200.fast_matmul import MatMul, MatMulError
    k, n = 1024, 2048
    wf = oracle.normal(50, (n, k), 0.0, 0.02)
    q = oracle.quantize_q8_0(wf)
    deq = oracle.dequant_q8_0(q, n, k)
    a = MatMul.from_qtensor(q, n, k)
    b = MatMul.from_tensor(deq)  # dequantized f32, as new_mm passes it
    assert np.array_equal(b.weight.to_q8_0(), q)  # lossless re-quantization
    assert np.array_equal(a.weight.to_q8_0(), q)
    x = oracle.normal(51, (2, 3, k))
    xt = torch.from_numpy(x).cuda()
    ya, yb = a.forward(xt), b.forward(xt)
    assert ya.shape == yb.shape == (2, 3, n)
    # from_qtensor: QTiledOp's semantics, bit-identical to the oracle's order
    assert np.array_equal(ya.reshape(6, n).cpu().numpy(), oracle.matmul_qtiled(x.reshape(6, k), q, n))
    # from_tensor: FbgemmBf16Op's semantics
    _check(oracle, yb.reshape(6, n).cpu().numpy(), _ref(oracle, x.reshape(6, k), q, n), "MatMul")
    with pytest.raises(MatMulError, match="not contiguous"):
        a.forward(xt.transpose(0, 1))
    with pytest.raises(MatMulError, match="only one dimension"):
        a.forward(xt[0, 0])
    with pytest.raises(MatMulError, match="incompatible"):
        a.forward(xt[..., :512].contiguous())
    with pytest.raises(MatMulError, match="only supports f32"):
        a.forward(xt.to(torch.bfloat16))


@pytest.mark.parametrize("m,k,n", [(1, 1024, 1024), (3, 96, 130), (16, 640, 2560), (17, 1024, 4096),
                                   (125, 4096, 1024), (200, 768, 2048), (1000, 160, 200)])
@pytest.mark.parametrize("xdt", ["f32", "bf16"])
def test_qtiled_mode_bit_identical_to_oracle(nq, oracle, m, k, n, xdt):
    """NQ_MODE_QTILED weights (MatMul::from_qtensor): x quantized per 32 to
    Q8_0 on the GPU, exact int8 block sums, f32 scaling in block order --
    bit-identical to REF_QTILED (oracle/nq8_oracle.c) on the same inputs."""
    from nspeech_b200.fast_matmul import QWeight
    q = oracle.quantize_q8_0(oracle.normal(70 + n, (n, k), 0.0, 0.02))
    w = QWeight.from_q8_0(q, n, k, flags=nq.NQ_MODE_QTILED)
    x = oracle.normal(71 + m, (m, k))
    if xdt == "bf16":
        x = _bf16_round(x)
    got = _run(w, x, torch.float32 if xdt == "f32" else torch.bfloat16)
    ref = oracle.matmul_qtiled(x, q, n)
    assert np.array_equal(got, ref), float(np.abs(got - ref).max())
    # against the exact product: the activation quantization is the difference
    assert oracle.max_rel_err(got, oracle.matmul_exact(x, q, n), 1.0) < 5e-2


@pytest.mark.parametrize("epi", [0, 1, 2, 5])
def test_qtiled_mode_bias_epilogue_and_edges(nq, oracle, epi):
    from nspeech_b200.fast_matmul import QWeight
    k, n, m = 640, 1000, 33
    xs = oracle.normal(81, (m, k))
    xs[3, :32] = 0.0          # an all-zero block: d = 0
    xs[4, 64:96] = 1e-30      # tiny values: f16 scale underflows to 0
    xs[5, 96:128] = 127.0     # d = 1 exactly
    xs[6, 128:160] = np.linspace(-0.5, 0.5, 32)  # rounding ties
    q = oracle.quantize_q8_0(oracle.normal(82, (n, k), 0.0, 0.05))
    bias = oracle.normal(83, (n,), 0.0, 0.1)
    w = QWeight.from_q8_0(q, n, k, flags=nq.NQ_MODE_QTILED)
    got = _run(w, xs, bias=bias, epi=epi)
    raw = oracle.matmul_qtiled(xs, q, n).astype(np.float64)
    ref = oracle.epilogue(raw, bias, epi)
    assert oracle.max_rel_err(got, ref, 1.0) < 1e-6
    # bf16 output
    got_b = _run(w, xs, bias=bias, epi=epi, out_dtype=torch.bfloat16)
    assert oracle.max_rel_err(got_b, ref, 1.0) < 5e-3
    assert nq.status() == 0


def test_qtiled_mode_rejections(nq, oracle):
    from nspeech_b200 import lib
    from nspeech_b200.fast_matmul import QWeight
    q = oracle.quantize_q8_0(oracle.normal(84, (256, 256), 0.0, 0.05))
    with pytest.raises(lib.NqError) as e:
        QWeight.from_q8_0(q, 256, 256, flags=nq.NQ_MODE_QTILED | nq.NQ_PACK_GLU)
    assert e.value.code == nq.NQ_ERR_UNSUPPORTED
    w = QWeight.from_q8_0(q, 256, 256, flags=nq.NQ_MODE_QTILED)
    x = torch.zeros((1, 256), device="cuda")
    y = torch.zeros((1, 256), device="cuda")
    L = nq.load()
    rc = L.nq_gemv_noalloc(w.handle, x.data_ptr(), 0, 1, 256, None, 0, y.data_ptr(), 0, 256, None)
    assert rc == nq.NQ_ERR_UNSUPPORTED
    plain = QWeight.from_q8_0(q, 256, 256)
    import ctypes
    outs = [torch.zeros((1, 256), device="cuda") for _ in range(3)]
    rc = L.nq_gemv_qkv_splitk(w.handle, plain.handle, w.handle, x.data_ptr(), 0, *[o.data_ptr() for o in outs], 0,
                              ctypes.c_void_p(0))
    assert rc == nq.NQ_ERR_ARG  # one call mixes the two semantics


def test_from_f32_keeps_bf16_for_non_q8_tensor(nq, oracle):
    """MatMul::from_tensor on an f32 tensor that is not a Q8_0 dequantization
    keeps it at bf16 precision, as the reference's PackedMatrixBf16 packing
    does (src/fast_matmul.rs:191-208): y = x . bf16(W)^T with f32 accumulation
    at every M (such a weight has no Q8_0 tiles; the bf16 GEMM serves all M).
    A Q8_0-derived tensor is still stored as Q8_0 (lossless)."""
    from nspeech_b200 import lib
    from nspeech_b200.fast_matmul import MatMul, QWeight
    n, k = 300, 640
    w = oracle.normal(85, (n, k), 0.0, 0.02)
    qw = QWeight.from_f32(w)
    wb = _bf16_round(w).astype(np.float64)
    bias = oracle.normal(86, (n,), 0.0, 0.01)
    for m in (1, 5, 16, 17, 200):
        x = oracle.normal(87 + m, (m, k))
        got = _run(qw, x, bias=bias, epi=1)
        ref = oracle.epilogue(x.astype(np.float64) @ wb.T, bias, 1)
        assert _check(oracle, got, ref, f"bf16-only m={m}") <= EXPECT_TOL
        gotb = _run(qw, _bf16_round(x), torch.bfloat16)
        refb = _bf16_round(x).astype(np.float64) @ wb.T
        assert _check(oracle, gotb, refb, f"bf16-only bf16 x m={m}") <= EXPECT_TOL
    with pytest.raises(lib.NqError) as e:
        qw.to_q8_0()
    assert e.value.code == nq.NQ_ERR_UNSUPPORTED
    with pytest.raises(lib.NqError) as e:
        qw.keep_bf16(False)
    assert e.value.code == nq.NQ_ERR_UNSUPPORTED
    with pytest.raises(lib.NqError) as e:
        QWeight.from_f32(w, flags=nq.NQ_MODE_QTILED)
    assert e.value.code == nq.NQ_ERR_DTYPE
    bad = w.copy()
    bad[7, 9] = np.nan
    with pytest.raises(lib.NqError) as e:
        MatMul.from_tensor(bad)
    assert e.value.code == nq.NQ_ERR_DTYPE
    deq = oracle.dequant_q8_0(oracle.quantize_q8_0(w), n, k)
    assert np.array_equal(QWeight.from_f32(deq).to_q8_0(), oracle.quantize_q8_0(w))
    # the MatMul mirror keeps the reference's f32 contract on such a weight
    mm = MatMul.from_tensor(w)
    x = oracle.normal(90, (2, 3, k))
    y = mm.forward(torch.from_numpy(x).cuda()).cpu().numpy().reshape(6, n)
    assert _check(oracle, y, x.reshape(6, k).astype(np.float64) @ wb.T, "MatMul bf16-only") <= EXPECT_TOL


def test_weight_roundtrip_and_fuse(nq, oracle):
    from nspeech_b200.fast_matmul import QWeight
    k = 96
    qa = oracle.quantize_q8_0(oracle.normal(60, (70, k), 0.0, 0.1))
    qb = oracle.quantize_q8_0(oracle.normal(61, (130, k), 0.0, 0.1))
    wa, wb = QWeight.from_q8_0(qa, 70, k), QWeight.from_q8_0(qb, 130, k)
    assert np.array_equal(wa.to_q8_0(), qa)
    f = QWeight.fuse([wa, wb])
    assert (f.n, f.k) == (200, k)
    assert np.array_equal(f.to_q8_0(), np.concatenate([qa, qb]))
    x = oracle.normal(62, (5, k))
    _check(oracle, _run(f, x), _ref(oracle, x, np.concatenate([qa, qb]), 200), "fused")


def test_gguf_load(nq, oracle, tmp_path):
    gguf = pytest.importorskip("gguf")
    from nspeech_b200 import lib
    from nspeech_b200.fast_matmul import QWeight
    n, k = 300, 640
    q = oracle.quantize_q8_0(oracle.normal(70, (n, k), 0.0, 0.02))
    p = tmp_path / "w.gguf"
    wr = gguf.GGUFWriter(str(p), arch="parakeet")
    wr.add_tensor("layers.0.feed_forward1.linear1.weight", q, raw_dtype=gguf.GGMLQuantizationType.Q8_0)
    wr.add_tensor("f32.weight", oracle.normal(71, (4, 32)))
    wr.write_header_to_file()
    wr.write_kv_data_to_file()
    wr.write_tensors_to_file()
    wr.close()
    w = QWeight.from_gguf(str(p), "layers.0.feed_forward1.linear1.weight")
    assert (w.n, w.k) == (n, k)
    assert np.array_equal(w.to_q8_0(), q)
    with pytest.raises(lib.NqError) as e:
        QWeight.from_gguf(str(p), "f32.weight")
    assert e.value.code == lib.NQ_ERR_DTYPE


def test_errors_fail_loudly(nq, oracle):
    import ctypes
    from nspeech_b200 import lib
    from nspeech_b200.fast_matmul import QWeight
    L = lib.load()
    h = ctypes.c_void_p()
    blob = np.zeros(34 * 4, np.uint8)
    assert L.nq_weight_from_q8_0(blob.ctypes.data, 4, 48, 0, ctypes.byref(h)) == lib.NQ_ERR_SHAPE
    q = oracle.quantize_q8_0(oracle.normal(80, (64, 64)))
    w = QWeight.from_q8_0(q, 64, 64)
    x = torch.zeros((4, 64), device="cuda")
    with pytest.raises(lib.NqError) as e:
        w.linear(x, epilogue=lib.NQ_EPI_GLU_SILU)
    assert e.value.code == lib.NQ_ERR_UNSUPPORTED
    y = torch.empty((0, 64), device="cuda")
    w.linear(torch.zeros((0, 64), device="cuda"), out=y)  # M = 0 is a no-op
    assert lib.status() == 0


def test_deterministic_split_k(nq, oracle):
    from nspeech_b200.fast_matmul import QWeight
    for (m, k, n) in [(1, 4096, 1024), (125, 4096, 1024), (8, 2560, 640)]:
        q = oracle.quantize_q8_0(oracle.normal(90, (n, k), 0.0, 0.02))
        w = QWeight.from_q8_0(q, n, k)
        x = torch.from_numpy(oracle.normal(91, (m, k))).cuda()
        a = w.linear(x).clone()
        b = w.linear(x).clone()
        assert torch.equal(a, b)


def test_full_size_row_sample_and_linearity(nq, oracle):
    """cfg5-sized M (12000 rows): oracle on a row sample + linearity in x."""
    from nspeech_b200.fast_matmul import QWeight
    m, k, n = 12000, 1024, 4096
    q = oracle.quantize_q8_0(oracle.normal(95, (n, k), 0.0, 0.02))
    w = QWeight.from_q8_0(q, n, k)
    x = torch.randn((m, k), generator=torch.Generator().manual_seed(96)).to(torch.bfloat16).cuda()
    y = w.linear(x, out_dtype=torch.float32)
    rows = np.random.default_rng(97).choice(m, 96, replace=False)
    xs = x[rows].float().cpu().numpy()
    _check(oracle, y[rows].cpu().numpy(), _ref(oracle, xs, q, n), "row sample")
    y2 = w.linear(x * 2, out_dtype=torch.float32)  # exact scaling in bf16
    assert torch.equal(y2, 2 * y)


def test_wait_timeout_reports_and_recovers(nq, oracle):
    """A bounded wait that nothing satisfies ends with a status bit, not a hang."""
    from nspeech_b200 import lib
    from nspeech_b200.fast_matmul import QWeight
    L = lib.load()
    try:
        lib.check(L.nq_set_wait_limit(2_000_000))  # ~1 ms
        lib.check(L.nq_debug_wait_timeout(None))
        bits = lib.status(0)
        assert bits & 0x2
        assert lib.status(0) == 0  # cleared
    finally:
        lib.check(L.nq_set_wait_limit(1 << 31))
    q = oracle.quantize_q8_0(oracle.normal(99, (256, 256), 0.0, 0.02))
    w = QWeight.from_q8_0(q, 256, 256)
    x = oracle.normal(98, (3, 256))
    _check(oracle, _run(w, x), _ref(oracle, x, q, 256), "after timeout")


@pytest.fixture
def gemv_path(nq):
    """Select the GEMV form for one test (nq_set_gemv_path), AUTO after it."""
    L = nq.load()

    def set_path(path):
        nq.check(L.nq_set_gemv_path(path))

    yield set_path
    nq.check(L.nq_set_gemv_path(nq.NQ_GEMV_AUTO))


# Both GEMV forms -- k split over all SMs + reduce launch, and each tile's k
# over a cluster with the partials added in distributed shared memory -- on
# the decoder's shapes and on shapes at the edges of the cluster rule (one k
# chunk; the lm_head's 256 tiles; 16 rows; f32 activations; GLU).
@pytest.mark.parametrize("m,k,n,flags,epi,dt", [
    (1, 640, 640, 0, 0, "bf16"), (1, 640, 1920, 0, 0, "bf16"), (1, 640, 5120, 1, 4, "bf16"),
    (1, 2560, 640, 0, 1, "bf16"), (1, 640, 32768, 0, 0, "bf16"), (8, 4096, 4096, 0, 2, "bf16"),
    (16, 1024, 3000, 0, 0, "f32"), (4, 64, 200, 0, 5, "f32"), (3, 512, 4096, 1, 3, "f32")])
def test_gemv_forms_match_oracle(nq, oracle, gemv_path, m, k, n, flags, epi, dt):
    from nspeech_b200.fast_matmul import QWeight
    q = oracle.quantize_q8_0(oracle.normal(70 + n + k, (n, k), 0.0, 0.02))
    w = QWeight.from_q8_0(q, n, k, flags=flags)
    x = oracle.normal(71, (m, k))
    bias = oracle.normal(72, (n,), 0.0, 0.1)
    if dt == "bf16":
        x = torch.from_numpy(x).to(torch.bfloat16).float().numpy()
    ref = _ref(oracle, x, q, n, bias, epi) if not flags else None
    outs = []
    for path in (1, 2):
        gemv_path(path)
        y = _run(w, x, torch.float32 if dt == "f32" else torch.bfloat16, bias=bias, epi=epi)
        y2 = _run(w, x, torch.float32 if dt == "f32" else torch.bfloat16, bias=bias, epi=epi)
        assert np.array_equal(y, y2)  # deterministic
        outs.append(y)
    if ref is not None:
        for got in outs:
            _check(oracle, got, ref, f"gemv {m}x{k}x{n}")
    # same products, f32 sums in another order
    scale = max(1.0, float(np.abs(outs[0]).max()))
    assert np.abs(outs[0] - outs[1]).max() <= 1e-3 * scale
    assert nq.status() == 0


# nq_gemv_resadd_ln: decoder-step GEMV with the fused residual add + LayerNorm
# (DecoderBackend::gemv_resadd_ln).  Moonshine decoder shapes (640 -> 640 O
# projections, 2560 -> 640 fc2), an odd width, and several rows; in-place
# residual, with and without bias / beta, bf16 and f32 outputs.
@pytest.mark.parametrize("path", [1, 2])  # NQ_GEMV_SPLIT, NQ_GEMV_CLUSTER
@pytest.mark.parametrize("m,k,n,bias,beta,inplace,odt", [
    (1, 640, 640, False, False, False, torch.bfloat16),
    (1, 2560, 640, True, False, True, torch.bfloat16),
    (4, 1024, 1000, True, True, False, torch.float32),
    (16, 640, 640, True, True, True, torch.float32),
    (1, 4096, 8192, False, True, False, torch.bfloat16),
])
def test_gemv_resadd_ln_matches_oracle(nq, oracle, gemv_path, m, k, n, bias, beta, inplace, odt, path):
    from nspeech_b200.fast_matmul import QWeight
    gemv_path(path)
    q = oracle.quantize_q8_0(oracle.normal(60 + n, (n, k), 0.0, 0.02))
    w = QWeight.from_q8_0(q, n, k)
    x = oracle.normal(61, (m, k))
    res = oracle.normal(62, (m, n))
    g = oracle.normal(63, (n,), 1.0, 0.1)
    b = oracle.normal(64, (n,), 0.0, 0.1) if beta else None
    bs = oracle.normal(65, (n,), 0.0, 0.01) if bias else None
    y = oracle.matmul_fbgemm_bf16(x, q, n).astype(np.float64) + (bs if bias else 0.0)
    r_ref, o_ref = oracle.resadd_layernorm(y, res, g, b, 1e-5)
    dev = lambda a: torch.from_numpy(a).cuda() if a is not None else None
    rin = dev(res)
    rout, out = w.gemv_resadd_ln(dev(x), rin, dev(g), beta=dev(b), bias=dev(bs), eps=1e-5,
                                 residual_out=rin if inplace else None, out_dtype=odt)
    torch.cuda.synchronize()
    if inplace:
        assert rout.data_ptr() == rin.data_ptr()
    r_got, o_got = rout.cpu().numpy(), out.float().cpu().numpy()
    err_r = oracle.max_rel_err(r_got, r_ref, 1.0)
    err_o = oracle.max_rel_err(o_got, o_ref, 1.0)
    assert np.isfinite(o_got).all()
    assert err_r <= EXPECT_TOL, err_r
    assert err_o <= (EXPECT_TOL if odt == torch.float32 else 1e-2), err_o
    # bit-reproducible: the same call again gives the same bits
    rout2, out2 = w.gemv_resadd_ln(dev(x), dev(res), dev(g), beta=dev(b), bias=dev(bs), eps=1e-5, out_dtype=odt)
    torch.cuda.synchronize()
    if not inplace:
        assert torch.equal(rout2, rout)
        assert torch.equal(out2, out)
    assert nq.status() == 0


def test_gemv_resadd_ln_rejects_bad_arguments(nq):
    from nspeech_b200 import lib
    from nspeech_b200.fast_matmul import QWeight, MatMulError
    q = np.zeros((8192 + 128, 64 // 32 * 34), dtype=np.uint8)
    wide = QWeight.from_q8_0(q, 8192 + 128, 64)
    x = torch.zeros((1, 64), device="cuda")
    r = torch.zeros((1, 8192 + 128), device="cuda")
    g = torch.ones(8192 + 128, device="cuda")
    with pytest.raises(lib.NqError) as e:
        wide.gemv_resadd_ln(x, r, g)
    assert e.value.code == lib.NQ_ERR_SHAPE
    w = QWeight.from_q8_0(np.zeros((64, 2 * 34), dtype=np.uint8), 64, 64)
    x17 = torch.zeros((17, 64), device="cuda")
    with pytest.raises(lib.NqError) as e:
        w.gemv_resadd_ln(x17, torch.zeros((17, 64), device="cuda"), torch.ones(64, device="cuda"))
    assert e.value.code == lib.NQ_ERR_SHAPE
    with pytest.raises(MatMulError):
        w.gemv_resadd_ln(torch.zeros((1, 64), device="cuda"), torch.zeros((1, 64), device="cuda", dtype=torch.float64),
                         torch.ones(64, device="cuda"))
    assert nq.status() == 0
