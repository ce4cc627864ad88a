"""Kokoro conv1d / conv_transpose1d (nq_conv1d, nq_conv_transpose1d) against
the CPU oracle.

Reference semantics: the decoder's convolutions on the weights the loader
dequantizes from Q8_0 (src/kokoro/model.rs:66-76, decoder.rs), lowered by the
reference's GPU path to im2col + matmul_bias (kernels/kokoro_kernels.py:182,
426; src/kokoro/gpu_backend.rs:59-110).  Here the weights multiply at bf16
precision (the fast_matmul packing of the dequantized values) with f32
accumulation, so the oracle is the float64 convolution of the bf16-rounded
weights (oracle.conv1d_ref / conv_transpose1d_ref, themselves checked against
torch.nn.functional in tests/test_oracle_vs_parakeet.py).  Contract: the
row-rms-normalised max relative error of the linear tests, <= 2e-3 for f32
inputs and outputs, <= 1e-2 with bf16 inputs or outputs.
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def nq():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from nspeech_b200 import lib
    lib.init(0)
    return lib


def _bf16(a):
    return torch.from_numpy(np.ascontiguousarray(a, np.float32)).to(torch.bfloat16).to(torch.float32).numpy()


def _err(oracle, got, ref):
    # rows are output channels, normalised by each channel's rms
    return oracle.max_rel_err(np.ascontiguousarray(got, np.float32), np.ascontiguousarray(ref, np.float64), 1.0)


# (c_in, c_out, K, stride, padding, dilation, leaky, T_in): resblock convs with
# dilations 1/3/5 (kernels 3/7/11), the conv_post (128 -> 22, K 7, leaky 0.01),
# the ASR projection (512 -> 64, K 1), the F0/N convs (1 -> 1, K 3, stride 2:
# a bf16-only weight, 3 is not a multiple of 32), a short sequence (T_out <= 16:
# the GEMV path) and a 22-channel noise conv.
CONV1D = [(128, 128, 3, 1, 1, 1, 1.0, 700), (128, 128, 7, 1, 9, 3, 0.1, 700), (64, 64, 11, 1, 25, 5, 0.1, 1500),
          (128, 22, 7, 1, 3, 1, 0.01, 2000), (512, 64, 1, 1, 0, 1, 1.0, 300), (1, 1, 3, 2, 1, 1, 1.0, 401),
          (256, 256, 3, 1, 1, 1, 1.0, 12), (22, 64, 7, 1, 3, 1, 1.0, 300)]


@pytest.mark.parametrize("cin,cout,k,stride,pad,dil,leaky,t_in", CONV1D)
@pytest.mark.parametrize("dt", ["f32", "bf16"])
def test_conv1d_matches_oracle(nq, oracle, cin, cout, k, stride, pad, dil, leaky, t_in, dt):
    from nspeech_b200 import conv as C
    from nspeech_b200.fast_matmul import QWeight
    rng = np.random.default_rng(cin * 7 + k + t_in)
    w3 = (rng.standard_normal((cout, cin, k)) * 0.05).astype(np.float32)
    w2 = w3.reshape(cout, cin * k)
    if (cin * k) % 32 == 0:
        q = oracle.quantize_q8_0(w2)  # the GGUF form: Q8_0 [C_out, C_in * K]
        w = QWeight.from_q8_0(q, cout, cin * k)
        wref = _bf16(oracle.dequant_q8_0(q, cout, cin * k)).reshape(cout, cin, k)
    else:
        w = QWeight.from_f32(w2)  # stays f32 in GGUF: kept at bf16 precision
        wref = _bf16(w2).reshape(cout, cin, k)
    bias = (rng.standard_normal(cout) * 0.1).astype(np.float32)
    x = rng.standard_normal((cin, t_in)).astype(np.float32)
    tdt = torch.float32 if dt == "f32" else torch.bfloat16
    if dt == "bf16":
        x = _bf16(x)
    xt = torch.from_numpy(x).cuda().to(tdt)
    y = C.conv1d(xt, w, torch.from_numpy(bias).cuda(), k, stride, pad, dil, x_leaky=leaky, out_dtype=torch.float32)
    torch.cuda.synchronize()
    ref = oracle.conv1d_ref(x, wref, bias, stride, pad, dil, leaky)
    assert y.shape == ref.shape
    err = _err(oracle, y.cpu().numpy(), ref)
    assert err <= (2e-3 if dt == "f32" else 1e-2), err
    assert nq.status() == 0


def test_conv1d_epilogue_bf16_out_and_strided_rows(nq, oracle):
    """SiLU epilogue, bf16 output, and x / y channel rows with padding (ldx, ldy)."""
    from nspeech_b200 import conv as C
    from nspeech_b200.fast_matmul import QWeight
    rng = np.random.default_rng(5)
    cin, cout, k, t_in = 256, 128, 3, 500
    w2 = (rng.standard_normal((cout, cin * k)) * 0.05).astype(np.float32)
    q = oracle.quantize_q8_0(w2)
    w = QWeight.from_q8_0(q, cout, cin * k)
    wref = _bf16(oracle.dequant_q8_0(q, cout, cin * k)).reshape(cout, cin, k)
    x = rng.standard_normal((cin, t_in)).astype(np.float32)
    xbig = torch.zeros((cin, t_in + 37), device="cuda")
    xbig[:, :t_in] = torch.from_numpy(x).cuda()
    ybig = torch.full((cout, 520), float("nan"), device="cuda", dtype=torch.bfloat16)
    C.conv1d(xbig[:, :t_in], w, None, k, 1, 1, 1, epilogue=nq.NQ_EPI_SILU, out=ybig[:, :500])
    torch.cuda.synchronize()
    ref = oracle.conv1d_ref(x, wref, None, 1, 1, 1)
    ref = ref / (1 + np.exp(-ref))
    got = ybig[:, :500].float().cpu().numpy()
    assert _err(oracle, got, ref) <= 1e-2
    assert torch.isnan(ybig[:, 500:].float()).all()  # nothing written past the output length


# Implicit-GEMM conv1d (stride 1, c_in a multiple of 64): (c_in, c_out, K,
# padding, dilation, leaky, T_in).  Many token tiles with dilation 5; a short
# sequence (tail split); c_out 22 (partial feature rows); no padding (T_out <
# T_in); padding beyond the kernel's reach (rows outside the input on both
# ends); 512 input channels.
IMPLICIT = [(128, 128, 11, 25, 5, 0.1, 3000), (256, 256, 7, 9, 3, 0.1, 1000), (512, 256, 3, 1, 1, 1.0, 300),
            (64, 22, 7, 3, 1, 0.01, 2000), (128, 64, 5, 0, 2, 1.0, 40), (64, 96, 3, 10, 1, 1.0, 150)]


@pytest.mark.parametrize("cin,cout,k,pad,dil,leaky,t_in", IMPLICIT)
@pytest.mark.parametrize("dt", ["f32", "bf16"])
def test_conv1d_implicit_matches_oracle_and_im2col(nq, oracle, cin, cout, k, pad, dil, leaky, t_in, dt):
    """The implicit GEMM (default for these shapes) against the oracle and
    against the im2col lowering (NQ_CONV_IM2COL) of the same weights; both
    sum the same products in different orders.  Repeated calls are
    bit-identical."""
    from nspeech_b200 import conv as C
    from nspeech_b200.fast_matmul import QWeight
    L = nq.load()
    rng = np.random.default_rng(cin + 3 * k + t_in)
    w2 = (rng.standard_normal((cout, cin * k)) * 0.05).astype(np.float32)
    q = oracle.quantize_q8_0(w2)
    w = QWeight.from_q8_0(q, cout, cin * k)
    wref = _bf16(oracle.dequant_q8_0(q, cout, cin * k)).reshape(cout, cin, k)
    bias = (rng.standard_normal(cout) * 0.1).astype(np.float32)
    x = rng.standard_normal((cin, t_in)).astype(np.float32)
    tdt = torch.float32 if dt == "f32" else torch.bfloat16
    if dt == "bf16":
        x = _bf16(x)
    xt = torch.from_numpy(x).cuda().to(tdt)
    bt = torch.from_numpy(bias).cuda()
    y = C.conv1d(xt, w, bt, k, 1, pad, dil, x_leaky=leaky, out_dtype=torch.float32)
    y_again = C.conv1d(xt, w, bt, k, 1, pad, dil, x_leaky=leaky, out_dtype=torch.float32)
    try:
        nq.check(L.nq_set_conv_path(nq.NQ_CONV_IM2COL))
        y_im2col = C.conv1d(xt, w, bt, k, 1, pad, dil, x_leaky=leaky, out_dtype=torch.float32)
    finally:
        nq.check(L.nq_set_conv_path(nq.NQ_CONV_AUTO))
    torch.cuda.synchronize()
    ref = oracle.conv1d_ref(x, wref, bias, 1, pad, dil, leaky)
    assert y.shape == ref.shape
    tol = 2e-3 if dt == "f32" else 1e-2
    assert _err(oracle, y.cpu().numpy(), ref) <= tol
    assert _err(oracle, y_im2col.cpu().numpy(), ref) <= tol
    assert torch.equal(y, y_again)
    # same bf16 products, f32 sums in another order
    assert (y - y_im2col).abs().max().item() <= 1e-3 * max(1.0, y_im2col.abs().max().item())
    assert nq.status() == 0


@pytest.mark.parametrize("unit", [64, 128, 256])
def test_conv1d_implicit_unit_widths_and_tail_split(nq, oracle, unit):
    """Forced unit widths and a forced tail split give the oracle's result
    on a short, wide conv (few token tiles)."""
    from nspeech_b200 import conv as C
    from nspeech_b200.fast_matmul import QWeight
    L = nq.load()
    rng = np.random.default_rng(unit)
    cin, cout, k, pad, dil, t_in = 256, 512, 3, 1, 1, 300
    w2 = (rng.standard_normal((cout, cin * k)) * 0.05).astype(np.float32)
    q = oracle.quantize_q8_0(w2)
    w = QWeight.from_q8_0(q, cout, cin * k)
    wref = _bf16(oracle.dequant_q8_0(q, cout, cin * k)).reshape(cout, cin, k)
    x = _bf16(rng.standard_normal((cin, t_in)).astype(np.float32))
    xt = torch.from_numpy(x).cuda().to(torch.bfloat16)
    ref = oracle.conv1d_ref(x, wref, None, 1, pad, dil)
    outs = []
    try:
        nq.check(L.nq_set_gemm_unit_tokens(unit))
        for split in (1, 4):
            nq.check(L.nq_set_gemm_tail_split(split))
            outs.append(C.conv1d(xt, w, None, k, 1, pad, dil, out_dtype=torch.float32))
    finally:
        nq.check(L.nq_set_gemm_unit_tokens(0))
        nq.check(L.nq_set_gemm_tail_split(0))
    torch.cuda.synchronize()
    for y in outs:
        assert _err(oracle, y.cpu().numpy(), ref) <= 1e-2
    assert nq.status() == 0


@pytest.mark.parametrize("pad_t", [0, 3])
def test_conv1d_implicit_bf16_rows_and_graph(nq, oracle, pad_t):
    """bf16 NCW output with 16-byte aligned rows (vector stores) and with
    odd row padding (element stores), nothing written past the output length;
    after a first call the conv replays inside a CUDA graph."""
    from nspeech_b200 import conv as C
    from nspeech_b200.fast_matmul import QWeight
    rng = np.random.default_rng(11 + pad_t)
    cin, cout, k, pad, dil, t_in = 128, 128, 7, 9, 3, 1200
    w2 = (rng.standard_normal((cout, cin * k)) * 0.05).astype(np.float32)
    q = oracle.quantize_q8_0(w2)
    w = QWeight.from_q8_0(q, cout, cin * k)
    wref = _bf16(oracle.dequant_q8_0(q, cout, cin * k)).reshape(cout, cin, k)
    x = _bf16(rng.standard_normal((cin, t_in)).astype(np.float32))
    xt = torch.from_numpy(x).cuda().to(torch.bfloat16)
    t_out = C.conv1d_out_len(t_in, k, 1, pad, dil)
    ybig = torch.full((cout, t_out + 8 + pad_t), float("nan"), device="cuda", dtype=torch.bfloat16)
    y = ybig[:, :t_out]
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        C.conv1d(xt, w, None, k, 1, pad, dil, x_leaky=0.1, epilogue=nq.NQ_EPI_RELU, out=y, stream=s)
    torch.cuda.synchronize()
    ref = np.maximum(oracle.conv1d_ref(x, wref, None, 1, pad, dil, 0.1), 0.0)
    assert _err(oracle, y.float().cpu().numpy(), ref) <= 1e-2
    assert torch.isnan(ybig[:, t_out:].float()).all()
    first = y.clone()
    y.zero_()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        C.conv1d(xt, w, None, k, 1, pad, dil, x_leaky=0.1, epilogue=nq.NQ_EPI_RELU, out=y, stream=s)
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(y, first)
    del g
    assert nq.status() == 0


# Kokoro generator upsampling (ConvTranspose1d 512 -> 256, K 20, stride 10,
# padding 5; 256 -> 128, K 12, stride 6, padding 3; leaky 0.1 on the input) and
# a small one with output padding.
CONVT = [(512, 256, 20, 10, 5, 0, 0.1, 80), (256, 128, 12, 6, 3, 0, 0.1, 300), (64, 48, 3, 2, 1, 1, 1.0, 9)]


@pytest.mark.parametrize("cin,cout,k,stride,pad,opad,leaky,t_in", CONVT)
@pytest.mark.parametrize("dt", ["f32", "bf16"])
def test_conv_transpose1d_matches_oracle(nq, oracle, cin, cout, k, stride, pad, opad, leaky, t_in, dt):
    from nspeech_b200 import conv as C
    rng = np.random.default_rng(cin + k)
    w = (rng.standard_normal((cin, cout, k)) * 0.05).astype(np.float32)
    wt = C.ConvTransposeWeight.from_f32(w)
    bias = (rng.standard_normal(cout) * 0.1).astype(np.float32)
    x = rng.standard_normal((cin, t_in)).astype(np.float32)
    tdt = torch.float32 if dt == "f32" else torch.bfloat16
    if dt == "bf16":
        x = _bf16(x)
    y = C.conv_transpose1d(torch.from_numpy(x).cuda().to(tdt), wt, torch.from_numpy(bias).cuda(), stride, pad, opad,
                           x_leaky=leaky, out_dtype=torch.float32)
    torch.cuda.synchronize()
    ref = oracle.conv_transpose1d_ref(x, _bf16(w), bias, stride, pad, opad, leaky)
    assert y.shape == ref.shape
    err = _err(oracle, y.cpu().numpy(), ref)
    assert err <= (2e-3 if dt == "f32" else 1e-2), err
    # deterministic: the overlap-add sums taps in a fixed order
    y2 = C.conv_transpose1d(torch.from_numpy(x).cuda().to(tdt), wt, torch.from_numpy(bias).cuda(), stride, pad, opad,
                            x_leaky=leaky, out_dtype=torch.float32)
    assert torch.equal(y, y2)
    assert nq.status() == 0


# Polyphase implicit GEMM (c_in a multiple of 64, more than 16 input
# positions): (c_in, c_out, K, stride, padding, output_padding, leaky, T_in).
# Kernels that are and are not multiples of the stride, output padding, no
# padding, and c_out * stride not a multiple of 128.
POLY = [(512, 256, 20, 10, 5, 0, 0.1, 300), (256, 128, 12, 6, 3, 0, 0.1, 700), (128, 48, 7, 3, 2, 1, 1.0, 60),
        (64, 40, 5, 2, 0, 1, 0.2, 33), (128, 64, 4, 4, 0, 0, 1.0, 50)]


@pytest.mark.parametrize("cin,cout,k,stride,pad,opad,leaky,t_in", POLY)
@pytest.mark.parametrize("dt", ["f32", "bf16"])
def test_conv_transpose1d_implicit_matches_oracle_and_col2im(nq, oracle, cin, cout, k, stride, pad, opad, leaky,
                                                             t_in, dt):
    """The polyphase implicit GEMM (default for these shapes) against the
    oracle and against the column GEMM + overlap-add (NQ_CONV_IM2COL)."""
    from nspeech_b200 import conv as C
    L = nq.load()
    rng = np.random.default_rng(cin + 5 * k + t_in)
    w = (rng.standard_normal((cin, cout, k)) * 0.05).astype(np.float32)
    wt = C.ConvTransposeWeight.from_f32(w)
    bias = (rng.standard_normal(cout) * 0.1).astype(np.float32)
    x = rng.standard_normal((cin, t_in)).astype(np.float32)
    tdt = torch.float32 if dt == "f32" else torch.bfloat16
    if dt == "bf16":
        x = _bf16(x)
    xt = torch.from_numpy(x).cuda().to(tdt)
    bt = torch.from_numpy(bias).cuda()
    y = C.conv_transpose1d(xt, wt, bt, stride, pad, opad, x_leaky=leaky, out_dtype=torch.float32)
    y2 = C.conv_transpose1d(xt, wt, bt, stride, pad, opad, x_leaky=leaky, out_dtype=torch.float32)
    try:
        nq.check(L.nq_set_conv_path(nq.NQ_CONV_IM2COL))
        yc = C.conv_transpose1d(xt, wt, bt, stride, pad, opad, x_leaky=leaky, out_dtype=torch.float32)
    finally:
        nq.check(L.nq_set_conv_path(nq.NQ_CONV_AUTO))
    torch.cuda.synchronize()
    ref = oracle.conv_transpose1d_ref(x, _bf16(w), bias, stride, pad, opad, leaky)
    assert y.shape == ref.shape
    tol = 2e-3 if dt == "f32" else 1e-2
    assert _err(oracle, y.cpu().numpy(), ref) <= tol
    assert _err(oracle, yc.cpu().numpy(), ref) <= tol
    assert torch.equal(y, y2)
    assert (y - yc).abs().max().item() <= 1e-3 * max(1.0, yc.abs().max().item())
    assert nq.status() == 0


def test_conv_rejects_bad_shapes(nq, oracle):
    from nspeech_b200 import conv as C
    from nspeech_b200.fast_matmul import MatMulError, QWeight
    q = oracle.quantize_q8_0(oracle.normal(3, (64, 128 * 3), 0.0, 0.05))
    w = QWeight.from_q8_0(q, 64, 128 * 3)
    x = torch.zeros((100, 50), device="cuda")  # 100 channels, weight expects 128 x 3
    with pytest.raises(nq.NqError) as e:
        C.conv1d(x, w, None, 3, 1, 1)
    assert e.value.code == nq.NQ_ERR_SHAPE
    with pytest.raises(MatMulError):
        C.conv1d(torch.zeros((128, 2), device="cuda"), w, None, 3, 1, 0)  # no output frames
    assert nq.status() == 0
