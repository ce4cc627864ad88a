"""Decode chain (nq_chain_*, nspeech_b200/decode.py): a decoder token's M = 1
projections run as one cooperative launch.

Reference: the Moonshine decoder token as a sequence of DecoderBackend::gemv
and ::gemv_resadd_ln calls (src/moonshine/decoder.rs,
src/moonshine/gpu_decoder.rs:67-70; kernels/moonshine_kernels.py:1039-1146).
Contract: every chain step computes what the op-by-op call it replaces
(QWeight.linear with one row, QWeight.gemv_resadd_ln) computes -- the same
bf16 weight products -- with f32 sums in another fixed order: the chain is
deterministic, and after several layers its outputs stay within a row-rms
relative error of 5e-2 (bf16 buffers) / 2e-2 (f32 buffers) of the op-by-op
path's: bf16 activations round at every step, so the two orders' last-bit
differences occasionally flip an activation by one bf16 ulp.  The op-by-op path's own parity with the oracle is tested in
test_linear_gpu.py; the chain's logits are also checked against the oracle's
matmul of the chain's final hidden vector.
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


D, FF, VOCAB = 640, 2560, 4096


def _weight(oracle, rng, n, k, flags=0):
    from nspeech_b200.fast_matmul import QWeight
    w = (rng.standard_normal((n, k)) * (1.0 / np.sqrt(k))).astype(np.float32)
    q = oracle.quantize_q8_0(w)
    return QWeight.from_q8_0(q, n, k, flags=flags), q


def _decoder(nq, oracle, layers, seed):
    rng = np.random.default_rng(seed)
    lay = []
    for _ in range(layers):
        L = {}
        L["qkv"], _ = _weight(oracle, rng, 3 * D, D)
        L["o"], _ = _weight(oracle, rng, D, D)
        L["cq"], _ = _weight(oracle, rng, D, D)
        L["co"], _ = _weight(oracle, rng, D, D)
        L["fc1"], _ = _weight(oracle, rng, 2 * FF, D, nq.NQ_PACK_GLU)
        L["fc2"], _ = _weight(oracle, rng, D, FF)
        vec = lambda n, s=0.1: torch.from_numpy((rng.standard_normal(n) * s).astype(np.float32)).cuda()  # noqa: E731
        L["bo"], L["b1"], L["b2"] = vec(D), vec(2 * FF), vec(D)
        for i in range(3):
            L[f"g{i}"] = 1.0 + vec(D)
            L[f"beta{i}"] = vec(D)
        lay.append(L)
    head, hq = _weight(oracle, rng, VOCAB, D)
    return lay, head, hq


class _Bufs:
    def __init__(self, x0, r0):
        self.x = x0.clone()
        self.res = r0.clone()
        self.qkv = torch.zeros(3 * D, device="cuda", dtype=torch.bfloat16)
        self.h = torch.zeros(D, device="cuda", dtype=torch.bfloat16)
        self.t = torch.zeros(FF, device="cuda", dtype=torch.bfloat16)
        self.logits = torch.zeros(VOCAB, device="cuda", dtype=torch.float32)


def _token_ops(nq, lay, head, b):
    """The op-by-op token (two launches per call)."""
    row = lambda v: v.view(1, -1)  # noqa: E731
    for L in lay:
        L["qkv"].linear(row(b.x), out=row(b.qkv))
        L["o"].gemv_resadd_ln(row(b.qkv[:D]), row(b.res), L["g0"], L["beta0"], bias=L["bo"], residual_out=row(b.res),
                              out=row(b.h))
        L["cq"].linear(row(b.h), out=row(b.qkv[:D]))
        L["co"].gemv_resadd_ln(row(b.qkv[:D]), row(b.res), L["g1"], L["beta1"], residual_out=row(b.res),
                               out=row(b.h))
        L["fc1"].linear(row(b.h), bias=L["b1"], epilogue=nq.NQ_EPI_GLU_SILU, out=row(b.t))
        L["fc2"].gemv_resadd_ln(row(b.t), row(b.res), L["g2"], L["beta2"], bias=L["b2"], residual_out=row(b.res),
                                out=row(b.x))
    head.linear(row(b.x), out=row(b.logits))


def _chain(nq, lay, head, b):
    from nspeech_b200.decode import DecodeChain
    c = DecodeChain(0)
    for L in lay:
        c.linear(L["qkv"], b.x, b.qkv)
        c.gemv_resadd_ln(L["o"], b.qkv[:D], b.res, L["g0"], L["beta0"], bias=L["bo"], out=b.h)
        c.linear(L["cq"], b.h, b.qkv[:D])
        c.gemv_resadd_ln(L["co"], b.qkv[:D], b.res, L["g1"], L["beta1"], out=b.h)
        c.linear(L["fc1"], b.h, b.t, bias=L["b1"], epilogue=nq.NQ_EPI_GLU_SILU)
        c.gemv_resadd_ln(L["fc2"], b.t, b.res, L["g2"], L["beta2"], bias=L["b2"], out=b.x)
    c.linear(head, b.x, b.logits)
    return c


NAMES = ("x", "res", "qkv", "h", "t", "logits")


def _close(oracle, a, b):
    # bf16 buffers: a one-ulp rounding flip of an element several times the
    # row's rms already reads a few percent of the rms; an indexing or
    # ordering error reads ~1.
    for name in NAMES:
        t = getattr(a, name)
        u = t.float().cpu().numpy()[None]
        v = getattr(b, name).float().cpu().numpy()[None].astype(np.float64)
        err = oracle.max_rel_err(u, v, 1.0)
        assert err <= (5e-2 if t.dtype == torch.bfloat16 else 2e-2), (name, err)


def _equal(a, b):
    for name in NAMES:
        assert torch.equal(getattr(a, name), getattr(b, name)), name


@pytest.mark.parametrize("layers", [1, 4])
def test_chain_matches_op_by_op(nq, oracle, layers):
    lay, head, hq = _decoder(nq, oracle, layers, 7 + layers)
    x0 = torch.randn(D, device="cuda").to(torch.bfloat16)
    r0 = torch.randn(D, device="cuda")
    ops, ch = _Bufs(x0, r0), _Bufs(x0, r0)
    c = _chain(nq, lay, head, ch)
    assert c.steps == 6 * layers + 1
    for _ in range(2):  # two tokens: the chain's counters re-arm between runs
        _token_ops(nq, lay, head, ops)
        c.run()
        torch.cuda.synchronize()
        _close(oracle, ch, ops)
    # deterministic: the same inputs give the same bits
    first = _Bufs(x0, r0)
    for name in NAMES:
        getattr(first, name).copy_(getattr(ch, name))
    again = _Bufs(x0, r0)
    c2 = _chain(nq, lay, head, again)
    for _ in range(2):
        c2.run()
    torch.cuda.synchronize()
    _equal(first, again)
    c2.close()
    # logits against the oracle's matmul (bf16 weights, f64 sums) of the
    # final hidden vector
    ref = oracle.matmul_fbgemm_bf16(ch.x.float().cpu().numpy()[None], hq, VOCAB).astype(np.float64)
    err = oracle.max_rel_err(ch.logits.cpu().numpy()[None], ref, 1.0)
    assert err <= 2e-3, err
    assert nq.status() == 0
    c.close()


def test_chain_replays_in_a_graph(nq, oracle):
    lay, head, _ = _decoder(nq, oracle, 2, 21)
    x0 = torch.randn(D, device="cuda").to(torch.bfloat16)
    r0 = torch.randn(D, device="cuda")
    ops, ch = _Bufs(x0, r0), _Bufs(x0, r0)
    c = _chain(nq, lay, head, ch)
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        c.run(s)  # the first run uploads the chain
    torch.cuda.synchronize()
    _token_ops(nq, lay, head, ops)
    torch.cuda.synchronize()
    _close(oracle, ch, ops)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        c.run(s)
    for _ in range(3):
        g.replay()
        _token_ops(nq, lay, head, ops)
    torch.cuda.synchronize()
    _close(oracle, ch, ops)
    del g
    assert nq.status() == 0
    c.close()


def test_chain_rejects_hazards(nq, oracle):
    from nspeech_b200.decode import DecodeChain
    from nspeech_b200.fast_matmul import QWeight
    rng = np.random.default_rng(3)
    w, _ = _weight(oracle, rng, D, D)
    g = torch.ones(D, device="cuda")
    a = torch.zeros(2 * D, device="cuda", dtype=torch.bfloat16)
    res = torch.zeros(D, device="cuda")
    c = DecodeChain(0)
    with pytest.raises(nq.NqError) as e:
        c.linear(w, a[:D], a[D // 2:D // 2 + D])  # output overlaps the input
    assert e.value.code == nq.NQ_ERR_UNSUPPORTED
    c.gemv_resadd_ln(w, a[:D], res, g, out=a[D:])
    with pytest.raises(nq.NqError) as e:
        c.gemv_resadd_ln(w, a[D:], res, g, out=a[:D])  # two residual steps in a row
    assert e.value.code == nq.NQ_ERR_UNSUPPORTED
    f32 = torch.zeros(D, device="cuda")
    c.linear(w, a[D:], f32)
    with pytest.raises(Exception):
        c.linear(w, f32.view(torch.bfloat16)[:D], a[:D])  # reads an f32 output as bf16
    bf16_only = QWeight.from_f32((rng.standard_normal((D, D)) * 0.3).astype(np.float32))
    with pytest.raises(nq.NqError) as e:
        c.linear(bf16_only, a[:D], a[D:])
    assert e.value.code == nq.NQ_ERR_UNSUPPORTED
    c.close()


def test_chain_wait_timeout_reports_and_recovers(nq, oracle):
    """Failure detection without a GPU fault: with a wait limit far below a
    step's duration, a bounded wait in the chain runs out, the kernel
    records a status bit and returns (every CTA stops at its next wait).
    nq_status reports it and re-arms the chain's counters; the next run
    with the normal limit gives the op-by-op result."""
    lay, head, _ = _decoder(nq, oracle, 2, 5)
    x0 = torch.randn(D, device="cuda").to(torch.bfloat16)
    r0 = torch.randn(D, device="cuda")
    ch = _Bufs(x0, r0)
    c = _chain(nq, lay, head, ch)
    c.run()  # upload with the normal limit
    torch.cuda.synchronize()
    assert nq.status() == 0
    L = nq.load()
    try:
        nq.check(L.nq_set_wait_limit(200))
        c.run()
        bits = nq.status(0)
        assert bits != 0
        assert nq.status(0) == 0  # cleared
    finally:
        nq.check(L.nq_set_wait_limit(1 << 31))
    # the counters were re-armed: a clean run from the same inputs
    ops = _Bufs(x0, r0)
    _token_ops(nq, lay, head, ops)
    ch.x.copy_(x0)
    ch.res.copy_(r0)
    c.run()
    torch.cuda.synchronize()
    _close(oracle, ch, ops)
    assert nq.status() == 0
    c.close()
