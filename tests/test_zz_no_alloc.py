"""nq_gemv_noalloc (static-scratch split-K GEMV) against nq_linear and the
CPU oracle.

Runs through the C ABI: the same weight and activations go through the
existing entry point (nq_linear, workspace scratch) and through
nq_gemv_noalloc (static device scratch); outputs must agree within the
linear contract's tolerance, on two calls in a row (the second call reuses
the array the first one left behind), and both must match the reference's
FbgemmBf16Op semantics computed by the oracle.  Collected last, and
self-contained so it also passes alone in a fresh process (its first call
sets up the scratch).
"""
import ctypes

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

TOL = 2e-3  # EXPECT_TOL of the linear parity tests (row-rms-normalised max rel err)


@pytest.fixture(scope="module")
def nq():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from nspeech_b200 import lib
    lib.init(0)
    return lib


def _rel(a, b):
    a = a.astype(np.float64)
    b = b.astype(np.float64)
    scale = np.maximum(np.abs(b), np.sqrt((b * b).mean(axis=1, keepdims=True)))
    return float((np.abs(a - b) / np.maximum(scale, 1e-30)).max())


def _weight(nq, rng, n, k, flags=0):
    from nspeech_b200.fast_matmul import QWeight
    q = rng.integers(0, 256, size=(n, k // 32, 34), dtype=np.uint8)
    q[:, :, :2] = (rng.random((n, k // 32)) * 2e-3 + 1e-4).astype(np.float16).view(np.uint8).reshape(n, k // 32, 2)
    return QWeight.from_q8_0(np.ascontiguousarray(q.reshape(n, -1)), n, k, flags=flags)


def _call(L, fn, w, x, m, bias, epi, y, y_dtype):
    s = torch.cuda.current_stream().cuda_stream
    x_dtype = 0 if x.dtype == torch.float32 else 1
    rc = fn(w._h, x.data_ptr(), x_dtype, m, x.stride(0), bias.data_ptr() if bias is not None else None, epi,
            y.data_ptr(), y_dtype, y.stride(0), ctypes.c_void_p(s))
    return rc


@pytest.mark.parametrize("m,k,n,epi,glu", [(1, 1024, 4096, 0, False), (4, 4096, 1024, 1, False),
                                           (16, 1024, 1024, 0, False), (1, 640, 1024, 4, True),
                                           (9, 2048, 3072, 2, False)])
@pytest.mark.parametrize("xdt", [torch.float32, torch.bfloat16])
def test_noalloc_matches_linear_twice(nq, oracle, m, k, n, epi, glu, xdt):
    L = nq.load()
    rng = np.random.default_rng(m * 31 + k + n)
    w = _weight(nq, rng, n, k, flags=nq.NQ_PACK_GLU if glu else 0)
    blocks = w.to_q8_0()
    n_out = n // 2 if glu else n
    bias_np = rng.standard_normal(n).astype(np.float32) * 0.1
    bias = torch.from_numpy(bias_np).cuda()
    ref = torch.empty((m, n_out), device="cuda")
    for call in range(2):
        x = torch.from_numpy(rng.standard_normal((m, k)).astype(np.float32)).cuda().to(xdt)
        nq.check(_call(L, L.nq_linear, w, x, m, bias, epi, ref, 0))
        got = torch.full((m, n_out), float("nan"), device="cuda")
        nq.check(_call(L, L.nq_gemv_noalloc, w, x, m, bias, epi, got, 0))
        torch.cuda.synchronize()
        g, r = got.cpu().numpy(), ref.cpu().numpy()
        assert np.isfinite(g).all(), call
        assert _rel(g, r) <= TOL, (call, _rel(g, r))
        # the reference's semantics on the same inputs (bf16 x as its values)
        want = oracle.epilogue(oracle.matmul_fbgemm_bf16(x.float().cpu().numpy(), blocks, n).astype(np.float64),
                               bias_np, epi)
        assert oracle.max_rel_err(g, want, 1.0) <= TOL, (call, oracle.max_rel_err(g, want, 1.0))
    assert nq.status() == 0


def test_noalloc_is_profiled_like_linear(nq):
    """One nq_gemv_noalloc call is one GEMV-class launch in the library's
    profiler, with the same algorithmic FLOPs and bytes as nq_linear's."""
    L = nq.load()
    rng = np.random.default_rng(9)
    w = _weight(nq, rng, 1024, 1024)
    x = torch.from_numpy(rng.standard_normal((2, 1024)).astype(np.float32)).cuda()
    y = torch.empty((2, 1024), device="cuda")
    nq.check(_call(L, L.nq_linear, w, x, 2, None, 0, y, 0))  # workspace sized outside the profile
    torch.cuda.synchronize()
    nq.profile_read(nq.NQ_KCLASS_GEMV, reset=True)
    nq.profile_enable(True)
    try:
        nq.check(_call(L, L.nq_linear, w, x, 2, None, 0, y, 0))
        a = nq.profile_read(nq.NQ_KCLASS_GEMV, reset=True)
        nq.check(_call(L, L.nq_gemv_noalloc, w, x, 2, None, 0, y, 0))
        b = nq.profile_read(nq.NQ_KCLASS_GEMV, reset=True)
    finally:
        nq.profile_enable(False)
    assert a["launches"] == b["launches"] == 1
    assert a["flops"] == b["flops"] and a["bytes"] == b["bytes"]


def test_noalloc_rejects_oversized_and_wide(nq):
    """Scratch beyond the static array, and M > 16, fail with a clear error."""
    L = nq.load()
    rng = np.random.default_rng(5)
    w = _weight(nq, rng, 256, 65536)  # f32 x of 16 rows: hi + lo planes of 4 MiB > 2 MiB
    x = torch.zeros((16, 65536), device="cuda")
    y = torch.zeros((16, 256), device="cuda")
    rc = _call(L, L.nq_gemv_noalloc, w, x, 16, None, 0, y, 0)
    assert rc == nq.NQ_ERR_SHAPE
    assert "static" in nq.last_error()
    w2 = _weight(nq, rng, 256, 256)
    x2 = torch.zeros((17, 256), device="cuda")
    y2 = torch.zeros((17, 256), device="cuda")
    assert _call(L, L.nq_gemv_noalloc, w2, x2, 17, None, 0, y2, 0) == nq.NQ_ERR_SHAPE
    assert nq.status() == 0
