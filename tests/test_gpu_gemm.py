"""The forward's prefill GEMM (tgkv_gemm.cu) through the C-ABI tg_fwd_gemm_f32.

The reference bridge runs its projections as cublasSgemm in fp32
(cuda/tgai_cuda.cu:473-479).  Here they run on the tensor cores with each fp32
operand split into its tf32 part and the exact remainder (three products), so
the result must be as accurate as an fp32 GEMM: every output is checked
against the float64 product, scaled by sum_k |x_k w_k| (the magnitude an
fp32 dot product's rounding error is proportional to).  Shapes cover one row
(the LM head), the router's 8 columns, K not a multiple of the 32-wide
k-block, partial tiles in both directions, and accumulation into the output
(the residual adds).
"""
import numpy as np
import pytest

import tgkv

pytestmark = pytest.mark.gpu

# per-output error / sum_k |x_k w_k|; an fp32 SGEMM of these sizes lands near
# 1e-7, one tf32 product alone near 1e-3
TOL = 2e-6


def _run(lib, devbuf, M, N, K, accumulate, seed, ldx_pad=0, ldo_pad=0):
    rng = np.random.default_rng(seed)
    ldx, ldo = K + ldx_pad, N + ldo_pad
    x = rng.standard_normal((M, ldx), dtype=np.float32)
    w = rng.standard_normal((N, K), dtype=np.float32) * np.float32(1.0 / np.sqrt(K))
    out0 = rng.standard_normal((M, ldo), dtype=np.float32)
    xd, wd, od = devbuf(x), devbuf(w), devbuf(out0)
    ok = lib.tg_fwd_gemm_f32(M, N, K, xd.ptr, ldx, wd.ptr, K, od.ptr, ldo, accumulate, None)
    assert ok, lib.tg_fwd_last_error().decode()
    got = od.get(np.float32, (M, ldo))
    x64, w64 = x[:, :K].astype(np.float64), w.astype(np.float64)
    ref = x64 @ w64.T + (out0[:, :N].astype(np.float64) if accumulate else 0.0)
    scale = np.abs(x64) @ np.abs(w64).T + (np.abs(out0[:, :N]) if accumulate else 0.0)
    err = float((np.abs(got[:, :N] - ref) / np.maximum(scale, 1e-30)).max())
    # columns past N in a padded output row are never written
    if ldo_pad:
        assert np.array_equal(got[:, N:].view(np.uint32), out0[:, N:].view(np.uint32))
    return err


@pytest.mark.parametrize("M,N,K,acc", [
    (1, 64, 64, 0),            # one row
    (5, 8, 1536, 0),           # the router: 8 experts
    (128, 128, 32, 0),         # one tile, one k-block
    (129, 200, 100, 0),        # partial tiles, K not a multiple of 32
    (512, 2560, 1536, 0),      # Q/K/V of the V2.7-shaped model, 512-token prefill
    (512, 1536, 1536, 1),      # out projection + residual
    (300, 5120, 1536, 0),      # dense W1/W2
    (300, 1536, 2560, 1),      # dense W3 + residual
    (37, 1000, 2048, 1),
])
def test_gemm_matches_float64(cuda, devbuf, M, N, K, acc):
    err = _run(cuda, devbuf, M, N, K, acc, 1000 + M + N + K)
    assert err < TOL, err
    assert cuda.tg_cuda_kv_device_error() == 0


def test_gemm_strided_rows(cuda, devbuf):
    """Input rows with a stride past K and output rows past N (the forward
    writes into wider buffers): only the first N columns are touched."""
    err = _run(cuda, devbuf, 70, 96, 256, 1, 77, ldx_pad=12, ldo_pad=8)
    assert err < TOL, err


def test_gemm_rejects_unsupported_shapes(cuda, devbuf):
    lib = cuda
    b = devbuf(nbytes=4096)
    assert not lib.tg_fwd_gemm_f32(4, 4, 6, b.ptr, 6, b.ptr, 6, b.ptr, 4, 0, None)
    assert b"multiples of 4" in lib.tg_fwd_last_error()
    assert not lib.tg_fwd_gemm_f32(0, 4, 4, b.ptr, 4, b.ptr, 4, b.ptr, 4, 0, None)
