"""GPU parity of the few-row W4A16 contraction (specdec_w4a16_gemv) against the
oracle, against the tcgen05 tile kernel on the same weights, and its
determinism: bit-identical on a second run, and mode 1 adds into Y."""
import numpy as np
import pytest

import oracle as O
import specdec as S
from helpers import dev, ptr, stream_ptr, sync, tile_w4, zeros

pytestmark = pytest.mark.gpu
TOL = 2e-3


def _case(M, N, K, seed):
    packed, scales = O.synth_w4(seed, 13, N, K)
    X16 = O.f16_bits(np.random.default_rng(seed + M).standard_normal((M, K)))
    d_tiled = dev(tile_w4(packed, scales, N, K))
    return packed, scales, X16, d_tiled


@pytest.mark.parametrize("M,N,K", [(1, 256, 512), (1, 4096, 4096), (3, 1000, 1376), (5, 4096, 14336), (8, 512, 512),
                                   (9, 2816, 512), (16, 768, 640), (17, 512, 4096), (31, 4096, 4096),
                                   (32, 4096, 4096), (33, 384, 384), (64, 1024, 4096), (64, 512, 128), (2, 128, 8)])
def test_w4a16_gemv_matches_oracle(cuda_device, M, N, K):
    import torch

    packed, scales, X16, d_tiled = _case(M, N, K, seed=M + N)
    ref = O.w4a16_gemm(X16, packed, scales)
    dX = dev(X16)
    Y = zeros((M, N), torch.float32)
    S.check(S.lib().specdec_w4a16_gemv(ptr(dX), M, K, ptr(d_tiled), N, K, ptr(Y), N, 0, stream_ptr()))
    sync()
    y = Y.cpu().numpy()
    np.testing.assert_allclose(y, ref, rtol=TOL, atol=TOL)
    # deterministic, and mode 1 adds
    Y2 = zeros((M, N), torch.float32)
    S.check(S.lib().specdec_w4a16_gemv(ptr(dX), M, K, ptr(d_tiled), N, K, ptr(Y2), N, 0, stream_ptr()))
    S.check(S.lib().specdec_w4a16_gemv(ptr(dX), M, K, ptr(d_tiled), N, K, ptr(Y), N, 1, stream_ptr()))
    sync()
    np.testing.assert_array_equal(Y2.cpu().numpy(), y)
    np.testing.assert_allclose(Y.cpu().numpy(), 2 * y, rtol=1e-6, atol=1e-6)


@pytest.mark.parametrize("M,N,K", [(4, 2048, 2048), (32, 4096, 4096), (64, 1536, 1024)])
def test_w4a16_gemv_matches_tcgen05_tiles(cuda_device, M, N, K):
    """The same weights through the GEMV and through the tensor-core tiles
    (one-unit tiles, k split 2): equal within fp32 summation order."""
    import torch

    _, _, X16, d_tiled = _case(M, N, K, seed=7)
    dX = dev(X16)
    Y1, Y2 = zeros((M, N), torch.float32), zeros((M, N), torch.float32)
    S.check(S.lib().specdec_w4a16_gemv(ptr(dX), M, K, ptr(d_tiled), N, K, ptr(Y1), N, 0, stream_ptr()))
    S.check(S.lib().specdec_w4a16_gemm_with_plan(ptr(dX), M, K, ptr(d_tiled), N, K, ptr(Y2), N, 0, 1, 2,
                                                 stream_ptr()))
    sync()
    np.testing.assert_allclose(Y1.cpu().numpy(), Y2.cpu().numpy(), rtol=1e-4, atol=1e-4)


def test_w4a16_gemv_strided_rows(cuda_device):
    """X and Y with row strides larger than K and N (as the engine's draft
    hidden chain [B, k, H] is read and written one head at a time)."""
    import torch

    M, N, K, ldx, ldy = 6, 768, 1024, 1024 * 3, 768 * 2
    packed, scales, X16, d_tiled = _case(M, N, K, seed=3)
    Xbig = np.zeros((M, ldx), np.uint16)
    Xbig[:, :K] = X16
    dX = dev(Xbig)
    Y = zeros((M, ldy), torch.float32)
    S.check(S.lib().specdec_w4a16_gemv(ptr(dX), M, ldx, ptr(d_tiled), N, K, ptr(Y), ldy, 0, stream_ptr()))
    sync()
    y = Y.cpu().numpy()
    np.testing.assert_allclose(y[:, :N], O.w4a16_gemm(X16, packed, scales), rtol=TOL, atol=TOL)
    assert np.all(y[:, N:] == 0)
