"""Shared helpers for the GPU parity tests (torch is used only for device memory)."""
import ctypes as C

import numpy as np

import oracle as O
import specdec as S


def dev(arr, device="cuda:0"):
    import torch

    return torch.from_numpy(np.ascontiguousarray(arr)).to(device)


def ptr(t):
    return C.c_void_p(t.data_ptr())


def stream_ptr():
    import torch

    return C.c_void_p(torch.cuda.current_stream().cuda_stream)


def empty(shape, dtype, device="cuda:0"):
    import torch

    return torch.empty(shape, dtype=dtype, device=device)


def zeros(shape, dtype, device="cuda:0"):
    import torch

    return torch.zeros(shape, dtype=dtype, device=device)


def sync():
    import torch

    torch.cuda.synchronize()


def tile_w4(packed: np.ndarray, scales: np.ndarray, N: int, K: int) -> np.ndarray:
    """numpy restatement of the tiled weight layout (8448-byte units)."""
    KG = (K + 127) // 128
    units_n = ((N + 255) // 256) * 2
    Npad, Kpad = units_n * 128, KG * 128
    u = np.full((Npad, Kpad), 8, np.uint32)
    lo = packed & 15
    hi = packed >> 4
    full = np.empty((N, K), np.uint32)
    full[:, 0::2] = lo[:, : (K + 1) // 2]
    full[:, 1::2] = hi[:, : K // 2]
    u[:N, :K] = full
    sc = np.zeros((Npad, KG), np.uint16)
    sc[:N, : scales.shape[1]] = scales
    out = np.zeros((units_n, KG, 8448), np.uint8)
    uu = u.reshape(units_n, 128, KG, 16, 8)  # [un, r, kg, kc, i]
    word = np.zeros((units_n, 128, KG, 16), np.uint32)
    for i in range(8):
        j = i >> 1
        sh = (4 * j + 16) if (i & 1) else (4 * j)
        word |= uu[..., i] << np.uint32(sh)
    words = word.transpose(0, 2, 3, 1)  # [un, kg, kc, r]
    out[:, :, :8192] = words.reshape(units_n, KG, 2048).view(np.uint8).reshape(units_n, KG, 8192)
    out[:, :, 8192:] = sc.reshape(units_n, 128, KG).transpose(0, 2, 1).copy().view(np.uint8).reshape(units_n, KG, 256)
    return out.reshape(-1)


def interleave_gu(gate, up, F: int):
    """Gate/up rows of the fused SwiGLU weight: 128-row blocks alternate
    gate rows 128t.. and up rows 128t.., zero rows (nibbles 8, scale 0) past
    F.  gate/up = (packed [F, K/2], scales [F, G]); returns (packed, scales, N)."""
    units = 2 * ((F + 127) // 128)
    N = 128 * units
    packed = np.full((N, gate[0].shape[1]), 0x88, np.uint8)
    scales = np.zeros((N, gate[1].shape[1]), gate[1].dtype)
    for t in range(units // 2):
        lo, hi = 128 * t, min(F, 128 * t + 128)
        for part, (p, s) in enumerate((gate, up)):
            r0 = 256 * t + 128 * part
            packed[r0:r0 + hi - lo] = p[lo:hi]
            scales[r0:r0 + hi - lo] = s[lo:hi]
    return packed, scales, N


def margin_ok(z: np.ndarray, thr: float = 1e-2) -> bool:
    top = np.sort(z)[-2:]
    return float(top[1] - top[0]) >= thr
