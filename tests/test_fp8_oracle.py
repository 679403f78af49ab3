"""CPU checks of the fp8 index path's oracle (oracle/dsa_oracle.c, fp8 section).

The path itself has no reference output to pin against (the reference declares
ModelArgs.dtype = "fp8" / scale_fmt = "ue8m0" but never runs it), so the oracle's
pieces are pinned against independent implementations: the e4m3 conversion
against torch's float8_e4m3fn cast, the rotation against a Sylvester Hadamard
matrix product, the ue8m0 scale against its definition, and the score against
a numpy restatement.
"""

import numpy as np
import torch

import oracle


def _bf16(a: np.ndarray) -> np.ndarray:
    return torch.from_numpy(np.ascontiguousarray(a, np.float32)).to(torch.bfloat16).view(
        torch.int16).numpy().view(np.uint16)


def _f32(u16: np.ndarray) -> np.ndarray:
    return (u16.astype(np.uint32) << 16).view(np.float32)


def test_e4m3_matches_torch_cast():
    g = np.random.default_rng(1)
    x = (g.standard_normal(100_000) * np.exp2(g.integers(-16, 10, 100_000))).astype(np.float32)
    edges = np.array([0.0, -0.0, 2 ** -10, 3 * 2 ** -10, 2 ** -9, 2 ** -6, 2 ** -6 * 0.999,
                      447.9, 448.0, 1.0625, 1.1875, -1.0625], np.float32)
    x = np.concatenate([x, edges])
    want = torch.from_numpy(np.clip(x, -448, 448)).to(torch.float8_e4m3fn).view(
        torch.uint8).numpy()
    assert np.array_equal(oracle.e4m3(x), want)
    # saturation: beyond 448 the oracle clamps (the kernels' satfinite)
    assert oracle.e4m3(np.array([1e9, -1e9], np.float32)).tolist() == [0x7E, 0xFE]


def _hadamard64() -> np.ndarray:
    h = np.array([[1.0]])
    for _ in range(6):
        h = np.block([[h, h], [h, -h]])
    return h


def test_quant_rows_rotation_and_scale():
    g = np.random.default_rng(2)
    x = g.standard_normal((500, 64)).astype(np.float32)
    x[0] = 0.0                       # all-zero row: amax clamps to 1e-4
    x[1] *= 1e-30                    # tiny row
    x[2] *= 1e30                     # huge row
    xb = _bf16(x)
    y, s = oracle.fp8_quant_rows(xb)
    # scales are powers of two >= amax / 448 and < 2 amax / 448
    h = _f32(_bf16((_f32(xb).astype(np.float64) @ _hadamard64().T * 0.125).astype(np.float32)))
    amax = np.maximum(np.abs(h).max(1), np.float32(1e-4))
    mant, _ = np.frexp(s)
    assert np.all(mant == 0.5)
    assert np.all(s >= amax / 448) and np.all(s < 2 * amax / 448)
    # dequantized values lie within half an e4m3 ulp of the rotated row
    deq = torch.from_numpy(y.copy()).view(torch.float8_e4m3fn).float().numpy() * s[:, None]
    tol = np.maximum(np.abs(h) * 2.0 ** -4, s[:, None] * 2.0 ** -10) * 1.0001
    ok = np.abs(deq - h) <= tol
    # rows whose fp32 butterflies rounded (wide exponent spread) may differ from
    # the fp64 matrix product by a bf16 ulp before quantization
    assert ok[3:].mean() > 0.999
    assert np.all(y[0] == 0)


def test_index_scores_match_numpy_restatement():
    g = np.random.default_rng(3)
    B, S, T, H, D, K = 2, 40, 10, 16, 64, 6
    q8, qs = oracle.fp8_quant_rows(_bf16(g.standard_normal((B * S * H, D))))
    k8, ks = oracle.fp8_quant_rows(_bf16(g.standard_normal((B * T, D))))
    wq = (g.standard_normal(B * S * H) * 0.1).astype(np.float32) * qs
    idx, sc = oracle.index_topk_fp8(q8, wq, k8, ks, B, S, H, D, T, K, 0, 4, 5,
                                    want_scores=True)
    qd = torch.from_numpy(q8.copy()).view(torch.float8_e4m3fn).double().numpy().reshape(
        B, S, H, D)
    kd = torch.from_numpy(k8.copy()).view(torch.float8_e4m3fn).double().numpy().reshape(B, T, D)
    dots = np.einsum("bshd,btd->bsht", qd, kd).astype(np.float32)
    w = wq.reshape(B, S, H)
    acc = np.zeros((B, S, T), np.float32)
    for h in range(H):  # fma chain: fp64 product + accumulator, rounded once (exact fma)
        acc = (np.maximum(dots[:, :, h], 0).astype(np.float64) * w[:, :, h, None]
               + acc.astype(np.float64)).astype(np.float32)
    want = (acc * ks.reshape(B, 1, T)).reshape(B * S, T)
    t = np.arange(S)
    valid = (np.arange(T)[None, :] < np.minimum((t[:, None] + 1) // 4, T))
    valid = np.tile(valid, (B, 1))
    assert np.array_equal(sc[valid], want[valid])
    assert np.all(np.isneginf(sc[~valid]))
    for r in range(B * S):
        nv = int(valid[r].sum())
        order = sorted(range(nv), key=lambda k: (-(want[r, k] + 0.0), k))
        exp = [k + 5 for k in order[:K]] + [-1] * max(0, K - nv)
        assert idx[r].tolist() == exp[:K]
