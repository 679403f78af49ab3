"""CPU oracle for the DeepSeek sparse-attention operator path.

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and the
CPU-baseline leg of bench.py as the parity checker. The product package
(ascendc_kernel_b200/) never imports it.

numpy front-end over the C restatement in dsa_oracle.c (built by the Makefile
next to it into oracle/_build/libdsa_oracle.so). bf16 tensors are passed as
uint16 bit patterns.
"""

from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_DIR = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_DIR, "_build", "libdsa_oracle.so")
_LIB = None

_vp = ctypes.c_void_p
_i64 = ctypes.c_int64
_i32 = ctypes.c_int
_f32 = ctypes.c_float
_f64 = ctypes.c_double

_SIGS = {
    "oracle_num_threads": (_i32, []),
    "oracle_set_num_threads": (None, [_i32]),
    "oracle_sinkhorn": (None, [_vp, _vp, _i64, _i32, _i32, _f32]),
    "oracle_sparse_attn": (None, [_vp, _vp, _vp, _i32, _vp, _vp, _i64, _i64, _i32, _i32, _i32,
                                  _i32, _f64]),
    "oracle_linear_bf16": (None, [_vp, _vp, _vp, _i64, _i32, _i32]),
    "oracle_rope": (None, [_vp, _vp, _vp, _i64, _i32, _i32, _i32, _i64]),
    "oracle_scale_bf16": (None, [_vp, _i64, _f32]),
    "oracle_index_topk": (None, [_vp, _vp, _vp, _i64, _vp, _vp, _i64, _i64, _i32, _i32, _i64,
                                 _i32, _i64, _i32, _i64]),
    "oracle_e4m3_array": (None, [_vp, _i64, _vp]),
    "oracle_kv_writer": (None, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i32, _i32,
                                _i64, _i32]),
    "oracle_fp8_quant_rows": (None, [_vp, _i64, _vp, _vp]),
    "oracle_index_topk_fp8": (None, [_vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i32, _i32, _i64,
                                     _i32, _i64, _i32, _i64]),
}


def build() -> str:
    """Compiles dsa_oracle.c with the Makefile beside it (no-op when current)."""
    r = subprocess.run(["make", "-s", "-C", _DIR], capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"oracle build failed:\n{r.stdout}\n{r.stderr}")
    return LIB_PATH


def lib() -> ctypes.CDLL:
    global _LIB
    if _LIB is None:
        if not os.path.exists(LIB_PATH):
            build()
        h = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in _SIGS.items():
            f = getattr(h, name)
            f.restype = res
            f.argtypes = args
        _LIB = h
    return _LIB


def _p(a: np.ndarray) -> int:
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data


def num_threads() -> int:
    return lib().oracle_num_threads()


def set_num_threads(n: int) -> None:
    lib().oracle_set_num_threads(n)


def sinkhorn(x: np.ndarray, repeat: int = 10, eps: float = 1e-6) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    n = x.shape[-1]
    y = np.empty_like(x)
    lib().oracle_sinkhorn(_p(x), _p(y), x.size // (n * n), n, repeat, eps)
    return y


def sparse_attn(q: np.ndarray, kv: np.ndarray, idx: np.ndarray, sink: np.ndarray,
                scale: float) -> np.ndarray:
    """q [B,M,H,D] u16, kv [B,NKV,D] u16, idx [B,M,TOPK] int32/int64, sink [H] f32."""
    q = np.ascontiguousarray(q, dtype=np.uint16)
    kv = np.ascontiguousarray(kv, dtype=np.uint16)
    assert idx.dtype in (np.int32, np.int64)
    idx = np.ascontiguousarray(idx)
    sink = np.ascontiguousarray(sink, dtype=np.float32)
    B, M, H, D = q.shape
    out = np.empty_like(q)
    lib().oracle_sparse_attn(_p(q), _p(kv), _p(idx), idx.itemsize, _p(sink), _p(out), B, M, H,
                             D, kv.shape[1], idx.shape[-1], scale)
    return out


def linear_bf16(x: np.ndarray, w: np.ndarray) -> np.ndarray:
    """bf16(x @ w.T) correctly rounded; x [..., K] u16, w [N, K] u16."""
    x = np.ascontiguousarray(x, dtype=np.uint16)
    w = np.ascontiguousarray(w, dtype=np.uint16)
    K = x.shape[-1]
    N = w.shape[0]
    rows = x.size // K
    out = np.empty(x.shape[:-1] + (N,), dtype=np.uint16)
    lib().oracle_linear_bf16(_p(x), _p(w), _p(out), rows, K, N)
    return out


def rope(q: np.ndarray, cos: np.ndarray, sin: np.ndarray, n_heads: int, head_dim: int,
         rope_dim: int, seqlen: int) -> np.ndarray:
    """Returns a rotated copy of q [rows, n_heads*head_dim] u16."""
    q = np.array(q, dtype=np.uint16, copy=True, order="C")
    cos = np.ascontiguousarray(cos, dtype=np.float32)
    sin = np.ascontiguousarray(sin, dtype=np.float32)
    rows = q.size // (n_heads * head_dim)
    lib().oracle_rope(_p(q), _p(cos), _p(sin), rows, n_heads, head_dim, rope_dim, seqlen)
    return q


def scale_bf16(w: np.ndarray, scale: float) -> np.ndarray:
    w = np.array(w, dtype=np.uint16, copy=True, order="C")
    lib().oracle_scale_bf16(_p(w), w.size, scale)
    return w


def index_topk(q: np.ndarray, w: np.ndarray, kv: np.ndarray, batch: int, seqlen: int,
               n_heads: int, head_dim: int, n_cand: int, topk: int, start_pos: int, ratio: int,
               offset: int, want_scores: bool = False):
    """Scores + causal mask + top-k; returns (idx [B*S, K] int64, scores or None).

    kv is [B, >= n_cand, head_dim] u16 (batch stride taken from its shape).
    """
    q = np.ascontiguousarray(q, dtype=np.uint16)
    w = np.ascontiguousarray(w, dtype=np.uint16)
    kv = np.ascontiguousarray(kv, dtype=np.uint16)
    out = np.empty((batch * seqlen, topk), dtype=np.int64)
    scores = np.empty((batch * seqlen, n_cand), dtype=np.uint16) if want_scores else None
    lib().oracle_index_topk(_p(q), _p(w), _p(kv), kv.shape[1] * head_dim, _p(out),
                            _p(scores) if want_scores else None, batch, seqlen, n_heads,
                            head_dim, n_cand, topk, start_pos, ratio, offset)
    return out, scores


_index_topk = index_topk


def indexer_fwd(x, qr, wq, wp, cos, sin, kv, *, n_heads, head_dim, rope_dim, index_topk,
                start_pos, ratio, offset, w_scale, want_intermediates=False):
    """The whole Model.forward of reference/task2_v0_ref.py:123-144 on the CPU.

    x [B,S,dim] u16, qr [B,S,q_lora] u16, wq [H*Dh, q_lora] u16, wp [H, dim] u16,
    cos/sin [S, rope_dim/2] f32 (positions start_pos..), kv [B, >=T, Dh] u16.
    """
    B, S, _ = x.shape
    T = (start_pos + S) // ratio
    K = min(index_topk, T)
    q = linear_bf16(qr.reshape(B * S, -1), wq)
    q = rope(q, cos, sin, n_heads, head_dim, rope_dim, S)
    w = scale_bf16(linear_bf16(x.reshape(B * S, -1), wp), w_scale)
    idx, scores = _index_topk(q, w, kv, B, S, n_heads, head_dim, T, K, start_pos, ratio, offset,
                              want_scores=want_intermediates)
    idx = idx.reshape(B, S, K)
    if want_intermediates:
        return idx, {"q": q, "w": w, "scores": scores}
    return idx


# ----------------------------------------------------------- fp8 index path
def e4m3(x: np.ndarray) -> np.ndarray:
    """fp32 -> float8_e4m3fn bits (RNE, saturating to +-448)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.empty(x.shape, dtype=np.uint8)
    lib().oracle_e4m3_array(_p(x), x.size, _p(y))
    return y


def fp8_quant_rows(x: np.ndarray):
    """Hadamard rotation + ue8m0 e4m3 quantization of 64-wide bf16 rows.
    x [..., 64] u16. Returns (y u8 [rows, 64], scale f32 [rows])."""
    x = np.ascontiguousarray(x, dtype=np.uint16)
    rows = x.size // 64
    y = np.empty((rows, 64), dtype=np.uint8)
    s = np.empty(rows, dtype=np.float32)
    lib().oracle_fp8_quant_rows(_p(x), rows, _p(y), _p(s))
    return y, s


def index_topk_fp8(q8, wq, k8, ks, batch, seqlen, n_heads, head_dim, n_cand, topk, start_pos,
                   ratio, offset, want_scores=False):
    """fp8 scores + mask + top-k; q8 [B*S*H, Dh] u8, wq [B*S*H] f32, k8 [B*T, Dh] u8,
    ks [B*T] f32. Returns (idx [B*S, K] int64, scores f32 [B*S, T] or None)."""
    q8 = np.ascontiguousarray(q8, dtype=np.uint8)
    wq = np.ascontiguousarray(wq, dtype=np.float32)
    k8 = np.ascontiguousarray(k8, dtype=np.uint8)
    ks = np.ascontiguousarray(ks, dtype=np.float32)
    out = np.empty((batch * seqlen, topk), dtype=np.int64)
    scores = np.empty((batch * seqlen, n_cand), dtype=np.float32) if want_scores else None
    lib().oracle_index_topk_fp8(_p(q8), _p(wq), _p(k8), _p(ks), _p(out),
                                _p(scores) if want_scores else None, batch, seqlen, n_heads,
                                head_dim, n_cand, topk, start_pos, ratio, offset)
    return out, scores


def indexer_fwd_fp8(x, qr, wq, wp, cos, sin, kv, *, n_heads, head_dim, rope_dim, index_topk,
                    start_pos, ratio, offset, w_scale, want_intermediates=False):
    """The fp8 index path end to end: the bf16 projections and RoPE of
    indexer_fwd, then rotation + quantization of q (weights times the q rows'
    scales) and of kv rows 0 .. T-1 of every batch, then index_topk_fp8."""
    B, S, _ = x.shape
    T = (start_pos + S) // ratio
    K = min(index_topk, T)
    q = linear_bf16(qr.reshape(B * S, -1), wq)
    q = rope(q, cos, sin, n_heads, head_dim, rope_dim, S)
    w = scale_bf16(linear_bf16(x.reshape(B * S, -1), wp), w_scale)
    q8, qs = fp8_quant_rows(q.reshape(-1, head_dim))
    wqs = ((w.reshape(-1).astype(np.uint32) << 16).view(np.float32) * qs).astype(np.float32)
    k8, ks = fp8_quant_rows(np.ascontiguousarray(kv[:, :T]).reshape(-1, head_dim))
    idx, scores = index_topk_fp8(q8, wqs, k8, ks, B, S, n_heads, head_dim, T, K, start_pos,
                                 ratio, offset, want_scores=want_intermediates)
    idx = idx.reshape(B, S, K)
    if want_intermediates:
        return idx, {"q": q, "w": w, "q8": q8, "wq": wqs, "k8": k8, "ks": ks, "scores": scores}
    return idx


# --------------------------------------------------------- kv_cache writer
def kv_writer(x, wk, g, b, cos, sin, kv, *, rope_dim, start_pos, ratio):
    """Writes the compressed index keys of x [B, S, dim] u16 into a copy of kv
    [B, T, 64] u16 (entries start_pos/ratio .. start_pos/ratio + S/ratio - 1);
    wk [64, dim] u16, g/b [64] f32, cos/sin [S, rope_dim/2] f32. Returns the copy."""
    x = np.ascontiguousarray(x, dtype=np.uint16)
    wk = np.ascontiguousarray(wk, dtype=np.uint16)
    g = np.ascontiguousarray(g, dtype=np.float32)
    b = np.ascontiguousarray(b, dtype=np.float32)
    cos = np.ascontiguousarray(cos, dtype=np.float32)
    sin = np.ascontiguousarray(sin, dtype=np.float32)
    out = np.array(kv, dtype=np.uint16, copy=True, order="C")
    B, S, dim = x.shape
    lib().oracle_kv_writer(_p(x), _p(wk), _p(g), _p(b), _p(cos), _p(sin), _p(out),
                           out.shape[1] * 64, B, S, dim, rope_dim, start_pos, ratio)
    return out
