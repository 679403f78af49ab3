"""SparseAttention drop-in for the reference's Task 1 operator.

Mirrors ``reference/task1_v0_ref.py`` (``sparse_attn_ref``, ``Model``,
``get_inputs``, ``get_init_inputs``) and the v1 ``ModelNew`` of
``src/task1_sparse_attn.py:666-804``: same constructor arguments, same
``attn_sink`` parameter, same ``forward(q, kv, topk_idxs)`` signature. The
compute runs in the fused sm_100a kernel behind ``dsa_sparse_attn_fwd``.

Shape preconditions are checked with ``assert`` like the reference v1
(``src/task1_sparse_attn.py:757-761``); CUDA-level failures raise DsaError.
"""

from __future__ import annotations

import torch
import torch.nn as nn

from ._native import call

SUPPORTED_HEADS = (16, 32, 64, 128)


def sparse_attn(q: torch.Tensor, kv: torch.Tensor, attn_sink: torch.Tensor,
                topk_idxs: torch.Tensor, softmax_scale: float,
                out: torch.Tensor | None = None) -> torch.Tensor:
    """out[b,t,h] = sum_j softmax_j(q.kv[idx_j] * scale ++ sink[h]) kv[idx_j].

    q [b, m, h, 128] bf16, kv [b, n_kv, 128] bf16, topk_idxs [b, m, topk]
    int32 or int64 (negative = masked), attn_sink [h] fp32. Returns bf16 like q.
    Same semantics as ``sparse_attn_ref`` (reference/task1_v0_ref.py:5-24).
    Two kernels: n_kv <= 32 with topk <= 128 (the BASELINE shape), and a chunked
    one for long kv pools (n_kv <= 4096, any topk, 64 or 128 heads).
    """
    assert q.is_cuda and kv.is_cuda and topk_idxs.is_cuda, "inputs must be CUDA tensors"
    assert q.dtype == torch.bfloat16 and kv.dtype == torch.bfloat16, "q and kv must be bf16"
    assert topk_idxs.dtype in (torch.int32, torch.int64), "topk_idxs must be int32 or int64"
    b, m, h, d = q.shape
    assert kv.dim() == 3 and kv.shape[0] == b and kv.shape[2] == d, "kv must be [b, n_kv, d]"
    assert topk_idxs.shape[:2] == (b, m), "topk_idxs must be [b, m, topk]"
    assert d == 128, "kernel specialised to head_dim == 128"
    assert h in SUPPORTED_HEADS, f"kernel specialised to n_heads in {SUPPORTED_HEADS}"
    topk = topk_idxs.shape[-1]
    if kv.shape[1] <= 32 and topk <= 128:
        assert (topk * topk_idxs.element_size()) % 16 == 0, \
            "topk * sizeof(index) must be a multiple of 16 bytes"
    else:
        assert kv.shape[1] <= 4096 and h in (64, 128), \
            "long kv pools: n_kv <= 4096 and n_heads in (64, 128)"
    q = q.contiguous()
    kv = kv.contiguous()
    topk_idxs = topk_idxs.contiguous()
    sink = attn_sink.detach()
    if sink.device != q.device or sink.dtype != torch.float32 or not sink.is_contiguous():
        sink = sink.to(device=q.device, dtype=torch.float32).contiguous()
    assert sink.numel() == h, "attn_sink must have n_heads entries"
    if out is None:
        out = torch.empty_like(q)
    stream = torch.cuda.current_stream(q.device).cuda_stream
    with torch.cuda.device(q.device):
        call("dsa_sparse_attn_fwd", q.data_ptr(), kv.data_ptr(), topk_idxs.data_ptr(),
             topk_idxs.element_size(), sink.data_ptr(), out.data_ptr(), b, m, h, d, kv.shape[1],
             topk, float(softmax_scale), stream)
    return out


class ModelNew(nn.Module):
    """Drop-in for ``Model`` of reference/task1_v0_ref.py:27-36."""

    def __init__(self, n_heads: int, head_dim: int):
        super().__init__()
        self.n_heads = n_heads
        self.head_dim = head_dim
        self.softmax_scale = head_dim ** -0.5
        self.attn_sink = nn.Parameter(torch.zeros(n_heads, dtype=torch.float32))
        self._sink_cache = None  # (device, version, tensor)

    def _sink_on(self, device: torch.device) -> torch.Tensor:
        ver = self.attn_sink._version
        c = self._sink_cache
        if c is None or c[0] != device or c[1] != ver or c[3] is not self.attn_sink:
            t = self.attn_sink.detach().to(device=device, dtype=torch.float32).contiguous()
            self._sink_cache = (device, ver, t, self.attn_sink)
        return self._sink_cache[2]

    def forward(self, q: torch.Tensor, kv: torch.Tensor, topk_idxs: torch.Tensor) -> torch.Tensor:
        assert q.shape[2] == self.n_heads and q.shape[3] == self.head_dim
        return sparse_attn(q, kv, self._sink_on(q.device), topk_idxs, self.softmax_scale)


# Reference configuration (reference/task1_v0_ref.py:39-55).
batch_size = 8
seq_len = 2600
n_kv = 32
n_heads = 64
head_dim = 128
topk = 16


def get_inputs():
    q = torch.randn(batch_size, seq_len, n_heads, head_dim, dtype=torch.bfloat16)
    kv = torch.randn(batch_size, n_kv, head_dim, dtype=torch.bfloat16)
    topk_idxs = torch.randint(0, n_kv, (batch_size, seq_len, topk), dtype=torch.int32)
    return [q, kv, topk_idxs]


def get_init_inputs():
    return [n_heads, head_dim]
