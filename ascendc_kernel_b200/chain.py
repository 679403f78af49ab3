"""Chained long-context path: the Lightning Indexer's top-k selection feeding
SparseAttention over a kv pool, in one native call (``dsa_chain_fwd``).

In the reference the two modules run one after the other:
``sa_model(q, kv, ix_model(x, qr, start_pos, offset))`` (the indexer's int64 output,
reference/task2_v0_ref.py:123-144, is the attention's ``topk_idxs``,
reference/task1_v0_ref.py:5-24). Attention in the multiplicity form depends only on
WHICH pool rows a token selected, so the fused call hands the selection over as one
bitmap per token and skips both the sort and the int64 index list; its output is
identical to the two-call sequence on this library.
"""
from __future__ import annotations

import torch

from ._native import call, lib
from . import indexer as _ix
from . import sparse_attn as _sa


def indexer_sparse_attn(ix_model: "_ix.ModelNew", sa_model: "_sa.ModelNew", x: torch.Tensor,
                        qr: torch.Tensor, start_pos: int, offset: int, q: torch.Tensor,
                        kv: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """``sa_model(q, kv, ix_model(x, qr, start_pos, offset))`` in one call.

    x [b, s, dim] and qr [b, s, q_lora_rank] bf16 as for the indexer; q [b, s, heads, 128]
    and kv [b, n_kv, 128] bf16 as for the attention (heads 64 or 128, n_kv <= 4096).
    """
    bsz, seqlen, _ = x.size()
    dev = x.device
    ratio = ix_model.compress_ratio
    T = (start_pos + seqlen) // ratio
    K = min(ix_model.index_topk, T)
    assert x.is_cuda and qr.is_cuda and q.is_cuda and kv.is_cuda, "inputs must be CUDA tensors"
    assert x.dtype == torch.bfloat16 and qr.dtype == torch.bfloat16
    assert q.dtype == torch.bfloat16 and kv.dtype == torch.bfloat16
    assert ix_model.n_local_heads == 16 and ix_model.head_dim == 64, \
        "indexer kernel specialised to index_n_heads == 16, index_head_dim == 64"
    assert 1 <= K and T <= 8192, "1 .. 8192 indexer candidates"
    assert q.shape[0] == bsz and q.shape[1] == seqlen and q.shape[3] == 128
    assert q.shape[2] == sa_model.n_heads and q.shape[2] in (64, 128)
    assert kv.shape[0] == bsz and kv.shape[2] == 128 and 1 <= kv.shape[1] <= 4096
    kvc = ix_model.kv_cache
    assert kvc.is_cuda and kvc.dtype == torch.bfloat16 and kvc.device == dev
    assert kvc.shape[0] >= bsz and kvc.shape[1] >= T and kvc.shape[2] == ix_model.head_dim
    assert kvc.stride(2) == 1 and kvc.stride(1) == ix_model.head_dim
    x, qr, q, kv = x.contiguous(), qr.contiguous(), q.contiguous(), kv.contiguous()
    wq, wp = ix_model._weights_on(dev)
    cos, sin = ix_model._rope_tables(start_pos, seqlen, dev)
    sink = sa_model._sink_on(dev)
    nbytes = lib().dsa_chain_workspace_bytes(bsz, seqlen, ix_model.n_heads, ix_model.head_dim, T)
    # room for a second projection scratch: the q and w projections run concurrently
    nbytes += lib().dsa_indexer_overlap_extra_bytes(bsz * seqlen, ix_model.n_heads,
                                                    ix_model.head_dim)
    ws = ix_model._workspace(nbytes, dev)
    if out is None:
        out = torch.empty_like(q)
    w_scale = ix_model.softmax_scale * ix_model.n_heads ** -0.5
    stream = torch.cuda.current_stream(dev).cuda_stream
    with torch.cuda.device(dev):
        call("dsa_chain_fwd", x.data_ptr(), qr.data_ptr(), wq.data_ptr(), wp.data_ptr(),
             cos.data_ptr(), sin.data_ptr(), kvc.data_ptr(), kvc.stride(0), bsz, seqlen,
             ix_model.dim, ix_model.q_lora_rank, ix_model.n_heads, ix_model.head_dim,
             ix_model.rope_head_dim, ix_model.index_topk, start_pos, ratio, offset,
             float(w_scale), q.data_ptr(), kv.data_ptr(), kv.shape[1], q.shape[2], q.shape[3],
             sink.data_ptr(), float(sa_model.softmax_scale), out.data_ptr(), ws.data_ptr(),
             ws.numel(), stream)
    return out
