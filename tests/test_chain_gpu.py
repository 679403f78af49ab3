"""The fused chained path (indexer top-k set -> SparseAttention, one call) against
the two-call sequence it replaces, sa(q, kv, indexer(x, qr, start_pos, offset)):
the outputs must be bit-identical (attention in the multiplicity form depends only
on the selected set, which both paths select with the same canonical rule)."""
import pytest
import torch

from ascendc_kernel_b200 import _native
from ascendc_kernel_b200 import chain
from ascendc_kernel_b200 import indexer as ix
from ascendc_kernel_b200 import sparse_attn as sa

pytestmark = pytest.mark.gpu


def make_case(dev, b, s, t_cache, topk, n_pool, heads, start_pos=0, seed=0, tie_levels=None):
    torch.manual_seed(seed)
    args = ix.ModelArgs(max_batch_size=b, max_seq_len=start_pos + s, dim=1024, index_n_heads=16,
                        index_head_dim=64, index_topk=topk, q_lora_rank=256, rope_head_dim=32)
    freqs = ix.make_freqs_cis(32, start_pos + s)
    g = torch.Generator(device=dev)
    g.manual_seed(seed + 1)
    if tie_levels:
        # few distinct kv_cache values: many candidates share a score
        kvc = torch.randint(-tie_levels, tie_levels + 1, (b, t_cache, 64), device=dev,
                            generator=g).to(torch.bfloat16)
    else:
        kvc = torch.randn(b, t_cache, 64, device=dev, generator=g).to(torch.bfloat16)
    ixm = ix.ModelNew(args, freqs, kvc, 4).to(dev)
    sam = sa.ModelNew(heads, 128).to(dev)
    with torch.no_grad():
        sam.attn_sink.copy_(torch.randn(heads, generator=torch.Generator().manual_seed(seed)))
    x = torch.randn(b, s, 1024, device=dev, generator=g).to(torch.bfloat16)
    qr = torch.randn(b, s, 256, device=dev, generator=g).to(torch.bfloat16)
    q = torch.randn(b, s, heads, 128, device=dev, generator=g).to(torch.bfloat16)
    kv = torch.randn(b, n_pool, 128, device=dev, generator=g).to(torch.bfloat16)
    return ixm, sam, x, qr, q, kv


@pytest.mark.parametrize("b,s,t_cache,topk,n_pool,heads,start_pos,offset,ties", [
    (2, 1024, 256, 64, 256, 64, 0, 0, None),       # causal, n <= k and n > k rows
    (1, 1024, 256, 64, 256, 128, 0, 0, 2),         # heavy score ties at the boundary
    (2, 8, 512, 128, 1024, 64, 2040, 100, None),   # decode: no causal mask, index offset
    (1, 8192, 2048, 512, 2048, 64, 0, 0, 1),       # 2048 candidates, ties
])
def test_chain_equals_two_calls(cuda_device, b, s, t_cache, topk, n_pool, heads, start_pos,
                                offset, ties):
    ixm, sam, x, qr, q, kv = make_case(cuda_device, b, s, t_cache, topk, n_pool, heads,
                                       start_pos=start_pos, tie_levels=ties)
    want = sam(q, kv, ixm(x, qr, start_pos, offset))
    got = chain.indexer_sparse_attn(ixm, sam, x, qr, start_pos, offset, q, kv)
    torch.cuda.synchronize()
    assert torch.equal(got, want)
    assert _native.device_error(cuda_device.index) == 0
    # a second call reuses the cached workspace
    got2 = chain.indexer_sparse_attn(ixm, sam, x, qr, start_pos, offset, q, kv)
    assert torch.equal(got2, want)


def test_chain_long_context_shape(cuda_device):
    """BASELINE configs[3] at batch 1: 16384 tokens, 4096 candidates, top-2048."""
    ixm, sam, x, qr, q, kv = make_case(cuda_device, 1, 16384, 4096, 2048, 4096, 64, seed=3)
    want = sam(q, kv, ixm(x, qr, 0, 0))
    got = chain.indexer_sparse_attn(ixm, sam, x, qr, 0, 0, q, kv)
    torch.cuda.synchronize()
    assert torch.equal(got, want)
    assert _native.device_error(cuda_device.index) == 0


def _oracle_chain(ixm, sam, x, qr, start_pos, offset, q, kv, rows):
    """sparse_attn_ref(q, kv, sink, Model.forward(x, qr, start_pos, offset)) on the CPU
    oracle (reference/task2_v0_ref.py:123-144 feeding reference/task1_v0_ref.py:5-24),
    the attention evaluated on the token positions `rows` only."""
    import numpy as np

    import oracle
    from tests.helpers import to_u16

    b, s = x.shape[:2]
    fc = torch.view_as_real(ixm.freqs_cis[start_pos:start_pos + s].cpu())
    idx = oracle.indexer_fwd(
        to_u16(x), to_u16(qr), to_u16(ixm.wq_b.weight), to_u16(ixm.weights_proj.weight),
        fc[..., 0].contiguous().numpy(), fc[..., 1].contiguous().numpy(), to_u16(ixm.kv_cache),
        n_heads=16, head_dim=64, rope_dim=32, index_topk=ixm.index_topk, start_pos=start_pos,
        ratio=ixm.compress_ratio, offset=offset,
        w_scale=ixm.softmax_scale * ixm.n_heads ** -0.5)
    qs = np.ascontiguousarray(to_u16(q)[:, rows])
    ids = np.ascontiguousarray(idx[:, rows])
    return oracle.sparse_attn(qs, to_u16(kv), ids, sam.attn_sink.detach().cpu().numpy(),
                              sam.softmax_scale)


@pytest.mark.parametrize("b,s,t_cache,topk,n_pool,heads,start_pos,offset,ties,n_rows", [
    # causal, 2048 candidates at the last token, top-512, integer kv_cache: ties
    (1, 8192, 2048, 512, 2048, 64, 0, 0, 1, 192),
    # decode: 2048 candidates for every token, top-1024, index offset into the pool
    (2, 32, 2048, 1024, 2304, 64, 8160, 256, 2, 32),
    # the chained configuration's selection: 4096 candidates, top-2048, 128 heads
    (1, 16, 4096, 2048, 4096, 128, 16368, 0, None, 16),
])
def test_chain_matches_oracle(cuda_device, b, s, t_cache, topk, n_pool, heads, start_pos,
                              offset, ties, n_rows):
    """The fused call against the oracle's indexer -> attention sequence (the
    bitmap hand-off is the part only the fused path has)."""
    import numpy as np

    from tests.helpers import bf16_compare, to_u16

    ixm, sam, x, qr, q, kv = make_case(cuda_device, b, s, t_cache, topk, n_pool, heads,
                                       start_pos=start_pos, seed=11, tie_levels=ties)
    got = chain.indexer_sparse_attn(ixm, sam, x, qr, start_pos, offset, q, kv)
    torch.cuda.synchronize()
    assert _native.device_error(cuda_device.index) == 0
    # rows: the last tokens (most candidates) and an even spread over the rest
    rows = np.unique(np.concatenate([np.linspace(0, s - 1, n_rows // 2).astype(np.int64),
                                     np.arange(max(0, s - n_rows // 2), s)]))
    want = _oracle_chain(ixm, sam, x.cpu(), qr.cpu(), start_pos, offset, q.cpu(), kv.cpu(), rows)
    r = bf16_compare(np.ascontiguousarray(to_u16(got)[:, rows]), want, 1e-2, 1e-2)
    # long-pool attention tolerance (two-piece bf16 P): see test_sparse_attn_gpu.py
    assert r["allclose"], r
    assert r["bit_mismatch"] <= max(4, r["n"] * 1e-2), r
    assert r["max_abs"] <= 4e-3, r
