"""kv_cache writer (KVCacheWriter, dsa_kv_cache_write) against the CPU oracle
(oracle.kv_writer), and the written cache read back by the indexer (ModelNew).

The key projection runs on the tensor cores with fp32 accumulation, whose
internal rounding order is not specified, while the oracle rounds each exact
dot product once. So:
- with inputs whose dot products are exact in any fp32 order (small integers
  times multiples of 1/16), the whole chain -- projection, LayerNorm, RoPE,
  block mean -- must be bit-exact;
- with N(0, 1) inputs, outputs must be within atol = rtol = 1e-2 and differ
  from the oracle in at most 1 % of elements (a projection that lands on the
  other side of a bf16 rounding boundary), by at most 2^-7 absolute: one bf16
  step of a projected key near magnitude 1, which LayerNorm carries to the
  normalised key whatever that key's own magnitude (so near zero the difference
  is several of the output's own ulps).
Rows outside the written blocks must be untouched in every case.
"""

import numpy as np
import pytest
import torch

import oracle
from ascendc_kernel_b200 import _native
from ascendc_kernel_b200 import indexer as ix
from tests.helpers import bf16_compare, to_u16

pytestmark = pytest.mark.gpu


def _writer(dim, rope_dim, ratio, exact, seed):
    g = torch.Generator().manual_seed(seed)
    args = ix.ModelArgs(dim=dim, index_head_dim=64, rope_head_dim=rope_dim)
    w = ix.KVCacheWriter(args, ratio)
    with torch.no_grad():
        if exact:
            w.wk.weight.copy_((torch.randint(-8, 9, (64, dim), generator=g) / 16.0))
        else:
            w.wk.weight.copy_(torch.randn(64, dim, generator=g) * dim ** -0.5)
        w.k_norm_weight.copy_(1 + 0.1 * torch.randn(64, generator=g))
        w.k_norm_bias.copy_(0.1 * torch.randn(64, generator=g))
    return w


def _inputs(B, S, dim, T, exact, seed):
    g = torch.Generator().manual_seed(seed + 1)
    if exact:
        x = torch.randint(-3, 4, (B, S, dim), generator=g).to(torch.bfloat16)
    else:
        x = torch.randn(B, S, dim, generator=g).to(torch.bfloat16)
    kv = torch.randn(B, T, 64, generator=g).to(torch.bfloat16)
    return x, kv


def _oracle(w, x, kv, freqs, start_pos, rope_dim, ratio):
    S = x.shape[1]
    fc = torch.view_as_real(freqs[start_pos:start_pos + S])
    return oracle.kv_writer(to_u16(x), to_u16(w.wk.weight.detach()),
                            w.k_norm_weight.detach().numpy(), w.k_norm_bias.detach().numpy(),
                            fc[..., 0].contiguous().numpy(), fc[..., 1].contiguous().numpy(),
                            to_u16(kv), rope_dim=rope_dim, start_pos=start_pos, ratio=ratio)


CASES = [
    # B, S, dim, rope_dim, start_pos, ratio, T
    (2, 256, 1024, 32, 0, 4, 64),     # prefill, the BASELINE indexer's key shape
    (2, 300, 1024, 32, 8, 4, 200),    # offset start, tiles that cross a batch boundary
    (1, 257, 512, 64, 0, 4, 80),      # seqlen not a multiple of the ratio
    (3, 64, 256, 0, 0, 1, 70),        # ratio 1, no rotary dims
    (1, 130, 1024, 32, 16, 8, 40),    # ratio 8
    (1, 640, 2048, 32, 128, 128, 9),  # one block per 128-token tile
    (2, 200, 512, 6, 4, 4, 60),       # 3 rotary pairs: tables staged with scalar loads
]


@pytest.mark.parametrize("case", CASES)
def test_exact_sums_bit_exact(cuda_device, case):
    B, S, dim, rd, sp, r, T = case
    w = _writer(dim, rd, r, exact=True, seed=S + dim)
    x, kv = _inputs(B, S, dim, T, exact=True, seed=S)
    freqs = ix.make_freqs_cis(max(rd, 2), sp + S)
    kvd = kv.to(cuda_device)
    out = w.to(cuda_device)(x.to(cuda_device), sp, freqs, kvd)
    assert out.data_ptr() == kvd.data_ptr()
    assert np.array_equal(to_u16(out), _oracle(w.cpu(), x, kv, freqs, sp, rd, r))
    assert _native.device_error(0) == 0


@pytest.mark.parametrize("case", CASES[:3])
def test_random_within_tolerance(cuda_device, case):
    B, S, dim, rd, sp, r, T = case
    w = _writer(dim, rd, r, exact=False, seed=S + dim)
    x, kv = _inputs(B, S, dim, T, exact=False, seed=S)
    freqs = ix.make_freqs_cis(rd, sp + S)
    got = to_u16(w.to(cuda_device)(x.to(cuda_device), sp, freqs, kv.to(cuda_device)))
    want = _oracle(w.cpu(), x, kv, freqs, sp, rd, r)
    lo, hi = sp // r, sp // r + S // r
    cmp = bf16_compare(got[:, lo:hi], want[:, lo:hi])
    print(f"kv writer {case}: {cmp}")
    assert cmp["allclose"], cmp
    assert cmp["bit_mismatch"] <= cmp["n"] // 100, cmp
    assert cmp["max_abs"] <= 2.0 ** -7, cmp
    keep = np.ones(T, bool)
    keep[lo:hi] = False
    assert np.array_equal(got[:, keep], to_u16(kv)[:, keep])


@pytest.mark.parametrize("case", [
    (1, 4, 64, 32, 0, 4, 1),      # one block, one 64-wide k chunk
    (2, 3, 128, 32, 0, 4, 5),     # fewer tokens than a block: nothing written
    (3, 7, 256, 32, 4, 4, 9),     # decode-sized call: one block per batch, a partial one left
    (2, 128, 256, 64, 0, 128, 3), # one block of 128 tokens per batch
])
def test_small_and_degenerate_calls(cuda_device, case):
    """Edge sizes: a single block, fewer tokens than a block (the cache is left as
    it was), a decode-sized chunk, one 128-token block."""
    B, S, dim, rd, sp, r, T = case
    w = _writer(dim, rd, r, exact=True, seed=S + 7)
    x, kv = _inputs(B, S, dim, T, exact=True, seed=S + 3)
    freqs = ix.make_freqs_cis(rd, sp + S)
    kvd = kv.to(cuda_device)
    w.to(cuda_device)(x.to(cuda_device), sp, freqs, kvd)
    assert np.array_equal(to_u16(kvd), _oracle(w.cpu(), x, kv, freqs, sp, rd, r))
    if S < r:
        assert np.array_equal(to_u16(kvd), to_u16(kv))
    assert _native.device_error(0) == 0


def test_chunked_prefill_equals_one_call(cuda_device):
    """Writing 512 tokens in two calls (start_pos 0 and 256) gives the same cache
    as one call over all 512: every block depends only on its own tokens and
    positions."""
    dev = cuda_device
    w = _writer(1024, 32, 4, exact=False, seed=11).to(dev)
    x, kv = _inputs(2, 512, 1024, 160, exact=False, seed=12)
    freqs = ix.make_freqs_cis(32, 512)
    one = w(x.to(dev), 0, freqs, kv.to(dev).clone())
    two = kv.to(dev).clone()
    w(x[:, :256].contiguous().to(dev), 0, freqs, two)
    w(x[:, 256:].contiguous().to(dev), 256, freqs, two)
    assert torch.equal(one, two)


def test_written_cache_feeds_the_indexer(cuda_device):
    """Prefill: the writer fills kv_cache[:, :S/4]; ModelNew (the reference's
    Model.forward contract) then selects exactly the oracle's indices from that
    cache."""
    dev = cuda_device
    torch.manual_seed(5)
    args = ix.ModelArgs(max_batch_size=2, max_seq_len=512, dim=1024, index_n_heads=16,
                        index_head_dim=64, index_topk=64, q_lora_rank=256, rope_head_dim=32)
    freqs = ix.make_freqs_cis(args.rope_head_dim, args.max_seq_len)
    kv_cache = torch.zeros(2, 128, 64, dtype=torch.bfloat16, device=dev)
    writer = _writer(args.dim, args.rope_head_dim, 4, exact=False, seed=21).to(dev)
    model = ix.ModelNew(args, freqs.to(dev), kv_cache, 4)
    x = torch.randn(2, 512, args.dim).to(torch.bfloat16)
    qr = torch.randn(2, 512, args.q_lora_rank).to(torch.bfloat16)
    writer(x.to(dev), 0, freqs, kv_cache)
    got = model(x.to(dev), qr.to(dev), 0, 0).cpu().numpy()
    fc = torch.view_as_real(freqs)
    want = oracle.indexer_fwd(
        to_u16(x), to_u16(qr), to_u16(model.wq_b.weight.detach().cpu()),
        to_u16(model.weights_proj.weight.detach().cpu()), fc[..., 0].contiguous().numpy(),
        fc[..., 1].contiguous().numpy(), to_u16(kv_cache), n_heads=args.index_n_heads,
        head_dim=args.index_head_dim, rope_dim=args.rope_head_dim, index_topk=args.index_topk,
        start_pos=0, ratio=4, offset=0, w_scale=model.softmax_scale * args.index_n_heads ** -0.5)
    assert np.array_equal(got, want)
