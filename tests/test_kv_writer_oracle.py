"""The kv_cache writer's CPU oracle (oracle.kv_writer) against a torch restatement
of its public definition, DeepSeek-V3.2-Exp's indexer key path
(inference/model.py, Indexer.forward: k = wk(x); k = k_norm(k), a LayerNorm
with eps 1e-6 in fp32; RoPE on the rotary dims), with the rotary dims last as
the reference's q (reference/task2_v0_ref.py:131, apply_rotary_emb at :93-104)
and each block of compress_ratio tokens pooled by its mean into the cache rows
the reference's indexer reads (reference/task2_v0_ref.py:133,
kv_cache[:bsz, :end_pos // ratio]).

The torch side issues the ops of that definition (F.linear, F.layer_norm, the
reference's complex RoPE, mean) on the CPU; the oracle states each rounding
step in C, with the LayerNorm's mean and variance summed in index order.
torch's CPU layer_norm reduces in another order, so its fp32 variance can
differ in the last bit, and a normalised key that lands within that bit of a
bf16 rounding tie rounds the other way: the two agree to one bf16 ulp, and bit
for bit on all but a few in ten thousand elements. Rows outside the written
blocks must be left untouched.
"""

import numpy as np
import pytest
import torch

import oracle
from oracle.v0_torch import kv_writer_v32
from ascendc_kernel_b200 import indexer as ix
from tests.helpers import to_u16


def run_oracle(x, wk, gamma, beta, freqs_cis, kv, start_pos, ratio, rope_dim):
    S = x.shape[1]
    half = max(rope_dim // 2, 1)
    if rope_dim:
        fc = torch.view_as_real(freqs_cis[start_pos:start_pos + S])
        cos, sin = fc[..., 0].contiguous().numpy(), fc[..., 1].contiguous().numpy()
    else:
        cos = sin = np.zeros((S, half), np.float32)
    return oracle.kv_writer(to_u16(x), to_u16(wk), gamma.numpy(), beta.numpy(), cos, sin,
                            to_u16(kv), rope_dim=rope_dim, start_pos=start_pos, ratio=ratio)


def make_case(B, S, dim, rope_dim, start_pos, ratio, T, seed):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(B, S, dim, generator=g).to(torch.bfloat16)
    wk = (torch.randn(64, dim, generator=g) * dim ** -0.5).to(torch.bfloat16)
    gamma = (1 + 0.1 * torch.randn(64, generator=g)).float()
    beta = (0.1 * torch.randn(64, generator=g)).float()
    freqs = ix.make_freqs_cis(max(rope_dim, 2), start_pos + S)
    kv = torch.randn(B, T, 64, generator=g).to(torch.bfloat16)
    return x, wk, gamma, beta, freqs, kv


@pytest.mark.parametrize("B,S,dim,rope_dim,start_pos,ratio,T", [
    (2, 300, 1024, 32, 8, 4, 200),   # decode-style offset, ragged tail (300 % 4 == 0, 300 % 128)
    (1, 257, 512, 64, 0, 4, 80),     # seqlen not a multiple of the ratio: the last token is not pooled
    (3, 64, 256, 0, 0, 1, 70),       # ratio 1 (every token written), no rotary dims
    (1, 130, 1024, 32, 16, 8, 40),   # ratio 8
])
def test_oracle_matches_torch_restatement(B, S, dim, rope_dim, start_pos, ratio, T):
    x, wk, gamma, beta, freqs, kv = make_case(B, S, dim, rope_dim, start_pos, ratio, T, seed=S)
    got = run_oracle(x, wk, gamma, beta, freqs, kv, start_pos, ratio, rope_dim)
    want = to_u16(kv_writer_v32(x, wk, gamma, beta, freqs, kv, start_pos, ratio, rope_dim))
    ulps = np.abs(got.astype(np.int32) - want.astype(np.int32))
    assert ulps.max() <= 1
    assert (ulps != 0).sum() <= max(2, got.size // 2000)
    # rows outside [start_pos / ratio, start_pos / ratio + S // ratio) keep their contents
    lo, hi = start_pos // ratio, start_pos // ratio + S // ratio
    keep = np.ones(T, bool)
    keep[lo:hi] = False
    assert np.array_equal(got[:, keep], to_u16(kv)[:, keep])
