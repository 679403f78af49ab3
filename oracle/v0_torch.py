"""The reference's v0 operators restated as the same sequence of torch ops.

TEST INFRASTRUCTURE ONLY, like the rest of oracle/: imported by tests/ (the
G1 parity gate runs it on torch CUDA on the B200, where the reference itself
cannot travel) and by bench.py's reference arm / cpu_baseline leg (the
reference's PyTorch CPU path timed on the host cores). The product package
never imports it.

Each function issues the ATen ops of the cited v0 lines in the same order
with the same dtypes, so on one device it produces the reference's bits: the
CPU restatement is pinned against the reference's own CPU output by
tests/test_oracle_golden.py (index digests recorded by
tests/golden/make_golden.py). No shape assertion or tiling is added; the ops
run on whatever device their inputs live on.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F


def sparse_attn_v0(q: torch.Tensor, kv: torch.Tensor, sink: torch.Tensor,
                   topk_idxs: torch.Tensor, softmax_scale: float) -> torch.Tensor:
    """sparse_attn_ref (reference/task1_v0_ref.py:5-24): gather the top-k kv rows,
    fp32 scores with the sink logit in the max and the denominator, bf16 output."""
    b, m, h, _ = q.shape
    k = topk_idxs.shape[-1]
    ok = topk_idxs >= 0
    rows = topk_idxs.clamp(min=0).long()
    bsel = torch.arange(b, device=q.device)[:, None, None].expand(b, m, k)
    g = kv[bsel, rows].masked_fill(~ok.unsqueeze(-1), 0.0)
    s = torch.einsum("bmhd,bmtd->bmht", q.float(), g.float()) * softmax_scale
    s = s.masked_fill(~ok.unsqueeze(2), float("-inf"))
    sk = sink.float().view(1, 1, h, 1)
    mx = torch.maximum(torch.amax(s, dim=-1, keepdim=True), sk)
    e = torch.exp(s - mx).masked_fill(~ok.unsqueeze(2), 0.0)
    den = e.sum(dim=-1, keepdim=True) + torch.exp(sk - mx)
    return torch.einsum("bmht,bmtd->bmhd", e / den, g.float()).to(q.dtype)


def rotate_tail_(q: torch.Tensor, freqs_cis: torch.Tensor, rope_dim: int) -> None:
    """apply_rotary_emb on q[..., -rope_dim:] in place (reference/task2_v0_ref.py:93-104):
    interleaved pairs as complex64 times freqs_cis, copied back into the bf16 view."""
    y = q[..., -rope_dim:]
    z = torch.view_as_complex(y.float().unflatten(-1, (-1, 2)))
    f = freqs_cis.view(1, z.size(1), 1, z.size(-1))
    y.copy_(torch.view_as_real(z * f).flatten(-2))


def indexer_v0(wq_b: torch.Tensor, w_proj: torch.Tensor, freqs_cis: torch.Tensor,
               kv_cache: torch.Tensor, x: torch.Tensor, qr: torch.Tensor, start_pos: int,
               offset: int, *, n_heads: int, head_dim: int, rope_dim: int, index_topk: int,
               ratio: int, intermediates: bool = False):
    """Model.forward of reference/task2_v0_ref.py:123-144.

    wq_b [n_heads*head_dim, q_lora] and w_proj [n_heads, dim] bf16 (the
    ColumnParallelLinear weights, world_size 1), freqs_cis [max_seq, rope_dim/2]
    complex64, kv_cache [>=b, >=T, head_dim] bf16. Returns int64 [b, s, K]; with
    intermediates=True also (q after RoPE, weights, masked bf16 scores).
    """
    bsz, seqlen, _ = x.size()
    fc = freqs_cis[start_pos:start_pos + seqlen]
    end_pos = start_pos + seqlen
    q = F.linear(qr, wq_b).unflatten(-1, (n_heads, head_dim))
    rotate_tail_(q, fc, rope_dim)
    w = F.linear(x, w_proj) * (head_dim ** -0.5 * n_heads ** -0.5)
    sc = torch.einsum("bshd,btd->bsht", q, kv_cache[:bsz, :end_pos // ratio])
    sc = (sc.relu_() * w.unsqueeze(-1)).sum(dim=2)
    dev = x.device
    if start_pos == 0:
        lim = torch.arange(1, seqlen + 1, device=dev).unsqueeze(1) // ratio
        masked = torch.arange(seqlen // ratio, device=dev).repeat(seqlen, 1) >= lim
        sc += torch.where(masked, float("-inf"), 0)
    idx = sc.topk(min(index_topk, end_pos // ratio), dim=-1)[1]
    if start_pos == 0:
        lim = torch.arange(1, seqlen + 1, device=dev).unsqueeze(1) // ratio
        idx = torch.where(idx >= lim, -1, idx + offset)
    else:
        idx += offset
    if intermediates:
        return idx, (q, w, sc)
    return idx


def kv_writer_v32(x: torch.Tensor, wk: torch.Tensor, gamma: torch.Tensor, beta: torch.Tensor,
                  freqs_cis: torch.Tensor, kv_cache: torch.Tensor, start_pos: int, ratio: int,
                  rope_dim: int) -> torch.Tensor:
    """The compressed index-key cache the indexer reads (reference/task2_v0_ref.py:
    119,133, kv_cache[:bsz, :end_pos // ratio]; the reference holds no producer),
    after DeepSeek-V3.2-Exp's indexer key path (inference/model.py,
    Indexer.forward: k = wk(x); k = k_norm(k), LayerNorm eps 1e-6 in fp32; RoPE),
    with the rotary dims last as the reference's q (rotate_tail_ above) and each
    block of `ratio` tokens pooled by its mean. x [b, s, dim] bf16, wk [64, dim]
    bf16, gamma/beta [64] fp32, freqs_cis [max_seq, rope_dim/2] complex64. Returns
    a copy of kv_cache with rows start_pos/ratio .. + s//ratio - 1 written."""
    B, S, _ = x.shape
    k = F.linear(x.double(), wk.double()).to(torch.bfloat16)
    k = F.layer_norm(k.float(), (k.shape[-1],), gamma, beta, 1e-6).to(torch.bfloat16)
    if rope_dim:
        rotate_tail_(k.unsqueeze(2), freqs_cis[start_pos:start_pos + S], rope_dim)
    nb = S // ratio
    out = kv_cache.clone()
    if nb:
        pooled = k[:, :nb * ratio].float().view(B, nb, ratio, -1).mean(2).to(torch.bfloat16)
        out[:, start_pos // ratio:start_pos // ratio + nb] = pooled
    return out


def sinkhorn_v0(x: torch.Tensor, repeat: int = 10, eps: float = 1e-6) -> torch.Tensor:
    """Model.forward of reference/task3_v0_ref.py:8-14."""
    y = x.softmax(-1) + eps
    y = y / (y.sum(-2, keepdim=True) + eps)
    for _ in range(repeat - 1):
        y = y / (y.sum(-1, keepdim=True) + eps)
        y = y / (y.sum(-2, keepdim=True) + eps)
    return y
