"""Lightning Indexer drop-in for the reference's Task 2 operator.

Mirrors ``reference/task2_v0_ref.py`` -- ``ModelArgs``, ``Linear``,
``ColumnParallelLinear``, ``Model(args, freqs_cis, kv_cache, compress_ratio)``,
``forward(x, qr, start_pos, offset) -> int64``, ``_make_args``, ``get_inputs``,
``get_init_inputs`` -- and the v1 ``ModelNew`` of ``src/task2_indexer.py:1011-1349``.
Parameters are created in the reference's order (wq_b, then weights_proj, each
kaiming_uniform(a=sqrt(5))) so a seeded construction yields the same weights.

The forward is one call of ``dsa_indexer_fwd``: q projection + RoPE, weights
projection, then the fused score / causal mask / top-k kernel. Indices are
bit-exact to the rounding contract of include/dsa_b200.h, ties broken by
ascending candidate index.
"""

from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Literal, Tuple

import torch
import torch.nn.functional as F
from torch import nn

from ._native import call, lib

world_size = 1
rank = 0


@dataclass
class ModelArgs:
    """Configuration object with the fields of reference/task2_v0_ref.py:21-61.

    Only dim, index_n_heads, index_head_dim, rope_head_dim, index_topk and
    q_lora_rank are read by the indexer; the other fields are kept so that code
    written against the reference's dataclass keeps working.
    """

    max_batch_size: int = 4
    max_seq_len: int = 4096
    dtype: Literal["bf16", "fp8"] = "fp8"
    scale_fmt: Literal[None, "ue8m0"] = "ue8m0"
    expert_dtype: Literal[None, "fp4"] = None
    scale_dtype: Literal["fp32", "fp8"] = "fp8"
    vocab_size: int = 129280
    dim: int = 4096
    moe_inter_dim: int = 4096
    n_layers: int = 7
    n_hash_layers: int = 0
    n_mtp_layers: int = 1
    n_heads: int = 64
    n_routed_experts: int = 8
    n_shared_experts: int = 1
    n_activated_experts: int = 2
    score_func: Literal["softmax", "sigmoid", "sqrtsoftplus"] = "sqrtsoftplus"
    route_scale: float = 1.0
    swiglu_limit: float = 0.0
    q_lora_rank: int = 1024
    head_dim: int = 512
    rope_head_dim: int = 64
    norm_eps: float = 1e-6
    o_groups: int = 8
    o_lora_rank: int = 1024
    window_size: int = 128
    compress_ratios: Tuple[int, ...] = (0, 0, 4, 128, 4, 128, 4, 0)
    compress_rope_theta: float = 40000.0
    original_seq_len: int = 0
    rope_theta: float = 10000.0
    rope_factor: float = 40
    beta_fast: int = 32
    beta_slow: int = 1
    index_n_heads: int = 64
    index_head_dim: int = 128
    index_topk: int = 512
    hc_mult: int = 4
    hc_sinkhorn_iters: int = 20
    hc_eps: float = 1e-6


class Linear(nn.Module):
    """Bias-free bf16 linear layer with the reference's initialisation
    (reference/task2_v0_ref.py:63-80)."""

    def __init__(self, in_features: int, out_features: int, bias: bool = False, dtype=None):
        super().__init__()
        assert not bias, "the indexer's projections have no bias"
        self.in_features = in_features
        self.out_features = out_features
        self.weight = nn.Parameter(torch.empty(out_features, in_features,
                                               dtype=dtype or torch.bfloat16))
        nn.init.kaiming_uniform_(self.weight, a=math.sqrt(5))
        self.register_parameter("scale", None)
        self.register_parameter("bias", None)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return F.linear(x, self.weight)


class ColumnParallelLinear(Linear):
    """Column-split linear (reference/task2_v0_ref.py:85-91); world_size is 1."""

    def __init__(self, in_features, out_features, bias=False, dtype=None):
        assert out_features % world_size == 0
        self.part_out_features = out_features // world_size
        super().__init__(in_features, self.part_out_features, bias, dtype)


class ModelNew(nn.Module):
    """Drop-in for ``Model`` of reference/task2_v0_ref.py:106-144."""

    def __init__(self, args, freqs_cis: torch.Tensor, kv_cache: torch.Tensor,
                 compress_ratio: int = 4, fp8_index: bool = False):
        """``fp8_index=True`` selects the fp8 index path that ModelArgs.dtype =
        "fp8" / scale_fmt = "ue8m0" declares (reference/task2_v0_ref.py:25-26):
        q and kv_cache rows are Hadamard-rotated and quantized to e4m3 with
        power-of-two scales and scored on the fp8 tensor cores
        (dsa_indexer_fwd_fp8). The default is the reference's bf16 path
        (reference/task2_v0_ref.py:123-144), bit-exact."""
        super().__init__()
        self.fp8_index = bool(fp8_index)
        self.dim = args.dim
        self.n_heads = args.index_n_heads
        self.n_local_heads = args.index_n_heads // world_size
        self.head_dim = args.index_head_dim
        self.rope_head_dim = args.rope_head_dim
        self.index_topk = args.index_topk
        self.q_lora_rank = args.q_lora_rank
        self.wq_b = ColumnParallelLinear(self.q_lora_rank, self.n_heads * self.head_dim)
        self.weights_proj = ColumnParallelLinear(self.dim, self.n_heads, dtype=torch.bfloat16)
        self.softmax_scale = self.head_dim ** -0.5
        self.compress_ratio = compress_ratio
        self.kv_cache = kv_cache
        self.freqs_cis = freqs_cis
        self._dev_cache = {}

    # -- cached device-side operands ---------------------------------------
    def _weights_on(self, device):
        key = ("w", device)
        vers = (self.wq_b.weight._version, self.weights_proj.weight._version,
                id(self.wq_b.weight), id(self.weights_proj.weight))
        c = self._dev_cache.get(key)
        if c is None or c[0] != vers:
            wq = self.wq_b.weight.detach().to(device=device, dtype=torch.bfloat16).contiguous()
            wp = self.weights_proj.weight.detach().to(device=device,
                                                      dtype=torch.bfloat16).contiguous()
            c = (vers, wq, wp)
            self._dev_cache[key] = c
        return c[1], c[2]

    def _rope_tables(self, start_pos: int, seqlen: int, device):
        key = ("rope", start_pos, seqlen, device, id(self.freqs_cis))
        c = self._dev_cache.get(key)
        if c is None:
            fc = torch.view_as_real(self.freqs_cis[start_pos:start_pos + seqlen])
            cos = fc[..., 0].to(device=device, dtype=torch.float32).contiguous()
            sin = fc[..., 1].to(device=device, dtype=torch.float32).contiguous()
            c = (cos, sin)
            self._dev_cache[key] = c
        return c

    def _workspace(self, nbytes: int, device) -> torch.Tensor:
        key = ("ws", device)
        c = self._dev_cache.get(key)
        if c is None or c.numel() < nbytes:
            c = torch.empty(max(nbytes, 256), dtype=torch.uint8, device=device)
            self._dev_cache[key] = c
        return c

    def forward(self, x: torch.Tensor, qr: torch.Tensor, start_pos: int, offset: int):
        bsz, seqlen, _ = x.size()
        dev = x.device
        ratio = self.compress_ratio
        end_pos = start_pos + seqlen
        T = end_pos // ratio
        K = min(self.index_topk, T)
        assert x.is_cuda and qr.is_cuda, "inputs must be CUDA tensors"
        assert x.dtype == torch.bfloat16 and qr.dtype == torch.bfloat16
        assert self.n_local_heads == 16 and self.head_dim == 64, \
            "kernel specialised to index_n_heads == 16, index_head_dim == 64"
        assert self.rope_head_dim % 2 == 0 and self.rope_head_dim <= self.head_dim
        assert T <= (1024 if self.fp8_index else 8192), "candidate count above the kernels' limit"
        if self.fp8_index:
            assert K <= 256, "the fp8 path selects up to 256 candidates"
        assert K >= 1, "need at least one candidate (end_pos >= compress_ratio)"
        kv = self.kv_cache
        assert kv.is_cuda and kv.dtype == torch.bfloat16 and kv.device == dev
        assert kv.shape[0] >= bsz and kv.shape[1] >= T and kv.shape[2] == self.head_dim
        assert kv.stride(2) == 1 and kv.stride(1) == self.head_dim, \
            "kv_cache rows must be contiguous"
        x = x.contiguous()
        qr = qr.contiguous()
        wq, wp = self._weights_on(dev)
        cos, sin = self._rope_tables(start_pos, seqlen, dev)
        if self.fp8_index:
            nbytes = lib().dsa_indexer_fp8_workspace_bytes(bsz, seqlen, self.n_heads,
                                                           self.head_dim, T)
            fn = "dsa_indexer_fwd_fp8"
        else:
            nbytes = lib().dsa_indexer_workspace_bytes(bsz, seqlen, self.n_heads, self.head_dim,
                                                       T, K)
            fn = "dsa_indexer_fwd"
        # room for a second projection scratch: the q and w projections run concurrently
        nbytes += lib().dsa_indexer_overlap_extra_bytes(bsz * seqlen, self.n_heads, self.head_dim)
        ws = self._workspace(nbytes, dev)
        out = torch.empty(bsz, seqlen, K, dtype=torch.int64, device=dev)
        w_scale = self.softmax_scale * self.n_heads ** -0.5
        stream = torch.cuda.current_stream(dev).cuda_stream
        with torch.cuda.device(dev):
            call(fn, x.data_ptr(), qr.data_ptr(), wq.data_ptr(), wp.data_ptr(),
                 cos.data_ptr(), sin.data_ptr(), kv.data_ptr(), kv.stride(0), out.data_ptr(),
                 ws.data_ptr(), ws.numel(), bsz, seqlen, self.dim, self.q_lora_rank,
                 self.n_heads, self.head_dim, self.rope_head_dim, self.index_topk, start_pos,
                 ratio, offset, float(w_scale), stream)
        return out


class KVCacheWriter(nn.Module):
    """Producer of the compressed index-key cache that ``ModelNew`` reads
    (reference/task2_v0_ref.py:119,133 read kv_cache[:bsz, :end_pos // ratio];
    the reference holds no producer). After DeepSeek-V3.2-Exp's indexer key path
    (inference/model.py, Indexer.forward: wk, LayerNorm ``k_norm``, RoPE), with the
    rotary dims last as this reference's q and each block of ``compress_ratio``
    tokens pooled by its mean (dsa_kv_cache_write)."""

    def __init__(self, args, compress_ratio: int = 4):
        super().__init__()
        self.dim = args.dim
        self.head_dim = args.index_head_dim
        self.rope_head_dim = args.rope_head_dim
        self.compress_ratio = compress_ratio
        self.wk = Linear(self.dim, self.head_dim)
        self.k_norm_weight = nn.Parameter(torch.ones(self.head_dim, dtype=torch.float32))
        self.k_norm_bias = nn.Parameter(torch.zeros(self.head_dim, dtype=torch.float32))
        self._dev_cache = {}

    def _operands(self, freqs_cis: torch.Tensor, start_pos: int, seqlen: int, device):
        """Device copies of wk, the LayerNorm affine and the RoPE tables, cached
        until a parameter changes (the reference's weights live on the host)."""
        vers = tuple((p._version, id(p), p.data_ptr())
                     for p in (self.wk.weight, self.k_norm_weight, self.k_norm_bias))
        key = (device, start_pos, seqlen, id(freqs_cis), vers)
        c = self._dev_cache.get("ops")
        if c is None or c[0] != key:
            fc = torch.view_as_real(freqs_cis[start_pos:start_pos + seqlen])
            c = (key,
                 self.wk.weight.detach().to(device=device, dtype=torch.bfloat16).contiguous(),
                 self.k_norm_weight.detach().to(device=device, dtype=torch.float32).contiguous(),
                 self.k_norm_bias.detach().to(device=device, dtype=torch.float32).contiguous(),
                 fc[..., 0].to(device=device, dtype=torch.float32).contiguous(),
                 fc[..., 1].to(device=device, dtype=torch.float32).contiguous())
            self._dev_cache["ops"] = c
        return c[1:]

    def forward(self, x: torch.Tensor, start_pos: int, freqs_cis: torch.Tensor,
                kv_cache: torch.Tensor) -> torch.Tensor:
        """Writes kv_cache[:bsz, start_pos // r : (start_pos + seqlen) // r] (complete
        blocks of r = compress_ratio tokens; start_pos a multiple of r) and returns it."""
        bsz, seqlen, _ = x.size()
        r = self.compress_ratio
        dev = x.device
        assert x.is_cuda and x.dtype == torch.bfloat16 and kv_cache.dtype == torch.bfloat16
        assert kv_cache.device == dev
        assert kv_cache.stride(2) == 1 and kv_cache.stride(1) == self.head_dim
        assert start_pos % r == 0, "start_pos must be a multiple of compress_ratio"
        wk, g, b, cos, sin = self._operands(freqs_cis, start_pos, seqlen, dev)
        x = x.contiguous()
        stream = torch.cuda.current_stream(dev).cuda_stream
        with torch.cuda.device(dev):
            call("dsa_kv_cache_write", x.data_ptr(), wk.data_ptr(), g.data_ptr(), b.data_ptr(),
                 cos.data_ptr(), sin.data_ptr(), kv_cache.data_ptr(), kv_cache.stride(0),
                 kv_cache.shape[1], bsz, seqlen, self.dim, self.head_dim, self.rope_head_dim,
                 start_pos, r, stream)
        return kv_cache


def qproj_rope(qr: torch.Tensor, wq: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor,
               n_heads: int, head_dim: int, rope_dim: int, seqlen: int) -> torch.Tensor:
    """q = RoPE(bf16(qr @ wq.T)) with correctly rounded bf16 (dsa_indexer_qproj_rope).

    qr [rows, q_lora_rank] bf16, wq [n_heads*head_dim, q_lora_rank] bf16,
    cos/sin [seqlen, rope_dim/2] fp32 (row r at position r % seqlen).
    """
    qr = qr.contiguous()
    rows = qr.numel() // qr.shape[-1]
    out = torch.empty(rows, n_heads * head_dim, dtype=torch.bfloat16, device=qr.device)
    nbytes = lib().dsa_indexer_workspace_bytes(rows, 1, n_heads, head_dim, 0, 0)
    ws = torch.empty(nbytes, dtype=torch.uint8, device=qr.device)
    stream = torch.cuda.current_stream(qr.device).cuda_stream
    with torch.cuda.device(qr.device):
        call("dsa_indexer_qproj_rope", qr.data_ptr(), wq.contiguous().data_ptr(),
             cos.contiguous().data_ptr(), sin.contiguous().data_ptr(), out.data_ptr(), rows,
             qr.shape[-1], n_heads, head_dim, rope_dim, seqlen, ws.data_ptr(), nbytes, stream)
    return out


def wproj(x: torch.Tensor, wp: torch.Tensor, scale: float) -> torch.Tensor:
    """w = bf16(bf16(x @ wp.T) * scale) with correct rounding (dsa_indexer_wproj)."""
    x = x.contiguous()
    rows = x.numel() // x.shape[-1]
    out = torch.empty(rows, wp.shape[0], dtype=torch.bfloat16, device=x.device)
    nbytes = lib().dsa_indexer_wproj_workspace_bytes(rows, x.shape[-1])
    ws = torch.empty(max(nbytes, 256), dtype=torch.uint8, device=x.device)
    stream = torch.cuda.current_stream(x.device).cuda_stream
    with torch.cuda.device(x.device):
        call("dsa_indexer_wproj", x.data_ptr(), wp.contiguous().data_ptr(), out.data_ptr(), rows,
             x.shape[-1], wp.shape[0], float(scale), ws.data_ptr(), ws.numel(), stream)
    return out


def score_topk(q: torch.Tensor, w: torch.Tensor, kv_cache: torch.Tensor, batch: int,
               seqlen: int, n_cand: int, topk: int, start_pos: int, ratio: int,
               offset: int) -> torch.Tensor:
    """Scores, causal mask and top-k indices (dsa_indexer_score_topk).

    q [batch*seqlen, 16*64] bf16, w [batch*seqlen, 16] bf16, kv_cache [>=batch, >=n_cand, 64]
    bf16 with contiguous rows. Returns int64 [batch, seqlen, topk].
    """
    assert kv_cache.stride(2) == 1 and kv_cache.stride(1) == kv_cache.shape[2]
    out = torch.empty(batch, seqlen, topk, dtype=torch.int64, device=q.device)
    stream = torch.cuda.current_stream(q.device).cuda_stream
    with torch.cuda.device(q.device):
        nbytes = lib().dsa_indexer_score_workspace_bytes(batch, seqlen, n_cand, topk)
        ws = torch.empty(max(nbytes, 1), dtype=torch.uint8, device=q.device)
        call("dsa_indexer_score_topk", q.contiguous().data_ptr(), w.contiguous().data_ptr(),
             kv_cache.data_ptr(), kv_cache.stride(0), out.data_ptr(), batch, seqlen, 16, 64,
             n_cand, topk, start_pos, ratio, offset, ws.data_ptr(), nbytes, stream)
    return out


def fp8_quant_rows(x: torch.Tensor, w: torch.Tensor = None):
    """Hadamard rotation + ue8m0 e4m3 quantization of 64-wide bf16 rows
    (dsa_indexer_fp8_quant_rows). x [..., 64] bf16 contiguous. Returns (y uint8
    [rows, 64] e4m3 bits, scale f32 [rows]) and, with w (bf16, one per row),
    also w * scale (f32 [rows])."""
    x = x.contiguous()
    rows = x.numel() // 64
    y = torch.empty(rows, 64, dtype=torch.uint8, device=x.device)
    sc = torch.empty(rows, dtype=torch.float32, device=x.device)
    wo = None
    if w is not None:
        w = w.contiguous()
        assert w.numel() == rows and w.dtype == torch.bfloat16
        wo = torch.empty(rows, dtype=torch.float32, device=x.device)
    stream = torch.cuda.current_stream(x.device).cuda_stream
    with torch.cuda.device(x.device):
        call("dsa_indexer_fp8_quant_rows", x.data_ptr(), rows, rows, 0, 64, y.data_ptr(),
             sc.data_ptr(), w.data_ptr() if w is not None else None,
             wo.data_ptr() if wo is not None else None, stream)
    return (y, sc, wo) if w is not None else (y, sc)


def score_topk_fp8(q8: torch.Tensor, wq: torch.Tensor, k8: torch.Tensor, ks: torch.Tensor,
                   batch: int, seqlen: int, n_cand: int, topk: int, start_pos: int, ratio: int,
                   offset: int, want_scores: bool = False):
    """fp8 scores and top-k (dsa_indexer_score_topk_fp8). q8 [batch*seqlen*16, 64]
    uint8, wq [batch*seqlen, 16] f32, k8 [batch*n_cand, 64] uint8, ks [batch*n_cand]
    f32. Returns int64 [batch, seqlen, topk] (and the f32 scores [batch*seqlen,
    n_cand], NaN where masked, with want_scores)."""
    dev = q8.device
    out = torch.empty(batch, seqlen, topk, dtype=torch.int64, device=dev)
    scores = None
    if want_scores:
        scores = torch.full((batch * seqlen, n_cand), float("nan"), dtype=torch.float32,
                            device=dev)
    stream = torch.cuda.current_stream(dev).cuda_stream
    with torch.cuda.device(dev):
        call("dsa_indexer_score_topk_fp8", q8.contiguous().data_ptr(), wq.contiguous().data_ptr(),
             k8.contiguous().data_ptr(), ks.contiguous().data_ptr(), out.data_ptr(),
             scores.data_ptr() if scores is not None else None, batch, seqlen, 16, 64, n_cand,
             topk, start_pos, ratio, offset, stream)
    return (out, scores) if want_scores else out


def _make_args():
    """Reference configuration (reference/task2_v0_ref.py:147-150)."""
    return ModelArgs(max_batch_size=8, max_seq_len=2600, dim=1024, index_n_heads=16,
                     index_head_dim=64, index_topk=128, q_lora_rank=256, rope_head_dim=32)


def get_inputs(device: str = "cuda"):
    a = _make_args()
    batch_size = 8
    seq_len = 2600
    x = torch.randn(batch_size, seq_len, a.dim, dtype=torch.bfloat16).to(device)
    qr = torch.randn(batch_size, seq_len, a.q_lora_rank, dtype=torch.bfloat16).to(device)
    start_pos = 0
    offset = 0
    return [x, qr, start_pos, offset]


def make_freqs_cis(rope_head_dim: int, max_seq_len: int, rope_theta: float = 10000.0,
                   device: str = "cpu") -> torch.Tensor:
    """freqs_cis as built by reference/task2_v0_ref.py:162-168 (complex64)."""
    freqs = 1.0 / (rope_theta ** (torch.arange(0, rope_head_dim, 2)[:rope_head_dim // 2].float()
                                  / rope_head_dim))
    t = torch.arange(max_seq_len, dtype=torch.float32)
    freqs = torch.outer(t, freqs).float().to(device)
    return torch.polar(torch.ones_like(freqs), freqs).view(max_seq_len, -1)


def get_init_inputs(device: str = "cuda"):
    a = _make_args()
    compress_ratio = 4
    freqs_cis = make_freqs_cis(a.rope_head_dim, a.max_seq_len, 10000.0, device)
    kv_cache = torch.randn(a.max_batch_size, a.max_seq_len // compress_ratio, a.index_head_dim,
                           dtype=torch.bfloat16).to(device)
    return [a, freqs_cis, kv_cache, compress_ratio]
