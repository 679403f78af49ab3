"""The allocation-free indexer entry point (dsa_indexer_fwd_noalloc).

It serves callers that cannot allocate device memory when they call the
indexer -- e.g. a plug-in whose host framework owns all device memory, or a
latency-critical path that must not pay for cudaMalloc/cudaFree -- by keeping
the q and w intermediates in a fixed 128 MiB array inside the library. These
tests call it through the C ABI and check that two calls in a row (different
inputs, same shared array) return exactly the indices of the workspace-taking
entry point, dsa_indexer_fwd, and that the documented token limit is exact:
at 650 candidates per token, 25,981 tokens succeed and 25,982 are rejected.

This file is named so that pytest collects it last.
"""

import ctypes

import pytest
import torch

from ascendc_kernel_b200 import _native
from ascendc_kernel_b200 import indexer as ix

pytestmark = pytest.mark.gpu

DSA_ERR_WORKSPACE = 5
LIMIT_BYTES = 128 << 20  # the fixed in-library array


def _max_tokens():
    """Largest batch*seqlen whose workspace fits the fixed array (16 heads x 64)."""
    lib = _native.lib()
    lo, hi = 1, 1 << 20
    while lo < hi:
        mid = (lo + hi + 1) // 2
        if lib.dsa_indexer_workspace_bytes(1, mid, 16, 64, 650, 128) <= LIMIT_BYTES:
            lo = mid
        else:
            hi = mid - 1
    return lo


def _inputs(seed, dev, batch=8, seqlen=2600, start_pos=0):
    torch.manual_seed(seed)
    args, freqs_cis, kv_cache, ratio = ix.get_init_inputs(device="cpu")
    model = ix.ModelNew(args, freqs_cis, kv_cache, ratio)
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    x = torch.randn(batch, seqlen, args.dim, dtype=torch.bfloat16, device=dev, generator=g)
    qr = torch.randn(batch, seqlen, args.q_lora_rank, dtype=torch.bfloat16, device=dev,
                     generator=g)
    T = (start_pos + seqlen) // ratio
    if batch <= kv_cache.shape[0]:
        kv = kv_cache.to(dev)
    else:
        kv = torch.randn(batch, T, args.index_head_dim, dtype=torch.bfloat16, device=dev,
                         generator=g)
    fc = torch.view_as_real(freqs_cis[start_pos:start_pos + seqlen])
    return dict(
        x=x, qr=qr, wq=model.wq_b.weight.detach().to(dev).contiguous(),
        wp=model.weights_proj.weight.detach().to(dev).contiguous(),
        cos=fc[..., 0].contiguous().to(dev), sin=fc[..., 1].contiguous().to(dev),
        kv=kv, batch=batch, seqlen=seqlen, start_pos=start_pos, T=T, K=min(128, T),
        w_scale=model.softmax_scale * model.n_heads ** -0.5)


def _head(d, out):
    return [d["x"].data_ptr(), d["qr"].data_ptr(), d["wq"].data_ptr(), d["wp"].data_ptr(),
            d["cos"].data_ptr(), d["sin"].data_ptr(), d["kv"].data_ptr(), d["kv"].stride(0),
            out.data_ptr()]


def _tail(d, stream):
    return [d["batch"], d["seqlen"], 1024, 256, 16, 64, 32, 128, d["start_pos"], 4, 0,
            ctypes.c_float(d["w_scale"]), stream]


def _out(d, dev):
    return torch.empty(d["batch"], d["seqlen"], d["K"], dtype=torch.int64, device=dev)


def _with_workspace(d, dev):
    lib = _native.lib()
    out = _out(d, dev)
    nbytes = lib.dsa_indexer_workspace_bytes(d["batch"], d["seqlen"], 16, 64, d["T"], d["K"])
    ws = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev).cuda_stream
    st = lib.dsa_indexer_fwd(*_head(d, out), ws.data_ptr(), nbytes, *_tail(d, stream))
    assert st == 0, st
    return out


def _no_alloc(d, dev):
    lib = _native.lib()
    out = _out(d, dev)
    stream = torch.cuda.current_stream(dev).cuda_stream
    st = lib.dsa_indexer_fwd_noalloc(*_head(d, out), *_tail(d, stream))
    assert st == 0, st
    return out


def test_no_alloc_matches_workspace_entry_point(cuda_device):
    dev = cuda_device
    a = _inputs(1, dev)   # the reference configuration: 20,800 tokens
    b = _inputs(2, dev)
    want_a = _with_workspace(a, dev)
    want_b = _with_workspace(b, dev)
    got_a = _no_alloc(a, dev)   # first call: resolves the array's address
    got_b = _no_alloc(b, dev)   # second call reuses the array left by the first
    torch.cuda.synchronize()
    assert torch.equal(got_a, want_a)
    assert torch.equal(got_b, want_b)
    assert _native.device_error(dev.index) == 0


def test_no_alloc_limit_is_exact(cuda_device):
    """At 650 candidates (the reference's count) the array holds exactly
    _max_tokens() tokens: that many succeed with the indices of the workspace
    entry point, one more is rejected before any launch. The tokens are spread
    over the batch (seqlen 1 at start_pos 2599, so every token has 650
    candidates)."""
    dev = cuda_device
    n = _max_tokens()
    assert n == 25981, n  # the documented limit
    d = _inputs(4, dev, batch=n, seqlen=1, start_pos=2599)
    assert d["T"] == 650
    want = _with_workspace(d, dev)
    got = _no_alloc(d, dev)
    torch.cuda.synchronize()
    assert torch.equal(got, want)
    assert _native.device_error(dev.index) == 0
    del d, want, got
    e = _inputs(5, dev, batch=n + 1, seqlen=1, start_pos=2599)
    lib = _native.lib()
    out = _out(e, dev)
    stream = torch.cuda.current_stream(dev).cuda_stream
    assert lib.dsa_indexer_workspace_bytes(n + 1, 1, 16, 64, 650, 128) > LIMIT_BYTES
    assert lib.dsa_indexer_fwd_noalloc(*_head(e, out), *_tail(e, stream)) == DSA_ERR_WORKSPACE
