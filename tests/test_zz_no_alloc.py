"""The allocation-free indexer entry point (dsa_indexer_fwd_noalloc).

It serves callers that cannot allocate device memory when they call the
indexer -- e.g. a plug-in whose host framework owns all device memory, or a
latency-critical path that must not pay for cudaMalloc/cudaFree -- by keeping
the q and w intermediates in a fixed 128 MiB array inside the library. These
tests call it through the C ABI and check that two calls in a row (different
inputs, same shared array) return exactly the indices of the workspace-taking
entry point, dsa_indexer_fwd, and that an oversized request is rejected.

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


def _inputs(seed, dev, batch=8, seqlen=2600):
    torch.manual_seed(seed)
    args, freqs_cis, kv_cache, ratio = ix.get_init_inputs(device="cpu")
    model = ix.ModelNew(args, freqs_cis, kv_cache, ratio)
    x = torch.randn(batch, seqlen, args.dim, dtype=torch.bfloat16, device=dev)
    qr = torch.randn(batch, seqlen, args.q_lora_rank, dtype=torch.bfloat16, device=dev)
    fc = torch.view_as_real(freqs_cis[:seqlen])
    return dict(
        x=x, qr=qr, wq=model.wq_b.weight.detach().to(dev).contiguous(),
        wp=model.weights_proj.weight.detach().to(dev).contiguous(),
        cos=fc[..., 0].contiguous().to(dev), sin=fc[..., 1].contiguous().to(dev),
        kv=kv_cache.to(dev), batch=batch, seqlen=seqlen,
        w_scale=model.softmax_scale * model.n_heads ** -0.5)


def _common_args(d, out):
    T = d["seqlen"] // 4
    return [d["x"].data_ptr(), d["qr"].data_ptr(), d["wq"].data_ptr(), d["wp"].data_ptr(),
            d["cos"].data_ptr(), d["sin"].data_ptr(), d["kv"].data_ptr(), d["kv"].stride(0),
            out.data_ptr()], T


def _tail(d, stream):
    return [d["batch"], d["seqlen"], 1024, 256, 16, 64, 32, 128, 0, 4, 0,
            ctypes.c_float(d["w_scale"]), stream]


def _with_workspace(d, dev):
    lib = _native.lib()
    T = d["seqlen"] // 4
    out = torch.empty(d["batch"], d["seqlen"], min(128, T), dtype=torch.int64, device=dev)
    head, _ = _common_args(d, out)
    nbytes = lib.dsa_indexer_workspace_bytes(d["batch"], d["seqlen"], 16, 64, T, min(128, T))
    ws = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev).cuda_stream
    tail = _tail(d, stream)
    st = lib.dsa_indexer_fwd(*head, ws.data_ptr(), nbytes, *tail)
    assert st == 0, st
    return out


def _no_alloc(d, dev):
    lib = _native.lib()
    T = d["seqlen"] // 4
    out = torch.empty(d["batch"], d["seqlen"], min(128, T), dtype=torch.int64, device=dev)
    head, _ = _common_args(d, out)
    stream = torch.cuda.current_stream(dev).cuda_stream
    st = lib.dsa_indexer_fwd_noalloc(*head, *_tail(d, stream))
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


def test_no_alloc_rejects_requests_beyond_its_array(cuda_device):
    dev = cuda_device
    d = _inputs(3, dev, batch=1, seqlen=64)
    lib = _native.lib()
    out = torch.empty(1, 64, 16, dtype=torch.int64, device=dev)
    head, _ = _common_args(d, out)
    stream = torch.cuda.current_stream(dev).cuda_stream
    tail = _tail(d, stream)
    tail[0], tail[1] = 1, _max_tokens() + 1   # batch, seqlen beyond the fixed array
    assert lib.dsa_indexer_fwd_noalloc(*head, *tail) == DSA_ERR_WORKSPACE
