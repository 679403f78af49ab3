"""Host-side tests of the C ABI: the library loads on a machine without a GPU,
exports every symbol the header declares, and rejects bad arguments before any
CUDA work (the reference's asserts / TORCH_CHECKs map to status codes)."""

import ctypes
import os
import re

import pytest

from ascendc_kernel_b200 import _native

HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include",
                      "dsa_b200.h")

OK, INVALID, UNSUPPORTED, MISALIGNED = 0, 1, 2, 3


def declared_symbols():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(dsa_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    lib = _native.lib()
    syms = declared_symbols()
    assert len(syms) >= 10
    for s in syms:
        assert hasattr(lib, s), s
    assert set(syms) == set(_native.SIGNATURES), "ctypes signatures out of sync with the header"


def test_status_strings():
    lib = _native.lib()
    assert lib.dsa_status_string(0) == b"DSA_OK"
    assert lib.dsa_status_string(2) == b"DSA_ERR_UNSUPPORTED"
    assert lib.dsa_status_string(99) == b"DSA_ERR_UNKNOWN"
    assert lib.dsa_version() >= 100


FAKE = 0x1000  # 16-byte aligned, never dereferenced: every call below fails validation


def sa(**kw):
    a = dict(q=FAKE, kv=FAKE, idx=FAKE, eb=4, sink=FAKE, out=FAKE, b=8, m=2600, h=64, d=128,
             nkv=32, topk=16, scale=0.088, stream=None)
    a.update(kw)
    return _native.lib().dsa_sparse_attn_fwd(a["q"], a["kv"], a["idx"], a["eb"], a["sink"],
                                              a["out"], a["b"], a["m"], a["h"], a["d"], a["nkv"],
                                              a["topk"], a["scale"], a["stream"])


@pytest.mark.parametrize("kw,code", [
    (dict(q=None), INVALID),
    (dict(out=None), INVALID),
    (dict(b=-1), INVALID),
    (dict(eb=2), INVALID),
    (dict(d=64), UNSUPPORTED),
    (dict(h=48), UNSUPPORTED),
    (dict(nkv=33, h=16), UNSUPPORTED),    # long kv pools need 64 or 128 heads
    (dict(nkv=4097), UNSUPPORTED),        # long kv pools: at most 4096 rows
    (dict(topk=6), UNSUPPORTED),          # 24 bytes: not a multiple of 16
    (dict(topk=256, h=32), UNSUPPORTED),
    (dict(q=FAKE + 2), MISALIGNED),
    (dict(b=0), OK),                      # empty batch is a no-op
    (dict(m=0), OK),
])
def test_sparse_attn_argument_checks(kw, code):
    assert sa(**kw) == code


@pytest.mark.parametrize("args,code", [
    ((None, FAKE, 1024, 4, 10, 1e-6), INVALID),
    ((FAKE, FAKE, 1024, 5, 10, 1e-6), UNSUPPORTED),
    ((FAKE, FAKE, 1024, 4, 0, 1e-6), INVALID),
    ((FAKE + 4, FAKE, 1024, 4, 10, 1e-6), MISALIGNED),
    ((FAKE, FAKE, 0, 4, 10, 1e-6), OK),
])
def test_sinkhorn_argument_checks(args, code):
    x, y, n, mhc, rep, eps = args
    assert _native.lib().dsa_sinkhorn_fwd(x, y, n, mhc, rep, eps, None) == code


def test_error_carries_status_name():
    with pytest.raises(_native.DsaError, match="DSA_ERR_UNSUPPORTED"):
        _native.call("dsa_sinkhorn_fwd", FAKE, FAKE, 16, 5, 10, ctypes.c_float(1e-6), None)


def kvw(**kw):
    a = dict(x=FAKE, wk=FAKE, g=FAKE, b=FAKE, cos=FAKE, sin=FAKE, kv=FAKE, kvs=650 * 64,
             rows=650, batch=8, s=2600, dim=1024, hd=64, rd=32, sp=0, r=4, stream=None)
    a.update(kw)
    return _native.lib().dsa_kv_cache_write(a["x"], a["wk"], a["g"], a["b"], a["cos"], a["sin"],
                                            a["kv"], a["kvs"], a["rows"], a["batch"], a["s"],
                                            a["dim"], a["hd"], a["rd"], a["sp"], a["r"],
                                            a["stream"])


@pytest.mark.parametrize("kw,code", [
    (dict(x=None), INVALID),
    (dict(kv=None), INVALID),
    (dict(cos=None), INVALID),            # rotary dims need the tables
    (dict(rd=3), INVALID),                # odd rotary width
    (dict(r=0), INVALID),
    (dict(sp=2), INVALID),                # start_pos not a multiple of the ratio
    (dict(rows=649), INVALID),            # the written blocks do not fit the cache
    (dict(kvs=649 * 64), INVALID),        # batch stride shorter than the rows
    (dict(hd=128), UNSUPPORTED),
    (dict(dim=1000), UNSUPPORTED),
    (dict(r=3), UNSUPPORTED),             # the ratio must divide the 128-token tile
    (dict(x=FAKE + 2), MISALIGNED),
    (dict(kvs=650 * 64 + 4), MISALIGNED),
    (dict(batch=0), OK),                  # nothing to write
    (dict(s=3), OK),                      # fewer tokens than one block
    (dict(rd=0, cos=None, sin=None, batch=0), OK),
])
def test_kv_cache_write_argument_checks(kw, code):
    assert kvw(**kw) == code
