"""G1 parity gate: the Lightning Indexer against the reference's own v0 module run
on torch CUDA on the B200 (reference/task2_v0_ref.py:123-144, executed as the same
torch op sequence by oracle/v0_torch.py, which the CPU tests pin bit for bit to the
reference's CPU output).

The reference's arithmetic on CUDA is cuBLAS bf16 GEMMs with fp32 accumulation
(F.linear, the score einsum), an fp32 complex product for RoPE and an fp32 head sum.
None of them promises a correctly rounded bf16 result, while this library's
contract is correct rounding everywhere. So the gate has two parts:

- rows whose valid reference scores all equal the correctly rounded ones must
  select exactly this library's indices (same set, same order), which also pins the
  tie rule of torch CUDA topk at the BASELINE shape;
- every other row is attributed: it holds a reference score that differs from
  the correctly rounded value of the same formula, and the cause is split into the
  reference's q / w (projection GEMMs and RoPE) and its score einsum / head sum.

The counts are pinned for this torch build and GPU; the attribution assertions hold
for any cuBLAS algorithm choice.
"""

import json
import os

import numpy as np
import pytest
import torch

import oracle
from ascendc_kernel_b200 import indexer as ix
from oracle import v0_torch
from tests.helpers import to_u16

pytestmark = pytest.mark.gpu


def _report(name, data):
    path = os.environ.get("DSA_PARITY_REPORT_DIR")
    if path:
        os.makedirs(path, exist_ok=True)
        with open(os.path.join(path, name), "w") as f:
            json.dump(data, f, indent=1)
    print(name, json.dumps(data))


def _tie_rule(dev, n, k, rows=256, levels=6, seed=0):
    """torch CUDA topk on rows with heavy ties: does it take boundary ties by
    ascending index (the selected set), and order equal values by ascending index?"""
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    v = torch.randint(0, levels, (rows, n), device=dev, generator=g).to(torch.bfloat16)
    _, idx = v.topk(k, dim=-1)
    # canonical order: value descending, index ascending
    key = v.float() * (2 * n) - torch.arange(n, device=dev, dtype=torch.float32)
    canon = key.argsort(dim=-1, descending=True)[:, :k]
    same_set = (idx.sort(-1).values == canon.sort(-1).values).all(-1)
    same_order = (idx == canon).all(-1)
    return {"n": n, "k": k, "rows": rows, "levels": levels,
            "rows_set_ascending": int(same_set.sum()), "rows_order_ascending": int(same_order.sum())}


def test_torch_cuda_topk_tie_rule(cuda_device):
    """Measured tie rule of torch CUDA topk at the two selection shapes of the path."""
    res = [_tie_rule(cuda_device, 650, 128), _tie_rule(cuda_device, 4096, 2048)]
    _report("g1_topk_tie_rule.json", {"torch": torch.__version__, "cases": res})
    for r in res:
        # the selected set follows ascending index at the k-th value boundary, and
        # equal values come out in ascending index order: the canonical rule
        # (score descending, index ascending) this library implements
        assert r["rows_set_ascending"] == r["rows"], r
        assert r["rows_order_ascending"] == r["rows"], r


def _value_lists(idx, scores, T):
    """bf16 score bits of each selected index (masked slots -> -inf bits)."""
    rows = np.arange(idx.shape[0])[:, None]
    safe = np.clip(idx, 0, T - 1)
    return np.where(idx >= 0, scores[rows, safe], np.uint16(0xFF80)).astype(np.uint16)


def test_indexer_matches_reference_on_torch_cuda(cuda_device):
    dev = cuda_device
    torch.manual_seed(42)
    args, freqs_cis, kv_cache, ratio = ix.get_init_inputs(device="cpu")
    model = ix.ModelNew(args, freqs_cis, kv_cache, ratio)
    x, qr, start_pos, offset = ix.get_inputs(device="cpu")
    B, S = x.shape[:2]
    T = (start_pos + S) // ratio
    K = min(args.index_topk, T)
    wq = model.wq_b.weight.detach()
    wp = model.weights_proj.weight.detach()

    # the reference's module on torch CUDA
    with torch.no_grad():
        ref_idx, (ref_q, ref_w, ref_sc) = v0_torch.indexer_v0(
            wq.to(dev), wp.to(dev), freqs_cis.to(dev), kv_cache.to(dev), x.to(dev), qr.to(dev),
            start_pos, offset, n_heads=16, head_dim=64, rope_dim=32, index_topk=K,
            ratio=ratio, intermediates=True)
    # this library's drop-in
    model_d = ix.ModelNew(args, freqs_cis.to(dev), kv_cache.to(dev), ratio)
    model_d.load_state_dict(model.state_dict())
    got = model_d(x.to(dev), qr.to(dev), start_pos, offset)
    torch.cuda.synchronize()

    ref_idx = ref_idx.reshape(B * S, K).cpu().numpy()
    got_np = got.reshape(B * S, K).cpu().numpy()
    ref_q = to_u16(ref_q).reshape(B * S, -1)
    ref_w = to_u16(ref_w).reshape(B * S, -1)
    ref_sc = to_u16(ref_sc.to(torch.bfloat16)).reshape(B * S, T)

    # the contract's values: correctly rounded q, w and scores (CPU oracle)
    fc = torch.view_as_real(freqs_cis[start_pos:start_pos + S])
    cos, sin = fc[..., 0].contiguous().numpy(), fc[..., 1].contiguous().numpy()
    w_scale = model.softmax_scale * model.n_heads ** -0.5
    _, inter = oracle.indexer_fwd(
        to_u16(x), to_u16(qr), to_u16(wq), to_u16(wp), cos, sin, to_u16(kv_cache),
        n_heads=16, head_dim=64, rope_dim=32, index_topk=K, start_pos=start_pos, ratio=ratio,
        offset=offset, w_scale=w_scale, want_intermediates=True)
    # the contract's scores from the reference's own q and w: separates what the
    # reference's projections changed from what its einsum / head sum changed
    _, sc_from_ref_qw = oracle.index_topk(ref_q, ref_w, to_u16(kv_cache), B, S, 16, 64, T, K,
                                          start_pos, ratio, offset, want_scores=True)
    lim = np.minimum((np.arange(S) + 1) // ratio, T) if start_pos == 0 else np.full(S, T)
    valid = (np.arange(T)[None, :] < np.tile(lim, B)[:, None])

    q_mism = ref_q != inter["q"]
    rope_cols = np.zeros(16 * 64, bool)
    for h in range(16):
        rope_cols[h * 64 + 32:(h + 1) * 64] = True
    s_mism = (ref_sc != inter["scores"]) & valid
    s_from_qw = (sc_from_ref_qw != inter["scores"]) & valid
    s_from_gemm = (ref_sc != sc_from_ref_qw) & valid
    rows_s_mism = s_mism.any(axis=1)

    order_eq = (got_np == ref_idx).all(axis=1)
    set_eq = (np.sort(got_np, axis=1) == np.sort(ref_idx, axis=1)).all(axis=1)
    vals_eq = (_value_lists(got_np, inter["scores"], T)
               == _value_lists(ref_idx, ref_sc, T)).all(axis=1)
    rep = {
        "shape": [B, S, T, K], "torch": torch.__version__,
        "device": torch.cuda.get_device_name(dev),
        "rows": B * S,
        "rows_index_order_equal": int(order_eq.sum()),
        "rows_index_set_equal": int(set_eq.sum()),
        "rows_value_list_equal": int(vals_eq.sum()),
        "q_elements": int(q_mism.size), "q_mismatch": int(q_mism.sum()),
        "q_mismatch_rope_columns": int(q_mism[:, rope_cols].sum()),
        "q_mismatch_projection_only_columns": int(q_mism[:, ~rope_cols].sum()),
        "w_elements": int(ref_w.size), "w_mismatch": int((ref_w != inter["w"]).sum()),
        "score_elements_valid": int(valid.sum()),
        "score_mismatch": int(s_mism.sum()),
        "score_mismatch_from_ref_q_w": int(s_from_qw.sum()),
        "score_mismatch_from_ref_einsum_or_head_sum": int(s_from_gemm.sum()),
        "rows_with_score_mismatch": int(rows_s_mism.sum()),
        "rows_order_differs_without_score_mismatch": int((~order_eq & ~rows_s_mism).sum()),
        "rows_value_list_differs_without_score_mismatch": int((~vals_eq & ~rows_s_mism).sum()),
    }
    _report("g1_indexer_reference_cuda.json", rep)
    # Measured on a B200 with torch 2.11.0+cu128 (cuBLAS algorithm choice for these
    # shapes); the attribution assertions below hold whatever cuBLAS picks.
    pinned = {"rows_index_order_equal": 20692, "rows_index_set_equal": 20797,
              "rows_value_list_equal": 20554, "q_mismatch": 809, "w_mismatch": 45,
              "score_mismatch": 2845, "rows_with_score_mismatch": 472}
    if torch.__version__.startswith("2.11.0") and "B200" in rep["device"]:
        assert {k: rep[k] for k in pinned} == pinned, rep
    # every row whose reference scores are the correctly rounded ones selects
    # exactly this library's indices, in the same order
    assert rep["rows_order_differs_without_score_mismatch"] == 0, rep
    assert rep["rows_value_list_differs_without_score_mismatch"] == 0, rep
    # every score mismatch has a cause on the reference's side
    assert int((s_mism & ~(s_from_qw | s_from_gemm)).sum()) == 0


def _bf16_report(got, want):
    g = got.float().cpu().numpy().astype(np.float64)
    w = want.float().cpu().numpy().astype(np.float64)
    d = np.abs(g - w)
    gb, wb = to_u16(got).astype(np.int32), to_u16(want).astype(np.int32)
    go = np.where(gb & 0x8000, 0x8000 - (gb & 0x7FFF), 0x8000 + gb)
    wo = np.where(wb & 0x8000, 0x8000 - (wb & 0x7FFF), 0x8000 + wb)
    return {"n": int(d.size), "max_abs": float(d.max()), "bit_mismatch": int((go != wo).sum()),
            "over_1ulp": int((np.abs(go - wo) > 1).sum()),
            "allclose_1e-2": bool(np.all(d <= 1e-2 + 1e-2 * np.abs(w)))}


def test_sparse_attn_vs_reference_on_torch_cuda(cuda_device):
    """BASELINE configs[1] against sparse_attn_ref on torch CUDA (fp32 einsums there):
    max error reported, within the harness tolerance atol = rtol = 1e-2."""
    from ascendc_kernel_b200 import sparse_attn as sa

    dev = cuda_device
    torch.manual_seed(42)
    model = sa.ModelNew(*sa.get_init_inputs()).to(dev)
    q, kv, idx = (t.to(dev) for t in sa.get_inputs())
    got = model(q, kv, idx)
    with torch.no_grad():
        want = v0_torch.sparse_attn_v0(q, kv, model.attn_sink, idx, model.softmax_scale)
    rep = _bf16_report(got, want)
    _report("g1_sparse_attn_reference_cuda.json", rep)
    assert rep["allclose_1e-2"], rep
    assert rep["bit_mismatch"] <= rep["n"] * 1e-3, rep


def test_sinkhorn_vs_reference_on_torch_cuda(cuda_device):
    """Sinkhorn at the reference shape against Model.forward on torch CUDA."""
    from ascendc_kernel_b200 import sinkhorn as sk

    dev = cuda_device
    torch.manual_seed(42)
    (x,) = sk.get_inputs()
    x = x.to(dev)
    got = sk.ModelNew()(x)
    want = v0_torch.sinkhorn_v0(x, 10, 1e-6)
    d = (got.double() - want.double()).abs()
    rep = {"n": int(d.numel()), "max_abs": float(d.max()),
           "bit_mismatch": int((got.view(torch.int32) != want.view(torch.int32)).sum())}
    _report("g1_sinkhorn_reference_cuda.json", rep)
    assert rep["max_abs"] < 2e-6, rep
