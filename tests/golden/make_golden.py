"""Generates the golden fixtures in tests/golden/ from the reference's own v0 code.

Run once in a checkout that has the reference repository (default location
given by --ref); the outputs are committed so that the tests never need the
reference at run time:

    python tests/golden/make_golden.py --ref <path-to-reference-repo>

The reference modules (reference/task{1,2,3}_v0_ref.py) are imported
unmodified; their ``.cuda()`` calls are made identity so they run on the CPU.
Inputs follow the reference's order: torch.manual_seed(seed), then
get_init_inputs(), then the Model construction, then get_inputs().

Outputs
  sinkhorn.npz        full reference shape [1,1024,4,4] and a small case with
                      other repeat/eps.
  sparse_attn.npz     small cases: int32 indices / zero sink at h=64, and int64
                      indices with -1 entries, n_kv < 32, random sink at h=16.
  indexer.npz         small prefill (start_pos=0) and decode (start_pos>0)
                      cases with every intermediate (q after RoPE, weights,
                      masked bf16 scores) and the reference's top-k indices.
  indexer_full_pin.json / indexer_full_rows.npz
                      full BASELINE shape [8,2600]: the reference's per-row
                      top-k index lists and value lists (as digests) and the
                      comparison of the oracle against the reference at that size.
"""

from __future__ import annotations

import argparse
import hashlib
import importlib.util
import json
import os
import sys
import time

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)

import oracle  # noqa: E402


def _load(ref: str, name: str):
    path = os.path.join(ref, "reference", name)
    spec = importlib.util.spec_from_file_location(name[:-3], path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def u16(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).numpy().view(np.uint16).copy()


def make_sinkhorn(ref: str) -> dict:
    m = _load(ref, "task3_v0_ref.py")
    torch.manual_seed(42)
    model = m.Model(*m.get_init_inputs())
    (x,) = m.get_inputs()
    y = model(x)
    torch.manual_seed(7)
    xs = torch.randn(2, 8, 4, 4) * 3.0
    ys = m.Model(repeat=3, eps=1e-3)(xs)
    return {"full_x": x.numpy(), "full_y": y.numpy(), "small_x": xs.numpy(),
            "small_y": ys.numpy(), "small_repeat": np.int64(3), "small_eps": np.float64(1e-3)}


def make_sparse_attn(ref: str) -> dict:
    m = _load(ref, "task1_v0_ref.py")
    out = {}
    # case A: reference distributions, int32 indices, zero sink, h=64
    torch.manual_seed(42)
    model = m.Model(64, 128)
    q = torch.randn(2, 4, 64, 128, dtype=torch.bfloat16)
    kv = torch.randn(2, 32, 128, dtype=torch.bfloat16)
    idx = torch.randint(0, 32, (2, 4, 16), dtype=torch.int32)
    o = model(q, kv, idx)
    out.update(a_q=u16(q), a_kv=u16(kv), a_idx=idx.numpy(), a_sink=model.attn_sink.detach().numpy(),
               a_out=u16(o), a_scale=np.float64(model.softmax_scale))
    # case B: int64 indices with -1 entries (one token fully masked), n_kv = 20,
    # random sink, h = 16 -- the chained form fed by the indexer.
    torch.manual_seed(43)
    model = m.Model(16, 128)
    with torch.no_grad():
        model.attn_sink.copy_(torch.randn(16))
    q = torch.randn(2, 12, 16, 128, dtype=torch.bfloat16)
    kv = torch.randn(2, 20, 128, dtype=torch.bfloat16)
    idx = torch.randint(-1, 20, (2, 12, 16), dtype=torch.int64)
    idx[0, 3, :] = -1
    idx[1, 5, :8] = -1
    o = model(q, kv, idx)
    out.update(b_q=u16(q), b_kv=u16(kv), b_idx=idx.numpy(), b_sink=model.attn_sink.detach().numpy(),
               b_out=u16(o), b_scale=np.float64(model.softmax_scale))
    return out


def _indexer_case(m, args, batch, seqlen, start_pos, offset, seed, prefix):
    """Runs the reference indexer and records inputs and every intermediate."""
    torch.manual_seed(seed)
    rope_theta = 10000.0
    freqs = 1.0 / (rope_theta ** (torch.arange(0, args.rope_head_dim, 2)[:args.rope_head_dim // 2]
                                  .float() / args.rope_head_dim))
    t = torch.arange(args.max_seq_len, dtype=torch.float32)
    freqs = torch.outer(t, freqs).float()
    freqs_cis = torch.polar(torch.ones_like(freqs), freqs).view(args.max_seq_len, -1)
    ratio = 4
    kv_cache = torch.randn(args.max_batch_size, args.max_seq_len // ratio, args.index_head_dim,
                           dtype=torch.bfloat16)
    model = m.Model(args, freqs_cis, kv_cache, ratio)
    x = torch.randn(batch, seqlen, args.dim, dtype=torch.bfloat16)
    qr = torch.randn(batch, seqlen, args.q_lora_rank, dtype=torch.bfloat16)
    with torch.no_grad():
        idx = model(x, qr, start_pos, offset)
        # Intermediates, replaying the reference forward (task2_v0_ref.py:124-137).
        fc = freqs_cis[start_pos:start_pos + seqlen]
        end_pos = start_pos + seqlen
        rd = args.rope_head_dim
        q = model.wq_b(qr).unflatten(-1, (model.n_local_heads, model.head_dim))
        m.apply_rotary_emb(q[..., -rd:], fc)
        w = model.weights_proj(x) * (model.softmax_scale * model.n_heads ** -0.5)
        sc = torch.einsum("bshd,btd->bsht", q, kv_cache[:batch, :end_pos // ratio])
        sc = (sc.relu_() * w.unsqueeze(-1)).sum(dim=2)
        if start_pos == 0:
            mask = (torch.arange(seqlen // ratio).repeat(seqlen, 1)
                    >= torch.arange(1, seqlen + 1).unsqueeze(1) // ratio)
            sc += torch.where(mask, float("-inf"), 0)
    pre = prefix
    return {
        pre + "x": u16(x), pre + "qr": u16(qr), pre + "wq": u16(model.wq_b.weight.detach()),
        pre + "wp": u16(model.weights_proj.weight.detach()),
        pre + "cos": torch.view_as_real(fc)[..., 0].contiguous().numpy(),
        pre + "sin": torch.view_as_real(fc)[..., 1].contiguous().numpy(),
        pre + "kv": u16(kv_cache), pre + "q": u16(q.reshape(batch * seqlen, -1)),
        pre + "w": u16(w.reshape(batch * seqlen, -1)),
        pre + "scores": u16(sc.reshape(batch * seqlen, -1).to(torch.bfloat16)),
        pre + "idx": idx.numpy(),
        pre + "meta": np.array([batch, seqlen, start_pos, offset, ratio, args.dim,
                                args.q_lora_rank, args.index_n_heads, args.index_head_dim,
                                args.rope_head_dim, args.index_topk], dtype=np.int64),
        pre + "w_scale": np.float64(model.softmax_scale * model.n_heads ** -0.5),
    }


def make_indexer(ref: str) -> dict:
    m = _load(ref, "task2_v0_ref.py")
    torch.Tensor.cuda = lambda self, *a, **k: self  # the reference calls .cuda()
    args = m.ModelArgs(max_batch_size=2, max_seq_len=64, dim=256, index_n_heads=16,
                       index_head_dim=64, index_topk=8, q_lora_rank=128, rope_head_dim=32)
    out = {}
    out.update(_indexer_case(m, args, 2, 64, 0, 0, 11, "p_"))
    out.update(_indexer_case(m, args, 2, 32, 16, 5, 12, "d_"))
    return out


def _row_digest(values: np.ndarray) -> np.ndarray:
    """8-byte digest of each row of a [rows, K] array (its raw bytes)."""
    out = np.empty(values.shape[0], dtype=np.uint64)
    for i, row in enumerate(values):
        out[i] = np.frombuffer(hashlib.blake2b(row.tobytes(), digest_size=8).digest(),
                               dtype=np.uint64)[0]
    return out


def make_indexer_full(ref: str) -> tuple[dict, dict]:
    """Full BASELINE shape: reference vs oracle, recorded as digests + stats."""
    m = _load(ref, "task2_v0_ref.py")
    torch.Tensor.cuda = lambda self, *a, **k: self
    torch.manual_seed(42)
    init = m.get_init_inputs()
    model = m.Model(*init)
    x, qr, start_pos, offset = m.get_inputs()
    args, freqs_cis, kv_cache, ratio = init
    t0 = time.time()
    with torch.no_grad():
        idx = model(x, qr, start_pos, offset)
        B, S, _ = x.shape
        end_pos = start_pos + S
        rd = args.rope_head_dim
        q = model.wq_b(qr).unflatten(-1, (model.n_local_heads, model.head_dim))
        m.apply_rotary_emb(q[..., -rd:], freqs_cis[start_pos:end_pos])
        w = model.weights_proj(x) * (model.softmax_scale * model.n_heads ** -0.5)
        sc = torch.einsum("bshd,btd->bsht", q, kv_cache[:B, :end_pos // ratio])
        sc = (sc.relu_() * w.unsqueeze(-1)).sum(dim=2)
        mask = (torch.arange(S // ratio).repeat(S, 1)
                >= torch.arange(1, S + 1).unsqueeze(1) // ratio)
        sc += torch.where(mask, float("-inf"), 0)
    ref_s = time.time() - t0
    T = end_pos // ratio
    K = idx.shape[-1]
    ref_idx = idx.reshape(B * S, K).numpy()
    ref_scores = u16(sc.reshape(B * S, T))
    ref_q = u16(q.reshape(B * S, -1))
    ref_w = u16(w.reshape(B * S, -1))
    # value list of the reference's selection (masked slots -> 0xFF80 = -inf)
    rows = np.arange(B * S)[:, None]
    safe = np.where(ref_idx >= 0, ref_idx, 0)
    ref_vals = np.where(ref_idx >= 0, ref_scores[rows, safe], np.uint16(0xFF80)).astype(np.uint16)

    fc = freqs_cis[start_pos:end_pos]
    cos = torch.view_as_real(fc)[..., 0].contiguous().numpy()
    sin = torch.view_as_real(fc)[..., 1].contiguous().numpy()
    t0 = time.time()
    o_idx, inter = oracle.indexer_fwd(
        u16(x), u16(qr), u16(model.wq_b.weight.detach()), u16(model.weights_proj.weight.detach()),
        cos, sin, u16(kv_cache), n_heads=16, head_dim=64, rope_dim=rd, index_topk=128,
        start_pos=start_pos, ratio=ratio, offset=offset,
        w_scale=model.softmax_scale * model.n_heads ** -0.5, want_intermediates=True)
    or_s = time.time() - t0
    o_idx = o_idx.reshape(B * S, K)
    o_scores = inter["scores"]
    o_vals = np.where(o_idx >= 0, o_scores[rows, np.where(o_idx >= 0, o_idx, 0)],
                      np.uint16(0xFF80)).astype(np.uint16)
    # bf16 value order for comparison of value lists (descending, -0 == +0)
    q_mism = int((inter["q"] != ref_q).sum())
    w_mism = int((inter["w"] != ref_w).sum())
    valid = ref_scores != 0xFF80
    s_mism_mask = (o_scores != ref_scores) & valid
    s_mism = int(s_mism_mask.sum())
    rows_with_score_diff = np.where(s_mism_mask.any(axis=1))[0]
    vals_equal = (o_vals == ref_vals).all(axis=1)
    sets_equal = np.array([np.array_equal(np.sort(a), np.sort(b)) for a, b in zip(o_idx, ref_idx)])
    idx_equal = (o_idx == ref_idx).all(axis=1)
    stats = {
        "shape": [B, S, T, K],
        "reference_cpu_seconds": round(ref_s, 3),
        "oracle_cpu_seconds": round(or_s, 3),
        "oracle_threads": oracle.num_threads(),
        "q_elements": int(ref_q.size), "q_mismatch": q_mism,
        "w_elements": int(ref_w.size), "w_mismatch": w_mism,
        "score_elements_valid": int(valid.sum()), "score_mismatch": s_mism,
        "rows": B * S,
        "rows_value_list_equal": int(vals_equal.sum()),
        "rows_index_set_equal": int(sets_equal.sum()),
        "rows_index_order_equal": int(idx_equal.sum()),
        "rows_with_score_mismatch": int(rows_with_score_diff.size),
        "rows_value_list_diff_without_score_mismatch":
            int((~vals_equal & ~s_mism_mask.any(axis=1)).sum()),
        "input_sha": hashlib.sha1(u16(x).tobytes() + u16(qr).tobytes() + u16(kv_cache).tobytes()
                                  ).hexdigest(),
    }
    arrays = {
        "ref_value_digest": _row_digest(ref_vals),
        "ref_index_digest": _row_digest(ref_idx),
        "rows_with_score_mismatch": rows_with_score_diff.astype(np.int64),
    }
    return stats, arrays


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("DSA_REFERENCE_DIR"),
                    help="checkout of the reference repository (or set DSA_REFERENCE_DIR)")
    ap.add_argument("--skip-full", action="store_true")
    a = ap.parse_args()
    if not a.ref:
        ap.error("give --ref or DSA_REFERENCE_DIR: the reference checkout to import")
    torch.set_num_threads(os.cpu_count() or 1)
    np.savez_compressed(os.path.join(HERE, "sinkhorn.npz"), **make_sinkhorn(a.ref))
    np.savez_compressed(os.path.join(HERE, "sparse_attn.npz"), **make_sparse_attn(a.ref))
    np.savez_compressed(os.path.join(HERE, "indexer.npz"), **make_indexer(a.ref))
    if not a.skip_full:
        stats, arrays = make_indexer_full(a.ref)
        with open(os.path.join(HERE, "indexer_full_pin.json"), "w") as f:
            json.dump(stats, f, indent=1)
        np.savez_compressed(os.path.join(HERE, "indexer_full_rows.npz"), **arrays)
        print(json.dumps(stats, indent=1))


if __name__ == "__main__":
    main()
