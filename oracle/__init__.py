"""CPU oracle for the ReSS/HeSS selection path -- TEST INFRASTRUCTURE ONLY.

This package is the checker the CUDA path is compared against.  Only
``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline legs of
``bench.py`` may import it; the product package (``ress_b200``) never does and
has no CPU fallback.

The arithmetic lives in ``ress_oracle.c`` (a restatement of the reference's
torch functions with a fixed operation order; its header lists the reference
file:line each function follows).  This module only marshals CPU tensors and
chains the steps the way ``ress_attention_forward``
(reference ``src/ress/models/attention.py:446-581``) chains them.
"""

from __future__ import annotations

import ctypes
import math
import os
import subprocess

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "libress_oracle.so")
_lib = None

F32, BF16 = 0, 1
KS_Q, KS_K = 128, 64


def build() -> str:
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        _lib = ctypes.CDLL(_LIB_PATH)
        _lib.ro_hess_adjust.restype = ctypes.c_int
        _lib.ro_num_threads.restype = ctypes.c_int
    return _lib


def num_threads() -> int:
    return lib().ro_num_threads()


def _p(t: torch.Tensor):
    assert t.device.type == "cpu" and t.is_contiguous(), "oracle wants contiguous CPU tensors"
    return ctypes.c_void_p(t.data_ptr())


def _dt(t: torch.Tensor) -> int:
    if t.dtype == torch.float32:
        return F32
    if t.dtype == torch.bfloat16:
        return BF16
    raise TypeError(f"oracle supports float32/bfloat16, got {t.dtype}")


def _f(x: float):
    return ctypes.c_float(x)


# --------------------------------------------------------------------------- steps

def pool_mean(x: torch.Tensor, blk: int) -> torch.Tensor:
    """(rows, T, D) -> (rows, ceil(T/blk), D): avg_pool1d(ceil_mode=True)."""
    x = x.contiguous()
    rows, T, D = x.shape
    out = torch.empty(rows, -(-T // blk), D, dtype=x.dtype)
    lib().ro_pool_mean(_dt(x), _p(x), rows, T, D, blk, _p(out))
    return out


def predict(qbar: torch.Tensor, kbar: torch.Tensor) -> torch.Tensor:
    rows, nq, D = qbar.shape
    nk = kbar.shape[1]
    out = torch.empty(rows, nq, nk, dtype=qbar.dtype)
    qc, kc = qbar.contiguous(), kbar.contiguous()
    lib().ro_predict(_dt(qc), _p(qc), _p(kc), rows, nq, nk, D, _p(out))
    return out


def attn_cond(attn: torch.Tensor, n_cand: int) -> torch.Tensor:
    attn = attn.contiguous()
    nk = attn.shape[-1]
    rows = attn.numel() // nk
    out = torch.empty(attn.shape[:-1] + (n_cand,), dtype=attn.dtype)
    lib().ro_attn_cond(_dt(attn), _p(attn), rows, nk, n_cand, _p(out))
    return out


def cdf_value(cdf_threshold: float, eps: float = 1e-5) -> float:
    """The fp32 value searchsorted compares against (attention.py:283-285)."""
    return float(torch.as_tensor(cdf_threshold) + eps)


def baseline(cond: torch.Tensor, sparse_ratio=None, cdf_threshold=None) -> torch.Tensor:
    cond = cond.contiguous()
    n = cond.shape[-1]
    rows = cond.numel() // n
    topk = int(n * (1 - sparse_ratio)) if sparse_ratio is not None else -1
    use_cdf = cdf_threshold is not None
    cv = cdf_value(cdf_threshold) if use_cdf else 0.0
    out = torch.empty(cond.shape[:-1], dtype=torch.int32)
    lib().ro_baseline(_dt(cond), _p(cond), rows, n, int(use_cdf), _f(cv), topk, _p(out))
    return out


def scores_norm(head_scores: torch.Tensor) -> torch.Tensor:
    """head_scores / head_scores.sum() with a sequential fp32 sum, or uniform
    when the sum is not finite or not positive (_proportional.py:184-188)."""
    hs = head_scores.float().contiguous()
    s = torch.zeros((), dtype=torch.float32)
    for v in hs:
        s = s + v
    if not torch.isfinite(s) or s <= 0:
        return torch.full_like(hs, 1.0 / hs.numel())
    return hs / s


def hess_adjust(counts: torch.Tensor, snorm: torch.Tensor, max_val: int, beta: float = 1.0,
                min_clamp: int = 0, max_iters: int = 1000) -> torch.Tensor:
    c = counts.to(torch.int32).contiguous()
    B, nh, nq = c.shape
    out = torch.empty_like(c)
    omb = float(torch.tensor(1 - beta, dtype=torch.float32))
    sn = snorm.float().contiguous()
    st = lib().ro_hess_adjust(_p(c), _p(sn), B, nh, nq, max_val, _f(omb),
                              _f(float(beta)), max_iters, min_clamp, _p(out))
    if st != 0:
        raise RuntimeError(f"adjust_attention_selection did not converge in {max_iters} iterations")
    return out


def vbar_metric(vbar_bf16: torch.Tensor, M: torch.Tensor, n_cand: int) -> torch.Tensor:
    vb = vbar_bf16.contiguous().view(torch.int16)
    rows, nkp, _ = vb.shape
    nh = M.shape[0]
    tk = torch.empty(rows, n_cand, dtype=torch.int16)
    Mf = M.float().contiguous()
    lib().ro_vbar_metric(_p(vb), _p(Mf), rows, nh, nkp, n_cand, _p(tk))
    return tk.view(torch.bfloat16)


def round_fracs(n_iters: int, restore_frac: float = 0.5, decay: float = 0.5) -> torch.Tensor:
    """Each round's fraction of num_to_select, as the fp32 the reference
    multiplies with (projected.py:845, 897-899)."""
    out, remaining = [], restore_frac
    for _ in range(n_iters):
        this = remaining * decay
        remaining -= this
        out.append(this)
    return torch.tensor(out, dtype=torch.float32)


def restore_swap(attn_full: torch.Tensor, vbar_bf16: torch.Tensor, M: torch.Tensor,
                 nts: torch.Tensor, n_cand: int, n_iters: int = 5, track_best: bool = True,
                 restore_frac: float = 0.5, decay: float = 0.5):
    """Returns (drop (rows, n_cand) bool, s (rows, n_cand) bf16)."""
    a = attn_full.contiguous()
    rows = a.numel() // a.shape[-1]
    nkp = a.shape[-1]
    heads = vbar_bf16.numel() // (nkp * 64)
    nq = rows // heads
    vb = vbar_bf16.contiguous()
    tk = vbar_metric(vb, M, n_cand)
    nh = M.shape[0]
    fr = round_fracs(n_iters, restore_frac, decay)
    drop = torch.empty(rows, n_cand, dtype=torch.uint8)
    s = torch.empty(rows, n_cand, dtype=torch.int16)
    nt = nts.to(torch.int32).contiguous().view(-1)
    vbi, Mf, tki = vb.view(torch.int16), M.float().contiguous(), tk.view(torch.int16)
    lib().ro_restore_swap(_dt(a), _p(a), _p(vbi), _p(Mf),
                          _p(tki), _p(nt), rows, nq, nh, nkp, n_cand, n_iters, _p(fr),
                          int(track_best), _p(drop), _p(s))
    return drop.bool(), s.view(torch.bfloat16)


def top_m_mask(q: torch.Tensor, counts: torch.Tensor, largest: bool = True) -> torch.Tensor:
    q = q.contiguous()
    n = q.shape[-1]
    rows = q.numel() // n
    out = torch.empty(q.shape, dtype=torch.uint8)
    c = counts.to(torch.int32).clamp(min=0).contiguous().view(-1)
    lib().ro_top_m_mask(_dt(q), _p(q), _p(c), rows, n, int(largest), _p(out))
    return out.bool()


def keep_lists(keep: torch.Tensor, sink_blocks: int, lead_blocks: int = 0):
    k = keep.to(torch.uint8).contiguous()
    n_cand = k.shape[-1]
    rows = k.numel() // n_cand
    width = n_cand + sink_blocks
    lists = torch.full((rows, width), -1, dtype=torch.int32)
    counts = torch.empty(rows, dtype=torch.int32)
    lib().ro_keep_lists(_p(k), rows, n_cand, sink_blocks, lead_blocks, _p(lists), _p(counts))
    return lists, counts


def quant_blocks(x16: torch.Tensor, blk: int):
    """x16 (rows, T, 64) fp32 holding fp16-rounded values -> (int8, scales)."""
    x = x16.float().contiguous()
    rows, T, _ = x.shape
    nb = -(-T // blk)
    q = torch.empty(rows, T, 64, dtype=torch.int8)
    sc = torch.empty(rows, nb, dtype=torch.float32)
    lib().ro_quant_blocks(_p(x), rows, T, blk, _p(q), _p(sc))
    return q, sc


def key_mean(k16: torch.Tensor) -> torch.Tensor:
    x = k16.float().contiguous()
    rows, T, _ = x.shape
    km = torch.empty(rows, 64, dtype=torch.float32)
    lib().ro_key_mean(_p(x), rows, T, _p(km))
    return km


def quantize_qk(q_patch: torch.Tensor, key: torch.Tensor):
    """run_block_sparse_kernel's quantisation (attention.py:226-233):
    fp16 casts, km over all keys, per-block int8 of q (128) and k - km (64)."""
    rows = q_patch.shape[0] * q_patch.shape[1]
    q16 = q_patch.reshape(rows, -1, 64).to(torch.float16).float()
    k16 = key.reshape(rows, -1, 64).to(torch.float16).float()
    km = key_mean(k16)
    kc = (k16 - km.unsqueeze(1)).to(torch.float16).float()
    q8, qs = quant_blocks(q16, KS_Q)
    k8, ks = quant_blocks(kc, KS_K)
    return q8, qs, k8, ks, km


def sparse_attn_rows(q8, qs, k8, ks, v16, lists, counts, samples, sm_scale=None):
    """fp64 reference attention for sampled (row, q-block) pairs.  Returns
    (n_samples, 128, 64) fp32."""
    rows, Tq, _ = q8.shape
    Tk = k8.shape[1]
    if sm_scale is None:
        sm_scale = 1.0 / math.sqrt(64)
    sr = torch.tensor([s[0] for s in samples], dtype=torch.int32)
    sq = torch.tensor([s[1] for s in samples], dtype=torch.int32)
    out = torch.zeros(len(samples), 128, 64, dtype=torch.float32)
    keep = [q8.contiguous(), k8.contiguous(), v16.float().contiguous(), qs.contiguous(), ks.contiguous(),
            lists.to(torch.int32).contiguous(), counts.to(torch.int32).contiguous()]
    lib().ro_sparse_attn_rows(_p(keep[0]), _p(keep[1]), _p(keep[2]),
                              _p(keep[3]), _p(keep[4]), Tq, Tk,
                              _p(keep[5]), _p(keep[6]),
                              lists.shape[-1], _p(sr), _p(sq), len(samples), _f(sm_scale), _p(out))
    return out


def gathered_attention_fp32(q_patch, key, value, lists, counts, sm_scale=None, threads=None):
    """Block-sparse attention in fp32 on the host cores, the CPU form of
    run_block_sparse_kernel (attention.py:217-243): for every (head, 128-query
    block) row, the listed 64-key blocks of K and V are gathered and
    softmax(Q K^T * sm_scale) V is computed with torch's fp32 matmuls; keys
    past Tk are masked.  q_patch (B, H, Tq, 64), key/value (B, H, Tk, 64) in
    any float dtype; lists/counts as ress_b200 emits them, rows = B*H*nq.
    Returns (B*H, Tq, 64) fp32.  A timing baseline, not a parity reference
    (the GPU path quantises Q and K to int8 as SpargeAttn does)."""
    if threads is not None:
        torch.set_num_threads(threads)
    B, H, Tq, D = q_patch.shape
    BH = B * H
    Tk = key.shape[-2]
    nq = -(-Tq // KS_Q)
    nkb = -(-Tk // KS_K)
    pad = nkb * KS_K - Tk
    if sm_scale is None:
        sm_scale = 1.0 / math.sqrt(D)
    qf = q_patch.reshape(BH, Tq, D).float()
    kb = torch.nn.functional.pad(key.reshape(BH, Tk, D).float(), (0, 0, 0, pad)).view(BH, nkb, KS_K, D)
    vb = torch.nn.functional.pad(value.reshape(BH, Tk, D).float(), (0, 0, 0, pad)).view(BH, nkb, KS_K, D)
    lists = lists.view(BH, nq, -1)
    counts = counts.view(BH, nq)
    out = torch.zeros(BH, Tq, D, dtype=torch.float32)
    for h in range(BH):
        for b in range(nq):
            c = int(counts[h, b])
            if c <= 0:
                continue
            idx = lists[h, b, :c].long()
            s = (qf[h, b * KS_Q:(b + 1) * KS_Q] @ kb[h, idx].reshape(-1, D).T) * sm_scale
            if pad and int(idx[-1]) == nkb - 1:
                s[:, -pad:] = float("-inf")
            out[h, b * KS_Q:(b + 1) * KS_Q] = torch.softmax(s, -1) @ vb[h, idx].reshape(-1, D)
    return out


# --------------------------------------------------------------------------- layer

def layer_select(q_patch, k_patch, v_patch, n_special_keys, M, head_scores=None, mode="ress",
                 sparse_ratio=0.5, cdf_threshold=None, n_iters=5, track_best=True,
                 restore_frac=0.5, decay=0.5, beta=1.0):
    """One layer's selection, chained like ress_attention_forward
    (attention.py:446-581).  Inputs (B, nh, T, 64) CPU tensors in the layer
    dtype.  mode: "ress" (restore-swap order) or "prob" (probability order).
    head_scores: (nh,) or None for a uniform budget.  Returns a dict."""
    B, nh, Tp, D = q_patch.shape
    rows = B * nh
    qp = q_patch.reshape(rows, Tp, D)
    kp = k_patch.reshape(rows, Tp, D)
    vp = v_patch.reshape(rows, Tp, D)
    qbar = pool_mean(qp, KS_Q)
    kbar = pool_mean(kp, KS_K)
    attn_full = predict(qbar, kbar)
    has_special = n_special_keys > 0
    n_cand = Tp // KS_K if has_special else -(-Tp // KS_K)
    cond = attn_cond(attn_full, n_cand)
    nq = attn_full.shape[1]
    base = baseline(cond, sparse_ratio, cdf_threshold).view(B, nh, nq)
    if head_scores is not None:
        nts = hess_adjust(base, scores_norm(head_scores), n_cand, beta=beta,
                          min_clamp=min(2, n_cand))
    else:
        nts = base.clamp(min=min(2, n_cand))
    Tk = Tp + n_special_keys
    sink_blocks = -(-Tk // KS_K) - n_cand
    out = dict(qbar=qbar, kbar=kbar, attn_full=attn_full, attn_cond=cond, baseline=base, nts=nts,
               n_cand=n_cand, sink_blocks=sink_blocks)
    if mode == "ress":
        vbar = pool_mean(vp, KS_K)
        vbar_bf16 = vbar.to(torch.bfloat16)
        drop, s = restore_swap(attn_full, vbar_bf16, M, nts.view(-1), n_cand, n_iters, track_best,
                               restore_frac, decay)
        keep = ~drop
        out.update(vbar=vbar, drop=drop, s=s)
    else:
        keep = top_m_mask(cond.view(rows * nq, n_cand), nts.view(-1))
    lists, counts = keep_lists(keep.view(rows * nq, n_cand), sink_blocks)
    out.update(keep=keep.view(B, nh, nq, n_cand), lists=lists, counts=counts)
    return out
