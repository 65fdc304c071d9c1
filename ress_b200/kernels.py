"""Tensor-level wrappers over the C ABI (include/ress_sm100.h).

Each wrapper checks its torch CUDA tensors, allocates the outputs with the
torch caching allocator, and enqueues the library's kernels on the current
stream.  None of them synchronises.  Device-side conditions (HeSS
non-convergence, an expired bounded wait, a keep-list overflow) are OR-ed
into a per-device status word that ``check_status`` reads.
"""

from __future__ import annotations

import ctypes
import math
from dataclasses import dataclass

import torch

from . import _lib
from ._lib import RESS_BF16, RESS_F32, RessError, check

KS_Q, KS_K, HD = 128, 64, 64

_status = {}


def _dev_ok(*ts):
    for t in ts:
        if t is None:
            continue
        if not t.is_cuda:
            raise RessError("ress_b200 kernels run on CUDA tensors only (no CPU fallback)")


def _ptr(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _stream(device=None):
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def _dtype_code(dt) -> int:
    if dt == torch.float32:
        return RESS_F32
    if dt == torch.bfloat16:
        return RESS_BF16
    raise RessError(f"unsupported dtype {dt} (float32 or bfloat16)")


def status_word(device) -> torch.Tensor:
    device = torch.device(device)
    if device.index is None:
        device = torch.device("cuda", torch.cuda.current_device())
    t = _status.get(device)
    if t is None:
        t = torch.zeros(1, dtype=torch.int32, device=device)
        _status[device] = t
    return t


def check_status(device=None, reset: bool = True) -> int:
    """Read (synchronising) and clear the device status word; raise on errors."""
    st = status_word(device if device is not None else "cuda")
    v = int(st.item())
    if reset and v:
        st.zero_()
    if v & _lib.STATUS_HESS_NO_CONVERGENCE:
        raise RuntimeError("adjust_attention_selection did not converge in 1000 iterations")
    if v & _lib.STATUS_ATTN_WAIT_TIMEOUT:
        raise RessError("sparse attention kernel: a bounded wait expired (result invalid)")
    if v & _lib.STATUS_LIST_OVERFLOW:
        raise RessError("keep list longer than its buffer")
    return v


def workspace(device, BH, Tp, Tk, n_cand) -> torch.Tensor:
    n = _lib.load().ress_workspace_size(BH, Tp, Tk, n_cand)
    return torch.empty(n, dtype=torch.uint8, device=device)


@dataclass(frozen=True)
class Layout:
    """Token layout of a (B, H, frames*(special+hw), 64) layer tensor."""

    B: int
    H: int
    frames: int
    special: int
    hw: int

    @property
    def Tp(self):
        return self.frames * self.hw

    @property
    def Ts(self):
        return self.frames * self.special

    @property
    def Tk(self):
        return self.Tp + self.Ts

    @property
    def nq(self):
        return -(-self.Tp // KS_Q)

    @property
    def nkp(self):
        return -(-self.Tp // KS_K)

    @property
    def nkb(self):
        return -(-self.Tk // KS_K)

    @property
    def n_cand(self):
        # attention.py:453-456 with sink protection on
        return self.Tp // KS_K if self.special > 0 else self.nkp

    @property
    def sink_blocks(self):
        return self.nkb - self.n_cand

    @staticmethod
    def plain(x: torch.Tensor) -> "Layout":
        B, H, T, _ = x.shape
        return Layout(B, H, 1, 0, T)


def _strides(x: torch.Tensor, L: Layout):
    if x.dim() != 4 or x.shape[-1] != HD or x.stride(-1) != 1:
        raise RessError("layer tensors must be (B, H, T, 64) with a contiguous last dim")
    if x.shape[0] != L.B or x.shape[1] != L.H or x.shape[2] != L.frames * (L.special + L.hw):
        raise RessError(f"tensor shape {tuple(x.shape)} does not match layout {L}")
    return x.stride(0), x.stride(1), x.stride(2)


# ----------------------------------------------------------------- scoring
def pool_quant_q(q, L: Layout, pool=True, quant=True):
    _dev_ok(q)
    sb, sh, st = _strides(q, L)
    BH = L.B * L.H
    qbar = torch.empty(BH, L.nq, HD, dtype=q.dtype, device=q.device) if pool else None
    q8 = torch.empty(BH, L.Tp, HD, dtype=torch.int8, device=q.device) if quant else None
    qs = torch.empty(BH, L.nq, dtype=torch.float32, device=q.device) if quant else None
    check(_lib.load().ress_pool_quant_q(_ptr(q), _dtype_code(q.dtype), L.B, L.H, L.frames, L.special, L.hw,
                                        sb, sh, st, _ptr(qbar), _ptr(q8), _ptr(qs), _stream(q.device)),
          "ress_pool_quant_q")
    return qbar, q8, qs


def qkv_prologue_scored(qkv, L: Layout, qn_weight=None, qn_bias=None, kn_weight=None, kn_bias=None, eps=1e-5,
                        pos=None, rope_cos=None, rope_sin=None):
    """bf16 (B, T, 3*H*64) qkv Linear output of a global layer (layout L) ->
    dict(k, v: (B, H, T, 64) bf16; q_special: (B*H, frames*S, 64) bf16 or
    None; qbar, q8, qs as pool_quant_q on qkv_prologue's q).  The patch
    tokens' q is normalised, rotated, pooled and quantised in one pass and
    never written (ress_qkv_prologue_scored)."""
    _dev_ok(qkv)
    B, T, C3 = qkv.shape
    H = L.H
    if qkv.dtype != torch.bfloat16 or C3 != 3 * H * HD or not qkv.is_contiguous():
        raise RessError("qkv must be contiguous bf16 (B, T, 3*H*64)")
    if B != L.B or T != L.frames * (L.special + L.hw):
        raise RessError("qkv does not hold the layout's tokens")
    dev = qkv.device
    k, v = (torch.empty(B, H, T, HD, dtype=qkv.dtype, device=dev) for _ in range(2))
    q_special = torch.empty(B * H, L.frames * L.special, HD, dtype=qkv.dtype, device=dev) if L.special else None
    qbar = torch.empty(B * H, L.nq, HD, dtype=qkv.dtype, device=dev)
    q8 = torch.empty(B * H, L.Tp, HD, dtype=torch.int8, device=dev)
    qs = torch.empty(B * H, L.nq, dtype=torch.float32, device=dev)
    f32 = lambda t: None if t is None else t.detach().to(device=dev, dtype=torch.float32).contiguous()
    qw, qb, kw, kb = f32(qn_weight), f32(qn_bias), f32(kn_weight), f32(kn_bias)
    rope_len = 0
    if rope_cos is not None:
        rope_cos, rope_sin = rope_cos.contiguous(), rope_sin.contiguous()
        if rope_cos.dtype != qkv.dtype or rope_cos.shape[-1] != 32:
            raise RessError("rotary tables must be (max_pos, 32) in the qkv dtype")
        rope_len = rope_cos.shape[0]
        pos = pos.to(dtype=torch.int64).contiguous()
    check(_lib.load().ress_qkv_prologue_scored(_ptr(qkv), B, T, H, L.special, L.hw, _ptr(qw), _ptr(qb), _ptr(kw),
                                               _ptr(kb), ctypes.c_float(eps), _ptr(pos), _ptr(rope_cos),
                                               _ptr(rope_sin), rope_len, _ptr(q_special), _ptr(k), _ptr(v),
                                               _ptr(qbar), _ptr(q8), _ptr(qs), _stream(dev)),
          "ress_qkv_prologue_scored")
    return dict(k=k, v=v, q_special=q_special, qbar=qbar, q8=q8, qs=qs)


def pool_quant_kv(k, v, L: Layout, pool=True, quant=True, ws=None):
    _dev_ok(k, v)
    if k.stride() != v.stride() or k.dtype != v.dtype:
        raise RessError("k and v must share strides and dtype")
    sb, sh, st = _strides(k, L)
    BH = L.B * L.H
    dev = k.device
    kbar = torch.empty(BH, L.nkp, HD, dtype=k.dtype, device=dev) if pool else None
    vbar = torch.empty(BH, L.nkp, HD, dtype=k.dtype, device=dev) if pool else None
    k8 = torch.empty(BH, L.Tk, HD, dtype=torch.int8, device=dev) if quant else None
    ks = torch.empty(BH, L.nkb, dtype=torch.float32, device=dev) if quant else None
    v16 = torch.empty(BH, L.Tk, HD, dtype=torch.float16, device=dev) if quant else None
    km = torch.empty(BH, HD, dtype=torch.float32, device=dev) if quant else None
    if quant and ws is None:
        ws = workspace(dev, BH, L.Tp, L.Tk, max(1, L.n_cand))
    check(_lib.load().ress_pool_quant_kv(_ptr(k), _ptr(v), _dtype_code(k.dtype), L.B, L.H, L.frames, L.special,
                                         L.hw, sb, sh, st, _ptr(kbar), _ptr(vbar), _ptr(k8), _ptr(ks), _ptr(v16),
                                         _ptr(km), _ptr(ws if quant else None), _stream(dev)),
          "ress_pool_quant_kv")
    return kbar, vbar, k8, ks, v16, km


def predict(qbar, kbar, n_cand, full=True, cond=True):
    """(BH, nq, 64), (BH, nkp, 64) -> attn_full (BH, nq, nkp), attn_cond (BH, nq, n_cand)."""
    _dev_ok(qbar, kbar)
    BH, nq, _ = qbar.shape
    nkp = kbar.shape[1]
    af = torch.empty(BH, nq, nkp, dtype=qbar.dtype, device=qbar.device) if full else None
    ac = torch.empty(BH, nq, n_cand, dtype=qbar.dtype, device=qbar.device) if cond else None
    qc, kc = qbar.contiguous(), kbar.contiguous()
    check(_lib.load().ress_predict(_dtype_code(qc.dtype), _ptr(qc), _ptr(kc), BH, nq, nkp, n_cand, _ptr(af), _ptr(ac),
                                   _stream(qbar.device)), "ress_predict")
    return af, ac


def cdf_value(cdf_threshold: float, eps: float = 1e-5) -> float:
    """The fp32 value the reference's searchsorted compares (attention.py:283-285)."""
    return float(torch.as_tensor(cdf_threshold, dtype=torch.float32) + eps)


def baseline(cond, sparse_ratio=None, cdf_threshold=None):
    """compute_baseline_num_to_select on (..., n) -> (...) int32."""
    _dev_ok(cond)
    if sparse_ratio is None and cdf_threshold is None:
        raise AssertionError("at least one of sparse_ratio/cdf_threshold required")
    c = cond.contiguous()
    n = c.shape[-1]
    rows = c.numel() // n
    topk = int(n * (1 - sparse_ratio)) if sparse_ratio is not None else -1
    out = torch.empty(c.shape[:-1], dtype=torch.int32, device=c.device)
    use = cdf_threshold is not None
    cv = cdf_value(cdf_threshold) if use else 0.0
    check(_lib.load().ress_baseline(_dtype_code(c.dtype), _ptr(c), rows, n, int(use), ctypes.c_float(cv), topk,
                                    _ptr(out), _stream(c.device)), "ress_baseline")
    return out


def scores_norm(head_scores: torch.Tensor) -> torch.Tensor:
    """head_scores / head_scores.sum(), the sum taken sequentially in fp32, or
    the uniform 1/H when that sum is not finite or not positive
    (_proportional.py:184-188).  Host-side (H scalars)."""
    hs = head_scores.detach().float().cpu().contiguous()
    s = torch.zeros((), dtype=torch.float32)
    for x in hs:
        s = s + x
    if not bool(torch.isfinite(s)) or float(s) <= 0:
        return torch.full_like(hs, 1.0 / hs.numel())
    return hs / s


def hess_adjust(base, snorm, max_val, beta=1.0, min_clamp=0, max_iters=1000):
    """base (B, H, nq) int -> (B, H, nq) int32; snorm (H,) fp32 (any device)."""
    _dev_ok(base)
    b = base.to(torch.int32).contiguous()
    B, H, nq = b.shape
    sn = snorm.to(device=b.device, dtype=torch.float32).contiguous()
    out = torch.empty_like(b)
    omb = float(torch.tensor(1 - beta, dtype=torch.float32))
    check(_lib.load().ress_hess_adjust(_ptr(b), _ptr(sn), B, H, nq, int(max_val), ctypes.c_float(omb),
                                       ctypes.c_float(float(beta)), int(max_iters), int(min_clamp), _ptr(out),
                                       _ptr(status_word(b.device)), _stream(b.device)), "ress_hess_adjust")
    return out


def round_fracs(n_iters, restore_frac=0.5, decay=0.5):
    """Per-round fraction of num_to_select, as the fp32 values the reference
    multiplies with (projected.py:845, 897-899)."""
    out, remaining = [], restore_frac
    for _ in range(n_iters):
        this = remaining * decay
        remaining -= this
        out.append(float(torch.tensor(this, dtype=torch.float32)))
    return out


def restore_swap(attn_full, vbar, M, nts, n_cand, n_iters=5, track_best=True, restore_frac=0.5, decay=0.5,
                 sink_blocks=0, lead_blocks=0, want_drop=False, want_s=False, want_lists=True, ws=None,
                 list_width=None):
    """attn_full (B, H, nq, nkp) or (BH, nq, nkp); vbar (.., nkp, 64); M (H, 64, 64) fp32;
    nts (rows,) int.  Returns dict(drop, s, lists, counts)."""
    _dev_ok(attn_full, vbar, M, nts)
    nkp = attn_full.shape[-1]
    nq = attn_full.shape[-2]
    H = M.shape[0]
    BH = attn_full.numel() // (nq * nkp)
    if BH % H:
        raise RessError("head count of M does not divide the rows")
    B = BH // H
    rows = BH * nq
    dev = attn_full.device
    af = attn_full.contiguous()
    vb = vbar.to(af.dtype).contiguous()
    fr = round_fracs(n_iters, restore_frac, decay)
    fr_c = (ctypes.c_float * max(1, len(fr)))(*fr) if fr else None
    nt = nts.to(device=dev, dtype=torch.int32).contiguous().view(-1)
    if nt.numel() != rows:
        raise RessError("num_to_select has the wrong number of rows")
    drop = torch.empty(rows, n_cand, dtype=torch.uint8, device=dev) if want_drop else None
    s = torch.empty(rows, n_cand, dtype=torch.bfloat16, device=dev) if want_s else None
    width = list_width or (n_cand + sink_blocks)
    lists = torch.empty(rows, width, dtype=torch.int32, device=dev) if want_lists else None
    counts = torch.empty(rows, dtype=torch.int32, device=dev) if want_lists else None
    if ws is None:
        ws = workspace(dev, BH, nkp * KS_K, nkp * KS_K, n_cand)
    Mf = M.float().contiguous()
    check(_lib.load().ress_restore_swap(_dtype_code(af.dtype), _ptr(af), _ptr(vb), _ptr(Mf),
                                        _ptr(nt), B, H, nq, nkp, n_cand, n_iters, fr_c, int(track_best), _ptr(drop),
                                        _ptr(s), _ptr(lists), _ptr(counts), width, sink_blocks, lead_blocks,
                                        _ptr(status_word(dev)), _ptr(ws), _stream(dev)), "ress_restore_swap")
    return dict(drop=drop, s=s, lists=lists, counts=counts)


def select_prob(cond, nts, sink_blocks=0, lead_blocks=0, want_keep=False, want_lists=True, list_width=None):
    _dev_ok(cond, nts)
    c = cond.contiguous()
    n = c.shape[-1]
    rows = c.numel() // n
    nt = nts.to(device=c.device, dtype=torch.int32).contiguous().view(-1)
    keep = torch.empty(rows, n, dtype=torch.uint8, device=c.device) if want_keep else None
    width = list_width or (n + sink_blocks)
    lists = torch.empty(rows, width, dtype=torch.int32, device=c.device) if want_lists else None
    counts = torch.empty(rows, dtype=torch.int32, device=c.device) if want_lists else None
    check(_lib.load().ress_select_prob(_dtype_code(c.dtype), _ptr(c), _ptr(nt), rows, n, _ptr(keep), _ptr(lists),
                                       _ptr(counts), width, sink_blocks, lead_blocks, _ptr(status_word(c.device)),
                                       _stream(c.device)), "ress_select_prob")
    return dict(keep=keep, lists=lists, counts=counts)


def top_m_mask(q, counts, largest=True):
    _dev_ok(q)
    qc = q.contiguous()
    n = qc.shape[-1]
    rows = qc.numel() // n
    cn = counts.to(device=qc.device, dtype=torch.int32).contiguous().view(-1)
    out = torch.empty(qc.shape, dtype=torch.uint8, device=qc.device)
    if rows == 0:
        return out.bool()
    if qc.dtype not in (torch.float32, torch.bfloat16):
        qc = qc.float()
    check(_lib.load().ress_top_m_mask(_dtype_code(qc.dtype), _ptr(qc), _ptr(cn), rows, n, int(largest), _ptr(out),
                                      _stream(qc.device)), "ress_top_m_mask")
    return out.view(torch.bool)


def round_step(P, term_k, s_sq, term_q, drop, per_iter, raw_bf16, q_bf16, g_norm_sq=None, kept_mass=None,
               k_eps=1e-6):
    _dev_ok(P, term_k, s_sq, term_q, drop, per_iter)
    p = P.contiguous()
    tk = term_k.to(p.dtype).contiguous()
    ss = s_sq.contiguous()
    n = p.shape[-1]
    rows = p.numel() // n
    tq = term_q.float().contiguous()
    dm = drop.contiguous().view(torch.uint8)
    pic = per_iter.to(torch.int32).contiguous()
    knorm = g_norm_sq is not None
    gn = g_norm_sq.float().contiguous() if knorm else None
    km = kept_mass.float().contiguous() if knorm else None
    new = torch.empty(p.shape, dtype=torch.uint8, device=p.device)
    cnt = torch.empty(p.shape[:-1], dtype=torch.int32, device=p.device)
    check(_lib.load().ress_round_step(_ptr(p), _ptr(tk), _ptr(ss), _dtype_code(p.dtype), _dtype_code(ss.dtype),
                                      _ptr(tq), _ptr(dm), _ptr(pic), _ptr(gn), _ptr(km), rows, n, int(raw_bf16),
                                      int(q_bf16), int(knorm), ctypes.c_float(k_eps), _ptr(new), _ptr(cnt),
                                      _stream(p.device)), "ress_round_step")
    return new.view(torch.bool), cnt


def map_to_lists(block_map):
    _dev_ok(block_map)
    m = block_map.contiguous().view(torch.uint8) if block_map.dtype == torch.bool else block_map.to(torch.uint8).contiguous()
    width = m.shape[-1]
    rows = m.numel() // width
    lists = torch.empty(rows, width, dtype=torch.int32, device=m.device)
    counts = torch.empty(rows, dtype=torch.int32, device=m.device)
    check(_lib.load().ress_map_to_lists(_ptr(m), rows, width, _ptr(lists), _ptr(counts), width,
                                        _ptr(status_word(m.device)), _stream(m.device)), "ress_map_to_lists")
    return lists, counts


def lists_to_map(lists, counts, width):
    """Dense bool map (rows, width) from keep lists (torch glue for API
    compatibility; not on the fused path)."""
    rows, lw = lists.shape
    ar = torch.arange(lw, device=lists.device)
    valid = ar.unsqueeze(0) < counts.unsqueeze(1)
    m = torch.zeros(rows, width + 1, dtype=torch.bool, device=lists.device)
    idx = torch.where(valid, lists.long(), torch.full_like(lists, width).long())
    m.scatter_(1, idx, True)
    return m[:, :width]


_SM_COUNT = {}


def _sm_count(dev) -> int:
    i = dev.index if dev.index is not None else torch.cuda.current_device()
    if i not in _SM_COUNT:
        _SM_COUNT[i] = torch.cuda.get_device_properties(i).multi_processor_count
    return _SM_COUNT[i]


# A launch with fewer rows than this many waves of CTAs (two per SM) splits
# its long rows (split=None); with more, the descending-length schedule alone
# keeps the last wave short.
SPLIT_WAVES = 3
SPLIT_MAX = 2  # pieces per row at most (attn.cu)
SPLIT_MAX_WIDTH = 16384  # widest keep list the split launch takes (attn.cu ORDER_MAX_WIDTH: one sort bin per count)


def split_piece(rows: int, list_width: int, sm_count: int, schedule: bool = True):
    """sparse_attn's split=None decision: the piece size in key blocks for a
    launch of ``rows`` rows with keep lists ``list_width`` wide on
    ``sm_count`` SMs, or False for one CTA per row.  Only launches of fewer
    than SPLIT_WAVES waves of CTAs (two per SM) split; a row longer than the
    piece then runs as up to SPLIT_MAX pieces."""
    if schedule and rows < SPLIT_WAVES * 2 * sm_count and list_width <= SPLIT_MAX_WIDTH:
        return max(32, (list_width + SPLIT_MAX - 1) // SPLIT_MAX)
    return False


def sparse_attn(q8, qscale, k8, kscale, v16, lists, counts, out=None, out_layout=None, sm_scale=None,
                schedule=True, split=False):
    """Block-sparse attention.  q8 (BH, Tq, 64); k8/v16 (BH, Tk, 64).
    out: fp32 tensor; with out_layout (a Layout) rows land at their full-layout
    positions of a (B, H, frames*(special+hw), 64) tensor.
    split: False (default) runs one CTA per row, the same bits whatever the
    launch; None lets launches of few rows (under SPLIT_WAVES waves) run rows
    longer than half the list width as two pieces on separate CTAs (outputs
    within the attention tolerance of the unsplit launch; split_piece
    decides); an int forces that piece size."""
    _dev_ok(q8, k8, v16, lists, counts)
    BH, Tq, _ = q8.shape
    Tk = k8.shape[1]
    dev = q8.device
    if out is None:
        out = torch.empty(BH, Tq, HD, dtype=torch.float32, device=dev)
    if out.dtype != torch.float32 or out.stride(-1) != 1:
        raise RessError("sparse_attn output must be fp32 with a contiguous last dim")
    if out_layout is None:
        o_sh, o_st, o_hw, o_sp = out.stride(0), out.stride(1), Tq, 0
    else:
        o_sh, o_st, o_hw, o_sp = out.stride(1), out.stride(2), out_layout.hw, out_layout.special
        if out_layout.B != 1:
            o_sh = out.stride(1)
            if out.stride(0) != out.stride(1) * out_layout.H:
                raise RessError("batched full-layout output must have stride(0) == H * stride(1)")
    if sm_scale is None:
        sm_scale = 1.0 / math.sqrt(HD)
    lw = lists.shape[-1]
    rows = counts.numel()
    if split is None:
        split = split_piece(rows, lw, _sm_count(dev), schedule)
    if split is not False:
        item_order = torch.empty(SPLIT_MAX * rows, dtype=torch.int32, device=dev)
        partial = torch.empty(rows * SPLIT_MAX * 128 * 68, dtype=torch.float32, device=dev)
        row_done = torch.zeros(rows, dtype=torch.int32, device=dev)
        check(_lib.load().ress_sparse_attn_split(_ptr(q8), _ptr(qscale), _ptr(k8), _ptr(kscale), _ptr(v16), BH, Tq,
                                                 Tk, _ptr(lists), _ptr(counts), lw, ctypes.c_float(sm_scale), _ptr(out),
                                                 o_sh, o_st, o_hw, o_sp, _ptr(status_word(dev)), _ptr(item_order),
                                                 int(split), _ptr(partial), _ptr(row_done), _stream(dev)),
              "ress_sparse_attn_split")
        return out
    if schedule:
        # rows launched in descending kept-block count (same bits as the plain order)
        order = torch.empty(counts.numel(), dtype=torch.int32, device=dev)
        check(_lib.load().ress_sparse_attn_sched(_ptr(q8), _ptr(qscale), _ptr(k8), _ptr(kscale), _ptr(v16), BH, Tq,
                                                 Tk, _ptr(lists), _ptr(counts), lw, ctypes.c_float(sm_scale), _ptr(out),
                                                 o_sh, o_st, o_hw, o_sp, _ptr(status_word(dev)), _ptr(order),
                                                 _stream(dev)), "ress_sparse_attn_sched")
        return out
    check(_lib.load().ress_sparse_attn(_ptr(q8), _ptr(qscale), _ptr(k8), _ptr(kscale), _ptr(v16), BH, Tq, Tk,
                                       _ptr(lists), _ptr(counts), lw, ctypes.c_float(sm_scale), _ptr(out), o_sh, o_st,
                                       o_hw, o_sp, _ptr(status_word(dev)), _stream(dev)), "ress_sparse_attn")
    return out


def dense_attn(q, k, v, out=None, out_bf16=None, sm_scale=None, out_rows=None):
    """Dense non-causal attention, bf16 on the tensor cores (ress_dense_attn).
    q (S, Tq, 64), k/v (S, Tk, 64) bf16 with a contiguous last dim and one
    stride per sequence and per row (e.g. (B*H) sequences of a contiguous
    (B, H, T, 64) tensor, viewed as (B*H, T, 64)).
    out: None -> a new (S, Tq, 64) tensor (bf16 unless out_bf16 is False);
    otherwise written in place, addressed by out_rows = (out_heads, out_sb,
    out_sh, out_st, group, period, offset) (see include/ress_sm100.h)."""
    _dev_ok(q, k, v)
    if q.dtype != torch.bfloat16 or k.dtype != torch.bfloat16 or v.dtype != torch.bfloat16:
        raise RessError("dense_attn takes bf16 q, k, v")
    if q.dim() != 3 or k.dim() != 3 or v.dim() != 3 or q.shape[-1] != HD or k.stride() != v.stride():
        raise RessError("dense_attn takes (S, T, 64) q, k, v with k and v sharing strides")
    if q.stride(-1) != 1 or k.stride(-1) != 1:
        raise RessError("dense_attn needs a contiguous last dim")
    S, Tq, _ = q.shape
    Tk = k.shape[1]
    dev = q.device
    if out is None:
        bf = True if out_bf16 is None else bool(out_bf16)
        out = torch.empty(S, Tq, HD, dtype=torch.bfloat16 if bf else torch.float32, device=dev)
        rows = (S, 0, out.stride(0), out.stride(1), Tq, 0, 0)
    else:
        bf = out.dtype == torch.bfloat16
        if not bf and out.dtype != torch.float32:
            raise RessError("dense_attn output must be fp32 or bf16")
        rows = out_rows if out_rows is not None else (S, 0, out.stride(0), out.stride(1), Tq, 0, 0)
    if sm_scale is None:
        sm_scale = 1.0 / math.sqrt(HD)
    heads, sb, sh, st, grp, period, off = rows
    check(_lib.load().ress_dense_attn(_ptr(q), _ptr(k), _ptr(v), S, Tq, Tk, q.stride(1), q.stride(0), k.stride(1),
                                      k.stride(0), ctypes.c_float(sm_scale), _ptr(out), int(bf), heads, sb, sh, st, grp,
                                      period, off, _ptr(status_word(dev)), _stream(dev)), "ress_dense_attn")
    return out


def qkv_prologue(qkv, H, qn_weight=None, qn_bias=None, kn_weight=None, kn_bias=None, eps=1e-5, pos=None,
                 rope_cos=None, rope_sin=None):
    """(B, T, 3*H*64) qkv Linear output -> q, k, v (B, H, T, 64): q/k LayerNorm
    (fp32 weights) and the optional 2-D rotary embedding in one pass."""
    _dev_ok(qkv)
    B, T, C3 = qkv.shape
    if C3 != 3 * H * HD or not qkv.is_contiguous():
        raise RessError("qkv must be contiguous (B, T, 3*H*64)")
    dev = qkv.device
    q, k, v = (torch.empty(B, H, T, HD, dtype=qkv.dtype, device=dev) for _ in range(3))
    f32 = lambda t: None if t is None else t.detach().to(device=dev, dtype=torch.float32).contiguous()
    qw, qb, kw, kb = f32(qn_weight), f32(qn_bias), f32(kn_weight), f32(kn_bias)
    rope_len = 0
    if rope_cos is not None:
        rope_cos, rope_sin = rope_cos.contiguous(), rope_sin.contiguous()
        if rope_cos.dtype != qkv.dtype or rope_cos.shape[-1] != 32:
            raise RessError("rotary tables must be (max_pos, 32) in the qkv dtype")
        rope_len = rope_cos.shape[0]
        pos = pos.to(dtype=torch.int64).contiguous()
    check(_lib.load().ress_qkv_prologue(_ptr(qkv), _dtype_code(qkv.dtype), B, T, H, _ptr(qw), _ptr(qb), _ptr(kw),
                                        _ptr(kb), ctypes.c_float(eps), _ptr(pos), _ptr(rope_cos), _ptr(rope_sin),
                                        rope_len, _ptr(q), _ptr(k), _ptr(v), _stream(dev)), "ress_qkv_prologue")
    return q, k, v
