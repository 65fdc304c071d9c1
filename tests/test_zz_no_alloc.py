"""ress_restore_swap_noalloc: the restore-swap entry point for callers that
cannot allocate device memory (a plain C/FFI host program without a device
allocator, or a process that reserves all device memory up front and may not
call cudaMalloc later).  It takes no workspace and uses a 4 MiB static
device array inside the library instead.

These tests call it through the C ABI with raw pointers, exactly as such a
caller would, and require its outputs to equal those of ress_restore_swap
(which is given a workspace allocated here) bit for bit, on two calls in a
row: the shared array keeps the previous call's contents, and the second call
must not depend on them.  Two layers are covered: a 6-frame, 16-head layer,
whose pooled values fit in shared memory, and a 60-frame, 2-head layer, which
runs the large-layer kernel that also keeps a transposed copy of the pooled
values in the array.  Collected last so that a stop-at-first-failure run has
run every other test first; it also passes alone in a fresh process."""

import ctypes

import pytest
import torch

from ress_b200 import _lib
from ress_b200 import kernels as K
from ress_b200 import synth


def _p(t):
    return ctypes.c_void_p(0 if t is None else t.data_ptr())


def _host_ptrs(n):
    """Non-null host addresses standing in for device pointers in calls that
    must be refused before any pointer is used."""
    buf = (ctypes.c_char * 64)()
    return [ctypes.c_void_p(ctypes.addressof(buf) + 8 * i) for i in range(n)], buf


def test_oversized_problem_is_rejected_before_launch():
    """A problem whose scratch exceeds the static array returns RESS_E_SCRATCH
    without touching any pointer or the device."""
    lib = _lib.load()
    fr = (ctypes.c_float * 5)(*K.round_fracs(5))
    (af, vb, M, nts, drop, s, lists, counts, status), keep = _host_ptrs(9)
    rc = lib.ress_restore_swap_noalloc(1, af, vb, M, nts, 1, 16, 2140, 4279, 4278, 5, fr, 1, drop, s, lists,
                                       counts, 4294, 16, 0, status, None)
    assert rc == _lib.RESS_E_SCRATCH
    assert b"static array" in lib.ress_error_string(rc)


def test_argument_errors_come_before_the_size_check():
    """Invalid arguments give the same code as ress_restore_swap even when the
    problem would also be too large for the array."""
    lib = _lib.load()
    fr = (ctypes.c_float * 5)(*K.round_fracs(5))
    (af, vb, M, nts, drop, s, lists, counts, status), keep = _host_ptrs(9)
    # n_cand > nkp
    rc = lib.ress_restore_swap_noalloc(1, af, vb, M, nts, 1, 16, 2140, 4279, 4280, 5, fr, 1, drop, s, lists,
                                       counts, 4294, 16, 0, status, None)
    assert rc == _lib.RESS_E_ARG
    # a null input pointer
    rc = lib.ress_restore_swap_noalloc(1, None, vb, M, nts, 1, 16, 2140, 4279, 4278, 5, fr, 1, drop, s, lists,
                                       counts, 4294, 16, 0, status, None)
    assert rc == _lib.RESS_E_ARG
    # more rounds than the kernels take
    fr40 = (ctypes.c_float * 40)(*([0.1] * 40))
    rc = lib.ress_restore_swap_noalloc(1, af, vb, M, nts, 1, 16, 2140, 4279, 4278, 40, fr40, 1, drop, s, lists,
                                       counts, 4294, 16, 0, status, None)
    assert rc == _lib.RESS_E_ARG
    # heads x q-blocks past the int range
    rc = lib.ress_restore_swap_noalloc(1, af, vb, M, nts, 1 << 16, 1 << 16, 2, 4, 4, 5, fr, 1, drop, s, lists,
                                       counts, 8, 0, 0, status, None)
    assert rc == _lib.RESS_E_SHAPE


def _layer(frames, heads, seed, sr):
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    shape = synth.LayerShape(n_frames=frames)
    q, k, v = (t[:, :heads].contiguous() for t in synth.layer_qkv(shape, seed=seed, dtype=torch.bfloat16,
                                                                  device=dev))
    L = K.Layout(1, heads, shape.n_frames, shape.n_special, shape.hw)
    qbar, _, _ = K.pool_quant_q(q, L, quant=False)
    kbar, vbar, _, _, _, _ = K.pool_quant_kv(k, v, L, quant=False)
    attn_full, attn_cond = K.predict(qbar, kbar, L.n_cand)
    hs = synth.fisher_table(seed=1)[0, 2, :heads]
    nts = K.hess_adjust(K.baseline(attn_cond, sr).view(1, heads, -1), K.scores_norm(hs), L.n_cand,
                        min_clamp=2).view(-1)
    M = synth.metric_from_weight(synth.out_proj_weight())[:heads].contiguous().to(dev)
    return dev, L, attn_full, vbar, M, nts


@pytest.mark.gpu
@pytest.mark.parametrize("frames,heads,seed,sr", [(6, 16, 0, 0.5), (60, 2, 3, 0.6)])
def test_noalloc_matches_restore_swap_twice(frames, heads, seed, sr):
    lib = _lib.load()
    dev, L, attn_full, vbar, M, nts = _layer(frames, heads, seed, sr)
    need = lib.ress_workspace_size(heads, L.Tp, L.Tk, L.n_cand)
    assert need <= _lib.NOALLOC_SCRATCH_BYTES
    rows, width = heads * L.nq, L.n_cand + L.sink_blocks
    fr = (ctypes.c_float * 5)(*K.round_fracs(5))
    stream = ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
    status = torch.zeros(1, dtype=torch.int32, device=dev)

    def outputs():
        return (torch.full((rows, L.n_cand), 7, dtype=torch.uint8, device=dev),
                torch.zeros(rows, L.n_cand, dtype=torch.bfloat16, device=dev),
                torch.full((rows, width), -1, dtype=torch.int32, device=dev),
                torch.zeros(rows, dtype=torch.int32, device=dev))

    ref = outputs()
    ws = K.workspace(dev, heads, L.Tp, L.Tk, L.n_cand)
    rc = lib.ress_restore_swap(_lib.RESS_BF16, _p(attn_full), _p(vbar), _p(M), _p(nts), 1, heads, L.nq, L.nkp,
                               L.n_cand, 5, fr, 1, _p(ref[0]), _p(ref[1]), _p(ref[2]), _p(ref[3]), width,
                               L.sink_blocks, 0, _p(status), _p(ws), stream)
    assert rc == 0
    for call in range(2):
        got = outputs()
        rc = lib.ress_restore_swap_noalloc(_lib.RESS_BF16, _p(attn_full), _p(vbar), _p(M), _p(nts), 1, heads,
                                           L.nq, L.nkp, L.n_cand, 5, fr, 1, _p(got[0]), _p(got[1]), _p(got[2]),
                                           _p(got[3]), width, L.sink_blocks, 0, _p(status), stream)
        assert rc == 0, lib.ress_error_string(rc)
        torch.cuda.synchronize()
        assert int(status.item()) == 0
        for a, b in zip(ref, got):
            assert torch.equal(a, b), f"call {call}: output differs from ress_restore_swap"
