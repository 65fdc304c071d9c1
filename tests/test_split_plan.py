"""Host-side launch planning, no GPU: the decision of the split attention
launch (kernels.split_piece, the split=None path of kernels.sparse_attn:
which launches spread their longest rows over two CTAs, and with what piece
size), and the token and block counts kernels.Layout gives the benchmark
configurations.  The kernel side is covered by tests/test_gpu_kernels.py."""

import pytest

from ress_b200 import kernels as K

SMS = 148  # B200


@pytest.mark.parametrize("rows,width,expect", [
    (16 * 343, 687, False),       # cfg2 on one GPU: 5,488 rows, many waves
    (8 * 343, 687, False),        # heads over 2 GPUs
    (4 * 343, 687, False),        # heads over 4 GPUs: 1,372 rows, still >= 3 waves of 296 CTAs
    (2 * 343, 687, 344),          # heads over 8 GPUs: 686 rows split at half the width
    (16 * 43, 86, 43),            # a 4-frame layer: 688 rows
    (100, 40, 32),                # the piece never goes below 32 blocks
    (100, K.SPLIT_MAX_WIDTH + 1, False),
])
def test_split_piece_on_a_b200(rows, width, expect):
    assert K.split_piece(rows, width, SMS) == expect


def test_unscheduled_launches_never_split():
    assert K.split_piece(10, 687, SMS, schedule=False) is False


def test_wave_threshold():
    limit = K.SPLIT_WAVES * 2 * SMS
    assert K.split_piece(limit - 1, 687, SMS) == 344
    assert K.split_piece(limit, 687, SMS) is False


def test_no_row_needs_more_than_split_max_pieces():
    # a row holds at most the list width of blocks, so ceil(count / piece)
    # never exceeds the kernel's piece limit
    for width in range(1, 3000, 7):
        piece = K.split_piece(1, width, SMS)
        assert piece >= 32
        assert -(-width // piece) <= K.SPLIT_MAX


@pytest.mark.parametrize("frames,Tp,Tk,nq,nkp,n_cand,nkb,sinks", [
    (4, 5476, 5496, 43, 86, 85, 86, 1),              # config 1
    (32, 43808, 43968, 343, 685, 684, 687, 3),       # configs 2 and 3
    (200, 273800, 274800, 2140, 4279, 4278, 4294, 16),  # config 4
])
def test_layout_of_the_configs(frames, Tp, Tk, nq, nkp, n_cand, nkb, sinks):
    """Token and block counts of the VGGT global layer (5 special tokens and
    37 x 37 patches per frame; attention.py:446-491 for the candidate/sink
    split) for the benchmark configurations."""
    L = K.Layout(1, 16, frames, 5, 37 * 37)
    assert (L.Tp, L.Tk, L.nq, L.nkp, L.n_cand, L.nkb, L.sink_blocks) == (Tp, Tk, nq, nkp, n_cand, nkb, sinks)
