"""Host-side checks of native logic that needs no GPU."""

import os
import subprocess

import numpy as np
import pytest

from conftest import GOLDEN, REPO

CSRC = os.path.join(REPO, "blockstreamer_b200", "csrc")


@pytest.fixture(scope="module")
def e2m1_check(tmp_path_factory):
    exe = str(tmp_path_factory.mktemp("native") / "e2m1_host_check")
    src = os.path.join(REPO, "tests", "native", "e2m1_host_check.cu")
    subprocess.run(["nvcc", "-std=c++17", "-O2", "-I", os.path.join(REPO, "include"), "-I", CSRC,
                    src, "-o", exe], check=True)
    res = subprocess.run([exe], capture_output=True, text=True)
    return res


def test_e2m1_decode_matches_reference_sweep(e2m1_check):
    """The library's general e2m1 decode equals the reference dequant for every
    byte under every e8m0 scale (golden sweep from dequantize_expert)."""
    lines = e2m1_check.stdout.splitlines()
    tab = np.array([[int(v, 16) for v in ln.split()] for ln in lines[: 256 * 256]], dtype=np.uint16)
    tab = tab.reshape(256, 256, 2)  # [scale][byte][lo/hi]
    golden = np.load(os.path.join(GOLDEN, "dequant_sweep.npz"))["bits"]  # [512 k, 256 rows=scale]
    # golden row r uses scale r; element k comes from byte k//2 (low nibble for even k)
    k = np.arange(512)
    byte = k // 2
    half = k % 2
    for s in range(256):
        assert np.array_equal(tab[s, byte, half], golden[:, s]), f"scale {s}"


def test_e2m1_fast_decode_equals_general(e2m1_check):
    last = e2m1_check.stdout.splitlines()[-1]
    assert last.startswith("MISMATCHES 0"), last
    assert e2m1_check.returncode == 0


def _stream_k_pieces(n_items, nkc, G):
    """The decode experts' stream-K split, restated from decode_mx_kernel
    (csrc/decode.cu): CTA c takes stages [n_st c / G, n_st (c + 1) / G) of the
    items' stages laid out item after item and works through its pieces from
    the top down; a piece holding an item's last stage owns it and adds the
    partial sums of CTAs [c_first, c) with non-empty ranges."""
    n_st = n_items * nkc
    rl = lambda c: n_st * c // G
    pieces = {}
    for c in range(G):
        lo, hi = rl(c), rl(c + 1)
        top = (hi - 1) // nkc if hi > lo else 0
        n_pc = top - lo // nkc + 1 if hi > lo else 0
        out = []
        for pc in range(n_pc):
            item = top - pc
            s0 = item * nkc
            kc0 = lo - s0 if lo > s0 else 0
            kc1 = hi - s0 if hi - s0 < nkc else nkc
            owner = kc1 == nkc
            c_first = ((item * nkc + 1) * G - 1) // n_st if owner and kc0 > 0 else c
            contrib = [c2 for c2 in range(c_first, c) if n_st >= G or rl(c2) < rl(c2 + 1)]
            out.append((item, kc0, kc1, owner, contrib))
        pieces[c] = out
    return pieces


@pytest.mark.parametrize("n_items", [1, 2, 5, 17, 90, 92, 180, 500])
@pytest.mark.parametrize("nkc", [1, 2, 3, 11, 12])
@pytest.mark.parametrize("G", [1, 7, 148])
def test_stream_k_split_covers_every_stage_once(n_items, nkc, G):
    """Every (item, stage) belongs to exactly one piece; only a CTA's first
    piece can be a head piece (not the owner); an owner's contributors are
    exactly the other CTAs holding stages of its item, all below it and each
    holding that item as its single head piece -- the facts the kernel's
    partial-sum flags (one per CTA, waited on only by higher CTAs) rely on."""
    pieces = _stream_k_pieces(n_items, nkc, G)
    cover, head = {}, {}
    for c, ps in pieces.items():
        for pc, (item, kc0, kc1, owner, _) in enumerate(ps):
            assert 0 <= kc0 < kc1 <= nkc
            for kc in range(kc0, kc1):
                assert (item, kc) not in cover
                cover[(item, kc)] = c
            if not owner:
                assert pc == 0
                head[c] = item
    assert len(cover) == n_items * nkc
    for c, ps in pieces.items():
        for item, kc0, kc1, owner, contrib in ps:
            if not owner:
                continue
            holders = sorted({cover[(item, kc)] for kc in range(nkc)} - {c})
            assert contrib == holders
            assert all(c2 < c and head[c2] == item for c2 in contrib)
