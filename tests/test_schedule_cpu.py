"""The split-last-wave schedule's arithmetic, restated from
fastdialoguesidon_b200/csrc/attn_kernel.cuh (TileSeq, piece_range,
build_items, finish_part's neighbour search) and csrc/fds_capi.cu
(plan_schedule), checked on the CPU for the invariants the kernel relies on,
and against the C library's own plan (fds_attn_schedule, no GPU needed when
grid_ctas is given):

* every (unit, KV tile) step belongs to exactly one CTA;
* the first (waves - 1) x G CTAs hold one whole unit each, in unit order;
* a piece is non-empty and touches at most kMaxItems units;
* a cut unit has at most kMaxParts parts, on contiguous pieces, and the
  neighbour search of finish_part finds exactly those pieces;
* pieces weigh about the same.
"""

import itertools
import math

import pytest

from fastdialoguesidon_b200 import _native as N

K_BLOCK = 128
ROWS_PER_CTA = 256
W2, W1 = 5, 3          # kWeightTwoTiles, kWeightOneTile
C0_MAX = 20            # kWeightUnitStart: the weight of starting a unit, capped at n * W2 / 6


def c0_of(n):
    return min(C0_MAX, n * W2 // 6)
MAX_ITEMS = 3          # kMaxItems
MAX_PARTS = 4          # kMaxParts
SLOT_BYTES = 256 * 68 * 4


def geometry(batch, heads, L):
    R = math.ceil(L / ROWS_PER_CTA)
    n = math.ceil(L / K_BLOCK)
    U = batch * heads * R
    w_last = W2 if (R - 1) * ROWS_PER_CTA + 128 < L else W1
    per_bh = (R - 1) * (c0_of(n) + n * W2) + c0_of(n) + n * w_last
    return R, n, U, w_last, per_bh


def unit_pos(u, R, n, per_bh):
    return (u // R) * per_bh + (u % R) * (c0_of(n) + n * W2)


def tile_at(x, R, n, w_last, per_bh):
    c0 = c0_of(n)
    full = (R - 1) * (c0 + n * W2)
    bh, rem = divmod(x, per_bh)
    if rem < full:
        r, q = divmod(rem, c0 + n * W2)
        w = W2
    else:
        r, q, w = R - 1, rem - full, w_last
    t = 0 if q < c0 else (q - c0) // w
    return (bh * R + r) * n + t


def ws_bytes(G):
    return 1024 * 8 * 4 + G * MAX_ITEMS * SLOT_BYTES   # fixed count region (kMaxPieces), then the slots


def plan(batch, heads, L, G, forced=True, has_ws=True, has_kv=False):
    R, n, U, w_last, per_bh = geometry(batch, heads, L)
    if not has_ws or has_kv or G <= 0 or G > 1024:
        return U, U, 0
    waves = -(-U // G)
    if not forced and U / (waves * G) >= 0.97:
        return U, U, 0
    whole = (waves - 1) * G
    total = unit_pos(U, R, n, per_bh)
    wt = total - unit_pos(whole, R, n, per_bh)
    w_min, w_max = wt // G, -(-wt // G)
    c0 = c0_of(n)
    if (w_min >= c0 + W2 and 3 * w_min >= c0 + n * W2 and w_max <= 2 * (c0 + n * w_last)
            and G * total < 2 ** 31):
        return whole + G, whole, G
    return U, U, 0


def piece_range(k, whole, P, batch, heads, L):
    R, n, U, w_last, per_bh = geometry(batch, heads, L)
    x0 = unit_pos(whole, R, n, per_bh)
    wt = unit_pos(U, R, n, per_bh) - x0
    first = tile_at(x0 + k * wt // P, R, n, w_last, per_bh)
    last = U * n if k + 1 == P else tile_at(x0 + (k + 1) * wt // P, R, n, w_last, per_bh)
    return first, last


def items_of_piece(k, whole, P, batch, heads, L):
    R, n, U, w_last, per_bh = geometry(batch, heads, L)
    first, last = piece_range(k, whole, P, batch, heads, L)
    out = []
    u = first // n
    while u * n < last and len(out) < MAX_ITEMS:
        tb = first - u * n if first > u * n else 0
        te = last - u * n if last - u * n < n else n
        out.append((u, tb, te))
        u += 1
    return out


def neighbour_parts(k, u, whole, P, batch, heads, L):
    """finish_part's search for the pieces touching unit u around piece k."""
    R, n, *_ = geometry(batch, heads, L)
    lo, hi = u * n, u * n + n
    kf = kl = k
    while kf > 0 and k - kf + 1 < MAX_PARTS and piece_range(kf - 1, whole, P, batch, heads, L)[1] > lo:
        kf -= 1
    while kl + 1 < P and kl - k + 1 < MAX_PARTS and piece_range(kl + 1, whole, P, batch, heads, L)[0] < hi:
        kl += 1
    return kf, kl


def check_plan(batch, heads, L, G):
    R, n, U, w_last, per_bh = geometry(batch, heads, L)
    grid, whole, P = plan(batch, heads, L, G)
    assert P > 0, "split expected"
    assert whole % G == 0 and grid == whole + P
    owner = {}
    for cta in range(whole):
        for t in range(n):
            owner[(cta, t)] = cta
    cover = {}
    weights = []
    for k in range(P):
        its = items_of_piece(k, whole, P, batch, heads, L)
        assert 0 < len(its) <= MAX_ITEMS
        w = 0
        for u, tb, te in its:
            assert whole <= u < U and 0 <= tb < te <= n
            for t in range(tb, te):
                assert (u, t) not in owner
                owner[(u, t)] = whole + k
            cover.setdefault(u, []).append(k)
            w += (te - tb) * (w_last if u % R == R - 1 else W2) + (c0_of(n) if tb == 0 else 0)
        weights.append(w)
    assert len(owner) == U * n
    for u, ks in cover.items():
        assert ks == list(range(ks[0], ks[-1] + 1)) and len(ks) <= MAX_PARTS
        if len(ks) > 1:
            for k in ks:
                assert neighbour_parts(k, u, whole, P, batch, heads, L) == (ks[0], ks[-1])
    assert max(weights) - min(weights) <= 2 * (W2 + c0_of(n))


CASES = [(1, 6000, 16, 148), (1, 6000, 16, 100), (1, 1000, 16, 5), (1, 1000, 16, 37), (1, 1000, 16, 64),
         (1, 1100, 8, 9), (1, 1000, 12, 7), (2, 600, 12, 20), (1, 1000, 4, 6), (4, 6000, 16, 148),
         (2, 3000, 16, 148), (1, 6016, 6, 60), (2, 2500, 4, 140), (1, 3333, 16, 148)]


@pytest.mark.parametrize("B,L,H,G", CASES)
def test_split_last_wave_invariants(B, L, H, G):
    check_plan(B, H, L, G)


def test_auto_choice_on_the_bench_shapes():
    """With one CTA per SM (148): the encoder layer (384 units, 2.59 waves) is
    split; the DiT layer (288 units, 97% of two waves) is not."""
    assert plan(1, 16, 6000, 148, forced=False)[2] == 148
    assert plan(1, 12, 6000, 148, forced=False)[2] == 0
    assert plan(1, 16, 6000, 148, forced=False, has_kv=True)[2] == 0
    assert plan(1, 16, 6000, 148, forced=False, has_ws=False)[2] == 0


@pytest.mark.parametrize("B,L,H", list(itertools.product([1, 2], [129, 1000, 2500, 6000], [1, 4, 16])))
def test_every_accepted_grid_keeps_the_invariants(B, L, H):
    for G in range(1, 149):
        if plan(B, H, L, G)[2]:
            check_plan(B, H, L, G)


@pytest.mark.parametrize("B,L,H,G", CASES + [(2, 333, 16, 7), (3, 129, 4, 11), (1, 100, 2, 3)])
def test_c_library_plan_matches(B, L, H, G):
    got = N.schedule(B, H, L, False, ws_bytes(G), G)
    assert got == plan(B, H, L, G), (got, plan(B, H, L, G))
    U = geometry(B, H, L)[2]
    assert N.schedule(B, H, L, False, 0, G) == (U, U, 0)
    assert N.schedule(B, H, L, True, ws_bytes(G), G)[2] == 0
    assert N.load().fds_attn_workspace_bytes(G) == ws_bytes(G)


# the forced splits of tests/test_balanced_gpu.py must be accepted shapes
GPU_SPLIT_CASES = [(1, 1000, 16, 5), (1, 1000, 16, 37), (1, 1000, 16, 64), (2, 333, 16, 13), (1, 1100, 8, 9),
                   (3, 129, 4, 7), (1, 1000, 16, 13), (1, 1000, 16, 17), (1, 1000, 12, 7), (2, 600, 12, 20),
                   (1, 1000, 4, 6)]


@pytest.mark.parametrize("B,L,H,G", GPU_SPLIT_CASES)
def test_gpu_test_shapes_split(B, L, H, G):
    check_plan(B, H, L, G)
