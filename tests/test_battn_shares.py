"""The batched attention's cost-weighted shares (BaShares, csrc/q3_battn.cuh)
restated on the CPU.

Chunk u of the flattened (b, h, chunk) list starts at unit
Cs(u) = K u + A (8 b + h + 1); CTA g of G takes the chunks whose start unit
lies in [g C / G, (g+1) C / G), C = K T + 8 B A, with A dropped to 0 unless
C / G >= K + A.  The kernel finds a share's first chunk with a search over the
(b, h) starts (battn_share_lo) and the CTA of a chunk directly
(battn_share_of); the cross-CTA merge relies on both agreeing, on the shares
being contiguous and on no share being empty (a CTA with nothing to publish
between two others of a (b, h) would leave its merge counter short).
"""
import pathlib
import random
import re

HDR = pathlib.Path(__file__).resolve().parents[1] / "qwen3-iree_b200" / "csrc" / "q3_battn.cuh"


def _constants():
    src = HDR.read_text()
    k = int(re.search(r"constexpr long long kBaChunkUnits = (\d+);", src).group(1))
    a = int(re.search(r"constexpr int kBaPieceUnits = (\d+);", src).group(1))
    # the kernel's division by kBaChunkUnits is a shift by 3
    assert ">> 3);  // / kBaChunkUnits" in src and k == 8
    return k, a


def shares(nch, grid, A, K):
    """(lo[0..G], share_of) as the kernel computes them."""
    B = len(nch)
    pre = [0]
    for n in nch:
        pre.append(pre[-1] + 8 * n)
    T = pre[-1]
    G = min(grid, T)
    A = max(A, 0)
    C = K * T + 8 * B * A
    if C // G < K + A:
        A, C = 0, K * T

    def unit(b, h):
        return K * (pre[b] + h * nch[b]) + A * (8 * b + h + 1)

    def lo(g):  # battn_share_lo
        if g <= 0:
            return 0
        if g >= G:
            return T
        if A == 0:
            return (g * T + G - 1) // G
        t = (g * C + G - 1) // G
        bs = [b for b in range(B) if unit(b, 0) <= t]
        if not bs:
            return 0
        b = bs[-1]
        h = [hh for hh in range(8) if unit(b, hh) <= t][-1]
        s0 = pre[b] + h * nch[b]
        return min(s0 + (t - unit(b, h) + K - 1) // K, s0 + nch[b])

    def share_of(u):  # battn_share_of
        b = max(bb for bb in range(B) if pre[bb] <= u)
        h = (u - pre[b]) // nch[b]
        return (K * u + A * (8 * b + h + 1)) * G // C

    return [lo(g) for g in range(G + 1)], share_of, A


def test_shares_are_contiguous_nonempty_and_consistent():
    K, A0 = _constants()
    rng = random.Random(11)
    weighted = 0
    for _ in range(300):
        B = rng.randint(1, 64)
        nch = [rng.randint(1, rng.choice([2, 8, 64, 130])) for _ in range(B)]
        grid = rng.choice([1, 7, 148, 296])
        A = rng.choice([0, A0, 2 * A0, 8])
        los, share_of, used = shares(nch, grid, A, K)
        weighted += used > 0
        assert los[0] == 0 and los[-1] == 8 * sum(nch)
        for g in range(len(los) - 1):
            assert los[g] < los[g + 1], "empty share"
            for u in range(los[g], los[g + 1]):
                assert share_of(u) == g
    assert weighted > 100


def test_pieces_even_out_the_cost():
    """With the piece cost, a share's chunks + A/K per piece varies less
    than with equal chunk counts (the B=32 configuration's shapes)."""
    K, A0 = _constants()
    rng = random.Random(32)
    nch = [rng.randint(128, 2048) // 32 + 1 for _ in range(32)]
    starts = []
    s = 0
    for n in nch:
        for _ in range(8):
            starts.append((s, s + n))
            s += n

    def cost_spread(A):
        los, _, _ = shares(nch, 296, A, K)
        costs = []
        for g in range(len(los) - 1):
            pieces = sum(1 for a, b in starts if a < los[g + 1] and b > los[g])
            costs.append((los[g + 1] - los[g]) + pieces * A0 / K)
        return max(costs) - min(costs)

    assert cost_spread(A0) < cost_spread(0)
