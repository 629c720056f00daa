"""Index arithmetic of the stream-K GEMM grid (hc_gemm_tc.cu, k_q4_gemm_tc
with SK), restated and checked by brute force on the host, no GPU.  CTA c of
G takes the (tile, 128-K stage) units [c U / G, (c + 1) U / G) of U = tiles x
nk; its run falls into one piece per tile it touches; the piece holding a
tile's first stage owns the tile, and the owner finds the last CTA holding
the rest of the tile as ceil((tile + 1) nk G / U) - 1.  Checked here: the
pieces cover every unit once; a piece that does not start its tile is the
first piece of its CTA (so one workspace slot per CTA suffices); the owner's
contributors are exactly the CTAs whose first piece lies in the tile; each
issuer (stages of one parity) knows whether it had a stage in a piece; and
with the launcher's rule (runs of at least one tile) every contributor piece
is shorter than its CTA's run, i.e. published before that run ends."""
import pytest


def runs(tiles, nk, G):
    U = tiles * nk
    return U, [(c * U // G, (c + 1) * U // G) for c in range(G)]


def pieces(b, e, nk):
    """(tile, first unit, end unit) of the pieces of the run [b, e)."""
    out = []
    for tp in range(b // nk, (e - 1) // nk + 1):
        out.append((tp, max(b, tp * nk), min(e, (tp + 1) * nk)))
    return out


SHAPES = [(tiles, nk, nsm) for tiles in (1, 2, 9, 32, 48, 112, 160, 224, 300, 501, 1002)
          for nk in (1, 2, 4, 8, 32, 112) for nsm in (148, 132)]


@pytest.mark.parametrize("tiles,nk,nsm", SHAPES)
def test_stream_k_partition(tiles, nk, nsm):
    U, rs = runs(tiles, nk, min(nsm, tiles * nk))
    G = len(rs)
    covered = [0] * U
    first_piece_tile = {}
    for c, (b, e) in enumerate(rs):
        assert e > b  # every CTA has work (G <= U)
        ps = pieces(b, e, nk)
        for k, (tp, us, ue) in enumerate(ps):
            for u in range(us, ue):
                covered[u] += 1
            owner = us == tp * nk
            if not owner:
                assert k == 0, "only a CTA's first piece can start inside a tile"
                first_piece_tile[c] = tp
            # issuer i (stages j = i mod 2 of the CTA's counter) had a stage
            j0, j1 = us - b, ue - b
            has = [(ue - us) >= 2 or (j0 & 1) == i for i in (0, 1)]
            brute = [any(j % 2 == i for j in range(j0, j1)) for i in (0, 1)]
            assert has == brute
    assert all(v == 1 for v in covered)
    # owners: the contributors cta + 1 .. last hold the rest of the tile, in K order
    for c, (b, e) in enumerate(rs):
        for tp, us, ue in pieces(b, e, nk):
            if us != tp * nk:
                continue
            last = ((tp + 1) * nk * G + U - 1) // U - 1
            x = (tp + 1) * nk - 1
            assert rs[last][0] <= x < rs[last][1]
            contributors = [cc for cc in range(c + 1, last + 1)]
            assert all(first_piece_tile.get(cc) == tp for cc in contributors)
            assert sorted(cc for cc, t in first_piece_tile.items() if t == tp) == contributors
            # the tile's units are exactly the owner's piece plus the contributors' first pieces
            got = (ue - us) + sum(min(rs[cc][1], (tp + 1) * nk) - rs[cc][0] for cc in contributors)
            assert got == nk
    # the launcher takes stream-K only for runs of at least one tile: then a
    # contributor's piece ends before its CTA's run does
    if U // G >= nk:
        for c, tp in first_piece_tile.items():
            b, e = rs[c]
            assert min(e, (tp + 1) * nk) - b < e - b
