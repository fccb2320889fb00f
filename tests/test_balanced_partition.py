"""The balanced streaming launch's cut of a batch into per-CTA shares (CPU only).

A restatement of ``f_seg`` (``pagedbatch_b200/csrc/pb_stream.cuh``) and of the host's grid and
workspace sizing (``balanced_grid`` / ``ws_need`` in ``pb_sample.cu``), checked for the properties
the kernel relies on: every body vector, head and tail element of every row is streamed by exactly
one segment; a row's pieces sit at CTAs ``gf..gl`` with record indices ``row + g`` that are distinct
and inside the workspace; only a CTA's segments 0 and 1 can be pieces; every 16-byte copy starts
inside its row.
"""

import itertools

import pytest

SEG_MIN = 2048
F_SREC = 256


def record_bytes(cap):
    return 16 + 8 * cap


def align256(n):
    return (n + 255) & ~255


def cta_of(P, N, G):
    return ((P + 1) * G - 1) // N


CTAS_PER_SM = 1  # F_CPS in pb_stream.cuh


def grid_for(n_rows, vocab, es, sms):
    epv = 16 // es
    N = n_rows * ((vocab + epv - 1) // epv)
    return max(1, min(CTAS_PER_SM * sms, N // SEG_MIN))


def ws_need(n_rows, grid):
    return align256(n_rows * 8) + (n_rows + grid) * record_bytes(F_SREC)


def row_geometry(base_bytes, vocab, es):
    """(head_n, nvec, tail_e0, tail_n) of a row starting at byte address base_bytes (f_row)."""
    epv = 16 // es
    head = ((16 - (base_bytes & 15)) & 15) // es
    head = min(head, vocab)
    nvec = (vocab - head) // epv
    tail_e0 = head + nvec * epv
    return head, nvec, tail_e0, vocab - tail_e0


def segments(g, G, n_rows, vocab, es, geo):
    epv = 16 // es
    U = (vocab + epv - 1) // epv
    N = n_rows * U
    A0, A1 = g * N // G, (g + 1) * N // G
    rf, rl = A0 // U, (A1 - 1) // U
    out = []
    for i in itertools.count():
        if i > rl - rf:
            break
        row = rl if i == 0 else rf + i - 1
        head, nvec, tail_e0, tail_n = geo[row]
        u0 = max(A0, row * U) - row * U
        u1 = min(A1, (row + 1) * U) - row * U
        gf, gl = cta_of(row * U, N, G), cta_of(row * U + U - 1, N, G)
        out.append(dict(i=i, row=row, v0=min(u0, nvec), v1=min(u1, nvec), h=head if u0 == 0 else 0,
                        t=tail_n if u1 == U else 0, nseg=gl - gf + 1, first_rec=row + gf, rec=row + g, g=g))
    return out


CASES = [
    (256, 128256, 4, 148, 513024),   # config 2
    (1024, 128256, 2, 148, 256512),  # config 3
    (256, 49152, 2, 148, 98304),     # config 1
    (8, 49152, 4, 148, 196608),      # config 0: fewer rows than CTAs
    (3, 4099, 4, 148, 16396 + 4),    # odd vocabulary, rows not 16-byte aligned
    (1, 2 ** 20, 2, 148, 2 ** 21),   # one long row over every CTA
    (5000, 1000, 4, 148, 4000),      # many short rows
    (7, 32768, 2, 132, 65536 + 6),   # another SM count, unaligned stride
]


@pytest.mark.parametrize("n_rows,vocab,es,sms,stride_bytes", CASES)
def test_segments_cover_every_element_once(n_rows, vocab, es, sms, stride_bytes):
    G = grid_for(n_rows, vocab, es, sms)
    epv = 16 // es
    U = (vocab + epv - 1) // epv
    assert n_rows * U // G >= 1 and (G == 1 or n_rows * U // G >= SEG_MIN)
    geo = [row_geometry(r * stride_bytes, vocab, es) for r in range(n_rows)]
    seen_vec = [[] for _ in range(n_rows)]
    heads = [0] * n_rows
    tails = [0] * n_rows
    recs = set()
    by_row = {}
    for g in range(G):
        segs = segments(g, G, n_rows, vocab, es, geo)
        assert segs, "every CTA has a share"
        for s in segs:
            r = s["row"]
            assert 0 <= s["v0"] <= s["v1"] <= geo[r][1]
            seen_vec[r].append((s["v0"], s["v1"]))
            heads[r] += s["h"]
            tails[r] += s["t"]
            if s["nseg"] > 1:
                assert s["i"] in (0, 1), "only a CTA's first two segments can be pieces"
                assert s["rec"] not in recs
                recs.add(s["rec"])
                assert s["first_rec"] <= s["rec"] < s["first_rec"] + s["nseg"]
                assert 0 <= s["rec"] < n_rows + G
                off = align256(n_rows * 8) + s["rec"] * record_bytes(F_SREC)
                assert off + record_bytes(F_SREC) <= ws_need(n_rows, G) and off % 16 == 0
            by_row.setdefault(r, []).append(s)
    for r in range(n_rows):
        head, nvec, _, tail_n = geo[r]
        iv = sorted(seen_vec[r])
        pos = 0
        for a, b in iv:
            assert a == pos or (a == b == min(a, nvec)), f"row {r}: gap or overlap at {a} (expected {pos})"
            pos = max(pos, b)
        assert pos == nvec
        assert heads[r] == head and tails[r] == tail_n
        segs = by_row[r]
        assert len(segs) == segs[0]["nseg"], "nseg counts exactly the CTAs that hold a piece of the row"
        assert sorted(s["g"] for s in segs) == list(range(segs[0]["first_rec"] - r, segs[0]["first_rec"] - r + len(segs)))


def test_workspace_fits_the_noalloc_array_for_config_2_and_3():
    cap = 32 << 20
    assert ws_need(256, CTAS_PER_SM * 148) <= cap
    assert ws_need(1024, CTAS_PER_SM * 148) <= cap
