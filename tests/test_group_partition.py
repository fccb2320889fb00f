"""The two-pass launch's geometry (CPU only).

A restatement of ``group_plan`` (``pagedbatch_b200/csrc/pb_sample.cu``), of pass 1's task walk
(``group_max_kernel`` in ``pagedbatch_b200/csrc/pb_groups.cuh``: equal contiguous runs of 4-group
tasks per warp, each lane's (row, group) advanced by 4 groups per task) and of pass 2's key layout
(``cidx``: runs of 4 keys, the CTA's 256 threads side by side), checked for what the kernels rely
on: every group key of every row is written exactly once, inside the workspace; every 16-byte load
of pass 1 starts inside its row and the partial ones end at the row's end; pass 2 reads every key
of a row exactly once, with 16-byte loads inside the row's stride of keys; the no-alloc array holds
the group keys of the batches the header names.
"""

import numpy as np
import pytest

GM_GB = 128
GM_THREADS = 256
GM_WARPS = GM_THREADS // 32
GS_THREADS = 256
GS_NPT = 16
GS_MAXG = GS_THREADS * GS_NPT
NOALLOC = 32 << 20


def align256(n):
    return (n + 255) & ~255


def group_plan(n_rows, vocab, es):
    ge = GM_GB // es
    ngr = (vocab + ge - 1) // ge
    ngs = (ngr + 3) & ~3
    return dict(ngr=ngr, ngs=ngs, ntasks=(n_rows * ngr + 3) // 4, coarse=(ngr + GS_MAXG - 1) // GS_MAXG,
                bytes=align256(n_rows * ngs * 4))


def pass1_grid(ntasks, per_sm=4, sms=148):
    return max(1, min(per_sm * sms, (ntasks + GM_WARPS - 1) // GM_WARPS))


def walk_pass1(n_rows, vocab, es, grid):
    """Every (gmax index, first element, element count) pass 1's lanes write / read, in order."""
    g = group_plan(n_rows, vocab, es)
    ngr, ngs, ntasks = g["ngr"], g["ngs"], g["ntasks"]
    ge, epv = GM_GB // es, 16 // es
    W = grid * GM_WARPS
    writes, reads = [], []
    for w in range(W):
        t0, t1 = w * ntasks // W, (w + 1) * ntasks // W
        for sub in range(4):
            gid = 4 * t0 + sub
            row, j = divmod(gid, ngr)
            for _t in range(t0, t1):
                if row < n_rows:
                    writes.append(row * ngs + j)
                    for part in range(8):
                        e0 = j * ge + part * epv
                        if e0 < vocab:
                            reads.append((row, e0, min(epv, vocab - e0)))
                j += 4
                while j >= ngr:
                    j -= ngr
                    row += 1
    return g, writes, reads


CASES = [
    (3, 4099, 4),    # partial last vector, rows of 129 groups
    (5, 1, 4),       # one element per row: a group per row, tasks span rows
    (7, 17, 2),      # bf16 sub-group rows
    (4, 95, 4),      # 3 groups per row (fewer than a task)
    (2, 5000, 2),
    (9, 63, 2),
]


@pytest.mark.parametrize("n_rows,vocab,es", CASES)
@pytest.mark.parametrize("grid", [1, 3, None])
def test_pass1_writes_every_group_once(n_rows, vocab, es, grid):
    g = group_plan(n_rows, vocab, es)
    grid = pass1_grid(g["ntasks"]) if grid is None else grid
    g, writes, reads = walk_pass1(n_rows, vocab, es, grid)
    want = sorted(r * g["ngs"] + j for r in range(n_rows) for j in range(g["ngr"]))
    assert sorted(writes) == want, "each row's group keys written exactly once"
    assert max(writes) * 4 + 4 <= g["bytes"]
    seen = {}
    for row, e0, n in reads:
        assert 0 <= e0 and e0 + n <= vocab and n >= 1
        assert (e0 * es) % 16 == 0, "a full or partial vector starts on a 16-byte boundary of the row"
        seen.setdefault(row, []).append((e0, n))
    for row in range(n_rows):
        iv = sorted(seen[row])
        pos = 0
        for e0, n in iv:
            assert e0 == pos
            pos += n
        assert pos == vocab, "every element of every row is read exactly once"


def test_pass1_row_walk_matches_division():
    # the incremental (row, j) of a lane equals divmod(group, ngr) after any number of tasks
    for ngr in (1, 2, 3, 4, 5, 1002, 4008):
        for start in (0, 1, 7, 4 * 333 + 2):
            row, j = divmod(start, ngr)
            gid = start
            for _ in range(50):
                assert (row, j) == divmod(gid, ngr)
                gid += 4
                j += 4
                while j >= ngr:
                    j -= ngr
                    row += 1


def cidx(i, tid):
    return ((i >> 2) * GS_THREADS + tid) * 4 + (i & 3)


def test_pass2_key_layout_covers_each_row_once():
    idx = sorted(cidx(i, t) for t in range(GS_THREADS) for i in range(GS_NPT))
    assert idx == list(range(GS_MAXG))
    for vocab, es in ((128256, 4), (128256, 2), (49152, 2), (4099, 4), (1, 4)):
        g = group_plan(1, vocab, es)
        nc = (g["ngr"] + g["coarse"] - 1) // g["coarse"]
        assert nc <= GS_MAXG
        for t in range(GS_THREADS):
            for i in range(0, GS_NPT, 4):
                c = cidx(i, t)
                assert c % 4 == 0
                if g["coarse"] == 1 and c < g["ngr"]:
                    assert c + 4 <= g["ngs"], "a 16-byte load of keys stays inside the row's stride"


def test_workspace_sizes():
    assert group_plan(256, 128256, 4)["ngr"] == 4008
    assert group_plan(1 << 10, 128256, 2)["ngr"] == 2004
    assert group_plan(1, (1 << 20) + 5, 4)["coarse"] == 9
    # the no-alloc array holds the group keys of up to 2092 rows of 128256 fp32 logits, 4185 of bf16
    assert group_plan(2092, 128256, 4)["bytes"] <= NOALLOC < group_plan(2093, 128256, 4)["bytes"]
    assert group_plan(4185, 128256, 2)["bytes"] <= NOALLOC < group_plan(4186, 128256, 2)["bytes"]
