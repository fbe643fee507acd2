"""CTC greedy decode and detokenize (the steps beside the token loop).

CPU tests pin the oracle restatements (oracle/oracle.cpp: orc_ctc_greedy_window
restating src/parakeet_ctc.cpp:1831-1865, orc_detokenize restating
src/sentencepiece_bpe.cpp:9-37) on hand-worked cases. GPU tests compare the
library's batched kernels with the oracle on seeded inputs: bit-exact tokens,
frames, carried argmax and text bytes.
"""
import ctypes as C

import numpy as np
import pytest

MARK = "▁"


@pytest.fixture(scope="module")
def built(pk):
    pk.build()
    return pk


def ref_ctc_window(logits, blank, prev):
    """Pure-Python `>` scan of ctc_greedy_decode_window (NaN-aware, no fast-math)."""
    toks, frs = [], []
    for t, row in enumerate(logits):
        best, score = 0, float(row[0])
        for i in range(1, len(row)):
            if float(row[i]) > score:
                score, best = float(row[i]), i
        if best != blank and best != prev:
            toks.append(best)
            frs.append(t)
        prev = best
    return toks, frs, prev


# ---- CPU: the oracle on known answers ------------------------------------------

def test_oracle_ctc_known_answer(orc):
    L = np.array([[0, 5, 1], [0, 1, 5], [9, 1, 1], [0, 0, 0], [1, 2, 3], [1, 2, 3], [0, 0, 0]], np.float32)
    toks, frs, prev = orc.ctc_greedy_window(L, blank_id=0)
    assert toks.tolist() == [1, 2, 2] and frs.tolist() == [0, 1, 4] and prev == 0
    # the previous window's last argmax suppresses a repeat at the window start
    toks, frs, prev = orc.ctc_greedy_window(L, blank_id=0, prev=1)
    assert toks.tolist() == [2, 2] and frs.tolist() == [1, 4]
    # ties go to the first index; an empty window keeps prev
    toks, _, prev = orc.ctc_greedy_window(np.zeros((0, 3), np.float32), blank_id=0, prev=7)
    assert len(toks) == 0 and prev == 7


def test_oracle_ctc_matches_python_scan(orc):
    rng = np.random.default_rng(3)
    L = rng.integers(-3, 4, size=(200, 17)).astype(np.float32)   # many ties
    for prev in (-1, 0, 5):
        toks, frs, pv = orc.ctc_greedy_window(L, blank_id=16, prev=prev)
        et, ef, ep = ref_ctc_window(L, 16, prev)
        assert toks.tolist() == et and frs.tolist() == ef and pv == ep


def _random_vocab(rng, n):
    alphabet = [b"a", b"b", b"c", b" ", MARK.encode(), "é".encode(), "中".encode(), b"\xe2\x96", b"\x81"]
    pieces = []
    for v in range(n):
        k = int(rng.integers(0, 6))
        pieces.append(b"".join(alphabet[int(i)] for i in rng.integers(0, len(alphabet), size=k)))
    return pieces


def test_oracle_detokenize_matches_reference_build(orc):
    """orc_detokenize against the reference's own detokenize, compiled from its sources
    into oracle/_ref (oracle/Makefile target `ref`)."""
    if orc.ref_detokenize(["a"], [0]) is None:
        pytest.skip("oracle/_ref/libref_detok.so not built (the reference tree is absent)")
    rng = np.random.default_rng(41)
    for trial in range(20):
        pieces = _random_vocab(rng, int(rng.integers(1, 300)))
        n = len(pieces)
        ids = {k: int(rng.integers(-1, n)) for k in ("blank_id", "bos_id", "eos_id", "pad_id")}
        toks = rng.integers(-3, n + 3, size=int(rng.integers(0, 500))).astype(np.int32)
        assert orc.detokenize(pieces, toks, **ids) == orc.ref_detokenize(pieces, toks, **ids), trial


def test_oracle_detokenize_known_answer(orc):
    P = ["<blk>", MARK + "hel", "lo", MARK + "wor", "ld", MARK, "x" + MARK + "y", "<s>"]
    out = orc.detokenize(P, [5, 5, 1, 2, 3, 4, 0, 7, 6, 99, -3], blank_id=0, bos_id=7)
    assert out == b"hello worldx y"
    assert orc.detokenize(P, [], blank_id=0) == b""
    assert orc.detokenize(P, [5, 5, 0], blank_id=0) == b""          # only spaces
    # a piece ending in the first two bytes of U+2581 keeps them as they are
    P2 = [b"a\xe2\x96", b"\x81b", MARK.encode() + b"c"]
    assert orc.detokenize(P2, [0, 1, 2]) == b"a\xe2\x96\x81b c"


# ---- GPU: the library against the oracle --------------------------------------

def _ctc_case(rng, B, V, max_T, ties=False):
    T = rng.integers(0, max_T + 1, size=B).astype(np.int32)
    T[0] = 0                                      # an empty utterance
    offs = np.zeros(B, np.int64)
    offs[1:] = np.cumsum(T[:-1])
    F = int(T.sum())
    if ties:
        L = rng.integers(-2, 3, size=(F, V)).astype(np.float32)
    else:
        L = rng.standard_normal((F, V)).astype(np.float32)
    return T, offs, L


@pytest.mark.gpu
@pytest.mark.parametrize("ties", [False, True])
def test_ctc_greedy_matches_oracle(built, orc, ties):
    pk = built
    rng = np.random.default_rng(11 + int(ties))
    B, V = 37, 1025
    blank = V - 1
    T, offs, L = _ctc_case(rng, B, V, 300, ties)
    if not ties:
        # make blank and repeats common, as in real CTC output
        L[:, blank] += 1.5
        L[1::3] = L[0::3][:len(L[1::3])]
    ctc = pk.CtcGreedy(V, blank)
    prev0 = rng.integers(-1, V, size=B).astype(np.int32)
    toks, frs, prev = ctc.decode(L, offs, T, prev=prev0, with_frames=True)
    for b in range(B):
        et, ef, ep = orc.ctc_greedy_window(L[offs[b]:offs[b] + T[b]], blank, int(prev0[b]))
        assert np.array_equal(toks[b], et) and np.array_equal(frs[b], ef), b
        assert prev[b] == ep, b
    ctc.close()


@pytest.mark.gpu
def test_ctc_greedy_windows_carry(built, orc):
    """Two windows per utterance with the carried argmax equal one whole window."""
    pk = built
    rng = np.random.default_rng(21)
    B, V = 9, 129
    T, offs, L = _ctc_case(rng, B, V, 80, ties=True)
    ctc = pk.CtcGreedy(V, 0)
    cut = (T // 2).astype(np.int32)
    t1, _, p1 = ctc.decode(L, offs, cut)
    t2, _, p2 = ctc.decode(L, offs + cut, T - cut, prev=p1)
    whole, _, pw = ctc.decode(L, offs, T)
    for b in range(B):
        assert np.array_equal(np.concatenate([t1[b], t2[b]]), whole[b])
    assert np.array_equal(p2, pw)


@pytest.mark.gpu
def test_ctc_greedy_special_values(built):
    """NaN, infinities and signed zeros follow the reference's `>` scan."""
    pk = built
    V = 70
    rows = []
    r = np.zeros(V, np.float32); r[0] = np.nan; r[5] = 3.0; rows.append(r)           # NaN first: index 0
    r = np.zeros(V, np.float32); r[3] = np.nan; r[9] = 2.0; rows.append(r)           # other NaN skipped
    r = np.full(V, -np.inf, np.float32); rows.append(r)                              # all -inf: index 0
    r = np.zeros(V, np.float32); r[0] = -0.0; r[40] = 0.0; rows.append(r)           # -0 == +0: first wins
    r = np.zeros(V, np.float32); r[66] = np.inf; r[67] = np.inf; rows.append(r)      # first +inf
    r = np.full(V, np.nan, np.float32); r[0] = 1.0; rows.append(r)                   # all NaN but index 0
    L = np.stack(rows)
    ctc = pk.CtcGreedy(V, V - 1)
    toks, frs, prev = ctc.decode(L, [0], [len(rows)], with_frames=True)
    et, ef, ep = ref_ctc_window(L, V - 1, -1)
    assert toks[0].tolist() == et and frs[0].tolist() == ef and prev[0] == ep


@pytest.mark.gpu
def test_ctc_greedy_device_input_and_capacity(built, orc):
    import torch
    pk = built
    rng = np.random.default_rng(5)
    B, V = 6, 257
    T, offs, L = _ctc_case(rng, B, V, 50)
    ctc = pk.CtcGreedy(V, 3)
    dl = torch.from_numpy(L).cuda()
    td, _, pd = ctc.decode(dl.data_ptr(), offs, T, on_device=True)
    th, _, ph = ctc.decode(L, offs, T)
    assert all(np.array_equal(a, b) for a, b in zip(td, th)) and np.array_equal(pd, ph)
    # a too-small output buffer reports the size needed and leaves prev alone
    n = np.ascontiguousarray(T, np.int32)
    fo = np.ascontiguousarray(offs, np.int64)
    prev = np.full(B, -1, np.int32)
    toks = np.zeros(1, np.int32)
    toff = np.zeros(B + 1, np.int64)
    need = C.c_int64(0)
    P = C.c_void_p
    rc = pk.lib().pk_ctc_greedy(ctc._h, P(L.ctypes.data), 0, P(fo.ctypes.data), P(n.ctypes.data), B,
                                P(prev.ctypes.data), P(toks.ctypes.data), 0, P(toff.ctypes.data), None,
                                C.byref(need))
    total = sum(len(t) for t in th)
    assert rc == 7 and need.value == total and (prev == -1).all()


def _vocab(rng, n):
    return _random_vocab(rng, n)


@pytest.mark.gpu
def test_detokenize_matches_oracle(built, orc):
    pk = built
    rng = np.random.default_rng(7)
    pieces = _vocab(rng, 500)
    specials = dict(blank_id=499, bos_id=1, eos_id=2, pad_id=-1)
    voc = pk.Vocab(pieces, **specials)
    B = 50
    lists = []
    for b in range(B):
        n = int(rng.integers(0, 400)) if b % 7 else 0
        t = rng.integers(-5, 520, size=n).astype(np.int32)      # includes invalid ids
        if b % 5 == 1 and n > 3:
            t[:3] = pieces.index(b" ") if b" " in pieces else t[:3]   # leading spaces
        lists.append(t)
    got = voc.detokenize(lists)
    for b in range(B):
        assert got[b] == orc.detokenize(pieces, lists[b], **specials), b
        ref = orc.ref_detokenize(pieces, lists[b], **specials)   # the reference's own build, when present
        assert ref is None or got[b] == ref, b
    voc.close()


@pytest.mark.gpu
def test_detokenize_edges(built, orc):
    pk = built
    P = ["<blk>", MARK + "hel", "lo", MARK + "wor", "ld", MARK, "x" + MARK + "y", "<s>"]
    voc = pk.Vocab(P, blank_id=0, bos_id=7)
    lists = [[5, 5, 1, 2, 3, 4, 0, 7, 6, 99, -3], [], [5, 5, 0], [0, 7], [1]]
    got = voc.detokenize(lists)
    assert got == [b"hello worldx y", b"", b"", b"", b"hel"]
    for b, t in enumerate(lists):
        assert got[b] == orc.detokenize(P, t, blank_id=0, bos_id=7)
