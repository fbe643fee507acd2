"""The C++17 drop-in decoder (parakeet.cpp_b200/shim/parakeet_decoder_cuda.cpp).

It keeps the reference's declarations of tdt_prepare_runtime / tdt_init_state /
tdt_decode_window / tdt_greedy_decode and the eou_* four (src/parakeet_tdt.h:185-205,
src/parakeet_eou.h:82-107) over libparakeet_cuda. tests/shim/libpk_shim_test.so is
that translation unit compiled against the reference's own headers, plus a small C
driver that calls it the way the Engine does (src/parakeet_engine.cpp:403-457: one
state carried across windows). These tests compare what it returns, window by window,
with the CPU oracle (which is pinned to the reference build) and the golden fixtures.
"""
import ctypes as C
import os

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLDEN = os.path.join(ROOT, "tests", "golden")
LIB = os.path.join(ROOT, "tests", "shim", "libpk_shim_test.so")
CASES = ["tdt_small", "tdt_msym2", "eou_small"]

needs_lib = pytest.mark.skipif(not os.path.exists(LIB), reason="tests/shim/libpk_shim_test.so not built "
                               "(make -C tests/shim with PARAKEET_REFERENCE_DIR set)")

_lib = None


def shim_lib(pk):
    global _lib
    if _lib is None:
        pk.lib()   # libparakeet_cuda.so first (the harness links it)
        L = C.CDLL(LIB)
        P, I32 = C.c_void_p, C.c_int32
        L.shim_open.restype = P
        L.shim_open.argtypes = [P, P]
        L.shim_close.argtypes = [P]
        L.shim_init_state.restype = I32
        L.shim_init_state.argtypes = [P]
        L.shim_window.restype = I32
        L.shim_window.argtypes = [P, P, I32, I32, I32, P, I32, P, P, P, I32, P]
        L.shim_state.argtypes = [P, P, P, P, P]
        L.shim_greedy.restype = I32
        L.shim_greedy.argtypes = [P, P, I32, I32, I32, P, I32, P, P, P, I32, P, P, I32, P]
        _lib = L
    return _lib


def _p(a):
    return C.c_void_p(a.ctypes.data)


class Shim:
    def __init__(self, pk, model):
        self.L = shim_lib(pk)
        self.desc = pk.abi.ModelDesc(model)
        rc = C.c_int32(-1)
        h = self.L.shim_open(self.desc.ref(), C.byref(rc))
        self.rc = rc.value
        self.h = C.c_void_p(h) if h else None
        self.m = model

    def close(self):
        if self.h:
            self.L.shim_close(self.h)
            self.h = None

    def window(self, enc, msym, d_enc=None, cap=100000):
        enc = np.ascontiguousarray(enc, np.float32)
        toks = np.zeros(cap, np.int32)
        bnd = np.zeros(max(1, len(enc)), np.int32)
        nt, st, nb = C.c_int32(0), C.c_int32(0), C.c_int32(0)
        rc = self.L.shim_window(self.h, _p(enc) if len(enc) else None, len(enc),
                                self.m.d_enc if d_enc is None else d_enc, msym, _p(toks), cap, C.byref(nt),
                                C.byref(st), _p(bnd), len(bnd), C.byref(nb))
        return rc, toks[:nt.value].copy(), st.value, bnd[:nb.value].copy()

    def state(self):
        Lh = (self.m.n_layers, self.m.pred_hidden)
        h, c = np.zeros(Lh, np.float32), np.zeros(Lh, np.float32)
        p, ints = np.zeros(self.m.pred_hidden, np.float32), np.zeros(5, np.int32)
        self.L.shim_state(self.h, _p(h), _p(c), _p(p), _p(ints))
        return h, c, p, ints

    def greedy(self, enc, msym):
        enc = np.ascontiguousarray(enc, np.float32)
        cap = max(1, len(enc) * msym)
        toks, bnd = np.zeros(cap, np.int32), np.zeros(max(1, len(enc)), np.int32)
        text = C.create_string_buffer(1 << 16)
        nt, st, nb, tl = C.c_int32(0), C.c_int32(0), C.c_int32(0), C.c_int32(0)
        rc = self.L.shim_greedy(self.h, _p(enc) if len(enc) else None, len(enc), self.m.d_enc, msym, _p(toks), cap,
                                C.byref(nt), C.byref(st), _p(bnd), len(bnd), C.byref(nb), text, 1 << 16, C.byref(tl))
        return rc, toks[:nt.value].copy(), st.value, bnd[:nb.value].copy(), text.raw[:tl.value]


def load_case(pk, name):
    m = pk.synth.read_gguf(os.path.join(GOLDEN, f"{name}.gguf"))
    return m, dict(np.load(os.path.join(GOLDEN, f"{name}.npz")))


def split(flat, counts):
    out, pos = [], 0
    for c in counts:
        out.append(flat[pos:pos + c])
        pos += c
    return out


@needs_lib
def test_harness_exports(pk):
    """CPU: the harness library (and through it libparakeet_cuda) loads and binds."""
    L = shim_lib(pk)
    for name in ("shim_open", "shim_close", "shim_init_state", "shim_window", "shim_state", "shim_greedy"):
        assert hasattr(L, name)


@needs_lib
@pytest.mark.gpu
@pytest.mark.parametrize("name", CASES)
def test_shim_windows_match_oracle(pk, orc, name):
    """Mode-2 streaming through the drop-in: one TdtDecodeState / EouDecodeState carried
    across the fixture's windows (carry_frames, symbols_this_step, EOU resets and
    boundaries in the running token count), as src/parakeet_engine.cpp:403-457 drives it.
    Tokens, steps and boundaries equal the golden windows; the carried state equals the
    oracle's within the tensor-core tolerance (2e-3)."""
    m, g = load_case(pk, name)
    sh = Shim(pk, m)
    assert sh.rc == 0 and sh.h
    o = orc.Oracle(m)
    ost = o.new_state()
    msym = int(g["max_symbols"])
    e0 = g["enc"][:g["n_frames"][0]]
    wt = split(g["win_tokens"], g["win_token_counts"])
    wb = split(g["win_bounds"], g["win_bound_counts"])
    assert sh.L.shim_init_state(sh.h) == 0
    pos, ntok = 0, 0
    running = []
    for k, w in enumerate(g["windows"]):
        rc, toks, steps, bnd = sh.window(e0[pos:pos + w], msym)
        ro = o.decode_window(e0[pos:pos + w], st=ost, max_symbols=msym, n_tokens_before=ntok)
        pos += w
        assert rc == 0
        new = toks[ntok:]
        ntok = len(toks)
        running.append(new)
        assert np.array_equal(new, wt[k]), f"{name} window {k}"
        if m.model_type == "tdt" and w <= 0:
            continue
        assert steps == g["win_steps"][k], f"{name} window {k} steps"
        assert np.array_equal(bnd, wb[k]), f"{name} window {k} boundaries"
        h, c, p, ints = sh.state()
        assert np.abs(h - ost["h"]).max() < 2e-3 and np.abs(c - ost["c"]).max() < 2e-3
        assert np.array_equal(p, h[-1])
        assert ints[0] == ost["s"].symbols_this_step and ints[1] == 1
        if m.model_type == "tdt":
            assert ints[2] == ost["s"].carry_frames
        else:
            assert ints[3] == ost["s"].last_token and ints[4] == ost["s"].segment_start_token
    sh.close()


@needs_lib
@pytest.mark.gpu
@pytest.mark.parametrize("name", CASES)
def test_shim_greedy_matches_golden(pk, orc, name):
    """tdt_greedy_decode / eou_greedy_decode through the drop-in: tokens, steps and
    boundaries equal the golden fixture; the text is the reference's detokenize of the
    tokens (joined by segment for EOU)."""
    m, g = load_case(pk, name)
    sh = Shim(pk, m)
    toks = split(g["tokens"], g["token_counts"])
    bnds = split(g["bounds"], g["bound_counts"])
    msym = int(g["max_symbols"])
    for b, T in enumerate(g["n_frames"]):
        e = g["enc"][g["offsets"][b]:g["offsets"][b] + T]
        rc, t, steps, bnd, text = sh.greedy(e, msym)
        assert rc == 0
        assert np.array_equal(t, toks[b]) and steps == g["steps"][b], f"{name} utterance {b}"
        if m.model_type == "eou":
            assert np.array_equal(bnd, bnds[b])
        else:
            pieces = ["<s%d>" % i if s else "p%d" % i for i, s in enumerate(m.special_mask())]
            assert text == orc.detokenize(pieces, t, blank_id=m.blank_id)
    sh.close()


@needs_lib
@pytest.mark.gpu
def test_shim_return_codes(pk):
    """The reference's return codes: 1 for an encoder width that differs from the
    model's (parakeet_tdt.cpp:874-878), 0 and no state change for an empty TDT window
    (:879), and eou_prepare_runtime's 1 for a model that is not EOU (parakeet_eou.cpp:173)."""
    m, g = load_case(pk, "tdt_small")
    sh = Shim(pk, m)
    assert sh.L.shim_init_state(sh.h) == 0
    rc, toks, steps, _ = sh.window(g["enc"][:5], 10, d_enc=m.d_enc + 1)
    assert rc == 1 and len(toks) == 0 and steps == 0
    rc, toks, steps, _ = sh.window(np.zeros((0, m.d_enc), np.float32), 10)
    assert rc == 0 and len(toks) == 0 and steps == 0
    sh.close()
