"""The oracle pinned to the reference itself (CPU).

oracle/_ref/libref_decoder.so is src/parakeet_tdt.cpp and src/parakeet_eou.cpp
built unchanged against a host-only ggml stand-in (``make -C oracle ref``); it runs
the reference's CPU branch (tdt_decode_window :865-981, eou_decode_window
src/parakeet_eou.cpp:206-336). These tests check that the oracle restatement
(oracle/oracle.cpp), which every GPU parity test uses for logits, margins and
teacher forcing, gives the reference build's results:

* every golden fixture (tests/golden/*.npz): whole utterances and window by window,
  tokens, steps, EOU boundaries, and the carried decoder state (h, c, pred_out,
  symbols_this_step, carry_frames, last_token, segment_start_token) after each window;
* configuration 1 (TDT-0.6b q8_0, T = 125) and configuration 3 (EOU-120m f16,
  256 utterances) whole, and samples of configurations 2, 4 and 5 spread over the
  length quantiles (configuration 5 at blank bias +2 with its longest utterance,
  3750 frames), against the reference build's
  fixtures in tests/golden/full/ and, for a few utterances, against the build
  directly (final state within 1e-5).

Skipped when the reference build is absent (it is made where the reference tree is).
"""
import importlib.util
import os

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
GOLDEN = os.path.join(HERE, "golden")
FULL = os.path.join(GOLDEN, "full")
CASES = ["tdt_small", "tdt_msym2", "eou_small"]
STATE_TOL = 1e-5


@pytest.fixture(scope="module")
def ref(orc):
    if not orc.ref_decoder_available():
        pytest.skip("oracle/_ref/libref_decoder.so not built (make -C oracle ref with PARAKEET_REFERENCE_DIR)")
    return orc


@pytest.fixture(scope="module")
def full_cases(pk):
    spec = importlib.util.spec_from_file_location("make_full_golden", os.path.join(GOLDEN, "make_full_golden.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod, mod.cases(pk)


def _split(flat, counts):
    out, pos = [], 0
    for c in counts:
        out.append(flat[pos:pos + c])
        pos += c
    return out


def _same_state(o_st, r_st, where):
    """Oracle state dict (arrays + orc_state struct) against RefState.get()."""
    s = o_st["s"]
    assert s.initialized == r_st["initialized"], where
    if not s.initialized:
        return
    assert s.symbols_this_step == r_st["symbols_this_step"], where
    assert s.carry_frames == r_st["carry_frames"], where
    for k, rk in (("h", "h"), ("c", "c"), ("pred", "pred")):
        err = float(np.max(np.abs(o_st[k] - r_st[rk]))) if o_st[k].size else 0.0
        assert err <= STATE_TOL, f"{where}: {k} differs by {err}"


@pytest.mark.parametrize("name", CASES)
def test_reference_matches_golden_and_oracle(pk, ref, name):
    m = pk.synth.read_gguf(os.path.join(GOLDEN, f"{name}.gguf"))
    g = dict(np.load(os.path.join(GOLDEN, f"{name}.npz")))
    R, O = ref.Reference(m), ref.Oracle(m)
    msym = int(g["max_symbols"])
    toks = _split(g["tokens"], g["token_counts"])
    bnds = _split(g["bounds"], g["bound_counts"])
    for b, T in enumerate(g["n_frames"]):
        e = g["enc"][g["offsets"][b]:g["offsets"][b] + T]
        r = R.decode_window(e, max_symbols=msym)
        o = O.decode_window(e, max_symbols=msym)
        assert r["rc"] == 0 and o["rc"] == 0
        assert np.array_equal(r["tokens"], toks[b]), f"{name} utt {b}: reference vs golden"
        assert r["steps"] == g["steps"][b]
        assert np.array_equal(o["tokens"], r["tokens"]) and o["steps"] == r["steps"]
        if m.model_type == "eou":
            assert np.array_equal(r["bounds"], bnds[b]) and np.array_equal(o["bounds"], r["bounds"])
        _same_state(o["state"], r["state"].get(), f"{name} utt {b}")
    # mode-2 streaming: one state carried across windows
    rs, os_ = R.new_state(), O.new_state()
    e0 = g["enc"][:g["n_frames"][0]]
    wt = _split(g["win_tokens"], g["win_token_counts"])
    wb = _split(g["win_bounds"], g["win_bound_counts"])
    pos, before = 0, np.zeros(0, np.int32)
    for k, w in enumerate(g["windows"]):
        r = R.decode_window(e0[pos:pos + w], st=rs, max_symbols=msym, tokens_before=before)
        o = O.decode_window(e0[pos:pos + w], st=os_, max_symbols=msym, n_tokens_before=len(before))
        pos += w
        assert np.array_equal(r["tokens"], wt[k]), f"{name} window {k}: reference vs golden"
        assert r["steps"] == g["win_steps"][k]
        assert np.array_equal(r["bounds"], wb[k])
        assert np.array_equal(o["tokens"], r["tokens"]) and np.array_equal(o["bounds"], r["bounds"])
        rst = rs.get()
        _same_state(os_, rst, f"{name} window {k}")
        if m.model_type == "eou":
            assert os_["s"].last_token == rst["last_token"]
            assert os_["s"].segment_start_token == rst["segment_start_token"]
        before = np.concatenate([before, r["tokens"]]).astype(np.int32)


def test_config1_reference_state(pk, ref):
    """Configuration 1 (TDT-0.6b q8_0, B = 1, T = 125): same tokens and steps, and the
    decoder state after the utterance within 1e-5."""
    m = pk.synth.tdt_0_6b(seed=1234)
    enc, _ = pk.synth.encoder_batch(np.array([125], np.int32), 1024, seed=99)
    r = ref.Reference(m).decode_window(enc)
    o = ref.Oracle(m).decode_window(enc)
    assert r["rc"] == 0 and o["rc"] == 0
    assert np.array_equal(o["tokens"], r["tokens"]) and o["steps"] == r["steps"]
    assert len(r["tokens"]) > 0
    _same_state(o["state"], r["state"].get(), "config 1")


def _sample(T, n, longest):
    """n utterances spread over the length quantiles below the top 2 %, plus the
    longest when asked (the single longest costs more oracle time than the rest)."""
    order = np.argsort(T, kind="stable")
    top = int(0.98 * (len(T) - 1))
    pick = order[np.linspace(0, top, n).round().astype(int)]
    if longest:
        pick = np.concatenate([pick, [int(np.argmax(T))]])
    return np.unique(pick)


def _hash(mod, a):
    return mod.tok_hash(np.asarray(a, np.int32))


@pytest.mark.parametrize("name,n,longest", [("config3", None, False), ("config2", 16, False),
                                            ("config4_q8_0", 6, False), ("config5_bias2", 48, True),
                                            ("config5_bias0", 16, False), ("config5_bias4", 16, False)])
def test_oracle_matches_reference_fixtures(pk, ref, full_cases, name, n, longest):
    """The oracle on (a sample of) a whole BASELINE configuration against the reference
    build's per-utterance outputs (tests/golden/full/<name>.npz): token hashes, counts,
    steps and EOU boundaries identical."""
    mod, todo = full_cases
    mk_model, mk_input, _ = todo[name]
    fx = dict(np.load(os.path.join(FULL, f"{name}.npz")))
    m = mk_model()
    if name.startswith("config5"):
        # only the sampled utterances' frames (the whole batch is 5.7 GB)
        idx = _sample(mod.config5_lengths(pk.synth), n, longest)
        enc, offs_s, T_s = mk_input(idx)
    else:
        enc, offs, T = mk_input()
        idx = np.arange(len(T)) if n is None else _sample(T, n, longest)
        offs_s, T_s = offs[idx], T[idx]
    o = ref.Oracle(m)
    r = o.decode_batch(enc, offs_s, T_s)
    for k, u in enumerate(idx):
        assert len(r["tokens"][k]) == fx["n_tok"][u], f"{name} utt {u}: token count"
        assert r["steps"][k] == fx["steps"][u], f"{name} utt {u}: steps"
        assert _hash(mod, r["tokens"][k]) == fx["tok_hash"][u], f"{name} utt {u}: tokens"
        if "bnd_hash" in fx:
            assert _hash(mod, r["bounds"][k]) == fx["bnd_hash"][u], f"{name} utt {u}: boundaries"
    if "tokens" in fx:   # small configurations keep the ids themselves
        ids = _split(fx["tokens"], fx["n_tok"])
        for k, u in enumerate(idx):
            assert np.array_equal(r["tokens"][k], ids[u])
    # a few utterances directly against the build: final decoder state
    R = ref.Reference(m)
    for k in range(min(2, len(idx))):
        e = enc[offs_s[k]:offs_s[k] + T_s[k]]
        rr, oo = R.decode_window(e), o.decode_window(e)
        assert np.array_equal(rr["tokens"], oo["tokens"])
        _same_state(oo["state"], rr["state"].get(), f"{name} utt {idx[k]}")
