"""CPU tests of the oracle (the CPU restatement of the reference decoder).

Checked here against (1) gguf-py's dequantization of the same q8_0/f16 bytes and
(2) golden vectors from an independent float64 numpy restatement
(tests/golden/make_golden.py). The pin against the reference's own decoder, built
unchanged from its sources, is tests/test_ref_pin.py. The reference's own test
fixtures need real GGUF models and NeMo dumps that are not available here.
"""
import os

import numpy as np
import pytest

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
CASES = ["tdt_small", "tdt_msym2", "eou_small"]


def load_case(pk, name):
    m = pk.synth.read_gguf(os.path.join(GOLDEN, f"{name}.gguf"))
    g = dict(np.load(os.path.join(GOLDEN, f"{name}.npz")))
    return m, g


def split(flat, counts):
    out, pos = [], 0
    for c in counts:
        out.append(flat[pos:pos + c])
        pos += c
    return out


def test_q8_0_known_answer(pk, orc):
    # One hand-built q8_0 block: d = 0.5 (binary16 0x3800), qs = -128..127 step 8.
    blk = np.zeros(34, np.uint8)
    blk[0:2] = np.frombuffer(np.float16(0.5).tobytes(), np.uint8)
    qs = np.arange(-128, 128, 8, dtype=np.int8)
    blk[2:] = qs.view(np.uint8)
    t = pk.synth.Tensor(blk, pk.synth.GGML_Q8_0, 32, 1)
    got = orc.dequantize(t).reshape(-1)
    assert np.array_equal(got, qs.astype(np.float32) * 0.5)
    assert np.array_equal(got, pk.synth.dequantize(t).reshape(-1))


@pytest.mark.parametrize("wtype", ["q8_0", "f16", "f32"])
def test_dequant_matches_gguf_py(pk, orc, wtype):
    rng = np.random.default_rng(3)
    a = rng.standard_normal((37, 96), dtype=np.float32) * 0.07
    t = pk.synth.encode_2d(a, wtype)
    assert np.array_equal(orc.dequantize(t), pk.synth.dequantize(t))


def test_f16_subnormal_and_special_values(pk, orc):
    vals = np.array([0.0, -0.0, 6.0e-8, -5.96e-8, 6.1e-5, 65504.0, -2.0, np.inf, -np.inf],
                    np.float16)
    t = pk.synth.Tensor(vals.view(np.uint8).copy(), pk.synth.GGML_F16, len(vals), 1)
    got = orc.dequantize(t).reshape(-1)
    assert np.array_equal(got.view(np.uint32), vals.astype(np.float32).view(np.uint32))


@pytest.mark.parametrize("name", CASES)
def test_oracle_matches_golden(pk, orc, name):
    m, g = load_case(pk, name)
    o = orc.Oracle(m)
    toks = split(g["tokens"], g["token_counts"])
    bnds = split(g["bounds"], g["bound_counts"])
    msym = int(g["max_symbols"])
    for b, T in enumerate(g["n_frames"]):
        e = g["enc"][g["offsets"][b]:g["offsets"][b] + T]
        r = o.decode_window(e, max_symbols=msym)
        assert r["rc"] == 0
        assert np.array_equal(r["tokens"], toks[b]), f"{name} utt {b}"
        assert r["steps"] == g["steps"][b]
        if m.model_type == "eou":
            assert np.array_equal(r["bounds"], bnds[b])


@pytest.mark.parametrize("name", CASES)
def test_oracle_windows_match_golden(pk, orc, name):
    """Mode-2 streaming: one state carried across windows (carry_frames, EOU resets)."""
    m, g = load_case(pk, name)
    o = orc.Oracle(m)
    st = o.new_state()
    e0 = g["enc"][:g["n_frames"][0]]
    wt = split(g["win_tokens"], g["win_token_counts"])
    wb = split(g["win_bounds"], g["win_bound_counts"])
    pos, ntok = 0, 0
    for k, w in enumerate(g["windows"]):
        r = o.decode_window(e0[pos:pos + w], st=st, max_symbols=int(g["max_symbols"]),
                            n_tokens_before=ntok)
        pos += w
        ntok += len(r["tokens"])
        assert np.array_equal(r["tokens"], wt[k]), f"{name} window {k}"
        assert r["steps"] == g["win_steps"][k]
        assert np.array_equal(r["bounds"], wb[k])
    # windows concatenated give the single-window decode for TDT (carry_frames)
    if m.model_type == "tdt":
        full = split(g["tokens"], g["token_counts"])[0]
        assert np.array_equal(np.concatenate(wt), full)


def test_batch_threads_match_sequential(pk, orc):
    m, g = load_case(pk, "tdt_small")
    o = orc.Oracle(m)
    r = o.decode_batch(g["enc"], g["offsets"], g["n_frames"], n_threads=3,
                       max_symbols=int(g["max_symbols"]))
    toks = split(g["tokens"], g["token_counts"])
    for b in range(len(g["n_frames"])):
        assert np.array_equal(r["tokens"][b], toks[b])
    assert np.array_equal(r["steps"], g["steps"])


def test_eou_batch_bounds(pk, orc):
    m, g = load_case(pk, "eou_small")
    o = orc.Oracle(m)
    r = o.decode_batch(g["enc"], g["offsets"], g["n_frames"], n_threads=2)
    bnds = split(g["bounds"], g["bound_counts"])
    for b in range(len(g["n_frames"])):
        assert np.array_equal(r["bounds"][b], bnds[b])


def test_dmodel_mismatch_and_empty(pk, orc):
    m, g = load_case(pk, "tdt_small")
    o = orc.Oracle(m)
    e = g["enc"][:5]
    assert o.decode_window(e, d_enc=m.d_enc + 1)["rc"] == 1          # parakeet_tdt.cpp:874-878
    st = o.new_state()
    r = o.decode_window(np.zeros((0, m.d_enc), np.float32), st=st)   # n_frames <= 0: no init
    assert r["rc"] == 0 and r["steps"] == 0 and st["s"].initialized == 0


def test_trace_margins_and_state(pk, orc):
    m, g = load_case(pk, "tdt_small")
    o = orc.Oracle(m)
    e = g["enc"][:g["n_frames"][0]]
    r = o.decode_window(e, trace_steps=200)
    assert len(r["token"]) == r["steps"]
    lg = r["logits"]
    V1 = m.vocab_size + 1
    assert np.array_equal(np.argmax(lg[:, :V1], axis=1), r["token"])
    srt = np.sort(lg[:, :V1], axis=1)
    assert np.allclose(srt[:, -1] - srt[:, -2], r["margin_tok"])
    # the state after the last step equals the final decoder state
    assert np.array_equal(r["h"][-1], r["state"]["h"])
