"""Parity harness shared by the GPU tests, smoke() and bench.py's parity line.

Bar (north_star): emitted token/duration sequences identical to the CPU oracle
except at steps where the oracle's top-2 logit margin is below 1e-3 (counted and
reported); logits and LSTM states within 2e-3 max-abs. Comparisons are made step
by step in teacher-forced mode: the device replays the oracle's decisions and
reports its own logits, argmax and state at each step.
"""
import numpy as np

LOGIT_TOL = 2e-3
STATE_TOL = 2e-3
TIE_MARGIN = 1e-3


def teacher_forced(dec, o, enc_utt, max_symbols=None):
    """Compare one utterance step by step. Returns a dict of error statistics."""
    T = int(enc_utt.shape[0])
    r = o.decode_window(enc_utt, max_symbols=max_symbols, trace_steps=max(1, T * 12 + 8))
    S = r["steps"]
    if S == 0:
        return {"steps": 0, "logit_err": 0.0, "h_err": 0.0, "c_err": 0.0, "near_ties": 0,
                "bad_mismatch": 0, "mismatch": 0, "oracle": r}
    g = dec.trace(enc_utt, [0], [T], max_steps=S, forced_token=[r["token"]],
                  forced_dur=[r["dur_idx"]], max_symbols=max_symbols)
    nl = r["logits"].shape[1]
    lg = g["logits"][0, :S, :nl]
    logit_err = float(np.max(np.abs(lg - r["logits"])))
    h_err = float(np.max(np.abs(g["h"][0, :S] - r["h"])))
    c_err = float(np.max(np.abs(g["c"][0, :S] - r["c"])))
    at = g["argmax_token"][0, :S]
    ad = g["argmax_dur_idx"][0, :S]
    tok_mis = at != r["token"]
    dur_mis = (ad != r["dur_idx"]) if o.is_tdt else np.zeros(S, bool)
    near = (r["margin_tok"] < TIE_MARGIN) | (o.is_tdt & (r["margin_dur"] < TIE_MARGIN))
    mis = tok_mis | dur_mis
    per_step = np.max(np.abs(lg - r["logits"]), axis=1)
    bad = np.nonzero(per_step > LOGIT_TOL)[0]
    detail = ""
    if len(bad):
        s0 = int(bad[0])
        detail = (f"first bad step {s0} of {S} ({len(bad)} bad): oracle frame {int(r['frame'][s0])}, "
                  f"oracle token {int(r['token'][s0])}, device argmax {int(at[s0])}, "
                  f"device row all-zero {bool(np.all(lg[s0] == 0))}, err {per_step[s0]:.3g}, "
                  f"bad steps {bad[:12].tolist()}, frames {[int(r['frame'][k]) for k in bad[:12]]}")
    return {"steps": S, "logit_err": logit_err, "h_err": h_err, "c_err": c_err,
            "near_ties": int(np.sum(near)), "mismatch": int(np.sum(mis)),
            "bad_mismatch": int(np.sum(mis & ~near)), "oracle": r, "detail": detail}


def assert_tf_ok(st, what=""):
    assert st["logit_err"] <= LOGIT_TOL, f"{what} logits max-abs {st['logit_err']:.3g}; {st.get('detail', '')}"
    assert st["h_err"] <= STATE_TOL, f"{what} h max-abs {st['h_err']:.3g}"
    assert st["c_err"] <= STATE_TOL, f"{what} c max-abs {st['c_err']:.3g}"
    assert st["bad_mismatch"] == 0, f"{what} {st['bad_mismatch']} argmax mismatches at margin >= 1e-3"


def compare_free_running(dec, o, enc, offs, n_frames, gpu_tokens, oracle_tokens,
                         max_symbols=None, gpu_bounds=None, oracle_bounds=None):
    """Free-running sequences must be identical; a divergence is accepted only when
    the teacher-forced replay of that utterance shows a near-tie (margin < 1e-3)
    where the device's argmax differs. Returns the number of excused utterances."""
    excused = 0
    for b in range(len(n_frames)):
        same = np.array_equal(gpu_tokens[b], oracle_tokens[b])
        if same and gpu_bounds is not None:
            same = np.array_equal(gpu_bounds[b], oracle_bounds[b])
        if same:
            continue
        e = enc[int(offs[b]):int(offs[b]) + int(n_frames[b])]
        st = teacher_forced(dec, o, e, max_symbols)
        assert_tf_ok(st, f"utterance {b}")
        assert st["mismatch"] > 0, f"utterance {b} differs with no argmax mismatch under forcing"
        excused += 1
    return excused
