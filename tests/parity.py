"""Parity harness shared by the GPU tests and smoke().

Bar (north_star): emitted token/duration sequences identical to the CPU oracle
(which is bit-identical to the reference's own decoder build) except where the
sequences first part at a step whose oracle top-2 logit margin is below 1e-3
(counted and reported); logits and LSTM states within 2e-3 max-abs. Logits and
state are compared step by step in teacher-forced mode: the device replays the
oracle's decisions and reports its own logits, argmax and state at each step.
"""
import numpy as np

LOGIT_TOL = 2e-3
STATE_TOL = 2e-3
TIE_MARGIN = 1e-3


def oracle_trace(o, enc_utt, max_symbols=None):
    """The oracle's free-running decode of one utterance with every step traced."""
    T = int(enc_utt.shape[0])
    msym = o.model.max_symbols_per_step if max_symbols is None else max_symbols
    return o.decode_window(enc_utt, max_symbols=max_symbols, trace_steps=max(1, T * (msym + 1) + 8))


def teacher_forced(dec, o, enc_utt, max_symbols=None, trace=None):
    """Compare one utterance step by step (trace: its oracle_trace, if already made).
    Returns a dict of error statistics."""
    T = int(enc_utt.shape[0])
    r = trace if trace is not None else oracle_trace(o, enc_utt, max_symbols)
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


def emitted_steps(o, tokens):
    """Steps of an oracle trace whose decision appended a token to the output
    (TDT: any non-blank; EOU: not blank, <EOB>, <EOU> or a "<...>" piece)."""
    m = o.model
    tok = np.asarray(tokens)
    if o.is_tdt:
        return tok != m.blank_id
    special = m.special_mask()
    sp = np.zeros(len(tok), bool)
    inr = (tok >= 0) & (tok < len(special))
    sp[inr] = special[tok[inr]] != 0
    return (tok != m.blank_id) & (tok != m.eob_id) & (tok != m.eou_id) & ~sp


def divergence_at_near_tie(o, enc_utt, gpu_tokens, max_symbols=None, trace=None):
    """Where a free-running device decode first parts from the oracle's: the
    oracle steps from its last common emitted token to the next one (the whole
    trace when the token lists are equal). For TDT the window starts AT the step
    that emitted the last common token, whose duration choice may differ while
    its token agrees; for EOU it starts after it. Returns (near_tie_in_window,
    (first_step, last_step)): whether one of those steps has an oracle token or
    duration margin below 1e-3, i.e. the first differing decision is a near-tie."""
    r = trace if trace is not None else oracle_trace(o, enc_utt, max_symbols)
    S = r["steps"]
    em = np.nonzero(emitted_steps(o, r["token"][:S]))[0]
    ot, gt = r["tokens"], np.asarray(gpu_tokens)
    n = min(len(ot), len(gt))
    diff = np.nonzero(ot[:n] != gt[:n])[0]
    k = int(diff[0]) if len(diff) else n
    if k == len(ot) and k == len(gt):
        lo, hi = 0, S - 1
    else:
        lo = (int(em[k - 1]) + (0 if o.is_tdt else 1)) if k > 0 else 0
        hi = int(em[k]) if k < len(em) else S - 1
    near = r["margin_tok"][lo:hi + 1] < TIE_MARGIN
    if o.is_tdt:
        near = near | (r["margin_dur"][lo:hi + 1] < TIE_MARGIN)
    return bool(np.any(near)), (lo, hi)


def compare_free_running(dec, o, enc, offs, n_frames, gpu_tokens, oracle_tokens,
                         max_symbols=None, gpu_bounds=None, oracle_bounds=None, tf_decoders=None,
                         gpu_steps=None, oracle_steps=None):
    """Free-running sequences must be identical; an utterance that differs is
    accepted only when its first differing decision falls on an oracle near-tie
    (margin < 1e-3) and, teacher forced on each of the device's step loops
    (tf_decoders: the decoders to replay it on, default [dec]), its logits and
    state stay within tolerance with no argmax mismatch away from near-ties.
    Returns the number of such (excused) utterances."""
    excused = 0
    decs = tf_decoders if tf_decoders is not None else [dec]
    for b in range(len(n_frames)):
        same = np.array_equal(gpu_tokens[b], oracle_tokens[b])
        if same and gpu_bounds is not None:
            same = np.array_equal(gpu_bounds[b], oracle_bounds[b])
        if same and gpu_steps is not None:
            same = int(gpu_steps[b]) == int(oracle_steps[b])
        if same:
            continue
        e = enc[int(offs[b]):int(offs[b]) + int(n_frames[b])]
        tr = oracle_trace(o, e, max_symbols)
        near, win = divergence_at_near_tie(o, e, gpu_tokens[b], max_symbols, trace=tr)
        assert near, f"utterance {b}: first differing decision (oracle steps {win}) is not at a near-tie"
        for d in decs:
            st = teacher_forced(d, o, e, max_symbols, trace=tr)
            assert_tf_ok(st, f"utterance {b}")
        excused += 1
    return excused
