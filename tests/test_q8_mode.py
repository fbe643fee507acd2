"""PK_MATH_Q8: the q8_0-activation mode (ggml's vec_dot_q8_0_q8_0 arithmetic).

Optional and never the default. The step loop's activations (LSTM inputs, the
pred-proj input and the joint hidden layer) are quantised to q8_0 blocks as ggml's
quantize_row_q8_0 does (per 32 values d = max|x| / 127, q = round(x / d), d kept as
binary16), and each block's product with the q8_0 weights is one int8 tensor-core
product scaled by both blocks' d -- the arithmetic of the reference's graph path
(ggml mul_mat on q8_0 weights, src/parakeet_tdt.cpp:193-321), against which the
reference's CPU path (the parity target, f32 activations) differs by the
quantisation error. So this mode is measured against the f32 oracle with its own,
looser bars, reported rather than held to the 2e-3 parity bar:
  * teacher forced on TDT-0.6b q8_0 (configuration 1): logit error well above the
    exact path's (the mode is really quantising) and below 0.1;
  * teacher forced on configuration-2-length utterances: few argmax mismatches;
    free running: token counts close to the oracle's;
  * models with f16 step-loop weights reject the mode.
"""
import numpy as np
import pytest

import parity

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def built(pk):
    pk.build()
    return pk


def test_q8_rejected_without_q8_0_weights(built):
    pk = built
    dec = pk.Decoder(pk.synth.eou_120m(seed=1234))          # f16 weights
    with pytest.raises(pk.PkError) as e:
        dec.set_option(pk.abi.PK_OPT_MATH, pk.abi.PK_MATH_Q8)
    assert e.value.status == pk.abi.PK_ERR_INVALID
    dec.close()


def test_q8_teacher_forced_error(built, orc):
    pk = built
    m = pk.synth.tdt_0_6b(seed=1234)
    o = orc.Oracle(m)
    enc, _ = pk.synth.encoder_batch(np.array([125], np.int32), m.d_enc, seed=99)
    tr = parity.oracle_trace(o, enc)
    res = {}
    for math in ("tc", "q8"):
        dec = pk.Decoder(m, math=math)
        res[math] = parity.teacher_forced(dec, o, enc, trace=tr)
        dec.close()
    q, t = res["q8"], res["tc"]
    print(f"\nq8_0 activations, configuration 1 teacher forced ({q['steps']} steps): logit max-abs "
          f"{q['logit_err']:.3g} (exact path {t['logit_err']:.3g}), h {q['h_err']:.3g}, c {q['c_err']:.3g}, "
          f"argmax mismatches {q['mismatch']} ({q['bad_mismatch']} at margins >= 1e-3)")
    assert t["logit_err"] <= parity.LOGIT_TOL
    assert q["logit_err"] > 10 * t["logit_err"]          # the activations are quantised
    assert q["logit_err"] < 0.1
    assert q["h_err"] < 0.05 and q["c_err"] < 0.1
    assert q["mismatch"] <= max(2, q["steps"] // 20)


def test_q8_mismatch_rate(built, orc):
    """Teacher forced on four configuration-2-length utterances: argmax mismatches
    against the f32 oracle stay rare (counted, with the near-ties among them);
    free running on the same batch, the per-utterance token counts stay close (a
    free-running utterance that departs once from the oracle differs from there on,
    so identical utterances are reported, not required)."""
    pk = built
    m = pk.synth.tdt_0_6b(seed=1234)
    o = orc.Oracle(m)
    T = pk.synth.lengths_uniform(4, 120, 300, seed=7)
    enc, offs = pk.synth.encoder_batch(T, m.d_enc, seed=99)
    dec = pk.Decoder(m, math="q8")
    steps = mis = near = bad = 0
    err = 0.0
    for b in range(len(T)):
        st = parity.teacher_forced(dec, o, enc[offs[b]:offs[b] + T[b]])
        steps += st["steps"]
        mis += st["mismatch"]
        bad += st["bad_mismatch"]
        err = max(err, st["logit_err"])
    r = dec.decode_batch(enc, offs, T)
    assert r["bulk_iterations"] == 0                       # persistent loop only
    ro = o.decode_batch(enc, offs, T)
    same = sum(np.array_equal(a, b) for a, b in zip(r["tokens"], ro["tokens"]))
    n_q8 = np.array([len(a) for a in r["tokens"]])
    n_or = np.array([len(a) for a in ro["tokens"]])
    print(f"\nq8_0 activations, {len(T)} utterances teacher forced: {steps} steps, {mis} argmax mismatches "
          f"({bad} at margins >= 1e-3), logit max-abs {err:.3g}; free running: {same} identical, "
          f"tokens {int(n_q8.sum())} vs {int(n_or.sum())}")
    assert mis <= max(3, steps // 25)
    assert err < 0.1
    assert np.all(np.abs(n_q8 - n_or) <= np.maximum(3, n_or // 5))
    dec.close()
