"""The tcgen05 bulk loop (csrc/pk_bulk.cu) against the CPU oracle.

The bulk loop runs the iterations of a fresh batch while at least
PK_OPT_BULK_MIN_LIVE utterances are live (two-dimensional tensor-memory GEMM tiles);
the persistent loop continues from its state. These tests force it for every
iteration (threshold 1) on small and full geometries, for TDT and EOU, q8_0 and
f16 weights, and check the hand-over to the persistent loop, with the parity bar of
the rest of the suite: tokens, steps and EOU boundaries identical to the oracle
except where teacher forcing shows a near-tie (top-2 margin < 1e-3), and logits and
LSTM state within 2e-3 step by step under teacher forcing (the trace runs on the bulk
loop too).
"""
import numpy as np
import pytest

import parity

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def built(pk):
    pk.build()
    return pk


def small_model(pk, kind, wtype):
    if kind == "tdt":
        return pk.synth.make_decoder("tdt", vocab_size=300, d_enc=128, pred_hidden=128, joint_hidden=128,
                                     n_layers=2, wtype=wtype, blank_bias=1.0, seed=5)
    return pk.synth.make_decoder("eou", vocab_size=300, d_enc=128, pred_hidden=128, joint_hidden=128,
                                 n_layers=1, wtype=wtype, blank_bias=1.0, seed=5, eou_id=297, eob_id=298)


def check_batch(dec, o, enc, offs, T, r, max_excused):
    ro = o.decode_batch(enc, offs, T)
    gb = r.get("bounds")
    ob = ro.get("bounds")
    excused = parity.compare_free_running(dec, o, enc, offs, T, r["tokens"], ro["tokens"],
                                          gpu_bounds=gb, oracle_bounds=ob)
    assert excused <= max_excused, f"{excused} utterances diverge at near-ties"
    same = [np.array_equal(a, b) for a, b in zip(r["tokens"], ro["tokens"])]
    assert all(r["steps"][b] == ro["steps"][b] for b in range(len(T)) if same[b])
    return excused


@pytest.mark.parametrize("kind", ["tdt", "eou"])
@pytest.mark.parametrize("wtype", ["q8_0", "f16"])
@pytest.mark.parametrize("screen", [0, 1])
def test_bulk_every_iteration_matches_oracle(built, orc, kind, wtype, screen):
    """Threshold 1: every iteration of the batch on the bulk loop (including the
    init step of every utterance, empty utterances and the last iteration), with the
    joint screened in every iteration (PK_OPT_BULK_SCREEN = 1) or never (0)."""
    pk = built
    m = small_model(pk, kind, wtype)
    dec = pk.Decoder(m, bulk_min_live=1)
    dec.set_option(pk.abi.PK_OPT_BULK_SCREEN, screen)
    T = pk.synth.lengths_uniform(40, 1, 60, seed=3)
    T[7] = 0
    enc, offs = pk.synth.encoder_batch(T, m.d_enc, seed=11)
    r = dec.decode_batch(enc, offs, T)
    assert r["bulk_iterations"] > 0 and r["bulk_iterations"] == r["loop_iterations"]
    check_batch(dec, orc.Oracle(m), enc, offs, T, r, max_excused=2)
    dec.close()


@pytest.mark.parametrize("which", ["tdt_0_6b", "eou_120m"])
def test_bulk_teacher_forced_full_geometry(built, orc, which):
    """Logits and LSTM state of the bulk loop, step by step against the oracle, on the
    benchmark geometries (TDT-0.6b q8_0: 8198 joint rows over 33 tiles; EOU-120m f16)."""
    pk = built
    m = getattr(pk.synth, which)(seed=1234)
    dec = pk.Decoder(m, bulk_min_live=1)
    o = orc.Oracle(m)
    T = np.array([90], np.int32)
    enc, _ = pk.synth.encoder_batch(T, m.d_enc, seed=21)
    st = parity.teacher_forced(dec, o, enc)
    assert st["steps"] > 0
    parity.assert_tf_ok(st, f"{which} bulk")
    dec.close()


def test_bulk_hands_over_to_persistent_loop(built, orc):
    """Threshold 24 on 48 utterances of TDT-0.6b: the bulk loop runs the first
    iterations, the persistent loop finishes the ragged tail from its state."""
    pk = built
    m = pk.synth.tdt_0_6b(seed=1234)
    dec = pk.Decoder(m, bulk_min_live=24)
    T = pk.synth.lengths_uniform(48, 20, 300, seed=9)
    enc, offs = pk.synth.encoder_batch(T, m.d_enc, seed=31)
    r = dec.decode_batch(enc, offs, T)
    assert 0 < r["bulk_iterations"] < r["loop_iterations"]
    check_batch(dec, orc.Oracle(m), enc, offs, T, r, max_excused=2)
    # the same batch on the persistent loop alone agrees except at near-ties
    dec0 = pk.Decoder(m, bulk_min_live=0)
    r0 = dec0.decode_batch(enc, offs, T)
    assert r0["bulk_iterations"] == 0
    diff = sum(not np.array_equal(a, b) for a, b in zip(r["tokens"], r0["tokens"]))
    assert diff <= 2
    dec.close()
    dec0.close()


def _tie_model(pk):
    """Small TDT model whose joint.out rows 40-43 are one row and rows 200 and 260
    another, each group's bias raised so that it often wins: exact ties among up to
    four tokens of one N tile (the screened joint recomputes that whole tile) and
    between two tiles (two top-1 candidates). argmax_f32 takes the first index."""
    m = small_model(pk, "tdt", "q8_0")
    p = m.prefix
    W = pk.synth.dequantize(m.tensors[f"{p}.joint.out.weight"]).copy()
    b = pk.synth.dequantize(m.tensors[f"{p}.joint.out.bias"]).reshape(-1).copy()
    for group in ([40, 41, 42, 43], [200, 260]):
        W[group] = W[group[0]]
        b[group] = 1.2
    m.tensors[f"{p}.joint.out.weight"] = pk.synth.encode_2d(W, "q8_0")
    m.tensors[f"{p}.joint.out.bias"] = pk.synth.encode_f32(b)
    return m


def test_screened_joint_exact_ties(built, orc):
    """Every iteration on the bulk loop with the screened joint: tied tokens resolve to
    the first index, as in the oracle (identical rows give identical f32 sums); four
    tied tokens in one N tile take the whole-tile recomputation."""
    pk = built
    m = _tie_model(pk)
    dec = pk.Decoder(m, bulk_min_live=1)
    dec.set_option(pk.abi.PK_OPT_BULK_SCREEN, 1)
    T = pk.synth.lengths_uniform(48, 5, 80, seed=13)
    enc, offs = pk.synth.encoder_batch(T, m.d_enc, seed=17)
    r = dec.decode_batch(enc, offs, T)
    assert r["bulk_iterations"] == r["loop_iterations"] > 0
    toks = np.concatenate(r["tokens"])
    assert np.count_nonzero(toks == 40) > 0 and np.count_nonzero(toks == 200) > 0
    assert not np.isin(toks, [41, 42, 43, 260]).any()
    check_batch(dec, orc.Oracle(m), enc, offs, T, r, max_excused=2)
    dec.close()


def test_screened_joint_matches_three_product_joint(built, orc):
    """TDT-0.6b geometry, every iteration on the bulk loop: the screened joint (one f16
    product, f32 recomputation of the candidates) and the three-product joint give the
    same tokens except at near-ties, and both match the oracle."""
    pk = built
    m = pk.synth.tdt_0_6b(seed=1234)
    T = pk.synth.lengths_uniform(160, 20, 240, seed=19)
    enc, offs = pk.synth.encoder_batch(T, m.d_enc, seed=23)
    o = orc.Oracle(m)
    outs = []
    for screen in (1, 0):                      # every iteration screened / none
        dec = pk.Decoder(m, bulk_min_live=1)
        dec.set_option(pk.abi.PK_OPT_BULK_SCREEN, screen)
        r = dec.decode_batch(enc, offs, T)
        assert r["bulk_iterations"] == r["loop_iterations"] > 0
        check_batch(dec, o, enc, offs, T, r, max_excused=3)
        outs.append(r)
        dec.close()
    diff = sum(not np.array_equal(a, b) for a, b in zip(outs[0]["tokens"], outs[1]["tokens"]))
    assert diff <= 3
