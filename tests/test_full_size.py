"""GPU parity at the full sizes of the benchmark configurations.

Each test decodes a whole batch with a configuration's geometry, weight type, batch
size and length distribution (random-init weights, seeded N(0,1) encoder outputs,
the same generators bench.py uses) and checks it two ways:

* against the CPU oracle on a sample of its utterances: the oracle decodes each
  utterance on its own, so a sample is an exact check of those utterances (a
  divergence is excused only where teacher forcing shows a near-tie, margin < 1e-3);
* through properties that do not depend on size: an utterance's tokens (and EOU
  boundaries) do not depend on the batch around it (the batch decoded in reverse
  order, and a shard of it decoded as its own batch, give the same sequences), and
  every utterance's step count stays within the loop's bound.
"""
import numpy as np
import pytest

import parity

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def built(pk):
    pk.build()
    return pk


def _oracle_sample(dec, o, enc, offs, T, r, idx):
    """The oracle on utterances idx of a decoded batch; returns the excused count."""
    idx = np.asarray(idx, np.int64)
    so, sT = np.ascontiguousarray(offs[idx]), np.ascontiguousarray(T[idx])
    ro = o.decode_batch(enc, so, sT)
    gb = ob = None
    if "bounds" in r:
        gb, ob = [r["bounds"][i] for i in idx], ro["bounds"]
    return parity.compare_free_running(dec, o, enc, so, sT, [r["tokens"][i] for i in idx], ro["tokens"],
                                       gpu_bounds=gb, oracle_bounds=ob)


def _same_sequences(a, b, ia, ib, what):
    for x, y in zip(ia, ib):
        assert np.array_equal(a["tokens"][x], b["tokens"][y]), f"{what}: utterance {x} tokens differ"
        assert a["steps"][x] == b["steps"][y], f"{what}: utterance {x} steps differ"
        if "bounds" in a:
            assert np.array_equal(a["bounds"][x], b["bounds"][y]), f"{what}: utterance {x} bounds differ"


def _batch_properties(dec, enc, offs, T, r, msym, shard):
    B = len(T)
    # step bound: at most max_symbols + 1 decode steps per frame
    assert np.all(r["steps"] <= T.astype(np.int64) * (msym + 1))
    assert np.all(r["steps"][T == 0] == 0)
    assert all(len(r["tokens"][b]) <= r["steps"][b] for b in range(B))
    # reverse order: every utterance lands in other passes, record blocks and lists
    rev = np.arange(B)[::-1]
    rr = dec.decode_batch(enc, np.ascontiguousarray(offs[rev]), np.ascontiguousarray(T[rev]))
    _same_sequences(r, rr, rev, np.arange(B), "reversed batch")
    # a shard as its own batch (what one rank of a multi-GPU run decodes)
    sh = np.arange(shard[0], shard[1])
    rs = dec.decode_batch(enc, np.ascontiguousarray(offs[sh]), np.ascontiguousarray(T[sh]))
    _same_sequences(r, rs, sh, np.arange(len(sh)), "shard")


def test_config1_full(built, orc):
    """TDT-0.6b q8_0, B = 1, T = 125: the whole utterance against the oracle, free
    running and teacher forced (logits and LSTM state per step)."""
    pk = built
    m = pk.synth.tdt_0_6b(seed=1234)
    dec = pk.Decoder(m, math="tc")
    o = orc.Oracle(m)
    T = np.full(1, 125, np.int32)
    enc, offs = pk.synth.encoder_batch(T, m.d_enc, seed=99)
    r = dec.decode_batch(enc, offs, T)
    assert r["total_steps"] > 0
    _oracle_sample(dec, o, enc, offs, T, r, [0])
    parity.assert_tf_ok(parity.teacher_forced(dec, o, enc), "config 1")


def test_config2_full(built, orc):
    """TDT-0.6b q8_0, B = 64, T ~ U[60, 1875]: the shortest utterances and one of
    median length against the oracle; reverse order and a 16-utterance shard."""
    pk = built
    m = pk.synth.tdt_0_6b(seed=1234)
    dec = pk.Decoder(m, math="tc")
    o = orc.Oracle(m)
    T = pk.synth.lengths_uniform(64, 60, 1875, seed=7)
    enc, offs = pk.synth.encoder_batch(T, m.d_enc, seed=99)
    r = dec.decode_batch(enc, offs, T)
    order = np.argsort(T, kind="stable")
    _oracle_sample(dec, o, enc, offs, T, r, list(order[:3]) + [int(order[32])])
    _batch_properties(dec, enc, offs, T, r, m.max_symbols_per_step, (24, 40))


def test_config3_full(built, orc):
    """EOU-120m f16, B = 256, T = 50: every utterance's tokens and EOU boundaries
    against the oracle (the loop starts in leader decisions, more live utterances
    than a CTA keeps in shared memory, and finishes in replicated ones)."""
    pk = built
    m = pk.synth.eou_120m(seed=1234)
    dec = pk.Decoder(m, math="tc")
    o = orc.Oracle(m)
    T = np.full(256, 50, np.int32)
    enc, offs = pk.synth.encoder_batch(T, m.d_enc, seed=99)
    r = dec.decode_batch(enc, offs, T)
    _oracle_sample(dec, o, enc, offs, T, r, np.arange(256))
    _batch_properties(dec, enc, offs, T, r, m.max_symbols_per_step, (100, 164))


@pytest.mark.parametrize("wtype", ["q8_0", "f16"])
def test_config4_full(built, orc, wtype):
    """TDT-1.1b, B = 1024, T = 750, q8_0 and f16 weights. The 1024 encoder outputs
    are 750-frame windows at distinct offsets into one seeded N(0,1) pool of 16,384
    frames (overlapping frame ranges are valid input), so the loop runs at the full
    batch and length while the host holds 64 MB instead of 3 GB."""
    pk = built
    m = pk.synth.tdt_1_1b(seed=1234, wtype=wtype)
    dec = pk.Decoder(m, math="tc")
    o = orc.Oracle(m)
    B, TT, pool = 1024, 750, 16384
    enc = np.random.default_rng(99).standard_normal((pool, m.d_enc), dtype=np.float32)
    offs = (np.arange(B, dtype=np.int64) * 613) % (pool - TT + 1)
    assert len(np.unique(offs)) == B
    T = np.full(B, TT, np.int32)
    r = dec.decode_batch(enc, offs, T)
    _oracle_sample(dec, o, enc, offs, T, r, [0, 511, 1023])
    _batch_properties(dec, enc, offs, T, r, m.max_symbols_per_step, (384, 512))


@pytest.mark.parametrize("blank_bias", [0.0, 2.0, 4.0])
def test_config5_full(built, orc, blank_bias):
    """TDT-0.6b q8_0, one GPU's 512 utterances of the 4096 batch, T log-normal
    (median 250, sigma 0.8, clipped to [25, 3750]), blank bias swept over {0, 2, 4}
    (few to many blanks): the three shortest utterances and one of median length
    against the oracle; reverse order and a 64-utterance shard."""
    pk = built
    m = pk.synth.tdt_0_6b(seed=1234, blank_bias=blank_bias)
    dec = pk.Decoder(m, math="tc")
    o = orc.Oracle(m)
    T = pk.synth.lengths_lognormal(512, 250.0, 0.8, 25, 3750, seed=7)
    enc, offs = pk.synth.encoder_batch(T, m.d_enc, seed=99)
    r = dec.decode_batch(enc, offs, T)
    order = np.argsort(T, kind="stable")
    _oracle_sample(dec, o, enc, offs, T, r, list(order[:3]) + [int(order[256])])
    _batch_properties(dec, enc, offs, T, r, m.max_symbols_per_step, (64, 128))
