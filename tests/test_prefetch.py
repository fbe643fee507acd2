"""pk_prefetch_batch: host encoder outputs copied ahead on the context's copy
stream and used by the next decode call with the same input; any other host
input empties the queue. Every decode must return what a plain decode returns."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def built(pk):
    pk.build()
    return pk


@pytest.fixture(scope="module")
def model(built):
    return built.synth.make_decoder("tdt", vocab_size=128, d_enc=96, pred_hidden=64, joint_hidden=64,
                                    n_layers=2, wtype="q8_0", seed=41, blank_bias=0.5)


def _batch(pk, m, seed, B=6):
    T = pk.synth.lengths_uniform(B, 5, 60, seed=seed)
    enc, offs = pk.synth.encoder_batch(T, m.d_enc, seed=seed + 100)
    return enc, offs, T


def _same(a, b):
    assert len(a["tokens"]) == len(b["tokens"])
    for x, y in zip(a["tokens"], b["tokens"]):
        assert np.array_equal(x, y)
    assert np.array_equal(a["steps"], b["steps"])


def test_pipeline_matches_plain_decode(built, model):
    """prefetch(b0); for k: prefetch(b[k+1]); decode(b[k]) over distinct batches."""
    pk = built
    dec = pk.Decoder(model)
    bs = [_batch(pk, model, s) for s in (1, 2, 3, 4)]
    plain = [dec.decode_batch(*b) for b in bs]
    dec.prefetch(*bs[0])
    for k in range(len(bs)):
        if k + 1 < len(bs):
            dec.prefetch(*bs[k + 1])
        _same(dec.decode_batch(*bs[k]), plain[k])


def test_decode_uses_the_prefetched_copy(built, model):
    """Pageable input is copied before prefetch returns, so changing the host array
    afterwards shows which copy the decode used: the staged one (the contract says
    the array must not change; the test breaks it on purpose, on the host)."""
    pk = built
    dec = pk.Decoder(model)
    enc, offs, T = _batch(pk, model, 5)
    enc2 = np.ascontiguousarray(enc[::-1])
    want_old = dec.decode_batch(enc, offs, T)
    want_new = dec.decode_batch(enc2.copy(), offs, T)
    assert any(not np.array_equal(x, y) for x, y in zip(want_old["tokens"], want_new["tokens"]))
    buf = enc.copy()
    dec.prefetch(buf, offs, T)
    buf[:] = enc2                       # after the copy has been made
    _same(dec.decode_batch(buf, offs, T), want_old)
    # the queue is empty now: the next decode copies the array as it is
    _same(dec.decode_batch(buf, offs, T), want_new)


def test_same_array_queued_twice(built, model):
    pk = built
    dec = pk.Decoder(model)
    enc, offs, T = _batch(pk, model, 6)
    want = dec.decode_batch(enc, offs, T)
    dec.prefetch(enc, offs, T)
    dec.prefetch(enc, offs, T)
    _same(dec.decode_batch(enc, offs, T), want)
    _same(dec.decode_batch(enc, offs, T), want)


def test_out_of_order_and_replaced_copies(built, model):
    """A decode whose input is not the queue head drops the queue and copies its own
    input; a third prefetch replaces the oldest; a prefetch covering fewer frames
    than the decode needs is not used."""
    pk = built
    dec = pk.Decoder(model)
    A, Bb, Cc = (_batch(pk, model, s) for s in (7, 8, 9))
    want = [dec.decode_batch(*x) for x in (A, Bb, Cc)]
    dec.prefetch(*A)
    dec.prefetch(*Bb)
    _same(dec.decode_batch(*Bb), want[1])          # head is A: dropped, direct copy
    _same(dec.decode_batch(*A), want[0])
    for x in (A, Bb, Cc):
        dec.prefetch(*x)                            # C replaces A
    for x, w in zip((A, Bb, Cc), want):
        _same(dec.decode_batch(*x), w)
    enc, offs, T = A
    dec.prefetch(enc, offs[:2], T[:2])             # fewer frames than the whole batch
    _same(dec.decode_batch(*A), want[0])


def test_device_input_leaves_the_queue(built, model):
    import torch
    pk = built
    dec = pk.Decoder(model)
    A, Bb = _batch(pk, model, 10), _batch(pk, model, 11)
    want_a, want_b = dec.decode_batch(*A), dec.decode_batch(*Bb)
    dec.prefetch(*A)
    ed = torch.from_numpy(Bb[0]).cuda()
    torch.cuda.synchronize()
    _same(dec.decode_batch(ed.data_ptr(), Bb[1], Bb[2], enc_on_device=True), want_b)
    _same(dec.decode_batch(*A), want_a)
    b, _ = dec.make_batch(ed.data_ptr(), Bb[1], Bb[2], enc_on_device=True)
    assert dec.prefetch_raw(b) == pk.abi.PK_ERR_INVALID


def test_stream_window_uses_prefetch(built, model):
    pk = built
    dec = pk.Decoder(model)
    enc, _, T = _batch(pk, model, 12, B=1)
    s0 = dec.stream()
    want = s0.window(enc)
    assert not np.array_equal(dec.stream().window(np.ascontiguousarray(enc[::-1]))["tokens"], want["tokens"])
    s1 = dec.stream()
    buf = enc.copy()
    dec.prefetch(buf, np.zeros(1, np.int64), T)
    buf[:] = enc[::-1]                  # after the copy: the window must see the staged copy
    got = s1.window(buf)
    assert np.array_equal(got["tokens"], want["tokens"]) and got["steps"] == want["steps"]
