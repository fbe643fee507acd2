"""pk_prefetch_batch: host encoder outputs copied ahead on the context's copy
stream; the ticket it returns names the staged copy, and a decode whose batch
carries the ticket reads that copy. Every decode must return what a plain decode
of the same frames returns; misuse of a ticket fails loudly."""
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


def _differs(a, b):
    return any(not np.array_equal(x, y) for x, y in zip(a["tokens"], b["tokens"]))


def test_pipeline_matches_plain_decode(built, model):
    """t0 = prefetch(b0); for k: t[k+1] = prefetch(b[k+1]); decode(b[k], t[k])."""
    pk = built
    dec = pk.Decoder(model)
    bs = [_batch(pk, model, s) for s in (1, 2, 3, 4)]
    plain = [dec.decode_batch(*b) for b in bs]
    tickets = [dec.prefetch(*bs[0])]
    for k in range(len(bs)):
        if k + 1 < len(bs):
            tickets.append(dec.prefetch(*bs[k + 1]))
        _same(dec.decode_batch(*bs[k], ticket=tickets[k]), plain[k])
    assert len(set(tickets)) == len(tickets) and 0 not in tickets


def test_refilled_buffer_reads_the_staged_copy(built, model):
    """A server refills its (pageable) buffer with the next request right after the
    prefetch: the decode with the ticket still reads the frames as they were; a
    decode without a ticket reads the buffer as it is now."""
    pk = built
    dec = pk.Decoder(model)
    enc, offs, T = _batch(pk, model, 5)
    enc2 = np.ascontiguousarray(enc[::-1])
    want_old = dec.decode_batch(enc, offs, T)
    want_new = dec.decode_batch(enc2.copy(), offs, T)
    assert _differs(want_old, want_new)
    buf = enc.copy()
    t = dec.prefetch(buf, offs, T)
    buf[:] = enc2                       # pageable: the copy was made before prefetch returned
    _same(dec.decode_batch(buf, offs, T), want_new)          # no ticket: the buffer as it is
    _same(dec.decode_batch(buf, offs, T, ticket=t), want_old)


def test_ticket_is_used_once(built, model):
    pk = built
    dec = pk.Decoder(model)
    enc, offs, T = _batch(pk, model, 6)
    want = dec.decode_batch(enc, offs, T)
    t = dec.prefetch(enc, offs, T)
    _same(dec.decode_batch(enc, offs, T, ticket=t), want)
    with pytest.raises(pk.PkError) as e:
        dec.decode_batch(enc, offs, T, ticket=t)
    assert e.value.status == pk.abi.PK_ERR_INVALID and "not staged" in str(e.value)
    with pytest.raises(pk.PkError):
        dec.decode_batch(enc, offs, T, ticket=12345)             # never issued


def test_out_of_order_and_replaced_copies(built, model):
    """Staged copies are used in any order; a third prefetch replaces the oldest
    staged copy, whose ticket then fails; a ticket covering fewer frames than the
    batch reads fails; a failed decode leaves the other staged copy usable."""
    pk = built
    dec = pk.Decoder(model)
    A, Bb, Cc = (_batch(pk, model, s) for s in (7, 8, 9))
    want = [dec.decode_batch(*x) for x in (A, Bb, Cc)]
    ta, tb = dec.prefetch(*A), dec.prefetch(*Bb)
    _same(dec.decode_batch(*Bb, ticket=tb), want[1])
    _same(dec.decode_batch(*A, ticket=ta), want[0])
    ta, tb, tc = (dec.prefetch(*x) for x in (A, Bb, Cc))          # C replaces A
    with pytest.raises(pk.PkError):
        dec.decode_batch(*A, ticket=ta)
    _same(dec.decode_batch(*Cc, ticket=tc), want[2])
    _same(dec.decode_batch(*Bb, ticket=tb), want[1])
    enc, offs, T = A
    tshort = dec.prefetch(enc, offs[:2], T[:2])                   # fewer frames than the whole batch
    with pytest.raises(pk.PkError) as e:
        dec.decode_batch(*A, ticket=tshort)
    assert "frames" in str(e.value)
    _same(dec.decode_batch(enc, offs[:2], T[:2], ticket=tshort), {"tokens": want[0]["tokens"][:2],
                                                                   "steps": want[0]["steps"][:2]})


def test_calls_without_ticket_leave_staged_copies(built, model):
    """Device input, host input without a ticket and stream windows neither use nor
    drop a staged copy; a device batch with a ticket and a device prefetch are
    rejected."""
    import torch
    pk = built
    dec = pk.Decoder(model)
    A, Bb = _batch(pk, model, 10), _batch(pk, model, 11)
    want_a, want_b = dec.decode_batch(*A), dec.decode_batch(*Bb)
    ta = dec.prefetch(*A)
    ed = torch.from_numpy(Bb[0]).cuda()
    torch.cuda.synchronize()
    _same(dec.decode_batch(ed.data_ptr(), Bb[1], Bb[2], enc_on_device=True), want_b)
    _same(dec.decode_batch(*Bb), want_b)
    dec.stream().window(np.ascontiguousarray(Bb[0][:20]))
    with pytest.raises(pk.PkError):
        dec.decode_batch(ed.data_ptr(), Bb[1], Bb[2], enc_on_device=True, ticket=ta)
    _same(dec.decode_batch(*A, ticket=ta), want_a)
    b, _ = dec.make_batch(ed.data_ptr(), Bb[1], Bb[2], enc_on_device=True)
    rc, t = dec.prefetch_raw(b)
    assert rc == pk.abi.PK_ERR_INVALID and t == 0


def test_pinned_pipeline_overlaps_refill(built, model):
    """Pinned input (asynchronous copy): a two-buffer ring where each buffer is
    refilled once the second later prefetch has returned, as the header allows;
    every decode matches the plain decode of its request."""
    import torch
    pk = built
    dec = pk.Decoder(model)
    reqs = [_batch(pk, model, 20 + s, B=4) for s in range(6)]
    rows = max(int(max(o + t for o, t in zip(r[1], r[2]))) for r in reqs)
    ring = [torch.zeros((rows, model.d_enc), dtype=torch.float32).pin_memory() for _ in range(2)]
    plain = [dec.decode_batch(*r) for r in reqs]
    tickets = []
    for k, (enc, offs, T) in enumerate(reqs):
        buf = ring[k % 2].numpy()
        buf[:enc.shape[0]] = enc
        tickets.append(dec.prefetch(buf, offs, T))
        if k >= 1:
            _same(dec.decode_batch(ring[(k - 1) % 2].numpy(), reqs[k - 1][1], reqs[k - 1][2],
                                   ticket=tickets[k - 1]), plain[k - 1])
    _same(dec.decode_batch(ring[(len(reqs) - 1) % 2].numpy(), reqs[-1][1], reqs[-1][2],
                           ticket=tickets[-1]), plain[-1])
