"""CPU tests of the C-ABI library: it loads, exports every declared symbol, and
its host-only logic (sharding, capacity, error paths without a device) works.
No compute is called here."""
import ctypes as C
import os
import re

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "parakeet_cuda.h")


def declared_symbols():
    txt = open(HEADER).read()
    return sorted(set(re.findall(r"^PK_API[^;(]*?\b(pk_\w+)\s*\(", txt, flags=re.M)))


def test_header_and_binding_agree(pk):
    assert declared_symbols() == sorted(pk.abi.EXPORTED_SYMBOLS)


def test_library_exports_every_declared_symbol(pk):
    L = C.CDLL(pk.LIB_PATH)
    for name in declared_symbols():
        assert hasattr(L, name), name
    assert pk.lib().pk_abi_version() == 1


def test_struct_sizes_match_header(pk):
    # pk_tensor: ptr + 2 x i32 + 2 x i64 + u64 = 40 bytes on LP64
    assert C.sizeof(pk.abi.pk_tensor) == 40
    assert C.sizeof(pk.abi.pk_lstm_layer) == 160


def test_shard_lpt_balances(pk):
    T = pk.synth.lengths_lognormal(4096, seed=5)
    for world in (1, 2, 4, 8):
        owner = pk.shard_lpt(T, world)
        loads = np.bincount(owner, weights=T, minlength=world)
        assert owner.min() >= 0 and owner.max() < world
        assert loads.max() - loads.min() <= T.max()
        # deterministic
        assert np.array_equal(owner, pk.shard_lpt(T, world))


def test_shard_lpt_matches_python_lpt(pk):
    T = np.array([5, 9, 9, 1, 0, 7, 3], np.int32)
    order = sorted(range(len(T)), key=lambda i: (-T[i], i))
    load = [0, 0, 0]
    exp = np.zeros(len(T), np.int32)
    for i in order:
        k = int(np.argmin(load))
        exp[i] = k
        load[k] += T[i]
    assert np.array_equal(pk.shard_lpt(T, 3), exp)


def _interp(x, y, v):
    """pk_shard_balanced's piecewise-linear interpolation, the same operations in the same order."""
    if v <= x[0]:
        return y[0]
    for i in range(1, len(x)):
        if v <= x[i]:
            return y[i - 1] + (y[i] - y[i - 1]) * (v - x[i - 1]) / (x[i] - x[i - 1])
    m = len(x)
    return y[m - 1] + (y[m - 1] - y[m - 2]) * (v - x[m - 1]) / (x[m - 1] - x[m - 2])


def _iteration_cost(n):
    """pk_shard_balanced's per-iteration cost model (microseconds vs live count)."""
    if n <= 0:
        return 0.0
    if n < 128:
        return _interp([1.0, 16.0, 32.0, 64.0, 127.0], [19.1, 21.7, 34.0, 43.6, 76.8], float(n))
    return _interp([128.0, 256.0, 1024.0, 4096.0], [70.9, 84.5, 141.0, 346.2], float(n))


_FRAME_COST = 0.0095   # enc-proj per frame in the model's units


def _modelled_time(T):
    """sum over loop iterations of the cost at that iteration's live count, steps = frames."""
    T = np.sort(np.asarray(T, np.int64))[::-1]
    if len(T) == 0 or T[0] <= 0:
        return 0.0
    cnt = np.bincount(T, minlength=int(T[0]) + 1)
    live = len(T) - np.cumsum(cnt)[:-1]
    return float(sum(_iteration_cost(int(n)) for n in live))


def _ffd_bisect(T, world):
    """The partition restated: first fit decreasing against a bound on every shard's
    modelled time, the bound bisected to the smallest that places every utterance."""
    order = sorted(range(len(T)), key=lambda i: (-int(T[i]), i))

    def place(M):
        tm, cnt, out = [0.0] * world, [0] * world, [0] * len(T)
        for i in order:
            t = float(max(int(T[i]), 0))
            for k in range(world):
                after = tm[k] + t * (_iteration_cost(cnt[k] + 1) - _iteration_cost(cnt[k])) + _FRAME_COST * t
                if after <= M:
                    tm[k], out[i] = after, k
                    cnt[k] += 1
                    break
            else:
                return None
        return out

    lo = float(max(int(T[order[0]]), 0)) * (_iteration_cost(1) + _FRAME_COST)
    hi = 0.0
    for r, i in enumerate(order):
        hi += float(max(int(T[i]), 0)) * (_iteration_cost(r + 1) - _iteration_cost(r) + _FRAME_COST)
    best = place(hi)
    it = 0
    while it < 64 and hi - lo > 1e-9 * hi:
        mid = 0.5 * (lo + hi)
        p = place(mid)
        if p is not None:
            hi, best = mid, p
        else:
            lo = mid
        it += 1
    return np.array(best, np.int32)


def test_shard_balanced_matches_python_restatement(pk):
    for T, world in ((np.array([5, 9, 9, 1, 0, 7, 3], np.int32), 3),
                     (pk.synth.lengths_lognormal(300, seed=3), 4),
                     (np.array([40, 40, 40], np.int32), 8)):
        assert np.array_equal(pk.shard_balanced(T, world), _ffd_bisect(T, world))


def test_shard_balanced_evens_modelled_time(pk):
    """On configuration 5's lengths the balanced partition's slowest shard is modelled
    well below LPT's, and the shard with the longest utterance holds fewer than an
    equal share; every utterance is placed once, deterministically."""
    T = pk.synth.lengths_lognormal(4096, 250.0, 0.8, 25, 3750, seed=7)
    for world in (2, 4, 8):
        bal, lpt = pk.shard_balanced(T, world), pk.shard_lpt(T, world)
        assert bal.min() >= 0 and bal.max() < world and len(bal) == len(T)
        assert np.array_equal(bal, pk.shard_balanced(T, world))
        t_bal = max(_modelled_time(T[bal == k]) for k in range(world))
        t_lpt = max(_modelled_time(T[lpt == k]) for k in range(world))
        assert t_bal < t_lpt
        assert np.sum(bal == bal[int(np.argmax(T))]) < len(T) // world
    assert np.array_equal(pk.shard_balanced(T, 1), np.zeros(len(T), np.int32))
    assert len(pk.shard_balanced(np.zeros(0, np.int32), 3)) == 0
    # as many equal utterances as shards: one each
    assert sorted(pk.shard_balanced(np.full(4, 100, np.int32), 4).tolist()) == [0, 1, 2, 3]


def test_tokens_capacity(pk):
    T = np.array([3, 0, 10], np.int32)
    f = pk.lib().pk_tokens_capacity
    assert f(T.ctypes.data, 3, 10) == 130
    assert f(T.ctypes.data, 3, 0) == 13


def test_invalid_arguments_report_status(pk):
    L = pk.lib()
    assert L.pk_shard_lpt(None, 3, 0, None) == pk.abi.PK_ERR_INVALID
    assert "sharding" in pk.last_error()
    assert L.pk_shard_balanced(None, 3, 0, None) == pk.abi.PK_ERR_INVALID
    assert L.pk_create(None, 0, None) == pk.abi.PK_ERR_INVALID
    assert L.pk_prefetch_batch(None, None, None) == pk.abi.PK_ERR_INVALID


def test_create_without_device_fails_cleanly(pk):
    import torch
    if torch.cuda.is_available():
        pytest.skip("a CUDA device is present")
    m = pk.synth.make_decoder("tdt", vocab_size=32, d_enc=32, pred_hidden=32, joint_hidden=32)
    with pytest.raises(pk.PkError) as e:
        pk.Decoder(m)
    assert e.value.status in (pk.abi.PK_ERR_NO_DEVICE, pk.abi.PK_ERR_CUDA)


def test_text_entry_points_check_arguments(pk):
    """pk_ctc_* / pk_vocab_* / pk_detokenize reject bad arguments before touching a device."""
    L = pk.lib()
    E = pk.abi
    h = C.c_void_p()
    assert L.pk_ctc_create(0, 0, 0, C.byref(h)) == E.PK_ERR_INVALID            # empty vocabulary
    assert L.pk_ctc_create(0, 10, 10, C.byref(h)) == E.PK_ERR_INVALID          # blank out of range
    assert L.pk_ctc_create(0, 10, 3, None) == E.PK_ERR_INVALID
    assert L.pk_ctc_greedy(None, None, 0, None, None, 1, None, None, 0, None, None, None) == E.PK_ERR_INVALID
    offs = np.array([0, 2, 1], np.int64)                                         # decreasing
    assert L.pk_vocab_create(0, None, offs.ctypes.data, 2, -1, -1, -1, -1, C.byref(h)) == E.PK_ERR_INVALID
    assert L.pk_detokenize(None, None, 0, None, 1, None, 0, None, None) == E.PK_ERR_INVALID
    L.pk_ctc_destroy(None)
    L.pk_vocab_destroy(None)


def test_text_create_without_device_fails_cleanly(pk):
    import torch
    if torch.cuda.is_available():
        pytest.skip("a CUDA device is present")
    with pytest.raises(pk.PkError) as e:
        pk.CtcGreedy(10, 3)
    assert e.value.status == pk.abi.PK_ERR_NO_DEVICE
    with pytest.raises(pk.PkError) as e:
        pk.Vocab(["a", "b"])
    assert e.value.status == pk.abi.PK_ERR_NO_DEVICE


def test_gguf_round_trip(pk, tmp_path):
    m = pk.synth.make_decoder("eou", vocab_size=40, d_enc=32, pred_hidden=32, joint_hidden=64,
                              n_layers=1, wtype="f16", eou_id=36, eob_id=37)
    p = str(tmp_path / "m.gguf")
    pk.synth.write_gguf(m, p)
    m2 = pk.synth.read_gguf(p)
    assert (m2.model_type, m2.vocab_size, m2.blank_id, m2.eou_id, m2.eob_id) == ("eou", 40, 40, 36, 37)
    assert m2.pieces == m.pieces
    for k, t in m.tensors.items():
        t2 = m2.tensors[k]
        assert (t.type, t.ne0, t.ne1) == (t2.type, t2.ne0, t2.ne1)
        assert np.array_equal(t.data, t2.data)
