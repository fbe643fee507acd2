"""GPU parity tests: libparakeet_cuda (through its C ABI) against the CPU oracle
and the golden fixtures. Run on a B200 with `pytest -m gpu`."""
import os

import numpy as np
import pytest

import parity

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
CASES = ["tdt_small", "tdt_msym2", "eou_small"]
MATHS = ["tc", "f32"]


def split(flat, counts):
    out, pos = [], 0
    for c in counts:
        out.append(flat[pos:pos + c])
        pos += c
    return out


@pytest.fixture(scope="module")
def built(pk):
    pk.build()
    return pk


def load_case(pk, name):
    m = pk.synth.read_gguf(os.path.join(GOLDEN, f"{name}.gguf"))
    return m, dict(np.load(os.path.join(GOLDEN, f"{name}.npz")))


@pytest.mark.parametrize("name", CASES)
@pytest.mark.parametrize("math", MATHS)
def test_golden_batch(built, name, math):
    pk = built
    m, g = load_case(pk, name)
    dec = pk.Decoder(m, math=math)
    r = dec.decode_batch(g["enc"], g["offsets"], g["n_frames"], max_symbols=int(g["max_symbols"]))
    toks = split(g["tokens"], g["token_counts"])
    for b in range(len(g["n_frames"])):
        assert np.array_equal(r["tokens"][b], toks[b]), f"{name} utt {b}"
    assert np.array_equal(r["steps"], g["steps"])
    if m.model_type == "eou":
        bnds = split(g["bounds"], g["bound_counts"])
        for b in range(len(g["n_frames"])):
            assert np.array_equal(r["bounds"][b], bnds[b])


@pytest.mark.parametrize("name", CASES)
@pytest.mark.parametrize("math", MATHS)
def test_golden_stream_windows(built, name, math):
    pk = built
    m, g = load_case(pk, name)
    dec = pk.Decoder(m, math=math)
    s = dec.stream()
    e0 = g["enc"][:g["n_frames"][0]]
    wt = split(g["win_tokens"], g["win_token_counts"])
    wb = split(g["win_bounds"], g["win_bound_counts"])
    pos = 0
    for k, w in enumerate(g["windows"]):
        r = s.window(e0[pos:pos + w], max_symbols=int(g["max_symbols"]))
        pos += w
        assert np.array_equal(r["tokens"], wt[k]), f"{name} window {k}"
        assert r["steps"] == g["win_steps"][k]
        assert np.array_equal(r["bounds"], wb[k])


@pytest.mark.parametrize("math", MATHS)
def test_tdt_0_6b_teacher_forced(built, orc, math):
    """Config 1 geometry (TDT-0.6b-v3, q8_0, B=1, T=125): per-step logits and
    LSTM state within 2e-3, argmax identical except at margins < 1e-3."""
    pk = built
    m = pk.synth.tdt_0_6b(seed=1234)
    dec = pk.Decoder(m, math=math)
    o = orc.Oracle(m)
    enc, _ = pk.synth.encoder_batch([125], m.d_enc, seed=99)
    st = parity.teacher_forced(dec, o, enc)
    parity.assert_tf_ok(st, "0.6b")
    assert st["steps"] > 20
    r = dec.decode_batch(enc, [0], [125])
    parity.compare_free_running(dec, o, enc, [0], [125], r["tokens"], [st["oracle"]["tokens"]])


@pytest.mark.parametrize("math", MATHS)
def test_tdt_0_6b_ragged_batch(built, orc, math):
    pk = built
    m = pk.synth.tdt_0_6b(seed=7)
    dec = pk.Decoder(m, math=math)
    o = orc.Oracle(m)
    T = np.array([125, 60, 1, 0, 90, 33, 200, 7], np.int32)
    enc, offs = pk.synth.encoder_batch(T, m.d_enc, seed=5)
    r = dec.decode_batch(enc, offs, T)
    ro = o.decode_batch(enc, offs, T)
    parity.compare_free_running(dec, o, enc, offs, T, r["tokens"], ro["tokens"])
    same = [np.array_equal(a, b) for a, b in zip(r["tokens"], ro["tokens"])]
    assert np.array_equal(r["steps"][same], ro["steps"][same])
    assert r["steps"][3] == 0 and len(r["tokens"][3]) == 0


def test_tdt_0_6b_two_block_passes(built, orc):
    """40 live utterances: 32-utterance passes (two m16 blocks) in every phase, and a
    joint slice of 7 tiles per CTA that the GEMM covers in two calls on one staged tile."""
    pk = built
    m = pk.synth.tdt_0_6b(seed=17)
    dec = pk.Decoder(m, math="tc")
    o = orc.Oracle(m)
    T = pk.synth.lengths_uniform(40, 20, 70, seed=4)
    enc, offs = pk.synth.encoder_batch(T, m.d_enc, seed=6)
    r = dec.decode_batch(enc, offs, T)
    ro = o.decode_batch(enc, offs, T)
    parity.compare_free_running(dec, o, enc, offs, T, r["tokens"], ro["tokens"])


def test_joint_slice_in_several_calls(built, orc):
    """A 9000-piece vocabulary gives each CTA 61 joint rows (8 tiles): 32-utterance
    passes cover them in two GEMM calls on one staged tile."""
    pk = built
    m = pk.synth.make_decoder("tdt", vocab_size=9000, d_enc=128, pred_hidden=128, joint_hidden=128,
                              seed=23, blank_bias=1.0)
    dec = pk.Decoder(m, math="tc")
    o = orc.Oracle(m)
    T = pk.synth.lengths_uniform(40, 10, 40, seed=8)
    enc, offs = pk.synth.encoder_batch(T, m.d_enc, seed=12)
    r = dec.decode_batch(enc, offs, T)
    ro = o.decode_batch(enc, offs, T)
    parity.compare_free_running(dec, o, enc, offs, T, r["tokens"], ro["tokens"])


@pytest.mark.parametrize("wtype", ["f16", "q8_0"])
@pytest.mark.parametrize("math", MATHS)
def test_tdt_1_1b(built, orc, wtype, math):
    pk = built
    m = pk.synth.tdt_1_1b(seed=3, wtype=wtype)
    dec = pk.Decoder(m, math=math)
    o = orc.Oracle(m)
    T = pk.synth.lengths_uniform(12, 1, 90, seed=4)
    enc, offs = pk.synth.encoder_batch(T, m.d_enc, seed=6)
    r = dec.decode_batch(enc, offs, T)
    ro = o.decode_batch(enc, offs, T)
    parity.compare_free_running(dec, o, enc, offs, T, r["tokens"], ro["tokens"])
    st = parity.teacher_forced(dec, o, enc[:T[0]])
    parity.assert_tf_ok(st, "1.1b")


@pytest.mark.parametrize("math", MATHS)
def test_eou_120m_batch(built, orc, math):
    """Config 3 geometry: EOU f16, 1-layer LSTM, no duration head, T=50."""
    pk = built
    m = pk.synth.eou_120m(seed=5)
    dec = pk.Decoder(m, math=math)
    o = orc.Oracle(m)
    T = np.full(24, 50, np.int32)
    enc, offs = pk.synth.encoder_batch(T, m.d_enc, seed=8)
    r = dec.decode_batch(enc, offs, T)
    ro = o.decode_batch(enc, offs, T)
    parity.compare_free_running(dec, o, enc, offs, T, r["tokens"], ro["tokens"],
                                gpu_bounds=r["bounds"], oracle_bounds=ro["bounds"])
    st = parity.teacher_forced(dec, o, enc[:50])
    parity.assert_tf_ok(st, "eou")


def test_eou_leader_then_replicated_decisions(built, orc):
    """300 EOU utterances: the loop starts with more live utterances than a CTA keeps
    in shared memory (leader decisions), then switches to decisions every CTA makes
    itself as utterances finish; tokens and EOU boundaries must match the oracle."""
    pk = built
    m = pk.synth.make_decoder("eou", vocab_size=64, d_enc=64, pred_hidden=64, joint_hidden=64,
                              n_layers=1, wtype="f16", seed=29, blank_bias=0.5)
    dec = pk.Decoder(m, math="tc")
    o = orc.Oracle(m)
    T = pk.synth.lengths_uniform(300, 1, 60, seed=31)
    enc, offs = pk.synth.encoder_batch(T, m.d_enc, seed=33)
    r = dec.decode_batch(enc, offs, T)
    ro = o.decode_batch(enc, offs, T)
    parity.compare_free_running(dec, o, enc, offs, T, r["tokens"], ro["tokens"],
                                gpu_bounds=r["bounds"], oracle_bounds=ro["bounds"])
    assert sum(len(b) for b in ro["bounds"]) > 0      # the case does reach EOU


@pytest.mark.parametrize("math", MATHS)
def test_many_chunks_small_model(built, orc, math):
    """B=300 crosses several 32-utterance chunks and exercises live-list compaction."""
    pk = built
    m = pk.synth.make_decoder("tdt", vocab_size=200, d_enc=128, pred_hidden=128, joint_hidden=128,
                              seed=31, blank_bias=1.5)
    dec = pk.Decoder(m, math=math)
    o = orc.Oracle(m)
    T = pk.synth.lengths_uniform(300, 0, 60, seed=9)
    enc, offs = pk.synth.encoder_batch(T, m.d_enc, seed=10)
    r = dec.decode_batch(enc, offs, T)
    ro = o.decode_batch(enc, offs, T)
    parity.compare_free_running(dec, o, enc, offs, T, r["tokens"], ro["tokens"])
    r2 = dec.decode_batch(enc, offs, T)
    assert all(np.array_equal(a, b) for a, b in zip(r["tokens"], r2["tokens"]))  # determinism


@pytest.mark.parametrize("math", MATHS)
def test_stream_state_matches_oracle(built, orc, math):
    pk = built
    m, g = load_case(pk, "tdt_small")
    dec = pk.Decoder(m, math=math)
    o = orc.Oracle(m)
    s = dec.stream()
    ost = o.new_state()
    e0 = g["enc"][:g["n_frames"][0]]
    pos = 0
    for w in g["windows"]:
        s.window(e0[pos:pos + w])
        o.decode_window(e0[pos:pos + w], st=ost)
        pos += w
        gs = s.get_state()
        assert np.max(np.abs(gs["h"] - ost["h"])) <= parity.STATE_TOL
        assert np.max(np.abs(gs["c"] - ost["c"])) <= parity.STATE_TOL
        assert gs["carry_frames"] == ost["s"].carry_frames
        assert gs["symbols_this_step"] == ost["s"].symbols_this_step
    # export / import round trip into a fresh stream continues identically
    s2 = dec.stream()
    s2.set_state(s.get_state())
    e1 = g["enc"][g["offsets"][3]:g["offsets"][3] + g["n_frames"][3]]
    assert np.array_equal(s.window(e1)["tokens"], s2.window(e1)["tokens"])


def test_stream_reset_matches_init_state(built, orc):
    pk = built
    m, g = load_case(pk, "eou_small")
    dec = pk.Decoder(m)
    o = orc.Oracle(m)
    s = dec.stream()
    s.reset()
    ost = o.new_state()
    o.init_state(ost)
    gs = s.get_state()
    assert gs["initialized"] == 1 and gs["last_token"] == -1
    assert np.max(np.abs(gs["h"] - ost["h"])) <= parity.STATE_TOL
    assert np.max(np.abs(gs["pred"] - ost["pred"])) <= parity.STATE_TOL


def test_device_resident_input(built):
    import torch
    pk = built
    m, g = load_case(pk, "tdt_small")
    dec = pk.Decoder(m)
    ref = dec.decode_batch(g["enc"], g["offsets"], g["n_frames"])
    t = torch.from_numpy(g["enc"]).cuda()
    r = dec.decode_batch(t.data_ptr(), g["offsets"], g["n_frames"], enc_on_device=True)
    torch.cuda.synchronize()
    assert all(np.array_equal(a, b) for a, b in zip(ref["tokens"], r["tokens"]))


def test_device_input_encproj_paths(built, orc):
    """TDT-0.6b geometry runs the tensor-core enc-proj for host input and for a 16-byte
    aligned device pointer, and the CUDA-core enc-proj for a device pointer that is only
    4-byte aligned; all three must agree with the oracle."""
    import torch
    pk = built
    m = pk.synth.tdt_0_6b(seed=21)
    dec = pk.Decoder(m)
    o = orc.Oracle(m)
    T = np.array([70, 45, 96], np.int32)
    enc, offs = pk.synth.encoder_batch(T, m.d_enc, seed=8)
    ro = o.decode_batch(enc, offs, T)
    r_host = dec.decode_batch(enc, offs, T)
    t = torch.from_numpy(enc).cuda()
    r_al = dec.decode_batch(t.data_ptr(), offs, T, enc_on_device=True)
    t2 = torch.zeros(enc.size + 1, dtype=torch.float32, device="cuda")
    t2[1:] = t.reshape(-1)
    torch.cuda.synchronize()
    r_mis = dec.decode_batch(t2.data_ptr() + 4, offs, T, enc_on_device=True)
    torch.cuda.synchronize()
    for r in (r_host, r_al, r_mis):
        parity.compare_free_running(dec, o, enc, offs, T, r["tokens"], ro["tokens"])
    assert all(np.array_equal(a, b) for a, b in zip(r_host["tokens"], r_al["tokens"]))


def test_error_paths(built):
    pk = built
    m, g = load_case(pk, "tdt_small")
    dec = pk.Decoder(m)
    with pytest.raises(pk.PkError) as e:
        dec.decode_batch(g["enc"], g["offsets"], g["n_frames"], d_enc=m.d_enc + 1)
    assert e.value.status == pk.abi.PK_ERR_DMODEL
    # a caller buffer too small reports the size needed
    import ctypes as C
    b, keep = dec.make_batch(g["enc"], g["offsets"], g["n_frames"])
    toks = np.zeros(2, np.int32)
    offs = np.zeros(len(g["n_frames"]) + 1, np.int64)
    r = pk.abi.pk_result()
    r.tokens, r.tokens_cap, r.token_offsets = C.c_void_p(toks.ctypes.data), 2, C.c_void_p(offs.ctypes.data)
    assert dec.decode_batch_raw(b, r) == pk.abi.PK_ERR_CAPACITY
    assert r.tokens_needed == int(g["token_counts"].sum())
    # one CTA never reaches the barrier (a flag nothing sets): the bounded waits of
    # the others run out after 20 ms, the call returns PK_ERR_TIMEOUT and the
    # context stays usable
    dec.set_option(pk.abi.PK_OPT_TIMEOUT_US, 20_000)
    dec.set_option(pk.abi.PK_OPT_TEST_STALL, 1)
    with pytest.raises(pk.PkError) as e:
        dec.decode_batch(g["enc"], g["offsets"], g["n_frames"])
    assert e.value.status == pk.abi.PK_ERR_TIMEOUT
    dec.set_option(pk.abi.PK_OPT_TIMEOUT_US, 5_000_000)
    r2 = dec.decode_batch(g["enc"], g["offsets"], g["n_frames"])
    assert np.array_equal(np.concatenate(r2["tokens"]), g["tokens"])
