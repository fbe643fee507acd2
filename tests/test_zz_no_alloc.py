"""pk_decode_noalloc: the decode entry point that allocates no device memory.

It exists for callers that cannot call cudaMalloc while they decode: a process
running under a fixed device-memory budget whose allocator refuses new device
memory after start-up, or a latency-critical audio thread that cannot afford
cudaMalloc's implicit device synchronisation or its failure. Its scratch lives
in one fixed-size device array inside the library, shared by every call.

The tests check the entry point, through the C ABI, against the existing
pk_decode_batch on the same inputs -- token ids and step counts must be
identical (the same kernels do the same arithmetic) -- on two calls in a row,
so leftovers of a previous call in the shared array would show up; against the
CPU oracle directly; and that two calls made right after pk_create leave the
device's free memory unchanged. The file name makes pytest collect it after
every other test.
"""
import ctypes as C
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


@pytest.fixture(scope="module")
def built(pk):
    pk.build()
    f = pk.lib().pk_decode_noalloc
    f.argtypes = [C.c_void_p, C.c_void_p, C.c_int32, C.c_int32, C.c_int32, C.c_void_p, C.c_int32,
                  C.c_void_p, C.c_void_p]
    f.restype = C.c_int32
    return pk


def outputs(T, msym, cap=None):
    import torch
    cap = max(1, T * max(1, msym)) if cap is None else cap
    tok = torch.full((max(cap, 1),), -7, dtype=torch.int32, device="cuda")
    n = torch.full((1,), -1, dtype=torch.int32, device="cuda")
    st = torch.full((1,), -1, dtype=torch.int32, device="cuda")
    return cap, tok, n, st


def noalloc(pk, dec, enc_dev, T, msym, cap=None, d_enc=None, out=None):
    import torch
    cap, tok, n, st = outputs(T, msym, cap) if out is None else out
    # the buffers were filled on torch's stream; the library decodes on its own
    torch.cuda.synchronize()
    rc = pk.lib().pk_decode_noalloc(dec.h, C.c_void_p(enc_dev.data_ptr() if enc_dev is not None else 0),
                                    T, dec.info.d_enc if d_enc is None else d_enc, msym,
                                    C.c_void_p(tok.data_ptr()), cap, C.c_void_p(n.data_ptr()),
                                    C.c_void_p(st.data_ptr()))
    torch.cuda.synchronize()
    if rc != 0:
        return rc, None, None
    k = int(n.item())
    return rc, tok[:k].cpu().numpy(), int(st.item())


def check_model(pk, m, enc, offs, T, msym):
    import torch
    # the no-alloc entry point runs the CUDA-core f32 step loop: compare with the
    # same kernel variant of pk_decode_batch
    dec = pk.Decoder(m, math="f32")
    ref = dec.decode_batch(enc, offs, T, max_symbols=msym)
    # two calls in a row per utterance, longest first so a short call follows a long one
    for b in sorted(range(len(T)), key=lambda i: -int(T[i])):
        e = torch.from_numpy(np.ascontiguousarray(enc[int(offs[b]):int(offs[b]) + int(T[b])])).cuda()
        for _ in range(2):
            rc, toks, steps = noalloc(pk, dec, e, int(T[b]), msym)
            assert rc == 0, pk.last_error()
            assert np.array_equal(toks, ref["tokens"][b]), f"utterance {b}"
            assert steps == int(ref["steps"][b])
    dec.close()


@pytest.mark.parametrize("name", ["tdt_small", "eou_small"])
def test_noalloc_matches_decode_batch_golden(built, name):
    pk = built
    m = pk.synth.read_gguf(os.path.join(GOLDEN, f"{name}.gguf"))
    g = dict(np.load(os.path.join(GOLDEN, f"{name}.npz")))
    check_model(pk, m, g["enc"], g["offsets"], g["n_frames"], int(g["max_symbols"]))


def test_noalloc_matches_decode_batch_tdt_0_6b(built):
    pk = built
    m = pk.synth.tdt_0_6b(seed=1234)
    T = np.array([125, 300, 17], np.int32)
    enc, offs = pk.synth.encoder_batch(T, m.d_enc, seed=99)
    check_model(pk, m, enc, offs, T, m.max_symbols_per_step)


def test_noalloc_matches_oracle_and_allocates_nothing(built, orc):
    """Right after pk_create, two calls on one TDT-0.6b utterance leave the device's
    free memory unchanged (no allocation, not even a lazily loaded module) and give
    the CPU oracle's tokens and steps (the oracle is pinned to the reference build)."""
    import torch
    pk = built
    m = pk.synth.tdt_0_6b(seed=1234)
    T = np.array([160], np.int32)
    enc, offs = pk.synth.encoder_batch(T, m.d_enc, seed=5)
    e = torch.from_numpy(enc).cuda()
    out = outputs(int(T[0]), m.max_symbols_per_step)
    dec = pk.Decoder(m)                       # default math mode: noalloc still runs the f32 loop
    torch.cuda.synchronize()
    free0 = torch.cuda.mem_get_info()[0]
    got = [noalloc(pk, dec, e, int(T[0]), m.max_symbols_per_step, out=out) for _ in range(2)]
    torch.cuda.synchronize()
    free1 = torch.cuda.mem_get_info()[0]
    assert free1 == free0, f"device free memory changed by {free0 - free1} bytes"
    ro = orc.Oracle(m).decode_batch(enc, offs, T)
    for rc, toks, steps in got:
        assert rc == 0, pk.last_error()
        assert np.array_equal(toks, ro["tokens"][0]) and steps == int(ro["steps"][0])
    dec.close()


def test_noalloc_rejects_oversize(built):
    import torch
    pk = built
    m = pk.synth.read_gguf(os.path.join(GOLDEN, "tdt_small.gguf"))
    dec = pk.Decoder(m)
    T = 4097                                           # one frame above the stated maximum
    e = torch.zeros((T, m.d_enc), dtype=torch.float32, device="cuda")
    rc, _, _ = noalloc(pk, dec, e, T, 10)
    assert rc == pk.abi.PK_ERR_INVALID
    assert "4096" in pk.last_error()
    rc, _, _ = noalloc(pk, dec, e[:10], 10, 10, cap=5)  # token buffer below T * max_symbols
    assert rc == pk.abi.PK_ERR_CAPACITY
    rc, _, _ = noalloc(pk, dec, e[:10], 10, 10, d_enc=m.d_enc + 1)
    assert rc == pk.abi.PK_ERR_DMODEL
    dec.close()
