"""world_size-2 gloo test of the multi-GPU host path: the partition (balanced or
LPT) computed on every rank, per-rank decode of a disjoint shard, gather of token
lists to rank 0.
The per-rank decode here is the CPU oracle (the sharding/gather logic is what is
tested); on GPUs bench.py runs the same logic with libparakeet_cuda."""
import os
import sys

import numpy as np
import pytest
import torch.multiprocessing as mp

HERE = os.path.dirname(os.path.abspath(__file__))


def _worker(rank, world, port, q, policy):
    import torch.distributed as dist
    sys.path.insert(0, HERE)
    from conftest import load_oracle, load_pkg
    pk = load_pkg()
    orc = load_oracle()
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        m = pk.synth.make_decoder("tdt", vocab_size=64, d_enc=32, pred_hidden=32, joint_hidden=32,
                                  n_layers=2, seed=21, blank_bias=1.5)
        T = pk.synth.lengths_uniform(9, 0, 30, seed=2)
        enc, offs = pk.synth.encoder_batch(T, 32, seed=4)
        idx = pk.multi.shard_indices(T, world, policy)[rank]
        sub = pk.multi.sub_batch(enc, offs, T, idx)
        o = orc.Oracle(m)
        r = o.decode_batch(*sub, n_threads=1)
        parts = [None] * world
        dist.all_gather_object(parts, {"idx": idx.tolist(), "tokens": [t.tolist() for t in r["tokens"]]})
        if rank == 0:
            got = pk.multi.gather_in_order(len(T), parts)
            ref = o.decode_batch(enc, offs, T, n_threads=1)["tokens"]
            ok = all(np.array_equal(a, b) for a, b in zip(got, ref))
            q.put(("ok" if ok else "mismatch", sorted(len(p["idx"]) for p in parts)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("policy", ["balanced", "lpt"])
def test_two_rank_shard_and_gather(policy):
    import socket
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q, policy)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    status, sizes = q.get(timeout=5)
    assert status == "ok"
    assert sum(sizes) == 9 and min(sizes) >= 1
