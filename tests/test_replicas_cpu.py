"""Replica decode on two gloo ranks (CPU, no GPU): the ranks' disjoint slices
cover the batch, each rank's greedy streams equal the single-process run of the
same sequences, and the timing reduction takes the max over ranks and sums the
tokens -- the host logic bench.py runs around the CUDA library on N GPUs."""
import os
import socket

import numpy as np
import pytest

torch = pytest.importorskip("torch")
import torch.distributed as dist  # noqa: E402
import torch.multiprocessing as mp  # noqa: E402

from krikil_rs_b200 import replicas, synth  # noqa: E402

WORLD, SEQS_PER_RANK, PLEN, NEW = 2, 2, 5, 3


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, port, out_q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=WORLD, timeout=datetime.timedelta(seconds=60))
    try:
        import oracle as O
        prompts = replicas.shard(synth.decode_prompts(WORLD * SEQS_PER_RANK, PLEN, seed=1), WORLD, rank)
        model = O.OracleModel(synth.make_weights(0))
        streams = [O.generate_greedy(model, O.OracleState(64), p.tolist(), NEW, eos=None)[0] for p in prompts]
        times, tokens = replicas.reduce_timings(dist, "cpu", [10.0 + rank, 5.0 - rank], sum(map(len, streams)))
        gathered = [None] * WORLD
        dist.all_gather_object(gathered, [p.tolist() for p in prompts] + streams)
        out_q.put((rank, times, tokens, gathered))
    finally:
        dist.destroy_process_group()


def test_shard_splits_evenly_and_rejects_ragged():
    items = list(range(12))
    parts = [replicas.shard(items, 3, r) for r in range(3)]
    assert sum(parts, []) == items
    with pytest.raises(ValueError):
        replicas.shard(items, 5, 0)
    with pytest.raises(ValueError):
        replicas.shard(items, 2, 2)


def test_single_process_reduction_is_identity():
    assert replicas.reduce_timings(dist, "cpu", [1.5, 2.5], 7) == ([1.5, 2.5], 7)


def test_two_gloo_ranks_match_single_process():
    import oracle as O
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, port, q)) for r in range(WORLD)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in range(WORLD)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    res.sort()
    for rank, times, tokens, gathered in res:
        assert times == [11.0, 5.0]  # max over ranks of each entry
        assert tokens == WORLD * SEQS_PER_RANK * NEW
    gathered = res[0][3]
    all_prompts = synth.decode_prompts(WORLD * SEQS_PER_RANK, PLEN, seed=1)
    model = O.OracleModel(synth.make_weights(0))
    for r in range(WORLD):
        got_prompts, got_streams = gathered[r][:SEQS_PER_RANK], gathered[r][SEQS_PER_RANK:]
        for i in range(SEQS_PER_RANK):
            b = r * SEQS_PER_RANK + i
            assert got_prompts[i] == all_prompts[b].tolist()
            ref, _ = O.generate_greedy(model, O.OracleState(64), all_prompts[b].tolist(), NEW, eos=None)
            assert got_streams[i] == ref
    assert np.unique(np.concatenate([np.array(g[:SEQS_PER_RANK]) for g in gathered]), axis=0).shape[0] == 4
