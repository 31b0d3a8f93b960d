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


# ---- failures: a rank that raises, a rank that never joins ------------------
def test_phase_single_process():
    with replicas.Phase(None):
        pass
    with pytest.raises(replicas.ReplicaFailure) as e:
        with replicas.Phase(None):
            raise ValueError("planted")
    assert e.value.failed == {0: "ValueError: planted"}
    with pytest.raises(KeyboardInterrupt):  # not an Exception: passes through untouched
        with replicas.Phase(None):
            raise KeyboardInterrupt


def _failing_rank_main(rank, port, out_q, fail_rank, mode):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime
    import time
    dist.init_process_group("gloo", rank=rank, world_size=WORLD, timeout=datetime.timedelta(seconds=5))
    t0 = time.monotonic()
    try:
        with replicas.Phase(dist):  # set-up: fine on every rank
            pass
        if mode == "exit" and rank == fail_rank:
            os._exit(0)  # dies without reaching the next exchange
        with replicas.Phase(dist):
            if rank == fail_rank:
                raise ValueError(f"planted on rank {rank}")
        replicas.reduce_timings(dist, "cpu", [1.0], 1)
        out_q.put((rank, "finished", None, time.monotonic() - t0))
    except replicas.ReplicaFailure as e:
        out_q.put((rank, "ReplicaFailure", e.failed, time.monotonic() - t0))
    except Exception as e:  # the process group's error when a peer is gone
        out_q.put((rank, "error", type(e).__name__, time.monotonic() - t0))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def _run_failing(fail_rank, mode):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_failing_rank_main, args=(r, port, q, fail_rank, mode)) for r in range(WORLD)]
    for p in procs:
        p.start()
    n = WORLD if mode == "raise" else WORLD - 1
    res = sorted(q.get(timeout=120) for _ in range(n))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    return res


@pytest.mark.parametrize("fail_rank", [0, 1])
def test_failed_rank_is_reported_on_every_rank(fail_rank):
    """A rank whose phase raises still takes the phase's exchange: every rank
    then raises ReplicaFailure naming it, and no rank reaches the timing
    reduction (same collective steps on every rank)."""
    res = _run_failing(fail_rank, "raise")
    assert [r[0] for r in res] == [0, 1]
    for rank, kind, failed, _ in res:
        assert kind == "ReplicaFailure"
        assert failed == {fail_rank: f"ValueError: planted on rank {fail_rank}"}


def test_rank_that_never_joins_ends_the_others_exchange():
    """A rank that dies between phases: the survivor's exchange ends with an
    error (peer gone, or the 5 s process-group timeout) instead of waiting."""
    res = _run_failing(1, "exit")
    assert len(res) == 1
    rank, kind, _, elapsed = res[0]
    assert rank == 0 and kind == "error" and elapsed < 60
