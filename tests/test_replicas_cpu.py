"""Multi-rank host logic of the replica path, on CPU ranks (gloo, world size 2).

The data path of N GPUs is N independent replicas (no collective); what the
ranks share is the host logic in gpt2b200.replicas: the sequence partition,
the max-over-ranks timing and the gather of token streams on rank 0.  Here
two spawned processes decode their sequences with the oracle (standing in for
one GPU each) and rank 0's gathered streams must equal a single-process run.
"""
import os
import socket

import numpy as np
import pytest

import oracle
from gpt2b200 import replicas, synth

torch = pytest.importorskip("torch")


def test_shard_strong_covers_every_sequence_once():
    for n in (0, 1, 5, 32, 33):
        for world in (1, 2, 3, 4, 8):
            got = [i for r in range(world) for i in replicas.shard(n, world, r)]
            assert got == list(range(n)), (n, world)
            sizes = [len(replicas.shard(n, world, r)) for r in range(world)]
            assert max(sizes) - min(sizes) <= 1


def test_shard_weak_gives_each_rank_its_own_block():
    blocks = [replicas.shard(32, 4, r, "weak") for r in range(4)]
    assert [len(b) for b in blocks] == [32] * 4
    assert sorted(i for b in blocks for i in b) == list(range(128))


def test_shard_rejects_bad_arguments():
    with pytest.raises(ValueError):
        replicas.shard(4, 2, 2)
    with pytest.raises(ValueError):
        replicas.shard(4, 0, 0)
    with pytest.raises(ValueError):
        replicas.shard(4, 2, 0, "diagonal")


def test_single_process_helpers_without_process_group():
    assert replicas.max_over_ranks([1.5, 2.0]) == [1.5, 2.0]
    assert replicas.gather_streams({1: [3, 4], 0: [1, 2]}) == [[1, 2], [3, 4]]


N_SEQ, PROMPT, N_NEW = 5, 6, 5


def _oracle_generate(model_dir):
    def gen(prompts):
        ref = oracle.RefModel(model_dir)
        try:
            return [[int(t) for t in ref.generate(np.array(p, np.int32), N_NEW)] for p in prompts]
        finally:
            ref.close()
    return gen


def _rank_main(rank, world, port, model_dir, out_path):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        local = replicas.run_replica(_oracle_generate(model_dir), lambda i: synth.prompt_ids(100 + i, PROMPT), N_SEQ)
        # every rank reports a different "time"; the job's time is the largest
        t = replicas.max_over_ranks([1.0 + rank, 10.0 - rank])
        streams = replicas.gather_streams(local)
        if rank == 0:
            np.save(out_path, np.array(streams, np.int64))
            np.save(out_path + ".t.npy", np.array(t))
        else:
            assert streams is None
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_two_gloo_ranks_match_single_process(tiny_model, tmp_path):
    import torch.multiprocessing as mp
    out = str(tmp_path / "streams.npy")
    mp.start_processes(_rank_main, args=(2, _free_port(), tiny_model, out), nprocs=2, join=True,
                       start_method="spawn")
    got = np.load(out)
    assert list(np.load(out + ".t.npy")) == [2.0, 10.0]
    want = _oracle_generate(tiny_model)([synth.prompt_ids(100 + i, PROMPT) for i in range(N_SEQ)])
    assert got.tolist() == want
