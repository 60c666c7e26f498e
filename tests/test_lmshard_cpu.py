"""Host logic of the LM head split by vocabulary rows (gpt2b200.lmshard), on
CPU ranks (gloo, world size 2).

The GPU part (Engine.lm_head_rows) is tested in test_gpu_lmshard.py; here the
ranks stand in for it with numpy: every rank holds its own rows, all-gathers
them, computes logits over its vocabulary range only, and the exchange of
per-row bests must reproduce the reference's first maximum over the whole
vocabulary (main.c:1898-1904), ties across ranges included.
"""
import os
import socket

import numpy as np
import pytest

from gpt2b200 import lmshard

torch = pytest.importorskip("torch")


def test_vocab_ranges_cover_the_vocabulary_once():
    for V in (1, 127, 128, 50257, 50304):
        for world in (1, 2, 3, 8):
            rs = [lmshard.vocab_range(V, world, r) for r in range(world)]
            got = [v for a, b in rs for v in range(a, b)]
            assert got == list(range(V)), (V, world)
            for a, b in rs:
                assert a <= b and (a % 128 == 0 or a == b)   # an empty range may start at V
    with pytest.raises(ValueError):
        lmshard.vocab_range(100, 2, 2)


def test_merge_prefers_larger_value_then_smaller_index():
    v = torch.tensor([[1.0, 5.0, 2.0, 3.0], [1.0, 4.0, 2.5, 3.0]])
    i = torch.tensor([[7, 1, 2, 9], [3, 8, 4, 2]])
    bv, bi = lmshard.merge_best(v, i)
    assert bv.tolist() == [1.0, 5.0, 2.5, 3.0]
    assert bi.tolist() == [3, 1, 4, 2]


def first_argmax(logits):
    """Per row the first maximum (np.argmax already returns the first)."""
    return np.argmax(logits, axis=1)


B, E, V = 5, 16, 1000


def _problem():
    # small integers: every dot product is exact in any summation order, so the
    # ranges' logits equal the whole head's bit for bit and ties are exact (and common)
    rng = np.random.default_rng(3)
    W = rng.integers(-3, 4, size=(V, E)).astype(np.float32)
    W[640] = W[300]            # equal logits on both sides of the 2-rank boundary (512)
    W[900] = W[10]             # and within one range
    rows = rng.integers(-3, 4, size=(2 * B, E)).astype(np.float32)
    rows[1] = W[300] * 4       # rows whose maximum is one of the tied pairs
    rows[B + 2] = W[10] * 4
    return W, rows


def _rank_main(rank, world, port, out_path):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        W, rows = _problem()
        mine = torch.from_numpy(rows[rank * B:(rank + 1) * B].copy())
        all_rows = lmshard.gather_rows(mine).numpy()
        assert np.array_equal(all_rows, rows)
        v0, v1 = lmshard.vocab_range(V, world, rank)
        logits = all_rows @ W[v0:v1].T
        best_i = torch.from_numpy((np.argmax(logits, axis=1) + v0).astype(np.int32))
        best_v = torch.from_numpy(logits[np.arange(len(logits)), best_i.numpy() - v0].astype(np.float32))
        _, got = lmshard.exchange_best(best_v, best_i, slice(rank * B, (rank + 1) * B))
        np.save(f"{out_path}.{rank}.npy", got.numpy())
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_two_gloo_ranks_reproduce_the_first_maximum(tmp_path):
    import torch.multiprocessing as mp
    out = str(tmp_path / "best")
    mp.start_processes(_rank_main, args=(2, _free_port(), out), nprocs=2, join=True, start_method="spawn")
    W, rows = _problem()
    want = first_argmax(rows @ W.T)
    got = np.concatenate([np.load(f"{out}.{r}.npy") for r in range(2)])
    assert got.tolist() == want.tolist()
    assert want[1] == 300 and want[B + 2] == 10   # the planted ties resolve to the smaller index
