"""The LM head split by vocabulary rows on the GPU (Engine.decode_batch_rows,
Engine.lm_head_rows, gpt2b200.lmshard).

* On one GPU: the head over several ranges of wte rows, merged by the first-
  maximum rule, gives the unsplit head's greedy tokens (g2_decode_batch +
  g2_argmax) and values within the kernel tolerance; one range [0, V) too.
* generate_batch_sharded without a process group equals generate_batch.
* On two GPUs (skipped with fewer): two NCCL ranks, each decoding its own
  sequences with the head split between them, give every sequence the tokens
  of an unsplit run on one GPU.
"""
import os
import socket

import numpy as np
import pytest

from gpt2b200 import lmshard, synth

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

TOL = {"f32": 1e-5, "f16": 1e-3}


@pytest.fixture(scope="module")
def g2():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import gpt2b200
    return gpt2b200


def _model(dtype):
    from conftest import MODEL_CACHE
    return synth.ensure_model(os.path.join(MODEL_CACHE, f"tiny_affine_s1_{dtype}"), synth.TINY, seed=1, affine=True,
                              dtype=dtype)


def _prompts(n):
    return [synth.prompt_ids(40 + i, 9 + 3 * i) for i in range(n)]


@pytest.mark.parametrize("dtype", ["f32", "f16"])
def test_ranges_merged_equal_the_unsplit_head(g2, dtype):
    d, kind = _model(dtype), g2.G2_F32 if dtype == "f32" else g2.G2_F16
    prompts = _prompts(4)
    slots = np.arange(4, dtype=np.int32)
    pos = np.array([len(p) for p in prompts], np.int32)
    with g2.Engine(d, max_batch=4, dtype=kind) as full, g2.Engine(d, max_batch=4, dtype=kind) as split:
        toks = []
        for s, p in enumerate(prompts):
            full.prefill(p, slot=s)
            split.prefill(p, slot=s)
            toks.append(full.argmax(s)[0])
        toks = np.array(toks, np.int32)
        full.decode_batch(slots, toks, pos)
        want = [full.argmax(s) for s in range(4)]
        logits = [full.logits(s) for s in range(4)]
        E, V = split.cfg.n_embd, split.cfg.vocab_size
        rows = torch.empty((4, E), device="cuda")
        split.decode_batch_rows(slots, toks, pos, rows)
        for world in (1, 2, 3):
            vals, idxs = [], []
            for r in range(world):
                v0, v1 = lmshard.vocab_range(V, world, r)
                bv = torch.empty(4, device="cuda")
                bi = torch.empty(4, dtype=torch.int32, device="cuda")
                split.lm_head_rows(rows, 4, v0, v1, bv, bi)
                assert all(v0 <= int(i) < v1 for i in bi.tolist())
                vals.append(bv)
                idxs.append(bi)
            bv, bi = lmshard.merge_best(torch.stack(vals), torch.stack(idxs))
            for s in range(4):
                assert int(bi[s]) == want[s][0], (world, s)
                scale = float(np.abs(logits[s][:V]).max())
                assert abs(float(bv[s]) - logits[s][want[s][0]]) <= TOL[dtype] * scale


def test_rejects_bad_ranges(g2):
    d = _model("f32")
    with g2.Engine(d, max_batch=2) as eng:
        rows = torch.zeros((2, eng.cfg.n_embd), device="cuda")
        bv = torch.empty(2, device="cuda")
        bi = torch.empty(2, dtype=torch.int32, device="cuda")
        for v0, v1 in ((2, 100), (0, eng.cfg.vocab_size + 1), (100, 100), (-4, 8)):
            with pytest.raises(g2.G2Error):
                eng.lm_head_rows(rows, 2, v0, v1, bv, bi)
        with pytest.raises(g2.G2Error):
            eng.lm_head_rows(rows, 100000, 0, 128, bv, bi)


def test_sharded_generation_on_one_rank_equals_generate_batch(g2):
    d = _model("f32")
    prompts = _prompts(3)
    with g2.Engine(d, max_batch=3) as a:
        want = a.generate_batch(prompts, 12)
    with g2.Engine(d, max_batch=3) as b:
        got = lmshard.generate_batch_sharded(b, prompts, 12, torch.device("cuda"))
    assert np.array(got).tolist() == want.tolist()


def _rank_main(rank, world, port, model_dir, out_path):
    import torch.distributed as dist
    import gpt2b200 as g2m
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank))
    try:
        prompts = [synth.prompt_ids(200 + 10 * rank + i, 7 + i) for i in range(3)]
        with g2m.Engine(model_dir, device=rank, max_batch=3) as eng:
            got = lmshard.generate_batch_sharded(eng, prompts, 10, torch.device("cuda", rank))
        with g2m.Engine(model_dir, device=rank, max_batch=3) as eng:
            want = eng.generate_batch(prompts, 10)
        np.save(f"{out_path}.{rank}.npy", np.array([got, want.tolist()]))
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_two_nccl_ranks_split_the_head(g2, tmp_path):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    out = str(tmp_path / "gen")
    mp.start_processes(_rank_main, args=(2, port, _model("f32"), out), nprocs=2, join=True, start_method="spawn")
    for r in range(2):
        got, want = np.load(f"{out}.{r}.npy")
        assert got.tolist() == want.tolist(), r
