"""Tensor-parallel weight sharding (velo_cuda_shard_weight / _strategy)
against the oracle's restatement of src/metal/sharding.rs, and the N > 1 path
of the host logic as two gloo ranks on the CPU: each rank shards every tensor
of a model for itself, the shards are all-gathered, and reassembling them
gives back the full tensors."""
import os

import numpy as np
import pytest

import synthetic
import velo_cuda
import vo

NAMES = ["attention.wq", "attention.wk", "attention.wv", "attention.wo", "feed_forward.w1",
         "feed_forward.w2", "feed_forward.w3"]


def test_strategy_names_match_reference():
    for n in NAMES:
        name = f"layers.3.{n}.weight"
        assert velo_cuda.shard_strategy(name) == vo.shard_strategy(name)
    for name in ["output.weight", "token_embd.weight", "output_norm.weight",
                 "layers.0.attention_norm.weight", "layers.0.ffn_norm.weight"]:
        assert velo_cuda.shard_strategy(name) == vo.shard_strategy(name)
    assert velo_cuda.shard_strategy("output.weight") == 1
    assert velo_cuda.shard_strategy("layers.0.attention.wo.weight") == 2


@pytest.mark.parametrize("tp", [2, 4, 8])
@pytest.mark.parametrize("strategy", [0, 1, 2])
def test_shard_bytes_match_oracle(tp, strategy):
    rows, cols = 64, 512
    q4 = synthetic.q4_0_weights(rows, cols, seed=tp)
    f32 = synthetic.rng(tp, 70).normal(0, 1, (rows, cols)).astype(np.float32)
    for dt, data in ((2, q4), (0, f32)):
        for rank in range(tp):
            got, r, c = velo_cuda.shard_weight("w", dt, data, rows, cols, strategy, tp, rank)
            ref, rr, rc = vo.shard_weight(dt, data, rows, cols, strategy, tp, rank)
            assert (r, c) == (rr, rc)
            assert np.array_equal(got, ref)


def test_shard_errors_like_reference():
    q4 = synthetic.q4_0_weights(10, 64, seed=1)
    with pytest.raises(velo_cuda.VeloError):
        velo_cuda.shard_weight("w", 2, q4, 10, 64, 1, 4, 0)   # rows 10 % 4
    with pytest.raises(ValueError):
        vo.shard_weight(2, q4, 10, 64, 1, 4, 0)
    with pytest.raises(velo_cuda.VeloError):
        velo_cuda.shard_weight("w", 2, q4, 10, 64, 2, 4, 0)   # 16-wide q4_0 shard
    with pytest.raises(ValueError):
        vo.shard_weight(2, q4, 10, 64, 2, 4, 0)


def _gloo_rank(rank, world, port, out_q):
    import torch
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        meta, tensors = synthetic.llama_q4_model(256, 256, 1, 2, 2, 512, seed=9)
        ok = True
        for name, (dt, arr, rows, cols) in tensors.items():
            strat = velo_cuda.shard_strategy(name)
            mine, r, c = velo_cuda.shard_weight(name, dt, arr, rows, cols, strat, world, rank)
            t = torch.from_numpy(mine.copy())
            parts = [torch.empty_like(t) for _ in range(world)]
            dist.all_gather(parts, t)
            full = np.ascontiguousarray(arr).view(np.uint8).reshape(rows, -1)
            if strat == 1:
                back = np.concatenate([p.numpy().reshape(r, -1) for p in parts], axis=0)
            elif strat == 2:
                back = np.concatenate([p.numpy().reshape(rows, -1) for p in parts], axis=1)
            else:
                back = parts[rank].numpy().reshape(rows, -1)
            ok &= np.array_equal(back, full)
        out_q.put((rank, bool(ok)))
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_reassemble_every_tensor():
    import multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29500 + os.getpid() % 1000
    ps = [ctx.Process(target=_gloo_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = dict(q.get(timeout=120) for _ in ps)
    for p in ps:
        p.join(timeout=60)
    assert res == {0: True, 1: True}
