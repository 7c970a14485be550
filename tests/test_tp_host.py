"""Tensor-parallel host logic on CPU: shard arithmetic (mirror of llama_model_create)
and the IPC-handle exchange over a world-size-2 gloo process group."""
import os
import socket

import pytest

torch = pytest.importorskip("torch")
import torch.distributed as dist  # noqa: E402
import torch.multiprocessing as mp  # noqa: E402

from fp4x import engine, tp  # noqa: E402


@pytest.mark.parametrize("world", [2, 4, 8])
def test_shards_cover_the_model(world):
    cfg = engine.LLAMA3_8B
    parts = [tp.shard_ranges(cfg, r, world) for r in range(world)]
    for key, total in (("heads", cfg["n_heads"]), ("kv_heads", cfg["n_kv_heads"]), ("ffn", cfg["ffn"]),
                       ("vocab", cfg["vocab"])):
        spans = [p[key] for p in parts]
        assert spans[0][0] == 0 and spans[-1][1] == total
        assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
    assert all((p["ffn"][1] - p["ffn"][0]) % 32 == 0 for p in parts)  # down columns split on scale blocks
    assert all(p["vocab"][0] % 16 == 0 for p in parts)


def test_shards_reject_uneven_split():
    with pytest.raises(ValueError):
        tp.shard_ranges(dict(engine.TINYLLAMA), 0, 8)  # 4 KV heads over 8 ranks


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, result):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        mine = bytes([rank]) * 64
        got = tp.exchange_handles(mine)
        result[rank] = got == [bytes([r]) * 64 for r in range(world)]
    finally:
        dist.destroy_process_group()


def test_handle_exchange_gloo_world2():
    world = 2
    with mp.get_context("spawn").Manager() as man:
        result = man.dict()
        mp.spawn(_worker, args=(world, _free_port(), result), nprocs=world, join=True)
        assert dict(result) == {0: True, 1: True}
