"""Tensor parallelism on 2 GPUs (one process per GPU): every rank's weight shards
equal the oracle's slices bit-exactly, every rank's logits slice matches the
oracle within 1e-2, and greedy generation reproduces the oracle's tokens.  The
allreduce and argmax run inside the decode graph over NVLink peer memory."""
import os
import socket

import numpy as np
import pytest

torch = pytest.importorskip("torch")
import torch.distributed as dist  # noqa: E402
import torch.multiprocessing as mp  # noqa: E402

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                                 reason="needs 2 GPUs")]

TINY = dict(n_layers=2, dim=256, ffn=512, n_heads=8, n_kv_heads=2, head_dim=64, vocab=1000, max_seq=64,
            rope_theta=10000.0, eps=1e-5, seed=1234)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _rel(got, ref):
    rms = np.sqrt(np.mean(ref.astype(np.float64) ** 2)) + 1e-30
    return float(np.max(np.abs(got.astype(np.float64) - ref)) / rms)


def _worker(rank, world, port, cfg, path, result):
    import datetime
    import oracle
    from fp4x import tp
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120))
    out = {}
    try:
        ref = oracle.Model(cfg)
        m = tp.create_model(cfg)
        m.set_path(path)
        sh = tp.shard_ranges(cfg, rank, world)
        hd = cfg["head_dim"]
        q0, q1 = sh["heads"][0] * hd, sh["heads"][1] * hd
        k0, k1 = sh["kv_heads"][0] * hd, sh["kv_heads"][1] * hd
        f0, f1 = sh["ffn"]
        v0, v1 = sh["vocab"]
        assert m.shard() == (v0, v1 - v0)
        qd, kvd = cfg["n_heads"] * hd, cfg["n_kv_heads"] * hd
        checks = {1: ((v0, v1), None)}
        base = 16 + 8 * (cfg["n_layers"] - 1)
        checks.update({base + 0: ((q0, q1), None), base + 1: ((k0, k1), None), base + 2: ((k0, k1), None),
                       base + 3: (None, (q0, q1)), base + 4: ((f0, f1), None), base + 5: ((f0, f1), None),
                       base + 6: (None, (f0, f1))})
        shapes = {0: (qd, cfg["dim"]), 1: (kvd, cfg["dim"]), 2: (kvd, cfg["dim"]), 3: (cfg["dim"], qd),
                  4: (cfg["ffn"], cfg["dim"]), 5: (cfg["ffn"], cfg["dim"]), 6: (cfg["dim"], cfg["ffn"])}
        for tid, (rows, cols) in checks.items():
            n, k = (cfg["vocab"], cfg["dim"]) if tid == 1 else shapes[(tid - 16) % 8]
            rp, rs = ref.tensor(tid, n, k)
            if rows:
                rp, rs = rp[rows[0]:rows[1]], rs[rows[0]:rows[1]]
            if cols:
                rp, rs = rp[:, cols[0] // 2:cols[1] // 2], rs[:, cols[0] // 32:cols[1] // 32]
            gp, gs = m.export_tensor(tid)
            np.testing.assert_array_equal(gs, rs, err_msg=f"scales {tid}")
            np.testing.assert_array_equal(gp, rp, err_msg=f"nibbles {tid}")
        toks = oracle.uniform_ids(5, cfg["vocab"], 12)
        worst = 0.0
        for pos, t in enumerate(toks):
            gn, gl = m.forward(int(t), pos)
            rn, rl = ref.forward(int(t), pos)
            worst = max(worst, _rel(gl, rl[v0:v1]))
            assert gn == rn or abs(float(np.sort(rl)[-1] - np.sort(rl)[-2])) < 1e-2 * np.sqrt(np.mean(rl ** 2))
        out["logits_err"] = worst
        prompt = oracle.uniform_ids(3, cfg["vocab"], 6)
        m.reset()
        ref2 = oracle.Model(cfg)
        want = ref2.generate(prompt, 16)
        got, _, _ = m.generate(prompt, 16)
        out["generate_equal"] = bool(np.array_equal(got, want))
        torch.cuda.synchronize()
        m.close()
        ref.close()
        ref2.close()
        result[rank] = out
    finally:
        dist.barrier()
        dist.destroy_process_group()


@pytest.mark.parametrize("path", ["graph", "tensor"])
def test_tp2_matches_oracle(path):
    """graph: per-layer kernels + the in-graph peer-memory allreduce kernel;
    tensor: the persistent tcgen05 kernel adding its row-parallel outputs into every
    rank's residual over NVLink, with cross-rank grid barriers."""
    world = 2
    with mp.get_context("spawn").Manager() as man:
        result = man.dict()
        mp.spawn(_worker, args=(world, _free_port(), TINY, path, result), nprocs=world, join=True)
        res = dict(result)
    assert set(res) == {0, 1}
    for r, out in res.items():
        assert out["logits_err"] <= 1e-2, (r, out)
        assert out["generate_equal"], (r, out)


def _batch_worker(rank, world, port, cfg, result):
    """Batched engine at TP=2 against the same engine at TP=1 (this process's GPU):
    per-sequence logits slices within 1e-2, identical greedy tokens."""
    import datetime
    import oracle
    from fp4x import engine, tp
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120))
    out = {}
    try:
        prompts = [oracle.uniform_ids(40 + i, cfg["vocab"], n) for i, n in enumerate((5, 9, 2))]
        runs = {}
        for mode in ("tp", "single"):
            m = tp.create_model(cfg) if mode == "tp" else engine.Model(cfg)
            b = tp.create_batch(m, 4) if mode == "tp" else engine.Batch(m, 4)
            logits = []
            for s, p in enumerate(prompts):
                b.prefill(s, p)
                logits.append(b.logits()[0])
            for _ in range(5):
                b.decode(1)
                logits.append(b.logits()[:3])
            toks = [b.tokens(s) for s in range(3)]
            runs[mode] = (logits, toks, m.shard())
            b.close()
            m.close()
        (lt, tt, (v0, nv)), (ls, ts, _) = runs["tp"], runs["single"]
        worst = 0.0
        for a, c in zip(lt, ls):
            worst = max(worst, _rel(np.asarray(a), np.asarray(c)[..., v0:v0 + nv]))
        out["logits_err"] = worst
        out["tokens_equal"] = all(np.array_equal(x, y) for x, y in zip(tt, ts))
        result[rank] = out
    finally:
        dist.barrier()
        dist.destroy_process_group()


def test_tp2_batched_engine_matches_single_gpu():
    world = 2
    with mp.get_context("spawn").Manager() as man:
        result = man.dict()
        mp.spawn(_batch_worker, args=(world, _free_port(), TINY, result), nprocs=world, join=True)
        res = dict(result)
    assert set(res) == {0, 1}
    for r, out in res.items():
        assert out["logits_err"] <= 1e-2, (r, out)
        assert out["tokens_equal"], (r, out)


def _stall_worker(rank, world, port, cfg, path, result):
    """Rank 1 stops issuing after one step (it waits on the host, its exchange area
    still mapped); rank 0 runs one more step with a short flag-wait limit.  The
    device-side waits for rank 1's flags run out, the kernels return, and rank 0
    reads FP4X_ETIMEOUT from fp4x_device_error on a context that still works."""
    import ctypes
    import datetime
    import oracle
    import fp4x
    from fp4x import Fp4xError, ops, tp
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120))
    out = {}
    L = fp4x.lib()
    try:
        toks = oracle.uniform_ids(7, cfg["vocab"], 2)
        m = tp.create_model(cfg)
        m.set_path(path)
        m.forward(int(toks[0]), 0, want_logits=False)  # a normal step on both ranks
        torch.cuda.synchronize()
        dist.barrier()
        if rank == 0:
            assert L.fp4x_set_wait_limit(4096) == 0
            try:
                m.forward(int(toks[1]), 1, want_logits=False)
                out["forward"] = "returned"
            except Fp4xError as e:  # the call may already report the expired wait
                out["forward"] = str(e)
            bits = ctypes.c_uint32(0)
            out["status"] = L.fp4x_device_error(torch.cuda.current_stream().cuda_stream, ctypes.byref(bits))
            out["bits"] = bits.value
            assert L.fp4x_set_wait_limit(0) == 0
            x = ops.fill_normal(1 << 16, seed=5)
            torch.cuda.synchronize()
            out["usable"] = bool(torch.isfinite(x).all().item())
        dist.barrier()  # rank 1 keeps its area mapped until rank 0's step has ended
        m.close()
        torch.cuda.synchronize()
        result[rank] = out
    finally:
        dist.barrier()
        dist.destroy_process_group()


@pytest.mark.parametrize("path", ["graph", "tensor"])
def test_tp2_stalled_rank_wait_expires(path):
    world = 2
    with mp.get_context("spawn").Manager() as man:
        result = man.dict()
        mp.spawn(_stall_worker, args=(world, _free_port(), TINY, path, result), nprocs=world, join=True)
        res = dict(result)
    assert set(res) == {0, 1}
    r0 = res[0]
    assert r0["status"] == 3, r0  # FP4X_ETIMEOUT
    assert r0["bits"] & 2, r0  # DEVERR_FLAG_TIMEOUT
    assert r0["usable"], r0
