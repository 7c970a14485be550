"""Batched engine (llama_batch_*) vs the CPU oracle: several sequences prefilled
in multi-token passes (causal attention inside a pass) and decoded together, each
sequence's logits within 1e-2 of the oracle's single-sequence forward and the
same greedy tokens.  All calls go through the C ABI."""
import numpy as np
import pytest

import oracle
from test_gpu_engine import TINY, TINY128, compare_logits

torch = pytest.importorskip("torch")
from fp4x import Fp4xError, engine  # noqa: E402

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("cfg", [TINY, TINY128], ids=["hd64", "hd128"])
def test_batch_prefill_and_decode_vs_oracle(cfg):
    rows = 4
    prompts = [oracle.uniform_ids(100 + i, cfg["vocab"], n) for i, n in enumerate((5, 9, 3))]
    refs = [oracle.Model(cfg) for _ in prompts]
    with engine.Model(cfg) as m, engine.Batch(m, rows) as b:
        nxt = []
        for s, (p, ref) in enumerate(zip(prompts, refs)):
            b.prefill(s, p)  # 9 tokens -> passes of 4 + 4 + 1 rows
            got = b.logits()
            assert got.shape == (1, cfg["vocab"])
            for pos, t in enumerate(p):
                rn, rl = ref.forward(int(t), pos)
            compare_logits(got[0], rl)
            toks = b.tokens(s)
            np.testing.assert_array_equal(toks[:len(p)], p)
            assert len(toks) == len(p) + 1 and toks[-1] == int(np.argmax(got[0]))
            nxt.append(int(toks[-1]))
        pos = [len(p) for p in prompts]
        for step in range(6):
            b.decode(1)
            got = b.logits()
            assert got.shape == (rows, cfg["vocab"])
            for s, ref in enumerate(refs):
                rn, rl = ref.forward(nxt[s], pos[s])
                compare_logits(got[s], rl)
                toks = b.tokens(s)
                assert len(toks) == pos[s] + 2
                assert toks[-1] == int(np.argmax(got[s]))
                nxt[s] = int(toks[-1])
                pos[s] += 1
    for r in refs:
        r.close()


def test_batch_greedy_tokens_match_oracle_generate():
    cfg = TINY
    # prompts whose 16 oracle greedy steps have no near-tie (top-2 margin > 3e-3 rms)
    prompts = [oracle.uniform_ids(11, cfg["vocab"], 4), oracle.uniform_ids(20, cfg["vocab"], 6)]
    with engine.Model(cfg) as m, engine.Batch(m, 2) as b:
        for s, p in enumerate(prompts):
            b.prefill(s, p)
        b.decode(15)
        got = [b.tokens(s)[len(p):] for s, p in enumerate(prompts)]
    for p, g in zip(prompts, got):
        ref = oracle.Model(cfg)
        want = ref.generate(p, 16)
        ref.close()
        np.testing.assert_array_equal(g, want)


def test_batch_decode_graph_repeats_and_prefill_after_decode():
    """Multi-step decode equals single steps; a sequence can be extended by a
    prefill after decoding (its cache continues at its own length)."""
    cfg = TINY
    p = oracle.uniform_ids(3, cfg["vocab"], 6)
    with engine.Model(cfg) as m:
        with engine.Batch(m, 2) as b1:
            b1.prefill(0, p)
            b1.decode(5)
            t1 = b1.tokens(0)
        with engine.Batch(m, 2) as b2:
            b2.prefill(0, p)
            for _ in range(5):
                b2.decode(1)
            np.testing.assert_array_equal(b2.tokens(0), t1)
            extra = oracle.uniform_ids(4, cfg["vocab"], 3)
            b2.prefill(0, extra)
            t2 = b2.tokens(0)
    assert len(t2) == len(t1) - 1 + 3 + 1
    np.testing.assert_array_equal(t2[:len(t1) - 1], t1[:-1])
    ref = oracle.Model(cfg)
    seq = list(t1[:-1]) + list(extra)
    for pos, t in enumerate(seq):
        rn, _ = ref.forward(int(t), pos)
    ref.close()
    assert t2[-1] == rn


def test_batch_rejects_bad_arguments():
    with engine.Model(TINY) as m:
        with pytest.raises(Fp4xError):
            engine.Batch(m, 0)
        with engine.Batch(m, 2) as b:
            with pytest.raises(Fp4xError):
                b.prefill(2, [1, 2])  # no such sequence
            with pytest.raises(Fp4xError):
                b.prefill(0, np.arange(TINY["max_seq"]))  # longer than the cache
            with pytest.raises(Fp4xError):
                b.prefill(0, [TINY["vocab"]])  # token out of range
            b.set_length(1, TINY["max_seq"] - 3, 5)
            with pytest.raises(Fp4xError):
                b.decode(3)  # would run sequence 1 past its cache
            b.decode(2)


def test_batch_tinyllama_shape_agrees_with_batch1_engine():
    """BASELINE config-1 shape: three copies of one 16-token prompt, prefilled in
    one pass each and decoded together, agree with each other and with the
    batch-1 engine fed the same tokens (two 8-term/fp32 paths, bound 2e-2)."""
    cfg = dict(engine.TINYLLAMA, max_seq=64)
    prompt = oracle.uniform_ids(11, cfg["vocab"], 16)
    with engine.Model(cfg) as m, engine.Batch(m, 3) as b:
        for s in range(3):
            b.prefill(s, prompt)
        got = [b.logits()[0]]
        for _ in range(3):
            b.decode(1)
            lg = b.logits()
            for s in (1, 2):  # same inputs; split-K red.add order and bf16 KV rounding differ
                compare_logits(lg[s], lg[0])
            got.append(lg[0])
        toks = b.tokens(0)
        for pos in range(len(prompt) + 3):
            _, ref = m.forward(int(toks[pos]), pos)
            if pos >= len(prompt) - 1:
                compare_logits(got[pos - len(prompt) + 1], ref, tol=2e-2)


@pytest.mark.parametrize("terms,tol", [("8", 1e-2), ("4", 3e-2)])
def test_batch_tinyllama_shape_vs_oracle(terms, tol, monkeypatch):
    """BASELINE config-1 shape (22 layers) against the oracle: a 16-token prompt
    prefilled in one pass, then 3 decode steps.  8-term activations (the default)
    meet the 1e-2 logits bar (measured 2.8e-3); the opt-in 4-term mode is held to
    its own measured bound (1.6e-2 measured, 3e-2 gate)."""
    monkeypatch.setenv("FP4X_BATCH_TERMS", terms)
    cfg = dict(engine.TINYLLAMA, max_seq=64)
    prompt = oracle.uniform_ids(11, cfg["vocab"], 16)
    ref = oracle.Model(cfg)
    with engine.Model(cfg) as m, engine.Batch(m, 2) as b:
        b.prefill(0, prompt)
        got = [b.logits()[0]]
        for _ in range(3):
            b.decode(1)
            got.append(b.logits()[0])
        toks = b.tokens(0)
    errs = []
    for pos in range(len(prompt) + 3):
        _, rl = ref.forward(int(toks[pos]), pos)
        if pos >= len(prompt) - 1:
            errs.append(compare_logits(got[pos - len(prompt) + 1], rl, tol=tol))
    ref.close()
    print(f"terms {terms}: max logits err {max(errs):.3e}")
