"""The continuous-batching engine's scheduling on CPU, with a stand-in
handle whose per-sequence state is an integer hash of the tokens it has
seen: every request served among others, in whichever slot, must produce
exactly the tokens it produces served alone (reference serve.py
generate_stream: prompt, then sample / append / step until max_tokens, the
end-of-sequence id (not emitted) or a stop id)."""
from __future__ import annotations

import numpy as np
import pytest

from sunnynet_b200.serve import BatchEngine, sample_token

V = 97


class FakeHandle:
    """n sequences; logits are a deterministic function of each sequence's
    state, the state a hash of its tokens."""

    def __init__(self, n):
        self.n, self.vocab = n, V
        self.st = np.zeros(n, np.int64)

    def _logits(self, rows):
        v = np.arange(V)
        return np.stack([np.cos(0.37 * ((self.st[i] * 13 + v * 7) % 101)) for i in rows]
                        ).astype(np.float32)

    def reset(self):
        self.st[:] = 0

    def prefill(self, toks, chunk=256):
        toks = np.asarray(toks)
        for i, row in enumerate(toks):
            for t in row:
                self.st[i] = (self.st[i] * 31 + int(t) + 1) % 1000003
        return self._logits(range(toks.shape[0]))

    def step(self, toks):
        for i, t in enumerate(np.asarray(toks)):
            self.st[i] = (self.st[i] * 31 + int(t) + 1) % 1000003
        return self._logits(range(len(toks)))

    def step_argmax(self, toks):
        return self.step(toks).argmax(1).astype(np.int32)

    def get_state_at(self, seq0, n):
        return self.st[seq0:seq0 + n].reshape(n, 1, 1).copy(), np.zeros((n, 1, 1, 1))

    def set_state_at(self, seq0, s, h):
        self.st[seq0:seq0 + len(s)] = np.asarray(s).reshape(-1)


def _alone(prompt, max_tokens, eos=None, stop=(), **samp):
    h = FakeHandle(1)
    rng = np.random.default_rng(samp.pop("seed", None))
    lg = h.prefill(np.array([prompt]))[0]
    out = []
    while True:
        t = sample_token(lg, samp.get("temperature", 0.0), samp.get("top_p", 1.0),
                         samp.get("top_k", 0), rng)
        if eos is not None and t == eos:
            break
        out.append(t)
        if t in stop or len(out) >= max_tokens:
            break
        lg = h.step(np.array([t]))[0]
    return out


def test_requests_served_together_equal_served_alone():
    rng = np.random.default_rng(0)
    reqs = [(list(rng.integers(0, V, n)), m) for n, m in
            [(5, 6), (9, 4), (9, 8), (17, 5), (3, 10), (30, 3), (9, 7), (1, 1), (2, 12)]]
    eng = BatchEngine(slots=3, handle_factory=FakeHandle)
    handles = [eng.submit(p, m) for p, m in reqs]
    done = eng.run()
    assert sorted(r.id for r in done) == list(range(len(reqs)))
    for r, (p, m) in zip(handles, reqs):
        assert r.done and r.finish_reason == "length"
        assert r.tokens == _alone(p, m), r.id
    assert all(s is None for s in eng.slots)


def test_eos_stop_ids_and_seeded_sampling():
    rng = np.random.default_rng(1)
    eng = BatchEngine(slots=2, eos=5, handle_factory=FakeHandle)
    specs = []
    for k in range(6):
        p = list(rng.integers(0, V, 4 + k))
        samp = dict(temperature=0.8, top_p=0.9, top_k=20, seed=100 + k)
        stop = (7, 11) if k % 2 else ()
        specs.append((p, samp, stop, eng.submit(p, 40, stop_ids=stop, **samp)))
    eng.run()
    for p, samp, stop, r in specs:
        assert r.tokens == _alone(p, 40, eos=5, stop=stop, **dict(samp))
        assert r.finish_reason in ("eos", "stop", "length")
        assert 5 not in r.tokens


def test_sample_token_rules():
    lg = np.array([0.0, 3.0, 3.0, -1.0], np.float32)
    assert sample_token(lg, 0.0) == 1  # greedy, lowest id on ties
    rng = np.random.default_rng(0)
    draws = {sample_token(lg, 1.0, top_k=2, rng=rng) for _ in range(200)}
    assert draws == {1, 2}
    draws = {sample_token(np.array([5.0, 0.0, 0.0]), 1.0, top_p=0.5, rng=rng) for _ in range(50)}
    assert draws == {0}  # the most probable token alone covers top_p


def test_rejects_empty_prompt_and_zero_budget():
    eng = BatchEngine(slots=1, handle_factory=FakeHandle)
    with pytest.raises(ValueError):
        eng.submit([], 3)
    with pytest.raises(ValueError):
        eng.submit([1], 0)
