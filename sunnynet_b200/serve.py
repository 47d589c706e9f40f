"""Serving SunnyNet on a B200: the reference's per-request engine contract and
a continuous-batching engine over one batched handle.

Reference: sunnynet/serve.py -- ``Engine`` (encode / decode / init_state /
step, :60-79), the C-runtime engine that owns one sequence and resets it per
request (``GGUFCEngine``, :177-207), the sampling rule (``sample_logits``,
:30-57) and the generation loop (``generate_stream``, :254-281).

``CudaSunnyEngine`` keeps that contract for one sequence at a time, so the
reference's HTTP front end can use it unchanged. ``BatchEngine`` is what the
batched step is for: requests join and leave a fixed set of slots (sequences
of one ``SunnyBatch``) between steps, so one decode step serves every live
request:

* admission: waiting requests take free slots; their prompts run through a
  second handle's chunked prefill (requests of equal prompt length share one
  call), and each request's state is copied device-to-device into its slot;
  the first token is sampled from the prefill's last logits;
* decode: one batched step over slots [0, highest live slot]; slots without a
  live request are fed token 0 and their outputs ignored (their state is
  overwritten when a request takes the slot);
* a request ends at ``max_tokens`` generated tokens, at the end-of-sequence
  id (not emitted, as in the reference loop) or at one of its stop ids; its
  slot is free for the next step's admission.

Sampling follows the reference: temperature <= 0 is greedy (lowest id on
ties); otherwise logits / temperature, top-k, then nucleus top-p (the most
probable token always kept), drawn with the request's numpy generator. When
every live request is greedy the step returns only the argmax ids from the
device instead of all logits.
"""
from __future__ import annotations

import collections
import itertools
from dataclasses import dataclass, field

import numpy as np

from .model import SunnyBatch

__all__ = ["sample_token", "CudaSunnyEngine", "Request", "BatchEngine"]


def sample_token(logits, temperature=1.0, top_p=1.0, top_k=0, rng=None) -> int:
    """Next token id from one row of logits (the reference's sampling rule)."""
    x = np.asarray(logits, np.float64)
    if temperature is None or temperature <= 0:
        return int(np.argmax(x))
    z = x / float(temperature)
    if top_k and 0 < top_k < z.size:
        kth = np.partition(z, z.size - int(top_k))[z.size - int(top_k)]
        z = np.where(z >= kth, z, -np.inf)
    if 0.0 < top_p < 1.0:
        order = np.argsort(-z, kind="stable")
        zs = z[order]
        w = np.exp(zs - zs[0])
        w /= w.sum()
        before = np.concatenate(([0.0], np.cumsum(w)[:-1]))  # mass ahead of each token
        zs = np.where(before < top_p, zs, -np.inf)               # the first is always kept
        z = np.full_like(z, -np.inf)
        z[order] = zs
    w = np.exp(z - np.max(z))
    tot = w.sum()
    if not np.isfinite(tot) or tot <= 0:
        return int(np.argmax(x))
    rng = rng or np.random.default_rng()
    return int(rng.choice(z.size, p=w / tot))


class CudaSunnyEngine:
    """The reference ``Engine`` contract for one sequence at a time on the GPU
    (like its C-runtime engine, the state lives in the handle: init_state
    resets it and the returned state object is a placeholder)."""

    name = "sunnynet-cuda"

    def __init__(self, blob, tokenizer=None, eos=None):
        self.model = SunnyBatch(blob, 1)
        self.vocab = self.model.vocab
        self.tok = tokenizer
        self.eos = eos

    def encode(self, text: str) -> list:
        if self.tok is None:
            raise NotImplementedError("no tokenizer given")
        return list(self.tok.encode(text))

    def decode(self, ids) -> str:
        if self.tok is None:
            raise NotImplementedError("no tokenizer given")
        return self.tok.decode([int(i) for i in ids])

    def init_state(self):
        self.model.reset()
        return {}

    def step(self, token, state):
        return self.model.step(np.array([int(token)], np.int32))[0].copy(), state


@dataclass
class Request:
    prompt: list
    max_tokens: int
    temperature: float = 0.0
    top_p: float = 1.0
    top_k: int = 0
    seed: int | None = None
    stop_ids: tuple = ()
    record_logits: bool = False  # keep the logits each token was drawn from (testing)
    id: int = -1
    tokens: list = field(default_factory=list)
    logits: list = field(default_factory=list)
    slot: int = -1
    done: bool = False
    finish_reason: str | None = None

    def __post_init__(self):
        self._rng = np.random.default_rng(self.seed)


class BatchEngine:
    """Continuous batching over `slots` sequences of one batched handle.

    ``handle_factory(n)`` makes a handle of n sequences (default: a
    ``SunnyBatch`` of `blob`); it must offer prefill, step, step_argmax,
    get_state_at, set_state_at and reset.
    """

    def __init__(self, blob=None, slots: int = 16, eos: int | None = None,
                 prefill_chunk: int = 256, handle_factory=None):
        factory = handle_factory or (lambda n: SunnyBatch(blob, n))
        self.main = factory(slots)
        self.pre = factory(slots)
        self.vocab = self.main.vocab
        self.eos = eos
        self.chunk = prefill_chunk
        self.slots: list = [None] * slots
        self.waiting: collections.deque = collections.deque()
        self.finished: list = []
        self._ids = itertools.count()

    # ------------------------------------------------------------- requests
    def submit(self, prompt, max_tokens: int, **sampling) -> Request:
        if len(prompt) == 0:
            raise ValueError("a request needs at least one prompt token")
        if max_tokens <= 0:
            raise ValueError("max_tokens must be positive")
        r = Request(list(int(t) for t in prompt), int(max_tokens), **sampling)
        r.id = next(self._ids)
        self.waiting.append(r)
        return r

    def busy(self) -> bool:
        return bool(self.waiting) or any(r is not None for r in self.slots)

    # ---------------------------------------------------------------- steps
    def _finish(self, r: Request, reason: str):
        r.done, r.finish_reason = True, reason
        self.slots[r.slot] = None
        self.finished.append(r)

    def _take(self, r: Request, logits_row=None, token=None, events=None):
        """Choose r's next token from its logits (or the device's argmax)."""
        if logits_row is not None:
            if r.record_logits:
                r.logits.append(np.array(logits_row, np.float32))
            token = sample_token(logits_row, r.temperature, r.top_p, r.top_k, r._rng)
        if self.eos is not None and token == self.eos:
            self._finish(r, "eos")
            return
        r.tokens.append(int(token))
        if events is not None:
            events.append((r, int(token)))
        if int(token) in r.stop_ids:
            self._finish(r, "stop")
        elif len(r.tokens) >= r.max_tokens:
            self._finish(r, "length")

    def _admit(self, events):
        free = [i for i, r in enumerate(self.slots) if r is None]
        batch = []
        while free and self.waiting:
            r = self.waiting.popleft()
            r.slot = free.pop(0)
            self.slots[r.slot] = r
            batch.append(r)
        by_len = collections.defaultdict(list)
        for r in batch:
            by_len[len(r.prompt)].append(r)
        for T, group in sorted(by_len.items()):
            n = len(group)
            self.pre.reset()
            lg = np.asarray(self.pre.prefill(np.array([r.prompt for r in group], np.int32),
                                             chunk=self.chunk))
            s, h = self.pre.get_state_at(0, n)
            for j, r in enumerate(group):
                self.main.set_state_at(r.slot, s[j:j + 1], h[j:j + 1])
                self._take(r, logits_row=lg[j], events=events)

    def step(self) -> list:
        """Admit waiting requests, then one decode step for every live
        request. Returns the (request, token) pairs produced."""
        events: list = []
        self._admit(events)
        live = [r for r in self.slots if r is not None]
        if not live:
            return events
        B = max(r.slot for r in live) + 1
        toks = np.zeros(B, np.int32)
        for r in live:
            toks[r.slot] = r.tokens[-1]
        if all(r.temperature is None or r.temperature <= 0 for r in live) and \
                not any(r.record_logits for r in live):
            nxt = np.asarray(self.main.step_argmax(toks))
            for r in live:
                self._take(r, token=int(nxt[r.slot]), events=events)
        else:
            lg = np.asarray(self.main.step(toks))
            for r in live:
                self._take(r, logits_row=lg[r.slot], events=events)
        return events

    def run(self) -> list:
        """Step until every submitted request has finished; the finished
        requests in completion order."""
        while self.busy():
            self.step()
        return self.finished
