"""Continuous batching (smollm2_triton/scheduler.py): slot reuse, streaming,
eos, failures -- host logic on CPU with a stand-in session; on the GPU the
batched answers equal the single-request path."""

from __future__ import annotations

import threading

import numpy as np
import pytest

from smollm2_triton.scheduler import BatchScheduler

V = 97


class _Arr:
    def __init__(self, n):
        self.a = np.zeros(n, np.int32)

    def to_numpy(self):
        return self.a.copy()

    def from_numpy(self, x):
        self.a[...] = np.asarray(x, np.int32)


class FakeSession:
    """Next token = f(current token, position), the same rule per slot."""

    def __init__(self, B, S, fail_at=None):
        self.B, self.S = B, S
        self.ids, self.pos, self.lens = _Arr(B), _Arr(B), _Arr(B)
        self.steps = 0
        self.fail_at = fail_at
        self.prefills = []

    @staticmethod
    def first(prompt):
        return int(np.sum(prompt) * 7 + len(prompt)) % V

    @staticmethod
    def nxt(tok, pos):
        return (tok * 31 + pos * 3 + 1) % V

    def prefill(self, prompts, slots=None):
        self.prefills.append(list(slots))
        logits = np.zeros((len(prompts), V), np.float32)
        for i, (p, s) in enumerate(zip(prompts, slots)):
            t = self.first(p)
            logits[i, t] = 1.0
            self.ids.a[s] = t
            self.pos.a[s] = len(p)
        return logits

    def capture(self):
        pass

    def step(self):
        self.steps += 1
        if self.fail_at is not None and self.steps >= self.fail_at:
            raise RuntimeError("GPU runtime error (cuda): injected")
        for b in range(self.B):
            self.ids.a[b] = self.nxt(self.ids.a[b], self.pos.a[b])
            self.pos.a[b] += 1


def expected(prompt, n, eos=None):
    out = [FakeSession.first(prompt)]
    pos = len(prompt)
    while len(out) < n and (eos is None or out[-1] != eos):
        out.append(FakeSession.nxt(out[-1], pos))
        pos += 1
    return list(prompt) + out


def test_concurrent_requests_share_slots():
    sched = BatchScheduler(lambda B, S: FakeSession(B, S), max_batch=3, max_seq=64)
    rng = np.random.default_rng(0)
    prompts = [rng.integers(0, V, int(rng.integers(1, 9))).tolist() for _ in range(10)]
    lengths = [int(rng.integers(1, 12)) for _ in prompts]
    results = [None] * len(prompts)

    def worker(i):
        results[i] = sched.generate(prompts[i], lengths[i]).tolist()

    threads = [threading.Thread(target=worker, args=(i,)) for i in range(len(prompts))]
    for t in threads:
        t.start()
    for t in threads:
        t.join(30)
    sched.close()
    for p, n, got in zip(prompts, lengths, results):
        assert got == expected(p, n)


def test_stream_eos_and_single_token():
    sched = BatchScheduler(lambda B, S: FakeSession(B, S), max_batch=2, max_seq=64)
    p = [3, 1, 4]
    full = expected(p, 10)
    eos = full[len(p) + 2]
    got = [t for t, _ in sched.submit(p, 10, eos_token_id=eos).stream()]
    assert got == expected(p, 10, eos)[len(p):]
    assert sched.generate([5], 1).tolist() == expected([5], 1)
    sched.close()


def test_rejects_and_failures():
    sched = BatchScheduler(lambda B, S: FakeSession(B, S, fail_at=3), max_batch=2, max_seq=16)
    with pytest.raises(ValueError):
        sched.submit([], 4)
    with pytest.raises(ValueError):
        sched.submit([1] * 10, 10)          # beyond max_seq
    r = sched.submit([1, 2], 8)
    with pytest.raises(RuntimeError):
        list(r.stream())                    # the step fails on its third call
    sched.close()
    with pytest.raises(RuntimeError):
        sched.submit([1], 2)

    def bad_factory(B, S):
        raise MemoryError("no room for the cache")

    with pytest.raises(MemoryError):
        BatchScheduler(bad_factory, max_batch=2, max_seq=16)


@pytest.mark.gpu
def test_batched_generation_equals_single_requests():
    import os
    import sys
    sys.path.insert(0, os.path.join(os.path.dirname(__file__), "golden"))
    import inputs
    from smollm2_triton import SmolLM2Config, SmolLM2ForCausalLM
    w = inputs.round_linear_weights_bf16(inputs.llama_weights(inputs.SMOL_TINY, 0))
    cfg = SmolLM2Config(**inputs.SMOL_TINY.config_kwargs())
    single = SmolLM2ForCausalLM(cfg, w, dtype="bfloat16")
    batched = SmolLM2ForCausalLM(cfg, w, dtype="bfloat16")
    batched.enable_batching(max_batch=3, max_seq=128)
    rng = np.random.default_rng(3)
    prompts = [rng.integers(0, 100, int(n)).tolist() for n in (1, 5, 9, 3, 12)]
    want = [single.generate_gpu(np.array([p], np.int32), 12, temperature=0.0)[0].tolist()
            for p in prompts]
    got = [None] * len(prompts)

    def worker(i):
        got[i] = batched.generate_gpu(np.array([prompts[i]], np.int32), 12,
                                      temperature=0.0)[0].tolist()

    ts = [threading.Thread(target=worker, args=(i,)) for i in range(len(prompts))]
    for t in ts:
        t.start()
    for t in ts:
        t.join(120)
    batched.disable_batching()
    assert got == want
