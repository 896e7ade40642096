"""Continuous batching behind generate_gpu / generate_stream_gpu.

The reference server (scripts/serve_model.py:385-518) calls the model's
generate_gpu / generate_stream_gpu from worker threads, one request at a
time and without a lock. ``BatchScheduler`` lets those calls share the GPU:
each request takes a free sequence slot of one batched LlamaSession, its
prompt is prefilled into that slot, and one decode step (a CUDA graph
replay) advances every active request at once; tokens stream back to each
caller as they are produced, and a finished request frees its slot for the
next one. All GPU work runs on the scheduler's own thread.

Greedy decoding only (the reference's temperature sampling draws from the
host RNG in request order, which a shared batch cannot reproduce).
"""

from __future__ import annotations

import queue
import threading
import time
from dataclasses import dataclass, field

import numpy as np


@dataclass
class Request:
    prompt: np.ndarray
    max_new_tokens: int
    eos_token_id: int | None
    tokens: "queue.Queue" = field(default_factory=queue.Queue)   # (tok, dt) or None
    error: BaseException | None = None
    slot: int = -1
    produced: int = 0
    last: int = -1
    t_last: float = 0.0

    def stream(self):
        """Yield (token, seconds since the previous token) until done."""
        while True:
            item = self.tokens.get()
            if item is None:
                if self.error is not None:
                    raise self.error
                return
            yield item


class BatchScheduler:
    """Serve greedy requests from any thread on ``max_batch`` shared slots.

    ``session_factory(batch, max_seq)`` builds the session (a LlamaSession
    or a stand-in with ``prefill(prompts, slots=...)``, ``step()``,
    ``capture()``, and ``ids`` / ``pos`` device arrays with ``to_numpy`` /
    ``from_numpy``).
    """

    def __init__(self, session_factory, max_batch: int, max_seq: int,
                 use_graph: bool = True, idle_wait: float = 0.05):
        self.B, self.S = int(max_batch), int(max_seq)
        self._factory = session_factory
        self._use_graph = use_graph
        self._idle = idle_wait
        self._waiting: "queue.Queue[Request]" = queue.Queue()
        self._pending: list[Request] = []     # taken off the queue, not admitted
        self._active: dict[int, Request] = {}
        self._stop = threading.Event()
        self._lock = threading.Lock()     # submit vs close
        self._thread = threading.Thread(target=self._run, name="tllm-batch", daemon=True)
        self._session = None
        self._started = threading.Event()
        self._start_error: BaseException | None = None
        self._thread.start()
        self._started.wait()
        if self._start_error is not None:
            raise self._start_error

    # ---- client side -------------------------------------------------
    def submit(self, prompt, max_new_tokens: int, eos_token_id: int | None = None) -> Request:
        prompt = np.asarray(prompt, np.int32).reshape(-1)
        if prompt.size == 0:
            raise ValueError("the prompt needs at least one token")
        if max_new_tokens < 1:
            raise ValueError("max_new_tokens must be >= 1")
        if prompt.size + max_new_tokens > self.S:
            raise ValueError(f"{prompt.size} + {max_new_tokens} tokens exceed the "
                             f"scheduler's {self.S} positions")
        r = Request(prompt, int(max_new_tokens), eos_token_id)
        with self._lock:
            if self._stop.is_set():
                raise RuntimeError("the batch scheduler is closed")
            self._waiting.put(r)
        return r

    def generate(self, prompt, max_new_tokens: int, eos_token_id: int | None = None):
        """Prompt + generated tokens (int32), blocking."""
        r = self.submit(prompt, max_new_tokens, eos_token_id)
        toks = [t for t, _ in r.stream()]
        return np.concatenate([r.prompt, np.array(toks, np.int32)])

    def close(self):
        """Stop the loop; requests not finished yet end with an error."""
        with self._lock:
            self._stop.set()
        self._thread.join()

    # ---- scheduler thread ----------------------------------------------
    def _run(self):
        try:
            self._session = self._factory(self.B, self.S)
        except BaseException as e:   # noqa: BLE001 -- reported to the creator
            self._start_error = e
            self._started.set()
            return
        self._started.set()
        s = self._session
        graph = False
        pos = np.zeros(self.B, np.int32)
        while not self._stop.is_set():
            try:
                self._admit(pos)
                if not self._active:
                    try:   # idle: sleep until a request arrives
                        self._pending.append(self._waiting.get(timeout=self._idle))
                    except queue.Empty:
                        pass
                    continue
                if self._use_graph and not graph:
                    s.capture()
                    graph = True
                # free slots keep position 0 (their writes land in slots
                # that are prefilled again before use)
                s.pos.from_numpy(pos)
                s.lens.from_numpy(pos)
                s.step()
                ids = s.ids.to_numpy()
                now = time.perf_counter()
                for slot, r in list(self._active.items()):
                    pos[slot] += 1
                    self._deliver(r, int(ids[slot]), now)
                    if self._finished(r):
                        self._release(r, pos)
            except BaseException as e:   # noqa: BLE001 -- fail every request
                self._fail_all(e)
                graph = False
        self._fail_all(RuntimeError("the batch scheduler was closed"))

    def _admit(self, pos):
        free = [b for b in range(self.B) if b not in self._active]
        while len(self._pending) < len(free):
            try:
                self._pending.append(self._waiting.get_nowait())
            except queue.Empty:
                break
        batch, self._pending = self._pending[:len(free)], self._pending[len(free):]
        if not batch:
            return
        slots = free[:len(batch)]
        s = self._session
        logits = s.prefill([r.prompt for r in batch], slots=slots)
        now = time.perf_counter()
        for r, slot, lg in zip(batch, slots, logits):
            r.slot = slot
            r.t_last = now
            self._active[slot] = r
            pos[slot] = len(r.prompt)
            self._deliver(r, int(np.argmax(lg)), now)
            if self._finished(r):
                self._release(r, pos)

    def _deliver(self, r: Request, tok: int, now: float):
        r.tokens.put((tok, now - r.t_last))
        r.t_last = now
        r.produced += 1
        r.last = tok

    def _finished(self, r: Request) -> bool:
        return r.produced >= r.max_new_tokens or (
            r.eos_token_id is not None and r.last == r.eos_token_id)

    def _release(self, r: Request, pos):
        self._active.pop(r.slot, None)
        pos[r.slot] = 0
        r.tokens.put(None)

    def _fail_all(self, e: BaseException):
        for r in list(self._active.values()) + self._pending:
            r.error = e
            r.tokens.put(None)
        self._active.clear()
        self._pending = []
        while True:
            try:
                r = self._waiting.get_nowait()
            except queue.Empty:
                break
            r.error = e
            r.tokens.put(None)
