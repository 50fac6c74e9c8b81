"""Continuous-batching generation on top of the multi-session runtime.

The reference serves one request at a time: `InferenceSession::infer_batch`
(woolly-core/src/session.rs:260-277) loops over its sequences and the server's
decode loop (woolly-server/src/handlers/inference.rs:371-438) calls
`InferenceEngine::infer` once per generated token, re-reading one shared KV
cache.  Here every request owns a session (its own paged KV cache on the
GPU); `BatchEngine.step()` admits waiting requests, prefills them, and then
runs ONE batched decode forward over every running request, so requests join
and leave the batch between steps (continuous batching).

Sampling follows the server's `sample_next_token` (inference.rs:441-483) and
its helpers (softmax_with_temperature, apply_top_k_filtering,
apply_top_p_filtering: inference.rs:551-630): temperature floor 0.01, top-k
by the k-th largest probability, top-p by the first prefix whose cumulative
probability exceeds p, greedy (temperature == 0) as the last index of the
largest probability, and a stop on token ids below 3 (inference.rs:414-418).
"""
from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np

from ._lib import WL_ERR_OUT_OF_MEMORY, WoollyError


@dataclass
class GenerationConfig:
    """The server's generation knobs (inference.rs:25-27, 180-182)."""
    max_tokens: int = 16
    temperature: float = 0.0   # 0: greedy
    top_k: int = 0             # 0: off
    top_p: float = 1.0         # 1: off
    eos_below: int = 3         # stop once a token id < eos_below is produced (0: never)
    seed: int = 0              # per-request sampling stream


def softmax_with_temperature(logits: np.ndarray, temperature: float) -> np.ndarray:
    """inference.rs:551-565 (f32, max-subtracted)."""
    t = np.float32(max(temperature, 0.01))
    x = np.asarray(logits, np.float32)
    e = np.exp((x - x.max()) / t).astype(np.float32)
    return (e / e.sum(dtype=np.float32)).astype(np.float32)


def apply_top_k(probs: np.ndarray, k: int) -> np.ndarray:
    """inference.rs:568-591: zero probabilities below the k-th largest, renormalise."""
    if k == 0 or k >= probs.size:
        return probs
    thr = np.sort(probs)[::-1][k - 1]
    p = np.where(probs < thr, np.float32(0), probs).astype(np.float32)
    s = p.sum(dtype=np.float32)
    return (p / s).astype(np.float32) if s > 0 else p


def apply_top_p(probs: np.ndarray, top_p: float) -> np.ndarray:
    """inference.rs:594-630: keep the shortest prefix (by descending
    probability) whose cumulative sum exceeds p; when no prefix exceeds p the
    reference keeps nothing (all zeros), and so does this."""
    if top_p >= 1.0:
        return probs
    order = np.argsort(-probs, kind="stable")
    cum = np.float32(0)
    cut = 0
    for i, idx in enumerate(order):
        cum = np.float32(cum + probs[idx])
        if cum > top_p:
            cut = i + 1
            break
    p = np.zeros_like(probs)
    keep = order[:cut]
    p[keep] = probs[keep]
    s = p.sum(dtype=np.float32)
    return (p / s).astype(np.float32) if s > 0 else p


def sample_next_token(logits: np.ndarray, cfg: GenerationConfig, rng: np.random.Generator) -> int:
    """sample_next_token (inference.rs:441-483) on one row of logits."""
    probs = softmax_with_temperature(logits, cfg.temperature)
    if cfg.top_k > 0:
        probs = apply_top_k(probs, cfg.top_k)
    if cfg.top_p < 1.0:
        probs = apply_top_p(probs, cfg.top_p)
    if cfg.temperature == 0.0:
        m = probs.max()
        return int(np.flatnonzero(probs == m)[-1])  # Rust max_by keeps the last maximum
    return sample_from_distribution(probs, rng)


def sample_from_distribution(probs: np.ndarray, rng: np.random.Generator) -> int:
    """inference.rs:638-654: first index whose f32 running sum exceeds a
    uniform draw in [0, 1); the last index when none does (e.g. all zeros)."""
    u = np.float32(rng.random(dtype=np.float32))
    cum = np.cumsum(probs, dtype=np.float32)
    hit = np.flatnonzero(cum > u)
    return int(hit[0]) if hit.size else probs.size - 1


@dataclass
class Request:
    rid: int
    prompt: list
    cfg: GenerationConfig
    rng: np.random.Generator
    tokens: list = field(default_factory=list)
    logits: list = field(default_factory=list)
    session: object = None
    done: bool = False
    reason: str = ""
    on_token: object = None  # callable(rid, token, done, reason) per produced token


class BatchEngine:
    """Continuous batching over a CudaTransformer (or any object with the same
    `forward_sessions` / `vocab_size` / `max_batch` interface).

    submit() queues a request; step() admits queued requests while sessions
    and batch room allow (each prefilled on its own, which yields its first
    token), then decodes one token for every other running request in one
    batched forward; run() steps until every request has finished.  A request
    finishes after cfg.max_tokens tokens, on a token id below cfg.eos_below,
    or when its session's context is full.  Its session is released at once,
    so a waiting request can take the slot on the next step.
    """

    def __init__(self, model, max_batch: int | None = None, session_factory=None,
                 max_context: int | None = None, keep_logits: bool = False,
                 device_sampling: bool = False):
        self.model = model
        self.max_batch = max_batch or model.max_batch
        if session_factory is None:
            from .model import Session
            session_factory = lambda: Session(model)  # noqa: E731
        self.new_session = session_factory
        self.max_context = max_context or getattr(model, "max_context", None)
        self.keep_logits = keep_logits
        # decode steps sample on the GPU (CudaTransformer.decode_sample): only
        # token ids cross to the host; the uniform draws still come from each
        # request's own stream, in the same order as host sampling
        self.device_sampling = device_sampling and not keep_logits and hasattr(model, "decode_sample")
        self.waiting: list[Request] = []
        self.running: list[Request] = []
        self.finished: dict[int, Request] = {}
        self._next = 0

    def submit(self, prompt, cfg: GenerationConfig | None = None, on_token=None) -> int:
        """Queues a request; `on_token(rid, token, done, reason)`, if given, is
        called as each of its tokens is produced (the server's streaming
        responses, inference.rs:271-357, forward tokens this way)."""
        prompt = [int(t) for t in prompt]
        if not prompt:
            raise ValueError("empty prompt (the reference's EMPTY_INPUT)")
        cfg = cfg or GenerationConfig()
        r = Request(self._next, prompt, cfg, np.random.default_rng(cfg.seed), on_token=on_token)
        self._next += 1
        self.waiting.append(r)
        return r.rid

    # ---------------------------------------------------------------- internals
    def _emit(self, r: Request, row: np.ndarray) -> None:
        tok = sample_next_token(row, r.cfg, r.rng)
        if self.keep_logits:
            r.logits.append(np.array(row, np.float32, copy=True))
        self._emit_token(r, tok)

    def _emit_token(self, r: Request, tok: int) -> None:
        r.tokens.append(int(tok))
        if len(r.tokens) >= r.cfg.max_tokens:
            r.done, r.reason = True, "length"
        elif r.cfg.eos_below and tok < r.cfg.eos_below:
            r.done, r.reason = True, "eos"
        elif self.max_context is not None and len(r.session) + 1 > self.max_context:
            r.done, r.reason = True, "context"
        if r.on_token is not None:
            r.on_token(r.rid, int(tok), r.done, r.reason)

    def _retire(self) -> None:
        keep = []
        for r in self.running:
            if r.done:
                r.session.close()
                r.session = None
                self.finished[r.rid] = r
            else:
                keep.append(r)
        self.running = keep

    def _admit(self) -> list[Request]:
        new = []
        while self.waiting and len(self.running) + len(new) < self.max_batch:
            r = self.waiting[0]
            if self.max_context is not None and len(r.prompt) >= self.max_context:
                self.waiting.pop(0)
                r.done, r.reason = True, "context"
                self.finished[r.rid] = r
                continue
            try:
                r.session = self.new_session()
            except WoollyError as e:
                if e.code == WL_ERR_OUT_OF_MEMORY:  # every session slot is taken
                    break
                raise
            self.waiting.pop(0)
            new.append(r)
        return new

    # ---------------------------------------------------------------- public
    def step(self) -> int:
        """One scheduler iteration; returns the number of tokens produced."""
        produced = 0
        decoding = [r for r in self.running if not r.done]
        new = self._admit()
        for r in new:  # prefill: the prompt's last row gives the first token
            row = self.model.forward_sessions([r.session], [r.prompt])[0]
            self._emit(r, np.asarray(row).reshape(-1)[-self.model.vocab_size():])
            produced += 1
        if decoding and self.device_sampling:
            cf = [r.cfg for r in decoding]
            u = [np.float32(r.rng.random(dtype=np.float32)) if r.cfg.temperature != 0.0 else 0.0
                 for r in decoding]
            toks = self.model.decode_sample([r.session for r in decoding],
                                            [r.tokens[-1] for r in decoding],
                                            [c.temperature for c in cf], [c.top_k for c in cf],
                                            [c.top_p for c in cf], u)
            for r, tok in zip(decoding, toks):
                self._emit_token(r, tok)
                produced += 1
        elif decoding:
            outs = self.model.forward_sessions([r.session for r in decoding],
                                               [[r.tokens[-1]] for r in decoding])
            for r, row in zip(decoding, outs):
                self._emit(r, np.asarray(row).reshape(-1))
                produced += 1
        self.running += new
        self._retire()
        return produced

    def idle(self) -> bool:
        return not self.waiting and not self.running

    def run(self, max_steps: int = 1_000_000) -> dict[int, list]:
        for _ in range(max_steps):
            if self.idle():
                break
            self.step()
        return {rid: r.tokens for rid, r in sorted(self.finished.items())}

    def stream(self, prompt, cfg: GenerationConfig | None = None):
        """Submits a request and yields its tokens as they are produced,
        stepping the whole engine (other requests advance in the same batched
        steps)."""
        got: list = []
        rid = self.submit(prompt, cfg, on_token=lambda _r, tok, _d, _why: got.append(tok))
        while rid not in self.finished:
            self.step()
            while got:
                yield got.pop(0)
        while got:
            yield got.pop(0)

    def close(self) -> None:
        for r in self.running:
            if r.session is not None:
                r.session.close()
                r.session = None
        self.running = []
