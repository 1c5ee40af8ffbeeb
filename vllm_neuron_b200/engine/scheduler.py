"""Continuous-batching scheduler with chunked prefill over the paged block manager.

Policy (per step, token budget ``max_num_batched_tokens``):
  1. running requests first, in admission order: a decode needs one token, a partially
     prefilled prompt gets its next chunk; if blocks run out, the most recently admitted
     running request is preempted (blocks freed, recomputed later);
  2. then waiting requests FCFS while the budget, ``max_num_seqs`` and free blocks allow,
     reusing cached prefix blocks when prefix caching is on.

Prefill chunks and decodes share one batch (the B200 runner handles mixed batches in one
forward).  The reference forbids mixing and allows one prefill per batch
(vllm_neuron/vllm/core/scheduler.py:203,774-780); ``mixed_batches=False`` reproduces that
behaviour for API parity.  Bucket padding statistics for ``num_batched_tokens_buckets`` /
``num_seqs_buckets`` are recorded as metrics (reference: scheduler.py:618-792).
"""
from __future__ import annotations

from collections import deque
from dataclasses import dataclass, field

from ..utils.buckets import bucket_for  # noqa: F401 (re-exported)
from .block_manager import BlockManager
from .request import Request, RequestStatus


@dataclass
class ScheduledRequest:
    req: Request
    start: int          # first token position computed this step
    num_tokens: int     # tokens computed this step
    samples: bool       # reaches the end of the known tokens -> produces a new token
    spec: list = field(default_factory=list)  # draft tokens verified this step (after the last token)

    @property
    def num_logits(self) -> int:
        """Logits rows this request needs: one per verified draft plus one, or one."""
        if not self.samples:
            return 0
        return len(self.spec) + 1 if self.spec else 1


@dataclass
class SchedulerOutput:
    scheduled: list[ScheduledRequest] = field(default_factory=list)
    num_tokens: int = 0
    preempted: list[str] = field(default_factory=list)
    padded_tokens: int = 0
    padded_seqs: int = 0

    @property
    def is_pure_decode(self) -> bool:
        return bool(self.scheduled) and all(s.num_tokens == 1 for s in self.scheduled)

    @property
    def empty(self) -> bool:
        return not self.scheduled


class Scheduler:
    def __init__(self, block_manager: BlockManager, max_num_seqs: int, max_num_batched_tokens: int,
                 max_model_len: int, enable_chunked_prefill: bool = True, mixed_batches: bool = True,
                 num_batched_tokens_buckets: list[int] | None = None,
                 num_seqs_buckets: list[int] | None = None, metrics=None):
        self.bm = block_manager
        self.max_num_seqs = max_num_seqs
        self.max_num_batched_tokens = max_num_batched_tokens
        self.max_model_len = max_model_len
        self.enable_chunked_prefill = enable_chunked_prefill
        self.mixed_batches = mixed_batches
        self.tok_buckets = num_batched_tokens_buckets
        self.seq_buckets = num_seqs_buckets
        self.metrics = metrics
        self.waiting: deque[Request] = deque()
        self.running: list[Request] = []
        self.requests: dict[str, Request] = {}

    # --------------------------------------------------------------------- queue ops
    def add_request(self, req: Request):
        if req.num_prompt_tokens >= self.max_model_len:
            raise ValueError(f"prompt of {req.num_prompt_tokens} tokens does not fit max_model_len "
                             f"{self.max_model_len}")
        self.requests[req.request_id] = req
        self.waiting.append(req)

    def abort_request(self, request_id: str):
        req = self.requests.pop(request_id, None)
        if req is None:
            return
        if req in self.running:
            self.running.remove(req)
        elif req in self.waiting:
            self.waiting.remove(req)
        self.bm.free_request(req)
        req.status = RequestStatus.FINISHED_ABORTED

    def finish_request(self, req: Request, status: RequestStatus, now: float | None = None):
        """Finish a running request outside the token stop checks (e.g. a completed grammar)."""
        req.status = status
        req.finish_time = now
        if req in self.running:
            self.running.remove(req)
        self.bm.free_request(req)
        self.requests.pop(req.request_id, None)

    def has_unfinished(self) -> bool:
        return bool(self.waiting or self.running)

    def _preempt(self, req: Request, out: SchedulerOutput):
        self.bm.free_request(req)
        req.num_computed_tokens = 0
        req.status = RequestStatus.PREEMPTED
        self.waiting.appendleft(req)
        out.preempted.append(req.request_id)

    # --------------------------------------------------------------------- schedule
    def schedule(self) -> SchedulerOutput:
        out = SchedulerOutput()
        budget = self.max_num_batched_tokens
        scheduled_ids = set()
        has_decode = has_prefill = False
        i = 0
        while i < len(self.running) and budget > 0:
            req = self.running[i]
            n = req.num_tokens_scheduled - req.num_computed_tokens
            if n <= 0 or len(req.output_token_ids) + req.num_pending >= req.max_tokens:
                # nothing to compute, or its last token is already being sampled
                i += 1
                continue
            is_prefill = n > 1 or req.num_computed_tokens < req.num_prompt_tokens
            if not self.mixed_batches and ((is_prefill and has_decode) or (not is_prefill and has_prefill)
                                           or (is_prefill and has_prefill)):
                i += 1
                continue
            n = min(n, budget)
            if n < req.num_tokens_scheduled - req.num_computed_tokens and not self.enable_chunked_prefill:
                i += 1
                continue
            spec = []
            if n == 1 and getattr(req, "spec_token_ids", None):
                room = min(budget - 1, self.max_model_len - req.num_tokens - 1,
                           req.max_tokens - len(req.output_token_ids) - 1)
                spec = list(req.spec_token_ids[:max(0, room)])
                n += len(spec)
            ok = True
            while not self.bm.allocate(req, req.num_computed_tokens + n):
                victim = self.running.pop()
                self._preempt(victim, out)
                if victim is req:
                    ok = False
                    break
            if not ok:
                break
            out.scheduled.append(ScheduledRequest(req, req.num_computed_tokens, n,
                                                  req.num_computed_tokens + n >= req.num_tokens_scheduled,
                                                  spec))
            scheduled_ids.add(req.request_id)
            budget -= n
            has_prefill |= is_prefill
            has_decode |= not is_prefill
            i += 1
        if not out.preempted:
            while self.waiting and budget > 0 and len(self.running) < self.max_num_seqs:
                if not self.mixed_batches and (has_decode or has_prefill):
                    break
                req = self.waiting[0]
                if req.num_pending:
                    break  # a preempted request whose last token is still in flight
                if not req.block_ids:
                    cached = self.bm.match_prefix(req)
                    req.num_computed_tokens = cached
                    req.num_cached_tokens = cached
                n = req.num_tokens - req.num_computed_tokens
                if n > budget and not self.enable_chunked_prefill:
                    break
                n = min(n, budget)
                if not self.bm.allocate(req, req.num_computed_tokens + n):
                    if req.num_cached_tokens:
                        self.bm.free_request(req)
                        req.num_computed_tokens = 0
                        req.num_cached_tokens = 0
                    break
                self.waiting.popleft()
                req.status = RequestStatus.RUNNING
                self.running.append(req)
                out.scheduled.append(ScheduledRequest(req, req.num_computed_tokens, n,
                                                      req.num_computed_tokens + n >= req.num_tokens_scheduled))
                budget -= n
                has_prefill = True
        # The KV of scheduled tokens is written by this step, and sampling rows add a
        # placeholder token until their result comes back (asynchronous scheduling).
        for sr in out.scheduled:
            sr.req.num_computed_tokens = sr.start + sr.num_tokens
            if sr.samples:
                sr.req.num_pending += 1
        out.num_tokens = sum(s.num_tokens for s in out.scheduled)
        out.padded_tokens = bucket_for(self.tok_buckets, out.num_tokens)
        out.padded_seqs = bucket_for(self.seq_buckets, len(out.scheduled))
        if self.metrics is not None and out.scheduled:
            self.metrics.observe_padding(out.num_tokens, out.padded_tokens, len(out.scheduled), out.padded_seqs)
        return out

    # --------------------------------------------------------------------- update
    def update_spec(self, out: SchedulerOutput, tokens: list[list[int]],
                    now: float | None = None) -> list[Request]:
        """Apply a speculative step: ``tokens[i]`` are the accepted tokens (1..k+1) of the
        i-th sampling request.  The KV of rejected drafts is dropped by rolling back
        ``num_computed_tokens`` (their slots are rewritten by later steps)."""
        finished = []
        k = 0
        for s in out.scheduled:
            req = s.req
            if not s.samples:
                if not req.status.finished:
                    self.bm.commit_full_blocks(req)
                continue
            toks = tokens[k]
            k += 1
            req.num_pending -= 1
            if req.status.finished:
                continue
            if s.spec:
                req.num_computed_tokens = s.start + len(toks)
                req.spec_accepted = getattr(req, "spec_accepted", 0) + len(toks) - 1
                req.spec_proposed = getattr(req, "spec_proposed", 0) + len(s.spec)
            for tok in toks:
                req.output_token_ids.append(int(tok))
                if now is not None:
                    if req.first_token_time is None:
                        req.first_token_time = now
                    req.token_times.append(now)
                if req.check_stop(self.max_model_len):
                    req.finish_time = now
                    finished.append(req)
                    break
            self.bm.commit_full_blocks(req)
        for req in finished:
            if req in self.running:
                self.running.remove(req)
            req.freed_block_ids = list(req.block_ids)  # KV hand-off (disaggregated prefill)
            self.bm.free_request(req)
            self.requests.pop(req.request_id, None)
        return finished

    def update(self, out: SchedulerOutput, sampled: list[int], logprobs: list[float] | None = None,
               now: float | None = None) -> list[Request]:
        """Apply one step's results; returns the requests that finished."""
        finished = []
        k = 0
        for s in out.scheduled:
            req = s.req
            if not s.samples:
                if not req.status.finished:
                    self.bm.commit_full_blocks(req)
                continue
            tok = int(sampled[k])
            lp = float(logprobs[k]) if logprobs is not None else None
            k += 1
            req.num_pending -= 1
            if req.status.finished:
                continue  # stopped by an earlier token; this one was computed speculatively
            if lp is not None:
                req.output_logprobs.append(lp)
            req.output_token_ids.append(tok)
            self.bm.commit_full_blocks(req)
            if now is not None:
                if req.first_token_time is None:
                    req.first_token_time = now
                req.token_times.append(now)
            if req.check_stop(self.max_model_len):
                req.finish_time = now
                finished.append(req)
        for req in finished:
            if req in self.running:
                self.running.remove(req)
            req.freed_block_ids = list(req.block_ids)  # KV hand-off (disaggregated prefill)
            self.bm.free_request(req)
            self.requests.pop(req.request_id, None)
        return finished
