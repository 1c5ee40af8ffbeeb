"""Request state tracked by the scheduler and the runner."""
from __future__ import annotations

import enum
import time
from dataclasses import dataclass, field

from .sampling_params import SamplingParams


class RequestStatus(enum.Enum):
    WAITING = 0
    RUNNING = 1
    PREEMPTED = 2
    FINISHED_STOPPED = 3
    FINISHED_LENGTH = 4
    FINISHED_ABORTED = 5

    @property
    def finished(self) -> bool:
        return self.value >= 3


@dataclass
class Request:
    request_id: str
    prompt_token_ids: list[int]
    sampling_params: SamplingParams
    eos_token_id: int | None = None
    arrival_time: float = field(default_factory=time.perf_counter)
    prompt_embeds: object | None = None
    mm: object | None = None    # MultiModalInputs (images of a vision-language model)
    output_token_ids: list[int] = field(default_factory=list)
    output_logprobs: list[float] = field(default_factory=list)
    status: RequestStatus = RequestStatus.WAITING
    num_computed_tokens: int = 0
    num_cached_tokens: int = 0  # prefix-cache hits of the current admission
    num_pending: int = 0        # tokens sampled by launched steps whose results are not back yet
    slot: int = -1              # device slot holding this request's last sampled token
    block_ids: list[int] = field(default_factory=list)
    first_token_time: float | None = None
    finish_time: float | None = None
    token_times: list[float] = field(default_factory=list)
    stop_reason: str | None = None

    @property
    def num_prompt_tokens(self) -> int:
        return len(self.prompt_token_ids)

    @property
    def num_tokens(self) -> int:
        """Tokens known on the host (prompt + received outputs)."""
        return len(self.prompt_token_ids) + len(self.output_token_ids)

    @property
    def num_tokens_scheduled(self) -> int:
        """Tokens including those still being sampled by in-flight steps."""
        return len(self.prompt_token_ids) + len(self.output_token_ids) + self.num_pending

    def token_at(self, i: int) -> int:
        n = len(self.prompt_token_ids)
        return self.prompt_token_ids[i] if i < n else self.output_token_ids[i - n]

    def all_token_ids(self) -> list[int]:
        return self.prompt_token_ids + self.output_token_ids

    @property
    def max_tokens(self) -> int:
        mt = self.sampling_params.max_tokens
        return mt if mt is not None else 1 << 30

    def check_stop(self, max_model_len: int) -> bool:
        """Update status after a new token; returns True when the request finished."""
        sp = self.sampling_params
        n_out = len(self.output_token_ids)
        if n_out == 0:
            return False
        last = self.output_token_ids[-1]
        if n_out >= sp.min_tokens:
            if not sp.ignore_eos and self.eos_token_id is not None and last == self.eos_token_id:
                self.status, self.stop_reason = RequestStatus.FINISHED_STOPPED, "eos"
                return True
            if last in sp.stop_token_ids:
                self.status, self.stop_reason = RequestStatus.FINISHED_STOPPED, "stop"
                return True
        if n_out >= self.max_tokens or self.num_tokens >= max_model_len:
            self.status, self.stop_reason = RequestStatus.FINISHED_LENGTH, "length"
            return True
        return False
