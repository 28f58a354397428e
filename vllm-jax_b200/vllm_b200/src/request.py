"""Request state (vllm/src/request.py:8-37 of vllm-jax).

Ids come from one process-wide counter, as in the reference; `slot` is this
build's index of the request's rows in the device-resident token and block
tables (assigned by the engine)."""
from __future__ import annotations

import itertools
from copy import copy
from enum import Enum, auto

from ..sampling_params import SamplingParams


class Status(Enum):
    WAITING = auto()
    RUNNING = auto()
    FINISHED = auto()


class Request:
    counter = itertools.count()

    def __init__(self, token_ids: list[int], sampling_params: SamplingParams,
                 eos_token_id: int | None):
        self.id = next(Request.counter)
        self.status = Status.WAITING
        self.sampling_params = sampling_params
        self.ignore_eos = sampling_params.ignore_eos
        self.max_new_tokens = sampling_params.max_new_tokens
        self.eos_token_id = eos_token_id
        self.token_ids = copy(list(token_ids))
        self.num_prompt_tokens = len(token_ids)
        self.num_completion_tokens = 0
        self.slot = -1
        self.num_computed_tokens = 0   # chunked mode: positions whose KV is cached
        # sampling stream: Philox key (seed, stream id); the engine sets the
        # stream id to the request's index in its generate() call
        self.sample_stream = self.id

    def is_finished(self) -> bool:
        return self.status == Status.FINISHED

    def get_last_token_id(self) -> int:
        return self.token_ids[-1]

    def __len__(self) -> int:
        return self.num_prompt_tokens + self.num_completion_tokens

    @classmethod
    def reset_ids(cls) -> None:
        """Restart the id counter (tests replaying a reference trace)."""
        cls.counter = itertools.count()
