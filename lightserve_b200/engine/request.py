"""Request state, the subset of lightserve's ``engine/request.py:48-117`` the
block manager and decode runner use: prompt/output token lists, status, the
block table, and ``num_blocks_needed = ceil(len / block_size)`` (``:95-99``).
"""
from __future__ import annotations

from dataclasses import dataclass, field
from enum import Enum, auto
from typing import Optional


class RequestStatus(Enum):
    WAITING = auto()
    RUNNING = auto()
    PREEMPTED = auto()
    FINISHED_STOPPED = auto()
    FINISHED_LENGTH_CAPPED = auto()
    FINISHED_ABORTED = auto()

    @property
    def finished(self) -> bool:
        return self.name.startswith("FINISHED")


@dataclass
class SamplingParams:
    max_tokens: int = 16
    eos_token_id: Optional[int] = None


@dataclass
class Request:
    request_id: str
    prompt_token_ids: list
    sampling_params: SamplingParams = field(default_factory=SamplingParams)
    arrival_time: float = 0.0
    output_token_ids: list = field(default_factory=list)
    status: RequestStatus = RequestStatus.WAITING
    block_table: list = field(default_factory=list)
    num_computed_tokens: int = 0

    def all_token_ids(self) -> list:
        return list(self.prompt_token_ids) + list(self.output_token_ids)

    def get_len(self) -> int:
        return len(self.prompt_token_ids) + len(self.output_token_ids)

    def get_num_new_tokens(self) -> int:
        return self.get_len() - self.num_computed_tokens

    def is_prefill(self) -> bool:
        return self.num_computed_tokens < len(self.prompt_token_ids)

    def num_blocks_needed(self, block_size: int) -> int:
        return -(-self.get_len() // block_size)

    def is_finished(self) -> bool:
        return self.status.finished

    def maybe_finish(self) -> None:
        if self.status.finished:
            return
        eos = self.sampling_params.eos_token_id
        if eos is not None and self.output_token_ids and self.output_token_ids[-1] == eos:
            self.status = RequestStatus.FINISHED_STOPPED
        elif len(self.output_token_ids) >= self.sampling_params.max_tokens:
            self.status = RequestStatus.FINISHED_LENGTH_CAPPED
