"""Continuous-batching scheduler with lightserve's policy and API
(``engine/scheduler.py:82-247``), feeding this package's model runner.

Per ``schedule()`` call:

* running requests first, in their order: each needs one new token's KV
  (``get_num_new_tokens``); when its next token needs a block and none is
  free, the lowest-priority running request not yet decided this step is
  preempted (``:141-149``) -- itself if it is the last one;
* then, only when nothing was preempted this step (``:110-115``), waiting
  requests in FIFO order while the sequence cap, the token budget and
  ``BlockManager.can_allocate`` allow; the first one that does not fit stops
  the scan (head-of-line blocking, ``:175-181``);
* preemption is by recompute (``:187-203``): blocks freed, computed-token
  count reset, status PREEMPTED, requeued at the FRONT of ``waiting``, so its
  next admission is a prefill over prompt + tokens generated so far.

Like the reference, ``schedule()`` commits its decision (block tables and
``num_computed_tokens`` advance before the forward pass runs).
"""
from __future__ import annotations

from collections import deque
from dataclasses import dataclass, field

from .block_manager import BlockManager
from .config import CacheConfig, SchedulerConfig
from .request import Request, RequestStatus


@dataclass
class ScheduledRequest:
    """One request's share of a step: ``num_scheduled_tokens`` > 1 is a prefill
    (the whole sequence so far), 1 is a decode step."""
    request: Request
    num_scheduled_tokens: int


@dataclass
class SchedulerOutput:
    scheduled_new: list = field(default_factory=list)      # admitted this step (prefill)
    scheduled_running: list = field(default_factory=list)  # already running (decode)
    preempted: list = field(default_factory=list)          # bumped back to waiting this step

    @property
    def is_empty(self) -> bool:
        return not self.scheduled_new and not self.scheduled_running

    @property
    def total_num_scheduled_tokens(self) -> int:
        return sum(s.num_scheduled_tokens for s in self.scheduled_new + self.scheduled_running)


class Scheduler:
    def __init__(self, cache_config: CacheConfig, scheduler_config: SchedulerConfig):
        self.cache_config = cache_config
        self.scheduler_config = scheduler_config
        self.block_manager = BlockManager(block_size=cache_config.block_size,
                                          num_gpu_blocks=cache_config.num_gpu_blocks,
                                          watermark_blocks=cache_config.watermark_blocks)
        self.waiting: deque = deque()
        self.running: list = []
        self.requests: dict = {}

    # ------------------------------------------------------------- intake --
    def add_request(self, request: Request) -> None:
        if request.request_id in self.requests:
            raise ValueError(f"duplicate request_id {request.request_id!r}")
        request.status = RequestStatus.WAITING
        self.requests[request.request_id] = request
        self.waiting.append(request)

    def get_num_unfinished_requests(self) -> int:
        return len(self.waiting) + len(self.running)

    def has_unfinished_requests(self) -> bool:
        return bool(self.waiting or self.running)

    # ----------------------------------------------------------- decision --
    def schedule(self) -> SchedulerOutput:
        out = SchedulerOutput()
        budget = self._schedule_running(out, self.scheduler_config.max_num_batched_tokens)
        if not out.preempted:
            self._schedule_waiting(out, budget)
        return out

    def _schedule_running(self, out: SchedulerOutput, budget: int) -> int:
        undecided = deque(self.running)
        kept = []
        while undecided:
            req = undecided.popleft()
            n = req.get_num_new_tokens()
            if n <= 0 or n > budget:
                kept.append(req)  # nothing to compute, or over budget: stays running, retried next step
                continue
            victim_is_self = False
            while not self.block_manager.can_append_slot(req):
                if undecided:
                    self._preempt(undecided.pop(), out)
                else:
                    self._preempt(req, out)
                    victim_is_self = True
                    break
            if victim_is_self:
                continue
            self.block_manager.append_slot(req)
            req.num_computed_tokens = req.get_len()
            out.scheduled_running.append(ScheduledRequest(req, n))
            budget -= n
            kept.append(req)
        self.running = kept
        return budget

    def _schedule_waiting(self, out: SchedulerOutput, budget: int) -> int:
        while self.waiting:
            req = self.waiting[0]
            n = req.get_num_new_tokens()
            if (len(self.running) >= self.scheduler_config.max_num_seqs or n > budget
                    or not self.block_manager.can_allocate(req)):
                break  # FIFO: nothing behind the head of the line goes first
            self.waiting.popleft()
            self.block_manager.allocate(req)
            req.status = RequestStatus.RUNNING
            req.num_computed_tokens = req.get_len()
            out.scheduled_new.append(ScheduledRequest(req, n))
            budget -= n
            self.running.append(req)
        return budget

    def _preempt(self, req: Request, out: SchedulerOutput) -> None:
        self.block_manager.free(req)
        req.num_computed_tokens = 0
        req.status = RequestStatus.PREEMPTED
        self.waiting.appendleft(req)
        out.preempted.append(req)

    # ----------------------------------------------------------- teardown --
    def free_finished_requests(self) -> list:
        """Releases the blocks of running requests marked finished
        (``Request.maybe_finish``); returns them."""
        done = [r for r in self.running if r.is_finished()]
        if done:
            self.running = [r for r in self.running if not r.is_finished()]
            for r in done:
                self.block_manager.free(r)
                del self.requests[r.request_id]
        return done

    def abort_requests(self, request_ids) -> list:
        """Cancels waiting or running requests (unknown ids are ignored);
        returns the newly aborted ones."""
        ids = set(request_ids)
        aborted = [r for r in self.waiting if r.request_id in ids]
        for r in aborted:
            r.status = RequestStatus.FINISHED_ABORTED
            del self.requests[r.request_id]
        self.waiting = deque(r for r in self.waiting if r.request_id not in ids)
        for r in self.running:
            if r.request_id in ids:
                r.status = RequestStatus.FINISHED_ABORTED
        return aborted + self.free_finished_requests()
