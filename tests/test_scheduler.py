"""Continuous-batching scheduler: the policy of lightserve's
engine/scheduler.py (its engine/tests/test_scheduler.py scenarios), on CPU."""
import pytest

from lightserve_b200.engine import (CacheConfig, Request, RequestStatus, SamplingParams, Scheduler,
                                    SchedulerConfig)


def _sched(blocks=64, seqs=8, tokens=4096, bs=4, watermark=0):
    return Scheduler(CacheConfig(block_size=bs, num_gpu_blocks=blocks, watermark_blocks=watermark),
                     SchedulerConfig(max_num_seqs=seqs, max_num_batched_tokens=tokens))


def _req(i, n, max_tokens=16, eos=None):
    return Request(f"r{i}", list(range(1, n + 1)), SamplingParams(max_tokens=max_tokens, eos_token_id=eos))


def _emit(req, tok=7):
    """What the model runner does after a forward: append the sampled token."""
    req.output_token_ids.append(tok)
    req.maybe_finish()


def test_new_request_waits():
    s = _sched()
    r = _req(0, 5)
    s.add_request(r)
    assert list(s.waiting) == [r] and s.running == [] and r.status == RequestStatus.WAITING
    assert s.has_unfinished_requests() and s.get_num_unfinished_requests() == 1


def test_duplicate_id_rejected():
    s = _sched()
    s.add_request(_req(0, 3))
    with pytest.raises(ValueError):
        s.add_request(_req(0, 4))


def test_admission_is_a_whole_prompt_prefill():
    s = _sched()
    r = _req(0, 10)
    s.add_request(r)
    out = s.schedule()
    assert [x.request for x in out.scheduled_new] == [r] and out.scheduled_new[0].num_scheduled_tokens == 10
    assert r.status == RequestStatus.RUNNING and r.num_computed_tokens == 10
    assert len(s.block_manager.get_block_table(r)) == 3 and out.total_num_scheduled_tokens == 10


def test_fifo_order_and_sequence_cap():
    s = _sched(seqs=2)
    rs = [_req(i, 3) for i in range(3)]
    for r in rs:
        s.add_request(r)
    out = s.schedule()
    assert [x.request for x in out.scheduled_new] == rs[:2] and list(s.waiting) == [rs[2]]


def test_token_budget_and_head_of_line_blocking():
    s = _sched(tokens=10)
    big, small = _req(0, 8), _req(1, 2)
    s.add_request(_req(2, 5))
    s.add_request(big)
    s.add_request(small)
    out = s.schedule()
    # 5 fit, the 8-token head of the line does not, and the 2-token one may not overtake it.
    assert [x.request.request_id for x in out.scheduled_new] == ["r2"]
    assert list(s.waiting) == [big, small]


def test_decode_step_is_one_token_and_grows_table_at_block_boundary():
    s = _sched(bs=4)
    r = _req(0, 4)
    s.add_request(r)
    s.schedule()
    assert len(s.block_manager.get_block_table(r)) == 1
    _emit(r)  # length 5 -> needs a second block at the next step
    out = s.schedule()
    assert [(x.request, x.num_scheduled_tokens) for x in out.scheduled_running] == [(r, 1)]
    assert len(s.block_manager.get_block_table(r)) == 2 and r.num_computed_tokens == 5
    for _ in range(3):  # lengths 6..8 fit in two blocks
        _emit(r)
        s.schedule()
    assert len(s.block_manager.get_block_table(r)) == 2


def test_preemption_frees_blocks_and_requeues_at_front():
    s = _sched(blocks=2, bs=4)
    a, b, c = _req(0, 4), _req(1, 4), _req(2, 1)
    for r in (a, b):
        s.add_request(r)
    s.schedule()
    s.add_request(c)
    for r in (a, b):
        _emit(r)  # both need a new block, none is free
    out = s.schedule()
    assert out.preempted == [b] and b.status == RequestStatus.PREEMPTED
    assert b.num_computed_tokens == 0 and s.block_manager.get_block_table(b) == []
    assert [x.request for x in out.scheduled_running] == [a]
    assert list(s.waiting) == [b, c] and out.scheduled_new == []  # no admission after a preemption


def test_preempted_request_resumes_as_prefill_of_everything_so_far():
    s = _sched(blocks=2, bs=4)
    a, b = _req(0, 4, max_tokens=1), _req(1, 4)
    s.add_request(a)
    s.add_request(b)
    s.schedule()
    _emit(b)
    _emit(a)  # a finishes (length cap 1) but still holds its block this step
    out = s.schedule()
    assert out.preempted == [b]
    assert s.free_finished_requests() == [a]
    out = s.schedule()
    assert [(x.request, x.num_scheduled_tokens) for x in out.scheduled_new] == [(b, 5)]
    assert b.status == RequestStatus.RUNNING and b.num_computed_tokens == 5


def test_self_preemption_when_alone():
    s = _sched(blocks=1, bs=4)
    r = _req(0, 4)
    s.add_request(r)
    s.schedule()
    _emit(r)
    out = s.schedule()
    assert out.preempted == [r] and out.scheduled_running == [] and list(s.waiting) == [r]


def test_finish_on_length_cap_and_eos():
    r = _req(0, 2, max_tokens=2)
    _emit(r)
    assert not r.is_finished()
    _emit(r)
    assert r.status == RequestStatus.FINISHED_LENGTH_CAPPED
    e = _req(1, 2, eos=9)
    _emit(e, tok=9)
    assert e.status == RequestStatus.FINISHED_STOPPED


def test_free_finished_releases_blocks():
    s = _sched(blocks=8)
    r = _req(0, 3, max_tokens=1)
    s.add_request(r)
    s.schedule()
    free0 = s.block_manager.num_free_blocks
    _emit(r)
    assert s.free_finished_requests() == [r]
    assert s.running == [] and s.block_manager.num_free_blocks == free0 + 1 and "r0" not in s.requests


def test_abort_waiting_running_and_unknown():
    s = _sched(seqs=1)
    a, b = _req(0, 3), _req(1, 3)
    s.add_request(a)
    s.add_request(b)
    s.schedule()
    assert s.abort_requests(["r1"]) == [b] and b.status == RequestStatus.FINISHED_ABORTED
    free0 = s.block_manager.num_free_blocks
    assert s.abort_requests(["r0", "nope"]) == [a]
    assert s.block_manager.num_free_blocks > free0 and not s.has_unfinished_requests()
    assert s.abort_requests(["nope"]) == []
