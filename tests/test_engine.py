"""Block manager behaviour (the behaviours lightserve's
engine/tests/test_block_manager.py checks), plus the int32 table packing the
paged decode kernel reads."""
import pytest
import torch

from lightserve_b200.engine import BlockManager, OutOfMemoryError, Request


def req(rid="r0", prompt_len=10, num_output=0):
    r = Request(request_id=rid, prompt_token_ids=list(range(prompt_len)))
    r.output_token_ids = list(range(num_output))
    return r


def test_ceil_div_allocation_and_writeback():
    bm = BlockManager(block_size=4, num_gpu_blocks=10)
    r = req(prompt_len=9)
    assert bm.can_allocate(r)
    bm.allocate(r)
    assert len(bm.get_block_table(r)) == 3 and bm.num_free_blocks == 7
    assert r.block_table == bm.get_block_table(r)
    r2 = req("r1", prompt_len=8)
    bm.allocate(r2)
    assert len(bm.get_block_table(r2)) == 2


def test_watermark_only_at_admission():
    bm = BlockManager(block_size=4, num_gpu_blocks=10, watermark_blocks=2)
    assert bm.can_allocate(req(prompt_len=32))
    assert not bm.can_allocate(req("r1", prompt_len=33))


def test_oom_and_double_allocate():
    bm = BlockManager(block_size=4, num_gpu_blocks=2)
    r = req(prompt_len=9)
    assert not bm.can_allocate(r)
    with pytest.raises(OutOfMemoryError):
        bm.allocate(r)
    bm2 = BlockManager(block_size=4, num_gpu_blocks=10)
    r = req(prompt_len=4)
    bm2.allocate(r)
    with pytest.raises(ValueError):
        bm2.allocate(r)


def test_append_slot_grows_only_at_block_boundary():
    bm = BlockManager(block_size=4, num_gpu_blocks=10)
    r = req(prompt_len=4)
    bm.allocate(r)
    assert len(r.block_table) == 1
    sizes = []
    for i in range(9):
        r.output_token_ids.append(i)
        bm.append_slot(r)
        sizes.append(len(bm.get_block_table(r)))
    assert sizes == [2, 2, 2, 2, 3, 3, 3, 3, 4]
    with pytest.raises(ValueError):
        bm.append_slot(req("nope"))


def test_append_slot_pool_exhausted():
    bm = BlockManager(block_size=4, num_gpu_blocks=1)
    r = req(prompt_len=4)
    bm.allocate(r)
    r.output_token_ids.append(0)
    assert not bm.can_append_slot(r)
    with pytest.raises(OutOfMemoryError):
        bm.append_slot(r)


def test_free_idempotent_and_reusable():
    bm = BlockManager(block_size=4, num_gpu_blocks=4)
    r = req(prompt_len=16)
    bm.allocate(r)
    assert bm.num_free_blocks == 0
    bm.free(r)
    assert bm.num_free_blocks == 4 and r.block_table == []
    bm.free(r)
    bm.free(req("never"))
    assert bm.num_free_blocks == 4
    r2 = req("r2", prompt_len=16)
    bm.allocate(r2)
    assert sorted(r2.block_table) == [0, 1, 2, 3]


def test_as_tensor_packs_tables():
    bm = BlockManager(block_size=16, num_gpu_blocks=8)
    a, b = req("a", prompt_len=20), req("b", prompt_len=5)
    bm.allocate(a); bm.allocate(b)
    t = bm.as_tensor([a, b], max_blocks=3)
    assert t.dtype == torch.int32 and t.shape == (2, 3)
    assert t[0, :2].tolist() == a.block_table and t[0, 2] == -1
    assert t[1, 0] == b.block_table[0] and t[1, 1:].tolist() == [-1, -1]
    with pytest.raises(ValueError):
        bm.as_tensor([a], max_blocks=1)
