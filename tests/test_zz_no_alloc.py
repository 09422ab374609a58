"""The allocation-free paged decode entry point, called through the C ABI.

lsb_paged_decode_static_scratch exists for callers that cannot allocate device
memory themselves (runtimes whose own pool owns the GPU's memory, FFI bindings
with no access to the host framework's allocator). It keeps its split-context
scratch in a fixed array inside the library. This test checks it against the
workspace-taking lsb_paged_decode on the same inputs, twice in a row (the
shared array keeps the previous call's contents, which must not leak into the
next result), and that oversized requests are refused. The file name sorts
last so a run that stops at the first failure has run every other test first.
"""
import pytest
import torch

from lightserve_b200 import _lib
from oracle.llama import paged_decode_ref

pytestmark = pytest.mark.gpu


def _inputs(seed, lens, S=6, H=4, D=128, bs=16, dtype=torch.bfloat16):
    g = torch.Generator().manual_seed(seed)
    max_blocks = max(-(-l // bs) for l in lens)
    nb = S * max_blocks + 5
    perm = torch.randperm(nb, generator=g)
    bt = torch.full((S, max_blocks), -1, dtype=torch.int32)
    for s, l in enumerate(lens):
        n = -(-l // bs)
        bt[s, :n] = perm[s * max_blocks: s * max_blocks + n].to(torch.int32)
    kc = torch.randn(nb, H, bs, D, generator=g).to(dtype).cuda()
    vc = torch.randn(nb, H, bs, D, generator=g).to(dtype).cuda()
    q = torch.randn(S, H, D, generator=g).to(dtype).cuda()
    return q, kc, vc, bt.cuda(), torch.tensor(lens, dtype=torch.int32).cuda(), max_blocks, bs, nb


def _args(q, kc, vc, bt, cl, o, max_blocks, bs, nb):
    S, H, D = q.shape
    return (q.data_ptr(), kc.data_ptr(), vc.data_ptr(), bt.data_ptr(), cl.data_ptr(), o.data_ptr(),
            S, H, D, max_blocks, bs, nb, q.stride(0), q.stride(1), o.stride(0), o.stride(1),
            1.0 / D ** 0.5, _lib.DTYPE_BF16)


def test_static_scratch_matches_workspace_entry_point_twice():
    lib = _lib.load()
    stream = torch.cuda.current_stream().cuda_stream
    for seed, lens in ((0, [1, 511, 513, 1500, 2049, 4000]), (1, [3000, 17, 700, 1024, 1, 2600])):
        q, kc, vc, bt, cl, max_blocks, bs, nb = _inputs(seed, lens)
        S, H, D = q.shape
        need = lib.lsb_paged_decode_workspace_size(S, H, D, max_blocks, bs)
        assert 0 < need <= lib.lsb_paged_decode_static_scratch_capacity()
        ws = torch.empty(need // 4, dtype=torch.float32, device="cuda")
        ref = torch.empty_like(q)
        _lib.check(lib.lsb_paged_decode(*_args(q, kc, vc, bt, cl, ref, max_blocks, bs, nb),
                                        ws.data_ptr(), need, stream), "lsb_paged_decode")
        out = torch.full_like(q, float("nan"))
        _lib.check(lib.lsb_paged_decode_static_scratch(
            *_args(q, kc, vc, bt, cl, out, max_blocks, bs, nb), stream),
            "lsb_paged_decode_static_scratch")
        torch.cuda.synchronize()
        # Same kernels, same launch shape, same inputs: bit-identical. The
        # second case runs over the array as the first case left it.
        assert torch.equal(out, ref)
        torch.testing.assert_close(out.float().cpu(), paged_decode_ref(q, kc, vc, bt.cpu(), cl.cpu()),
                                   atol=2e-2, rtol=2e-2)


def test_static_scratch_rejects_oversized_requests():
    lib = _lib.load()
    cap = lib.lsb_paged_decode_static_scratch_capacity()
    S, H, D, bs, max_blocks = 4096, 32, 128, 16, 4096
    assert lib.lsb_paged_decode_workspace_size(S, H, D, max_blocks, bs) > cap
    rc = lib.lsb_paged_decode_static_scratch(None, None, None, None, None, None, S, H, D, max_blocks,
                                             bs, 1, 0, 0, 0, 0, 1.0, _lib.DTYPE_BF16, None)
    assert rc == _lib.LSB_ERR_INVALID and "maximum" in _lib.last_error()
