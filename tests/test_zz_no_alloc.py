"""gsa_indexer_topk_noalloc, the entry point that allocates no device memory.

Some callers cannot call cudaMalloc: a plugin running inside a host engine
that owns all device memory, or a runtime that fixes its memory budget at
start-up (an allocation can synchronise the device and fragment the pool).
They cannot pass gsa_indexer_topk the scratch it takes as `workspace`, so
this variant keeps that scratch in a buffer built into the library (16 MiB per
GPU).  The test calls it through the C ABI and checks its outputs against
gsa_indexer_topk with a caller workspace, on two calls in a row.  The second
call uses other shapes, so it also shows that the scores the first call left
in the shared buffer do not leak into the second.  It also checks that a call
needing more scratch than the built-in buffer holds is refused with a clear
message.

The file name sorts last, so a run that stops at the first failure has run
every other test before this one."""
import pytest
import torch

from gsa_gdn_benchmarkstudy_b200 import _lib
from gsa_gdn_benchmarkstudy_b200.build import build

pytestmark = pytest.mark.gpu
torch.set_grad_enabled(False)

GSA_ERR_UNSUPPORTED = 3


def _inputs(B, Tq, Tkv, seed):
    g = torch.Generator().manual_seed(seed)
    q = (torch.randn(B, Tq, 4 * 64, generator=g) * 0.9).bfloat16().cuda()
    k = (torch.randn(B, Tkv, 64, generator=g) * 0.9).bfloat16().cuda()
    w = torch.randn(B, Tq, 4, generator=g).bfloat16().cuda()
    bias = (torch.randn(4, generator=g) * 0.1).float().cuda()
    return q, k, w, bias


def _outputs(B, Tq, k_sel, words):
    return (torch.full((B, Tq, k_sel), -7, dtype=torch.int32, device="cuda"),
            torch.full((B, Tq, k_sel), 9, dtype=torch.uint8, device="cuda"),
            torch.full((B, Tq, words), -1, dtype=torch.int32, device="cuda"))


def _run(lib, noalloc, q, k, w, bias, Tkv, q_pos0, k_sel):
    B, Tq = q.shape[0], q.shape[1]
    words = lib.gsa_bitmask_words(Tkv)
    idx, msk, bm = _outputs(B, Tq, k_sel, words)
    stream = torch.cuda.current_stream().cuda_stream
    common = (q.data_ptr(), q.stride(1), k.data_ptr(), k.stride(1), w.data_ptr(), w.stride(1),
              bias.data_ptr(), 0.125, 0, B, Tq, Tkv, q_pos0, 4, 64, k_sel)
    if noalloc:
        rc = lib.gsa_indexer_topk_noalloc(*common, idx.data_ptr(), msk.data_ptr(),
                                          bm.data_ptr(), words, stream)
    else:
        need = lib.gsa_indexer_topk_workspace_size(B, Tq, Tkv)
        ws = torch.empty(need, dtype=torch.uint8, device="cuda")
        rc = lib.gsa_indexer_topk(*common, ws.data_ptr(), need, idx.data_ptr(), msk.data_ptr(),
                                  bm.data_ptr(), words, stream)
    assert rc == 0, lib.gsa_last_error_string().decode()
    torch.cuda.synchronize()
    return idx.cpu(), msk.cpu(), bm.cpu()


def test_noalloc_matches_workspace_entry_on_two_calls_in_a_row():
    build()
    lib = _lib.load()
    cases = [(1, 700, 1500, 800, 256, 11), (2, 160, 160, 0, 48, 12)]
    for B, Tq, Tkv, q_pos0, k_sel, seed in cases:
        q, k, w, bias = _inputs(B, Tq, Tkv, seed)
        got = _run(lib, True, q, k, w, bias, Tkv, q_pos0, k_sel)
        ref = _run(lib, False, q, k, w, bias, Tkv, q_pos0, k_sel)
        # same kernels on the same inputs: identical indices, mask and bitmask
        for a, b in zip(got, ref):
            assert torch.equal(a, b)
    assert _lib.device_error() == 0


def test_noalloc_refuses_calls_beyond_its_buffer():
    build()
    lib = _lib.load()
    B, Tq, Tkv = 1, 4096, 4096  # 64 MiB of scores > 16 MiB built in
    assert lib.gsa_indexer_topk_workspace_size(B, Tq, Tkv) > 16 << 20
    q, k, w, bias = _inputs(B, Tq, Tkv, 13)
    words = lib.gsa_bitmask_words(Tkv)
    _, _, bm = _outputs(B, Tq, 16, words)
    rc = lib.gsa_indexer_topk_noalloc(q.data_ptr(), q.stride(1), k.data_ptr(), k.stride(1),
                                      w.data_ptr(), w.stride(1), bias.data_ptr(), 0.125, 0, B, Tq,
                                      Tkv, 0, 4, 64, 16, None, None, bm.data_ptr(), words,
                                      torch.cuda.current_stream().cuda_stream)
    assert rc == GSA_ERR_UNSUPPORTED
    assert b"built-in" in lib.gsa_last_error_string()
