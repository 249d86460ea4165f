"""The allocation-free Freivalds entry point (ima_freivalds_fp8_noalloc).

Callers that cannot allocate device memory -- a verifier living in a process whose
device memory is reserved by another allocator, or a latency-sensitive path that must
not pay for cudaMalloc/cudaFree -- use this variant, whose scratch vector lives in a
fixed device array inside the library.  This test calls it through the C ABI and checks
it against the allocating entry point (ima_freivalds_fp8) on two calls in a row: a
correct product (no rejected rows) and the same product with corrupted entries (the same
rejected rows as the allocating check).  The file is named to be collected last.
"""

from __future__ import annotations

import ctypes

import pytest
import torch

from int_model_approximation_b200 import _native as nat
from int_model_approximation_b200 import codebook, synthetic
from int_model_approximation_b200.freivalds import freivalds_vector

pytestmark = pytest.mark.gpu


def _product(device, m, k, n, seed):
    x = synthetic.student_t_activations(m, k, seed=seed).to(device)
    w, _ws = synthetic.normal_fp8_weights(n, k, seed=seed + 1)
    w = w.to(device)
    q, _s, _cb, _cs, planes = codebook.per_token_fp8(x, planes=True)
    b, _ = codebook.codebook_planes_from_fp8(w)
    c, _ = codebook.int_gemm(planes, b)
    r = freivalds_vector(n, seed=seed + 2, device=device)
    return q.view(torch.uint8), w.view(torch.uint8), c, r


def _allocating(q, w, c, r):
    m, k = q.shape
    n = w.shape[0]
    out = torch.zeros((1,), dtype=torch.int32, device=c.device)
    ws = torch.empty((k,), dtype=torch.int64, device=c.device)
    nat.call("ima_freivalds_fp8", q.data_ptr(), k, w.data_ptr(), k, c.data_ptr(), n, r.data_ptr(), m, n, k,
             ws.data_ptr(), out.data_ptr(), nat.stream_of(c.device))
    return int(out.item())


def _noalloc(q, w, c, r):
    m, k = q.shape
    n = w.shape[0]
    out = torch.zeros((1,), dtype=torch.int32, device=c.device)
    nat.call("ima_freivalds_fp8_noalloc", q.data_ptr(), k, w.data_ptr(), k, c.data_ptr(), n, r.data_ptr(), m, n,
             k, out.data_ptr(), nat.stream_of(c.device))
    return int(out.item())


def test_noalloc_freivalds_matches_the_allocating_check_on_two_calls(cuda_device):
    q, w, c, r = _product(cuda_device, 77, 4864, 300, seed=5)
    # first call: a correct product
    assert _noalloc(q, w, c, r) == _allocating(q, w, c, r) == 0
    # second call in a row (the scratch keeps the first call's contents): corrupted rows
    bad = c.clone()
    bad[3, 7] += 1
    bad[40, 299] -= 9
    expected = _allocating(q, w, bad, r)
    assert expected == int(r[7].item() != 0) + int(r[299].item() != 0) == 2
    assert _noalloc(q, w, bad, r) == expected
    # a different, smaller product afterwards still agrees
    q2, w2, c2, r2 = _product(cuda_device, 5, 96, 40, seed=9)
    c2[0, 0] += 3
    assert _noalloc(q2, w2, c2, r2) == _allocating(q2, w2, c2, r2) == 1


def test_noalloc_freivalds_on_two_streams_ordered_by_an_event(cuda_device):
    """Two calls on different streams, the second ordered after the first by an event, agree
    with the allocating check (the shared array is cleared by each call)."""
    q, w, c, r = _product(cuda_device, 64, 896, 130, seed=13)
    bad = c.clone()
    bad[10, 5] += 2
    outs = [torch.zeros((1,), dtype=torch.int32, device=cuda_device) for _ in range(2)]
    s1, s2 = torch.cuda.Stream(cuda_device), torch.cuda.Stream(cuda_device)
    s1.wait_stream(torch.cuda.current_stream(cuda_device))
    m, k = q.shape
    n = w.shape[0]
    with torch.cuda.stream(s1):
        nat.call("ima_freivalds_fp8_noalloc", q.data_ptr(), k, w.data_ptr(), k, bad.data_ptr(), n, r.data_ptr(), m,
                 n, k, outs[0].data_ptr(), s1.cuda_stream)
    done = torch.cuda.Event()
    done.record(s1)
    s2.wait_event(done)
    with torch.cuda.stream(s2):
        nat.call("ima_freivalds_fp8_noalloc", q.data_ptr(), k, w.data_ptr(), k, c.data_ptr(), n, r.data_ptr(), m,
                 n, k, outs[1].data_ptr(), s2.cuda_stream)
    torch.cuda.synchronize(cuda_device)
    assert int(outs[0].item()) == _allocating(q, w, bad, r) == int(r[5].item() != 0)
    assert int(outs[1].item()) == _allocating(q, w, c, r) == 0


def test_noalloc_freivalds_refuses_operands_off_the_current_device(cuda_device):
    """A host pointer among the operands is refused before any launch (the call would
    otherwise pair the current device's scratch array with memory the kernels cannot use)."""
    q, w, c, r = _product(cuda_device, 8, 64, 16, seed=17)
    m, k = q.shape
    n = w.shape[0]
    out = torch.zeros((1,), dtype=torch.int32, device=cuda_device)
    host_c = c.cpu()
    lib = nat.lib()
    stream = ctypes.c_void_p(nat.stream_of(cuda_device))
    status = lib.ima_freivalds_fp8_noalloc(q.data_ptr(), k, w.data_ptr(), k, host_c.data_ptr(), n, r.data_ptr(), m,
                                           n, k, out.data_ptr(), stream)
    assert status == nat.IMA_ERR_INVALID_ARGUMENT
    host_out = torch.zeros((1,), dtype=torch.int32)
    status = lib.ima_freivalds_fp8_noalloc(q.data_ptr(), k, w.data_ptr(), k, c.data_ptr(), n, r.data_ptr(), m, n, k,
                                           host_out.data_ptr(), stream)
    assert status == nat.IMA_ERR_INVALID_ARGUMENT
    torch.cuda.synchronize(cuda_device)
    assert int(out.item()) == 0 and int(host_out.item()) == 0
    # the same call with device operands still works afterwards
    assert _noalloc(q, w, c, r) == 0


def test_noalloc_freivalds_rejects_sizes_beyond_its_scratch(cuda_device):
    lib = nat.lib()
    max_k = 65536
    dummy = torch.zeros((16,), dtype=torch.int64, device=cuda_device)
    status = lib.ima_freivalds_fp8_noalloc(dummy.data_ptr(), max_k + 1, dummy.data_ptr(), max_k + 1,
                                           dummy.data_ptr(), 1, dummy.data_ptr(), 1, 1, max_k + 1,
                                           dummy.data_ptr(), ctypes.c_void_p(nat.stream_of(cuda_device)))
    assert status == nat.IMA_ERR_UNSUPPORTED
