"""The allocation-free lm_head entry point, nd_head_logits_noalloc.

It serves callers that cannot call cudaMalloc — a process whose GPU memory
is owned by another allocator, or a serving loop that must not take
cudaMalloc's implicit device synchronisation — by keeping its int8
activations in one static device array of the library. This file sits last
in collection order so that a run stopping at its first failure has already
run every other test. It checks the entry point, called through the C ABI
with device buffers, against the allocating nd_head_logits on the same
inputs, for calls in a row (each with a different row count and values,
since every call shares the one array): 3 rows (the warp-per-row kernel),
7 rows (one partial 64-row tensor-core tile) and 64 rows (the largest
request, which fills the array to its last byte). Requests of 0 or 65 rows
are refused with a message.
"""

import ctypes

import numpy as np
import pytest

from parity_tools import bits_equal, describe_diff

pytestmark = pytest.mark.gpu


def _bind():
    import needle_b200 as nb

    lib = nb.lib()
    fn = lib.nd_head_logits_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p]
    return fn


def test_noalloc_head_logits_matches_allocating_entry(small_archive, cuda_device):
    import torch

    import needle_b200 as nb

    fn = _bind()
    model = nb.Model(small_archive, cuda_device)
    batch = model.batch(2, 64)  # room for 64 rows in the allocating entry
    dev = torch.device("cuda", cuda_device)
    stream = torch.cuda.current_stream(dev)
    rng = np.random.default_rng(99)
    for rows, scale in ((3, 1.0), (7, 25.0), (64, 4.0), (3, 0.5)):
        h = (rng.standard_normal((rows, model.d_model)) * scale).astype(np.float32)
        h_dev = torch.from_numpy(h).to(dev)
        out_dev = torch.full((rows, model.out_rows), float("nan"), dtype=torch.float32, device=dev)
        rc = fn(model._h, h_dev.data_ptr(), rows, out_dev.data_ptr(), stream.cuda_stream)
        assert rc == 0, nb.lib().nd_last_error().decode()
        torch.cuda.synchronize(dev)
        got = out_dev.cpu().numpy()
        want = batch.head_logits(h)
        assert bits_equal(got, want), describe_diff("noalloc logits", got, want)


def test_noalloc_rejects_oversized_requests(small_archive, cuda_device):
    import torch

    import needle_b200 as nb

    fn = _bind()
    model = nb.Model(small_archive, cuda_device)
    dev = torch.device("cuda", cuda_device)
    h_dev = torch.zeros((65, model.d_model), dtype=torch.float32, device=dev)
    out_dev = torch.zeros((65, model.out_rows), dtype=torch.float32, device=dev)
    for rows in (65, 0, -1):
        assert fn(model._h, h_dev.data_ptr(), rows, out_dev.data_ptr(), None) == -1
        assert b"rows must be in [1, 64]" in nb.lib().nd_last_error()
